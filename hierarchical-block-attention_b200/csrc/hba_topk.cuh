// Block-wide top-k over up to kTopkMaxItems (score, index) pairs held in
// shared memory, under the library's total order: higher score first, then
// lower index.  Radix select on the order-preserving 32-bit image of the
// score: four passes of an 8-bit digit histogram (warp-aggregated shared
// atomics) find the k-th largest key v; keys > v are taken, and the remaining
// slots go to keys == v by ascending index (a scan is needed only when there
// are more such ties than free slots).  The <= 32 survivors are ranked.
#pragma once

#include <climits>

#include "hba_common.cuh"

namespace hba {

constexpr int kTopkMaxItems = 2048;

// Monotone map float -> uint32 (a > b  <=>  key(a) > key(b)); -inf -> small.
HBA_DEVICE uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct TopkScratch {
  int hist[256];
  int digit;
  int k_rem;
  int ties;
  int n_sel;
  int sel_idx[32];
  float sel_score[32];
};

// Every thread of the block must call this (contains barriers).  Writes the
// selected entries, best first, to ts.sel_idx / ts.sel_score[0..n) and
// returns n = min(k, R, 32).  NT = blockDim.x.  id == nullptr means the
// candidate's id is its position j (callers whose ids grow with j map the
// returned positions to ids afterwards).
template <int NT>
HBA_DEVICE int block_topk(const float* __restrict__ sc, const int* __restrict__ id, int R, int k,
                          TopkScratch& ts) {
  constexpr int E = (kTopkMaxItems + NT - 1) / NT;
  const int tid = threadIdx.x, lane = tid & 31;
  if (k > 32) k = 32;
  const int take = min(k, R);
  if (take <= 0) {
    if (tid == 0) ts.n_sel = 0;
    __syncthreads();
    return 0;
  }
  uint32_t key[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int j = tid + e * NT;
    key[e] = j < R ? order_key(sc[j]) : 0u;
  }
  uint32_t prefix = 0, pmask = 0;
  int k_rem = take;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += NT) ts.hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int j = tid + e * NT;
      const bool in = j < R && (key[e] & pmask) == prefix;
      const unsigned act = __ballot_sync(0xffffffffu, in);
      if (in) {
        const int bin = (key[e] >> shift) & 0xFF;
        const unsigned peers = __match_any_sync(act, bin);
        if ((__ffs(peers) - 1) == lane) atomicAdd(&ts.hist[bin], __popc(peers));
      }
    }
    __syncthreads();
    if (tid < 32) {
      // lane l owns bins [255 - 8l - 7, 255 - 8l], scanned from the top
      int c[8], tot = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = ts.hist[255 - 8 * lane - i];
        tot += c[i];
      }
      int incl = tot;  // inclusive prefix over lanes = elements in bins above and at this lane's range
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int nv = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += nv;
      }
      const int before = incl - tot;  // elements in strictly higher bins
      if (before < k_rem && k_rem <= incl) {
        int acc = before;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (acc < k_rem && k_rem <= acc + c[i]) {
            ts.digit = 255 - 8 * lane - i;
            ts.k_rem = k_rem - acc;
            ts.ties = c[i];
          }
          acc += c[i];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)ts.digit << shift;
    pmask |= 0xFFu << shift;
    k_rem = ts.k_rem;
  }
  const uint32_t v = prefix;  // the take-th largest key
  const int need_ties = k_rem;
  const bool all_ties = ts.ties == need_ties;
  if (tid == 0) ts.n_sel = 0;
  __syncthreads();
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int j = tid + e * NT;
    if (j < R) {
      bool pick = key[e] > v;
      if (!pick && key[e] == v) {
        if (all_ties) {
          pick = true;
        } else {  // genuine ties at the boundary: keep the lowest indices
          int before = 0;
          for (int i = 0; i < R; ++i)
            if (order_key(sc[i]) == v && (id ? id[i] : i) < (id ? id[j] : j)) ++before;
          pick = before < need_ties;
        }
      }
      if (pick) {
        const int slot = atomicAdd(&ts.n_sel, 1);
        ts.sel_idx[slot] = j;  // position in sc/id, ranked below
      }
    }
  }
  __syncthreads();
  const int n = ts.n_sel;
  int my_pos = -1, my_id = 0;
  float my_s = 0.f;
  if (tid < n) {
    const int j = ts.sel_idx[tid];
    my_s = sc[j];
    my_id = id ? id[j] : j;
    int r = 0;
    for (int i = 0; i < n; ++i) {
      const int ji = ts.sel_idx[i];
      const float si = sc[ji];
      const int ii = id ? id[ji] : ji;
      r += (si > my_s) || (si == my_s && ii < my_id);
    }
    my_pos = r;
  }
  __syncthreads();
  if (tid < n) {
    ts.sel_idx[my_pos] = my_id;
    ts.sel_score[my_pos] = my_s;
  }
  __syncthreads();
  return n;
}

}  // namespace hba
