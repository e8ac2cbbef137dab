// Block-wide top-k over up to kTopkMaxItems (score, index) pairs held in
// shared memory, under the library's total order: higher score first, then
// lower index.  Radix select: 32 bisection steps on the order-preserving
// integer image of the score find the k-th largest score, ties at that score
// are taken by ascending index, and the <= k survivors are ranked.  Cost
// O(R/threads) per step with two barriers per step, independent of k.
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
  int warp_cnt[2][32];
  int n_sel;
  int sel_idx[32];
  float sel_score[32];
};

// Every thread of the block must call this (contains barriers).  Writes the
// selected entries, best first, to out_idx/out_score[0..k) (-1 / -inf padding)
// of `ts`, and returns the number of valid picks.  NT = blockDim.x.
template <int NT>
HBA_DEVICE int block_topk(const float* __restrict__ sc, const int* __restrict__ id, int R, int k,
                          TopkScratch& ts) {
  constexpr int NW = NT / 32;
  constexpr int E = (kTopkMaxItems + NT - 1) / NT;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t key[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int j = tid + e * NT;
    key[e] = j < R ? order_key(sc[j]) : 0u;
  }
  auto block_count = [&](uint32_t thr, bool strict, int buf) -> int {
    int c = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int j = tid + e * NT;
      if (j < R) c += strict ? (key[e] > thr) : (key[e] >= thr);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) ts.warp_cnt[buf][warp] = c;
    __syncthreads();
    int t = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) t += ts.warp_cnt[buf][w];
    return t;
  };
  if (k > 32) k = 32;
  int take = min(k, R);
  if (tid == 0) ts.n_sel = 0;
  if (take <= 0) {
    __syncthreads();
    return 0;
  }
  // largest threshold v with count(key >= v) >= take  ==  the take-th largest key
  uint32_t v = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = v | (1u << bit);
    if (block_count(cand, false, bit & 1) >= take) v = cand;
  }
  const int greater = block_count(v, true, 1);  // the last bisection step used buffer 0
  const int need_ties = take - greater;  // ties at v taken by ascending index
  __syncthreads();
  // compact: all keys > v, and ties at v whose index rank among ties < need_ties
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int j = tid + e * NT;
    if (j < R) {
      bool pick = key[e] > v;
      if (!pick && key[e] == v) {
        int before = 0;  // ties at v with a lower index (ties are rare: linear scan)
        for (int i = 0; i < R; ++i)
          if (order_key(sc[i]) == v && id[i] < id[j]) ++before;
        pick = before < need_ties;
      }
      if (pick) {
        const int slot = atomicAdd(&ts.n_sel, 1);
        ts.sel_idx[slot] = j;  // position in sc/id, ranked below
      }
    }
  }
  __syncthreads();
  // rank the survivors (<= 32) by (score desc, index asc)
  const int n = ts.n_sel;
  int my_pos = -1, my_id = 0;
  float my_s = 0.f;
  if (tid < n) {
    const int j = ts.sel_idx[tid];
    my_s = sc[j];
    my_id = id[j];
    int r = 0;
    for (int i = 0; i < n; ++i) {
      const int ji = ts.sel_idx[i];
      const float si = sc[ji];
      const int ii = id[ji];
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
