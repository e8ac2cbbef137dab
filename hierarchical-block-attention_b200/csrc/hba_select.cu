// Routed-block selection: flat scan, super level and child level of the
// two-level beam descent.  Bandwidth/latency-bound: no tensor cores.
//
// One CTA per (split, query, batch*kv-head).  The CTA (1) builds the grouped
// routing query -- QKNorm'd query heads of the KV group, each rounded to bf16,
// summed in fp32 in head order and rounded to bf16 (reference
// src/hba/summarizer.py:50-54 on bf16 tensors) -- (2) scores its slice of the
// candidates, one warp per candidate, with 16-byte coalesced summary loads:
// score = max_slot(qg . S[slot]) * scale (summarizer.py:45-47), and (3) keeps
// a warp-cooperative top-k of (score desc, block index asc) that it writes as
// one partial list.  The next kernel merges the partial lists.
#include <climits>

#include "hba_common.cuh"
#include "hba_internal.h"

namespace hba {

constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kMaxCandPerCta = 2048;

HBA_DEVICE void query_position(const QueryPos& qp, int b, int t, int& pos, int& nctx, float& scale) {
  if (qp.seq_lens != nullptr) {
    nctx = qp.seq_lens[b];
    pos = nctx - 1;
    scale = qp.scales[b];
  } else {
    nctx = qp.n_fixed;
    pos = t;
    scale = qp.scale_fixed;
  }
}

// Candidate blocks of the query at `pos`: 1 .. bmax (reference
// attention.py:250-256: b >= 1 and (b+1)*Bk <= pos - W + 1); 0 when none.
HBA_DEVICE int last_candidate(int pos, int W, int Bk) {
  const int lim = pos - W + 1;
  return lim >= 2 * Bk ? lim / Bk - 1 : 0;
}

// max over slots of qg . S[slot] for one summary row of m*DH bf16 values.
// Lane l takes 16-byte vectors l, l+32, ...; each group of DH/8 lanes covers
// one slot of one vector round.
template <int DH>
HBA_DEVICE float slot_score(const __nv_bfloat16* __restrict__ S, const float* __restrict__ qg, int m) {
  constexpr int LPS = DH / 8;
  const int lane = threadIdx.x & 31;
  const int nvec = m * DH / 8;
  float best = neg_inf();
  for (int v0 = 0; v0 < nvec; v0 += 32) {
    const int v = v0 + lane;
    float part = 0.f;
    if (v < nvec) {
      float f[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(S) + v), f);
      const int d0 = (v * 8) % DH;
#pragma unroll
      for (int j = 0; j < 8; ++j) part = fmaf(f[j], qg[d0 + j], part);
    }
#pragma unroll
    for (int o = 1; o < LPS; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (v < nvec) best = fmaxf(best, part);
  }
  return warp_max(best);
}

template <int DH>
__global__ void __launch_bounds__(kSelThreads) select_kernel(SelParams p) {
  const Geom& geo = p.geo;
  const int split = blockIdx.x, t = blockIdx.y, bg = blockIdx.z;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  __shared__ float qc_s[16][DH];
  __shared__ float qg_s[DH];
  __shared__ float sc_s[kMaxCandPerCta];
  __shared__ int id_s[kMaxCandPerCta];
  __shared__ int sup_lo[32], sup_off[32], sup_cnt[32];
  __shared__ int n_children;

  int pos, nctx;
  float scale;
  query_position(p.qp, b, t, pos, nctx, scale);
  const size_t list_base = (((size_t)bg * geo.nq + t) * p.splits + split) * p.list_k;
  const bool ok_pos = (nctx >= 1 && nctx <= geo.n_cap);

  // ---- grouped routing query ----
  constexpr int PER = DH / 32;
  for (int h = warp; h < geo.G; h += kSelWarps) {
    const int hq = g * geo.G + h;
    float v[PER];
    load_head_row<DH>(p.q + (((size_t)b * geo.nq + t) * geo.Hq + hq) * DH, v);
    if (geo.qknorm) qknorm_lane<DH>(v, p.q_gain[hq], geo.eps);
#pragma unroll
    for (int i = 0; i < PER; ++i) qc_s[h][lane * PER + i] = v[i];
  }
  __syncthreads();
  for (int d = tid; d < DH; d += kSelThreads) {
    float s = 0.f;
    for (int h = 0; h < geo.G; ++h) s += qc_s[h][d];
    qg_s[d] = round_bf16(s);
  }

  const int nb = ok_pos ? nctx / geo.Bk : 0;
  const int bmax = ok_pos ? min(last_candidate(pos, geo.W, geo.Bk), nb - 1) : 0;
  const int F = geo.F;

  // ---- this CTA's candidate slice ----
  int C = 0;       // candidates of this query (all splits)
  int id_lo = 0;   // flat/super: id of candidate j is id_lo + j
  if (p.mode == kSelFlat) {
    C = bmax;
    id_lo = 1;
  } else if (p.mode == kSelSuper) {
    if (bmax >= 1) {
      id_lo = (F == 1) ? 1 : 0;
      C = bmax / F - id_lo + 1;
    }
  } else {
    // merge the super lists: top b_eff supers, then enumerate their candidate children
    const int ns = (nb + F - 1) / F;
    const int b_eff = min(geo.beam, ns);
    if (warp == 0) {
      WarpTopK top;
      top.init();
      const int total = p.in_lists * geo.beam;
      const size_t base = ((size_t)bg * geo.nq + t) * total;
      for (int e0 = 0; e0 < total; e0 += 32) {
        const int e = e0 + lane;
        float s = neg_inf();
        int i = INT_MAX;
        if (e < total) {
          const int ii = p.in_idx[base + e];
          if (ii >= 0) {
            s = p.in_score[base + e];
            i = ii;
          }
        }
        if (b_eff > 0) top.offer(s, i, b_eff);
      }
      const bool valid = lane < b_eff && top.i != INT_MAX;
      int lo = 0, cnt = 0;
      if (valid) {
        lo = max(1, top.i * F);
        const int hi = min(bmax, top.i * F + F - 1);
        cnt = max(0, hi - lo + 1);
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int nv = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += nv;
      }
      sup_lo[lane] = lo;
      sup_cnt[lane] = cnt;
      sup_off[lane] = incl - cnt;
      if (lane == 31) n_children = incl;
    }
    __syncthreads();
    C = n_children;
  }
  const int j0 = (int)(((long long)C * split) / p.splits);
  const int j1 = (int)(((long long)C * (split + 1)) / p.splits);
  const int R = j1 - j0;  // host guarantees R <= kMaxCandPerCta

  // ---- score ----
  const __nv_bfloat16* src;
  int rows_cap;
  if (p.mode == kSelSuper) {
    src = p.supers;
    rows_cap = geo.ns_cap;
  } else {
    src = p.summ;
    rows_cap = geo.nb_cap;
  }
  const size_t row_elems = (size_t)geo.m * DH;
  const __nv_bfloat16* base = src + ((size_t)bg * rows_cap) * row_elems;
  __syncthreads();
  for (int r = warp; r < R; r += kSelWarps) {
    const int j = j0 + r;
    int id;
    if (p.mode == kSelChild) {
      int s = 0;
      while (s < 31 && j >= sup_off[s] + sup_cnt[s]) ++s;
      id = sup_lo[s] + (j - sup_off[s]);
    } else {
      id = id_lo + j;
    }
    const float sc = slot_score<DH>(base + (size_t)id * row_elems, qg_s, geo.m) * scale;
    if (lane == 0) {
      sc_s[r] = sc;
      id_s[r] = id;
    }
  }
  __syncthreads();

  // ---- partial top-k of this slice ----
  if (warp == 0) {
    WarpTopK top;
    top.init();
    const int k = p.list_k;
    for (int e0 = 0; e0 < R; e0 += 32) {
      const int e = e0 + lane;
      const float s = e < R ? sc_s[e] : neg_inf();
      const int i = e < R ? id_s[e] : INT_MAX;
      top.offer(s, i, k);
    }
    if (lane < k) {
      const bool valid = top.i != INT_MAX;
      p.out_score[list_base + lane] = valid ? top.s : neg_inf();
      p.out_idx[list_base + lane] = valid ? top.i : -1;
    }
  }
}

cudaError_t launch_select(const SelParams& p, int dh, cudaStream_t st) {
  dim3 grid(p.splits, p.geo.nq, p.geo.B * p.geo.Hkv);
  if (dh == 64)
    select_kernel<64><<<grid, kSelThreads, 0, st>>>(p);
  else
    select_kernel<128><<<grid, kSelThreads, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace hba
