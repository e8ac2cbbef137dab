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
#include "hba_score.cuh"

namespace hba {

constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kMaxCandPerCta = 2048;

template <int DH, int VPL>
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

  // let the next kernel of the chain start launching; a child-level kernel
  // reads the super lists of the previous kernel, so it waits for it first
  grid_dep_launch_dependents();
  if (p.pdl) grid_dep_wait();
  if (p.counters != nullptr && split == 0 && t == 0 && tid == 0) p.counters[bg] = 0;

  int pos, nctx;
  float scale;
  query_position(p.qp, b, t, pos, nctx, scale);
  const size_t list_base = (((size_t)bg * geo.nq + t) * p.splits + split) * p.list_k;
  const bool ok_pos = (nctx >= 1 && nctx <= p.n_limit);
  const int nb = ok_pos ? nctx / geo.Bk : 0;
  const int bmax = ok_pos ? min(last_candidate(pos, geo.W, geo.Bk), nb - 1) : 0;
  const int F = geo.F;

  // ---- candidate range (flat / super known from the position alone),
  // intersected with the blocks (supers) this shard owns ----
  const int own_slo = p.own_blo / F;
  const int own_shi = p.own_bhi == INT_MAX ? INT_MAX : p.own_bhi / F;
  int C = 0, id_lo = 0;
  if (p.mode == kSelFlat) {
    id_lo = max(1, p.own_blo);
    C = max(0, min(bmax, p.own_bhi - 1) - id_lo + 1);
  } else if (p.mode == kSelSuper) {
    if (bmax >= 1) {
      id_lo = max((F == 1) ? 1 : 0, own_slo);
      C = max(0, min(bmax / F, own_shi - 1) - id_lo + 1);
    }
  }
  const __nv_bfloat16* src;
  int rows_cap, row_base;
  if (p.mode == kSelSuper) {
    src = p.supers;
    rows_cap = geo.ns_cap;
    row_base = own_slo;
  } else {
    src = p.summ;
    rows_cap = geo.nb_cap;
    row_base = p.own_blo;
  }
  const size_t row_elems = (size_t)geo.m * DH;
  // row of candidate id: id - row_base
  const __nv_bfloat16* base = src + ((ptrdiff_t)bg * rows_cap - row_base) * (ptrdiff_t)row_elems;
  const int nvec = geo.m * DH / 8;
  SummaryLoads<DH, VPL, kSelWarps> ld;
  constexpr int GROUP = kSelWarps * SummaryLoads<DH, VPL, kSelWarps>::U;
  auto flat_id = [&](int r) { return id_lo + (int)(((long long)C * split) / p.splits) + r; };
  int R = 0;
  if (p.mode != kSelChild) {
    R = (int)(((long long)C * (split + 1)) / p.splits) - (int)(((long long)C * split) / p.splits);
    ld.load(base, row_elems, nvec, 0, R, flat_id);  // in flight during the query prologue
  }

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
    float sacc = 0.f;
    for (int h = 0; h < geo.G; ++h) sacc += qc_s[h][d];
    qg_s[d] = round_bf16(sacc);
  }

  if (p.mode == kSelChild) {
    // merge the super lists: top b_eff supers, then enumerate their candidate children
    const int ns = (nb + F - 1) / F;
    const int b_eff = min(geo.beam, ns);
    if (warp == 0) {
      WarpTopK top;
      top.init();
      const int total = p.in_lists * geo.beam;
      const size_t lbase = ((size_t)bg * geo.nq + t) * total;
      for (int e0 = 0; e0 < total; e0 += 32) {
        const int e = e0 + lane;
        float sv = neg_inf();
        int i = INT_MAX;
        if (e < total) {
          const int ii = __ldcg(p.in_idx + lbase + e);
          if (ii >= 0) {
            sv = __ldcg(p.in_score + lbase + e);
            i = ii;
          }
        }
        if (b_eff > 0) top.offer(sv, i, b_eff);
      }
      const bool valid = lane < b_eff && top.i != INT_MAX;
      int lo = 0, cnt = 0;
      if (valid) {
        lo = max(max(1, top.i * F), p.own_blo);
        const int hi = min(min(bmax, top.i * F + F - 1), p.own_bhi - 1);
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
  __syncthreads();
  const int j0 = (int)(((long long)C * split) / p.splits);
  R = (int)(((long long)C * (split + 1)) / p.splits) - j0;  // host guarantees R <= kMaxCandPerCta
  auto child_id = [&](int r) {
    const int j = j0 + r;
    int sidx = 0;
    while (sidx < 31 && j >= sup_off[sidx] + sup_cnt[sidx]) ++sidx;
    return sup_lo[sidx] + (j - sup_off[sidx]);
  };

  // ---- score ----
  if (p.mode == kSelChild) {
    for (int rb = 0; rb < R; rb += GROUP) {
      ld.load(base, row_elems, nvec, rb, R, child_id);
      ld.score(qg_s, nvec, rb, R, scale, child_id, sc_s, id_s);
    }
  } else {
    for (int rb = 0; rb < R; rb += GROUP) {
      if (rb > 0) ld.load(base, row_elems, nvec, rb, R, flat_id);
      ld.score(qg_s, nvec, rb, R, scale, flat_id, sc_s, id_s);
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
      const float sv = e < R ? sc_s[e] : neg_inf();
      const int i = e < R ? id_s[e] : INT_MAX;
      top.offer(sv, i, k);
    }
    if (lane < k) {
      const bool valid = top.i != INT_MAX;
      p.out_score[list_base + lane] = valid ? top.s : neg_inf();
      p.out_idx[list_base + lane] = valid ? top.i : -1;
    }
  }
}

template <int DH, int VPL>
static cudaError_t launch_select_t(const SelParams& p, cudaStream_t st) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(p.splits, p.geo.nq, p.geo.B * p.geo.Hkv);
  lc.blockDim = dim3(kSelThreads);
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = p.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&lc, select_kernel<DH, VPL>, p);
}

cudaError_t launch_select(const SelParams& p, int dh, cudaStream_t st) {
  const int nvec = p.geo.m * dh / 8;  // 16-byte vectors per summary row
  const int vpl = (nvec + 31) / 32;
  if (dh == 64) {
    if (vpl <= 1) return launch_select_t<64, 1>(p, st);
    return launch_select_t<64, 2>(p, st);
  }
  if (vpl <= 1) return launch_select_t<128, 1>(p, st);
  if (vpl <= 2) return launch_select_t<128, 2>(p, st);
  return launch_select_t<128, 4>(p, st);
}

}  // namespace hba
