// Summary scoring shared by the selection kernels and the fused decode
// kernel, so that every path computes bit-identical routing scores.
#pragma once

#include "hba_common.cuh"
#include "hba_internal.h"

namespace hba {

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

// One warp scores candidates r = rbase + warp + NWARPS*u, u < U: lane l
// holds 16-byte vectors l, l+32, ... (VPL per candidate) of the candidate's
// m*DH bf16 summary row; loads for all U candidates are issued before any is
// used.  score = max over slots of qg . S[slot] (each group of DH/8 lanes of
// one vector round covers one slot), times the union scale.
template <int DH, int VPL, int NWARPS>
struct SummaryLoads {
  static constexpr int U = 8 / VPL;
  uint4 buf[U][VPL];

  template <typename IdFn>
  HBA_DEVICE void load(const __nv_bfloat16* __restrict__ base, size_t row_elems, int nvec, int rbase, int R,
                       IdFn id_of) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int r = rbase + warp + NWARPS * u;
      if (r < R) {
        const uint4* src = reinterpret_cast<const uint4*>(base + (size_t)id_of(r) * row_elems);
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          const int vv = lane + 32 * v;
          if (vv < nvec) buf[u][v] = __ldg(src + vv);
        }
      }
    }
  }

  template <typename IdFn>
  HBA_DEVICE void score(const float* __restrict__ qg, int nvec, int rbase, int R, float scale, IdFn id_of,
                        float* sc_s, int* id_s) {
    constexpr int LPS = DH / 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int r = rbase + warp + NWARPS * u;
      if (r < R) {  // warp-uniform
        float best = neg_inf();
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          const int vv = lane + 32 * v;
          float part = 0.f;
          if (vv < nvec) {
            float f[8];
            unpack8(buf[u][v], f);
            const int d0 = (vv * 8) % DH;
#pragma unroll
            for (int j = 0; j < 8; ++j) part = fmaf(f[j], qg[d0 + j], part);
          }
#pragma unroll
          for (int o = 1; o < LPS; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
          if (vv < nvec) best = fmaxf(best, part);
        }
        best = warp_max(best);
        if (lane == 0) {
          sc_s[r] = best * scale;
          id_s[r] = id_of(r);
        }
      }
    }
  }
};

}  // namespace hba
