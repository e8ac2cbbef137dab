// Prefill routed-block selection, flat scan, tiled over queries.
//
// One CTA per (64 consecutive query positions, sequence x kv head).  The
// summary rows of the candidate blocks stream through shared memory in
// stages of 64 blocks (1-D bulk copies, double-buffered), and every staged
// row is used by all 64 queries of the tile -- instead of every query
// re-reading every candidate row from L2 (select_kernel).  Each of the 512
// threads scores 4 queries x 2 blocks per stage.
//
// Scores are bit-identical to select_kernel / SummaryLoads::score
// (hba_score.cuh): routing query qg = bf16(fp32 sum, in head order, of the
// group's bf16 QKNorm'd heads); per 16-byte vector of a slot an 8-term fma
// chain from 0; the vectors of a slot added in the pairwise tree ((v0+v1) +
// (v2+v3)) + ...; max over slots; times the union scale.  Candidates: blocks
// 1 .. bmax(i), bmax(i) = min((i - W + 1)/Bk - 1, nb - 1) (reference
// src/hba/attention.py:250-256, :694-698).  Each warp keeps, for 4 of the
// tile's queries, the best 32 (score desc, block asc) in shared memory
// (hba_warpsort.cuh) and writes the top k as the query's single list.
#include <climits>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_score.cuh"
#include "hba_sm100.cuh"
#include "hba_warpsort.cuh"

namespace hba {

using namespace sm100;

constexpr int kTsQ = 64;          // queries per CTA
constexpr int kTsB = 64;          // summary blocks per stage
constexpr int kTsThreads = 512;
constexpr int kTsWarps = kTsThreads / 32;
constexpr int kTsQpw = kTsQ / kTsWarps;  // queries per warp in the prologue and the top-k
constexpr int kTsStageBytes = 65536;  // kTsB rows of m * dh bf16 (m * dh <= 512)

template <int DH>
struct TsSmem {
  alignas(1024) unsigned char stage[2][kTsStageBytes];
  // bf16 routing queries: 16-byte chunk c (elements 8c .. 8c+7) of row r at c ^ ((r >> 2) & 7); one
  // 128-bit load per query vector (a 128-bit shared load costs a wavefront per quarter-warp)
  alignas(16) uint4 qg[kTsQ][DH / 8];
  float sc[kTsQ][kTsB + 1];
  float ls[kTsQ][32];  // per-query running best 32 (score desc, block asc)
  int li[kTsQ][32];
  uint64_t full[2];
};

template <int DH>
__global__ void __launch_bounds__(kTsThreads, 1) select_tile_kernel(SelParams p, int* err) {
  using SM = TsSmem<DH>;
  constexpr int VPR = DH / 8;  // 16-byte vectors per slot
  constexpr int PER = DH / 32;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  SM& sm = *reinterpret_cast<SM*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ntile = gridDim.x;
  const int tile = ntile - 1 - blockIdx.x;  // the longest (latest) tiles first
  const int bg = blockIdx.y;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const int i0 = tile * kTsQ;
  const int nq = geo.nq;
  const int m = geo.m;
  const int row_elems = m * DH;
  const int row_bytes = row_elems * 2;
  const float scale = p.qp.scale_fixed;
  const int nctx = p.qp.n_fixed;
  const int nb = nctx / geo.Bk;
  auto bmax_of = [&](int i) { return i < nq ? min(last_candidate(i, geo.W, geo.Bk), nb - 1) : 0; };
  const int bmax_tile = bmax_of(min(i0 + kTsQ, nq) - 1);  // grows with i: the tile's largest
  const int nstage = bmax_tile >= 1 ? (bmax_tile + kTsB - 1) / kTsB : 0;
  const __nv_bfloat16* summ_bg = p.summ + (size_t)bg * geo.nb_cap * row_elems;

  // ---- stage copies issued first, so they overlap the query prologue ----
  auto issue = [&](int s) {
    const int lo = 1 + s * kTsB, hi = min(lo + kTsB, bmax_tile + 1);
    const uint32_t bytes = (uint32_t)((hi - lo) * row_bytes);
    mbar_arrive_expect_tx(&sm.full[s & 1], bytes);
    bulk_load(sm.stage[s & 1], summ_bg + (size_t)lo * row_elems, bytes, &sm.full[s & 1]);
  };
  if (tid == 0) {
    mbar_init(&sm.full[0], 1);
    mbar_init(&sm.full[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    for (int s = 0; s < min(2, nstage); ++s) issue(s);
  }

  // ---- routing queries of the tile (warp w: queries kTsQpw*w ..) ----
  for (int r = warp * kTsQpw; r < warp * kTsQpw + kTsQpw; ++r) {
    const int i = i0 + r;
    float acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.f;
    if (i < nq) {
      for (int h = 0; h < geo.G; ++h) {
        const int hq = g * geo.G + h;
        float v[PER];
        load_head_row<DH>(p.q + (((size_t)b * nq + i) * geo.Hq + hq) * DH, v);
        if (geo.qknorm && !p.q_normed) qknorm_lane<DH>(v, p.q_gain[hq], geo.eps);
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] += v[e];
      }
    }
    // lane holds elements lane*PER .. +PER of the row: qg = bf16(sum)
    const int d0 = lane * PER;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(&sm.qg[r][(d0 / 8) ^ ((r >> 2) & 7)]) + (d0 % 8);
#pragma unroll
    for (int e = 0; e < PER; ++e) dst[e] = __float2bfloat16_rn(acc[e]);
  }
  __syncthreads();

  // ---- per-query running lists (shared memory): warp w owns queries kTsQpw*w .. ----
#pragma unroll
  for (int u = 0; u < kTsQpw; ++u) {
    sm.ls[warp * kTsQpw + u][lane] = neg_inf();
    sm.li[warp * kTsQpw + u][lane] = INT_MAX;
  }
  const int k = p.list_k;
  const int qgrp = tid & 15, bgrp = tid >> 4;  // this thread's 4 queries x 2 blocks
  const int qsw = qgrp & 7;                    // swizzle of its qg rows (row >> 2 == qgrp)
  bool ok = true;

  for (int s = 0; s < nstage; ++s) {
    const int blo = 1 + s * kTsB;
    const int nblk = min(kTsB, bmax_tile + 1 - blo);
    if (!mbar_wait(&sm.full[s & 1], (s >> 1) & 1, err)) ok = false;
    const unsigned char* st = sm.stage[s & 1];
    float best[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 2; ++j) best[i][j] = neg_inf();
    int jr[2];  // staged row of each of the thread's blocks (clamped; masked below)
#pragma unroll
    for (int j = 0; j < 2; ++j) jr[j] = min(2 * bgrp + j, nblk - 1);
    for (int sl = 0; sl < m; ++sl) {
      float a[4][2], s1[4][2], s2[4][2], s3[4][2];
#pragma unroll 2  // (by 4: 128 registers and a spill)
      for (int v = 0; v < VPR; ++v) {
        uint4 sw[2];
#pragma unroll
        for (int j = 0; j < 2; ++j)
          sw[j] = *reinterpret_cast<const uint4*>(st + (size_t)jr[j] * row_bytes + (sl * VPR + v) * 16);
        float pv[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 qw = sm.qg[4 * qgrp + i][v ^ qsw];
#pragma unroll
          for (int j = 0; j < 2; ++j) pv[i][j] = dot8_bf16(sw[j], qw);  // the 8-term fmaf chain
        }
        // pairwise tree over the slot's vectors, built as they arrive
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if ((v & 1) == 0) {
              a[i][j] = pv[i][j];
            } else {
              const float l1 = a[i][j] + pv[i][j];
              if ((v & 2) == 0) {
                s1[i][j] = l1;
              } else {
                const float l2 = s1[i][j] + l1;
                if ((v & 4) == 0) {
                  s2[i][j] = l2;
                } else {
                  const float l3 = s2[i][j] + l2;
                  if (VPR == 8) {
                    best[i][j] = fmaxf(best[i][j], l3);
                  } else if ((v & 8) == 0) {
                    s3[i][j] = l3;
                  } else {
                    best[i][j] = fmaxf(best[i][j], s3[i][j] + l3);
                  }
                }
              }
            }
          }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = 4 * qgrp + i;
      const int bm = bmax_of(i0 + qi);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int bl = 2 * bgrp + j;
        sm.sc[qi][bl] = (bl < nblk && blo + bl <= bm) ? best[i][j] * scale : neg_inf();
      }
    }
    __syncthreads();  // stage buffer read, scores written
    if (tid == 0 && s + 2 < nstage) issue(s + 2);
    // one rolled copy of the sort network (unrolled copies thrash the instruction cache)
#pragma unroll 1
    for (int u = 0; u < kTsQpw; ++u) {
      const int qi = warp * kTsQpw + u;
      float ls = sm.ls[qi][lane];
      int li = sm.li[qi][lane];
#pragma unroll 1
      for (int h = 0; h < kTsB / 32; ++h) {
        const int bl = 32 * h + lane;
        const float cs = sm.sc[qi][bl];
        const bool valid = cs != neg_inf();
        warp_offer(ls, li, valid ? cs : neg_inf(), valid ? blo + bl : INT_MAX, k);
      }
      sm.ls[qi][lane] = ls;
      sm.li[qi][lane] = li;
    }
    __syncthreads();  // scores consumed
  }
  if (!ok && tid == 0) atomicExch(err, 1);

  // ---- lists out: [bg, query, 1, k] ----
  for (int u = 0; u < kTsQpw; ++u) {
    const int qi = warp * kTsQpw + u, i = i0 + qi;
    if (i < nq && lane < k) {
      const size_t o = ((size_t)bg * nq + i) * k + lane;
      const int id = sm.li[qi][lane];
      p.out_score[o] = id != INT_MAX ? sm.ls[qi][lane] : neg_inf();
      p.out_idx[o] = id != INT_MAX ? id : -1;
    }
  }
}

bool select_tile_supported(const Geom& geo, int dh, const void* summ) {
  return !geo.hier && (dh == 64 || dh == 128) && geo.m * dh <= 512 && geo.K <= 32 &&
         (reinterpret_cast<uintptr_t>(summ) & 15u) == 0;
}

template <int DH>
static cudaError_t launch_tile_t(const SelParams& p, int* err, cudaStream_t st) {
  const size_t smem = sizeof(TsSmem<DH>) + 1024;
  static const cudaError_t attr =
      cudaFuncSetAttribute(select_tile_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (attr != cudaSuccess) return attr;
  const dim3 grid((p.geo.nq + kTsQ - 1) / kTsQ, p.geo.B * p.geo.Hkv);
  select_tile_kernel<DH><<<grid, kTsThreads, smem, st>>>(p, err);
  return cudaGetLastError();
}

cudaError_t launch_select_tile(const SelParams& p, int dh, int* err, cudaStream_t st) {
  return dh == 64 ? launch_tile_t<64>(p, err, st) : launch_tile_t<128>(p, err, st);
}

}  // namespace hba
