// Block summaries (SlotSummarizer) and super-summaries (build_super).
//
// summarize: one CTA per (block group, kv head, sequence); the head's probes
// and projection stay in shared memory while the CTA walks its blocks.  Per
// block (reference src/hba/summarizer.py:38-42):
//   att[m][t] = softmax_t(probes[m] . k[t] * dh^-1/2)
//   pooled[m] = sum_t att[m][t] k[t]
//   S[m]      = pooled[m] @ proj           (stored bf16)
// supers: per-slot mean of up to F children (reference attention.py:202-214).
#include "hba_common.cuh"
#include "hba_internal.h"

namespace hba {

constexpr int kSumThreads = 256;
constexpr int kSumRound = 4;       // blocks whose pooled rows are projected together
constexpr int kBlocksPerCta = 16;  // blocks per CTA (the projection is staged once per CTA)

// First/last block completed by appending tokens [p, p+t) (inclusive range,
// empty when lo > hi).
HBA_DEVICE void completed_blocks(int p, int t, int Bk, int& lo, int& hi) {
  lo = (p + 1 + Bk - 1) / Bk - 1;  // block whose last token is the first >= p
  hi = (p + t) / Bk - 1;
}

// Per block, in shared memory: the keys (fp32 rows of DH + 4 floats, so a
// row is 16-byte aligned and 8 lanes' float4 reads of 8 rows hit distinct
// banks), the slot logits, the pooled rows of a round of kSumRound blocks
// (transposed: [DH][rows]).  The projection then runs once per round, each
// thread 2 rows x DH/32 columns (one float2 of pooled values and one vector
// of projection columns per d).  Every sum runs in the same order as the
// reference formula's loops (d, then tokens, then d), in fp32.
template <int DH>
__global__ void __launch_bounds__(kSumThreads, 2) summarize_kernel(Geom geo, const __nv_bfloat16* __restrict__ kc,
                                                                   const float* __restrict__ probes,
                                                                   const float* __restrict__ proj,
                                                                   __nv_bfloat16* __restrict__ summ, int blk_begin,
                                                                   int blk_end, const int32_t* __restrict__ pos,
                                                                   int t, float rsd, int tiled) {
  extern __shared__ __align__(16) float smem[];
  constexpr int KS = DH + 4;
  constexpr int CP = DH / 32;  // projection columns per thread
  const int m = geo.m, Bk = geo.Bk;
  const int R = kSumRound * m;             // pooled rows of a round
  float* proj_s = smem;                    // [DH][DH]
  float* probe_s = proj_s + DH * DH;       // [m][DH]
  float* k_s = probe_s + m * DH;           // [Bk][KS]
  float* att_s = k_s + Bk * KS;            // [m][Bk]
  float* pool_s = att_s + m * Bk;          // [DH][R]
  const int g = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;

  int lo = blk_begin, hi = blk_end - 1;
  if (pos != nullptr) {
    const int p0 = pos[b];
    if (p0 < 0 || p0 >= geo.n_cap) return;  // the append kernel skipped these tokens too
    int clo, chi;
    completed_blocks(p0, t, Bk, clo, chi);
    lo = clo;
    hi = min(chi, geo.nb_cap - 1);
  }
  const int first = lo + blockIdx.x * kBlocksPerCta;
  const int last = min(hi, first + kBlocksPerCta - 1);
  if (first > last) return;

  for (int e = tid; e < DH * DH / 4; e += kSumThreads)
    reinterpret_cast<float4*>(proj_s)[e] = reinterpret_cast<const float4*>(proj + (size_t)g * DH * DH)[e];
  for (int e = tid; e < m * DH; e += kSumThreads) probe_s[e] = probes[(size_t)g * m * DH + e];
  __nv_bfloat16* summ_bg = summ + (((size_t)b * geo.Hkv + g) * geo.nb_cap) * (size_t)m * DH;

  for (int b0 = first; b0 <= last; b0 += kSumRound) {
    const int nr = min(kSumRound, last - b0 + 1);
    for (int jb = 0; jb < nr; ++jb) {
      const int blk = b0 + jb;
      __syncthreads();  // k_s / att_s free (and, first time, proj_s / probe_s written)
      for (int e = tid; e < Bk * (DH / 8); e += kSumThreads) {
        const int row = e / (DH / 8), c8 = e % (DH / 8);
        const size_t off =
            tiled ? tiled_offset<DH>(((size_t)b * geo.Hkv + g) * (size_t)geo.n_cap * DH, blk * Bk + row, c8 * 8)
                  : (((size_t)b * geo.n_cap + (size_t)blk * Bk + row) * geo.Hkv + g) * DH + c8 * 8;
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(kc + off), f);
        float4* dst = reinterpret_cast<float4*>(k_s + row * KS + c8 * 8);
        dst[0] = make_float4(f[0], f[1], f[2], f[3]);
        dst[1] = make_float4(f[4], f[5], f[6], f[7]);
      }
      __syncthreads();
      // att[mi][tok] = probes[mi] . k[tok] * dh^-1/2 (an fma chain over d)
      for (int e = tid; e < m * Bk; e += kSumThreads) {
        const int mi = e / Bk, tok = e % Bk;
        const float4* pr = reinterpret_cast<const float4*>(probe_s + mi * DH);
        const float4* kr = reinterpret_cast<const float4*>(k_s + tok * KS);
        float acc = 0.f;
#pragma unroll 8
        for (int d4 = 0; d4 < DH / 4; ++d4) {
          const float4 a = pr[d4], k4 = kr[d4];
          acc = fmaf(a.x, k4.x, acc);
          acc = fmaf(a.y, k4.y, acc);
          acc = fmaf(a.z, k4.z, acc);
          acc = fmaf(a.w, k4.w, acc);
        }
        att_s[e] = acc * rsd;
      }
      __syncthreads();
      // softmax over the block's tokens, one warp per slot
      for (int mi = tid / 32; mi < m; mi += kSumThreads / 32) {
        const int lane = tid & 31;
        float mx = neg_inf();
        for (int j = lane; j < Bk; j += 32) mx = fmaxf(mx, att_s[mi * Bk + j]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int j = lane; j < Bk; j += 32) {
          const float e = expf(att_s[mi * Bk + j] - mx);
          att_s[mi * Bk + j] = e;
          sum += e;
        }
        sum = warp_sum(sum);
        for (int j = lane; j < Bk; j += 32) att_s[mi * Bk + j] /= sum;
      }
      __syncthreads();
      // pooled[mi][d] = sum_tok att[mi][tok] k[tok][d] -> pool_s[d][jb * m + mi]
      for (int e = tid; e < m * DH; e += kSumThreads) {
        const int mi = e / DH, d = e % DH;
        const float* a = att_s + mi * Bk;
        float acc = 0.f;
        for (int tok = 0; tok < Bk; ++tok) acc = fmaf(a[tok], k_s[tok * KS + d], acc);
        pool_s[d * R + jb * m + mi] = acc;
      }
    }
    __syncthreads();
    // S[row][col] = pooled[row] @ proj, rows = the round's (block, slot) pairs
    const int rows = nr * m;
    const int cg = tid & 31, rg = tid >> 5;
    for (int r0 = 2 * rg; r0 < rows; r0 += 2 * (kSumThreads / 32)) {
      const bool two = r0 + 1 < rows;
      float acc0[CP], acc1[CP];
#pragma unroll
      for (int c = 0; c < CP; ++c) acc0[c] = acc1[c] = 0.f;
#pragma unroll 4
      for (int d = 0; d < DH; ++d) {
        const float p0 = pool_s[d * R + r0], p1 = two ? pool_s[d * R + r0 + 1] : 0.f;
        float w[CP];
        if constexpr (CP == 4) {
          const float4 v = reinterpret_cast<const float4*>(proj_s + d * DH)[cg];
          w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
        } else {
          const float2 v = reinterpret_cast<const float2*>(proj_s + d * DH)[cg];
          w[0] = v.x; w[1] = v.y;
        }
#pragma unroll
        for (int c = 0; c < CP; ++c) {
          acc0[c] = fmaf(p0, w[c], acc0[c]);
          acc1[c] = fmaf(p1, w[c], acc1[c]);
        }
      }
      // row r = block b0 + r / m, slot r % m: rows of consecutive blocks are consecutive in summ
      __nv_bfloat16* d0 = summ_bg + ((size_t)b0 * m + r0) * DH + cg * CP;
#pragma unroll
      for (int c = 0; c < CP; ++c) d0[c] = f2bf(acc0[c]);
      if (two) {
#pragma unroll
        for (int c = 0; c < CP; ++c) d0[DH + c] = f2bf(acc1[c]);
      }
    }
  }
}

// supers[s] = mean of children [sF, min(sF+F, nb)), per slot and dim.
template <int DH>
__global__ void __launch_bounds__(128) supers_kernel(Geom geo, int nb_fixed, const __nv_bfloat16* __restrict__ summ,
                                                     __nv_bfloat16* __restrict__ sup, int s_begin, int s_end,
                                                     const int32_t* __restrict__ pos, int t) {
  const int g = blockIdx.y, b = blockIdx.z, F = geo.F;
  int lo = s_begin, hi = s_end - 1, nb = nb_fixed;
  if (pos != nullptr) {
    const int p0 = pos[b];
    if (p0 < 0 || p0 >= geo.n_cap) return;
    int clo, chi;
    completed_blocks(p0, t, geo.Bk, clo, chi);
    chi = min(chi, geo.nb_cap - 1);
    if (clo > chi) return;
    lo = clo / F;
    hi = chi / F;
    nb = min((p0 + t) / geo.Bk, geo.nb_cap);
  }
  nb = min(nb, geo.nb_cap);
  const int s = lo + blockIdx.x;
  if (s > hi || s >= geo.ns_cap) return;
  const int c0 = s * F, c1 = min(c0 + F, nb);
  if (c1 <= c0) return;
  const float inv_cnt = 1.0f / (float)(c1 - c0);
  const int per = geo.m * DH;
  const __nv_bfloat16* src = summ + (((size_t)b * geo.Hkv + g) * geo.nb_cap) * per;
  __nv_bfloat16* dst = sup + ((((size_t)b * geo.Hkv + g) * geo.ns_cap) + s) * per;
  for (int e = threadIdx.x; e < per; e += blockDim.x) {
    float acc = 0.f;
    for (int c = c0; c < c1; ++c) acc += bf2f(src[(size_t)c * per + e]);
    dst[e] = f2bf(acc * inv_cnt);
  }
}

static size_t summarize_smem(int dh, int m, int Bk) {
  return sizeof(float) * ((size_t)dh * dh + (size_t)m * dh + (size_t)Bk * (dh + 4) + (size_t)m * Bk +
                          (size_t)dh * kSumRound * m);
}

cudaError_t launch_summarize(const Geom& geo, int dh, const __nv_bfloat16* k_cache, const float* probes,
                             const float* proj, __nv_bfloat16* summ, int blk_begin, int blk_end,
                             const int32_t* pos, int t, cudaStream_t st, bool tiled) {
  int nblk = blk_end - blk_begin;
  if (pos != nullptr) nblk = t / geo.Bk + 2;  // upper bound on blocks completed by t tokens
  if (nblk <= 0) return cudaSuccess;
  const size_t smem = summarize_smem(dh, geo.m, geo.Bk);
  dim3 grid((nblk + kBlocksPerCta - 1) / kBlocksPerCta, geo.Hkv, geo.B);
  const float rsd = (float)(1.0 / sqrt((double)dh));
  cudaError_t e;
  if (dh == 64) {
    static const cudaError_t attr64 =
        cudaFuncSetAttribute(summarize_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if ((e = attr64) != cudaSuccess) return e;
    summarize_kernel<64><<<grid, kSumThreads, smem, st>>>(geo, k_cache, probes, proj, summ, blk_begin, blk_end,
                                                         pos, t, rsd, tiled ? 1 : 0);
  } else {
    static const cudaError_t attr128 =
        cudaFuncSetAttribute(summarize_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if ((e = attr128) != cudaSuccess) return e;
    summarize_kernel<128><<<grid, kSumThreads, smem, st>>>(geo, k_cache, probes, proj, summ, blk_begin, blk_end,
                                                          pos, t, rsd, tiled ? 1 : 0);
  }
  return cudaGetLastError();
}

cudaError_t launch_supers(const Geom& geo, int dh, int nb_fixed, const __nv_bfloat16* summ, __nv_bfloat16* supers,
                          int s_begin, int s_end, const int32_t* pos, int t, cudaStream_t st) {
  int ns = s_end - s_begin;
  if (pos != nullptr) ns = (t / geo.Bk + 2) / geo.F + 2;
  if (ns <= 0) return cudaSuccess;
  dim3 grid(ns, geo.Hkv, geo.B);
  if (dh == 64)
    supers_kernel<64><<<grid, 128, 0, st>>>(geo, nb_fixed, summ, supers, s_begin, s_end, pos, t);
  else
    supers_kernel<128><<<grid, 128, 0, st>>>(geo, nb_fixed, summ, supers, s_begin, s_end, pos, t);
  return cudaGetLastError();
}

}  // namespace hba
