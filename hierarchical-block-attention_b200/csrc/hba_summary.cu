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

constexpr int kSumThreads = 128;
constexpr int kBlocksPerCta = 8;

// First/last block completed by appending tokens [p, p+t) (inclusive range,
// empty when lo > hi).
HBA_DEVICE void completed_blocks(int p, int t, int Bk, int& lo, int& hi) {
  lo = (p + 1 + Bk - 1) / Bk - 1;  // block whose last token is the first >= p
  hi = (p + t) / Bk - 1;
}

template <int DH>
__global__ void __launch_bounds__(kSumThreads) summarize_kernel(Geom geo, const __nv_bfloat16* __restrict__ kc,
                                                                const float* __restrict__ probes,
                                                                const float* __restrict__ proj,
                                                                __nv_bfloat16* __restrict__ summ, int blk_begin,
                                                                int blk_end, const int32_t* __restrict__ pos,
                                                                int t, float rsd) {
  extern __shared__ float smem[];
  const int m = geo.m, Bk = geo.Bk;
  float* proj_s = smem;                    // [DH][DH]
  float* probe_s = proj_s + DH * DH;       // [m][DH]
  float* k_s = probe_s + m * DH;           // [Bk][DH+1]
  float* att_s = k_s + Bk * (DH + 1);      // [m][Bk]
  float* pool_s = att_s + m * Bk;          // [m][DH]
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

  for (int e = tid; e < DH * DH; e += kSumThreads) proj_s[e] = proj[(size_t)g * DH * DH + e];
  for (int e = tid; e < m * DH; e += kSumThreads) probe_s[e] = probes[(size_t)g * m * DH + e];

  for (int blk = first; blk <= last; ++blk) {
    __syncthreads();
    // keys of the block -> fp32 smem (row stride DH+1: conflict-free column reads)
    for (int e = tid; e < Bk * (DH / 8); e += kSumThreads) {
      const int row = e / (DH / 8), c8 = e % (DH / 8);
      const size_t off = (((size_t)b * geo.n_cap + (size_t)blk * Bk + row) * geo.Hkv + g) * DH + c8 * 8;
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(kc + off), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) k_s[row * (DH + 1) + c8 * 8 + j] = f[j];
    }
    __syncthreads();
    for (int e = tid; e < m * Bk; e += kSumThreads) {
      const int mi = e / Bk, tok = e % Bk;
      const float* pr = probe_s + mi * DH;
      const float* kr = k_s + tok * (DH + 1);
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < DH; ++d) acc = fmaf(pr[d], kr[d], acc);
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
    for (int e = tid; e < m * DH; e += kSumThreads) {
      const int mi = e / DH, d = e % DH;
      const float* a = att_s + mi * Bk;
      float acc = 0.f;
      for (int tok = 0; tok < Bk; ++tok) acc = fmaf(a[tok], k_s[tok * (DH + 1) + d], acc);
      pool_s[e] = acc;
    }
    __syncthreads();
    __nv_bfloat16* dst = summ + ((((size_t)b * geo.Hkv + g) * geo.nb_cap + blk) * m) * DH;
    for (int e = tid; e < m * DH; e += kSumThreads) {
      const int mi = e / DH, col = e % DH;
      const float* pl = pool_s + mi * DH;
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < DH; ++d) acc = fmaf(pl[d], proj_s[d * DH + col], acc);
      dst[e] = f2bf(acc);
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
  return sizeof(float) * ((size_t)dh * dh + (size_t)m * dh + (size_t)Bk * (dh + 1) + (size_t)m * Bk + (size_t)m * dh);
}

cudaError_t launch_summarize(const Geom& geo, int dh, const __nv_bfloat16* k_cache, const float* probes,
                             const float* proj, __nv_bfloat16* summ, int blk_begin, int blk_end,
                             const int32_t* pos, int t, cudaStream_t st) {
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
                                                         pos, t, rsd);
  } else {
    static const cudaError_t attr128 =
        cudaFuncSetAttribute(summarize_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if ((e = attr128) != cudaSuccess) return e;
    summarize_kernel<128><<<grid, kSumThreads, smem, st>>>(geo, k_cache, probes, proj, summ, blk_begin, blk_end,
                                                          pos, t, rsd);
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
