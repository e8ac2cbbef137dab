// QKNorm (per-head RMS normalisation with a scalar gain) and the KV-cache
// append.  Both are memory-bound elementwise passes: one warp per (row, head),
// 16-byte vector loads, fp32 math.
#include "hba_common.cuh"
#include "hba_internal.h"

namespace hba {

// y = bf16(x / sqrt(max(mean(x^2), eps)) * gain), the order of operations of
// _HeadRMSNorm.forward (reference src/hba/attention.py:90-94).
template <int DH>
HBA_DEVICE void rmsnorm_row(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, float gain,
                            float eps) {
  constexpr int PER = DH / 32;
  const int lane = threadIdx.x & 31;
  float v[PER];
  load_head_row<DH>(x, v);
  qknorm_lane<DH>(v, gain, eps);
  if constexpr (PER == 2) {
    reinterpret_cast<__nv_bfloat162*>(y)[lane] = __floats2bfloat162_rn(v[0], v[1]);
  } else {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    h[0] = __floats2bfloat162_rn(v[0], v[1]);
    h[1] = __floats2bfloat162_rn(v[2], v[3]);
    reinterpret_cast<uint2*>(y)[lane] = u;
  }
}

template <int DH>
__global__ void __launch_bounds__(256) qknorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                     __nv_bfloat16* __restrict__ y,
                                                     const float* __restrict__ gain, int64_t rows, int heads,
                                                     float eps) {
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (w >= rows * heads) return;
  const int h = (int)(w % heads);
  rmsnorm_row<DH>(x + w * DH, y + w * DH, gain[h], eps);
}

// Writes new tokens into the cache: k QKNorm'd (or copied when qknorm is
// off), v copied.  One warp per (batch, token, kv head).
template <int DH>
__global__ void __launch_bounds__(256) append_kernel(Geom geo, int t, const int32_t* __restrict__ pos,
                                                     const __nv_bfloat16* __restrict__ k_new,
                                                     const __nv_bfloat16* __restrict__ v_new,
                                                     const float* __restrict__ k_gain,
                                                     __nv_bfloat16* __restrict__ k_cache,
                                                     __nv_bfloat16* __restrict__ v_cache) {
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int64_t total = (int64_t)geo.B * t * geo.Hkv;
  if (w >= total) return;
  const int g = (int)(w % geo.Hkv);
  const int tau = (int)((w / geo.Hkv) % t);
  const int b = (int)(w / ((int64_t)geo.Hkv * t));
  const int p = pos[b] + tau;
  if (p < 0 || p >= geo.n_cap) return;  // host validated; never write out of the cache
  const __nv_bfloat16* ks = k_new + w * DH;
  const __nv_bfloat16* vs = v_new + w * DH;
  const int64_t dst = (((int64_t)b * geo.n_cap + p) * geo.Hkv + g) * DH;
  const int lane = threadIdx.x & 31;
  if (geo.qknorm) {
    rmsnorm_row<DH>(ks, k_cache + dst, k_gain[g], geo.eps);
  } else {
    for (int d = lane; d < DH / 2; d += 32)
      reinterpret_cast<__nv_bfloat162*>(k_cache + dst)[d] = reinterpret_cast<const __nv_bfloat162*>(ks)[d];
  }
  for (int d = lane; d < DH / 2; d += 32)
    reinterpret_cast<__nv_bfloat162*>(v_cache + dst)[d] = reinterpret_cast<const __nv_bfloat162*>(vs)[d];
}

cudaError_t launch_qknorm(const __nv_bfloat16* x, __nv_bfloat16* y, const float* gain, int64_t rows, int heads,
                          int dh, float eps, cudaStream_t st) {
  const int64_t warps = rows * heads;
  const int64_t blocks = (warps + 7) / 8;
  if (blocks == 0) return cudaSuccess;
  if (dh == 64)
    qknorm_kernel<64><<<(unsigned)blocks, 256, 0, st>>>(x, y, gain, rows, heads, eps);
  else
    qknorm_kernel<128><<<(unsigned)blocks, 256, 0, st>>>(x, y, gain, rows, heads, eps);
  return cudaGetLastError();
}

cudaError_t launch_append(const Geom& geo, int t, const int32_t* pos, const __nv_bfloat16* k_new,
                          const __nv_bfloat16* v_new, const float* k_gain, __nv_bfloat16* k_cache,
                          __nv_bfloat16* v_cache, int dh, cudaStream_t st) {
  const int64_t warps = (int64_t)geo.B * t * geo.Hkv;
  const int64_t blocks = (warps + 7) / 8;
  if (blocks == 0) return cudaSuccess;
  if (dh == 64)
    append_kernel<64><<<(unsigned)blocks, 256, 0, st>>>(geo, t, pos, k_new, v_new, k_gain, k_cache, v_cache);
  else
    append_kernel<128><<<(unsigned)blocks, 256, 0, st>>>(geo, t, pos, k_new, v_new, k_gain, k_cache, v_cache);
  return cudaGetLastError();
}

}  // namespace hba
