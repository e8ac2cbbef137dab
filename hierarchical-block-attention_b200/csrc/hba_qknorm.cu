// QKNorm (per-head RMS normalisation with a scalar gain) and the KV-cache
// append.  Both are memory-bound elementwise passes: one warp per (row, head),
// 16-byte vector loads, fp32 math.
#include <cstdint>

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

// RoPE of one head row held in the warp layout of load_head_row (lane l has
// elements [l*DH/32, (l+1)*DH/32)): y = x*cos + rot_half(x)*sin with
// rot_half(x) = (-x[DH/2:], x[:DH/2]) (reference attention.py:35-44).  The
// partner element d +- DH/2 sits in lane l ^ 16.
template <int DH>
HBA_DEVICE void rope_lane(const float* x, float* y, const float* __restrict__ cos_row,
                          const float* __restrict__ sin_row) {
  constexpr int PER = DH / 32;
  const int lane = threadIdx.x & 31;
  const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int d = lane * PER + i;
    const float partner = __shfl_xor_sync(0xffffffffu, x[i], 16);
    y[i] = rope_elem(x[i], sign * partner, cos_row[d], sin_row[d]);
  }
}

template <int DH>
HBA_DEVICE void store_head_row(__nv_bfloat16* __restrict__ y, const float* v) {
  constexpr int PER = DH / 32;
  const int lane = threadIdx.x & 31;
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

// One key head row: kc = QKNorm(k) (or k), kr = bf16(RoPE(kc) at position p).
template <int DH>
HBA_DEVICE void key_row(const __nv_bfloat16* __restrict__ ks, __nv_bfloat16* __restrict__ kc,
                        __nv_bfloat16* __restrict__ kr, float gain, float eps, bool qknorm,
                        const float* __restrict__ cos_row, const float* __restrict__ sin_row) {
  constexpr int PER = DH / 32;
  float v[PER], r[PER];
  load_head_row<DH>(ks, v);
  if (qknorm) qknorm_lane<DH>(v, gain, eps);
  store_head_row<DH>(kc, v);
  rope_lane<DH>(v, r, cos_row, sin_row);
  store_head_row<DH>(kr, r);
}

// A lane's PER consecutive elements (d = lane * PER ...) stored at their
// chunk-tiled positions (contiguous: they sit in one 16-byte group).
template <int DH>
HBA_DEVICE void store_chunked(__nv_bfloat16* __restrict__ y, size_t row_base, int t, const float* v) {
  constexpr int PER = DH / 32;
  const int lane = threadIdx.x & 31;
  __nv_bfloat16* dst = y + tiled_offset<DH>(row_base, t, lane * PER);
  if constexpr (PER == 2) {
    *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(v[0], v[1]);
  } else {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    h[0] = __floats2bfloat162_rn(v[0], v[1]);
    h[1] = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(dst) = u;
  }
}

// Writes new tokens into the cache: k QKNorm'd (or copied when qknorm is
// off) and its RoPE'd copy at the token's position, v copied.  One warp per
// (batch, token, kv head).
template <int DH>
__global__ void __launch_bounds__(256) append_kernel(Geom geo, int t, const int32_t* __restrict__ pos,
                                                     const __nv_bfloat16* __restrict__ k_new,
                                                     const __nv_bfloat16* __restrict__ v_new,
                                                     const float* __restrict__ k_gain, const float* __restrict__ cos,
                                                     const float* __restrict__ sin,
                                                     __nv_bfloat16* __restrict__ k_cache,
                                                     __nv_bfloat16* __restrict__ kr_cache,
                                                     __nv_bfloat16* __restrict__ v_cache) {
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int64_t total = (int64_t)geo.B * t * geo.Hkv;
  if (w >= total) return;
  const int g = (int)(w % geo.Hkv);
  const int tau = (int)((w / geo.Hkv) % t);
  const int b = (int)(w / ((int64_t)geo.Hkv * t));
  const int p = pos[b] + tau;
  if (p < 0 || p >= geo.n_cap) return;  // host validated; never write out of the cache
  // the cache is chunk-tiled per (sequence, kv head): [n_cap/64][dh/64][64 x 64]
  const size_t head_base = ((size_t)b * geo.Hkv + g) * (size_t)geo.n_cap * DH;
  constexpr int PER = DH / 32;
  float x[PER], r[PER], vv[PER];
  load_head_row<DH>(k_new + w * DH, x);
  load_head_row<DH>(v_new + w * DH, vv);
  if (geo.qknorm) qknorm_lane<DH>(x, k_gain[g], geo.eps);
  store_chunked<DH>(k_cache, head_base, p, x);
  rope_lane<DH>(x, r, cos + (size_t)p * DH, sin + (size_t)p * DH);
  store_chunked<DH>(kr_cache, head_base, p, r);
  store_chunked<DH>(v_cache, head_base, p, vv);
}

// kc and kr for every (batch, token, kv head) of a [B, n, Hkv, dh] tensor.
// With kc_sw != nullptr (the tensor-core prefill): kc as above, and kc, its
// RoPE'd copy and v (when given) also in the chunk-tiled layout [B, Hkv,
// n/64, dh/64, 64 x 64] (kr itself is then not written).  A warp handles
// kQkRows consecutive rows and issues all their loads before any math, so
// enough bytes are in flight per SM for this pure streaming pass.
constexpr int kQkRows = 4;

template <int DH>
__global__ void __launch_bounds__(256) qknorm_rope_kernel(Geom geo, int n, const __nv_bfloat16* __restrict__ k,
                                                          const float* __restrict__ k_gain,
                                                          const float* __restrict__ cos,
                                                          const float* __restrict__ sin,
                                                          __nv_bfloat16* __restrict__ kc,
                                                          __nv_bfloat16* __restrict__ kr,
                                                          const __nv_bfloat16* __restrict__ v,
                                                          __nv_bfloat16* __restrict__ kc_sw,
                                                          __nv_bfloat16* __restrict__ kr_sw,
                                                          __nv_bfloat16* __restrict__ v_sw, int pos0) {
  constexpr int PER = DH / 32;
  const int64_t total = (int64_t)geo.B * n * geo.Hkv;
  const int64_t w0 = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * kQkRows;
  if (w0 >= total) return;
  // row w = (b * n + token) * Hkv + head: one division per warp (the host
  // keeps B * n * Hkv below 2^31), then the kQkRows rows by increments
  const int H = geo.Hkv;
  int bt = (int)w0 / H;      // b * n + token of the first row
  int g0 = (int)w0 - bt * H;  // its head
  float x[kQkRows][PER], vv[kQkRows][PER];
#pragma unroll
  for (int r = 0; r < kQkRows; ++r)
    if (w0 + r < total) load_head_row<DH>(k + (w0 + r) * DH, x[r]);
  const bool tiled = kc_sw != nullptr;
  if (tiled && v != nullptr) {
#pragma unroll
    for (int r = 0; r < kQkRows; ++r)
      if (w0 + r < total) load_head_row<DH>(v + (w0 + r) * DH, vv[r]);
  }
  int b_ = bt / n, tok = bt - b_ * n;
#pragma unroll
  for (int r = 0; r < kQkRows; ++r) {
    const int64_t w = w0 + r;
    if (w >= total) break;  // warp-uniform
    if (r > 0 && ++g0 == H) {  // next row: next head, or the next token's head 0
      g0 = 0;
      if (++tok == n) {
        tok = 0;
        ++b_;
      }
    }
    const int g = g0;
    const int p = pos0 + tok;  // the row's position (RoPE tables row)
    float rr[PER];
    if (geo.qknorm) qknorm_lane<DH>(x[r], k_gain[g], geo.eps);
    store_head_row<DH>(kc + w * DH, x[r]);
    rope_lane<DH>(x[r], rr, cos + (size_t)p * DH, sin + (size_t)p * DH);
    if (!tiled) {
      store_head_row<DH>(kr + w * DH, rr);
      continue;
    }
    const size_t row_base = ((size_t)b_ * geo.Hkv + g) * (size_t)n * DH;  // n % 64 == 0, pos0 == 0
    store_chunked<DH>(kc_sw, row_base, p, x[r]);
    store_chunked<DH>(kr_sw, row_base, p, rr);
    if (v != nullptr) store_chunked<DH>(v_sw, row_base, p, vv[r]);
  }
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
                          const __nv_bfloat16* v_new, const float* k_gain, const float* cos, const float* sin,
                          __nv_bfloat16* k_cache, __nv_bfloat16* kr_cache, __nv_bfloat16* v_cache, int dh,
                          cudaStream_t st) {
  const int64_t warps = (int64_t)geo.B * t * geo.Hkv;
  const int64_t blocks = (warps + 7) / 8;
  if (blocks == 0) return cudaSuccess;
  if (dh == 64)
    append_kernel<64><<<(unsigned)blocks, 256, 0, st>>>(geo, t, pos, k_new, v_new, k_gain, cos, sin, k_cache,
                                                         kr_cache, v_cache);
  else
    append_kernel<128><<<(unsigned)blocks, 256, 0, st>>>(geo, t, pos, k_new, v_new, k_gain, cos, sin, k_cache,
                                                          kr_cache, v_cache);
  return cudaGetLastError();
}

cudaError_t launch_qknorm_rope(const Geom& geo, int n, const __nv_bfloat16* k, const float* k_gain,
                               const float* cos, const float* sin, __nv_bfloat16* kc, __nv_bfloat16* kr, int dh,
                               cudaStream_t st, const __nv_bfloat16* v, __nv_bfloat16* kc_sw,
                               __nv_bfloat16* kr_sw, __nv_bfloat16* v_sw, int pos0) {
  const int64_t warps = ((int64_t)geo.B * n * geo.Hkv + kQkRows - 1) / kQkRows;
  const int64_t blocks = (warps + 7) / 8;
  if (blocks == 0) return cudaSuccess;
  if (kc_sw != nullptr && (n % 64 != 0 || pos0 != 0 || kr_sw == nullptr || (v != nullptr && v_sw == nullptr)))
    return cudaErrorInvalidValue;
  if ((int64_t)geo.B * n * geo.Hkv + kQkRows >= (int64_t)INT32_MAX) return cudaErrorInvalidValue;  // 32-bit row math
  if (dh == 64)
    qknorm_rope_kernel<64><<<(unsigned)blocks, 256, 0, st>>>(geo, n, k, k_gain, cos, sin, kc, kr, v, kc_sw, kr_sw,
                                                              v_sw, pos0);
  else
    qknorm_rope_kernel<128><<<(unsigned)blocks, 256, 0, st>>>(geo, n, k, k_gain, cos, sin, kc, kr, v, kc_sw, kr_sw,
                                                               v_sw, pos0);
  return cudaGetLastError();
}

}  // namespace hba
