// Shared device helpers for the HBA B200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hba_b200.h"

#define HBA_DEVICE __device__ __forceinline__

namespace hba {

constexpr float kLog2e = 1.4426950408889634f;

HBA_DEVICE float neg_inf() { return __int_as_float(0xff800000); }

HBA_DEVICE float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
HBA_DEVICE __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }
HBA_DEVICE float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Element offset of (token t, dim d) of one (sequence, kv head) in the
// chunk-tiled layout [n/64][dh/64][64 tokens x 64 dims]: per 64-token block
// and 64-dim group the 8 KB image a 128-byte-swizzled TMA box leaves in
// shared memory (the 16-byte unit u of row r sits at unit u ^ (r & 7)), so
// one 1-D bulk copy of a block's group lands as a UMMA operand.  head_base =
// the (sequence, head)'s first element; the 8 elements of a 16-byte unit
// (d % 8 == 0 .. 7) stay contiguous.  The KV cache (K, RoPE'd K, V) and the
// prefill's chunk-tiled copies use it.
template <int DH>
HBA_DEVICE size_t tiled_offset(size_t head_base, int t, int d) {
  constexpr int GROUPS = DH / 64;
  const int r = t & 63;
  const int c = d & 63;
  const uint32_t off = (uint32_t)(r * 64 + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7));
  return head_base + ((size_t)(t >> 6) * GROUPS + (d >> 6)) * 4096 + off;
}

// One element of RoPE, y = x*cos + rot*sin (rot = the rot_half partner, sign
// included), with every rounding fixed: rn(rn(x*cos) + rn(rot*sin)), no fused
// multiply-add.  x and rot are bf16 values and every caller rounds y to bf16
// once, so the window operands are bit-reproducible (the test oracle computes
// the same float32 expression).
HBA_DEVICE float rope_elem(float x, float rot, float c, float s) { return __fadd_rn(__fmul_rn(x, c), __fmul_rn(rot, s)); }

// unpack 8 bf16 held in a uint4 into floats (a bf16 is the upper half of
// the fp32 with the same value, so the widening is exact bit placement)
HBA_DEVICE void unpack8(uint4 u, float* f) {
  f[0] = __uint_as_float(u.x << 16);
  f[1] = __uint_as_float(u.x & 0xffff0000u);
  f[2] = __uint_as_float(u.y << 16);
  f[3] = __uint_as_float(u.y & 0xffff0000u);
  f[4] = __uint_as_float(u.z << 16);
  f[5] = __uint_as_float(u.z & 0xffff0000u);
  f[6] = __uint_as_float(u.w << 16);
  f[7] = __uint_as_float(u.w & 0xffff0000u);
}

// Two independent IEEE fp32 fmas in one instruction (sm_100 fma.rn.f32x2):
// (x, y) = (a0 * b0 + x, a1 * b1 + y), each rounded exactly as fmaf.
HBA_DEVICE void fma2(float& x, float& y, float a0, float a1, float b0, float b1) {
  unsigned long long a, b, c, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(x), "f"(y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(d));
}

// The 8-term fma chain from 0 over two 16-byte vectors of 8 bf16 each, in
// element order (element 2k is the low half of word k): the same value as
// unpack8 of both and fmaf(a[e], b[e], acc) for e = 0..7, since sm_100's
// mixed-precision fma.rn.f32.bf16 widens its bf16 operands exactly and
// rounds a * b + c once -- without the widening instructions.
HBA_DEVICE float dot8_bf16(uint4 a, uint4 b) {
  float d;
  asm("{\n"
      " .reg .b16 a0, a1, a2, a3, a4, a5, a6, a7, b0, b1, b2, b3, b4, b5, b6, b7;\n"
      " mov.b32 {a0, a1}, %1;\n mov.b32 {a2, a3}, %2;\n mov.b32 {a4, a5}, %3;\n mov.b32 {a6, a7}, %4;\n"
      " mov.b32 {b0, b1}, %5;\n mov.b32 {b2, b3}, %6;\n mov.b32 {b4, b5}, %7;\n mov.b32 {b6, b7}, %8;\n"
      " mov.b32 %0, 0;\n"
      " fma.rn.f32.bf16 %0, a0, b0, %0;\n fma.rn.f32.bf16 %0, a1, b1, %0;\n"
      " fma.rn.f32.bf16 %0, a2, b2, %0;\n fma.rn.f32.bf16 %0, a3, b3, %0;\n"
      " fma.rn.f32.bf16 %0, a4, b4, %0;\n fma.rn.f32.bf16 %0, a5, b5, %0;\n"
      " fma.rn.f32.bf16 %0, a6, b6, %0;\n fma.rn.f32.bf16 %0, a7, b7, %0;\n"
      "}\n"
      : "=f"(d)
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w));
  return d;
}

HBA_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

HBA_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

HBA_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- cp.async (Ampere-style async copies; 16 bytes, L2-only caching) ----
HBA_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
HBA_DEVICE void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
HBA_DEVICE void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(sz));
}
HBA_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
HBA_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---- bf16 tensor-core MMA, m16n8k16, fp32 accumulate ----
HBA_DEVICE void mma_bf16_16816(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

HBA_DEVICE void ldmatrix_x4_trans(uint32_t* r, const void* smem) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(smem)));
}

// Loads one head row of DH bf16 values, lane l holding elements
// [l*DH/32, (l+1)*DH/32), and optionally QKNorms it in place:
// v = bf16(v / sqrt(max(mean(v^2), eps)) * gain) (reference attention.py:90-94).
// Every kernel that needs q uses this so all of them see identical bits.
template <int DH>
HBA_DEVICE void load_head_row(const __nv_bfloat16* __restrict__ x, float* v) {
  constexpr int PER = DH / 32;
  const int lane = threadIdx.x & 31;
  if constexpr (PER == 2) {
    float2 t = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(x)[lane]);
    v[0] = t.x;
    v[1] = t.y;
  } else {
    uint2 u = reinterpret_cast<const uint2*>(x)[lane];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
}

template <int DH>
HBA_DEVICE void qknorm_lane(float* v, float gain, float eps) {
  constexpr int PER = DH / 32;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float rms = sqrtf(fmaxf(ss / (float)DH, eps));
#pragma unroll
  for (int i = 0; i < PER; ++i) v[i] = round_bf16((v[i] / rms) * gain);
}

// Warp-cooperative running top-k (k <= 32) under the order `beats`: lane l
// holds the l-th best (score, id); empty slots hold (-inf, INT_MAX).
struct WarpTopK {
  float s;
  int i;
  HBA_DEVICE void init() {
    s = neg_inf();
    i = 0x7fffffff;
  }
  // every lane passes the same (xs, xi); caller guarantees it beats entry k-1
  HBA_DEVICE void insert(float xs, int xi) {
    const int lane = threadIdx.x & 31;
    const bool better = beats_(s, i, xs, xi);
    const int at = __popc(__ballot_sync(0xffffffffu, better));
    const float ps = __shfl_up_sync(0xffffffffu, s, 1);
    const int pi = __shfl_up_sync(0xffffffffu, i, 1);
    if (lane == at) {
      s = xs;
      i = xi;
    } else if (lane > at) {
      s = ps;
      i = pi;
    }
  }
  // each lane offers its own candidate; keeps the best k seen so far
  HBA_DEVICE void offer(float cs, int ci, int k) {
    float ts = __shfl_sync(0xffffffffu, s, k - 1);
    int ti = __shfl_sync(0xffffffffu, i, k - 1);
    unsigned m = __ballot_sync(0xffffffffu, beats_(cs, ci, ts, ti));
    while (m) {
      const int src = __ffs(m) - 1;
      m &= m - 1;
      const float xs = __shfl_sync(0xffffffffu, cs, src);
      const int xi = __shfl_sync(0xffffffffu, ci, src);
      ts = __shfl_sync(0xffffffffu, s, k - 1);
      ti = __shfl_sync(0xffffffffu, i, k - 1);
      if (beats_(xs, xi, ts, ti)) insert(xs, xi);
    }
  }
  static HBA_DEVICE bool beats_(float sa, int ia, float sb, int ib) { return (sa > sb) || (sa == sb && ia < ib); }
};

// Programmatic dependent launch: a kernel launched with the PDL attribute may
// start before its predecessor finishes; it must call grid_dep_wait() before
// reading anything the predecessor writes.  Both are no-ops without PDL.
HBA_DEVICE void grid_dep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
HBA_DEVICE void grid_dep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// Total order used for every top-k in this library: higher score first, then
// lower block index.  Matches the oracle's (score desc, index asc) order.
HBA_DEVICE bool beats(float sa, int ia, float sb, int ib) {
  return (sa > sb) || (sa == sb && ia < ib);
}

}  // namespace hba
