// sm_100a primitives: mbarriers, TMA tile loads, tcgen05 (TMEM allocation,
// UMMA issue/commit, TMEM loads) and the UMMA shared-memory / instruction
// descriptors.  Inline PTX, no library code.  Every wait is bounded in time:
// after kWaitNs of the global timer it records an error in *err and returns
// false (a legitimate wait in these kernels lasts microseconds).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "hba_common.cuh"

namespace hba {
namespace sm100 {

constexpr unsigned long long kWaitNs = 200ull * 1000 * 1000;  // 200 ms

HBA_DEVICE unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

HBA_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
HBA_DEVICE void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
HBA_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
HBA_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
HBA_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that may suspend the thread until the phase completes or hint_ns
// elapse: a waiting warp sleeps instead of spinning (a spin of mbarrier
// probes keeps the shared-memory pipe busy, which slows the shuffles and
// shared loads of the warps doing the work).
HBA_DEVICE bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Non-blocking test (try_wait may suspend the thread for a while).
HBA_DEVICE bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity; false (and *err set) on timeout.
HBA_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (global_ns() - t0 > kWaitNs) break;
  }
  if (err != nullptr) atomicExch(err, 1);
  return false;
}

// 64-bit words another GPU writes over NVLink: single-copy-atomic relaxed
// system-scope store / load (the load bypasses L1, which peers do not update).
HBA_DEVICE void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
HBA_DEVICE unsigned long long ld_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Limit of a wait on another rank's words: ranks may arrive at a step apart
// by host-side work (a first launch that loads its module, the interpreter),
// so this limit is longer than the in-CTA one; still bounded.
constexpr unsigned long long kPeerWaitNs = 2000ull * 1000 * 1000;  // 2 s

// Bounded wait for N self-validating words p[i * stride] (i < N), loaded
// together and re-polled while any lacks the tag; w[i] = the words.  Once
// *err is set (an earlier wait of this launch expired) it does not wait again.
template <int N>
HBA_DEVICE void wait_tagged_n(const unsigned long long* p, size_t stride, int n, int shift,
                              unsigned long long mask, unsigned long long tag, unsigned long long (&w)[N], int* err) {
  bool all = true;
#pragma unroll
  for (int i = 0; i < N; ++i) w[i] = i < n ? ld_relaxed_sys(p + i * stride) : 0ull;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < n) all = all && ((w[i] >> shift) & mask) == tag;
  if (all) return;
  if (err != nullptr && *reinterpret_cast<volatile int*>(err) != 0) return;
  const unsigned long long t0 = global_ns();
  for (uint32_t k = 1;; ++k) {
    __nanosleep(32);
    all = true;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      if (i < n && ((w[i] >> shift) & mask) != tag) {
        w[i] = ld_relaxed_sys(p + i * stride);
        all = all && ((w[i] >> shift) & mask) == tag;
      }
    }
    if (all) return;
    if ((k & 15) == 0) {
      if (global_ns() - t0 > kPeerWaitNs) break;
      if (err != nullptr && *reinterpret_cast<volatile int*>(err) != 0) return;
    }
  }
  if (err != nullptr) atomicExch(err, 1);
}

// Shared-memory writes by threads must be made visible to the async proxy
// (TMA, tensor cores) before the consumer is signalled.
HBA_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

HBA_DEVICE void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tiled TMA load into shared memory, completion counted on `bar` (bytes).
HBA_DEVICE void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load into shared memory, completion counted on `bar` (bytes).
HBA_DEVICE void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple
// of 16), completion counted on `bar` (bytes).  Never multicast.
HBA_DEVICE void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ---- tcgen05 ----
HBA_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
HBA_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n"); }
HBA_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
HBA_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
HBA_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 in, fp32 accumulate), one CTA.
HBA_DEVICE void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], kind::f16: A (M x K bf16, K-major) read from
// tensor memory -- row i in lane i, two K-consecutive elements per 32-bit column.
HBA_DEVICE void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// One lane of the (converged) warp is elected: true there, false elsewhere.
// Code that runs on the whole warp keeps its operands warp-uniform and
// issues a single-thread instruction (tcgen05.mma, a TMA copy) from the
// elected lane.
HBA_DEVICE bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .b32 r;\n .reg .pred p;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread is complete.
HBA_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (32x32b shape).
HBA_DEVICE void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
HBA_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
// 16 consecutive fp32 columns of this thread's TMEM lane, not waited (tmem_ld_wait).
HBA_DEVICE void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 2^x by the MUFU instruction (ex2.approx.ftz: relative error ~2^-22, far
// below the bf16 rounding of the probabilities it feeds)
HBA_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two fp32 lanes in one 64-bit register pair, and sm_100's packed fp32 ops
// on them (each lane rounded exactly as the scalar fmaf / add).
HBA_DEVICE unsigned long long f2pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
HBA_DEVICE void f2unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
HBA_DEVICE unsigned long long ffma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
HBA_DEVICE unsigned long long fadd2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// N fp32 columns of this thread's TMEM lane (32x32b shape), waited.
template <int N>
HBA_DEVICE void tmem_ld_row(uint32_t taddr, float* v) {
  uint32_t r[N];
  if constexpr (N == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = __uint_as_float(r[i]);
}

// N fp32 columns written to this thread's TMEM lane (32x32b shape), waited:
// the values are in TMEM before the caller's tcgen05 fence + thread sync.
template <int N>
HBA_DEVICE void tmem_st_row(uint32_t taddr, const float* v) {
  static_assert(N == 8 || N == 16 || N == 32, "tmem_st_row: 8, 16 or 32 columns");
  if constexpr (N == 8) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr),
                 "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
                 : "memory");
  } else if constexpr (N == 16) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::
            "r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
        "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
        : "memory");
  } else {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
        "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]),
        "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]),
        "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
  }
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// 32 raw 32-bit columns written to this thread's TMEM lane (32x32b shape), waited.
template <int N>
HBA_DEVICE void tmem_st_u32(uint32_t taddr, const uint32_t* v) {
  static_assert(N == 32, "tmem_st_u32: 32 columns");
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// 16 raw 32-bit columns written to this thread's TMEM lane (32x32b shape),
// not waited: the caller issues tmem_st_wait() before its tcgen05 fence.
HBA_DEVICE void tmem_st16_nowait(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
// 8 raw 32-bit columns written to this thread's TMEM lane, not waited.
HBA_DEVICE void tmem_st8_nowait(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
HBA_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// Maximum of x over the full warp in one instruction (sm_100a redux.sync
// .f32; -inf is the identity, a NaN input is ignored).
HBA_DEVICE float warp_max_f32(float x) {
  float y;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;\n" : "=f"(y) : "f"(x));
  return y;
}

// Softmax reference maxima of the tensor-core kernels, in log2 units.  A
// QKNorm bound m2 <= kBoundedLog2 serves as a fixed maximum for the whole
// union: no logit exceeds it and none lies below -m2, so p = 2^(s - m2) >=
// 2^-120 never flushes to zero.  Above it the kernels keep a running maximum,
// raised (with O and l rescaled) only when a chunk's maximum passes it by
// more than kRescaleLog2, so every p <= 2^kRescaleLog2.
constexpr float kBoundedLog2 = 60.f;
constexpr float kRescaleLog2 = 8.f;

// UMMA instruction descriptor, kind::f16: D fp32, A and B bf16, M x N tile,
// A/B K-major unless the *_mn flag selects MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// UMMA shared-memory descriptor for a 128-byte-swizzled operand whose
// swizzle atoms (8 rows x 128 B) start on 1024-byte boundaries.
// lbo/sbo in bytes: K-major -> sbo = stride between 8-row groups (lbo unused);
// MN-major -> lbo = stride between 64-element MN groups, sbo = stride between
// 8-row K groups.
HBA_DEVICE uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Byte offset of element (row, col) of a [rows x 64] bf16 tile stored with the
// 128-byte swizzle (the layout TMA SWIZZLE_128B writes and UMMA SW128 reads).
HBA_DEVICE uint32_t sw128_offset(int row, int col) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}

}  // namespace sm100
}  // namespace hba
