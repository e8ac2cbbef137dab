// Prefill union softmax on the 5th-generation tensor cores (tcgen05 + TMEM,
// operands fed by TMA), the full-sequence forward of the HBA path.
//
// One CTA per (sequence, kv head, query tile).  A tile is QT = 128/G
// consecutive queries x the G query heads of the KV group = the 128 rows of
// the UMMA M dimension (row r = query r/G, head r%G).  Its keys are walked in
// 64-key chunks: [sinks (keys 0..63, NoPE) | the tile's RoPE window | the
// union of the blocks its queries selected (NoPE)] -- a routed block is
// computed once for the whole tile and masked per row by a bitmask of the
// queries that selected it (reference semantics: src/hba/attention.py:676-711;
// the reference's fused path builds the same union at 128x128 granularity,
// :438-475).
//
// Roles (192 threads):
//   warps 0-3  one thread per row: QKNorm + RoPE of the tile's queries into
//              128-byte-swizzled shared memory (no separate q pass), then per
//              chunk: S row from TMEM -> mask -> p = exp2(s*scale*log2e - M)
//              -> P row (bf16, swizzled) for the PV MMA; epilogue O/l -> out.
//              M is the row's QKNorm bound of the logits (|s| <=
//              scale*|q|*|k|, |k| = sqrt(dh)*k_gain) when that bound is small
//              enough that no p can flush to zero (kBoundedLog2): no running
//              max, O never rescaled.  Otherwise M is the row's running max,
//              raised lazily: when a chunk's max passes it by more than
//              kRescaleLog2, the warp waits for the previous PV and rescales
//              its rows of O in TMEM (and l) before writing P.
//   warp 4     TMEM allocation; one thread issues tcgen05.mma:
//              S[c%2] = Q K_c^T (M=128, N=64, K=dh), O += P_c V_c (M=128,
//              N=dh, K=64, V as an MN-major operand).
//   warp 5     one thread issues the TMA loads of K_c, V_c (3-stage ring).
// Every mbarrier wait is bounded; a timeout sets *err and drains.
#include <climits>
#include <cudaTypedefs.h>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_sm100.cuh"

namespace hba {

using namespace sm100;

constexpr int kTcThreads = 192;
constexpr int kTcSlots = 6;  // ring of K or V tiles: K(c) = item 2c, V(c) = item 2c + 1
constexpr int kTcKeys = 64;            // keys per chunk
constexpr int kTcMaxBlocks = 2048;     // routed block union capacity (nb <= 2048)
constexpr int kTcMaxChunks = 1 + 20 + kTcMaxBlocks;

enum ChunkType : uint32_t { kSink = 0, kWindow = 1, kRouted = 2 };

template <int DH>
struct TcSmem {
  static constexpr int HALVES = DH / 64;
  static constexpr int QBYTES = HALVES * 128 * 128;     // [128 rows x DH] bf16, swizzled halves
  static constexpr int KBYTES = HALVES * 64 * 128;      // [64 keys x DH]
  alignas(1024) unsigned char qc[QBYTES];
  alignas(1024) unsigned char qr[QBYTES];
  alignas(1024) unsigned char ring[kTcSlots][KBYTES];  // a K tile is free once its S MMA is done
  alignas(1024) unsigned char p[2][128 * 128];          // [128 rows x 64 keys] bf16, swizzled
  uint2 chunks[kTcMaxChunks];                           // (key base | type << 28, query mask)
  uint64_t q_ready, o_full;
  uint64_t full[kTcSlots], empty[kTcSlots];
  uint64_t s_full[2], p_full[2], p_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  int n_chunks;
  int scan[kTcThreads];
};

struct PrefillTcParams {
  Geom geo;
  int n;
  float scale;
  int QT;              // queries per tile
  int tiles;           // tiles per (sequence, kv head)
  const float* k_gain;
  const int32_t* sel;       // [B*Hkv, n, list_stride] final picks (-1 = none)
  int list_stride;
  __nv_bfloat16* out;       // [B, n, Hq, dh]
  float* lse;               // [B, Hq, n] or null
  int* err;
  unsigned long long* trace;  // debug: 16 global-timer stamps for the last tile of (sequence, kv head) < trace_rows
  long long trace_rows;
};

template <int DH>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_kc, const __grid_constant__ CUtensorMap tm_kr,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_qc,
                      const __grid_constant__ CUtensorMap tm_qr, PrefillTcParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // dynamic shared memory is only 16-byte aligned by default: align by hand
  unsigned char* base_ptr =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  TcSmem<DH>& sm = *reinterpret_cast<TcSmem<DH>*>(base_ptr);
  constexpr int HALVES = DH / 64;
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = geo.G, QT = p.QT, n = p.n;
  const int bg = blockIdx.x / p.tiles, tile = blockIdx.x % p.tiles;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const int i0 = tile * QT;
  const int nq = min(QT, n - i0);
  const int nb = n / geo.Bk;
  unsigned long long* trace =
      (p.trace != nullptr && tile == p.tiles - 1 && bg < p.trace_rows) ? p.trace + (size_t)bg * 16 : nullptr;
  auto stamp = [&](int s) {
    if (trace != nullptr) trace[s] = global_ns();
  };
  if (tid == 0) stamp(0);

  // ---- chunk list: sinks, window, routed union (all threads) ----
  uint32_t* mask = reinterpret_cast<uint32_t*>(sm.p[0]);  // [nb] query bitmasks, overlays P before use
  for (int i = tid; i < nb; i += kTcThreads) mask[i] = 0u;
  __syncthreads();
  {
    const int32_t* sel = p.sel + ((size_t)bg * n + i0) * p.list_stride;
    for (int e = tid; e < nq * p.list_stride; e += kTcThreads) {
      const int blk = sel[e];
      if (blk >= 0 && blk < nb) atomicOr(&mask[blk], 1u << (e / p.list_stride));
    }
  }
  __syncthreads();
  const int jlo = max(geo.S, i0 - geo.W + 1);
  const int jhi = i0 + nq - 1;
  const int nw = max(0, jhi - jlo + 1);
  const int nwc = (nw + kTcKeys - 1) / kTcKeys;
  const int nsc = geo.S > 0 ? 1 : 0;
  {
    const int per = (nb + kTcThreads - 1) / kTcThreads;
    const int lo = tid * per, hi = min(nb, lo + per);
    int cnt = 0;
    for (int i = lo; i < hi; ++i) cnt += mask[i] != 0u;
    // exclusive prefix of the per-thread counts: within each warp, then over the warp totals
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int nv = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += nv;
    }
    if (lane == 31) sm.scan[warp] = incl;
    __syncthreads();
    int wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += sm.scan[w];
    if (tid == kTcThreads - 1) sm.n_chunks = nsc + nwc + wbase + incl;
    int o = nsc + nwc + wbase + incl - cnt;
    for (int i = lo; i < hi; ++i)
      if (mask[i] != 0u) sm.chunks[o++] = make_uint2((uint32_t)(i * geo.Bk) | (kRouted << 28), mask[i]);
    if (tid == 0 && nsc) sm.chunks[0] = make_uint2(0u | (kSink << 28), 0u);
    for (int c = tid; c < nwc; c += kTcThreads)
      sm.chunks[nsc + c] = make_uint2((uint32_t)(jlo + c * kTcKeys) | (kWindow << 28), 0u);
  }
  if (tid == 0) {
    mbar_init(&sm.q_ready, 1);  // the query tile's TMA
    mbar_init(&sm.o_full, 1);
    for (int s = 0; s < kTcSlots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 128);
      mbar_init(&sm.p_free[s], 1);
    }
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(&sm.tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int NCH = sm.n_chunks;
  if (tid == 0) stamp(1);
  const uint32_t t_s0 = tmem, t_o = tmem + 128;

  if (warp == 5) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tm_kc);
      prefetch_tmap(&tm_kr);
      prefetch_tmap(&tm_v);
      // the query tile: rows r = query * G + head, QKNorm'd (qc) and RoPE'd (qr) by the pre-pass
      // a box is G heads x QT queries (G * QT <= 128 rows: 126 when G = 7) of 128 bytes, per half
      mbar_arrive_expect_tx(&sm.q_ready, (uint32_t)(2 * HALVES * G * QT * 128));
      for (int h = 0; h < HALVES; ++h) {
        tma_load_4d(sm.qc + h * 16384, &tm_qc, h * 64, g * G, i0, b, &sm.q_ready);
        tma_load_4d(sm.qr + h * 16384, &tm_qr, h * 64, g * G, i0, b, &sm.q_ready);
      }
      for (int it = 0; it < 2 * NCH; ++it) {
        const int st = it % kTcSlots, u = it / kTcSlots;
        if (it >= kTcSlots && !mbar_wait(&sm.empty[st], (u - 1) & 1, p.err)) break;
        const uint2 e = sm.chunks[it >> 1];
        const int kb = (int)(e.x & 0x0FFFFFFFu);
        const uint32_t type = e.x >> 28;
        mbar_arrive_expect_tx(&sm.full[st], TcSmem<DH>::KBYTES);
        const CUtensorMap* m = (it & 1) ? &tm_v : (type == kWindow ? &tm_kr : &tm_kc);
        for (int h = 0; h < HALVES; ++h) tma_load_4d(sm.ring[st] + h * 8192, m, h * 64, g, kb, b, &sm.full[st]);
      }
    }
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(128, kTcKeys, false, false);
      constexpr uint32_t idesc_o = idesc_bf16(128, DH, false, true);
      bool ok = mbar_wait(&sm.q_ready, 0, p.err);
      tc_fence_after();
      auto pv = [&](int c) -> bool {
        const int sb = c & 1, iv = 2 * c + 1, st = iv % kTcSlots;
        if (!mbar_wait(&sm.p_full[sb], (c >> 1) & 1, p.err)) return false;
        if (!mbar_wait(&sm.full[st], (iv / kTcSlots) & 1, p.err)) return false;
        tc_fence_after();
        const uint32_t pa = smem_u32(sm.p[sb]), va = smem_u32(sm.ring[st]);
#pragma unroll
        for (int kk = 0; kk < kTcKeys / 16; ++kk)
          umma_f16(t_o, sdesc_sw128(pa + kk * 32, 16, 1024), sdesc_sw128(va + kk * 2048, 8192, 1024), idesc_o,
                   (c > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&sm.empty[st]);
        umma_commit(&sm.p_free[sb]);
        return true;
      };
      for (int c = 0; ok && c < NCH; ++c) {
        const int sb = c & 1, ik = 2 * c, st = ik % kTcSlots;
        if (!mbar_wait(&sm.full[st], (ik / kTcSlots) & 1, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t type = sm.chunks[c].x >> 28;
        const uint32_t qa = smem_u32(type == kWindow ? sm.qr : sm.qc), ka = smem_u32(sm.ring[st]);
        if (c == 4) stamp(13);
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const int h = kk >> 2, ko = (kk & 3) * 32;
          umma_f16(t_s0 + sb * kTcKeys, sdesc_sw128(qa + h * 16384 + ko, 16, 1024),
                   sdesc_sw128(ka + h * 8192 + ko, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full[sb]);
        umma_commit(&sm.empty[st]);  // the K tile is free once S is done
        if (c >= 1 && !pv(c - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && NCH >= 1) ok = pv(NCH - 1);
      umma_commit(&sm.o_full);
      // drain: every MMA issued above is complete before TMEM can be released
      umma_commit(&sm.drain);
      mbar_wait(&sm.drain, 0, p.err);
    }
  } else {
    // ---------------- softmax / epilogue, one thread per row ----------------
    const int r = tid;
    const int qt = r / G, hh = r % G;
    const int i = i0 + qt;
    const bool row_ok = (r < QT * G) && (qt < nq);
    const int hq = g * G + hh;
    // the query tile arrives by TMA; this row's logit bound from its QKNorm'd values
    float M2 = 0.f;
    bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_ready, 0, p.err));
    if (row_ok) {
      float qn2 = 0.f;
#pragma unroll
      for (int d8 = 0; d8 < DH / 8; ++d8) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(sm.qc + (d8 / 8) * 16384 + sw128_offset(r, (d8 % 8) * 8)), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) qn2 = fmaf(f[e], f[e], qn2);
      }
      const float kmax = sqrtf((float)DH) * p.k_gain[g] * (1.f + 1.f / 64.f);
      M2 = p.scale * sqrtf(qn2) * kmax * kLog2e;
    }
    // the row's reference maximum: its bound (fixed), or a running max that starts empty
    const bool bounded = M2 <= kBoundedLog2;
    float M = bounded ? M2 : neg_inf();
    if (r == 0) stamp(2);
    const float sl2 = p.scale * kLog2e;
    const int win_lo = max(geo.S, i - geo.W + 1);
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float l = 0.f;
    for (int c = 0; ok && c < NCH; ++c) {
      const int sb = c & 1;
      // a failed wait leaves the whole warp together (the TMEM accesses are warp-collective)
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[sb], (c >> 1) & 1, p.err))) {
        ok = false;
        break;
      }
      const int ts0 = (c == 4) ? 3 : ((c == NCH - 8) ? 8 : -1);  // debug trace slots of two chunks
      if (r == 0 && ts0 >= 0) stamp(ts0);
      tc_fence_after();
      float s[kTcKeys];
      tmem_ld32(t_s0 + sb * kTcKeys + lane_off, s);
      tmem_ld32(t_s0 + sb * kTcKeys + 32 + lane_off, s + 32);
      tmem_ld_wait();
      if (r == 0 && ts0 >= 0) stamp(ts0 + 1);
      if (c >= 2 && !__all_sync(0xffffffffu, mbar_wait(&sm.p_free[sb], ((c - 2) >> 1) & 1, p.err))) {
        ok = false;
        break;
      }
      if (r == 0 && ts0 >= 0) stamp(ts0 + 2);
      const uint2 e = sm.chunks[c];
      const int kb = (int)(e.x & 0x0FFFFFFFu);
      const uint32_t type = e.x >> 28;
      // this row's valid columns [cl, ch) of the chunk, worked out once
      int cl = 0, ch = 0;
      if (row_ok) {
        if (type == kRouted) {
          ch = ((e.y >> qt) & 1u) ? kTcKeys : 0;  // a picked block is wholly before i - W + 1
        } else if (type == kSink) {
          ch = min(geo.S, i + 1) - kb;
        } else {
          cl = max(win_lo - kb, 0);
          ch = min(i - kb + 1, kTcKeys);
        }
      }
      if (!__all_sync(0xffffffffu, bounded)) {
        // running max: this row's chunk max over its valid columns
        float mx = neg_inf();
        if (ch > cl) {
#pragma unroll
          for (int col = 0; col < kTcKeys; ++col) mx = fmaxf(mx, (col >= cl && col < ch) ? s[col] : neg_inf());
        }
        const float mn = bounded ? M : fmaxf(M, mx * sl2);
        const bool need = mn > M + kRescaleLog2;  // -inf + 8 = -inf: the first valid value
        if (__any_sync(0xffffffffu, need)) {
          const float al = need ? (M == neg_inf() ? 0.f : ex2_approx(M - mn)) : 1.f;
          if (c >= 1) {
            // O holds PV(0 .. c-1): wait for the last one, rescale the warp's 32 rows
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.p_free[(c - 1) & 1], ((c - 1) >> 1) & 1, p.err))) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int cb = 0; cb < DH / 32; ++cb) {
              float o[32];
              tmem_ld32(t_o + cb * 32 + lane_off, o);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) o[j] *= al;
              tmem_st_row<32>(t_o + cb * 32 + lane_off, o);
            }
          }
          if (need) {
            l *= al;
            M = mn;
          }
        }
      }
      unsigned char* prow = sm.p[sb];
      if (ch <= cl) {  // nothing of this chunk for this row (most rows of a block few queries picked)
#pragma unroll
        for (int c8 = 0; c8 < kTcKeys / 8; ++c8)
          *reinterpret_cast<uint4*>(prow + sw128_offset(r, c8 * 8)) = make_uint4(0u, 0u, 0u, 0u);
      } else {
#pragma unroll
        for (int c8 = 0; c8 < kTcKeys / 8; ++c8) {
          uint32_t w[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float pv2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int col = c8 * 8 + 2 * t + u;
              float pe = ex2_approx(fmaf(s[col], sl2, -M));
              pe = (col >= cl && col < ch) ? pe : 0.f;
              l += pe;
              pv2[u] = pe;
            }
            w[t] = pack_bf16x2(pv2[0], pv2[1]);
          }
          *reinterpret_cast<uint4*>(prow + sw128_offset(r, c8 * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      if (r == 0 && ts0 >= 0) stamp(ts0 + 3);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.p_full[sb]);
      if (r == 0 && ts0 >= 0) stamp(ts0 + 4);
    }
    if (r == 0) stamp(14);
    if (__all_sync(0xffffffffu, ok && mbar_wait(&sm.o_full, 0, p.err))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int cb = 0; cb < DH / 32; ++cb) {
        float o[32];
        tmem_ld32(t_o + cb * 32 + lane_off, o);
        tmem_ld_wait();
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + (((size_t)b * n + i) * geo.Hq + hq) * DH + cb * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(pack_bf16x2(o[q4 * 8 + 0] * inv, o[q4 * 8 + 1] * inv),
                                 pack_bf16x2(o[q4 * 8 + 2] * inv, o[q4 * 8 + 3] * inv),
                                 pack_bf16x2(o[q4 * 8 + 4] * inv, o[q4 * 8 + 5] * inv),
                                 pack_bf16x2(o[q4 * 8 + 6] * inv, o[q4 * 8 + 7] * inv));
        }
      }
      if (row_ok && p.lse != nullptr)
        p.lse[((size_t)b * geo.Hq + hq) * n + i] =
            l > 0.f ? (M + log2f(l)) * 0.6931471805599453f : neg_inf();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tmem, 256);
  if (tid == 0) stamp(15);
}

// ---------------------------------------------------------------- host ----
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// [B, n, H, dh] bf16 as a 4-D map {dh, H, n, B}, box {64, 1, 64, 1}, 128-byte swizzle.
// [B, n, H, dh] bf16 tensor; a box is 64 elements of dh x box_h heads x box_n tokens
static bool make_map(CUtensorMap* m, const void* base, int B, int n, int H, int dh, int box_h = 1, int box_n = 64) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[4] = {(cuuint64_t)dh, (cuuint64_t)H, (cuuint64_t)n, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)dh * 2, (cuuint64_t)H * dh * 2, (cuuint64_t)n * H * dh * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_h, (cuuint32_t)box_n, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  // L2 fills no wider than a head's slice of a token row (dh * 2 bytes)
  const CUtensorMapL2promotion promo = dh * 2 >= 256 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
                                                     : CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool prefill_tc_supported(const Geom& geo, int dh, int n, bool qknorm) {
  const int G = geo.G;
  return qknorm && (dh == 64 || dh == 128) && geo.Bk == kTcKeys && G >= 4 && G <= 16 && (128 / G) * G >= 64 &&
         n / geo.Bk <= kTcMaxBlocks && geo.W <= 1024 && encode_fn() != nullptr;
}

cudaError_t launch_prefill_tc(const Geom& geo, int dh, int n, float scale, const __nv_bfloat16* qc,
                              const __nv_bfloat16* qr, const float* k_gain, const __nv_bfloat16* kc,
                              const __nv_bfloat16* kr, const __nv_bfloat16* v,
                              const int32_t* sel, int list_stride, __nv_bfloat16* out, float* lse, int* err,
                              unsigned long long* trace, long long trace_rows, cudaStream_t st) {
  CUtensorMap m_kc, m_kr, m_v, m_qc, m_qr;
  const int QT = 128 / geo.G;
  if (!make_map(&m_kc, kc, geo.B, n, geo.Hkv, dh) || !make_map(&m_kr, kr, geo.B, n, geo.Hkv, dh) ||
      !make_map(&m_v, v, geo.B, n, geo.Hkv, dh) || !make_map(&m_qc, qc, geo.B, n, geo.Hq, dh, geo.G, QT) ||
      !make_map(&m_qr, qr, geo.B, n, geo.Hq, dh, geo.G, QT))
    return cudaErrorInvalidValue;
  PrefillTcParams p{};
  p.geo = geo;
  p.n = n;
  p.scale = scale;
  p.QT = 128 / geo.G;
  p.tiles = (n + p.QT - 1) / p.QT;
  p.k_gain = k_gain;
  p.sel = sel;
  p.list_stride = list_stride;
  p.out = out;
  p.lse = lse;
  p.err = err;
  p.trace = trace;
  p.trace_rows = trace_rows;
  const long long grid = (long long)geo.B * geo.Hkv * p.tiles;
  if (dh == 64) {
    const size_t smem = sizeof(TcSmem<64>) + 1024;
    static const cudaError_t attr = cudaFuncSetAttribute(prefill_tc_kernel<64>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (attr != cudaSuccess) return attr;
    prefill_tc_kernel<64><<<(unsigned)grid, kTcThreads, smem, st>>>(m_kc, m_kr, m_v, m_qc, m_qr, p);
  } else {
    const size_t smem = sizeof(TcSmem<128>) + 1024;
    static const cudaError_t attr = cudaFuncSetAttribute(prefill_tc_kernel<128>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (attr != cudaSuccess) return attr;
    prefill_tc_kernel<128><<<(unsigned)grid, kTcThreads, smem, st>>>(m_kc, m_kr, m_v, m_qc, m_qr, p);
  }
  return cudaGetLastError();
}

}  // namespace hba
