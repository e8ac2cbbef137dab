// Prefill union softmax on the 5th-generation tensor cores (tcgen05 + TMEM,
// operands fed by TMA), the full-sequence forward of the HBA path.
//
// One CTA per (sequence, kv head, pair of query tiles).  A tile is QT = 128/G
// consecutive queries x the G query heads of the KV group = the 128 rows of
// the UMMA M dimension (row r = query r/G, head r%G); the CTA's two tiles (T =
// 0, 1: queries [i0, i0+QT) and [i0+QT, i0+2QT)) share one stream of 64-key
// chunks: [sinks (keys 0..63, NoPE) | the pair's RoPE window | the union of
// the blocks their queries selected (NoPE)] -- a routed block is loaded once
// for both tiles and masked per row by a bitmask of the queries that selected
// it; a chunk that no query of a tile needs is skipped for that tile
// (reference semantics: src/hba/attention.py:676-711; the reference's fused
// path builds the same union at 128x128 granularity, :438-475).
//
// Per tile T, TMEM columns [256T, 256T + 256): S [0, 64) fp32, two P buffers
// [64, 96) and [96, 128) (64 bf16 probabilities per row, two per column), O
// [128, 128 + dh) fp32.  With two P buffers a row's softmax of chunk j waits
// only for PV(j - 2) before storing P.
//   S_T = Q_T K_c^T   (M 128, N 64, K dh; A = the swizzled query tile)
//   O_T += P_T V_c    (M 128, N dh, K 64; A = P_T from TMEM, V MN-major)
// While one tile's softmax warps turn S into P, the tensor cores run the other
// tile's MMAs (and the next chunk's S), so the tensor pipe and the two
// softmax groups overlap.
//
// Roles (352 threads):
//   warps 4T .. 4T+3  softmax / epilogue of tile T, one thread per row (TMEM
//              lane): S row -> mask -> p = exp2(s*scale*log2e - M) -> P row
//              (bf16, tcgen05.st) for the PV MMA; epilogue O/l -> out.  M is
//              the row's QKNorm bound of the logits (|s| <= scale*|q|*|k|,
//              |k| = sqrt(dh)*k_gain) when that bound is small enough that no
//              p can flush to zero (kBoundedLog2): no running max, O never
//              rescaled.  Otherwise M is the row's running max, raised lazily:
//              when a chunk's max passes it by more than kRescaleLog2, the warp
//              rescales its rows of O in TMEM (and l) before writing P.
//   warps 8, 10  one thread each issues tile 0's / tile 1's tcgen05.mma
//              (warp 8 also owns the TMEM allocation).
//   warp 9     one thread issues the loads: the query tiles (TMA), then K_c
//              and V_c through a 5-slot ring, each one 1-D bulk copy of a
//              contiguous chunk of the pre-pass's chunk-tiled K / RoPE'd K /
//              V copies (the 128-byte-swizzled image of a [64 keys x 64
//              dims] box per half, so the ring holds UMMA operands as a
//              tiled TMA load would leave them, at the bulk engine's higher
//              per-SM rate).  Window chunks are 64-key aligned (the row masks
//              cut the window's ragged first chunk).
// Every mbarrier wait is bounded; a timeout sets *err and drains.
#include <climits>
#include <cudaTypedefs.h>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_sm100.cuh"

namespace hba {

using namespace sm100;

constexpr int kTcThreads = 352;
// ring of K or V tiles: K(c) = item 2c, V(c) = item 2c + 1 in slot item % 5.
// With an odd slot count, V(c + 2) reuses K(c)'s slot (free once S(c) is
// done) and K(c + 3) reuses V(c)'s (free once PV(c) is done): the load that
// waits for a PV has three chunk periods to land.
constexpr int kTcSlots = 5;
constexpr int kTcKeys = 64;            // keys per chunk
constexpr int kTcMaxRouted = 1024;     // routed union capacity of a tile pair
constexpr int kTcMma = 8;              // MMA warp of tile 0 (and TMEM owner)
constexpr int kTcMma2 = 10;            // MMA warp of tile 1
constexpr int kTcTma = 9;              // TMA warp

enum ChunkType : uint32_t { kSink = 0, kWindow = 1, kRouted = 2 };

template <int DH>
struct TcSmem {
  static constexpr int HALVES = DH / 64;
  static constexpr int QBYTES = HALVES * 128 * 128;     // [128 rows x DH] bf16, swizzled halves
  static constexpr int KBYTES = HALVES * 64 * 128;      // [64 keys x DH]
  alignas(1024) unsigned char qc[2][QBYTES];            // per tile: QKNorm'd queries (NoPE chunks)
  alignas(1024) unsigned char qr[2][QBYTES];            // per tile: the same RoPE'd (window chunks)
  alignas(1024) unsigned char ring[kTcSlots][KBYTES];   // a K tile is free once its S MMAs are done
  // the routed union: block ids and the pair's query masks (bit q: query i0 + q picked it)
  unsigned long long rmask[kTcMaxRouted];
  uint16_t rblk[kTcMaxRouted];
  uint64_t q_ready, drain[2];
  uint64_t full[kTcSlots], empty[kTcSlots];
  uint64_t s_full[2], s_free[2], o_full[2];
  uint64_t p_full[2][2], p_free[2][2];  // [tile][P buffer]
  uint32_t tmem_base;
  int n_chunks;
  int scan[kTcThreads / 32];
};

static_assert(sizeof(TcSmem<128>) + 1024 <= 232448, "prefill tile set exceeds the 227 KB of shared memory");

struct PrefillTcParams {
  Geom geo;            // geo.nq local queries (positions q_off ..) over n keys
  int n;
  int q_off;
  float scale;
  int QT;              // queries per tile
  int pairs;           // tile pairs per (sequence, kv head)
  const float* k_gain;
  const int32_t* sel;       // [B*Hkv, n, list_stride] final picks (-1 = none)
  const __nv_bfloat16* kc;  // chunk-tiled QKNorm'd keys, RoPE'd keys, values (pre-pass)
  const __nv_bfloat16* kr;
  const __nv_bfloat16* v;
  int list_stride;
  __nv_bfloat16* out;       // [B, n, Hq, dh]
  float* lse;               // [B, Hq, n] or null
  int* err;
  unsigned long long* trace;  // debug: 16 global-timer stamps for the last pair of (sequence, kv head) < trace_rows
  long long trace_rows;
};

template <int DH>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_qc, const __grid_constant__ CUtensorMap tm_qr,
                      PrefillTcParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // dynamic shared memory is only 16-byte aligned by default: align by hand
  unsigned char* base_ptr =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  TcSmem<DH>& sm = *reinterpret_cast<TcSmem<DH>*>(base_ptr);
  constexpr int HALVES = DH / 64;
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = geo.G, QT = p.QT, n = p.n;
  const int pair = p.pairs - 1 - (int)(blockIdx.x % p.pairs);  // the latest (longest) pairs first
  const int bg = blockIdx.x / p.pairs;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const int nql = geo.nq;                      // local queries; local query t sits at position q_off + t
  const int li0 = pair * 2 * QT;               // the pair's first local query
  const int i0 = p.q_off + li0;                // ... and its position
  const int nq2 = min(2 * QT, nql - li0);      // queries of the pair
  const int nq0 = min(QT, nq2), nq1 = max(0, nq2 - QT);  // queries of tile 0, tile 1
  auto nqt = [&](int t) { return t == 0 ? nq0 : nq1; };
  const int nb = n / geo.Bk;
  unsigned long long* trace =
      (p.trace != nullptr && pair == p.pairs - 1 && bg < p.trace_rows) ? p.trace + (size_t)bg * 16 : nullptr;
  auto stamp = [&](int s) {
    if (trace != nullptr) trace[s] = global_ns();
  };
  if (tid == 0) stamp(0);

  // ---- barriers, then the query tiles' TMA, which needs no chunk list and
  // lands while the list is built ----
  if (tid == kTcTma * 32) {
    mbar_init(&sm.q_ready, 1);
    mbar_init(&sm.drain[0], 1);
    mbar_init(&sm.drain[1], 1);
    for (int s = 0; s < kTcSlots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 2);  // one commit per MMA issuer
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.s_free[t], 128);
      mbar_init(&sm.o_full[t], 1);
      for (int u = 0; u < 2; ++u) {
        mbar_init(&sm.p_full[t][u], 128);
        mbar_init(&sm.p_free[t][u], 1);
      }
    }
    fence_barrier_init();
    // rows r = query * G + head, QKNorm'd (qc) and RoPE'd (qr) by the pre-pass;
    // a box is G heads x QT queries (G * QT <= 128 rows: 126 when G = 7) of 128 bytes, per half
    const int ntile = nq1 > 0 ? 2 : 1;
    mbar_arrive_expect_tx(&sm.q_ready, (uint32_t)(ntile * 2 * HALVES * G * QT * 128));
    for (int t = 0; t < ntile; ++t)
      for (int h = 0; h < HALVES; ++h) {
        tma_load_4d(sm.qc[t] + h * 16384, &tm_qc, h * 64, g * G, li0 + t * QT, b, &sm.q_ready);
        tma_load_4d(sm.qr[t] + h * 16384, &tm_qr, h * 64, g * G, li0 + t * QT, b, &sm.q_ready);
      }
  }

  // ---- chunk list: sinks, window, routed union (all threads) ----
  // [nb] 64-bit query masks of the pair, overlaying the ring before its first use
  unsigned long long* mask = reinterpret_cast<unsigned long long*>(sm.ring[0]);
  for (int i = tid; i < nb; i += kTcThreads) mask[i] = 0ull;
  __syncthreads();
  {
    const int32_t* sel = p.sel + ((size_t)bg * nql + li0) * p.list_stride;
    for (int e = tid; e < nq2 * p.list_stride; e += kTcThreads) {
      const int blk = sel[e];
      if (blk >= 0 && blk < nb) atomicOr(&mask[blk], 1ull << (e / p.list_stride));
    }
  }
  __syncthreads();
  // the pair's window keys [jlo, jhi], walked in 64-key aligned chunks from jla
  const int jlo = max(geo.S, i0 - geo.W + 1);
  const int jhi = i0 + nq2 - 1;
  const int jla = jlo & ~(kTcKeys - 1);
  const int nwc = jhi >= jlo ? (jhi - jla) / kTcKeys + 1 : 0;
  const int nsc = geo.S > 0 ? 1 : 0;
  const uint32_t qmask_t = QT >= 32 ? 0xffffffffu : ((1u << QT) - 1u);
  {
    const int per = (nb + kTcThreads - 1) / kTcThreads;
    const int lo = tid * per, hi = min(nb, lo + per);
    int cnt = 0;
    for (int i = lo; i < hi; ++i) cnt += mask[i] != 0ull;
    // exclusive prefix of the per-thread counts: within each warp, then over the warp totals
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int nv = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += nv;
    }
    if (lane == 31) sm.scan[warp] = incl;
    __syncthreads();
    int wbase = 0, total_routed = 0;
    for (int w = 0; w < kTcThreads / 32; ++w) {
      if (w < warp) wbase += sm.scan[w];
      total_routed += sm.scan[w];
    }
    // the host admits only 2 * QT * k <= kTcMaxRouted, so the union always fits
    if (tid == 0) sm.n_chunks = nsc + nwc + min(total_routed, kTcMaxRouted);
    int o = wbase + incl - cnt;
    for (int i = lo; i < hi; ++i) {
      const unsigned long long mk = mask[i];
      if (mk != 0ull) {
        if (o < kTcMaxRouted) {
          sm.rblk[o] = (uint16_t)i;
          sm.rmask[o] = mk;
        }
        ++o;
      }
    }
  }
  if (warp == kTcMma) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();  // the chunk list is complete (and the mask overlay dead) from here on
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int NCH = sm.n_chunks;
  if (tid == 0) stamp(1);
  // chunk c: [sinks | window (aligned) | routed union]: first key, type, the
  // query masks of the two tiles (routed) and the tiles that need it
  struct Chunk {
    int kb;
    uint32_t type, m0, m1, need;
  };
  auto chunk = [&](int c) -> Chunk {
    Chunk ch;
    ch.m0 = ch.m1 = 0u;
    if (c < nsc) {
      ch.kb = 0;
      ch.type = kSink;
      ch.need = 1u | (nq1 > 0 ? 2u : 0u);
    } else if (c < nsc + nwc) {
      ch.kb = jla + (c - nsc) * kTcKeys;
      ch.type = kWindow;
      ch.need = 0u;
      // tile t needs it if it meets the tile's window keys [max(S, first - W + 1), last]
      for (int t = 0; t < 2; ++t) {
        if (nqt(t) == 0) continue;
        const int first = i0 + t * QT, last = first + nqt(t) - 1;
        const int lo_t = max(geo.S, first - geo.W + 1);
        if (ch.kb + kTcKeys - 1 >= lo_t && ch.kb <= last) ch.need |= 1u << t;
      }
    } else {
      const int r = c - nsc - nwc;
      const unsigned long long mk = sm.rmask[r];
      ch.kb = (int)sm.rblk[r] * geo.Bk;
      ch.type = kRouted;
      ch.m0 = (uint32_t)mk & qmask_t;
      ch.m1 = (uint32_t)(mk >> QT) & qmask_t;
      ch.need = (ch.m0 != 0u ? 1u : 0u) | (ch.m1 != 0u ? 2u : 0u);
    }
    return ch;
  };
  constexpr int KB = TcSmem<DH>::KBYTES;
  const size_t head_elems = (size_t)n * DH;  // one (sequence, head) of the chunk-tiled copies
  const __nv_bfloat16* kc_bg = p.kc + (size_t)bg * head_elems;
  const __nv_bfloat16* kr_bg = p.kr + (size_t)bg * head_elems;
  const __nv_bfloat16* v_bg = p.v + (size_t)bg * head_elems;

  if (warp == kTcTma) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int it = 0; it < 2 * NCH; ++it) {
        const int st = it % kTcSlots, u = it / kTcSlots;
        if (it >= kTcSlots && !mbar_wait(&sm.empty[st], (u - 1) & 1, p.err)) break;
        const Chunk ck = chunk(it >> 1);
        const __nv_bfloat16* src = (it & 1) ? v_bg : (ck.type == kWindow ? kr_bg : kc_bg);
        mbar_arrive_expect_tx(&sm.full[st], KB);
        bulk_load(sm.ring[st], src + (size_t)(ck.kb / kTcKeys) * (KB / 2), KB, &sm.full[st]);
      }
    }
  } else if (warp == kTcMma || warp == kTcMma2) {
    // ---------------- MMA issuers: one thread per tile ----------------
    // Each tile's S and PV MMAs are issued by its own thread, so a tile whose
    // softmax is ready is never held behind the other tile's issue; a K or V
    // slot is released once both issuers have committed it.  An issuer waits
    // for every item to land, also one its tile skips, before committing it:
    // so neither can commit a slot's next use before the other's arrival
    // for the current one (the empty barriers count two arrivals a phase).
    if (lane == 0) {
      const int t = warp == kTcMma ? 0 : 1;
      constexpr uint32_t idesc_s = idesc_bf16(128, kTcKeys, false, false);
      constexpr uint32_t idesc_o = idesc_bf16(128, DH, false, true);
      const uint32_t tt = tmem + (uint32_t)(t * 256);
      bool ok = mbar_wait(&sm.q_ready, 0, p.err);
      tc_fence_after();
      int ns = 0, np = 0;  // S and PV MMAs this tile has issued
      auto pv = [&](int c) -> bool {
        const int iv = 2 * c + 1, st = iv % kTcSlots;
        if (!mbar_wait(&sm.full[st], (iv / kTcSlots) & 1, p.err)) return false;
        if ((chunk(c).need >> t) & 1u) {
          const int pb = np & 1;  // P buffer of this tile's np-th chunk
          if (!mbar_wait(&sm.p_full[t][pb], (np >> 1) & 1, p.err)) return false;
          tc_fence_after();
          const uint32_t va = smem_u32(sm.ring[st]);
#pragma unroll
          for (int kk = 0; kk < kTcKeys / 16; ++kk)  // K = 16 keys = 8 packed columns of P per MMA
            umma_f16_ts(tt + 128, tt + 64 + pb * 32 + kk * 8, sdesc_sw128(va + kk * 2048, 8192, 1024), idesc_o,
                        (np > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&sm.p_free[t][pb]);
          ++np;
        }
        umma_commit(&sm.empty[st]);  // this issuer is done with the V tile
        return true;
      };
      for (int c = 0; ok && c < NCH; ++c) {
        const int ik = 2 * c, st = ik % kTcSlots;
        const Chunk ck = chunk(c);
        if (!mbar_wait(&sm.full[st], (ik / kTcSlots) & 1, p.err)) {
          ok = false;
          break;
        }
        if ((ck.need >> t) & 1u) {
          // the tile's S buffer is free once its softmax has read the previous S
          if (ns > 0 && !mbar_wait(&sm.s_free[t], (ns - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qa = smem_u32(ck.type == kWindow ? sm.qr[t] : sm.qc[t]);
          const uint32_t ka = smem_u32(sm.ring[st]);
#pragma unroll
          for (int kk = 0; kk < DH / 16; ++kk) {
            const int h = kk >> 2, ko = (kk & 3) * 32;
            umma_f16(tt, sdesc_sw128(qa + h * 16384 + ko, 16, 1024), sdesc_sw128(ka + h * 8192 + ko, 16, 1024),
                     idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&sm.s_full[t]);
          ++ns;
        }
        umma_commit(&sm.empty[st]);  // this issuer is done with the K tile
        if (c >= 1 && !pv(c - 1)) ok = false;
      }
      if (ok && NCH >= 1) ok = pv(NCH - 1);
      umma_commit(&sm.o_full[t]);
      // drain: every MMA this thread issued is complete before TMEM can be released
      umma_commit(&sm.drain[t]);
      mbar_wait(&sm.drain[t], 0, p.err);
    }
  } else {
    // ---------------- softmax / epilogue of tile t, one thread per row ----------------
    const int t = warp >> 2;
    const int r = tid - 128 * t;
    const int qt = r / G, hh = r % G;
    const int i = i0 + t * QT + qt;          // position
    const int li = li0 + t * QT + qt;        // local query
    const bool row_ok = (r < QT * G) && (qt < nqt(t));
    const int hq = g * G + hh;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + (uint32_t)(t * 256), t_p = t_s + 64, t_o = t_s + 128;  // S, P buffer 0, O
    // the query tiles arrive by TMA; this row's logit bound from its QKNorm'd values
    float M2 = 0.f;
    bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_ready, 0, p.err));
    if (row_ok) {
      float qn2 = 0.f;
#pragma unroll
      for (int d8 = 0; d8 < DH / 8; ++d8) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(sm.qc[t] + (d8 / 8) * 16384 + sw128_offset(r, (d8 % 8) * 8)), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) qn2 = fmaf(f[e], f[e], qn2);
      }
      const float kmax = sqrtf((float)DH) * p.k_gain[g] * (1.f + 1.f / 64.f);
      M2 = p.scale * sqrtf(qn2) * kmax * kLog2e;
    }
    // the row's reference maximum: its bound (fixed), or a running max that starts empty
    const bool bounded = M2 <= kBoundedLog2;
    const bool warp_bounded = __all_sync(0xffffffffu, bounded);
    float M = bounded ? M2 : neg_inf();
    if (r == 0 && t == 0) stamp(2);
    const float sl2 = p.scale * kLog2e;
    const int win_lo = max(geo.S, i - geo.W + 1);
    float l = 0.f;
    int j = 0;  // chunks this tile has processed
    for (int c = 0; ok && c < NCH; ++c) {
      const Chunk ck = chunk(c);
      if (!((ck.need >> t) & 1u)) continue;
      // a failed wait leaves the whole warp together (the TMEM accesses are warp-collective)
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], j & 1, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kTcKeys];
      tmem_ld32(t_s + lane_off, s);
      tmem_ld32(t_s + 32 + lane_off, s + 32);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&sm.s_free[t]);  // the next S MMA of this tile may overwrite S
      const int kb = ck.kb;
      const uint32_t type = ck.type;
      // this row's valid columns [cl, ch) of the chunk, worked out once
      int cl = 0, ch = 0;
      if (row_ok) {
        if (type == kRouted) {
          const uint32_t qm = t == 0 ? ck.m0 : ck.m1;
          ch = ((qm >> qt) & 1u) ? kTcKeys : 0;  // a picked block is wholly before i - W + 1
        } else if (type == kSink) {
          ch = min(geo.S, i + 1) - kb;
        } else {
          cl = max(win_lo - kb, 0);
          ch = min(i - kb + 1, kTcKeys);
        }
      }
      if (!warp_bounded) {
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
          if (j >= 1) {
            // O holds PV(0 .. j-1): wait for the last one, rescale the warp's rows
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.p_free[t][(j - 1) & 1], ((j - 1) >> 1) & 1, p.err))) {
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
              for (int q = 0; q < 32; ++q) o[q] *= al;
              tmem_st_row<32>(t_o + cb * 32 + lane_off, o);
            }
          }
          if (need) {
            l *= al;
            M = mn;
          }
        }
      }
      uint32_t pk[kTcKeys / 2];
      if (ch <= cl) {  // nothing of this chunk for this row (most rows of a block few queries picked)
#pragma unroll
        for (int q = 0; q < kTcKeys / 2; ++q) pk[q] = 0u;
      } else {
#pragma unroll
        for (int q = 0; q < kTcKeys / 2; ++q) {
          float pv2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = 2 * q + u;
            float pe = ex2_approx(fmaf(s[col], sl2, -M));
            pe = (col >= cl && col < ch) ? pe : 0.f;
            l += pe;
            pv2[u] = pe;
          }
          pk[q] = pack_bf16x2(pv2[0], pv2[1]);
        }
      }
      // P buffer j & 1 is free once PV(j - 2) of this tile has completed
      const int pb = j & 1;
      if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(&sm.p_free[t][pb], ((j - 2) >> 1) & 1, p.err))) {
        ok = false;
        break;
      }
      tmem_st_u32<32>(t_p + pb * 32 + lane_off, pk);
      tc_fence_before();
      mbar_arrive(&sm.p_full[t][pb]);
      ++j;
    }
    if (r == 0 && t == 0) stamp(14);
    if (__all_sync(0xffffffffu, ok && (j == 0 || mbar_wait(&sm.o_full[t], 0, p.err)))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int cb = 0; cb < DH / 32; ++cb) {
        float o[32];
        if (j > 0) {
          tmem_ld32(t_o + cb * 32 + lane_off, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) o[q] = 0.f;
        }
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + (((size_t)b * nql + li) * geo.Hq + hq) * DH + cb * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(pack_bf16x2(o[q4 * 8 + 0] * inv, o[q4 * 8 + 1] * inv),
                                 pack_bf16x2(o[q4 * 8 + 2] * inv, o[q4 * 8 + 3] * inv),
                                 pack_bf16x2(o[q4 * 8 + 4] * inv, o[q4 * 8 + 5] * inv),
                                 pack_bf16x2(o[q4 * 8 + 6] * inv, o[q4 * 8 + 7] * inv));
        }
      }
      if (row_ok && p.lse != nullptr)
        p.lse[((size_t)b * geo.Hq + hq) * nql + li] = l > 0.f ? (M + log2f(l)) * 0.6931471805599453f : neg_inf();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kTcMma) tmem_dealloc(tmem, 512);
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

// [B, n, H, dh] bf16 tensor as a 4-D map {dh, H, n, B}; a box is 64 elements
// of dh x box_h heads x box_n tokens, 128-byte swizzle (the query tiles).
static bool make_map(CUtensorMap* m, const void* base, int B, int n, int H, int dh, int box_h, int box_n) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[4] = {(cuuint64_t)dh, (cuuint64_t)H, (cuuint64_t)n, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)dh * 2, (cuuint64_t)H * dh * 2, (cuuint64_t)n * H * dh * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_h, (cuuint32_t)box_n, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool prefill_tc_supported(const Geom& geo, int dh, int n, bool qknorm) {
  const int G = geo.G;
  const int QT = 128 / G;
  // the routed union of a tile pair (2 QT queries x k picks) fits the chunk list; its
  // block masks (nb x 8 bytes) fit the K/V ring they overlay while the list is built
  return qknorm && (dh == 64 || dh == 128) && geo.Bk == kTcKeys && G >= 4 && G <= 16 && QT * G >= 64 &&
         2 * QT * geo.K <= kTcMaxRouted && (size_t)(n / geo.Bk) * 8 <= sizeof(TcSmem<64>::ring) &&
         geo.W <= 1024 && encode_fn() != nullptr;
}

cudaError_t launch_prefill_tc(const Geom& geo, int dh, int n, int q_off, float scale, const __nv_bfloat16* qc,
                              const __nv_bfloat16* qr, const float* k_gain, const __nv_bfloat16* kc_sw,
                              const __nv_bfloat16* kr_sw, const __nv_bfloat16* v_sw,
                              const int32_t* sel, int list_stride, __nv_bfloat16* out, float* lse, int* err,
                              unsigned long long* trace, long long trace_rows, cudaStream_t st) {
  CUtensorMap m_qc, m_qr;
  const int QT = 128 / geo.G;
  if (n % kTcKeys != 0 || ((reinterpret_cast<uintptr_t>(kc_sw) | reinterpret_cast<uintptr_t>(kr_sw) |
                            reinterpret_cast<uintptr_t>(v_sw)) & 15u) != 0 ||
      !make_map(&m_qc, qc, geo.B, geo.nq, geo.Hq, dh, geo.G, QT) ||
      !make_map(&m_qr, qr, geo.B, geo.nq, geo.Hq, dh, geo.G, QT))
    return cudaErrorInvalidValue;
  PrefillTcParams p{};
  p.kc = kc_sw;
  p.kr = kr_sw;
  p.v = v_sw;
  p.geo = geo;
  p.n = n;
  p.q_off = q_off;
  p.scale = scale;
  p.QT = 128 / geo.G;
  p.pairs = (geo.nq + 2 * p.QT - 1) / (2 * p.QT);
  p.k_gain = k_gain;
  p.sel = sel;
  p.list_stride = list_stride;
  p.out = out;
  p.lse = lse;
  p.err = err;
  p.trace = trace;
  p.trace_rows = trace_rows;
  const long long grid = (long long)geo.B * geo.Hkv * p.pairs;
  if (dh == 64) {
    const size_t smem = sizeof(TcSmem<64>) + 1024;
    static const cudaError_t attr = cudaFuncSetAttribute(prefill_tc_kernel<64>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (attr != cudaSuccess) return attr;
    prefill_tc_kernel<64><<<(unsigned)grid, kTcThreads, smem, st>>>(m_qc, m_qr, p);
  } else {
    const size_t smem = sizeof(TcSmem<128>) + 1024;
    static const cudaError_t attr = cudaFuncSetAttribute(prefill_tc_kernel<128>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (attr != cudaSuccess) return attr;
    prefill_tc_kernel<128><<<(unsigned)grid, kTcThreads, smem, st>>>(m_qc, m_qr, p);
  }
  return cudaGetLastError();
}

}  // namespace hba
