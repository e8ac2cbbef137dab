// Prefill union softmax on the 5th-generation tensor cores (tcgen05 + TMEM,
// operands fed by TMA and bulk copies), the full-sequence forward of the HBA
// path.
//
// One CTA per (sequence, kv head, pair of query tiles).  A tile is QT = 128/G
// consecutive queries x the G query heads of the KV group = the 128 rows of
// the UMMA M dimension (row r = query r/G, head r%G); the CTA's two tiles (T =
// 0, 1: queries [i0, i0+QT) and [i0+QT, i0+2QT)) share one stream of 128-key
// chunks, each two 64-key halves:
//   [the pair's RoPE window, 64-aligned, two consecutive blocks per chunk |
//    NoPE blocks in pairs: the sink block, then the union of the blocks the
//    pair's queries selected, those both tiles need first, then tile 0's,
//    then tile 1's]
// A routed block is loaded once for both tiles and masked per row by a
// bitmask of the queries that selected it; a chunk that no query of a tile
// needs is skipped for that tile (reference semantics:
// src/hba/attention.py:676-711; the reference's fused path builds the same
// union at 128x128 granularity, :438-475).
//
// Per tile T, TMEM columns [256T, 256T + 256): S [0, 128) fp32, P (128 bf16
// probabilities per row, two per column: keys [64h, 64h + 64) in columns
// [64h, 64h + 32)) written over S, O [128, 128 + dh) fp32.
//   S_T = Q_T K_c^T   (M 128, N 128, K dh; A = the swizzled query tile)
//   O_T += P_T V_c    (M 128, N dh, K 128; A = P_T from TMEM, V MN-major)
// One warp issues all MMAs, per chunk c in the order PV_0(c-1), S_0(c),
// PV_1(c-1), S_1(c): S_t(c) may overwrite P_t(c-1) because tcgen05.mma
// operations of one thread execute in issue order, and the commit of S_t(c)
// also tells tile t's softmax that PV_t(c-1) is complete (so O may be
// rescaled then).  S_0(c) completes half a step before S_1(c), so each tile's
// softmax runs while the tensor cores run the other tile's PV and S.
//
// The query tile holds the RoPE'd queries for the window chunks and is
// reloaded with the QKNorm'd ones before the tile's first NoPE chunk (issued
// once its last window S is complete, so the load overlaps that chunk's
// softmax).
//
// Roles (576 threads):
//   warps 8T .. 8T+7  softmax / epilogue of tile T: row = TMEM lane, warps
//              8T + 4h + q take lane quarter q and the chunk's 64-column half
//              h: S -> mask -> p = exp2(s*scale*log2e - M) -> P (bf16,
//              tcgen05.st) for the PV MMA, in pieces of 16 columns with the
//              next piece's TMEM load in flight; epilogue O/l -> out, each
//              warp its half of O's columns.  M is the row's QKNorm bound of
//              the logits (|s| <= scale*|q|*|k|, |k| = sqrt(dh)*k_gain) when
//              that bound is small enough that no p can flush to zero
//              (kBoundedLog2): no running max, O never rescaled.  Otherwise M
//              is the row's running max, raised lazily: when a chunk's max
//              (over both halves, exchanged through shared memory) passes it
//              by more than kRescaleLog2, the warps rescale their parts of O
//              in TMEM (and l) before writing P.  Two warps per row group
//              keep the MUFU units busy: one warp's exponentials alone are
//              latency-bound.
//   warp 16    one thread issues the loads: the RoPE'd query tiles (TMA),
//              then K_c and V_c through a ring of 128-key slots, each half of
//              a slot one 1-D bulk copy per 64-dim group from the pre-pass's
//              chunk-tiled K / RoPE'd K / V copies (the 128-byte-swizzled
//              image of a [64 keys x 64 dims] box), so the ring holds UMMA
//              operands as a tiled TMA load would leave them, at the bulk
//              engine's higher per-SM rate.
//   warp 17    issues every tcgen05.mma (one elected lane; the loop runs on
//              the whole warp so its operands stay warp-uniform) and the
//              query reloads; it owns the TMEM allocation.
// Every mbarrier wait is bounded; a timeout sets *err and drains.
#include <climits>
#include <cudaTypedefs.h>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_sm100.cuh"

namespace hba {

using namespace sm100;

constexpr int kTcThreads = 576;
constexpr int kTcBlock = 64;           // keys per routed block = per half chunk
constexpr int kTcKeys = 128;           // keys per chunk (UMMA N of S, K of PV)
constexpr int kTcMaxEntries = 1040;    // NoPE list capacity: the sink block + the routed union of a tile pair
constexpr int kTcMaxChunks = 544;      // window chunks (<= 9 for W <= 1024) + NoPE chunks (<= 520)
constexpr int kTcSoftmaxWarps = 16;    // two warps per row group of a tile (one per 64-column half)
constexpr int kTcTma = 16;             // load warp
constexpr int kTcMma = 17;             // MMA warp (and TMEM owner)

enum HalfType : uint32_t { kSink = 0, kWindow = 1, kRouted = 2, kPad = 3 };

template <int DH>
struct TcSmem {
  static constexpr int HALVES = DH / 64;                // 64-dim groups
  static constexpr int QBYTES = HALVES * 128 * 128;     // [128 rows x DH] bf16, swizzled per dim group
  static constexpr int GBYTES = kTcKeys * 128;          // one dim group of a K or V chunk: 128 rows of 128 B
  static constexpr int KT = HALVES * GBYTES;            // [128 keys x DH]
  // K(c) is ring item 2c, V(c) item 2c + 1, slot item % NSLOT: a K slot is
  // free once both tiles' S(c) are done, a V slot once both PV(c) are
  static constexpr int NSLOT = DH == 64 ? 8 : 4;
  alignas(1024) unsigned char q[2][QBYTES];             // per tile: RoPE'd, then QKNorm'd queries
  alignas(1024) unsigned char ring[NSLOT][KT];
  // NoPE blocks: ids and the pair's query masks (bit q: query i0 + q picked it)
  unsigned long long emask[kTcMaxEntries];
  uint16_t eblk[kTcMaxEntries];
  uint64_t q_ready, qn_read[2], qc_ready[2], drain[2];
  uint64_t full[NSLOT], empty[NSLOT];
  uint64_t s_full[2], p_full[2], o_full[2];
  // the two softmax warps of a row group (tile t, lane quarter): chunk maxima
  // exchanged in the running-max mode (by chunk parity), and the row sums
  uint64_t mx_bar[2][4][2], l_bar[2][4];
  float mx_x[2][2][2][128];  // [tile][column half][chunk parity][row]
  float l_x[2][2][128];      // [tile][column half][row]
  uint32_t tmem_base;
  int n_entries;
  int scan[3][kTcThreads / 32];
  alignas(4) uint8_t cneed[kTcMaxChunks];  // per chunk: the tiles (bit t) with a query that needs it
};

static_assert(sizeof(TcSmem<128>) + 1024 <= 232448 && sizeof(TcSmem<64>) + 1024 <= 232448,
              "prefill tile set exceeds the 227 KB of shared memory");

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
  using SM = TcSmem<DH>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // dynamic shared memory is only 16-byte aligned by default: align by hand
  unsigned char* base_ptr =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SM& sm = *reinterpret_cast<SM*>(base_ptr);
  constexpr int HALVES = SM::HALVES;
  constexpr int NSLOT = SM::NSLOT;
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
  const int nb = n / kTcBlock;
  const uint32_t qbox_bytes = (uint32_t)(HALVES * G * QT * 128);  // a tile's query box (G*QT <= 128 rows)
  unsigned long long* trace =
      (p.trace != nullptr && pair == p.pairs - 1 && bg < p.trace_rows) ? p.trace + (size_t)bg * 16 : nullptr;
  auto stamp = [&](int s) {
    if (trace != nullptr) trace[s] = global_ns();
  };
  if (tid == 0) stamp(0);

  // ---- barriers, then the RoPE'd query tiles' TMA, which needs no chunk list
  // and lands while the list is built ----
  if (tid == kTcTma * 32) {
    mbar_init(&sm.q_ready, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.qn_read[t], 256);
      for (int q = 0; q < 4; ++q) {
        mbar_init(&sm.mx_bar[t][q][0], 64);
        mbar_init(&sm.mx_bar[t][q][1], 64);
        mbar_init(&sm.l_bar[t][q], 64);
      }
      mbar_init(&sm.qc_ready[t], 1);
      mbar_init(&sm.drain[t], 1);
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_full[t], 256);
      mbar_init(&sm.o_full[t], 1);
    }
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    fence_barrier_init();
    // rows r = query * G + head, RoPE'd by the pre-pass; a box is G heads x QT
    // queries (G * QT <= 128 rows: 126 when G = 7) of 128 bytes, per dim group
    const int ntile = nq1 > 0 ? 2 : 1;
    mbar_arrive_expect_tx(&sm.q_ready, (uint32_t)ntile * qbox_bytes);
    for (int t = 0; t < ntile; ++t)
      for (int h = 0; h < HALVES; ++h)
        tma_load_4d(sm.q[t] + h * 16384, &tm_qr, h * 64, g * G, li0 + t * QT, b, &sm.q_ready);
  }

  // ---- NoPE list: the sink block, then the routed union by class (all threads) ----
  // [nb] 64-bit query masks of the pair, overlaying the ring before its first use
  unsigned long long* mask = reinterpret_cast<unsigned long long*>(sm.ring[0]);
  for (int i = tid; i < nb; i += kTcThreads) mask[i] = 0ull;
  __syncthreads();
  {
    const int32_t* sel = p.sel + ((size_t)bg * nql + li0) * p.list_stride;
    for (int e = tid; e < nq2 * p.list_stride; e += kTcThreads) {
      const int blk = sel[e];
      if (blk >= 1 && blk < nb) atomicOr(&mask[blk], 1ull << (e / p.list_stride));
    }
  }
  __syncthreads();
  const uint32_t qmask_t = QT >= 32 ? 0xffffffffu : ((1u << QT) - 1u);
  const int nsk = geo.S > 0 ? 1 : 0;  // the sink block heads the NoPE list
  {
    // class of a routed block: 0 = both tiles need it, 1 = tile 0 only, 2 = tile 1 only
    auto cls_of = [&](unsigned long long mk) {
      const bool a = ((uint32_t)mk & qmask_t) != 0u, c = ((uint32_t)(mk >> QT) & qmask_t) != 0u;
      return a && c ? 0 : (a ? 1 : 2);
    };
    const int per = (nb + kTcThreads - 1) / kTcThreads;
    const int lo = tid * per, hi = min(nb, lo + per);
    int cnt[3] = {0, 0, 0};
    for (int i = lo; i < hi; ++i) {
      const unsigned long long mk = mask[i];
      if (mk != 0ull) {
        const int k = cls_of(mk);
        cnt[0] += k == 0;
        cnt[1] += k == 1;
        cnt[2] += k == 2;
      }
    }
    // exclusive prefix of the per-thread counts of each class: within each warp, then over the warp totals
    int incl[3] = {cnt[0], cnt[1], cnt[2]};
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int nv = __shfl_up_sync(0xffffffffu, incl[k], o);
        if (lane >= o) incl[k] += nv;
      }
    }
    if (lane == 31) {
#pragma unroll
      for (int k = 0; k < 3; ++k) sm.scan[k][warp] = incl[k];
    }
    __syncthreads();
    int wbase[3] = {0, 0, 0}, total[3] = {0, 0, 0};
    for (int w = 0; w < kTcThreads / 32; ++w)
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        if (w < warp) wbase[k] += sm.scan[k][w];
        total[k] += sm.scan[k][w];
      }
    // the host admits only 1 + 2 * QT * k <= kTcMaxEntries, so the list always fits
    if (tid == 0) {
      sm.n_entries = min(nsk + total[0] + total[1] + total[2], kTcMaxEntries);
      if (nsk) {
        sm.eblk[0] = 0;
        sm.emask[0] = 0ull;
      }
    }
    int o[3];
    o[0] = nsk + wbase[0] + incl[0] - cnt[0];
    o[1] = nsk + total[0] + wbase[1] + incl[1] - cnt[1];
    o[2] = nsk + total[0] + total[1] + wbase[2] + incl[2] - cnt[2];
    for (int i = lo; i < hi; ++i) {
      const unsigned long long mk = mask[i];
      if (mk != 0ull) {
        const int k = cls_of(mk);
        const int e = k == 0 ? o[0]++ : (k == 1 ? o[1]++ : o[2]++);
        if (e < kTcMaxEntries) {
          sm.eblk[e] = (uint16_t)i;
          sm.emask[e] = mk;
        }
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
  const int NE = sm.n_entries;
  // the pair's window keys [jlo, jhi], in 64-key blocks from jla, two per chunk
  const int jlo = max(geo.S, i0 - geo.W + 1);
  const int jhi = i0 + nq2 - 1;
  const int jla = jlo & ~(kTcBlock - 1);
  const int nwb = jhi >= jlo ? (jhi - jla) / kTcBlock + 1 : 0;
  const int nwc = (nwb + 1) / 2;
  const int NCH = min(nwc + (NE + 1) / 2, kTcMaxChunks);  // the host's limits keep it below the cap
  if (tid == 0) stamp(1);

  // half h of chunk c: its type, first key and the query masks of the two tiles (routed)
  struct Half {
    int kb;
    uint32_t type, m0, m1;
  };
  auto half_of = [&](int c, int h) -> Half {
    Half x;
    x.m0 = x.m1 = 0u;
    if (c < nwc) {
      const int w = 2 * c + h;
      x.kb = jla + w * kTcBlock;
      x.type = w < nwb ? kWindow : kPad;
    } else {
      const int e = 2 * (c - nwc) + h;
      if (e >= NE) {
        x.kb = 0;
        x.type = kPad;
      } else {
        x.kb = (int)sm.eblk[e] * kTcBlock;
        if (nsk && e == 0) {
          x.type = kSink;
        } else {
          const unsigned long long mk = sm.emask[e];
          x.type = kRouted;
          x.m0 = (uint32_t)mk & qmask_t;
          x.m1 = (uint32_t)(mk >> QT) & qmask_t;
        }
      }
    }
    return x;
  };
  // the tiles (bit t) with a query that needs a half / a chunk
  auto half_need = [&](const Half& x) -> uint32_t {
    uint32_t nd = 0u;
    for (int t = 0; t < 2; ++t) {
      if (nqt(t) == 0) continue;
      bool need = false;
      if (x.type == kWindow) {
        const int first = i0 + t * QT, last = first + nqt(t) - 1;
        const int lo_t = max(geo.S, first - geo.W + 1);
        need = x.kb + kTcBlock - 1 >= lo_t && x.kb <= last;
      } else if (x.type == kSink) {
        need = true;
      } else if (x.type == kRouted) {
        need = (t == 0 ? x.m0 : x.m1) != 0u;
      }
      if (need) nd |= 1u << t;
    }
    return nd;
  };
  auto chunk_need = [&](int c) { return half_need(half_of(c, 0)) | half_need(half_of(c, 1)); };
  // once per CTA, so the issuer and the softmax warps skip chunks by one shared-memory byte
  for (int c = tid; c < NCH; c += kTcThreads) sm.cneed[c] = (uint8_t)chunk_need(c);
  __syncthreads();
  const size_t head_elems = (size_t)n * DH;  // one (sequence, head) of the chunk-tiled copies
  const __nv_bfloat16* kc_bg = p.kc + (size_t)bg * head_elems;
  const __nv_bfloat16* kr_bg = p.kr + (size_t)bg * head_elems;
  const __nv_bfloat16* v_bg = p.v + (size_t)bg * head_elems;

  if (warp == kTcTma) {
    // ---------------- load producer ----------------
    if (lane == 0) {
      for (int it = 0; it < 2 * NCH; ++it) {
        const int st = it % NSLOT, u = it / NSLOT;
        if (it >= NSLOT && !mbar_wait(&sm.empty[st], (u - 1) & 1, p.err)) break;
        const int c = it >> 1;
        const __nv_bfloat16* src = (it & 1) ? v_bg : (c < nwc ? kr_bg : kc_bg);
        const Half x0 = half_of(c, 0), x1 = half_of(c, 1);
        // a padding half loads the chunk's other block again (finite values, masked to p = 0)
        const int blk0 = x0.kb / kTcBlock, blk1 = x1.type == kPad ? blk0 : x1.kb / kTcBlock;
        mbar_arrive_expect_tx(&sm.full[st], SM::KT);
#pragma unroll
        for (int dg = 0; dg < HALVES; ++dg) {
          unsigned char* dst = sm.ring[st] + dg * SM::GBYTES;
          bulk_load(dst, src + ((size_t)blk0 * HALVES + dg) * 4096, 8192, &sm.full[st]);
          bulk_load(dst + 8192, src + ((size_t)blk1 * HALVES + dg) * 4096, 8192, &sm.full[st]);
        }
      }
    }
  } else if (warp == kTcMma) {
    // ---------------- MMA issuer: one thread for both tiles ----------------
    // Step c issues, per tile t: the PV of t's pending chunk (once t's
    // softmax has written its P), then S_t(c) if t needs chunk c.  The
    // tensor pipe so runs PV_0, S_0, PV_1, S_1 per chunk: S_0(c) completes
    // half a step before S_1(c), and each tile's softmax overlaps the other
    // tile's MMAs.  K(c) is released after step c (both S(c) issued), V(c)
    // after step c + 1 (both PV(c) issued); an extra step NCH issues the
    // last PVs.  A tile's first NoPE chunk reloads its query tile: the TMA is
    // issued once its last window S is complete, before waiting for that
    // chunk's P, so the load overlaps the softmax.
    // The whole warp runs the loop, so every operand (descriptors, TMEM
    // addresses) is warp-uniform; one elected lane issues each tcgen05 op.
    {
      constexpr uint32_t idesc_s = idesc_bf16(128, kTcKeys, false, false);
      constexpr uint32_t idesc_o = idesc_bf16(128, DH, false, true);
      auto wwait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err));
      };
      bool ok = wwait(&sm.q_ready, 0);
      tc_fence_after();
      int pend[2] = {-1, -1};  // chunk whose PV is still to issue, per tile
      int np[2] = {0, 0}, ns[2] = {0, 0};
      bool nope[2] = {false, false};  // the query tile holds the QKNorm'd queries
      auto wait_item = [&](int it) { return wwait(&sm.full[it % NSLOT], (it / NSLOT) & 1); };
      // the need bits are read four chunks at a time; items a tile has waited for are not tested again
      uint32_t needw = 0u, prev_need = 0u;
      for (int c = 0; ok && c <= NCH; ++c) {
        if ((c & 3) == 0 && c < NCH) needw = *reinterpret_cast<const uint32_t*>(&sm.cneed[c]);
        const uint32_t need = c < NCH ? (needw >> (8 * (c & 3))) & 3u : 0u;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint32_t tt = tmem + (uint32_t)(t * 256);
          const bool s_t = ok && ((need >> t) & 1u);
          const bool reload = s_t && c >= nwc && !nope[t];
          if (reload) {
            // Q is free once the tile's last S is complete and the softmax has read it for its bound
            if ((ns[t] > 0 && !wwait(&sm.s_full[t], (ns[t] - 1) & 1)) || !wwait(&sm.qn_read[t], 0)) {
              ok = false;
              break;
            }
            if (elect_one_sync()) {
              mbar_arrive_expect_tx(&sm.qc_ready[t], qbox_bytes);
              for (int h = 0; h < HALVES; ++h)
                tma_load_4d(sm.q[t] + h * 16384, &tm_qc, h * 64, g * G, li0 + t * QT, b, &sm.qc_ready[t]);
            }
            __syncwarp();
          }
          if (ok && pend[t] >= 0) {
            const int iv = 2 * pend[t] + 1;
            if (!wait_item(iv) || !wwait(&sm.p_full[t], np[t] & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t vdesc = sdesc_sw128(smem_u32(sm.ring[iv % NSLOT]), SM::GBYTES, 1024);
            if (elect_one_sync()) {
#pragma unroll
              // K = 16 keys = 8 packed columns of P per MMA; P of keys [64h, 64h + 64) in columns [64h, 64h + 32)
              for (int kk = 0; kk < kTcKeys / 16; ++kk)
                umma_f16_ts(tt + 128, tt + (kk >> 2) * 64 + (kk & 3) * 8, vdesc + (uint64_t)(kk * 2048 >> 4), idesc_o,
                            (np[t] > 0 || kk > 0) ? 1u : 0u);
            }
            __syncwarp();
            ++np[t];
            pend[t] = -1;
          }
          if (s_t) {
            if (reload) {
              if (!wwait(&sm.qc_ready[t], 0)) {
                ok = false;
                break;
              }
              nope[t] = true;
            }
            if (!wait_item(2 * c)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t qdesc = sdesc_sw128(smem_u32(sm.q[t]), 16, 1024);
            const uint64_t kdesc = sdesc_sw128(smem_u32(sm.ring[(2 * c) % NSLOT]), 16, 1024);
            if (elect_one_sync()) {
#pragma unroll
              for (int kk = 0; kk < DH / 16; ++kk) {
                const int h = kk >> 2, ko = (kk & 3) * 32;
                umma_f16(tt, qdesc + (uint64_t)((h * 16384 + ko) >> 4), kdesc + (uint64_t)((h * SM::GBYTES + ko) >> 4),
                         idesc_s, kk > 0 ? 1u : 0u);
              }
              umma_commit(&sm.s_full[t]);
            }
            __syncwarp();
            ++ns[t];
            pend[t] = c;
          }
        }
        if (!ok) break;
        // release K(c) and V(c - 1) once landed (a tile that used one has waited for it)
        if (c < NCH) {
          if (need == 0u && !wait_item(2 * c)) break;
          if (elect_one_sync()) umma_commit(&sm.empty[(2 * c) % NSLOT]);
          __syncwarp();
        }
        if (c >= 1) {
          if (prev_need == 0u && !wait_item(2 * c - 1)) break;
          if (elect_one_sync()) umma_commit(&sm.empty[(2 * c - 1) % NSLOT]);
          __syncwarp();
        }
        prev_need = need;
      }
      if (elect_one_sync()) {
        umma_commit(&sm.o_full[0]);
        umma_commit(&sm.o_full[1]);
        // drain: every MMA is complete before TMEM can be released
        umma_commit(&sm.drain[0]);
      }
      __syncwarp();
      wwait(&sm.drain[0], 0);
    }
  } else if (warp < kTcSoftmaxWarps) {
    // ---------------- softmax / epilogue: tile t, row = TMEM lane, one 64-column half ----------------
    // Two warps share each row group (the same TMEM lane quarter): warp
    // half hc turns S columns [64hc, 64hc + 64) (the chunk's half hc) into P
    // columns [64hc, 64hc + 32), which only it has read, and owns O columns
    // [hc dh/2, (hc + 1) dh/2) in the epilogue.  The row's maximum (running-max
    // mode) and its sum are combined through shared memory and an mbarrier of
    // the pair (bounded waits, like every other).
    const int t = warp >> 3;
    const int hc = (warp >> 2) & 1;
    const int lq = warp & 3;
    const int r = lq * 32 + lane;
    const int qt = r / G, hh = r % G;
    const int i = i0 + t * QT + qt;          // position
    const int li = li0 + t * QT + qt;        // local query
    const bool row_ok = (r < QT * G) && (qt < nqt(t));
    const int hq = g * G + hh;
    const uint32_t lane_off = (uint32_t)(lq * 32) << 16;
    const uint32_t t_s = tmem + (uint32_t)(t * 256), t_o = t_s + 128;  // S (P in its columns [0,32) and [64,96)), O
    // the query tiles arrive by TMA; this row's logit bound from its (RoPE'd:
    // a rotation, same norm up to rounding) values
    float M2 = 0.f;
    bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_ready, 0, p.err));
    if (row_ok) {
      float qn2 = 0.f;
#pragma unroll
      for (int d8 = 0; d8 < DH / 8; ++d8) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(sm.q[t] + (d8 / 8) * 16384 + sw128_offset(r, (d8 % 8) * 8)), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) qn2 = fmaf(f[e], f[e], qn2);
      }
      // without QKNorm no bound: the running maximum from the first chunk
      M2 = geo.qknorm ? p.scale * sqrtf(qn2) * (sqrtf((float)DH) * p.k_gain[g] * (1.f + 1.f / 64.f)) * kLog2e
                      : __int_as_float(0x7f800000);
    }
    mbar_arrive(&sm.qn_read[t]);  // the tile may be reloaded from here on
    // the row's reference maximum: its bound (fixed), or a running max that starts empty
    const bool bounded = M2 <= kBoundedLog2;
    const bool warp_bounded = __all_sync(0xffffffffu, bounded);  // the same in both warps of the pair
    float M = bounded ? M2 : neg_inf();
    if (r == 0 && t == 0 && hc == 0) stamp(2);
    const float sl2 = p.scale * kLog2e;
    const int win_lo = max(geo.S, i - geo.W + 1);
    // this row's valid columns [lo, hi) of a half (hi <= lo: none)
    auto row_range = [&](const Half& x, int& lo, int& hi) {
      lo = 0;
      hi = 0;
      if (!row_ok) return;
      if (x.type == kWindow) {
        lo = max(win_lo - x.kb, 0);
        hi = min(i - x.kb + 1, kTcBlock);
      } else if (x.type == kSink) {
        hi = min(geo.S, i + 1);
      } else if (x.type == kRouted) {
        hi = ((((t == 0 ? x.m0 : x.m1)) >> qt) & 1u) ? kTcBlock : 0;  // a picked block is wholly before i - W + 1
      }
    };
    // this thread's sum of p over even and odd columns, one packed pair (sm_100's
    // paired fp32 fma / add keep the instructions around the exponentials few)
    unsigned long long lsum = f2pack(0.f, 0.f);
    // P of piece pc of this half (16 columns of S) -> TMEM columns [64hc + 8pc, +8); valid columns [lo, hi)
    auto piece = [&](const float* s, int pc, int lo, int hi) {
      uint32_t pk[8];
      const unsigned long long sl2x2 = f2pack(sl2, sl2), nm2 = f2pack(-M, -M);
      if (hi - lo == 16) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float x0, x1;
          f2unpack(ffma2(f2pack(s[2 * q], s[2 * q + 1]), sl2x2, nm2), x0, x1);
          const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
          lsum = fadd2(lsum, f2pack(p0, p1));
          pk[q] = pack_bf16x2(p0, p1);
        }
      } else if (hi > lo) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float x0, x1;
          f2unpack(ffma2(f2pack(s[2 * q], s[2 * q + 1]), sl2x2, nm2), x0, x1);
          float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
          p0 = (2 * q >= lo && 2 * q < hi) ? p0 : 0.f;
          p1 = (2 * q + 1 >= lo && 2 * q + 1 < hi) ? p1 : 0.f;
          lsum = fadd2(lsum, f2pack(p0, p1));
          pk[q] = pack_bf16x2(p0, p1);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) pk[q] = 0u;
      }
      tmem_st8_nowait(t_s + (uint32_t)(64 * hc + 8 * pc) + lane_off, pk);
    };
    int j = 0;  // chunks this tile has processed
    uint32_t needw = 0u;
    for (int c = 0; ok && c < NCH; ++c) {
      if ((c & 3) == 0) needw = *reinterpret_cast<const uint32_t*>(&sm.cneed[c]);
      if (!((needw >> (8 * (c & 3) + t)) & 1u)) continue;
      const Half x = half_of(c, hc);
      // a failed wait leaves the whole warp together (the TMEM accesses are warp-collective)
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], j & 1, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      int lo, hi;
      row_range(x, lo, hi);
      if (!warp_bounded) {
        // running max: the chunk max of the row's valid columns of this half, then of both halves
        float mx = neg_inf();
        if (__any_sync(0xffffffffu, hi > lo)) {
          float s[kTcBlock];
          tmem_ld32(t_s + hc * 64 + lane_off, s);
          tmem_ld32(t_s + hc * 64 + 32 + lane_off, s + 32);
          tmem_ld_wait();
#pragma unroll
          for (int col = 0; col < kTcBlock; ++col) mx = fmaxf(mx, (col >= lo && col < hi) ? s[col] : neg_inf());
        }
        sm.mx_x[t][hc][j & 1][r] = mx;
        mbar_arrive(&sm.mx_bar[t][lq][j & 1]);
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.mx_bar[t][lq][j & 1], (j >> 1) & 1, p.err))) {
          ok = false;
          break;
        }
        mx = fmaxf(sm.mx_x[t][0][j & 1][r], sm.mx_x[t][1][j & 1][r]);
        const float mn = bounded ? M : fmaxf(M, mx * sl2);
        const bool need = mn > M + kRescaleLog2;  // -inf + 8 = -inf: the first valid value
        if (__any_sync(0xffffffffu, need)) {
          const float al = need ? (M == neg_inf() ? 0.f : ex2_approx(M - mn)) : 1.f;
          if (j >= 1) {
            // O holds PV(0 .. j-1), complete: S(j) was issued after PV(j-1); this warp's half of O
#pragma unroll
            for (int cb = 0; cb < DH / 64; ++cb) {
              const uint32_t oc = t_o + (uint32_t)(hc * (DH / 2) + cb * 32) + lane_off;
              float o[32];
              tmem_ld32(oc, o);
              tmem_ld_wait();
#pragma unroll
              for (int q = 0; q < 32; ++q) o[q] *= al;
              tmem_st_row<32>(oc, o);
            }
          }
          if (need) {
            lsum = ffma2(lsum, f2pack(al, al), f2pack(0.f, 0.f));
            M = mn;
          }
        }
      }
      // four pieces of 16 columns, the next one's TMEM load in flight while one is turned into P
      {
        const uint32_t sc = t_s + (uint32_t)(hc * 64) + lane_off;
        float sa[16], sb[16];
        tmem_ld16(sc, sa);
        tmem_ld_wait();
        tmem_ld16(sc + 16, sb);
        piece(sa, 0, lo, min(hi, 16));
        tmem_ld_wait();
        tmem_ld16(sc + 32, sa);
        piece(sb, 1, max(lo - 16, 0), min(hi, 32) - 16);
        tmem_ld_wait();
        tmem_ld16(sc + 48, sb);
        piece(sa, 2, max(lo - 32, 0), min(hi, 48) - 32);
        tmem_ld_wait();
        piece(sb, 3, max(lo - 48, 0), hi - 48);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sm.p_full[t]);
      ++j;
    }
    if (r == 0 && t == 0 && hc == 0) stamp(14);
    // the row's sum over both halves (in the same order in both warps)
    {
      float a0, a1;
      f2unpack(lsum, a0, a1);
      sm.l_x[t][hc][r] = a0 + a1;
      mbar_arrive(&sm.l_bar[t][lq]);
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.l_bar[t][lq], 0, p.err)) && ok;
    }
    const float l = sm.l_x[t][0][r] + sm.l_x[t][1][r];
    if (__all_sync(0xffffffffu, ok && (j == 0 || mbar_wait(&sm.o_full[t], 0, p.err)))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int cb = 0; cb < DH / 64; ++cb) {
        const int col0 = hc * (DH / 2) + cb * 32;
        float o[32];
        if (j > 0) {
          tmem_ld32(t_o + (uint32_t)col0 + lane_off, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) o[q] = 0.f;
        }
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + (((size_t)b * nql + li) * geo.Hq + hq) * DH + col0);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(pack_bf16x2(o[q4 * 8 + 0] * inv, o[q4 * 8 + 1] * inv),
                                 pack_bf16x2(o[q4 * 8 + 2] * inv, o[q4 * 8 + 3] * inv),
                                 pack_bf16x2(o[q4 * 8 + 4] * inv, o[q4 * 8 + 5] * inv),
                                 pack_bf16x2(o[q4 * 8 + 6] * inv, o[q4 * 8 + 7] * inv));
        }
      }
      if (row_ok && hc == 0 && p.lse != nullptr)
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
// of dh x box_h heads x box_n tokens, 128-byte swizzle (the query tiles; the
// backward's query and output-gradient tiles too).
bool make_map(CUtensorMap* m, const void* base, int B, int n, int H, int dh, int box_h, int box_n) {
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
  // the sink block and the routed union of a tile pair (2 QT queries x k picks) fit the
  // NoPE list; its block masks (nb x 8 bytes) fit the K/V ring they overlay while the list is built
  (void)qknorm;  // without QKNorm the softmax keeps a running maximum
  return (dh == 64 || dh == 128) && geo.Bk == kTcBlock && G >= 4 && G <= 16 && QT * G >= 64 &&
         1 + 2 * QT * geo.K <= kTcMaxEntries && (size_t)(n / geo.Bk) * 8 <= sizeof(TcSmem<64>::ring) &&
         (size_t)(n / geo.Bk) * 8 <= sizeof(TcSmem<128>::ring) && geo.W <= 1024 && encode_fn() != nullptr;
}

cudaError_t launch_prefill_tc(const Geom& geo, int dh, int n, int q_off, float scale, const __nv_bfloat16* qc,
                              const __nv_bfloat16* qr, const float* k_gain, const __nv_bfloat16* kc_sw,
                              const __nv_bfloat16* kr_sw, const __nv_bfloat16* v_sw,
                              const int32_t* sel, int list_stride, __nv_bfloat16* out, float* lse, int* err,
                              unsigned long long* trace, long long trace_rows, cudaStream_t st) {
  CUtensorMap m_qc, m_qr;
  const int QT = 128 / geo.G;
  if (n % kTcBlock != 0 || ((reinterpret_cast<uintptr_t>(kc_sw) | reinterpret_cast<uintptr_t>(kr_sw) |
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
