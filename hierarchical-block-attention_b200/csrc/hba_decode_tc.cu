// Decode on the 5th-generation tensor cores: one CTA per (sequence, kv head)
// does the selection on CUDA cores and the union softmax with tcgen05 MMAs
// whose accumulators live in TMEM, K/V tiles fed by 1-D bulk copies from the
// chunk-tiled cache.  With QKNorm off there is no logit bound: the softmax
// keeps the running maximum described below from the first chunk.
//
// The G query heads of a KV group are few (4-16), so the MMAs are swapped:
// keys are the M dimension.  For a 128-key chunk
//     S^T[128 keys x 16] = K[128 x dh] . Q^T          (A = K, B = Q, K-major)
//     O^T[dh x 16]      += V^T[dh x 128] . P^T         (A = V^T MN-major, B = P^T)
// One softmax thread per key reads its 16 head scores from TMEM and writes
// p = exp2(s*scale*log2e - M[h]) into P^T; l[h] are per-thread partial sums
// reduced once at the end.  M[h] is the per-head QKNorm bound of the logits
// (|s| <= scale*|q_h|*sqrt(dh)*k_gain) when every head's bound is small
// enough that no p can flush to zero (kBoundedLog2): then there is no max
// and O^T is never rescaled.  With larger bounds (trained QKNorm gains) M[h]
// is a lazily raised running max: the 4 softmax warps exchange their chunk
// maxima, and when one passes M[h] by more than kRescaleLog2 the warps wait
// for the previous PV, rescale their O^T rows in TMEM and l, and go on.
//
// Roles and phases:
//  warp 3 (lane 0) produces from the first instruction on: summary pages by
//    1-D bulk copies, then the window/sink K/V tiles by TMA (they need no
//    selection), then the routed tiles once the picks are known.
//  A (the other 7 warps) query prologue (its loads are issued before any bulk
//    copy); each warp scores whole pages, 4 rows at a time, keeping a running
//    top-k; one warp merges the 7 lists (flat, or supers then children of
//    the beam).
//  B warp 1: TMEM owner and single-thread MMA issuer; warps 4-7: softmax
//    (TMEM lane quarter = warp % 4).
//  C warps 4-7 reduce l, read O^T from TMEM, write out, LSE.
// Reference semantics: src/hba/attention.py:663-711 at cs = n-1.
#include <climits>
#include <cudaTypedefs.h>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_score.cuh"
#include "hba_sm100.cuh"
#include "hba_topk.cuh"
#include "hba_warpsort.cuh"

namespace hba {

using namespace sm100;

constexpr int kDtThreads = 256;
constexpr int kDtKeys = 128;  // keys per chunk (UMMA M)
constexpr int kDtProducer = 3;    // warp that feeds the ring from the first instruction on
constexpr int kDtScoreWarps = 7;  // every other warp scores summary pages
constexpr int kXListW = 32;       // entries per exchanged list slot

// barrier of the 7 scoring warps (the producer warp never joins it)
HBA_DEVICE void score_bar() { asm volatile("bar.sync 2, 224;\n" ::: "memory"); }



// One ring of NSLOT slots of one K (or V) tile each carries every byte the
// CTA reads, in this order: summary pages (128/m rows each; the flat scan, or
// the super rows then the children of the beam), then per 128-key chunk of
// [window | sinks | routed block pairs] its K tile and its V tile.  Thread 0
// keeps the ring full from the first instruction on, so the window tiles
// load while the pages are scored and the top-k runs.  A page slot is freed
// once all warps have scored it, a K slot when the softmax has seen its S MMA
// complete (an arrival, not another commit for the MMA thread to issue), a V
// slot when its PV MMA completes.
template <int DH>
struct DtcSmem {
  static constexpr int HALVES = DH / 64;
  static constexpr int KT = kDtKeys * DH * 2;               // one K or V tile = one slot
  static constexpr int NSLOT = DH == 64 ? 12 : 6;
  alignas(1024) unsigned char ring[NSLOT][KT];              // K/V: halves of [128 x 64] SW128
  alignas(1024) unsigned char qc[HALVES][16 * 128];         // Q rows (16 heads) [16 x 64] SW128 per half
  alignas(1024) unsigned char qr[HALVES][16 * 128];
  alignas(1024) unsigned char pt[2][2][16 * 128];           // P^T [buffer][key half][16 heads x 64 keys]
  alignas(16) __nv_bfloat16 qg[DH];  // routing query (bf16 values), read as packed 16-byte vectors
  float m2[16];      // per-head QKNorm logit bound (log2 units)
  float mfin[16];    // per-head softmax reference maximum at the end of the union
  float cmax[2][4][16];  // per-chunk maxima of the 4 softmax warps (running-max mode)
  float lsum[4][16];
  float xl[16];  // fused shard: l of every head merged over the ranks
  float xm[16];  // fused shard: the ranks' largest reference maximum per head
  float xw[kShardMaxRanks][16];  // fused shard: weight 2^(m_rank - xm) of each rank's partial
  float wl_s[kDtScoreWarps][32];  // per-warp top-k lists
  int wl_i[kDtScoreWarps][32];
  float xs[kDtScoreWarps][32];    // a scoring warp's batch candidates and list, for its rank update
  int xi[kDtScoreWarps][32];
  float ys[kDtScoreWarps][32];
  int yi[kDtScoreWarps][32];
  float sel_s[32];                // merged picks, best first
  int sel_i[32];
  int nsel;
  uint32_t thr;
  int sup_lo[32], sup_off[32], sup_cnt[32];
  int n_children;
  uint64_t full[NSLOT], empty[NSLOT];
  uint64_t s_full[2], p_full[2], p_free[2], cm_full[2];
  uint64_t s_free[2];  // the 4 softmax warps have read S buffer [b] (flat: the S issuer may reuse it)
  uint64_t o_full, drain, child_ready, sel_ready, lists_ready;
  uint32_t tmem_base;
  int issued;  // ring items the producer has issued (published after each)
};

static_assert(sizeof(DtcSmem<64>) + 1024 <= 232448 && sizeof(DtcSmem<128>) + 1024 <= 232448,
              "decode tile set exceeds the 227 KB of shared memory per CTA");

struct DecodeTcParams {
  DecodeAttnParams a;
  const __nv_bfloat16* summ;
  const __nv_bfloat16* supers;
  const float* k_gain;
  int* err;
  // KV-range shard mode (mode 1): this CTA's caches hold global tokens
  // [tok_lo, tok_lo + n_cap); the picks are the global top-k of the n_in
  // candidate entries per (sequence, kv head) in in_idx / in_score (every
  // shard's local lists); the union over the owned tokens is written as the
  // unnormalised O, l and the logit bound m2 (identical on every shard).
  int32_t mode;
  int32_t tok_lo;
  int32_t n_in;
  const int32_t* in_idx;  // [B*Hkv, n_in] global block ids, -1 = none
  const float* in_score;
  float* part_o;          // [B, Hq, dh]
  float* part_l;          // [B, Hq]
  float* part_m2;         // [B, Hq]
  // Fused shard mode (mode 2): as mode 1 for the owned tokens, but the CTA
  // selects itself (owned candidates, exact scores) and exchanges with the
  // same CTA of every other rank over NVLink: it writes its list (and later
  // its (O, l) partial) into slot [rank] of every rank's exchange buffer
  // (xpeer[r], IPC-mapped; xpeer[rank] is its own) as epoch-tagged 64-bit
  // words (x_layout) and waits for this step's tag in every rank's slot of
  // its own buffer.  Every rank merges the same global top-k and sums the
  // same partials in rank order.
  int32_t world, rank;
  const int32_t* epoch;   // this step's epoch, bumped on the stream before the launch
  unsigned char* xpeer[kShardMaxRanks];
};

template <int DH, int HB>
__global__ void __launch_bounds__(kDtThreads, 1)
    decode_tc_kernel(DecodeTcParams P) {
  using SM = DtcSmem<DH>;
  constexpr int HALVES = SM::HALVES;
  constexpr int NSLOT = SM::NSLOT;
  constexpr int NSW = kDtScoreWarps;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base_ptr =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SM& sm = *reinterpret_cast<SM*>(base_ptr);
  const DecodeAttnParams& p = P.a;
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int PER = DH / 32;
  const int G = geo.G;
  const int bg = blockIdx.x;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const bool shard = P.mode >= 1;   // owned tokens [tok_lo, tok_hi) only
  const bool fused = P.mode == 2;   // ... selecting and exchanging in-kernel
  const bool hier = geo.hier != 0 && P.mode != 1;  // mode 1 gets its picks from the lists
  const int tok_lo = shard ? P.tok_lo : 0;    // global token of local row 0
  const int tok_hi = tok_lo + geo.n_cap;      // end of the owned tokens
  unsigned long long* trace = (p.trace != nullptr && bg < p.trace_ctas) ? p.trace + (size_t)bg * 16 : nullptr;
  auto stamp = [&](int i) {
    if (trace != nullptr && tid == 0) trace[i] = global_ns();
  };
  auto stamp_any = [&](int i) {  // from the calling thread
    if (trace != nullptr) trace[i] = global_ns();
  };
  stamp(0);

  const int nctx = p.qp.seq_lens[b];
  const float scale = p.qp.scales[b];
  const bool ok = nctx >= 1 && (shard || nctx <= geo.n_cap);
  const int pos = ok ? nctx - 1 : -1;
  const int nb = ok ? nctx / geo.Bk : 0;
  const int bmax = ok ? min(last_candidate(pos, geo.W, geo.Bk), nb - 1) : 0;
  int kfinal = min(geo.K, nb);
  const int ns = (nb + geo.F - 1) / geo.F;
  if (geo.hier) kfinal = min(kfinal, min(geo.beam, ns) * geo.F);  // shards too: the global k
  // owned part of the window [wlo, whi] (global tokens) and of the sinks
  const int wlo = max(max(geo.S, pos - geo.W + 1), tok_lo);
  const int whi = min(pos, tok_hi - 1);
  const int nw = ok ? max(0, whi - wlo + 1) : 0;
  // window chunks start on a 64-token block (the cache's tile): [wla, whi], keys before wlo masked
  const int wla = wlo & ~63;
  const int nsink = (ok && tok_lo == 0) ? min(geo.S, pos + 1) : 0;
  const int NCw = nw > 0 ? (whi - wla) / kDtKeys + 1 : 0;
  const int NCs = nsink > 0 ? 1 : 0;
  const bool producer = warp == kDtProducer;
  const int sw = warp < kDtProducer ? warp : warp - 1;  // scoring-warp index (producer excluded)

  // ---- A.0 query rows, RoPE row and gains: issued before any bulk copy ----
  uint32_t qraw[3][PER / 2];
  float cr[PER], sr[PER], qgain[3];
  float kg = 0.f;
  if (!producer && ok) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      cr[i] = p.cos[(size_t)pos * DH + lane * PER + i];
      sr[i] = p.sin[(size_t)pos * DH + lane * PER + i];
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int h = sw + NSW * j;
      if (h < G) {
        const uint32_t* src =
            reinterpret_cast<const uint32_t*>(p.q + ((size_t)b * geo.Hq + g * G + h) * DH) + lane * (PER / 2);
#pragma unroll
        for (int k = 0; k < PER / 2; ++k) qraw[j][k] = src[k];
        qgain[j] = geo.qknorm ? p.q_gain[g * G + h] : 1.f;
      }
    }
    kg = geo.qknorm ? P.k_gain[g] : 0.f;
  }

  // ---- selection geometry (known from the position alone) ----
  const int row_elems = geo.m * DH;
  const int row_bytes = row_elems * 2;
  const int PB = SM::KT / row_bytes;  // summary rows per page
  const __nv_bfloat16* summ_bg = P.summ + (size_t)bg * geo.nb_cap * row_elems;
  // this (sequence, kv head)'s chunk-tiled K, RoPE'd K and V: [n_cap/64][dh/64][64 x 64]
  const size_t kv_head = (size_t)bg * geo.n_cap * DH;
  const __nv_bfloat16* k_bg = p.k + kv_head;
  const __nv_bfloat16* kr_bg = p.kr + kv_head;
  const __nv_bfloat16* v_bg = p.v + kv_head;
  const __nv_bfloat16* sup_bg = hier ? P.supers + (size_t)bg * geo.ns_cap * row_elems : nullptr;
  // phase-A candidates, ids id0 .. id0 + Ra - 1: flat blocks 1..bmax, or
  // supers ida..bmax/F, of them the owned ones (blocks [blo, bhi), supers
  // [blo/F, bhi/F); local row = id - first owned id)
  const int blo = tok_lo / geo.Bk, bhi = tok_hi / geo.Bk;
  int Ra = 0, id0 = 1;
  if (P.mode == 1) {
    Ra = 0;  // picks come from the lists
  } else if (!hier) {
    id0 = max(1, blo);
    Ra = max(0, min(bmax, bhi - 1) - id0 + 1);
  } else if (bmax >= 1) {
    const int ida = (geo.F == 1) ? 1 : 0;
    id0 = max(ida, blo / geo.F);
    Ra = max(0, min(bmax / geo.F, bhi / geo.F - 1) - id0 + 1);
  }
  const __nv_bfloat16* rows_a = hier ? sup_bg + (size_t)(id0 - blo / geo.F) * row_elems
                                     : summ_bg + (size_t)(id0 - blo) * row_elems;
  const int NPa = (Ra + PB - 1) / PB;
  // Ring item order: [NPa phase-A pages][K,V of chunks 0 .. WA-1][NPb child
  // pages][K,V of chunks WA ..].  Flat: WA = all window/sink chunks (no child
  // pages).  Hier: a few window chunks go ahead of the child pages, so the
  // attention warps have work (and the memory pipe traffic) while the super
  // top-k runs.
  const int NCk = NCw + NCs;  // window + sink chunks: known before any selection
  const int WA = hier ? min(NCk, SM::NSLOT / 3) : NCk;
  auto item_of_chunk = [&](int c, int npb) { return c < WA ? NPa + 2 * c : NPa + 2 * WA + npb + 2 * (c - WA); };

  // ---- barriers, TMEM ----
  if (producer && lane == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 128);
      mbar_init(&sm.p_free[s], 1);
      mbar_init(&sm.cm_full[s], 4);  // one arrival per softmax warp
      mbar_init(&sm.s_free[s], 4);
    }
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.drain, 1);
    mbar_init(&sm.child_ready, 1);
    mbar_init(&sm.sel_ready, 1);
    mbar_init(&sm.lists_ready, kDtScoreWarps);
    sm.issued = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;  // cols [0,16) S0, [16,32) S1, [32,48) O^T
  // A consumer of ring item i first sees it issued, then tests full[i % NSLOT]
  // by parity: a parity test is only unambiguous once the slot's previous
  // item has landed, which the producer's empty wait before issuing item i
  // guarantees (that item was consumed).
  auto issued_past = [&](int i) { return *reinterpret_cast<volatile int*>(&sm.issued) > i; };
  auto wait_full = [&](int i) -> bool {
    if (!issued_past(i)) {
      const unsigned long long t0 = global_ns();
      for (uint32_t k = 1; !issued_past(i); ++k) {
        __nanosleep(32);
        if ((k & 63) == 0 && global_ns() - t0 > kWaitNs) {
          atomicExch(P.err, 1);
          return false;
        }
      }
    }
    return mbar_wait(&sm.full[i % NSLOT], (i / NSLOT) & 1, P.err);
  };

  if (producer) {
    // ---- ring producer: the items in the order described at item_of_chunk ----
    if (lane == 0) {
      int NPb = 0, R2 = 0, nsel = 0, issued = 0;
      auto issue_item = [&](int i) {
        unsigned char* dst = sm.ring[i % NSLOT];
        uint64_t* fb = &sm.full[i % NSLOT];
        const int cp0 = NPa + 2 * WA;  // first child page item
        if (i < NPa) {
          const int j0 = i * PB, nr = min(PB, Ra - j0);
          mbar_arrive_expect_tx(fb, (uint32_t)(nr * row_bytes));
          bulk_load(dst, rows_a + (size_t)j0 * row_elems, (uint32_t)(nr * row_bytes), fb);
        } else if (i >= cp0 && i < cp0 + NPb) {  // children of the beam: one bulk copy per contiguous span
          const int j0 = (i - cp0) * PB, j1 = min(R2, j0 + PB);
          mbar_arrive_expect_tx(fb, (uint32_t)((j1 - j0) * row_bytes));
          for (int si = 0; si < 32; ++si) {
            const int lo = max(j0, sm.sup_off[si]), hi = min(j1, sm.sup_off[si] + sm.sup_cnt[si]);
            if (lo < hi)
              bulk_load(dst + (size_t)(lo - j0) * row_bytes,
                        summ_bg + (size_t)(sm.sup_lo[si] + lo - sm.sup_off[si] - blo) * row_elems,
                        (uint32_t)((hi - lo) * row_bytes), fb);
          }
        } else {
          const int e = i < cp0 ? i - NPa : i - NPb - NPa;  // 2 * chunk + (V ? 1 : 0)
          const int c = e >> 1, is_v = e & 1;
          // the chunk's two 64-token blocks (local); a half past the keys
          // loads a valid block again, its keys masked
          int kind, b0, b1;
          if (c < NCw) {
            kind = 0;
            b0 = (wla - tok_lo + c * kDtKeys) >> 6;
            b1 = min(b0 + 1, geo.n_cap / 64 - 1);
          } else if (c < NCw + NCs) {
            kind = 1;
            b0 = b1 = 0;
          } else {
            kind = 2;
            const int q = (c - NCw - NCs) * 2;
            b0 = sm.sel_i[q];
            b1 = q + 1 < nsel ? sm.sel_i[q + 1] : b0;  // odd count: a valid block, masked
          }
          mbar_arrive_expect_tx(fb, SM::KT);
          const __nv_bfloat16* src = is_v ? v_bg : (kind == 0 ? kr_bg : k_bg);
          // per 64-dim group one 8 KB tile per block: rows [0, 64) of the
          // slot's group from b0, rows [64, 128) from b1
#pragma unroll
          for (int h = 0; h < HALVES; ++h) {
            bulk_load(dst + h * (kDtKeys * 128), src + ((size_t)b0 * HALVES + h) * 4096, 8192, fb);
            bulk_load(dst + h * (kDtKeys * 128) + 64 * 128, src + ((size_t)b1 * HALVES + h) * 4096, 8192, fb);
          }
        }
      };
      auto pump_to = [&](int upto) -> bool {
        for (; issued < upto; ++issued) {
          if (issued >= NSLOT &&
              !mbar_wait(&sm.empty[issued % NSLOT], ((issued / NSLOT) - 1) & 1, P.err))
            return false;
          issue_item(issued);
          __threadfence_block();
          *reinterpret_cast<volatile int*>(&sm.issued) = issued + 1;
        }
        return true;
      };
      bool okp = pump_to(NPa + 2 * WA);  // window/sink tiles need no selection
      if (hier && okp) {
        okp = mbar_wait(&sm.child_ready, 0, P.err);
        R2 = sm.n_children;
        NPb = (R2 + PB - 1) / PB;
        okp = okp && pump_to(NPa + NPb + 2 * NCk);
      }
      if (okp && mbar_wait(&sm.sel_ready, 0, P.err)) {
        stamp_any(12);
        nsel = sm.nsel;
        pump_to(NPa + NPb + 2 * (NCk + (nsel * geo.Bk + kDtKeys - 1) / kDtKeys));
      }
    }
  } else {
    // ---- A.1 QKNorm, RoPE, Q tiles (SW128), per-head logit bounds ----
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int h = sw + NSW * j;  // warp-uniform
      if (h < 16) {
        float v[PER], r[PER];
        float qn2 = 0.f;
        if (h < G && ok) {
#pragma unroll
          for (int k = 0; k < PER / 2; ++k) {
            const float2 t2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qraw[j][k]));
            v[2 * k] = t2.x;
            v[2 * k + 1] = t2.y;
          }
          if (geo.qknorm) qknorm_lane<DH>(v, qgain[j], geo.eps);
          const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
          for (int i = 0; i < PER; ++i) {
            const float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
            r[i] = rope_elem(v[i], sign * partner, cr[i], sr[i]);
            qn2 = fmaf(v[i], v[i], qn2);
          }
        } else {
#pragma unroll
          for (int i = 0; i < PER; ++i) v[i] = r[i] = 0.f;
        }
        qn2 = warp_sum(qn2);
        // element d -> half d/64, column d%64 of row h
#pragma unroll
        for (int i = 0; i < PER; i += 2) {
          const int d = lane * PER + i;
          const uint32_t off = sw128_offset(h, d % 64);
          *reinterpret_cast<uint32_t*>(sm.qc[d / 64] + off) = pack_bf16x2(v[i], v[i + 1]);
          *reinterpret_cast<uint32_t*>(sm.qr[d / 64] + off) = pack_bf16x2(r[i], r[i + 1]);
        }
        if (lane == 0) {
          const float kmax = sqrtf((float)DH) * kg * (1.f + 1.f / 64.f);
          const float m2 = scale * sqrtf(qn2) * kmax * kLog2e;
          // without QKNorm no bound: the running maximum from the first chunk
          sm.m2[h] = (h < G && ok) ? (geo.qknorm ? m2 : __int_as_float(0x7f800000)) : 0.f;
        }
      }
    }
    score_bar();
    // routing query: bf16(fp32 sum of the bf16 QKNorm'd heads, in head order)
    for (int d = sw * 32 + lane; d < DH; d += NSW * 32) {
      float acc = 0.f;
      for (int h = 0; h < G; ++h) acc += bf2f(*reinterpret_cast<const __nv_bfloat16*>(sm.qc[d / 64] + sw128_offset(h, d % 64)));
      sm.qg[d] = __float2bfloat16_rn(acc);
    }
    if constexpr (HB < 16) {  // P^T rows of heads >= HB stay zero for the whole kernel
      // 4 tiles [buffer][key half] of 16 rows x 128 B; rows 8-15 = the second
      // 1024-byte swizzle atom = 64 chunks of 16 B per tile
      for (int e = sw * 32 + lane; e < 4 * 64; e += NSW * 32) {
        const int tile = e >> 6, rem = e & 63;
        *reinterpret_cast<uint4*>(sm.pt[tile >> 1][tile & 1] + 1024 + rem * 16) = make_uint4(0, 0, 0, 0);
      }
    }
    fence_proxy_async_smem();  // Q and P^T tiles are read by the tensor cores
    score_bar();
    stamp(1);

    // ---- A.2 selection: each scoring warp owns pages sw, sw + 7, ... ----
    // One summary row per lane.  A lane reads the LPS 16-byte vectors of a
    // slot in the order q ^ (lane & 7) -- conflict-free across the 8 lanes of
    // a shared-memory phase -- and adds the per-vector partials in the
    // pairwise tree of SummaryLoads::score (hba_score.cuh); XOR relabelling
    // within aligned groups keeps every pair of that tree, so the scores are
    // bit-identical to the other decode paths.  Each warp keeps its best 32
    // (score desc, id asc) in registers: a 32-row batch that beats the k-th
    // entry is bitonic-sorted and merged in.
    constexpr int LPS = DH / 8;  // 16-byte vectors per slot
    // dh 64: the query in fp32 registers and two vectors' chains in packed
    // f32x2 fmas.  dh 128: each 8-term chain is dot8_bf16 (mixed-precision
    // fmas on the packed bf16 halves, the same value as the fp32 fmaf chain
    // over the widened vectors); measured, each form is the faster one for
    // its head size.
    constexpr bool kQgRegs = DH == 64;  // this lane's permuted copy of qg in registers
    const int m_slots = geo.m;
    const int o = lane & 7;
    float qgp[kQgRegs ? LPS : 1][8];
    if constexpr (kQgRegs) {
#pragma unroll
      for (int q = 0; q < LPS; ++q) unpack8(*reinterpret_cast<const uint4*>(&sm.qg[(q ^ o) * 8]), qgp[q]);
    }
    float ls = neg_inf();
    int li = INT_MAX;
    if (tid == 0) sm.thr = 0u;  // order_key of the best k-th score any warp has reached
    score_bar();
    int pg_first = sw, pg_stride = NSW;  // which pages this warp scores
    auto score_pages = [&](int i0, int np, int R, int k, auto id_of) {
      for (int pg = pg_first; pg < np; pg += pg_stride) {
        const int i = i0 + pg;
        wait_full(i);
        const unsigned char* src = sm.ring[i % NSLOT];
        const int nr = min(PB, R - pg * PB);
        for (int rg = 0; rg < nr; rg += 32) {
          const int r = rg + lane;
          float cs = neg_inf();
          int ci = INT_MAX;
          if (r < nr) {
            const unsigned char* row = src + (size_t)r * row_bytes;
            float best = neg_inf();
            if constexpr (DH == 64) {
              for (int sl = 0; sl < m_slots; ++sl) {
                float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;  // pending sums of the pairwise tree
#pragma unroll
                for (int q = 0; q < LPS; q += 2) {
                  // vectors q, q + 1: two independent chains in packed f32x2 fmas
                  // (each half is the fmaf chain)
                  float f0[8], f1[8];
                  unpack8(*reinterpret_cast<const uint4*>(row + (sl * LPS + (q ^ o)) * 16), f0);
                  unpack8(*reinterpret_cast<const uint4*>(row + (sl * LPS + ((q + 1) ^ o)) * 16), f1);
                  float p0 = 0.f, p1 = 0.f;
#pragma unroll
                  for (int jj = 0; jj < 8; ++jj) fma2(p0, p1, f0[jj], f1[jj], qgp[q][jj], qgp[q + 1][jj]);
                  t0 = p0;
                  const float part = p1;
                  {
                    const float l1 = t0 + part;
                    if ((q & 2) == 0) {
                      t1 = l1;
                    } else {
                      const float l2 = t1 + l1;
                      if ((q & 4) == 0) {
                        t2 = l2;
                      } else {
                        const float l3 = t2 + l2;
                        if (LPS == 8) {
                          best = fmaxf(best, l3);
                        } else if ((q & 8) == 0) {
                          t3 = l3;
                        } else {
                          best = fmaxf(best, t3 + l3);
                        }
                      }
                    }
                  }
                }
              }
            } else {
              for (int sl = 0; sl < m_slots; ++sl) {
                float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;  // pending sums of the pairwise tree
#pragma unroll
                for (int q = 0; q < LPS; ++q) {
                  const int vq = q ^ o;
                  const float part = dot8_bf16(*reinterpret_cast<const uint4*>(row + (sl * LPS + vq) * 16),
                                               *reinterpret_cast<const uint4*>(&sm.qg[vq * 8]));
                  // fold into the tree as the vectors arrive: ((p0+p1)+(p2+p3))+...
                  if ((q & 1) == 0) {
                    t0 = part;
                  } else {
                    const float l1 = t0 + part;
                    if ((q & 2) == 0) {
                      t1 = l1;
                    } else {
                      const float l2 = t1 + l1;
                      if ((q & 4) == 0) {
                        t2 = l2;
                      } else {
                        const float l3 = t2 + l2;
                        if (LPS == 8) {
                          best = fmaxf(best, l3);
                        } else if ((q & 8) == 0) {
                          t3 = l3;
                        } else {
                          best = fmaxf(best, t3 + l3);
                        }
                      }
                    }
                  }
                }
            }
            }
            cs = best * scale;
            ci = id_of(pg * PB + r);
          }
          if (rg + 32 >= nr) {  // the page's last rows are scored: free its slot before the top-k work
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[i % NSLOT]);
          }
          // keep the batch entries that can still reach the final top-k
          const float ts = __shfl_sync(0xffffffffu, ls, k - 1);
          const int ti = __shfl_sync(0xffffffffu, li, k - 1);
          const uint32_t thr = *reinterpret_cast<volatile uint32_t*>(&sm.thr);
          const bool cand = beats(cs, ci, ts, ti) && order_key(cs) >= thr;
          const unsigned mask = __ballot_sync(0xffffffffu, cand);
          if (mask == 0u) continue;
          // The list keeps its top k (lanes >= k: fillers).  Every entry gets
          // its exact rank: an old one moves down by the candidates that beat
          // it, a candidate counts the old entries ahead of it (binary search
          // of the sorted list; entry k - 1 is behind it) and the candidates
          // ahead of it.  The top k of list and batch, in a few steps (a
          // bitonic sort of the batch costs ~2,600 cycles).
          const int n = __popc(mask);
          float* xs_ = sm.xs[sw];
          int* xi_ = sm.xi[sw];
          float* ys_ = sm.ys[sw];
          int* yi_ = sm.yi[sw];
          if (cand) {
            const int at = __popc(mask & ((1u << lane) - 1u));
            xs_[at] = cs;
            xi_[at] = ci;
          }
          ys_[lane] = ls;
          yi_[lane] = li;
          __syncwarp();
          int opos = lane;
          for (int j = 0; j < n; ++j) opos += beats(xs_[j], xi_[j], ls, li);
          int npos = k;
          float ns = 0.f;
          int ni = 0;
          if (lane < n) {
            ns = xs_[lane];
            ni = xi_[lane];
            int lo = 0;
#pragma unroll
            for (int step = 16; step > 0; step >>= 1)
              if (lo + step <= k && beats(ys_[lo + step - 1], yi_[lo + step - 1], ns, ni)) lo += step;
            for (int j = 0; j < n; ++j) lo += beats(xs_[j], xi_[j], ns, ni);
            npos = lo;
          }
          __syncwarp();
          if (lane < k && opos < k) {
            ys_[opos] = ls;
            yi_[opos] = li;
          }
          if (npos < k) {
            ys_[npos] = ns;
            yi_[npos] = ni;
          }
          __syncwarp();
          ls = lane < k ? ys_[lane] : neg_inf();
          li = lane < k ? yi_[lane] : INT_MAX;
          const int kth = __shfl_sync(0xffffffffu, li, k - 1);
          const float kts = __shfl_sync(0xffffffffu, ls, k - 1);
          if (lane == 0 && kth != INT_MAX) atomicMax(&sm.thr, order_key(kts));
        }
      }
    };
    int nsel = 0, NPb = 0;
    // warp 0, from the global top-k (gs, gi) (best first): the picks out,
    // and the owned ones as local block ids in sm.sel_i, their count nsel
    auto own_picks = [&](float gs, int gi) {
      const bool valid = lane < kfinal && gi != INT_MAX;
      if (p.sel_idx != nullptr && lane < geo.K) {
        p.sel_idx[(size_t)bg * geo.K + lane] = valid ? gi : -1;
        p.sel_score[(size_t)bg * geo.K + lane] = valid ? gs : neg_inf();
      }
      const bool own = valid && gi >= blo && gi < bhi;
      const unsigned om = __ballot_sync(0xffffffffu, own);
      if (own) sm.sel_i[__popc(om & ((1u << lane) - 1u))] = gi - blo;
      nsel = __popc(om);
      if (lane == 0) sm.nsel = nsel;
    };
    // Fused shard (warp 0): publish lanes [0, kx) of (ls, li) as this rank's
    // list of exchange x in every rank's buffer, wait for every rank's, and
    // return in (ls, li) the best 32 of their union, best first.
    const XLayout xl = x_layout(geo.B * geo.Hkv, fused ? P.world : 1, DH);
    const uint32_t epoch = fused ? (uint32_t)*P.epoch : 0u;
    // list entry: score bits | block id (0xffff: none) << 32 | epoch (16 bits) << 48
    const unsigned long long etag = epoch & 0xffffu;
    auto exchange_lists = [&](int x, int kx, float& ls_, int& li_) {
      const bool has = lane < kx && li_ != INT_MAX;
      const unsigned long long mine = (unsigned long long)__float_as_uint(has ? ls_ : neg_inf()) |
                                      ((unsigned long long)(has ? (uint32_t)li_ & 0xffffu : 0xffffu) << 32) |
                                      (etag << 48);
      for (int r = 0; r < P.world; ++r)
        st_relaxed_sys(reinterpret_cast<unsigned long long*>(P.xpeer[r] + xl.list[x]) +
                           ((size_t)bg * P.world + P.rank) * kXListW + lane,
                       mine);
      const unsigned long long* lists =
          reinterpret_cast<const unsigned long long*>(P.xpeer[P.rank] + xl.list[x]) + (size_t)bg * P.world * kXListW;
      unsigned long long e[kShardMaxRanks];  // this lane's entry of every rank's list, loaded together
      wait_tagged_n<kShardMaxRanks>(lists + lane, kXListW, P.world, 48, 0xffffu, etag, e, P.err);
      float gs = neg_inf();
      int gi = INT_MAX;
#pragma unroll
      for (int r = 0; r < kShardMaxRanks; ++r) {  // each rank's list is sorted: merge them
        if (r < P.world) {
          const uint32_t id = (uint32_t)(e[r] >> 32) & 0xffffu;
          warp_merge32(gs, gi, id == 0xffffu ? neg_inf() : __uint_as_float((uint32_t)e[r]),
                       id == 0xffffu ? INT_MAX : (int)id);
        }
      }
      if (lane == 0) stamp_any(14 + x);
      ls_ = gs;
      li_ = gi;
    };
    if (P.mode == 1) {
      // global top-k of every shard's lists, then the owned picks (local block ids)
      if (warp == 0) {
        const int kk = max(1, kfinal);
        for (int e0 = 0; e0 < P.n_in; e0 += 32) {
          const int e = e0 + lane;
          float cs = neg_inf();
          int ci = INT_MAX;
          if (e < P.n_in) {
            const int id = P.in_idx[(size_t)bg * P.n_in + e];
            if (id >= 0) {
              cs = P.in_score[(size_t)bg * P.n_in + e];
              ci = id;
            }
          }
          const float ts = __shfl_sync(0xffffffffu, ls, kk - 1);
          const int ti = __shfl_sync(0xffffffffu, li, kk - 1);
          if (__any_sync(0xffffffffu, beats(cs, ci, ts, ti))) {
            warp_sort32(cs, ci);
            warp_merge32(ls, li, cs, ci);
          }
        }
        own_picks(ls, li);
      }
      score_bar();
      nsel = sm.nsel;
      stamp(5);
    } else if (!hier) {
      // each warp publishes its list; warp 0 alone merges them, while the MMA
      // and softmax warps go on to the window and sink chunks
      if (kfinal > 0) score_pages(0, NPa, Ra, kfinal, [&](int j) { return id0 + j; });
      stamp(5);
      sm.wl_s[sw][lane] = ls;
      sm.wl_i[sw][lane] = li;
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.lists_ready);
      if (warp == 0) {
        mbar_wait(&sm.lists_ready, 0, P.err);
        float fs = sm.wl_s[0][lane];
        int fi = sm.wl_i[0][lane];
        for (int w = 1; w < NSW; ++w) warp_merge32(fs, fi, sm.wl_s[w][lane], sm.wl_i[w][lane]);
        if (fused) {  // this rank's top-k -> every rank -> the global top-k
          exchange_lists(0, kfinal, fs, fi);
          own_picks(fs, fi);
        } else {
          nsel = __popc(__ballot_sync(0xffffffffu, lane < kfinal && fi != INT_MAX));
          sm.sel_i[lane] = fi;
          sm.sel_s[lane] = fs;
          if (lane == 0) sm.nsel = nsel;
        }
      }
      stamp(6);
    } else if (warp == 0 || warp == 2) {
      // hierarchical: warps 0 and 2 select (a level has a few pages); warps 1
      // and 4-7 go on to the window chunks (phase B) at once
      const int hw = warp >> 1;
      pg_first = hw;
      pg_stride = 2;
      auto pair_bar = []() { asm volatile("bar.sync 3, 64;\n" ::: "memory"); };
      auto merge2 = [&](int k) -> int {  // the two lists -> best-first picks in sm.sel_i / sel_s
        sm.wl_s[hw][lane] = ls;
        sm.wl_i[hw][lane] = li;
        pair_bar();
        if (warp == 0) {
          float fs = sm.wl_s[0][lane];
          int fi = sm.wl_i[0][lane];
          warp_merge32(fs, fi, sm.wl_s[1][lane], sm.wl_i[1][lane]);
          const int n = __popc(__ballot_sync(0xffffffffu, lane < k && fi != INT_MAX));
          sm.sel_i[lane] = fi;
          sm.sel_s[lane] = fs;
          if (lane == 0) sm.nsel = n;
        }
        pair_bar();
        return sm.nsel;
      };
      const int kb = max(1, min(geo.beam, ns));
      score_pages(0, NPa, Ra, kb, [&](int j) { return id0 + j; });
      stamp(5);
      int nsup = merge2(kb);
      if (warp == 0) {  // the beam's supers in ascending order; their children as contiguous spans
        if (fused) {  // this rank's top-beam -> every rank -> the global beam
          float fs = lane < nsup ? sm.sel_s[lane] : neg_inf();
          int fi = lane < nsup ? sm.sel_i[lane] : INT_MAX;
          exchange_lists(0, kb, fs, fi);
          nsup = __popc(__ballot_sync(0xffffffffu, lane < kb && fi != INT_MAX));
          __syncwarp();
          sm.sel_i[lane] = fi;
          __syncwarp();
        }
        const bool valid = lane < nsup;
        const int sidx = valid ? sm.sel_i[lane] : INT_MAX;
        int rank = 0;
        for (int o = 0; o < 32; ++o) rank += __shfl_sync(0xffffffffu, sidx, o) < sidx;
        __syncwarp();
        if (valid) sm.sup_lo[rank] = sidx;
        __syncwarp();
        const int s = lane < nsup ? sm.sup_lo[lane] : 0;
        __syncwarp();
        int lo = 0, cnt = 0;
        if (lane < nsup) {
          lo = max(1, s * geo.F);
          cnt = max(0, min(bmax, s * geo.F + geo.F - 1) - lo + 1);
          if (s < blo / geo.F || s >= bhi / geo.F) cnt = 0;  // children on another rank
        }
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int nv = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += nv;
        }
        sm.sup_lo[lane] = lo;
        sm.sup_cnt[lane] = cnt;
        sm.sup_off[lane] = incl - cnt;
        if (lane == 31) sm.n_children = incl;
        if (lane == 0) sm.thr = 0u;  // child scores start a new threshold
        __syncwarp();
        __threadfence_block();
        if (lane == 0) mbar_arrive(&sm.child_ready);
      }
      pair_bar();
      const int R2 = sm.n_children;
      NPb = (R2 + PB - 1) / PB;
      stamp(6);
      auto child_id = [&](int j) -> int {
        int si = 0;
        while (si < 31 && j >= sm.sup_off[si] + sm.sup_cnt[si]) ++si;
        return sm.sup_lo[si] + (j - sm.sup_off[si]);
      };
      ls = neg_inf();
      li = INT_MAX;
      if (kfinal > 0) score_pages(NPa + 2 * WA, NPb, R2, kfinal, child_id);
      stamp(7);
      nsel = merge2(max(1, kfinal));
      if (fused && warp == 0) {  // this rank's top-k of its children -> every rank -> the global top-k
        float fs = lane < nsel ? sm.sel_s[lane] : neg_inf();
        int fi = lane < nsel ? sm.sel_i[lane] : INT_MAX;
        exchange_lists(1, kfinal, fs, fi);
        __syncwarp();
        own_picks(fs, fi);
      }
    }
    if (warp == 0) {  // (flat: only warp 0 knows nsel here; the others read it after sel_ready)
      const bool valid = lane < nsel;
      if (!shard && p.sel_idx != nullptr && lane < geo.K) {
        p.sel_idx[(size_t)bg * geo.K + lane] = valid ? sm.sel_i[lane] : -1;
        p.sel_score[(size_t)bg * geo.K + lane] = valid ? sm.sel_s[lane] : neg_inf();
      }
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        mbar_arrive(&sm.sel_ready);  // picks and count are in shared memory
      }
    }
    // chunks [window | sinks] are known now; the routed ones once sel_ready completes
    const int NCk = NCw + NCs;
    auto routed_chunks = [&]() -> int {  // waits for the picks (a no-op wait once they are in)
      if (!mbar_wait(&sm.sel_ready, 0, P.err)) return 0;
      nsel = sm.nsel;
      return (nsel * geo.Bk + kDtKeys - 1) / kDtKeys;
    };
    stamp(2);

    // ---- B. union softmax ----
    if (warp == 1 || (warp == 2 && !hier)) {
      // MMA issue.  Flat selection: warp 2 (free once the lists are merged)
      // issues the S MMAs, up to both S buffers ahead, and warp 1 the PV MMAs,
      // so each warp's waits overlap the other's issue (the tensor pipe takes
      // one of these small MMAs every ~22 ns; the waits and bookkeeping around
      // them were most of a chunk's time).  Hierarchical selection keeps warps
      // 0 and 2 busy: warp 1 issues both, S(c) before PV(c-1).  Each loop runs
      // on the whole warp (warp-uniform descriptors and waits); one elected
      // lane issues each tcgen05 op.
      const bool do_s = warp == 2 || hier, do_pv = warp == 1;
      {
        constexpr uint32_t idesc_s = idesc_bf16(128, 16, false, false);
        constexpr uint32_t idesc_o = idesc_bf16(128, 16, true, false);
        auto wwait = [&](uint64_t* bar, uint32_t parity) {
          return __all_sync(0xffffffffu, mbar_wait(bar, parity, P.err));
        };
        auto wfull = [&](int i) { return __all_sync(0xffffffffu, wait_full(i)); };
        bool okw = true;
        int npb = 0;  // child pages ahead of chunk WA (hier: known at child_ready)
        // dh 64: M = 128 reads a second MN group at LBO 0 (rows 64-127 of O^T duplicate 0-63, unused)
        constexpr uint32_t lbo = DH == 128 ? kDtKeys * 128 : 0;
        const uint64_t pdesc0 = sdesc_sw128(smem_u32(sm.pt[0][0]), 16, 1024);
        const uint64_t pdesc1 = sdesc_sw128(smem_u32(sm.pt[1][0]), 16, 1024);
        const uint64_t qc_desc = sdesc_sw128(smem_u32(sm.qc[0]), 16, 1024);
        const uint64_t qr_desc = sdesc_sw128(smem_u32(sm.qr[0]), 16, 1024);
        constexpr uint32_t qhalf = 16 * 128;  // bytes between the Q tiles' 64-dim halves
        auto pv = [&](int c) -> bool {
          const int sb = c & 1, iv = item_of_chunk(c, npb) + 1;
          if (!wwait(&sm.p_full[sb], (c >> 1) & 1) || !wfull(iv)) return false;
          tc_fence_after();
          const uint64_t vdesc = sdesc_sw128(smem_u32(sm.ring[iv % NSLOT]), lbo, 1024);
          if (elect_one_sync()) {
#pragma unroll
            for (int kk = 0; kk < kDtKeys / 16; ++kk)
              umma_f16(tmem + 32, vdesc + (uint64_t)((kk * 2048) >> 4),
                       (sb ? pdesc1 : pdesc0) + (uint64_t)(((kk >> 2) * 2048 + (kk & 3) * 32) >> 4), idesc_o,
                       (c > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&sm.empty[iv % NSLOT]);  // the V tile is free once PV is done
            umma_commit(&sm.p_free[sb]);
          }
          __syncwarp();
          return true;
        };
        int NC = NCk;
        bool picks_in = false;
        for (int c = 0; okw; ++c) {
          if (c == NC && !picks_in) {  // window and sinks issued: now the routed chunks
            NC += __shfl_sync(0xffffffffu, routed_chunks(), 0);
            picks_in = true;
          }
          if (c >= NC) break;
          if (hier && c == WA) {  // chunks from here on sit behind the child pages in the ring
            if (!wwait(&sm.child_ready, 0)) {
              okw = false;
              break;
            }
            npb = (sm.n_children + PB - 1) / PB;
          }
          const int sb = c & 1;
          if (do_s) {
            const int ik = item_of_chunk(c, npb);
            // flat: S buffer sb is free once the softmax has read S(c - 2)
            if (!wfull(ik) || (!hier && c >= 2 && !wwait(&sm.s_free[sb], ((c - 2) >> 1) & 1))) {
              okw = false;
              break;
            }
            if (lane == 0) {
              if (c == 0) stamp_any(8);
              if (c == NCk - 1) stamp_any(9);
              if (c == NCk) stamp_any(10);
            }
            tc_fence_after();
            const uint64_t kdesc = sdesc_sw128(smem_u32(sm.ring[ik % NSLOT]), 16, 1024);
            const uint64_t qdesc = c < NCw ? qr_desc : qc_desc;
            if (elect_one_sync()) {
#pragma unroll
              for (int kk = 0; kk < DH / 16; ++kk) {
                const int h = kk >> 2, ko = (kk & 3) * 32;
                umma_f16(tmem + sb * 16, kdesc + (uint64_t)((h * (kDtKeys * 128) + ko) >> 4),
                         qdesc + (uint64_t)((h * qhalf + ko) >> 4), idesc_s, kk > 0 ? 1u : 0u);
              }
              umma_commit(&sm.s_full[sb]);  // the softmax frees the K slot once it has seen this
            }
            __syncwarp();
          }
          if (do_pv) {
            if (hier) {
              if (c >= 1 && !pv(c - 1)) {
                okw = false;
                break;
              }
            } else if (!pv(c)) {
              okw = false;
              break;
            }
          }
        }
        if (do_pv) {
          if (hier && okw && NC >= 1) okw = pv(NC - 1);
          if (lane == 0) stamp_any(11);
          if (elect_one_sync()) {
            umma_commit(&sm.o_full);
            umma_commit(&sm.drain);
          }
          __syncwarp();
          wwait(&sm.drain, 0);
        }
      }
    } else if (warp >= 4) {
      const int t = tid - 128;  // key row of the chunk / TMEM lane
      const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
      const float sl2 = scale * kLog2e;
      // mr[h]: the reference maximum of head h (log2 units), uniform over the
      // 128 softmax threads.  bounded: the QKNorm bounds, fixed; otherwise a
      // running max that starts empty.
      float lp[HB], mr[HB];
      bool bounded = true;
#pragma unroll
      for (int h = 0; h < HB; ++h) {
        lp[h] = 0.f;
        mr[h] = sm.m2[h];
        bounded = bounded && mr[h] <= kBoundedLog2;
      }
      if (!bounded) {
#pragma unroll
        for (int h = 0; h < HB; ++h) mr[h] = neg_inf();
      }
      bool okw = true;
      int NC = NCk;
      bool picks_in = false;
      int npb_s = 0;  // child pages ahead of chunk WA (hier), for the ring items this warp releases
      for (int c = 0;; ++c) {
        if (c == NC && !picks_in) {
          NC += routed_chunks();
          picks_in = true;
        }
        if (c >= NC) break;
        if (hier && c == WA) {
          if (!__all_sync(0xffffffffu, mbar_wait(&sm.child_ready, 0, P.err))) {
            okw = false;
            break;
          }
          npb_s = (sm.n_children + PB - 1) / PB;
        }
        const int sb = c & 1;
        // a failed wait leaves the whole warp together (the TMEM accesses below are warp-collective)
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[sb], (c >> 1) & 1, P.err))) {
          okw = false;
          break;
        }
        tc_fence_after();
        float s[HB];
        tmem_ld_row<HB>(tmem + sb * 16 + lane_off, s);
        // S(c) is complete and read: its K tile's slot and (flat) its TMEM buffer are free
        if (t == 0) mbar_arrive(&sm.empty[item_of_chunk(c, npb_s) % NSLOT]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free[sb]);
        if (c >= 2 && !__all_sync(0xffffffffu, mbar_wait(&sm.p_free[sb], ((c - 2) >> 1) & 1, P.err))) {
          okw = false;
          break;
        }
        bool valid;
        if (c < NCw) {
          const int key = wla + c * kDtKeys + t;
          valid = key >= wlo && key <= whi;
        }
        else if (c < NCw + NCs) valid = t < nsink;
        else valid = (c - NCw - NCs) * kDtKeys + t < nsel * geo.Bk;
        if (!bounded) {
          // chunk maxima: warp max, then the 4 warps' through shared memory
          // (an mbarrier of 4 arrivals per buffer; a warp writes buffer c & 1
          // again at chunk c + 2 only after every warp arrived for c + 1,
          // i.e. read chunk c's values)
          float cm[HB];
#pragma unroll
          for (int h = 0; h < HB; ++h) cm[h] = warp_max_f32((valid && h < G) ? s[h] * sl2 : neg_inf());
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int h = 0; h < HB; ++h) sm.cmax[sb][warp & 3][h] = cm[h];
            mbar_arrive(&sm.cm_full[sb]);
          }
          if (!__all_sync(0xffffffffu, mbar_wait(&sm.cm_full[sb], (c >> 1) & 1, P.err))) {
            okw = false;
            break;
          }
          float mn[HB];
          bool need = false;
#pragma unroll
          for (int h = 0; h < HB; ++h) {
            const float x = fmaxf(fmaxf(sm.cmax[sb][0][h], sm.cmax[sb][1][h]),
                                  fmaxf(sm.cmax[sb][2][h], sm.cmax[sb][3][h]));
            mn[h] = fmaxf(mr[h], x);
            need = need || mn[h] > mr[h] + kRescaleLog2;  // -inf + 8 = -inf: the first valid value
          }
          if (need) {  // uniform: every softmax thread computed it from the same values
            float al[HB];
#pragma unroll
            for (int h = 0; h < HB; ++h) al[h] = mr[h] == neg_inf() ? 0.f : ex2_approx(mr[h] - mn[h]);
            if (c >= 1) {
              // O^T holds PV(0 .. c-1): wait for the last one, rescale this lane's row
              if (!__all_sync(0xffffffffu, mbar_wait(&sm.p_free[(c - 1) & 1], ((c - 1) >> 1) & 1, P.err))) {
                okw = false;
                break;
              }
              tc_fence_after();
              float o[HB];
              tmem_ld_row<HB>(tmem + 32 + lane_off, o);
#pragma unroll
              for (int h = 0; h < HB; ++h) o[h] *= al[h];
              tmem_st_row<HB>(tmem + 32 + lane_off, o);
            }
#pragma unroll
            for (int h = 0; h < HB; ++h) {
              lp[h] *= al[h];
              mr[h] = mn[h];
            }
          }
        }
        unsigned char* pdst = sm.pt[sb][t >> 6];
        // branch-free over the HB head rows (rows >= HB were zeroed in the prologue)
#pragma unroll
        for (int h = 0; h < HB; ++h) {
          float pe = ex2_approx(fmaf(s[h], sl2, -mr[h]));
          pe = (valid && h < G) ? pe : 0.f;
          lp[h] += pe;
          *reinterpret_cast<__nv_bfloat16*>(pdst + sw128_offset(h, t & 63)) = f2bf(pe);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&sm.p_full[sb]);
      }
      if (t == 0) {
#pragma unroll
        for (int h = 0; h < HB; ++h) sm.mfin[h] = mr[h];
      }
      // ---- C. epilogue ----
      if (trace != nullptr && t == 0) {
        unsigned long long ts;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ts));
        trace[3] = ts;
      }
#pragma unroll
      for (int h = 0; h < HB; ++h) lp[h] = warp_sum(lp[h]);
      if (lane == 0)
#pragma unroll
        for (int h = 0; h < HB; ++h) sm.lsum[warp & 3][h] = lp[h];
      asm volatile("bar.sync 1, 128;\n" ::: "memory");  // the 4 softmax warps
      const bool have_o = __all_sync(0xffffffffu, okw && mbar_wait(&sm.o_full, 0, P.err));
      uint32_t r[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) r[h] = 0u;
      if (have_o) {
        tc_fence_after();
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
            "[%16];\n"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(tmem + 32 + lane_off));
        tmem_ld_wait();
      }
      if (fused) {
        // (O, l, M) of the owned tokens -> slot [rank] of every rank's
        // buffer; then the max-rescaled merge over the ranks' slots in rank
        // order (the same on every rank): M* = max_r M_r, w_r = 2^(M_r - M*),
        // out = sum w_r O_r / sum w_r l_r, lse = (M* + log2 sum w_r l_r) ln 2.
        // Every value is tagged with the epoch: (fp32 bits | epoch << 32).
        const size_t xs = 16 * DH + 32;
        const unsigned long long ptag = (unsigned long long)epoch << 32;
        for (int rr = 0; rr < P.world; ++rr) {
          unsigned long long* dst =
              reinterpret_cast<unsigned long long*>(P.xpeer[rr] + xl.parts) + ((size_t)bg * P.world + P.rank) * xs;
          if (t < DH) {
#pragma unroll
            for (int h = 0; h < 16; ++h)
              if (h < G)  // no owned keys: zero
                st_relaxed_sys(dst + h * DH + t, ptag | __float_as_uint(NC > 0 ? __uint_as_float(r[h]) : 0.f));
          }
          if (t < G) {
            st_relaxed_sys(dst + 16 * DH + t,
                           ptag | __float_as_uint(sm.lsum[0][t] + sm.lsum[1][t] + sm.lsum[2][t] + sm.lsum[3][t]));
            st_relaxed_sys(dst + 16 * DH + 16 + t, ptag | __float_as_uint(sm.mfin[t]));
          }
        }
        const unsigned long long* parts =
            reinterpret_cast<const unsigned long long*>(P.xpeer[P.rank] + xl.parts) + (size_t)bg * P.world * xs;
        // thread t < G: head t's (l, M) of every rank -> M*, the weights, the
        // merged l; then each thread t < DH merges its O^T row over the ranks,
        // a rank's G words at a time
        if (t < G) {
          unsigned long long wl[kShardMaxRanks], wm[kShardMaxRanks];
          wait_tagged_n<kShardMaxRanks>(parts + 16 * DH + t, xs, P.world, 32, 0xffffffffull, epoch, wl, P.err);
          wait_tagged_n<kShardMaxRanks>(parts + 16 * DH + 16 + t, xs, P.world, 32, 0xffffffffull, epoch, wm, P.err);
          float M = neg_inf();
#pragma unroll
          for (int rr = 0; rr < kShardMaxRanks; ++rr)
            if (rr < P.world) M = fmaxf(M, __uint_as_float((uint32_t)wm[rr]));
          float L = 0.f;
#pragma unroll
          for (int rr = 0; rr < kShardMaxRanks; ++rr) {
            if (rr < P.world) {
              const float mr_ = __uint_as_float((uint32_t)wm[rr]);
              const float w = (mr_ == neg_inf()) ? 0.f : ex2_approx(mr_ - M);
              sm.xw[rr][t] = w;
              L += w * __uint_as_float((uint32_t)wl[rr]);
            }
          }
          sm.xl[t] = L;
          sm.xm[t] = M;
        }
        asm volatile("bar.sync 1, 128;\n" ::: "memory");
        float O[HB];
#pragma unroll
        for (int h = 0; h < HB; ++h) O[h] = 0.f;
        if (t < DH) {
          for (int rr = 0; rr < P.world; ++rr) {
            unsigned long long w[HB];
            wait_tagged_n<HB>(parts + rr * xs + t, DH, G, 32, 0xffffffffull, epoch, w, P.err);
#pragma unroll
            for (int h = 0; h < HB; ++h)
              if (h < G) O[h] += sm.xw[rr][h] * __uint_as_float((uint32_t)w[h]);
          }
#pragma unroll
          for (int h = 0; h < HB; ++h) {
            if (h < G) {
              const float L = sm.xl[h];
              p.out[((size_t)b * geo.Hq + g * G + h) * DH + t] = f2bf(L > 0.f ? O[h] / L : 0.f);
            }
          }
        }
        if (t < G && p.lse != nullptr) {
          const float L = sm.xl[t];
          p.lse[(size_t)b * geo.Hq + g * G + t] = L > 0.f ? (sm.xm[t] + log2f(L)) * 0.6931471805599453f : neg_inf();
        }
        if (t == 0) stamp_any(13);
      } else if (have_o) {
        if (P.mode == 1) {  // unnormalised partial of the owned tokens and its reference max
          if (t < DH) {
#pragma unroll
            for (int h = 0; h < 16; ++h)
              if (h < G)  // no owned keys: O^T was never written
                P.part_o[((size_t)b * geo.Hq + g * G + h) * DH + t] = NC > 0 ? __uint_as_float(r[h]) : 0.f;
          }
          if (t < G) {
            const float L = sm.lsum[0][t] + sm.lsum[1][t] + sm.lsum[2][t] + sm.lsum[3][t];
            P.part_l[(size_t)b * geo.Hq + g * G + t] = L;
            P.part_m2[(size_t)b * geo.Hq + g * G + t] = sm.mfin[t];
          }
        } else {
          if (t < DH) {
#pragma unroll
            for (int h = 0; h < 16; ++h) {
              if (h < G) {
                const float L = sm.lsum[0][h] + sm.lsum[1][h] + sm.lsum[2][h] + sm.lsum[3][h];
                const float O = __uint_as_float(r[h]);
                p.out[((size_t)b * geo.Hq + g * G + h) * DH + t] = f2bf(L > 0.f ? O / L : 0.f);
              }
            }
          }
          if (t < G && p.lse != nullptr) {
            const float L = sm.lsum[0][t] + sm.lsum[1][t] + sm.lsum[2][t] + sm.lsum[3][t];
            p.lse[(size_t)b * geo.Hq + g * G + t] = L > 0.f ? (sm.mfin[t] + log2f(L)) * 0.6931471805599453f : neg_inf();
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 64);
  stamp(4);
}

// ---------------------------------------------------------------- host ----
bool decode_tc_supported(const Geom& geo, int dh, const void* k, const void* kr, const void* v, const void* summ,
                         const void* supers) {
  // 1-D bulk copies start on 16-byte boundaries
  const bool aligned = ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(kr) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(summ) |
                         reinterpret_cast<uintptr_t>(geo.hier ? supers : summ)) & 15u) == 0;
  return (dh == 64 || dh == 128) && geo.Bk == 64 && geo.n_cap % 64 == 0 && geo.m >= 1 &&
         128 % geo.m == 0 && geo.G <= 16 && geo.nb_cap <= kTopkMaxItems &&
         (!geo.hier || (geo.ns_cap <= kTopkMaxItems && geo.beam * geo.F <= kTopkMaxItems)) && aligned;
}

template <int DH, int HB>
static cudaError_t launch_dtc_t(const DecodeTcParams& P, cudaStream_t st) {
  const size_t smem = sizeof(DtcSmem<DH>) + 1024;
  static const cudaError_t attr =
      cudaFuncSetAttribute(decode_tc_kernel<DH, HB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (attr != cudaSuccess) return attr;
  decode_tc_kernel<DH, HB><<<P.a.geo.B * P.a.geo.Hkv, kDtThreads, smem, st>>>(P);
  return cudaGetLastError();
}

static cudaError_t launch_dtc(DecodeTcParams P, int dh, cudaStream_t st) {
  const Geom& geo = P.a.geo;
  if (geo.n_cap % 64 != 0) return cudaErrorInvalidValue;  // whole 64-token tiles
  // softmax head rows: 8 when the group fits, else all 16 of the MMA's N
  if (dh == 64) return geo.G <= 8 ? launch_dtc_t<64, 8>(P, st) : launch_dtc_t<64, 16>(P, st);
  return geo.G <= 8 ? launch_dtc_t<128, 8>(P, st) : launch_dtc_t<128, 16>(P, st);
}


cudaError_t launch_decode_tc(const DecodeAttnParams& p, const __nv_bfloat16* summ, const __nv_bfloat16* supers,
                             const float* k_gain, int* err, int dh, cudaStream_t st) {
  DecodeTcParams P{};
  P.a = p;
  P.summ = summ;
  P.supers = supers;
  P.k_gain = k_gain;
  P.err = err;
  P.mode = 0;
  return launch_dtc(P, dh, st);
}

cudaError_t launch_decode_tc_shard(const DecodeAttnParams& p, const float* k_gain, int* err, int dh, int tok_lo,
                                   const int32_t* in_idx, const float* in_score, int n_in, float* part_o,
                                   float* part_l, float* part_m2, cudaStream_t st) {
  DecodeTcParams P{};
  P.a = p;
  P.k_gain = k_gain;
  P.err = err;
  P.mode = 1;
  P.tok_lo = tok_lo;
  P.n_in = n_in;
  P.in_idx = in_idx;
  P.in_score = in_score;
  P.part_o = part_o;
  P.part_l = part_l;
  P.part_m2 = part_m2;
  return launch_dtc(P, dh, st);
}

__global__ void epoch_bump_kernel(int32_t* epoch) { *epoch += 1; }

cudaError_t launch_decode_tc_fused(const DecodeAttnParams& p, const __nv_bfloat16* summ, const __nv_bfloat16* supers,
                                   const float* k_gain, int* err, int dh, int tok_lo, int world, int rank,
                                   int32_t* epoch, void* const* xbufs, cudaStream_t st) {
  if (world < 1 || world > kShardMaxRanks || rank < 0 || rank >= world) return cudaErrorInvalidValue;
  epoch_bump_kernel<<<1, 1, 0, st>>>(epoch);  // this step's epoch, the same count on every rank
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  DecodeTcParams P{};
  P.a = p;
  P.summ = summ;
  P.supers = supers;
  P.k_gain = k_gain;
  P.err = err;
  P.mode = 2;
  P.tok_lo = tok_lo;
  P.world = world;
  P.rank = rank;
  P.epoch = epoch;
  for (int r = 0; r < world; ++r) P.xpeer[r] = static_cast<unsigned char*>(xbufs[r]);
  return launch_dtc(P, dh, st);
}

// The max-rescaled merge of the ranks' partials (gathered rank-major, per
// rank [m | l | O] over `rows` = B * Hq rows): M = max_r m_r,
// w_r = 2^(m_r - M), out = sum_r w_r O_r / sum_r w_r l_r (bf16),
// lse = (M + log2 sum_r w_r l_r) ln 2, summed in rank order.
__global__ void __launch_bounds__(128) shard_finish_kernel(int rows, int dh, int world,
                                                           const float* __restrict__ parts,
                                                           __nv_bfloat16* __restrict__ out, float* __restrict__ lse) {
  const size_t row = blockIdx.x;
  const size_t stride = (size_t)rows * (dh + 2);  // one rank's partials
  float M = neg_inf();
  for (int r = 0; r < world; ++r) M = fmaxf(M, parts[r * stride + row]);
  float L = 0.f;
  for (int r = 0; r < world; ++r) {
    const float m = parts[r * stride + row];
    if (m != neg_inf()) L += ex2_approx(m - M) * parts[r * stride + rows + row];
  }
  for (int d = threadIdx.x; d < dh; d += blockDim.x) {
    float o = 0.f;
    for (int r = 0; r < world; ++r) {
      const float m = parts[r * stride + row];
      if (m != neg_inf()) o += ex2_approx(m - M) * parts[r * stride + 2 * (size_t)rows + row * dh + d];
    }
    out[row * dh + d] = f2bf(L > 0.f ? o / L : 0.f);
  }
  if (threadIdx.x == 0 && lse != nullptr) lse[row] = L > 0.f ? (M + log2f(L)) * 0.6931471805599453f : neg_inf();
}

cudaError_t launch_shard_finish(int rows, int dh, int world, const float* parts, __nv_bfloat16* out, float* lse,
                                cudaStream_t st) {
  shard_finish_kernel<<<rows, 128, 0, st>>>(rows, dh, world, parts, out, lse);
  return cudaGetLastError();
}

}  // namespace hba
