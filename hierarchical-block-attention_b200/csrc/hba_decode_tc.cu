// Decode on the 5th-generation tensor cores: one CTA per (sequence, kv head)
// does the selection on CUDA cores and the union softmax with tcgen05 MMAs
// whose accumulators live in TMEM, K/V tiles fed by TMA.  Used with QKNorm
// (the logit bound below needs it); other configurations use the mma.sync
// fused kernel.
//
// The G query heads of a KV group are few (4-16), so the MMAs are swapped:
// keys are the M dimension.  For a 128-key chunk
//     S^T[128 keys x 16] = K[128 x dh] . Q^T          (A = K, B = Q, K-major)
//     O^T[dh x 16]      += V^T[dh x 128] . P^T         (A = V^T MN-major, B = P^T)
// One softmax thread per key reads its 16 head scores from TMEM and writes
// p = exp2(s*scale*log2e - M2[h]) into P^T.  M2[h] is a per-head upper bound
// of the logits (QKNorm: |s| <= scale*|q_h|*sqrt(dh)*k_gain), so there is no
// running max and O^T is never rescaled; l[h] are per-thread partial sums
// reduced once at the end.
//
// Phases:
//  A (all 8 warps) query prologue; TMA of the first window chunks issued at
//    once (they need no selection); summary pages stream through a 2-page
//    cp.async ring and are scored; block-wide radix-select top-k (flat, or
//    supers then children for the hierarchical beam).
//  B (roles) warp 0: TMA producer of the K/V ring [window | sinks | routed
//    block pairs]; warp 1: TMEM owner and single-thread MMA issuer;
//    warps 4-7: softmax (TMEM lane quarter = warp % 4); warps 2-3 idle.
//  C warps 4-7 reduce l, read O^T from TMEM, write out, LSE, the picks.
// Reference semantics: src/hba/attention.py:663-711 at cs = n-1.
#include <climits>
#include <cudaTypedefs.h>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_score.cuh"
#include "hba_sm100.cuh"
#include "hba_topk.cuh"

namespace hba {

using namespace sm100;

constexpr int kDtThreads = 256;
constexpr int kDtWarps = 8;
constexpr int kDtKeys = 128;  // keys per chunk (UMMA M)

template <int DH>
struct DtcSmem {
  static constexpr int HALVES = DH / 64;
  static constexpr int KT = kDtKeys * DH * 2;               // one K or V tile
  static constexpr int NKV = DH == 64 ? 3 : 2;              // K/V ring stages
  static constexpr int PAGE = DH == 64 ? 32768 : 16384;     // summary page bytes
  alignas(1024) unsigned char kv[NKV][2][KT];               // [stage][K|V], halves of [128 x 64] SW128
  static constexpr int NPG = 3;                             // summary page ring
  alignas(1024) unsigned char pages[NPG][PAGE];
  alignas(1024) unsigned char qc[HALVES][16 * 128];         // Q rows (16 heads) [16 x 64] SW128 per half
  alignas(1024) unsigned char qr[HALVES][16 * 128];
  alignas(1024) unsigned char pt[2][2][16 * 128];           // P^T [buffer][key half][16 heads x 64 keys]
  float qg[DH];
  float m2[16];
  float lsum[4][16];
  float sc[kTopkMaxItems];
  int id[kTopkMaxItems];
  TopkScratch ts;
  int blocks[32];
  int sup_lo[32], sup_off[32], sup_cnt[32];
  int n_children;
  uint64_t kv_full[NKV], kv_empty[NKV];
  uint64_t s_full[2], p_full[2], p_free[2];
  uint64_t o_full, drain;
  uint32_t tmem_base;
};

struct DecodeTcParams {
  DecodeAttnParams a;
  const __nv_bfloat16* summ;
  const __nv_bfloat16* supers;
  const float* k_gain;
  int* err;
};

template <int DH, int VPL>
__global__ void __launch_bounds__(kDtThreads, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tm_kc, const __grid_constant__ CUtensorMap tm_kr,
                     const __grid_constant__ CUtensorMap tm_v, DecodeTcParams P) {
  using SM = DtcSmem<DH>;
  constexpr int HALVES = SM::HALVES;
  constexpr int NKV = SM::NKV;
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
  const bool hier = geo.hier != 0;
  unsigned long long* trace = (p.trace != nullptr && bg < p.trace_ctas) ? p.trace + (size_t)bg * 8 : nullptr;
  auto stamp = [&](int i) {
    if (trace != nullptr && tid == 0) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      trace[i] = t;
    }
  };
  stamp(0);

  const int nctx = p.qp.seq_lens[b];
  const float scale = p.qp.scales[b];
  const bool ok = nctx >= 1 && nctx <= geo.n_cap;
  const int pos = ok ? nctx - 1 : -1;
  const int nb = ok ? nctx / geo.Bk : 0;
  const int bmax = ok ? min(last_candidate(pos, geo.W, geo.Bk), nb - 1) : 0;
  int kfinal = min(geo.K, nb);
  const int ns = (nb + geo.F - 1) / geo.F;
  if (hier) kfinal = min(kfinal, min(geo.beam, ns) * geo.F);
  const int w0 = max(geo.S, pos - geo.W + 1);
  const int nw = ok ? max(0, pos - w0 + 1) : 0;
  const int nsink = ok ? min(geo.S, pos + 1) : 0;
  const int NCw = (nw + kDtKeys - 1) / kDtKeys;
  const int NCs = nsink > 0 ? 1 : 0;

  // ---- barriers, TMEM ----
  if (tid == 0) {
    for (int s = 0; s < NKV; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 128);
      mbar_init(&sm.p_free[s], 1);
    }
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.drain, 1);
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

  // K/V chunk c -> (kind, token of its first / second 64-row half)
  int nsel = 0, NCr = 0;
  auto chunk_src = [&](int c, int& kind, int& t0, int& t1) {
    if (c < NCw) {
      kind = 0;
      t0 = w0 + c * kDtKeys;
      t1 = t0 + 64;
    } else if (c < NCw + NCs) {
      kind = 1;
      t0 = 0;
      t1 = 64;
    } else {
      kind = 2;
      const int i = (c - NCw - NCs) * 2;
      t0 = sm.blocks[i] * 64;
      t1 = (i + 1 < nsel ? sm.blocks[i + 1] : sm.blocks[i]) * 64;  // odd count: reload a valid block (masked)
    }
  };
  int issued = 0;  // producer thread only
  auto produce = [&](int upto) {  // issue chunks [issued, upto) into the ring (warp 0, lane 0)
    for (; issued < upto; ++issued) {
      const int c = issued, st = c % NKV, u = c / NKV;
      if (c >= NKV && !mbar_wait(&sm.kv_empty[st], (u - 1) & 1, P.err)) return;
      int kind, t0, t1;
      chunk_src(c, kind, t0, t1);
      mbar_arrive_expect_tx(&sm.kv_full[st], 2 * SM::KT);
      const CUtensorMap* km = kind == 0 ? &tm_kr : &tm_kc;
#pragma unroll
      for (int h = 0; h < HALVES; ++h) {
        unsigned char* kd = sm.kv[st][0] + h * (kDtKeys * 128);
        unsigned char* vd = sm.kv[st][1] + h * (kDtKeys * 128);
        tma_load_4d(kd, km, h * 64, g, t0, b, &sm.kv_full[st]);
        tma_load_4d(kd + 64 * 128, km, h * 64, g, t1, b, &sm.kv_full[st]);
        tma_load_4d(vd, &tm_v, h * 64, g, t0, b, &sm.kv_full[st]);
        tma_load_4d(vd + 64 * 128, &tm_v, h * 64, g, t1, b, &sm.kv_full[st]);
      }
    }
  };
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_kc);
    prefetch_tmap(&tm_kr);
    prefetch_tmap(&tm_v);
    produce(min(NKV, NCw + NCs));  // window/sink chunks need no selection
  }

  // ---- A.1 query prologue: Q rows (SW128), qg, per-head logit bounds ----
  for (int h = warp; h < 16; h += kDtWarps) {
    float v[PER], r[PER];
    float qn2 = 0.f;
    if (h < G && ok) {
      const int hq = g * G + h;
      float cr[PER], sr[PER];  // issued together with the query load
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        cr[i] = p.cos[(size_t)pos * DH + lane * PER + i];
        sr[i] = p.sin[(size_t)pos * DH + lane * PER + i];
      }
      load_head_row<DH>(p.q + ((size_t)b * geo.Hq + hq) * DH, v);
      qknorm_lane<DH>(v, p.q_gain[hq], geo.eps);
      const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
        r[i] = v[i] * cr[i] + sign * partner * sr[i];
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
      const float kmax = sqrtf((float)DH) * P.k_gain[g] * (1.f + 1.f / 64.f);
      const float m2 = scale * sqrtf(qn2) * kmax * kLog2e;
      sm.m2[h] = (h < G && ok) ? m2 : 0.f;
      if (m2 > 120.f) atomicExch(P.err, 2);
    }
  }
  __syncthreads();
  for (int d = tid; d < DH; d += kDtThreads) {
    float acc = 0.f;
    for (int h = 0; h < G; ++h) {
      acc += bf2f(*reinterpret_cast<const __nv_bfloat16*>(sm.qc[d / 64] + sw128_offset(h, d % 64)));
    }
    sm.qg[d] = round_bf16(acc);
  }
  fence_proxy_async_smem();  // Q tiles are read by the tensor cores
  __syncthreads();
  stamp(1);

  // ---- A.2 selection: summary pages through a 2-page cp.async ring ----
  const int row_bytes = geo.m * DH * 2;
  const int row_pieces = row_bytes / 16;
  const int PB = SM::PAGE / row_bytes;
  const __nv_bfloat16* summ_bg = P.summ + (size_t)bg * geo.nb_cap * geo.m * DH;
  const __nv_bfloat16* sup_bg = hier ? P.supers + (size_t)bg * geo.ns_cap * geo.m * DH : nullptr;
  const int nvec = row_pieces;
  constexpr int LPS = DH / 8;
  auto child_id = [&](int j) -> int {
    int si = 0;
    while (si < 31 && j >= sm.sup_off[si] + sm.sup_cnt[si]) ++si;
    return sm.sup_lo[si] + (j - sm.sup_off[si]);
  };
  // scores candidates [0, R): id_fn(j) is the candidate's row in `rows`.
  // Each warp scores 4 rows at a time with the per-row arithmetic of
  // SummaryLoads::score (hba_score.cuh), so every decode path selects from
  // bit-identical scores.
  float qgr[VPL][8];
  auto load_qg = [&]() {
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int d0 = ((lane + 32 * v) * 8) % DH;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) qgr[v][jj] = sm.qg[d0 + jj];
    }
  };
  auto score_phase = [&](const __nv_bfloat16* rows, int R, auto id_fn) {
    constexpr int NPG = SM::NPG;
    const int np = (R + PB - 1) / PB;
    auto issue_page = [&](int pg) {
      if (pg < np) {
        const int nr = min(PB, R - pg * PB);
        unsigned char* dst = sm.pages[pg % NPG];
        for (int e = tid; e < nr * row_pieces; e += kDtThreads) {
          const int r = e / row_pieces, pc = e % row_pieces;
          cp_async16(dst + r * row_bytes + pc * 16, rows + (size_t)id_fn(pg * PB + r) * geo.m * DH + pc * 8);
        }
      }
      cp_async_commit();
    };
    for (int pg = 0; pg < NPG - 1; ++pg) issue_page(pg);
    for (int pg = 0; pg < np; ++pg) {
      issue_page(pg + NPG - 1);
      cp_async_wait<NPG - 1>();
      __syncthreads();
      const unsigned char* src = sm.pages[pg % NPG];
      const int nr = min(PB, R - pg * PB);
      for (int r0 = warp * 4; r0 < nr; r0 += kDtWarps * 4) {
        float part[4][VPL];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int v = 0; v < VPL; ++v) {
            const int vv = lane + 32 * v;
            part[u][v] = 0.f;
            if (r0 + u < nr && vv < nvec) {
              float f[8];
              unpack8(*reinterpret_cast<const uint4*>(src + (r0 + u) * row_bytes + vv * 16), f);
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) part[u][v] = fmaf(f[jj], qgr[v][jj], part[u][v]);
            }
          }
#pragma unroll
        for (int ox = 1; ox < LPS; ox <<= 1)
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int v = 0; v < VPL; ++v) part[u][v] += __shfl_xor_sync(0xffffffffu, part[u][v], ox);
        float best[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          best[u] = neg_inf();
#pragma unroll
          for (int v = 0; v < VPL; ++v)
            if (lane + 32 * v < nvec) best[u] = fmaxf(best[u], part[u][v]);
        }
#pragma unroll
        for (int ox = 16; ox > 0; ox >>= 1)
#pragma unroll
          for (int u = 0; u < 4; ++u) best[u] = fmaxf(best[u], __shfl_xor_sync(0xffffffffu, best[u], ox));
        if (lane == 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (r0 + u < nr) {
              const int j = pg * PB + r0 + u;
              sm.sc[j] = best[u] * scale;
              sm.id[j] = id_fn(j);
            }
        }
      }
      __syncthreads();
    }
    cp_async_wait<0>();
  };
  load_qg();
  if (!hier) {
    const int R = max(0, bmax);
    score_phase(summ_bg, R, [&](int j) { return 1 + j; });
    stamp(5);
    nsel = block_topk<kDtThreads>(sm.sc, sm.id, R, kfinal, sm.ts);
    stamp(6);
  } else {
    int R1 = 0, s_lo = 0;
    if (bmax >= 1) {
      s_lo = (geo.F == 1) ? 1 : 0;
      R1 = bmax / geo.F - s_lo + 1;
    }
    score_phase(sup_bg, R1, [&](int j) { return s_lo + j; });
    stamp(5);
    const int nsup = block_topk<kDtThreads>(sm.sc, sm.id, R1, min(geo.beam, ns), sm.ts);
    if (warp == 0) {
      const bool valid = lane < nsup;
      int lo = 0, cnt = 0;
      if (valid) {
        const int sidx = sm.ts.sel_idx[lane];
        lo = max(1, sidx * geo.F);
        cnt = max(0, min(bmax, sidx * geo.F + geo.F - 1) - lo + 1);
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
    }
    __syncthreads();
    const int R2 = sm.n_children;
    stamp(6);
    score_phase(summ_bg, R2, [&](int j) { return child_id(j); });
    stamp(7);
    nsel = block_topk<kDtThreads>(sm.sc, sm.id, R2, kfinal, sm.ts);
  }
  if (tid < 32) {
    const bool valid = tid < nsel;
    sm.blocks[tid] = valid ? sm.ts.sel_idx[tid] : 0;
    if (p.sel_idx != nullptr && tid < geo.K) {
      p.sel_idx[(size_t)bg * geo.K + tid] = valid ? sm.ts.sel_idx[tid] : -1;
      p.sel_score[(size_t)bg * geo.K + tid] = valid ? sm.ts.sel_score[tid] : neg_inf();
    }
  }
  __syncthreads();
  NCr = (nsel * geo.Bk + kDtKeys - 1) / kDtKeys;
  const int NC = NCw + NCs + NCr;
  stamp(2);

  // ---- B. union softmax ----
  if (warp == 0) {
    if (lane == 0) produce(NC);
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(128, 16, false, false);
      constexpr uint32_t idesc_o = idesc_bf16(128, 16, true, false);
      bool okw = true;
      auto pv = [&](int c) -> bool {
        const int sb = c & 1, st = c % NKV;
        if (!mbar_wait(&sm.p_full[sb], (c >> 1) & 1, P.err)) return false;
        tc_fence_after();
        const uint32_t va = smem_u32(sm.kv[st][1]);
        const uint32_t pa = smem_u32(sm.pt[sb][0]);
        // dh 64: M = 128 reads a second MN group at LBO 0 (rows 64-127 of O^T duplicate 0-63, unused)
        const uint32_t lbo = DH == 128 ? kDtKeys * 128 : 0;
#pragma unroll
        for (int kk = 0; kk < kDtKeys / 16; ++kk)
          umma_f16(tmem + 32, sdesc_sw128(va + kk * 2048, lbo, 1024),
                   sdesc_sw128(pa + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), idesc_o,
                   (c > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&sm.kv_empty[st]);
        umma_commit(&sm.p_free[sb]);
        return true;
      };
      for (int c = 0; okw && c < NC; ++c) {
        const int st = c % NKV, sb = c & 1;
        if (!mbar_wait(&sm.kv_full[st], (c / NKV) & 1, P.err)) {
          okw = false;
          break;
        }
        tc_fence_after();
        const bool window = c < NCw;
        const uint32_t ka = smem_u32(sm.kv[st][0]);
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const int h = kk >> 2, ko = (kk & 3) * 32;
          const uint32_t qa = smem_u32(window ? sm.qr[h] : sm.qc[h]);
          umma_f16(tmem + sb * 16, sdesc_sw128(ka + h * (kDtKeys * 128) + ko, 16, 1024),
                   sdesc_sw128(qa + ko, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full[sb]);
        if (c >= 1 && !pv(c - 1)) {
          okw = false;
          break;
        }
      }
      if (okw && NC >= 1) okw = pv(NC - 1);
      umma_commit(&sm.o_full);
      umma_commit(&sm.drain);
      mbar_wait(&sm.drain, 0, P.err);
    }
  } else if (warp >= 4) {
    const int t = tid - 128;  // key row of the chunk / TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const float sl2 = scale * kLog2e;
    float lp[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) lp[h] = 0.f;
    float m2[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) m2[h] = sm.m2[h];
    bool okw = true;
    for (int c = 0; c < NC; ++c) {
      const int sb = c & 1;
      if (!mbar_wait(&sm.s_full[sb], (c >> 1) & 1, P.err)) {
        okw = false;
        break;
      }
      tc_fence_after();
      float s[16];
      {
        uint32_t r[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
            "[%16];\n"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(tmem + sb * 16 + lane_off));
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 16; ++h) s[h] = __uint_as_float(r[h]);
      }
      if (c >= 2 && !mbar_wait(&sm.p_free[sb], ((c - 2) >> 1) & 1, P.err)) {
        okw = false;
        break;
      }
      bool valid;
      if (c < NCw) valid = w0 + c * kDtKeys + t <= pos;
      else if (c < NCw + NCs) valid = t < nsink;
      else valid = (c - NCw - NCs) * kDtKeys + t < nsel * geo.Bk;
      unsigned char* pdst = sm.pt[sb][t >> 6];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float pe = (valid && h < G) ? exp2f(fmaf(s[h], sl2, -m2[h])) : 0.f;
        lp[h] += pe;
        *reinterpret_cast<__nv_bfloat16*>(pdst + sw128_offset(h, t & 63)) = f2bf(pe);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.p_full[sb]);
    }
    // ---- C. epilogue ----
    if (trace != nullptr && t == 0) {
      unsigned long long ts;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ts));
      trace[3] = ts;
    }
#pragma unroll
    for (int h = 0; h < 16; ++h) lp[h] = warp_sum(lp[h]);
    if (lane == 0)
#pragma unroll
      for (int h = 0; h < 16; ++h) sm.lsum[warp & 3][h] = lp[h];
    asm volatile("bar.sync 1, 128;\n" ::: "memory");  // the 4 softmax warps
    if (okw && mbar_wait(&sm.o_full, 0, P.err)) {
      tc_fence_after();
      uint32_t r[16];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
          "[%16];\n"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
            "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
          : "r"(tmem + 32 + lane_off));
      tmem_ld_wait();
      if (t < DH) {
        for (int h = 0; h < G; ++h) {
          const float L = sm.lsum[0][h] + sm.lsum[1][h] + sm.lsum[2][h] + sm.lsum[3][h];
          const float O = __uint_as_float(r[h]);
          p.out[((size_t)b * geo.Hq + g * G + h) * DH + t] = f2bf(L > 0.f ? O / L : 0.f);
        }
      }
      if (t < G && p.lse != nullptr) {
        const float L = sm.lsum[0][t] + sm.lsum[1][t] + sm.lsum[2][t] + sm.lsum[3][t];
        p.lse[(size_t)b * geo.Hq + g * G + t] = L > 0.f ? (sm.m2[t] + log2f(L)) * 0.6931471805599453f : neg_inf();
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
static PFN_cuTensorMapEncodeTiled_v12000 dtc_encode_fn() {
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

static bool dtc_map(CUtensorMap* m, const void* base, int B, int n, int H, int dh) {
  auto fn = dtc_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[4] = {(cuuint64_t)dh, (cuuint64_t)H, (cuuint64_t)n, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)dh * 2, (cuuint64_t)H * dh * 2, (cuuint64_t)n * H * dh * 2};
  cuuint32_t box[4] = {64, 1, 64, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool decode_tc_supported(const Geom& geo, int dh, const void* k, const void* kr, const void* v) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(kr) |
                         reinterpret_cast<uintptr_t>(v)) & 15u) == 0;
  return geo.qknorm && (dh == 64 || dh == 128) && geo.Bk == 64 && geo.G <= 16 && geo.nb_cap <= kTopkMaxItems &&
         (!geo.hier || (geo.ns_cap <= kTopkMaxItems && geo.beam * geo.F <= kTopkMaxItems)) && aligned &&
         dtc_encode_fn() != nullptr;
}

template <int DH, int VPL>
static cudaError_t launch_dtc_t(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c,
                                const DecodeTcParams& P, cudaStream_t st) {
  const size_t smem = sizeof(DtcSmem<DH>) + 1024;
  static const cudaError_t attr =
      cudaFuncSetAttribute(decode_tc_kernel<DH, VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (attr != cudaSuccess) return attr;
  decode_tc_kernel<DH, VPL><<<P.a.geo.B * P.a.geo.Hkv, kDtThreads, smem, st>>>(a, b, c, P);
  return cudaGetLastError();
}

cudaError_t launch_decode_tc(const DecodeAttnParams& p, const __nv_bfloat16* summ, const __nv_bfloat16* supers,
                             const float* k_gain, int* err, int dh, cudaStream_t st) {
  CUtensorMap m_kc, m_kr, m_v;
  const Geom& geo = p.geo;
  if (!dtc_map(&m_kc, p.k, geo.B, geo.n_cap, geo.Hkv, dh) || !dtc_map(&m_kr, p.kr, geo.B, geo.n_cap, geo.Hkv, dh) ||
      !dtc_map(&m_v, p.v, geo.B, geo.n_cap, geo.Hkv, dh))
    return cudaErrorInvalidValue;
  DecodeTcParams P{p, summ, supers, k_gain, err};
  const int vpl = (geo.m * dh / 8 + 31) / 32;
  if (dh == 64) {
    if (vpl <= 1) return launch_dtc_t<64, 1>(m_kc, m_kr, m_v, P, st);
    return launch_dtc_t<64, 2>(m_kc, m_kr, m_v, P, st);
  }
  if (vpl <= 1) return launch_dtc_t<128, 1>(m_kc, m_kr, m_v, P, st);
  if (vpl <= 2) return launch_dtc_t<128, 2>(m_kc, m_kr, m_v, P, st);
  return launch_dtc_t<128, 4>(m_kc, m_kr, m_v, P, st);
}

}  // namespace hba
