// Fused decode: selection and the union softmax in one kernel, one CTA per
// (sequence, kv head) -- the large-batch decode path.  Nothing goes through
// global scratch: the CTA scores the candidate summaries, selects the top-k
// and gathers the selected blocks itself.
//
// Per CTA (256 threads = 8 warps):
//   1. the first K/V chunks of the RoPE window (cp.async, from the RoPE'd key
//      cache) are put in flight -- they depend neither on the query nor on the
//      selection;
//   2. query prologue: the G heads QKNorm'd (qc) and RoPE'd (qr) into shared
//      memory; routing query qg = bf16(sum of the bf16 qc heads, fp32, in
//      head order) (reference src/hba/summarizer.py:50-54);
//   3. scoring: every candidate block summary (flat), or the super-summaries
//      then the beam's children (hierarchical, attention.py:217-246), 8
//      16-byte loads in flight per lane; scores max_slot(qg . S) * scale;
//   4. block-wide radix-select top-k (score desc, block index asc);
//   5. union softmax over 128-key chunks [window | sinks | routed blocks],
//      each warp 16 keys per chunk on m16n8k16 bf16 tensor-core tiles (the G
//      heads are the 16 rows), online softmax in the log2 domain;
// Steps 3 and 5 share one cp.async ring (5 stages of 32 KB for dh 64, 3 of
// 64 KB for dh 128): summary pages, window chunks, the beam's child pages,
// the sink chunk and the routed chunks stream through it in that order, so
// ~128 KB stay in flight per CTA and the top-k runs while the window loads
// are already landing.
//   6. warps merge (max, sum, O); the CTA writes out, the natural-log LSE and
//      the selected blocks.
#include <climits>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_score.cuh"
#include "hba_topk.cuh"

namespace hba {

constexpr int kFThreads = 256;
constexpr int kFWarps = kFThreads / 32;
constexpr int kFChunk = 128;  // keys per K/V chunk: 8 warps x 16

// One ring stage holds a K/V chunk [2][128 keys][DH] or a page of summary rows.
template <int DH>
struct FusedCfg {
  static constexpr int kStageBytes = 2 * kFChunk * DH * 2;  // 32 KB (dh 64) / 64 KB (dh 128)
  static constexpr int kStages = DH == 64 ? 5 : 3;
};

template <int DH>
struct FusedSmem {
  alignas(128) unsigned char ring[FusedCfg<DH>::kStages][FusedCfg<DH>::kStageBytes];
  __nv_bfloat16 qc[16][DH + 8];
  __nv_bfloat16 qr[16][DH + 8];
  float qg[DH];
  float sc[kTopkMaxItems];
  int id[kTopkMaxItems];
  TopkScratch ts;
  int blocks[32];
  int sup_lo[32], sup_off[32], sup_cnt[32];
  int n_children;
};

template <int DH>
struct FusedCombine {  // overlays the ring after the item loop
  float m[kFWarps][16];
  float l[kFWarps][16];
  float o[kFWarps][16][DH];
};

// byte offset of (row, 16-byte piece) in a swizzled [rows x DH] bf16 tile
template <int DH>
HBA_DEVICE uint32_t swz(int row, int piece) {
  return (uint32_t)(row * DH * 2 + ((piece ^ (row & 7)) << 4));
}

HBA_DEVICE void cp_async_wait_dyn(int pending) {
  switch (pending) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    default: cp_async_wait<4>(); break;
  }
}

enum FusedItem : int { kPageScore = 0, kPageChild = 1, kChunkWindow = 2, kChunkSink = 3, kChunkRouted = 4 };

template <int DH, int VPL>
__global__ void __launch_bounds__(kFThreads, 1) decode_fused_kernel(DecodeAttnParams p, const __nv_bfloat16* summ,
                                                                    const __nv_bfloat16* supers) {
  using FC = FusedCfg<DH>;
  constexpr int NS = FC::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  FusedSmem<DH>& sm = *reinterpret_cast<FusedSmem<DH>*>(smem_raw);
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  constexpr int PER = DH / 32;
  constexpr int PIECES = DH / 8;
  const int G = geo.G;
  const int bg = blockIdx.x;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const bool hier = geo.hier != 0;

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
  const size_t head_base = ((size_t)b * geo.Hkv + g) * (size_t)geo.n_cap * DH;  // the chunk-tiled cache
  const __nv_bfloat16* kbase = p.k + head_base;
  const __nv_bfloat16* krbase = p.kr + head_base;
  const __nv_bfloat16* vbase = p.v + head_base;
  const int row_bytes = geo.m * DH * 2;                 // one summary row
  const int row_pieces = row_bytes / 16;
  const int PB = FC::kStageBytes / row_bytes;           // summary rows per page
  const __nv_bfloat16* summ_bg = summ + (size_t)bg * geo.nb_cap * geo.m * DH;
  const __nv_bfloat16* sup_bg = hier ? supers + (size_t)bg * geo.ns_cap * geo.m * DH : nullptr;

  // ---- item counts (later ones become known at the top-k points) ----
  int R1 = 0, id_lo = 1;  // first scoring phase: candidate blocks (flat) or supers (hier)
  if (!hier) {
    R1 = max(0, bmax);
  } else if (bmax >= 1) {
    id_lo = (geo.F == 1) ? 1 : 0;
    R1 = bmax / geo.F - id_lo + 1;
  }
  const int P1 = (R1 + PB - 1) / PB;
  const int NCw = (nw + kFChunk - 1) / kFChunk;
  const int NCs = nsink > 0 ? 1 : 0;
  int R2 = 0, P2 = 0;    // hier: children of the selected supers
  int nsel = 0, NCr = 0;
  bool phase1_done = false, final_done = false;

  // item order: [phase-1 pages | window | child pages | sink | routed]
  auto kind_of = [&](int it, int& idx) -> int {
    if (it < P1) { idx = it; return kPageScore; }
    it -= P1;
    if (it < NCw) { idx = it; return kChunkWindow; }
    it -= NCw;
    if (it < P2) { idx = it; return kPageChild; }
    it -= P2;
    if (it < NCs) { idx = it; return kChunkSink; }
    idx = it - NCs;
    return kChunkRouted;
  };
  auto issuable = [&](int kind) -> bool {
    if (kind == kPageChild) return phase1_done;
    if (kind == kChunkSink || kind == kChunkRouted) return final_done;  // item positions need P2 (hier)
    return true;
  };
  auto child_id = [&](int j) -> int {
    int si = 0;
    while (si < 31 && j >= sm.sup_off[si] + sm.sup_cnt[si]) ++si;
    return sm.sup_lo[si] + (j - sm.sup_off[si]);
  };
  auto chunk_rows = [&](int kind, int idx) -> int {
    if (kind == kChunkWindow) return min(kFChunk, nw - idx * kFChunk);
    if (kind == kChunkSink) return nsink;
    return max(0, min(kFChunk, nsel * geo.Bk - idx * kFChunk));
  };
  auto page_rows = [&](int kind, int idx) -> int {
    const int R = kind == kPageScore ? R1 : R2;
    return min(PB, R - idx * PB);
  };
  auto issue = [&](int it, int stage) {
    int idx;
    const int kind = kind_of(it, idx);
    unsigned char* st = sm.ring[stage];
    if (kind == kPageScore || kind == kPageChild) {
      const int rows = page_rows(kind, idx);
      for (int e = tid; e < rows * row_pieces; e += kFThreads) {
        const int r = e / row_pieces, pc = e % row_pieces;
        const int j = idx * PB + r;
        const __nv_bfloat16* src;
        if (kind == kPageScore) src = (hier ? sup_bg : summ_bg) + (size_t)(id_lo + j) * geo.m * DH;
        else src = summ_bg + (size_t)child_id(j) * geo.m * DH;
        cp_async16(st + r * row_bytes + pc * 16, src + pc * 8);
      }
    } else {
      const int cnt = chunk_rows(kind, idx);
      const __nv_bfloat16* ksrc = kind == kChunkWindow ? krbase : kbase;
      for (int e = tid; e < kFChunk * PIECES; e += kFThreads) {
        const int r = e / PIECES, pc = e % PIECES;
        const bool valid = r < cnt;
        int tok = 0;
        if (valid) {
          if (kind == kChunkWindow) tok = w0 + idx * kFChunk + r;
          else if (kind == kChunkSink) tok = r;
          else {
            const int key = idx * kFChunk + r;
            tok = sm.blocks[key / geo.Bk] * geo.Bk + key % geo.Bk;
          }
        }
        const size_t off = tiled_offset<DH>(0, tok, pc * 8);
        cp_async16_zfill(st + swz<DH>(r, pc), ksrc + off, valid);
        cp_async16_zfill(st + kFChunk * DH * 2 + swz<DH>(r, pc), vbase + off, valid);
      }
    }
    cp_async_commit();
  };

  int issued = 0;  // items issued (one cp.async group each, in order)
  auto total_items = [&]() { return P1 + NCw + P2 + NCs + NCr; };
  auto pump = [&](int upto) {  // issue items < upto that are issuable, in order
    const int lim = min(upto, final_done ? total_items() : (phase1_done ? P1 + NCw + P2 : P1 + NCw));
    while (issued < lim) {
      int idx;
      if (!issuable(kind_of(issued, idx))) break;
      issue(issued, issued % NS);
      ++issued;
    }
  };

  pump(NS - 1);  // summary pages and window chunks first

  // ---- query prologue: qc, qr (RoPE at pos) and the routing query qg ----
  for (int h = warp; h < 16; h += kFWarps) {
    float v[PER], r[PER];
    if (h < G && ok) {
      const int hq = g * G + h;
      load_head_row<DH>(p.q + ((size_t)b * geo.Hq + hq) * DH, v);
      if (geo.qknorm) {
        qknorm_lane<DH>(v, p.q_gain[hq], geo.eps);
      } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) v[i] = round_bf16(v[i]);
      }
      const float* cr = p.cos + (size_t)pos * DH;
      const float* sr = p.sin + (size_t)pos * DH;
      const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int d = lane * PER + i;
        const float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
        r[i] = rope_elem(v[i], sign * partner, cr[d], sr[d]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < PER; ++i) v[i] = r[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      sm.qc[h][lane * PER + i] = f2bf(v[i]);
      sm.qr[h][lane * PER + i] = f2bf(r[i]);
    }
  }
  __syncthreads();
  for (int d = tid; d < DH; d += kFThreads) {
    float acc = 0.f;
    for (int h = 0; h < G; ++h) acc += bf2f(sm.qc[h][d]);
    sm.qg[d] = round_bf16(acc);
  }
  __syncthreads();

  // ---- top-k points ----
  auto final_topk = [&](int R) {
    nsel = block_topk<kFThreads>(sm.sc, sm.id, R, kfinal, sm.ts);
    if (tid < 32) {
      const bool valid = tid < nsel;
      sm.blocks[tid] = valid ? sm.ts.sel_idx[tid] : -1;
      if (p.sel_idx != nullptr && tid < geo.K) {
        p.sel_idx[(size_t)bg * geo.K + tid] = valid ? sm.ts.sel_idx[tid] : -1;
        p.sel_score[(size_t)bg * geo.K + tid] = valid ? sm.ts.sel_score[tid] : neg_inf();
      }
    }
    __syncthreads();
    NCr = (nsel * geo.Bk + kFChunk - 1) / kFChunk;
    final_done = true;
  };
  auto super_topk = [&]() {
    const int b_eff = min(geo.beam, ns);
    const int nsup = block_topk<kFThreads>(sm.sc, sm.id, R1, b_eff, sm.ts);
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
    R2 = sm.n_children;
    P2 = (R2 + PB - 1) / PB;
    phase1_done = true;
  };
  if (P1 == 0) {
    if (!hier) {
      final_topk(0);
    } else {
      super_topk();
      if (P2 == 0) final_topk(0);
    }
  }

  float m0 = neg_inf(), m1 = neg_inf(), l0 = 0.f, l1 = 0.f;
  float o[DH / 8][4];
#pragma unroll
  for (int n = 0; n < DH / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const float sl2 = scale * kLog2e;
  const int key0 = warp * 16;
  const int nvec = row_pieces;
  constexpr int LPS = DH / 8;

  for (int it = 0; it < total_items(); ++it) {
    pump(it + NS);           // keep NS - 1 items ahead
    if (issued <= it) pump(it + 1);
    cp_async_wait_dyn(issued - it - 1);
    __syncthreads();
    const int stage = it % NS;
    int idx;
    const int kind = kind_of(it, idx);
    const unsigned char* st = sm.ring[stage];
    if (kind == kPageScore || kind == kPageChild) {
      // ---- score a page of summary rows from shared memory ----
      const int rows = page_rows(kind, idx);
      for (int r = warp; r < rows; r += kFWarps) {
        const int j = idx * PB + r;
        float best = neg_inf();
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          const int vv = lane + 32 * v;
          float part = 0.f;
          if (vv < nvec) {
            float f[8];
            unpack8(*reinterpret_cast<const uint4*>(st + r * row_bytes + vv * 16), f);
            const int d0 = (vv * 8) % DH;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) part = fmaf(f[jj], sm.qg[d0 + jj], part);
          }
#pragma unroll
          for (int ox = 1; ox < LPS; ox <<= 1) part += __shfl_xor_sync(0xffffffffu, part, ox);
          if (vv < nvec) best = fmaxf(best, part);
        }
        best = warp_max(best);
        if (lane == 0) {
          sm.sc[j] = best * scale;
          sm.id[j] = kind == kPageScore ? id_lo + j : child_id(j);
        }
      }
    } else {
      const int cnt = chunk_rows(kind, idx);
      if (key0 < cnt) {
        const unsigned char* kt = st;
        const unsigned char* vt = st + kFChunk * DH * 2;
        const __nv_bfloat16(*Q)[DH + 8] = kind == kChunkWindow ? sm.qr : sm.qc;
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kd = 0; kd < DH; kd += 16) {
          uint32_t a[4];
          a[0] = *reinterpret_cast<const uint32_t*>(&Q[gid][kd + tig * 2]);
          a[1] = *reinterpret_cast<const uint32_t*>(&Q[gid + 8][kd + tig * 2]);
          a[2] = *reinterpret_cast<const uint32_t*>(&Q[gid][kd + 8 + tig * 2]);
          a[3] = *reinterpret_cast<const uint32_t*>(&Q[gid + 8][kd + 8 + tig * 2]);
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int row = key0 + 8 * jj + gid;
            uint32_t bb[2];
            bb[0] = *reinterpret_cast<const uint32_t*>(kt + swz<DH>(row, kd / 8) + tig * 4);
            bb[1] = *reinterpret_cast<const uint32_t*>(kt + swz<DH>(row, kd / 8 + 1) + tig * 4);
            mma_bf16_16816(s[jj], a, bb);
          }
        }
#pragma unroll
        for (int jj = 0; jj < 2; ++jj)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = key0 + 8 * jj + tig * 2 + (e & 1);
            s[jj][e] = key < cnt ? s[jj][e] * sl2 : neg_inf();
          }
        float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
        float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float mu0 = (mn0 == neg_inf()) ? 0.f : mn0;
        const float mu1 = (mn1 == neg_inf()) ? 0.f : mn1;
        const float al0 = exp2f(m0 - mu0), al1 = exp2f(m1 - mu1);
        m0 = mn0;
        m1 = mn1;
        float pr[2][4];
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          pr[jj][0] = exp2f(s[jj][0] - mu0);
          pr[jj][1] = exp2f(s[jj][1] - mu0);
          pr[jj][2] = exp2f(s[jj][2] - mu1);
          pr[jj][3] = exp2f(s[jj][3] - mu1);
        }
        l0 = l0 * al0 + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
        l1 = l1 * al1 + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
#pragma unroll
        for (int n = 0; n < DH / 8; ++n) {
          o[n][0] *= al0;
          o[n][1] *= al0;
          o[n][2] *= al1;
          o[n][3] *= al1;
        }
        uint32_t pa[4];
        pa[0] = pack_bf16x2(pr[0][0], pr[0][1]);
        pa[1] = pack_bf16x2(pr[0][2], pr[0][3]);
        pa[2] = pack_bf16x2(pr[1][0], pr[1][1]);
        pa[3] = pack_bf16x2(pr[1][2], pr[1][3]);
        const int vrow = key0 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int vpiece = lane >> 4;
#pragma unroll
        for (int nd = 0; nd < DH; nd += 16) {
          uint32_t bv[4];
          ldmatrix_x4_trans(bv, vt + swz<DH>(vrow, nd / 8 + vpiece));
          mma_bf16_16816(o[nd / 8], pa, bv);
          mma_bf16_16816(o[nd / 8 + 1], pa, bv + 2);
        }
      }
    }
    __syncthreads();
    // ---- top-k points (after the page that completes a scoring phase) ----
    if (kind == kPageScore && idx == P1 - 1) {
      if (!hier) {
        final_topk(R1);
      } else {
        super_topk();
        if (P2 == 0) final_topk(0);
      }
    } else if (kind == kPageChild && idx == P2 - 1) {
      final_topk(R2);
    }
  }
  cp_async_wait<0>();

  // ---- merge the 8 warps, write the output ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  __syncthreads();
  FusedCombine<DH>& cb = *reinterpret_cast<FusedCombine<DH>*>(&sm.ring[0][0]);
  if (tig == 0) {
    cb.m[warp][gid] = m0;
    cb.m[warp][gid + 8] = m1;
    cb.l[warp][gid] = l0;
    cb.l[warp][gid + 8] = l1;
  }
#pragma unroll
  for (int n = 0; n < DH / 8; ++n) {
    cb.o[warp][gid][n * 8 + tig * 2] = o[n][0];
    cb.o[warp][gid][n * 8 + tig * 2 + 1] = o[n][1];
    cb.o[warp][gid + 8][n * 8 + tig * 2] = o[n][2];
    cb.o[warp][gid + 8][n * 8 + tig * 2 + 1] = o[n][3];
  }
  __syncthreads();
  for (int e = tid; e < G * DH; e += kFThreads) {
    const int r = e / DH, d = e % DH;
    float M = neg_inf();
#pragma unroll
    for (int w = 0; w < kFWarps; ++w) M = fmaxf(M, cb.m[w][r]);
    const float Mu = (M == neg_inf()) ? 0.f : M;
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kFWarps; ++w) {
      const float f = exp2f(cb.m[w][r] - Mu);
      L += cb.l[w][r] * f;
      O += cb.o[w][r][d] * f;
    }
    const int hq = g * G + r;
    p.out[((size_t)b * geo.Hq + hq) * DH + d] = f2bf(L > 0.f ? O / L : 0.f);
    if (d == 0 && p.lse != nullptr)
      p.lse[(size_t)b * geo.Hq + hq] = L > 0.f ? (M + log2f(L)) * 0.6931471805599453f : neg_inf();
  }
}

template <int DH, int VPL>
static cudaError_t launch_fused_t(const DecodeAttnParams& p, const __nv_bfloat16* summ, const __nv_bfloat16* supers,
                                  cudaStream_t st) {
  const size_t smem = sizeof(FusedSmem<DH>);
  static const cudaError_t attr = cudaFuncSetAttribute(decode_fused_kernel<DH, VPL>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (attr != cudaSuccess) return attr;
  decode_fused_kernel<DH, VPL><<<p.geo.B * p.geo.Hkv, kFThreads, smem, st>>>(p, summ, supers);
  return cudaGetLastError();
}

cudaError_t launch_decode_fused(const DecodeAttnParams& p, const __nv_bfloat16* summ, const __nv_bfloat16* supers,
                                int dh, cudaStream_t st) {
  const int vpl = (p.geo.m * dh / 8 + 31) / 32;
  if (dh == 64) {
    if (vpl <= 1) return launch_fused_t<64, 1>(p, summ, supers, st);
    return launch_fused_t<64, 2>(p, summ, supers, st);
  }
  if (vpl <= 1) return launch_fused_t<128, 1>(p, summ, supers, st);
  if (vpl <= 2) return launch_fused_t<128, 2>(p, summ, supers, st);
  return launch_fused_t<128, 4>(p, summ, supers, st);
}

size_t decode_fused_smem(int dh) { return dh == 64 ? sizeof(FusedSmem<64>) : sizeof(FusedSmem<128>); }

}  // namespace hba
