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
//      3-stage cp.async pipeline into 128-byte-swizzled tiles, each warp 16
//      keys per chunk on m16n8k16 bf16 tensor-core tiles (the G heads are the
//      16 rows), online softmax in the log2 domain;
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
constexpr int kFChunk = 128;  // keys per chunk: 8 warps x 16
constexpr int kFStages = 3;

template <int DH>
struct FusedSmem {
  __nv_bfloat16 kv[kFStages][2][kFChunk * DH];  // [stage][K|V] swizzled rows of DH bf16
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
struct FusedCombine {  // overlays the K/V stages after the chunk loop
  float m[kFWarps][16];
  float l[kFWarps][16];
  float o[kFWarps][16][DH];
};

// byte offset of (row, 16-byte piece) in a swizzled [rows x DH] bf16 tile
template <int DH>
HBA_DEVICE uint32_t swz(int row, int piece) {
  return (uint32_t)(row * DH * 2 + ((piece ^ (row & 7)) << 4));
}

template <int DH, int VPL>
__global__ void __launch_bounds__(kFThreads, 1) decode_fused_kernel(DecodeAttnParams p, const __nv_bfloat16* summ,
                                                                    const __nv_bfloat16* supers) {
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

  const int nctx = p.qp.seq_lens[b];
  const float scale = p.qp.scales[b];
  const bool ok = nctx >= 1 && nctx <= geo.n_cap;
  const int pos = ok ? nctx - 1 : -1;
  const int nb = ok ? nctx / geo.Bk : 0;
  const int bmax = ok ? min(last_candidate(pos, geo.W, geo.Bk), nb - 1) : 0;
  int kfinal = min(geo.K, nb);
  const int ns = (nb + geo.F - 1) / geo.F;
  if (geo.hier) kfinal = min(kfinal, min(geo.beam, ns) * geo.F);
  const int w0 = max(geo.S, pos - geo.W + 1);
  const int nw = ok ? max(0, pos - w0 + 1) : 0;
  const int nsink = ok ? min(geo.S, pos + 1) : 0;
  const int NCw = (nw + kFChunk - 1) / kFChunk;
  const int NCs = nsink > 0 ? 1 : 0;
  const size_t tok_stride = (size_t)geo.Hkv * DH;
  const size_t head_base = ((size_t)b * geo.n_cap) * tok_stride + (size_t)g * DH;
  const __nv_bfloat16* kbase = p.k + head_base;
  const __nv_bfloat16* krbase = p.kr + head_base;
  const __nv_bfloat16* vbase = p.v + head_base;
  int nsel = 0;  // valid routed picks (set after the top-k)

  auto chunk_rows = [&](int c) -> int {
    if (c < NCw) return min(kFChunk, nw - c * kFChunk);
    if (c < NCw + NCs) return nsink;
    return max(0, min(kFChunk, nsel * geo.Bk - (c - NCw - NCs) * kFChunk));
  };
  auto row_token = [&](int c, int r) -> int {
    if (c < NCw) return w0 + c * kFChunk + r;
    if (c < NCw + NCs) return r;
    const int key = (c - NCw - NCs) * kFChunk + r;
    return sm.blocks[key / geo.Bk] * geo.Bk + key % geo.Bk;
  };
  auto issue = [&](int c, int stage) {
    const int cnt = chunk_rows(c);
    if (cnt > 0) {
      const __nv_bfloat16* ksrc = c < NCw ? krbase : kbase;
      unsigned char* kt = reinterpret_cast<unsigned char*>(sm.kv[stage][0]);
      unsigned char* vt = reinterpret_cast<unsigned char*>(sm.kv[stage][1]);
      for (int e = tid; e < kFChunk * PIECES; e += kFThreads) {
        const int r = e / PIECES, pc = e % PIECES;
        const bool valid = r < cnt;
        const size_t off = (size_t)(valid ? row_token(c, r) : 0) * tok_stride + pc * 8;
        cp_async16_zfill(kt + swz<DH>(r, pc), ksrc + off, valid);
        cp_async16_zfill(vt + swz<DH>(r, pc), vbase + off, valid);
      }
    }
    cp_async_commit();
  };

  // ---- 1. window / sink chunks first ----
  const int early = min(kFStages - 1, NCw + NCs);
  for (int s = 0; s < early; ++s) issue(s, s);

  // ---- 2. query prologue ----
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
        r[i] = v[i] * cr[d] + sign * partner * sr[d];
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

  // ---- 3./4. scoring and top-k ----
  const size_t row_elems = (size_t)geo.m * DH;
  const int nvec = geo.m * DH / 8;
  SummaryLoads<DH, VPL, kFWarps> ld;
  constexpr int GROUP = kFWarps * SummaryLoads<DH, VPL, kFWarps>::U;
  auto score_range = [&](const __nv_bfloat16* base, int R, auto id_of) {
    for (int rb = 0; rb < R; rb += GROUP) {
      ld.load(base, row_elems, nvec, rb, R, id_of);
      ld.score(sm.qg, nvec, rb, R, scale, id_of, sm.sc, sm.id);
    }
    __syncthreads();
  };
  const __nv_bfloat16* summ_bg = summ + (size_t)bg * geo.nb_cap * row_elems;
  if (!geo.hier) {
    const int R = max(0, bmax);  // candidates 1..bmax
    score_range(summ_bg, R, [&](int r) { return 1 + r; });
    nsel = block_topk<kFThreads>(sm.sc, sm.id, R, kfinal, sm.ts);
  } else {
    const int F = geo.F;
    int R1 = 0, s_lo = 0;
    if (bmax >= 1) {
      s_lo = (F == 1) ? 1 : 0;
      R1 = bmax / F - s_lo + 1;
    }
    const __nv_bfloat16* sup_bg = supers + (size_t)bg * geo.ns_cap * row_elems;
    score_range(sup_bg, R1, [&](int r) { return s_lo + r; });
    const int b_eff = min(geo.beam, ns);
    const int nsup = block_topk<kFThreads>(sm.sc, sm.id, R1, b_eff, sm.ts);
    if (warp == 0) {
      const bool valid = lane < nsup;
      int lo = 0, cnt = 0;
      if (valid) {
        const int sidx = sm.ts.sel_idx[lane];
        lo = max(1, sidx * F);
        cnt = max(0, min(bmax, sidx * F + F - 1) - lo + 1);
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
    score_range(summ_bg, R2, [&](int r) {
      int si = 0;
      while (si < 31 && r >= sm.sup_off[si] + sm.sup_cnt[si]) ++si;
      return sm.sup_lo[si] + (r - sm.sup_off[si]);
    });
    nsel = block_topk<kFThreads>(sm.sc, sm.id, R2, kfinal, sm.ts);
  }
  if (tid < 32) {
    const bool valid = tid < nsel;
    sm.blocks[tid] = valid ? sm.ts.sel_idx[tid] : -1;
    if (p.sel_idx != nullptr && tid < geo.K) {
      p.sel_idx[(size_t)bg * geo.K + tid] = valid ? sm.ts.sel_idx[tid] : -1;
      p.sel_score[(size_t)bg * geo.K + tid] = valid ? sm.ts.sel_score[tid] : neg_inf();
    }
  }
  __syncthreads();

  // ---- 5. union softmax over the chunks ----
  const int NCr = (nsel * geo.Bk + kFChunk - 1) / kFChunk;
  const int NC = NCw + NCs + NCr;
  for (int s = early; s < kFStages - 1; ++s) {
    if (s < NC) issue(s, s);
    else cp_async_commit();
  }
  float m0 = neg_inf(), m1 = neg_inf(), l0 = 0.f, l1 = 0.f;
  float o[DH / 8][4];
#pragma unroll
  for (int n = 0; n < DH / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const float sl2 = scale * kLog2e;
  const int key0 = warp * 16;

  for (int c = 0; c < NC; ++c) {
    const int stage = c % kFStages;
    const int j = c + kFStages - 1;
    if (j < NC) issue(j, j % kFStages);
    else cp_async_commit();
    cp_async_wait<kFStages - 1>();
    __syncthreads();
    const int cnt = chunk_rows(c);
    if (key0 < cnt) {
      const unsigned char* kt = reinterpret_cast<const unsigned char*>(sm.kv[stage][0]);
      const unsigned char* vt = reinterpret_cast<const unsigned char*>(sm.kv[stage][1]);
      const __nv_bfloat16(*Q)[DH + 8] = c < NCw ? sm.qr : sm.qc;
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
    __syncthreads();
  }
  cp_async_wait<0>();

  // ---- 6. merge the 8 warps, write the output ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  __syncthreads();
  FusedCombine<DH>& cb = *reinterpret_cast<FusedCombine<DH>*>(&sm.kv[0][0][0]);
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
