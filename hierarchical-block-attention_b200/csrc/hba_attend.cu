// Fused union softmax: one online log-sum-exp over
//   [routed blocks (NoPE) | RoPE window | sinks (NoPE)]
// for each (query, kv head), the G query heads of the group stacked as the 16
// rows of an m16n8k16 bf16 tensor-core tile (reference
// src/hba/attention.py:676-711, which builds the same union with a
// concatenated softmax).
//
// One CTA per (query, batch*kv-head), 4 warps (the per-query prefill path).
// The CTA merges the partial selection lists into the final top-k, lays the
// union out as 64-key chunks (routed blocks first, then the window, then the
// sinks), and walks the chunks: cp.async double-buffered K/V gathers of whole
// 64-key chunks driven by the block list (window keys from the RoPE'd key
// copy), then per warp 16 keys: S = Q K^T, online softmax, O += P V.  Warps
// merge their (max, sum, O) through shared memory and the CTA writes the
// normalised output and the natural-log LSE.
#include <climits>

#include "hba_common.cuh"
#include "hba_internal.h"

namespace hba {

constexpr int kChunk = 64;
constexpr int kAttnThreads = 128;

template <int DH>
struct AttnSmem {
  __nv_bfloat16 qc[16][DH + 8];  // QKNorm'd query rows (NoPE branches)
  __nv_bfloat16 qr[16][DH + 8];  // RoPE'd query rows (window branch)
  __nv_bfloat16 k[2][kChunk][DH + 8];
  __nv_bfloat16 v[2][kChunk][DH + 8];
  int blocks[32];
  int nsel;
};

template <int DH>
struct AttnCombine {  // reuses the K/V buffers after the chunk loop
  float m[4][16];
  float l[4][16];
  float o[4][16][DH];
};

HBA_DEVICE void query_position_a(const QueryPos& qp, int b, int t, int& pos, int& nctx, float& scale) {
  if (qp.seq_lens != nullptr) {
    nctx = qp.seq_lens[b];
    pos = nctx - 1;
    scale = qp.scales[b];
  } else {
    nctx = qp.n_fixed;
    pos = t;
    scale = qp.scale_fixed;
  }
}

template <int DH>
__global__ void __launch_bounds__(kAttnThreads) attend_kernel(AttnParams p) {
  const Geom& geo = p.geo;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  AttnSmem<DH>& sm = *reinterpret_cast<AttnSmem<DH>*>(smem_raw);
  const int split = blockIdx.x, t = blockIdx.y, bg = blockIdx.z;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;

  int pos, nctx;
  float scale;
  query_position_a(p.qp, b, t, pos, nctx, scale);
  const bool ok_pos = (nctx >= 1 && nctx <= geo.n_cap);
  if (!ok_pos) pos = -1;
  const int nb = ok_pos ? nctx / geo.Bk : 0;
  const int kk = min(geo.K, nb);
  int kfinal = kk;
  if (geo.hier) {
    const int ns = (nb + geo.F - 1) / geo.F;
    kfinal = min(kk, min(geo.beam, ns) * geo.F);
  }

  // ---- final top-k from the partial lists (every CTA of the query agrees) ----
  if (warp == 0) {
    WarpTopK top;
    top.init();
    const int total = p.in_lists * p.list_k;
    const size_t base = ((size_t)bg * geo.nq + t) * total;
    if (kfinal > 0) {
      for (int e0 = 0; e0 < total; e0 += 32) {
        const int e = e0 + lane;
        float s = neg_inf();
        int i = INT_MAX;
        if (e < total) {
          const int ii = p.in_idx[base + e];
          if (ii >= 0) {
            s = p.in_score[base + e];
            i = ii;
          }
        }
        top.offer(s, i, kfinal);
      }
    }
    const bool valid = lane < kfinal && top.i != INT_MAX;
    const unsigned vm = __ballot_sync(0xffffffffu, valid);
    if (valid) sm.blocks[lane] = top.i;
    if (lane == 0) sm.nsel = __popc(vm);
    if (split == 0 && p.sel_idx != nullptr && lane < geo.K) {
      const size_t o = (((size_t)bg * geo.nq + t) * geo.K) + lane;
      p.sel_idx[o] = valid ? top.i : -1;
      p.sel_score[o] = valid ? top.s : neg_inf();
    }
  }

  // ---- query rows: QKNorm'd (qc) and RoPE'd (qr), rows >= G zero ----
  constexpr int PER = DH / 32;
  constexpr int HALF = DH / 2;
  for (int h = warp; h < 16; h += 4) {
    float v[PER];
    if (h < geo.G && ok_pos) {
      const int hq = g * geo.G + h;
      load_head_row<DH>(p.q + (((size_t)b * geo.nq + t) * geo.Hq + hq) * DH, v);
      if (geo.qknorm) qknorm_lane<DH>(v, p.q_gain[hq], geo.eps);
    } else {
#pragma unroll
      for (int i = 0; i < PER; ++i) v[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) sm.qc[h][lane * PER + i] = f2bf(v[i]);
  }
  __syncthreads();
  for (int e = tid; e < 16 * HALF; e += kAttnThreads) {
    const int h = e / HALF, d = e % HALF;
    float y1 = 0.f, y2 = 0.f;
    if (h < geo.G && ok_pos) {
      const float x1 = bf2f(sm.qc[h][d]), x2 = bf2f(sm.qc[h][d + HALF]);
      const float* cr = p.cos + (size_t)pos * DH;
      const float* sr = p.sin + (size_t)pos * DH;
      y1 = rope_elem(x1, -x2, cr[d], sr[d]);
      y2 = rope_elem(x2, x1, cr[d + HALF], sr[d + HALF]);
    }
    sm.qr[h][d] = f2bf(y1);
    sm.qr[h][d + HALF] = f2bf(y2);
  }
  __syncthreads();

  // ---- union layout: routed | window | sinks, in 64-key chunks ----
  const int nsel = sm.nsel;
  const int Lr = nsel * geo.Bk;
  const int w0 = max(geo.S, pos - geo.W + 1);
  const int nw = ok_pos ? max(0, pos - w0 + 1) : 0;
  const int nsink = ok_pos ? min(geo.S, pos + 1) : 0;
  const int NCr = (Lr + kChunk - 1) / kChunk;
  const int NCw = (nw + kChunk - 1) / kChunk;
  const int NC = NCr + NCw + (nsink > 0 ? 1 : 0);
  const int c_begin = (int)(((long long)NC * split) / p.splits);
  const int c_end = (int)(((long long)NC * (split + 1)) / p.splits);

  const size_t tok_stride = (size_t)geo.Hkv * DH;
  const size_t head_base = ((size_t)b * geo.n_cap) * tok_stride + (size_t)g * DH;
  const __nv_bfloat16* kbase = p.k + head_base;
  const __nv_bfloat16* krbase = p.kr + head_base;
  const __nv_bfloat16* vbase = p.v + head_base;

  // token of row r of chunk c, -1 when the row is past the segment's end
  auto row_token = [&](int c, int r) -> int {
    if (c < NCr) {
      const int key = c * kChunk + r;
      return key < Lr ? sm.blocks[key / geo.Bk] * geo.Bk + key % geo.Bk : -1;
    }
    if (c < NCr + NCw) {
      const int key = (c - NCr) * kChunk + r;
      return key < nw ? w0 + key : -1;
    }
    return r < nsink ? r : -1;
  };
  auto issue = [&](int c, int buf) {
    constexpr int PIECES = DH / 8;
    const __nv_bfloat16* ksrc = (c >= NCr && c < NCr + NCw) ? krbase : kbase;  // window keys come RoPE'd
    for (int e = tid; e < kChunk * PIECES; e += kAttnThreads) {
      const int r = e / PIECES, pc = e % PIECES;
      const int tok = row_token(c, r);
      const bool valid = tok >= 0;
      const size_t off = (size_t)(valid ? tok : 0) * tok_stride + pc * 8;
      cp_async16_zfill(&sm.k[buf][r][pc * 8], ksrc + off, valid);
      cp_async16_zfill(&sm.v[buf][r][pc * 8], vbase + off, valid);
    }
    cp_async_commit();
  };

  float m0 = neg_inf(), m1 = neg_inf(), l0 = 0.f, l1 = 0.f;
  float o[DH / 8][4];
#pragma unroll
  for (int n = 0; n < DH / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const float sl2 = scale * kLog2e;

  if (c_begin < c_end) issue(c_begin, 0);
  for (int c = c_begin; c < c_end; ++c) {
    const int buf = (c - c_begin) & 1;
    if (c + 1 < c_end) {
      issue(c + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const bool window = (c >= NCr) && (c < NCr + NCw);
    int cnt;
    if (c < NCr) cnt = min(kChunk, Lr - c * kChunk);
    else if (window) cnt = min(kChunk, nw - (c - NCr) * kChunk);
    else cnt = nsink;
    // ---- S = Q K^T for this warp's 16 keys ----
    const __nv_bfloat16(*Q)[DH + 8] = window ? sm.qr : sm.qc;
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int key0 = warp * 16;
#pragma unroll
    for (int kd = 0; kd < DH; kd += 16) {
      uint32_t a[4];
      a[0] = *reinterpret_cast<const uint32_t*>(&Q[gid][kd + tig * 2]);
      a[1] = *reinterpret_cast<const uint32_t*>(&Q[gid + 8][kd + tig * 2]);
      a[2] = *reinterpret_cast<const uint32_t*>(&Q[gid][kd + 8 + tig * 2]);
      a[3] = *reinterpret_cast<const uint32_t*>(&Q[gid + 8][kd + 8 + tig * 2]);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t bb[2];
        bb[0] = *reinterpret_cast<const uint32_t*>(&sm.k[buf][key0 + 8 * j + gid][kd + tig * 2]);
        bb[1] = *reinterpret_cast<const uint32_t*>(&sm.k[buf][key0 + 8 * j + gid][kd + 8 + tig * 2]);
        mma_bf16_16816(s[j], a, bb);
      }
    }
    // ---- scale, mask, online softmax (log2 domain) ----
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + 8 * j + tig * 2 + (e & 1);
        s[j][e] = key < cnt ? s[j][e] * sl2 : neg_inf();
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
    for (int j = 0; j < 2; ++j) {
      pr[j][0] = exp2f(s[j][0] - mu0);
      pr[j][1] = exp2f(s[j][1] - mu0);
      pr[j][2] = exp2f(s[j][2] - mu1);
      pr[j][3] = exp2f(s[j][3] - mu1);
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
    // ---- O += P V ----
    uint32_t pa[4];
    pa[0] = pack_bf16x2(pr[0][0], pr[0][1]);
    pa[1] = pack_bf16x2(pr[0][2], pr[0][3]);
    pa[2] = pack_bf16x2(pr[1][0], pr[1][1]);
    pa[3] = pack_bf16x2(pr[1][2], pr[1][3]);
    const int vrow = key0 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int vcol = (lane >> 4) * 8;
#pragma unroll
    for (int nd = 0; nd < DH; nd += 16) {
      uint32_t bv[4];
      ldmatrix_x4_trans(bv, &sm.v[buf][vrow][nd + vcol]);
      mma_bf16_16816(o[nd / 8], pa, bv);
      mma_bf16_16816(o[nd / 8 + 1], pa, bv + 2);
    }
    __syncthreads();
  }

  // ---- merge the 4 warps ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  AttnCombine<DH>& cb = *reinterpret_cast<AttnCombine<DH>*>(&sm.k[0][0][0]);
  __syncthreads();
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
  const int G = geo.G;
  for (int e = tid; e < G * DH; e += kAttnThreads) {
    const int r = e / DH, d = e % DH;
    float M = neg_inf();
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, cb.m[w][r]);
    const float Mu = (M == neg_inf()) ? 0.f : M;
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = exp2f(cb.m[w][r] - Mu);
      L += cb.l[w][r] * f;
      O += cb.o[w][r][d] * f;
    }
    const int hq = g * G + r;
    p.out[(((size_t)b * geo.nq + t) * geo.Hq + hq) * DH + d] = f2bf(L > 0.f ? O / L : 0.f);
    if (d == 0 && p.lse != nullptr)
      p.lse[((size_t)b * geo.Hq + hq) * geo.nq + t] = L > 0.f ? (M + log2f(L)) * 0.6931471805599453f : neg_inf();
  }
}

cudaError_t launch_attend(const AttnParams& p, int dh, cudaStream_t st) {
  dim3 grid(p.splits, p.geo.nq, p.geo.B * p.geo.Hkv);
  cudaError_t e;
  if (dh == 64) {
    const size_t smem = sizeof(AttnSmem<64>);
    static_assert(sizeof(AttnCombine<64>) <= sizeof(__nv_bfloat16) * 4 * kChunk * (64 + 8), "combine fits");
    static const cudaError_t attr = cudaFuncSetAttribute(attend_kernel<64>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if ((e = attr) != cudaSuccess) return e;
    attend_kernel<64><<<grid, kAttnThreads, smem, st>>>(p);
  } else {
    const size_t smem = sizeof(AttnSmem<128>);
    static_assert(sizeof(AttnCombine<128>) <= sizeof(__nv_bfloat16) * 4 * kChunk * (128 + 8), "combine fits");
    static const cudaError_t attr = cudaFuncSetAttribute(attend_kernel<128>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if ((e = attr) != cudaSuccess) return e;
    attend_kernel<128><<<grid, kAttnThreads, smem, st>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace hba
