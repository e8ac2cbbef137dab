// Decode attention: the fused union softmax for one new query per sequence,
// balanced over the whole GPU.
//
// For every (sequence, kv head) the union is laid out as `nchunk` 64-key
// chunk slots: [RoPE window (ncw slots) | sinks (1) | routed blocks (ncr)].
// All B*Hkv*nchunk slots form one sequence that is cut into gridDim.x equal
// contiguous ranges (grid sized to be resident at once), so every CTA moves
// the same number of bytes whatever the batch or head count.  A CTA walks its
// range one (sequence, kv head) segment at a time:
//   * query prologue: the G query heads QKNorm'd (qc) and RoPE'd (qr) into
//     shared memory, the group stacked as the rows of m16n8k16 bf16 tiles;
//   * a 3-stage cp.async pipeline of 64-key K/V gathers (window keys from the
//     RoPE'd key cache, routed keys block by block from the selected list),
//     window first so that routed chunks -- the only ones that need the
//     selection -- come last: the kernel is launched as a programmatic
//     dependent of the selection kernel and waits for it (griddepcontrol)
//     only when the pipeline reaches the first routed chunk;
//   * per warp 16 keys per chunk: S = Q K^T, online softmax in the log2
//     domain, O += P V; warps combine through shared memory;
//   * the segment's (max, sum, O) partial goes to the workspace; the CTA that
//     completes a (sequence, kv head) last (atomic counter, zeroed by the
//     selection kernel of the same call) merges the partials into the output
//     and the natural-log LSE and writes the selected block list.
// Reference semantics: src/hba/attention.py:676-711 at cs = n-1.
#include <climits>

#include "hba_common.cuh"
#include "hba_internal.h"

namespace hba {

constexpr int kDChunk = 64;
constexpr int kDThreads = 128;
constexpr int kDStages = 3;

template <int DH>
struct DecSmem {
  __nv_bfloat16 qc[16][DH + 8];
  __nv_bfloat16 qr[16][DH + 8];
  __nv_bfloat16 k[kDStages][kDChunk][DH + 8];
  __nv_bfloat16 v[kDStages][kDChunk][DH + 8];
  int blocks[32];
  float bscore[32];
  int nsel;
  int last;
};

template <int DH>
struct DecCombine {  // overlays the K/V stages after a segment's chunk loop
  float m[4][16];
  float l[4][16];
  float o[4][16][DH];
};

// CTA that owns global chunk slot a when T slots are cut into N ranges
// [floor(c*T/N), floor((c+1)*T/N)).
HBA_DEVICE int owner_cta(long long a, long long T, int N) { return (int)(((a + 1) * N - 1) / T); }

template <int DH>
__global__ void __launch_bounds__(kDThreads) decode_attend_kernel(DecodeAttnParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  DecSmem<DH>& sm = *reinterpret_cast<DecSmem<DH>*>(smem_raw);
  DecCombine<DH>& cb = *reinterpret_cast<DecCombine<DH>*>(&sm.k[0][0][0]);
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  constexpr int PER = DH / 32;
  constexpr int HALF = DH / 2;
  constexpr int PIECES = DH / 8;
  const int G = geo.G;
  const int N = gridDim.x;
  const long long T = (long long)geo.B * geo.Hkv * p.nchunk;
  const long long g0 = T * blockIdx.x / N, g1 = T * (blockIdx.x + 1) / N;
  bool waited = false;

  for (long long gc = g0; gc < g1;) {
    const int bg = (int)(gc / p.nchunk);
    const int c0 = (int)(gc % p.nchunk);
    const long long rem = g1 - gc;
    const int c1 = (int)(rem < (long long)(p.nchunk - c0) ? c0 + rem : p.nchunk);
    gc += c1 - c0;
    const int b = bg / geo.Hkv, g = bg % geo.Hkv;

    const int nctx = p.qp.seq_lens[b];
    const float scale = p.qp.scales[b];
    const bool ok = nctx >= 1 && nctx <= geo.n_cap;
    const int pos = ok ? nctx - 1 : -1;
    const int nb = ok ? nctx / geo.Bk : 0;
    int kfinal = min(geo.K, nb);
    if (geo.hier) kfinal = min(kfinal, min(geo.beam, (nb + geo.F - 1) / geo.F) * geo.F);
    const int w0 = max(geo.S, pos - geo.W + 1);
    const int nw = ok ? max(0, pos - w0 + 1) : 0;
    const int nsink = ok ? min(geo.S, pos + 1) : 0;
    const size_t head_base = ((size_t)b * geo.Hkv + g) * (size_t)geo.n_cap * DH;  // the chunk-tiled cache
    const __nv_bfloat16* kbase = p.k + head_base;
    const __nv_bfloat16* krbase = p.kr + head_base;
    const __nv_bfloat16* vbase = p.v + head_base;

    __syncthreads();  // the previous segment is done with shared memory
    bool lists_ready = false;
    auto ensure_lists = [&]() {
      if (lists_ready) return;
      if (!waited) {
        grid_dep_wait();
        waited = true;
      }
      if (warp == 0) {
        WarpTopK top;
        top.init();
        const int total = p.in_lists * p.list_k;
        const size_t base = (size_t)bg * total;
        if (kfinal > 0) {
          for (int e0 = 0; e0 < total; e0 += 32) {
            const int e = e0 + lane;
            float s = neg_inf();
            int i = INT_MAX;
            if (e < total) {
              const int ii = __ldcg(p.in_idx + base + e);
              if (ii >= 0) {
                s = __ldcg(p.in_score + base + e);
                i = ii;
              }
            }
            top.offer(s, i, kfinal);
          }
        }
        const bool valid = lane < kfinal && top.i != INT_MAX;
        const unsigned vm = __ballot_sync(0xffffffffu, valid);
        sm.blocks[lane] = valid ? top.i : -1;
        sm.bscore[lane] = valid ? top.s : neg_inf();
        if (lane == 0) sm.nsel = __popc(vm);
      }
      __syncthreads();
      lists_ready = true;
    };
    // valid rows of chunk slot c (routed slots need the lists)
    auto chunk_rows = [&](int c) -> int {
      if (c < p.ncw) return max(0, min(kDChunk, nw - c * kDChunk));
      if (c == p.ncw) return nsink;
      return max(0, min(kDChunk, sm.nsel * geo.Bk - (c - p.ncw - 1) * kDChunk));
    };
    auto row_token = [&](int c, int r) -> int {
      if (c < p.ncw) return w0 + c * kDChunk + r;
      if (c == p.ncw) return r;
      const int key = (c - p.ncw - 1) * kDChunk + r;
      return sm.blocks[key / geo.Bk] * geo.Bk + key % geo.Bk;
    };
    auto issue = [&](int c, int stage) {
      if (c > p.ncw) ensure_lists();
      const int cnt = chunk_rows(c);
      if (cnt > 0) {
        const __nv_bfloat16* ksrc = c < p.ncw ? krbase : kbase;
        for (int e = tid; e < kDChunk * PIECES; e += kDThreads) {
          const int r = e / PIECES, pc = e % PIECES;
          const bool valid = r < cnt;
          const size_t off = tiled_offset<DH>(0, valid ? row_token(c, r) : 0, pc * 8);
          cp_async16_zfill(&sm.k[stage][r][pc * 8], ksrc + off, valid);
          cp_async16_zfill(&sm.v[stage][r][pc * 8], vbase + off, valid);
        }
      }
      cp_async_commit();
    };

    const int nc = c1 - c0;
    // window/sink loads depend neither on the query nor on the selection:
    // start them first (they are a prefix of the chunk order)
    for (int s = 0; s < kDStages - 1; ++s)
      if (s < nc && c0 + s <= p.ncw) issue(c0 + s, s);
    // ---- query rows ----
    for (int h = warp; h < 16; h += 4) {
      float v[PER];
      if (h < G && ok) {
        const int hq = g * G + h;
        load_head_row<DH>(p.q + ((size_t)b * geo.Hq + hq) * DH, v);
        if (geo.qknorm) qknorm_lane<DH>(v, p.q_gain[hq], geo.eps);
      } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) v[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) sm.qc[h][lane * PER + i] = f2bf(v[i]);
    }
    __syncthreads();
    for (int e = tid; e < 16 * HALF; e += kDThreads) {
      const int h = e / HALF, d = e % HALF;
      float y1 = 0.f, y2 = 0.f;
      if (h < G && ok) {
        const float x1 = bf2f(sm.qc[h][d]), x2 = bf2f(sm.qc[h][d + HALF]);
        const float* cr = p.cos + (size_t)pos * DH;
        const float* sr = p.sin + (size_t)pos * DH;
        y1 = rope_elem(x1, -x2, cr[d], sr[d]);
        y2 = rope_elem(x2, x1, cr[d + HALF], sr[d + HALF]);
      }
      sm.qr[h][d] = f2bf(y1);
      sm.qr[h][d + HALF] = f2bf(y2);
    }
    // then routed chunks among the first stages (their lists may need the wait),
    // then empty groups, so that cp.async groups stay in chunk order
    for (int s = 0; s < kDStages - 1; ++s) {
      if (s < nc) {
        if (c0 + s > p.ncw) issue(c0 + s, s);
      } else {
        cp_async_commit();
      }
    }
    __syncthreads();

    float m0 = neg_inf(), m1 = neg_inf(), l0 = 0.f, l1 = 0.f;
    float o[DH / 8][4];
#pragma unroll
    for (int n = 0; n < DH / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    const float sl2 = scale * kLog2e;

    for (int i = 0; i < nc; ++i) {
      const int c = c0 + i, stage = i % kDStages;
      const int j = i + kDStages - 1;
      if (j < nc) issue(c0 + j, j % kDStages);
      else cp_async_commit();
      cp_async_wait<kDStages - 1>();
      __syncthreads();
      const int cnt = chunk_rows(c);
      if (cnt > 0) {
        const __nv_bfloat16(*Q)[DH + 8] = c < p.ncw ? sm.qr : sm.qc;
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
          for (int jj = 0; jj < 2; ++jj) {
            uint32_t bb[2];
            bb[0] = *reinterpret_cast<const uint32_t*>(&sm.k[stage][key0 + 8 * jj + gid][kd + tig * 2]);
            bb[1] = *reinterpret_cast<const uint32_t*>(&sm.k[stage][key0 + 8 * jj + gid][kd + 8 + tig * 2]);
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
        const int vcol = (lane >> 4) * 8;
#pragma unroll
        for (int nd = 0; nd < DH; nd += 16) {
          uint32_t bv[4];
          ldmatrix_x4_trans(bv, &sm.v[stage][vrow][nd + vcol]);
          mma_bf16_16816(o[nd / 8], pa, bv);
          mma_bf16_16816(o[nd / 8 + 1], pa, bv + 2);
        }
      }
      __syncthreads();
    }
    cp_async_wait<0>();

    // ---- combine the 4 warps, write this segment's partial ----
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
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
    const int cfirst = owner_cta((long long)bg * p.nchunk, T, N);
    const int clast = owner_cta((long long)(bg + 1) * p.nchunk - 1, T, N);
    const int nseg = clast - cfirst + 1;
    const int seg = blockIdx.x - cfirst;
    float* part_bg = p.part + (size_t)bg * p.max_seg * G * (DH + 2);
    for (int e = tid; e < G * DH; e += kDThreads) {
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
      float* pr = part_bg + ((size_t)seg * G + r) * (DH + 2);
      pr[2 + d] = O;
      if (d == 0) {
        pr[0] = M;
        pr[1] = L;
      }
    }
    if (!waited) {  // the counters are zeroed by the selection kernel of this call
      grid_dep_wait();
      waited = true;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) sm.last = (atomicAdd(p.counters + bg, 1) == nseg - 1);
    __syncthreads();
    if (sm.last) {
      __threadfence();
      for (int e = tid; e < G * DH; e += kDThreads) {
        const int r = e / DH, d = e % DH;
        float M = neg_inf();
        for (int k = 0; k < nseg; ++k) M = fmaxf(M, __ldcg(part_bg + ((size_t)k * G + r) * (DH + 2)));
        const float Mu = (M == neg_inf()) ? 0.f : M;
        float L = 0.f, O = 0.f;
        for (int k = 0; k < nseg; ++k) {
          const float* pr = part_bg + ((size_t)k * G + r) * (DH + 2);
          const float f = exp2f(__ldcg(pr) - Mu);
          L += __ldcg(pr + 1) * f;
          O += __ldcg(pr + 2 + d) * f;
        }
        const int hq = g * G + r;
        p.out[((size_t)b * geo.Hq + hq) * DH + d] = f2bf(L > 0.f ? O / L : 0.f);
        if (d == 0 && p.lse != nullptr)
          p.lse[(size_t)b * geo.Hq + hq] = L > 0.f ? (M + log2f(L)) * 0.6931471805599453f : neg_inf();
      }
      if (p.sel_idx != nullptr) {
        ensure_lists();
        if (warp == 0 && lane < geo.K) {
          p.sel_idx[(size_t)bg * geo.K + lane] = lane < kfinal ? sm.blocks[lane] : -1;
          p.sel_score[(size_t)bg * geo.K + lane] = lane < kfinal ? sm.bscore[lane] : neg_inf();
        }
      }
      if (tid == 0) p.counters[bg] = 0;
    }
  }
}

// Resident CTAs of the decode attention kernel on the current device,
// computed on the first call per head size (make that call before any graph
// capture; later calls only read the cached value).
template <int DH>
static int resident_ctas() {
  static int cap = -1;
  if (cap < 0) {
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = sizeof(DecSmem<DH>);
    cudaFuncSetAttribute(decode_attend_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_attend_kernel<DH>, kDThreads, smem);
    cap = sms * (per_sm > 0 ? per_sm : 1);
  }
  return cap;
}

int decode_attend_grid(int dh, int total_chunks) {
  const int cap = dh == 64 ? resident_ctas<64>() : resident_ctas<128>();
  return total_chunks < cap ? (total_chunks > 0 ? total_chunks : 1) : cap;
}

cudaError_t launch_decode_attend(const DecodeAttnParams& p, int dh, int grid, cudaStream_t st) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(kDThreads);
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  if (dh == 64) {
    lc.dynamicSmemBytes = sizeof(DecSmem<64>);
    return cudaLaunchKernelEx(&lc, decode_attend_kernel<64>, p);
  }
  lc.dynamicSmemBytes = sizeof(DecSmem<128>);
  return cudaLaunchKernelEx(&lc, decode_attend_kernel<128>, p);
}

}  // namespace hba
