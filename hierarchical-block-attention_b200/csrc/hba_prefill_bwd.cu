// Backward of the prefill union softmax on the 5th-generation tensor cores
// (tcgen05 + TMEM), the gradient of the training path's attention
// (reference: hba_attention_fused, src/hba/attention.py:552-607, and the
// dense path it agrees with, :306-389; the QKNorm it differentiates through,
// :88-94).  The block selection is a top-k and has no gradient: the kernels
// take the forward's picks.
//
// Per row (query i, head h) of a (sequence, kv head) with P the union
// softmax over [sinks (NoPE) | window (RoPE) | routed blocks (NoPE)],
// logits scale * q.k:
//   D = sum_d dout * out,  dP = dout . v,  dS = P * (dP - D)
//   dq = scale * sum_keys dS k,  dk = scale * sum_rows dS q,  dv = sum_rows P dout
// with the window's q and k the RoPE'd ones (their gradients rotated back by
// RoPE's transpose) and the rest the QKNorm'd ones; then QKNorm's own
// gradient (and the per-head gains').
//
// Kernels, in order:
//   bwd_delta_kernel     D per row (CUDA cores)
//   prefill_bwd_kernel   one CTA per (sequence, kv head, query tile of QT =
//                        128/G queries x G heads = the 128 rows); it walks the
//                        same chunk list as the forward (window chunks with
//                        the RoPE'd tiles, then the sink block and the routed
//                        union in 128-key chunks) and, per chunk, on the
//                        tensor cores, keys on the TMEM lanes:
//                          S^T  = K Q^T,   dP^T = V dO^T      (M 128 keys, N 128 rows, K dh)
//                          P^T, dS^T (bf16) written back into TMEM over S^T / dP^T
//                          dV_c = P^T dO,  dK_c = dS^T Q      (A from TMEM, M 128 keys, N dh, K 128 rows)
//                          dQ  += dS K                        (dS from shared memory, M 128 rows, N dh, K 128 keys)
//                        dV_c and dK_c (dK_c rotated back for window keys)
//                        are added into fp32 accumulators with vector
//                        reductions; dQ stays in TMEM per phase (window,
//                        then NoPE) and is written once per row.
//   bwd_norm_kernel      QKNorm's backward (q and k sides, gains by per-CTA
//                        sums), or a plain conversion, fp32 -> bf16.
//
// Roles of prefill_bwd_kernel (320 threads):
//   warps 0-7   gradient warps: lane quarter lq = warp & 3 of the TMEM lanes,
//               column group hc = warp >> 2 of the 128 row columns
//               (elementwise step) or of the dh columns (read-outs)
//               (kBwColGroups = 2; 4 groups ran no faster: the chain is not
//               bound by the per-warp work)
//   warp 8      loads: the query and dO tiles (TMA), K / V chunks (1-D bulk
//               copies of the chunk-tiled pre-pass copies) through a ring
//   warp 9      issues every tcgen05.mma (one elected lane, whole-warp loop)
//               and owns the TMEM allocation
// TMEM columns: S^T [0, 128) (P^T packed over [64h, 64h + 32)), dP^T [128,
// 256) (dS^T likewise), dQ [256, 256 + dh), dV_c / dK_c: dh 64 in [320, 384)
// and [384, 448); dh 128 one shared region [384, 512) used for dV_c, then
// dK_c.  Every mbarrier wait is bounded; a timeout sets *err and drains.
#include <climits>
#include <cudaTypedefs.h>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_sm100.cuh"

namespace hba {

using namespace sm100;

constexpr int kBwColGroups = 2;                   // gradient warps per TMEM lane quarter
constexpr int kBwGradWarps = 4 * kBwColGroups;
constexpr int kBwGradThreads = 32 * kBwGradWarps;
constexpr int kBwThreads = kBwGradThreads + 64;
constexpr int kBwLoad = kBwGradWarps;              // load warp
constexpr int kBwMma = kBwGradWarps + 1;           // MMA warp (and TMEM owner)
constexpr int kBwCols = 128 / kBwColGroups;        // a gradient warp's S^T / dP^T columns (rows of the tile)
// P^T / dS^T, bf16 pairs, are written over S^T / dP^T: the 16 rows of piece
// pc of column group cq go to the 8 columns kBwCols cq + 8 pc, inside what
// that warp has already read; the TMEM address of MMA K-step kk (rows
// 16 kk .. 16 kk + 15):
__host__ __device__ constexpr uint32_t bw_packed_col(int kk) {
  return (uint32_t)(kBwCols * (16 * kk / kBwCols) + 8 * ((16 * kk % kBwCols) / 16));
}
constexpr int kBwBlock = 64;         // keys per routed block = per half chunk
constexpr int kBwKeys = 128;         // keys per chunk
constexpr int kBwMaxEntries = 520;   // NoPE list: the sink block + the routed union of one tile (1 + QT k)
constexpr int kBwMaxHeads = 128;     // bwd_norm_kernel's per-CTA gain sums

enum BwHalfType : uint32_t { kBwSink = 0, kBwWindow = 1, kBwRouted = 2, kBwPad = 3 };

template <int DH>
struct BwSmem {
  static constexpr int HALVES = DH / 64;
  static constexpr int QBYTES = HALVES * 16384;         // [128 rows x DH], swizzled per 64-dim group
  static constexpr int GBYTES = kBwKeys * 128;          // one dim group of a K or V chunk
  static constexpr int KT = HALVES * GBYTES;            // [128 keys x DH]
  static constexpr int NSLOT = DH == 64 ? 6 : 3;        // K(c) is ring item 2c, V(c) item 2c + 1
  alignas(1024) unsigned char q[QBYTES];                // RoPE'd (window phase), then QKNorm'd queries
  alignas(1024) unsigned char dout[QBYTES];
  alignas(1024) unsigned char ds[2][16384];             // dS, MN-major for the dQ MMA: [row half][128 keys x 64 rows]
  alignas(1024) unsigned char ring[NSLOT][KT];
  uint32_t emask[kBwMaxEntries];                        // routed blocks: bit q = query i0 + q picked it
  uint16_t eblk[kBwMaxEntries];
  float2 rowc[128];                                     // per row: (LSE in log2 units, D)
  uint8_t rq[128];                                      // per row: its query in the tile (32: padding row)
  uint64_t q_ready, qc_ready;
  uint64_t full[NSLOT], empty[NSLOT];
  uint64_t s_full, p_full, dv_full, dk_full, tmp_free, dq_full, dq_free, fin;
  uint32_t tmem_base;
  int n_entries;
  int scan[kBwThreads / 32];
};

static_assert(sizeof(BwSmem<128>) + 1024 <= 232448 && sizeof(BwSmem<64>) + 1024 <= 232448,
              "backward tile set exceeds the 227 KB of shared memory");

struct PrefillBwdParams {
  Geom geo;
  int n;
  float scale;
  int QT;                    // queries per tile
  int tiles;                 // tiles per (sequence, kv head)
  const int32_t* sel;        // [B*Hkv, n, list_stride] the forward's picks (-1 = none)
  int list_stride;
  const __nv_bfloat16* kc;   // chunk-tiled QKNorm'd keys, RoPE'd keys, values
  const __nv_bfloat16* kr;
  const __nv_bfloat16* v;
  const float* lse;          // [B, Hq, n] natural log
  const float* delta;        // [B, Hq, n]
  // fp32 gradients in the q / k layouts: w.r.t. the QKNorm'd q (NoPE keys)
  // and the RoPE'd q (window keys), written once per row; w.r.t. the QKNorm'd
  // k (NoPE rows), the RoPE'd k (window rows) and v, by reductions (zeroed by
  // the host).  The RoPE transpose and QKNorm's backward run afterwards.
  float* dq_acc;             // [B, n, Hq, DH]
  float* dqr_acc;
  float* dk_acc;             // [B, n, Hkv, DH]
  float* dkr_acc;
  float* dv_acc;
  int* err;
};

HBA_DEVICE void red_add4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d));
}

// D[b, h, t] = sum_d dout * out, one warp per row (b, t, h) of [B, n, H, DH].
template <int DH>
__global__ void __launch_bounds__(256) bwd_delta_kernel(int64_t rows, int n, int H,
                                                        const __nv_bfloat16* __restrict__ dout,
                                                        const __nv_bfloat16* __restrict__ out,
                                                        float* __restrict__ delta) {
  constexpr int PER = DH / 32;
  const int64_t w = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < PER; e += 2) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dout + w * DH + lane * PER + e));
    const float2 o = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(out + w * DH + lane * PER + e));
    acc = fmaf(a.x, o.x, fmaf(a.y, o.y, acc));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    const int64_t bt = w / H;
    const int h = (int)(w - bt * H);
    const int64_t b = bt / n, t = bt - b * n;
    delta[(b * H + h) * n + t] = acc;
  }
}

// One warp per row (b, t, h) of [B, n, H, DH]: the gradient w.r.t. the
// QKNorm'd tensor, dy + RoPE^T(dyr) (dyr: the gradient w.r.t. its RoPE'd
// copy at position t; rope(x) = x cos + rot_half(x) sin with rot_half(x) =
// (-x2, x1), so RoPE^T(g)[d] = g[d] cos[d] + g[d + h] sin[d + h] for d < h
// and g[d] cos[d] - g[d - h] sin[d - h] above, h = DH / 2), then QKNorm's
// backward (attention.py:88-94: y = x / rms * g, rms = sqrt(max(mean(x^2),
// eps))): dx = (g / rms) (dy - u mean(dy u)) with u = x / rms (dx = (g /
// rms) dy where the mean is clamped), dg[h] += sum_d dy u; without QKNorm
// dx = dy.  fp32 in, bf16 out; the gain sums go through shared memory, then
// one atomic per head per CTA.
template <int DH>
__global__ void __launch_bounds__(256) bwd_norm_kernel(int64_t rows, int n, int H, const __nv_bfloat16* __restrict__ x,
                                                       const float* __restrict__ dy, const float* __restrict__ dyr,
                                                       const float* __restrict__ cos, const float* __restrict__ sin,
                                                       const float* __restrict__ gain, float eps, int qknorm,
                                                       __nv_bfloat16* __restrict__ dx, float* __restrict__ dgain) {
  constexpr int PER = DH / 32;
  static_assert(PER % 2 == 0, "two columns per access");
  __shared__ float gs[kBwMaxHeads];
  for (int h = threadIdx.x; h < kBwMaxHeads; h += blockDim.x) gs[h] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * 8;
  for (int64_t w = (int64_t)blockIdx.x * 8 + threadIdx.x / 32; w < rows; w += nwarps) {
    // lane l holds columns [l PER, l PER + PER), PER = 2 or 4: 8-byte (float2) accesses
    float d[PER], xv[PER], o[PER];
    const float2* dp = reinterpret_cast<const float2*>(dy + w * DH + lane * PER);
#pragma unroll
    for (int e = 0; e < PER; e += 2) {
      const float2 f = dp[e / 2];
      d[e] = f.x;
      d[e + 1] = f.y;
    }
    if (dyr != nullptr) {
      // the RoPE partner columns (d +- DH / 2) of lane l sit in lane l ^ 16
      const int64_t t = (w / H) % n;
      const float2* rp = reinterpret_cast<const float2*>(dyr + w * DH + lane * PER);
      const float2* cp = reinterpret_cast<const float2*>(cos + t * DH + lane * PER);
      const float2* sp = reinterpret_cast<const float2*>(sin + t * DH + lane * PER);
#pragma unroll
      for (int e = 0; e < PER; e += 2) {
        const float2 g2 = rp[e / 2], c2 = cp[e / 2], s2 = sp[e / 2];
        const float gv[2] = {g2.x, g2.y}, cv[2] = {c2.x, c2.y}, sv[2] = {s2.x, s2.y};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float og = __shfl_xor_sync(0xffffffffu, gv[j] * sv[j], 16);  // partner's g * sin
          d[e + j] += lane < 16 ? fmaf(gv[j], cv[j], og) : fmaf(gv[j], cv[j], -og);
        }
      }
    }
    if (qknorm) {
#pragma unroll
      for (int e = 0; e < PER; e += 2) {
        const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(x + w * DH + lane * PER + e));
        xv[e] = t.x;
        xv[e + 1] = t.y;
      }
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) ss = fmaf(xv[e], xv[e], ss);
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s);
      const float ms = ss / (float)DH;
      const float rms = sqrtf(fmaxf(ms, eps));
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        xv[e] = xv[e] / rms;  // u
        dot = fmaf(d[e], xv[e], dot);
      }
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, s);
      const int h = (int)(w % H);
      const float gr = gain[h] / rms;
      const float proj = ms > eps ? dot / (float)DH : 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) o[e] = gr * fmaf(-xv[e], proj, d[e]);
      if (lane == 0) atomicAdd(&gs[h], dot);
    } else {
#pragma unroll
      for (int e = 0; e < PER; ++e) o[e] = d[e];
    }
#pragma unroll
    for (int e = 0; e < PER; e += 2)
      *reinterpret_cast<__nv_bfloat162*>(dx + w * DH + lane * PER + e) = __floats2bfloat162_rn(o[e], o[e + 1]);
  }
  __syncthreads();
  if (qknorm && dgain != nullptr)
    for (int h = threadIdx.x; h < H; h += blockDim.x)
      if (gs[h] != 0.f) atomicAdd(&dgain[h], gs[h]);
}

template <int DH>
__global__ void __launch_bounds__(kBwThreads, 1)
    prefill_bwd_kernel(const __grid_constant__ CUtensorMap tm_qc, const __grid_constant__ CUtensorMap tm_qr,
                       const __grid_constant__ CUtensorMap tm_do, PrefillBwdParams p) {
  using SM = BwSmem<DH>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base_ptr =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SM& sm = *reinterpret_cast<SM*>(base_ptr);
  constexpr int HALVES = SM::HALVES;
  constexpr int NSLOT = SM::NSLOT;
  constexpr int HD = DH / kBwColGroups;  // a gradient warp's columns in the read-outs
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = geo.G, QT = p.QT, n = p.n;
  // the latest (longest) tiles first, one (sequence, kv head) after the
  // other: the CTAs running together add their dK / dV into one head's
  // accumulators (~50 MB at dh 128, 32K), which stay in L2 (interleaving the
  // heads instead spread the reductions over all heads' accumulators: 1.6x
  // slower at cfg2)
  const int tile = p.tiles - 1 - (int)(blockIdx.x % p.tiles);
  const int bg = blockIdx.x / p.tiles;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const int i0 = tile * QT;                 // the tile's first query
  const int nq = min(QT, n - i0);           // its queries
  const int nb = n / kBwBlock;
  const uint32_t qbox_bytes = (uint32_t)(HALVES * G * QT * 128);
  // the tile's window keys [jlo, jhi], in 64-key blocks from jla, two per chunk
  const int jlo = max(geo.S, i0 - geo.W + 1);
  const int jhi = i0 + nq - 1;
  const int jla = jlo & ~(kBwBlock - 1);
  const int nwb = jhi >= jlo ? (jhi - jla) / kBwBlock + 1 : 0;
  const int nwc = (nwb + 1) / 2;

  // ---- barriers; the query (RoPE'd when there is a window) and dO tiles ----
  if (tid == kBwLoad * 32) {
    mbar_init(&sm.q_ready, 1);
    mbar_init(&sm.qc_ready, 1);
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.p_full, kBwGradThreads);
    mbar_init(&sm.dv_full, 1);
    mbar_init(&sm.dk_full, 1);
    mbar_init(&sm.tmp_free, kBwGradThreads);
    mbar_init(&sm.dq_full, 1);
    mbar_init(&sm.dq_free, kBwGradThreads);
    mbar_init(&sm.fin, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&sm.q_ready, 2 * qbox_bytes);
    const CUtensorMap* tq = nwc > 0 ? &tm_qr : &tm_qc;
    for (int h = 0; h < HALVES; ++h) {
      tma_load_4d(sm.q + h * 16384, tq, h * 64, g * G, i0, b, &sm.q_ready);
      tma_load_4d(sm.dout + h * 16384, &tm_do, h * 64, g * G, i0, b, &sm.q_ready);
    }
  }
  // rows past the G * QT the boxes fill (G = 7: 126) are zero, so that a
  // masked P or dS of 0 never meets a non-finite value in the MMAs
  for (int r = G * QT + tid / 16; r < 128; r += kBwThreads / 16) {
    const int c16 = tid & 15;  // 16-byte chunk of the row's 256 bytes (dh 128) / 128 bytes (dh 64)
    if (c16 < HALVES * 8) {
      const int h = c16 / 8, ch = c16 % 8;
      const uint32_t off = (uint32_t)(h * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + ch * 16);
      *reinterpret_cast<uint4*>(sm.q + off) = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(sm.dout + off) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  fence_proxy_async_smem();
  // per row: query, LSE (log2 units), D
  if (tid < 128) {
    const int r = tid;
    const int qt = r / G, hh = r - (r / G) * G;
    if (r < G * QT && qt < nq) {
      const size_t ri = ((size_t)b * geo.Hq + g * G + hh) * n + i0 + qt;
      sm.rq[r] = (uint8_t)qt;
      sm.rowc[r] = make_float2(p.lse[ri] * kLog2e, p.delta[ri]);
    } else {
      sm.rq[r] = 32;
      sm.rowc[r] = make_float2(0.f, 0.f);
    }
  }

  // ---- NoPE list: the sink block, then the routed blocks the tile's queries picked (ascending) ----
  uint32_t* mask = reinterpret_cast<uint32_t*>(sm.ring[0]);  // [nb] query masks, overlaying the ring
  for (int i = tid; i < nb; i += kBwThreads) mask[i] = 0u;
  __syncthreads();
  {
    const int32_t* sel = p.sel + ((size_t)bg * n + i0) * p.list_stride;
    for (int e = tid; e < nq * p.list_stride; e += kBwThreads) {
      const int blk = sel[e];
      if (blk >= 1 && blk < nb) atomicOr(&mask[blk], 1u << (e / p.list_stride));
    }
  }
  __syncthreads();
  const int nsk = geo.S > 0 ? 1 : 0;
  {
    const int per = (nb + kBwThreads - 1) / kBwThreads;
    const int lo = tid * per, hi = min(nb, lo + per);
    int cnt = 0;
    for (int i = lo; i < hi; ++i) cnt += mask[i] != 0u;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int nv = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += nv;
    }
    if (lane == 31) sm.scan[warp] = incl;
    __syncthreads();
    int base = 0, total = 0;
    for (int w = 0; w < kBwThreads / 32; ++w) {
      if (w < warp) base += sm.scan[w];
      total += sm.scan[w];
    }
    // the host admits only 1 + QT * k <= kBwMaxEntries
    if (tid == 0) {
      sm.n_entries = min(nsk + total, kBwMaxEntries);
      if (nsk) {
        sm.eblk[0] = 0;
        sm.emask[0] = 0u;
      }
    }
    int o = nsk + base + incl - cnt;
    for (int i = lo; i < hi; ++i) {
      const uint32_t mk = mask[i];
      if (mk != 0u) {
        if (o < kBwMaxEntries) {
          sm.eblk[o] = (uint16_t)i;
          sm.emask[o] = mk;
        }
        ++o;
      }
    }
  }
  if (warp == kBwMma) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();  // the list is complete (and the mask overlay dead) from here on
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int NE = sm.n_entries;
  const int NCH = nwc + (NE + 1) / 2;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dq = tmem + 256;
  const uint32_t t_dv = tmem + (DH == 64 ? 320 : 384), t_dk = tmem + 384;

  // half h of chunk c: type, first key, the tile's query mask (routed)
  struct Half {
    int kb;
    uint32_t type, m;
  };
  auto half_of = [&](int c, int h) -> Half {
    Half x;
    x.m = 0u;
    if (c < nwc) {
      const int w = 2 * c + h;
      x.kb = jla + w * kBwBlock;
      x.type = w < nwb ? kBwWindow : kBwPad;
    } else {
      const int e = 2 * (c - nwc) + h;
      if (e >= NE) {
        x.kb = 0;
        x.type = kBwPad;
      } else {
        x.kb = (int)sm.eblk[e] * kBwBlock;
        x.type = (nsk && e == 0) ? kBwSink : kBwRouted;
        x.m = sm.emask[e];
      }
    }
    return x;
  };
  const size_t head_elems = (size_t)n * DH;  // one (sequence, kv head) of the chunk-tiled copies
  const __nv_bfloat16* kc_bg = p.kc + (size_t)bg * head_elems;
  const __nv_bfloat16* kr_bg = p.kr + (size_t)bg * head_elems;
  const __nv_bfloat16* v_bg = p.v + (size_t)bg * head_elems;
  if (warp == kBwLoad) {
    // ---------------- load producer: K(c), V(c) through the ring ----------------
    if (lane == 0) {
      for (int it = 0; it < 2 * NCH; ++it) {
        const int st = it % NSLOT, u = it / NSLOT;
        if (it >= NSLOT && !mbar_wait(&sm.empty[st], (u - 1) & 1, p.err)) break;
        const int c = it >> 1;
        const __nv_bfloat16* src = (it & 1) ? v_bg : (c < nwc ? kr_bg : kc_bg);
        const Half x0 = half_of(c, 0), x1 = half_of(c, 1);
        // a padding half loads the chunk's other block again (finite values, masked to P = 0)
        const int blk0 = x0.kb / kBwBlock, blk1 = x1.type == kBwPad ? blk0 : x1.kb / kBwBlock;
        mbar_arrive_expect_tx(&sm.full[st], SM::KT);
#pragma unroll
        for (int dg = 0; dg < HALVES; ++dg) {
          unsigned char* dst = sm.ring[st] + dg * SM::GBYTES;
          bulk_load(dst, src + ((size_t)blk0 * HALVES + dg) * 4096, 8192, &sm.full[st]);
          bulk_load(dst + 8192, src + ((size_t)blk1 * HALVES + dg) * 4096, 8192, &sm.full[st]);
        }
      }
    }
  } else if (warp == kBwMma) {
    // ---------------- MMA issuer ----------------
    // per chunk: S^T, dP^T (commit s_full; V free); after the gradient
    // warps' P^T / dS^T: dV_c, dQ (+ dK_c at dh 64) (commit dv_full), at dh
    // 128 dK_c once dV_c is read (commit dk_full); K free.  In-order
    // execution of one thread's MMAs keeps S^T(c+1) behind dV_c / dK_c,
    // which read the P^T / dS^T it overwrites.
    constexpr uint32_t idesc_t = idesc_bf16(128, 128, false, false);  // S^T, dP^T: both operands K-major
    constexpr uint32_t idesc_kv = idesc_bf16(128, DH, false, true);   // dV_c, dK_c: A in TMEM, B MN-major
    constexpr uint32_t idesc_q = idesc_bf16(128, DH, true, true);     // dQ: A = dS and B = K, both MN-major
    auto wwait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err));
    };
    auto wait_item = [&](int it) { return wwait(&sm.full[it % NSLOT], (it / NSLOT) & 1); };
    const uint64_t qdesc = sdesc_sw128(smem_u32(sm.q), 16, 1024);
    const uint64_t odesc = sdesc_sw128(smem_u32(sm.dout), 16, 1024);
    const uint64_t q_mn = sdesc_sw128(smem_u32(sm.q), 16384, 1024);     // Q as B (K = rows, N = dh)
    const uint64_t o_mn = sdesc_sw128(smem_u32(sm.dout), 16384, 1024);  // dO likewise
    const uint64_t ds_mn = sdesc_sw128(smem_u32(sm.ds[0]), 16384, 1024);
    bool ok = wwait(&sm.q_ready, 0);
    tc_fence_after();
    int tmp_uses = 0;
    bool dq_acc = false;  // dQ holds this phase's partial sums
    for (int c = 0; ok && c < NCH; ++c) {
      if (c == nwc && nwc > 0) {
        // window -> NoPE: every MMA that read the RoPE'd queries or wrote the
        // window part of dQ is complete, then the QKNorm'd tile comes in
        if (elect_one_sync()) umma_commit(&sm.dq_full);
        __syncwarp();
        if (!wwait(&sm.dq_full, 0)) break;
        if (elect_one_sync()) {
          mbar_arrive_expect_tx(&sm.qc_ready, qbox_bytes);
          for (int h = 0; h < HALVES; ++h) tma_load_4d(sm.q + h * 16384, &tm_qc, h * 64, g * G, i0, b, &sm.qc_ready);
        }
        __syncwarp();
        if (!wwait(&sm.qc_ready, 0)) break;
        tc_fence_after();
        dq_acc = false;
      }
      const int ik = 2 * c, iv = 2 * c + 1;
      if (!wait_item(ik) || !wait_item(iv)) break;
      tc_fence_after();
      const uint64_t kdesc = sdesc_sw128(smem_u32(sm.ring[ik % NSLOT]), 16, 1024);
      const uint64_t vdesc = sdesc_sw128(smem_u32(sm.ring[iv % NSLOT]), 16, 1024);
      if (elect_one_sync()) {
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const int h = kk >> 2, ko = (kk & 3) * 32;
          umma_f16(t_s, kdesc + (uint64_t)((h * SM::GBYTES + ko) >> 4), qdesc + (uint64_t)((h * 16384 + ko) >> 4),
                   idesc_t, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const int h = kk >> 2, ko = (kk & 3) * 32;
          umma_f16(t_dp, vdesc + (uint64_t)((h * SM::GBYTES + ko) >> 4), odesc + (uint64_t)((h * 16384 + ko) >> 4),
                   idesc_t, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full);
        umma_commit(&sm.empty[iv % NSLOT]);  // V is read by dP^T only
      }
      __syncwarp();
      if (!wwait(&sm.p_full, c & 1)) break;
      if (tmp_uses > 0 && !wwait(&sm.tmp_free, (tmp_uses - 1) & 1)) break;
      if (c == nwc && nwc > 0 && !wwait(&sm.dq_free, 0)) break;  // the window part of dQ has been read
      tc_fence_after();
      const uint64_t k_mn = sdesc_sw128(smem_u32(sm.ring[ik % NSLOT]), SM::GBYTES, 1024);  // K as B (K = keys)
      if (elect_one_sync()) {
        // K = 16 rows (keys) = 8 packed columns per MMA; rows [64h, 64h + 64) in columns [64h, 64h + 32)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ts(t_dv, t_s + bw_packed_col(kk), o_mn + (uint64_t)(kk * 2048 >> 4),
                      idesc_kv, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(t_dq, ds_mn + (uint64_t)(kk * 2048 >> 4), k_mn + (uint64_t)(kk * 2048 >> 4), idesc_q,
                   (dq_acc || kk > 0) ? 1u : 0u);
        if (DH == 64) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16_ts(t_dk, t_dp + bw_packed_col(kk), q_mn + (uint64_t)(kk * 2048 >> 4),
                        idesc_kv, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.dv_full);
      }
      __syncwarp();
      dq_acc = true;
      ++tmp_uses;
      if (DH == 128) {
        if (!wwait(&sm.tmp_free, (tmp_uses - 1) & 1)) break;  // dV_c has been read out
        tc_fence_after();
        if (elect_one_sync()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16_ts(t_dk, t_dp + bw_packed_col(kk), q_mn + (uint64_t)(kk * 2048 >> 4),
                        idesc_kv, kk > 0 ? 1u : 0u);
          umma_commit(&sm.dk_full);
        }
        __syncwarp();
        ++tmp_uses;
      }
      if (elect_one_sync()) umma_commit(&sm.empty[ik % NSLOT]);  // K: its S^T and dQ MMAs are done
      __syncwarp();
    }
    // drain: every MMA is complete before the final dQ read and the TMEM release
    if (elect_one_sync()) umma_commit(&sm.fin);
    __syncwarp();
    wwait(&sm.fin, 0);
  } else {
    // ---------------- gradient warps ----------------
    const int lq = warp & 3, hc = warp >> 2;  // lane quarter, column group
    const uint32_t lane_off = (uint32_t)(lq * 32) << 16;
    const int kap = lq * 32 + lane;  // key of the chunk (elementwise step, dV / dK read-outs)
    const int hk = lq >> 1;          // its half of the chunk
    const float sl2 = p.scale * kLog2e;
    const int rows_valid = G * nq;   // rows [0, G nq) hold queries of the tile
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err));
    };
    // HD consecutive TMEM columns of this thread's lane, one wait
    auto ld_cols = [&](uint32_t taddr, float* f) {
      if constexpr (HD >= 32) {
#pragma unroll
        for (int q32 = 0; q32 < HD / 32; ++q32) tmem_ld32(taddr + (uint32_t)(32 * q32), f + 32 * q32);
      } else {
        tmem_ld16(taddr, f);
      }
      tmem_ld_wait();
    };
    // read-out of a [128 x DH] fp32 accumulator with keys on the lanes: this
    // warp's DH / 2 columns of key `kap`, scaled, added into acc (null: the
    // key has no valid row); one TMEM wait for all of them
    auto kv_out = [&](uint32_t tcol, float* acc, float mul) {
      float f[HD];
      ld_cols(tcol + (uint32_t)(hc * HD) + lane_off, f);
      if (acc != nullptr) {
        float* a = acc + hc * HD;
#pragma unroll
        for (int e = 0; e < HD; e += 4) red_add4(a + e, f[e] * mul, f[e + 1] * mul, f[e + 2] * mul, f[e + 3] * mul);
      }
    };
    // read-out of dQ (rows on the lanes): this warp's DH / 2 columns of row
    // r, scaled, stored to one row of dst (or zeros)
    const int r = kap;
    const int rqt = sm.rq[r];
    const bool row_ok = rqt < 32;
    const size_t qrow = row_ok ? (((size_t)b * n + i0 + rqt) * geo.Hq + g * G + (r % G)) * DH + hc * HD : 0;
    auto dq_out = [&](float* dst, bool zero) {
      float f[HD];
      if (!zero) ld_cols(t_dq + (uint32_t)(hc * HD) + lane_off, f);
      if (row_ok) {
        float4* d4 = reinterpret_cast<float4*>(dst + qrow);
#pragma unroll
        for (int e = 0; e < HD; e += 4)
          d4[e / 4] = zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                           : make_float4(f[e] * p.scale, f[e + 1] * p.scale, f[e + 2] * p.scale, f[e + 3] * p.scale);
      }
    };
    bool ok = true;
    for (int c = 0; c < NCH; ++c) {
      const Half x = half_of(c, hk);
      const int s = x.kb + (kap & (kBwBlock - 1));  // the key's token
      // the rows of this warp's 64 row columns [64hc, 64hc + 64) this key is
      // valid for, as a bit mask: window / sink keys a range of queries, a
      // routed block the queries that picked it (G rows each)
      unsigned long long rmask = 0ull;
      bool key_live = false;
      {
        int qlo = 1, qhi = 0;
        if (x.type == kBwWindow && s >= geo.S) {
          qlo = max(0, s - i0);
          qhi = min(nq - 1, s + geo.W - 1 - i0);
        } else if (x.type == kBwSink && s < geo.S) {
          qlo = max(0, s - i0);
          qhi = nq - 1;
        }
        auto add_rows = [&](int r0, int r1) {  // rows [r0, r1) of the tile into the 64-row window
          r0 = max(r0, kBwCols * hc);
          r1 = min(min(r1, rows_valid), kBwCols * hc + kBwCols);
          if (r1 > r0) {
            const int lo = r0 - kBwCols * hc, len = r1 - r0;
            rmask |= (len >= 64 ? ~0ull : ((1ull << len) - 1ull)) << lo;
          }
        };
        if (x.type == kBwRouted) {
          key_live = x.m != 0u;
          for (uint32_t m = x.m; m != 0u; m &= m - 1u) {
            const int q = __ffs(m) - 1;
            add_rows(q * G, q * G + G);
          }
        } else if (qlo <= qhi) {
          key_live = true;
          add_rows(qlo * G, qhi * G + G);
        }
      }
      if (!wait_all(&sm.s_full, c & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // S^T / dP^T columns [kBwCols hc, + kBwCols) (rows) of this key, in pieces of 16
#pragma unroll 1
      for (int pc = 0; pc < kBwCols / 16; ++pc) {
        const int row0 = kBwCols * hc + 16 * pc;  // the piece's first row
        float sv[16], dv[16];
        tmem_ld16(t_s + (uint32_t)row0 + lane_off, sv);
        tmem_ld16(t_dp + (uint32_t)row0 + lane_off, dv);
        tmem_ld_wait();
        const uint32_t bits = (uint32_t)(rmask >> (16 * pc)) & 0xffffu;
        uint32_t pk[8], dk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          float pv[2], dsv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float2 rc = sm.rowc[row0 + e + u];
            const bool valid = (bits >> (e + u)) & 1u;
            pv[u] = valid ? ex2_approx(fmaf(sv[e + u], sl2, -rc.x)) : 0.f;
            dsv[u] = pv[u] * (dv[e + u] - rc.y);
          }
          pk[e / 2] = pack_bf16x2(pv[0], pv[1]);
          dk[e / 2] = pack_bf16x2(dsv[0], dsv[1]);
        }
        tmem_st8_nowait(t_s + (uint32_t)(kBwCols * hc + 8 * pc) + lane_off, pk);
        tmem_st8_nowait(t_dp + (uint32_t)(kBwCols * hc + 8 * pc) + lane_off, dk);
        unsigned char* dsh = sm.ds[row0 >> 6];
        *reinterpret_cast<uint4*>(dsh + sw128_offset(kap, row0 & 63)) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
        *reinterpret_cast<uint4*>(dsh + sw128_offset(kap, (row0 & 63) + 8)) = make_uint4(dk[4], dk[5], dk[6], dk[7]);
      }
      tmem_st_wait();
      fence_proxy_async_smem();  // dS in shared memory, for the dQ MMA
      tc_fence_before();
      mbar_arrive(&sm.p_full);
      // dV_c and dK_c into the accumulators (window keys: the RoPE'd keys' gradient)
      const size_t krow = (((size_t)b * n + s) * geo.Hkv + g) * DH;
      float* dv_row = key_live ? p.dv_acc + krow : nullptr;
      float* dk_row = key_live ? (x.type == kBwWindow ? p.dkr_acc : p.dk_acc) + krow : nullptr;
      if (!wait_all(&sm.dv_full, c & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      kv_out(t_dv, dv_row, 1.f);
      if (DH == 128) {
        tc_fence_before();
        mbar_arrive(&sm.tmp_free);
        if (!wait_all(&sm.dk_full, c & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      kv_out(t_dk, dk_row, p.scale);
      tc_fence_before();
      mbar_arrive(&sm.tmp_free);
      if (c == nwc - 1 && NCH > nwc) {
        // the window part of dQ (w.r.t. the RoPE'd queries), before the NoPE chunks reuse the accumulator
        if (!wait_all(&sm.dq_full, 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        dq_out(p.dqr_acc, false);
        tc_fence_before();
        mbar_arrive(&sm.dq_free);
      }
    }
    if (ok && wait_all(&sm.fin, 0)) {
      tc_fence_after();
      // every row gets exactly one store into each of dq_acc (NoPE) and dqr_acc (window)
      const bool has_w = nwc > 0, has_n = NCH > nwc;
      if (has_n) {
        dq_out(p.dq_acc, false);
        if (!has_w) dq_out(p.dqr_acc, true);
      } else {
        dq_out(p.dqr_acc, !has_w);
        dq_out(p.dq_acc, true);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kBwMma) tmem_dealloc(tmem, 512);
}


// ---------------------------------------------------------------- host ----
bool make_map(CUtensorMap* m, const void* base, int B, int n, int H, int dh, int box_h, int box_n);

bool prefill_bwd_supported(const Geom& geo, int dh, int n) {
  const int G = geo.G;
  const int QT = 128 / G;
  // the sink block and the routed union of one tile (QT x k picks) fit the
  // NoPE list; the block masks (nb x 4 bytes) fit the ring they overlay
  return !geo.hier && (dh == 64 || dh == 128) && geo.Bk == kBwBlock && G >= 4 && G <= 16 && QT * G >= 64 &&
         1 + QT * geo.K <= kBwMaxEntries && n % kBwBlock == 0 &&
         (size_t)(n / kBwBlock) * 4 <= sizeof(BwSmem<128>::ring) && geo.Hq <= kBwMaxHeads;
}

cudaError_t launch_bwd_delta(int64_t rows, int n, int H, int dh, const __nv_bfloat16* dout, const __nv_bfloat16* out,
                             float* delta, cudaStream_t st) {
  const int64_t blocks = (rows + 7) / 8;
  if (blocks == 0) return cudaSuccess;
  if (dh == 64)
    bwd_delta_kernel<64><<<(unsigned)blocks, 256, 0, st>>>(rows, n, H, dout, out, delta);
  else
    bwd_delta_kernel<128><<<(unsigned)blocks, 256, 0, st>>>(rows, n, H, dout, out, delta);
  return cudaGetLastError();
}

cudaError_t launch_bwd_norm(int64_t rows, int n, int H, int dh, const __nv_bfloat16* x, const float* dy,
                            const float* dyr, const float* cos, const float* sin, const float* gain, float eps,
                            bool qknorm, __nv_bfloat16* dx, float* dgain, cudaStream_t st) {
  const int64_t blocks = std::min<int64_t>((rows + 7) / 8, 148 * 16);
  if (blocks == 0) return cudaSuccess;
  if (H > kBwMaxHeads || (dyr != nullptr && (cos == nullptr || sin == nullptr))) return cudaErrorInvalidValue;
  if (dh == 64)
    bwd_norm_kernel<64><<<(unsigned)blocks, 256, 0, st>>>(rows, n, H, x, dy, dyr, cos, sin, gain, eps, qknorm ? 1 : 0,
                                                           dx, dgain);
  else
    bwd_norm_kernel<128><<<(unsigned)blocks, 256, 0, st>>>(rows, n, H, x, dy, dyr, cos, sin, gain, eps,
                                                            qknorm ? 1 : 0, dx, dgain);
  return cudaGetLastError();
}

cudaError_t launch_prefill_bwd(const Geom& geo, int dh, int n, float scale, const __nv_bfloat16* qc,
                               const __nv_bfloat16* qr, const __nv_bfloat16* dout, const __nv_bfloat16* kc_sw,
                               const __nv_bfloat16* kr_sw, const __nv_bfloat16* v_sw, const int32_t* sel,
                               int list_stride, const float* lse, const float* delta, float* dq_acc,
                               float* dqr_acc, float* dk_acc, float* dkr_acc, float* dv_acc, int* err,
                               cudaStream_t st) {
  const int QT = 128 / geo.G;
  CUtensorMap m_qc, m_qr, m_do;
  if (((reinterpret_cast<uintptr_t>(kc_sw) | reinterpret_cast<uintptr_t>(kr_sw) | reinterpret_cast<uintptr_t>(v_sw) |
        reinterpret_cast<uintptr_t>(dq_acc) | reinterpret_cast<uintptr_t>(dk_acc) |
        reinterpret_cast<uintptr_t>(dv_acc) | reinterpret_cast<uintptr_t>(dqr_acc) |
        reinterpret_cast<uintptr_t>(dkr_acc)) &
       15u) != 0 ||
      !make_map(&m_qc, qc, geo.B, n, geo.Hq, dh, geo.G, QT) || !make_map(&m_qr, qr, geo.B, n, geo.Hq, dh, geo.G, QT) ||
      !make_map(&m_do, dout, geo.B, n, geo.Hq, dh, geo.G, QT))
    return cudaErrorInvalidValue;
  PrefillBwdParams p{};
  p.geo = geo;
  p.n = n;
  p.scale = scale;
  p.QT = QT;
  p.tiles = (n + QT - 1) / QT;
  p.sel = sel;
  p.list_stride = list_stride;
  p.kc = kc_sw;
  p.kr = kr_sw;
  p.v = v_sw;
  p.lse = lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dqr_acc = dqr_acc;
  p.dk_acc = dk_acc;
  p.dkr_acc = dkr_acc;
  p.dv_acc = dv_acc;
  p.err = err;
  const long long grid = (long long)geo.B * geo.Hkv * p.tiles;
  if (grid <= 0) return cudaSuccess;
  if (grid > INT32_MAX) return cudaErrorInvalidValue;
  if (dh == 64) {
    const size_t smem = sizeof(BwSmem<64>) + 1024;
    static const cudaError_t attr =
        cudaFuncSetAttribute(prefill_bwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (attr != cudaSuccess) return attr;
    prefill_bwd_kernel<64><<<(unsigned)grid, kBwThreads, smem, st>>>(m_qc, m_qr, m_do, p);
  } else {
    const size_t smem = sizeof(BwSmem<128>) + 1024;
    static const cudaError_t attr =
        cudaFuncSetAttribute(prefill_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (attr != cudaSuccess) return attr;
    prefill_bwd_kernel<128><<<(unsigned)grid, kBwThreads, smem, st>>>(m_qc, m_qr, m_do, p);
  }
  return cudaGetLastError();
}

}  // namespace hba
