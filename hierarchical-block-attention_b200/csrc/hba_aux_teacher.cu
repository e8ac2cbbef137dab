// The summarizer's auxiliary-loss teacher on the 5th-generation tensor cores
// (reference: _teacher_chunk / _aux_kl_chunked, src/hba/attention.py:476-529;
// the same distribution as hba_attention_dense's teacher, :364-369).
//
// For query i of a KV head, over the NoPE logits scale * qc_h . kc of every
// key of its candidate blocks (blocks 1 .. bmax(i), wholly before the
// window), head h's softmax mass of block b is
//     p_h(i, b) = sum_{keys j in b} exp(s_h(i, j) - LSE_h(i)),
// LSE_h(i) the log-sum-exp over all candidate keys (the reference's softmax
// over blockwise LSEs); the teacher is the mean over the group's G heads,
// pstar(i, b) = mean_h p_h(i, b).  It sums to 1 over blocks by construction
// (the reference's renormalisation only corrects rounding, and is not
// repeated here); non-candidate blocks and queries with no candidate are 0.
//
// One CTA per (sequence, kv head, tile of QT = 128/G queries x G heads = the
// 128 rows of the UMMA M dimension).  The tile's candidate blocks are walked
// twice in 128-key chunks (two 64-key blocks each): S = Q K^T (M 128 rows, N
// 128 keys, K dh) into one of two TMEM buffers, so the next chunk's MMA runs
// while the row warps read one.
//   pass 1: per row the running maximum and sum of 2^(s log2e - m) over its
//           valid keys -> LSE (log2 units);
//   pass 2: per row and block the mass 2^(s log2e - LSE), then the mean over
//           the G rows of each query (through shared memory) -> pstar.
// Roles (320 threads): warps 0-7 the rows (TMEM lane = row), two warps per
// lane quarter, one per 64-key block of the chunk (one warp's exponentials
// alone are latency-bound on the MUFU); warp 8 loads (the query tile by TMA,
// K chunks by 1-D bulk copies of the pre-pass's chunk-tiled keys through a
// ring); warp 9 issues the MMAs and owns
// TMEM.  Every mbarrier wait is bounded; a timeout sets *err and drains.
#include <algorithm>
#include <climits>
#include <cudaTypedefs.h>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_score.cuh"
#include "hba_sm100.cuh"

namespace hba {

using namespace sm100;

constexpr int kAtThreads = 320;
constexpr int kAtRowThreads = 256;  // warps 0-7: two per TMEM lane quarter, one per 64-key block of a chunk
constexpr int kAtLoad = 8;
constexpr int kAtMma = 9;
constexpr int kAtBlock = 64;
constexpr int kAtKeys = 128;
constexpr size_t kAuxScratchCap = size_t(1) << 30;  // single-pass scratch: at most 1 GiB (the host slices the queries)

template <int DH>
struct AtSmem {
  static constexpr int HALVES = DH / 64;
  static constexpr int QBYTES = HALVES * 16384;  // [128 rows x DH], swizzled per 64-dim group
  static constexpr int GBYTES = kAtKeys * 128;   // one dim group of a K chunk
  static constexpr int KT = HALVES * GBYTES;
  static constexpr int NSLOT = DH == 64 ? 8 : 4;
  alignas(1024) unsigned char q[QBYTES];
  alignas(1024) unsigned char ring[NSLOT][KT];
  float mass[2][2][128];  // pass 2: [chunk parity][block half][row]
  float ml[2][2][128];    // end of pass 1: [block half][m, l][row]
  float trow[128];        // single pass: the row's total mass
  uint64_t q_ready, full[NSLOT], empty[NSLOT], s_full[2], s_free[2], mass_full[2], ml_full, drain;
  uint32_t tmem_base;
};

static_assert(sizeof(AtSmem<128>) + 1024 <= 232448 && sizeof(AtSmem<64>) + 1024 <= 232448,
              "teacher tile set exceeds the 227 KB of shared memory");

struct AuxTeacherParams {
  Geom geo;
  int n;
  float scale;
  int QT;
  int tiles;
  const __nv_bfloat16* kc;  // chunk-tiled QKNorm'd (or raw) keys
  float* pstar;             // [B, Hkv, n, nb], zeroed by the host
  int* err;
  // queries [q0, q0 + nsl) of every sequence (a slice; the host loops)
  int q0, nsl;
  // single pass (QKNorm, bounded logits): k_gain bounds the keys' norms;
  // scratch [B*Hkv, nsl, nb, G] fp32 holds each head row's block masses
  const float* k_gain;
  float* scratch;
};

template <int DH>
__global__ void __launch_bounds__(kAtThreads, 1)
    aux_teacher_kernel(const __grid_constant__ CUtensorMap tm_q, AuxTeacherParams p) {
  using SM = AtSmem<DH>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  SM& sm = *reinterpret_cast<SM*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int HALVES = SM::HALVES;
  constexpr int NSLOT = SM::NSLOT;
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = geo.G, QT = p.QT, n = p.n;
  const int tile = p.tiles - 1 - (int)(blockIdx.x % p.tiles);  // the latest (longest) tiles first
  const int bg = blockIdx.x / p.tiles;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const int i0 = p.q0 + tile * QT;
  const int nq = min(QT, p.q0 + p.nsl - i0);
  const int nb = n / kAtBlock;
  auto bmax_of = [&](int i) { return min(last_candidate(i, geo.W, kAtBlock), nb - 1); };
  const int bmaxT = bmax_of(i0 + nq - 1);      // the tile's last candidate block (0: none)
  const int NCH = bmaxT >= 1 ? (bmaxT + 1) / 2 : 0;  // chunk c: blocks 1 + 2c, 2 + 2c
  if (NCH == 0) return;                         // no candidate anywhere in the tile: pstar stays 0

  if (tid == kAtLoad * 32) {
    mbar_init(&sm.q_ready, 1);
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], kAtRowThreads);
      mbar_init(&sm.mass_full[s], kAtRowThreads);
    }
    mbar_init(&sm.ml_full, kAtRowThreads);
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&sm.q_ready, (uint32_t)(HALVES * G * QT * 128));
    for (int h = 0; h < HALVES; ++h) tma_load_4d(sm.q + h * 16384, &tm_q, h * 64, g * G, i0, b, &sm.q_ready);
  }
  if (warp == kAtMma) {
    tmem_alloc(&sm.tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // One pass when every row's logits are bounded (QKNorm: |s| <= scale |q|
  // sqrt(dh) k_gain, with a 1/64 margin for the bf16 keys; the forward's
  // bounded mode): masses 2^(s log2e - M2) never flush to zero, and each
  // row's total normalises them at the end.  Otherwise two passes (the row
  // LSE, then the masses).  Every thread waits for the query tile to decide.
  const float sl2 = p.scale * kLog2e;
  float M2 = 0.f;
  bool unbounded = !geo.qknorm || p.scratch == nullptr;
  if (!__all_sync(0xffffffffu, mbar_wait(&sm.q_ready, 0, p.err))) unbounded = true;
  if (!unbounded && tid < 128) {
    const int qt = tid / G;
    if (tid < G * QT && qt < nq) {
      float qn2 = 0.f;
#pragma unroll
      for (int d8 = 0; d8 < DH / 8; ++d8) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(sm.q + (d8 / 8) * 16384 + sw128_offset(tid, (d8 % 8) * 8)), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) qn2 = fmaf(f[e], f[e], qn2);
      }
      M2 = p.scale * sqrtf(qn2) * (sqrtf((float)DH) * p.k_gain[g] * (1.f + 1.f / 64.f)) * kLog2e;
      unbounded = !(M2 <= kBoundedLog2);
    }
  }
  const bool single = !__syncthreads_or(unbounded ? 1 : 0);
  if (tid < 128) sm.trow[tid] = M2;  // the row's bound, read by its two row warps
  __syncthreads();
  const int NIT = single ? NCH : 2 * NCH;  // item it: chunk it % NCH, pass it / NCH

  if (warp == kAtLoad) {
    if (lane == 0) {
      const __nv_bfloat16* kc_bg = p.kc + (size_t)bg * n * DH;
      for (int it = 0; it < NIT; ++it) {
        const int st = it % NSLOT;
        if (it >= NSLOT && !mbar_wait(&sm.empty[st], ((it / NSLOT) - 1) & 1, p.err)) break;
        const int c = it % NCH;
        const int blk0 = 1 + 2 * c, blk1 = min(2 + 2 * c, bmaxT);  // past the last candidate: a valid block, masked
        mbar_arrive_expect_tx(&sm.full[st], SM::KT);
#pragma unroll
        for (int dg = 0; dg < HALVES; ++dg) {
          unsigned char* dst = sm.ring[st] + dg * SM::GBYTES;
          bulk_load(dst, kc_bg + ((size_t)blk0 * HALVES + dg) * 4096, 8192, &sm.full[st]);
          bulk_load(dst + 8192, kc_bg + ((size_t)blk1 * HALVES + dg) * 4096, 8192, &sm.full[st]);
        }
      }
    }
  } else if (warp == kAtMma) {
    constexpr uint32_t idesc = idesc_bf16(128, kAtKeys, false, false);
    auto wwait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.err));
    };
    bool ok = wwait(&sm.q_ready, 0);
    const uint64_t qdesc = sdesc_sw128(smem_u32(sm.q), 16, 1024);
    for (int it = 0; ok && it < NIT; ++it) {
      const int st = it % NSLOT, sb = it & 1;
      if (!wwait(&sm.full[st], (it / NSLOT) & 1)) break;
      if (it >= 2 && !wwait(&sm.s_free[sb], ((it - 2) >> 1) & 1)) break;
      tc_fence_after();
      const uint64_t kdesc = sdesc_sw128(smem_u32(sm.ring[st]), 16, 1024);
      if (elect_one_sync()) {
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const int h = kk >> 2, ko = (kk & 3) * 32;
          umma_f16(tmem + (uint32_t)(sb * kAtKeys), qdesc + (uint64_t)((h * 16384 + ko) >> 4),
                   kdesc + (uint64_t)((h * SM::GBYTES + ko) >> 4), idesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full[sb]);
        umma_commit(&sm.empty[st]);
      }
      __syncwarp();
    }
    if (elect_one_sync()) umma_commit(&sm.drain);
    __syncwarp();
    wwait(&sm.drain, 0);
  } else {
    // ---------------- row warps: row r = TMEM lane, warp half hb = block 1 + 2c + hb ----------------
    const int lq = warp & 3, hb = warp >> 2;
    const int r = lq * 32 + lane;
    const int qt = r / G;
    const bool row_ok = r < G * QT && qt < nq;
    const int bmax = row_ok ? bmax_of(i0 + qt) : 0;  // the row's last candidate block (0: none)
    const uint32_t lane_off = (uint32_t)(lq * 32) << 16;
    const float m2row = sm.trow[r];
    float m = neg_inf(), l = 0.f, lse2 = neg_inf();
    float tot = 0.f;  // single pass: the row's mass over this warp's blocks
    bool ok = true;
    // single pass: this row's slot in the scratch ([bg, query - q0, blk, head])
    float* srow = single && row_ok
                      ? p.scratch + ((size_t)bg * p.nsl + (i0 + qt - p.q0)) * nb * G + (r - qt * G)
                      : nullptr;
    for (int it = 0; it < NIT; ++it) {
      const int sb = it & 1, c = it % NCH;
      const bool pass2 = !single && it >= NCH;
      if (pass2 && it == NCH) {
        // the row's LSE over both halves' keys (log2 units)
        sm.ml[hb][0][r] = m;
        sm.ml[hb][1][r] = l;
        mbar_arrive(&sm.ml_full);
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.ml_full, 0, p.err))) {
          ok = false;
          break;
        }
        const float m0 = sm.ml[0][0][r], l0 = sm.ml[0][1][r], m1 = sm.ml[1][0][r], l1 = sm.ml[1][1][r];
        const float mm = fmaxf(m0, m1);
        const float ll = (l0 > 0.f ? l0 * ex2_approx(m0 - mm) : 0.f) + (l1 > 0.f ? l1 * ex2_approx(m1 - mm) : 0.f);
        lse2 = ll > 0.f ? mm + log2f(ll) : neg_inf();
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[sb], (it >> 1) & 1, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[64];
      tmem_ld32(tmem + (uint32_t)(sb * kAtKeys + 64 * hb) + lane_off, v);
      tmem_ld32(tmem + (uint32_t)(sb * kAtKeys + 64 * hb + 32) + lane_off, v + 32);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&sm.s_free[sb]);  // the buffer may take chunk it + 2's scores
      const bool valid = 1 + 2 * c + hb <= bmax;  // the half is one block
      float mass = 0.f;
      if (single) {
        if (valid) {
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int e = 0; e < 64; e += 2) {
            s0 += ex2_approx(fmaf(v[e], sl2, -m2row));
            s1 += ex2_approx(fmaf(v[e + 1], sl2, -m2row));
          }
          mass = s0 + s1;
          tot += mass;
        }
        const int blk = 1 + 2 * c + hb;
        if (srow != nullptr && blk <= bmaxT) srow[(size_t)blk * G] = mass;
        continue;
      }
      if (valid) {
        if (!pass2) {
          float mx = neg_inf();
#pragma unroll
          for (int e = 0; e < 64; ++e) mx = fmaxf(mx, v[e]);
          const float mn = fmaxf(m, mx * sl2);
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int e = 0; e < 64; e += 2) {
            s0 += ex2_approx(fmaf(v[e], sl2, -mn));
            s1 += ex2_approx(fmaf(v[e + 1], sl2, -mn));
          }
          l = l * ex2_approx(m - mn) + (s0 + s1);  // m = -inf at the first valid block: 2^-inf = 0
          m = mn;
        } else {
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int e = 0; e < 64; e += 2) {
            s0 += ex2_approx(fmaf(v[e], sl2, -lse2));
            s1 += ex2_approx(fmaf(v[e + 1], sl2, -lse2));
          }
          mass = s0 + s1;
        }
      }
      if (pass2) {
        // the mean over the G rows (heads) of each query -> pstar.  The
        // arrays alternate by chunk parity: every row thread waits for chunk
        // j's masses before writing chunk j + 1's, so chunk j + 2 overwrites
        // parity j only after every thread has read chunk j.
        const int j = c, pj = j & 1;
        sm.mass[pj][hb][r] = mass;
        mbar_arrive(&sm.mass_full[pj]);
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.mass_full[pj], (j >> 1) & 1, p.err))) {
          ok = false;
          break;
        }
        for (int e = tid; e < 2 * nq; e += kAtRowThreads) {
          const int q_ = e >> 1, h = e & 1;
          const int blk = 1 + 2 * c + h;
          if (blk <= bmaxT) {
            float sum = 0.f;
            for (int hh = 0; hh < G; ++hh) sum += sm.mass[pj][h][q_ * G + hh];
            p.pstar[((size_t)bg * n + i0 + q_) * nb + blk] = sum / (float)G;
          }
        }
      }
    }
    if (single && ok) {
      // each row's total over both halves, then per (query, block) the mean
      // over the G head rows of mass / total -> pstar
      sm.ml[hb][1][r] = tot;
      mbar_arrive(&sm.ml_full);
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.ml_full, 0, p.err));
      if (ok) {
        const float* sbase = p.scratch + ((size_t)bg * p.nsl + (i0 - p.q0)) * nb * G;
        const int per_q = bmaxT;  // blocks 1 .. bmaxT
        for (int e = tid; e < nq * per_q; e += kAtRowThreads) {
          const int q_ = e / per_q, blk = 1 + e % per_q;
          float sum = 0.f;
          for (int hh = 0; hh < G; ++hh) {
            const int rr = q_ * G + hh;
            const float t = sm.ml[0][1][rr] + sm.ml[1][1][rr];
            if (t > 0.f) sum += sbase[((size_t)q_ * nb + blk) * G + hh] / t;
          }
          p.pstar[((size_t)bg * n + i0 + q_) * nb + blk] = sum / (float)G;
        }
      }
    }
    if (!ok && tid == 0) atomicExch(p.err, 1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kAtMma) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------- host ----
bool make_map(CUtensorMap* m, const void* base, int B, int n, int H, int dh, int box_h, int box_n);

bool aux_teacher_supported(const Geom& geo, int dh, int n) {
  return !geo.hier && (dh == 64 || dh == 128) && geo.Bk == kAtBlock && n % kAtBlock == 0 && geo.G >= 1 &&
         geo.G <= 16;
}

size_t aux_teacher_scratch_bytes(const Geom& geo, int n) {
  const size_t per_query = (size_t)geo.B * geo.Hq * (n / kAtBlock) * sizeof(float);
  const size_t all = per_query * (size_t)n;
  return std::min(all, std::max(kAuxScratchCap, per_query * (size_t)(128 / geo.G)));
}

cudaError_t launch_aux_teacher(const Geom& geo, int dh, int n, float scale, const __nv_bfloat16* qc,
                               const __nv_bfloat16* kc_sw, const float* k_gain, float* scratch,
                               size_t scratch_bytes, float* pstar, int* err, cudaStream_t st) {
  const int QT = 128 / geo.G;
  CUtensorMap m_q;
  if ((reinterpret_cast<uintptr_t>(kc_sw) & 15u) != 0 || !make_map(&m_q, qc, geo.B, n, geo.Hq, dh, geo.G, QT))
    return cudaErrorInvalidValue;
  AuxTeacherParams p{};
  p.geo = geo;
  p.n = n;
  p.scale = scale;
  p.QT = QT;
  p.kc = kc_sw;
  p.pstar = pstar;
  p.err = err;
  p.k_gain = k_gain;
  // the single pass keeps [slice queries x nb x Hq] masses: slices of whole tiles fitting the scratch
  const size_t per_query = (size_t)geo.B * geo.Hq * (n / kAtBlock) * sizeof(float);
  int nsl = n;
  if (geo.qknorm && k_gain != nullptr && scratch != nullptr && scratch_bytes >= per_query * QT) {
    nsl = (int)std::min<size_t>((size_t)n, (scratch_bytes / per_query) / QT * QT);
    p.scratch = scratch;
  }
  const size_t smem = (dh == 64 ? sizeof(AtSmem<64>) : sizeof(AtSmem<128>)) + 1024;
  static const cudaError_t attr64 =
      cudaFuncSetAttribute(aux_teacher_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)(sizeof(AtSmem<64>) + 1024));
  static const cudaError_t attr128 =
      cudaFuncSetAttribute(aux_teacher_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)(sizeof(AtSmem<128>) + 1024));
  if ((dh == 64 ? attr64 : attr128) != cudaSuccess) return dh == 64 ? attr64 : attr128;
  for (int q0 = 0; q0 < n; q0 += nsl) {
    p.q0 = q0;
    p.nsl = std::min(nsl, n - q0);
    p.tiles = (p.nsl + QT - 1) / QT;
    const long long grid = (long long)geo.B * geo.Hkv * p.tiles;
    if (grid <= 0) continue;
    if (grid > INT32_MAX) return cudaErrorInvalidValue;
    if (dh == 64)
      aux_teacher_kernel<64><<<(unsigned)grid, kAtThreads, smem, st>>>(m_q, p);
    else
      aux_teacher_kernel<128><<<(unsigned)grid, kAtThreads, smem, st>>>(m_q, p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace hba
