// Prefill routed-block selection on the 5th-generation tensor cores: the
// flat scan, and the two passes of the hierarchical selection (reference
// hier_select, src/hba/attention.py:217-246): a super pass that keeps the
// top-beam super-summaries of each query (a super is a candidate when one of
// its children is), then a child pass that scores the blocks exactly like
// the flat scan (a child's score is its block score) and keeps, per query,
// only the children of its own beam.
//
// One CTA per (128 consecutive query positions, sequence x kv head).  The
// routing queries of the tile form the A operand (M = 128 rows, K = dh) and
// each stage of candidate summaries the B operand: BPS blocks x m slots = 128
// summary rows (N = 128, K-major, TMA 128-byte swizzle straight from the
// summary tensor [B*Hkv, nb*m, dh]), so one stage's scores
//     D[query, block*m + slot] = qg . S[block, slot]     (fp32, in TMEM)
// take dh/16 tcgen05.mma instructions.  Two stages of summaries and two TMEM
// accumulators are in flight: while the epilogue reads stage s's scores the
// tensor cores compute stage s+1.
//
// Roles (192 threads):
//   warps 0-3  one thread per query row: the routing query (bf16 of the fp32
//              sum, in head order, of the group's QKNorm'd heads) into the
//              swizzled A tile; then per stage: 32-column TMEM loads, max over
//              the m slots, x scale, the candidate mask (blocks 1 .. bmax(i),
//              reference src/hba/attention.py:250-256) and a running top-k in
//              registers (score desc, block asc, as torch.topk's set with the
//              oracle's tie order; :694-698).
//   warp 4     TMEM allocation; one thread issues the MMAs.
//   warp 5     one thread issues the TMA loads of the stages.
// Scores are the tensor core's fp32 sums of exact bf16 products: they agree
// with the CUDA-core scoring order to ~1e-7 relative, so picks equal the
// oracle's up to the 1e-6-logit tie rule.  Every wait is bounded; a timeout
// sets *err and drains.
#include <climits>
#include <cudaTypedefs.h>

#include "hba_common.cuh"
#include "hba_internal.h"
#include "hba_score.cuh"
#include "hba_sm100.cuh"

namespace hba {

using namespace sm100;

constexpr int kStThreads = 192;
constexpr int kStQ = 128;  // queries per tile (UMMA M)
constexpr int kStN = 128;  // summary rows per stage (UMMA N)

template <int DH>
struct StSmem {
  static constexpr int HALVES = DH / 64;
  alignas(1024) unsigned char qg[HALVES][kStQ * 128];     // [128 queries x 64] bf16 SW128 per half
  alignas(1024) unsigned char st[2][HALVES][kStN * 128];  // [128 summary rows x 64] bf16 SW128 per half
  uint64_t s_full[2], s_empty[2], acc_full[2], acc_free[2], q_ready, drain;
  uint32_t tmem_base;
};

// KM: register list length (>= k); the list keeps the KM best, the first k
// are written.  MS: summary slots per block (m, a divisor of 32).
template <int DH, int KM, int MS>
__global__ void __launch_bounds__(kStThreads, 2)
    select_tc_kernel(const __grid_constant__ CUtensorMap tm_s, SelParams p, int* err) {
  using SM = StSmem<DH>;
  constexpr int HALVES = SM::HALVES;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  SM& sm = *reinterpret_cast<SM*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Geom& geo = p.geo;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ntile = gridDim.x;
  const int tile = ntile - 1 - blockIdx.x;  // the longest (latest) tiles first
  const int bg = blockIdx.y;
  const int b = bg / geo.Hkv, g = bg % geo.Hkv;
  const int i0 = tile * kStQ;
  const int nq = geo.nq;
  constexpr int m = MS;
  constexpr int BPS = kStN / MS;  // blocks per stage
  const float scale = p.qp.scale_fixed;
  const int nb = p.qp.n_fixed / geo.Bk;
  const bool sup_mode = p.mode == kSelSuper, child_mode = p.mode == kSelChild;
  const int F = geo.F;
  // local query i sits at position q_off + i (a query range of the sequence)
  auto bmax_of = [&](int i) { return i < nq ? min(last_candidate(p.q_off + i, geo.W, geo.Bk), nb - 1) : 0; };
  // items: blocks 1 .. bmax(i) (flat, child), or supers first .. bmax(i) / F,
  // the supers with a candidate child (super 0 holds block 0 alone when F = 1)
  const int first = sup_mode ? (F == 1 ? 1 : 0) : 1;
  auto imax_of = [&](int i) {
    const int bm = bmax_of(i);
    return sup_mode ? (bm >= 1 ? bm / F : -1) : bm;
  };
  const int imax_tile = imax_of(min(i0 + kStQ, nq) - 1);  // grows with i: the tile's largest
  const int NS = imax_tile >= first ? (imax_tile - first + BPS) / BPS : 0;
  const int k = p.list_k;

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_empty[s], 1);
      mbar_init(&sm.acc_full[s], 1);
      mbar_init(&sm.acc_free[s], 128);
    }
    mbar_init(&sm.q_ready, 128);
    mbar_init(&sm.drain, 1);
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(&sm.tmem_base, 2 * kStN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 5) {
    // ---------------- TMA producer: stage s = blocks [1 + s*BPS, 1 + (s+1)*BPS) ----------------
    if (lane == 0 && NS > 0) {
      prefetch_tmap(&tm_s);
      for (int s = 0; s < NS; ++s) {
        const int sb = s & 1;
        if (s >= 2 && !mbar_wait(&sm.s_empty[sb], ((s - 2) >> 1) & 1, err)) break;
        mbar_arrive_expect_tx(&sm.s_full[sb], (uint32_t)(HALVES * kStN * 128));
        const int row0 = (first + s * BPS) * m;  // rows past the tensor are filled with zeros (masked)
        for (int h = 0; h < HALVES; ++h) tma_load_3d(sm.st[sb][h], &tm_s, h * 64, row0, bg, &sm.s_full[sb]);
      }
    }
  } else if (warp == 4) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && NS > 0) {
      constexpr uint32_t idesc = idesc_bf16(kStQ, kStN, false, false);
      bool ok = mbar_wait(&sm.q_ready, 0, err);
      for (int s = 0; ok && s < NS; ++s) {
        const int sb = s & 1;
        if (!mbar_wait(&sm.s_full[sb], (s >> 1) & 1, err)) break;
        if (s >= 2 && !mbar_wait(&sm.acc_free[sb], ((s - 2) >> 1) & 1, err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const int h = kk >> 2, ko = (kk & 3) * 32;
          umma_f16(tmem + sb * kStN, sdesc_sw128(smem_u32(sm.qg[h]) + ko, 16, 1024),
                   sdesc_sw128(smem_u32(sm.st[sb][h]) + ko, 16, 1024), idesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_empty[sb]);
        umma_commit(&sm.acc_full[sb]);
      }
      // drain: every MMA issued above is complete before TMEM can be released
      umma_commit(&sm.drain);
      mbar_wait(&sm.drain, 0, err);
    }
  } else {
    // ---------------- routing queries, then per-row scoring and top-k ----------------
    const int r = tid;  // query row = TMEM lane
    const int i = i0 + r;
    const bool row_ok = i < nq;
    {
      // qg = bf16(sum over the G heads, in head order, of the bf16 QKNorm'd
      // query), 8 dims (one 16-byte chunk) at a time, into row r of the
      // 128-byte-swizzled A tile
      const __nv_bfloat16* qrow = p.q + (((size_t)b * nq + (row_ok ? i : 0)) * geo.Hq + (size_t)g * geo.G) * DH;
#pragma unroll 4
      for (int c = 0; c < DH / 8; ++c) {
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
        if (row_ok) {
          for (int h = 0; h < geo.G; ++h) {
            float f[8];
            unpack8(*reinterpret_cast<const uint4*>(qrow + (size_t)h * DH + c * 8), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] += f[e];
          }
        }
        const uint4 w = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                   pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
        *reinterpret_cast<uint4*>(sm.qg[c / 8] + sw128_offset(r, (c % 8) * 8)) = w;
      }
      fence_proxy_async_smem();  // the tile is read by the tensor cores
      mbar_arrive(&sm.q_ready);
    }
    const int imax = imax_of(i);
    // child pass: the row's beam (the super pass's list, -1 = none)
    int par[KM];
    const int nbeam = child_mode ? min(geo.beam, KM) : 0;
#pragma unroll
    for (int j = 0; j < KM; ++j)
      par[j] = (child_mode && row_ok && j < nbeam) ? p.in_idx[((size_t)bg * nq + i) * geo.beam + j] : -1;
    float ls[KM];
    int li[KM];
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      ls[j] = neg_inf();
      li[j] = INT_MAX;
    }
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    bool ok = true;
    for (int s = 0; s < NS; ++s) {
      const int sb = s & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.acc_full[sb], (s >> 1) & 1, err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int blo = first + s * BPS;
#pragma unroll 1
      for (int cb = 0; cb < kStN / 32; ++cb) {
        float v[32];
        tmem_ld32(tmem + sb * kStN + cb * 32 + lane_off, v);
        tmem_ld_wait();
        constexpr int bpc = 32 / MS;  // blocks in this 32-column chunk
#pragma unroll
        for (int jb = 0; jb < bpc; ++jb) {
          const int blk = blo + cb * bpc + jb;
          float best = v[jb * m];
#pragma unroll
          for (int sl = 1; sl < MS; ++sl) best = fmaxf(best, v[jb * MS + sl]);
          const float cs = best * scale;
          // candidate and better than the list's last entry (ascending items: a tie never beats)
          bool take = blk <= imax && cs > ls[KM - 1];
          if (child_mode && take) {  // a child of the row's beam
            const int sup = blk / F;
            bool in = false;
#pragma unroll
            for (int j = 0; j < KM; ++j) in |= par[j] == sup;
            take = in;
          }
          if (take) {
            // insert at the first position whose entry it beats, shifting the
            // rest down (descending j reads entry j - 1 before it moves)
#pragma unroll
            for (int j = KM - 1; j >= 0; --j) {
              const bool here = cs > ls[j];                        // beats entry j
              const bool above = j > 0 ? (cs > ls[j - 1]) : false;  // and entry j - 1
              if (here) {
                ls[j] = above ? ls[j - 1] : cs;
                li[j] = above ? li[j - 1] : blk;
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_free[sb]);
    }
    if (!ok && tid == 0) atomicExch(err, 1);
    if (row_ok) {  // lists out: [bg, query, 1, k]
      const size_t o = ((size_t)bg * nq + i) * k;
#pragma unroll
      for (int j = 0; j < KM; ++j) {
        if (j < k) {
          p.out_score[o + j] = li[j] != INT_MAX ? ls[j] : neg_inf();
          p.out_idx[o + j] = li[j] != INT_MAX ? li[j] : -1;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tmem, 2 * kStN);
}

// ---------------------------------------------------------------- host ----
static PFN_cuTensorMapEncodeTiled_v12000 st_encode_fn() {
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

bool select_tc_supported(const Geom& geo, int dh, const void* summ, const void* q, const void* supers) {
  // m | 32: a block's slots never straddle a 32-column TMEM load; hierarchical:
  // the beam fits the register list, the supers are 16-byte aligned
  return (dh == 64 || dh == 128) && (geo.m == 1 || geo.m == 2 || geo.m == 4 || geo.m == 8) && geo.K >= 1 &&
         geo.K <= 32 && (reinterpret_cast<uintptr_t>(summ) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(q) & 15u) == 0 &&
         (!geo.hier || (supers != nullptr && geo.beam >= 1 && geo.beam <= 32 && geo.F >= 1 &&
                        (reinterpret_cast<uintptr_t>(supers) & 15u) == 0)) &&
         st_encode_fn() != nullptr;
}

template <int DH, int KM, int MS>
static cudaError_t launch_st_t(const CUtensorMap& m, const SelParams& p, int* err, cudaStream_t st) {
  const size_t smem = sizeof(StSmem<DH>) + 1024;
  static const cudaError_t attr =
      cudaFuncSetAttribute(select_tc_kernel<DH, KM, MS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (attr != cudaSuccess) return attr;
  const dim3 grid((p.geo.nq + kStQ - 1) / kStQ, p.geo.B * p.geo.Hkv);
  select_tc_kernel<DH, KM, MS><<<grid, kStThreads, smem, st>>>(m, p, err);
  return cudaGetLastError();
}

template <int DH, int KM>
static cudaError_t launch_st_m(const CUtensorMap& map, const SelParams& p, int* err, cudaStream_t st) {
  switch (p.geo.m) {
    case 1: return launch_st_t<DH, KM, 1>(map, p, err, st);
    case 2: return launch_st_t<DH, KM, 2>(map, p, err, st);
    case 4: return launch_st_t<DH, KM, 4>(map, p, err, st);
    case 8: return launch_st_t<DH, KM, 8>(map, p, err, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_select_tc(const SelParams& p, int dh, int* err, cudaStream_t st) {
  auto fn = st_encode_fn();
  if (fn == nullptr) return cudaErrorInvalidValue;
  const Geom& geo = p.geo;
  // summaries [B*Hkv, nb_cap*m, dh] (super pass: supers [B*Hkv, ns_cap*m, dh])
  // bf16: box {64 dims, 128 rows, 1}, 128-byte swizzle
  const bool sup = p.mode == kSelSuper;
  const __nv_bfloat16* base = sup ? p.supers : p.summ;
  const long long rows = (long long)(sup ? geo.ns_cap : geo.nb_cap) * geo.m;
  if (base == nullptr || rows <= 0 || (p.mode == kSelChild && p.in_idx == nullptr)) return cudaErrorInvalidValue;
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)dh, (cuuint64_t)rows, (cuuint64_t)geo.B * geo.Hkv};
  cuuint64_t strides[2] = {(cuuint64_t)dh * 2, (cuuint64_t)rows * dh * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)kStN, 1};
  cuuint32_t es[3] = {1, 1, 1};
  if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16*>(base), dims, strides, box, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  // the register list holds the output list (k or the beam) and, in the child pass, the beam
  const int need = std::max(p.list_k, geo.hier ? geo.beam : 1);
  if (p.list_k < 1 || need > 32) return cudaErrorInvalidValue;
  if (dh == 64) return need <= 16 ? launch_st_m<64, 16>(map, p, err, st) : launch_st_m<64, 32>(map, p, err, st);
  return need <= 16 ? launch_st_m<128, 16>(map, p, err, st) : launch_st_m<128, 32>(map, p, err, st);
}

}  // namespace hba
