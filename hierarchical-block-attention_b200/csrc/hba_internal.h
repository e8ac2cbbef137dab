// Internal parameter blocks and launcher declarations shared by the kernel
// translation units and the C-ABI layer (hba_api.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hba {

constexpr int kShardMaxRanks = 8;

// Exchange buffer of the fused shard decode (one per rank, IPC-mapped by the
// others), for BH = B * Hkv (sequence, kv head) rows and `world` ranks:
// two list regions [BH][world][32] and the (O, l, M) partials
// [BH][world][16 * dh + 32] (O^T [16 heads][dh], l [16], the reference
// maximum M [16]), all of self-validating 64-bit words -- a list
// entry is (score bits | block id (16 bits) << 32 | epoch (16 bits) << 48),
// a partial value (fp32 bits | epoch << 32) -- written by one aligned 64-bit
// store each, so a reader that sees this step's epoch in a word has its data
// (no fence, no flag).
struct XLayout {
  size_t list[2], parts, total;
};
__host__ __device__ inline XLayout x_layout(int BH, int world, int dh) {
  XLayout l;
  size_t o = 0;
  for (int x = 0; x < 2; ++x) {
    l.list[x] = o;
    o += (size_t)BH * world * 32 * 8;
  }
  l.parts = o;
  o += (size_t)BH * world * (16 * dh + 32) * 8;
  l.total = o;
  return l;
}

// Where a query sits: decode (one query per sequence at seq_lens[b]-1 over a
// cache of seq_lens[b] tokens, per-sequence scale) or prefill (query t of a
// length-n sequence at position t, one scale).
struct QueryPos {
  const int32_t* seq_lens;  // decode: [B]; prefill: nullptr
  const float* scales;      // decode: [B]; prefill: nullptr
  int32_t n_fixed;          // prefill sequence length
  float scale_fixed;        // prefill scale
};

// Geometry shared by selection and attention kernels.
struct Geom {
  int32_t B, Hq, Hkv, G, m, Bk, W, S, K, F, beam, hier, qknorm;
  float eps;
  int32_t nq;      // queries per sequence in this launch (decode 1, prefill n)
  int32_t n_cap;   // token capacity of the key/value buffers
  int32_t nb_cap;  // block capacity of the summary buffer
  int32_t ns_cap;  // super capacity of the super buffer
};

enum SelMode : int32_t { kSelFlat = 0, kSelSuper = 1, kSelChild = 2 };

struct SelParams {
  Geom geo;
  QueryPos qp;
  int32_t mode;
  int32_t splits;      // gridDim.x
  int32_t list_k;      // entries per output list (K, or beam for supers)
  int32_t in_lists;    // child mode: super lists per query
  const __nv_bfloat16* q;       // [B, nq, Hq, dh]
  const float* q_gain;          // [Hq]
  const __nv_bfloat16* summ;    // [B, Hkv, nb_cap, m, dh]
  const __nv_bfloat16* supers;  // [B, Hkv, ns_cap, m, dh]
  const float* in_score;        // child mode: [B*Hkv, nq, in_lists, beam]
  const int32_t* in_idx;
  float* out_score;             // [B*Hkv, nq, splits, list_k]
  int32_t* out_idx;
  int32_t* counters;            // decode: [B*Hkv] merge counters zeroed here, or null
  int32_t pdl;                  // launched as a programmatic dependent of the previous kernel
  // KV-range shard: candidate blocks restricted to [own_blo, own_bhi) (supers
  // to [own_blo/F, own_bhi/F)); summary row r of this shard holds block
  // own_blo + r (super own_blo/F + r).  One GPU: 0, INT_MAX.
  int32_t own_blo, own_bhi;
  int32_t n_limit;  // longest valid context (one GPU: n_cap; a shard: the global capacity)
  int32_t q_normed;  // q is already QKNorm'd (select_tile_kernel only)
  int32_t q_off;     // position of local query 0 (select_tc_kernel: a query range of the sequence)
};

struct AttnParams {
  Geom geo;
  QueryPos qp;
  int32_t splits;      // gridDim.x (key-range partitions per query)
  int32_t in_lists;    // selection lists per query to merge
  int32_t list_k;      // entries per selection list
  const __nv_bfloat16* q;   // [B, nq, Hq, dh] raw
  const float* q_gain;
  const __nv_bfloat16* k;   // [B, n_cap, Hkv, dh] QKNorm'd NoPE keys
  const __nv_bfloat16* kr;  // [B, n_cap, Hkv, dh] the same keys RoPE'd at their positions
  const __nv_bfloat16* v;   // [B, n_cap, Hkv, dh]
  const float* cos;         // [n_cap, dh] (query rotation)
  const float* sin;
  const float* in_score;    // [B*Hkv, nq, in_lists, list_k]
  const int32_t* in_idx;
  __nv_bfloat16* out;       // [B, nq, Hq, dh]      (splits == 1)
  float* lse;               // [B, Hq, nq] or null  (splits == 1)
  float* part;              // [B*Hkv, nq, splits, 16, dh + 2] (splits > 1)
  int32_t* sel_idx;         // [B, Hkv, nq, K] or null
  float* sel_score;
};

// Decode attention over a flattened chunk sequence: for every (sequence, kv
// head) `nchunk` 64-key chunk slots [window | sinks | routed]; CTA c takes the
// contiguous slots [c*T/N, (c+1)*T/N) of the T = B*Hkv*nchunk total.
struct DecodeAttnParams {
  Geom geo;
  unsigned long long* trace;  // debug: 16 global-timer stamps per CTA, or null
  long long trace_ctas;
  QueryPos qp;
  int32_t ncw;          // window chunk slots per (sequence, kv head)
  int32_t ncr;          // routed chunk slots
  int32_t nchunk;       // ncw + 1 + ncr
  int32_t in_lists;     // selection lists per query to merge
  int32_t list_k;
  int32_t max_seg;      // partial slots per (sequence, kv head)
  const __nv_bfloat16* q;
  const float* q_gain;
  const __nv_bfloat16* k;
  const __nv_bfloat16* kr;
  const __nv_bfloat16* v;
  const float* cos;
  const float* sin;
  const float* in_score;
  const int32_t* in_idx;
  __nv_bfloat16* out;   // [B, Hq, dh]
  float* lse;           // [B, Hq] or null
  int32_t* sel_idx;     // [B, Hkv, K] or null
  float* sel_score;
  float* part;          // [B*Hkv, max_seg, G, dh + 2]
  int32_t* counters;    // [B*Hkv], zeroed by the selection kernel of this call
};

cudaError_t launch_qknorm(const __nv_bfloat16* x, __nv_bfloat16* y, const float* gain, int64_t rows,
                          int heads, int dh, float eps, cudaStream_t st);
cudaError_t launch_append(const Geom& geo, int t, const int32_t* pos, const __nv_bfloat16* k_new,
                          const __nv_bfloat16* v_new, const float* k_gain, const float* cos, const float* sin,
                          __nv_bfloat16* k_cache, __nv_bfloat16* kr_cache, __nv_bfloat16* v_cache, int dh,
                          cudaStream_t st);
// k (QKNorm'd, or copied) and kr = RoPE(k) for a whole [B, n, Hkv, dh] tensor.
// With kc_sw: kc, plus kc, RoPE(kc) and v (when given) in the chunk-tiled
// layout of the tensor-core prefill ([B, Hkv, n/64, dh/64] tiles of the
// 8 KB 128-byte-swizzled [64 tokens x 64 dims] image; n % 64 == 0), kr unused.
cudaError_t launch_qknorm_rope(const Geom& geo, int n, const __nv_bfloat16* k, const float* k_gain,
                               const float* cos, const float* sin, __nv_bfloat16* kc, __nv_bfloat16* kr, int dh,
                               cudaStream_t st, const __nv_bfloat16* v = nullptr, __nv_bfloat16* kc_sw = nullptr,
                               __nv_bfloat16* kr_sw = nullptr, __nv_bfloat16* v_sw = nullptr, int pos0 = 0);
// Summaries of blocks [blk_begin, blk_end) for every sequence; if pos/t are
// given (append), only blocks completed by tokens [pos[b], pos[b]+t) of
// sequence b are rebuilt.
// k_cache token-major [B, n_cap, Hkv, dh], or (tiled) the KV cache's chunk-tiled layout
cudaError_t launch_summarize(const Geom& geo, int dh, const __nv_bfloat16* k_cache, const float* probes,
                             const float* proj, __nv_bfloat16* summ, int blk_begin, int blk_end,
                             const int32_t* pos, int t, cudaStream_t st, bool tiled = false);
cudaError_t launch_supers(const Geom& geo, int dh, int nb_fixed, const __nv_bfloat16* summ,
                          __nv_bfloat16* supers, int s_begin, int s_end, const int32_t* pos, int t,
                          cudaStream_t st);
cudaError_t launch_select(const SelParams& p, int dh, cudaStream_t st);
cudaError_t launch_attend(const AttnParams& p, int dh, cudaStream_t st);
cudaError_t launch_decode_attend(const DecodeAttnParams& p, int dh, int grid, cudaStream_t st);
// One CTA per (sequence, kv head): selection and attention fused (no scratch).
cudaError_t launch_decode_fused(const DecodeAttnParams& p, const __nv_bfloat16* summ, const __nv_bfloat16* supers,
                                int dh, cudaStream_t st);
size_t decode_fused_smem(int dh);
// tcgen05 decode (hba_decode_tc.cu): one CTA per (sequence, kv head), QKNorm only.
// Prefill flat selection tiled over 64 queries per CTA (scores identical to
// select_kernel's); writes one list of p.list_k per query.
bool select_tile_supported(const Geom& geo, int dh, const void* summ);
cudaError_t launch_select_tile(const SelParams& p, int dh, int* err, cudaStream_t st);
// Prefill flat selection on tcgen05 (hba_select_tc.cu): 128 queries per CTA,
// scores as a UMMA GEMM per stage of summaries, top-k from TMEM; p.q holds the
// QKNorm'd queries.  Writes one list of p.list_k per query.
bool select_tc_supported(const Geom& geo, int dh, const void* summ, const void* q, const void* supers);
cudaError_t launch_select_tc(const SelParams& p, int dh, int* err, cudaStream_t st);
// KV-range shard: the union over this shard's tokens [tok_lo, tok_lo + n_cap)
// as unnormalised partials (O, l, m) -- m the softmax reference maximum in
// log2 units -- after merging n_in candidate picks per (sequence, kv head)
// into the global top-k; and the max-rescaled merge of every rank's partials.
cudaError_t launch_decode_tc_shard(const DecodeAttnParams& p, const float* k_gain, int* err, int dh, int tok_lo,
                                   const int32_t* in_idx, const float* in_score, int n_in, float* part_o,
                                   float* part_l, float* part_m2, cudaStream_t st);
// Fused KV-range shard (mode 2): selection of the owned candidates, the list
// and partial exchanges with the other ranks over their IPC-mapped exchange
// buffers xbufs[0 .. world) (x_layout), and the union of the owned tokens, in
// one launch after a one-thread epoch bump.
cudaError_t launch_decode_tc_fused(const DecodeAttnParams& p, const __nv_bfloat16* summ, const __nv_bfloat16* supers,
                                   const float* k_gain, int* err, int dh, int tok_lo, int world, int rank,
                                   int32_t* epoch, void* const* xbufs, cudaStream_t st);
// parts: [world][rows * (dh + 2)] fp32, per rank [m (rows) | l (rows) | O (rows x dh)].
cudaError_t launch_shard_finish(int rows, int dh, int world, const float* parts, __nv_bfloat16* out, float* lse,
                                cudaStream_t st);
bool decode_tc_supported(const Geom& geo, int dh, const void* k, const void* kr, const void* v, const void* summ,
                         const void* supers);
cudaError_t launch_decode_tc(const DecodeAttnParams& p, const __nv_bfloat16* summ, const __nv_bfloat16* supers,
                             const float* k_gain, int* err, int dh, cudaStream_t st);
// tcgen05/TMEM prefill union softmax (hba_prefill_tc.cu).
bool prefill_tc_supported(const Geom& geo, int dh, int n, bool qknorm);
// qc / qr: the queries QKNorm'd and RoPE'd by the pre-pass, [B, n, Hq, dh] bf16;
// kc_sw / kr_sw / v_sw: the keys QKNorm'd, RoPE'd, and the values, in the
// pre-pass's chunk-tiled layout.
// geo.nq local queries at positions q_off .. over n keys.
cudaError_t launch_prefill_tc(const Geom& geo, int dh, int n, int q_off, float scale, const __nv_bfloat16* qc,
                              const __nv_bfloat16* qr, const float* k_gain, const __nv_bfloat16* kc_sw,
                              const __nv_bfloat16* kr_sw, const __nv_bfloat16* v_sw,
                              const int32_t* sel, int list_stride, __nv_bfloat16* out, float* lse, int* err,
                              unsigned long long* trace, long long trace_rows, cudaStream_t st);
// CTAs the decode attention grid should have for this device (all resident at once).
int decode_attend_grid(int dh, int total_chunks);
// The summarizer's aux-KL teacher (hba_aux_teacher.cu): qc [B, n, Hq, dh]
// bf16 (QKNorm'd or raw queries), kc_sw the chunk-tiled keys; pstar [B, Hkv,
// n, nb] fp32, zeroed first.
bool aux_teacher_supported(const Geom& geo, int dh, int n);
// scratch (aux_teacher_scratch_bytes, may be null: two passes) lets rows
// with bounded logits (QKNorm, k_gain) run in one pass.
size_t aux_teacher_scratch_bytes(const Geom& geo, int n);
cudaError_t launch_aux_teacher(const Geom& geo, int dh, int n, float scale, const __nv_bfloat16* qc,
                               const __nv_bfloat16* kc_sw, const float* k_gain, float* scratch,
                               size_t scratch_bytes, float* pstar, int* err, cudaStream_t st);
// Backward of the prefill union softmax (hba_prefill_bwd.cu).
bool prefill_bwd_supported(const Geom& geo, int dh, int n);
// delta[b, h, t] = sum_d dout * out over rows (b, t, h) of [B, n, H, dh] bf16.
cudaError_t launch_bwd_delta(int64_t rows, int n, int H, int dh, const __nv_bfloat16* dout, const __nv_bfloat16* out,
                             float* delta, cudaStream_t st);
// dx (bf16) = QKNorm's backward of dy + RoPE^T(dyr) (fp32; dyr may be null)
// at x, dgain[h] += sum dy * x / rms; or that sum alone without QKNorm.
cudaError_t launch_bwd_norm(int64_t rows, int n, int H, int dh, const __nv_bfloat16* x, const float* dy,
                            const float* dyr, const float* cos, const float* sin, const float* gain, float eps,
                            bool qknorm, __nv_bfloat16* dx, float* dgain, cudaStream_t st);
// qc / qr: the pre-pass's QKNorm'd / RoPE'd queries, dout [B, n, Hq, dh] bf16;
// kc_sw / kr_sw / v_sw chunk-tiled; sel the forward's picks [B*Hkv, n,
// list_stride]; lse / delta [B, Hq, n]; dq_acc / dqr_acc (w.r.t. the
// QKNorm'd / RoPE'd queries) written, dk_acc / dkr_acc / dv_acc accumulated
// (zero them first), all fp32 in the q / k layouts.
cudaError_t launch_prefill_bwd(const Geom& geo, int dh, int n, float scale, const __nv_bfloat16* qc,
                               const __nv_bfloat16* qr, const __nv_bfloat16* dout, const __nv_bfloat16* kc_sw,
                               const __nv_bfloat16* kr_sw, const __nv_bfloat16* v_sw, const int32_t* sel,
                               int list_stride, const float* lse, const float* delta, float* dq_acc,
                               float* dqr_acc, float* dk_acc, float* dkr_acc, float* dv_acc, int* err,
                               cudaStream_t st);

}  // namespace hba
