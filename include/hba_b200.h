/*
 * hba_b200.h -- C ABI of the B200 (sm_100a) implementation of the
 * Hierarchical Block Attention (HBA) hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t,
 * enqueues its kernels on that stream, and returns an hba_b200_status; none
 * aborts the process and none allocates device memory (scratch space comes
 * from the caller's `workspace`).  All tensors are dense, row-major, in the
 * layouts documented per argument (the reference's token-major
 * [B, n, H, dh] for q/k/v/out and [B, Hkv, nb, m, dh] for block summaries).
 *
 * Reference = nealxpatel/hierarchical-block-attention, file paths relative to
 * that project.  Each entry point names the reference interface it replaces.
 */
#ifndef HBA_B200_H
#define HBA_B200_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum hba_b200_status {
  HBA_B200_OK = 0,
  HBA_B200_ERR_INVALID_ARGUMENT = 1,   /* null pointer, non-positive size, inconsistent heads */
  HBA_B200_ERR_NOT_BLOCK_MULTIPLE = 2, /* n % block != 0 (reference: assert n % Bk == 0) */
  HBA_B200_ERR_WORKSPACE = 3,          /* workspace smaller than the *_workspace_size query */
  HBA_B200_ERR_UNSUPPORTED = 4,        /* knob outside the compiled kernels' range */
  HBA_B200_ERR_CUDA = 5,               /* a kernel launch or stream operation failed */
  HBA_B200_ERR_DEVICE_TIMEOUT = 6      /* a bounded device-side wait expired */
} hba_b200_status;

/* Architecture knobs, mirroring HBAConfig (src/hba/config.py:105-184). */
typedef struct hba_b200_config {
  int32_t n_heads;   /* Hq, query heads                                   */
  int32_t n_kv;      /* Hkv, KV heads (GQA); G = Hq / Hkv <= 16           */
  int32_t head_dim;  /* dh: 64 or 128                                     */
  int32_t block;     /* Bk, routing block size: 16, 32 or 64              */
  int32_t window;    /* W, RoPE local window (>= 0)                       */
  int32_t sinks;     /* S, NoPE sink tokens (0 <= S <= Bk)                */
  int32_t k_blocks;  /* routed top-k budget (1..32)                       */
  int32_t slots;     /* m, summary slots per block (1..8)                 */
  int32_t fanout;    /* F, children per super-summary (hier)              */
  int32_t beam;      /* super-summaries kept by the beam (hier)           */
  int32_t hier;      /* 0: flat scan; 1: two-level beam descent           */
  int32_t qknorm;    /* 1: RMS-normalise q and k with per-head gains      */
  float eps;         /* QKNorm clamp on mean(x^2) (reference: 1e-6)       */
} hba_b200_config;

/* Human-readable name of a status code (static storage). */
const char* hba_b200_status_string(int status);

/* Library version, major*10000 + minor*100 + patch. */
int hba_b200_version(void);

/*
 * Per-head RMS normalisation with a scalar gain per head:
 *   y = bf16( x / sqrt(max(mean(x^2), eps)) * gain[h] ), math in fp32.
 * x, y: [rows, heads, head_dim] bf16 (may alias); gain: [heads] fp32.
 * Replaces _HeadRMSNorm.forward (src/hba/attention.py:88-94), i.e. the
 * QKNorm applied by _content_qk (src/hba/attention.py:173-198).
 */
int hba_b200_qknorm(const void* x, void* y, const float* gain, int64_t rows, int32_t heads,
                    int32_t head_dim, float eps, cudaStream_t stream);

/*
 * Learned slot summaries of complete key blocks [blk_begin, blk_end):
 *   att = softmax_t(probes[g] . k_t * dh^-1/2); S = (att @ k) @ proj[g]
 * k_cache:   [batch, n_cap, Hkv, dh] bf16, QKNorm'd NoPE keys
 * probes:    [Hkv, m, dh] fp32;  proj: [Hkv, dh, dh] fp32
 * summaries: [batch, Hkv, nb_cap, m, dh] bf16, nb_cap = n_cap / block
 * Replaces SlotSummarizer.summarize (src/hba/summarizer.py:34-42).
 */
int hba_b200_summarize(const hba_b200_config* cfg, int32_t batch, int32_t n_cap, const void* k_cache,
                       const float* probes, const float* proj, void* summaries, int32_t blk_begin,
                       int32_t blk_end, cudaStream_t stream);

/*
 * Super-summaries over the first nb blocks: per-slot mean of `fanout`
 * children, the last group averaged over the children present.  Writes
 * supers [s_begin, s_end) of [batch, Hkv, ns_cap, m, dh] bf16,
 * ns_cap = ceil(nb_cap / fanout).
 * Replaces build_super (src/hba/attention.py:202-214).
 */
int hba_b200_build_supers(const hba_b200_config* cfg, int32_t batch, int32_t nb_cap, int32_t nb,
                          const void* summaries, void* supers, int32_t s_begin, int32_t s_end,
                          cudaStream_t stream);

/*
 * Append `t` new tokens per sequence at positions pos[b] .. pos[b]+t-1 of a
 * KV/summary cache: k is QKNorm'd (k_gain) and stored, its RoPE'd copy (at
 * the token's position, cos/sin [n_cap, dh] fp32) stored in k_rope_cache, v
 * stored, and the summaries of blocks completed by the append (plus the
 * super-summaries that contain them, when `supers` is not NULL) are rebuilt.
 * k_new, v_new: [batch, t, Hkv, dh] bf16 raw; pos: [batch] int32 device;
 * k_cache, k_rope_cache, v_cache: the KV cache, bf16, chunk-tiled per
 *   (sequence, kv head): [batch, Hkv, n_cap/64, dh/64, 64, 64] -- per 64-token
 *   block and 64-dim group the 8 KB image a 128-byte-swizzled TMA box leaves
 *   in shared memory: element (token t, dim d) at ((t/64)*(dh/64) + d/64)*4096
 *   + (t%64)*64 + (((d%64)/8) ^ (t%8))*8 + d%8 of the head's run, so a decode
 *   moves a block with one 1-D bulk copy.  n_cap is a multiple of 64.
 * Has no single counterpart in the reference, which recomputes QKNorm and
 * every summary on each call (src/hba/attention.py:631,659); it produces the
 * same cache contents incrementally.
 */
int hba_b200_append_kv(const hba_b200_config* cfg, int32_t batch, int32_t n_cap, int32_t t,
                       const int32_t* pos, const void* k_new, const void* v_new, const float* k_gain,
                       const float* cos, const float* sin, const float* probes, const float* proj,
                       void* k_cache, void* k_rope_cache, void* v_cache, void* summaries, void* supers,
                       cudaStream_t stream);

/* Bytes of scratch needed by hba_b200_decode for this batch and cache capacity
 * (0 when the configuration is rejected). */
size_t hba_b200_decode_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n_cap);

/*
 * One decode step: the newest token of every sequence (position
 * seq_lens[b]-1) attends over its cached context with one union softmax over
 * sinks (NoPE), the RoPE window and the top-k routed blocks (NoPE), routed by
 * QKNorm'd grouped-query scores against the cached block summaries (flat
 * scan, or the two-level beam over `supers` when cfg->hier).
 *   seq_lens:  [batch] int32 device, 1 <= seq_lens[b] <= n_cap
 *   scales:    [batch] fp32 device, union logit scale (content scale x tau(n))
 *   q:         [batch, Hq, dh] bf16 raw query;  q_gain: [Hq], k_gain: [Hkv] fp32
 *              (the QKNorm gains; k_gain bounds the logits of the tensor-core path)
 *   k_cache, v_cache: the chunk-tiled KV cache of hba_b200_append_kv (keys
 *              QKNorm'd, NoPE); n_cap a multiple of 64
 *   k_rope_cache: the same keys RoPE'd at their positions, same layout
 *              (hba_b200_append_kv writes both); the window reads it
 *   summaries: [batch, Hkv, n_cap/block, m, dh] bf16
 *   supers:    [batch, Hkv, ceil(n_cap/block/F), m, dh] bf16 (hier only)
 *   cos, sin:  [n_cap, dh] fp32 RoPE tables (rope_tables layout)
 *   out:       [batch, Hq, dh] bf16;  lse: [batch, Hq] fp32 natural-log or NULL
 *   sel_idx:   [batch, Hkv, k_blocks] int32 (-1: no pick) or NULL
 *   sel_score: [batch, Hkv, k_blocks] fp32 or NULL
 * The first 4 bytes of the workspace hold a sticky device status: the caller
 * zeroes them once (and whenever it clears an error); a decode whose bounded
 * device wait times out sets 1 and later calls leave it set.  No per-call
 * reset keeps a decode step at one kernel launch.  Read it with
 * hba_b200_device_status(workspace, ...) after the step: this call returns
 * when the work is enqueued, before the device could report.
 * Replaces the per-query body of hba_attention_eval
 * (src/hba/attention.py:663-711) at cs = n-1, flat (:694-698) or
 * hierarchical (:690-693, hier_select :217-246).
 */
int hba_b200_decode(const hba_b200_config* cfg, int32_t batch, int32_t n_cap, const int32_t* seq_lens,
                    const float* scales, const void* q, const float* q_gain, const float* k_gain,
                    const void* k_cache,
                    const void* k_rope_cache, const void* v_cache, const void* summaries, const void* supers,
                    const float* cos, const float* sin, void* out, float* lse, int32_t* sel_idx,
                    float* sel_score, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * hba_b200_decode without a workspace argument, for callers that cannot
 * allocate device memory when they decode (an engine whose arena owns all of
 * HBM, a plugin host without an allocator, code where cudaMalloc is not
 * allowed).  It allocates nothing: its scratch is a fixed 8 MiB __device__
 * array inside the library, held on every GPU that loads the library until
 * the process exits.  Requests whose hba_b200_decode_workspace_size exceeds
 * 8 MiB return HBA_B200_ERR_WORKSPACE (use hba_b200_decode instead).  The
 * array's device address is looked up on the first call made on each device,
 * so make that call before any stream capture.  All calls on a device share
 * the array: calls whose kernels may overlap on the GPU race on it.  The
 * request size counts the split path's partials whatever path runs, so the
 * limit is about batch x context <= 8 MiB of hba_b200_decode_workspace_size.
 * No counterpart in the reference.
 */
int hba_b200_decode_noalloc(const hba_b200_config* cfg, int32_t batch, int32_t n_cap, const int32_t* seq_lens,
                            const float* scales, const void* q, const float* q_gain, const float* k_gain,
                            const void* k_cache,
                            const void* k_rope_cache, const void* v_cache, const void* summaries,
                            const void* supers, const float* cos, const float* sin, void* out, float* lse,
                            int32_t* sel_idx, float* sel_score, cudaStream_t stream);

/*
 * The sticky device status of hba_b200_decode_noalloc on the current device
 * (the word sits in the library's scratch array, out of the caller's reach):
 * waits for `stream`, reads it, zeroes it when `clear` is non-zero, and
 * returns what hba_b200_device_status returns for it.  The word starts at
 * zero when the library loads.  No counterpart in the reference.
 */
int hba_b200_decode_noalloc_status(int32_t clear, cudaStream_t stream);

/* Bytes of scratch needed by hba_b200_prefill (0 when rejected). */
size_t hba_b200_prefill_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n);

/*
 * Full HBA attention forward over n tokens (n % block == 0): QKNorm, block
 * summaries, (super-summaries), per-query top-k selection and the fused union
 * softmax with one online log-sum-exp.
 *   q: [batch, n, Hq, dh], k, v: [batch, n, Hkv, dh] bf16 raw projections
 *   scale: union logit scale (content_scale x tau(n), or dh^-1/2 without QKNorm)
 *   cos, sin: [n, dh] fp32; q_gain: [Hq], k_gain: [Hkv] fp32
 *   probes: [Hkv, m, dh], proj: [Hkv, dh, dh] fp32 (SlotSummarizer weights)
 *   out: [batch, n, Hq, dh] bf16; lse: [batch, Hq, n] fp32 or NULL
 *   sel_idx / sel_score: [batch, Hkv, n, k_blocks] or NULL
 * The flat selection runs as a tcgen05 GEMM of 128 routing queries against
 * 128 summary rows per stage.  With QKNorm, block 64 and G >= 4 the union
 * softmax runs on the tcgen05 tensor cores (two 128-row tiles of 128/G
 * queries x G heads per CTA sharing one K/V stream, the routed blocks of
 * their queries computed once and masked per row); other configurations use
 * the per-query gather kernel.  The first 4 bytes of the
 * workspace receive a device status (zeroed by the call; 1 = a bounded device
 * wait timed out), read by hba_b200_device_status(workspace, ...).
 * Replaces hba_attention_eval (src/hba/attention.py:610-713, hier or flat)
 * and the forward of hba_attention_fused / hba_attention_dense
 * (src/hba/attention.py:552-607, :306-389), which compute the same union.
 */
int hba_b200_prefill(const hba_b200_config* cfg, int32_t batch, int32_t n, float scale, const void* q,
                     const void* k, const void* v, const float* cos, const float* sin, const float* q_gain,
                     const float* k_gain, const float* probes, const float* proj, void* out, float* lse,
                     int32_t* sel_idx, float* sel_score, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream);

/*
 * The forward for a range of query positions [q_lo, q_lo + n_q) of
 * sequences whose keys and values [0, n) are given: the rows q_lo .. of
 * hba_b200_prefill over the n tokens (same summaries, same selection, same
 * union; `scale` is the caller's -- content scale x tau of the whole
 * sequence's length, as every row of the reference's forward uses).  For a
 * prefill split by token range over ranks: rank r passes its queries and
 * the keys / values of tokens [0, its last position].
 *   q: [batch, n_q, Hq, dh]; k, v: [batch, n, Hkv, dh]; cos, sin: [n, dh]
 *   out: [batch, n_q, Hq, dh]; lse: [batch, Hq, n_q]; sel: [batch, Hkv, n_q, k]
 * Runs on the tensor-core selection and union (flat selection, QKNorm, block
 * 64, G >= 4); HBA_B200_ERR_UNSUPPORTED otherwise.  No counterpart in the
 * reference, which runs one device.
 */
size_t hba_b200_prefill_range_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n, int32_t n_q);
int hba_b200_prefill_range(const hba_b200_config* cfg, int32_t batch, int32_t n, int32_t q_lo, int32_t n_q,
                           float scale, const void* q, const void* k, const void* v, const float* cos,
                           const float* sin, const float* q_gain, const float* k_gain, const float* probes,
                           const float* proj, void* out, float* lse, int32_t* sel_idx, float* sel_score,
                           void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * The summarizer's auxiliary-loss teacher (reference: _teacher_chunk /
 * _aux_kl_chunked, src/hba/attention.py:476-529): for every query position i
 * and kv head, the mean over the group's query heads of each candidate
 * block's share of the softmax over all candidate keys (NoPE logits scale *
 * QKNorm(q) . QKNorm(k), candidates the blocks 1 .. wholly before the
 * window).  pstar: [batch, Hkv, n, n / block] fp32, written whole (0 for
 * non-candidate blocks and for queries with no candidate, where the
 * reference's rows are NaN and its loss skips them).  scale: the union's
 * (content scale x tau(n) under QKNorm, dh**-0.5 without).  cos / sin feed
 * the shared key pre-pass.  Block 64, dh 64 / 128, flat configs;
 * HBA_B200_ERR_UNSUPPORTED otherwise.  O(n^2): training only.  The
 * workspace includes up to 1 GiB for the one-pass mode's block masses
 * (QKNorm with bounded logits); larger batches x lengths run in query
 * slices of that size.
 */
size_t hba_b200_aux_teacher_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n);
int hba_b200_aux_teacher(const hba_b200_config* cfg, int32_t batch, int32_t n, float scale, const void* q,
                         const void* k, const float* cos, const float* sin, const float* q_gain, const float* k_gain,
                         float* pstar, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Backward of the prefill union softmax: the gradients that autograd takes
 * through the reference's training attention, hba_attention_fused
 * (src/hba/attention.py:552-607; equal to hba_attention_dense, :306-389),
 * for the forward's block selection (a top-k: no gradient through it).
 *   q, k, v, cos, sin, gains, scale: the forward's arguments (hba_b200_prefill)
 *   out: [batch, n, Hq, dh] bf16 and lse: [batch, Hq, n] fp32, the forward's outputs
 *   sel_idx: [batch, Hkv, n, k] int32, the forward's picks (-1 = none)
 *   dout: [batch, n, Hq, dh] bf16, the gradient of out
 * Writes dq [batch, n, Hq, dh], dk, dv [batch, n, Hkv, dh] (bf16) and, with
 * QKNorm, dq_gain [Hq] and dk_gain [Hkv] (fp32; overwritten, not added to).
 * Flat selection, block 64, dh 64 / 128, G = Hq / Hkv in 4 .. 16, and a
 * query tile's routed union (1 + (128 / G) * k blocks) within 520 -- k <= 16
 * at G = 4; HBA_B200_ERR_UNSUPPORTED otherwise.  Replaces the flex-attention backward
 * (torch autograd) of the reference's training path.
 */
size_t hba_b200_prefill_backward_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n);
int hba_b200_prefill_backward(const hba_b200_config* cfg, int32_t batch, int32_t n, float scale, const void* q,
                              const void* k, const void* v, const float* cos, const float* sin, const float* q_gain,
                              const float* k_gain, const void* out, const float* lse, const int32_t* sel_idx,
                              const void* dout, void* dq, void* dk, void* dv, float* dq_gain, float* dk_gain,
                              void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Device status readout (no counterpart in the reference, whose torch calls
 * are synchronous).  The kernels report a failed bounded device-side wait by
 * writing 1 into a status word instead of hanging or trapping: the first 4
 * bytes of the decode / prefill workspace, or a shard call's dev_status.
 * This waits for `stream`, reads the word, zeroes it when `clear` is
 * non-zero, and returns HBA_B200_OK (word 0), HBA_B200_ERR_DEVICE_TIMEOUT
 * (word 1) or HBA_B200_ERR_CUDA (any other value, or a failed copy).
 */
int hba_b200_device_status(void* status_word, int32_t clear, cudaStream_t stream);

/*
 * Profiling hook (no counterpart in the reference).  With count > 0, each
 * later hba_b200_decode / hba_b200_prefill call records events[0] before its
 * first kernel and events[i] after its i-th kernel, up to `count` events (at
 * most 16), on the call's stream; hba_b200_profile_events_recorded() returns
 * how many the last call recorded.  count == 0 turns it off.  Process-global,
 * not thread-safe; leave it off in production and during graph capture.
 */
int hba_b200_set_profile_events(void* const* events, int32_t count);
int hba_b200_profile_events_recorded(void);

/*
 * Debug hook (no counterpart in the reference): with a non-NULL device
 * buffer, later tcgen05 decode kernels write 16 uint64 global-timer stamps
 * per CTA to buffer[blockIdx * 16 + i], for CTAs with blockIdx * 128 < bytes:
 * 0 kernel start, 1 after the query prologue, 2 after selection, 3 after the
 * union softmax, 4 end, 5-7 selection sub-phases, 8 / 9 / 10 the MMA warp
 * sees the first window tile / the last window-or-sink tile / the first
 * routed tile land, 11 last PV issued, 12 the producer sees the picks;
 * fused shard decode: 14 / 15 the first / second list exchange complete,
 * 13 the partial exchange complete.  The
 * prefill union kernel writes stamps for the last pair of query tiles of each
 * (sequence, kv head) row r < bytes / 128 at buffer[r * 16 + i]: 0 start,
 * 1 chunk list built, 2 query tiles ready, 14 the first tile's softmax done,
 * 15 end.  NULL turns it off.
 */
int hba_b200_set_debug_trace(void* device_buffer, int64_t bytes);

/*
 * KV-range sharded decode (no counterpart in the reference, which runs on one
 * device; the result is the decode of src/hba/attention.py:663-711 at
 * cs = n-1 over the whole context).  Rank r of P holds global tokens
 * [tok_lo, tok_lo + n_cap_local) of every sequence -- K/V/RoPE'd-K caches of
 * that range in local rows 0.., the summaries (and supers) of its blocks --
 * with bounds on block (hier: super) multiples.  seq_lens are the global
 * context lengths.  One step, with collectives done by the caller:
 *   flat: shard_select(level 0) -> all-gather the [B*Hkv, K] lists ->
 *         shard_attend(every shard's lists) -> all-gather the (m2, l, O)
 *         partials -> shard_finish.
 *   hier: shard_select(level 1, local top-beam supers) -> all-gather ->
 *         shard_select(level 2, in = every shard's beam lists, children
 *         this shard owns) -> all-gather -> shard_attend -> ... as flat.
 * Every rank computes the same global top-k (score desc, block asc) from
 * exact per-shard scores, so the picks equal the one-device picks.
 *
 * shard_select: out_idx/out_score [B*Hkv, K] (level 1: [B*Hkv, beam]) global
 *   block (super) ids, -1 = none; in lists [B*Hkv, n_in_lists, beam].
 * shard_attend: in [B*Hkv, n_in] candidate picks; the union over the owned
 *   tokens as an unnormalised partial: part_o [B, Hq, dh], part_l [B, Hq] and
 *   part_m2 [B, Hq] fp32, the softmax reference maximum (log2 units) the
 *   partial is scaled by -- the QKNorm logit bound while it is small, else a
 *   running maximum of the owned logits, so it differs between shards;
 *   sel_idx/sel_score (optional) get the global picks; dev_status: one device
 *   int, zeroed by the call, 1 = a bounded wait timed out.
 *   Needs the tensor-core decode path (QKNorm, block 64, head dim 64/128).
 * shard_finish: the max-rescaled merge of every rank's partial.  parts
 *   [world][B*Hq*(dh+2)] fp32, rank-major (an all-gather of each rank's
 *   contiguous [m2 | l | O] = [B*Hq | B*Hq | B*Hq*dh]); out [B, Hq, dh] bf16
 *   = sum_r w_r O_r / sum_r w_r l_r with w_r = 2^(m2_r - max m2), lse
 *   (optional) natural log.
 */
int hba_b200_decode_shard_select(const hba_b200_config* cfg, int32_t batch, int32_t n_cap_local, int32_t tok_lo,
                                 int32_t level, const int32_t* seq_lens, const float* scales, const void* q,
                                 const float* q_gain, const void* summaries, const void* supers,
                                 const int32_t* in_idx, const float* in_score, int32_t n_in_lists, int32_t* out_idx,
                                 float* out_score, cudaStream_t stream);
int hba_b200_decode_shard_attend(const hba_b200_config* cfg, int32_t batch, int32_t n_cap_local, int32_t tok_lo,
                                 const int32_t* seq_lens, const float* scales, const void* q, const float* q_gain,
                                 const float* k_gain, const void* k_cache, const void* k_rope_cache,
                                 const void* v_cache, const float* cos, const float* sin, const int32_t* in_idx,
                                 const float* in_score, int32_t n_in, float* part_o, float* part_l, float* part_m2,
                                 int32_t* sel_idx, float* sel_score, int32_t* dev_status, cudaStream_t stream);
int hba_b200_decode_shard_finish(const hba_b200_config* cfg, int32_t batch, int32_t world, const float* parts,
                                 void* out, float* lse, cudaStream_t stream);

/*
 * Fused KV-range sharded decode (no counterpart in the reference; same
 * result as the three calls above): ONE launch per step on each rank does
 * the owned selection, the list exchanges and the union over the owned
 * tokens, exchanging with the same (sequence, kv head) CTA of every other
 * rank over NVLink through the ranks' exchange buffers -- each rank writes
 * its lists and its (O, l) partial into slot [rank] of every buffer as
 * 64-bit words tagged with the step's epoch, and readers wait for the tag
 * (no fence, no flag) -- so there is no collective library call.
 * Every rank returns the full out / lse / picks.
 *   xbuf_bytes   size of one rank's exchange buffer (-1 on bad arguments).
 *   peer_alloc   cudaMalloc + zero a buffer on the current device and write
 *                its 64-byte CUDA IPC handle to ipc_handle.
 *   peer_open    map another process's buffer from its handle (same node,
 *                peer access enabled); peer_close unmaps, peer_free frees.
 *   decode_shard_fused  xbufs[r] = rank r's buffer as mapped in this process
 *                (xbufs[rank] = its own); epoch = a device int32, zero at
 *                start, bumped by the call on `stream` (every rank must make
 *                the same calls); dev_status is sticky (zero it once; 1 = a
 *                wait gave up, e.g. a rank that never arrived).  Bounds fall
 *                on block (hier: block * fanout) multiples; world <= 8 and
 *                world * n_cap_local / block < 65535 (16-bit block ids).
 * Every wait is bounded in time; a rank that never arrives turns into a
 * status, not a hang.
 */
int64_t hba_b200_shard_xbuf_bytes(const hba_b200_config* cfg, int32_t batch, int32_t world);

/*
 * Zero-copy host I/O (no counterpart in the reference): pinned host memory
 * mapped into the device address space (cudaHostAlloc mapped; dev_ptr from
 * cudaHostGetDevicePointer, so an unmapped pointer is a host-side error).
 * hba_b200_decode / _decode_noalloc accept dev_ptr for q, out and lse: the
 * decode kernel then reads the query from and writes the result to host
 * memory directly, with no copy before or after the launch -- the serving
 * path for a decode step whose I/O is a few hundred KB.
 */
int hba_b200_host_alloc(int64_t bytes, void** host_ptr, void** dev_ptr);
int hba_b200_host_free(void* host_ptr);
int hba_b200_peer_alloc(int64_t bytes, void** dptr, void* ipc_handle);
int hba_b200_peer_open(const void* ipc_handle, void** dptr);
int hba_b200_peer_close(void* dptr);
int hba_b200_peer_free(void* dptr);
int hba_b200_decode_shard_fused(const hba_b200_config* cfg, int32_t batch, int32_t n_cap_local, int32_t tok_lo,
                                int32_t world, int32_t rank, void* const* xbufs, int32_t* epoch,
                                const int32_t* seq_lens, const float* scales, const void* q, const float* q_gain,
                                const float* k_gain, const void* summaries, const void* supers, const void* k_cache,
                                const void* k_rope_cache, const void* v_cache, const float* cos, const float* sin,
                                void* out, float* lse, int32_t* sel_idx, float* sel_score, int32_t* dev_status,
                                cudaStream_t stream);

/*
 * Introspection (no counterpart in the reference): the kernels the last
 * hba_b200_decode / _decode_noalloc / _prefill call of this process launched,
 * in launch order joined by '+', as a static string (e.g. "decode_tc_kernel";
 * "" before the first call).  The profile marks fall between them.
 */
const char* hba_b200_last_kernels(void);

#ifdef __cplusplus
}
#endif

#endif /* HBA_B200_H */
