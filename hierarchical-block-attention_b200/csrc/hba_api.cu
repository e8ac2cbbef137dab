// C ABI of the HBA B200 library: argument validation, workspace layout and
// kernel orchestration.  No entry point allocates device memory.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "hba_b200.h"
#include "hba_internal.h"

using hba::Geom;

namespace {

constexpr size_t kAlign = 256;
constexpr int kMaxCandPerCta = 2048;  // must match hba_select.cu

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Optional event marks at kernel boundaries (hba_b200_set_profile_events).
struct ProfileHook {
  cudaEvent_t ev[16];
  int count = 0;
  int next = 0;
};
ProfileHook g_prof;
unsigned long long* g_trace = nullptr;  // hba_b200_set_debug_trace
long long g_trace_ctas = 0;
const char* g_last_kernels = "";  // hba_b200_last_kernels

void prof_begin(cudaStream_t st) {
  g_prof.next = 0;
  if (g_prof.count > 0) cudaEventRecord(g_prof.ev[g_prof.next++], st);
}
void prof_mark(cudaStream_t st) {
  if (g_prof.count > 0 && g_prof.next < g_prof.count) cudaEventRecord(g_prof.ev[g_prof.next++], st);
}

bool config_ok(const hba_b200_config* c, int* status) {
  if (c == nullptr) {
    *status = HBA_B200_ERR_INVALID_ARGUMENT;
    return false;
  }
  if (c->n_heads <= 0 || c->n_kv <= 0 || c->n_heads % c->n_kv != 0 || c->slots <= 0 || c->k_blocks <= 0 ||
      c->block <= 0 || c->window < 0 || c->sinks < 0 || !(c->eps >= 0.f)) {
    *status = HBA_B200_ERR_INVALID_ARGUMENT;
    return false;
  }
  const int G = c->n_heads / c->n_kv;
  if ((c->head_dim != 64 && c->head_dim != 128) || G > 16 || (c->block != 16 && c->block != 32 && c->block != 64) ||
      c->sinks > c->block || c->k_blocks > 32 || c->slots > 8) {
    *status = HBA_B200_ERR_UNSUPPORTED;
    return false;
  }
  if (c->hier) {
    if (c->fanout <= 0 || c->beam <= 0) {
      *status = HBA_B200_ERR_INVALID_ARGUMENT;
      return false;
    }
    if (c->beam > 32) {
      *status = HBA_B200_ERR_UNSUPPORTED;
      return false;
    }
  }
  return true;
}

Geom make_geom(const hba_b200_config* c, int B, int nq, int n_cap) {
  Geom g{};
  g.B = B;
  g.Hq = c->n_heads;
  g.Hkv = c->n_kv;
  g.G = c->n_heads / c->n_kv;
  g.m = c->slots;
  g.Bk = c->block;
  g.W = c->window;
  g.S = c->sinks;
  g.K = c->k_blocks;
  g.F = c->hier ? c->fanout : 1;
  g.beam = c->hier ? c->beam : 1;
  g.hier = c->hier ? 1 : 0;
  g.qknorm = c->qknorm ? 1 : 0;
  g.eps = c->eps;
  g.nq = nq;
  g.n_cap = n_cap;
  g.nb_cap = n_cap / c->block;
  g.ns_cap = c->hier ? (g.nb_cap + c->fanout - 1) / c->fanout : 0;
  return g;
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return HBA_B200_OK;
  fprintf(stderr, "hba_b200: CUDA error: %s\n", cudaGetErrorString(e));
  return HBA_B200_ERR_CUDA;
}

// Split plan shared by the decode and prefill paths.
struct Plan {
  int sel_splits;    // flat lists, or super lists (hier)
  int sel_list_k;    // K, or beam (hier)
  int child_splits;  // hier only
  int attn_splits;   // prefill: key-range splits per query (1)
  int ncw, ncr, nchunk, max_seg;  // decode attention chunk slots and partial segments
};

constexpr int kMinChunksPerCta = 4;

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

Plan make_plan(const hba_b200_config* c, int nb_cap, int bh, bool decode) {
  Plan p{};
  const int max_cand = nb_cap;  // blocks 1..nb-2 at most
  const int per_cta = decode ? 128 : kMaxCandPerCta;
  if (c->hier) {
    const int max_sup = (nb_cap + c->fanout - 1) / c->fanout;
    p.sel_splits = std::max(1, std::max(ceil_div(max_sup, decode ? 64 : kMaxCandPerCta),
                                        ceil_div(max_sup, kMaxCandPerCta)));
    p.sel_list_k = c->beam;
    const int max_child = c->beam * c->fanout;
    p.child_splits = std::max(1, std::max(ceil_div(max_child, decode ? 64 : kMaxCandPerCta),
                                          ceil_div(max_child, kMaxCandPerCta)));
  } else {
    p.sel_splits = std::max(1, std::max(ceil_div(max_cand, per_cta), ceil_div(max_cand, kMaxCandPerCta)));
    p.sel_list_k = c->k_blocks;
    p.child_splits = 0;
  }
  p.attn_splits = 1;
  p.ncw = ceil_div(c->window, 64);
  p.ncr = ceil_div((long long)c->k_blocks * c->block, 64);
  p.nchunk = p.ncw + 1 + p.ncr;
  // decode attention: every CTA owns >= kMinChunksPerCta chunk slots, so a
  // (sequence, kv head) is split into at most nchunk / kMinChunksPerCta + 2 segments
  p.max_seg = p.nchunk / kMinChunksPerCta + 2;
  (void)bh;
  (void)decode;
  return p;
}

struct Lists {
  float* score;
  int32_t* idx;
};

// Carves [score f32 | idx i32] for `entries` list entries from the workspace.
Lists carve_lists(unsigned char*& ws, size_t entries) {
  Lists l;
  l.score = reinterpret_cast<float*>(ws);
  ws += align_up(entries * sizeof(float));
  l.idx = reinterpret_cast<int32_t*>(ws);
  ws += align_up(entries * sizeof(int32_t));
  return l;
}

size_t lists_bytes(size_t entries) { return align_up(entries * sizeof(float)) + align_up(entries * sizeof(int32_t)); }

size_t selection_bytes(const hba_b200_config* c, const Plan& p, size_t queries) {
  size_t b = lists_bytes(queries * p.sel_splits * p.sel_list_k);
  if (c->hier) b += lists_bytes(queries * p.child_splits * c->k_blocks);
  return b;
}

// Runs selection (flat, or super then child) for nq queries per sequence and
// returns the final lists through `fin`.  `counters` (decode) are zeroed by
// the last selection kernel; with `pdl` the child kernel is launched as a
// programmatic dependent of the super kernel.
int run_select(const hba_b200_config* c, const Geom& geo, const hba::QueryPos& qp, const Plan& plan,
               const __nv_bfloat16* q, const float* q_gain, const __nv_bfloat16* summ,
               const __nv_bfloat16* supers, unsigned char*& ws, int32_t* counters, Lists& fin, int& fin_lists,
               int& fin_k, cudaStream_t st) {
  const int dh = c->head_dim;
  const size_t queries = (size_t)geo.B * geo.Hkv * geo.nq;
  Lists l1 = carve_lists(ws, queries * plan.sel_splits * plan.sel_list_k);
  hba::SelParams sp{};
  sp.geo = geo;
  sp.qp = qp;
  sp.q = q;
  sp.q_gain = q_gain;
  sp.summ = summ;
  sp.supers = supers;
  sp.mode = c->hier ? hba::kSelSuper : hba::kSelFlat;
  sp.splits = plan.sel_splits;
  sp.list_k = plan.sel_list_k;
  sp.out_score = l1.score;
  sp.out_idx = l1.idx;
  sp.counters = c->hier ? nullptr : counters;
  sp.pdl = 0;
  sp.own_blo = 0;
  sp.own_bhi = INT_MAX;
  sp.n_limit = geo.n_cap;
  cudaError_t e = hba::launch_select(sp, dh, st);
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(st);
  fin = l1;
  fin_lists = plan.sel_splits;
  fin_k = plan.sel_list_k;
  if (c->hier) {
    Lists l2 = carve_lists(ws, queries * plan.child_splits * c->k_blocks);
    sp.mode = hba::kSelChild;
    sp.in_score = l1.score;
    sp.in_idx = l1.idx;
    sp.in_lists = plan.sel_splits;
    sp.splits = plan.child_splits;
    sp.list_k = c->k_blocks;
    sp.out_score = l2.score;
    sp.out_idx = l2.idx;
    sp.counters = counters;
    sp.pdl = 1;
    e = hba::launch_select(sp, dh, st);
    if (e != cudaSuccess) return cuda_status(e);
    prof_mark(st);
    fin = l2;
    fin_lists = plan.child_splits;
    fin_k = c->k_blocks;
  }
  return HBA_B200_OK;
}

// Decode path choice.  Fused (one CTA per sequence and kv head, selection and
// attention in one kernel, no scratch) when there are enough (sequence, kv
// head) pairs to fill the GPU and the candidate lists fit its shared-memory
// top-k; otherwise the split path (selection kernels, then the stream-K
// attention kernel with partial merges).  HBA_B200_DECODE_PATH=fused|split
// forces one (tests use it to cover both).
constexpr long long kFusedMinPairs = 96;
constexpr int kFusedMaxItems = 2048;  // must match kTopkMaxItems (hba_topk.cuh)

enum DecodePath { kDecodeSplit = 0, kDecodeFused = 1, kDecodeTc = 2 };

// Large batches: one CTA per (sequence, kv head) -- on tcgen05 when QKNorm
// bounds the logits (kDecodeTc), else the mma.sync fused kernel; small
// batches: the split path.  HBA_B200_DECODE_PATH=tc|fused|split forces one
// (falling back to split when the forced kernel cannot run the configuration).
int decode_path(const hba_b200_config* c, const Geom& geo, size_t bh, const void* k, const void* kr, const void* v,
                const void* summ, const void* supers) {
  const char* force = getenv("HBA_B200_DECODE_PATH");
  bool fits = geo.nb_cap <= kFusedMaxItems;
  if (c->hier) fits = fits && geo.ns_cap <= kFusedMaxItems && (long long)c->beam * c->fanout <= kFusedMaxItems;
  const bool tc_ok = fits && hba::decode_tc_supported(geo, c->head_dim, k, kr, v, summ, supers);
  if (force != nullptr) {
    if (strcmp(force, "split") == 0) return kDecodeSplit;
    if (strcmp(force, "fused") == 0) return fits ? kDecodeFused : kDecodeSplit;
    if (strcmp(force, "tc") == 0) return tc_ok ? kDecodeTc : kDecodeSplit;
  }
  // the tensor-core kernel whenever it runs: at small batches too (one CTA per
  // (sequence, kv head) took ~31 us at cfg1 geometry for B = 1, 4 and 16,
  // the split path over all SMs 48-56 us); else the fused mma.sync kernel for
  // enough (sequence, kv head) pairs, the split path below that
  if (tc_ok) return kDecodeTc;
  if (!fits || (long long)bh < kFusedMinPairs) return kDecodeSplit;
  return kDecodeFused;
}

// decode split path: per-(sequence, kv head) softmax partials and merge counters
size_t decode_state_bytes(const hba_b200_config* c, const Plan& p, size_t bh) {
  const size_t G = (size_t)(c->n_heads / c->n_kv);
  return align_up(bh * p.max_seg * G * (size_t)(c->head_dim + 2) * sizeof(float)) + align_up(bh * sizeof(int32_t));
}

// The tensor-core union runs for this configuration (before the pointer checks).
bool prefill_tc_config(const hba_b200_config* cfg, int32_t batch, int32_t n) {
  const Geom geo = make_geom(cfg, batch, n, n);
  return hba::prefill_tc_supported(geo, cfg->head_dim, n, cfg->qknorm != 0);
}

}  // namespace

extern "C" {

const char* hba_b200_status_string(int s) {
  switch (s) {
    case HBA_B200_OK: return "ok";
    case HBA_B200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case HBA_B200_ERR_NOT_BLOCK_MULTIPLE: return "sequence length is not a multiple of the block size";
    case HBA_B200_ERR_WORKSPACE: return "workspace too small";
    case HBA_B200_ERR_UNSUPPORTED: return "configuration outside the compiled kernels' range";
    case HBA_B200_ERR_CUDA: return "CUDA error";
    case HBA_B200_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

int hba_b200_version(void) { return 200; }

int hba_b200_device_status(void* status_word, int32_t clear, cudaStream_t stream) {
  if (status_word == nullptr) return HBA_B200_ERR_INVALID_ARGUMENT;
  int32_t word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, status_word, sizeof(word), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && clear) {
    e = cudaMemsetAsync(status_word, 0, sizeof(word), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  }
  if (e != cudaSuccess) return cuda_status(e);
  if (word == 0) return HBA_B200_OK;
  return word == 1 ? HBA_B200_ERR_DEVICE_TIMEOUT : HBA_B200_ERR_CUDA;
}

int hba_b200_set_profile_events(void* const* events, int32_t count) {
  if (count < 0 || count > 16 || (count > 0 && events == nullptr)) return HBA_B200_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < count; ++i) g_prof.ev[i] = static_cast<cudaEvent_t>(events[i]);
  g_prof.count = count;
  g_prof.next = 0;
  return HBA_B200_OK;
}

int hba_b200_profile_events_recorded(void) { return g_prof.next; }

const char* hba_b200_last_kernels(void) { return g_last_kernels; }

int hba_b200_set_debug_trace(void* device_buffer, int64_t bytes) {
  if (bytes < 0 || (device_buffer == nullptr && bytes != 0)) return HBA_B200_ERR_INVALID_ARGUMENT;
  g_trace = static_cast<unsigned long long*>(device_buffer);
  g_trace_ctas = device_buffer == nullptr ? 0 : bytes / 128;
  return HBA_B200_OK;
}

int hba_b200_qknorm(const void* x, void* y, const float* gain, int64_t rows, int32_t heads, int32_t head_dim,
                    float eps, cudaStream_t stream) {
  if (x == nullptr || y == nullptr || gain == nullptr || rows < 0 || heads <= 0) return HBA_B200_ERR_INVALID_ARGUMENT;
  if (head_dim != 64 && head_dim != 128) return HBA_B200_ERR_UNSUPPORTED;
  return cuda_status(hba::launch_qknorm(static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), gain,
                                        rows, heads, head_dim, eps, stream));
}

int hba_b200_summarize(const hba_b200_config* cfg, int32_t batch, int32_t n_cap, const void* k_cache,
                       const float* probes, const float* proj, void* summaries, int32_t blk_begin, int32_t blk_end,
                       cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || n_cap <= 0 || k_cache == nullptr || probes == nullptr || proj == nullptr ||
      summaries == nullptr || blk_begin < 0 || blk_end < blk_begin || blk_end > n_cap / cfg->block)
    return HBA_B200_ERR_INVALID_ARGUMENT;
  Geom geo = make_geom(cfg, batch, 1, n_cap);
  return cuda_status(hba::launch_summarize(geo, cfg->head_dim, static_cast<const __nv_bfloat16*>(k_cache), probes,
                                           proj, static_cast<__nv_bfloat16*>(summaries), blk_begin, blk_end,
                                           nullptr, 0, stream));
}

int hba_b200_build_supers(const hba_b200_config* cfg, int32_t batch, int32_t nb_cap, int32_t nb,
                          const void* summaries, void* supers, int32_t s_begin, int32_t s_end, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (!cfg->hier && cfg->fanout <= 0) return HBA_B200_ERR_INVALID_ARGUMENT;
  const int F = cfg->fanout;
  if (batch <= 0 || nb_cap <= 0 || nb < 0 || nb > nb_cap || summaries == nullptr || supers == nullptr ||
      s_begin < 0 || s_end < s_begin || s_end > (nb_cap + F - 1) / F)
    return HBA_B200_ERR_INVALID_ARGUMENT;
  hba_b200_config c2 = *cfg;
  c2.hier = 1;
  if (c2.beam <= 0) c2.beam = 1;
  Geom geo = make_geom(&c2, batch, 1, nb_cap * cfg->block);
  return cuda_status(hba::launch_supers(geo, cfg->head_dim, nb, static_cast<const __nv_bfloat16*>(summaries),
                                        static_cast<__nv_bfloat16*>(supers), s_begin, s_end, nullptr, 0, stream));
}

int hba_b200_append_kv(const hba_b200_config* cfg, int32_t batch, int32_t n_cap, int32_t t, const int32_t* pos,
                       const void* k_new, const void* v_new, const float* k_gain, const float* cos, const float* sin,
                       const float* probes, const float* proj, void* k_cache, void* k_rope_cache, void* v_cache,
                       void* summaries, void* supers, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || n_cap <= 0 || n_cap % 64 != 0 || t <= 0 || pos == nullptr || k_new == nullptr ||
      v_new == nullptr || k_cache == nullptr || k_rope_cache == nullptr || v_cache == nullptr || cos == nullptr ||
      sin == nullptr || (cfg->qknorm && k_gain == nullptr))
    return HBA_B200_ERR_INVALID_ARGUMENT;  // the chunk-tiled cache holds whole 64-token blocks
  if (summaries != nullptr && (probes == nullptr || proj == nullptr)) return HBA_B200_ERR_INVALID_ARGUMENT;
  Geom geo = make_geom(cfg, batch, 1, n_cap);
  const int dh = cfg->head_dim;
  cudaError_t e = hba::launch_append(geo, t, pos, static_cast<const __nv_bfloat16*>(k_new),
                                     static_cast<const __nv_bfloat16*>(v_new), k_gain, cos, sin,
                                     static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(k_rope_cache),
                                     static_cast<__nv_bfloat16*>(v_cache), dh, stream);
  if (e != cudaSuccess) return cuda_status(e);
  if (summaries != nullptr) {
    e = hba::launch_summarize(geo, dh, static_cast<const __nv_bfloat16*>(k_cache), probes, proj,
                              static_cast<__nv_bfloat16*>(summaries), 0, 0, pos, t, stream, /*tiled=*/true);
    if (e != cudaSuccess) return cuda_status(e);
    if (supers != nullptr && cfg->hier) {
      e = hba::launch_supers(geo, dh, 0, static_cast<const __nv_bfloat16*>(summaries),
                             static_cast<__nv_bfloat16*>(supers), 0, 0, pos, t, stream);
      if (e != cudaSuccess) return cuda_status(e);
    }
  }
  return HBA_B200_OK;
}

size_t hba_b200_decode_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n_cap) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st) || batch <= 0 || n_cap <= 0 || n_cap % cfg->block != 0) return 0;
  const Plan plan = make_plan(cfg, n_cap / cfg->block, batch * cfg->n_kv, true);
  const size_t bh = (size_t)batch * cfg->n_kv;
  return kAlign + selection_bytes(cfg, plan, bh) + decode_state_bytes(cfg, plan, bh);  // status word first
}

int hba_b200_decode(const hba_b200_config* cfg, int32_t batch, int32_t n_cap, const int32_t* seq_lens,
                    const float* scales, const void* q, const float* q_gain, const float* k_gain,
                    const void* k_cache,
                    const void* k_rope_cache, const void* v_cache, const void* summaries, const void* supers,
                    const float* cos, const float* sin, void* out, float* lse, int32_t* sel_idx, float* sel_score,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || n_cap <= 0 || seq_lens == nullptr || scales == nullptr || q == nullptr || k_cache == nullptr ||
      k_rope_cache == nullptr || v_cache == nullptr || summaries == nullptr || cos == nullptr || sin == nullptr ||
      out == nullptr || (cfg->qknorm && (q_gain == nullptr || k_gain == nullptr)) ||
      (cfg->hier && supers == nullptr) ||
      ((sel_idx == nullptr) != (sel_score == nullptr)))
    return HBA_B200_ERR_INVALID_ARGUMENT;
  if (n_cap % cfg->block != 0 || n_cap % 64 != 0) return HBA_B200_ERR_NOT_BLOCK_MULTIPLE;  // whole cache tiles
  const size_t need = hba_b200_decode_workspace_size(cfg, batch, n_cap);
  if (workspace == nullptr || workspace_bytes < need) return HBA_B200_ERR_WORKSPACE;
  Geom geo = make_geom(cfg, batch, 1, n_cap);
  const Plan plan = make_plan(cfg, geo.nb_cap, batch * cfg->n_kv, true);
  const size_t bh = (size_t)batch * cfg->n_kv;
  const int G = cfg->n_heads / cfg->n_kv;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  int* dev_status = reinterpret_cast<int*>(ws);  // sticky device status word (bounded waits)
  ws += kAlign;
  // split-path state: partials, then counters
  float* part = reinterpret_cast<float*>(ws);
  ws += align_up(bh * plan.max_seg * G * (size_t)(cfg->head_dim + 2) * sizeof(float));
  int32_t* counters = reinterpret_cast<int32_t*>(ws);
  ws += align_up(bh * sizeof(int32_t));
  hba::QueryPos qp{seq_lens, scales, 0, 0.f};
  prof_begin(stream);
  const int path = decode_path(cfg, geo, bh, k_cache, k_rope_cache, v_cache, summaries, supers);
  if (path != kDecodeSplit) {
    hba::DecodeAttnParams dp{};
    dp.geo = geo;
    dp.trace = g_trace;
    dp.trace_ctas = g_trace_ctas;
    dp.qp = qp;
    dp.q = static_cast<const __nv_bfloat16*>(q);
    dp.q_gain = q_gain;
    dp.k = static_cast<const __nv_bfloat16*>(k_cache);
    dp.kr = static_cast<const __nv_bfloat16*>(k_rope_cache);
    dp.v = static_cast<const __nv_bfloat16*>(v_cache);
    dp.cos = cos;
    dp.sin = sin;
    dp.out = static_cast<__nv_bfloat16*>(out);
    dp.lse = lse;
    dp.sel_idx = sel_idx;
    dp.sel_score = sel_score;
    cudaError_t e;
    if (path == kDecodeTc) {  // the status word is sticky: no per-call reset (one launch per step)
      e = hba::launch_decode_tc(dp, static_cast<const __nv_bfloat16*>(summaries),
                                static_cast<const __nv_bfloat16*>(supers), k_gain, dev_status, cfg->head_dim,
                                stream);
    } else {
      e = hba::launch_decode_fused(dp, static_cast<const __nv_bfloat16*>(summaries),
                                   static_cast<const __nv_bfloat16*>(supers), cfg->head_dim, stream);
    }
    if (e != cudaSuccess) return cuda_status(e);
    g_last_kernels = path == kDecodeTc ? "decode_tc_kernel" : "decode_fused_kernel";
    prof_mark(stream);
    return HBA_B200_OK;
  }
  g_last_kernels = "select_kernel+decode_attend_kernel";
  Lists fin{};
  int fin_lists = 0, fin_k = 0;
  st = run_select(cfg, geo, qp, plan, static_cast<const __nv_bfloat16*>(q), q_gain,
                  static_cast<const __nv_bfloat16*>(summaries), static_cast<const __nv_bfloat16*>(supers), ws,
                  counters, fin, fin_lists, fin_k, stream);
  if (st != HBA_B200_OK) return st;
  hba::DecodeAttnParams dp{};
  dp.geo = geo;
  dp.qp = qp;
  dp.ncw = plan.ncw;
  dp.ncr = plan.ncr;
  dp.nchunk = plan.nchunk;
  dp.in_lists = fin_lists;
  dp.list_k = fin_k;
  dp.max_seg = plan.max_seg;
  dp.q = static_cast<const __nv_bfloat16*>(q);
  dp.q_gain = q_gain;
  dp.k = static_cast<const __nv_bfloat16*>(k_cache);
  dp.kr = static_cast<const __nv_bfloat16*>(k_rope_cache);
  dp.v = static_cast<const __nv_bfloat16*>(v_cache);
  dp.cos = cos;
  dp.sin = sin;
  dp.in_score = fin.score;
  dp.in_idx = fin.idx;
  dp.out = static_cast<__nv_bfloat16*>(out);
  dp.lse = lse;
  dp.sel_idx = sel_idx;
  dp.sel_score = sel_score;
  dp.part = part;
  dp.counters = counters;
  const long long total = (long long)bh * plan.nchunk;
  int grid = hba::decode_attend_grid(cfg->head_dim, (int)std::max<long long>(1, total / kMinChunksPerCta));
  cudaError_t e = hba::launch_decode_attend(dp, cfg->head_dim, grid, stream);
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  return HBA_B200_OK;
}

size_t hba_b200_prefill_range_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n, int32_t n_q) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st) || batch <= 0 || n <= 0 || n % cfg->block != 0 || n_q <= 0 || n_q > n) return 0;
  const int dh = cfg->head_dim;
  const size_t nb = (size_t)n / cfg->block;
  const size_t ns = cfg->hier ? (nb + cfg->fanout - 1) / cfg->fanout : 0;
  const Plan plan = make_plan(cfg, (int)nb, batch * cfg->n_kv, false);
  const size_t queries = (size_t)batch * cfg->n_kv * n_q;
  size_t b = kAlign;                                                      // device status word
  b += 2 * align_up((size_t)batch * n * cfg->n_kv * dh * 2);              // QKNorm'd keys and their RoPE'd copy
  b += 2 * align_up((size_t)batch * n_q * cfg->n_heads * dh * 2);         // the same for the queries
  b += align_up((size_t)batch * cfg->n_kv * nb * cfg->slots * dh * 2);    // summaries
  b += align_up((size_t)batch * cfg->n_kv * ns * cfg->slots * dh * 2);    // supers
  if (prefill_tc_config(cfg, batch, n))                                    // chunk-tiled K, RoPE'd K, V
    b += 3 * align_up((size_t)batch * n * cfg->n_kv * dh * 2);
  b += selection_bytes(cfg, plan, queries);
  return b;
}

size_t hba_b200_prefill_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n) {
  return hba_b200_prefill_range_workspace_size(cfg, batch, n, n);
}

int hba_b200_prefill(const hba_b200_config* cfg, int32_t batch, int32_t n, float scale, const void* q, const void* k,
                     const void* v, const float* cos, const float* sin, const float* q_gain, const float* k_gain,
                     const float* probes, const float* proj, void* out, float* lse, int32_t* sel_idx,
                     float* sel_score, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return hba_b200_prefill_range(cfg, batch, n, 0, n, scale, q, k, v, cos, sin, q_gain, k_gain, probes, proj, out, lse,
                                sel_idx, sel_score, workspace, workspace_bytes, stream);
}

int hba_b200_prefill_range(const hba_b200_config* cfg, int32_t batch, int32_t n, int32_t q_lo, int32_t n_q,
                           float scale, const void* q, const void* k, const void* v, const float* cos,
                           const float* sin, const float* q_gain, const float* k_gain, const float* probes,
                           const float* proj, void* out, float* lse, int32_t* sel_idx, float* sel_score,
                           void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || n <= 0 || q == nullptr || k == nullptr || v == nullptr || cos == nullptr || sin == nullptr ||
      probes == nullptr || proj == nullptr || out == nullptr || (cfg->qknorm && (q_gain == nullptr || k_gain == nullptr)) ||
      ((sel_idx == nullptr) != (sel_score == nullptr)) || !std::isfinite(scale) || q_lo < 0 || n_q <= 0 ||
      q_lo > n - n_q)
    return HBA_B200_ERR_INVALID_ARGUMENT;
  if (n % cfg->block != 0) return HBA_B200_ERR_NOT_BLOCK_MULTIPLE;
  const bool ranged = q_lo != 0 || n_q != n;
  const size_t need = hba_b200_prefill_range_workspace_size(cfg, batch, n, n_q);
  if (workspace == nullptr || workspace_bytes < need) return HBA_B200_ERR_WORKSPACE;
  const int dh = cfg->head_dim;
  const size_t nb = (size_t)n / cfg->block;
  const size_t ns = cfg->hier ? (nb + cfg->fanout - 1) / cfg->fanout : 0;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  int* dev_status = reinterpret_cast<int*>(ws);
  ws += kAlign;
  __nv_bfloat16* kc = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += align_up((size_t)batch * n * cfg->n_kv * dh * 2);
  __nv_bfloat16* kr = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += align_up((size_t)batch * n * cfg->n_kv * dh * 2);
  __nv_bfloat16* qcn = reinterpret_cast<__nv_bfloat16*>(ws);  // queries QKNorm'd
  ws += align_up((size_t)batch * n_q * cfg->n_heads * dh * 2);
  __nv_bfloat16* qrn = reinterpret_cast<__nv_bfloat16*>(ws);  // and RoPE'd at their positions
  ws += align_up((size_t)batch * n_q * cfg->n_heads * dh * 2);
  __nv_bfloat16* summ = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += align_up((size_t)batch * cfg->n_kv * nb * cfg->slots * dh * 2);
  __nv_bfloat16* sup = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += align_up((size_t)batch * cfg->n_kv * ns * cfg->slots * dh * 2);
  __nv_bfloat16 *kc_sw = nullptr, *kr_sw = nullptr, *v_sw = nullptr;  // chunk-tiled copies (tensor-core union)
  if (prefill_tc_config(cfg, batch, n)) {
    const size_t kv_bytes = align_up((size_t)batch * n * cfg->n_kv * dh * 2);
    kc_sw = reinterpret_cast<__nv_bfloat16*>(ws);
    kr_sw = reinterpret_cast<__nv_bfloat16*>(ws + kv_bytes);
    v_sw = reinterpret_cast<__nv_bfloat16*>(ws + 2 * kv_bytes);
    ws += 3 * kv_bytes;
  }

  Geom geo = make_geom(cfg, batch, n_q, n);  // n_q queries per sequence over n keys
  const Plan plan = make_plan(cfg, (int)nb, batch * cfg->n_kv, false);
  // selection: the tcgen05 selection GEMM; HBA_B200_SELECT_PATH=tile forces the
  // query-tiled CUDA-core kernel, =scan the per-query kernel
  const char* force_sel = getenv("HBA_B200_SELECT_PATH");
  const bool no_tc = force_sel != nullptr && (strcmp(force_sel, "scan") == 0 || strcmp(force_sel, "tile") == 0);
  const bool tc_sel = !no_tc && hba::select_tc_supported(geo, dh, summ, qcn, sup);
  const bool tile_sel = !tc_sel && !(force_sel != nullptr && strcmp(force_sel, "scan") == 0) &&
                        hba::select_tile_supported(geo, dh, summ);
  const int n_lists = (tc_sel || tile_sel) ? 1 : (cfg->hier ? plan.child_splits : plan.sel_splits);
  // union: the tensor-core kernel unless HBA_B200_PREFILL_PATH=gather forces the per-query kernel
  const char* force = getenv("HBA_B200_PREFILL_PATH");
  const bool want_tc = !(force != nullptr && strcmp(force, "gather") == 0);
  const bool v_aligned = (reinterpret_cast<uintptr_t>(v) & 15u) == 0;
  const bool use_tc = want_tc && v_aligned && kc_sw != nullptr && n_lists == 1;
  // the per-query selection and gather kernels put the query index in gridDim.y;
  // a query range runs on the tensor-core selection and union only
  if ((n > 65535 || ranged) && !(tc_sel && use_tc)) return HBA_B200_ERR_UNSUPPORTED;

  prof_begin(stream);
  cudaError_t e = cudaMemsetAsync(dev_status, 0, sizeof(int), stream);
  if (e != cudaSuccess) return cuda_status(e);
  e = hba::launch_qknorm_rope(geo, n, static_cast<const __nv_bfloat16*>(k), k_gain, cos, sin, kc, kr, dh, stream,
                              use_tc ? static_cast<const __nv_bfloat16*>(v) : nullptr, use_tc ? kc_sw : nullptr,
                              kr_sw, v_sw);
  if (e == cudaSuccess) {  // the same pre-pass over the query heads (the gain per query head), at positions q_lo..
    Geom gq = geo;
    gq.Hkv = geo.Hq;
    e = hba::launch_qknorm_rope(gq, n_q, static_cast<const __nv_bfloat16*>(q), q_gain, cos, sin, qcn, qrn, dh, stream,
                                nullptr, nullptr, nullptr, nullptr, q_lo);
  }
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  e = hba::launch_summarize(geo, dh, kc, probes, proj, summ, 0, (int)nb, nullptr, 0, stream);
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  if (cfg->hier) {
    e = hba::launch_supers(geo, dh, (int)nb, summ, sup, 0, (int)ns, nullptr, 0, stream);
    if (e != cudaSuccess) return cuda_status(e);
    prof_mark(stream);
  }
  hba::QueryPos qp{nullptr, nullptr, n, scale};  // n keys; local query t sits at position q_lo + t
  Lists fin{};
  int fin_lists = 0, fin_k = 0;
  if (tc_sel || tile_sel) {
    fin = carve_lists(ws, (size_t)batch * cfg->n_kv * n_q * cfg->k_blocks);
    hba::SelParams sp{};
    sp.geo = geo;
    sp.qp = qp;
    sp.q = qcn;  // already QKNorm'd: the kernel skips its own norm (same arithmetic)
    sp.q_normed = 1;
    sp.q_gain = q_gain;
    sp.summ = summ;
    sp.mode = hba::kSelFlat;
    sp.splits = 1;
    sp.list_k = cfg->k_blocks;
    sp.out_score = fin.score;
    sp.out_idx = fin.idx;
    sp.own_blo = 0;
    sp.own_bhi = INT_MAX;
    sp.n_limit = geo.n_cap;
    sp.q_off = q_lo;
    if (cfg->hier) {
      // the super pass (top-beam supers per query), then the child pass over
      // the block summaries, each row keeping the children of its own beam
      Lists beam = carve_lists(ws, (size_t)batch * cfg->n_kv * n_q * cfg->beam);
      sp.supers = sup;
      sp.mode = hba::kSelSuper;
      sp.list_k = cfg->beam;
      sp.out_score = beam.score;
      sp.out_idx = beam.idx;
      e = hba::launch_select_tc(sp, dh, dev_status, stream);
      if (e != cudaSuccess) return cuda_status(e);
      prof_mark(stream);
      sp.mode = hba::kSelChild;
      sp.list_k = cfg->k_blocks;
      sp.in_lists = 1;
      sp.in_score = beam.score;
      sp.in_idx = beam.idx;
      sp.out_score = fin.score;
      sp.out_idx = fin.idx;
    }
    e = tc_sel ? hba::launch_select_tc(sp, dh, dev_status, stream) : hba::launch_select_tile(sp, dh, dev_status, stream);
    if (e != cudaSuccess) return cuda_status(e);
    prof_mark(stream);
    fin_lists = 1;
    fin_k = cfg->k_blocks;
  } else {
    st = run_select(cfg, geo, qp, plan, static_cast<const __nv_bfloat16*>(q), q_gain, summ, sup, ws, nullptr, fin,
                    fin_lists, fin_k, stream);
    if (st != HBA_B200_OK) return st;
  }
  if (use_tc) {
    if (fin_lists != 1) return HBA_B200_ERR_UNSUPPORTED;  // (n_lists predicted it: never taken)
    e = hba::launch_prefill_tc(geo, dh, n, q_lo, scale, qcn, qrn, k_gain, kc_sw, kr_sw, v_sw, fin.idx,
                               fin_lists * fin_k, static_cast<__nv_bfloat16*>(out), lse, dev_status, g_trace,
                               g_trace_ctas, stream);
    if (e != cudaSuccess) return cuda_status(e);
    prof_mark(stream);
    g_last_kernels = cfg->hier ? (tc_sel ? "qknorm_rope_kernel+summarize_kernel+supers_kernel+select_tc_kernel+"
                                           "select_tc_kernel+prefill_tc_kernel"
                                         : "qknorm_rope_kernel+summarize_kernel+supers_kernel+select_kernel+"
                                           "select_kernel+prefill_tc_kernel")
                               : (tc_sel ? "qknorm_rope_kernel+summarize_kernel+select_tc_kernel+prefill_tc_kernel"
                                         : (tile_sel ? "qknorm_rope_kernel+summarize_kernel+select_tile_kernel+"
                                                       "prefill_tc_kernel"
                                                     : "qknorm_rope_kernel+summarize_kernel+select_kernel+"
                                                       "prefill_tc_kernel"));
    if (sel_idx != nullptr) {  // the single-split lists are the final picks, layout [B, Hkv, n_q, K]
      const size_t bytes = (size_t)batch * cfg->n_kv * n_q * cfg->k_blocks * sizeof(int32_t);
      e = cudaMemcpyAsync(sel_idx, fin.idx, bytes, cudaMemcpyDeviceToDevice, stream);
      if (e == cudaSuccess) e = cudaMemcpyAsync(sel_score, fin.score, bytes, cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return cuda_status(e);
    }
    return HBA_B200_OK;
  }
  hba::AttnParams ap{};
  ap.geo = geo;
  ap.qp = qp;
  ap.splits = 1;
  ap.in_lists = fin_lists;
  ap.list_k = fin_k;
  ap.q = static_cast<const __nv_bfloat16*>(q);
  ap.q_gain = q_gain;
  ap.k = kc;
  ap.kr = kr;
  ap.v = static_cast<const __nv_bfloat16*>(v);
  ap.cos = cos;
  ap.sin = sin;
  ap.in_score = fin.score;
  ap.in_idx = fin.idx;
  ap.out = static_cast<__nv_bfloat16*>(out);
  ap.lse = lse;
  ap.sel_idx = sel_idx;
  ap.sel_score = sel_score;
  e = hba::launch_attend(ap, dh, stream);
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  g_last_kernels = cfg->hier ? (tc_sel ? "qknorm_rope_kernel+summarize_kernel+supers_kernel+select_tc_kernel+"
                                         "select_tc_kernel+attend_kernel"
                                       : "qknorm_rope_kernel+summarize_kernel+supers_kernel+select_kernel+"
                                         "select_kernel+attend_kernel")
                             : (tc_sel ? "qknorm_rope_kernel+summarize_kernel+select_tc_kernel+attend_kernel"
                                       : (tile_sel ? "qknorm_rope_kernel+summarize_kernel+select_tile_kernel+"
                                                     "attend_kernel"
                                                   : "qknorm_rope_kernel+summarize_kernel+select_kernel+attend_kernel"));
  return HBA_B200_OK;
}


// ---- the summarizer's aux-KL teacher ----

size_t hba_b200_aux_teacher_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st) || cfg->hier || batch <= 0 || n <= 0 || n % cfg->block != 0) return 0;
  const Geom geo = make_geom(cfg, batch, n, n);
  if (!hba::aux_teacher_supported(geo, cfg->head_dim, n)) return 0;
  const size_t kv = (size_t)batch * n * cfg->n_kv * cfg->head_dim;
  const size_t qv = (size_t)batch * n * cfg->n_heads * cfg->head_dim;
  // status; keys plain, chunk-tiled, RoPE'd tiled; queries; the single pass's block masses
  return kAlign + 3 * align_up(kv * 2) + align_up(qv * 2) + align_up(hba::aux_teacher_scratch_bytes(geo, n));
}

int hba_b200_aux_teacher(const hba_b200_config* cfg, int32_t batch, int32_t n, float scale, const void* q,
                         const void* k, const float* cos, const float* sin, const float* q_gain, const float* k_gain,
                         float* pstar, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || n <= 0 || q == nullptr || k == nullptr || cos == nullptr || sin == nullptr || pstar == nullptr ||
      (cfg->qknorm && (q_gain == nullptr || k_gain == nullptr)) || !std::isfinite(scale))
    return HBA_B200_ERR_INVALID_ARGUMENT;
  if (n % cfg->block != 0) return HBA_B200_ERR_NOT_BLOCK_MULTIPLE;
  if (cfg->hier) return HBA_B200_ERR_UNSUPPORTED;
  const int dh = cfg->head_dim;
  const Geom geo = make_geom(cfg, batch, n, n);
  if (!hba::aux_teacher_supported(geo, dh, n)) return HBA_B200_ERR_UNSUPPORTED;
  const size_t need = hba_b200_aux_teacher_workspace_size(cfg, batch, n);
  if (workspace == nullptr || workspace_bytes < need) return HBA_B200_ERR_WORKSPACE;
  const size_t kv = (size_t)batch * n * cfg->n_kv * dh;
  const size_t qv = (size_t)batch * n * cfg->n_heads * dh;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  int* dev_status = reinterpret_cast<int*>(ws);
  ws += kAlign;
  auto carve = [&](size_t bytes) {
    unsigned char* p = ws;
    ws += align_up(bytes);
    return p;
  };
  auto* kc = reinterpret_cast<__nv_bfloat16*>(carve(kv * 2));
  auto* kc_sw = reinterpret_cast<__nv_bfloat16*>(carve(kv * 2));
  auto* kr_sw = reinterpret_cast<__nv_bfloat16*>(carve(kv * 2));
  auto* qcn = reinterpret_cast<__nv_bfloat16*>(carve(qv * 2));
  const size_t scratch_bytes = hba::aux_teacher_scratch_bytes(geo, n);
  auto* scratch = reinterpret_cast<float*>(carve(scratch_bytes));
  const size_t nb = (size_t)n / cfg->block;
  prof_begin(stream);
  cudaError_t e = cudaMemsetAsync(dev_status, 0, sizeof(int), stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(pstar, 0, (size_t)batch * cfg->n_kv * n * nb * sizeof(float), stream);
  if (e == cudaSuccess)
    e = hba::launch_qknorm_rope(geo, n, static_cast<const __nv_bfloat16*>(k), k_gain, cos, sin, kc, nullptr, dh, stream,
                                nullptr, kc_sw, kr_sw, nullptr);
  const __nv_bfloat16* qsrc = static_cast<const __nv_bfloat16*>(q);
  if (e == cudaSuccess && cfg->qknorm) {
    e = hba::launch_qknorm(qsrc, qcn, q_gain, (int64_t)batch * n, cfg->n_heads, dh, cfg->eps, stream);
    qsrc = qcn;
  }
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  e = hba::launch_aux_teacher(geo, dh, n, scale, qsrc, kc_sw, k_gain, scratch, scratch_bytes, pstar, dev_status,
                              stream);
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  g_last_kernels = cfg->qknorm ? "qknorm_rope_kernel+qknorm_kernel+aux_teacher_kernel" : "qknorm_rope_kernel+aux_teacher_kernel";
  return HBA_B200_OK;
}

// ---- prefill backward ----

size_t hba_b200_prefill_backward_workspace_size(const hba_b200_config* cfg, int32_t batch, int32_t n) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st) || cfg->hier || batch <= 0 || n <= 0 || n % cfg->block != 0) return 0;
  const Geom geo = make_geom(cfg, batch, n, n);
  if (!hba::prefill_bwd_supported(geo, cfg->head_dim, n)) return 0;
  const size_t kv = (size_t)batch * n * cfg->n_kv * cfg->head_dim;
  const size_t qv = (size_t)batch * n * cfg->n_heads * cfg->head_dim;
  size_t b = kAlign;                        // device status word
  b += 4 * align_up(kv * 2);                // QKNorm'd keys; chunk-tiled QKNorm'd keys, RoPE'd keys, values
  b += 2 * align_up(qv * 2);                // queries QKNorm'd, RoPE'd
  b += align_up((size_t)batch * cfg->n_heads * n * 4);  // D per row
  b += 2 * align_up(qv * 4);                // dq w.r.t. the QKNorm'd and the RoPE'd queries (fp32)
  b += 3 * align_up(kv * 4);                // dk (NoPE, RoPE'd), dv (fp32 accumulators)
  return b;
}

int hba_b200_prefill_backward(const hba_b200_config* cfg, int32_t batch, int32_t n, float scale, const void* q,
                              const void* k, const void* v, const float* cos, const float* sin, const float* q_gain,
                              const float* k_gain, const void* out, const float* lse, const int32_t* sel_idx,
                              const void* dout, void* dq, void* dk, void* dv, float* dq_gain, float* dk_gain,
                              void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || n <= 0 || q == nullptr || k == nullptr || v == nullptr || cos == nullptr || sin == nullptr ||
      out == nullptr || lse == nullptr || sel_idx == nullptr || dout == nullptr || dq == nullptr || dk == nullptr ||
      dv == nullptr || (cfg->qknorm && (q_gain == nullptr || k_gain == nullptr)) || !std::isfinite(scale))
    return HBA_B200_ERR_INVALID_ARGUMENT;
  if (n % cfg->block != 0) return HBA_B200_ERR_NOT_BLOCK_MULTIPLE;
  if (cfg->hier) return HBA_B200_ERR_UNSUPPORTED;  // the training path selects flat
  const int dh = cfg->head_dim;
  const Geom geo = make_geom(cfg, batch, n, n);
  if (!hba::prefill_bwd_supported(geo, dh, n)) return HBA_B200_ERR_UNSUPPORTED;
  const size_t need = hba_b200_prefill_backward_workspace_size(cfg, batch, n);
  if (workspace == nullptr || workspace_bytes < need) return HBA_B200_ERR_WORKSPACE;
  const size_t kv = (size_t)batch * n * cfg->n_kv * dh;
  const size_t qv = (size_t)batch * n * cfg->n_heads * dh;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  int* dev_status = reinterpret_cast<int*>(ws);
  ws += kAlign;
  auto carve = [&](size_t bytes) {
    unsigned char* p = ws;
    ws += align_up(bytes);
    return p;
  };
  auto* kc = reinterpret_cast<__nv_bfloat16*>(carve(kv * 2));
  auto* kc_sw = reinterpret_cast<__nv_bfloat16*>(carve(kv * 2));
  auto* kr_sw = reinterpret_cast<__nv_bfloat16*>(carve(kv * 2));
  auto* v_sw = reinterpret_cast<__nv_bfloat16*>(carve(kv * 2));
  auto* qcn = reinterpret_cast<__nv_bfloat16*>(carve(qv * 2));
  auto* qrn = reinterpret_cast<__nv_bfloat16*>(carve(qv * 2));
  auto* delta = reinterpret_cast<float*>(carve((size_t)batch * cfg->n_heads * n * 4));
  auto* dq_acc = reinterpret_cast<float*>(carve(qv * 4));
  auto* dqr_acc = reinterpret_cast<float*>(carve(qv * 4));
  auto* dk_acc = reinterpret_cast<float*>(carve(kv * 4));
  auto* dkr_acc = reinterpret_cast<float*>(carve(kv * 4));
  auto* dv_acc = reinterpret_cast<float*>(carve(kv * 4));
  const auto* kb = static_cast<const __nv_bfloat16*>(k);
  const auto* qb = static_cast<const __nv_bfloat16*>(q);

  prof_begin(stream);
  cudaError_t e = cudaMemsetAsync(dev_status, 0, sizeof(int), stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(dk_acc, 0, kv * 4, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(dkr_acc, 0, kv * 4, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(dv_acc, 0, kv * 4, stream);
  if (e == cudaSuccess && dq_gain != nullptr) e = cudaMemsetAsync(dq_gain, 0, cfg->n_heads * sizeof(float), stream);
  if (e == cudaSuccess && dk_gain != nullptr) e = cudaMemsetAsync(dk_gain, 0, cfg->n_kv * sizeof(float), stream);
  // the forward's pre-pass again: the same QKNorm'd / RoPE'd operands, bit for bit
  if (e == cudaSuccess)
    e = hba::launch_qknorm_rope(geo, n, kb, k_gain, cos, sin, kc, nullptr, dh, stream,
                                static_cast<const __nv_bfloat16*>(v), kc_sw, kr_sw, v_sw);
  if (e == cudaSuccess) {
    Geom gq = geo;
    gq.Hkv = geo.Hq;
    e = hba::launch_qknorm_rope(gq, n, qb, q_gain, cos, sin, qcn, qrn, dh, stream, nullptr, nullptr, nullptr,
                                nullptr);
  }
  if (e == cudaSuccess)
    e = hba::launch_bwd_delta((int64_t)batch * n * cfg->n_heads, n, cfg->n_heads, dh,
                              static_cast<const __nv_bfloat16*>(dout), static_cast<const __nv_bfloat16*>(out), delta,
                              stream);
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  e = hba::launch_prefill_bwd(geo, dh, n, scale, qcn, qrn, static_cast<const __nv_bfloat16*>(dout), kc_sw, kr_sw, v_sw,
                              sel_idx, cfg->k_blocks, lse, delta, dq_acc, dqr_acc, dk_acc, dkr_acc, dv_acc,
                              dev_status, stream);
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  e = hba::launch_bwd_norm((int64_t)batch * n * cfg->n_heads, n, cfg->n_heads, dh, qb, dq_acc, dqr_acc, cos, sin,
                           q_gain, cfg->eps, cfg->qknorm != 0, static_cast<__nv_bfloat16*>(dq), dq_gain, stream);
  if (e == cudaSuccess)
    e = hba::launch_bwd_norm((int64_t)batch * n * cfg->n_kv, n, cfg->n_kv, dh, kb, dk_acc, dkr_acc, cos, sin, k_gain,
                             cfg->eps, cfg->qknorm != 0, static_cast<__nv_bfloat16*>(dk), dk_gain, stream);
  if (e == cudaSuccess)
    e = hba::launch_bwd_norm((int64_t)batch * n * cfg->n_kv, n, cfg->n_kv, dh, nullptr, dv_acc, nullptr, nullptr,
                             nullptr, nullptr, cfg->eps, false, static_cast<__nv_bfloat16*>(dv), nullptr, stream);
  if (e != cudaSuccess) return cuda_status(e);
  prof_mark(stream);
  g_last_kernels = "qknorm_rope_kernel+bwd_delta_kernel+prefill_bwd_kernel+bwd_norm_kernel";
  return HBA_B200_OK;
}


// ---- KV-range sharded decode ----

int hba_b200_decode_shard_select(const hba_b200_config* cfg, int32_t batch, int32_t n_cap_local, int32_t tok_lo,
                                 int32_t level, const int32_t* seq_lens, const float* scales, const void* q,
                                 const float* q_gain, const void* summaries, const void* supers,
                                 const int32_t* in_idx, const float* in_score, int32_t n_in_lists, int32_t* out_idx,
                                 float* out_score, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  const int F = cfg->hier ? cfg->fanout : 1;
  if (batch <= 0 || n_cap_local <= 0 || tok_lo < 0 || seq_lens == nullptr || scales == nullptr || q == nullptr ||
      (cfg->qknorm && q_gain == nullptr) || out_idx == nullptr || out_score == nullptr || level < 0 || level > 2 ||
      (level == 0 && cfg->hier) || (level > 0 && !cfg->hier) || (level == 1 && supers == nullptr) ||
      (level != 1 && summaries == nullptr) || (level == 2 && (in_idx == nullptr || in_score == nullptr || n_in_lists <= 0)))
    return HBA_B200_ERR_INVALID_ARGUMENT;
  // shard bounds on block (hier: super) boundaries, so no block or super straddles two shards
  const long long unit = (long long)cfg->block * F;
  if (n_cap_local % unit != 0 || tok_lo % unit != 0) return HBA_B200_ERR_NOT_BLOCK_MULTIPLE;
  const int nb_local = n_cap_local / cfg->block;
  if (nb_local > 2048 || (long long)cfg->beam * F > 2048 || n_in_lists * cfg->beam > 4096)
    return HBA_B200_ERR_UNSUPPORTED;  // one CTA per (sequence, kv head) scores at most 2048 rows
  Geom geo = make_geom(cfg, batch, 1, n_cap_local);
  hba::SelParams sp{};
  sp.geo = geo;
  sp.qp = hba::QueryPos{seq_lens, scales, 0, 0.f};
  sp.q = static_cast<const __nv_bfloat16*>(q);
  sp.q_gain = q_gain;
  sp.summ = static_cast<const __nv_bfloat16*>(summaries);
  sp.supers = static_cast<const __nv_bfloat16*>(supers);
  sp.mode = level == 0 ? hba::kSelFlat : (level == 1 ? hba::kSelSuper : hba::kSelChild);
  sp.splits = 1;
  sp.list_k = level == 1 ? cfg->beam : cfg->k_blocks;
  sp.in_lists = level == 2 ? n_in_lists : 0;
  sp.in_idx = in_idx;
  sp.in_score = in_score;
  sp.out_idx = out_idx;
  sp.out_score = out_score;
  sp.counters = nullptr;
  sp.pdl = 0;
  sp.own_blo = tok_lo / cfg->block;
  sp.own_bhi = (tok_lo + n_cap_local) / cfg->block;
  sp.n_limit = INT_MAX;  // contexts run past this shard
  return cuda_status(hba::launch_select(sp, cfg->head_dim, stream));
}

int hba_b200_decode_shard_attend(const hba_b200_config* cfg, int32_t batch, int32_t n_cap_local, int32_t tok_lo,
                                 const int32_t* seq_lens, const float* scales, const void* q, const float* q_gain,
                                 const float* k_gain, const void* k_cache, const void* k_rope_cache,
                                 const void* v_cache, const float* cos, const float* sin, const int32_t* in_idx,
                                 const float* in_score, int32_t n_in, float* part_o, float* part_l, float* part_m2,
                                 int32_t* sel_idx, float* sel_score, int32_t* dev_status, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || n_cap_local <= 0 || tok_lo < 0 || seq_lens == nullptr || scales == nullptr || q == nullptr ||
      q_gain == nullptr || k_gain == nullptr || k_cache == nullptr || k_rope_cache == nullptr || v_cache == nullptr ||
      cos == nullptr || sin == nullptr || in_idx == nullptr || in_score == nullptr || n_in <= 0 ||
      part_o == nullptr || part_l == nullptr || part_m2 == nullptr || dev_status == nullptr ||
      ((sel_idx == nullptr) != (sel_score == nullptr)))
    return HBA_B200_ERR_INVALID_ARGUMENT;
  if (n_cap_local % cfg->block != 0 || tok_lo % cfg->block != 0 || n_cap_local % 64 != 0 || tok_lo % 64 != 0)
    return HBA_B200_ERR_NOT_BLOCK_MULTIPLE;
  if (tok_lo > 0 && tok_lo < cfg->sinks) return HBA_B200_ERR_UNSUPPORTED;  // the sinks live on one shard
  Geom geo = make_geom(cfg, batch, 1, n_cap_local);
  if (!hba::decode_tc_supported(geo, cfg->head_dim, k_cache, k_rope_cache, v_cache, nullptr, nullptr))
    return HBA_B200_ERR_UNSUPPORTED;  // the shard partials come from the tensor-core kernel
  hba::DecodeAttnParams dp{};
  dp.geo = geo;
  dp.qp = hba::QueryPos{seq_lens, scales, 0, 0.f};
  dp.q = static_cast<const __nv_bfloat16*>(q);
  dp.q_gain = q_gain;
  dp.k = static_cast<const __nv_bfloat16*>(k_cache);
  dp.kr = static_cast<const __nv_bfloat16*>(k_rope_cache);
  dp.v = static_cast<const __nv_bfloat16*>(v_cache);
  dp.cos = cos;
  dp.sin = sin;
  dp.sel_idx = sel_idx;
  dp.sel_score = sel_score;
  cudaError_t e = cudaMemsetAsync(dev_status, 0, sizeof(int32_t), stream);
  if (e == cudaSuccess)
    e = hba::launch_decode_tc_shard(dp, k_gain, dev_status, cfg->head_dim, tok_lo, in_idx, in_score, n_in, part_o,
                                    part_l, part_m2, stream);
  return cuda_status(e);
}

int hba_b200_decode_shard_finish(const hba_b200_config* cfg, int32_t batch, int32_t world, const float* parts,
                                 void* out, float* lse, cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || world < 1 || parts == nullptr || out == nullptr) return HBA_B200_ERR_INVALID_ARGUMENT;
  return cuda_status(hba::launch_shard_finish(batch * cfg->n_heads, cfg->head_dim, world, parts,
                                              static_cast<__nv_bfloat16*>(out), lse, stream));
}

int hba_b200_host_alloc(int64_t bytes, void** host_ptr, void** dev_ptr) {
  if (bytes <= 0 || host_ptr == nullptr || dev_ptr == nullptr) return HBA_B200_ERR_INVALID_ARGUMENT;
  *host_ptr = nullptr;
  *dev_ptr = nullptr;
  cudaError_t e = cudaHostAlloc(host_ptr, (size_t)bytes, cudaHostAllocMapped);
  if (e == cudaSuccess) e = cudaHostGetDevicePointer(dev_ptr, *host_ptr, 0);
  if (e != cudaSuccess && *host_ptr != nullptr) {
    cudaFreeHost(*host_ptr);
    *host_ptr = nullptr;
    *dev_ptr = nullptr;
  }
  return cuda_status(e);
}

int hba_b200_host_free(void* host_ptr) { return host_ptr == nullptr ? HBA_B200_OK : cuda_status(cudaFreeHost(host_ptr)); }

int64_t hba_b200_shard_xbuf_bytes(const hba_b200_config* cfg, int32_t batch, int32_t world) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st) || batch <= 0 || world < 1 || world > hba::kShardMaxRanks) return -1;
  return (int64_t)hba::x_layout(batch * cfg->n_kv, world, cfg->head_dim).total;
}

int hba_b200_peer_alloc(int64_t bytes, void** dptr, void* ipc_handle) {
  if (bytes <= 0 || dptr == nullptr || ipc_handle == nullptr) return HBA_B200_ERR_INVALID_ARGUMENT;
  *dptr = nullptr;
  cudaError_t e = cudaMalloc(dptr, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(*dptr, 0, (size_t)bytes);  // flags start below every epoch
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), *dptr);
  if (e != cudaSuccess && *dptr != nullptr) {
    cudaFree(*dptr);
    *dptr = nullptr;
  }
  return cuda_status(e);
}

int hba_b200_peer_open(const void* ipc_handle, void** dptr) {
  if (ipc_handle == nullptr || dptr == nullptr) return HBA_B200_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int hba_b200_peer_close(void* dptr) { return dptr == nullptr ? HBA_B200_OK : cuda_status(cudaIpcCloseMemHandle(dptr)); }

int hba_b200_peer_free(void* dptr) { return dptr == nullptr ? HBA_B200_OK : cuda_status(cudaFree(dptr)); }

int hba_b200_decode_shard_fused(const hba_b200_config* cfg, int32_t batch, int32_t n_cap_local, int32_t tok_lo,
                                int32_t world, int32_t rank, void* const* xbufs, int32_t* epoch,
                                const int32_t* seq_lens, const float* scales, const void* q, const float* q_gain,
                                const float* k_gain, const void* summaries, const void* supers, const void* k_cache,
                                const void* k_rope_cache, const void* v_cache, const float* cos, const float* sin,
                                void* out, float* lse, int32_t* sel_idx, float* sel_score, int32_t* dev_status,
                                cudaStream_t stream) {
  int st = HBA_B200_OK;
  if (!config_ok(cfg, &st)) return st;
  if (batch <= 0 || n_cap_local <= 0 || tok_lo < 0 || world < 1 || world > hba::kShardMaxRanks || rank < 0 ||
      rank >= world || xbufs == nullptr || epoch == nullptr || seq_lens == nullptr || scales == nullptr ||
      q == nullptr || q_gain == nullptr || k_gain == nullptr || summaries == nullptr ||
      (cfg->hier && supers == nullptr) || k_cache == nullptr || k_rope_cache == nullptr || v_cache == nullptr ||
      cos == nullptr || sin == nullptr || out == nullptr || dev_status == nullptr ||
      ((sel_idx == nullptr) != (sel_score == nullptr)))
    return HBA_B200_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < world; ++r)
    if (xbufs[r] == nullptr) return HBA_B200_ERR_INVALID_ARGUMENT;
  const int unit = cfg->block * (cfg->hier ? cfg->fanout : 1);  // no block (super) straddles two ranks
  if (n_cap_local % unit != 0 || tok_lo % unit != 0 || n_cap_local % 64 != 0 || tok_lo % 64 != 0)
    return HBA_B200_ERR_NOT_BLOCK_MULTIPLE;
  if (tok_lo > 0 && tok_lo < cfg->sinks) return HBA_B200_ERR_UNSUPPORTED;  // the sinks live on one shard
  if ((int64_t)world * n_cap_local / cfg->block >= 0xffff) return HBA_B200_ERR_UNSUPPORTED;  // 16-bit block ids
  Geom geo = make_geom(cfg, batch, 1, n_cap_local);
  if (!hba::decode_tc_supported(geo, cfg->head_dim, k_cache, k_rope_cache, v_cache, summaries, supers))
    return HBA_B200_ERR_UNSUPPORTED;
  hba::DecodeAttnParams dp{};
  dp.geo = geo;
  dp.trace = g_trace;
  dp.trace_ctas = g_trace_ctas;
  dp.qp = hba::QueryPos{seq_lens, scales, 0, 0.f};
  dp.q = static_cast<const __nv_bfloat16*>(q);
  dp.q_gain = q_gain;
  dp.k = static_cast<const __nv_bfloat16*>(k_cache);
  dp.kr = static_cast<const __nv_bfloat16*>(k_rope_cache);
  dp.v = static_cast<const __nv_bfloat16*>(v_cache);
  dp.cos = cos;
  dp.sin = sin;
  dp.out = static_cast<__nv_bfloat16*>(out);
  dp.lse = lse;
  dp.sel_idx = sel_idx;
  dp.sel_score = sel_score;
  return cuda_status(hba::launch_decode_tc_fused(dp, static_cast<const __nv_bfloat16*>(summaries),
                                                 static_cast<const __nv_bfloat16*>(supers), k_gain, dev_status,
                                                 cfg->head_dim, tok_lo, world, rank, epoch, xbufs, stream));
}

}  // extern "C"
