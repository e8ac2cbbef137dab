// Allocation-free decode entry point.
//
// Some callers cannot allocate device memory at the moment they decode: a
// serving engine that hands every byte of HBM to its own arena at start-up,
// a plugin host that exposes no allocator to its plugins, or code that runs
// where cudaMalloc is forbidden (inside a signal-driven or real-time loop).
// hba_b200_decode needs a caller-provided workspace; this variant instead uses
// a fixed scratch array that lives in the library's own device image, so the
// caller passes only inputs and outputs and nothing is allocated per call.
//
// The scratch is a file-scope __device__ array of kScratchBytes (8 MiB); every
// GPU that loads the library holds it until the process exits.  Its device
// address is looked up once per device (cudaGetSymbolAddress with that device
// current) on the first call made while that device is current, so make that
// first call before any stream capture.  All calls on a device share the one
// array and it keeps the last call's contents: decode writes every scratch
// byte it reads (its merge counters are zeroed by the call's own selection
// kernel), so nothing needs clearing, but calls whose kernels overlap on
// the GPU (different streams, no ordering between them) race on it.
#include <mutex>

#include "hba_b200.h"

namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array for the current device, looked up once.
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

int hba_b200_decode_noalloc(const hba_b200_config* cfg, int32_t batch, int32_t n_cap, const int32_t* seq_lens,
                            const float* scales, const void* q, const float* q_gain, const float* k_gain,
                            const void* k_cache,
                            const void* k_rope_cache, const void* v_cache, const void* summaries,
                            const void* supers, const float* cos, const float* sin, void* out, float* lse,
                            int32_t* sel_idx, float* sel_score, cudaStream_t stream) {
  const size_t need = hba_b200_decode_workspace_size(cfg, batch, n_cap);
  if (need > kScratchBytes) return HBA_B200_ERR_WORKSPACE;  // batch x context too large for the fixed scratch
  void* scratch = nullptr;
  const cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) return HBA_B200_ERR_CUDA;
  return hba_b200_decode(cfg, batch, n_cap, seq_lens, scales, q, q_gain, k_gain, k_cache, k_rope_cache, v_cache,
                         summaries,
                         supers, cos, sin, out, lse, sel_idx, sel_score, scratch, kScratchBytes, stream);
}

int hba_b200_decode_noalloc_status(int32_t clear, cudaStream_t stream) {
  // the decode's sticky status word is the first 4 bytes of its workspace,
  // here the scratch array
  void* scratch = nullptr;
  const cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) return HBA_B200_ERR_CUDA;
  return hba_b200_device_status(scratch, clear, stream);
}

}  // extern "C"
