// Decode entry point for callers that cannot allocate device memory.
//
// Some callers of this library have no way to hand it a workspace: code running where
// cudaMalloc is unavailable or forbidden (a host runtime with its own fixed memory
// pool, an inference server that pre-plans every device byte at start-up, a plugin
// interface that only passes input and output pointers). For them this file provides
// cernels_moe_experts_decode_noalloc(): the same decode kernels as
// cernels_moe_experts_decode(), with their scratch (fp32 activation rows, fp32 per-pair
// output rows, per-block arrival counters) taken from one file-scope __device__ array of
// kNoAllocScratchBytes instead of a caller-provided workspace. No cudaMalloc, cudaFree
// or allocating library routine is called.
//
// The array exists once per device that loads the library and is held until the process
// exits. Host code cannot use the array's name as a device address (in host code it names
// a host-side stand-in), so the device address is looked up once per device with
// cudaGetSymbolAddress while that device is current, on the first call made on it.
#include <mutex>

#include "moe_internal.h"

namespace cernels {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_decode_scratch on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CERNELS_E_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return CERNELS_E_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (err != cudaSuccess || p == nullptr) return CERNELS_E_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return CERNELS_OK;
}

}  // namespace

int noalloc_scratch(void** out) { return scratch_for_current_device(out); }

}  // namespace cernels

using namespace cernels;

extern "C" int cernels_moe_experts_decode_noalloc(const cernels_moe_shape* shape, const void* x,
                                                  const void* gate_up_proj, const float* gate_up_bias,
                                                  const void* down_proj, const float* down_bias,
                                                  const int32_t* indices, const float* weights, void* out,
                                                  void* stream) {
  if (!shape) return CERNELS_E_NULL;
  const cernels_moe_shape s = *shape;
  size_t need = 0;
  int rc = cernels_moe_workspace_bytes(&s, 1, &need);
  if (rc) return rc;
  if (static_cast<long long>(s.tokens) * s.topk > kDecodeMaxPairs) return CERNELS_E_UNSUPPORTED;
  if (need > kNoAllocScratchBytes) return CERNELS_E_UNSUPPORTED;  // beyond the static scratch
  if (s.tokens == 0) return CERNELS_OK;
  void* scratch = nullptr;
  rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  // The decode kernels write every scratch element they later read, the first kernel
  // zeroes the arrival counters itself, and the decode entry point clears the status word
  // (read back with cernels_workspace_status(shape, 1, NULL, ...)), so nothing else has to
  // be cleared here.
  return cernels_moe_experts_decode(&s, x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, out,
                                    scratch, kNoAllocScratchBytes, stream);
}
