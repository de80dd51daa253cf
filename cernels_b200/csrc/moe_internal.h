// Internal (not exported) declarations shared between the kernel translation
// units and the C-ABI layer: the workspace layout and the kernel launchers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstddef>
#include <cstdint>

#include "../../include/cernels_b200.h"

namespace cernels {

// Routing works on chunks of flat (token, slot) entries, one CTA per chunk: 256 entries for
// small batches (more CTAs), kRouteChunk for large ones.
constexpr int kRouteChunk = 1024;
constexpr int kRouteSmallChunk = 256;
inline int route_chunk(long long total) { return total <= 16384 ? kRouteSmallChunk : kRouteChunk; }
constexpr int kRouteThreads = 256;
constexpr int kMaxExperts = 2048;

// Grouped-GEMM tile shape (rows of the permuted token matrix per tile).
constexpr int kBlockM = 128;

// Decode path limits: total (token, slot) pairs per call.
constexpr int kDecodeMaxPairs = 1024;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Limit of the bounded waits inside kernels, in ns: `default_ns` unless
// cernels_set_wait_limit_ns() set one. Read by every launcher and passed as an argument.
unsigned long long wait_limit_ns(unsigned long long default_ns);

// Runs `set` (a cudaFuncSetAttribute call) once per device: kernel attributes belong to a
// device context, so a process that drives several GPUs needs them on each.
struct PerDeviceOnce {
  std::atomic<unsigned long long> done{0};
  template <class F>
  cudaError_t run(F&& set) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= 64) return set();
    const unsigned long long bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    err = set();  // two host threads may both get here: setting an attribute twice is harmless
    if (err == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return err;
  }
};

// Device pointers carved out of one caller-provided workspace allocation.
struct PrefillWorkspace {
  int* status;          // [1] device status word (cernels::DeviceStatus)
  int* block_counts;    // [n_chunks * E] per-chunk histograms, then per-chunk bases
  int* offsets;         // [E + 1] row offset of each expert in the permuted order
  int* mtile_offsets;   // [E + 1] cumulative count of 128-row tiles per expert
  int* perm_flat;       // [Tk] flat (token * topk + slot) index of each permuted row
  int* perm_token;      // [Tk] token id of each permuted row
  float* perm_weight;   // [Tk] router weight of each permuted row
  int* inv;             // [Tk] permuted row of each flat entry (-1 when skipped)
  __nv_bfloat16* gathered;  // [Tk, H] token rows in permuted (expert-major) order
  __nv_bfloat16* glu;       // [Tk, F] activation output of the gate/up GEMM
  __nv_bfloat16* down_out;  // [Tk, H] output of the down GEMM (unweighted)
};

struct DecodeWorkspace {
  int* status;       // [1]
  int* counters;     // [max(H, F) / 8 + 1] arrival counters of the down stage
  float* glu;        // [Tk, F] fp32 activation rows (flat (token, slot) order)
  float* partial;    // [s2, Tk, H] fp32 per-pair down-projection rows, one slab per K split
  float* pre;        // [s1, Tk, 2F] fp32 gate/up split sums (only when s1 > 1)
};

// K splits of the GPTOSS decode kernels (gate/up s1, down s2): enough CTAs to keep every
// SM's load pipeline full when only a few experts are touched. A function of the shape
// only, so workspace sizing and launch agree.
struct DecodeSplits {
  int s1, s2;
};
DecodeSplits decode_splits(int tokens, int topk, int experts, int hidden, int inter, int layout);

size_t prefill_workspace_bytes(const cernels_moe_shape& s);
PrefillWorkspace carve_prefill_workspace(const cernels_moe_shape& s, void* base);
size_t decode_workspace_bytes(const cernels_moe_shape& s);
DecodeWorkspace carve_decode_workspace(const cernels_moe_shape& s, void* base);

// ---- launchers (return cudaError_t of the launch)
cudaError_t launch_route(const int32_t* indices, const float* weights, int tokens, int topk, int experts,
                         const PrefillWorkspace& ws, cudaStream_t stream);
// Copies rows [0, rows) (and only those below *row_count when row_count is non-null).
cudaError_t launch_gather(const __nv_bfloat16* x, const int* perm_token, int rows, const int* row_count,
                          int hidden, __nv_bfloat16* gathered, cudaStream_t stream);
// Row groups given by counts: offsets[g] = sum of counts before g, mtile_offsets likewise in
// 128-row tiles. `scratch` holds `groups` ints.
cudaError_t launch_segments(const int* counts, int groups, int* scratch, int* offsets, int* mtile_offsets,
                            cudaStream_t stream);
cudaError_t launch_combine(const __nv_bfloat16* down_out, const int* inv, const float* weights, int tokens,
                           int topk, int hidden, __nv_bfloat16* out, cudaStream_t stream);

struct GroupedGemmArgs {
  const __nv_bfloat16* a;      // [rows, K] permuted activations
  const __nv_bfloat16* b;      // expert weights (layout per mode)
  const float* bias;           // [E, N] fp32 or nullptr
  __nv_bfloat16* out;          // [rows, out_cols]
  const int* offsets;          // [E + 1]
  const int* mtile_offsets;    // [E + 1]
  int* status;
  int rows;                    // Tk (row count of a / out)
  int experts;
  int k;                       // reduction length
  int n;                       // columns of the weight product (2F or H)
  int out_cols;                // F for gate/up, H for down
  int weight_experts;          // experts in the weight tensors; row group g uses expert g % weight_experts
  unsigned long long wait_ns;  // limit of each bounded mbarrier wait
  const int* group_rows;       // optional [groups]: rows of group g (default offsets[g+1] - offsets[g])
  // Optional always-on extra group (a shared expert): group `extra_group` takes its weights
  // from b_extra (one slab, same layout as b) instead of b. Unused when b_extra is null.
  const __nv_bfloat16* b_extra;
  int extra_group;
  // Optional per-row output rows (indexed like the rows of a): when set, row r's outputs go to
  // row_out[r] (any device-visible address, a peer GPU's included; null = not written) instead
  // of out + r * out_cols.
  __nv_bfloat16* const* row_out;
  // Optional arrival wait (expert parallelism): before loading the first tile of group g, the
  // producer waits (bounded) until the 32-bit flag at ready + s * ready_stride + 4 * g equals
  // the step's epoch for every source s != ready_self (ready_epoch, or *ready_epoch_dev + 1 when
  // ready_epoch is 0). Null: no wait.
  const uint8_t* ready;
  size_t ready_stride;
  int ready_sources, ready_self;
  uint32_t ready_epoch;
  const uint32_t* ready_epoch_dev;
};

enum GemmMode : int {
  kGateUpLinear = 0,   // B = gate_up_proj [E, 2F, H] (K-major), chunked gate|up, SiLU
  kGateUpGptOss = 1,   // B = gate_up_proj [E, H, 2F] (N-major), interleaved, clamped SwiGLU + bias
  kDownLinear = 2,     // B = down_proj [E, H, F] (K-major)
  kDownGptOss = 3,     // B = down_proj [E, F, H] (N-major), + bias
};

cudaError_t launch_grouped_gemm(GemmMode mode, const GroupedGemmArgs& args, int num_sms, cudaStream_t stream);

struct DecodeArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w1;
  const float* b1;
  const __nv_bfloat16* w2;
  const float* b2;
  const int32_t* indices;
  const float* weights;
  __nv_bfloat16* out;
  int tokens, hidden, experts, inter, topk, layout;
};
cudaError_t launch_decode(const DecodeArgs& a, const DecodeWorkspace& ws, cudaStream_t stream);

// Router tail (router.cu). mode 0: top-k of the logits, softmax over the k values rounded to
// bf16; mode 1: softmax over all experts (fp32), top-k, optional renormalisation.
cudaError_t launch_router_topk(const void* logits, int bf16, int tokens, int experts, int topk, int mode, int renorm,
                               int shared_gate, int32_t* idx, float* w, cudaStream_t stream);

int device_sm_count();

// Tiled bf16 TMA map with 128-byte swizzle (grouped_gemm.cu).
bool encode_bf16_map(CUtensorMap* map, const void* ptr, int rank, const uint64_t* dims, const uint64_t* byte_strides,
                     const uint32_t* box);

// Fused router GEMM + top-k tail (router_gemm.cu): column split of the logits over a cluster
// of nc CTAs (bn columns each), 128-token tiles.
struct RouterPlan {
  int nc, bn, kmax, tmem_cols, m_tiles;
};
RouterPlan router_plan(int tokens, int experts, int weight_rows, int gate, int topk);
cudaError_t launch_router_gemm(const void* x, int tokens, int hidden, const void* w, int weight_rows,
                               const void* bias, int experts, int topk, int mode, int renorm, int gate,
                               int32_t* indices, float* weights, void* logits, int* status, cudaStream_t stream);

// Device address of the static decode scratch of cernels_moe_experts_decode_noalloc on the
// current device (looked up on first use per device). Returns a CERNELS_* code.
int noalloc_scratch(void** out);

}  // namespace cernels
