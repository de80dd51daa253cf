// C ABI: argument validation, workspace carving and the launch sequence of each entry
// point. Validation mirrors the reference's TORCH_CHECKs
// (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:213-216,253-257) as return codes.
#include <cstdio>
#include <cstring>

#include "moe_internal.h"

namespace cernels {

namespace {

constexpr size_t kAlign = 256;

struct Carver {
  uint8_t* base;
  size_t off = 0;
  template <class T>
  T* take(size_t count) {
    off = align_up(off, kAlign);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

template <class F>
PrefillWorkspace carve_prefill(const cernels_moe_shape& s, void* base, F&& done) {
  Carver c{static_cast<uint8_t*>(base)};
  const size_t tk = static_cast<size_t>(s.tokens) * s.topk;
  const size_t chunk = static_cast<size_t>(route_chunk(static_cast<long long>(tk)));
  const size_t n_chunks = (tk + chunk - 1) / chunk;
  PrefillWorkspace w;
  w.status = c.take<int>(1);
  w.block_counts = c.take<int>(n_chunks * s.experts + 1);
  w.offsets = c.take<int>(s.experts + 1);
  w.mtile_offsets = c.take<int>(s.experts + 1);
  w.perm_flat = c.take<int>(tk + 1);
  w.perm_token = c.take<int>(tk + 1);
  w.perm_weight = c.take<float>(tk + 1);
  w.inv = c.take<int>(tk + 1);
  w.gathered = c.take<__nv_bfloat16>(tk * s.hidden + 8);
  w.glu = c.take<__nv_bfloat16>(tk * s.intermediate + 8);
  w.down_out = c.take<__nv_bfloat16>(tk * s.hidden + 8);
  done(c.off);
  return w;
}

template <class F>
DecodeWorkspace carve_decode(const cernels_moe_shape& s, void* base, F&& done) {
  Carver c{static_cast<uint8_t*>(base)};
  const size_t tk = static_cast<size_t>(s.tokens) * s.topk;
  DecodeWorkspace w;
  w.status = c.take<int>(1);
  w.counters = c.take<int>(static_cast<size_t>(s.hidden) + 8);
  const DecodeSplits sp = decode_splits(s.tokens, s.topk, s.experts, s.hidden, s.intermediate, s.layout);
  w.glu = c.take<float>(tk * s.intermediate + 4);
  w.partial = c.take<float>(static_cast<size_t>(sp.s2) * tk * s.hidden + 4);
  w.pre = sp.s1 > 1 ? c.take<float>(static_cast<size_t>(sp.s1) * tk * 2 * s.intermediate + 4) : nullptr;
  done(c.off);
  return w;
}

int check_shape(const cernels_moe_shape* s) {
  if (!s) return CERNELS_E_NULL;
  if (s->tokens < 0 || s->hidden <= 0 || s->experts <= 0 || s->intermediate <= 0 || s->topk <= 0)
    return CERNELS_E_INVALID_SHAPE;
  if (s->layout != CERNELS_LAYOUT_LINEAR && s->layout != CERNELS_LAYOUT_GPTOSS) return CERNELS_E_INVALID_SHAPE;
  if (s->experts > kMaxExperts) return CERNELS_E_UNSUPPORTED;
  if (static_cast<long long>(s->tokens) * s->topk > (1ll << 30)) return CERNELS_E_UNSUPPORTED;
  // 16-byte rows for vector loads and TMA strides.
  if (s->hidden % 8 != 0 || s->intermediate % 8 != 0) return CERNELS_E_ALIGNMENT;
  return CERNELS_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int cuda_rc(cudaError_t e) {
  if (e == cudaSuccess) return CERNELS_OK;
  std::fprintf(stderr, "cernels_b200: CUDA error: %s\n", cudaGetErrorString(e));
  return CERNELS_E_CUDA;
}

std::atomic<unsigned long long> g_wait_limit_ns{0};

int sm_count_cached() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  static int counts[64] = {0};
  if (dev < 0 || dev >= 64) return 0;
  if (counts[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n;
  }
  return counts[dev];
}

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CERNELS_E_CUDA;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) return CERNELS_E_UNSUPPORTED;  // built for sm_100a only
  return CERNELS_OK;
}

}  // namespace

size_t prefill_workspace_bytes(const cernels_moe_shape& s) {
  size_t n = 0;
  carve_prefill(s, nullptr, [&](size_t off) { n = off; });
  return n;
}
PrefillWorkspace carve_prefill_workspace(const cernels_moe_shape& s, void* base) {
  return carve_prefill(s, base, [](size_t) {});
}
size_t decode_workspace_bytes(const cernels_moe_shape& s) {
  size_t n = 0;
  carve_decode(s, nullptr, [&](size_t off) { n = off; });
  return n;
}
DecodeWorkspace carve_decode_workspace(const cernels_moe_shape& s, void* base) {
  return carve_decode(s, base, [](size_t) {});
}

int device_sm_count() { return sm_count_cached(); }

unsigned long long wait_limit_ns(unsigned long long default_ns) {
  const unsigned long long v = g_wait_limit_ns.load(std::memory_order_relaxed);
  return v ? v : default_ns;
}

}  // namespace cernels

using namespace cernels;

extern "C" {

const char* cernels_error_string(int code) {
  switch (code) {
    case CERNELS_OK: return "ok";
    case CERNELS_E_INVALID_SHAPE: return "invalid or unsupported shape";
    case CERNELS_E_ALIGNMENT: return "H and F must be multiples of 8 and pointers 16-byte aligned";
    case CERNELS_E_WORKSPACE: return "workspace missing or too small";
    case CERNELS_E_CUDA: return "CUDA call failed";
    case CERNELS_E_UNSUPPORTED: return "unsupported device or size limit of this build";
    case CERNELS_E_NULL: return "required pointer is NULL";
  }
  return "unknown error";
}

int cernels_version(void) { return 200; }

int cernels_set_wait_limit_ns(uint64_t ns) {
  g_wait_limit_ns.store(ns, std::memory_order_relaxed);
  return CERNELS_OK;
}

int cernels_moe_workspace_bytes(const cernels_moe_shape* shape, int decode, size_t* bytes) {
  const int rc = check_shape(shape);
  if (rc) return rc;
  if (!bytes) return CERNELS_E_NULL;
  *bytes = decode ? decode_workspace_bytes(*shape) : prefill_workspace_bytes(*shape);
  return CERNELS_OK;
}

static int validate_common(const cernels_moe_shape* shape, const void* x, const void* w1, const void* w2,
                           const int32_t* indices, const float* weights, void* out, void* workspace,
                           size_t ws_bytes, size_t need) {
  int rc = check_shape(shape);
  if (rc) return rc;
  if (shape->tokens == 0) return CERNELS_OK;
  if (!x || !w1 || !w2 || !indices || !weights || !out) return CERNELS_E_NULL;
  if (!aligned16(x) || !aligned16(w1) || !aligned16(w2) || !aligned16(out)) return CERNELS_E_ALIGNMENT;
  if (!workspace || ws_bytes < need) return CERNELS_E_WORKSPACE;
  if (!aligned16(workspace)) return CERNELS_E_ALIGNMENT;
  return check_device();
}

// Launch sequence of the prefill path. When `events` is non-null, events[i] is recorded
// before stage i and events[5] after the last stage.
// With shared_w1 / shared_w2 (one always-on expert, same F), `shape` describes the routed
// experts and top-k; indices / weights carry topk + 1 columns, the last one routing every
// token to expert id E (the shared expert) with its gate weight.
static int run_prefill(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                       const float* gate_up_bias, const void* down_proj, const float* down_bias,
                       const int32_t* indices, const float* weights, void* out, void* workspace,
                       size_t workspace_bytes, cudaStream_t stream, cudaEvent_t* events,
                       const void* shared_w1 = nullptr, const void* shared_w2 = nullptr) {
  const int rc0 = check_shape(shape);
  if (rc0) return rc0;
  const bool has_shared = shared_w1 != nullptr;
  const int routed_experts = shape->experts;
  cernels_moe_shape s = *shape;
  if (has_shared) {
    if (!shared_w2) return CERNELS_E_NULL;
    if (s.layout != CERNELS_LAYOUT_LINEAR) return CERNELS_E_UNSUPPORTED;
    if (!aligned16(shared_w1) || !aligned16(shared_w2)) return CERNELS_E_ALIGNMENT;
    s.experts += 1;  // expert id E is the shared expert
    s.topk += 1;     // its slot is the last column
    if (check_shape(&s)) return check_shape(&s);
  }
  int rc = validate_common(&s, x, gate_up_proj, down_proj, indices, weights, out, workspace, workspace_bytes,
                           prefill_workspace_bytes(s));
  if (rc || s.tokens == 0) return rc;
  const PrefillWorkspace ws = carve_prefill_workspace(s, workspace);
  const int tk = s.tokens * s.topk;
  const bool gptoss = s.layout == CERNELS_LAYOUT_GPTOSS;
  auto mark = [&](int i) {
    if (events) cudaEventRecord(events[i], stream);
  };
  cudaError_t err = cudaMemsetAsync(ws.status, 0, sizeof(int), stream);
  if (err != cudaSuccess) return cuda_rc(err);

  mark(0);
  err = launch_route(indices, weights, s.tokens, s.topk, s.experts, ws, stream);
  if (err != cudaSuccess) return cuda_rc(err);
  mark(1);
  // Rows at or past offsets[E] belong to no expert (skipped ids): not gathered, never read.
  err = launch_gather(static_cast<const __nv_bfloat16*>(x), ws.perm_token, tk, ws.offsets + s.experts, s.hidden,
                      ws.gathered, stream);
  if (err != cudaSuccess) return cuda_rc(err);
  mark(2);
  const int sms = device_sm_count();
  GroupedGemmArgs g1{};
  g1.a = ws.gathered;
  g1.b = static_cast<const __nv_bfloat16*>(gate_up_proj);
  g1.bias = gptoss ? gate_up_bias : nullptr;
  g1.out = ws.glu;
  g1.offsets = ws.offsets;
  g1.mtile_offsets = ws.mtile_offsets;
  g1.status = ws.status;
  g1.rows = tk;
  g1.experts = s.experts;
  g1.k = s.hidden;
  g1.n = 2 * s.intermediate;
  g1.out_cols = s.intermediate;
  g1.weight_experts = routed_experts;
  if (has_shared) {
    g1.b_extra = static_cast<const __nv_bfloat16*>(shared_w1);
    g1.extra_group = routed_experts;
  }
  err = launch_grouped_gemm(gptoss ? kGateUpGptOss : kGateUpLinear, g1, sms, stream);
  if (err != cudaSuccess) return cuda_rc(err);
  mark(3);
  GroupedGemmArgs g2{};
  g2.a = ws.glu;
  g2.b = static_cast<const __nv_bfloat16*>(down_proj);
  g2.bias = gptoss ? down_bias : nullptr;
  g2.out = ws.down_out;
  g2.offsets = ws.offsets;
  g2.mtile_offsets = ws.mtile_offsets;
  g2.status = ws.status;
  g2.rows = tk;
  g2.experts = s.experts;
  g2.k = s.intermediate;
  g2.n = s.hidden;
  g2.out_cols = s.hidden;
  g2.weight_experts = routed_experts;
  if (has_shared) {
    g2.b_extra = static_cast<const __nv_bfloat16*>(shared_w2);
    g2.extra_group = routed_experts;
  }
  err = launch_grouped_gemm(gptoss ? kDownGptOss : kDownLinear, g2, sms, stream);
  if (err != cudaSuccess) return cuda_rc(err);
  mark(4);
  err = launch_combine(ws.down_out, ws.inv, weights, s.tokens, s.topk, s.hidden, static_cast<__nv_bfloat16*>(out),
                       stream);
  mark(5);
  return cuda_rc(err);
}

int cernels_moe_experts(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                        const float* gate_up_bias, const void* down_proj, const float* down_bias,
                        const int32_t* indices, const float* weights, void* out, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return run_prefill(shape, x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, out, workspace,
                     workspace_bytes, static_cast<cudaStream_t>(stream), nullptr);
}

int cernels_moe_experts_shared(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                               const void* down_proj, const void* shared_gate_up_proj, const void* shared_down_proj,
                               const int32_t* indices, const float* weights, void* out, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!shared_gate_up_proj || !shared_down_proj) return CERNELS_E_NULL;
  return run_prefill(shape, x, gate_up_proj, nullptr, down_proj, nullptr, indices, weights, out, workspace,
                     workspace_bytes, static_cast<cudaStream_t>(stream), nullptr, shared_gate_up_proj,
                     shared_down_proj);
}

int cernels_moe_experts_profiled(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                                 const float* gate_up_bias, const void* down_proj, const float* down_bias,
                                 const int32_t* indices, const float* weights, void* out, void* workspace,
                                 size_t workspace_bytes, void* stream_ptr, float* stage_ms) {
  if (!stage_ms) return CERNELS_E_NULL;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaEvent_t ev[6];
  for (int i = 0; i < 6; ++i)
    if (cudaEventCreate(&ev[i]) != cudaSuccess) return CERNELS_E_CUDA;
  int rc = run_prefill(shape, x, gate_up_proj, gate_up_bias, down_proj, down_bias, indices, weights, out, workspace,
                       workspace_bytes, stream, ev);
  if (rc == CERNELS_OK && shape->tokens > 0) {
    cudaError_t err = cudaEventSynchronize(ev[5]);
    for (int i = 0; i < 5 && err == cudaSuccess; ++i) err = cudaEventElapsedTime(&stage_ms[i], ev[i], ev[i + 1]);
    rc = cuda_rc(err);
  }
  for (int i = 0; i < 6; ++i) cudaEventDestroy(ev[i]);
  return rc;
}

int cernels_moe_experts_decode(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                               const float* gate_up_bias, const void* down_proj, const float* down_bias,
                               const int32_t* indices, const float* weights, void* out, void* workspace,
                               size_t workspace_bytes, void* stream_ptr) {
  const int rc0 = check_shape(shape);
  if (rc0) return rc0;
  const cernels_moe_shape s = *shape;
  if (static_cast<long long>(s.tokens) * s.topk > kDecodeMaxPairs) return CERNELS_E_UNSUPPORTED;
  int rc = validate_common(shape, x, gate_up_proj, down_proj, indices, weights, out, workspace, workspace_bytes,
                           decode_workspace_bytes(s));
  if (rc || s.tokens == 0) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const DecodeWorkspace ws = carve_decode_workspace(s, workspace);
  const cudaError_t zero = cudaMemsetAsync(ws.status, 0, sizeof(int), stream);
  if (zero != cudaSuccess) return cuda_rc(zero);
  DecodeArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.w1 = static_cast<const __nv_bfloat16*>(gate_up_proj);
  a.b1 = s.layout == CERNELS_LAYOUT_GPTOSS ? gate_up_bias : nullptr;
  a.w2 = static_cast<const __nv_bfloat16*>(down_proj);
  a.b2 = s.layout == CERNELS_LAYOUT_GPTOSS ? down_bias : nullptr;
  a.indices = indices;
  a.weights = weights;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.tokens = s.tokens;
  a.hidden = s.hidden;
  a.experts = s.experts;
  a.inter = s.intermediate;
  a.topk = s.topk;
  a.layout = s.layout;
  return cuda_rc(launch_decode(a, ws, stream));
}

int cernels_moe_grouped_experts(const cernels_moe_shape* shape, int32_t groups, const int32_t* group_counts,
                                const void* rows_in, const void* gate_up_proj, const float* gate_up_bias,
                                const void* down_proj, const float* down_bias, void* rows_out, void* workspace,
                                size_t workspace_bytes, void* stream_ptr) {
  int rc = check_shape(shape);
  if (rc) return rc;
  const cernels_moe_shape s = *shape;
  if (groups <= 0 || groups > kMaxExperts || groups % s.experts != 0) return CERNELS_E_INVALID_SHAPE;
  if (s.tokens == 0) return CERNELS_OK;
  if (!group_counts || !rows_in || !gate_up_proj || !down_proj || !rows_out) return CERNELS_E_NULL;
  if (!aligned16(rows_in) || !aligned16(rows_out) || !aligned16(gate_up_proj) || !aligned16(down_proj))
    return CERNELS_E_ALIGNMENT;
  cernels_moe_shape ws_shape = s;
  ws_shape.experts = groups;
  ws_shape.topk = 1;
  if (!workspace || workspace_bytes < prefill_workspace_bytes(ws_shape)) return CERNELS_E_WORKSPACE;
  if ((rc = check_device())) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const PrefillWorkspace ws = carve_prefill_workspace(ws_shape, workspace);
  const bool gptoss = s.layout == CERNELS_LAYOUT_GPTOSS;
  cudaError_t err = cudaMemsetAsync(ws.status, 0, sizeof(int), stream);
  if (err == cudaSuccess) err = launch_segments(group_counts, groups, ws.block_counts, ws.offsets, ws.mtile_offsets, stream);
  if (err != cudaSuccess) return cuda_rc(err);
  const int sms = device_sm_count();
  GroupedGemmArgs g1{};
  g1.a = static_cast<const __nv_bfloat16*>(rows_in);
  g1.b = static_cast<const __nv_bfloat16*>(gate_up_proj);
  g1.bias = gptoss ? gate_up_bias : nullptr;
  g1.out = ws.glu;
  g1.offsets = ws.offsets;
  g1.mtile_offsets = ws.mtile_offsets;
  g1.status = ws.status;
  g1.rows = s.tokens;
  g1.experts = groups;
  g1.k = s.hidden;
  g1.n = 2 * s.intermediate;
  g1.out_cols = s.intermediate;
  g1.weight_experts = s.experts;
  err = launch_grouped_gemm(gptoss ? kGateUpGptOss : kGateUpLinear, g1, sms, stream);
  if (err != cudaSuccess) return cuda_rc(err);
  GroupedGemmArgs g2 = g1;
  g2.a = ws.glu;
  g2.b = static_cast<const __nv_bfloat16*>(down_proj);
  g2.bias = gptoss ? down_bias : nullptr;
  g2.out = static_cast<__nv_bfloat16*>(rows_out);
  g2.k = s.intermediate;
  g2.n = s.hidden;
  g2.out_cols = s.hidden;
  return cuda_rc(launch_grouped_gemm(gptoss ? kDownGptOss : kDownLinear, g2, sms, stream));
}

int cernels_router_topk(const void* logits, int32_t logits_bf16, int32_t tokens, int32_t experts, int32_t topk,
                        int32_t mode, int32_t renorm, int32_t shared_gate, int32_t* indices, float* weights,
                        void* stream) {
  if (tokens < 0 || experts <= 0 || experts > 1024 || topk <= 0 || topk > 32 || topk > experts)
    return CERNELS_E_INVALID_SHAPE;
  if (mode != CERNELS_ROUTER_TOPK_SOFTMAX && mode != CERNELS_ROUTER_SOFTMAX_TOPK) return CERNELS_E_INVALID_SHAPE;
  if (tokens == 0) return CERNELS_OK;
  if (!logits || !indices || !weights) return CERNELS_E_NULL;
  return cuda_rc(launch_router_topk(logits, logits_bf16 != 0, tokens, experts, topk, mode, renorm != 0,
                                    shared_gate != 0, indices, weights, static_cast<cudaStream_t>(stream)));
}

int cernels_router(const void* x, int32_t tokens, int32_t hidden, const void* router_weight, int32_t weight_rows,
                   const void* router_bias, int32_t experts, int32_t topk, int32_t mode, int32_t renorm,
                   int32_t shared_gate, int32_t* indices, float* weights, void* logits_out, void* stream) {
  if (tokens < 0 || hidden <= 0 || experts <= 0 || topk <= 0 || topk > 16 || topk > experts)
    return CERNELS_E_INVALID_SHAPE;
  if (mode != CERNELS_ROUTER_TOPK_SOFTMAX && mode != CERNELS_ROUTER_SOFTMAX_TOPK) return CERNELS_E_INVALID_SHAPE;
  const int cols = experts + (shared_gate ? 1 : 0);
  if (weight_rows < cols || cols > 8 * 256) return CERNELS_E_INVALID_SHAPE;
  if (hidden % 8) return CERNELS_E_ALIGNMENT;
  if (tokens == 0) return CERNELS_OK;
  if (!x || !router_weight || !indices || !weights) return CERNELS_E_NULL;
  if (!aligned16(x) || !aligned16(router_weight)) return CERNELS_E_ALIGNMENT;
  if (const int rc = check_device()) return rc;
  return cuda_rc(launch_router_gemm(x, tokens, hidden, router_weight, weight_rows, router_bias, experts, topk, mode,
                                    renorm != 0, shared_gate != 0, indices, weights, logits_out, nullptr,
                                    static_cast<cudaStream_t>(stream)));
}

int cernels_moe_route(const cernels_moe_shape* shape, const int32_t* indices, const float* weights,
                      int32_t* offsets, int32_t* perm_token, float* perm_weight, int32_t* inv, void* workspace,
                      size_t workspace_bytes, void* stream_ptr) {
  int rc = check_shape(shape);
  if (rc) return rc;
  const cernels_moe_shape s = *shape;
  if (!offsets || !perm_token || !perm_weight || !inv) return CERNELS_E_NULL;
  if (s.tokens > 0 && (!indices || !weights)) return CERNELS_E_NULL;
  if (!workspace || workspace_bytes < prefill_workspace_bytes(s)) return CERNELS_E_WORKSPACE;
  if ((rc = check_device())) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  PrefillWorkspace ws = carve_prefill_workspace(s, workspace);
  // Route straight into the caller's arrays.
  ws.offsets = offsets;
  ws.perm_token = perm_token;
  ws.perm_weight = perm_weight;
  ws.inv = inv;
  return cuda_rc(launch_route(indices, weights, s.tokens, s.topk, s.experts, ws, stream));
}

int cernels_moe_gather(const void* x, const int32_t* perm_token, int32_t rows, int32_t hidden, void* rows_out,
                       void* stream_ptr) {
  if (rows < 0 || hidden <= 0) return CERNELS_E_INVALID_SHAPE;
  if (hidden % 8) return CERNELS_E_ALIGNMENT;
  if (rows == 0) return CERNELS_OK;
  if (!x || !perm_token || !rows_out) return CERNELS_E_NULL;
  if (!aligned16(x) || !aligned16(rows_out)) return CERNELS_E_ALIGNMENT;
  return cuda_rc(launch_gather(static_cast<const __nv_bfloat16*>(x), perm_token, rows, nullptr, hidden,
                               static_cast<__nv_bfloat16*>(rows_out), static_cast<cudaStream_t>(stream_ptr)));
}

int cernels_moe_combine(const void* rows, const int32_t* inv, const float* weights, int32_t tokens, int32_t topk,
                        int32_t hidden, void* out, void* stream_ptr) {
  if (tokens < 0 || topk <= 0 || hidden <= 0) return CERNELS_E_INVALID_SHAPE;
  if (hidden % 8) return CERNELS_E_ALIGNMENT;
  if (tokens == 0) return CERNELS_OK;
  if (!inv || !weights || !out) return CERNELS_E_NULL;
  if (!aligned16(out) || (rows && !aligned16(rows))) return CERNELS_E_ALIGNMENT;
  return cuda_rc(launch_combine(static_cast<const __nv_bfloat16*>(rows), inv, weights, tokens, topk, hidden,
                                static_cast<__nv_bfloat16*>(out), static_cast<cudaStream_t>(stream_ptr)));
}

int cernels_workspace_status(const cernels_moe_shape* shape, int decode, const void* workspace, int* status,
                             void* stream_ptr) {
  const int rc = check_shape(shape);
  if (rc) return rc;
  if (!status) return CERNELS_E_NULL;
  if (!workspace) {
    // decode with no workspace: the scratch of cernels_moe_experts_decode_noalloc
    if (!decode) return CERNELS_E_NULL;
    void* scratch = nullptr;
    if (const int rc2 = noalloc_scratch(&scratch)) return rc2;
    workspace = scratch;
  }
  const int* dev = decode ? carve_decode_workspace(*shape, const_cast<void*>(workspace)).status
                          : carve_prefill_workspace(*shape, const_cast<void*>(workspace)).status;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaError_t err = cudaMemcpyAsync(status, dev, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
  return cuda_rc(err);
}

}  // extern "C"
