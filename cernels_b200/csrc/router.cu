// Router tail: top-k selection and routing weights from router logits, one launch.
//
// The reference loaders run the transformers routers in torch in the timed path
// (src/kops/registry/gpt_oss_moe_experts.py:35, src/kops/registry/qwen3_next_moe_experts.py:28),
// then cast indices to int32 and scores to fp32 (:25-26 of the cohere2 loader). The
// routers (transformers 5.5.0):
//   gpt-oss  models/gpt_oss/modeling_gpt_oss.py:117-131: logits = x W^T + b (bf16);
//            top-k of the logits; softmax over the k values in the logits' dtype (bf16)
//   qwen3    models/qwen3_next/modeling_qwen3_next.py:761-780: softmax over all experts in
//            fp32; top-k of the probabilities; optional renormalisation to sum 1
// After the logits GEMM (kept in cuBLAS via torch), everything else — selection, softmax,
// renormalisation and the dtype casts — is this one kernel. One warp per token; lane l
// holds logits l, l+32, ...; k rounds of warp arg-max (ties: lower expert id).
#include "moe_internal.h"

namespace cernels {
namespace {

constexpr int kRouterWarps = 8;
constexpr int kMaxPerLane = 32;  // E <= 1024

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T, int kPerLane>
__global__ void __launch_bounds__(kRouterWarps * 32) router_topk_kernel(const T* __restrict__ logits, int tokens,
                                                                        int experts, int topk, int mode, int renorm,
                                                                        int shared_gate,
                                                                        int32_t* __restrict__ indices,
                                                                        float* __restrict__ weights) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kRouterWarps + warp;
  if (t >= tokens) return;
  // With a shared-gate column, logits rows hold experts + 1 values (the last is the gate),
  // padded to a multiple of 8 columns (16-byte rows for the router GEMM).
  const int row_stride = shared_gate ? ((experts + 1 + 7) / 8) * 8 : experts;
  const T* row = logits + static_cast<size_t>(t) * row_stride;
  const int out_stride = topk + shared_gate;
  float v[kPerLane];
#pragma unroll
  for (int j = 0; j < kPerLane; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < experts ? to_f32(row[e]) : -INFINITY;
  }
  float row_max = -INFINITY, row_sum = 0.f;
  if (mode == 1) {  // softmax over all experts (fp32)
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) row_max = fmaxf(row_max, v[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) row_max = fmaxf(row_max, __shfl_xor_sync(0xffffffffu, row_max, o));
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) row_sum += (lane + 32 * j < experts) ? __expf(v[j] - row_max) : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) row_sum += __shfl_xor_sync(0xffffffffu, row_sum, o);
  }
  float sel_v = 0.f;  // lane j < topk keeps the j-th selected value
  int sel_e = 0;
  for (int r = 0; r < topk; ++r) {
    float best = -INFINITY;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int e = lane + 32 * j;
      if (e < experts && (v[j] > best || (v[j] == best && e < best_e))) {
        best = v[j];
        best_e = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    if (lane == r) {
      sel_v = best;
      sel_e = best_e;
    }
    if ((best_e & 31) == lane) {  // owner removes it
#pragma unroll
      for (int j = 0; j < kPerLane; ++j)
        if (lane + 32 * j == best_e) v[j] = -INFINITY;
    }
  }
  float w;
  if (mode == 0) {
    // softmax over the k selected logits, result rounded to bf16 (the logits' dtype)
    const float m = __shfl_sync(0xffffffffu, sel_v, 0);  // selection is descending
    float ex = lane < topk ? __expf(sel_v - m) : 0.f;
    float s = ex;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    w = __bfloat162float(__float2bfloat16_rn(ex / s));
  } else {
    float p = lane < topk ? __expf(sel_v - row_max) / row_sum : 0.f;
    if (renorm) {
      float s = p;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      p = p / s;
    }
    w = p;
  }
  if (lane < topk) {
    indices[static_cast<size_t>(t) * out_stride + lane] = sel_e;
    weights[static_cast<size_t>(t) * out_stride + lane] = w;
  }
  if (shared_gate && lane == 0) {  // always-on shared expert: id `experts`, weight sigmoid(gate)
    const float gl = to_f32(row[experts]);
    indices[static_cast<size_t>(t) * out_stride + topk] = experts;
    weights[static_cast<size_t>(t) * out_stride + topk] = 1.0f / (1.0f + __expf(-gl));
  }
}

template <typename T>
cudaError_t launch_t(const void* logits, int tokens, int experts, int topk, int mode, int renorm, int shared,
                     int32_t* idx, float* w, cudaStream_t stream) {
  const int blocks = (tokens + kRouterWarps - 1) / kRouterWarps;
  const T* l = static_cast<const T*>(logits);
  if (experts <= 64)
    router_topk_kernel<T, 2><<<blocks, kRouterWarps * 32, 0, stream>>>(l, tokens, experts, topk, mode, renorm, shared, idx, w);
  else if (experts <= 256)
    router_topk_kernel<T, 8><<<blocks, kRouterWarps * 32, 0, stream>>>(l, tokens, experts, topk, mode, renorm, shared, idx, w);
  else
    router_topk_kernel<T, kMaxPerLane><<<blocks, kRouterWarps * 32, 0, stream>>>(l, tokens, experts, topk, mode,
                                                                                 renorm, shared, idx, w);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_router_topk(const void* logits, int bf16, int tokens, int experts, int topk, int mode, int renorm,
                               int shared_gate, int32_t* idx, float* w, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  const int sg = shared_gate ? 1 : 0;
  return bf16 ? launch_t<__nv_bfloat16>(logits, tokens, experts, topk, mode, renorm, sg, idx, w, stream)
              : launch_t<float>(logits, tokens, experts, topk, mode, renorm, sg, idx, w, stream);
}

}  // namespace cernels
