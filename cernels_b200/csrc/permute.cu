// Row gather into routed order and the weighted, deterministic un-permute/combine.
//
// Reference: gather_kernel (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:58-65)
// copies one bf16 per thread; scatter_add_f32_kernel (:85-94, gpt-oss variant adds the
// down bias first, src/kops/gpt_oss_moe_experts/csrc/gpt_oss_moe_experts.cu:104-117)
// accumulates with fp32 atomics into a [T, H] fp32 buffer that is then cast to bf16.
// Here both are HBM-streaming kernels with one warp per row and 16-byte accesses; the
// combine gathers the topk rows of a token through the inverse permutation and sums
// them in fixed slot order, so the result does not depend on scheduling.
#include "moe_internal.h"

namespace cernels {
namespace {

constexpr int kRowThreads = 256;
constexpr int kRowsPerBlock = kRowThreads / 32;

__global__ void __launch_bounds__(kRowThreads) gather_rows_kernel(const uint4* __restrict__ x,
                                                                  const int* __restrict__ perm_token, int rows,
                                                                  const int* __restrict__ row_count,
                                                                  int vec_per_row, uint4* __restrict__ out) {
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  if (row_count && row >= *row_count) return;  // rows of skipped (invalid-id) entries
  const int lane = threadIdx.x & 31;
  const int t = perm_token[row];
  const uint4* src = x + static_cast<size_t>(t) * vec_per_row;
  uint4* dst = out + static_cast<size_t>(row) * vec_per_row;
  // up to 8 loads per lane in flight before their stores
  for (int v0 = 0; v0 < vec_per_row; v0 += 32 * 8) {
    uint4 r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int v = v0 + j * 32 + lane;
      if (v < vec_per_row) r[j] = src[v];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int v = v0 + j * 32 + lane;
      if (v < vec_per_row) dst[v] = r[j];
    }
  }
}

__device__ __forceinline__ void accumulate_bf16x8(float (&acc)[8], const uint4& v, float w) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    acc[2 * i] = fmaf(w, f.x, acc[2 * i]);
    acc[2 * i + 1] = fmaf(w, f.y, acc[2 * i + 1]);
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&acc)[8]) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
  return r;
}

// One warp per token; each lane owns 8 consecutive columns per step.
template <int kMaxTopk>
__global__ void __launch_bounds__(kRowThreads) combine_kernel(const uint4* __restrict__ rows,
                                                              const int* __restrict__ inv,
                                                              const float* __restrict__ weights, int tokens,
                                                              int topk, int vec_per_row, uint4* __restrict__ out) {
  const int t = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const int lane = threadIdx.x & 31;
  int src[kMaxTopk];
  float w[kMaxTopk];
#pragma unroll
  for (int j = 0; j < kMaxTopk; ++j) {
    src[j] = j < topk ? inv[static_cast<size_t>(t) * topk + j] : -1;
    w[j] = j < topk ? weights[static_cast<size_t>(t) * topk + j] : 0.f;
  }
  for (int v = lane; v < vec_per_row; v += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    uint4 vals[kMaxTopk];
#pragma unroll
    for (int j = 0; j < kMaxTopk; ++j)
      if (src[j] >= 0) vals[j] = rows[static_cast<size_t>(src[j]) * vec_per_row + v];
#pragma unroll
    for (int j = 0; j < kMaxTopk; ++j)
      if (src[j] >= 0) accumulate_bf16x8(acc, vals[j], w[j]);
    out[static_cast<size_t>(t) * vec_per_row + v] = pack_bf16x8(acc);
  }
}

// Generic-topk variant (loop, no unrolled register arrays).
__global__ void __launch_bounds__(kRowThreads) combine_kernel_any(const uint4* __restrict__ rows,
                                                                  const int* __restrict__ inv,
                                                                  const float* __restrict__ weights, int tokens,
                                                                  int topk, int vec_per_row,
                                                                  uint4* __restrict__ out) {
  const int t = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const int lane = threadIdx.x & 31;
  for (int v = lane; v < vec_per_row; v += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < topk; ++j) {
      const int s = inv[static_cast<size_t>(t) * topk + j];
      if (s < 0) continue;
      accumulate_bf16x8(acc, rows[static_cast<size_t>(s) * vec_per_row + v],
                        weights[static_cast<size_t>(t) * topk + j]);
    }
    out[static_cast<size_t>(t) * vec_per_row + v] = pack_bf16x8(acc);
  }
}

}  // namespace

cudaError_t launch_gather(const __nv_bfloat16* x, const int* perm_token, int rows, const int* row_count,
                          int hidden, __nv_bfloat16* gathered, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  gather_rows_kernel<<<blocks, kRowThreads, 0, stream>>>(reinterpret_cast<const uint4*>(x), perm_token, rows,
                                                         row_count, hidden / 8, reinterpret_cast<uint4*>(gathered));
  return cudaGetLastError();
}

cudaError_t launch_combine(const __nv_bfloat16* down_out, const int* inv, const float* weights, int tokens,
                           int topk, int hidden, __nv_bfloat16* out, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  const int blocks = (tokens + kRowsPerBlock - 1) / kRowsPerBlock;
  const uint4* rows = reinterpret_cast<const uint4*>(down_out);
  uint4* o = reinterpret_cast<uint4*>(out);
  const int vec = hidden / 8;
  if (topk <= 4) {
    combine_kernel<4><<<blocks, kRowThreads, 0, stream>>>(rows, inv, weights, tokens, topk, vec, o);
  } else if (topk <= 8) {
    combine_kernel<8><<<blocks, kRowThreads, 0, stream>>>(rows, inv, weights, tokens, topk, vec, o);
  } else if (topk <= 12) {
    combine_kernel<12><<<blocks, kRowThreads, 0, stream>>>(rows, inv, weights, tokens, topk, vec, o);
  } else if (topk <= 16) {
    combine_kernel<16><<<blocks, kRowThreads, 0, stream>>>(rows, inv, weights, tokens, topk, vec, o);
  } else {
    combine_kernel_any<<<blocks, kRowThreads, 0, stream>>>(rows, inv, weights, tokens, topk, vec, o);
  }
  return cudaGetLastError();
}

}  // namespace cernels
