// Decode path: fused gather-GEMV for a handful of tokens.
//
// Reference: cohere2_moe_experts_decode
// (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:106-236) launches one CTA per
// (token, slot) pair and output tile, so an expert chosen by several tokens is streamed
// from HBM once per pair, and it accumulates the output with fp32 atomics.
//
// Here each CTA owns (unique expert g, output block). Every CTA rebuilds the grouping of
// the T*topk (token, slot) pairs by expert in shared memory from `indices` (a bitmap of
// touched experts; group g = g-th smallest touched expert id; pairs of a group in flat
// order), so no routing launch is needed and each touched expert's weights are read once
// for all of its tokens.
//   decode_gate_up_*  : glu[pair, f]  (fp32) = act(x[t] . W1[e] gate/up rows or columns)
//   decode_down_*     : partial[pair, h] (fp32) = glu[pair] . W2[e] (+ b2)
//                       the last CTA to finish an h-block (arrival counter) sums the
//                       topk partials of every token in slot order and writes bf16 out.
// LINEAR weights ([E,2F,H], [E,H,F]) are K-contiguous: one warp per output row pair,
// 16-byte loads along K and a warp-shuffle reduction. GPTOSS weights ([E,H,2F], [E,F,H])
// are N-contiguous: each lane owns 8 adjacent output columns, warps split K and reduce
// through shared memory.
#include "moe_internal.h"

namespace cernels {
namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kTokBatch = 8;          // tokens of one group processed per weight pass
constexpr int kRowsPerWarp = 2;       // LINEAR: output rows per warp
constexpr int kRowsPerCta = kDecWarps * kRowsPerWarp;  // 16
constexpr int kColsPerCta = 256;      // GPTOSS: output columns per CTA (32 lanes x 8)
constexpr float kLimit = 7.0f;
constexpr float kAlpha = 1.702f;

struct Grouping {
  int expert;     // expert id of this CTA's group (-1: no such group)
  int n_groups;   // number of touched experts
  int n_pairs;    // pairs of this group
};

// Builds, in shared memory, the list of flat pair indices routed to the g-th smallest
// touched expert. `bitmap` needs (experts + 31) / 32 words; `list` up to `total` ints.
__device__ Grouping build_group(const int32_t* __restrict__ indices, int total, int experts, int g,
                                unsigned* bitmap, int* list, int* scratch) {
  const int words = (experts + 31) >> 5;
  for (int w = threadIdx.x; w < words; w += blockDim.x) bitmap[w] = 0u;
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int e = indices[i];
    if (e >= 0 && e < experts) atomicOr(&bitmap[e >> 5], 1u << (e & 31));
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // Warp 0: find the g-th set bit and the group count.
    const int lane = threadIdx.x;
    int seen = 0;
    int found = -1;
    for (int w0 = 0; w0 < words; w0 += 32) {
      const int w = w0 + lane;
      const unsigned bits = w < words ? bitmap[w] : 0u;
      const int c = __popc(bits);
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const int excl = seen + incl - c;
      if (found < 0 && g >= excl && g < excl + c) {
        unsigned b = bits;
        for (int r = g - excl; r > 0; --r) b &= b - 1u;
        found = w * 32 + (__ffs(b) - 1);
      }
      seen += __shfl_sync(0xffffffffu, incl, 31);
    }
    // Broadcast the (unique) finder's result.
    const unsigned who = __ballot_sync(0xffffffffu, found >= 0);
    const int expert = who ? __shfl_sync(0xffffffffu, found, __ffs(who) - 1) : -1;
    // Pairs of that expert, flat order.
    int cnt = 0;
    if (expert >= 0) {
      for (int b = 0; b < total; b += 32) {
        const int i = b + lane;
        const bool hit = i < total && indices[i] == expert;
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        if (hit) list[cnt + __popc(m & ((1u << lane) - 1u))] = i;
        cnt += __popc(m);
      }
    }
    if (lane == 0) {
      scratch[0] = expert;
      scratch[1] = seen;
      scratch[2] = cnt;
    }
  }
  __syncthreads();
  Grouping gr;
  gr.expert = scratch[0];
  gr.n_groups = scratch[1];
  gr.n_pairs = scratch[2];
  return gr;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __bfloat1622float2(h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float act_linear(float g, float u) { return g / (1.0f + __expf(-g)) * u; }
__device__ __forceinline__ float act_gptoss(float g, float u) {
  g = fminf(g, kLimit);
  u = fmaxf(-kLimit, fminf(u, kLimit));
  return (u + 1.0f) * (g / (1.0f + __expf(-g * kAlpha)));
}

// Shared-memory layout common to all decode kernels:
//   bitmap [kMaxExperts/32] | list [kDecodeMaxPairs] | scratch [4] | operand rows...
constexpr int kBitmapWords = kMaxExperts / 32;
constexpr size_t kHeaderBytes = (kBitmapWords + kDecodeMaxPairs + 4) * sizeof(int);

// ---------------------------------------------------------------- LINEAR gate/up
__global__ void __launch_bounds__(kDecThreads) decode_gate_up_linear(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w1, const int32_t* __restrict__ indices,
    int total, int topk, int experts, int H, int F, float* __restrict__ glu, int* __restrict__ counters,
    int n_counters) {
  extern __shared__ __align__(16) int dsm[];
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm);
  int* list = dsm + kBitmapWords;
  int* scratch = list + kDecodeMaxPairs;
  uint4* xs = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(dsm) + kHeaderBytes);  // [kTokBatch, H/8]

  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0;

  const Grouping gr = build_group(indices, total, experts, blockIdx.y, bitmap, list, scratch);
  if (gr.expert < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hv = H / 8;
  const int f0 = blockIdx.x * kRowsPerCta + warp * kRowsPerWarp;
  const uint4* wg = reinterpret_cast<const uint4*>(w1 + (static_cast<size_t>(gr.expert) * 2 * F) * H);

  for (int p0 = 0; p0 < gr.n_pairs; p0 += kTokBatch) {
    const int nb = min(kTokBatch, gr.n_pairs - p0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * hv; i += blockDim.x) {
      const int r = i / hv, v = i - r * hv;
      const int t = list[p0 + r] / topk;
      xs[r * hv + v] = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H)[v];
    }
    __syncthreads();
    float acc[2 * kRowsPerWarp][kTokBatch];
#pragma unroll
    for (int r = 0; r < 2 * kRowsPerWarp; ++r)
#pragma unroll
      for (int b = 0; b < kTokBatch; ++b) acc[r][b] = 0.f;
    // rows: gate f0, f0+1, up F+f0, F+f0+1 (clamped to valid rows)
    size_t row_off[2 * kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const int f = min(f0 + r, F - 1);
      row_off[r] = static_cast<size_t>(f) * hv;
      row_off[kRowsPerWarp + r] = static_cast<size_t>(F + f) * hv;
    }
#pragma unroll 2
    for (int v = lane; v < hv; v += 32) {
      uint4 wv[2 * kRowsPerWarp];
#pragma unroll
      for (int r = 0; r < 2 * kRowsPerWarp; ++r) wv[r] = __ldg(wg + row_off[r] + v);
      float wf[2 * kRowsPerWarp][8];
#pragma unroll
      for (int r = 0; r < 2 * kRowsPerWarp; ++r) bf16x8_to_f32(wv[r], wf[r]);
#pragma unroll
      for (int b = 0; b < kTokBatch; ++b) {
        if (b < nb) {
          float xf[8];
          bf16x8_to_f32(xs[b * hv + v], xf);
#pragma unroll
          for (int r = 0; r < 2 * kRowsPerWarp; ++r)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[r][b] = fmaf(wf[r][i], xf[i], acc[r][b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < kTokBatch; ++b) {
      if (b < nb) {
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          const float g = warp_sum(acc[r][b]);
          const float u = warp_sum(acc[kRowsPerWarp + r][b]);
          const int f = f0 + r;
          if (lane == 0 && f < F) glu[static_cast<size_t>(list[p0 + b]) * F + f] = act_linear(g, u);
        }
      }
    }
  }
}

// Last-arriving CTA of an output block combines the partial rows of every token.
__device__ void finish_block(const float* __restrict__ partial, const int32_t* __restrict__ indices,
                             const float* __restrict__ weights, int tokens, int topk, int experts, int H, int c0,
                             int c1, int n_groups, int* __restrict__ counters, __nv_bfloat16* __restrict__ out,
                             int* flag) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&counters[blockIdx.x], 1);
    *flag = prev == n_groups - 1;
  }
  __syncthreads();
  if (!*flag) return;
  __threadfence();
  const int width = c1 - c0;
  for (int i = threadIdx.x; i < tokens * width; i += blockDim.x) {
    const int t = i / width, c = c0 + (i - t * width);
    float s = 0.f;
    for (int j = 0; j < topk; ++j) {
      const int p = t * topk + j;
      const int e = indices[p];
      if (e < 0 || e >= experts) continue;
      s = fmaf(weights[p], __ldcg(partial + static_cast<size_t>(p) * H + c), s);
    }
    out[static_cast<size_t>(t) * H + c] = __float2bfloat16_rn(s);
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0;
}

// Tokens whose every slot is skipped, or calls with no valid slot at all, still need
// zero rows: CTA row 0 writes zeros when there is no group.
__device__ void zero_block_if_empty(const Grouping& gr, int tokens, int H, int c0, int c1,
                                    __nv_bfloat16* __restrict__ out) {
  if (gr.n_groups != 0 || blockIdx.y != 0) return;
  const int width = c1 - c0;
  for (int i = threadIdx.x; i < tokens * width; i += blockDim.x) {
    const int t = i / width, c = c0 + (i - t * width);
    out[static_cast<size_t>(t) * H + c] = __float2bfloat16_rn(0.f);
  }
}

// ---------------------------------------------------------------- LINEAR down
__global__ void __launch_bounds__(kDecThreads) decode_down_linear(
    const float* __restrict__ glu, const __nv_bfloat16* __restrict__ w2, const int32_t* __restrict__ indices,
    const float* __restrict__ weights, int tokens, int topk, int experts, int H, int F, float* __restrict__ partial,
    int* __restrict__ counters, __nv_bfloat16* __restrict__ out) {
  extern __shared__ __align__(16) int dsm[];
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm);
  int* list = dsm + kBitmapWords;
  int* scratch = list + kDecodeMaxPairs;
  float4* gs = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(dsm) + kHeaderBytes);  // [kTokBatch, F/4]
  const int total = tokens * topk;
  const Grouping gr = build_group(indices, total, experts, blockIdx.y, bitmap, list, scratch);
  const int c0 = blockIdx.x * kRowsPerCta, c1 = min(H, c0 + kRowsPerCta);
  zero_block_if_empty(gr, tokens, H, c0, c1, out);
  if (gr.expert < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int fv = F / 8;  // 16-byte weight vectors per row
  const int h0 = c0 + warp * kRowsPerWarp;
  const uint4* wd = reinterpret_cast<const uint4*>(w2 + static_cast<size_t>(gr.expert) * H * F);
  size_t row_off[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) row_off[r] = static_cast<size_t>(min(h0 + r, H - 1)) * fv;

  for (int p0 = 0; p0 < gr.n_pairs; p0 += kTokBatch) {
    const int nb = min(kTokBatch, gr.n_pairs - p0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * (F / 4); i += blockDim.x) {
      const int r = i / (F / 4), v = i - r * (F / 4);
      gs[r * (F / 4) + v] = reinterpret_cast<const float4*>(glu + static_cast<size_t>(list[p0 + r]) * F)[v];
    }
    __syncthreads();
    float acc[kRowsPerWarp][kTokBatch];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
      for (int b = 0; b < kTokBatch; ++b) acc[r][b] = 0.f;
#pragma unroll 2
    for (int v = lane; v < fv; v += 32) {
      float wf[kRowsPerWarp][8];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) bf16x8_to_f32(__ldg(wd + row_off[r] + v), wf[r]);
#pragma unroll
      for (int b = 0; b < kTokBatch; ++b) {
        if (b < nb) {
          const float4 ga = gs[b * (F / 4) + 2 * v];
          const float4 gb = gs[b * (F / 4) + 2 * v + 1];
          const float gf[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
          for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[r][b] = fmaf(wf[r][i], gf[i], acc[r][b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < kTokBatch; ++b) {
      if (b < nb) {
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          const float s = warp_sum(acc[r][b]);
          if (lane == 0 && h0 + r < H) partial[static_cast<size_t>(list[p0 + b]) * H + h0 + r] = s;
        }
      }
    }
  }
  finish_block(partial, indices, weights, tokens, topk, experts, H, c0, c1, gr.n_groups, counters, out,
               scratch + 3);
}

// ---------------------------------------------------------------- GPTOSS gate/up
// W1[e] is [H, 2F] (columns interleaved gate/up). CTA covers 256 weight columns
// (128 glu columns); lane owns 8 adjacent columns; warps split the H rows.
__global__ void __launch_bounds__(kDecThreads) decode_gate_up_gptoss(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w1, const float* __restrict__ b1,
    const int32_t* __restrict__ indices, int total, int topk, int experts, int H, int F, float* __restrict__ glu,
    int* __restrict__ counters, int n_counters) {
  extern __shared__ __align__(16) int dsm[];
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm);
  int* list = dsm + kBitmapWords;
  int* scratch = list + kDecodeMaxPairs;
  float* xs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(dsm) + kHeaderBytes);  // [kTokBatch, H]
  float* red = xs + kTokBatch * H;  // [kDecWarps, kColsPerCta]

  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0;
  const Grouping gr = build_group(indices, total, experts, blockIdx.y, bitmap, list, scratch);
  if (gr.expert < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int two_f = 2 * F;
  const int col = blockIdx.x * kColsPerCta + lane * 8;  // first of this lane's 8 columns
  const bool col_ok = col < two_f;
  const __nv_bfloat16* wbase = w1 + static_cast<size_t>(gr.expert) * H * two_f;

  for (int p0 = 0; p0 < gr.n_pairs; p0 += kTokBatch) {
    const int nb = min(kTokBatch, gr.n_pairs - p0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * H; i += blockDim.x) {
      const int r = i / H, k = i - r * H;
      xs[r * H + k] = __bfloat162float(x[static_cast<size_t>(list[p0 + r] / topk) * H + k]);
    }
    __syncthreads();
    float acc[kTokBatch][8];
#pragma unroll
    for (int b = 0; b < kTokBatch; ++b)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[b][i] = 0.f;
    if (col_ok) {
#pragma unroll 4
      for (int k = warp; k < H; k += kDecWarps) {
        float wf[8];
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(wbase + static_cast<size_t>(k) * two_f + col)), wf);
#pragma unroll
        for (int b = 0; b < kTokBatch; ++b) {
          if (b < nb) {
            const float xv = xs[b * H + k];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[b][i] = fmaf(wf[i], xv, acc[b][i]);
          }
        }
      }
    }
    for (int b = 0; b < nb; ++b) {
#pragma unroll
      for (int i = 0; i < 8; ++i) red[warp * kColsPerCta + lane * 8 + i] = acc[b][i];
      __syncthreads();
      // 128 glu outputs per CTA: thread i < 128 reduces the (gate, up) column pair i.
      if (threadIdx.x < kColsPerCta / 2) {
        const int c = 2 * threadIdx.x;
        const int wc = blockIdx.x * kColsPerCta + c;
        if (wc < two_f) {
          float g = 0.f, u = 0.f;
#pragma unroll
          for (int w = 0; w < kDecWarps; ++w) {
            g += red[w * kColsPerCta + c];
            u += red[w * kColsPerCta + c + 1];
          }
          if (b1) {
            g += b1[static_cast<size_t>(gr.expert) * two_f + wc];
            u += b1[static_cast<size_t>(gr.expert) * two_f + wc + 1];
          }
          glu[static_cast<size_t>(list[p0 + b]) * F + wc / 2] = act_gptoss(g, u);
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------- GPTOSS down
// W2[e] is [F, H]. CTA covers 256 output columns; warps split the F rows.
__global__ void __launch_bounds__(kDecThreads) decode_down_gptoss(
    const float* __restrict__ glu, const __nv_bfloat16* __restrict__ w2, const float* __restrict__ b2,
    const int32_t* __restrict__ indices, const float* __restrict__ weights, int tokens, int topk, int experts, int H,
    int F, float* __restrict__ partial, int* __restrict__ counters, __nv_bfloat16* __restrict__ out) {
  extern __shared__ __align__(16) int dsm[];
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm);
  int* list = dsm + kBitmapWords;
  int* scratch = list + kDecodeMaxPairs;
  float* gs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(dsm) + kHeaderBytes);  // [kTokBatch, F]
  float* red = gs + kTokBatch * F;  // [kDecWarps, kColsPerCta]
  const int total = tokens * topk;
  const Grouping gr = build_group(indices, total, experts, blockIdx.y, bitmap, list, scratch);
  const int c0 = blockIdx.x * kColsPerCta, c1 = min(H, c0 + kColsPerCta);
  zero_block_if_empty(gr, tokens, H, c0, c1, out);
  if (gr.expert < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = c0 + lane * 8;
  const bool col_ok = col < H;
  const __nv_bfloat16* wbase = w2 + static_cast<size_t>(gr.expert) * F * H;

  for (int p0 = 0; p0 < gr.n_pairs; p0 += kTokBatch) {
    const int nb = min(kTokBatch, gr.n_pairs - p0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * F; i += blockDim.x) {
      const int r = i / F, k = i - r * F;
      gs[r * F + k] = glu[static_cast<size_t>(list[p0 + r]) * F + k];
    }
    __syncthreads();
    float acc[kTokBatch][8];
#pragma unroll
    for (int b = 0; b < kTokBatch; ++b)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[b][i] = 0.f;
    if (col_ok) {
#pragma unroll 4
      for (int k = warp; k < F; k += kDecWarps) {
        float wf[8];
        bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(wbase + static_cast<size_t>(k) * H + col)), wf);
#pragma unroll
        for (int b = 0; b < kTokBatch; ++b) {
          if (b < nb) {
            const float gv = gs[b * F + k];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[b][i] = fmaf(wf[i], gv, acc[b][i]);
          }
        }
      }
    }
    for (int b = 0; b < nb; ++b) {
#pragma unroll
      for (int i = 0; i < 8; ++i) red[warp * kColsPerCta + lane * 8 + i] = acc[b][i];
      __syncthreads();
      const int c = c0 + threadIdx.x;
      if (threadIdx.x < kColsPerCta && c < H) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) s += red[w * kColsPerCta + threadIdx.x];
        if (b2) s += b2[static_cast<size_t>(gr.expert) * H + c];
        partial[static_cast<size_t>(list[p0 + b]) * H + c] = s;
      }
      __syncthreads();
    }
  }
  finish_block(partial, indices, weights, tokens, topk, experts, H, c0, c1, gr.n_groups, counters, out,
               scratch + 3);
}

}  // namespace

cudaError_t launch_decode(const DecodeArgs& a, const DecodeWorkspace& ws, cudaStream_t stream) {
  const int total = a.tokens * a.topk;
  if (a.tokens <= 0) return cudaSuccess;
  const int max_groups = total < a.experts ? total : a.experts;
  const int H = a.hidden, F = a.inter;
  cudaError_t err;
  if (a.layout == CERNELS_LAYOUT_LINEAR) {
    const size_t smem1 = kHeaderBytes + static_cast<size_t>(kTokBatch) * H * 2;
    const size_t smem2 = kHeaderBytes + static_cast<size_t>(kTokBatch) * F * 4;
    const int n_hblocks = (H + kRowsPerCta - 1) / kRowsPerCta;
    if ((err = cudaFuncSetAttribute(decode_gate_up_linear, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem1))) != cudaSuccess)
      return err;
    if ((err = cudaFuncSetAttribute(decode_down_linear, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem2))) != cudaSuccess)
      return err;
    dim3 g1((F + kRowsPerCta - 1) / kRowsPerCta, max_groups);
    decode_gate_up_linear<<<g1, kDecThreads, smem1, stream>>>(a.x, a.w1, a.indices, total, a.topk, a.experts, H, F,
                                                              ws.glu, ws.counters, n_hblocks);
    dim3 g2(n_hblocks, max_groups);
    decode_down_linear<<<g2, kDecThreads, smem2, stream>>>(ws.glu, a.w2, a.indices, a.weights, a.tokens, a.topk,
                                                           a.experts, H, F, ws.partial, ws.counters, a.out);
  } else {
    const size_t smem1 = kHeaderBytes + (static_cast<size_t>(kTokBatch) * H + kDecWarps * kColsPerCta) * 4;
    const size_t smem2 = kHeaderBytes + (static_cast<size_t>(kTokBatch) * F + kDecWarps * kColsPerCta) * 4;
    const int n_hblocks = (H + kColsPerCta - 1) / kColsPerCta;
    if ((err = cudaFuncSetAttribute(decode_gate_up_gptoss, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem1))) != cudaSuccess)
      return err;
    if ((err = cudaFuncSetAttribute(decode_down_gptoss, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem2))) != cudaSuccess)
      return err;
    dim3 g1((2 * F + kColsPerCta - 1) / kColsPerCta, max_groups);
    decode_gate_up_gptoss<<<g1, kDecThreads, smem1, stream>>>(a.x, a.w1, a.b1, a.indices, total, a.topk, a.experts,
                                                              H, F, ws.glu, ws.counters, n_hblocks);
    dim3 g2(n_hblocks, max_groups);
    decode_down_gptoss<<<g2, kDecThreads, smem2, stream>>>(ws.glu, a.w2, a.b2, a.indices, a.weights, a.tokens,
                                                           a.topk, a.experts, H, F, ws.partial, ws.counters, a.out);
  }
  return cudaGetLastError();
}

size_t decode_counter_count(int hidden) { return static_cast<size_t>(hidden / 16 + 1); }

}  // namespace cernels
