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
#include <algorithm>

#include "moe_internal.h"
#include "sm100_primitives.cuh"

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

__device__ __forceinline__ unsigned long long global_timer_ns_dec() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

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
// `partial` holds `splits` slabs of [total, H] (down-projection partial sums over disjoint
// K ranges); the last of `arrivals` CTAs of this output block sums, per output element,
// slot by slot and within a slot slab by slab, so the result does not depend on timing.
__device__ void finish_block(const float* __restrict__ partial, const int32_t* __restrict__ indices,
                             const float* __restrict__ weights, int tokens, int topk, int experts, int H, int c0,
                             int c1, int arrivals, int splits, int* __restrict__ counters,
                             __nv_bfloat16* __restrict__ out, int* flag) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&counters[blockIdx.x], 1);
    *flag = prev == arrivals - 1;
  }
  __syncthreads();
  if (!*flag) return;
  __threadfence();
  const int width = c1 - c0;
  const size_t slab = static_cast<size_t>(tokens) * topk * H;
  for (int i = threadIdx.x; i < tokens * width; i += blockDim.x) {
    const int t = i / width, c = c0 + (i - t * width);
    float s = 0.f;
    for (int j = 0; j < topk; ++j) {
      const int p = t * topk + j;
      const int e = indices[p];
      if (e < 0 || e >= experts) continue;
      const float* src = partial + static_cast<size_t>(p) * H + c;
      float v = __ldcg(src);
      for (int z = 1; z < splits; ++z) v += __ldcg(src + z * slab);
      s = fmaf(weights[p], v, s);
    }
    out[static_cast<size_t>(t) * H + c] = __float2bfloat16_rn(s);
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0;
}

// Tokens whose every slot is skipped, or calls with no valid slot at all, still need
// zero rows: CTA row 0 writes zeros when there is no group.
__device__ void zero_block_if_empty(const Grouping& gr, int tokens, int H, int c0, int c1,
                                    __nv_bfloat16* __restrict__ out) {
  if (gr.n_groups != 0 || blockIdx.y != 0 || blockIdx.z != 0) return;
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
  finish_block(partial, indices, weights, tokens, topk, experts, H, c0, c1, gr.n_groups, 1, counters, out,
               scratch + 3);
}

// Rows of one K split, rounded up to 4 floats so the reduction buffer after the operand
// rows stays 16-byte aligned.
__host__ __device__ inline int split_rows(int k, int splits) { return (((k + splits - 1) / splits) + 3) & ~3; }

// ---------------------------------------------------------------- GPTOSS gate/up
// W1[e] is [H, 2F] (columns interleaved gate/up). CTA (column block, group, K split)
// covers 256 weight columns (128 glu columns) over the rows [k0, k1) of its split; lane
// owns 8 adjacent columns; warps split the rows. Each warp issues kUnroll independent
// 16-byte loads before it consumes them, so a CTA keeps 8 x kUnroll x 512 B in flight.
// splits == 1: writes glu = act(sum + b1) directly. splits > 1: writes the raw split sums
// to pre[z, pair, 2F]; the down kernel adds them in split order, adds b1 and applies act.
template <int kTB>
__global__ void __launch_bounds__(kDecThreads) decode_gate_up_gptoss(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w1, const float* __restrict__ b1,
    const int32_t* __restrict__ indices, int total, int topk, int experts, int H, int F, int splits,
    float* __restrict__ glu, float* __restrict__ pre, int* __restrict__ counters, int n_counters) {
  constexpr int kUnroll = kTB == 8 ? 4 : 8;  // 8 tokens: 64 accumulators leave room for 4 loads
  extern __shared__ __align__(16) int dsm[];
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm);
  int* list = dsm + kBitmapWords;
  int* scratch = list + kDecodeMaxPairs;
  const int k0 = static_cast<int>((static_cast<long long>(H) * blockIdx.z) / splits);
  const int k1 = static_cast<int>((static_cast<long long>(H) * (blockIdx.z + 1)) / splits);
  const int kr = k1 - k0;
  float* xs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(dsm) + kHeaderBytes);  // [kTB, kr]
  float* red = xs + kTB * split_rows(H, splits);  // [kDecWarps, kColsPerCta]

  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
    for (int i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0;
  const Grouping gr = build_group(indices, total, experts, blockIdx.y, bitmap, list, scratch);
  if (gr.expert < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int two_f = 2 * F;
  const int col = blockIdx.x * kColsPerCta + lane * 8;  // first of this lane's 8 columns
  const bool col_ok = col < two_f;
  const __nv_bfloat16* wbase = w1 + static_cast<size_t>(gr.expert) * H * two_f + col;

  for (int p0 = 0; p0 < gr.n_pairs; p0 += kTB) {
    const int nb = min(kTB, gr.n_pairs - p0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * kr; i += blockDim.x) {
      const int r = i / kr, k = i - r * kr;
      xs[r * kr + k] = __bfloat162float(x[static_cast<size_t>(list[p0 + r] / topk) * H + k0 + k]);
    }
    __syncthreads();
    float acc[kTB][8];
#pragma unroll
    for (int b = 0; b < kTB; ++b)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[b][i] = 0.f;
    if (col_ok) {
      for (int kb = k0 + warp; kb < k1; kb += kDecWarps * kUnroll) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int k = kb + u * kDecWarps;
          v[u] = k < k1 ? __ldg(reinterpret_cast<const uint4*>(wbase + static_cast<size_t>(k) * two_f))
                        : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int k = kb + u * kDecWarps;
          if (k < k1) {
            float wf[8];
            bf16x8_to_f32(v[u], wf);
#pragma unroll
            for (int b = 0; b < kTB; ++b) {
              if (b < nb) {
                const float xv = xs[b * kr + (k - k0)];
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[b][i] = fmaf(wf[i], xv, acc[b][i]);
              }
            }
          }
        }
      }
    }
    for (int b = 0; b < nb; ++b) {
      float4* rw = reinterpret_cast<float4*>(red + warp * kColsPerCta + lane * 8);
      rw[0] = make_float4(acc[b][0], acc[b][1], acc[b][2], acc[b][3]);
      rw[1] = make_float4(acc[b][4], acc[b][5], acc[b][6], acc[b][7]);
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
          const int pair = list[p0 + b];
          if (splits == 1) {
            if (b1) {
              g += b1[static_cast<size_t>(gr.expert) * two_f + wc];
              u += b1[static_cast<size_t>(gr.expert) * two_f + wc + 1];
            }
            glu[static_cast<size_t>(pair) * F + wc / 2] = act_gptoss(g, u);
          } else {
            *reinterpret_cast<float2*>(pre + (static_cast<size_t>(blockIdx.z) * total + pair) * two_f + wc) =
                make_float2(g, u);
          }
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------- GPTOSS down
// W2[e] is [F, H]. CTA (column block, group, K split) covers 256 output columns over the
// rows [f0, f1) of its split; warps split the rows. Its glu operand is built in shared
// memory: glu[pair, f0:f1] (gate/up splits == 1) or act(sum_z pre[z, pair, 2f..2f+1] + b1)
// (gate/up splits > 1, summed in split order). Down partial sums go to
// partial[z, pair, H] (b2 added by split 0); the last of the n_groups x splits CTAs of a
// column block writes the combined bf16 rows.
template <int kTB>
__global__ void __launch_bounds__(kDecThreads) decode_down_gptoss(
    const float* __restrict__ glu, const float* __restrict__ pre, const float* __restrict__ b1, int pre_splits,
    const __nv_bfloat16* __restrict__ w2, const float* __restrict__ b2, const int32_t* __restrict__ indices,
    const float* __restrict__ weights, int tokens, int topk, int experts, int H, int F, int splits,
    float* __restrict__ partial, int* __restrict__ counters, __nv_bfloat16* __restrict__ out) {
  constexpr int kUnroll = kTB == 8 ? 4 : 8;  // 8 tokens: 64 accumulators leave room for 4 loads
  extern __shared__ __align__(16) int dsm[];
  unsigned* bitmap = reinterpret_cast<unsigned*>(dsm);
  int* list = dsm + kBitmapWords;
  int* scratch = list + kDecodeMaxPairs;
  const int f0 = static_cast<int>((static_cast<long long>(F) * blockIdx.z) / splits);
  const int f1 = static_cast<int>((static_cast<long long>(F) * (blockIdx.z + 1)) / splits);
  const int fr = f1 - f0;
  float* gs = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(dsm) + kHeaderBytes);  // [kTB, fr]
  float* red = gs + kTB * split_rows(F, splits);  // [kDecWarps, kColsPerCta]
  const int total = tokens * topk;
  const Grouping gr = build_group(indices, total, experts, blockIdx.y, bitmap, list, scratch);
  const int c0 = blockIdx.x * kColsPerCta, c1 = min(H, c0 + kColsPerCta);
  zero_block_if_empty(gr, tokens, H, c0, c1, out);
  if (gr.expert < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = c0 + lane * 8;
  const bool col_ok = col < H;
  const __nv_bfloat16* wbase = w2 + static_cast<size_t>(gr.expert) * F * H + col;
  const int two_f = 2 * F;

  for (int p0 = 0; p0 < gr.n_pairs; p0 += kTB) {
    const int nb = min(kTB, gr.n_pairs - p0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * fr; i += blockDim.x) {
      const int r = i / fr, f = f0 + (i - r * fr);
      const int pair = list[p0 + r];
      float v;
      if (pre_splits == 1) {
        v = glu[static_cast<size_t>(pair) * F + f];
      } else {
        const float* src = pre + static_cast<size_t>(pair) * two_f + 2 * f;
        float2 gu = __ldcg(reinterpret_cast<const float2*>(src));
        for (int z = 1; z < pre_splits; ++z) {
          const float2 t = __ldcg(reinterpret_cast<const float2*>(src + static_cast<size_t>(z) * total * two_f));
          gu.x += t.x;
          gu.y += t.y;
        }
        if (b1) {
          gu.x += b1[static_cast<size_t>(gr.expert) * two_f + 2 * f];
          gu.y += b1[static_cast<size_t>(gr.expert) * two_f + 2 * f + 1];
        }
        v = act_gptoss(gu.x, gu.y);
      }
      gs[r * fr + (f - f0)] = v;
    }
    __syncthreads();
    float acc[kTB][8];
#pragma unroll
    for (int b = 0; b < kTB; ++b)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[b][i] = 0.f;
    if (col_ok) {
      for (int kb = f0 + warp; kb < f1; kb += kDecWarps * kUnroll) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int k = kb + u * kDecWarps;
          v[u] = k < f1 ? __ldg(reinterpret_cast<const uint4*>(wbase + static_cast<size_t>(k) * H))
                        : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int k = kb + u * kDecWarps;
          if (k < f1) {
            float wf[8];
            bf16x8_to_f32(v[u], wf);
#pragma unroll
            for (int b = 0; b < kTB; ++b) {
              if (b < nb) {
                const float gv = gs[b * fr + (k - f0)];
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[b][i] = fmaf(wf[i], gv, acc[b][i]);
              }
            }
          }
        }
      }
    }
    for (int b = 0; b < nb; ++b) {
      float4* rw = reinterpret_cast<float4*>(red + warp * kColsPerCta + lane * 8);
      rw[0] = make_float4(acc[b][0], acc[b][1], acc[b][2], acc[b][3]);
      rw[1] = make_float4(acc[b][4], acc[b][5], acc[b][6], acc[b][7]);
      __syncthreads();
      const int c = c0 + threadIdx.x;
      if (threadIdx.x < kColsPerCta && c < H) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) s += red[w * kColsPerCta + threadIdx.x];
        if (b2 && blockIdx.z == 0) s += b2[static_cast<size_t>(gr.expert) * H + c];
        partial[(static_cast<size_t>(blockIdx.z) * total + list[p0 + b]) * H + c] = s;
      }
      __syncthreads();
    }
  }
  finish_block(partial, indices, weights, tokens, topk, experts, H, c0, c1, gr.n_groups * splits, splits, counters,
               out, scratch + 3);
}

// ---------------------------------------------------------------- grouping for the streaming kernel
// Every CTA of the streaming decode kernel builds the same grouping of the (token, slot)
// pairs by touched expert, in shared memory, at most kFusedMaxPairs pairs.
constexpr int kFusedMaxPairs = 256;

struct FusedGroups {
  int n_groups;
  int expert[kFusedMaxPairs];
  int start[kFusedMaxPairs + 1];
  int count[kFusedMaxPairs];
  int list[kFusedMaxPairs];
  int eidx[kFusedMaxPairs];
  int word_prefix[kBitmapWords];
  unsigned bitmap[kBitmapWords];
  int flag;
};

__device__ void build_groups_fused(const int32_t* __restrict__ indices, int total, int experts, FusedGroups& G) {
  const int words = (experts + 31) >> 5;
  for (int w = threadIdx.x; w < words; w += blockDim.x) G.bitmap[w] = 0u;
  for (int i = threadIdx.x; i < total; i += blockDim.x) G.count[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int e = indices[i];
    if (e >= 0 && e < experts) atomicOr(&G.bitmap[e >> 5], 1u << (e & 31));
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int carry = 0;
    for (int w0 = 0; w0 < words; w0 += 32) {
      const int w = w0 + lane;
      const int c = w < words ? __popc(G.bitmap[w]) : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (w < words) G.word_prefix[w] = carry + incl - c;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) G.n_groups = carry;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int e = indices[i];
    if (e < 0 || e >= experts) continue;
    const int g = G.word_prefix[e >> 5] + __popc(G.bitmap[e >> 5] & ((1u << (e & 31)) - 1u));
    G.expert[g] = e;
    atomicAdd(&G.count[g], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int g = 0; g < G.n_groups; ++g) {
      G.start[g] = acc;
      acc += G.count[g];
    }
    G.start[G.n_groups] = acc;
  }
  __syncthreads();
  // Pairs of a group in flat order. Every CTA must build the identical list: token batches
  // of one group are split across CTAs by position in this list.
  for (int i = threadIdx.x; i < total; i += blockDim.x) G.eidx[i] = indices[i];
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int e = G.eidx[i];
    if (e < 0 || e >= experts) continue;
    const int g = G.word_prefix[e >> 5] + __popc(G.bitmap[e >> 5] & ((1u << (e & 31)) - 1u));
    int before = 0;
    for (int j = 0; j < i; ++j) before += G.eidx[j] == e;
    G.list[G.start[g] + before] = i;
  }
  __syncthreads();
}

// Grid-wide barrier for a cooperative launch. bar[0] = arrivals, bar[1] = generation.
// Bounded: gives up after limit_ns, records `code` in *status and returns false.
__device__ bool grid_barrier_bounded(unsigned* bar, unsigned n_blocks, int* status, int code, int* flag,
                                     unsigned long long limit_ns) {
  __syncthreads();
  if (threadIdx.x == 0) {
    *flag = 1;
    volatile unsigned* vgen = bar + 1;
    const unsigned gen = *vgen;
    __threadfence();
    const unsigned arrived = atomicAdd(bar, 1u);
    if (arrived == n_blocks - 1) {
      atomicExch(bar, 0u);
      __threadfence();
      atomicAdd(bar + 1, 1u);
    } else {
      const unsigned long long t0 = global_timer_ns_dec();
      while (*vgen == gen) {
        if (global_timer_ns_dec() - t0 > limit_ns) {
          if (status) atomicCAS(status, 0, code);
          *flag = 0;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  return *flag != 0;
}

#ifndef CERNELS_STREAM_STAGES
#define CERNELS_STREAM_STAGES 3
#define CERNELS_STREAM_STAGE_KB 48
#endif
constexpr int kStreamStages = CERNELS_STREAM_STAGES;
constexpr int kStreamStageBytes = CERNELS_STREAM_STAGE_KB * 1024;
constexpr int kStreamConsumers = 8;
constexpr int kStreamThreads = (kStreamConsumers + 1) * 32;
constexpr int kStreamCThreads = kStreamConsumers * 32;  // consumer threads
constexpr int kStreamMaxR1 = 8;                          // gate/up pairs per stage
constexpr int kStreamMaxR2 = 16;                         // down rows per stage
constexpr int kStreamMaxPairs = 12;
constexpr size_t kL2PrefetchBudget = size_t(64) << 20;    // bytes of down rows prefetched into L2

#ifdef CERNELS_DECODE_TRACE
// Debug builds only: %globaltimer stamps at phase boundaries, per CTA (thread 0).
__device__ unsigned long long g_decode_trace[1024][8];
#define DECODE_TRACE(slot) \
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_decode_trace[blockIdx.x][slot] = global_timer_ns_dec();
#else
#define DECODE_TRACE(slot)
#endif

struct StreamPlan {
  int r1, nfr;  // phase 1: gate/up row pairs per stage, stages per (group, token batch)
  int r2, nhr;  // phase 2: down rows per stage, stages per (group, token batch)
};

__host__ __device__ inline StreamPlan make_stream_plan(int H, int F) {
  StreamPlan p;
  p.r1 = kStreamStageBytes / (4 * H);
  if (p.r1 > kStreamMaxR1) p.r1 = kStreamMaxR1;
  p.nfr = p.r1 > 0 ? (F + p.r1 - 1) / p.r1 : 0;
  p.r2 = kStreamStageBytes / (2 * F);
  if (p.r2 > kStreamMaxR2) p.r2 = kStreamMaxR2;
  p.nhr = p.r2 > 0 ? (H + p.r2 - 1) / p.r2 : 0;
  return p;
}

struct StreamShared {
  FusedGroups G;
  int batch_prefix[kFusedMaxPairs + 1];  // token batches (of <= kTokBatch) before group g
  uint64_t full[kStreamStages];
  uint64_t empty[kStreamStages];
  float red[kStreamConsumers][2 * kStreamMaxR1 > kStreamMaxR2 ? 2 * kStreamMaxR1 : kStreamMaxR2];
  int abort;
};

__device__ __forceinline__ int find_group(const int* prefix, int n_groups, int q) {
  int lo = 0, hi = n_groups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= q) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Consumer-warps-only barrier (named barrier 1; the producer warp does not take part).
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kStreamConsumers * 32) : "memory");
}


// Reduces 16 per-lane values over the warp with 16 shuffles (transposing butterfly).
// On return, v[0] of every even lane l holds the warp-wide sum of row
// 8*bit4(l) + 4*bit3(l) + 2*bit2(l) + bit1(l).
__device__ __forceinline__ void warp_reduce16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool hi = lane & 16;
    const float send = hi ? v[i] : v[i + 8];
    const float keep = hi ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool hi = lane & 8;
    const float send = hi ? v[i] : v[i + 4];
    const float keep = hi ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool hi = lane & 4;
    const float send = hi ? v[i] : v[i + 2];
    const float keep = hi ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool hi = lane & 2;
    const float send = hi ? v[0] : v[1];
    const float keep = hi ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
}

struct UnitCoord {
  int g, p0, nb, r0, rows;
};

__device__ __forceinline__ UnitCoord unit_coord(const StreamShared& S, int u, int per_batch, int rows_per_unit,
                                                int rows_total, int n_groups) {
  const FusedGroups& G = S.G;
  UnitCoord c;
  const int q = u / per_batch, r = u - q * per_batch;
  c.g = find_group(S.batch_prefix, n_groups, q);
  c.p0 = G.start[c.g] + (q - S.batch_prefix[c.g]) * kTokBatch;
  c.nb = min(kTokBatch, G.start[c.g + 1] - c.p0);
  c.r0 = r * rows_per_unit;
  c.rows = min(rows_per_unit, rows_total - c.r0);
  return c;
}

// Streaming LINEAR decode: one cooperative launch, one CTA per SM, 9 warps. Warp 8 (one
// lane) streams weight rows with cp.async.bulk into a ring of kStreamStages x
// kStreamStageBytes of shared memory (mbarrier completion); warps 0-7 compute from shared
// memory. Phase-1 units are grid-strided (all SMs sweep neighbouring rows together);
// each CTA owns a contiguous range of phase-2 units, so its glu batch rarely changes.
//   phase 1  units (group, token batch <= 8, r1 gate/up row pairs) -> glu[pair, f] fp32
//   barrier  (bounded, grid-wide); the producer has already queued its first phase-2
//            weight stages, which do not depend on phase 1
//            (and, when they fit in L2, has prefetched its share of them into L2)
//   phase 2  units (group, token batch, r2 down rows); the batch's fp32 glu rows sit in a
//            per-CTA buffer reloaded when the unit's (group, batch) changes -> partial[pair, h]
//   barrier  (bounded, grid-wide), then every CTA combines a share of the output rows:
//            out[t, h] = bf16(sum_j w[t, j] * partial[(t, j), h]) in slot order j
// Every stage is split over all 256 consumer threads by columns (each thread owns 16-byte
// vectors of every row in the stage), then reduced per row with shuffles + shared memory.
__global__ void __launch_bounds__(kStreamThreads, 1) decode_stream_linear(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w1, const __nv_bfloat16* __restrict__ w2,
    const int32_t* __restrict__ indices, const float* __restrict__ weights, int tokens, int topk, int experts, int H,
    int F, float* __restrict__ glu, float* __restrict__ partial, unsigned* __restrict__ barrier,
    int* __restrict__ status, __nv_bfloat16* __restrict__ out, unsigned long long wait_ns) {
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  StreamShared& S = *reinterpret_cast<StreamShared*>(dsm_raw);
  uint8_t* ring = dsm_raw + ((sizeof(StreamShared) + 127) & ~size_t(127));
  uint8_t* opnd = ring + kStreamStages * kStreamStageBytes;  // x rows (phase 1) / glu batch (phase 2)
  uint4* xs = reinterpret_cast<uint4*>(opnd);                 // [tokens, H/8] bf16
  float4* gls = reinterpret_cast<float4*>(opnd);              // [kTokBatch, F/4] fp32
  FusedGroups& G = S.G;
  const int total = tokens * topk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hv = H / 8, fv = F / 8;
  const StreamPlan plan = make_stream_plan(H, F);
  volatile int* abort_flag = &S.abort;
  DECODE_TRACE(0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStreamStages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], kStreamConsumers);
    }
    S.abort = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < tokens * hv; i += blockDim.x) xs[i] = reinterpret_cast<const uint4*>(x)[i];
  build_groups_fused(indices, total, experts, G);  // ends with __syncthreads
  const int n_groups = G.n_groups;
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int g = 0; g < n_groups; ++g) {
      S.batch_prefix[g] = acc;
      acc += (G.start[g + 1] - G.start[g] + kTokBatch - 1) / kTokBatch;
    }
    S.batch_prefix[n_groups] = acc;
  }
  __syncthreads();
  DECODE_TRACE(1);
  const int n_batches = S.batch_prefix[n_groups];
  const int units1 = n_batches * plan.nfr, units2 = n_batches * plan.nhr;
  // contiguous unit ranges per CTA
  const int u2_begin = static_cast<int>((static_cast<long long>(units2) * blockIdx.x) / gridDim.x);
  const int u2_end = static_cast<int>((static_cast<long long>(units2) * (blockIdx.x + 1)) / gridDim.x);
  int stage = 0;
  uint32_t phase = 0;
  long long issued = 0;  // producer: stages loaded so far
  auto advance = [&]() {
    ++issued;
    if (++stage == kStreamStages) {
      stage = 0;
      phase ^= 1u;
    }
  };
  // Producer, when giving up: wait (bounded) for the copies still in flight (at most the
  // last kStreamStages stages) so none lands in shared memory after the CTA exits.
  auto drain = [&]() {
    for (long long i = issued > kStreamStages ? issued - kStreamStages : 0; i < issued; ++i)
      mbar_drain(&S.full[i % kStreamStages], static_cast<uint32_t>((i / kStreamStages) & 1), wait_ns);
  };
  const size_t row1 = static_cast<size_t>(H) * 2;  // bytes of one gate/up row
  const size_t row2 = static_cast<size_t>(F) * 2;  // bytes of one down row
  bool ok = true;

  if (warp == kStreamConsumers) {
    // ------------------------------------------------------------ producer
    int prefetched = 0;
    if (lane == 0) {
      // When this launch's down-projection rows fit comfortably in L2, prefetch this CTA's
      // share into L2 while phase 1 streams, so HBM stays busy across the grid barrier.
      const bool prefetch = static_cast<size_t>(units2) * plan.r2 * row2 <= kL2PrefetchBudget;
      const int n1 = (units1 - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
      const int n2 = u2_end - u2_begin;
      int i1 = 0, pf = u2_begin + kStreamStages;  // the first stages are loaded into smem directly
      for (int u = blockIdx.x; u < units1 && ok; u += gridDim.x, ++i1) {
        if (prefetch && n1 > 0) {
          const int pf_end = u2_begin + static_cast<int>((static_cast<long long>(n2) * (i1 + 1)) / n1);
          for (; pf < pf_end; ++pf) {
            const UnitCoord c2 = unit_coord(S, pf, plan.nhr, plan.r2, H, n_groups);
            bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(w2) + (static_cast<size_t>(G.expert[c2.g]) * H + c2.r0) * row2,
                             static_cast<uint32_t>(c2.rows * row2));
          }
        }
        const UnitCoord c = unit_coord(S, u, plan.nfr, plan.r1, F, n_groups);
        const int e = G.expert[c.g];
        if (!mbar_wait_bounded(&S.empty[stage], phase ^ 1u, status, kStatusTimeoutProducer, abort_flag, wait_ns)) {
          ok = false;
          break;
        }
        uint8_t* dst = ring + stage * kStreamStageBytes;
        mbar_arrive_expect_tx(&S.full[stage], static_cast<uint32_t>(2 * c.rows * row1));
        const uint8_t* base = reinterpret_cast<const uint8_t*>(w1) + (static_cast<size_t>(e) * 2 * F) * row1;
        bulk_copy_g2s(dst, base + c.r0 * row1, static_cast<uint32_t>(c.rows * row1), &S.full[stage]);
        bulk_copy_g2s(dst + plan.r1 * row1, base + (F + c.r0) * row1, static_cast<uint32_t>(c.rows * row1),
                      &S.full[stage]);
        advance();
      }
      // phase-2 weight rows do not depend on phase 1: queue the first stages now
      for (int u = u2_begin; u < u2_end && prefetched < kStreamStages && ok; ++u, ++prefetched) {
        const UnitCoord c = unit_coord(S, u, plan.nhr, plan.r2, H, n_groups);
        if (!mbar_wait_bounded(&S.empty[stage], phase ^ 1u, status, kStatusTimeoutProducer, abort_flag, wait_ns)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&S.full[stage], static_cast<uint32_t>(c.rows * row2));
        bulk_copy_g2s(ring + stage * kStreamStageBytes,
                      reinterpret_cast<const uint8_t*>(w2) + (static_cast<size_t>(G.expert[c.g]) * H + c.r0) * row2,
                      static_cast<uint32_t>(c.rows * row2), &S.full[stage]);
        advance();
      }
    }
    if (!grid_barrier_bounded(barrier, gridDim.x, status, kStatusTimeoutOther, &G.flag, wait_ns) || *abort_flag) {
      if (lane == 0) drain();
      return;
    }
    if (lane == 0 && ok) {
      for (int u = u2_begin + prefetched; u < u2_end; ++u) {
        const UnitCoord c = unit_coord(S, u, plan.nhr, plan.r2, H, n_groups);
        if (!mbar_wait_bounded(&S.empty[stage], phase ^ 1u, status, kStatusTimeoutProducer, abort_flag, wait_ns)) {
          drain();
          break;
        }
        mbar_arrive_expect_tx(&S.full[stage], static_cast<uint32_t>(c.rows * row2));
        bulk_copy_g2s(ring + stage * kStreamStageBytes,
                      reinterpret_cast<const uint8_t*>(w2) + (static_cast<size_t>(G.expert[c.g]) * H + c.r0) * row2,
                      static_cast<uint32_t>(c.rows * row2), &S.full[stage]);
        advance();
      }
    }
  } else {
    // ------------------------------------------------------------ consumers, phase 1
    for (int u = blockIdx.x; u < units1; u += gridDim.x) {
      const UnitCoord c = unit_coord(S, u, plan.nfr, plan.r1, F, n_groups);
      if (!mbar_wait_bounded(&S.full[stage], phase, status, kStatusTimeoutOther, abort_flag, wait_ns)) {
        ok = false;
        break;
      }
      const uint8_t* st = ring + stage * kStreamStageBytes;
      // All 256 consumer threads split the columns; each owns 16-byte vectors of every
      // row of the stage (2 * r1 independent FMA chains), then rows are reduced.
      for (int b = 0; b < c.nb; ++b) {
        const int pair = G.list[c.p0 + b];
        const uint4* xrow = xs + static_cast<size_t>(pair / topk) * hv;
        float acc[2 * kStreamMaxR1];
#pragma unroll
        for (int r = 0; r < 2 * kStreamMaxR1; ++r) acc[r] = 0.f;
        for (int v = threadIdx.x; v < hv; v += kStreamCThreads) {
          float xf[8];
          bf16x8_to_f32(xrow[v], xf);
#pragma unroll
          for (int r = 0; r < 2 * kStreamMaxR1; ++r) {
            const int rr = r < kStreamMaxR1 ? r : plan.r1 + (r - kStreamMaxR1);  // gate r / up r
            if ((r < kStreamMaxR1 ? r : r - kStreamMaxR1) < c.rows) {
              float wf[8];
              bf16x8_to_f32(reinterpret_cast<const uint4*>(st + rr * row1)[v], wf);
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[r] = fmaf(wf[i], xf[i], acc[r]);
            }
          }
        }
        warp_reduce16(acc, lane);
        // row index of this lane's sum: bit 4 -> v[i] vs v[i+8], bit 3 -> +4, bit 2 -> +2, bit 1 -> +1
        if ((lane & 1) == 0) S.red[warp][((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 +
                                          ((lane >> 1) & 1)] = acc[0];
        consumers_sync();
        if (threadIdx.x < c.rows) {
          float gs = 0.f, us = 0.f;
#pragma unroll
          for (int w = 0; w < kStreamConsumers; ++w) {
            gs += S.red[w][threadIdx.x];
            us += S.red[w][kStreamMaxR1 + threadIdx.x];
          }
          glu[static_cast<size_t>(pair) * F + c.r0 + threadIdx.x] = act_linear(gs, us);
        }
        consumers_sync();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[stage]);
      advance();
    }
    DECODE_TRACE(2);
    if (!grid_barrier_bounded(barrier, gridDim.x, status, kStatusTimeoutOther, &G.flag, wait_ns) || *abort_flag) return;
    DECODE_TRACE(3);
    // ------------------------------------------------------------ consumers, phase 2
    int cur_g = -1, cur_p0 = -1;
    for (int u = u2_begin; u < u2_end && ok; ++u) {
      const UnitCoord c = unit_coord(S, u, plan.nhr, plan.r2, H, n_groups);
      if (c.g != cur_g || c.p0 != cur_p0) {  // (group, batch) changed: reload its glu rows
        consumers_sync();
        for (int i = threadIdx.x; i < c.nb * (F / 4); i += kStreamConsumers * 32) {
          const int b = i / (F / 4), v = i - b * (F / 4);
          gls[b * (F / 4) + v] = __ldcg(reinterpret_cast<const float4*>(glu + static_cast<size_t>(G.list[c.p0 + b]) * F) + v);
        }
        consumers_sync();
        cur_g = c.g;
        cur_p0 = c.p0;
      }
      if (!mbar_wait_bounded(&S.full[stage], phase, status, kStatusTimeoutOther, abort_flag, wait_ns)) break;
      const uint8_t* st = ring + stage * kStreamStageBytes;
      for (int b = 0; b < c.nb; ++b) {
        float acc[kStreamMaxR2];
#pragma unroll
        for (int r = 0; r < kStreamMaxR2; ++r) acc[r] = 0.f;
        for (int v = threadIdx.x; v < fv; v += kStreamCThreads) {
          const float4 ga = gls[b * (F / 4) + 2 * v];
          const float4 gb = gls[b * (F / 4) + 2 * v + 1];
#pragma unroll
          for (int r = 0; r < kStreamMaxR2; ++r) {
            if (r < c.rows) {
              float wf[8];
              bf16x8_to_f32(reinterpret_cast<const uint4*>(st + r * row2)[v], wf);
              acc[r] = fmaf(wf[0], ga.x, acc[r]);
              acc[r] = fmaf(wf[1], ga.y, acc[r]);
              acc[r] = fmaf(wf[2], ga.z, acc[r]);
              acc[r] = fmaf(wf[3], ga.w, acc[r]);
              acc[r] = fmaf(wf[4], gb.x, acc[r]);
              acc[r] = fmaf(wf[5], gb.y, acc[r]);
              acc[r] = fmaf(wf[6], gb.z, acc[r]);
              acc[r] = fmaf(wf[7], gb.w, acc[r]);
            }
          }
        }
        warp_reduce16(acc, lane);
        if ((lane & 1) == 0) S.red[warp][((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 +
                                          ((lane >> 1) & 1)] = acc[0];
        consumers_sync();
        if (threadIdx.x < c.rows) {
          float sum = 0.f;
#pragma unroll
          for (int w = 0; w < kStreamConsumers; ++w) sum += S.red[w][threadIdx.x];
          partial[static_cast<size_t>(G.list[c.p0 + b]) * H + c.r0 + threadIdx.x] = sum;
        }
        consumers_sync();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[stage]);
      advance();
    }
    DECODE_TRACE(4);
  }
  // Every partial row is written: one more grid barrier, then all CTAs combine the output rows,
  // out[t, h] = bf16(sum_j w[t, j] * partial[(t, j), h]) over valid slots in order j = 0..topk-1
  // (zero rows when no slot is valid). One grid barrier costs less than a last-arriver combine
  // per phase-2 unit (a fence, an atomic and two CTA-wide syncs for every unit).
  if (!grid_barrier_bounded(barrier, gridDim.x, status, kStatusTimeoutOther, &G.flag, wait_ns)) {
    if (warp == kStreamConsumers && lane == 0) drain();
    return;
  }
  DECODE_TRACE(5);
  const int h4 = H / 4;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < tokens * h4; i += gridDim.x * blockDim.x) {
    const int t = i / h4, q = i - t * h4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < topk; ++j) {
      const int p = t * topk + j;
      const int e = indices[p];
      if (e < 0 || e >= experts) continue;
      const float w = weights[p];
      const float4 v = __ldcg(reinterpret_cast<const float4*>(partial + static_cast<size_t>(p) * H) + q);
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * H + 4 * q) = packed;
  }
  DECODE_TRACE(6);
}

}  // namespace

template <int kTB>
cudaError_t launch_gptoss(const DecodeArgs& a, const DecodeWorkspace& ws, const DecodeSplits& sp, int max_groups,
                          cudaStream_t stream) {
  const int H = a.hidden, F = a.inter, total = a.tokens * a.topk;
  const size_t smem1 = kHeaderBytes + (static_cast<size_t>(kTB) * split_rows(H, sp.s1) + kDecWarps * kColsPerCta) * 4;
  const size_t smem2 = kHeaderBytes + (static_cast<size_t>(kTB) * split_rows(F, sp.s2) + kDecWarps * kColsPerCta) * 4;
  const int n_hblocks = (H + kColsPerCta - 1) / kColsPerCta;
  cudaError_t err;
  if ((err = cudaFuncSetAttribute(decode_gate_up_gptoss<kTB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem1))) != cudaSuccess)
    return err;
  if ((err = cudaFuncSetAttribute(decode_down_gptoss<kTB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem2))) != cudaSuccess)
    return err;
  dim3 g1((2 * F + kColsPerCta - 1) / kColsPerCta, max_groups, sp.s1);
  decode_gate_up_gptoss<kTB><<<g1, kDecThreads, smem1, stream>>>(a.x, a.w1, a.b1, a.indices, total, a.topk,
                                                                 a.experts, H, F, sp.s1, ws.glu, ws.pre, ws.counters,
                                                                 n_hblocks);
  dim3 g2(n_hblocks, max_groups, sp.s2);
  decode_down_gptoss<kTB><<<g2, kDecThreads, smem2, stream>>>(ws.glu, ws.pre, a.b1, sp.s1, a.w2, a.b2, a.indices,
                                                              a.weights, a.tokens, a.topk, a.experts, H, F, sp.s2,
                                                              ws.partial, ws.counters, a.out);
  return cudaGetLastError();
}

DecodeSplits decode_splits(int tokens, int topk, int experts, int hidden, int inter, int layout) {
  DecodeSplits sp{1, 1};
  const long long total = static_cast<long long>(tokens) * topk;
  if (layout != CERNELS_LAYOUT_GPTOSS || total <= 0) return sp;
  const long long groups = total < experts ? total : experts;
  // About one resident wave on a 148-SM part (3 CTAs per SM; 4 for single-token batches,
  // whose CTAs are shortest), each split keeping >= 64 rows. Measured on gpt-oss-20b
  // shapes: 2, 6 and 8 CTAs per SM, or up to 16 splits, were slower.
  const long long kTargetCtas = (tokens == 1 ? 4 : 3) * 148;
  constexpr int kMaxSplits = 8;
  auto pick = [&](long long ctas, int rows) {
    long long s = (kTargetCtas + ctas - 1) / ctas;
    if (s > kMaxSplits) s = kMaxSplits;
    if (s > rows / 64) s = rows / 64;
    return s < 1 ? 1 : static_cast<int>(s);
  };
  sp.s1 = pick(groups * ((2LL * inter + kColsPerCta - 1) / kColsPerCta), hidden);
  sp.s2 = pick(groups * ((hidden + kColsPerCta - 1) / kColsPerCta), inter);
  return sp;
}

cudaError_t launch_decode(const DecodeArgs& a, const DecodeWorkspace& ws, cudaStream_t stream) {
  const int total = a.tokens * a.topk;
  if (a.tokens <= 0) return cudaSuccess;
  const int max_groups = total < a.experts ? total : a.experts;
  const int H = a.hidden, F = a.inter;
  cudaError_t err;
  // The streaming kernel wins only for a few pairs (each touched expert costs a grid-wide
  // pass); larger decode batches use the two-kernel path below.
  if (a.layout == CERNELS_LAYOUT_LINEAR && total <= kStreamMaxPairs) {
    const StreamPlan plan = make_stream_plan(H, F);
    const size_t opnd = std::max(static_cast<size_t>(a.tokens) * H * 2, static_cast<size_t>(kTokBatch) * F * 4);
    const size_t smem = ((sizeof(StreamShared) + 127) & ~size_t(127)) +
                        static_cast<size_t>(kStreamStages) * kStreamStageBytes + opnd;
    if (plan.r1 > 0 && plan.r2 > 0 && smem <= 220 * 1024) {
      static PerDeviceOnce smem_attr;
      if ((err = smem_attr.run([] {
             return cudaFuncSetAttribute(decode_stream_linear, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
           })) != cudaSuccess)
        return err;
      int per_sm = 0;
      if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_stream_linear, kStreamThreads,
                                                                smem)) != cudaSuccess)
        return err;
      const int units = max_groups * std::max(plan.nfr, plan.nhr);
      int grid = std::min(per_sm * device_sm_count(), units);
      if (grid < 1) grid = 1;
      // the grid barrier's words start at zero
      if ((err = cudaMemsetAsync(ws.counters, 0, 2 * sizeof(int), stream)) != cudaSuccess) return err;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(grid);
      cfg.blockDim = dim3(kStreamThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      err = cudaLaunchKernelEx(&cfg, decode_stream_linear, a.x, a.w1, a.w2, a.indices, a.weights, a.tokens, a.topk,
                               a.experts, H, F, ws.glu, ws.partial, reinterpret_cast<unsigned*>(ws.counters),
                               ws.status, a.out, wait_limit_ns(kWaitLimitNs));
      if (err != cudaSuccess) return err;
      return cudaGetLastError();
    }
  }
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
    const DecodeSplits sp = decode_splits(a.tokens, a.topk, a.experts, H, F, a.layout);
    // Pairs of one group never exceed the token count (a token picks an expert once), so
    // the operand batch is sized to it. Results do not depend on the batch size chosen.
    const int tb = a.tokens >= 8 ? 8 : a.tokens >= 3 ? 4 : a.tokens;
    switch (tb) {
      case 1: err = launch_gptoss<1>(a, ws, sp, max_groups, stream); break;
      case 2: err = launch_gptoss<2>(a, ws, sp, max_groups, stream); break;
      case 4: err = launch_gptoss<4>(a, ws, sp, max_groups, stream); break;
      default: err = launch_gptoss<8>(a, ws, sp, max_groups, stream); break;
    }
    if (err != cudaSuccess) return err;
  }
  return cudaGetLastError();
}

size_t decode_counter_count(int hidden) { return static_cast<size_t>(hidden / 16 + 1); }

}  // namespace cernels

#ifdef CERNELS_DECODE_TRACE
extern "C" int cernels_debug_decode_trace(unsigned long long* host, int rows) {
  return cudaMemcpyFromSymbol(host, cernels::g_decode_trace, sizeof(unsigned long long) * 8 * rows) == cudaSuccess ? 0 : 4;
}
#endif
