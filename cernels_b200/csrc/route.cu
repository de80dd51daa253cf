// Routing: per-expert histogram, expert offsets and a stable permutation of the
// flat (token, slot) entries into expert-major order, plus the inverse map used
// by the deterministic combine.
//
// Reference semantics (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:29-55):
// count_tokens_kernel histograms indices with global atomics, at::cumsum turns the
// histogram into offsets, build_perm_kernel places each entry with an atomic cursor
// (order inside an expert = atomic arrival order). Ids outside [0, E) are skipped.
// Here the order inside an expert is the flat index t*topk+j (a stable counting sort,
// identical to torch.sort(indices.flatten(), stable=True) restricted to valid ids),
// computed without global atomics:
//   1. route_count_kernel  — one CTA per chunk (256 or 1024 entries), shared-memory histogram
//   2. route_scan_kernel   — one CTA: per-expert prefix over chunks, offsets, tile offsets
//   3. route_place_kernel  — one CTA per chunk; warp __match_any_sync ranks entries of
//                            the same expert, a cross-warp prefix in shared memory keeps
//                            the flat order, chunk bases come from step 2.
#include "moe_internal.h"

namespace cernels {
namespace {

__global__ void __launch_bounds__(kRouteThreads) route_count_kernel(const int32_t* __restrict__ indices, int total,
                                                                    int chunk, int experts,
                                                                    int* __restrict__ block_counts) {
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < experts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int base = blockIdx.x * chunk;
  const int end = min(base + chunk, total);
  for (int i = base + threadIdx.x; i < end; i += blockDim.x) {
    const int e = indices[i];
    if (e >= 0 && e < experts) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  int* dst = block_counts + static_cast<size_t>(blockIdx.x) * experts;
  for (int e = threadIdx.x; e < experts; e += blockDim.x) dst[e] = hist[e];
}

// Exclusive block-wide scan of one int per thread (blockDim.x == 1024).
__device__ int block_exclusive_scan_1024(int v, int* warp_tot, int* total_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_tot[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    warp_tot[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) *total_out = wi;
  }
  __syncthreads();
  const int r = warp_tot[warp] + incl - v;
  __syncthreads();
  return r;
}

// One CTA of 1024 threads. block_counts [n_chunks, E] is rewritten in place into the
// absolute first row of each (chunk, expert) run.
__global__ void __launch_bounds__(1024) route_scan_kernel(int* __restrict__ block_counts, int n_chunks, int experts,
                                                          int* __restrict__ offsets, int* __restrict__ mtile_offsets) {
  __shared__ int warp_tot[32];
  __shared__ int total_rows, total_tiles;
  __shared__ int carry_rows, carry_tiles;
  extern __shared__ int expert_base[];  // [experts]
  if (threadIdx.x == 0) {
    carry_rows = 0;
    carry_tiles = 0;
  }
  __syncthreads();
  // Experts are scanned in rounds of 1024 (one expert per thread).
  for (int e0 = 0; e0 < experts; e0 += 1024) {
    const int e = e0 + threadIdx.x;
    int count = 0;
    if (e < experts) {
      // exclusive prefix over chunks, within the expert; loads batched 8 at a time so the
      // chain of global reads does not serialise on memory latency
      constexpr int kBatch = 8;
      for (int b0 = 0; b0 < n_chunks; b0 += kBatch) {
        int c[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
          c[j] = b0 + j < n_chunks ? block_counts[static_cast<size_t>(b0 + j) * experts + e] : 0;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          if (b0 + j < n_chunks) block_counts[static_cast<size_t>(b0 + j) * experts + e] = count;
          count += c[j];
        }
      }
    }
    const int tiles = (count + kBlockM - 1) / kBlockM;
    const int row_off = block_exclusive_scan_1024(count, warp_tot, &total_rows);
    const int tile_off = block_exclusive_scan_1024(tiles, warp_tot, &total_tiles);
    if (e < experts) {
      offsets[e] = carry_rows + row_off;
      mtile_offsets[e] = carry_tiles + tile_off;
      expert_base[e] = carry_rows + row_off;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      carry_rows += total_rows;
      carry_tiles += total_tiles;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    offsets[experts] = carry_rows;
    mtile_offsets[experts] = carry_tiles;
  }
  for (int e = threadIdx.x; e < experts; e += blockDim.x) {
    const int base = expert_base[e];
    for (int b = 0; b < n_chunks; ++b) block_counts[static_cast<size_t>(b) * experts + e] += base;
  }
}

__global__ void __launch_bounds__(kRouteThreads) route_place_kernel(
    const int32_t* __restrict__ indices, const float* __restrict__ weights, int total, int chunk, int topk, int experts,
    const int* __restrict__ chunk_base, int* __restrict__ perm_flat, int* __restrict__ perm_token,
    float* __restrict__ perm_weight, int* __restrict__ inv) {
  constexpr int kWarps = kRouteThreads / 32;
  extern __shared__ int smem[];
  int* running = smem;             // [experts] entries of each expert placed so far in this chunk
  int* warp_cnt = smem + experts;  // [kWarps, experts] entries of each expert in this round per warp
  for (int i = threadIdx.x; i < experts * (kWarps + 1); i += blockDim.x) smem[i] = 0;
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int* base_row = chunk_base + static_cast<size_t>(blockIdx.x) * experts;
  const int chunk0 = blockIdx.x * chunk;
  const unsigned lanes_below = (1u << lane) - 1u;

  for (int r0 = 0; r0 < chunk; r0 += kRouteThreads) {
    const int i = chunk0 + r0 + threadIdx.x;
    int e = -1;
    if (i < total) {
      e = indices[i];
      if (e < 0 || e >= experts) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lanes_below);
    const bool leader = rank == 0;
    if (e >= 0 && leader) warp_cnt[warp * experts + e] = __popc(peers);
    __syncthreads();
    int pos = -1;
    bool first_warp = false;
    int round_total = 0;
    if (e >= 0) {
      int before = 0;
      for (int w = 0; w < kWarps; ++w) {
        const int c = warp_cnt[w * experts + e];
        if (w < warp) before += c;
        round_total += c;
      }
      first_warp = before == 0;
      pos = base_row[e] + running[e] + before + rank;
    }
    __syncthreads();
    if (e >= 0 && leader) {
      if (first_warp) running[e] += round_total;
      warp_cnt[warp * experts + e] = 0;
    }
    if (i < total) {
      inv[i] = pos;
      if (pos >= 0) {
        perm_flat[pos] = i;
        perm_token[pos] = i / topk;
        perm_weight[pos] = weights[i];
      }
    }
    __syncthreads();
  }
}

}  // namespace

cudaError_t launch_route(const int32_t* indices, const float* weights, int tokens, int topk, int experts,
                         const PrefillWorkspace& ws, cudaStream_t stream) {
  const int total = tokens * topk;
  const int chunk = route_chunk(total);
  const int n_chunks = (total + chunk - 1) / chunk;
  const size_t hist_smem = static_cast<size_t>(experts) * sizeof(int);
  const size_t place_smem = static_cast<size_t>(experts) * (kRouteThreads / 32 + 1) * sizeof(int);
  cudaError_t err;
  if (place_smem > 48 * 1024) {
    err = cudaFuncSetAttribute(route_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(place_smem));
    if (err != cudaSuccess) return err;
  }
  if (n_chunks > 0) {
    route_count_kernel<<<n_chunks, kRouteThreads, hist_smem, stream>>>(indices, total, chunk, experts,
                                                                       ws.block_counts);
  }
  route_scan_kernel<<<1, 1024, hist_smem, stream>>>(ws.block_counts, n_chunks, experts, ws.offsets,
                                                    ws.mtile_offsets);
  if (n_chunks > 0) {
    route_place_kernel<<<n_chunks, kRouteThreads, place_smem, stream>>>(
        indices, weights, total, chunk, topk, experts, ws.block_counts, ws.perm_flat, ws.perm_token,
        ws.perm_weight, ws.inv);
  }
  return cudaGetLastError();
}

cudaError_t launch_segments(const int* counts, int groups, int* scratch, int* offsets, int* mtile_offsets,
                            cudaStream_t stream) {
  cudaError_t err = cudaMemcpyAsync(scratch, counts, static_cast<size_t>(groups) * sizeof(int),
                                    cudaMemcpyDeviceToDevice, stream);
  if (err != cudaSuccess) return err;
  // One "chunk" whose histogram is the given counts.
  route_scan_kernel<<<1, 1024, static_cast<size_t>(groups) * sizeof(int), stream>>>(scratch, 1, groups, offsets,
                                                                                    mtile_offsets);
  return cudaGetLastError();
}

}  // namespace cernels
