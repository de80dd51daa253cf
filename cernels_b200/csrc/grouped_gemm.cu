// Persistent grouped GEMM over ragged expert groups on sm_100a tensor cores.
//
// Reference: the host loop over experts in cohere2_moe_experts
// (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:302-358) syncs offsets to
// the host and issues, per non-empty expert, cublasGemmEx (gate/up), swiglu_kernel,
// cublasGemmEx (down) and scatter_add; gpt-oss adds add_gateup_bias_kernel and the
// clamped interleaved SwiGLU (src/kops/gpt_oss_moe_experts/csrc/gpt_oss_moe_experts.cu:75-117,185-242).
//
// Here one launch covers every expert. Rows of the permuted token matrix are grouped by
// expert (offsets from the routing kernel); tile t of the launch maps to
// (expert e, n-tile, m-tile) through the per-expert tile prefix mtile_offsets, read on
// the device, so there is no host synchronisation. Each CTA (one per SM) runs:
//   warp 0      TMA producer: A tile [128 x 64] and B tile [256 x 64] per stage
//               (128-byte swizzle, 4-stage ring of 48 KB stages)
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and issues
//               tcgen05.mma (M=128, N=256, K=16) from one thread; tcgen05.commit frees
//               smem stages and publishes finished accumulators
//   warps 2-5   epilogue: tcgen05.ld of the accumulator quarter owned by the warp,
//               fused bias + activation (gate/up) or bias (down), bf16 stores
// Accumulators are double-buffered so the epilogue of tile i overlaps the MMAs of i+1.
#include "moe_internal.h"
#include "sm100_primitives.cuh"

#include <cudaTypedefs.h>

namespace cernels {
namespace {

constexpr int BM = kBlockM;  // 128
constexpr int BN_MAX = 256;  // widest N tile; 192 is used when it divides N and 256 does not
constexpr int BK = 64;       // 64 bf16 = 128 bytes = one swizzle row
constexpr int kStages = 4;
constexpr int kABytes = BM * BK * 2;  // 16 KB
constexpr int kBBytesMax = BN_MAX * BK * 2;  // 32 KB
constexpr int kBoxBytes = 64 * BK * 2;         // one 64-column N-major box [64 K rows x 128 B]
constexpr int kAccStride = 256;                // TMEM column offset between the two accumulators
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kBarrierBytes = 256;
constexpr int kStageRow = 64 * 2 + 16;              // staging row: 64 bf16 outputs + 16 B pad (no bank conflicts)
constexpr int kStageBytes = 4 * 32 * kStageRow;     // 4 epilogue warps x 32 rows
__host__ __device__ constexpr size_t smem_fixed(int bn) {
  return static_cast<size_t>(kStages) * (kABytes + bn * BK * 2) + kBarrierBytes + kStageBytes;
}

constexpr float kGptOssLimit = 7.0f;
constexpr float kGptOssAlpha = 1.702f;

__host__ __device__ constexpr bool mode_is_gptoss(int mode) { return mode == kGateUpGptOss || mode == kDownGptOss; }

// Number of n-tiles of one expert's output.
__host__ __device__ inline int n_tiles_for(int mode, int n, int bn) {
  // Linear gate/up pairs 128 gate rows with 128 up rows per tile: n = 2F, F/128 tiles.
  if (mode == kGateUpLinear) return (n / 2 + 127) / 128;
  return (n + bn - 1) / bn;
}

struct TileCoord {
  int expert, m_tile, n_tile;
};

__device__ __forceinline__ TileCoord decode_tile(int t, int n_tiles, const int* s_mt, int experts) {
  const int q = t / n_tiles;
  int lo = 0, hi = experts - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_mt[mid] <= q) lo = mid; else hi = mid - 1;
  }
  TileCoord c;
  c.expert = lo;
  const int nm = s_mt[lo + 1] - s_mt[lo];
  const int local = t - s_mt[lo] * n_tiles;
  c.n_tile = local / nm;
  c.m_tile = local - c.n_tile * nm;
  return c;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

__device__ __forceinline__ float gptoss_glu(float gate, float up) {
  gate = fminf(gate, kGptOssLimit);
  up = fmaxf(-kGptOssLimit, fminf(up, kGptOssLimit));
  const float glu = gate / (1.0f + __expf(-gate * kGptOssAlpha));
  return (up + 1.0f) * glu;
}

template <int kMode, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_b_extra, GroupedGemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + kStages * kABytes;
  constexpr int kBBytes = BN * BK * 2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * (kABytes + kBBytes));
  uint64_t* full_bar = bars;                  // [kStages]
  uint64_t* empty_bar = bars + kStages;       // [kStages]
  uint64_t* tfull_bar = bars + 2 * kStages;   // [2]
  uint64_t* tempty_bar = bars + 2 * kStages + 2;  // [2]
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  uint8_t* epi_stage = smem + kStages * (kABytes + kBBytes) + kBarrierBytes;       // [kStageBytes]
  int* s_mt = reinterpret_cast<int*>(epi_stage + kStageBytes);                      // [E + 1]

  const int experts = args.experts;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i <= experts; i += blockDim.x) s_mt[i] = args.mtile_offsets[i];
  const int n_tiles = n_tiles_for(kMode, args.n, BN);
  __syncthreads();
  const int total_tiles = s_mt[experts] * n_tiles;
  if (static_cast<int>(blockIdx.x) >= total_tiles) return;  // uniform per CTA

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (args.b_extra != nullptr) tma_prefetch_desc(&tmap_b_extra);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  const int k_blocks = (args.k + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      long long issued = 0;  // stages loaded so far
      int ready_group = -1;  // group whose rows are known to have arrived
      const uint32_t epoch = args.ready == nullptr ? 0u
                             : args.ready_epoch ? args.ready_epoch
                                                : *reinterpret_cast<const volatile uint32_t*>(args.ready_epoch_dev) + 1u;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileCoord c = decode_tile(t, n_tiles, s_mt, experts);
        const bool local_group = args.b_extra != nullptr && c.expert == args.extra_group;  // rows from this GPU
        if (args.ready != nullptr && c.expert != ready_group && !local_group) {
          // rows of this group come from other GPUs: wait until every source has delivered them
          const unsigned long long t0 = global_timer_ns();
          for (int src = 0; src < args.ready_sources && ok; ++src) {
            if (src == args.ready_self) continue;
            const uint32_t* flag =
                reinterpret_cast<const uint32_t*>(args.ready + src * args.ready_stride + 4 * static_cast<size_t>(c.expert));
            uint32_t v;
            while (true) {
              asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
              if (v == epoch) break;
              if (*abort_flag || global_timer_ns() - t0 > args.wait_ns) {
                if (args.status) atomicCAS(args.status, 0, kStatusTimeoutProducer);
                *abort_flag = 1;
                ok = false;
                break;
              }
            }
          }
          if (!ok) break;
          fence_proxy_async_global();  // the peer-written rows are read next by TMA
          ready_group = c.expert;
        }
        const int row0 = args.offsets[c.expert] + c.m_tile * BM;
        const bool extra = args.b_extra != nullptr && c.expert == args.extra_group;
        const CUtensorMap* bmap = extra ? &tmap_b_extra : &tmap_b;
        const int we = extra ? 0 : c.expert % args.weight_experts;  // weight slab of this row group
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, args.status, kStatusTimeoutProducer, abort_flag, args.wait_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kABytes + kBBytes);
          uint8_t* a_dst = smem_a + stage * kABytes;
          uint8_t* b_dst = smem_b + stage * kBBytes;
          tma_load_2d(a_dst, &tmap_a, &full_bar[stage], kb * BK, row0, kCacheEvictNormal);
          if constexpr (kMode == kGateUpLinear) {
            const int f0 = c.n_tile * 128;
            const int half_f = args.n / 2;
            tma_load_3d(b_dst, bmap, &full_bar[stage], kb * BK, f0, we, kCacheEvictNormal);
            tma_load_3d(b_dst + kBBytes / 2, bmap, &full_bar[stage], kb * BK, half_f + f0, we,
                        kCacheEvictNormal);
          } else if constexpr (kMode == kDownLinear) {
            tma_load_3d(b_dst, bmap, &full_bar[stage], kb * BK, c.n_tile * BN, we, kCacheEvictNormal);
          } else {
            // N-major weights: BN/64 boxes of 64 columns, each [64 K rows x 128 bytes].
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(b_dst + j * kBoxBytes, bmap, &full_bar[stage], c.n_tile * BN + 64 * j, kb * BK,
                          we, kCacheEvictNormal);
          }
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Giving up: let the loads still in flight (at most the last kStages) land before
        // this CTA exits, so none writes shared memory the CTA no longer owns.
        for (long long i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
          mbar_drain(&full_bar[i % kStages], static_cast<uint32_t>((i / kStages) & 1), args.wait_ns);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, 0, mode_is_gptoss(kMode) ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1u, args.status, kStatusTimeoutMma, abort_flag, args.wait_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kAccStride);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, args.status, kStatusTimeoutMma, abort_flag, args.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem_a + stage * kABytes);
          const uint32_t b_addr = smem_u32(smem_b + stage * kBBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t a_desc = make_smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            uint64_t b_desc;
            if constexpr (mode_is_gptoss(kMode)) {
              b_desc = make_smem_desc_sw128(b_addr + kk * 2048, kBoxBytes, 1024);
            } else {
              b_desc = make_smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            }
            umma_bf16(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    int local = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, args.status, kStatusTimeoutEpilogue, abort_flag, args.wait_ns)) break;
      tc_fence_after();
      const TileCoord c = decode_tile(t, n_tiles, s_mt, experts);
      const int e = (args.b_extra != nullptr && c.expert == args.extra_group) ? 0 : c.expert % args.weight_experts;
      const int row_begin = args.offsets[c.expert];
      const int rows_e = args.group_rows ? args.group_rows[c.expert] : args.offsets[c.expert + 1] - row_begin;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kAccStride);

      // Outputs go through this warp's staging tile (32 rows x 64 bf16 columns) so that global
      // stores write whole 128-byte row segments: 8 lanes per row, 4 rows per instruction.
      uint8_t* stg = epi_stage + quarter * 32 * kStageRow;
      const int tile_row0 = c.m_tile * BM + quarter * 32;  // first row of this warp, within the group
      auto flush = [&](int col0) {
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int idx = it * 32 + lane;
          const int r = idx >> 3, piece = idx & 7;
          const int col = col0 + piece * 8;
          if (tile_row0 + r < rows_e && col < args.out_cols) {
            const uint4 v = *reinterpret_cast<const uint4*>(stg + r * kStageRow + piece * 16);
            __nv_bfloat16* dst;
            if (args.row_out) {
              dst = args.row_out[row_begin + tile_row0 + r];
              if (dst == nullptr) continue;
            } else {
              dst = args.out + static_cast<size_t>(row_begin + tile_row0 + r) * args.out_cols;
            }
            *reinterpret_cast<uint4*>(dst + col) = v;
          }
        }
        __syncwarp();
      };
      auto stage8 = [&](int wcol, const float* r8) {  // 8 outputs at window column wcol of this lane's row
        uint4 q;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(r8[2 * i], r8[2 * i + 1]);
        *reinterpret_cast<uint4*>(stg + lane * kStageRow + wcol * 2) = q;
      };
      // Per 32-column TMEM chunk: LINEAR gate/up and down produce 32 outputs, gpt-oss gate/up 16;
      // a window of 64 outputs is flushed once full, the last one after the accumulator is
      // released to the MMA warp.
      constexpr int kOutPerChunk = kMode == kGateUpGptOss ? 16 : 32;
      constexpr int kChunks = kMode == kGateUpLinear ? 4 : BN / 32;
      constexpr int kChunksPerWindow = 64 / kOutPerChunk;
      const int out0 = kMode == kGateUpLinear ? c.n_tile * 128 : kMode == kGateUpGptOss ? c.n_tile * BN / 2 : c.n_tile * BN;
      const float* bias = nullptr;
      if constexpr (kMode == kGateUpGptOss) bias = args.bias ? args.bias + static_cast<size_t>(e) * args.n : nullptr;
      if constexpr (kMode == kDownGptOss || kMode == kDownLinear)
        bias = args.bias ? args.bias + static_cast<size_t>(e) * args.out_cols : nullptr;
#pragma unroll 1
      for (int ch = 0; ch < kChunks; ++ch) {
        const int c0 = ch * 32;
        const int wbase = (ch % kChunksPerWindow) * kOutPerChunk;  // window column of this chunk's first output
        if constexpr (kMode == kGateUpLinear) {
          float g[32], u[32];
          tmem_ld_32x32b_x32(t_row + c0, g);
          tmem_ld_32x32b_x32(t_row + 128 + c0, u);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            float r[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = silu(g[8 * v + i]) * u[8 * v + i];
            stage8(wbase + 8 * v, r);
          }
        } else if constexpr (kMode == kGateUpGptOss) {
          float a[32];
          tmem_ld_32x32b_x32(t_row + c0, a);
          const int wcol = c.n_tile * BN + c0;  // weight column (even = gate, odd = up)
          if (bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i) a[i] += (wcol + i < args.n) ? __ldg(bias + wcol + i) : 0.f;
          }
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            float r[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = gptoss_glu(a[16 * v + 2 * i], a[16 * v + 2 * i + 1]);
            stage8(wbase + 8 * v, r);
          }
        } else {
          float a[32];
          tmem_ld_32x32b_x32(t_row + c0, a);
          const int col = c.n_tile * BN + c0;
          if (bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i) a[i] += (col + i < args.out_cols) ? __ldg(bias + col + i) : 0.f;
          }
#pragma unroll
          for (int v = 0; v < 4; ++v) stage8(wbase + 8 * v, a + 8 * v);
        }
        if ((ch + 1) % kChunksPerWindow == 0 && ch + 1 < kChunks)
          flush(out0 + (ch / kChunksPerWindow) * 64);
      }
      // every TMEM read of this accumulator is done: hand it back, then write the last window
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      flush(out0 + ((kChunks - 1) / kChunksPerWindow) * 64);
    }
  }

  // Outputs written through row_out may live on another GPU: make them visible system-wide
  // before the kernel ends, so that a flag raised by a later kernel is ordered after them.
  if (args.row_out != nullptr) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool encode_map(CUtensorMap* map, const void* ptr, int rank, const uint64_t* dims, const uint64_t* byte_strides,
                const uint32_t* box) {
  auto fn = get_encode_fn();
  if (!fn) return false;
  cuuint32_t elem_strides[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(ptr),
                        reinterpret_cast<const cuuint64_t*>(dims), reinterpret_cast<const cuuint64_t*>(byte_strides),
                        reinterpret_cast<const cuuint32_t*>(box), elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

bool encode_bf16_map(CUtensorMap* map, const void* ptr, int rank, const uint64_t* dims, const uint64_t* byte_strides,
                     const uint32_t* box) {
  return encode_map(map, ptr, rank, dims, byte_strides, box);
}

namespace {

template <int kMode, int BN>
cudaError_t launch_mode(const GroupedGemmArgs& args, int num_sms, cudaStream_t stream) {
  CUtensorMap map_a, map_b;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(args.rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(args.k) * 2};
    const uint32_t box[2] = {BK, BM};
    if (!encode_map(&map_a, args.a, 2, dims, strides, box)) return cudaErrorInvalidValue;
  }
  auto encode_b = [&](CUtensorMap* map, const __nv_bfloat16* ptr, uint64_t E) -> bool {
    if constexpr (kMode == kGateUpLinear || kMode == kDownLinear) {
      // Weight [E, N, K] (K contiguous): dims (K, N, E).
      const uint64_t dims[3] = {static_cast<uint64_t>(args.k), static_cast<uint64_t>(args.n), E};
      const uint64_t strides[2] = {static_cast<uint64_t>(args.k) * 2, static_cast<uint64_t>(args.k) * args.n * 2};
      const uint32_t box[3] = {BK, kMode == kGateUpLinear ? 128u : static_cast<uint32_t>(BN), 1};
      return encode_map(map, ptr, 3, dims, strides, box);
    } else {
      // Weight [E, K, N] (N contiguous): dims (N, K, E), 64-column boxes.
      const uint64_t dims[3] = {static_cast<uint64_t>(args.n), static_cast<uint64_t>(args.k), E};
      const uint64_t strides[2] = {static_cast<uint64_t>(args.n) * 2, static_cast<uint64_t>(args.k) * args.n * 2};
      const uint32_t box[3] = {64, BK, 1};
      return encode_map(map, ptr, 3, dims, strides, box);
    }
  };
  CUtensorMap map_b_extra;
  if (!encode_b(&map_b, args.b, static_cast<uint64_t>(args.weight_experts))) return cudaErrorInvalidValue;
  if (args.b_extra != nullptr) {
    if (!encode_b(&map_b_extra, args.b_extra, 1)) return cudaErrorInvalidValue;
  } else {
    map_b_extra = map_b;
  }
  const size_t smem = smem_fixed(BN) + 1024 + static_cast<size_t>(args.experts + 1) * sizeof(int);
  static PerDeviceOnce attr;
  cudaError_t err = attr.run([] {
    return cudaFuncSetAttribute(grouped_gemm_kernel<kMode, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem_fixed(BN) + 1024 + (kMaxExperts + 1) * sizeof(int)));
  });
  if (err != cudaSuccess) return err;
  const int n_tiles = n_tiles_for(kMode, args.n, BN);
  const long long max_mtiles = (static_cast<long long>(args.rows) + BM - 1) / BM + args.experts;
  const long long max_tiles = max_mtiles * n_tiles;
  const int grid = static_cast<int>(max_tiles < num_sms ? max_tiles : num_sms);
  if (grid <= 0) return cudaSuccess;
  GroupedGemmArgs a = args;
  a.wait_ns = wait_limit_ns(kWaitLimitNs);
  grouped_gemm_kernel<kMode, BN><<<grid, kThreads, smem, stream>>>(map_a, map_b, map_b_extra, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_grouped_gemm(GemmMode mode, const GroupedGemmArgs& args, int num_sms, cudaStream_t stream) {
  // 192-wide N tiles avoid the padded last tile when 192 divides N and 256 does not, but on
  // B200 they measured slower than 256-wide tiles with that padding (A re-read per FLOP rises
  // by a third): gpt-oss gate/up 1.77 vs 1.58 ms, down 0.91 vs 0.89 ms. Kept selectable.
  const bool narrow = false;
  switch (mode) {
    case kGateUpLinear: return launch_mode<kGateUpLinear, 256>(args, num_sms, stream);
    case kGateUpGptOss:
      return narrow ? launch_mode<kGateUpGptOss, 192>(args, num_sms, stream)
                    : launch_mode<kGateUpGptOss, 256>(args, num_sms, stream);
    case kDownLinear:
      return narrow ? launch_mode<kDownLinear, 192>(args, num_sms, stream)
                    : launch_mode<kDownLinear, 256>(args, num_sms, stream);
    case kDownGptOss:
      return narrow ? launch_mode<kDownGptOss, 192>(args, num_sms, stream)
                    : launch_mode<kDownGptOss, 256>(args, num_sms, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace cernels
