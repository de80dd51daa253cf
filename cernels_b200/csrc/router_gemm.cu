// Fused router: logits = x W^T (+ b) on tcgen05 tensor cores, with the top-k / softmax /
// renormalisation tail in the epilogue, so the logits never reach HBM.
//
// Reference: the loaders run the transformers routers in torch in the timed path
// (src/kops/registry/gpt_oss_moe_experts.py:35 -> GptOssTopKRouter, a bf16 F.linear with
// bias, top-k of the logits, softmax over the k values in bf16;
// src/kops/registry/qwen3_next_moe_experts.py:28 -> Qwen3NextTopKRouter, a bf16 F.linear,
// softmax over all experts in fp32, top-k, renormalisation), then cast the ids to int32 and
// the scores to fp32 (src/kops/registry/cohere2_moe_experts.py:25-26).
//
// One CTA computes a 128-token x BN-logit tile (BN <= 256): warp 0 streams x and router-weight
// tiles with TMA (128-byte swizzle), warp 1 issues tcgen05.mma (M=128, N=BN, K=16) into one
// TMEM accumulator, warps 2-5 each own 32 token rows. Epilogue per row, in one thread: add
// the bias, round to bf16 (the transformers linear's output dtype), keep a running top-k
// (ties to the lower expert id) and, for the softmax-over-all mode, the row max and sum of
// exponentials. When the experts do not fit one tile, a cluster of NC CTAs splits the
// columns; every CTA pushes its per-row candidates (top-k, max, sum, shared-gate logit) into
// the shared memory of cluster rank 0 (DSMEM stores + one remote mbarrier arrive), and rank 0
// merges them and writes int32 ids / fp32 weights. No TMA multicast is used.
#include "moe_internal.h"
#include "sm100_primitives.cuh"

namespace cernels {
namespace {

constexpr int RBM = 128;
constexpr int RBK = 64;
constexpr int kRThreads = 320;  // producer, MMA, 8 epilogue warps
constexpr int kRABytes = RBM * RBK * 2;  // 16 KB
constexpr int kTop = 16;                 // candidates kept per row (topk <= 16)

}  // namespace
#ifdef ROUTER_TRACE
// Debug builds only: %globaltimer stamps per CTA at phase boundaries (thread of the epilogue's row 0).
__device__ unsigned long long g_router_trace[4096][8];
#define RTRACE(slot) \
  if (threadIdx.x == 64 && blockIdx.x + gridDim.x * blockIdx.y < 4096) \
    g_router_trace[blockIdx.x + gridDim.x * blockIdx.y][slot] = clock64();
#else
#define RTRACE(slot)
#endif
namespace {

struct RouterArgs {
  const __nv_bfloat16* bias;  // [experts] or null
  int32_t* indices;           // [T, topk + gate]
  float* weights;             // [T, topk + gate]
  __nv_bfloat16* logits;      // optional [T, logits_ld]
  int* status;                // optional
  unsigned long long wait_ns;
  int tokens, hidden, experts, topk, mode, renorm, gate, bn, nc, stages, logits_ld, tmem_cols;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of `local_smem` in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local_smem, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Named barriers: 1 over the eight epilogue warps, 2 over the first four of them.
__device__ __forceinline__ void epilogue_sync_all() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ void epilogue_sync_half() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}


// A candidate (bf16 logit, expert id) packed into one unsigned key that orders like "larger
// logit first, then lower expert id": the logit's bf16 bits mapped to an order-preserving
// unsigned code in the high half, 0xFFFF - id in the low half. Key 0 ranks below every
// real candidate. Top-k selection then needs only unsigned min / max.
__device__ __forceinline__ uint32_t bf16_bits_rne(float f) {  // round to nearest even (no NaN inputs)
  uint32_t u = __float_as_uint(f);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return u >> 16;
}
__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits) { return __uint_as_float(bits << 16); }
__device__ __forceinline__ uint32_t make_key(uint32_t bits, int e) {
  const uint32_t ord = (bits & 0x8000u) ? (~bits & 0xFFFFu) : (bits | 0x8000u);
  return (ord << 16) | (0xFFFFu - static_cast<uint32_t>(e));
}
__device__ __forceinline__ float key_value(uint32_t key) {
  const uint32_t ord = key >> 16;
  return bf16_bits_to_float((ord & 0x8000u) ? (ord & 0x7FFFu) : (~ord & 0xFFFFu));
}
__device__ __forceinline__ int key_id(uint32_t key) { return static_cast<int>(0xFFFFu - (key & 0xFFFFu)); }

// Bitonic sorting network over 16 keys, largest first. Every index is a compile-time constant
// (the keys stay in registers) and each stage's 8 min / max pairs are independent.
__device__ __forceinline__ void sort16(uint32_t (&k)[16]) {
#pragma unroll
  for (int size = 2; size <= 16; size <<= 1) {
#pragma unroll
    for (int stride = size / 2; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const uint32_t hi = max(k[i], k[j]), lo = min(k[i], k[j]);
          const bool desc = (i & size) == 0 || size == 16;
          k[i] = desc ? hi : lo;
          k[j] = desc ? lo : hi;
        }
      }
    }
  }
}

// Running top-16 keys of one row, largest first (callers use the first k <= 16). A sorted block
// merges in with the larger of list[i] and block[15 - i] (a bitonic sequence holding the best
// 16 of both) and a 4-stage half-cleaner.
struct Top16 {
  uint32_t k[16];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int j = 0; j < 16; ++j) k[j] = 0u;
  }
  __device__ __forceinline__ void merge_sorted(const uint32_t (&b)[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) k[i] = max(k[i], b[15 - i]);
#pragma unroll
    for (int stride = 8; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const uint32_t hi = max(k[i], k[j]), lo = min(k[i], k[j]);
          k[i] = hi;
          k[j] = lo;
        }
      }
    }
  }
};

// Per-row candidate records (sum of exponentials against the list's best logit, shared-gate
// logit, top-16 keys), structure-of-arrays: slot c holds column chunk c's candidates.
struct Records {
  float* sum;     // [slots][128]
  float* gate;    // [slots][128] (NaN when the chunk has no gate column)
  uint32_t* key;  // [slots][16][128]
  __device__ Records(uint8_t* base, int slots) {
    sum = reinterpret_cast<float*>(base);
    gate = sum + slots * RBM;
    key = reinterpret_cast<uint32_t*>(gate + slots * RBM);
  }
  __host__ __device__ static size_t bytes(int slots) { return static_cast<size_t>(slots) * RBM * (2 + kTop) * 4; }
  __device__ void store(int row, int slot, float s, float g, const Top16& top) {
    sum[slot * RBM + row] = s;
    gate[slot * RBM + row] = g;
#pragma unroll
    for (int j = 0; j < kTop; ++j) key[(slot * kTop + j) * RBM + row] = top.k[j];
  }
  // Merges slot `slot`'s candidates of `row` into (s, g, top); s is a sum of exp(l - max) where
  // max is the best logit of the list it belongs to.
  __device__ void merge_into(int row, int slot, float& s, float& g, Top16& top) const {
    uint32_t b[kTop];
#pragma unroll
    for (int j = 0; j < kTop; ++j) b[j] = key[(slot * kTop + j) * RBM + row];
    if (b[0] != 0u) {
      const float m0 = top.k[0] ? key_value(top.k[0]) : -INFINITY;
      const float m1 = key_value(b[0]);
      const float mm = fmaxf(m0, m1);
      s = (top.k[0] ? s * __expf(m0 - mm) : 0.f) + sum[slot * RBM + row] * __expf(m1 - mm);
    }
    const float g1 = gate[slot * RBM + row];
    if (!isnan(g1)) g = g1;
    top.merge_sorted(b);
  }
};

__global__ void __launch_bounds__(kRThreads, 1)
    router_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                       RouterArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const int b_bytes = a.bn * RBK * 2;
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + S * kRABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_b + S * b_bytes);
  uint64_t* full_bar = bars;            // [S]
  uint64_t* empty_bar = bars + S;       // [S]
  uint64_t* tfull_bar = bars + 2 * S;   // [1]
  uint64_t* merge_bar = tfull_bar + 1;  // [1] arrivals of the other cluster ranks
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(merge_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* rec_base = reinterpret_cast<uint8_t*>(bars) + 256;
  Records rec(rec_base, a.nc);                          // the cluster's chunks (rank 0 reads)
  Records hrec(rec_base + Records::bytes(a.nc), 1);     // the upper column half of this CTA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = a.nc > 1 ? cluster_ctarank() : 0;
  const int chunk = blockIdx.x;  // column chunk (== cluster rank when nc > 1)
  const int m0 = blockIdx.y * RBM;
  const int k_blocks = (a.hidden + RBK - 1) / RBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(merge_bar, a.nc > 1 ? a.nc - 1 : 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  RTRACE(0);
  // every CTA of the cluster has initialised its barriers before any remote arrive
  if (a.nc > 1) cluster_sync_all();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, a.status, kStatusTimeoutProducer, abort_flag,
                               a.wait_ns)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[stage], kRABytes + b_bytes);
        tma_load_2d(smem_a + stage * kRABytes, &tmap_x, &full_bar[stage], kb * RBK, m0, kCacheEvictNormal);
        tma_load_2d(smem_b + stage * b_bytes, &tmap_w, &full_bar[stage], kb * RBK, chunk * a.bn, kCacheEvictLast);
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok)
        for (long long i = issued > S ? issued - S : 0; i < issued; ++i)
          mbar_drain(&full_bar[i % S], static_cast<uint32_t>((i / S) & 1), a.wait_ns);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = make_idesc_bf16(RBM, a.bn, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait_bounded(&full_bar[stage], phase, a.status, kStatusTimeoutMma, abort_flag, a.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem_a + stage * kRABytes);
        const uint32_t b_addr = smem_u32(smem_b + stage * b_bytes);
#pragma unroll
        for (int kk = 0; kk < RBK / 16; ++kk)
          umma_bf16(tmem, make_smem_desc_sw128(a_addr + kk * 32, 16, 1024),
                    make_smem_desc_sw128(b_addr + kk * 32, 16, 1024), idesc, (kb | kk) != 0 ? 1u : 0u);
        umma_commit(&empty_bar[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(tfull_bar);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    // Warps q+2 and q+6 read TMEM lane quarter q (rows 32q..32q+31): the first takes the
    // lower half of the tile's columns, the second the upper half; the halves merge in
    // shared memory, then the first half continues alone.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;  // TMEM lane == tile row
    const int t = m0 + row;
    const bool have_acc = mbar_wait_bounded(tfull_bar, 0, a.status, kStatusTimeoutEpilogue, abort_flag, a.wait_ns);
    RTRACE(1);
    tc_fence_after();
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int col0 = chunk * a.bn;
    const int k = a.topk;
    const int split = min(a.bn, (a.bn / 2 + 15) / 16 * 16);
    const int c_begin = half ? split : 0, c_end = half ? a.bn : split;
    Top16 top;
    top.init();
    float gate = __int_as_float(0x7fc00000), sum = 0.f;
    if (have_acc) {
      for (int c0 = c_begin; c0 < c_end; c0 += 16) {
        float acc[16];
        uint32_t key[16];
        tmem_ld_32x32b_x16(t_row + c0, acc);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = col0 + c0 + i;
          const bool in = c0 + i < c_end;
          const uint32_t bits = bf16_bits_rne(acc[i] + (a.bias && in && e < a.experts ? __bfloat162float(a.bias[e]) : 0.f));
          key[i] = (in && e < a.experts) ? make_key(bits, e) : 0u;
          if (in && a.gate && e == a.experts) gate = bf16_bits_to_float(bits);
          if (a.logits && in && e <= a.experts - 1 + a.gate && t < a.tokens)
            a.logits[static_cast<size_t>(t) * a.logits_ld + e] = __ushort_as_bfloat16(static_cast<unsigned short>(bits));
        }
        sort16(key);
        top.merge_sorted(key);
      }
      RTRACE(2);
      if (a.mode == 1 && top.k[0] != 0u) {  // sum of exp over these columns, against their max
        const float mx = key_value(top.k[0]);
        for (int c0 = c_begin; c0 < c_end; c0 += 16) {
          float acc[16];
          tmem_ld_32x32b_x16(t_row + c0, acc);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = col0 + c0 + i;
            if (c0 + i < c_end && e < a.experts)
              sum += __expf(bf16_bits_to_float(bf16_bits_rne(acc[i] + (a.bias ? __bfloat162float(a.bias[e]) : 0.f))) - mx);
          }
        }
      }
    }
    // ---- merge the two column halves of each row
    if (half == 1) hrec.store(row, 0, sum, gate, top);
    epilogue_sync_all();
    if (half == 0) {
      hrec.merge_into(row, 0, sum, gate, top);
      if (a.nc > 1 && rank != 0) {
        // push this chunk's candidates into rank 0's slot `rank`, then one remote arrive
        const uint32_t base = map_to_rank(smem_u32(rec.sum), 0);
        const uint32_t slot_off = static_cast<uint32_t>(rank) * RBM + row;
        st_cluster_f32(base + slot_off * 4, sum);
        st_cluster_f32(base + (a.nc * RBM + slot_off) * 4, gate);
        const uint32_t key_base = base + 2 * a.nc * RBM * 4;
#pragma unroll
        for (int j = 0; j < kTop; ++j)
          st_cluster_u32(key_base + ((static_cast<uint32_t>(rank) * kTop + j) * RBM + row) * 4, top.k[j]);
        epilogue_sync_half();
        if (row == 0) mbar_arrive_remote(map_to_rank(smem_u32(merge_bar), 0));
      } else {
        bool merged_ok = true;
        if (a.nc > 1) {
          // wait (bounded) for the other ranks' candidates, then merge them
          if (row == 0) {
            const unsigned long long t0 = global_timer_ns();
            while (!mbar_try_wait_cluster(merge_bar, 0)) {
              if (global_timer_ns() - t0 > a.wait_ns) {
                if (a.status) atomicCAS(a.status, 0, kStatusTimeoutOther);
                *abort_flag = 1;
                break;
              }
            }
          }
          epilogue_sync_half();
          merged_ok = *abort_flag == 0;
          if (merged_ok)
            for (int c = 1; c < a.nc; ++c) rec.merge_into(row, c, sum, gate, top);
        }
        RTRACE(3);
        if (t < a.tokens) {
          const int stride = k + a.gate;
          int32_t* oi = a.indices + static_cast<size_t>(t) * stride;
          float* ow = a.weights + static_cast<size_t>(t) * stride;
          if (!have_acc || !merged_ok) {
            for (int j = 0; j < stride; ++j) {  // failed: route the token nowhere (ids skipped downstream)
              oi[j] = -1;
              ow[j] = 0.f;
            }
          } else {
            // mode 0: softmax over the k selected logits, rounded to bf16 (the logits' dtype);
            // mode 1: softmax over all experts, optionally renormalised over the k selected
            const float best = key_value(top.k[0]);
            float w[kTop];
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < kTop; ++j) {
              w[j] = 0.f;
              if (j < k) {  // k is uniform: a real branch, not predication
                w[j] = __expf(key_value(top.k[j]) - best);
                s += w[j];
              }
            }
            const float scale = a.mode == 0 ? 1.0f / s : (a.renorm ? 1.0f / s : 1.0f / sum);
#pragma unroll
            for (int j = 0; j < kTop; ++j) {
              if (j < k) {
                const float wj = a.mode == 0 ? bf16_bits_to_float(bf16_bits_rne(w[j] * scale)) : w[j] * scale;
                oi[j] = key_id(top.k[j]);
                ow[j] = wj;
              }
            }
            if (a.gate) {
              oi[k] = a.experts;
              ow[k] = 1.0f / (1.0f + __expf(-gate));
            }
          }
        }
      }
    }
  }

  RTRACE(4);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

cudaError_t launch_kernel(const CUtensorMap& mx, const CUtensorMap& mw, const RouterArgs& a, int m_tiles, size_t smem,
                          cudaStream_t stream) {
  static PerDeviceOnce attr;
  cudaError_t err = attr.run([] {
    return cudaFuncSetAttribute(router_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nc, m_tiles);
  cfg.blockDim = dim3(kRThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = a.nc;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, router_gemm_kernel, mx, mw, a);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace

RouterPlan router_plan(int tokens, int experts, int weight_rows, int gate, int topk) {
  RouterPlan p{};
  const int cols = experts + (gate ? 1 : 0);
  const int m_tiles = (tokens + RBM - 1) / RBM;
  int nc = (cols + 255) / 256;
  // split columns further while that fills more of the 148 SMs (cluster size <= 8)
  while (nc < 8 && (nc + 1) * m_tiles <= 148 && (cols + nc) / (nc + 1) >= 32) ++nc;
  int bn = (cols + nc - 1) / nc;
  bn = (bn + 15) / 16 * 16;
  if (bn < 16) bn = 16;
  p.nc = nc;
  p.bn = bn;
  p.kmax = 16;
  (void)topk;
  p.tmem_cols = 32;
  while (p.tmem_cols < bn) p.tmem_cols <<= 1;
  p.m_tiles = m_tiles;
  (void)weight_rows;
  return p;
}

cudaError_t launch_router_gemm(const void* x, int tokens, int hidden, const void* w, int weight_rows,
                               const void* bias, int experts, int topk, int mode, int renorm, int gate,
                               int32_t* indices, float* weights, void* logits, int* status, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  const RouterPlan p = router_plan(tokens, experts, weight_rows, gate, topk);
  CUtensorMap mx, mw;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(tokens)};
    const uint64_t strides[1] = {static_cast<uint64_t>(hidden) * 2};
    const uint32_t box[2] = {RBK, RBM};
    if (!encode_bf16_map(&mx, x, 2, dims, strides, box)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(weight_rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(hidden) * 2};
    const uint32_t box[2] = {RBK, static_cast<uint32_t>(p.bn)};
    if (!encode_bf16_map(&mw, w, 2, dims, strides, box)) return cudaErrorInvalidValue;
  }
  RouterArgs a{};
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.indices = indices;
  a.weights = weights;
  a.logits = static_cast<__nv_bfloat16*>(logits);
  a.status = status;
  a.wait_ns = wait_limit_ns(kWaitLimitNs);
  a.tokens = tokens;
  a.hidden = hidden;
  a.experts = experts;
  a.topk = topk;
  a.mode = mode;
  a.renorm = renorm;
  a.gate = gate ? 1 : 0;
  a.bn = p.bn;
  a.nc = p.nc;
  a.logits_ld = weight_rows;
  a.tmem_cols = p.tmem_cols;
  const size_t rec_bytes = static_cast<size_t>(p.nc + 1) * RBM * (2 + 16) * 4;  // cluster + half records
  const size_t fixed = 1024 + 256 + rec_bytes;
  const size_t per_stage = kRABytes + static_cast<size_t>(p.bn) * RBK * 2;
  int stages = static_cast<int>((227 * 1024 - fixed) / per_stage);
  if (stages > 6) stages = 6;
  if (stages < 2) return cudaErrorInvalidValue;
  a.stages = stages;
  return launch_kernel(mx, mw, a, p.m_tiles, fixed + stages * per_stage, stream);
}

}  // namespace cernels

#ifdef ROUTER_TRACE
extern "C" int cernels_debug_router_trace(unsigned long long* host, int rows) {
  return cudaMemcpyFromSymbol(host, cernels::g_router_trace, sizeof(unsigned long long) * 8 * rows) == cudaSuccess ? 0 : 4;
}
#endif
