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
constexpr int kRThreads = 192;
constexpr int kRABytes = RBM * RBK * 2;  // 16 KB

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
__device__ __forceinline__ void st_cluster_s32(uint32_t addr, int v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
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
// Named barrier over the four epilogue warps (barrier 1; warps 0-1 do not take part).
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// a ranks before b: larger value, ties to the lower expert id
__device__ __forceinline__ bool better(float av, int ai, float bv, int bi) {
  return av > bv || (av == bv && ai < bi);
}

template <int KMAX>
struct TopK {
  float v[KMAX];
  int id[KMAX];
  float kth_v;  // the k-th entry (kept apart so no register array is indexed at run time)
  int kth_id;
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      v[j] = -INFINITY;
      id[j] = 0x7fffffff;
    }
    kth_v = -INFINITY;
    kth_id = 0x7fffffff;
  }
  // Inserts (val, e) keeping the first k entries sorted best-first.
  __device__ __forceinline__ void insert(float val, int e, int k) {
    if (!better(val, e, kth_v, kth_id)) return;
    float cv = val;
    int ci = e;
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j < k && better(cv, ci, v[j], id[j])) {
        const float tv = v[j];
        const int ti = id[j];
        v[j] = cv;
        id[j] = ci;
        cv = tv;
        ci = ti;
      }
      if (j == k - 1) {
        kth_v = v[j];
        kth_id = id[j];
      }
    }
  }
};

// Per-row candidate records of the NC column chunks, structure-of-arrays in rank 0's shared
// memory: slot c holds chunk c's candidates.
template <int KMAX>
struct Records {
  float* mx;    // [nc][128]
  float* sum;   // [nc][128]
  float* gate;  // [nc][128] (NaN when the chunk has no gate column)
  float* v;     // [nc][KMAX][128]
  int* id;      // [nc][KMAX][128]
  __device__ Records(uint8_t* base, int nc) {
    mx = reinterpret_cast<float*>(base);
    sum = mx + nc * RBM;
    gate = sum + nc * RBM;
    v = gate + nc * RBM;
    id = reinterpret_cast<int*>(v + nc * KMAX * RBM);
  }
  __host__ __device__ static size_t bytes(int nc) { return static_cast<size_t>(nc) * RBM * (3 + 2 * KMAX) * 4; }
};

template <int KMAX>
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
  uint64_t* full_bar = bars;           // [S]
  uint64_t* empty_bar = bars + S;      // [S]
  uint64_t* tfull_bar = bars + 2 * S;  // [1]
  uint64_t* merge_bar = tfull_bar + 1; // [1] arrivals of the other cluster ranks
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(merge_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  Records<KMAX> rec(reinterpret_cast<uint8_t*>(bars) + 256, a.nc);

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
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane == tile row
    const int t = m0 + row;
    const bool have_acc = mbar_wait_bounded(tfull_bar, 0, a.status, kStatusTimeoutEpilogue, abort_flag, a.wait_ns);
    tc_fence_after();
    const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int col0 = chunk * a.bn;
    const int k = a.topk;
    TopK<KMAX> top;
    top.init();
    float mx = -INFINITY, gate = __int_as_float(0x7fc00000), sum = 0.f;
    if (have_acc) {
      for (int c0 = 0; c0 < a.bn; c0 += 32) {
        float acc[32];
        tmem_ld_32x32b_x32(t_row + c0, acc);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = c0 + i;
          const int e = col0 + c;
          if (c < a.bn) {
            if (e < a.experts) {
              const float l = bf16_round(acc[i] + (a.bias ? __bfloat162float(a.bias[e]) : 0.f));
              mx = fmaxf(mx, l);
              top.insert(l, e, k);
              if (a.logits && t < a.tokens) a.logits[static_cast<size_t>(t) * a.logits_ld + e] = __float2bfloat16_rn(l);
            } else if (a.gate && e == a.experts) {
              gate = bf16_round(acc[i]);
              if (a.logits && t < a.tokens) a.logits[static_cast<size_t>(t) * a.logits_ld + e] = __float2bfloat16_rn(gate);
            }
          }
        }
      }
      if (a.mode == 1) {  // sum of exp over this chunk's logits, against the chunk max
        for (int c0 = 0; c0 < a.bn; c0 += 32) {
          float acc[32];
          tmem_ld_32x32b_x32(t_row + c0, acc);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int e = col0 + c0 + i;
            if (c0 + i < a.bn && e < a.experts)
              sum += __expf(bf16_round(acc[i] + (a.bias ? __bfloat162float(a.bias[e]) : 0.f)) - mx);
          }
        }
      }
    }
    if (a.nc > 1 && rank != 0) {
      // push this chunk's candidates into rank 0's slot `rank`, then one remote arrive
      const uint32_t base = map_to_rank(smem_u32(rec.mx), 0);
      const uint32_t slot_off = static_cast<uint32_t>(rank) * RBM + row;
      const uint32_t mx_a = base + slot_off * 4;
      const uint32_t sum_a = base + (a.nc * RBM + slot_off) * 4;
      const uint32_t gate_a = base + (2 * a.nc * RBM + slot_off) * 4;
      st_cluster_f32(mx_a, mx);
      st_cluster_f32(sum_a, sum);
      st_cluster_f32(gate_a, gate);
      const uint32_t v_base = base + 3 * a.nc * RBM * 4;
      const uint32_t id_base = v_base + a.nc * KMAX * RBM * 4;
#pragma unroll
      for (int j = 0; j < KMAX; ++j) {
        const uint32_t off = ((static_cast<uint32_t>(rank) * KMAX + j) * RBM + row) * 4;
        st_cluster_f32(v_base + off, top.v[j]);
        st_cluster_s32(id_base + off, top.id[j]);
      }
      epilogue_sync();
      if (row == 0) mbar_arrive_remote(map_to_rank(smem_u32(merge_bar), 0));
    } else {
      bool merged_ok = true;
      if (a.nc > 1) {
        // wait (bounded) for the other ranks' candidates, then merge them in chunk order
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
        epilogue_sync();
        merged_ok = *abort_flag == 0;
        if (merged_ok) {
          float m_all = mx;
          for (int c = 1; c < a.nc; ++c) m_all = fmaxf(m_all, rec.mx[c * RBM + row]);
          float s_all = mx == -INFINITY ? 0.f : sum * __expf(mx - m_all);
          for (int c = 1; c < a.nc; ++c) {
            const float mc = rec.mx[c * RBM + row];
            if (mc != -INFINITY) s_all += rec.sum[c * RBM + row] * __expf(mc - m_all);
            const float gc = rec.gate[c * RBM + row];
            if (!isnan(gc)) gate = gc;
            for (int j = 0; j < k; ++j)
              top.insert(rec.v[(c * KMAX + j) * RBM + row], rec.id[(c * KMAX + j) * RBM + row], k);
          }
          mx = m_all;
          sum = s_all;
        }
      }
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
          float w[KMAX];
          float s = 0.f;
          if (a.mode == 0) {
            // softmax over the k selected logits, rounded to bf16 (the logits' dtype)
#pragma unroll
            for (int j = 0; j < KMAX; ++j) {
              w[j] = j < k ? __expf(top.v[j] - top.v[0]) : 0.f;
              s += w[j];
            }
#pragma unroll
            for (int j = 0; j < KMAX; ++j) w[j] = bf16_round(w[j] / s);
          } else {
#pragma unroll
            for (int j = 0; j < KMAX; ++j) {
              w[j] = j < k ? __expf(top.v[j] - mx) / sum : 0.f;
              s += w[j];
            }
            if (a.renorm) {
#pragma unroll
              for (int j = 0; j < KMAX; ++j) w[j] = w[j] / s;
            }
          }
#pragma unroll
          for (int j = 0; j < KMAX; ++j) {
            if (j < k) {
              oi[j] = top.id[j];
              ow[j] = w[j];
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

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

template <int KMAX>
cudaError_t launch_k(const CUtensorMap& mx, const CUtensorMap& mw, const RouterArgs& a, int m_tiles, size_t smem,
                     cudaStream_t stream) {
  static PerDeviceOnce attr;
  cudaError_t err = attr.run([] {
    return cudaFuncSetAttribute(router_gemm_kernel<KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
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
  err = cudaLaunchKernelEx(&cfg, router_gemm_kernel<KMAX>, mx, mw, a);
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
  p.kmax = topk <= 4 ? 4 : topk <= 8 ? 8 : 16;
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
  const size_t rec_bytes = static_cast<size_t>(p.nc) * RBM * (3 + 2 * p.kmax) * 4;
  const size_t fixed = 1024 + 256 + rec_bytes;
  const size_t per_stage = kRABytes + static_cast<size_t>(p.bn) * RBK * 2;
  int stages = static_cast<int>((227 * 1024 - fixed) / per_stage);
  if (stages > 6) stages = 6;
  if (stages < 2) return cudaErrorInvalidValue;
  a.stages = stages;
  const size_t smem = fixed + stages * per_stage;
  switch (p.kmax) {
    case 4: return launch_k<4>(mx, mw, a, p.m_tiles, smem, stream);
    case 8: return launch_k<8>(mx, mw, a, p.m_tiles, smem, stream);
    default: return launch_k<16>(mx, mw, a, p.m_tiles, smem, stream);
  }
}

}  // namespace cernels
