// Expert-parallel dispatch / return over NVLink peer memory (no NCCL, no host sync).
//
// The reference is single-GPU; expert parallelism is this build's multi-GPU scheme. Each
// rank owns one device window (cudaMalloc), mapped into every other rank's address space
// with CUDA IPC:
//   hdr[R]          one EpHeader per peer rank (its counts and flags for this rank)
//   recv[R*cap][H]  rows routed to this rank's experts, expert-contiguous: all sources' rows of
//                   local expert 0 (source 0 first), then expert 1, ...
//   back[cap][H]    expert outputs of this rank's own routed rows, written by their owners
// One step (epoch e; kernels on the caller's stream unless marked "side"):
//   ep_counts    source, one CTA per destination d: writes its per-expert row counts into
//                d.hdr[me], release-stores count_epoch = e, waits (acquire, bounded) until
//                every source's counts for e are in d's window, and computes where its rows
//                of each expert start in d's receive region
//   ep_dispatch  (side stream) source: copies its rows for the other ranks, expert by expert,
//                and release-stores d.hdr[me].arrived[e] = e once all its rows of (d, e) are in
//   ep_dispatch  source: copies its rows for itself (in stream order before its GEMMs)
//   ep_segments  destination: grouped-GEMM tables from the counts (one group per local expert,
//                all sources' rows contiguous: no partial tiles between sources)
//   ep_rowmap    destination: the return address (source's back row) of every received row
//   gate/up grouped GEMM (tcgen05/TMA on recv, in place): before the first tile of expert e its
//                producer waits (bounded) for arrived[e] == e from every other source, so the
//                GEMMs of early experts overlap the transfer of later ones
//   down grouped GEMM: its epilogue stores each result row straight into its source's back
//                region over NVLink
//   ep_results   destination: release-stores s.hdr[me].result_epoch = e for every source
//   ep_combine   source (after joining the side stream): waits (acquire, bounded) for
//                result_epoch == e from every destination,
//                out[t] = bf16(sum_j w[t, j] * back[inv[t, j]]) in slot order
// The side-stream copy kernel waits for nothing, and its CTAs fit beside a resident GEMM CTA
// (little shared memory, 256 threads), so the GEMMs that wait on other ranks' copies never
// keep this rank's copies from running.
// A rank starts step e+1 only after its combine of step e saw every destination's results,
// and a destination signals results only after its GEMMs finished reading recv, so no slot
// or header is overwritten while in use. Loads and stores are plain accesses (no TMA and no
// multicast on peer memory). Every wait gives up after a limit (5 s unless
// cernels_set_wait_limit_ns set another) and records a status.
#include <cstdio>
#include <cstddef>
#include <cstdlib>
#include <cstring>

#include "moe_internal.h"
#include "sm100_primitives.cuh"

namespace cernels {
namespace {

constexpr int kEpMaxRanks = 16;
constexpr int kEpMaxLocalExperts = 512;
constexpr unsigned long long kEpWaitNs = 5000000000ull;
constexpr int kEpThreads = 256;

struct __align__(256) EpHeader {
  int32_t counts[kEpMaxLocalExperts];  // rows per local expert sent by this peer
  int32_t seg_start;                   // first routed row of this segment at the source
  int32_t n_rows;                      // rows in the segment
  uint32_t count_epoch;                // counts above are those of this step (written by the source)
  uint32_t result_epoch;               // written by the destination (source's window)
  uint32_t arrived[kEpMaxLocalExperts];  // arrived[e] == epoch: all of this source's rows of expert e are in
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *flag == epoch. Returns false (and records `code`) on timeout.
__device__ bool wait_epoch(const uint32_t* flag, uint32_t epoch, int* status, int code, unsigned long long limit_ns) {
  if (ld_acquire_sys(flag) == epoch) return true;
  const unsigned long long t0 = global_timer_ns();
  while (ld_acquire_sys(flag) != epoch) {
    if (global_timer_ns() - t0 > limit_ns) {
      atomicCAS(status, 0, code);
      return false;
    }
  }
  return true;
}

// The epoch of the current step: an explicit nonzero argument, or (argument 0) one past the
// last step this rank completed, kept in device memory so that a step can be replayed from a
// CUDA graph.
__device__ __forceinline__ uint32_t step_epoch(const uint32_t* epoch_dev, uint32_t arg) {
  return arg ? arg : *reinterpret_cast<const volatile uint32_t*>(epoch_dev) + 1u;
}

// Copies one row of `vec` 16-byte pieces with the whole warp: up to 8 loads per lane in flight
// before their stores.
__device__ __forceinline__ void copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int vec, int lane) {
  for (int v0 = 0; v0 < vec; v0 += 32 * 8) {
    uint4 r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int v = v0 + j * 32 + lane;
      if (v < vec) r[j] = __ldcs(src + v);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int v = v0 + j * 32 + lane;
      if (v < vec) __stcs(dst + v, r[j]);  // streaming: the copy is not re-read from this L2
    }
  }
}

__device__ __forceinline__ EpHeader* hdr_of(uint8_t* window, int peer) {
  return reinterpret_cast<EpHeader*>(window) + peer;
}

struct EpGeometry {
  int rank, world, local_experts, cap, hidden;
  int shared_cap;  // rows reserved after the routed ones for an always-on local (shared) expert
  size_t recv_offset, back_offset;
  unsigned long long wait_ns;  // limit of each bounded wait
};

// Marks this CTA done; the last CTA of the grid returns true (counter reset for the next launch).
__device__ bool last_cta_done(unsigned* counter) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(counter, 1u);
    last = old == gridDim.x - 1;
    if (last) *counter = 0u;
  }
  __syncthreads();
  return last != 0;
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024); returns the thread's
// exclusive prefix and writes the block total to *total.
__device__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
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
    const int nw = (blockDim.x + 31) >> 5;
    const int wv = lane < nw ? warp_tot[lane] : 0;
    int wi = wv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    warp_tot[lane] = wi - wv;
    if (lane == 31) warp_tot[32] = wi;
  }
  __syncthreads();
  const int excl = warp_tot[warp] + incl - v;
  *total = warp_tot[32];
  __syncthreads();
  return excl;
}

// Step 1 of a dispatch, one CTA per destination d: publish this rank's per-expert row counts in
// d's window, wait (bounded) until every source has published its counts for this step, and
// compute where this rank's rows go in d's expert-contiguous receive region:
//   dest_off[d][e] = rows of d's experts < e from all sources + rows of expert e from sources < me.
__global__ void __launch_bounds__(kEpThreads) ep_counts_kernel(uint8_t* const* __restrict__ peers, EpGeometry g,
                                                               const int* __restrict__ offsets, uint32_t epoch_arg,
                                                               const uint32_t* epoch_dev, int* __restrict__ dest_off,
                                                               int* __restrict__ done, int* status) {
  const uint32_t epoch = step_epoch(epoch_dev, epoch_arg);
  for (int e = threadIdx.x; e < g.local_experts; e += blockDim.x) done[blockIdx.x * kEpMaxLocalExperts + e] = 0;
  __shared__ int cnt[kEpMaxLocalExperts];  // per expert: rows from all sources
  __shared__ int before[kEpMaxLocalExperts];  // per expert: rows from sources < me
  __shared__ int warp_tot[33];
  __shared__ int ok;
  const int d = blockIdx.x, El = g.local_experts;
  EpHeader* h = hdr_of(peers[d], g.rank);
  for (int e = threadIdx.x; e < El; e += blockDim.x) h->counts[e] = offsets[d * El + e + 1] - offsets[d * El + e];
  if (threadIdx.x == 0) {
    h->seg_start = offsets[d * El];
    h->n_rows = offsets[(d + 1) * El] - offsets[d * El];
    ok = 1;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) st_release_sys(&h->count_epoch, epoch);
  if (threadIdx.x < g.world)
    if (!wait_epoch(&hdr_of(peers[d], threadIdx.x)->count_epoch, epoch, status, kStatusTimeoutOther, g.wait_ns))
      ok = 0;
  __syncthreads();
  for (int e = threadIdx.x; e < El; e += blockDim.x) {
    int tot = 0, bef = 0;
    if (ok)
      for (int s = 0; s < g.world; ++s) {
        const int c = __ldcv(&hdr_of(peers[d], s)->counts[e]);
        tot += c;
        if (s < g.rank) bef += c;
      }
    cnt[e] = tot;
    before[e] = bef;
  }
  __syncthreads();
  int carry = 0;
  for (int e0 = 0; e0 < El; e0 += blockDim.x) {
    const int e = e0 + threadIdx.x;
    int total = 0;
    const int excl = block_exclusive_scan(e < El ? cnt[e] : 0, warp_tot, &total);
    if (e < El) dest_off[d * kEpMaxLocalExperts + e] = carry + excl + before[e];
    carry += total;
  }
}

// Step 2: copy every routed row x[perm_token[p]] to its slot in its owner's receive region.
// `remote` selects the destinations: every other rank (run on a side stream, concurrently with
// the owner-side GEMMs that consume the rows) or this rank alone (in stream order before them).
// Work is ordered by local expert, so that every destination receives all of expert 0's rows
// first, then expert 1's, ...; inside an expert it is interleaved over destinations starting at
// rank + 1. When the last row of (destination d, expert e) has been written (a per-(d, e) row
// counter, after a system-scope fence by the writing warp), d.hdr[me].arrived[e] is
// release-stored with the epoch; the owner's GEMM waits on these flags per expert.
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(uint8_t* const* __restrict__ peers, EpGeometry g,
                                                                 const uint4* __restrict__ x,
                                                                 const int* __restrict__ perm_token,
                                                                 const int* __restrict__ offsets,
                                                                 const int* __restrict__ dest_off, uint32_t epoch_arg,
                                                                 const uint32_t* epoch_dev, int* __restrict__ done,
                                                                 int remote, int shared_tokens, int* status) {
  __shared__ int item_prefix[kEpMaxLocalExperts + 1];
  __shared__ int warp_tot[33];
  const uint32_t epoch = step_epoch(epoch_dev, epoch_arg);
  const int El = g.local_experts, R = g.world;
  const int nd = remote ? R - 1 : 1;  // destinations served
  // items of expert e: (most rows any served destination gets of e) x nd
  int carry = 0;
  for (int e0 = 0; e0 < El; e0 += blockDim.x) {
    const int e = e0 + threadIdx.x;
    int items = 0;
    if (e < El && nd > 0) {
      int mx = 0;
      for (int j = 0; j < nd; ++j) {
        const int d = remote ? (g.rank + 1 + j) % R : g.rank;
        mx = max(mx, offsets[d * El + e + 1] - offsets[d * El + e]);
      }
      items = mx * nd;
    }
    int total = 0;
    const int excl = block_exclusive_scan(items, warp_tot, &total);
    if (e < El) item_prefix[e] = carry + excl;
    carry += total;
  }
  if (threadIdx.x == 0) item_prefix[El] = carry;
  __syncthreads();
  const int vec = g.hidden / 8;
  const long long cap_rows = static_cast<long long>(R) * g.cap;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int n_warps = (gridDim.x * blockDim.x) >> 5;
  for (int q = warp; q < carry; q += n_warps) {
    int e = 0, hi = El - 1;  // expert: last e with item_prefix[e] <= q
    while (e < hi) {
      const int m = (e + hi + 1) >> 1;
      if (item_prefix[m] <= q) e = m; else hi = m - 1;
    }
    const int r = q - item_prefix[e];
    const int i = r / nd;
    const int d = remote ? (g.rank + 1 + r % nd) % R : g.rank;
    const int lo = offsets[d * El + e];
    const int n_de = offsets[d * El + e + 1] - lo;
    if (i >= n_de) continue;
    const long long dst_row = static_cast<long long>(dest_off[d * kEpMaxLocalExperts + e]) + i;
    if (dst_row >= 0 && dst_row < cap_rows) {  // cannot fail with consistent counts; never overrun
      copy_row(reinterpret_cast<uint4*>(peers[d] + g.recv_offset) + static_cast<size_t>(dst_row) * vec,
               x + static_cast<size_t>(perm_token[lo + i]) * vec, vec, lane);
    } else if (lane == 0) {
      atomicCAS(status, 0, kStatusTimeoutOther);
    }
    if (remote) {
      __threadfence_system();
      __syncwarp();
      if (lane == 0 && atomicAdd(&done[d * kEpMaxLocalExperts + e], 1) == n_de - 1) {
        __threadfence_system();
        st_release_sys(&hdr_of(peers[d], g.rank)->arrived[e], epoch);
      }
    }
  }
  // this rank's own rows for its shared expert: x[t] -> recv[world * cap + t]
  if (!remote)
    for (int t = warp; t < min(shared_tokens, g.shared_cap); t += n_warps)
      copy_row(reinterpret_cast<uint4*>(peers[g.rank] + g.recv_offset) + (cap_rows + t) * vec,
               x + static_cast<size_t>(t) * vec, vec, lane);
  // (destination, expert) pairs with no rows at all are complete from the start
  if (remote && blockIdx.x == 0)
    for (int idx = threadIdx.x; idx < nd * El; idx += blockDim.x) {
      const int d = (g.rank + 1 + idx / El) % R, e = idx % El;
      if (offsets[d * El + e + 1] == offsets[d * El + e]) st_release_sys(&hdr_of(peers[d], g.rank)->arrived[e], epoch);
    }
}

// One CTA of 1024 threads at the destination: the grouped-GEMM tables (group = local expert, rows of all sources contiguous) and, per source, the prefix of
// its segment by expert (for the return).
//   offsets[e], mtile_offsets[e]  (El + 1 entries)
//   src_prefix[s][e]              rows of source s's segment before expert e (El + 1 entries)
//   run_start[e][s]               first receive row of source s's rows of expert e
__global__ void __launch_bounds__(1024) ep_segments_kernel(uint8_t* __restrict__ window, EpGeometry g,
                                                           uint32_t epoch_arg, const uint32_t* epoch_dev,
                                                           int* __restrict__ offsets, int* __restrict__ group_rows,
                                                           int* __restrict__ mtile_offsets,
                                                           int* __restrict__ src_prefix, int* __restrict__ run_start,
                                                           int shared_tokens, int* status) {
  const uint32_t epoch = step_epoch(epoch_dev, epoch_arg);
  __shared__ int ok;
  __shared__ int warp_tot[33];
  const int El = g.local_experts, R = g.world;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  // the counts of this step are in place (ep_counts waited for them); the rows may still be on
  // their way: the GEMM waits for them per expert
  if (threadIdx.x < R)
    if (!wait_epoch(&hdr_of(window, threadIdx.x)->count_epoch, epoch, status, kStatusTimeoutOther, g.wait_ns)) ok = 0;
  __syncthreads();
  const long long cap_rows = static_cast<long long>(R) * g.cap;
  int carry_rows = 0, carry_tiles = 0;
  for (int e0 = 0; e0 < El; e0 += blockDim.x) {
    const int e = e0 + threadIdx.x;
    int rows = 0;
    if (e < El && ok)
      for (int s = 0; s < R; ++s) rows += max(hdr_of(window, s)->counts[e], 0);
    int total_rows = 0, total_tiles = 0;
    const int row_excl = block_exclusive_scan(rows, warp_tot, &total_rows);
    const int tiles = (rows + kBlockM - 1) / kBlockM;
    const int tile_excl = block_exclusive_scan(tiles, warp_tot, &total_tiles);
    if (e < El) {
      // clamp so that a bad header can never make the GEMM read past the receive region
      const long long start = min(static_cast<long long>(carry_rows + row_excl), cap_rows);
      offsets[e] = static_cast<int>(start);
      group_rows[e] = static_cast<int>(min(static_cast<long long>(rows), cap_rows - start));
      mtile_offsets[e] = carry_tiles + tile_excl;
      int r = static_cast<int>(start);
      for (int s = 0; s < R; ++s) {
        run_start[e * R + s] = r;
        r += ok ? max(hdr_of(window, s)->counts[e], 0) : 0;
      }
    }
    carry_rows += total_rows;
    carry_tiles += total_tiles;
  }
  for (int s = threadIdx.x; s < R; s += blockDim.x) {
    int acc = 0;
    for (int e = 0; e < El; ++e) {
      src_prefix[s * (El + 1) + e] = acc;
      acc += ok ? max(hdr_of(window, s)->counts[e], 0) : 0;
    }
    src_prefix[s * (El + 1) + El] = acc;
  }
  if (threadIdx.x == 0) {
    // group El, when present: this rank's own tokens for its shared expert, after the routed capacity
    const int sh = min(shared_tokens, g.shared_cap);
    offsets[El] = static_cast<int>(cap_rows);
    group_rows[El] = sh;
    mtile_offsets[El] = carry_tiles;
    mtile_offsets[El + 1] = carry_tiles + (sh + kBlockM - 1) / kBlockM;
  }
}

// Destination, before the down GEMM: the return address of every received row. Receive row r
// belongs to (expert e, source s): it is source s's segment row i = src_prefix[s][e] +
// (r - run_start[e][s]), whose result goes to s.back[seg_start + i]. The down GEMM's epilogue
// stores each result row straight there (NVLink peer stores), so no separate return pass runs.
__global__ void __launch_bounds__(kEpThreads) ep_rowmap_kernel(uint8_t* const* __restrict__ peers, EpGeometry g,
                                                               const int* __restrict__ offsets,
                                                               const int* __restrict__ group_rows,
                                                               const int* __restrict__ src_prefix,
                                                               const int* __restrict__ run_start,
                                                               __nv_bfloat16** __restrict__ row_out) {
  uint8_t* own = peers[g.rank];
  const int El = g.local_experts, R = g.world;
  const int total = offsets[El - 1] + group_rows[El - 1];  // routed rows (contiguous from 0)
  // shared-expert rows: results of this rank's own tokens go to back[cap + t]
  const long long cap_rows = static_cast<long long>(R) * g.cap;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < group_rows[El] && g.shared_cap > 0;
       t += gridDim.x * blockDim.x)
    row_out[cap_rows + t] = reinterpret_cast<__nv_bfloat16*>(own + g.back_offset) +
                            static_cast<size_t>(g.cap + t) * g.hidden;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < total; r += gridDim.x * blockDim.x) {
    int a = 0, b = El - 1;  // expert: last e with offsets[e] <= r
    while (a < b) {
      const int m = (a + b + 1) >> 1;
      if (offsets[m] <= r) a = m; else b = m - 1;
    }
    int s = R - 1;  // source: last s with run_start[a][s] <= r
    while (s > 0 && run_start[a * R + s] > r) --s;
    const int i = src_prefix[s * (El + 1) + a] + (r - run_start[a * R + s]);
    // headers come from another rank: clamp to the windows so a bad value cannot overrun them
    const int base = min(max(hdr_of(own, s)->seg_start, 0), g.cap);
    row_out[r] = (i >= 0 && base + i < g.cap)
                     ? reinterpret_cast<__nv_bfloat16*>(peers[s] + g.back_offset) + static_cast<size_t>(base + i) * g.hidden
                     : nullptr;
  }
}

// Destination, after the down GEMM (whose threads fenced their peer stores system-wide before
// the kernel ended): tell every source that its results for this step are in place.
__global__ void ep_results_kernel(uint8_t* const* __restrict__ peers, EpGeometry g, uint32_t epoch_arg,
                                  const uint32_t* epoch_dev) {
  const uint32_t epoch = step_epoch(epoch_dev, epoch_arg);
  __threadfence_system();
  if (threadIdx.x < g.world) st_release_sys(&hdr_of(peers[threadIdx.x], g.rank)->result_epoch, epoch);
}

// Last kernel of a step: with the device-side epoch (argument 0), its last CTA records the step
// as completed.
__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(uint8_t* __restrict__ window, EpGeometry g,
                                                                uint32_t epoch_arg, uint32_t* epoch_dev,
                                                                unsigned* __restrict__ counter,
                                                                const int* __restrict__ inv,
                                                                const float* __restrict__ weights, int tokens,
                                                                int topk, int shared, uint4* __restrict__ out,
                                                                int* status) {
  const uint32_t epoch = step_epoch(epoch_dev, epoch_arg);
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < g.world)
    if (!wait_epoch(&hdr_of(window, threadIdx.x)->result_epoch, epoch, status, kStatusTimeoutOther, g.wait_ns)) ok = 0;
  __syncthreads();
  const uint4* back = reinterpret_cast<const uint4*>(window + g.back_offset);
  const int vec = g.hidden / 8;
  const int warps = blockDim.x >> 5;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < tokens; t += gridDim.x * warps) {
    for (int v = threadIdx.x & 31; v < vec; v += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < topk && ok; ++j) {
        // with a shared expert, the last slot's row is this token's shared-expert result
        const int p = (shared && j == topk - 1) ? g.cap + t : inv[static_cast<size_t>(t) * topk + j];
        if (p < 0) continue;
        const uint4 r = __ldcv(back + static_cast<size_t>(p) * vec + v);
        const float w = weights[static_cast<size_t>(t) * topk + j];
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h2[q]);
          acc[2 * q] = fmaf(w, f.x, acc[2 * q]);
          acc[2 * q + 1] = fmaf(w, f.y, acc[2 * q + 1]);
        }
      }
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) oh[q] = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      out[static_cast<size_t>(t) * vec + v] = o;
    }
  }
  if (epoch_arg == 0 && last_cta_done(counter) && threadIdx.x == 0) *epoch_dev = epoch;
}

}  // namespace
}  // namespace cernels

using namespace cernels;

struct cernels_ep_ctx {
  EpGeometry geo;
  int device;
  size_t window_bytes;
  uint8_t* window;
  uint8_t* peers[kEpMaxRanks];
  uint8_t** d_peers;
  unsigned* d_counters;  // [0] dispatch, [1] return, [2] combine, [3] last completed epoch
  int* d_status;
  int* d_dest_off;       // [kEpMaxRanks][kEpMaxLocalExperts] this rank's write offsets per destination
  int* d_done;           // [kEpMaxRanks][kEpMaxLocalExperts] rows written per (destination, expert)
  cudaStream_t side;     // remote dispatch, concurrent with the owner-side work of the step
  cudaEvent_t ev_counts, ev_dispatched;
  bool connected;
};

namespace {

int rc_of(cudaError_t e) {
  if (e == cudaSuccess) return CERNELS_OK;
  std::fprintf(stderr, "cernels_b200 ep: CUDA error: %s\n", cudaGetErrorString(e));
  return CERNELS_E_CUDA;
}

// The geometry handed to a kernel, with the current wait limit.
EpGeometry geo_now(const cernels_ep_ctx* c) {
  EpGeometry g = c->geo;
  g.wait_ns = wait_limit_ns(kEpWaitNs);
  return g;
}

// CTAs of a row-copy kernel: 8 warps per CTA, a row per warp, at most `per_sm` CTAs per SM
// (CERNELS_EP_CTAS_PER_SM overrides the default of 4, for tuning).
int ep_grid(int rows) {
  static const int per_sm = [] {
    const char* v = std::getenv("CERNELS_EP_CTAS_PER_SM");
    const int n = v ? std::atoi(v) : 0;
    return n > 0 ? n : 4;
  }();
  const int sms = device_sm_count();
  const int want = (rows + 7) / 8;
  return want < 1 ? 1 : (want < per_sm * sms ? want : per_sm * sms);
}

}  // namespace

extern "C" {

int cernels_ep_create(int32_t rank, int32_t world, int32_t hidden, int32_t local_experts, int32_t max_rows,
                      int32_t shared_rows, void** ctx_out, void* handle_out) {
  if (!ctx_out || !handle_out) return CERNELS_E_NULL;
  if (world < 1 || world > kEpMaxRanks || rank < 0 || rank >= world) return CERNELS_E_INVALID_SHAPE;
  if (hidden <= 0 || hidden % 8 || local_experts <= 0 || local_experts > kEpMaxLocalExperts || max_rows <= 0 ||
      shared_rows < 0)
    return CERNELS_E_INVALID_SHAPE;
  if (world * local_experts > kMaxExperts) return CERNELS_E_UNSUPPORTED;
  auto* c = new cernels_ep_ctx();
  std::memset(c, 0, sizeof(*c));
  cudaGetDevice(&c->device);
  c->geo.rank = rank;
  c->geo.world = world;
  c->geo.local_experts = local_experts;
  c->geo.cap = max_rows;
  c->geo.hidden = hidden;
  const size_t hdr = align_up(sizeof(EpHeader) * world, 1024);
  const size_t row = static_cast<size_t>(hidden) * 2;
  c->geo.recv_offset = hdr;
  c->geo.shared_cap = shared_rows;
  c->geo.back_offset = align_up(hdr + (static_cast<size_t>(world) * max_rows + shared_rows) * row, 1024);
  c->window_bytes = c->geo.back_offset + (static_cast<size_t>(max_rows) + shared_rows) * row;
  cudaError_t err = cudaMalloc(&c->window, c->window_bytes);
  if (err == cudaSuccess) err = cudaMemset(c->window, 0, c->geo.recv_offset);
  if (err == cudaSuccess) err = cudaMalloc(&c->d_peers, sizeof(uint8_t*) * kEpMaxRanks);
  if (err == cudaSuccess) err = cudaMalloc(&c->d_counters, 4 * sizeof(unsigned) + sizeof(int));
  if (err == cudaSuccess) err = cudaMemset(c->d_counters, 0, 4 * sizeof(unsigned) + sizeof(int));
  if (err == cudaSuccess) err = cudaMalloc(&c->d_dest_off, sizeof(int) * kEpMaxRanks * kEpMaxLocalExperts);
  if (err == cudaSuccess) err = cudaMalloc(&c->d_done, sizeof(int) * kEpMaxRanks * kEpMaxLocalExperts);
  if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking);
  if (err == cudaSuccess) err = cudaEventCreateWithFlags(&c->ev_counts, cudaEventDisableTiming);
  if (err == cudaSuccess) err = cudaEventCreateWithFlags(&c->ev_dispatched, cudaEventDisableTiming);
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), c->window);
  if (err != cudaSuccess) {
    if (c->window) cudaFree(c->window);
    if (c->d_peers) cudaFree(c->d_peers);
    if (c->d_counters) cudaFree(c->d_counters);
    if (c->d_dest_off) cudaFree(c->d_dest_off);
    if (c->d_done) cudaFree(c->d_done);
    if (c->side) cudaStreamDestroy(c->side);
    if (c->ev_counts) cudaEventDestroy(c->ev_counts);
    if (c->ev_dispatched) cudaEventDestroy(c->ev_dispatched);
    delete c;
    return rc_of(err);
  }
  c->d_status = reinterpret_cast<int*>(c->d_counters + 4);
  c->peers[rank] = c->window;
  *ctx_out = c;
  return CERNELS_OK;
}

int cernels_ep_connect(void* ctx, const void* handles) {
  auto* c = static_cast<cernels_ep_ctx*>(ctx);
  if (!c || !handles) return CERNELS_E_NULL;
  const auto* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < c->geo.world; ++r) {
    if (r == c->geo.rank) continue;
    void* p = nullptr;
    const cudaError_t err = cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return rc_of(err);
    c->peers[r] = static_cast<uint8_t*>(p);
  }
  const cudaError_t err =
      cudaMemcpy(c->d_peers, c->peers, sizeof(uint8_t*) * kEpMaxRanks, cudaMemcpyHostToDevice);
  if (err != cudaSuccess) return rc_of(err);
  c->connected = true;
  return CERNELS_OK;
}

int cernels_ep_destroy(void* ctx) {
  auto* c = static_cast<cernels_ep_ctx*>(ctx);
  if (!c) return CERNELS_OK;
  for (int r = 0; r < c->geo.world; ++r)
    if (r != c->geo.rank && c->peers[r]) cudaIpcCloseMemHandle(c->peers[r]);
  cudaFree(c->window);
  cudaFree(c->d_peers);
  cudaFree(c->d_counters);
  cudaFree(c->d_dest_off);
  cudaFree(c->d_done);
  cudaStreamDestroy(c->side);
  cudaEventDestroy(c->ev_counts);
  cudaEventDestroy(c->ev_dispatched);
  delete c;
  return CERNELS_OK;
}

int cernels_ep_dispatch(void* ctx, const void* x, const int32_t* perm_token, const int32_t* offsets, int32_t rows,
                        int32_t shared_tokens, uint32_t epoch, void* stream) {
  auto* c = static_cast<cernels_ep_ctx*>(ctx);
  if (!c || !c->connected) return CERNELS_E_NULL;
  if (rows > c->geo.cap || shared_tokens < 0 || shared_tokens > c->geo.shared_cap) return CERNELS_E_UNSUPPORTED;
  if (rows > 0 && (!x || !perm_token || !offsets)) return CERNELS_E_NULL;
  if (x && (reinterpret_cast<uintptr_t>(x) & 15)) return CERNELS_E_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const EpGeometry g = geo_now(c);
  ep_counts_kernel<<<c->geo.world, kEpThreads, 0, st>>>(c->d_peers, g, offsets, epoch, c->d_counters + 3,
                                                        c->d_dest_off, c->d_done, c->d_status);
  cudaError_t err = cudaGetLastError();
  // rows for the other ranks go out on the side stream while this rank's own rows are copied
  // and its experts run on `stream` (cernels_ep_combine joins the side stream back)
  if (err == cudaSuccess) err = cudaEventRecord(c->ev_counts, st);
  if (err == cudaSuccess) err = cudaStreamWaitEvent(c->side, c->ev_counts, 0);
  if (err != cudaSuccess) return rc_of(err);
  static const bool overlap = [] {
    const char* v = std::getenv("CERNELS_EP_OVERLAP");  // 0: send on `stream` first (no overlap; for A/B)
    return !(v && v[0] == '0');
  }();
  if (c->geo.world > 1)
    ep_dispatch_kernel<<<ep_grid(rows), kEpThreads, 0, overlap ? c->side : st>>>(c->d_peers, g, static_cast<const uint4*>(x),
                                                                 perm_token, offsets, c->d_dest_off, epoch,
                                                                 c->d_counters + 3, c->d_done, 1, 0, c->d_status);
  if ((err = cudaEventRecord(c->ev_dispatched, c->side)) != cudaSuccess) return rc_of(err);
  ep_dispatch_kernel<<<ep_grid(rows / c->geo.world + shared_tokens + 1), kEpThreads, 0, st>>>(
      c->d_peers, g, static_cast<const uint4*>(x), perm_token, offsets, c->d_dest_off, epoch, c->d_counters + 3,
      c->d_done, 0, shared_tokens, c->d_status);
  return rc_of(cudaGetLastError());
}

namespace {
// Tables of the receive side, carved out of the experts workspace.
struct EpTables {
  int *offsets, *group_rows, *mtile, *src_prefix, *run_start;
  __nv_bfloat16** row_out;  // [rows] return address of each received row's result
  __nv_bfloat16* glu;
};
size_t ep_tables(const cernels_ep_ctx* c, int inter, uint8_t* base, EpTables* t) {
  const size_t rows = static_cast<size_t>(c->geo.world) * c->geo.cap + c->geo.shared_cap;
  const size_t El = c->geo.local_experts, R = c->geo.world;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = align_up(off, 256);
    uint8_t* p = base ? base + off : nullptr;
    off += bytes;
    return p;
  };
  uint8_t* p_off = take((El + 2) * 4);
  uint8_t* p_gr = take((El + 2) * 4);
  uint8_t* p_mt = take((El + 2) * 4);
  uint8_t* p_pre = take(R * (El + 1) * 4);
  uint8_t* p_run = take(R * El * 4);
  uint8_t* p_rows = take(rows * sizeof(void*));
  uint8_t* p_glu = take(rows * inter * 2);
  if (t) {
    t->offsets = reinterpret_cast<int*>(p_off);
    t->group_rows = reinterpret_cast<int*>(p_gr);
    t->mtile = reinterpret_cast<int*>(p_mt);
    t->src_prefix = reinterpret_cast<int*>(p_pre);
    t->run_start = reinterpret_cast<int*>(p_run);
    t->row_out = reinterpret_cast<__nv_bfloat16**>(p_rows);
    t->glu = reinterpret_cast<__nv_bfloat16*>(p_glu);
  }
  return off + 256;
}
}  // namespace

int cernels_ep_experts_workspace_bytes(void* ctx, const cernels_moe_shape* shape, size_t* bytes) {
  auto* c = static_cast<cernels_ep_ctx*>(ctx);
  if (!c || !shape || !bytes) return CERNELS_E_NULL;
  *bytes = ep_tables(c, shape->intermediate, nullptr, nullptr);
  return CERNELS_OK;
}

int cernels_ep_experts(void* ctx, const cernels_moe_shape* shape, const void* gate_up_proj, const float* gate_up_bias,
                       const void* down_proj, const float* down_bias, const void* shared_gate_up_proj,
                       const void* shared_down_proj, int32_t shared_tokens, uint32_t epoch, void* workspace,
                       size_t workspace_bytes, void* stream_ptr) {
  auto* c = static_cast<cernels_ep_ctx*>(ctx);
  if (!c || !c->connected || !shape || !gate_up_proj || !down_proj || !workspace) return CERNELS_E_NULL;
  const cernels_moe_shape s = *shape;
  if (s.hidden != c->geo.hidden || s.experts != c->geo.local_experts || s.intermediate <= 0 ||
      s.intermediate % 8)
    return CERNELS_E_INVALID_SHAPE;
  if (workspace_bytes < ep_tables(c, s.intermediate, nullptr, nullptr)) return CERNELS_E_WORKSPACE;
  const bool shared = shared_tokens > 0;
  if (shared_tokens < 0 || shared_tokens > c->geo.shared_cap) return CERNELS_E_UNSUPPORTED;
  if (shared && (!shared_gate_up_proj || !shared_down_proj)) return CERNELS_E_NULL;
  if (shared && s.layout != CERNELS_LAYOUT_LINEAR) return CERNELS_E_UNSUPPORTED;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  EpTables t;
  ep_tables(c, s.intermediate, static_cast<uint8_t*>(workspace), &t);
  const EpGeometry g = geo_now(c);
  const int El = c->geo.local_experts;
  const size_t rows = static_cast<size_t>(c->geo.world) * c->geo.cap + c->geo.shared_cap;

  ep_segments_kernel<<<1, 1024, 0, stream>>>(c->window, g, epoch, c->d_counters + 3, t.offsets, t.group_rows,
                                             t.mtile, t.src_prefix, t.run_start, shared_tokens, c->d_status);
  ep_rowmap_kernel<<<ep_grid(static_cast<int>(rows)), kEpThreads, 0, stream>>>(c->d_peers, g, t.offsets, t.group_rows,
                                                                              t.src_prefix, t.run_start, t.row_out);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return rc_of(err);
  const bool gptoss = s.layout == CERNELS_LAYOUT_GPTOSS;
  const int sms = device_sm_count();
  GroupedGemmArgs g1{};
  g1.a = reinterpret_cast<const __nv_bfloat16*>(c->window + c->geo.recv_offset);
  g1.b = static_cast<const __nv_bfloat16*>(gate_up_proj);
  g1.bias = gptoss ? gate_up_bias : nullptr;
  g1.out = t.glu;
  g1.offsets = t.offsets;
  g1.group_rows = t.group_rows;
  g1.mtile_offsets = t.mtile;
  g1.status = c->d_status;
  g1.rows = static_cast<int>(rows);
  g1.experts = El + (shared ? 1 : 0);  // group El: the shared expert on this rank's own tokens
  g1.k = s.hidden;
  g1.n = 2 * s.intermediate;
  g1.out_cols = s.intermediate;
  g1.weight_experts = El;
  if (shared) {
    g1.b_extra = static_cast<const __nv_bfloat16*>(shared_gate_up_proj);
    g1.extra_group = El;
  }
  // rows from other ranks may still be arriving: wait per expert for every source's flag
  g1.ready = c->window + offsetof(EpHeader, arrived);
  g1.ready_stride = sizeof(EpHeader);
  g1.ready_sources = c->geo.world;
  g1.ready_self = c->geo.rank;
  g1.ready_epoch = epoch;
  g1.ready_epoch_dev = c->d_counters + 3;
  if ((err = launch_grouped_gemm(gptoss ? kGateUpGptOss : kGateUpLinear, g1, sms, stream)) != cudaSuccess)
    return rc_of(err);
  GroupedGemmArgs g2 = g1;
  g2.ready = nullptr;
  g2.a = t.glu;
  g2.b = static_cast<const __nv_bfloat16*>(down_proj);
  if (shared) g2.b_extra = static_cast<const __nv_bfloat16*>(shared_down_proj);
  g2.bias = gptoss ? down_bias : nullptr;
  g2.out = nullptr;
  g2.row_out = t.row_out;  // results straight into the sources' return regions
  g2.k = s.intermediate;
  g2.n = s.hidden;
  g2.out_cols = s.hidden;
  if ((err = launch_grouped_gemm(gptoss ? kDownGptOss : kDownLinear, g2, sms, stream)) != cudaSuccess)
    return rc_of(err);
  ep_results_kernel<<<1, 32, 0, stream>>>(c->d_peers, g, epoch, c->d_counters + 3);
  return rc_of(cudaGetLastError());
}

int cernels_ep_combine(void* ctx, const int32_t* inv, const float* weights, int32_t tokens, int32_t topk,
                       int32_t shared, void* out, uint32_t epoch, void* stream) {
  auto* c = static_cast<cernels_ep_ctx*>(ctx);
  if (!c || !c->connected) return CERNELS_E_NULL;
  if (tokens < 0 || topk <= 0 || (shared && topk < 2)) return CERNELS_E_INVALID_SHAPE;
  if (shared && tokens > c->geo.shared_cap) return CERNELS_E_UNSUPPORTED;
  if (tokens > 0 && (!inv || !weights || !out)) return CERNELS_E_NULL;
  const int blocks = tokens > 0 ? ep_grid(tokens) : 1;
  const cudaError_t join = cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), c->ev_dispatched, 0);
  if (join != cudaSuccess) return rc_of(join);
  ep_combine_kernel<<<blocks, kEpThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      c->window, geo_now(c), epoch, c->d_counters + 3, c->d_counters + 2, inv, weights, tokens, topk,
      shared != 0, static_cast<uint4*>(out), c->d_status);
  return rc_of(cudaGetLastError());
}

int cernels_ep_status(void* ctx, int* status) {
  auto* c = static_cast<cernels_ep_ctx*>(ctx);
  if (!c || !status) return CERNELS_E_NULL;
  return rc_of(cudaMemcpy(status, c->d_status, sizeof(int), cudaMemcpyDeviceToHost));
}

}  // extern "C"
