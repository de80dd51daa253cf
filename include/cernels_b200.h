/*
 * cernels_b200 — C ABI of the B200 (sm_100a) mixture-of-experts "experts" operators.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (passed as
 * void*), launches asynchronously on that stream and returns 0 or a CERNELS_E_* code.
 * Apart from cernels_ep_create (the expert-parallel window), nothing here allocates device
 * memory: scratch comes from a caller-provided workspace whose size
 * cernels_moe_workspace_bytes() reports. No entry point synchronises the
 * stream or reads device memory on the host, so a call can be captured in a CUDA graph.
 *
 * Tensor conventions (all contiguous, row-major):
 *   x              [T, H]        bf16
 *   gate_up_proj   CERNELS_LAYOUT_LINEAR: [E, 2F, H] bf16  (F.linear layout, rows 0..F-1 gate, F..2F-1 up)
 *                  CERNELS_LAYOUT_GPTOSS: [E, H, 2F] bf16  (columns interleaved: even gate, odd up)
 *   gate_up_bias   [E, 2F] fp32, GPTOSS only (may be NULL)
 *   down_proj      CERNELS_LAYOUT_LINEAR: [E, H, F] bf16;  CERNELS_LAYOUT_GPTOSS: [E, F, H] bf16
 *   down_bias      [E, H] fp32, GPTOSS only (may be NULL)
 *   indices        [T, topk] int32 expert id per (token, slot); ids outside [0, E) are skipped
 *   weights        [T, topk] fp32 router weight per (token, slot)
 *   out            [T, H] bf16 (fully overwritten)
 *
 * Activation: LINEAR  glu = silu(gate) * up
 *             GPTOSS  g = min(gate, 7), u = clamp(up, -7, 7), glu = (u + 1) * g * sigmoid(1.702 g)
 * Output:     out[t] = sum_j weights[t, j] * (glu_j @ down[e_j] (+ down_bias[e_j]))   (fp32 accumulate)
 */
#ifndef CERNELS_B200_H_
#define CERNELS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CERNELS_LAYOUT_LINEAR 0
#define CERNELS_LAYOUT_GPTOSS 1

/* Return codes (mirroring the reference's TORCH_CHECK failures, as integers). */
#define CERNELS_OK 0
#define CERNELS_E_INVALID_SHAPE 1     /* non-positive or unsupported dimension            */
#define CERNELS_E_ALIGNMENT 2         /* H or F not a multiple of 8, or pointer misaligned */
#define CERNELS_E_WORKSPACE 3         /* workspace NULL or smaller than required          */
#define CERNELS_E_CUDA 4              /* a CUDA runtime / driver call failed              */
#define CERNELS_E_UNSUPPORTED 5       /* no sm_100 device, or a limit of this build       */
#define CERNELS_E_NULL 6              /* a required pointer is NULL                       */

typedef struct cernels_moe_shape {
  int32_t tokens;       /* T */
  int32_t hidden;       /* H */
  int32_t experts;      /* E */
  int32_t intermediate; /* F (per-expert moe_intermediate_size) */
  int32_t topk;         /* k */
  int32_t layout;       /* CERNELS_LAYOUT_* */
} cernels_moe_shape;

/* Human-readable text for a return code (static storage). */
const char* cernels_error_string(int code);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int cernels_version(void);

/* Limit, in nanoseconds, after which every bounded wait inside this library's kernels (an
 * mbarrier of a TMA / MMA pipeline, a grid barrier, a peer rank's flag) gives up, records a
 * nonzero status word and lets the kernel return. 0 restores the defaults (2 s for waits
 * inside one GPU, 5 s for waits on peer ranks). Applies to launches made after the call, from
 * any host thread. No counterpart in the reference (its kernels never wait). */
int cernels_set_wait_limit_ns(uint64_t ns);

/* Workspace bytes needed by cernels_moe_experts (decode == 0) or
 * cernels_moe_experts_decode (decode != 0) for this shape. */
int cernels_moe_workspace_bytes(const cernels_moe_shape* shape, int decode, size_t* bytes);

/* Prefill / general path: routing -> gather -> tcgen05 grouped GEMM (gate/up + fused
 * activation) -> tcgen05 grouped GEMM (down) -> deterministic weighted combine.
 * Replaces the host functions `cohere2_moe_experts`
 * (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:238),
 * `deepseek_ocr2_moe_experts` (src/kops/deepseek_ocr2_moe_experts/csrc/deepseek_ocr2_moe_experts.cu:240),
 * `qwen3_next_moe_experts` (src/kops/qwen3_next_moe_experts/csrc/qwen3_next_moe_experts.cu:97) and
 * `gpt_oss_moe_experts` (src/kops/gpt_oss_moe_experts/csrc/gpt_oss_moe_experts.cu:119). */
int cernels_moe_experts(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                        const float* gate_up_bias, const void* down_proj, const float* down_bias,
                        const int32_t* indices, const float* weights, void* out, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Routed experts plus one always-on shared expert in the same launches (LINEAR layout, shared
 * intermediate size = F): the shared expert is expert id E, every token routes to it in the last
 * of topk + 1 slots with its gate weight (cernels_router_topk with shared_gate produces that).
 * shape describes the routed experts (experts = E, topk = k); indices / weights are [T, k + 1];
 * shared_gate_up_proj [1, 2F, H], shared_down_proj [1, H, F]; workspace =
 * cernels_moe_workspace_bytes of the shape with experts + 1 and topk + 1. Replaces the routed op
 * plus the torch shared MLP, sigmoid gate and add of src/kops/registry/qwen3_next_moe_experts.py:31-44. */
int cernels_moe_experts_shared(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                               const void* down_proj, const void* shared_gate_up_proj, const void* shared_down_proj,
                               const int32_t* indices, const float* weights, void* out, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Decode path (T * topk <= 1024): fused gather-GEMV that streams each selected expert's
 * weights once, deduplicated across tokens. Replaces `cohere2_moe_experts_decode`
 * (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:199) and
 * `deepseek_ocr2_moe_experts_decode` (src/kops/deepseek_ocr2_moe_experts/csrc/deepseek_ocr2_moe_experts.cu:201). */
int cernels_moe_experts_decode(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                               const float* gate_up_bias, const void* down_proj, const float* down_bias,
                               const int32_t* indices, const float* weights, void* out, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---- Stage entry points (used by the expert-parallel host path and by tests). ---- */

/* Routing: per-expert histogram, offsets[E+1], and a permutation that is stable in the
 * flat index t*topk+j. Replaces count_tokens_kernel + at::cumsum + build_perm_kernel
 * (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:29-55,259-280).
 * Outputs (device, caller-allocated): offsets [E+1], perm_token [T*topk],
 * perm_weight [T*topk], inv [T*topk] (permuted row of each flat entry, -1 if skipped).
 * Entries past offsets[E] in perm_* are left untouched. */
int cernels_moe_route(const cernels_moe_shape* shape, const int32_t* indices, const float* weights,
                      int32_t* offsets, int32_t* perm_token, float* perm_weight, int32_t* inv,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Expert compute on rows already grouped into `groups` contiguous runs: run g holds
 * group_counts[g] rows (device int32 array) and uses expert g % shape->experts of the
 * weights (groups must be a multiple of shape->experts). Writes each row's unweighted expert
 * output (+ down_bias) to rows_out in the same order. shape->tokens is the row capacity of
 * rows_in / rows_out; shape->topk is ignored. Workspace: cernels_moe_workspace_bytes() of the
 * shape with experts = groups and topk = 1. This is the receive side of expert parallelism:
 * rows arrive from the dispatch all-to-all ordered by (source rank, local expert), so the
 * grouped GEMMs read them in place. Replaces, per expert, the two cublasGemmEx calls + bias +
 * SwiGLU of src/kops/gpt_oss_moe_experts/csrc/gpt_oss_moe_experts.cu:200-242. */
int cernels_moe_grouped_experts(const cernels_moe_shape* shape, int32_t groups, const int32_t* group_counts,
                                const void* rows_in, const void* gate_up_proj, const float* gate_up_bias,
                                const void* down_proj, const float* down_bias, void* rows_out, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Router tail: from router logits [T, E] (bf16 if logits_bf16, else fp32) to top-k expert ids
 * (int32 [T, topk], descending, ties to the lower id) and routing weights (fp32 [T, topk]).
 * mode CERNELS_ROUTER_TOPK_SOFTMAX: softmax over the k selected logits, rounded to bf16 — the
 *   transformers gpt-oss router (models/gpt_oss/modeling_gpt_oss.py:117-131);
 * mode CERNELS_ROUTER_SOFTMAX_TOPK: softmax over all E in fp32, top-k, renormalised to sum 1
 *   when renorm — the transformers qwen3-next router (models/qwen3_next/modeling_qwen3_next.py:761-780).
 * Replaces the torch topk / softmax / casts the reference loaders run
 * (src/kops/registry/gpt_oss_moe_experts.py:35-45, src/kops/registry/qwen3_next_moe_experts.py:28-37).
 * E <= 1024, topk <= 32. */
#define CERNELS_ROUTER_TOPK_SOFTMAX 0
#define CERNELS_ROUTER_SOFTMAX_TOPK 1
int cernels_router_topk(const void* logits, int32_t logits_bf16, int32_t tokens, int32_t experts, int32_t topk,
                        int32_t mode, int32_t renorm, int32_t shared_gate, int32_t* indices, float* weights,
                        void* stream);
/* shared_gate != 0: logits rows hold E + 1 values (row stride padded to a multiple of 8), column
 * E being a shared expert's gate logit;
 * indices / weights get topk + 1 columns, the last = (E, sigmoid(gate logit)) — the input of
 * cernels_moe_experts_shared. */

/* Fused router: logits = x router_weight^T (+ router_bias) computed on the tcgen05 tensor
 * cores, rounded to bf16 (the dtype the transformers linear produces), and the router tail of
 * cernels_router_topk (same modes, same tie rule) applied in the same kernel, so the logits
 * never reach global memory. x [T, H] bf16; router_weight [weight_rows, H] bf16 with
 * weight_rows >= experts (+ 1 with shared_gate, whose row `experts` is the shared expert's gate);
 * router_bias [experts] bf16 or NULL. Writes indices / weights [T, topk (+ 1)] as
 * cernels_router_topk does; logits_out, if not NULL, receives the bf16 logits [T, weight_rows]
 * (columns 0..experts (+ 1) - 1 only; for tests). topk <= 16, experts (+ 1) <= 2048.
 * Replaces the router linear + topk + softmax + casts of the reference loaders
 * (src/kops/registry/gpt_oss_moe_experts.py:35, src/kops/registry/qwen3_next_moe_experts.py:28). */
int cernels_router(const void* x, int32_t tokens, int32_t hidden, const void* router_weight, int32_t weight_rows,
                   const void* router_bias, int32_t experts, int32_t topk, int32_t mode, int32_t renorm,
                   int32_t shared_gate, int32_t* indices, float* weights, void* logits_out, void* stream);

/* Gather: rows_out[i, :] = x[perm_token[i], :] for i < rows ([rows, H] bf16). Replaces
 * gather_kernel (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:58-65). Used by
 * expert parallelism to build the dispatch send buffer in routed order. */
int cernels_moe_gather(const void* x, const int32_t* perm_token, int32_t rows, int32_t hidden, void* rows_out,
                       void* stream);

/* Weighted combine: out[t, :] = bf16( sum_j weights[t, j] * rows[inv[t*topk+j], :] ), fp32
 * accumulation in fixed slot order j = 0..topk-1, entries with inv < 0 skipped. Replaces
 * scatter_add_f32_kernel + the fp32->bf16 cast
 * (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:85-94,360), deterministically. */
int cernels_moe_combine(const void* rows, const int32_t* inv, const float* weights, int32_t tokens,
                        int32_t topk, int32_t hidden, void* out, void* stream);

/* Diagnostics: runs cernels_moe_experts once with CUDA events recorded on `stream`
 * between its stages and returns the device time of each stage in milliseconds:
 * stage_ms[0] routing, [1] gather, [2] gate/up grouped GEMM, [3] down grouped GEMM,
 * [4] combine. Synchronises `stream`. Not for the hot path. */
int cernels_moe_experts_profiled(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                                 const float* gate_up_bias, const void* down_proj, const float* down_bias,
                                 const int32_t* indices, const float* weights, void* out, void* workspace,
                                 size_t workspace_bytes, void* stream, float* stage_ms);

/* Decode without any caller-provided scratch, for callers that cannot allocate device
 * memory (no cudaMalloc available to them, or every device byte planned up front).
 * No counterpart in the reference. Same math and kernels as cernels_moe_experts_decode;
 * the scratch lives in a 4 MiB static __device__ array inside this library, held on each
 * device that loads the library until the process exits. The first call on a device looks
 * up that array's device address (cudaGetSymbolAddress), so make that first call before
 * any stream capture. Problems needing more than 4 MiB of decode scratch (the decode
 * workspace size that cernels_moe_workspace_bytes reports: T*topk*(F+H)*4 bytes plus a few
 * KB, and for the GPTOSS layout at small T up to 8 K-split slabs of T*topk*(2F) and
 * T*topk*H fp32 values), or T*topk > 1024, return CERNELS_E_UNSUPPORTED. All calls on a
 * device share the one array: calls whose kernels may overlap on the GPU (different
 * streams, or concurrent host threads) race and must be serialised by the caller. */
int cernels_moe_experts_decode_noalloc(const cernels_moe_shape* shape, const void* x, const void* gate_up_proj,
                                       const float* gate_up_bias, const void* down_proj, const float* down_bias,
                                       const int32_t* indices, const float* weights, void* out, void* stream);

/* ---- Expert parallelism over NVLink peer memory (no counterpart in the reference, which is
 * single-GPU). One context per rank (one process per GPU): a device window holding an
 * expert-contiguous receive region ([world * max_rows][H] bf16: every source's rows of local
 * expert 0, then of expert 1, ...), a return region ([max_rows][H]) and small headers, shared with
 * the other ranks through CUDA IPC. Per step:
 *   cernels_ep_dispatch  exchanges per-expert row counts with every rank, then copies the routed
 *                        rows (x[perm_token[p]], p < offsets[E]) to their owners' windows
 *   cernels_ep_experts   waits for all sources, grouped GEMMs on the received rows (one group per
 *                        local expert), returns each result row into its source's window
 *   cernels_ep_combine   waits for all results, out[t] = bf16(sum_j w[t,j] * row[inv[t,j]])
 * offsets/perm_token/inv come from cernels_moe_route over the GLOBAL expert ids (experts are
 * sharded contiguously: rank r owns [r*El, (r+1)*El)). `epoch` numbers the step: pass 0 to let the
 * context count steps on the device (the three calls of a step then replay correctly from a CUDA
 * graph), or the same nonzero, increasing value on every rank for every call of a step; do not mix
 * the two on one context. Waits inside the kernels give up after 5 s (see
 * cernels_set_wait_limit_ns) and record a nonzero status (cernels_ep_status). */
#define CERNELS_EP_HANDLE_BYTES 64
/* shared_rows > 0 reserves room for an always-on shared expert (the Qwen3-Next layout): up to
 * shared_rows of this rank's own tokens run through it inside the same grouped GEMMs, and
 * cernels_ep_combine adds it as the last routing slot. */
int cernels_ep_create(int32_t rank, int32_t world, int32_t hidden, int32_t local_experts, int32_t max_rows,
                      int32_t shared_rows, void** ctx, void* ipc_handle_out);
int cernels_ep_connect(void* ctx, const void* ipc_handles /* world * CERNELS_EP_HANDLE_BYTES, rank order */);
int cernels_ep_destroy(void* ctx);
/* shared_tokens: this rank's tokens (x rows 0..shared_tokens-1) for the shared expert, or 0. */
int cernels_ep_dispatch(void* ctx, const void* x, const int32_t* perm_token, const int32_t* offsets, int32_t rows,
                        int32_t shared_tokens, uint32_t epoch, void* stream);
int cernels_ep_experts_workspace_bytes(void* ctx, const cernels_moe_shape* shape, size_t* bytes);
/* shared_gate_up_proj [1, 2F, H] / shared_down_proj [1, H, F] (LINEAR layout, same F) with
 * shared_tokens > 0: the shared expert runs as one more group of the grouped GEMMs. */
int cernels_ep_experts(void* ctx, const cernels_moe_shape* shape, const void* gate_up_proj, const float* gate_up_bias,
                       const void* down_proj, const float* down_bias, const void* shared_gate_up_proj,
                       const void* shared_down_proj, int32_t shared_tokens, uint32_t epoch, void* workspace,
                       size_t workspace_bytes, void* stream);
/* shared != 0: slot topk - 1 of every token is its shared-expert result (its weight the gate),
 * the other slots routed as given by inv. */
int cernels_ep_combine(void* ctx, const int32_t* inv, const float* weights, int32_t tokens, int32_t topk,
                       int32_t shared, void* out, uint32_t epoch, void* stream);
int cernels_ep_status(void* ctx, int* status);

/* Device status word of the last call that used this workspace (0 = ok; nonzero when a
 * bounded wait inside a kernel gave up). Reads device memory: synchronises `stream`.
 * With decode != 0 and workspace == NULL it reads the status word of the last
 * cernels_moe_experts_decode_noalloc call on the current device. */
int cernels_workspace_status(const cernels_moe_shape* shape, int decode, const void* workspace, int* status,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CERNELS_B200_H_ */
