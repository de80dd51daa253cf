"""CPU oracle for the MoE-experts hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module, and only as the checker / CPU baseline. The product path
(``cernels_b200``) never calls it and fails loudly when its CUDA library is missing.

It restates, in numpy, the algorithm of the reference operators:

* routing — ``count_tokens_kernel`` / ``at::cumsum`` / ``build_perm_kernel``
  (src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:29-55,259-280): histogram of
  valid expert ids, exclusive prefix sum into ``offsets[E+1]``, and one permuted row per
  valid (token, slot) entry carrying its token id and router weight. Ids outside [0, E)
  are skipped (:35,49-50). The reference orders rows inside an expert by atomic arrival;
  the order defined here (and produced by the CUDA kernels) is the flat index t*topk+j,
  i.e. ``torch.sort(indices.flatten(), stable=True)`` — the per-expert row *set* equals
  the transformers eager loop's ``torch.where(expert_mask[e])`` token set
  (transformers 5.5.0 models/deepseek_v2/modeling_deepseek_v2.py:74).
* expert math — per expert e with rows R_e:
  LINEAR (cohere2 / deepseek_ocr2 / qwen3_next, src/kops/cohere2_moe_experts/csrc/cohere2_moe_experts.cu:5-17,70-82):
      gu = x[R_e] @ W1[e]^T ; gate, up = gu[:, :F], gu[:, F:] ; glu = silu(gate) * up
      y  = glu @ W2[e]^T
  GPTOSS (src/kops/gpt_oss_moe_experts/csrc/gpt_oss_moe_experts.cu:16-20,75-117):
      gu = x[R_e] @ W1[e] + b1[e] ; gate, up = gu[:, 0::2], gu[:, 1::2]
      gate = min(gate, 7) ; up = clamp(up, -7, 7) ; glu = (up + 1) * gate * sigmoid(1.702 gate)
      y  = glu @ W2[e] + b2[e]
  out[t] = sum_j w[t, j] * y_(t, j), accumulated in fp32 (reference scatter_add_f32_kernel,
  :85-94 / gpt_oss :104-117).

Arithmetic is float32 (numpy BLAS) on bf16-representable inputs — the "fp32 evaluation"
the parity bar is stated against (max |out - ref| / max |ref| <= 1e-2).
"""

from __future__ import annotations

import numpy as np

LAYOUT_LINEAR = 0
LAYOUT_GPTOSS = 1
GPTOSS_LIMIT = 7.0
GPTOSS_ALPHA = 1.702


def route(indices: np.ndarray, experts: int):
    """Stable counting sort of flat (token, slot) entries by expert id.

    Returns (offsets [E+1] int32, perm_flat [n_valid] int64, inv [T*k] int32 with -1 for
    skipped entries). perm_token = perm_flat // topk.
    """
    flat = np.asarray(indices, dtype=np.int64).reshape(-1)
    valid = (flat >= 0) & (flat < experts)
    counts = np.bincount(flat[valid], minlength=experts).astype(np.int64)
    offsets = np.zeros(experts + 1, dtype=np.int64)
    np.cumsum(counts, out=offsets[1:])
    # Stable sort by expert among valid entries == rank by (expert, flat index).
    idx_valid = np.nonzero(valid)[0]
    order = idx_valid[np.argsort(flat[idx_valid], kind="stable")]
    inv = np.full(flat.shape[0], -1, dtype=np.int64)
    inv[order] = np.arange(order.shape[0])
    return offsets.astype(np.int32), order, inv.astype(np.int32)


def _silu(g: np.ndarray) -> np.ndarray:
    return g / (1.0 + np.exp(-g))


def _gptoss_act(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    gate = np.minimum(gate, GPTOSS_LIMIT)
    up = np.clip(up, -GPTOSS_LIMIT, GPTOSS_LIMIT)
    return (up + 1.0) * (gate / (1.0 + np.exp(-gate * GPTOSS_ALPHA)))


def expert_rows(x_rows: np.ndarray, w1: np.ndarray, w2: np.ndarray, layout: int, b1=None, b2=None) -> np.ndarray:
    """Unweighted expert output for rows of one expert (float32)."""
    x_rows = x_rows.astype(np.float32, copy=False)
    if layout == LAYOUT_LINEAR:
        F = w1.shape[0] // 2
        gu = x_rows @ w1.astype(np.float32, copy=False).T
        glu = _silu(gu[:, :F]) * gu[:, F:]
        return glu @ w2.astype(np.float32, copy=False).T
    gu = x_rows @ w1.astype(np.float32, copy=False)
    if b1 is not None:
        gu = gu + b1.astype(np.float32, copy=False)
    glu = _gptoss_act(gu[:, 0::2], gu[:, 1::2])
    y = glu @ w2.astype(np.float32, copy=False)
    if b2 is not None:
        y = y + b2.astype(np.float32, copy=False)
    return y


def moe_experts(x, w1, w2, indices, weights, layout=LAYOUT_LINEAR, b1=None, b2=None, token_subset=None):
    """fp32 oracle of the experts operator: returns out [T, H] float32.

    x [T, H]; w1 LINEAR [E, 2F, H] / GPTOSS [E, H, 2F]; w2 LINEAR [E, H, F] / GPTOSS [E, F, H];
    indices [T, k] int; weights [T, k] float. Arrays may be any float dtype; math is fp32.
    ``token_subset`` (sorted token ids) restricts the computation to those tokens (the
    other rows of the result are zero) — used for bounded CPU samples of large configs.
    """
    x = np.asarray(x, dtype=np.float32)
    indices = np.asarray(indices)
    weights = np.asarray(weights, dtype=np.float32)
    T, H = x.shape
    E = w1.shape[0]
    k = indices.shape[1]
    out = np.zeros((T, H), dtype=np.float32)
    if token_subset is not None:
        mask = np.zeros(T, dtype=bool)
        mask[np.asarray(token_subset)] = True
        indices = np.where(mask[:, None], indices, -1)
    offsets, perm_flat, _ = route(indices, E)
    tok = perm_flat // k
    wts = weights.reshape(-1)[perm_flat]
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if lo == hi:
            continue
        rows = tok[lo:hi]
        y = expert_rows(x[rows], np.asarray(w1[e]), np.asarray(w2[e]), layout,
                        None if b1 is None else np.asarray(b1[e]), None if b2 is None else np.asarray(b2[e]))
        np.add.at(out, rows, y * wts[lo:hi, None])
    return out


def router_tail(logits: np.ndarray, topk: int, mode: int, renorm: bool = False):
    """Router tail restated from the transformers routers the reference loaders call
    (src/kops/registry/gpt_oss_moe_experts.py:35, src/kops/registry/qwen3_next_moe_experts.py:28):
    mode 0 (gpt-oss, transformers models/gpt_oss/modeling_gpt_oss.py:117-131): top-k of the logits,
    softmax over the k values; mode 1 (qwen3-next, models/qwen3_next/modeling_qwen3_next.py:761-780):
    softmax over all experts, top-k, optional renormalisation. Ties go to the lower expert id.
    Returns (indices [T, k] int64, weights [T, k] float32)."""
    logits = np.asarray(logits, dtype=np.float64)
    order = np.argsort(-logits, axis=1, kind="stable")[:, :topk]
    if mode == 0:
        v = np.take_along_axis(logits, order, axis=1)
        e = np.exp(v - v[:, :1])
        w = e / e.sum(axis=1, keepdims=True)
    else:
        p = np.exp(logits - logits.max(axis=1, keepdims=True))
        p = p / p.sum(axis=1, keepdims=True)
        w = np.take_along_axis(p, order, axis=1)
        if renorm:
            w = w / w.sum(axis=1, keepdims=True)
    return order, w.astype(np.float32)


def shared_expert(x, gate_proj, up_proj, down_proj, gate_w):
    """Qwen3-Next always-on shared expert: sigmoid(x @ g^T) * (silu(x Wg^T) * (x Wu^T)) Wd^T
    (src/kops/registry/qwen3_next_moe_experts.py:41-43). Returns float32 [T, H]."""
    x = np.asarray(x, dtype=np.float32)
    g = x @ np.asarray(gate_proj, dtype=np.float32).T
    u = x @ np.asarray(up_proj, dtype=np.float32).T
    y = (_silu(g) * u) @ np.asarray(down_proj, dtype=np.float32).T
    s = 1.0 / (1.0 + np.exp(-(x @ np.asarray(gate_w, dtype=np.float32).T)))
    return y * s


def rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max |out - ref| / max |ref| — the parity metric for expert outputs."""
    out = np.asarray(out, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    denom = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(out - ref))) / max(denom, 1e-30)
