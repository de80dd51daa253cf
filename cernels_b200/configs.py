"""Seeded synthetic workloads of the MoE-experts benchmark configurations.

Shapes and value distributions follow the reference's benchmark configs
(src/configs/registry/{cohere2,deepseek_ocr2,qwen3_next,gpt_oss}_moe_experts.py): expert
weights ~N(0, 0.02) bf16, hidden states ~N(0, 1) bf16, router logits ~N(0, 1); seed 0
for weights and seed 1 for activations / logits (cohere2_moe_experts.py:54,72).

Configurations (name: T, H, E, F, topk, routing):
  deepseek_v2_lite  C1  512, 2048, 64, 1408, 6   softmax over E, top-6, no renorm
  decode            C2  C1 at T in {1, 4, 8}
  qwen3_30b_a3b     C3  2048, 2048, 128, 768, 8  logits + 1.5*log(1/rank_e), softmax, top-8, renorm
  qwen3_next        C4  4096, 2048, 512, 512, 10 softmax, top-10, renorm; shared expert F=512
                        with sigmoid gate (router / gate / shared weights ~N(0, 0.02))
  gpt_oss_20b       C5  16384, 2880, 32, 2880, 4 top-4 of (x W_r^T + b_r), softmax over the 4;
                        interleaved gate/up with biases ~N(0, 0.01), clamped SwiGLU
"""

from __future__ import annotations

import dataclasses
import math

import torch

LAYOUT_LINEAR = 0
LAYOUT_GPTOSS = 1


@dataclasses.dataclass(frozen=True)
class MoeConfig:
    name: str
    tokens: int
    hidden: int
    experts: int
    inter: int
    topk: int
    layout: int = LAYOUT_LINEAR
    routing: str = "softmax_topk"   # softmax_topk | softmax_topk_renorm | zipf_renorm | router_linear | gptoss_router
    renorm: bool = False
    shared_inter: int = 0           # C4 shared expert
    ref_op: str = "cohere2_moe_experts"

    def with_tokens(self, t: int) -> "MoeConfig":
        return dataclasses.replace(self, tokens=int(t))

    def scaled(self, **kw) -> "MoeConfig":
        return dataclasses.replace(self, **kw)

    # ---- algorithmic cost (per call)
    def flops(self) -> float:
        f = 6.0 * self.hidden * self.inter * self.tokens * self.topk
        if self.shared_inter:
            f += 6.0 * self.hidden * self.shared_inter * self.tokens
        return f

    def bytes_moved(self, touched_experts: int | None = None) -> float:
        """Weights of touched experts + x read + out write + indices/weights (+ biases)."""
        e = self.experts if touched_experts is None else touched_experts
        b = 3.0 * self.hidden * self.inter * 2 * e
        b += 2.0 * self.tokens * self.hidden * 2
        b += self.tokens * self.topk * 8
        if self.layout == LAYOUT_GPTOSS:
            b += e * (2 * self.inter + self.hidden) * 4
        if self.shared_inter:
            b += 3.0 * self.hidden * self.shared_inter * 2
        return b


CONFIGS: dict[str, MoeConfig] = {
    "deepseek_v2_lite": MoeConfig("deepseek_v2_lite", 512, 2048, 64, 1408, 6, routing="softmax_topk",
                                  ref_op="deepseek_ocr2_moe_experts"),
    "decode": MoeConfig("decode", 8, 2048, 64, 1408, 6, routing="softmax_topk", ref_op="cohere2_moe_experts_decode"),
    "qwen3_30b_a3b": MoeConfig("qwen3_30b_a3b", 2048, 2048, 128, 768, 8, routing="zipf_renorm", renorm=True,
                               ref_op="cohere2_moe_experts"),
    "qwen3_next": MoeConfig("qwen3_next", 4096, 2048, 512, 512, 10, routing="router_linear", renorm=True,
                            shared_inter=512, ref_op="qwen3_next_moe_experts"),
    "gpt_oss_20b": MoeConfig("gpt_oss_20b", 16384, 2880, 32, 2880, 4, layout=LAYOUT_GPTOSS, routing="gptoss_router",
                             ref_op="gpt_oss_moe_experts"),
}


@dataclasses.dataclass
class MoeCase:
    cfg: MoeConfig
    x: torch.Tensor                  # [T, H] bf16
    w1: torch.Tensor                 # gate_up_proj
    w2: torch.Tensor                 # down_proj
    indices: torch.Tensor            # [T, k] int64 (as produced by torch.topk)
    weights: torch.Tensor            # [T, k] fp32
    b1: torch.Tensor | None = None   # [E, 2F] fp32 (gpt-oss)
    b2: torch.Tensor | None = None   # [E, H] fp32 (gpt-oss)
    router_w: torch.Tensor | None = None   # [E, H] bf16 (qwen3_next / gpt-oss router)
    router_b: torch.Tensor | None = None   # [E] bf16 (gpt-oss)
    shared: dict | None = None       # qwen3_next shared expert weights (bf16)

    def to(self, device) -> "MoeCase":
        def mv(t):
            return None if t is None else t.to(device)
        return MoeCase(self.cfg, mv(self.x), mv(self.w1), mv(self.w2), mv(self.indices), mv(self.weights),
                       mv(self.b1), mv(self.b2), mv(self.router_w), mv(self.router_b),
                       None if self.shared is None else {k: v.to(device) for k, v in self.shared.items()})


def _normal(gen: torch.Generator, shape, std: float, device) -> torch.Tensor:
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=gen)
    return t


def route_logits(cfg: MoeConfig, logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Turns fp32 router logits into (top-k indices int64, fp32 weights) per cfg.routing."""
    k = cfg.topk
    if cfg.routing == "gptoss_router":
        # transformers GptOssTopKRouter: top-k of the logits, softmax over the k values.
        top_v, top_i = torch.topk(logits, k, dim=-1)
        return top_i, torch.softmax(top_v, dim=-1)
    if cfg.routing == "zipf_renorm":
        rank = torch.arange(1, cfg.experts + 1, dtype=torch.float32, device=logits.device)
        logits = logits + 1.5 * torch.log(1.0 / rank)
    probs = torch.softmax(logits.float(), dim=-1)
    top_v, top_i = torch.topk(probs, k, dim=-1)
    if cfg.renorm:
        top_v = top_v / top_v.sum(dim=-1, keepdim=True)
    return top_i, top_v.float()


def router_forward(case: MoeCase, x: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Router of the module-level configs (qwen3_next, gpt_oss), torch ops as in the
    reference loaders (src/kops/registry/qwen3_next_moe_experts.py:28,
    src/kops/registry/gpt_oss_moe_experts.py:35)."""
    cfg = case.cfg
    x = case.x if x is None else x
    if cfg.routing == "gptoss_router":
        logits = torch.nn.functional.linear(x, case.router_w, case.router_b)
        return route_logits(cfg, logits.float())
    logits = torch.nn.functional.linear(x, case.router_w)
    return route_logits(cfg, logits.float())


def make_case(cfg: MoeConfig | str, device="cpu", seed_weights: int = 0, seed_inputs: int = 1) -> MoeCase:
    """Builds a seeded case. Weights from seed 0, x / logits from seed 1."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    T, H, E, F, k = cfg.tokens, cfg.hidden, cfg.experts, cfg.inter, cfg.topk
    gw = torch.Generator(device=device).manual_seed(seed_weights)
    bf = torch.bfloat16
    if cfg.layout == LAYOUT_LINEAR:
        w1 = _normal(gw, (E, 2 * F, H), 0.02, device).to(bf)
        w2 = _normal(gw, (E, H, F), 0.02, device).to(bf)
        b1 = b2 = None
    else:
        w1 = _normal(gw, (E, H, 2 * F), 0.02, device).to(bf)
        w2 = _normal(gw, (E, F, H), 0.02, device).to(bf)
        b1 = _normal(gw, (E, 2 * F), 0.01, device).to(bf).float()
        b2 = _normal(gw, (E, H), 0.01, device).to(bf).float()
    router_w = router_b = None
    shared = None
    if cfg.routing in ("router_linear", "gptoss_router"):
        router_w = _normal(gw, (E, H), 0.02, device).to(bf)
        if cfg.routing == "gptoss_router":
            router_b = _normal(gw, (E,), 0.02, device).to(bf)
    if cfg.shared_inter:
        Fs = cfg.shared_inter
        shared = {
            "gate_proj": _normal(gw, (Fs, H), 0.02, device).to(bf),
            "up_proj": _normal(gw, (Fs, H), 0.02, device).to(bf),
            "down_proj": _normal(gw, (H, Fs), 0.02, device).to(bf),
            "gate": _normal(gw, (1, H), 0.02, device).to(bf),
        }
    gi = torch.Generator(device=device).manual_seed(seed_inputs)
    x = _normal(gi, (T, H), 1.0, device).to(bf)
    case = MoeCase(cfg, x, w1, w2, None, None, b1, b2, router_w, router_b, shared)
    if router_w is None:
        logits = _normal(gi, (T, E), 1.0, device)
        idx, wts = route_logits(cfg, logits)
    else:
        idx, wts = router_forward(case)
    case.indices, case.weights = idx, wts.float()
    return case


def touched_experts(indices: torch.Tensor, experts: int) -> int:
    v = indices.reshape(-1)
    v = v[(v >= 0) & (v < experts)]
    return int(torch.unique(v).numel())


def describe(cfg: MoeConfig) -> str:
    return (f"{cfg.name}: T={cfg.tokens} H={cfg.hidden} E={cfg.experts} F={cfg.inter} k={cfg.topk} "
            f"layout={'gptoss' if cfg.layout else 'linear'} flops={cfg.flops() / 1e9:.1f}G "
            f"bytes={cfg.bytes_moved() / 1e9:.3f}GB intensity={cfg.flops() / cfg.bytes_moved():.0f}")


__all__ = ["MoeConfig", "MoeCase", "CONFIGS", "make_case", "route_logits", "router_forward", "touched_experts",
           "describe", "math"]
