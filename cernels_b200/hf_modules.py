"""Builds the transformers modules the reference benchmarks against, loaded with the
seeded weights of a :class:`cernels_b200.configs.MoeCase`.

The reference's ``baseline`` (op_eager) of each MoE config is the transformers module
called directly (src/configs/registry/*_moe_experts.py). transformers 5.5.0 ships
DeepseekV2Experts (the same F.linear-layout chunked-SwiGLU experts contract as
Cohere2MoeExperts / DeepseekOcr2TextExperts, which this version lacks),
Qwen3NextSparseMoeBlock and GptOssMLP. The loaders in ``cernels_b200.registry`` take
these modules as their weight storage, exactly as the reference loaders do.
"""

from __future__ import annotations

import torch

from .configs import LAYOUT_GPTOSS, MoeCase


def _assign(param: torch.nn.Parameter, value: torch.Tensor) -> None:
    with torch.no_grad():
        param.data = value.to(device=param.device, dtype=param.dtype).contiguous()


def build_module(case: MoeCase, device=None, dtype=torch.bfloat16):
    """Returns (kind, module) with kind in {"experts", "qwen3_next", "gpt_oss"}."""
    cfg = case.cfg
    device = case.x.device if device is None else torch.device(device)
    meta = torch.device("meta")
    if cfg.layout == LAYOUT_GPTOSS:
        from transformers.models.gpt_oss.configuration_gpt_oss import GptOssConfig
        from transformers.models.gpt_oss.modeling_gpt_oss import GptOssMLP

        hc = GptOssConfig(hidden_size=cfg.hidden, intermediate_size=cfg.inter, num_local_experts=cfg.experts,
                          num_experts_per_tok=cfg.topk)
        with meta:
            mod = GptOssMLP(hc)
        mod = mod.to_empty(device=device).to(dtype)
        _assign(mod.router.weight, case.router_w)
        _assign(mod.router.bias, case.router_b)
        _assign(mod.experts.gate_up_proj, case.w1)
        _assign(mod.experts.down_proj, case.w2)
        _assign(mod.experts.gate_up_proj_bias, case.b1)
        _assign(mod.experts.down_proj_bias, case.b2)
        return "gpt_oss", mod.eval()
    if cfg.shared_inter:
        from transformers.models.qwen3_next.configuration_qwen3_next import Qwen3NextConfig
        from transformers.models.qwen3_next.modeling_qwen3_next import Qwen3NextSparseMoeBlock

        hc = Qwen3NextConfig(hidden_size=cfg.hidden, moe_intermediate_size=cfg.inter,
                             shared_expert_intermediate_size=cfg.shared_inter, num_experts=cfg.experts,
                             num_experts_per_tok=cfg.topk, norm_topk_prob=cfg.renorm)
        with meta:
            blk = Qwen3NextSparseMoeBlock(hc)
        blk = blk.to_empty(device=device).to(dtype)
        _assign(blk.gate.weight, case.router_w)
        _assign(blk.experts.gate_up_proj, case.w1)
        _assign(blk.experts.down_proj, case.w2)
        _assign(blk.shared_expert.gate_proj.weight, case.shared["gate_proj"])
        _assign(blk.shared_expert.up_proj.weight, case.shared["up_proj"])
        _assign(blk.shared_expert.down_proj.weight, case.shared["down_proj"])
        _assign(blk.shared_expert_gate.weight, case.shared["gate"])
        return "qwen3_next", blk.eval()
    from transformers.models.deepseek_v2.configuration_deepseek_v2 import DeepseekV2Config
    from transformers.models.deepseek_v2.modeling_deepseek_v2 import DeepseekV2Experts

    hc = DeepseekV2Config(hidden_size=cfg.hidden, moe_intermediate_size=cfg.inter, n_routed_experts=cfg.experts,
                          num_experts_per_tok=cfg.topk, hidden_act="silu")
    with meta:
        mod = DeepseekV2Experts(hc)
    mod = mod.to_empty(device=device).to(dtype)
    _assign(mod.gate_up_proj, case.w1)
    _assign(mod.down_proj, case.w2)
    return "experts", mod.eval()


def reference_forward(kind: str, module, case: MoeCase, x: torch.Tensor | None = None,
                      indices: torch.Tensor | None = None, weights: torch.Tensor | None = None) -> torch.Tensor:
    """The reference benchmark's op_eager call for this config (returns [T, H])."""
    x = case.x if x is None else x
    with torch.no_grad():
        if kind == "gpt_oss":
            out, _ = module(x.unsqueeze(0))
            return out.reshape(x.shape)
        if kind == "qwen3_next":
            return module(x.unsqueeze(0)).reshape(x.shape)
        idx = case.indices if indices is None else indices
        w = case.weights if weights is None else weights
        return module(x, idx, w.to(x.dtype))
