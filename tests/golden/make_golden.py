"""Generates the golden fixtures in this directory from the reference's oracle modules.

The reference's op_eager baseline is the transformers experts module itself
(src/configs/registry/*_moe_experts.py ``baseline``). transformers 5.5.0 (installed)
provides DeepseekV2Experts (same contract and math as Cohere2MoeExperts /
DeepseekOcr2TextExperts: F.linear layout, chunked SwiGLU, bf16 index_add_),
Qwen3NextSparseMoeBlock and GptOssMLP. For each small seeded case this script stores the
inputs, the module's bf16 eager output (what the reference's verify() compares against)
and the same module evaluated in fp32 on the same bf16-representable values.

Run from the repository root:  python tests/golden/make_golden.py
Fixtures are .npz files; bf16 tensors are stored as their uint16 bit patterns.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def fill_(module: torch.nn.Module, seed: int, std: float = 0.02) -> None:
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * std)


def deepseek_case(name: str, T: int, H: int, E: int, F: int, k: int, invalid: bool = False) -> None:
    from transformers.models.deepseek_v2.configuration_deepseek_v2 import DeepseekV2Config
    from transformers.models.deepseek_v2.modeling_deepseek_v2 import DeepseekV2Experts

    cfg = DeepseekV2Config(hidden_size=H, moe_intermediate_size=F, n_routed_experts=E, num_experts_per_tok=k,
                           hidden_act="silu")
    mod = DeepseekV2Experts(cfg)
    fill_(mod, 0)
    mod = mod.to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    probs = logits.softmax(-1)
    w, idx = torch.topk(probs, k, dim=-1)
    with torch.no_grad():
        ref_bf16 = mod(x, idx, w.to(torch.bfloat16))
        mod32 = DeepseekV2Experts(cfg)
        mod32.load_state_dict({kk: v.float() for kk, v in mod.state_dict().items()})
        ref_fp32 = mod32.float()(x.float(), idx, w.to(torch.bfloat16).float())
    np.savez_compressed(
        OUT / f"{name}.npz", kind="linear", x=bf16_bits(x), w1=bf16_bits(mod.gate_up_proj), w2=bf16_bits(mod.down_proj),
        indices=idx.numpy().astype(np.int32), weights=w.to(torch.bfloat16).float().numpy(),
        ref_bf16=bf16_bits(ref_bf16), ref_fp32=ref_fp32.numpy())


def qwen3_next_case(name: str, T: int, H: int, E: int, F: int, Fs: int, k: int) -> None:
    from transformers.models.qwen3_next.configuration_qwen3_next import Qwen3NextConfig
    from transformers.models.qwen3_next.modeling_qwen3_next import Qwen3NextSparseMoeBlock

    cfg = Qwen3NextConfig(hidden_size=H, moe_intermediate_size=F, shared_expert_intermediate_size=Fs,
                          num_experts=E, num_experts_per_tok=k, norm_topk_prob=True)
    blk = Qwen3NextSparseMoeBlock(cfg)
    fill_(blk, 0)
    blk = blk.to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, T, H, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        ref_bf16 = blk(x)
        _, scores, idx = blk.gate(x.reshape(-1, H))
        blk32 = Qwen3NextSparseMoeBlock(cfg)
        blk32.load_state_dict({kk: v.float() for kk, v in blk.state_dict().items()})
        blk32 = blk32.float()
        # fp32 evaluation with the bf16 router's selection (same routing as ref_bf16)
        xf = x.reshape(T, H).float()
        ref_fp32 = blk32.experts(xf, idx, scores.float())
        ref_fp32 = ref_fp32 + torch.sigmoid(blk32.shared_expert_gate(xf)) * blk32.shared_expert(xf)
    sd = blk.state_dict()
    np.savez_compressed(
        OUT / f"{name}.npz", kind="qwen3_next", x=bf16_bits(x.reshape(T, H)),
        w1=bf16_bits(sd["experts.gate_up_proj"]), w2=bf16_bits(sd["experts.down_proj"]),
        router_w=bf16_bits(sd["gate.weight"]), shared_gate_proj=bf16_bits(sd["shared_expert.gate_proj.weight"]),
        shared_up_proj=bf16_bits(sd["shared_expert.up_proj.weight"]),
        shared_down_proj=bf16_bits(sd["shared_expert.down_proj.weight"]),
        shared_gate=bf16_bits(sd["shared_expert_gate.weight"]),
        indices=idx.numpy().astype(np.int32), weights=scores.float().numpy(),
        ref_bf16=bf16_bits(ref_bf16.reshape(T, H)), ref_fp32=ref_fp32.reshape(T, H).numpy())


def gpt_oss_case(name: str, T: int, H: int, E: int, F: int, k: int) -> None:
    from transformers.models.gpt_oss.configuration_gpt_oss import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssMLP

    # ref_fp32 evaluates the experts in fp32 on the bf16 router's selection, so that
    # it differs from ref_bf16 only by arithmetic precision.

    cfg = GptOssConfig(hidden_size=H, intermediate_size=F, num_local_experts=E, num_experts_per_tok=k)
    mlp = GptOssMLP(cfg)
    fill_(mlp, 0)
    with torch.no_grad():  # biases ~N(0, 0.01) as in the benchmark configuration
        gb = torch.Generator().manual_seed(2)
        mlp.experts.gate_up_proj_bias.copy_(torch.randn(mlp.experts.gate_up_proj_bias.shape, generator=gb) * 0.01)
        mlp.experts.down_proj_bias.copy_(torch.randn(mlp.experts.down_proj_bias.shape, generator=gb) * 0.01)
        # Larger gate/up weights so the clamp at +-7 is exercised.
        mlp.experts.gate_up_proj.mul_(60.0)
    mlp = mlp.to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, T, H, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        ref_bf16, _ = mlp(x)
        _, scores, idx = mlp.router(x.reshape(-1, H))
        mlp32 = GptOssMLP(cfg)
        mlp32.load_state_dict({kk: v.float() for kk, v in mlp.state_dict().items()})
        ref_fp32 = mlp32.float().experts(x.reshape(T, H).float(), idx, scores.float())
    sd = mlp.state_dict()
    np.savez_compressed(
        OUT / f"{name}.npz", kind="gpt_oss", x=bf16_bits(x.reshape(T, H)),
        w1=bf16_bits(sd["experts.gate_up_proj"]), w2=bf16_bits(sd["experts.down_proj"]),
        b1=sd["experts.gate_up_proj_bias"].float().numpy(), b2=sd["experts.down_proj_bias"].float().numpy(),
        router_w=bf16_bits(sd["router.weight"]), router_b=bf16_bits(sd["router.bias"]),
        indices=idx.numpy().astype(np.int32), weights=scores.float().numpy(),
        ref_bf16=bf16_bits(ref_bf16.reshape(T, H)), ref_fp32=ref_fp32.reshape(T, H).numpy())


def main() -> None:
    torch.manual_seed(0)
    deepseek_case("deepseek_small", T=24, H=64, E=8, F=48, k=3)
    deepseek_case("deepseek_ragged", T=37, H=128, E=13, F=40, k=6)
    qwen3_next_case("qwen3_next_small", T=20, H=64, E=16, F=32, Fs=48, k=4)
    gpt_oss_case("gpt_oss_small", T=18, H=64, E=6, F=40, k=2)
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
