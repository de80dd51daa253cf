"""cernels_b200 — B200-native (sm_100a) MoE-experts operators.

Drop-in for the reference's ``*_moe_experts`` operator family: same op schemas
(``cernels_b200.ops``), same loader entry points (``cernels_b200.registry``), backed by
hand-written CUDA kernels in ``cernels_b200/_C/libcernels_b200.so`` (C ABI in
``include/cernels_b200.h``).
"""

from . import ops  # noqa: F401  (registers torch.ops.cernels_b200.*)
from .ops import (  # noqa: F401
    cohere2_moe_experts,
    cohere2_moe_experts_decode,
    deepseek_ocr2_moe_experts,
    deepseek_ocr2_moe_experts_decode,
    gpt_oss_moe_experts,
    gpt_oss_moe_experts_decode,
    qwen3_next_moe_experts,
    qwen3_next_moe_experts_decode,
)

__version__ = "0.1.0"
