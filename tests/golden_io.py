"""Loading helpers for the golden fixtures in tests/golden (made by make_golden.py)."""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
NAMES = ["deepseek_small", "deepseek_ragged", "qwen3_next_small", "gpt_oss_small"]


def bf16_from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def load(name: str) -> dict:
    z = np.load(GOLDEN / f"{name}.npz", allow_pickle=False)
    out = {}
    for k in z.files:
        v = z[k]
        if v.dtype == np.uint16:
            out[k] = bf16_from_bits(v)
        elif v.dtype.kind == "U":
            out[k] = str(v)
        else:
            out[k] = torch.from_numpy(v.copy())
    return out
