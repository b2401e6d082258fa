"""Shared helpers for the tests: torch <-> oracle numpy conversions, seeded inputs."""
from __future__ import annotations

import numpy as np
import torch

import oracle


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> numpy uint16 bit patterns."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().reshape(-1) if t.dim() == 0 else \
        t.detach().contiguous().cpu().view(torch.uint8).numpy()


def randn_bf16(rows, cols, seed=0, scale=1.0, outliers=0.0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * scale
    if outliers > 0:
        n = int(x.numel() * outliers)
        idx = torch.randperm(x.numel(), generator=g)[:n]
        x.view(-1)[idx] *= 20.0
    return x.to(torch.bfloat16).to(device)


def student_t_bf16(rows, cols, seed=1, df=3.0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(rows, cols, generator=g)
    chi2 = torch.distributions.Chi2(torch.tensor(df)).sample((rows, cols)) if False else \
        torch.randn(rows, cols, int(df), generator=g).pow(2).sum(-1)
    t = z / torch.sqrt(chi2 / df)
    t = t / np.sqrt(df / (df - 2.0))  # unit variance
    return t.to(torch.bfloat16).to(device)


def eff_bits(ref: np.ndarray, approx: np.ndarray) -> float:
    ref = ref.astype(np.float64)
    approx = approx.astype(np.float64)
    err = ((ref - approx) ** 2).sum(-1) / (ref ** 2).sum(-1)
    return float(-np.log2(err.mean()) / 2)
