"""Shared helpers for the parity tests (CPU oracle on one side, C ABI on the other)."""
import math

import numpy as np
import torch

from oracle import bsroformer_ref as R


def snr_db(actual, reference) -> float:
    a = np.asarray(actual, dtype=np.float64).ravel()
    r = np.asarray(reference, dtype=np.float64).ravel()
    noise = float(((a - r) ** 2).sum())
    sig = float((r * r).sum())
    if noise == 0.0:
        return math.inf
    return 10.0 * math.log10(max(sig, 1e-300) / noise)


def rel_err(actual, reference) -> float:
    a = np.asarray(actual, dtype=np.float64).ravel()
    r = np.asarray(reference, dtype=np.float64).ravel()
    return float(np.linalg.norm(a - r) / max(np.linalg.norm(r), 1e-30))


def f16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float16).to(torch.float32)


def gen(seed: int):
    return torch.Generator().manual_seed(seed)


def randn(shape, seed, std=1.0):
    return torch.randn(shape, generator=gen(seed)) * std


def fold(a: torch.Tensor, T: int, nb: int, axis: int) -> torch.Tensor:
    """[M][H*64] (token t*nb+b) -> [seqs][H][S][64]."""
    a = a.reshape(T, nb, 8, 64)
    return a.permute(1, 2, 0, 3) if axis == 0 else a.permute(0, 2, 1, 3)


def unfold(a: torch.Tensor, T: int, nb: int, axis: int) -> torch.Tensor:
    if axis == 0:
        return a.permute(2, 0, 1, 3).reshape(T * nb, 512)
    return a.permute(0, 2, 1, 3).reshape(T * nb, 512)


def oracle_attention_gated(qkv: torch.Tensor, gates: torch.Tensor, T: int, nb: int, axis: int) -> torch.Tensor:
    """f16path attention + gate on the already-rotated qkv[M][1536] (fp32 values of fp16)."""
    o = R.Oracle({}, "f16path")
    q, k, v = (fold(qkv[:, i * 512:(i + 1) * 512], T, nb, axis) for i in range(3))
    out = unfold(o.attention(q, k, v), T, nb, axis)
    sig = R.sigmoid(gates).repeat_interleave(64, dim=1)
    return f16(out * sig)
