"""Seeded synthetic inputs for benchmarking without the real checkpoint or songs.

The reference benchmarks on its shipped `assets/model.safetensors` and real
songs, neither of which can be used here; these stand in with the same shapes:

* ``checkpoint(seed)``: every tensor the reference loader consumes
  (src/weights.rs:307-432, 1989 keys), ``*.weight`` / ``*.bias`` ~ N(0, std),
  RMSNorm gammas 1 (+ optional N(0, gamma_noise)), the shared QKV / out biases
  copied bit-identically into the 24 per-layer keys, and the analytic rotary
  frequencies 1/10000^(2i/64) the loader insists on;
* ``audio(length, seed)``: stereo planar [2][L] fp32, per channel eight sines
  between 50 Hz and 15 kHz plus N(0, 0.05) noise, normalised to peak 0.5.

Both are bit-identical to the generators the parity tests use, so a benchmark
run and a parity run see the same numbers.
"""
from __future__ import annotations

import numpy as np

DIM, DEPTH, HEADS, DIM_HEAD, STEMS, FF_DIM = 256, 12, 8, 64, 6, 1024
FREQS_PER_BAND = [2] * 24 + [4] * 12 + [12] * 8 + [24] * 8 + [48] * 8 + [128, 129]


def checkpoint_keys():
    """(name, shape) of every checkpoint tensor, in the loader's order."""
    keys = [("linear_62_bias_0", (3 * HEADS * DIM_HEAD,)), ("linear_64_bias_0", (DIM,))]
    for layer in range(DEPTH):
        for axis in range(2):
            attn = f"layers.{layer}.{axis}.layers.0.0"
            ff = f"layers.{layer}.{axis}.layers.0.1.net"
            keys += [(f"{attn}.norm.gamma", (DIM,)), (f"{attn}.to_qkv.weight", (3 * HEADS * DIM_HEAD, DIM)),
                     (f"{attn}.to_gates.weight", (HEADS, DIM)), (f"{attn}.to_gates.bias", (HEADS,)),
                     (f"{attn}.to_out.0.weight", (DIM, HEADS * DIM_HEAD)),
                     (f"{ff}.0.gamma", (DIM,)), (f"{ff}.1.weight", (FF_DIM, DIM)), (f"{ff}.1.bias", (FF_DIM,)),
                     (f"{ff}.4.weight", (DIM, FF_DIM)), (f"{ff}.4.bias", (DIM,)),
                     (f"{attn}.to_qkv.bias", (3 * HEADS * DIM_HEAD,)), (f"{attn}.to_out.0.bias", (DIM,)),
                     (f"{attn}.rotary_embed.freqs", (DIM_HEAD // 2,))]
    keys.append(("final_norm.gamma", (DIM,)))
    dims = [2 * 2 * f for f in FREQS_PER_BAND]  # complex x stereo per band
    for b, d in enumerate(dims):
        p = f"band_split.to_features.{b}"
        keys += [(f"{p}.0.gamma", (d,)), (f"{p}.1.weight", (DIM, d)), (f"{p}.1.bias", (DIM,))]
    for s in range(STEMS):
        for b, d in enumerate(dims):
            p = f"mask_estimators.{s}.to_freqs.{b}.0"
            keys += [(f"{p}.0.weight", (FF_DIM, DIM)), (f"{p}.0.bias", (FF_DIM,)),
                     (f"{p}.2.weight", (2 * d, FF_DIM)), (f"{p}.2.bias", (2 * d,))]
    return keys


def checkpoint(seed: int = 0, std: float = 0.02, gamma_noise: float = 0.0) -> dict:
    """{name: fp32 torch tensor} for every checkpoint key (torch's CPU generator
    drives the draws, one N(0,1) block per non-derived tensor in key order)."""
    import torch
    gen = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in checkpoint_keys():
        if name.endswith("rotary_embed.freqs"):
            i = torch.arange(DIM_HEAD // 2, dtype=torch.float32)
            out[name] = 1.0 / torch.pow(torch.tensor(10000.0), 2.0 * i / DIM_HEAD)
        elif name.endswith("to_qkv.bias"):
            out[name] = out["linear_62_bias_0"].clone()
        elif name.endswith("to_out.0.bias"):
            out[name] = out["linear_64_bias_0"].clone()
        elif name.endswith("gamma"):
            g = torch.ones(shape)
            if gamma_noise:
                g = g + torch.randn(shape, generator=gen) * gamma_noise
            out[name] = g
        else:
            out[name] = torch.randn(shape, generator=gen) * std
    return out


def audio(length: int, seed: int = 0, sr: int = 44100) -> np.ndarray:
    """Stereo planar [2][length] fp32 test signal."""
    rs = np.random.RandomState(seed)
    t = np.arange(length, dtype=np.float64) / sr
    out = np.empty((2, length), dtype=np.float32)
    for ch in range(2):
        f = rs.uniform(50.0, 15000.0, 8)
        ph = rs.uniform(0, 2 * np.pi, 8)
        a = rs.uniform(0.05, 0.15, 8)
        sig = (a[:, None] * np.sin(2 * np.pi * f[:, None] * t[None, :] + ph[:, None])).sum(0)
        out[ch] = sig + rs.normal(0.0, 0.05, length)
    peak = np.abs(out).max()
    return (out * (0.5 / max(peak, 1e-12))).astype(np.float32)
