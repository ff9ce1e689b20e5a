"""Regenerate the seeded inputs of the reference's parity generators.

Each function repeats the numpy ``RandomState`` draws of one generator in
``tools/dump_refs.py`` of the reference (same seeds, same call order, same
dtype casts), so the golden outputs stored in ``dump_refs_subset.npz`` can be
compared against this repository's CPU oracle without committing the inputs.
"""
import numpy as np

F32 = np.float32
FREQS_PER_BANDS = [2] * 24 + [4] * 12 + [12] * 8 + [24] * 8 + [48] * 8 + [128, 129]


def stft_input():
    """gen_stft (tools/dump_refs.py:26-44): x (2, 588800)."""
    rs = np.random.RandomState(42)
    return rs.randn(2, 588800).astype(F32) * F32(0.1)


def rmsnorm_input():
    """gen_rmsnorm (tools/dump_refs.py:47-57)."""
    rs = np.random.RandomState(7)
    x = rs.randn(4096, 256).astype(F32)
    gamma = (rs.randn(256) * 0.1 + 1.0).astype(F32)
    return x, gamma


def bandsplit_input():
    """gen_bandsplit (tools/dump_refs.py:65-88): x (1151, 4100) and per-band gamma/w/b."""
    rs = np.random.RandomState(11)
    x = rs.randn(1151, 2 * sum(FREQS_PER_BANDS) * 2).astype(F32) * F32(0.5)
    gammas, ws, bs = [], [], []
    for f in FREQS_PER_BANDS:
        d = 4 * f
        gammas.append((rs.randn(d) * 0.1 + 1.0).astype(F32))
        ws.append((rs.randn(256, d) * 0.05).astype(F32))
        bs.append((rs.randn(256) * 0.05).astype(F32))
    return x, gammas, ws, bs


def gemm_inputs():
    """gen_gemm (tools/dump_refs.py:91-104): [(x, w, bias)] for (K, N) shapes, M=2048."""
    rs = np.random.RandomState(13)
    out = []
    for k, n in [(256, 1536), (512, 256), (256, 1024), (1024, 256)]:
        x = (rs.randn(2048, k) * 0.3).astype(F32)
        w = (rs.randn(n, k) * 0.05).astype(F32)
        b = (rs.randn(n) * 0.05).astype(F32)
        out.append((x, w, b))
    return out


def qkvrope_input():
    """gen_qkv_rope (tools/dump_refs.py:107-138): x (2,64,256), gamma, w (1536,256), bias."""
    rs = np.random.RandomState(17)
    x = (rs.randn(2, 64, 256) * 0.5).astype(F32)
    gamma = (rs.randn(256) * 0.1 + 1.0).astype(F32)
    w = (rs.randn(1536, 256) * 0.05).astype(F32)
    bias = (rs.randn(1536) * 0.05).astype(F32)
    return x, gamma, w, bias


def attn_input(long: bool):
    """gen_attn_short / gen_attn_long (tools/dump_refs.py:141-165)."""
    if long:
        rs, shape = np.random.RandomState(23), (4, 256, 64)
    else:
        rs, shape = np.random.RandomState(19), (16, 62, 64)
    q = (rs.randn(*shape) * 0.3).astype(F32)
    k = (rs.randn(*shape) * 0.3).astype(F32)
    v = (rs.randn(*shape) * 0.3).astype(F32)
    return q, k, v


def gateff_input():
    """gen_gateout_ff (tools/dump_refs.py:168-197)."""
    rs = np.random.RandomState(29)
    M, dim, heads, dh, ff = 512, 256, 8, 64, 1024
    d = {}
    d["h"] = (rs.randn(M, dim) * 0.5).astype(F32)
    d["x_res"] = (rs.randn(M, dim) * 0.5).astype(F32)
    d["attn_raw"] = (rs.randn(M, heads * dh) * 0.3).astype(F32)
    d["wg"] = (rs.randn(heads, dim) * 0.1).astype(F32)
    d["bg"] = (rs.randn(heads) * 0.1).astype(F32)
    d["wo"] = (rs.randn(dim, heads * dh) * 0.05).astype(F32)
    d["bo"] = (rs.randn(dim) * 0.05).astype(F32)
    d["w1"] = (rs.randn(ff, dim) * 0.05).astype(F32)
    d["b1"] = (rs.randn(ff) * 0.05).astype(F32)
    d["w2"] = (rs.randn(dim, ff) * 0.05).astype(F32)
    d["b2"] = (rs.randn(dim) * 0.05).astype(F32)
    return d
