"""Per-op parity on the GPU: each C-ABI entry point against the CPU oracle.

Inputs are seeded; fp16 operands are exact fp16 values on both sides, so the
only differences are accumulation order (fp32 on the tensor cores vs the CPU)
and the occasional fp16 rounding flip that causes.  Tolerances are written per
test: relative L2 error, and max abs error against the output scale.
"""
import numpy as np
import pytest
import torch

from helpers import f16, fold, oracle_attention_gated, randn, rel_err, snr_db, unfold
from oracle import bsroformer_ref as R

pytestmark = pytest.mark.gpu

NB = 62


@pytest.fixture(scope="module")
def lb():
    import lbrr
    lbrr.lib()
    return lbrr


def cuda(t, dtype=None):
    return t.to(dtype or t.dtype).contiguous().cuda()


@pytest.mark.parametrize("M", [62, 2294, 71362])
def test_norm_gates(lb, M):
    x = randn((M, 256), 1, 0.7)
    gamma = 1.0 + randn((256,), 2, 0.1)
    gw, gb = randn((8, 256), 3, 0.05), randn((8,), 4, 0.05)
    h16 = torch.empty(M, 256, dtype=torch.float16, device="cuda")
    gates = torch.empty(M, 8, device="cuda")
    lb.norm_gates(cuda(x), cuda(gamma), cuda(gw), cuda(gb), h16, gates)
    lb.op_sync()
    hf = R.rmsnorm(x, gamma, "right")
    assert rel_err(h16.float().cpu(), f16(hf)) < 2e-3
    assert rel_err(gates.cpu(), hf @ gw.T + gb) < 1e-5


# (1151, 62): the full chunk, whose last tile has rows past the end; bands 1
# and 100 take the epilogue's global-memory RoPE path (a 32-row warp spans more
# than two frames / the table exceeds the shared-memory copy)
@pytest.mark.parametrize("T,axis,nb", [(1, 0, NB), (37, 0, NB), (259, 0, NB), (1151, 0, NB), (1, 1, NB), (37, 1, NB),
                                       (1151, 1, NB), (300, 0, 1), (9, 1, 100)])
def test_qkv_rope(lb, T, axis, nb):
    M = T * nb
    h = f16(randn((M, 256), 10 + T, 1.0))
    w = f16(randn((1536, 256), 11, 0.02))
    bias16 = f16(randn((1536,), 12, 0.02))
    P = T if axis == 0 else nb
    cos, sin = R.rope_tables(P)
    qkv = torch.empty(M, 1536, dtype=torch.float16, device="cuda")
    lb.qkv_rope(cuda(h, torch.float16), cuda(w, torch.float16), cuda(bias16), cuda(cos), cuda(sin), qkv, T, nb, axis)
    lb.op_sync()
    ref = f16(h @ w.T + bias16)
    q, k, v = ref[:, :512], ref[:, 512:1024], ref[:, 1024:]
    qr = unfold(f16(R.rope(fold(q, T, nb, axis), cos, sin)), T, nb, axis)
    kr = unfold(f16(R.rope(fold(k, T, nb, axis), cos, sin)), T, nb, axis)
    got = qkv.float().cpu()
    for sl, r in ((slice(0, 512), qr), (slice(512, 1024), kr), (slice(1024, 1536), v)):
        assert rel_err(got[:, sl], r) < 2e-3
        assert float((got[:, sl] - r).abs().max()) <= 4e-3 * float(r.abs().max())


@pytest.mark.parametrize("T,axis", [(1, 0), (37, 0), (129, 0), (200, 0), (259, 0), (300, 0), (1151, 0), (1, 1), (2, 1),
                                    (37, 1), (1151, 1)])
def test_attention(lb, T, axis):
    M = T * NB
    qkv = f16(randn((M, 1536), 20 + T, 1.0))
    gates = randn((M, 8), 21, 1.0)
    out = torch.empty(M, 512, dtype=torch.float16, device="cuda")
    lb.attention(cuda(qkv, torch.float16), cuda(gates), out, T, NB, axis)
    lb.op_sync()
    ref = oracle_attention_gated(qkv, gates, T, NB, axis)
    got = out.float().cpu()
    assert torch.isfinite(got).all()
    assert snr_db(got, ref) > 55.0, snr_db(got, ref)


@pytest.mark.parametrize("T,nb", [(5, 40), (3, 64), (4, 1)])
def test_attention_freq_band_counts(lb, T, nb):
    """Frequency axis with band counts other than 62: each frame's nb tokens
    sit at rows 0.. and 64.. of the packed tile, the padding rows zeroed."""
    M = T * nb
    qkv = f16(randn((M, 1536), 70 + nb, 1.0))
    gates = randn((M, 8), 71, 1.0)
    out = torch.empty(M, 512, dtype=torch.float16, device="cuda")
    lb.attention(cuda(qkv, torch.float16), cuda(gates), out, T, nb, 1)
    lb.op_sync()
    ref = oracle_attention_gated(qkv, gates, T, nb, 1)
    got = out.float().cpu()
    assert torch.isfinite(got).all()
    assert snr_db(got, ref) > 55.0, snr_db(got, ref)


def test_attention_max_jump(lb):
    """Time axis: keys of the second and third key tiles score far above the
    first tile's, so the row max grows by more than 2^8 in exp2 units mid-row
    (enough to overflow an fp16 P against the old max): the kernel must raise
    its reference max, rescale O and recompute those tiles' P."""
    T = 300
    M = T * NB
    qkv = randn((M, 1536), 33, 1.0)
    frame = torch.arange(M) // NB  # token = t * nb + b
    k = qkv[:, 512:1024]
    k[(frame >= 128) & (frame < 160)] *= 12.0
    k[frame >= 256] *= 30.0
    qkv = f16(qkv)
    gates = randn((M, 8), 34, 1.0)
    out = torch.empty(M, 512, dtype=torch.float16, device="cuda")
    lb.attention(cuda(qkv, torch.float16), cuda(gates), out, T, NB, 0)
    lb.op_sync()
    ref = oracle_attention_gated(qkv, gates, T, NB, 0)
    got = out.float().cpu()
    assert torch.isfinite(got).all()
    assert snr_db(got, ref) > 55.0, snr_db(got, ref)


@pytest.mark.parametrize("M", [62, 2294, 16058])
def test_outproj_norm(lb, M):
    s = f16(randn((M, 512), 30, 0.5))
    w = f16(randn((256, 512), 31, 0.02))
    bias = randn((256,), 32, 0.02)
    x = randn((M, 256), 33, 1.0)
    gamma = 1.0 + randn((256,), 34, 0.1)
    ao = torch.empty(M, 256, device="cuda")
    h16 = torch.empty(M, 256, dtype=torch.float16, device="cuda")
    lb.outproj_norm(cuda(s, torch.float16), cuda(w, torch.float16), cuda(bias), cuda(x), cuda(gamma), ao, h16)
    lb.op_sync()
    ref = s @ w.T + bias + x
    assert rel_err(ao.cpu(), ref) < 1e-5
    assert rel_err(h16.float().cpu(), f16(R.rmsnorm(ref, gamma, "left"))) < 2e-3


@pytest.mark.parametrize("M", [1, 37, 127, 129, 16058, 71362])
def test_ff1_gelu(lb, M):
    # the M list of the reference's FF1 regression (src/main.rs:8024)
    h = f16(randn((M, 256), 40, 1.0))
    w = f16(randn((1024, 256), 41, 0.05))
    b = randn((1024,), 42, 0.05)
    out = torch.empty(M, 1024, dtype=torch.float16, device="cuda")
    lb.ff1_gelu(cuda(h, torch.float16), cuda(w, torch.float16), cuda(b), out)
    lb.op_sync()
    ref = f16(R.gelu_as(h @ w.T + b))
    got = out.float().cpu()
    assert rel_err(got, ref) < 2e-3
    assert float((got - ref).abs().max()) <= 4e-3 * float(ref.abs().max())


@pytest.mark.parametrize("M", [1, 129, 16058])
def test_ff2_resid(lb, M):
    f = f16(randn((M, 1024), 50, 0.5))
    w = f16(randn((256, 1024), 51, 0.02))
    b = randn((256,), 52, 0.02)
    r = randn((M, 256), 53, 1.0)
    x = torch.empty(M, 256, device="cuda")
    lb.ff2_resid(cuda(f, torch.float16), cuda(w, torch.float16), cuda(b), cuda(r), x)
    lb.op_sync()
    assert rel_err(x.cpu(), f @ w.T + b + r) < 1e-5


@pytest.mark.parametrize("M", [1, 37, 129, 2294, 16058, 71362])
def test_feed_forward_fused(lb, M):
    """The fused FF kernel gives the two-kernel path (FF1 + GELU into an fp16
    buffer, then FF2 + bias + residual) bit for bit: same fp16 GELU values,
    same K order of the FF2 accumulation; and both match the fp32 model."""
    h = cuda(f16(randn((M, 256), 60, 1.0)), torch.float16)
    w1 = cuda(f16(randn((1024, 256), 61, 0.05)), torch.float16)
    b1 = cuda(randn((1024,), 62, 0.05))
    w2 = cuda(f16(randn((256, 1024), 63, 0.02)), torch.float16)
    b2 = cuda(randn((256,), 64, 0.02))
    r = cuda(randn((M, 256), 65, 1.0))
    ff1 = torch.empty(M, 1024, dtype=torch.float16, device="cuda")
    ref = torch.empty(M, 256, device="cuda")
    lb.ff1_gelu(h, w1, b1, ff1)
    lb.ff2_resid(ff1, w2, b2, r, ref)
    got = torch.full((M, 256), float("nan"), device="cuda")
    lb.feed_forward(h, w1, b1, w2, b2, r, got)
    lb.op_sync()
    assert torch.equal(got, ref)
    model = f16(R.gelu_as(h.float().cpu() @ w1.float().cpu().T + b1.cpu())) @ w2.float().cpu().T + b2.cpu() + r.cpu()
    assert rel_err(got.cpu(), model) < 1e-4


def test_invalid_arguments_are_rejected(lb):
    with pytest.raises(lb.LbrrError) as ei:
        lb.check(lb.lib().lbrr_op_attention(None, None, None, 10, 62, 0, None))
    assert ei.value.code == lb.ERR_INVALID
    with pytest.raises(lb.LbrrError):
        lb.check(lb.lib().lbrr_op_attention(1, 1, 1, 10, 100, 1, None))  # freq axis needs bands <= 64
