"""The feed-forward entry point that allocates no device memory.

Some callers cannot call cudaMalloc -- a real-time audio host calling from its
render thread, where an allocation can block, or an application that hands the
library a fixed device-memory budget -- so lbrr_op_feed_forward_noalloc keeps
its fp16 hidden activations in a static device array instead.  Through the C
ABI, two calls in a row must give exactly the output of the allocating path
(lbrr_op_ff1_gelu into a caller buffer, then lbrr_op_ff2_resid: the same two
kernels on the same operands, so bit-equal), and that output must match the
CPU oracle's feed-forward within the FF tolerance of the other op tests; row
counts beyond the static array are refused.  The file is collected last so a
failure here cannot hide the other results; it needs nothing from the other
test files and passes alone in a fresh process as well as after them.
"""
import pytest
import torch

from helpers import f16, rel_err
from oracle import bsroformer_ref as R

pytestmark = pytest.mark.gpu


def _inputs(rows, seed):
    g = torch.Generator().manual_seed(seed)
    h = f16(torch.randn(rows, 256, generator=g))
    w1 = f16(torch.randn(1024, 256, generator=g) * 0.05)
    b1 = torch.randn(1024, generator=g) * 0.05
    w2 = f16(torch.randn(256, 1024, generator=g) * 0.02)
    b2 = torch.randn(256, generator=g) * 0.02
    resid = torch.randn(rows, 256, generator=g)
    return h, w1, b1, w2, b2, resid


@pytest.mark.parametrize("rows", [129, 8192])
def test_noalloc_matches_allocating_path_twice(rows):
    import lbrr
    h, w1, b1, w2, b2, resid = _inputs(rows, 7 + rows)
    hd, w1d, w2d = h.half().cuda(), w1.half().cuda(), w2.half().cuda()
    b1d, b2d, rd = b1.cuda(), b2.cuda(), resid.cuda()
    ff1 = torch.empty(rows, 1024, dtype=torch.float16, device="cuda")
    ref = torch.empty(rows, 256, device="cuda")
    lbrr.ff1_gelu(hd, w1d, b1d, ff1)
    lbrr.ff2_resid(ff1, w2d, b2d, rd, ref)
    lbrr.op_sync()
    model = f16(R.gelu_as(h @ w1.T + b1)) @ w2.T + b2 + resid
    for _ in range(2):
        x = torch.full((rows, 256), float("nan"), device="cuda")
        lbrr.feed_forward_noalloc(hd, w1d, b1d, w2d, b2d, rd, x)
        assert torch.isfinite(x).all()
        assert torch.equal(x, ref)
        assert rel_err(x.cpu(), model) < 1e-4


def test_noalloc_rejects_rows_beyond_the_static_scratch():
    import lbrr
    h, w1, b1, w2, b2, resid = (t.cuda() for t in _inputs(8193, 3))
    x = torch.empty(8193, 256, device="cuda")
    with pytest.raises(lbrr.LbrrError) as ei:
        lbrr.feed_forward_noalloc(h.half(), w1.half(), b1, w2.half(), b2, resid, x)
    assert ei.value.code == lbrr.ERR_INVALID
    assert "8192" in str(ei.value)
