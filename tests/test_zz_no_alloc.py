"""The feed-forward entry point that allocates no device memory.

Some callers cannot call cudaMalloc -- a real-time audio host calling from its
render thread, or an application that hands the library a fixed device-memory
budget -- so lbrr_op_feed_forward_noalloc keeps its fp16 hidden activations in
a static device array instead.  This checks, through the C ABI, that two calls
in a row give the output of the allocating path (lbrr_op_ff1_gelu into a
caller buffer, then lbrr_op_ff2_resid) within the FF2 tolerance of the other
op tests, and that row counts beyond the static array are refused.  The file
is collected last so a failure here cannot hide the other results; it needs
nothing from the other test files.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


def _inputs(rows, seed):
    g = torch.Generator().manual_seed(seed)
    h = (torch.randn(rows, 256, generator=g)).half().cuda()
    w1 = (torch.randn(1024, 256, generator=g) * 0.05).half().cuda()
    b1 = (torch.randn(1024, generator=g) * 0.05).cuda()
    w2 = (torch.randn(256, 1024, generator=g) * 0.02).half().cuda()
    b2 = (torch.randn(256, generator=g) * 0.02).cuda()
    resid = torch.randn(rows, 256, generator=g).cuda()
    return h, w1, b1, w2, b2, resid


@pytest.mark.parametrize("rows", [129, 8192])
def test_noalloc_matches_allocating_path_twice(rows):
    import lbrr
    h, w1, b1, w2, b2, resid = _inputs(rows, 7 + rows)
    ff1 = torch.empty(rows, 1024, dtype=torch.float16, device="cuda")
    ref = torch.empty(rows, 256, device="cuda")
    lbrr.ff1_gelu(h, w1, b1, ff1)
    lbrr.ff2_resid(ff1, w2, b2, resid, ref)
    lbrr.op_sync()
    for _ in range(2):
        x = torch.full((rows, 256), float("nan"), device="cuda")
        lbrr.feed_forward_noalloc(h, w1, b1, w2, b2, resid, x)
        assert torch.isfinite(x).all()
        assert _rel(x.cpu(), ref.cpu()) < 1e-5


def test_noalloc_rejects_rows_beyond_the_static_scratch():
    import lbrr
    h, w1, b1, w2, b2, resid = _inputs(8193, 3)
    x = torch.empty(8193, 256, device="cuda")
    with pytest.raises(lbrr.LbrrError) as ei:
        lbrr.feed_forward_noalloc(h, w1, b1, w2, b2, resid, x)
    assert ei.value.code == lbrr.ERR_INVALID
    assert "8192" in str(ei.value)
