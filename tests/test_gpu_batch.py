"""Multi-chunk batching (lbrr_forward_chunks): several chunks of one length in
a single forward, every stage run once over the frames of all chunks.  Rows of
the GEMMs, the frequency-axis sequences and the mask estimator's frames do not
interact, and the time-axis attention keeps each chunk's frames apart, so each
chunk's stems must equal, bit for bit, lbrr_forward_chunk on that chunk alone;
one batched chunk is also checked against the CPU oracle (f16path, >= 60 dB).
"""
import numpy as np
import pytest
import torch

from helpers import snr_db
from oracle import bsroformer_ref as R

pytestmark = pytest.mark.gpu

FULL = 588800


@pytest.fixture(scope="module")
def weights():
    return R.make_weights(seed=0, gamma_noise=0.1)


@pytest.fixture(scope="module")
def engine(weights):
    import lbrr
    # room for two full chunks batched: 2 * 1151 frames
    e = lbrr.Engine(0, 2 * FULL + 512)
    e.upload_weights(weights)
    yield e
    e.close()


def _chunks(L, B, seed):
    audio = [R.synth_audio(L, seed=seed + b) for b in range(B)]
    x = torch.from_numpy(np.stack([np.ascontiguousarray(a.T) for a in audio])).cuda()
    return audio, x


def _singles(engine, x):
    B, L = x.shape[0], x.shape[1]
    outs = torch.empty(B, 6, 2, L, device="cuda")
    for b in range(B):
        engine.bench_forward(x[b], outs[b])
    engine.sync()
    return outs


@pytest.mark.parametrize("L,B", [(FULL, 2), (65537, 3), (20000, 4)])
def test_batched_chunks_equal_single_chunks(engine, L, B):
    """Full chunks (T = 1151, nine key tiles with a ragged last one), an odd
    length (the second chunk's samples start off a 16-byte boundary) and a
    short one (T = 40, a single key tile)."""
    _, x = _chunks(L, B, seed=40 + B)
    ref = _singles(engine, x)
    out = torch.empty(B, 6, 2, L, device="cuda")
    # direct launches, then the graph captured on the second call, then its replay
    for _ in range(3):
        out.fill_(float("nan"))
        engine.forward_chunks(x, out)
        engine.sync()
        for b in range(B):
            assert torch.equal(out[b], ref[b]), (L, B, b)


def test_batched_chunk_matches_oracle(engine, weights):
    L, B = 20000, 3
    audio, x = _chunks(L, B, seed=70)
    out = torch.empty(B, 6, 2, L, device="cuda")
    engine.forward_chunks(x, out)
    engine.sync()
    got = out[1].cpu().numpy()
    ref = R.Oracle(weights, "f16path").forward(torch.from_numpy(audio[1])).numpy()
    worst = min(snr_db(got[s], ref[s]) for s in range(6))
    assert worst >= 60.0, worst


def test_batched_chunks_cufft_backend_and_limits(engine):
    """With the cuFFT back end the chunks run one forward each (same bits as
    single calls with that back end); a batch whose frames exceed the engine's
    capacity is refused; the back end alone cannot rerun a batched forward;
    a single-chunk forward after a batch sets the engine back up."""
    import lbrr
    L, B = 20000, 2
    _, x = _chunks(L, B, seed=90)
    base = _singles(engine, x)
    engine.set_option(lbrr.OPT_FFT_BACKEND, 1)
    try:
        ref = _singles(engine, x)
        out = torch.empty(B, 6, 2, L, device="cuda")
        engine.forward_chunks(x, out)
        engine.sync()
        assert torch.equal(out, ref)
    finally:
        engine.set_option(lbrr.OPT_FFT_BACKEND, 0)
    out = torch.empty(B, 6, 2, L, device="cuda")
    engine.forward_chunks(x, out)
    engine.sync()
    with pytest.raises(lbrr.LbrrError) as ei:
        engine.forward_back(out[0])
    assert ei.value.code == lbrr.ERR_STATE
    # 3 x 1151 frames > 2302
    big = torch.zeros(3, FULL, 2, device="cuda")
    with pytest.raises(lbrr.LbrrError) as ei:
        engine.forward_chunks(big, torch.empty(3, 6, 2, FULL, device="cuda"))
    assert ei.value.code == lbrr.ERR_INVALID
    again = _singles(engine, x)
    assert torch.equal(again, base)


def test_batched_chunks_stay_apart_when_one_is_not_finite(engine):
    """A chunk whose samples hold NaN (data only: no index in the forward
    depends on a value) poisons its own stems and nothing else: both
    attention kernels read each chunk through its own coordinate of the
    tensor map, so the rows past a chunk's last frame are zero fill, never the
    next chunk's keys and values.  T = 41 is odd: the frequency axis's last
    frame pair of each chunk holds one frame (and would hold the next chunk's
    first frame if frames were paired across chunks)."""
    L, B = 20480, 3
    _, x = _chunks(L, B, seed=110)
    x[1, 5000:5100] = float("nan")
    ref = _singles(engine, x)
    out = torch.empty(B, 6, 2, L, device="cuda")
    engine.forward_chunks(x, out)
    engine.sync()
    assert torch.isnan(out[1]).any()
    for b in (0, 2):
        assert torch.isfinite(out[b]).all()
        assert torch.equal(out[b], ref[b]), b
