"""Whole-song separation on B200s: the rank-sharded driver (lbrr.song) over the
engine's device-buffer forward gives the oracle's chunked demix of the same
per-chunk model bit for bit, and the multi-engine C entry point
(lbrr_separate_song over two GPUs, chunks dealt round-robin, stitched on the
first) gives exactly the one-GPU result."""
import numpy as np
import pytest
import torch

from oracle import bsroformer_ref as R

pytestmark = pytest.mark.gpu

SONG = R.CHUNK + 300000  # two chunks of the reference plan


@pytest.fixture(scope="module")
def weights():
    return R.make_weights(seed=1, gamma_noise=0.1)


def _engine(device, weights):
    import lbrr
    e = lbrr.Engine(device, R.CHUNK)
    e.upload_weights(weights)
    return e


def test_separate_ranks_one_process_matches_demix(weights):
    from lbrr import song
    eng = _engine(0, weights)
    try:
        audio = R.synth_audio(SONG, seed=11)

        def forward(x, y):
            eng.bench_forward(x, y, stream=torch.cuda.current_stream())

        got = song.separate_ranks(forward, audio, 0, 1, None, "cuda")
        ref = R.demix(lambda c: eng.forward_host(np.ascontiguousarray(c.T)), audio)
        assert got.shape == (6, 2, SONG)
        assert np.array_equal(got, ref)
    finally:
        eng.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpus_match_one(weights):
    import lbrr
    e0, e1 = _engine(0, weights), _engine(1, weights)
    try:
        audio = R.synth_audio(2 * R.CHUNK + 12345, seed=13)  # 3 chunks: GPU 0 takes two
        one = lbrr.separate([e0], audio)
        two = lbrr.separate([e0, e1], audio)
        assert np.isfinite(one).all()
        assert np.array_equal(one, two)
    finally:
        e1.close()
        e0.close()
