"""Whole-song separation on B200s: the rank-sharded driver (lbrr.song) over the
engine's device-buffer forward gives the oracle's chunked demix of the same
per-chunk model bit for bit, and so does the multi-engine C entry point
(lbrr_separate_song: chunks dealt round-robin, each engine finishing its own
samples from its chunks and the previous chunk's overlap strip), for one
engine, two engines on one GPU and two GPUs alike."""
import numpy as np
import pytest
import torch

from helpers import snr_db
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


def test_two_engines_one_gpu_match_oracle(weights):
    # the overlap strips travel between engines even on one device
    import lbrr
    e0, e1 = _engine(0, weights), _engine(0, weights)
    try:
        audio = R.synth_audio(2 * R.CHUNK + 12345, seed=17)  # 3 chunks
        two = lbrr.separate([e0, e1], audio)
        one = lbrr.separate([e0], audio)
        ref = R.demix(lambda c: e0.forward_host(np.ascontiguousarray(c.T)), audio)
        assert np.array_equal(two, one)
        assert np.array_equal(one, ref)
    finally:
        e1.close()
        e0.close()


def test_short_song_and_serial_plan(weights):
    # one chunk (shorter than the plan's chunk), and a plan whose chunks overlap
    # by more than half (accumulated on one engine in chunk order)
    import lbrr
    e0 = _engine(0, weights)
    try:
        audio = R.synth_audio(50000, seed=19)
        got = lbrr.separate([e0], audio, chunk=65536, step=60000, border=5536)
        ref = R.demix(lambda c: e0.forward_host(np.ascontiguousarray(c.T)), audio, 65536, 60000, 5536)
        assert np.array_equal(got, ref)
        audio = R.synth_audio(200000, seed=23)
        got = lbrr.separate([e0], audio, chunk=65536, step=20000, border=8192)
        ref = R.demix(lambda c: e0.forward_host(np.ascontiguousarray(c.T)), audio, 65536, 20000, 8192)
        assert snr_db(got, ref) > 100.0
    finally:
        e0.close()


def test_hann50_plan_matches_oracle(weights):
    """BASELINE config 4's plan (50 % overlap, Hann-weighted overlap-add) through
    lbrr_separate_song with one and two engines: bit-equal to the oracle's
    chunk-order demix with the same per-chunk model and the same fp32 window."""
    import lbrr
    e0, e1 = _engine(0, weights), _engine(0, weights)
    try:
        audio = R.synth_audio(900000, seed=29)  # 4 chunks of the 50 % plan
        p = dict(lbrr.HANN50)
        one = lbrr.separate([e0], audio, **p)
        two = lbrr.separate([e0, e1], audio, **p)
        fade = p.pop("fade")
        ref = R.demix(lambda c: e0.forward_host(np.ascontiguousarray(c.T)), audio, **p, fade_kind=fade)
        assert np.array_equal(one, ref)
        assert np.array_equal(two, ref)
    finally:
        e1.close()
        e0.close()


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


def test_page_locked_song_buffers_same_bits(weights):
    """With a page-locked song and output array (lbrr.pinned_empty) interior
    chunks are uploaded straight from the song and finished regions are
    downloaded straight into the output; the bits are those of the staged path,
    for both plans and a song whose chunks include reflected edges."""
    import lbrr
    e0, e1 = _engine(0, weights), _engine(0, weights)
    try:
        audio = R.synth_audio(3 * R.CHUNK + 4321, seed=23)
        il = np.ascontiguousarray(audio.T)
        xh = lbrr.pinned_empty(il.shape)
        xh[:] = il
        for plan in ({}, lbrr.HANN50):
            ref = lbrr.separate([e0, e1], il, interleaved=True, **plan)
            out = lbrr.pinned_empty(ref.shape)
            out[:] = np.nan
            lbrr.separate([e0, e1], xh, interleaved=True, out=out, **plan)
            assert np.array_equal(out, ref)
            # pinned input with a pageable output, and the reverse
            assert np.array_equal(lbrr.separate([e0, e1], xh, interleaved=True, **plan), ref)
            out[:] = np.nan
            lbrr.separate([e0, e1], il, interleaved=True, out=out, **plan)
            assert np.array_equal(out, ref)
    finally:
        e1.close()
        e0.close()
