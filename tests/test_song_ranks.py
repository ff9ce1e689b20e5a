"""Whole-song separation sharded over ranks (lbrr.song.separate_ranks) on the
CPU with the gloo backend: the chunk dealing, the point-to-point exchange to
rank 0 and the chunk-order overlap-add must give the single-process demix
bit for bit (tools/bench_ref.py:47-65 as restated by the oracle, itself
pinned to the reference's identity-model golden vector), whatever the world
size.  A stand-in chunk model replaces the GPU forward, so these tests
exercise only the host-side sharding logic; a rank that fails must make the
others fail fast, not hang.
"""
import datetime

import numpy as np
import pytest
import torch.multiprocessing as mp

from lbrr import song, synthetic
from oracle import bsroformer_ref as R

PLAN = dict(chunk=8192, step=7168, border=1024)
LENGTH = 50000  # 7 chunks under PLAN


def fake_model(xc: np.ndarray) -> np.ndarray:
    """[2][chunk] -> [6][2][chunk]: per-stem gains plus a ramp over the chunk
    position, so a misplaced chunk or a wrong fade shows up."""
    chunk = xc.shape[-1]
    pos = np.arange(chunk, dtype=np.float32) / np.float32(chunk)
    gains = np.arange(1, 7, dtype=np.float32)[:, None, None] * np.float32(0.25)
    return (xc[None] * gains + pos * np.float32(0.01)).astype(np.float32)


def _worker(rank, world, init, audio, out_path, fail_rank, plan):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        def forward(x, y):
            if rank == fail_rank:
                raise RuntimeError(f"rank {rank}: injected chunk failure")
            y.copy_(torch.from_numpy(fake_model(x.numpy().T.copy())))

        res = song.separate_ranks(forward, audio, rank, world, dist, "cpu", **plan)
        if rank == 0:
            np.save(out_path, res)
    finally:
        dist.destroy_process_group()


def _run(world, tmp_path, audio, fail_rank=-1, plan=PLAN):
    out = tmp_path / f"song_w{world}.npy"
    # rendezvous through a file in the test's own directory: no port to race for
    init = f"file://{tmp_path / f'store_w{world}_f{fail_rank}'}"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, init, audio, str(out), fail_rank, plan))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    return out, codes


@pytest.fixture(scope="module")
def audio():
    return synthetic.audio(LENGTH, seed=7)


@pytest.fixture(scope="module")
def expected(audio):
    return R.demix(fake_model, audio, **PLAN)


def test_plan_matches_oracle():
    for length in (1, 1000, 8192 - 1024, 8192 - 1023, LENGTH, 10 ** 6):
        assert song.chunk_starts(length, **PLAN) == R.chunk_starts(length, **PLAN)
    assert song.chunk_starts(180 * 44100) == R.chunk_starts(180 * 44100)
    for i, n in ((0, 1), (0, 5), (2, 5), (4, 5)):
        w = song.chunk_weights(i, n, 8192, 1024)
        f = R.fade_window(8192, 1024).copy()
        if i == 0:
            f[:1024] = 1
        if i == n - 1:
            f[-1024:] = 1
        assert np.array_equal(w, f)
        w = song.chunk_weights(i, n, 8192, 4096, "hann")
        f = R.hann_fade(8192).copy()
        if i == 0:
            f[:4096] = 1
        if i == n - 1:
            f[-4096:] = 1
        assert np.array_equal(w, f)
    x = np.arange(10, dtype=np.float32)[None]
    assert np.array_equal(song.reflect_pad(x, 25, 31), R.reflect_pad(x, 25, 31))
    with pytest.raises(ValueError):
        song.chunk_starts(0)
    with pytest.raises(ValueError):
        song.chunk_starts(100, chunk=4096, step=5000, border=100)


def test_single_process(audio, expected):
    import torch

    def forward(x, y):
        y.copy_(torch.from_numpy(fake_model(x.numpy().T.copy())))

    got = song.separate_ranks(forward, audio, 0, 1, None, "cpu", **PLAN)
    assert got.shape == (6, 2, LENGTH)
    assert np.array_equal(got, expected)


@pytest.mark.parametrize("world", [2, 3])
def test_ranks_bit_identical(world, tmp_path, audio, expected):
    """The overlap-strip exchange between ranks (the library's lbrr_separate_song
    scheme) gives the chunk-order demix bit for bit."""
    out, codes = _run(world, tmp_path, audio)
    assert codes == [0] * world, codes
    got = np.load(out)
    assert np.array_equal(got, expected)


HANN50 = dict(chunk=8192, step=4096, border=4096, fade="hann")
DENSE = dict(chunk=8192, step=2048, border=1024)  # chunks overlap by more than half: gathered on rank 0


@pytest.mark.parametrize("plan", [HANN50, DENSE], ids=["hann50", "dense"])
def test_other_plans_bit_identical(plan, tmp_path, audio):
    p = dict(plan)
    fade = p.pop("fade", "linear")
    want = R.demix(fake_model, audio, **p, fade_kind=fade)
    out, codes = _run(2, tmp_path, audio, plan=plan)
    assert codes == [0, 0], codes
    assert np.array_equal(np.load(out), want)


def test_failed_rank_fails_fast(tmp_path, audio):
    out, codes = _run(2, tmp_path, audio, fail_rank=1)
    assert all(c not in (0, None) for c in codes), codes  # both ranks end with an error, none hangs
    assert not out.exists()
