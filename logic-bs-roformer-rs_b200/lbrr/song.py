"""Whole-song separation sharded over ranks (one process per GPU).

The reference separates a song on one GPU: it reflect-pads the audio by the
border, cuts chunks of ``chunk`` samples every ``step`` samples, runs the
model on each, and overlap-adds the stems with a linear fade of ``border``
samples, dividing by the accumulated fade energy (src/main.rs:7598-7819,
``ola_demix`` :5052-5123, chunk plan :7617-7641).

Here the chunks are independent units dealt round-robin over ``world`` ranks
(chunk i on rank i % world).  Each rank forwards its chunks back to back;
the only exchange is each finished chunk's waveform [6][2][chunk] fp32 sent
point-to-point to rank 0, which overlap-adds in chunk order, so the result
is bit-identical to the single-process demix whatever ``world`` is.  The
transport is whatever ``torch.distributed`` group is passed (NCCL over
NVLink between B200s; gloo on the CPU for tests).
"""
from __future__ import annotations

import numpy as np

CHUNK, STEP, BORDER = 588800, 559360, 29440


def chunk_starts(length: int, chunk: int = CHUNK, step: int = STEP, border: int = BORDER) -> list:
    """Chunk offsets into the padded signal covering [border, border+length)
    (src/main.rs:7617-7641)."""
    if length <= 0:
        raise ValueError("empty audio is unsupported")
    if not (chunk > 1024 and 0 < step <= chunk and 0 <= border and 2 * border <= chunk):
        raise ValueError(f"invalid chunk plan chunk={chunk} step={step} border={border}")
    needed = border + length
    last = max(0, (needed - chunk + step - 1) // step)
    return [i * step for i in range(last + 1)]


def reflect_pad(x: np.ndarray, left: int, right: int) -> np.ndarray:
    """Reflect-pad the last axis, folding as many periods as needed (short songs
    need more than one reflection of the border)."""
    length = x.shape[-1]
    if length == 0:
        raise ValueError("empty audio is unsupported")
    if length == 1:
        return np.repeat(x, left + length + right, axis=-1)
    idx = np.arange(-left, length + right) % (2 * (length - 1))
    idx = np.where(idx < length, idx, 2 * (length - 1) - idx)
    return x[..., idx]


def chunk_weights(index: int, count: int, chunk: int = CHUNK, border: int = BORDER) -> np.ndarray:
    """Linear fade in/out of width ``border``; the song's first chunk keeps full
    weight on its leading border and the last chunk on its trailing border."""
    w = np.ones(chunk, dtype=np.float32)
    if border == 0:
        return w
    ramp = np.arange(border, dtype=np.float32) / np.float32(border)
    if index != 0:
        w[:border] = ramp
    if index != count - 1:
        w[chunk - border:] = ramp[::-1]
    return w


def owned_chunks(n_chunks: int, rank: int, world: int) -> list:
    return list(range(rank, n_chunks, world))


def _reflect_pad_dev(x, left: int, right: int):
    """reflect_pad on a [2][L] torch tensor, as a gather on its own device."""
    import torch
    length = x.shape[-1]
    if length == 1:
        return x.expand(x.shape[0], left + 1 + right).contiguous()
    idx = torch.arange(-left, length + right, device=x.device, dtype=torch.int64) % (2 * (length - 1))
    idx = torch.where(idx < length, idx, 2 * (length - 1) - idx)
    return x.index_select(1, idx)


def separate_ranks(forward, audio_planar: np.ndarray, rank: int, world: int, dist=None, device="cpu",
                   chunk: int = CHUNK, step: int = STEP, border: int = BORDER):
    """Separate one song over ``world`` ranks.

    forward(x, out): x is a [chunk][2] fp32 tensor on ``device`` (interleaved
    stereo), out a [6][2][chunk] fp32 tensor it fills.  Every rank must call
    this with the same audio and plan.  The song is copied to ``device`` once
    (from pinned memory on a GPU) and padded and cut there.  Returns the stems
    [6][2][length] as a numpy array on rank 0 and None elsewhere.
    """
    import torch
    if world > 1 and dist is None:
        raise ValueError("world > 1 needs a torch.distributed module")
    length = audio_planar.shape[-1]
    starts = chunk_starts(length, chunk, step, border)
    needed = border + length
    dev = torch.device(device)
    on_gpu = dev.type == "cuda"
    x = torch.from_numpy(np.ascontiguousarray(audio_planar, dtype=np.float32))
    x = x.pin_memory().to(dev, non_blocking=True) if on_gpu else x
    xp = _reflect_pad_dev(x, border, starts[-1] + chunk - needed)
    mine = owned_chunks(len(starts), rank, world)

    def chunk_input(s):
        return xp[:, s:s + chunk].t().contiguous()

    # Non-zero ranks: forward every owned chunk, send each waveform to rank 0 in
    # chunk order (point-to-point pairs match because both sides walk the same
    # list in the same order).  One buffer per chunk, so a send in flight is
    # never overwritten by the next forward.
    if rank != 0:
        outs = []
        for i in mine:
            y = torch.empty(6, 2, chunk, dtype=torch.float32, device=dev)
            forward(chunk_input(starts[i]), y)
            outs.append(y)
            dist.send(y, dst=0)
        if on_gpu:
            torch.cuda.current_stream().synchronize()  # the sends read `outs` until here
        return None

    result = torch.zeros(12, needed, dtype=torch.float32, device=dev)
    counter = torch.zeros(needed, dtype=torch.float32, device=dev)
    own = torch.empty(6, 2, chunk, dtype=torch.float32, device=dev)
    recv = torch.empty(6, 2, chunk, dtype=torch.float32, device=dev)
    fades = {}
    for i, s in enumerate(starts):
        owner = i % world
        if owner == 0:
            forward(chunk_input(s), own)
            y = own
        else:
            dist.recv(recv, src=owner)
            y = recv
        key = (i == 0, i == len(starts) - 1)  # the fade depends only on these
        if key not in fades:
            fades[key] = torch.from_numpy(chunk_weights(i, len(starts), chunk, border)).to(dev)
        w = fades[key]
        take = min(chunk, needed - s)
        result[:, s:s + take] += y.reshape(12, chunk)[:, :take] * w[:take]
        counter[s:s + take] += w[:take] * w[:take]
    if not bool((counter[border:needed] > 0).all()):
        raise RuntimeError("uncovered audio tail")
    out = (result / counter.clamp_min(1e-8))[:, border:needed].reshape(6, 2, length)
    if not on_gpu:
        return out.numpy()
    host = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)
    host.copy_(out, non_blocking=True)
    torch.cuda.current_stream().synchronize()
    return host.numpy()
