"""Whole-song separation sharded over ranks (one process per GPU).

The reference separates a song on one GPU: it reflect-pads the audio by the
border, cuts chunks of ``chunk`` samples every ``step`` samples, runs the
model on each, and overlap-adds the stems with a linear fade of ``border``
samples, dividing by the accumulated fade energy (src/main.rs:7598-7819,
``ola_demix`` :5052-5123, chunk plan :7617-7641).

Here the chunks are independent units dealt round-robin over ``world`` ranks
(chunk c on rank c % world), the same exchange as the library's
lbrr_separate_song: each rank finishes the song samples its chunks start,
[s_c - border, s_{c+1} - border), from its own waveform and the previous
chunk's overlap strip (y*w and w*w over the chunk - step overlapping samples)
sent point-to-point by that chunk's rank; the finished regions go to rank 0,
which assembles the output.  Every sample is (0 + y_{c-1} w_{c-1} + y_c w_c)
/ max(0 + w_{c-1}^2 + w_c^2, 1e-8) with each operation rounded on its own,
the operations of chunk-order accumulation, so the result is bit-identical to
the single-process demix whatever ``world`` is.  Plans whose chunks overlap by
more than half fall back to sending every waveform to rank 0.  The transport
is whatever ``torch.distributed`` group is passed (NCCL over NVLink between
B200s; gloo on the CPU for tests).
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


def chunk_weights(index: int, count: int, chunk: int = CHUNK, border: int = BORDER, fade: str = "linear") -> np.ndarray:
    """Linear fade in/out of width ``border`` (or, fade="hann", a periodic Hann
    window over the chunk); the song's first chunk keeps full weight on its
    leading border and the last chunk on its trailing border."""
    if fade == "hann":
        n = np.arange(chunk, dtype=np.float64)
        w = (0.5 * (1.0 - np.cos(2.0 * np.pi * n / chunk))).astype(np.float32)
        if border:
            if index == 0:
                w[:border] = 1.0
            if index == count - 1:
                w[chunk - border:] = 1.0
        return w
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
                   chunk: int = CHUNK, step: int = STEP, border: int = BORDER, fade: str = "linear"):
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
    n = len(starts)
    needed = border + length
    dev = torch.device(device)
    on_gpu = dev.type == "cuda"
    x = torch.from_numpy(np.ascontiguousarray(audio_planar, dtype=np.float32))
    x = x.pin_memory().to(dev, non_blocking=True) if on_gpu else x
    xp = _reflect_pad_dev(x, border, starts[-1] + chunk - needed)
    fades = {}

    def weights(i):
        key = (i == 0, i == n - 1)  # the fade depends only on these
        if key not in fades:
            fades[key] = torch.from_numpy(chunk_weights(i, n, chunk, border, fade)).to(dev)
        return fades[key]

    def run_chunk(i):
        y = torch.empty(6, 2, chunk, dtype=torch.float32, device=dev)
        forward(xp[:, starts[i]:starts[i] + chunk].t().contiguous(), y)
        return y.reshape(12, chunk)

    if 2 * step < chunk:
        return _gather_all(run_chunk, weights, starts, rank, world, dist, dev, chunk, needed, border, length)

    ov = chunk - step
    owner = [i % world for i in range(n)]
    pending = []  # non-blocking sends and the tensors they read
    out = torch.empty(12, length, dtype=torch.float32, device=dev) if rank == 0 else None

    def region_of(i):
        o0 = 0 if i == 0 else starts[i] - border
        o1 = starts[i + 1] - border if i + 1 < n else length
        return o0, o1

    strip_keep = {}
    for i in range(n):
        if owner[i] != rank:
            if rank == 0:  # assemble a region finished on another rank
                o0, o1 = region_of(i)
                buf = torch.empty(12, o1 - o0, dtype=torch.float32, device=dev)
                dist.recv(buf, src=owner[i], tag=2 * i + 1)
                out[:, o0:o1] = buf
            continue
        y = run_chunk(i)
        w = weights(i)
        # the previous chunk's overlap strip: y*w (12 rows) and w*w
        prev = None
        if i > 0:
            if owner[i - 1] == rank:
                prev = strip_keep.pop(i - 1)
            else:
                prev = torch.empty(13, ov, dtype=torch.float32, device=dev)
                dist.recv(prev, src=owner[i - 1], tag=2 * i)
        o0, o1 = region_of(i)
        r0 = o0 + border - starts[i]
        rel = slice(r0, r0 + (o1 - o0))
        num = y[:, rel] * w[rel]
        den = w[rel] * w[rel]
        if prev is not None:
            h = min(ov - r0, o1 - o0)  # head samples also covered by the previous chunk
            if h > 0:
                num[:, :h] = prev[:12, r0:r0 + h] + num[:, :h]
                den[:h] = prev[12, r0:r0 + h] + den[:h]
        region = num / den.clamp_min(1e-8)
        if rank == 0:
            out[:, o0:o1] = region
        else:
            pending.append((dist.isend(region.contiguous(), dst=0, tag=2 * i + 1), region))
        if i + 1 < n:
            strip = torch.cat([y[:, step:] * w[step:], (w[step:] * w[step:])[None]], 0).contiguous()
            if owner[i + 1] == rank:
                strip_keep[i] = strip
            else:
                pending.append((dist.isend(strip, dst=owner[i + 1], tag=2 * (i + 1)), strip))
    for req, _ in pending:
        req.wait()
    if on_gpu:
        torch.cuda.current_stream().synchronize()
    if rank != 0:
        return None
    out = out.reshape(6, 2, length)
    if not on_gpu:
        return out.numpy()
    host = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)
    host.copy_(out, non_blocking=True)
    torch.cuda.current_stream().synchronize()
    return host.numpy()


def _gather_all(run_chunk, weights, starts, rank, world, dist, dev, chunk, needed, border, length):
    """Plans overlapping by more than half: every waveform goes to rank 0, which
    accumulates them in chunk order."""
    import torch
    n = len(starts)
    if rank != 0:
        outs = []
        for i in range(rank, n, world):
            y = run_chunk(i)
            outs.append(y)
            dist.send(y, dst=0, tag=2 * i + 1)
        if dev.type == "cuda":
            torch.cuda.current_stream().synchronize()
        return None
    result = torch.zeros(12, needed, dtype=torch.float32, device=dev)
    counter = torch.zeros(needed, dtype=torch.float32, device=dev)
    recv = torch.empty(12, chunk, dtype=torch.float32, device=dev)
    for i, s in enumerate(starts):
        if i % world == 0:
            y = run_chunk(i)
        else:
            dist.recv(recv, src=i % world, tag=2 * i + 1)
            y = recv
        w = weights(i)
        take = min(chunk, needed - s)
        result[:, s:s + take] += y[:, :take] * w[:take]
        counter[s:s + take] += w[:take] * w[:take]
    if not bool((counter[border:needed] > 0).all()):
        raise RuntimeError("uncovered audio tail")
    out = (result / counter.clamp_min(1e-8))[:, border:needed].reshape(6, 2, length)
    if dev.type != "cuda":
        return out.numpy()
    host = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)
    host.copy_(out, non_blocking=True)
    torch.cuda.current_stream().synchronize()
    return host.numpy()
