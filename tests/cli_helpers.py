"""Inputs for the host CLI tests: a model directory (training-style YAML and a
.safetensors checkpoint) and WAV files, written here in Python."""
import json
import struct
import subprocess
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parents[1] / "logic-bs-roformer-rs_b200"
CLI = PKG / "lbrr" / "lbrr_b200"

FREQS = [2] * 24 + [4] * 12 + [12] * 8 + [24] * 8 + [48] * 8 + [128, 129]


def model_yaml(depth=12, freqs=None, dim_freqs_in=1025, drop=(), instruments=None) -> str:
    """A config in the layout of the training YAML: a `!!python/tuple` list one
    level deeper, another at its key's own indentation, an inline list of
    quoted names, comments and keys the engine ignores."""
    freqs = FREQS if freqs is None else freqs
    instruments = instruments or ["bass", "drums", "other", "vocals", "guitar", "piano"]
    lines = ["audio:", "  chunk_size: 588800 # samples", "  n_fft: 2048", "  num_channels: 2",
             "  sample_rate: 44100", "", "model:", "  dim: 256", f"  depth: {depth}", "  stereo: true",
             "  num_stems: 6", "  freqs_per_bands: !!python/tuple"]
    lines += [f"    - {f}" for f in freqs]
    lines += ["  dim_head: 64", "  heads: 8", "  attn_dropout: 0.1", f"  dim_freqs_in: {dim_freqs_in}",
              "  stft_n_fft: 2048", "  stft_hop_length: 512", "  stft_win_length: 2048",
              "  multi_stft_resolutions_window_sizes: !!python/tuple", "  - 4096", "  - 2048",
              "  multi_stft_hop_size: 147", "  mlp_expansion_factor: 4", "  use_shared_bias: True",
              "training:", "  batch_size: 2",
              "  instruments: [" + ", ".join(f"'{n}'" for n in instruments) + "]", "  lr: 1.0e-5", ""]
    return "\n".join(l for l in lines if not any(l.strip().startswith(d + ":") for d in drop))


def write_safetensors(path, tensors: dict):
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        b = np.ascontiguousarray(np.asarray(a, dtype=np.float32)).tobytes()
        header[name] = {"dtype": "F32", "shape": list(np.shape(a)), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_wav(path, interleaved: np.ndarray, channels: int, rate=44100, fmt="f32"):
    """fmt: f32 (IEEE float), s16 or s24 (PCM, rounded toward zero from x * 2^15 / 2^23)."""
    x = np.asarray(interleaved, dtype=np.float32)
    if fmt == "f32":
        data, tag, bits = x.astype("<f4").tobytes(), 3, 32
    elif fmt == "s16":
        data, tag, bits = np.clip(x * 32768.0, -32768, 32767).astype("<i2").tobytes(), 1, 16
    else:
        v = np.clip(x * 8388608.0, -8388608, 8388607).astype("<i4")
        data, tag, bits = np.stack([v & 255, (v >> 8) & 255, (v >> 16) & 255], -1).astype(np.uint8).tobytes(), 1, 24
    ba = channels * bits // 8
    fmt_chunk = struct.pack("<HHIIHH", tag, channels, rate, rate * ba, ba, bits)
    extra = b"LIST" + struct.pack("<I", 4) + b"INFO"  # a chunk readers must skip
    body = b"WAVE" + b"fmt " + struct.pack("<I", 16) + fmt_chunk + extra + b"data" + struct.pack("<I", len(data)) + data
    Path(path).write_bytes(b"RIFF" + struct.pack("<I", len(body)) + body)


def read_wav_f32(path):
    b = Path(path).read_bytes()
    assert b[:4] == b"RIFF" and b[8:12] == b"WAVE"
    tag, ch, rate, _, _, bits = struct.unpack("<HHIIHH", b[20:36])
    assert (tag, bits) == (3, 32) and b[36:40] == b"data"
    n = struct.unpack("<I", b[40:44])[0]
    return rate, ch, np.frombuffer(b[44:44 + n], dtype="<f4")


def run_cli(*args, timeout=600):
    return subprocess.run([str(CLI), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def ensure_cli():
    import importlib.util
    if not CLI.exists():
        spec = importlib.util.spec_from_file_location("lbrr_build", PKG / "build.py")
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        m.build_cli()
    return CLI
