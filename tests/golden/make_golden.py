#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory from the reference's own code.

Run with ``--reference DIR`` naming a checkout of the reference repository
(read-only).  Two reference modules are imported and executed:

* ``tools/dump_refs.py`` -- the reference's seeded per-op parity generators
  (torch CPU): STFT, RMSNorm, band-split, the four trunk GEMM shapes, QKV+RoPE,
  short/long SDPA and gate/out-proj/FF.  Its ``OUT`` directory is redirected to
  a temporary folder; ``gen_e2e_mid`` (needs the absent checkpoint) is skipped.
* ``tools/bench_ref.py`` -- ``chunk_starts``, ``reflect_pad`` and ``demix`` of the
  song path, driven with an identity model exactly like ``tools/test_benchmark.py``.

The generators' inputs are seeded numpy draws; the fixtures keep the seeds'
outputs only as row subsets plus a few input spot values, and the tests
regenerate the inputs with the same ``RandomState`` call order
(``tests/golden/golden_inputs.py``).  Output: ``dump_refs_subset.npz`` and
``demix_identity.npz``.
"""
import argparse
import importlib.util
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.path.insert(0, str(path.parent))
    spec.loader.exec_module(mod)
    return mod


def dump_refs_subset(ref: Path) -> dict:
    import torch
    dr = load_module(ref / "tools" / "dump_refs.py", "lbrr_ref_dump_refs")
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        dr.OUT = Path(tmp)
        torch.manual_seed(0)
        for gen in (dr.gen_stft, dr.gen_rmsnorm, dr.gen_bandsplit, dr.gen_gemm, dr.gen_qkv_rope,
                    dr.gen_attn_short, dr.gen_attn_long, dr.gen_gateout_ff):
            gen()
        z = {n: np.load(Path(tmp) / f"{n}.npz") for n in
             ("stft", "rmsnorm", "bandsplit", "gemm", "qkvrope", "attn_short", "attn_long", "gateff")}
    # STFT: spec (CH, 1025, T, 2); keep frames at both reflect edges and the middle
    frames = np.array([0, 1, 2, 3, 575, 576, 1147, 1148, 1149, 1150])
    out["stft_frames"] = frames
    out["stft_spec"] = z["stft"]["spec"][:, :, frames, :].astype(np.float32)
    out["stft_x_head"] = z["stft"]["x"][:, :8]
    out["stft_window"] = z["stft"]["window"]
    # RMSNorm: first 64 rows
    out["rmsnorm_rows"] = np.int64(64)
    out["rmsnorm_out"] = z["rmsnorm"]["out"][:64]
    out["rmsnorm_gamma"] = z["rmsnorm"]["gamma"]
    # band split: (t, 62, 256) -> first 16 frames, all bands
    out["bandsplit_out"] = z["bandsplit"]["out"][:4]
    out["bandsplit_b"] = z["bandsplit"]["b"]
    # GEMMs: first 32 rows of each y
    for gi, (k, n) in enumerate([(256, 1536), (512, 256), (256, 1024), (1024, 256)]):
        out[f"gemm_y{gi}"] = z["gemm"][f"y{gi}"].reshape(2048, n)[:32]
        out[f"gemm_b{gi}"] = z["gemm"][f"b{gi}"]
    # QKV + RoPE: batch 0, first 16 positions (q/k/v are (b, seq, heads, dh))
    for key in ("q", "k", "v"):
        out[f"qkvrope_{key}"] = z["qkvrope"][key].reshape(2, 64, 8, 64)[:1, :16]
    for key in ("cos", "sin"):
        out[f"qkvrope_{key}"] = z["qkvrope"][key]
    # SDPA: first 4 of 16 (short) and first 1 of 4 (long) (b,h) groups
    out["attn_short_out"] = z["attn_short"]["out"].reshape(16, 62, 64)[:4]
    out["attn_long_out"] = z["attn_long"]["out"].reshape(4, 256, 64)[:1]
    # gate / out-proj / FF: first 32 rows
    out["gateff_attn_out"] = z["gateff"]["attn_out"].reshape(512, 256)[:32]
    out["gateff_ff1"] = z["gateff"]["ff1"].reshape(512, 1024)[:32]
    out["gateff_ff_out"] = z["gateff"]["ff_out"].reshape(512, 256)[:32]
    return out


def demix_identity(ref: Path) -> dict:
    import torch
    br = load_module(ref / "tools" / "bench_ref.py", "lbrr_ref_bench_ref")

    class Identity:
        def __call__(self, x):
            return x[:, None].expand(-1, 6, -1, -1)

    out = {}
    lengths = [1, 37, 44100 * 8, br.CHUNK, 44100 * 30, br.STEP * 3 + 91]
    out["lengths"] = np.array(lengths)
    for length in lengths:
        out[f"starts_{length}"] = np.array(br.chunk_starts(length))
    x = np.array([[1, 2, 3], [10, 20, 30]], dtype=np.float32)
    out["reflect_17_29"] = br.reflect_pad(torch.from_numpy(x), 17, 29).numpy()
    # identity-model demix on a seeded random stereo signal (exercises fades,
    # first/last overrides and the tail) -- keep strided samples
    for length in (37, br.CHUNK + 1000, br.STEP * 3 + 91):
        rs = np.random.RandomState(length % 1000)
        sig = rs.randn(1, 2, length).astype(np.float32)
        y = br.demix(Identity(), torch.from_numpy(sig)).numpy()[0]  # [6][2][L]
        idx = np.unique(np.concatenate([np.arange(0, length, max(1, length // 4000)),
                                        np.arange(max(0, length - 64), length)]))
        out[f"demix_idx_{length}"] = idx
        out[f"demix_y_{length}"] = y[:, :, idx]
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True,
                    help="root of a checkout of the reference repository (read-only)")
    a = ap.parse_args()
    np.savez_compressed(HERE / "dump_refs_subset.npz", **dump_refs_subset(a.reference))
    np.savez_compressed(HERE / "demix_identity.npz", **demix_identity(a.reference))
    print("wrote", HERE / "dump_refs_subset.npz", HERE / "demix_identity.npz")


if __name__ == "__main__":
    main()
