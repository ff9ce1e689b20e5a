"""The host CLI end to end on a B200: WAV in, a checkpoint from a model
directory, one float WAV per output target; the stems must be the ones the
library's own lbrr_separate_song produces for the same audio and weights, bit
for bit, and an instrumental mix their sum.  --bench prints its JSON line."""
import json

import numpy as np
import pytest

from cli_helpers import ensure_cli, model_yaml, read_wav_f32, run_cli, write_safetensors, write_wav

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup(tmp_path_factory):
    from lbrr import synthetic
    ensure_cli()
    d = tmp_path_factory.mktemp("cli")
    (d / "logic_bs_roformer.yaml").write_text(model_yaml())
    w = synthetic.checkpoint(seed=4)
    write_safetensors(d / "model.safetensors", {k: v.numpy() for k, v in w.items()})
    song = synthetic.audio(44100 * 16, seed=9)  # 16 s: two chunks, one overlap
    write_wav(d / "song.wav", np.ascontiguousarray(song.T).ravel(), 2)
    return d, w, song


def test_separate_matches_library(setup):
    import lbrr
    d, w, song = setup
    r = run_cli("--separate", "--model-dir", d, "--input", d / "song.wav", "--outdir", d / "out")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "6 tracks" in r.stdout
    eng = lbrr.Engine(0, 588800)
    try:
        eng.upload_weights(w)
        ref = lbrr.separate([eng], song)
    finally:
        eng.close()
    for i, name in enumerate(["bass", "drums", "other", "vocals", "guitar", "piano"]):
        rate, ch, x = read_wav_f32(d / "out" / f"{i}_{name}.wav")
        assert (rate, ch) == (44100, 2)
        got = x.reshape(-1, 2).T
        assert np.array_equal(got, ref[i]), name


def test_vocals_mode_mixes(setup):
    d, _, _ = setup
    r = run_cli("--model-dir", d, "--input", d / "song.wav", "--outdir", d / "voc", "--mode", "vocals")
    assert r.returncode == 0, r.stdout + r.stderr
    stems = [read_wav_f32(d / "out" / f"{i}_{n}.wav")[2]
             for i, n in enumerate(["bass", "drums", "other", "vocals", "guitar", "piano"])]
    assert np.array_equal(read_wav_f32(d / "voc" / "vocals.wav")[2], stems[3])
    inst = np.zeros_like(stems[0])
    for i in (0, 1, 2, 4, 5):  # summed in stem order, one fp32 rounding per addition
        inst = (inst + stems[i]).astype(np.float32)
    assert np.array_equal(read_wav_f32(d / "voc" / "instrumental.wav")[2], inst)


SCHEMA_V1 = {
    "schema_version", "identity", "shape", "pipeline", "backend", "precision", "timing_ms", "memory_bytes",
    "correctness", "ola_vs_host", "mfu"}
TIMING_KEYS = {
    "context_kernels", "weights_read", "weights_parse", "weights_pack_h2d", "weights_conversion",
    "weights_h2d_and_alloc", "fft_plan", "allocation_input_h2d", "prepare_algorithms", "warmup", "iterations",
    "host_total", "host_per_iteration", "cuda_event", "download_and_host_ola_check", "process_before_hashes", "rtf"}


def _write_npz_stored(path, **arrays):
    np.savez(path, **arrays)  # numpy.savez writes stored (uncompressed) zip entries


def test_bench_json(setup, tmp_path):
    """--bench writes the reference's schema-v1 report (src/main.rs:7336-7347)
    with per-stem correctness against a golden fixture: here the oracle's
    f16path forward of the short chunk, which the engine must match >= 60 dB."""
    import torch
    from oracle import bsroformer_ref as R
    d, w, _ = setup
    L = 132300
    audio = R.synth_audio(L, seed=12)
    ref = R.Oracle({k: torch.as_tensor(v) for k, v in w.items()}, "f16path").forward(torch.from_numpy(audio)).numpy()
    fixture = tmp_path / "golden" / "ref_output.npz"
    fixture.parent.mkdir()
    _write_npz_stored(fixture, inp=audio[None], out=ref[None])
    out = tmp_path / "bench.json"
    r = run_cli("--bench", "--model-dir", d, "--warmup", "2", "--iters", "3", "--bench-ref", fixture,
                "--bench-json", out)
    assert r.returncode == 0, r.stdout + r.stderr
    rep = json.loads(out.read_text())
    assert SCHEMA_V1 <= set(rep), SCHEMA_V1 - set(rep)
    assert rep["schema_version"] == 1
    assert set(rep["timing_ms"]) >= TIMING_KEYS
    assert len(rep["timing_ms"]["cuda_event"]) == 3 and rep["timing_ms"]["iterations"] == 3
    assert rep["shape"] == {"batch": 1, "channels": 2, "stems": 6, "samples": L, "T": 259, "bands": 62,
                            "sample_rate": 44100}
    assert rep["identity"]["model_sha256"] and len(rep["identity"]["source_sha256"]) == 64
    assert rep["identity"]["fixture_id"] == "golden"
    assert rep["ola_vs_host"]["finite"] and rep["ola_vs_host"]["max_abs_error"] <= 2e-6 * max(1.0, np.abs(ref).max())
    assert rep["mfu"]["matrix_flops"] == R.matrix_flops(259)  # the FLOP count follows the input length
    assert rep["memory_bytes"]["weights"] > 300e6
    c = rep["correctness"]
    assert c["finite"] and len(c["stems"]) == 6
    assert min(s["snr_db"] for s in c["stems"]) >= 60.0, c["stems"]
    assert "BENCH CUDA Event: median" in r.stdout


def test_kernel_regression_cli(tmp_path):
    """--kernel-regression: the reference's checkpoint-free checks restated for
    this build (STFT/OLA impulses, one-hot mask layout, QKV+RoPE boundaries,
    fused vs unfused feed-forward) all pass and the report is written."""
    ensure_cli()
    out = tmp_path / "kr.json"
    r = run_cli("--kernel-regression", "--bench-json", out, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "KERNEL_REGRESSION_OK" in r.stdout
    for line in ("STFT/OLA L=588800", "compact_mask T=1151", "QKV+RoPE T=1151", "FF M=71362 mode=ff_fused"):
        assert line in r.stdout, line
    rep = json.loads(out.read_text())
    assert rep["schema_version"] == 1 and len(rep["ff1"]) == 12
