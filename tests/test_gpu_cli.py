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


def test_bench_json(setup, tmp_path):
    d, _, _ = setup
    out = tmp_path / "bench.json"
    r = run_cli("--bench", "--model-dir", d, "--warmup", "2", "--iters", "3", "--bench-json", out)
    assert r.returncode == 0, r.stdout + r.stderr
    line = json.loads(out.read_text())
    assert line["metric"] == "ms/588800-sample chunk" and line["iters"] == 3
    assert 1.0 < line["ms_median"] < 1000.0
