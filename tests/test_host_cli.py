"""The host CLI (host/*.cpp, the reference CLI's modes over the C ABI) on the
CPU: the training-YAML reader behind --print-config, --check-weights on a full
synthetic checkpoint and on broken ones, and --dry-run over WAV inputs in the
three formats the reference reads (src/audio.rs:12-80), with the output plans
of src/plan.rs.  Separation itself runs in tests/test_gpu_cli.py."""
import numpy as np
import pytest

from cli_helpers import ensure_cli, model_yaml, run_cli, write_safetensors, write_wav


@pytest.fixture(scope="module", autouse=True)
def cli():
    return ensure_cli()


def model_dir(tmp_path, **kw):
    d = tmp_path / "model"
    d.mkdir(exist_ok=True)
    (d / "logic_bs_roformer.yaml").write_text(model_yaml(**kw))
    return d


def test_print_config(tmp_path):
    r = run_cli("--print-config", "--model-dir", model_dir(tmp_path))
    assert r.returncode == 0, r.stderr
    assert "dim=256 depth=12 heads=8 dim_head=64 bands=62 stems=[bass drums other vocals guitar piano]" in r.stdout
    assert "n_fft=2048 hop=512 win=2048 sample_rate=44100 dim_freqs_in=1025" in r.stdout
    assert "shared_bias=true chunk_size=588800" in r.stdout
    assert "engine   : supported" in r.stdout


@pytest.mark.parametrize("kw,needle", [
    (dict(drop=("heads",)), "missing key heads"),
    (dict(dim_freqs_in=1024), "freqs_per_bands sum 1025 != dim_freqs_in 1024"),
    (dict(depth=6), "not supported"),
    (dict(freqs=[2] * 24 + [4] * 12 + [12] * 8 + [24] * 8 + [48] * 8 + [257], dim_freqs_in=1025), "not supported"),
])
def test_print_config_rejects(tmp_path, kw, needle):
    r = run_cli("--print-config", "--model-dir", model_dir(tmp_path, **kw))
    assert r.returncode == 1
    assert needle in r.stdout + r.stderr


def test_missing_config(tmp_path):
    r = run_cli("--print-config", "--model-dir", tmp_path)
    assert r.returncode == 1 and "no logic_bs_roformer.yaml or config.yaml" in r.stderr


@pytest.fixture(scope="module")
def checkpoint_dir(tmp_path_factory):
    from lbrr import synthetic
    d = tmp_path_factory.mktemp("ckpt")
    (d / "logic_bs_roformer.yaml").write_text(model_yaml())
    write_safetensors(d / "model.safetensors", {k: v.numpy() for k, v in synthetic.checkpoint(seed=0).items()})
    return d


def test_check_weights(checkpoint_dir):
    r = run_cli("--check-weights", "--model-dir", checkpoint_dir)
    assert r.returncode == 0, r.stderr
    assert "weights OK: 12 layers, 62 bands, 6 stems; shared qkv bias len 1536" in r.stdout
    assert "all checkpoint keys consumed exactly once" in r.stdout


def test_check_weights_broken(tmp_path):
    d = model_dir(tmp_path)
    write_safetensors(d / "model.safetensors", {"linear_62_bias_0": np.zeros(1536, np.float32)})
    r = run_cli("--check-weights", "--model-dir", d)
    assert r.returncode == 1 and "missing tensor linear_64_bias_0" in r.stderr
    (d / "model.safetensors").write_bytes(b"\x05\x00\x00\x00\x00\x00\x00\x00{}")
    r = run_cli("--check-weights", "--model-dir", d)
    assert r.returncode == 1 and "truncated safetensors header" in r.stderr


def audio(n, seed, channels=2):
    rs = np.random.RandomState(seed)
    return (rs.uniform(-0.5, 0.5, n * channels)).astype(np.float32)


@pytest.mark.parametrize("fmt,channels", [("f32", 2), ("s16", 2), ("s24", 1)])
def test_dry_run_formats(tmp_path, fmt, channels):
    n = 44100 * 14  # 14 s: two chunks of the reference plan
    p = tmp_path / f"in_{fmt}.wav"
    write_wav(p, audio(n, 1, channels), channels, fmt=fmt)
    r = run_cli("--dry-run", "--input", p, "--model-dir", model_dir(tmp_path))
    assert r.returncode == 0, r.stderr
    assert "[44.1kHz stereo, 14.0s]" in r.stdout
    assert "chunks   : 2 of 588800 samples" in r.stdout
    assert "detailed stems (0_bass.wav, 1_drums.wav, 2_other.wav, 3_vocals.wav, 4_guitar.wav, 5_piano.wav)" in r.stdout


@pytest.mark.parametrize("args,needle", [
    (["--mode", "vocals"], "vocals / instrumental (vocals.wav, instrumental.wav)"),
    (["--mode", "karaoke"], "vocals / instrumental (vocals.wav, instrumental.wav)"),
    (["--stems", "vocals,1"], "detailed stems (1_drums.wav, 3_vocals.wav)"),
    (["--stems", "Piano; 0"], "detailed stems (0_bass.wav, 5_piano.wav)"),
])
def test_dry_run_plans(tmp_path, args, needle):
    p = tmp_path / "in.wav"
    write_wav(p, audio(1000, 2), 2)
    r = run_cli("--dry-run", p, "--model-dir", model_dir(tmp_path), *args)
    assert r.returncode == 0, r.stderr
    assert "chunks   : 1 of 588800" in r.stdout
    assert needle in r.stdout


@pytest.mark.parametrize("prep,needle", [
    ("rate", "convert it to 44.1 kHz stereo first"),
    ("text", "not a RIFF/WAVE file"),
    ("missing", "cannot open"),
])
def test_dry_run_bad_inputs(tmp_path, prep, needle):
    p = tmp_path / "bad.wav"
    if prep == "rate":
        write_wav(p, audio(1000, 3), 2, rate=48000)
    elif prep == "text":
        p.write_text("not audio")
    r = run_cli("--dry-run", "--input", p, "--model-dir", model_dir(tmp_path))
    assert r.returncode == 2 and needle in r.stderr


@pytest.mark.parametrize("args,needle", [
    (["--stems", "cowbell"], 'unknown stem "cowbell"'),
    (["--stems", "9"], "stem index 9 out of range"),
    (["--mode", "quad"], "bad output mode"),
    (["--bogus"], "unknown argument --bogus"),
])
def test_argument_errors(tmp_path, args, needle):
    p = tmp_path / "in.wav"
    write_wav(p, audio(100, 4), 2)
    r = run_cli("--dry-run", "--input", p, "--model-dir", model_dir(tmp_path), *args)
    assert r.returncode == 2 and needle in r.stderr
