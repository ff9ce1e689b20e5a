"""Pin the CPU oracle against the reference's own golden vectors.

Goldens come from the reference's ``tools/dump_refs.py`` (seeded per-op torch
generators) and ``tools/bench_ref.py`` (song demix with an identity model); see
``tests/golden/make_golden.py``.  Thresholds are the reference's per-op parity
gates (src/main.rs:5198, :5242, :5310, :5474, :5525, :5726, :5806-5854).
"""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import bsroformer_ref as R


def _maxerr(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


def test_stft_matches_reference_generator(golden):
    x = gi.stft_input()
    assert np.array_equal(x[:, :8], golden["stft_x_head"])
    # torch.hann_window evaluates cos in f32; src/stft.rs:25-29 rounds the f64 value once
    assert _maxerr(R.hann_window().numpy(), golden["stft_window"]) < 1e-6
    spec = R.stft(torch.from_numpy(x))  # [2][T][1025]
    got = torch.view_as_real(spec).permute(0, 2, 1, 3).numpy()[:, :, golden["stft_frames"], :]
    ref = golden["stft_spec"]
    # src/main.rs:5198: max err < 1e-5 * max|ref| + 1e-6
    assert _maxerr(got, ref) < 1e-5 * np.abs(ref).max() + 1e-6


def test_rmsnorm_matches_reference_generator(golden):
    x, gamma = gi.rmsnorm_input()
    assert np.array_equal(gamma, golden["rmsnorm_gamma"])
    for assoc in ("left", "right"):
        got = R.rmsnorm(torch.from_numpy(x[:64]), torch.from_numpy(gamma), assoc).numpy()
        ref = golden["rmsnorm_out"]
        assert _maxerr(got, ref) < 1e-5 * np.abs(ref).max()  # src/main.rs:5242


def test_bandsplit_matches_reference_generator(golden):
    x, gammas, ws, bs = gi.bandsplit_input()
    assert np.array_equal(np.concatenate(bs), golden["bandsplit_b"])
    w = {}
    for b in range(62):
        w[f"band_split.to_features.{b}.0.gamma"] = torch.from_numpy(gammas[b])
        w[f"band_split.to_features.{b}.1.weight"] = torch.from_numpy(ws[b])
        w[f"band_split.to_features.{b}.1.bias"] = torch.from_numpy(bs[b])
    o = R.Oracle(w, "fp32")
    got = o.band_split(torch.from_numpy(x[:4])).reshape(4, 62, 256).numpy()
    assert _maxerr(got, golden["bandsplit_out"]) < 1e-4  # src/main.rs:5310


@pytest.mark.parametrize("gi_idx", [0, 1, 2, 3])
def test_gemm_shapes_match_reference_generator(golden, gi_idx):
    x, w, b = gi.gemm_inputs()[gi_idx]
    assert np.array_equal(b, golden[f"gemm_b{gi_idx}"])
    o = R.Oracle({}, "fp32")
    got = (o._mm(torch.from_numpy(x[:32]), torch.from_numpy(w)) + torch.from_numpy(b)).numpy()
    assert _maxerr(got, golden[f"gemm_y{gi_idx}"]) < 1e-4


def test_qkv_rope_matches_reference_generator(golden):
    x, gamma, w, bias = gi.qkvrope_input()
    cos, sin = R.rope_tables(64)
    # the generator's tables are torch f32 math; ours round the f64 angle once
    assert _maxerr(cos.numpy().ravel(), golden["qkvrope_cos"]) < 1e-5
    assert _maxerr(sin.numpy().ravel(), golden["qkvrope_sin"]) < 1e-5
    h = R.rmsnorm(torch.from_numpy(x), torch.from_numpy(gamma), "left")
    qkv = h @ torch.from_numpy(w).T + torch.from_numpy(bias)
    q, k, v = qkv.view(2, 64, 3, 8, 64).unbind(2)          # (b, seq, heads, dh)
    qr = R.rope(q.permute(0, 2, 1, 3), cos, sin).permute(0, 2, 1, 3) * 0.125
    kr = R.rope(k.permute(0, 2, 1, 3), cos, sin).permute(0, 2, 1, 3)
    for got, key in ((qr, "q"), (kr, "k"), (v, "v")):
        assert _maxerr(got[:1, :16].numpy(), golden[f"qkvrope_{key}"]) < 1e-4  # src/main.rs:5474


@pytest.mark.parametrize("long", [False, True])
def test_attention_matches_reference_generator(golden, long):
    q, k, v = gi.attn_input(long)
    o = R.Oracle({}, "fp32")
    got = o.attention(*(torch.from_numpy(a)[None] for a in (q, k, v)))[0].numpy()
    if long:
        assert _maxerr(got[:1], golden["attn_long_out"]) < 1e-3   # src/main.rs:5726
    else:
        assert _maxerr(got[:4], golden["attn_short_out"]) < 1e-4  # src/main.rs:5525


def test_gate_outproj_ff_match_reference_generator(golden):
    d = {k: torch.from_numpy(v) for k, v in gi.gateff_input().items()}
    o = R.Oracle({}, "fp32")
    gates = d["h"] @ d["wg"].T + d["bg"]
    attn_out = o.gate_outproj(d["attn_raw"], gates, d["wo"], d["bo"], d["x_res"])
    assert _maxerr(attn_out[:32].numpy(), golden["gateff_attn_out"]) < 1e-4  # src/main.rs:5806
    ff1 = torch.nn.functional.gelu(attn_out @ d["w1"].T + d["b1"])
    assert _maxerr(ff1[:32].numpy(), golden["gateff_ff1"]) < 5e-4           # src/main.rs:5830
    ff_out = o.feed_forward(attn_out, d["w1"], d["b1"], d["w2"], d["b2"], attn_out)
    assert _maxerr(ff_out[:32].numpy(), golden["gateff_ff_out"]) < 1e-4     # src/main.rs:5854


def test_gelu_as_tracks_exact_erf():
    v = torch.linspace(-8, 8, 100001)
    # A&S 7.1.26 has |erf error| <= 1.5e-7, so |gelu error| <= 0.5*|v|*1.5e-7
    assert (R.gelu_as(v) - torch.nn.functional.gelu(v)).abs().max() < 0.5 * 8 * 1.6e-7 + 1e-6


def test_chunk_plan_and_reflect_pad_match_bench_ref(demix_golden):
    for length in demix_golden["lengths"]:
        assert R.chunk_starts(int(length)) == list(demix_golden[f"starts_{length}"])
    x = np.array([[1, 2, 3], [10, 20, 30]], dtype=np.float32)
    assert np.array_equal(R.reflect_pad(x, 17, 29), demix_golden["reflect_17_29"])
    assert np.array_equal(R.reflect_pad(x, 17, 29), np.pad(x, ((0, 0), (17, 29)), mode="reflect"))
    with pytest.raises(ValueError):
        R.chunk_starts(0)


@pytest.mark.parametrize("length", [37, R.CHUNK + 1000, R.STEP * 3 + 91])
def test_identity_demix_matches_bench_ref(demix_golden, length):
    rs = np.random.RandomState(length % 1000)
    sig = rs.randn(1, 2, length).astype(np.float32)[0]
    y = R.demix(lambda c: np.broadcast_to(c[None], (6,) + c.shape), sig)
    idx = demix_golden[f"demix_idx_{length}"]
    np.testing.assert_allclose(y[:, :, idx], demix_golden[f"demix_y_{length}"], rtol=0, atol=2e-6)


def test_flop_constants():
    # src/benchmark.rs:261-264
    assert R.matrix_flops(1151) == 6_069_010_774_016
    assert R.matrix_flops(259) == 1_013_639_108_608


def test_weight_keys_cover_checkpoint():
    keys = R.weight_keys()
    assert len(keys) == 1989 and len({k for k, _ in keys}) == 1989
    n = sum(int(np.prod(s)) for k, s in keys
            if not (k.endswith("to_qkv.bias") or k.endswith("to_out.0.bias") or k.endswith("rotary_embed.freqs")))
    assert n == 174_658_292


def test_metric_silence_and_nonfinite():
    # src/benchmark.rs:266-271
    m = R.metric(np.zeros(4, np.float32), np.zeros(4, np.float32))
    assert m["finite"] and m["bit_equal"] and m["snr_db"] is None
    assert not R.metric(np.array([np.nan], np.float32), np.zeros(1, np.float32))["finite"]
