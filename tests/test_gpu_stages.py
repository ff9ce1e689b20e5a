"""Stage-level parity of the chunk forward's back end on the GPU, through the
engine's diagnostic taps (lbrr_engine_read_buffer), plus the checkpoint-free
regressions of the reference's --kernel-regression mode (src/main.rs:7909-8052)
restated for this build's fused kernels:

* the mask estimator's hidden layer (all 6 x 62 (stem, band) MLPs) against the
  oracle, from the engine's own band-major final-norm output;
* the fused second mask GEMM + GLU + complex mask application (the C2R input)
  against the oracle, band by band, from the engine's own hidden layer;
* mask_layout_regression (src/main.rs:7967-8015): one-hot weights make every
  pre-GLU column identifiable, so every (stem, band, frame, bin, channel) slot
  of the masked spectrum is checked against its own expected value, twice with
  different biases so a slot the kernel failed to write cannot pass;
* ola_regression (src/main.rs:7943-7965): with an identity mask the forward is
  STFT -> C2R -> overlap-add, which must return the input impulses (and exact
  silence) to 1e-6 at L in {1025, 18944, 132300, 588800};
* the DC/Nyquist option: the reference's mask_apply keeps the imaginary parts
  of those two bins; the measured difference to the default is recorded.
"""
import json
import os

import numpy as np
import pytest
import torch

from helpers import rel_err, snr_db
from oracle import bsroformer_ref as R

pytestmark = pytest.mark.gpu

SHORT = 132300   # T = 259
FULL = 588800    # T = 1151
LAYOUT = R.BandLayout()


@pytest.fixture(scope="module")
def engine():
    import lbrr
    e = lbrr.Engine(0, FULL)
    yield e
    e.close()


def _forward(engine, audio):
    x = torch.from_numpy(np.ascontiguousarray(audio.T)).cuda()
    out = torch.full((6, 2, audio.shape[1]), float("nan"), device="cuda")
    engine.bench_forward(x, out)
    engine.sync()
    return out.cpu().numpy()


def _taps(engine, T):
    spec = engine.read_buffer("spec", (2, T, 1025), np.complex64)
    c2r = engine.read_buffer("c2r", (12, T, 1025), np.complex64)
    return spec, c2r


def _mask_keys(s, b):
    p = f"mask_estimators.{s}.to_freqs.{b}.0"
    return f"{p}.0.weight", f"{p}.0.bias", f"{p}.2.weight", f"{p}.2.bias"


def _apply_masks(spec, m_all, T):
    """masked[s*2+ch][t][f] = spec[ch][t][f] * (m_re + i m_im) from GLU
    outputs m_all[s][T][4100] laid out as d = fi*4 + ch*2 + c (mask_apply,
    src/main.rs:1776-1817), DC/Nyquist imaginary parts dropped (the default)."""
    m = m_all.reshape(6, T, 1025, 2, 2)
    mc = (m[..., 0] + 1j * m[..., 1]).transpose(0, 3, 1, 2)  # [s][ch][T][f]
    out = (spec[None].astype(np.complex128) * mc).reshape(12, T, 1025)
    out[:, :, 0] = out[:, :, 0].real
    out[:, :, 1024] = out[:, :, 1024].real
    return out


# ---------------------------------------------------------------------------
# mask estimator stages against the oracle
# ---------------------------------------------------------------------------
def test_mask_estimator_stages_match_oracle(engine):
    w = R.make_weights(seed=3, gamma_noise=0.1)
    engine.upload_weights(w)
    audio = R.synth_audio(SHORT, seed=31)
    T = R.num_frames(SHORT)
    _forward(engine, audio)
    xb16 = torch.from_numpy(engine.read_buffer("xb16", (62, T, 256), np.float16).astype(np.float32))
    hidden = engine.read_buffer("hidden", (6 * 62, T, 1024), np.float16)
    spec, c2r = _taps(engine, T)
    # layer 1 + tanh, every (stem, band) group, from the engine's own xb16
    worst = 0.0
    for s in range(6):
        for b in range(62):
            k1, kb1, _, _ = _mask_keys(s, b)
            ref = R.f16(torch.tanh(xb16[b] @ R.f16(w[k1]).T + w[kb1]))
            got = torch.from_numpy(hidden[s * 62 + b].astype(np.float32))
            err = rel_err(got, ref)
            worst = max(worst, err)
            assert err < 2e-3, (s, b, err)
            assert float((got - ref).abs().max()) <= 1.5e-3, (s, b)
    # layer 2 + GLU + complex mask, from the engine's own hidden layer
    m_all = np.zeros((6, T, LAYOUT.total), np.float64)
    hid = torch.from_numpy(hidden.astype(np.float32))
    for s in range(6):
        for b in range(62):
            _, _, k2, kb2 = _mask_keys(s, b)
            pre2 = (hid[s * 62 + b].double() @ R.f16(w[k2]).double().T + w[kb2].double()).numpy()
            d = LAYOUT.dims[b]
            m_all[s, :, LAYOUT.offs[b]:LAYOUT.offs[b + 1]] = pre2[:, :d] / (1.0 + np.exp(-pre2[:, d:]))
    ref = _apply_masks(spec, m_all, T)
    assert rel_err(c2r.view(np.float32), ref.astype(np.complex64).view(np.float32)) < 1e-5
    for b in range(62):
        f0, f1 = LAYOUT.f0[b], LAYOUT.f0[b] + LAYOUT.freqs[b]
        e = rel_err(c2r[:, :, f0:f1].view(np.float32), ref[:, :, f0:f1].astype(np.complex64).view(np.float32))
        assert e < 1e-4, (b, e)


@pytest.mark.parametrize("length", [SHORT, FULL])
def test_mask_layout_one_hot(engine, length):
    """mask_layout_regression (src/main.rs:7967-8015) through the fused mask
    kernels: W1 passes one input feature to hidden unit 0 (plus a per-stem
    bias), W2 copies hidden unit 0 into every pre-GLU column, and the pre-GLU
    biases differ per column, so each masked-spectrum slot has its own value."""
    T = R.num_frames(length)
    audio = R.synth_audio(length, seed=41)
    base = R.make_weights(seed=4)
    for offset in (0.0, 0.5):  # the second pass catches slots left from the first
        w = dict(base)
        for s in range(6):
            for b in range(62):
                k1, kb1, k2, kb2 = _mask_keys(s, b)
                d = LAYOUT.dims[b]
                w1 = torch.zeros(1024, 256)
                w1[0, 0] = 1.0
                b1 = torch.zeros(1024)
                b1[0] = s / 32.0
                w2 = torch.zeros(2 * d, 1024)
                w2[:, 0] = 1.0
                cols = torch.arange(2 * d, dtype=torch.float64) + 2 * LAYOUT.offs[b]
                w[k1], w[kb1], w[k2] = w1, b1, w2
                w[kb2] = (cols * 0.00003 + s / 16.0 + offset).float()
        engine.upload_weights(w)
        _forward(engine, audio)
        hidden = engine.read_buffer("hidden", (6 * 62, T, 1024), np.float16)
        assert not hidden.view(np.uint16)[:, :, 1:].any()  # units 1.. are tanh(0) = +0
        h0 = hidden[:, :, 0].astype(np.float32)
        del hidden
        spec, c2r = _taps(engine, T)
        m_all = np.zeros((6, T, LAYOUT.total), np.float64)
        for s in range(6):
            for b in range(62):
                d = LAYOUT.dims[b]
                b2 = w[_mask_keys(s, b)[3]].numpy().astype(np.float32)
                pre2 = (h0[s * 62 + b, :, None] + b2[None, :]).astype(np.float64)  # fp32 sum, as the epilogue
                m_all[s, :, LAYOUT.offs[b]:LAYOUT.offs[b + 1]] = pre2[:, :d] / (1.0 + np.exp(-pre2[:, d:]))
        ref = _apply_masks(spec, m_all, T)
        scale = np.abs(spec).astype(np.float64)[None].repeat(6, 0).reshape(12, T, 1025)
        bound = 2e-6 * scale * (np.abs(m_all.reshape(6, T, 1025, 2, 2)).sum(-1).transpose(0, 3, 1, 2)
                                .reshape(12, T, 1025)) + 1e-30
        assert np.isfinite(c2r.view(np.float32)).all()
        bad = np.abs(c2r.astype(np.complex128) - ref) > bound
        assert not bad.any(), np.argwhere(bad)[:5]


# ---------------------------------------------------------------------------
# STFT -> C2R -> OLA with an identity mask
# ---------------------------------------------------------------------------
def identity_mask_weights(seed=5):
    """Mask estimator weights whose masks are exactly 1 + 0i: W2 = 0, pre-GLU
    biases 1 (real) / 0 (imaginary) with gate biases 100 (sigmoid = 1 in fp32)."""
    w = R.make_weights(seed=seed)
    for s in range(6):
        for b in range(62):
            _, _, k2, kb2 = _mask_keys(s, b)
            d = LAYOUT.dims[b]
            w[k2] = torch.zeros(2 * d, 1024)
            a = torch.zeros(d)
            a[0::2] = 1.0  # d = fi*4 + ch*2 + c: c = 0 is the real part
            w[kb2] = torch.cat([a, torch.full((d,), 100.0)])
    return w


@pytest.mark.parametrize("backend", [0, 1], ids=["inhouse_fft", "cufft"])
@pytest.mark.parametrize("length", [1025, 18944, 132300, 588800])
def test_ola_impulses_identity_mask(engine, length, backend):
    """ola_regression (src/main.rs:7943-7965): impulses at both ends of both
    channels come back on every stem to 1e-6; silence stays silent; every
    output slot is written (the output starts as NaN) -- through the in-house
    fused FFT kernels and through the cuFFT back end."""
    import lbrr
    engine.upload_weights(identity_mask_weights())
    engine.set_option(lbrr.OPT_FFT_BACKEND, backend)
    try:
        for silent in (False, True):
            x = np.zeros((2, length), np.float32)
            if not silent:
                x[0, 0], x[0, length - 1], x[1, 31], x[1, length - 1] = 0.5, 1.0, -0.25, 0.125
            got = _forward(engine, x)
            assert np.isfinite(got).all()
            err = np.abs(got - x[None]).max()
            assert err <= 1e-6, (length, silent, err)
    finally:
        engine.set_option(lbrr.OPT_FFT_BACKEND, 0)


def test_inhouse_fft_matches_cufft_and_oracle(engine):
    """The fused in-house front end gives the oracle's spectrum (torch.fft in
    double) to fp32 accuracy, as cuFFT does; the whole forward through either
    FFT back end meets the 60 dB bar against the oracle, and the two agree."""
    import lbrr
    w = R.make_weights(seed=2, gamma_noise=0.1)
    engine.upload_weights(w)
    audio = R.synth_audio(SHORT, seed=13)
    T = R.num_frames(SHORT)
    ref_spec = R.stft(torch.from_numpy(audio)).numpy()
    outs, specs = {}, {}
    for backend in (0, 1):
        engine.set_option(lbrr.OPT_FFT_BACKEND, backend)
        outs[backend] = _forward(engine, audio)
        specs[backend] = engine.read_buffer("spec", (2, T, 1025), np.complex64)
    engine.set_option(lbrr.OPT_FFT_BACKEND, 0)
    for backend in (0, 1):
        e = rel_err(specs[backend].view(np.float32), ref_spec.view(np.float32))
        assert e < 2e-6, (backend, e)
    ref = R.Oracle(w, "f16path").forward(torch.from_numpy(audio)).numpy()
    for backend in (0, 1):
        worst = min(snr_db(outs[backend][s], ref[s]) for s in range(6))
        assert worst >= 60.0, (backend, worst)
    assert min(snr_db(outs[0][s], outs[1][s]) for s in range(6)) >= 60.0


# ---------------------------------------------------------------------------
# DC / Nyquist imaginary parts: the reference's choice, measured
# ---------------------------------------------------------------------------
def test_dc_nyquist_reference_semantics_recorded(engine):
    import lbrr
    w = R.make_weights(seed=0, gamma_noise=0.1)
    engine.upload_weights(w)
    audio = R.synth_audio(SHORT, seed=3)
    default = _forward(engine, audio)
    engine.set_option(lbrr.OPT_DC_NYQUIST_IMAG, 1)
    try:
        assert engine.get_option(lbrr.OPT_DC_NYQUIST_IMAG) == 1
        keep = _forward(engine, audio)
        T = R.num_frames(SHORT)
        c2r = engine.read_buffer("c2r", (12, T, 1025), np.complex64)
        assert np.abs(c2r[:, :, 0].imag).max() > 0.0  # the option reaches the kernel
    finally:
        engine.set_option(lbrr.OPT_DC_NYQUIST_IMAG, 0)
    again = _forward(engine, audio)
    assert np.array_equal(again, default)  # the option is undone exactly
    ref = R.Oracle(w, "f16path").forward(torch.from_numpy(audio)).numpy()
    rec = {
        "default_vs_oracle_db": min(snr_db(default[s], ref[s]) for s in range(6)),
        "reference_dc_nyquist_vs_oracle_db": min(snr_db(keep[s], ref[s]) for s in range(6)),
        "reference_dc_nyquist_vs_default_db": min(snr_db(keep[s], default[s]) for s in range(6)),
        "max_abs_reference_dc_nyquist_vs_default": float(np.abs(keep - default).max()),
    }
    print("DC_NYQUIST", json.dumps(rec))
    out = os.environ.get("LBRR_RECORD_DIR")
    if out:
        with open(os.path.join(out, "dc_nyquist.json"), "w") as f:
            json.dump(rec, f, indent=1)
    assert rec["default_vs_oracle_db"] >= 60.0
    assert np.isfinite(keep).all()
    assert rec["reference_dc_nyquist_vs_default_db"] > 20.0


# ---------------------------------------------------------------------------
# bounded device waits and the song's abort path (no device fault involved)
# ---------------------------------------------------------------------------
def test_bounded_wait_reports_and_engine_recovers(engine):
    import time
    import lbrr
    engine.upload_weights(R.make_weights(seed=0))
    audio = R.synth_audio(SHORT, seed=9)
    before = _forward(engine, audio)
    t0 = time.perf_counter()
    engine.wait_probe(50_000_000)  # 50 ms bound on a wait nothing ends
    with pytest.raises(lbrr.LbrrError) as ei:
        engine.sync()
    assert ei.value.code == lbrr.ERR_DEVICE
    assert "timed out" in str(ei.value)
    assert time.perf_counter() - t0 < 5.0
    engine.sync()  # the status was cleared
    assert np.array_equal(_forward(engine, audio), before)


def test_song_worker_failure_aborts_fast():
    import time
    import lbrr
    w = R.make_weights(seed=1)
    e0, e1 = lbrr.Engine(0, R.CHUNK), lbrr.Engine(0, R.CHUNK)
    try:
        e0.upload_weights(w)
        e1.upload_weights(w)
        audio = R.synth_audio(3 * R.STEP + 5000, seed=21)  # 4 chunks: engine 1 takes chunks 1 and 3
        ref = lbrr.separate([e0], audio)
        e1.set_option(lbrr.OPT_SONG_FAIL_CHUNK, 1)
        t0 = time.perf_counter()
        with pytest.raises(lbrr.LbrrError) as ei:
            lbrr.separate([e0, e1], audio)
        assert ei.value.code == lbrr.ERR_STATE
        assert "injected" in str(ei.value)
        assert time.perf_counter() - t0 < 20.0  # engine 0 stops waiting for the strip at once
        e1.set_option(lbrr.OPT_SONG_FAIL_CHUNK, -1)
        assert np.array_equal(lbrr.separate([e0, e1], audio), ref)  # both engines usable afterwards
    finally:
        e1.close()
        e0.close()
