"""The polynomial exp2 of the attention softmax (csrc/exp2_poly.cuh) against
its error bound: the device sequence (clamp, magic-number rounding, degree-4
polynomial in fp32 FMAs, exponent-field add) is replayed here in numpy fp32
and compared with the exact 2^x.  The coefficients in the header must be the
ones csrc/exp2_poly.py (Remez fit) produces."""
import importlib.util
import re
from pathlib import Path

import numpy as np

CSRC = Path(__file__).resolve().parents[1] / "logic-bs-roformer-rs_b200" / "csrc"


def _fit_module():
    spec = importlib.util.spec_from_file_location("exp2_poly", CSRC / "exp2_poly.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def header_coefficients():
    text = (CSRC / "exp2_poly.cuh").read_text()
    return [np.float32(float(v)) for v in re.findall(r"kC\d = ([0-9.e+-]+)f", text)]


def f32(v):
    return np.asarray(v, dtype=np.float32)


def fma32(a, b, c):
    # a*b is exact in float64 for fp32 inputs; one rounding of the sum to fp32
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly_replay(x):
    c = header_coefficients()
    x = np.maximum(f32(x), np.float32(-126.0))
    rnd = np.float32(12582912.0)
    t = (x + rnd).astype(np.float32)
    j = (t - rnd).astype(np.float32)
    f = fma32(j, f32(-1.0), x)
    p = fma32(f32(c[-1]), f, f32(c[-2]))
    for k in range(len(c) - 3, -1, -1):
        p = fma32(p, f, f32(c[k]))
    bits = p.view(np.int32).astype(np.int64) + ((t.view(np.int32).astype(np.int64) << 23) & 0xFFFFFFFF)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_header_matches_fit():
    m = _fit_module()
    got = header_coefficients()
    want = m.coefficients_f32()
    assert len(got) == 5
    assert np.array_equal(np.array(got, np.float32), want)
    assert m.max_rel_error(want) < 3e-6


def test_relative_error_bound():
    rs = np.random.RandomState(0)
    x = np.concatenate([np.linspace(-125.0, 8.0, 400001, dtype=np.float32),
                        rs.uniform(-30.0, 8.0, 200000).astype(np.float32),
                        np.arange(-125, 9, dtype=np.float32), np.arange(-125, 8, dtype=np.float32) + 0.5])
    got = exp2_poly_replay(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 3.2e-6, rel.max()


def test_clamp_and_fp16_rounding():
    x = f32([-np.inf, -1e30, -200.0, -126.0, 0.0, 8.0])
    y = exp2_poly_replay(x)
    assert np.all(np.isfinite(y))
    assert np.all(y[:4] <= np.float32(2.0 ** -125))
    assert np.all(y[:4].astype(np.float16) == 0)
    assert abs(float(y[4]) - 1.0) < 3e-6 and abs(float(y[5]) / 256.0 - 1.0) < 3e-6
