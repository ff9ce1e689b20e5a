"""Checkpoint validation on the host (no GPU): lbrr_check_weights and
lbrr_check_safetensors run the same checks lbrr_engine_load_weights /
lbrr_engine_load_safetensors run before any upload — the reference's
`--check-weights` mode (src/main.rs:332-365) over ModelWeights::load
(src/weights.rs:307-432) and SafeTensors::open (src/weights.rs:25-120).

Each failure case plants one defect in an otherwise valid checkpoint and
checks the call fails with LBRR_ERR_WEIGHTS and a message naming it.
"""
import json
import struct

import numpy as np
import pytest

import lbrr
from oracle import bsroformer_ref as R


@pytest.fixture(scope="module")
def weights():
    return {k: np.asarray(v, dtype=np.float32) for k, v in R.make_weights(seed=3).items()}


def _fails_with(fn, arg, needle):
    with pytest.raises(lbrr.LbrrError) as ei:
        fn(arg)
    assert ei.value.code == lbrr.ERR_WEIGHTS, ei.value
    assert needle in str(ei.value), str(ei.value)


def test_valid_checkpoint_passes(weights):
    assert len(weights) == 1989
    lbrr.check_weights(weights)


def test_missing_key(weights):
    w = dict(weights)
    del w["layers.7.1.layers.0.1.net.4.bias"]
    _fails_with(lbrr.check_weights, w, "missing tensor layers.7.1.layers.0.1.net.4.bias")


def test_wrong_numel(weights):
    w = dict(weights)
    w["band_split.to_features.5.1.weight"] = w["band_split.to_features.5.1.weight"][:-1]
    _fails_with(lbrr.check_weights, w, "band_split.to_features.5.1.weight: len")


def test_extra_key_is_unconsumed(weights):
    w = dict(weights)
    w["layers.0.0.layers.0.0.extra"] = np.zeros(4, np.float32)
    _fails_with(lbrr.check_weights, w, "unconsumed key layers.0.0.layers.0.0.extra")


def test_shared_qkv_bias_mismatch(weights):
    w = dict(weights)
    b = w["layers.3.0.layers.0.0.to_qkv.bias"].copy()
    b[100] = np.nextafter(b[100], np.float32(1))  # one ulp is enough: the check is bitwise
    w["layers.3.0.layers.0.0.to_qkv.bias"] = b
    _fails_with(lbrr.check_weights, w, "layers.3.0.layers.0.0.to_qkv.bias != linear_62_bias_0")


def test_shared_out_bias_mismatch(weights):
    w = dict(weights)
    b = w["layers.11.1.layers.0.0.to_out.0.bias"].copy()
    b[0] += 1.0
    w["layers.11.1.layers.0.0.to_out.0.bias"] = b
    _fails_with(lbrr.check_weights, w, "to_out.0.bias != linear_64_bias_0")


def test_rotary_freqs_not_analytic(weights):
    w = dict(weights)
    f = w["layers.2.1.layers.0.0.rotary_embed.freqs"].copy()
    f[31] *= 1.01
    w["layers.2.1.layers.0.0.rotary_embed.freqs"] = f
    _fails_with(lbrr.check_weights, w, "rotary freqs[31] != analytic in layers.2.1.layers.0.0")


def test_empty_checkpoint():
    _fails_with(lbrr.check_weights, {}, "missing tensor linear_62_bias_0")


# -- .safetensors parsing -----------------------------------------------------

def _write_safetensors(path, tensors, dtype="F32", header_extra=None, corrupt_len=0, raw_header=None):
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        b = np.ascontiguousarray(a, dtype=np.float32).tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(b) + corrupt_len]}
        blobs.append(b)
        off += len(b)
    if header_extra:
        header.update(header_extra)
    h = raw_header if raw_header is not None else json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def test_safetensors_parses_then_checks_keys(tmp_path, weights):
    # a well-formed file holding only the two shared biases parses, then fails
    # on the first layer key, which proves the header and data were read
    p = tmp_path / "partial.safetensors"
    _write_safetensors(p, {k: weights[k] for k in ("linear_62_bias_0", "linear_64_bias_0")},
                       header_extra={"__metadata__": {"format": "pt"}})
    _fails_with(lbrr.check_safetensors, p, "missing tensor layers.0.0.layers.0.0.norm.gamma")


def test_safetensors_wrong_dtype(tmp_path, weights):
    p = tmp_path / "f16.safetensors"
    _write_safetensors(p, {"linear_62_bias_0": weights["linear_62_bias_0"]}, dtype="F16")
    _fails_with(lbrr.check_safetensors, p, "linear_62_bias_0: expected F32, got F16")


def test_safetensors_byte_length_mismatch(tmp_path, weights):
    p = tmp_path / "len.safetensors"
    _write_safetensors(p, {"linear_64_bias_0": weights["linear_64_bias_0"]}, corrupt_len=4)
    _fails_with(lbrr.check_safetensors, p, "linear_64_bias_0: byte length mismatch")


def test_safetensors_header_too_large(tmp_path):
    p = tmp_path / "big.safetensors"
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", (64 << 20) + 1))
        f.write(b"{}")
    _fails_with(lbrr.check_safetensors, p, "safetensors header too large")


def test_safetensors_truncated_header(tmp_path):
    p = tmp_path / "trunc.safetensors"
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", 1000))
        f.write(b'{"a": ')
    _fails_with(lbrr.check_safetensors, p, "truncated safetensors header")


def test_safetensors_malformed_json(tmp_path):
    p = tmp_path / "bad.safetensors"
    _write_safetensors(p, {}, raw_header=b'{"x": {"dtype": "F32", "shape": [1], "data_offsets": [0]}}')
    _fails_with(lbrr.check_safetensors, p, "offsets len != 2")


def test_safetensors_missing_file(tmp_path):
    _fails_with(lbrr.check_safetensors, tmp_path / "nope.safetensors", "open ")
