"""CPU-side checks of the C ABI library: it loads and exports every symbol
include/lbrr_gpu.h declares; argument validation runs before any device work."""
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def header_symbols():
    text = (REPO / "include" / "lbrr_gpu.h").read_text()
    return sorted(set(re.findall(r"\b(lbrr_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    import lbrr
    L = lbrr.lib()
    syms = header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), s
    assert sorted(lbrr.HEADER_SYMBOLS) == syms


def test_abi_version_and_default_model():
    import lbrr
    assert lbrr.lib().lbrr_abi_version() == 2
    d = lbrr.default_model()
    assert (d.dim, d.depth, d.heads, d.dim_head, d.num_stems, d.num_bands) == (256, 12, 8, 64, 6, 62)
    freqs = [d.freqs_per_band[i] for i in range(62)]
    from oracle import bsroformer_ref as R
    assert freqs == R.FREQS_PER_BANDS and sum(freqs) == 1025


def test_invalid_arguments_fail_before_device_work():
    import lbrr
    L = lbrr.lib()
    assert L.lbrr_engine_create(0, None, 1000, None) == lbrr.ERR_INVALID
    assert b"NULL" in L.lbrr_last_error() or b"out" in L.lbrr_last_error()
    assert L.lbrr_forward_chunk(None, None, 0, None, None) == lbrr.ERR_INVALID
    assert L.lbrr_op_ff1_gelu(None, None, None, None, 0, None) == lbrr.ERR_INVALID
    assert L.lbrr_separate_song(None, 0, None, 0, None, None) == lbrr.ERR_INVALID


def test_fp16_packing_contract():
    # src/fp16.rs:121-181 bit contract: RNE, +-0, inf, NaN -> sign|0x7c01, subnormals
    import struct
    import lbrr
    import numpy as np
    f = lbrr.f32_to_f16_bits
    assert f(1.0) == 0x3C00 and f(-0.0) == 0x8000 and f(float("inf")) == 0x7C00
    nan = struct.unpack("<f", struct.pack("<I", 0x7FC01234))[0]
    nneg = struct.unpack("<f", struct.pack("<I", 0xFFC01234))[0]
    assert f(nan) == 0x7C01 and f(nneg) == 0xFC01
    for h in range(0, 1024, 7):
        assert f(h * 2.0 ** -24) == h
    # every normal half and its fp32 tie neighbours agree with numpy's RNE
    rs = np.random.RandomState(0)
    bits = ((np.arange(1, 31)[:, None] + 112) << 23 | (rs.randint(0, 1024, (30, 16)) << 13)).ravel()
    vals = []
    for b in bits:
        for d in (0, 0xFFF, 0x1000, 0x1001, 0x1FFF):
            vals.append(np.uint32(b + d).view(np.float32))
    vals = np.array(vals, np.float32)
    got = np.array([f(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, vals.astype(np.float16).view(np.uint16))
