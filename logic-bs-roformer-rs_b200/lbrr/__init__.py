"""Python binding of the B200 BS-RoFormer engine (ctypes over include/lbrr_gpu.h).

The names follow the reference's GPU pipeline in ``src/main.rs``:
``upload_weights`` (:6045-6077), ``bench_forward`` (:7014-7162, plus the
istft_ola of :7303-7306), ``separate`` (:7598-7819) and the per-op pieces of
``transformer_step`` (:6131-6268).  Device buffers are passed as torch CUDA
tensors (PyTorch is only the allocator and stream provider here); every
computation runs in ``liblbrr_b200.so``.  There is no fallback: if the library
is missing or a call fails, a ``LbrrError`` is raised.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "liblbrr_b200.so"

OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_WEIGHTS = -3
ERR_DEVICE = -4
ERR_STATE = -5
ERR_PEER = -6

CHUNK, STEP, BORDER = 588800, 559360, 29440
STEMS = 6
INSTRUMENTS = ["bass", "drums", "other", "vocals", "guitar", "piano"]


class LbrrError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"lbrr error {code}: {msg}")
        self.code = code


class ModelDesc(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("dim", "depth", "heads", "dim_head", "num_stems", "mlp_expansion",
                                         "n_fft", "hop", "sample_rate", "num_bands")] + \
               [("freqs_per_band", C.POINTER(C.c_int32))]


class WeightView(C.Structure):
    _fields_ = [("name", C.c_char_p), ("data", C.POINTER(C.c_float)), ("numel", C.c_int64)]


FADE_LINEAR, FADE_HANN = 0, 1
# BASELINE config 4's plan: 50 % overlap, Hann-weighted (28 chunks for 180.48 s)
HANN50 = dict(chunk=588800, step=294400, border=294400, fade="hann")


class ChunkPlan(C.Structure):
    _fields_ = [("chunk", C.c_int64), ("step", C.c_int64), ("border", C.c_int64), ("fade", C.c_int64)]


_lib = None


def lib() -> C.CDLL:
    """Load liblbrr_b200.so (built by logic-bs-roformer-rs_b200/build.py)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise LbrrError(ERR_STATE, f"{LIB_PATH} is missing: run logic-bs-roformer-rs_b200/build.py")
    L = C.CDLL(str(LIB_PATH))
    vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int32
    sig = {
        "lbrr_last_error": ([], C.c_char_p),
        "lbrr_abi_version": ([], C.c_int),
        "lbrr_host_alloc": ([C.c_size_t, C.POINTER(vp)], C.c_int),
        "lbrr_host_free": ([vp], C.c_int),
        "lbrr_default_model": ([C.POINTER(ModelDesc), C.POINTER(C.c_int32), i32], C.c_int),
        "lbrr_engine_create": ([C.c_int, C.POINTER(ModelDesc), i64, C.POINTER(vp)], C.c_int),
        "lbrr_engine_load_weights": ([vp, C.POINTER(WeightView), C.c_size_t], C.c_int),
        "lbrr_engine_load_safetensors": ([vp, C.c_char_p], C.c_int),
        "lbrr_check_weights": ([C.POINTER(WeightView), C.c_size_t], C.c_int),
        "lbrr_check_safetensors": ([C.c_char_p], C.c_int),
        "lbrr_forward_chunk": ([vp, vp, i64, vp, vp], C.c_int),
        "lbrr_forward_chunks": ([vp, vp, i64, i32, vp, vp], C.c_int),
        "lbrr_forward_chunk_host": ([vp, vp, i64, vp], C.c_int),
        "lbrr_forward_trunk": ([vp, vp, i64, C.c_int, vp, vp], C.c_int),
        "lbrr_forward_back": ([vp, i64, vp, vp], C.c_int),
        "lbrr_engine_sync": ([vp], C.c_int),
        "lbrr_engine_set_option": ([vp, C.c_int, i64], C.c_int),
        "lbrr_engine_get_option": ([vp, C.c_int, C.POINTER(i64)], C.c_int),
        "lbrr_engine_wait_probe": ([vp, i64], C.c_int),
        "lbrr_engine_read_buffer": ([vp, C.c_char_p, vp, i64], C.c_int),
        "lbrr_engine_memory": ([vp, C.POINTER(i64), C.POINTER(i64)], C.c_int),
        "lbrr_engine_destroy": ([vp], None),
        "lbrr_separate_song": ([C.POINTER(vp), C.c_int, vp, i64, C.POINTER(ChunkPlan), vp], C.c_int),
        "lbrr_op_norm_gates": ([vp, vp, vp, vp, vp, vp, i64, vp], C.c_int),
        "lbrr_op_qkv_rope": ([vp, vp, vp, vp, vp, vp, i64, i32, i32, vp], C.c_int),
        "lbrr_op_attention": ([vp, vp, vp, i64, i32, i32, vp], C.c_int),
        "lbrr_op_outproj_norm": ([vp, vp, vp, vp, vp, vp, vp, i64, vp], C.c_int),
        "lbrr_op_ff1_gelu": ([vp, vp, vp, vp, i64, vp], C.c_int),
        "lbrr_op_ff2_resid": ([vp, vp, vp, vp, vp, i64, vp], C.c_int),
        "lbrr_op_feed_forward": ([vp, vp, vp, vp, vp, vp, vp, i64, vp], C.c_int),
        "lbrr_op_sync": ([vp], C.c_int),
        "lbrr_op_feed_forward_noalloc": ([vp, vp, vp, vp, vp, vp, vp, i64, vp], C.c_int),
        "lbrr_f32_to_f16_bits": ([C.c_float], C.c_uint16),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


# Every symbol include/lbrr_gpu.h declares (checked by the CPU test suite).
HEADER_SYMBOLS = [
    "lbrr_last_error", "lbrr_abi_version", "lbrr_host_alloc", "lbrr_host_free", "lbrr_default_model", "lbrr_engine_create", "lbrr_engine_load_weights",
    "lbrr_engine_load_safetensors", "lbrr_check_weights", "lbrr_check_safetensors", "lbrr_forward_chunk", "lbrr_forward_chunks", "lbrr_forward_chunk_host", "lbrr_forward_trunk",
    "lbrr_forward_back",
    "lbrr_engine_sync", "lbrr_engine_set_option", "lbrr_engine_get_option", "lbrr_engine_wait_probe",
    "lbrr_engine_read_buffer", "lbrr_engine_memory", "lbrr_engine_destroy", "lbrr_separate_song", "lbrr_op_norm_gates",
    "lbrr_op_qkv_rope", "lbrr_op_attention", "lbrr_op_outproj_norm", "lbrr_op_ff1_gelu", "lbrr_op_ff2_resid",
    "lbrr_op_feed_forward", "lbrr_op_sync", "lbrr_op_feed_forward_noalloc",
]


def check(rc: int):
    if rc != OK:
        raise LbrrError(rc, lib().lbrr_last_error().decode(errors="replace"))


def _ptr(t):
    """Device (or host) address of a torch tensor / numpy array; None -> NULL."""
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


# engine options (include/lbrr_gpu.h)
OPT_DC_NYQUIST_IMAG = 1
OPT_SONG_FAIL_CHUNK = 2
OPT_FFT_BACKEND = 3
INFO_KERNELS_PER_FORWARD = 100

CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy: the legacy default stream named explicitly


def _stream(stream):
    """None -> NULL (the engine's own stream for engine calls).  A torch stream
    whose handle is 0 is the legacy default stream: it is passed as
    cudaStreamLegacy, because a NULL handle would put engine work on the
    engine's stream, unordered with the caller's default-stream work."""
    if stream is None:
        return None
    h = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    return h if h else CUDA_STREAM_LEGACY


def default_model():
    d = ModelDesc()
    freqs = (C.c_int32 * 62)()
    check(lib().lbrr_default_model(C.byref(d), freqs, 62))
    d._keep = freqs
    return d


def _weight_views(weights: dict):
    """fp32 copies of {name: array} and the lbrr_weight_view array pointing at them."""
    keep, views = [], (WeightView * len(weights))()
    for i, (name, t) in enumerate(weights.items()):
        a = np.ascontiguousarray(np.asarray(t.detach().cpu() if hasattr(t, "detach") else t, dtype=np.float32))
        keep.append(a)
        views[i].name = name.encode()
        views[i].data = a.ctypes.data_as(C.POINTER(C.c_float))
        views[i].numel = a.size
    return keep, views


def check_weights(weights: dict):
    """Validate a checkpoint on the host only (no GPU needed): the reference's
    `--check-weights` mode (src/main.rs:332-365, ModelWeights::load in
    src/weights.rs:307-447).  Raises LbrrError(ERR_WEIGHTS) naming the first
    bad tensor."""
    keep, views = _weight_views(weights)
    check(lib().lbrr_check_weights(views, len(weights)))
    del keep


def check_safetensors(path):
    """Parse and validate a .safetensors checkpoint on the host only."""
    check(lib().lbrr_check_safetensors(str(path).encode()))


class Engine:
    """One GPU's engine: weights, scratch, cuFFT plans and a stream."""

    def __init__(self, device: int = 0, max_chunk_samples: int = CHUNK):
        self.device = device
        self.max_chunk_samples = max_chunk_samples
        h = C.c_void_p()
        desc = default_model()
        check(lib().lbrr_engine_create(device, C.byref(desc), max_chunk_samples, C.byref(h)))
        self.handle = h

    # -- weights -------------------------------------------------------------
    def upload_weights(self, weights: dict):
        """Validate and upload a checkpoint given as {name: fp32 array/tensor}
        (ModelWeights::load + upload_weights, src/weights.rs:307-447, src/main.rs:6045-6077)."""
        keep, views = _weight_views(weights)
        check(lib().lbrr_engine_load_weights(self.handle, views, len(weights)))

    def load_safetensors(self, path):
        check(lib().lbrr_engine_load_safetensors(self.handle, str(path).encode()))

    # -- forward -------------------------------------------------------------
    def bench_forward(self, x_dev, out_dev, stream=None):
        """One chunk on device buffers: x [len][2] fp32 -> stems [6][2][len] fp32."""
        length = x_dev.numel() // 2
        check(lib().lbrr_forward_chunk(self.handle, _ptr(x_dev), length, _ptr(out_dev), _stream(stream)))

    def forward_chunks(self, x_dev, out_dev, stream=None):
        """Chunks of equal length batched in one forward: x [n][len][2] fp32 ->
        stems [n][6][2][len] fp32, each chunk bit-identical to bench_forward on it."""
        n = x_dev.shape[0]
        length = x_dev.numel() // (2 * n)
        check(lib().lbrr_forward_chunks(self.handle, _ptr(x_dev), length, n, _ptr(out_dev), _stream(stream)))

    def forward_host(self, x_host: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """End to end from host memory: x [len][2] fp32 -> stems [6][2][len] fp32
        (written into `out` when given: a C-contiguous fp32 array of that shape)."""
        x = np.ascontiguousarray(x_host, dtype=np.float32)
        length = x.shape[0]
        out = _out_array(out, (STEMS, 2, length))
        check(lib().lbrr_forward_chunk_host(self.handle, x.ctypes.data, length, out.ctypes.data))
        return out

    def forward_trunk(self, x_dev, n_steps: int, x_out_dev, stream=None):
        length = x_dev.numel() // 2
        check(lib().lbrr_forward_trunk(self.handle, _ptr(x_dev), length, n_steps, _ptr(x_out_dev), _stream(stream)))

    def forward_back(self, out_dev, stream=None):
        """Rerun the back end (mask estimator -> ISTFT) of the last forward."""
        length = out_dev.numel() // 12
        check(lib().lbrr_forward_back(self.handle, length, _ptr(out_dev), _stream(stream)))

    def sync(self):
        check(lib().lbrr_engine_sync(self.handle))

    def set_option(self, option: int, value: int):
        check(lib().lbrr_engine_set_option(self.handle, option, value))

    def get_option(self, option: int) -> int:
        v = C.c_int64()
        check(lib().lbrr_engine_get_option(self.handle, option, C.byref(v)))
        return v.value

    def wait_probe(self, limit_ns: int):
        """Launch the bounded-wait probe (a wait nothing ends, bounded by limit_ns)."""
        check(lib().lbrr_engine_wait_probe(self.handle, limit_ns))

    def read_buffer(self, name: str, shape, dtype) -> np.ndarray:
        """Host copy of an internal buffer of the last forward (diagnostic tap)."""
        out = np.empty(shape, dtype=dtype)
        check(lib().lbrr_engine_read_buffer(self.handle, name.encode(), out.ctypes.data, out.nbytes))
        return out

    def memory(self):
        w, s = C.c_int64(), C.c_int64()
        check(lib().lbrr_engine_memory(self.handle, C.byref(w), C.byref(s)))
        return w.value, s.value

    def close(self):
        if getattr(self, "handle", None):
            lib().lbrr_engine_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _PinnedBlock:
    """Owner of one lbrr_host_alloc block; frees it when the last array view goes."""

    def __init__(self, nbytes: int):
        p = C.c_void_p()
        check(lib().lbrr_host_alloc(nbytes, C.byref(p)))
        self.ptr = p.value

    def __del__(self):
        if getattr(self, "ptr", None) and _lib is not None:
            _lib.lbrr_host_free(self.ptr)
            self.ptr = None


def pinned_empty(shape, dtype=np.float32) -> np.ndarray:
    """An uninitialised C-contiguous array in page-locked host memory
    (lbrr_host_alloc): Engine.forward_host copies such arrays straight to and
    from the device."""
    dtype = np.dtype(dtype)
    n = int(np.prod(shape)) * dtype.itemsize
    block = _PinnedBlock(max(n, 1))
    buf = (C.c_char * max(n, 1)).from_address(block.ptr)
    buf._lbrr_block = block  # every numpy view holds buf, and buf holds the block
    return np.frombuffer(buf, dtype=np.uint8, count=n).view(dtype).reshape(shape)


def _out_array(out, shape):
    if out is None:
        return np.empty(shape, dtype=np.float32)
    if out.shape != shape or out.dtype != np.float32 or not out.flags["C_CONTIGUOUS"]:
        raise LbrrError(ERR_INVALID, f"out must be a C-contiguous float32 array of shape {shape}")
    return out


def separate(engines, audio: np.ndarray, chunk=CHUNK, step=STEP, border=BORDER, interleaved=False,
             out: np.ndarray | None = None, fade: str = "linear") -> np.ndarray:
    """Whole-song demix over one or more engines (separate(), src/main.rs:7598-7819).
    audio: planar [2][len] fp32, or interleaved [len][2] (the WAV layout the C
    ABI takes, passed without a copy) with interleaved=True -> stems
    [6][2][len] fp32, written into `out` when given.  Arrays from
    pinned_empty() move by DMA without host staging copies (same bits)."""
    if interleaved:
        x = np.ascontiguousarray(audio, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != 2:
            raise LbrrError(ERR_INVALID, "interleaved audio must have shape [len][2]")
    else:
        x = np.ascontiguousarray(np.asarray(audio, dtype=np.float32).T)
    length = x.shape[0]
    out = _out_array(out, (STEMS, 2, length))
    hs = (C.c_void_p * len(engines))(*[e.handle for e in engines])
    if fade not in ("linear", "hann"):
        raise LbrrError(ERR_INVALID, "fade must be 'linear' or 'hann'")
    plan = ChunkPlan(chunk, step, border, FADE_HANN if fade == "hann" else FADE_LINEAR)
    check(lib().lbrr_separate_song(hs, len(engines), x.ctypes.data, length, C.byref(plan), out.ctypes.data))
    return out


# ---------------------------------------------------------------------------
# Per-op entry points (torch CUDA tensors; fp16 tensors are torch.float16)
# ---------------------------------------------------------------------------
def op_sync(stream=None):
    check(lib().lbrr_op_sync(_stream(stream)))


def norm_gates(x, gamma, gate_w, gate_b, h16, gates, stream=None):
    check(lib().lbrr_op_norm_gates(_ptr(x), _ptr(gamma), _ptr(gate_w), _ptr(gate_b), _ptr(h16), _ptr(gates),
                                   x.shape[0], _stream(stream)))


def qkv_rope(h16, w16, bias16, cos, sin, qkv, frames, bands, axis, stream=None):
    check(lib().lbrr_op_qkv_rope(_ptr(h16), _ptr(w16), _ptr(bias16), _ptr(cos), _ptr(sin), _ptr(qkv), frames, bands,
                                 axis, _stream(stream)))


def attention(qkv, gates, out, frames, bands, axis, stream=None):
    check(lib().lbrr_op_attention(_ptr(qkv), _ptr(gates), _ptr(out), frames, bands, axis, _stream(stream)))


def outproj_norm(scaled16, w16, bias, resid, gamma, attn_out, h16, stream=None):
    check(lib().lbrr_op_outproj_norm(_ptr(scaled16), _ptr(w16), _ptr(bias), _ptr(resid), _ptr(gamma), _ptr(attn_out),
                                     _ptr(h16), scaled16.shape[0], _stream(stream)))


def ff1_gelu(h16, w16, b1, ff1, stream=None):
    check(lib().lbrr_op_ff1_gelu(_ptr(h16), _ptr(w16), _ptr(b1), _ptr(ff1), h16.shape[0], _stream(stream)))


def ff2_resid(ff1, w16, b2, resid, x, stream=None):
    check(lib().lbrr_op_ff2_resid(_ptr(ff1), _ptr(w16), _ptr(b2), _ptr(resid), _ptr(x), ff1.shape[0],
                                  _stream(stream)))


def feed_forward(h16, w1, b1, w2, b2, resid, x, stream=None):
    """FF1 + GELU -> FF2 + residual in one kernel (no [rows][1024] intermediate)."""
    check(lib().lbrr_op_feed_forward(_ptr(h16), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), _ptr(resid), _ptr(x),
                                     h16.shape[0], _stream(stream)))


def feed_forward_noalloc(h16, w1, b1, w2, b2, resid, x, stream=None):
    """FF1 + GELU -> FF2 + residual without any device allocation (static
    16 MiB scratch, at most 8192 rows); returns after the work finished."""
    check(lib().lbrr_op_feed_forward_noalloc(_ptr(h16), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), _ptr(resid),
                                             _ptr(x), h16.shape[0], _stream(stream)))


def f32_to_f16_bits(v: float) -> int:
    return int(lib().lbrr_f32_to_f16_bits(C.c_float(v)))
