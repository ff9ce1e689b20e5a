"""CPU oracle for the BS-RoFormer chunk forward and the whole-song demix.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or as the timed CPU baseline.  The product path
(the CUDA library behind ``include/lbrr_gpu.h``) never calls into it.

Why a restatement: the reference's own implementation cannot run here.  Its GPU
pipeline is Rust compiled by cuda-oxide (an empty git submodule, no rustc in the
image) and its PyTorch model class (``pymss_core`` BSRoformer) is not vendored.
This module restates, op by op, what ``bench_forward``/``transformer_step`` in
``src/main.rs`` compute, in two modes:

* ``"f16path"`` -- the reference GPU path: fp16 GEMM operands rounded (RNE) at
  exactly the boundaries where the reference packs f16x2 words, fp32 everywhere
  else (residual stream, gates, pre-GLU, GLU, STFT/ISTFT).
* ``"fp32"``    -- plain fp32 math with exact-erf GELU, i.e. the PyTorch fp32
  model that the reference's 60 dB golden gate compares against
  (``scripts/ci.sh:13``).

Pinning: the per-op formulas here are checked against golden vectors produced
by the reference's own generator ``tools/dump_refs.py`` (STFT, RMSNorm,
band-split, the four trunk GEMM shapes, QKV+RoPE, short/long SDPA,
gate/out-proj/FF), and the song demix against ``tools/bench_ref.py``
(``chunk_starts``/``reflect_pad``/``demix`` with an identity model).  The
fixtures live in ``tests/golden/`` with the script that made them.  The
cuDNN/cuBLASLt internals of the reference's production path have no fixture in
the reference tree (the checkpoint and ``ref_output.npz`` are not shipped), so
the model-level composition is pinned only through those per-op gates.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

# ---------------------------------------------------------------------------
# Model constants (assets/logic_bs_roformer.yaml:11-84, src/stft.rs:19-21)
# ---------------------------------------------------------------------------
N_FFT = 2048
HOP = 512
FREQ_BINS = N_FFT // 2 + 1
FREQS_PER_BANDS = [2] * 24 + [4] * 12 + [12] * 8 + [24] * 8 + [48] * 8 + [128, 129]
DIM = 256
DEPTH = 12
HEADS = 8
DIM_HEAD = 64
STEMS = 6
FF_DIM = 1024
INSTRUMENTS = ["bass", "drums", "other", "vocals", "guitar", "piano"]
# song chunking (src/main.rs:7617-7619, tools/bench_ref.py:13)
CHUNK = 588800
STEP = 559360
BORDER = 29440


def f16(x: torch.Tensor) -> torch.Tensor:
    """Round fp32 to fp16 (RNE) and back: the reference's cvt_f16x2_f32 / fp16::f32_to_f16_bits."""
    return x.to(torch.float16).to(torch.float32)


# ---------------------------------------------------------------------------
# Geometry helpers
# ---------------------------------------------------------------------------
@dataclass
class BandLayout:
    """Band geometry: d_b = 4*freqs, offs = prefix sums of d_b, f0 = offs/4.

    src/main.rs:7288-7292 (dims/offs/f0) and :7164-7166 (mask2 tile table).
    """

    freqs: list = field(default_factory=lambda: list(FREQS_PER_BANDS))

    def __post_init__(self):
        self.dims = [4 * f for f in self.freqs]
        self.offs = [0]
        for d in self.dims:
            self.offs.append(self.offs[-1] + d)
        self.f0 = [o // 4 for o in self.offs[:-1]]
        self.n = len(self.freqs)
        self.total = self.offs[-1]  # 4100


def num_frames(length: int) -> int:
    """Center-mode STFT frame count (src/stft.rs:32-34)."""
    return length // HOP + 1


def hann_window(n: int = N_FFT) -> torch.Tensor:
    """Periodic Hann computed in f64 then cast to f32 (src/stft.rs:25-29)."""
    i = np.arange(n, dtype=np.float64)
    return torch.from_numpy((0.5 * (1.0 - np.cos(2.0 * np.pi * i / n))).astype(np.float32))


def rope_tables(length: int):
    """cos/sin[pos][32]: angle = pos * 10000^(-2i/64) in f64, cast to f32, then cos/sin.

    src/main.rs:7678-7681 (song) and :7293 (bench) compute the angle in f64 and
    round it to f32 before the f32 cos/sin; the f32 cos/sin here are the
    correctly rounded values of the f32 angle.
    """
    p = np.arange(length, dtype=np.float64)[:, None]
    i = np.arange(32, dtype=np.float64)[None, :]
    ang = (p * (1.0 / np.power(10000.0, 2.0 * i / 64.0))).astype(np.float32).astype(np.float64)
    return (torch.from_numpy(np.cos(ang).astype(np.float32)),
            torch.from_numpy(np.sin(ang).astype(np.float32)))


# ---------------------------------------------------------------------------
# STFT front end
# ---------------------------------------------------------------------------
def stft_frames(x: torch.Tensor, window: torch.Tensor | None = None) -> torch.Tensor:
    """Reflect-padded framing times the window: frames[ch][t][j].

    x: planar [2][L] fp32.  Follows frame_hann_reflect (src/main.rs:396-429):
    g = t*hop + j; src = pad-g (g<pad), 2L+pad-2-g (g>=L+pad), else g-pad.
    """
    if window is None:
        window = hann_window()
    ch, length = x.shape
    t_frames = num_frames(length)
    pad = N_FFT // 2
    g = torch.arange(t_frames)[:, None] * HOP + torch.arange(N_FFT)[None, :]
    src = torch.where(g < pad, pad - g, torch.where(g >= length + pad, 2 * length + pad - 2 - g, g - pad))
    return x[:, src] * window[None, None, :]


def stft(x: torch.Tensor) -> torch.Tensor:
    """spec[ch][t][f] complex: rFFT of the framed signal (cuFFT R2C, src/stft.rs:55-57)."""
    frames = stft_frames(x).double()
    return torch.fft.rfft(frames, n=N_FFT, dim=-1).to(torch.complex64)


def spec_reorder(spec: torch.Tensor) -> torch.Tensor:
    """x_in[t][4f + 2ch + c] = spec[ch][t][f].c  (spec_reorder, src/main.rs:1649-1677)."""
    r = torch.view_as_real(spec)  # [2][T][1025][2]
    return r.permute(1, 2, 0, 3).reshape(r.shape[1], -1).contiguous()


# ---------------------------------------------------------------------------
# Norms and activations
# ---------------------------------------------------------------------------
def _rms_scale(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1]
    norm = torch.sqrt((x * x).sum(-1, keepdim=True))
    denom = torch.clamp(norm, min=1e-12)
    return torch.tensor(math.sqrt(d), dtype=torch.float32) / denom


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, assoc: str = "left") -> torch.Tensor:
    """x/max(||x||,1e-12)*sqrt(d)*gamma.

    assoc="left":  (v*scale)*gamma  -- rmsnorm / rmsnorm_h16 (src/main.rs:444-483, :536-540)
    assoc="right": v*(scale*gamma)  -- rmsnorm_gates_h16 (src/main.rs:672-675)
    """
    scale = _rms_scale(x)
    if assoc == "left":
        return (x * scale) * gamma
    return x * (scale * gamma)


def gelu_as(v: torch.Tensor) -> torch.Tensor:
    """GELU with the Abramowitz-Stegun 7.1.26 erf (src/main.rs:2928-2935)."""
    sign = torch.where(v < 0, -1.0, 1.0)
    a = v.abs() * 0.70710678
    t = 1.0 / (1.0 + 0.3275911 * a)
    poly = ((((1.061405429 * t - 1.453152027) * t + 1.421413741) * t - 0.284496736) * t + 0.254829592) * t
    erfa = sign * (1.0 - poly * torch.exp(-a * a))
    return 0.5 * v * (1.0 + erfa)


def sigmoid(v: torch.Tensor) -> torch.Tensor:
    """1/(1+exp(-v)) (sdpa_gate src/main.rs:3779, glu_scatter :4993)."""
    return 1.0 / (1.0 + torch.exp(-v))


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved RoPE on the last dim (64): (e*c - o*s, o*c + e*s) per pair.

    x: [..., S, 64] with positions along S; cos/sin: [S][32].
    rope_k16 / rope_q16_inplace (src/main.rs:3684-3754), tools/dump_refs.py:120-128.
    """
    e = x[..., 0::2]
    o = x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = e * cos - o * sin
    out[..., 1::2] = o * cos + e * sin
    return out


# ---------------------------------------------------------------------------
# Weights
# ---------------------------------------------------------------------------
def weight_keys(layout: BandLayout | None = None):
    """All 1989 checkpoint keys with shapes, in src/weights.rs:307-432 order."""
    layout = layout or BandLayout()
    keys = [("linear_62_bias_0", (3 * HEADS * DIM_HEAD,)), ("linear_64_bias_0", (DIM,))]
    for l in range(DEPTH):
        for a in range(2):
            p = f"layers.{l}.{a}.layers.0.0"
            keys += [
                (f"{p}.norm.gamma", (DIM,)),
                (f"{p}.to_qkv.weight", (3 * HEADS * DIM_HEAD, DIM)),
                (f"{p}.to_gates.weight", (HEADS, DIM)),
                (f"{p}.to_gates.bias", (HEADS,)),
                (f"{p}.to_out.0.weight", (DIM, HEADS * DIM_HEAD)),
            ]
            fp = f"layers.{l}.{a}.layers.0.1.net"
            keys += [
                (f"{fp}.0.gamma", (DIM,)),
                (f"{fp}.1.weight", (FF_DIM, DIM)),
                (f"{fp}.1.bias", (FF_DIM,)),
                (f"{fp}.4.weight", (DIM, FF_DIM)),
                (f"{fp}.4.bias", (DIM,)),
                (f"{p}.to_qkv.bias", (3 * HEADS * DIM_HEAD,)),
                (f"{p}.to_out.0.bias", (DIM,)),
                (f"{p}.rotary_embed.freqs", (DIM_HEAD // 2,)),
            ]
    keys.append(("final_norm.gamma", (DIM,)))
    for b in range(layout.n):
        d = layout.dims[b]
        keys += [
            (f"band_split.to_features.{b}.0.gamma", (d,)),
            (f"band_split.to_features.{b}.1.weight", (DIM, d)),
            (f"band_split.to_features.{b}.1.bias", (DIM,)),
        ]
    for s in range(STEMS):
        for b in range(layout.n):
            d = layout.dims[b]
            p = f"mask_estimators.{s}.to_freqs.{b}.0"
            keys += [
                (f"{p}.0.weight", (FF_DIM, DIM)),
                (f"{p}.0.bias", (FF_DIM,)),
                (f"{p}.2.weight", (2 * d, FF_DIM)),
                (f"{p}.2.bias", (2 * d,)),
            ]
    return keys


def make_weights(seed: int = 0, std: float = 0.02, gamma_noise: float = 0.0, layout: BandLayout | None = None):
    """Seeded synthetic checkpoint: every *.weight / *.bias ~ N(0, std), gammas = 1
    (+ optional N(0, gamma_noise) for op tests), shared biases duplicated bit-identically
    into the 24 per-layer keys, rotary freqs = 1/10000^(2i/64)."""
    gen = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in weight_keys(layout):
        if name.endswith("rotary_embed.freqs"):
            i = torch.arange(DIM_HEAD // 2, dtype=torch.float32)
            out[name] = 1.0 / torch.pow(torch.tensor(10000.0), 2.0 * i / DIM_HEAD)
        elif name.endswith("to_qkv.bias"):
            out[name] = out["linear_62_bias_0"].clone()
        elif name.endswith("to_out.0.bias"):
            out[name] = out["linear_64_bias_0"].clone()
        elif name.endswith("gamma"):
            g = torch.ones(shape)
            if gamma_noise:
                g = g + torch.randn(shape, generator=gen) * gamma_noise
            out[name] = g
        else:
            out[name] = torch.randn(shape, generator=gen) * std
    return out


# ---------------------------------------------------------------------------
# Model forward
# ---------------------------------------------------------------------------
class Oracle:
    """Chunk forward of the BS-RoFormer (src/main.rs:7014-7162 order and layouts)."""

    def __init__(self, weights: dict, mode: str = "f16path", layout: BandLayout | None = None):
        assert mode in ("f16path", "fp32")
        self.w = weights
        self.mode = mode
        self.L = layout or BandLayout()
        self.h = f16 if mode == "f16path" else (lambda t: t)

    # -- helpers -----------------------------------------------------------
    def _mm(self, a, w):
        """a @ w^T with fp32 accumulation (weights rounded to f16 in f16path)."""
        return a @ self.h(w).T

    # -- band split --------------------------------------------------------
    def band_split(self, x_in: torch.Tensor) -> torch.Tensor:
        """Per band RMSNorm(d_b) then Linear(d_b -> 256); output folded token t*62+b.

        bandsplit_norm (src/main.rs:792-828) + bandsplit_gemm_f16 (:4600-4699).
        """
        T = x_in.shape[0]
        out = torch.empty(T, self.L.n, DIM)
        for b in range(self.L.n):
            seg = x_in[:, self.L.offs[b]:self.L.offs[b + 1]]
            g = self.w[f"band_split.to_features.{b}.0.gamma"]
            v = rmsnorm(seg, g, "left")
            out[:, b] = self._mm(self.h(v), self.w[f"band_split.to_features.{b}.1.weight"]) + \
                self.w[f"band_split.to_features.{b}.1.bias"]
        return out.reshape(T * self.L.n, DIM)

    # -- attention ---------------------------------------------------------
    def attention(self, q, k, v):
        """softmax(q k^T * 0.125) v per (seq, head).  q,k,v: [B, H, S, 64].

        f16path: P rounded to f16 before P@V and the row sum kept in fp32, as the
        reference's own flash kernels do (attn_flash_tc, src/main.rs:3944-3994);
        output rounded to f16 (the f16 SDPA output of src/main.rs:6193-6196).
        """
        B = q.shape[0]
        outs = []
        step = max(1, int(2 ** 27 // max(1, q.shape[1] * q.shape[2] * k.shape[2])))
        for i in range(0, B, step):
            s = (q[i:i + step] @ k[i:i + step].transpose(-1, -2)) * 0.125
            m = s.amax(-1, keepdim=True)
            e = torch.exp(s - m)
            l = e.sum(-1, keepdim=True)
            if self.mode == "f16path":
                o = f16((f16(e) @ v[i:i + step]) / l)
            else:
                o = (e @ v[i:i + step]) / l
            outs.append(o)
        return torch.cat(outs, 0)

    # -- one transformer axis ---------------------------------------------
    def transformer_step(self, x: torch.Tensor, layer: int, axis: int, T: int) -> torch.Tensor:
        """One RoFormer axis on the folded token tensor x[M][256] (token = t*62 + b).

        transformer_step, src/main.rs:6131-6268.
        """
        nb = self.L.n
        p = f"layers.{layer}.{axis}.layers.0.0"
        fp = f"layers.{layer}.{axis}.layers.0.1.net"
        w = self.w
        hq = self.h
        # 1. pre-attention RMSNorm + gates (rmsnorm_gates_h16, :616-703)
        hf = rmsnorm(x, w[f"{p}.norm.gamma"], "right")
        gates = hf @ w[f"{p}.to_gates.weight"].T + w[f"{p}.to_gates.bias"]
        h16 = hq(hf)
        # 2. QKV with the shared bias pre-rounded to f16 (:5960-5962, :6157-6161)
        bias = hq(w["linear_62_bias_0"])
        qkv = hq(self._mm(h16, w[f"{p}.to_qkv.weight"]) + bias)
        q, k, v = qkv[:, :512], qkv[:, 512:1024], qkv[:, 1024:]
        # fold into sequences: time axis -> seq per band over t; freq -> seq per t over b
        def fold(a):
            a = a.reshape(T, nb, HEADS, DIM_HEAD)
            if axis == 0:
                return a.permute(1, 2, 0, 3)  # [62][H][T][64]
            return a.permute(0, 2, 1, 3)      # [T][H][62][64]

        def unfold(a):
            if axis == 0:
                return a.permute(2, 0, 1, 3).reshape(T * nb, HEADS * DIM_HEAD)
            return a.permute(0, 2, 1, 3).reshape(T * nb, HEADS * DIM_HEAD)

        S = T if axis == 0 else nb
        cos, sin = rope_tables(S)
        qf = hq(rope(fold(q), cos, sin))
        kf = hq(rope(fold(k), cos, sin))
        vf = fold(v)
        o = unfold(self.attention(qf, kf, vf))
        # 3. gate + out-proj + bias + residual (sdpa_gate :3769-3786, :6219-6223)
        attn_out = self.gate_outproj(o, gates, w[f"{p}.to_out.0.weight"], w["linear_64_bias_0"], x)
        # 4. FF (:6234-6259)
        hff = hq(rmsnorm(attn_out, w[f"{fp}.0.gamma"], "left"))
        return self.feed_forward(hff, w[f"{fp}.1.weight"], w[f"{fp}.1.bias"],
                                 w[f"{fp}.4.weight"], w[f"{fp}.4.bias"], attn_out)

    def gate_outproj(self, o, gates, wo, bo, resid):
        """o * sigmoid(gate[token][head]) (rounded to f16 in f16path), then
        out-proj + bias + residual (sdpa_gate src/main.rs:3769-3786; :6219-6223)."""
        sig = sigmoid(gates).repeat_interleave(DIM_HEAD, dim=1)
        scaled = self.h(o * sig)
        return self._mm(scaled, wo) + bo + resid

    def feed_forward(self, h, w1, b1, w2, b2, resid):
        """FF1 + GELU (A&S erf, rounded to f16, in f16path; exact erf in fp32) then
        FF2 + bias + residual (gemm_f16_gelu_a16w :2827-2949; :6255-6259)."""
        pre = self._mm(h, w1) + b1
        if self.mode == "f16path":
            ff1 = f16(gelu_as(pre))
        else:
            ff1 = torch.nn.functional.gelu(pre)
        return self._mm(ff1, w2) + b2 + resid

    # -- mask estimator ----------------------------------------------------
    def mask_estimator(self, xf: torch.Tensor, T: int) -> torch.Tensor:
        """Per stem, per band MLP: tanh(x W1^T + b1) W2^T + b2, then GLU.

        mask_gemm1_f16 (:4705-4843), mask_gemm2_f16 (:4849-4978), glu_scatter (:4984-4997).
        Returns masks[stem][T][4100] (layout d = fi*4 + ch*2 + c).
        """
        nb = self.L.n
        xb = self.h(xf).reshape(T, nb, DIM)
        out = torch.empty(STEMS, T, self.L.total)
        for s in range(STEMS):
            for b in range(nb):
                p = f"mask_estimators.{s}.to_freqs.{b}.0"
                pre1 = self._mm(xb[:, b], self.w[f"{p}.0.weight"]) + self.w[f"{p}.0.bias"]
                hid = self.h(torch.tanh(pre1))
                pre2 = self._mm(hid, self.w[f"{p}.2.weight"]) + self.w[f"{p}.2.bias"]
                d = self.L.dims[b]
                out[s, :, self.L.offs[b]:self.L.offs[b + 1]] = pre2[:, :d] * sigmoid(pre2[:, d:]) \
                    if self.mode == "f16path" else torch.nn.functional.glu(pre2, dim=-1)
        return out

    def mask_apply(self, spec: torch.Tensor, masks: torch.Tensor) -> torch.Tensor:
        """masked[stem][ch][t][f] = spec[ch][t][f] * (m_re + i m_im) (mask_apply, :1776-1817)."""
        T = spec.shape[1]
        m = masks.reshape(STEMS, T, FREQ_BINS, 2, 2)  # [s][t][f][ch][c]
        mc = torch.complex(m[..., 0], m[..., 1]).permute(0, 3, 1, 2)  # [s][ch][t][f]
        return spec[None] * mc

    # -- full chunk --------------------------------------------------------
    def trunk(self, x: torch.Tensor, T: int, layers: int = DEPTH) -> torch.Tensor:
        for layer in range(layers):
            for axis in range(2):
                x = self.transformer_step(x, layer, axis, T)
        return x

    def forward(self, audio: torch.Tensor, layers: int = DEPTH, return_parts: bool = False):
        """audio: planar [2][L] fp32 -> stems [6][2][L] fp32 (bench_forward + istft_ola)."""
        length = audio.shape[1]
        T = num_frames(length)
        spec = stft(audio)
        x = self.band_split(spec_reorder(spec))
        x = self.trunk(x, T, layers)
        xf = rmsnorm(x, self.w["final_norm.gamma"], "left")
        masks = self.mask_estimator(xf, T)
        masked = self.mask_apply(spec, masks)
        y = istft(masked.reshape(STEMS * 2, T, FREQ_BINS), length).reshape(STEMS, 2, length)
        if return_parts:
            return y, {"spec": spec, "x_trunk": x, "xf": xf, "masks": masks, "masked": masked}
        return y


def istft(spec: torch.Tensor, length: int) -> torch.Tensor:
    """torch.istft(center=True, hann, length=L) restated: irFFT (1/n), x window, OLA,
    divide by the window-square envelope, crop [n_fft/2, n_fft/2 + L).

    istft_ola (src/main.rs:5024-5039) + benchmark::istft_inverse (src/benchmark.rs:129-142).
    spec: [B][T][1025] complex -> [B][L].
    """
    B, T, _ = spec.shape
    win = hann_window().double()
    pcm = torch.fft.irfft(spec.to(torch.complex128), n=N_FFT, dim=-1) * win  # [B][T][2048]
    total = (T - 1) * HOP + N_FFT
    y = torch.zeros(B, total, dtype=torch.float64)
    env = torch.zeros(total, dtype=torch.float64)
    w2 = (hann_window() * hann_window()).double()
    for t in range(T):
        y[:, t * HOP:t * HOP + N_FFT] += pcm[:, t]
        env[t * HOP:t * HOP + N_FFT] += w2
    pad = N_FFT // 2
    y = y[:, pad:pad + length]
    e = env[pad:pad + length]
    inv = torch.where(e > 1e-8, 1.0 / e, torch.zeros_like(e))
    return (y * inv).to(torch.float32)


# ---------------------------------------------------------------------------
# Whole-song demix (src/main.rs:7617-7819, tools/bench_ref.py:33-65)
# ---------------------------------------------------------------------------
def chunk_starts(length: int, chunk: int = CHUNK, step: int = STEP, border: int = BORDER):
    """Chunk grid covering [border, border+length) (tools/bench_ref.py:33-37)."""
    if length <= 0:
        raise ValueError("empty audio is unsupported")
    needed = border + length
    last = max(0, (needed - chunk + step - 1) // step)
    return [i * step for i in range(last + 1)]


def reflect_pad(x: np.ndarray, left: int, right: int) -> np.ndarray:
    """numpy-style reflect padding with multiple periods (tools/bench_ref.py:39-45)."""
    length = x.shape[-1]
    if length == 0:
        raise ValueError("empty audio is unsupported")
    if length == 1:
        return np.repeat(x, left + length + right, axis=-1)
    p = np.arange(-left, length + right) % (2 * (length - 1))
    p = np.where(p < length, p, 2 * (length - 1) - p)
    return x[..., p]


def fade_window(chunk: int = CHUNK, border: int = BORDER) -> np.ndarray:
    """Linear fade in/out of width border (tools/bench_ref.py:50-52)."""
    fade = np.ones(chunk, dtype=np.float32)
    fade[:border] = np.arange(border, dtype=np.float32) / border
    fade[-border:] = fade[:border][::-1]
    return fade


def hann_fade(chunk: int) -> np.ndarray:
    """Periodic Hann window over the chunk, in f64 rounded to f32: the weight of
    BASELINE config 4's 50 %-overlap plan (not a reference plan; the reference
    only has the linear fade)."""
    n = np.arange(chunk, dtype=np.float64)
    return (0.5 * (1.0 - np.cos(2.0 * np.pi * n / chunk))).astype(np.float32)


def demix(model, x: np.ndarray, chunk: int = CHUNK, step: int = STEP, border: int = BORDER,
          fade_kind: str = "linear") -> np.ndarray:
    """Chunked overlap-add demix: model(xp[..., s:s+chunk]) -> [6][2][chunk].

    Fade-weighted accumulate with first/last border overrides, divide by the
    accumulated fade energy, crop the border (tools/bench_ref.py:47-65).
    fade_kind "hann" replaces the linear fade by hann_fade (same accumulation).
    x: planar [2][L].  Returns [6][2][L] fp32.
    """
    length = x.shape[-1]
    starts = chunk_starts(length, chunk, step, border)
    needed = border + length
    xp = reflect_pad(x, border, starts[-1] + chunk - needed)
    fade = fade_window(chunk, border) if fade_kind == "linear" else hann_fade(chunk)
    result = None
    counter = np.zeros(needed, dtype=np.float32)
    for i, s in enumerate(starts):
        y = np.asarray(model(xp[..., s:s + chunk]), dtype=np.float32)
        if result is None:
            result = np.zeros(y.shape[:-1] + (needed,), dtype=np.float32)
        w = fade.copy()
        if i == 0:
            w[:border] = 1
        if i == len(starts) - 1:
            w[-border:] = 1
        take = min(chunk, needed - s)
        result[..., s:s + take] += y[..., :take] * w[:take]
        counter[s:s + take] += w[:take] * w[:take]
    if not (counter[border:needed] > 0).all():
        raise RuntimeError("uncovered audio tail")
    return (result / np.maximum(counter, 1e-8))[..., border:needed]


# ---------------------------------------------------------------------------
# Synthetic inputs and metrics
# ---------------------------------------------------------------------------
def synth_audio(length: int, seed: int = 0, sr: int = 44100) -> np.ndarray:
    """Seeded synthetic stereo audio [2][L]: per channel 8 sines (50 Hz-15 kHz,
    random phase, amplitude U(0.05, 0.15)) + N(0, 0.05) noise, scaled to peak 0.5."""
    rs = np.random.RandomState(seed)
    t = np.arange(length, dtype=np.float64) / sr
    out = np.empty((2, length), dtype=np.float32)
    for ch in range(2):
        f = rs.uniform(50.0, 15000.0, 8)
        ph = rs.uniform(0, 2 * np.pi, 8)
        a = rs.uniform(0.05, 0.15, 8)
        sig = (a[:, None] * np.sin(2 * np.pi * f[:, None] * t[None, :] + ph[:, None])).sum(0)
        sig = sig + rs.normal(0.0, 0.05, length)
        out[ch] = sig
    peak = np.abs(out).max()
    return (out * (0.5 / max(peak, 1e-12))).astype(np.float32)


def metric(actual: np.ndarray, reference: np.ndarray) -> dict:
    """finite / rms / SNR dB / max-abs error / bit-equality (src/benchmark.rs:57-83)."""
    a = np.asarray(actual, dtype=np.float64).ravel()
    r = np.asarray(reference, dtype=np.float64).ravel()
    finite = bool(np.isfinite(a).all() and np.isfinite(r).all())
    signal = float((r * r).sum())
    d = a - r
    noise = float((d * d).sum()) if finite else float("nan")
    rms = math.sqrt(signal / max(1, r.size))
    return {
        "finite": finite,
        "reference_rms": rms,
        "snr_db": 10.0 * math.log10(signal / max(noise, 1e-300)) if finite and rms >= 1e-8 else None,
        "max_abs_error": float(np.abs(d).max()) if finite and d.size else 0.0,
        "bit_equal": bool(np.array_equal(np.asarray(actual, np.float32), np.asarray(reference, np.float32))),
    }


def matrix_flops(t: int) -> int:
    """Algorithmic FLOP per chunk (src/benchmark.rs:105-117)."""
    m = 62 * t
    trunk = 24 * (2 * m * 1536 * 256 + 2 * m * 256 * 512 + 2 * m * 1024 * 256 + 2 * m * 256 * 1024 + 2 * m * 8 * 256)
    attn = 12 * 4 * 62 * 8 * t * t * 64 + 12 * 4 * t * 8 * 62 * 62 * 64
    mask = 6 * (2 * m * 1024 * 256 + 2 * t * 8200 * 1024)
    return trunk + attn + mask + 2 * t * 4100 * 256
