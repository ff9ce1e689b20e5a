// In-house FFT for the STFT front end and the ISTFT back end, fused with the
// bandwidth work around them (replaces cuFFT R2C/C2R of the reference,
// src/stft.rs:36-57, src/main.rs:7033-7040, :7154-7160, together with
// frame_hann_reflect :396-429, spec_reorder :1649-1677, bandsplit_norm
// :792-828 and istft_ola :5024-5039).
//
// Both transforms are 2048-point real FFTs computed as one 1024-point complex
// FFT of z[m] = x[2m] + i x[2m+1] plus the usual split step
//   X[k] = E[k] + W^k O[k],  E[k] = (Z[k] + conj Z[1024-k]) / 2,
//   O[k] = (Z[k] - conj Z[1024-k]) / 2i,  W = exp(-2 pi i / 2048),
// and its inverse.  The 1024-point FFT is 32 x 32 (four-step): one warp owns a
// frame; lane b first runs a 32-point DFT over inputs 32a + b (a = 0..31) in
// registers, multiplies by w^(b c), and hands the result to lane c through a
// 33-column padded shared-memory transpose for the second 32-point DFT.  The
// 32-point DFTs are radix-2 decimation in frequency with twiddles folded into
// immediates; the 1024/2048-point twiddles come from a per-CTA table of
// exp(2 pi i k / 2048) computed in double precision on the host.
//
//   stft_front_kernel  reflect-padded Hann framing of both channels, forward
//                      FFT, spectrum out ([2][T][1025], needed by the mask
//                      stage) and the band RMSNorm of every band straight from
//                      shared memory into the fp16 band-split input xn.
//   istft_back_kernel  one channel, a run of 512-sample output blocks: the
//                      inverse FFT of every frame touching them (three frames
//                      of overlap recomputed by the neighbouring CTA), Hann
//                      window, overlap-add in frame order, division by the
//                      window-square envelope, crop -- one pass over the
//                      masked spectra and one write of the waveform.
// The DC and Nyquist bins are taken as real (their imaginary parts, which a
// real signal's spectrum does not have, are ignored), the torch.istft
// convention.
#include "common.cuh"
#include "kernels.h"

namespace lbrr {

namespace {

constexpr int kTwN = 2048;                 // twiddle table entries: exp(2 pi i k / 2048)
constexpr int kXpose = 32 * 33;            // padded 32 x 32 complex transpose (8448 B)
__device__ constexpr float kW32c[16] = {1.0f,           9.807852804e-01f, 9.238795325e-01f, 8.314696123e-01f,
                             7.071067812e-01f, 5.555702330e-01f, 3.826834324e-01f, 1.950903220e-01f,
                             0.0f,           -1.950903220e-01f, -3.826834324e-01f, -5.555702330e-01f,
                             -7.071067812e-01f, -8.314696123e-01f, -9.238795325e-01f, -9.807852804e-01f};
__device__ constexpr float kW32s[16] = {0.0f,           1.950903220e-01f, 3.826834324e-01f, 5.555702330e-01f,
                             7.071067812e-01f, 8.314696123e-01f, 9.238795325e-01f, 9.807852804e-01f,
                             1.0f,           9.807852804e-01f, 9.238795325e-01f, 8.314696123e-01f,
                             7.071067812e-01f, 5.555702330e-01f, 3.826834324e-01f, 1.950903220e-01f};

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }

__host__ __device__ constexpr int bitrev5(int i) {
  return ((i & 1) << 4) | ((i & 2) << 2) | (i & 4) | ((i & 8) >> 2) | ((i & 16) >> 4);
}

// In-register 32-point DFT, radix-2 decimation in frequency: on return v[i]
// holds output bitrev5(i).  INV selects exp(+2 pi i jk / 32) (inverse,
// unnormalised) over exp(-2 pi i jk / 32).
template <bool INV>
__device__ __forceinline__ void dft32(float2 (&v)[32]) {
#pragma unroll
  for (int span = 16; span >= 1; span >>= 1) {
#pragma unroll
    for (int start = 0; start < 32; start += 2 * span) {
#pragma unroll
      for (int j = 0; j < span; ++j) {
        const float2 a = v[start + j], b = v[start + j + span];
        v[start + j] = cadd(a, b);
        const float2 d = csub(a, b);
        const int k = j * (16 / span);  // twiddle W_32^k
        if (k == 0) {
          v[start + j + span] = d;
        } else if (k == 8) {
          v[start + j + span] = INV ? make_float2(-d.y, d.x) : make_float2(d.y, -d.x);
        } else {
          const float2 w = make_float2(kW32c[k], INV ? kW32s[k] : -kW32s[k]);
          v[start + j + span] = cmul(d, w);
        }
      }
    }
  }
}

// Twiddles come from a per-CTA shared-memory copy of tws[k] = exp(+2 pi i k /
// 2048) for k in [0, 1024) (8 KB; the second half of the circle is the first
// negated).
constexpr int kTwS = 1024;
__device__ __forceinline__ float2 twiddle(const float2* tws, int k) {
  const float2 w = tws[k & (kTwS - 1)];
  return (k & kTwS) ? make_float2(-w.x, -w.y) : w;
}
// 16-byte asynchronous global -> shared copies (no registers involved, all in
// flight at once), completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
// Copy the first kTwS entries of the global table into shared memory.
__device__ __forceinline__ void load_twiddles(float2* tws, const float2* __restrict__ twg) {
  for (int i = 2 * threadIdx.x; i < kTwS; i += 2 * blockDim.x) cp_async16(tws + i, twg + i);
}

// 1024-point complex FFT of one frame by one warp.  On entry lane b holds
// v[a] = input[32a + b]; on return lane c holds v[i] = output[c + 32 *
// bitrev5(i)].  `xp` is the warp's padded transpose buffer, `tw` the shared
// twiddle table.
template <bool INV>
__device__ __forceinline__ void fft1024_warp(float2 (&v)[32], float2* xp, const float2* tw, int lane) {
  dft32<INV>(v);
  // v[i] = U[b][c], c = bitrev5(i); times w^(b c), w = exp(+-2 pi i / 1024) = tw[2 b c]
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int c = bitrev5(i);
    float2 w = twiddle(tw, 2 * lane * c);
    if (!INV) w.y = -w.y;
    xp[c * 33 + lane] = c == 0 ? v[i] : cmul(v[i], w);
  }
  __syncwarp();
#pragma unroll
  for (int b = 0; b < 32; ++b) v[b] = xp[lane * 33 + b];
  __syncwarp();
  dft32<INV>(v);
}

}  // namespace

// ---------------------------------------------------------------------------
// Front end: one frame per CTA of four warps.  Warps 0 and 1 transform the two
// channels (each owning one 8.4 KB shared-memory slot that holds its
// transpose, then Z, then the spectrum X in place); then all four warps run
// the band RMSNorm of the frame's 62 bands.  17 KB of shared memory and at
// most 96 registers a thread: five CTAs per SM.
// ---------------------------------------------------------------------------
constexpr int kFrontWarps = 4;
constexpr int kFrontSmem = 2 * kXpose * 8 + kTwS * 8 + kNumBands * 8 * 4;

__global__ void __launch_bounds__(kFrontWarps * 32, 5) stft_front_kernel(const float* __restrict__ x,
                                                                     const float* __restrict__ win,
                                                                     const float2* __restrict__ twg,
                                                                     float2* __restrict__ spec,
                                                                     const float* __restrict__ gamma,
                                                                     const int* __restrict__ tab,
                                                                     __half* __restrict__ xn, int xn_cols, int len,
                                                                     int T, int nb) {
  extern __shared__ __align__(16) float2 fsm[];
  float2* tw = fsm + 2 * kXpose;
  int* stab = reinterpret_cast<int*>(tw + kTwS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // frame t of chunk blockIdx.y: that chunk's samples start len stereo pairs
  // further on; its frames are rows chunk*T.. of the chunks' common spectrum
  // planes (T * gridDim.y frames per channel) and band-split rows
  const int t = blockIdx.x;
  const int tg = blockIdx.y * T + t;
  const int Tp = T * gridDim.y;
  x += 2ll * len * blockIdx.y;
  const int pad = kNfft / 2;
  // Interior frames (no reflection) stage their 2048 interleaved stereo
  // samples, 16 KB contiguous and 16-byte aligned, with coalesced 16-byte loads
  // across both channels' slots; frames at the song edges gather per sample.
  const bool interior = t * kHop >= pad && t * kHop + kNfft <= len + pad &&
                        (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  if (interior) {
    const float4* src = reinterpret_cast<const float4*>(x + 2ll * (t * kHop - pad));
    float4* dst = reinterpret_cast<float4*>(fsm);
    for (int i = threadIdx.x; i < kNfft / 2; i += blockDim.x) cp_async16(dst + i, src + i);
  }
  for (int i = threadIdx.x; i < nb * 8; i += blockDim.x) stab[i] = __ldg(tab + i);
  load_twiddles(tw, twg);
  cp_async_wait_all();
  __syncthreads();
  if (warp < 2) {
    const int ch = warp;
    float2* xp = fsm + warp * kXpose;
    // z[m] = x[2m] + i x[2m+1] of the windowed, reflect-padded frame; lane b loads z[32a + b]
    float2 v[32];
    const float* staged = reinterpret_cast<const float*>(fsm);
#pragma unroll
    for (int a = 0; a < 32; ++a) {
      const int j = 64 * a + 2 * lane;
      const float2 w2 = __ldg(reinterpret_cast<const float2*>(win) + (j >> 1));
      float s2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (interior) {
          s2[e] = staged[2 * (j + e) + ch];
        } else {
          const int g = t * kHop + j + e;
          const int src = g < pad ? pad - g : (g >= len + pad ? 2 * len + pad - 2 - g : g - pad);
          s2[e] = __ldg(x + 2ll * src + ch);
        }
      }
      v[a] = make_float2(s2[0] * w2.x, s2[1] * w2.y);
    }
    // both channels have read the staged samples before either slot is reused
    asm volatile("bar.sync 1, 64;" ::: "memory");
    fft1024_warp<false>(v, xp, tw, lane);
    // Z[c + 32 d] (d = bitrev5(i)) into the slot, linear order
#pragma unroll
    for (int i = 0; i < 32; ++i) xp[lane + 32 * bitrev5(i)] = v[i];
    __syncwarp();
    // split step in place, one (k, 1024 - k) pair per lane and iteration:
    //   X[k] = E + W^k O,  X[1024-k] = conj E - exp(+2 pi i k / 2048) conj O
    for (int k = lane; k <= 512; k += 32) {
      const float2 z = xp[k], zr = xp[(1024 - k) & 1023];
      const float2 zc = cconj(zr);
      const float2 e = make_float2(0.5f * (z.x + zc.x), 0.5f * (z.y + zc.y));
      const float2 d = make_float2(0.5f * (z.x - zc.x), 0.5f * (z.y - zc.y));
      const float2 o = make_float2(d.y, -d.x);  // d / i
      const float2 w = twiddle(tw, k);          // exp(+2 pi i k / 2048)
      const float2 Xk = cadd(e, cmul(o, cconj(w)));
      if (k == 0) {
        xp[0] = make_float2(z.x + z.y, 0.f);     // E[0] + O[0]
        xp[1024] = make_float2(z.x - z.y, 0.f);  // E[0] - O[0]
      } else {
        xp[k] = Xk;
        if (k != 512) xp[1024 - k] = csub(cconj(e), cmul(w, cconj(o)));
      }
    }
    __syncwarp();
    float2* out = spec + (static_cast<size_t>(ch) * Tp + tg) * kBins;
    for (int k = lane; k < kBins; k += 32) out[k] = xp[k];
  }
  __syncthreads();
  // band RMSNorm (bandsplit_norm: v * sqrt(d_b) / max(|v|, 1e-12) * gamma,
  // zero-padded to the band's 64-aligned slot), one warp per band: the sum of
  // squares strided by lane, then the fp16 row two columns a lane
  const float* s0 = reinterpret_cast<const float*>(fsm);
  for (int b = warp; b < nb; b += kFrontWarps) {
    const int d = stab[b * 8 + 0], f0 = stab[b * 8 + 1], koff = stab[b * 8 + 2], kpad = stab[b * 8 + 3],
              goff = stab[b * 8 + 4];
    auto value = [&](int j) {  // x_in[j] of this band: spectrum bin f0 + j/4, channel (j/2)%2, re/im j%2
      return s0[((j >> 1) & 1) * (2 * kXpose) + 2 * (f0 + (j >> 2)) + (j & 1)];
    };
    float ss = 0.f;
    for (int j = lane; j < d; j += 32) {
      const float vv = value(j);
      ss += vv * vv;
    }
    ss = warp_sum(ss);
    const float scale = sqrtf(static_cast<float>(d)) / fmaxf(sqrtf(ss), 1e-12f);
    __half2* row = reinterpret_cast<__half2*>(xn + static_cast<long long>(tg) * xn_cols + koff);
    for (int j = 2 * lane; j < kpad; j += 64) {
      const float a0 = j < d ? __fmul_rn(__fmul_rn(value(j), scale), __ldg(gamma + goff + j)) : 0.f;
      const float a1 = j + 1 < d ? __fmul_rn(__fmul_rn(value(j + 1), scale), __ldg(gamma + goff + j + 1)) : 0.f;
      row[j >> 1] = __floats2half2_rn(a0, a1);
    }
  }
}

cudaError_t stft_front(const float* x, const float* window, const float2* twiddles, float2* spec, const float* gamma,
                       const int* band_tab, __half* xn, int xn_cols, int len, int T, int nb, int chunks,
                       cudaStream_t st) {
  if ((xn_cols & 1) != 0 || nb > kNumBands) return cudaErrorInvalidValue;  // half2 row stores, table size
  if (chunks < 1 || chunks > 65535) return cudaErrorInvalidValue;
  count_launch();
  stft_front_kernel<<<dim3(T, chunks), kFrontWarps * 32, kFrontSmem, st>>>(x, window, twiddles, spec, gamma, band_tab,
                                                                          xn, xn_cols, len, T, nb);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Back end: channel sc = blockIdx.y, output blocks [k0, k0 + kBackBlocks) of
// 512 padded samples, k0 = 2 + blockIdx.x * kBackBlocks.  Frames k0-3 ..
// k0+kBackBlocks-1 (one per warp) are inverse-transformed into shared memory
// (x[n] * w[n], already divided by 2048), then every output sample sums its
// (up to four) frames in frame order and takes the envelope.  12 warps and
// 101 KB of shared memory per CTA: two CTAs per SM.
// ---------------------------------------------------------------------------
constexpr int kBackWarps = 12;
constexpr int kBackBlocks = kBackWarps - 3;
constexpr int kBackSmem = kBackWarps * kXpose * 8 + kTwS * 8;

__global__ void __launch_bounds__(kBackWarps * 32, 2) istft_back_kernel(const float2* __restrict__ c2r,
                                                                     const float* __restrict__ win,
                                                                     const float2* __restrict__ twg,
                                                                     const float* __restrict__ inv_env,
                                                                     float* __restrict__ out, int len, int T) {
  extern __shared__ __align__(16) float2 bsm[];
  float2* tw = bsm + kBackWarps * kXpose;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // channel sc of chunk blockIdx.z: frames chunk*T.. of the chunks' common
  // spectrum planes (T * gridDim.z frames each), samples into out[chunk][sc]
  const int sc = blockIdx.y;
  const int Tp = T * gridDim.z;
  const int k0 = 2 + blockIdx.x * kBackBlocks;
  const int t = k0 - 3 + warp;
  const bool has_frame = t >= 0 && t < T;
  float2* xp = bsm + warp * kXpose;
  int shift = 0;  // the frame's first bin inside the slot (0 or 1: 16-byte aligned loads)
  if (has_frame) {
    // the frame's 1025 bins into its slot with coalesced 16-byte loads: the
    // 16-byte-aligned span holding them (at most 8 bytes before and after)
    const float2* X = c2r + (static_cast<size_t>(sc) * Tp + static_cast<size_t>(blockIdx.z) * T + t) * kBins;
    shift = static_cast<int>((reinterpret_cast<uintptr_t>(X) >> 3) & 1);
    const float4* src = reinterpret_cast<const float4*>(X - shift);
    float4* dst = reinterpret_cast<float4*>(xp);
    for (int i = lane; i < (shift + kBins + 1) / 2; i += 32) cp_async16(dst + i, src + i);
  }
  load_twiddles(tw, twg);
  cp_async_wait_all();
  __syncthreads();
  if (has_frame) {
    const float2* X = xp + shift;
    // Z'[k] = (X[k] + conj X[1024-k]) + i (X[k] - conj X[1024-k]) exp(+2 pi i k / 2048),
    // DC and Nyquist taken as real; lane b builds Z'[32a + b]
    float2 v[32];
#pragma unroll
    for (int a = 0; a < 32; ++a) {
      const int k = 32 * a + lane;
      float2 xk = X[k], xr = X[1024 - k];
      if (k == 0) {
        xk.y = 0.f;
        xr.y = 0.f;
      }
      const float2 xc = cconj(xr);
      const float2 e = cadd(xk, xc);
      const float2 o = cmul(csub(xk, xc), twiddle(tw, k));
      v[a] = make_float2(e.x - o.y, e.y + o.x);  // e + i o
    }
    __syncwarp();  // every lane has read the staged bins before the slot becomes the transpose buffer
    fft1024_warp<true>(v, xp, tw, lane);
    // y[c + 32 d] = 2048 (x[2m] + i x[2m+1]), m = c + 32 d: windowed samples (still
    // times 2048; the overlap-add scales once) into the slot
    float* fr = reinterpret_cast<float*>(xp);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int m = lane + 32 * bitrev5(i);
      const float2 w2 = __ldg(reinterpret_cast<const float2*>(win) + m);
      fr[2 * m] = v[i].x * w2.x;
      fr[2 * m + 1] = v[i].y * w2.y;
    }
  }
  __syncthreads();
  // overlap-add in frame order, envelope, crop to [n_fft/2, n_fft/2 + len)
  const int p_lo = max(k0 * kHop, kNfft / 2), p_hi = min((k0 + kBackBlocks) * kHop, kNfft / 2 + len);
  float* o = out + (static_cast<size_t>(blockIdx.z) * gridDim.y + sc) * len;
  for (int p = p_lo + threadIdx.x; p < p_hi; p += blockDim.x) {
    const int k = p / kHop;
    float sum = 0.f;
#pragma unroll
    for (int q = 3; q >= 0; --q) {
      const int tq = k - q;
      if (tq < 0 || tq >= T) continue;
      const float* fr = reinterpret_cast<const float*>(bsm + (tq - (k0 - 3)) * kXpose);
      sum += fr[p - tq * kHop];
    }
    o[p - kNfft / 2] = sum * ((1.0f / 2048.0f) * __ldg(inv_env + p));
  }
}

cudaError_t istft_back(const float2* c2r, const float* window, const float2* twiddles, const float* inv_env,
                       float* out, int len, int T, int channels, int chunks, cudaStream_t st) {
  static unsigned long long configured = 0;
  cudaError_t e = once_per_device(configured, [] {
    cudaError_t r = cudaFuncSetAttribute(istft_back_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBackSmem);
    // the whole unified L1/shared array as shared memory: two CTAs per SM
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(istft_back_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return r;
  });
  if (e != cudaSuccess) return e;
  const int k_last = (len + kNfft / 2 - 1) / kHop;  // last output block
  const int groups = (k_last - 2 + 1 + kBackBlocks - 1) / kBackBlocks;
  if (chunks < 1 || chunks > 65535) return cudaErrorInvalidValue;
  count_launch();
  istft_back_kernel<<<dim3(groups, channels, chunks), kBackWarps * 32, kBackSmem, st>>>(c2r, window, twiddles,
                                                                                         inv_env, out, len, T);
  return cudaGetLastError();
}

}  // namespace lbrr
