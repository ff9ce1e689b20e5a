// Bandwidth-bound kernels of the chunk forward: STFT framing, band RMSNorm
// (fused with the spectrum reorder), the stand-alone pre-attention RMSNorm +
// head gates (the forward fuses it into GEMM epilogues) and the single-chunk
// ISTFT overlap-add.  Also the TMA tensor-map helpers.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace lbrr {

// ---------------------------------------------------------------------------
// Tensor maps
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static CUtensorMapDataType map_dtype(MapElem e) {
  return e == MapElem::F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

cudaError_t make_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                        uint32_t box_inner, uint32_t box_outer, MapElem elem, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (row_bytes & 15u)) return cudaErrorMisalignedAddress;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, map_dtype(elem), 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_map_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
                        uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2, MapElem elem,
                        CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (s1_bytes & 15u) || (s2_bytes & 15u))
    return cudaErrorMisalignedAddress;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, map_dtype(elem), 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_map_4d(CUtensorMap* map, const void* base, const uint64_t dims[4], const uint64_t stride_bytes[3],
                        const uint32_t box[4]) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (reinterpret_cast<uintptr_t>(base) & 15u) return cudaErrorMisalignedAddress;
  cuuint64_t d[4], s[3];
  cuuint32_t b[4], estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < 4; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
  }
  for (int i = 0; i < 3; ++i) {
    if (stride_bytes[i] & 15u) return cudaErrorMisalignedAddress;
    s[i] = stride_bytes[i];
  }
  CUresult r = fn(map, map_dtype(MapElem::F16), 4, const_cast<void*>(base), d, s, b, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// STFT framing: frames[ch][t][j] = x[src][ch] * window[j] with torch/numpy
// reflect padding of n_fft/2 (frame_hann_reflect, src/main.rs:396-429).
// One thread writes 4 consecutive frame samples.
// ---------------------------------------------------------------------------
__global__ void frames_kernel(const float* __restrict__ x, const float* __restrict__ win, float* __restrict__ out,
                              int len, int T) {
  const long long i4 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total4 = 2ll * T * (kNfft / 4);
  if (i4 >= total4) return;
  const int j0 = static_cast<int>(i4 % (kNfft / 4)) * 4;
  const long long ct = i4 / (kNfft / 4);
  const int t = static_cast<int>(ct % T);
  const int ch = static_cast<int>(ct / T);
  const int pad = kNfft / 2;
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int g = t * kHop + j0 + k;
    const int src = g < pad ? pad - g : (g >= len + pad ? 2 * len + pad - 2 - g : g - pad);
    v[k] = __ldg(x + 2ll * src + ch) * __ldg(win + j0 + k);
  }
  reinterpret_cast<float4*>(out)[i4] = make_float4(v[0], v[1], v[2], v[3]);
}

cudaError_t stft_frames(const float* x, const float* window, float* frames, int len, int T, cudaStream_t st) {
  const long long total4 = 2ll * T * (kNfft / 4);
  const int threads = 256;
  count_launch();
  frames_kernel<<<static_cast<unsigned>((total4 + threads - 1) / threads), threads, 0, st>>>(x, window, frames, len,
                                                                                              T);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Band RMSNorm straight from the spectrum: for band b and frame t the input row
// is x_in[t][offs_b + j] = spec[ch][t][f0_b + j/4].(re|im) with ch = (j/2)%2
// (spec_reorder, src/main.rs:1649-1677); it is normalised as
// (v * sqrt(d_b)/max(|v|,1e-12)) * gamma (bandsplit_norm, :792-828) and stored
// fp16 at xn[t][koff_b + j], zero-padded to kpad_b (a multiple of 64) so every
// band is an independent zero-padded K range of the grouped GEMM.
// band_tab[b*8 + {0..4}] = {d_b, f0_b, koff_b, kpad_b, goff_b}.  One warp per (t, b).
// ---------------------------------------------------------------------------
__global__ void band_norm_kernel(const float2* __restrict__ spec, const float* __restrict__ gamma,
                                 const int* __restrict__ tab, __half* __restrict__ xn, int xn_cols, int T, int nb) {
  const long long task = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (task >= static_cast<long long>(T) * nb) return;
  const int t = static_cast<int>(task / nb), b = static_cast<int>(task % nb);
  const int d = tab[b * 8 + 0], f0 = tab[b * 8 + 1], koff = tab[b * 8 + 2], kpad = tab[b * 8 + 3],
            goff = tab[b * 8 + 4];
  float vals[17];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 17; ++i) {
    const int j = lane + 32 * i;
    float v = 0.f;
    if (j < d) {
      const int f = f0 + (j >> 2), ch = (j >> 1) & 1;
      const float2 s = __ldg(spec + (static_cast<long long>(ch) * T + t) * kBins + f);
      v = (j & 1) ? s.y : s.x;
    }
    vals[i] = v;
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float scale = sqrtf(static_cast<float>(d)) / fmaxf(sqrtf(ss), 1e-12f);
  __half* row = xn + static_cast<long long>(t) * xn_cols + koff;
#pragma unroll
  for (int i = 0; i < 17; ++i) {
    const int j = lane + 32 * i;
    if (j < kpad) {
      const float v = j < d ? __fmul_rn(__fmul_rn(vals[i], scale), __ldg(gamma + goff + j)) : 0.f;
      row[j] = __float2half_rn(v);
    }
  }
  for (int j = lane + 32 * 17; j < kpad; j += 32) row[j] = __float2half_rn(0.f);
}

cudaError_t band_norm(const float2* spec, const float* gamma, const int* band_tab, __half* xn, int xn_cols, int T,
                      int nb, cudaStream_t st) {
  const long long threads_total = static_cast<long long>(T) * nb * 32;
  count_launch();
  band_norm_kernel<<<static_cast<unsigned>((threads_total + 255) / 256), 256, 0, st>>>(spec, gamma, band_tab, xn,
                                                                                        xn_cols, T, nb);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Pre-attention RMSNorm + 8 head gates (rmsnorm_gates_h16, src/main.rs:616-703):
// h = v * (scale * gamma) in fp32, stored fp16; gates = h . Wg + bg from the
// fp32 h.  One warp per row; lane owns columns [8*lane, 8*lane+8).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) norm_gates_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                         const float* __restrict__ gw, const float* __restrict__ gb,
                                                         __half* __restrict__ h16, float* __restrict__ gates,
                                                         int rows) {
  __shared__ float sw[8 * 256];
  __shared__ float sg[256];
  for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) sw[i] = gw[i];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) sg[i] = gamma[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * 256 + lane * 8);
  const float4 a = xr[0], b = xr[1];
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) ss += v[k] * v[k];
  ss = warp_sum(ss);
  const float scale = 16.0f / fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(v[k], __fmul_rn(scale, sg[lane * 8 + k]));
  uint4 packed = make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]),
                            pack_f16x2(v[6], v[7]));
  reinterpret_cast<uint4*>(h16 + row * 256)[lane] = packed;
  float my_gate = 0.f;
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) dot += v[k] * sw[g * 256 + lane * 8 + k];
    dot = warp_sum(dot);
    if (lane == g) my_gate = dot + __ldg(gb + g);
  }
  if (lane < 8) gates[row * 8 + lane] = my_gate;
}

cudaError_t norm_gates(const float* x, const float* gamma, const float* gate_w, const float* gate_b, __half* h16,
                       float* gates, int rows, cudaStream_t st) {
  const int warps = 16;
  count_launch();
  norm_gates_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, st>>>(x, gamma, gate_w, gate_b, h16, gates, rows);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// ISTFT overlap-add, gather form: out[sc][i] = sum_t pcm[sc][t][p - 512t] *
// win[p - 512t] * (1/2048) * inv_env[p], p = i + 1024 (istft_ola,
// src/main.rs:5024-5039).  pcm is cuFFT's unnormalised C2R output.
// ---------------------------------------------------------------------------
__global__ void istft_kernel(const float* __restrict__ pcm, const float* __restrict__ win,
                             const float* __restrict__ inv, float* __restrict__ out, int len, int T, int channels) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(channels) * len) return;
  const int sc = static_cast<int>(i / len);
  const int pos = static_cast<int>(i % len) + kNfft / 2;
  const int first = (max(pos - (kNfft - 1), 0) + kHop - 1) / kHop;
  const int last = min(pos / kHop, T - 1);
  float sum = 0.f;
  for (int t = first; t <= last; ++t) {
    const int n = pos - t * kHop;
    sum += __ldg(pcm + (static_cast<long long>(sc) * T + t) * kNfft + n) * __ldg(win + n);
  }
  out[i] = sum * ((1.0f / 2048.0f) * __ldg(inv + pos));
}

cudaError_t istft_ola(const float* pcm, const float* window, const float* inv_env, float* out, int len, int T,
                      int channels, cudaStream_t st) {
  const long long n = static_cast<long long>(channels) * len;
  count_launch();
  istft_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(pcm, window, inv_env, out, len, T, channels);
  return cudaGetLastError();
}

}  // namespace lbrr
