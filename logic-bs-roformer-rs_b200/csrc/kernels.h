// Internal launcher interface between the CUDA kernels and the engine / C ABI.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Sets the thread-local message returned by lbrr_last_error and returns code
// (defined in engine.cu; used by the other translation units).
extern "C" int lbrr_set_error_for_host(int code, const char* msg);

namespace lbrr {

// Kernel launches issued by this library from the calling thread; the engine
// takes the difference around one forward to report its launches per chunk.
extern thread_local long long t_kernel_launches;
inline void count_launch() { ++t_kernel_launches; }

constexpr int kNumBands = 62;
constexpr int kDim = 256;
constexpr int kHeads = 8;
constexpr int kDimHead = 64;
constexpr int kFF = 1024;
constexpr int kStems = 6;
constexpr int kNfft = 2048;
constexpr int kHop = 512;
constexpr int kBins = 1025;
constexpr int kDepth = 12;

// One GEMM CTA tile (A rows [a_row, a_row+128), A columns from a_col, B rows
// [b_row, b_row+n), kblocks K-blocks of 64, epilogue rows row0.. with `rows`
// valid, `aux` epilogue-specific).
struct TileDesc {
  int a_row, a_col, b_row, kblocks;
  int n, row0, rows, aux;
};

// RMSNorm fused into an N = 256 fp32-row GEMM epilogue (out-projection, FF2,
// band split): kind 0 none, 1 pre-FF norm -> h16, 2 pre-attention norm -> h16
// plus the 8 head gates, 3 final norm -> band-major xb16.
struct RowNorm {
  int kind = 0;
  const float* gamma = nullptr;
  const float* gate_w = nullptr;
  const float* gate_b = nullptr;
  __half* h16 = nullptr;
  float* gates = nullptr;
  __half* xb16 = nullptr;
  int T = 0, nb = 0;
};

// TMA tensor maps (zero OOB fill).  Defaults: fp16 elements, 128-byte swizzle.
enum class MapElem { F16, F32 };
cudaError_t make_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                        uint32_t box_inner, uint32_t box_outer, MapElem elem = MapElem::F16,
                        CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B);
cudaError_t make_map_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
                        uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2, MapElem elem = MapElem::F16,
                        CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B);
// fp16, 128-byte swizzle
cudaError_t make_map_4d(CUtensorMap* map, const void* base, const uint64_t dims[4], const uint64_t stride_bytes[3],
                        const uint32_t box[4]);

// ---- GEMMs (gemm.cu) -------------------------------------------------------
cudaError_t gemm_qkv(const __half* h16, const __half* w, const float* bias16, const float* cos, const float* sin,
                     __half* qkv, int M, int nb, int axis, int* status, cudaStream_t st);
cudaError_t gemm_outproj_norm(const __half* scaled16, const __half* w, const float* bias, const float* resid,
                              const float* gamma, float* out, __half* h16, int M, int* status, cudaStream_t st);
cudaError_t gemm_ff1_gelu(const __half* h16, const __half* w1, const float* b1, __half* ff1, int M, int* status,
                          cudaStream_t st);
cudaError_t gemm_ff2_resid(const __half* ff1, const __half* w2, const float* b2, const float* resid, float* x, int M,
                           const RowNorm& next, int* status, cudaStream_t st);
// FF1 -> GELU -> FF2 + residual in one kernel, without the [M][1024] intermediate
cudaError_t gemm_ff_fused(const __half* h16, const __half* w1, const float* b1, const __half* w2, const float* b2,
                          const float* resid, float* x, int M, const RowNorm& next, int* status, cudaStream_t st);
cudaError_t gemm_bandsplit(const __half* xn, int xn_cols, const __half* wband, int wband_cols, const float* bias,
                           float* x, int T, int nb, const TileDesc* tiles, int n_tiles, const RowNorm& first,
                           int* status, cudaStream_t st);
cudaError_t gemm_mask1(const __half* xb16, const __half* w1, const float* b1, __half* hidden, int T, int groups,
                       const TileDesc* tiles, int n_tiles, int* status, cudaStream_t st);
cudaError_t gemm_mask2(const __half* hidden, const __half* w2, const float* b2, const int* band_f0,
                       const int* band_d, const int* band_o2, const float2* spec, float2* c2r, int T, int stems,
                       int n2tot, const TileDesc* tiles, int n_tiles, bool keep_dc_imag, int* status,
                       cudaStream_t st);

// ---- attention (attention.cu) ----------------------------------------------
// chunks: forwards batched along the frame axis (chunk c at frames c*T..);
// the time axis keeps their frames apart, the frequency axis sees T * chunks frames
cudaError_t attention_fwd(const __half* qkv, const float* gates, __half* out, int T, int nb, int axis, int chunks,
                          int* status, cudaStream_t st);

// ---- bandwidth kernels (spectral.cu) ---------------------------------------
cudaError_t stft_frames(const float* x_interleaved, const float* window, float* frames, int len, int T,
                        cudaStream_t st);
cudaError_t band_norm(const float2* spec, const float* gamma, const int* band_tab, __half* xn, int xn_cols, int T,
                      int nb, cudaStream_t st);
cudaError_t norm_gates(const float* x, const float* gamma, const float* gate_w, const float* gate_b, __half* h16,
                       float* gates, int rows, cudaStream_t st);
cudaError_t istft_ola(const float* pcm, const float* window, const float* inv_env, float* out, int len, int T,
                      int channels, cudaStream_t st);

// ---- in-house FFT, fused with its neighbours (fft.cu) ------------------------
// twiddles: [2048] exp(+2 pi i k / 2048) as float2
// chunks: x holds `chunks` interleaved inputs of len samples one after another;
// chunk c's frames are rows c*T.. of the spectrum planes ([2][T*chunks][1025])
// and of xn
cudaError_t stft_front(const float* x_interleaved, const float* window, const float2* twiddles, float2* spec,
                       const float* gamma, const int* band_tab, __half* xn, int xn_cols, int len, int T, int nb,
                       int chunks, cudaStream_t st);
// c2r planes [channels][T*chunks][1025] -> out [chunks][channels][len]
cudaError_t istft_back(const float2* c2r, const float* window, const float2* twiddles, const float* inv_env,
                       float* out, int len, int T, int channels, int chunks, cudaStream_t st);

// cudaFuncSetAttribute (the dynamic shared-memory opt-in) acts on the current
// device only.  Runs `setup` once per device (devices 0..63, bit d of `done`)
// before the first launch there; a failed setup is retried on the next call.
template <class Setup>
inline cudaError_t once_per_device(unsigned long long& done, Setup setup) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (bit && (__atomic_load_n(&done, __ATOMIC_ACQUIRE) & bit)) return cudaSuccess;
  e = setup();
  if (e == cudaSuccess && bit) __atomic_fetch_or(&done, bit, __ATOMIC_RELEASE);
  return e;
}

}  // namespace lbrr
