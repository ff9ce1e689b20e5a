// tcgen05 GEMMs of the BS-RoFormer forward.
//
// One kernel template computes D[128 x n] = A[128 x K] * B[n x K]^T per CTA
// tile with fp16 operands (both K-major, 128-byte swizzled, fed by TMA) and an
// fp32 accumulator in TMEM.  Warp roles (192 threads):
//   warp 0      TMA producer (one lane) over a STAGES-deep smem ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: one accumulator row per thread (tcgen05.ld 32x32b),
//               fused per use (bias, RoPE, residual, RMSNorm, GELU, tanh, GLU,
//               complex mask application).
// Every wait is time-bounded; a timeout sets the engine status word.
#include <cstdio>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace lbrr {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kBN = 256;
constexpr int kStages = 2;
constexpr int kABytes = kBM * kBK * 2;          // 16 KB
constexpr int kBBytes = kBN * kBK * 2;          // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;  // 48 KB
constexpr int kBarOff = kStages * kStageBytes;
constexpr int kGemmSmem = kBarOff + 256;
constexpr int kGemmThreads = 192;
constexpr uint32_t kTmemCols = 256;

// ---------------------------------------------------------------------------
// Tile resolvers
// ---------------------------------------------------------------------------
struct DenseTiles {
  int M, n_tiles, kblocks;
  __device__ TileDesc tile(int idx) const {
    TileDesc t;
    const int mt = idx / n_tiles, nt = idx % n_tiles;
    t.a_row = mt * kBM;
    t.a_col = 0;
    t.b_row = nt * kBN;
    t.kblocks = kblocks;
    t.n = kBN;
    t.row0 = mt * kBM;
    t.rows = min(kBM, M - t.row0);
    t.aux = nt * kBN;
    return t;
  }
};
struct TableTiles {
  const TileDesc* table;
  __device__ TileDesc tile(int idx) const { return table[idx]; }
};

// ---------------------------------------------------------------------------
// GELU with the Abramowitz-Stegun 7.1.26 erf approximation (the published
// formula the reference's FF1 epilogue uses, src/main.rs:2928-2935).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float gelu_as(float v) {
  const float a = fabsf(v) * 0.70710678f;
  const float t = __fdividef(1.0f, 1.0f + 0.3275911f * a);
  const float poly = ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
                      0.254829592f) * t;
  const float erfa = copysignf(1.0f - poly * __expf(-a * a), v);
  return 0.5f * v * (1.0f + erfa);
}

__device__ __forceinline__ void store16w(void* dst, const uint32_t (&w)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(w[0], w[1], w[2], w[3]);
  d[1] = make_uint4(w[4], w[5], w[6], w[7]);
  d[2] = make_uint4(w[8], w[9], w[10], w[11]);
  d[3] = make_uint4(w[12], w[13], w[14], w[15]);
}

// ---------------------------------------------------------------------------
// Epilogues
// ---------------------------------------------------------------------------
// QKV: qkv = f16(acc + f16(bias)); Q and K then rotated (interleaved RoPE at
// the token's position: frame t on the time axis, band b on the frequency axis)
// and rounded again -- the rounding points of cuBLASLt f16-out QKV followed by
// rope_q16_inplace / rope_k16 (src/main.rs:6157-6187, :3684-3754).
struct EpiQKV : DenseTiles {
  const float* bias16;  // [1536], values already rounded to fp16
  const float* cos;     // [P][32]
  const float* sin;
  __half* qkv;          // [M][1536]
  int nb, axis;
  __device__ void run(const TileDesc& t, int row, uint32_t tm) const {
    const int r = t.row0 + row;
    const bool valid = row < t.rows;
    const int pos = axis == 0 ? r / nb : r % nb;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tm + c, v);
      tmem_ld_wait(v);
      if (!valid) continue;
      const int col = t.aux + c;
      const bool rot = col < 1024;
      const int pair0 = (col & 63) >> 1;
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float e = f16_round(__uint_as_float(v[2 * j]) + __ldg(bias16 + col + 2 * j));
        float o = f16_round(__uint_as_float(v[2 * j + 1]) + __ldg(bias16 + col + 2 * j + 1));
        if (rot) {
          const float cs = __ldg(cos + pos * 32 + pair0 + j), sn = __ldg(sin + pos * 32 + pair0 + j);
          const float e2 = __fsub_rn(__fmul_rn(e, cs), __fmul_rn(o, sn));
          const float o2 = __fadd_rn(__fmul_rn(o, cs), __fmul_rn(e, sn));
          e = e2;
          o = o2;
        }
        w[j] = pack_f16x2(e, o);
      }
      store16w(qkv + static_cast<size_t>(r) * 1536 + col, w);
    }
  }
};

// Out-projection: attn_out = acc + bias + x (fp32), then the pre-FF RMSNorm of
// that row, (v*scale)*gamma rounded to fp16 (src/main.rs:6219-6234, :490-554).
struct EpiOutNorm : DenseTiles {
  const float* bias;   // [256]
  const float* resid;  // x [M][256]
  const float* gamma;  // [256]
  float* out;          // attn_out [M][256]
  __half* h16;         // [M][256]
  __device__ void run(const TileDesc& t, int row, uint32_t tm) const {
    const int r = t.row0 + row;
    const bool valid = row < t.rows;
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tm + c, v);
      tmem_ld_wait(v);
      if (valid) {
        const float4* rs = reinterpret_cast<const float4*>(resid + static_cast<size_t>(r) * 256 + c);
        float4* os = reinterpret_cast<float4*>(out + static_cast<size_t>(r) * 256 + c);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 x4 = rs[q];
          float4 o;
          o.x = __uint_as_float(v[4 * q + 0]) + __ldg(bias + c + 4 * q + 0) + x4.x;
          o.y = __uint_as_float(v[4 * q + 1]) + __ldg(bias + c + 4 * q + 1) + x4.y;
          o.z = __uint_as_float(v[4 * q + 2]) + __ldg(bias + c + 4 * q + 2) + x4.z;
          o.w = __uint_as_float(v[4 * q + 3]) + __ldg(bias + c + 4 * q + 3) + x4.w;
          os[q] = o;
          ss += o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
          v[4 * q + 0] = __float_as_uint(o.x);
          v[4 * q + 1] = __float_as_uint(o.y);
          v[4 * q + 2] = __float_as_uint(o.z);
          v[4 * q + 3] = __float_as_uint(o.w);
        }
      }
      tmem_st32(tm + c, v);
    }
    tmem_st_wait();
    const float scale = 16.0f / fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tm + c, v);
      tmem_ld_wait(v);
      if (!valid) continue;
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float a = __fmul_rn(__fmul_rn(__uint_as_float(v[2 * j]), scale), __ldg(gamma + c + 2 * j));
        const float b = __fmul_rn(__fmul_rn(__uint_as_float(v[2 * j + 1]), scale), __ldg(gamma + c + 2 * j + 1));
        w[j] = pack_f16x2(a, b);
      }
      store16w(h16 + static_cast<size_t>(r) * 256 + c, w);
    }
  }
};

// FF1: f16(gelu_AS(acc + b1)) (gemm_f16_gelu_a16w epilogue, src/main.rs:2918-2948).
struct EpiGelu : DenseTiles {
  const float* bias;  // [N]
  __half* out;        // [M][ldo]
  int ldo;
  __device__ void run(const TileDesc& t, int row, uint32_t tm) const {
    const int r = t.row0 + row;
    const bool valid = row < t.rows;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tm + c, v);
      tmem_ld_wait(v);
      if (!valid) continue;
      const int col = t.aux + c;
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float a = gelu_as(__uint_as_float(v[2 * j]) + __ldg(bias + col + 2 * j));
        const float b = gelu_as(__uint_as_float(v[2 * j + 1]) + __ldg(bias + col + 2 * j + 1));
        w[j] = pack_f16x2(a, b);
      }
      store16w(out + static_cast<size_t>(r) * ldo + col, w);
    }
  }
};

// FF2: x = acc + b2 + attn_out (fp32) (src/main.rs:6255-6259).
struct EpiResid : DenseTiles {
  const float* bias;
  const float* resid;
  float* out;
  int ldo;
  __device__ void run(const TileDesc& t, int row, uint32_t tm) const {
    const int r = t.row0 + row;
    const bool valid = row < t.rows;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tm + c, v);
      tmem_ld_wait(v);
      if (!valid) continue;
      const int col = t.aux + c;
      const float4* rs = reinterpret_cast<const float4*>(resid + static_cast<size_t>(r) * ldo + col);
      float4* os = reinterpret_cast<float4*>(out + static_cast<size_t>(r) * ldo + col);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 x4 = rs[q];
        float4 o;
        o.x = __uint_as_float(v[4 * q + 0]) + __ldg(bias + col + 4 * q + 0) + x4.x;
        o.y = __uint_as_float(v[4 * q + 1]) + __ldg(bias + col + 4 * q + 1) + x4.y;
        o.z = __uint_as_float(v[4 * q + 2]) + __ldg(bias + col + 4 * q + 2) + x4.z;
        o.w = __uint_as_float(v[4 * q + 3]) + __ldg(bias + col + 4 * q + 3) + x4.w;
        os[q] = o;
      }
    }
  }
};

// Band split: x[(t*nb + band)][n] = acc + bias[band][n]  (bandsplit_gemm_f16,
// src/main.rs:4686-4698).  Tile aux = band.
struct EpiBand : TableTiles {
  const float* bias;  // [nb][256]
  float* x;           // [T*nb][256]
  int nb;
  __device__ void run(const TileDesc& t, int row, uint32_t tm) const {
    const int r = t.row0 + row;
    const bool valid = row < t.rows;
    const int band = t.aux;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tm + c, v);
      tmem_ld_wait(v);
      if (!valid) continue;
      float4* os = reinterpret_cast<float4*>(x + (static_cast<size_t>(r) * nb + band) * 256 + c);
      const float* bb = bias + band * 256 + c;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 o;
        o.x = __uint_as_float(v[4 * q + 0]) + __ldg(bb + 4 * q + 0);
        o.y = __uint_as_float(v[4 * q + 1]) + __ldg(bb + 4 * q + 1);
        o.z = __uint_as_float(v[4 * q + 2]) + __ldg(bb + 4 * q + 2);
        o.w = __uint_as_float(v[4 * q + 3]) + __ldg(bb + 4 * q + 3);
        os[q] = o;
      }
    }
  }
};

// Mask estimator layer 1: hidden = f16(tanh(acc + b1)) (mask_gemm1_f16,
// src/main.rs:4816-4842).  Tile aux = group*4 + n-tile, group = stem*nb + band.
struct EpiTanh : TableTiles {
  const float* bias;  // [groups][1024]
  __half* hidden;     // [groups*T][1024]
  int T;
  __device__ void run(const TileDesc& t, int row, uint32_t tm) const {
    const int r = t.row0 + row;
    const bool valid = row < t.rows;
    const int group = t.aux >> 2, n0 = (t.aux & 3) * kBN;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tm + c, v);
      tmem_ld_wait(v);
      if (!valid) continue;
      const float* bb = bias + static_cast<size_t>(group) * 1024 + n0 + c;
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float a = tanhf(__uint_as_float(v[2 * j]) + __ldg(bb + 2 * j));
        const float b = tanhf(__uint_as_float(v[2 * j + 1]) + __ldg(bb + 2 * j + 1));
        w[j] = pack_f16x2(a, b);
      }
      store16w(hidden + (static_cast<size_t>(group) * T + r) * 1024 + n0 + c, w);
    }
  }
};

// Mask estimator layer 2 + GLU + mask application.  W2 rows are stored
// interleaved per band (a_0, g_0, a_1, g_1, ...), so every 8 accumulator
// columns are one frequency bin: (re, im) masks of both channels.  The
// epilogue writes the masked spectrum straight into the C2R input
// (glu_scatter + mask_apply, src/main.rs:4984-4997, :1776-1817).
// Tile aux = (stem << 16) | (band << 8) | n-tile.
struct EpiMask : TableTiles {
  const float* bias2;   // [stems][n2tot] permuted like W2
  const int* band_f0;   // [nb]
  const int* band_d;    // [nb] d_b
  const int* band_o2;   // [nb] row offset of the band inside one stem's permuted W2
  const float2* spec;   // [2][T][1025]
  float2* out;          // [stems*2][T][1025]
  int T, n2tot;
  __device__ void run(const TileDesc& t, int row, uint32_t tm) const {
    const int r = t.row0 + row;
    const bool valid = row < t.rows;
    const int stem = t.aux >> 16, band = (t.aux >> 8) & 255, n0 = (t.aux & 255) * kBN;
    const int d_b = band_d[band], f0 = band_f0[band];
    const float* bb = bias2 + static_cast<size_t>(stem) * n2tot + band_o2[band] + n0;
#pragma unroll 1
    for (int c = 0; c < t.n; c += 32) {
      uint32_t v[32];
      tmem_ld32(tm + c, v);
      tmem_ld_wait(v);
      if (!valid) continue;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int lc = c + q * 8;      // column inside this tile
        const int d0 = (n0 + lc) >> 1;  // first GLU index of this bin = fi*4
        if (lc < t.n && d0 < d_b) {
          float m[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float a = __uint_as_float(v[q * 8 + 2 * k]) + __ldg(bb + lc + 2 * k);
            const float g = __uint_as_float(v[q * 8 + 2 * k + 1]) + __ldg(bb + lc + 2 * k + 1);
            m[k] = __fdividef(a, 1.0f + __expf(-g));
          }
          const int f = f0 + (d0 >> 2);
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            const float2 s = spec[(static_cast<size_t>(ch) * T + r) * 1025 + f];
            const float mr = m[2 * ch], mi = m[2 * ch + 1];
            float2 o;
            o.x = s.x * mr - s.y * mi;
            // A real signal's DC and Nyquist bins are real: torch.istft drops
            // their imaginary parts, and cuFFT's C2R is only defined for such
            // Hermitian input, so the masked spectrum keeps them real.
            o.y = (f == 0 || f == 1024) ? 0.f : s.x * mi + s.y * mr;
            out[(static_cast<size_t>(stem * 2 + ch) * T + r) * 1025 + f] = o;
          }
        }
      }
    }
  }
};

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <class Epi>
__global__ void __launch_bounds__(kGemmThreads, 2)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Epi epi,
                   int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if ((smem_u32(smem) & 1023u) != 0) {  // uniform across the CTA: nothing allocated yet
    if (threadIdx.x == 0) report_status(status, kDevSmemMisaligned);
    return;
  }
  const TileDesc t = epi.tile(blockIdx.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < t.kblocks; ++kb) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, status)) break;
        uint8_t* sa = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(sa, &tmA, &full[s], t.a_col + kb * kBK, t.a_row);
        tma_load_2d(sa + kABytes, &tmB, &full[s], kb * kBK, t.b_row);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(kBM, t.n);
      for (int kb = 0; kb < t.kblocks; ++kb) {
        const int s = kb % kStages;
        const uint32_t ph = (kb / kStages) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * kStageBytes);
        const uint32_t sb = sa + kABytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          mma_f16_ss(tmem, sdesc_sw128(sa + k * 32, 1024, 16), sdesc_sw128(sb + k * 32, 1024, 16), idesc,
                     (kb | k) != 0 ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      mma_commit(acc_full);
    }
  } else {
    const int q = warp & 3;  // the TMEM lane quadrant this warp may access
    const bool ok = mbar_wait(acc_full, 0, abort_flag, status);
    tc_fence_after();
    if (ok && !*abort_flag) epi.run(t, q * 32 + lane, tmem + (static_cast<uint32_t>(q * 32) << 16));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <class Epi>
static cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const Epi& epi, int tiles, int* status,
                               cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  if (tiles <= 0) return cudaSuccess;
  gemm_tc_kernel<Epi><<<tiles, kGemmThreads, kGemmSmem, st>>>(a, b, epi, status);
  return cudaGetLastError();
}

static int dense_tiles(int M, int N) { return ((M + kBM - 1) / kBM) * (N / kBN); }

cudaError_t gemm_qkv(const __half* h16, const __half* w, const float* bias16, const float* cos, const float* sin,
                     __half* qkv, int M, int nb, int axis, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  cudaError_t e = make_map_2d(&ta, h16, 256, M, 256 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w, 256, 1536, 256 * 2, kBK, kBN);
  if (e != cudaSuccess) return e;
  EpiQKV ep;
  ep.M = M;
  ep.n_tiles = 1536 / kBN;
  ep.kblocks = 256 / kBK;
  ep.bias16 = bias16;
  ep.cos = cos;
  ep.sin = sin;
  ep.qkv = qkv;
  ep.nb = nb;
  ep.axis = axis;
  return launch_gemm(ta, tb, ep, dense_tiles(M, 1536), status, st);
}

cudaError_t gemm_outproj_norm(const __half* scaled16, const __half* w, const float* bias, const float* resid,
                              const float* gamma, float* out, __half* h16, int M, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  cudaError_t e = make_map_2d(&ta, scaled16, 512, M, 512 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w, 512, 256, 512 * 2, kBK, kBN);
  if (e != cudaSuccess) return e;
  EpiOutNorm ep;
  ep.M = M;
  ep.n_tiles = 1;
  ep.kblocks = 512 / kBK;
  ep.bias = bias;
  ep.resid = resid;
  ep.gamma = gamma;
  ep.out = out;
  ep.h16 = h16;
  return launch_gemm(ta, tb, ep, dense_tiles(M, 256), status, st);
}

cudaError_t gemm_ff1_gelu(const __half* h16, const __half* w1, const float* b1, __half* ff1, int M, int* status,
                          cudaStream_t st) {
  CUtensorMap ta, tb;
  cudaError_t e = make_map_2d(&ta, h16, 256, M, 256 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w1, 256, 1024, 256 * 2, kBK, kBN);
  if (e != cudaSuccess) return e;
  EpiGelu ep;
  ep.M = M;
  ep.n_tiles = 1024 / kBN;
  ep.kblocks = 256 / kBK;
  ep.bias = b1;
  ep.out = ff1;
  ep.ldo = 1024;
  return launch_gemm(ta, tb, ep, dense_tiles(M, 1024), status, st);
}

cudaError_t gemm_ff2_resid(const __half* ff1, const __half* w2, const float* b2, const float* resid, float* x, int M,
                           int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  cudaError_t e = make_map_2d(&ta, ff1, 1024, M, 1024 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w2, 1024, 256, 1024 * 2, kBK, kBN);
  if (e != cudaSuccess) return e;
  EpiResid ep;
  ep.M = M;
  ep.n_tiles = 1;
  ep.kblocks = 1024 / kBK;
  ep.bias = b2;
  ep.resid = resid;
  ep.out = x;
  ep.ldo = 256;
  return launch_gemm(ta, tb, ep, dense_tiles(M, 256), status, st);
}

cudaError_t gemm_bandsplit(const __half* xn, int xn_cols, const __half* wband, int wband_cols, const float* bias,
                           float* x, int T, int nb, const TileDesc* tiles, int n_tiles, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  cudaError_t e = make_map_2d(&ta, xn, xn_cols, T, static_cast<uint64_t>(xn_cols) * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, wband, wband_cols, static_cast<uint64_t>(nb) * 256,
                                        static_cast<uint64_t>(wband_cols) * 2, kBK, kBN);
  if (e != cudaSuccess) return e;
  EpiBand ep;
  ep.table = tiles;
  ep.bias = bias;
  ep.x = x;
  ep.nb = nb;
  return launch_gemm(ta, tb, ep, n_tiles, status, st);
}

cudaError_t gemm_mask1(const __half* xb16, const __half* w1, const float* b1, __half* hidden, int T, int groups,
                       const TileDesc* tiles, int n_tiles, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  const int nb_rows = groups;  // xb16 holds nb bands; w1 holds groups = stems*nb blocks
  (void)nb_rows;
  cudaError_t e = make_map_2d(&ta, xb16, 256, static_cast<uint64_t>(T) * kNumBands, 256 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w1, 256, static_cast<uint64_t>(groups) * 1024, 256 * 2, kBK, kBN);
  if (e != cudaSuccess) return e;
  EpiTanh ep;
  ep.table = tiles;
  ep.bias = b1;
  ep.hidden = hidden;
  ep.T = T;
  return launch_gemm(ta, tb, ep, n_tiles, status, st);
}

cudaError_t gemm_mask2(const __half* hidden, const __half* w2, const float* b2, const int* band_f0,
                       const int* band_d, const int* band_o2, const float2* spec, float2* c2r, int T, int stems,
                       int n2tot, const TileDesc* tiles, int n_tiles, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  cudaError_t e = make_map_2d(&ta, hidden, 1024, static_cast<uint64_t>(T) * kNumBands * stems, 1024 * 2, kBK, kBM);
  if (e == cudaSuccess)
    e = make_map_2d(&tb, w2, 1024, static_cast<uint64_t>(stems) * n2tot, 1024 * 2, kBK, kBN);
  if (e != cudaSuccess) return e;
  EpiMask ep;
  ep.table = tiles;
  ep.bias2 = b2;
  ep.band_f0 = band_f0;
  ep.band_d = band_d;
  ep.band_o2 = band_o2;
  ep.spec = spec;
  ep.out = c2r;
  ep.T = T;
  ep.n2tot = n2tot;
  return launch_gemm(ta, tb, ep, n_tiles, status, st);
}

}  // namespace lbrr
