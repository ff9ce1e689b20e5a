// tcgen05 GEMMs of the BS-RoFormer forward.
//
// One persistent kernel template computes, for every 128 x n output tile,
// D = A[128 x K] * B[n x K]^T with fp16 operands (both K-major, 128-byte
// swizzled, fed by TMA) and an fp32 accumulator in TMEM.  One CTA per SM
// walks the tile list with a static stride.  Warp roles (64 + 32 * kEpiWarps threads):
//   warp 0      TMA producer (one lane): 3-stage ring of 48 KB (A 16 KB + B 32 KB)
//   warp 1      TMEM allocator (all 512 columns) + single-thread tcgen05.mma
//               issuer into two 256-column accumulators (double buffer)
//   warps 2..9  epilogue: two warps per TMEM lane quadrant, each owning 128 of
//               the 256 columns, one accumulator row per thread.  Each 32 x 32
//               output block is written into a 4 KB per-warp staging buffer in
//               the TMA swizzle layout and leaves through a TMA tensor store, so
//               the LSU carries neither the transpose read-back nor the global
//               stores.  The epilogue of tile i overlaps the MMAs of tile i+1.
// Epilogues fuse bias, RoPE, residual, RMSNorm (+ head gates of the next
// transformer step), GELU, tanh, GLU and the complex mask application.
// Every wait is time-bounded; a timeout sets the engine status word.
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace lbrr {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kBN = 256;
constexpr int kStages = 3;
constexpr int kABytes = kBM * kBK * 2;          // 16 KB
constexpr int kBBytes = kBN * kBK * 2;          // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;  // 48 KB
constexpr int kEpiWarps = 8;
constexpr int kParts = kEpiWarps / 4;           // epilogue warps per TMEM lane quadrant
constexpr int kPartCols = kBN / kParts;         // accumulator columns per epilogue warp
constexpr int kStageWords = 32 * 32;            // per-warp staging buffer (4 KB)
constexpr int kStagingOff = kStages * kStageBytes;
// per-CTA copy of the epilogue's constant vectors (bias, gamma, gate weights,
// RoPE tables), loaded once when the kernel starts; read with shared-memory
// broadcasts instead of per-block global loads
constexpr int kConstFloats = 6144;
constexpr int kConstOff = kStagingOff + kEpiWarps * kStageWords * 4;
constexpr int kBarOff = kConstOff + kConstFloats * 4;
constexpr int kGemmSmem = kBarOff + 256;
constexpr int kGemmThreads = 64 + kEpiWarps * 32;
constexpr uint32_t kTmemCols = 512;
static_assert(kGemmSmem <= 232448, "exceeds the 227 KB per-CTA shared memory limit");

// ---------------------------------------------------------------------------
// Division by a launch constant: q = umulhi(x, m), m = ceil(2^32 / d), which is
// exact for x * d < 2^32 (|error| of x*m/2^32 - x/d stays below 1/d); the host
// leaves m = 0, meaning a plain division, when that bound does not hold.
// ---------------------------------------------------------------------------
struct FastDiv {
  uint32_t d = 1, m = 0;
  __device__ __forceinline__ int div(int x) const {
    const uint32_t u = static_cast<uint32_t>(x);
    return static_cast<int>(m ? __umulhi(u, m) : (d == 1 ? u : u / d));
  }
};
static inline FastDiv make_fastdiv(uint32_t d, uint64_t x_max) {
  FastDiv f;
  f.d = d;
  if (d > 1 && x_max * d < (1ull << 32)) f.m = static_cast<uint32_t>(((1ull << 32) + d - 1) / d);
  return f;
}

// ---------------------------------------------------------------------------
// Tile resolvers
// ---------------------------------------------------------------------------
struct EpiCtx;
struct DenseTiles {
  int M, n_tiles, kblocks;
  FastDiv ntd;  // division by n_tiles
  __device__ void load_consts(float*, int, int) const {}
  __device__ void prefetch(const TileDesc&, EpiCtx&) const {}
  __device__ TileDesc tile(int idx) const {
    TileDesc t;
    const int mt = ntd.div(idx), nt = idx - mt * n_tiles;
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
  __device__ void load_consts(float*, int, int) const {}
  __device__ void prefetch(const TileDesc&, EpiCtx&) const {}
  __device__ TileDesc tile(int idx) const { return table[idx]; }
};

// ---------------------------------------------------------------------------
// Per-warp staging buffer.  fp16 blocks (32 x 32 halves = 2 KB) alternate
// between the two 1024-aligned halves so a TMA store can drain one while the
// next block is written; fp32 blocks (4 KB) use the whole buffer.  Rows are
// stored with the TMA swizzle of their width (64 B rows: 16-byte vector v of
// row r at v ^ ((r >> 1) & 3); 128 B rows: v ^ (r & 7)), which also keeps the
// per-lane row writes free of bank conflicts.
// ---------------------------------------------------------------------------
struct Stager {
  uint32_t* base;
  int lane;
  int phase;
  bool last_f32;
  __device__ uint32_t* f16_buf() {
    if (lane == 0) {
      if (last_f32)
        tma_store_wait_read<0>();
      else
        tma_store_wait_read<1>();
    }
    __syncwarp();
    last_f32 = false;
    return base + ((phase++) & 1) * 512;
  }
  __device__ uint32_t* f32_buf() {
    if (lane == 0) tma_store_wait_read<0>();
    __syncwarp();
    last_f32 = true;
    return base;
  }
  __device__ void drain() {
    if (lane == 0) tma_store_wait_read<0>();
    __syncwarp();
  }
};

// Per-thread view handed to the epilogues.
struct EpiCtx {
  int lane, q, part;
  int c0;           // first accumulator column of this warp (part * kPartCols)
  int row;          // accumulator row (TMEM lane) 0..127
  uint32_t tm;      // TMEM address of this warp's lanes in the current accumulator
  Stager st;        // this warp's staging buffer
  uint32_t* quad;   // staging buffers of the kParts warps sharing these rows (part-major)
  int bar_id;       // named barrier shared by those warps
  float* consts;    // the epilogue's constants in shared memory (load_consts)
  int id;           // epilogue warp index 0..kEpiWarps-1 (part * 4 + q)
  int next_tile;    // index of this CTA's next tile, or -1
  float4 pre;       // epilogue data for the next tile, fetched during this one (Epi::prefetch)
};

// Write this lane's row (W = 16 words: 32 fp16, W = 32: 32 fp32) into buf.
template <int W>
__device__ __forceinline__ void stage_row(uint32_t* buf, const uint32_t* w, int lane) {
  constexpr int V = W / 4;
  const int sw = V == 8 ? (lane & 7) : ((lane >> 1) & 3);
#pragma unroll
  for (int k = 0; k < V; ++k)
    *reinterpret_cast<uint4*>(buf + lane * W + ((k ^ sw) << 2)) =
        make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
}
// Publish the staged block to the async proxy; lane 0 then issues the store.
__device__ __forceinline__ bool stage_publish(int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  return lane == 0;
}
__device__ __forceinline__ void store_2d(const CUtensorMap* m, const uint32_t* buf, int x, int y, int lane) {
  if (stage_publish(lane)) {
    tma_store_2d(m, buf, x, y);
    tma_store_commit();
  }
}
__device__ __forceinline__ void store_3d(const CUtensorMap* m, const uint32_t* buf, int x, int y, int z, int lane) {
  if (stage_publish(lane)) {
    tma_store_3d(m, buf, x, y, z);
    tma_store_commit();
  }
}
// Manual store of a staged fp16 block (rows with scattered destinations).
template <class RowPtr>
__device__ __forceinline__ void store_rows16_manual(const uint32_t* buf, int lane, RowPtr row_ptr) {
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + lane / 4, v = lane % 4;
    const uint4 val = *reinterpret_cast<const uint4*>(buf + r * 16 + ((v ^ ((r >> 1) & 3)) << 2));
    char* p = row_ptr(r);
    if (p) *reinterpret_cast<uint4*>(p + v * 16) = val;
  }
  __syncwarp();
}
// Coalesced load of a 32 x 32 fp32 block (rows rb.., columns c..) through the
// staging buffer; lane i receives row i.  Rows >= rows_valid read as zero.
__device__ __forceinline__ void load_rows32(uint32_t* buf, const float* src, size_t ld, int rows_valid, int lane,
                                            uint32_t (&out)[32]) {
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + lane / 8, v = lane % 8;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (r < rows_valid) val = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * ld + v * 4);
    *reinterpret_cast<uint4*>(buf + r * 32 + ((v ^ (r & 7)) << 2)) = val;
  }
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint4 val = *reinterpret_cast<const uint4*>(buf + lane * 32 + ((k ^ (lane & 7)) << 2));
    out[4 * k] = val.x;
    out[4 * k + 1] = val.y;
    out[4 * k + 2] = val.z;
    out[4 * k + 3] = val.w;
  }
  __syncwarp();
}

// Barrier over the kParts warps that own the same 32 accumulator rows.
__device__ __forceinline__ void quad_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kParts * 32) : "memory");
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
// 16-byte shared-memory load (p points into the constants region)
__device__ __forceinline__ float4 lds4(const float* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_u32(p)));
  return v;
}
// Copy n floats (n a multiple of 4, 16-byte aligned) into shared memory with the epilogue threads.
__device__ __forceinline__ void copy_consts(float* dst, const float* src, int n, int tid, int nthr) {
  for (int i = 4 * tid; i < n; i += 4 * nthr)
    *reinterpret_cast<float4*>(dst + i) = __ldg(reinterpret_cast<const float4*>(src + i));
}
// Run body(v, c) over this warp's kPartCols accumulator columns in blocks of
// 32, the TMEM load of block b+1 in flight while block b is processed.
template <class Body>
__device__ __forceinline__ void for_each_block(const EpiCtx& x, Body body) {
  static_assert(kPartCols % 64 == 0, "blocks are processed in pairs");
  uint32_t va[32], vb[32];
  tmem_ld32(x.tm + x.c0, va);
  tmem_ld_wait(va);
#pragma unroll
  for (int b = 0; b < kPartCols / 32; b += 2) {
    tmem_ld32(x.tm + x.c0 + 32 * (b + 1), vb);
    body(va, x.c0 + 32 * b);
    tmem_ld_wait(vb);
    if (b + 2 < kPartCols / 32) tmem_ld32(x.tm + x.c0 + 32 * (b + 2), va);
    body(vb, x.c0 + 32 * (b + 1));
    if (b + 2 < kPartCols / 32) tmem_ld_wait(va);
  }
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// GELU of two values with the Abramowitz-Stegun 7.1.26 erf approximation (the
// published formula the reference's FF1 epilogue uses, src/main.rs:2928-2935),
// written with packed fp32x2 FMA/MUL/ADD (same IEEE result per element as the
// scalar ops, half the instructions).
__device__ __forceinline__ float2 gelu_as2(float2 v) {
  const float2 a = __fmul2_rn(f2(fabsf(v.x), fabsf(v.y)), f2(0.70710678f, 0.70710678f));
  const float2 den = __ffma2_rn(a, f2(0.3275911f, 0.3275911f), f2(1.0f, 1.0f));
  const float2 t = f2(rcp_approx(den.x), rcp_approx(den.y));
  float2 p = __ffma2_rn(f2(1.061405429f, 1.061405429f), t, f2(-1.453152027f, -1.453152027f));
  p = __ffma2_rn(p, t, f2(1.421413741f, 1.421413741f));
  p = __ffma2_rn(p, t, f2(-0.284496736f, -0.284496736f));
  p = __ffma2_rn(p, t, f2(0.254829592f, 0.254829592f));
  p = __fmul2_rn(p, t);
  // exp(-a^2) = 2^(-a^2 * log2 e)
  const float2 arg = __fmul2_rn(__fmul2_rn(a, a), f2(-1.4426950408889634f, -1.4426950408889634f));
  const float2 e = f2(ex2_approx(arg.x), ex2_approx(arg.y));
  const float2 erfc = __fmul2_rn(p, e);
  const float2 erfa = f2(copysignf(1.0f - erfc.x, v.x), copysignf(1.0f - erfc.y, v.y));
  const float2 h = __fmul2_rn(v, f2(0.5f, 0.5f));
  return __ffma2_rn(h, erfa, h);  // 0.5 v (1 + erf)
}

// tanh accurate to ~1e-6 relative (far below the fp16 rounding of the
// mask estimator's hidden layer): odd Taylor series x(1 - x^2/3 + 2x^4/15)
// for |x| < 1/16 (truncation < 4e-10), else (1 - e)/(1 + e) with
// e = exp(-2|x|) from ex2, sign restored.
__device__ __forceinline__ float tanh_fast(float x) {
  const float ax = fabsf(x);
  const float e = ex2_approx(ax * -2.8853900817779268f);  // -2 log2(e)
  const float big = (1.0f - e) * rcp_approx(1.0f + e);
  const float x2 = x * x;
  const float small = ax * fmaf(x2, fmaf(x2, 0.13333333f, -0.33333333f), 1.0f);
  return copysignf(ax < 0.0625f ? small : big, x);
}

// ---------------------------------------------------------------------------
// Epilogues
// ---------------------------------------------------------------------------
// QKV: qkv = f16(acc + f16(bias)); Q and K then rotated (interleaved RoPE at
// the token's position: frame t on the time axis, band b on the frequency axis)
// and rounded again -- the rounding points of cuBLASLt f16-out QKV followed by
// rope_q16_inplace / rope_k16 (src/main.rs:6157-6187, :3684-3754).
struct EpiQKV : DenseTiles {
  CUtensorMap out_map;  // qkv [M][1536] fp16, box 64 x 32, 128-byte swizzle
  const float* bias16;  // [1536], values already rounded to fp16
  const float* cos;     // [P][32]
  const float* sin;
  int nb, axis;
  // constants: bias [0, 1536); RoPE rows from kRope as [pos][cos 32 | sin 32]:
  // frequency axis the whole table (nb <= kMaxNb positions, rows kRopeStride
  // floats apart so that the 32 lanes of a warp, 32 different band positions,
  // spread their 16-byte reads over all 32 banks), time axis a
  // per-warp cache of the (at most two) frames its 32 rows fall in
  static constexpr int kRope = 1536;
  static constexpr int kRopeStride = 68;
  static constexpr int kMaxNb = (kConstFloats - kRope) / kRopeStride;
  __device__ void load_consts(float* c, int tid, int nthr) const {
    copy_consts(c, bias16, 1536, tid, nthr);
    if (axis == 1 && nb <= kMaxNb)
      for (int i = tid; i < nb * 64; i += nthr) {
        const int pos = i >> 6, k = i & 63;
        c[kRope + pos * kRopeStride + k] = k < 32 ? __ldg(cos + pos * 32 + k) : __ldg(sin + pos * 32 + k - 32);
      }
  }
  FastDiv nbd;  // division by nb
  // Time axis: first frame and number of frames of the 32 rows of quadrant q.
  __device__ bool frames_of(const TileDesc& t, int q, int& p_lo, int& span) const {
    const int r_lo = t.row0 + q * 32;
    const int r_hi = min(r_lo + 31, t.row0 + t.rows - 1);
    if (r_lo > r_hi) return false;
    p_lo = nbd.div(r_lo);
    span = nbd.div(r_hi) - p_lo + 1;
    return true;
  }
  // Time axis: lane l's four floats of the cache rows p_lo, p_lo+1 of tile t
  // (row l/16, cos|sin column 4*(l%16)), fetched one tile ahead: a global load
  // in the middle of the GEMM's stores takes about a microsecond.
  __device__ void prefetch(const TileDesc& t, EpiCtx& x) const {
    int p_lo, span;
    x.pre = make_float4(0.f, 0.f, 0.f, 0.f);
    if (axis != 0 || !frames_of(t, x.q, p_lo, span) || span > 2) return;
    const int row = x.lane >> 4, k4 = (x.lane & 15) * 4;
    if (row < span) x.pre = ldg4((k4 < 32 ? cos + k4 : sin + (k4 - 32)) + (p_lo + row) * 32);
  }
  // V columns (n-tiles 4 and 5): bias only, no rotation and no RoPE rows
  __device__ void run_v(const TileDesc& t, EpiCtx& x) const {
    if (axis == 0 && x.next_tile >= 0) prefetch(tile(x.next_tile), x);
    uint32_t wp[32];
    for_each_block(x, [&](uint32_t(&v)[32], int c) {
      const int col = t.aux + c;
      const bool odd = ((c - x.c0) >> 5) & 1;  // block index within the warp's columns, known at compile time
      uint32_t* w = wp + (odd ? 16 : 0);
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 b = lds4(x.consts + col + 4 * j4);
        const float2 e0 = __fadd2_rn(f2(__uint_as_float(v[4 * j4]), __uint_as_float(v[4 * j4 + 1])), f2(b.x, b.y));
        const float2 e1 =
            __fadd2_rn(f2(__uint_as_float(v[4 * j4 + 2]), __uint_as_float(v[4 * j4 + 3])), f2(b.z, b.w));
        w[2 * j4] = pack_f16x2(e0.x, e0.y);
        w[2 * j4 + 1] = pack_f16x2(e1.x, e1.y);
      }
      if (odd) {
        uint32_t* buf = x.st.f32_buf();  // the whole 4 KB buffer
        stage_row<32>(buf, wp, x.lane);
        store_2d(&out_map, buf, col - 32, t.row0 + x.q * 32, x.lane);
      }
    });
  }
  __device__ void run(const TileDesc& t, EpiCtx& x) const {
    if (t.aux >= 1024) {
      run_v(t, x);
      return;
    }
    const int r = t.row0 + x.row;
    const bool valid = x.row < t.rows;
    const int pq = nbd.div(r);
    const int pos = valid ? (axis == 0 ? pq : r - pq * nb) : 0;
    // this thread's RoPE row: cos at rope[0..31], sin at rope[32..63]
    const float* rope = nullptr;
    bool rope_smem = false;
    if (axis == 1) {
      if (nb <= kMaxNb) {
        rope = x.consts + kRope + pos * kRopeStride;
        rope_smem = true;
      }
    } else {
      int p_lo, span;
      if (frames_of(t, x.q, p_lo, span) && span <= 2) {
        float* cache = x.consts + kRope + x.id * 128;
        __syncwarp();  // the previous tile's reads of the cache are done
        const int row = x.lane >> 4, k4 = (x.lane & 15) * 4;
        if (row < span) *reinterpret_cast<float4*>(cache + row * 64 + k4) = x.pre;
        __syncwarp();
        // rows past the end of the matrix (pos 0) read a valid cache row
        rope = cache + (valid ? pos - p_lo : 0) * 64;
        rope_smem = true;
      }
      if (x.next_tile >= 0) prefetch(tile(x.next_tile), x);
    }
    // Two 32-column blocks are staged together and leave as one 32 x 64 fp16
    // store: 128-byte rows, whole L2 lines, half as many stores as 32 x 32.
    uint32_t wp[32];
    for_each_block(x, [&](uint32_t(&v)[32], int c) {
      const int col = t.aux + c;
      const bool rot = col < 1024;
      const int pair0 = (col & 63) >> 1;
      const bool odd = ((c - x.c0) >> 5) & 1;  // block index within the warp's columns, known at compile time
      uint32_t* w = wp + (odd ? 16 : 0);
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) {
        const float4 b0 = lds4(x.consts + col + 8 * j4), b1 = lds4(x.consts + col + 8 * j4 + 4);
        float4 cs = make_float4(1.f, 1.f, 1.f, 1.f), sn = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rot) {
          if (rope_smem) {
            cs = lds4(rope + pair0 + 4 * j4);
            sn = lds4(rope + 32 + pair0 + 4 * j4);
          } else {
            cs = ldg4(cos + pos * 32 + pair0 + 4 * j4);
            sn = ldg4(sin + pos * 32 + pair0 + 4 * j4);
          }
        }
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const float cc[4] = {cs.x, cs.y, cs.z, cs.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int k = 8 * j4 + 2 * j;
          const float2 eo = __fadd2_rn(f2(__uint_as_float(v[k]), __uint_as_float(v[k + 1])), f2(bb[2 * j], bb[2 * j + 1]));
          if (rot) {
            // (e c - o s, o c + e s), products rounded separately like the
            // reference's rope kernels, applied to the fp32 pair and rounded to
            // fp16 once (the reference rounds before and after the rotation)
            const float2 p1 = __fmul2_rn(eo, f2(cc[j], cc[j]));
            const float2 p2 = __fmul2_rn(f2(eo.y, eo.x), f2(-ss[j], ss[j]));
            const float2 o2 = __fadd2_rn(p1, p2);
            w[4 * j4 + j] = pack_f16x2(o2.x, o2.y);
          } else {
            w[4 * j4 + j] = pack_f16x2(eo.x, eo.y);
          }
        }
      }
      if (odd) {
        uint32_t* buf = x.st.f32_buf();  // the whole 4 KB buffer
        stage_row<32>(buf, wp, x.lane);
        store_2d(&out_map, buf, col - 32, t.row0 + x.q * 32, x.lane);
      }
    });
  }
};

// FF1: f16(gelu_AS(acc + b1)) (gemm_f16_gelu_a16w epilogue, src/main.rs:2918-2948).
struct EpiGelu : DenseTiles {
  CUtensorMap out_map;  // ff1 [M][1024] fp16, box 32 x 32, 64-byte swizzle
  const float* bias;    // [N <= kConstFloats]
  int n;
  __device__ void load_consts(float* c, int tid, int nthr) const { copy_consts(c, bias, n, tid, nthr); }
  __device__ void run(const TileDesc& t, EpiCtx& x) const {
    for_each_block(x, [&](uint32_t(&v)[32], int c) {
      const int col = t.aux + c;
      uint32_t w[16];
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 b = lds4(x.consts + col + 4 * j4);
        const float2 g0 = gelu_as2(__fadd2_rn(f2(__uint_as_float(v[4 * j4]), __uint_as_float(v[4 * j4 + 1])), f2(b.x, b.y)));
        const float2 g1 =
            gelu_as2(__fadd2_rn(f2(__uint_as_float(v[4 * j4 + 2]), __uint_as_float(v[4 * j4 + 3])), f2(b.z, b.w)));
        w[2 * j4] = pack_f16x2(g0.x, g0.y);
        w[2 * j4 + 1] = pack_f16x2(g1.x, g1.y);
      }
      uint32_t* buf = x.st.f16_buf();
      stage_row<16>(buf, w, x.lane);
      store_2d(&out_map, buf, col, t.row0 + x.q * 32, x.lane);
    });
  }
};

// Shared body of the N = 256 fp32-row epilogues: v = acc + bias (+ resid), v
// stored as the fp32 output row, then an optional RMSNorm of the full row:
//   norm == 1: pre-FF norm (v*scale)*gamma -> fp16            (rmsnorm_h16, src/main.rs:490-554)
//   norm == 2: pre-attention norm v*(scale*gamma) -> fp16 plus
//              the 8 head gates h.Wg + bg from the fp32 h     (rmsnorm_gates_h16, :616-703)
//   norm == 3: final norm (v*scale)*gamma -> fp16, band-major (rmsnorm + transpose_band_major_h16,
//                                                              :444-483, :1755-1770)
// The warps of a row quadrant exchange partial sums through their staging
// buffers under a named barrier.  Dense rows use 2-D store maps; the band
// split's rows (t*nb + band) use 3-D maps over [T][nb][256].
struct RowNormParams {
  int norm;             // 0 none, 1 pre-FF, 2 pre-attention + gates, 3 final
  const float* gamma;   // [256]
  const float* gate_w;  // [8][256]   (norm 2)
  const float* gate_b;  // [8]        (norm 2)
  float* gates;         // [M][8]     (norm 2)
  __half* xb16;         // [nb][T][256] (norm 3)
  int T, nb;            //            (norm 3)
};

struct Row256Maps {
  CUtensorMap out_map;  // fp32 rows, box 32 x 32 (2-D) or 32 x 1 x 32 (3-D), 128-byte swizzle
  CUtensorMap h16_map;  // fp16 rows (norm 1, 2), box 64 x 32 (x 1), 128-byte swizzle
};

// Constants of the dense row epilogue in shared memory (EpiRow256::load_consts).
constexpr int kRowBias = 0, kRowGamma = 256, kRowGateW = 512, kRowGateB = 512 + 2048;

// kSmem: bias, gamma and gate_b are read from the constants region (x.consts,
// layout above) instead of global memory.  The gate weights always come from
// the constants region, transposed to [256][8] by load_gate_consts, so that one
// packed FMA updates two gates per column.
template <bool kBandRows, bool kSmem, class RowOf>
__device__ __forceinline__ void row256_epilogue(const TileDesc& t, EpiCtx& x, const float* bias, const float* resid,
                                                const Row256Maps& maps, const RowNormParams& np, int band,
                                                RowOf row_of) {
  auto ld4 = [](const float* p) { return kSmem ? lds4(p) : ldg4(p); };
  const float* gamma = kSmem ? x.consts + kRowGamma : np.gamma;
  const float* gate_wt = x.consts + kRowGateW;  // [256][8]: the 8 gate weights of each column together
  const float* gate_b = kSmem ? x.consts + kRowGateB : np.gate_b;
  if (kSmem) bias = x.consts + kRowBias;
  const bool valid = x.row < t.rows;
  const int my_row = valid ? row_of(x.row) : 0;  // global token row of this thread
  const int rb = x.q * 32;
  const int rows_valid = min(32, t.rows - rb);
  const int c0 = x.c0;
  auto store_out = [&](const CUtensorMap* m, const uint32_t* buf, int c) {
    if (kBandRows)
      store_3d(m, buf, c, band, t.row0 + rb, x.lane);
    else
      store_2d(m, buf, c, t.row0 + rb, x.lane);
  };
  // The residual (dense rows only) is read 32 rows x 32 columns at a time,
  // coalesced: 8 lanes per 128-byte row, 4 rows per instruction, one block
  // ahead.  Each block goes through the warp's staging buffer, where every
  // lane picks up its own row and then overwrites it with its output row.
  const int rl = x.lane >> 3, vl = x.lane & 7;
  const float* rbase = resid ? resid + static_cast<size_t>(t.row0 + rb) * 256 : nullptr;
  float4 pre[8];
  auto fetch = [&](int c) {
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int r = it * 4 + rl;
      pre[it] = r < rows_valid ? ldg4(rbase + static_cast<size_t>(r) * 256 + c + 4 * vl) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  if (rbase) fetch(c0);
  float ss = 0.f;
#pragma unroll 1
  for (int c = c0; c < c0 + kPartCols; c += 32) {
    const bool more = c + 32 < c0 + kPartCols;
    uint32_t v[32];
    tmem_ld32(x.tm + c, v);  // in flight while the residual is staged
    uint32_t* buf = x.st.f32_buf();
    float4 rr[8];
    if (rbase) {
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + rl;
        *reinterpret_cast<float4*>(buf + r * 32 + ((vl ^ (r & 7)) << 2)) = pre[it];
      }
      if (more) fetch(c + 32);
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 8; ++k)
        rr[k] = *reinterpret_cast<const float4*>(buf + x.lane * 32 + ((k ^ (x.lane & 7)) << 2));
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) rr[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    tmem_ld_wait(v);
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
      const float4 b = ld4(bias + c + 4 * j4);
      const float2 o01 = __fadd2_rn(__fadd2_rn(f2(__uint_as_float(v[4 * j4]), __uint_as_float(v[4 * j4 + 1])), f2(b.x, b.y)),
                                    f2(rr[j4].x, rr[j4].y));
      const float2 o23 =
          __fadd2_rn(__fadd2_rn(f2(__uint_as_float(v[4 * j4 + 2]), __uint_as_float(v[4 * j4 + 3])), f2(b.z, b.w)),
                     f2(rr[j4].z, rr[j4].w));
      const float2 sq = __ffma2_rn(o01, o01, __fmul2_rn(o23, o23));
      ss += sq.x + sq.y;
      v[4 * j4] = __float_as_uint(o01.x);
      v[4 * j4 + 1] = __float_as_uint(o01.y);
      v[4 * j4 + 2] = __float_as_uint(o23.x);
      v[4 * j4 + 3] = __float_as_uint(o23.y);
    }
    stage_row<32>(buf, v, x.lane);  // each lane rewrites only its own row
    store_out(&maps.out_map, buf, c);
    if (np.norm) tmem_st32(x.tm + c, v);
  }
  if (!np.norm) return;
  tmem_st_wait();
  // full-row sum of squares over the warps sharing these rows
  x.st.drain();
  x.st.base[x.lane] = __float_as_uint(ss);
  quad_sync(x.bar_id);
  ss = 0.f;
#pragma unroll
  for (int p = 0; p < kParts; ++p) ss += __uint_as_float(x.quad[p * kStageWords + x.lane]);
  quad_sync(x.bar_id);
  const float scale = 16.0f / fmaxf(sqrtf(ss), 1e-12f);
  // gate partial sums, (gate 2i, gate 2i+1) pairs, even and odd columns apart
  float2 ge[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
  float2 go[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
  // fp16 rows leave 64 columns at a time (32 x 64 blocks, 128-byte rows: whole
  // L2 lines); the band-major final norm scatters 32-column blocks by hand
#pragma unroll 1
  for (int c2 = c0; c2 < c0 + kPartCols; c2 += 64) {
    uint32_t wp[32];
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      const int c = c2 + 32 * hb;
      uint32_t v[32];
      tmem_ld32(x.tm + c, v);
      tmem_ld_wait(v);
      uint32_t* w = wp + 16 * hb;
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 gm = ld4(gamma + c + 4 * j4);
        const float gg[4] = {gm.x, gm.y, gm.z, gm.w};
        float h[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float vv = __uint_as_float(v[4 * j4 + k]);
          h[k] = np.norm == 2 ? __fmul_rn(vv, __fmul_rn(scale, gg[k])) : __fmul_rn(__fmul_rn(vv, scale), gg[k]);
        }
        if (np.norm == 2) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 wa = lds4(gate_wt + (c + 4 * j4 + k) * 8), wb = lds4(gate_wt + (c + 4 * j4 + k) * 8 + 4);
            const float2 hh = f2(h[k], h[k]);
            float2* acc = (k & 1) ? go : ge;
            acc[0] = __ffma2_rn(hh, f2(wa.x, wa.y), acc[0]);
            acc[1] = __ffma2_rn(hh, f2(wa.z, wa.w), acc[1]);
            acc[2] = __ffma2_rn(hh, f2(wb.x, wb.y), acc[2]);
            acc[3] = __ffma2_rn(hh, f2(wb.z, wb.w), acc[3]);
          }
        }
        w[2 * j4] = pack_f16x2(h[0], h[1]);
        w[2 * j4 + 1] = pack_f16x2(h[2], h[3]);
      }
      if (np.norm == 3) {
        uint32_t* buf = x.st.f16_buf();
        stage_row<16>(buf, w, x.lane);
        store_rows16_manual(buf, x.lane, [&](int r) -> char* {
          if (rb + r >= t.rows) return nullptr;
          const int tok = row_of(rb + r), tt = tok / np.nb, bb = tok % np.nb;
          return reinterpret_cast<char*>(np.xb16 + (static_cast<size_t>(bb) * np.T + tt) * 256 + c);
        });
      }
    }
    if (np.norm != 3) {
      uint32_t* buf = x.st.f32_buf();  // the whole 4 KB buffer
      stage_row<32>(buf, wp, x.lane);
      store_out(&maps.h16_map, buf, c2);
    }
  }
  if (np.norm == 2) {
    x.st.drain();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 gs = __fadd2_rn(ge[i], go[i]);
      x.st.base[(2 * i) * 32 + x.lane] = __float_as_uint(gs.x);
      x.st.base[(2 * i + 1) * 32 + x.lane] = __float_as_uint(gs.y);
    }
    quad_sync(x.bar_id);
    if (x.part == 0 && valid) {
      float tot[8];
#pragma unroll
      for (int gi = 0; gi < 8; ++gi) {
        tot[gi] = kSmem ? gate_b[gi] : __ldg(gate_b + gi);
#pragma unroll
        for (int p = 0; p < kParts; ++p) tot[gi] += __uint_as_float(x.quad[p * kStageWords + gi * 32 + x.lane]);
      }
      float4* dst = reinterpret_cast<float4*>(np.gates + static_cast<size_t>(my_row) * 8);
      dst[0] = make_float4(tot[0], tot[1], tot[2], tot[3]);
      dst[1] = make_float4(tot[4], tot[5], tot[6], tot[7]);
    }
    quad_sync(x.bar_id);
  }
}

// Gate weights into the constants region as [256][8] (the 8 weights of one
// column in two 16-byte vectors), plus the 8 gate biases.
__device__ __forceinline__ void load_gate_consts(float* c, const RowNormParams& np, int tid, int nthr) {
  for (int i = tid; i < 2048; i += nthr) c[kRowGateW + i] = __ldg(np.gate_w + (i & 7) * 256 + (i >> 3));
  if (tid < 8) c[kRowGateB + tid] = __ldg(np.gate_b + tid);
}

// Out-projection: attn_out = acc + bias + x, fused with the pre-FF RMSNorm
// (matmul_resid + rmsnorm_h16, src/main.rs:6219-6234).
// FF2: x = acc + b2 + attn_out (src/main.rs:6255-6259), fused with the next
// step's pre-attention RMSNorm + gates, or after the last step with the final
// norm in band-major fp16.
struct EpiRow256 : DenseTiles {
  Row256Maps maps;
  const float* bias;
  const float* resid;
  RowNormParams np;
  __device__ void load_consts(float* c, int tid, int nthr) const {
    copy_consts(c + kRowBias, bias, 256, tid, nthr);
    if (np.norm) copy_consts(c + kRowGamma, np.gamma, 256, tid, nthr);
    if (np.norm == 2) load_gate_consts(c, np, tid, nthr);
  }
  __device__ void run(const TileDesc& t, EpiCtx& x) const {
    row256_epilogue<false, true>(t, x, bias, resid, maps, np, 0, [&](int r) { return t.row0 + r; });
  }
};

// Band split: x[(t*nb + band)][n] = acc + bias[band][n] (bandsplit_gemm_f16,
// src/main.rs:4686-4698), fused with step 0's RMSNorm + gates.  Tile aux = band.
struct EpiBand : TableTiles {
  Row256Maps maps;  // 3-D maps over [T][nb][256]
  const float* bias;  // [nb][256]
  int nb;
  RowNormParams np;
  __device__ void load_consts(float* c, int tid, int nthr) const {
    if (np.norm == 2) load_gate_consts(c, np, tid, nthr);
  }
  __device__ void run(const TileDesc& t, EpiCtx& x) const {
    const int band = t.aux;
    row256_epilogue<true, false>(t, x, bias + band * 256, nullptr, maps, np, band,
                          [&](int r) { return (t.row0 + r) * nb + band; });
  }
};

// Mask estimator layer 1: hidden = f16(tanh(acc + b1)) (mask_gemm1_f16,
// src/main.rs:4816-4842).  Tile aux = group*4 + n-tile, group = stem*nb + band.
struct EpiTanh : TableTiles {
  CUtensorMap out_map;  // hidden [groups][T][1024] fp16, box 64 x 32 x 1, 128-byte swizzle
  const float* bias;    // [groups][1024]
  __device__ void run(const TileDesc& t, EpiCtx& x) const {
    const int group = t.aux >> 2, n0 = (t.aux & 3) * kBN;
    // 64 columns per store: 32 x 64 fp16 blocks, 128-byte rows (whole L2 lines)
#pragma unroll 1
    for (int c2 = x.c0; c2 < x.c0 + kPartCols; c2 += 64) {
      uint32_t wp[32];
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const int c = c2 + 32 * hb;
        uint32_t v[32];
        tmem_ld32(x.tm + c, v);
        tmem_ld_wait(v);
        const float* bb = bias + static_cast<size_t>(group) * 1024 + n0 + c;
        uint32_t* w = wp + 16 * hb;
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          const float4 b = ldg4(bb + 4 * j4);
          w[2 * j4] =
              pack_f16x2(tanh_fast(__uint_as_float(v[4 * j4]) + b.x), tanh_fast(__uint_as_float(v[4 * j4 + 1]) + b.y));
          w[2 * j4 + 1] = pack_f16x2(tanh_fast(__uint_as_float(v[4 * j4 + 2]) + b.z),
                                     tanh_fast(__uint_as_float(v[4 * j4 + 3]) + b.w));
        }
      }
      uint32_t* buf = x.st.f32_buf();  // the whole 4 KB buffer
      stage_row<32>(buf, wp, x.lane);
      store_3d(&out_map, buf, n0 + c2, t.row0 + x.q * 32, group, x.lane);
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
  int keep_dc_imag;     // 1: the DC/Nyquist bins keep the imaginary part the complex mask gives them
  __device__ void run(const TileDesc& t, EpiCtx& x) const {
    const bool valid = x.row < t.rows;
    const int rb = x.q * 32;                // this warp's first tile row
    const int rows_valid = min(32, t.rows - rb);
    const int r0 = t.row0 + rb;             // its first frame
    const int stem = t.aux >> 16, band = (t.aux >> 8) & 255, n0 = (t.aux & 255) * kBN;
    const int d_b = band_d[band], f0 = band_f0[band];
    const float* bb = bias2 + static_cast<size_t>(stem) * n2tot + band_o2[band] + n0;
    const int c_end = min(x.c0 + kPartCols, t.n);
    // A 32-column block is 4 bins of 32 frames.  Spectrum values go through
    // the warp's staging buffer ([2 channels][32 frames][4 bins] float2): read
    // with four lanes per frame (32 contiguous bytes), masked by the frame's
    // lane, written back the same way, instead of one 8-byte access per lane
    // at a stride of a whole frame.
    float2* sbuf = reinterpret_cast<float2*>(x.st.base);
    const int lrow = x.lane >> 2, lbin = x.lane & 3;
#pragma unroll 1
    for (int c = x.c0; c < c_end; c += 32) {
      uint32_t v[32];
      tmem_ld32(x.tm + c, v);
      // bins of this block with columns in the tile and inside the band (a prefix)
      int nbins = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) nbins += (c + q * 8 < t.n && ((n0 + c + q * 8) >> 1) < d_b) ? 1 : 0;
      const int fb = f0 + ((n0 + c) >> 3);  // first bin
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int row = it * 8 + lrow;
        if (row < rows_valid && lbin < nbins)
#pragma unroll
          for (int ch = 0; ch < 2; ++ch)
            sbuf[(ch * 32 + row) * 4 + lbin] = spec[(static_cast<size_t>(ch) * T + r0 + row) * 1025 + fb + lbin];
      }
      tmem_ld_wait(v);
      __syncwarp();
      if (valid) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q >= nbins) break;
          const int lc = c + q * 8;  // column inside this tile
          float m[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float a = __uint_as_float(v[q * 8 + 2 * k]) + __ldg(bb + lc + 2 * k);
            const float g = __uint_as_float(v[q * 8 + 2 * k + 1]) + __ldg(bb + lc + 2 * k + 1);
            m[k] = __fdividef(a, 1.0f + __expf(-g));
          }
          const int f = fb + q;
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            float2& slot = sbuf[(ch * 32 + x.lane) * 4 + q];
            const float2 sp = slot;
            const float mr = m[2 * ch], mi = m[2 * ch + 1];
            float2 o;
            o.x = sp.x * mr - sp.y * mi;
            // A real signal's DC and Nyquist bins are real: torch.istft drops
            // their imaginary parts, and a C2R transform is only defined for
            // such Hermitian input, so by default the masked spectrum keeps
            // them real.  keep_dc_imag reproduces the reference's mask_apply
            // (src/main.rs:1776-1817), which passes them on unchanged.
            o.y = ((f == 0 || f == 1024) && !keep_dc_imag) ? 0.f : sp.x * mi + sp.y * mr;
            slot = o;
          }
        }
      }
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int row = it * 8 + lrow;
        if (row < rows_valid && lbin < nbins)
#pragma unroll
          for (int ch = 0; ch < 2; ++ch)
            out[(static_cast<size_t>(stem * 2 + ch) * T + r0 + row) * 1025 + fb + lbin] =
                sbuf[(ch * 32 + row) * 4 + lbin];
      }
    }
    __syncwarp();
  }
};

// ---------------------------------------------------------------------------
// The persistent kernel
// ---------------------------------------------------------------------------
template <class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ Epi epi, int n_tiles, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if ((smem_u32(smem) & 1023u) != 0) {  // uniform across the CTA: nothing allocated yet
    if (threadIdx.x == 0) report_status(status, kDevSmemMisaligned);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], kEpiWarps);
    }
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
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t kbg = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        const TileDesc t = epi.tile(tile);
        for (int kb = 0; kb < t.kblocks; ++kb, ++kbg) {
          const int s = kbg % kStages;
          const uint32_t ph = (kbg / kStages) & 1;
          if (!(ok = mbar_wait(&empty[s], ph ^ 1u, abort_flag, status))) break;
          uint8_t* sa = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_2d(sa, &tmA, &full[s], t.a_col + kb * kBK, t.a_row);
          tma_load_2d(sa + kABytes, &tmB, &full[s], kb * kBK, t.b_row);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t kbg = 0;
      bool ok = true;
      int i = 0;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++i) {
        const TileDesc t = epi.tile(tile);
        const int slot = i & 1;
        if (!(ok = mbar_wait(&acc_empty[slot], ((i >> 1) & 1) ^ 1u, abort_flag, status))) break;
        tc_fence_after();
        const uint32_t d = tmem + slot * kBN;
        const uint32_t idesc = idesc_f16_f32(kBM, t.n);
        for (int kb = 0; kb < t.kblocks; ++kb, ++kbg) {
          const int s = kbg % kStages;
          const uint32_t ph = (kbg / kStages) & 1;
          if (!(ok = mbar_wait(&full[s], ph, abort_flag, status))) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16_ss(d, sdesc_sw128(sa + k * 32, 1024, 16), sdesc_sw128(sb + k * 32, 1024, 16), idesc,
                       (kb | k) != 0 ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[slot]);
      }
    }
  } else {
    // ---------------- epilogue warps ----------------
    const int ew = warp - 2;  // 0..kEpiWarps-1
    EpiCtx x;
    x.lane = lane;
    x.q = warp & 3;  // TMEM lane quadrant this warp may access
    x.part = ew >> 2;
    x.c0 = x.part * kPartCols;
    x.row = x.q * 32 + lane;
    uint32_t* staging = reinterpret_cast<uint32_t*>(smem + kStagingOff);
    // buffers are laid out quadrant-major so the kParts warps of a quadrant are contiguous
    x.quad = staging + x.q * kParts * kStageWords;
    x.st.base = x.quad + x.part * kStageWords;
    x.st.lane = lane;
    x.st.phase = 0;
    x.st.last_f32 = false;
    x.bar_id = 1 + x.q;
    float* consts = reinterpret_cast<float*>(smem + kConstOff);
    x.consts = consts;
    x.id = x.part * 4 + x.q;
    if (static_cast<int>(blockIdx.x) < n_tiles) epi.prefetch(epi.tile(blockIdx.x), x);
    epi.load_consts(consts, ew * 32 + lane, kEpiWarps * 32);
    // all epilogue warps, once, before any tile: the constants are complete
    asm volatile("bar.sync 5, %0;" ::"n"(kEpiWarps * 32) : "memory");
    int i = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++i) {
      const TileDesc t = epi.tile(tile);
      const int slot = i & 1;
      if (!mbar_wait(&acc_full[slot], (i >> 1) & 1, abort_flag, status)) break;
      tc_fence_after();
      x.tm = tmem + (static_cast<uint32_t>(x.q * 32) << 16) + slot * kBN;
      x.next_tile = tile + static_cast<int>(gridDim.x) < n_tiles ? tile + static_cast<int>(gridDim.x) : -1;
      epi.run(t, x);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[slot]);
    }
    if (lane == 0) tma_store_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Fused feed-forward: x = W2 f16(gelu(W1 h + b1)) + b2 + resid, then the row
// epilogue (next RMSNorm); the [M][1024] hidden activation never leaves the SM
// ---------------------------------------------------------------------------
// Per 128-row tile, FF1 runs in 4 chunks of 256 hidden units into a
// 256-column TMEM accumulator (acc1, columns 0..255).  The epilogue warps load
// a chunk into registers (which frees acc1 for the next chunk's FF1), turn it
// into f16(gelu(acc + b1)) (the values the unfused FF1 stores) and write it
// into shared memory as FF2's A operand G (K-major, 128-byte swizzle, four
// [128][64] tiles).  FF2 accumulates chunk by chunk into a second 256-column
// accumulator (acc2, columns 256..511) in the same K order as the unfused
// FF2; after the last chunk the epilogue warps run the N = 256 row epilogue,
// whose staging buffers reuse G.  All MMAs are
// 128 x 256 x 16 (an N = 128 MMA would read as many shared-memory bytes per
// FLOP as the SM can deliver).
// MMA order per tile: FF1(0), FF1(1), FF2(0), FF1(2), FF2(1), FF1(3),
// FF2(2), FF2(3), so each chunk's GELU overlaps the next chunk's FF1 and the
// previous chunk's FF2.  The weights stream through a 2-stage ring of 32 KB
// tiles ([256][64] fp16) in that order: W1 chunk c and W2 chunk c are 4
// K-blocks each.  Warps: 0..7 epilogue (two per TMEM lane quadrant, 128 of
// the 256 columns each), 8 weight loads, 9 TMEM allocation + MMA issue, 10
// h-tile loads (one [128][256] tile per 128 rows, reloaded once the tile's
// FF1 is done).  The epilogue warpgroups take 200 registers per thread and
// warpgroup 2 keeps 104 (setmaxnreg): a whole 128-column chunk row and its
// fp16 pairs fit without spilling.
constexpr int kFfChunk = 256;
constexpr int kFfChunks = 1024 / kFfChunk;
constexpr int kFfTileBytes = kBM * kBK * 2;   // 16 KB: [128][64] fp16
constexpr int kFfWBytes = kFfChunk * kBK * 2;  // 32 KB: [256][64] fp16
constexpr int kFfWStages = 2;
constexpr int kFfOffH = 0;                           // 4 tiles (K = 256)
constexpr int kFfOffG = kFfOffH + 4 * kFfTileBytes;  // 4 tiles (K = 256 hidden units of a chunk)
constexpr int kFfOffW = kFfOffG + 4 * kFfTileBytes;  // weight ring
constexpr int kFfOffConst = kFfOffW + kFfWStages * kFfWBytes;
constexpr int kFfConstFloats = 4096;
constexpr int kFfB1 = 3072;  // b1 in the constants region, after the row epilogue's constants
constexpr int kFfOffBar = kFfOffConst + kFfConstFloats * 4;
constexpr int kFfSmem = kFfOffBar + 256;
constexpr int kFfThreads = kEpiWarps * 32 + 128;
constexpr int kFfWarpW = kEpiWarps, kFfWarpMma = kEpiWarps + 1, kFfWarpH = kEpiWarps + 2;
constexpr int kFfRegsEpi = 200, kFfRegsOther = 104;
static_assert(kFfSmem <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
static_assert(kRowGateB + 8 <= kFfB1 && kFfB1 + 1024 <= kFfConstFloats, "constants overlap");
static_assert(kEpiWarps * kStageWords * 4 <= 4 * kFfTileBytes, "staging must fit in G");
static_assert(kEpiWarps == 8 && kPartCols == 128, "two epilogue warps per quadrant, 128 columns each");

__global__ void __launch_bounds__(kFfThreads, 1)
    ff_fused_kernel(const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmW1,
                    const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ EpiRow256 epi,
                    const float* b1, int n_tiles, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kFfOffBar);
  uint64_t* w_full = bars;                  // [kFfWStages]
  uint64_t* w_empty = w_full + kFfWStages;  // [kFfWStages]
  uint64_t* h_full = w_empty + kFfWStages;
  uint64_t* h_empty = h_full + 1;
  uint64_t* a1_full = h_empty + 1;   // FF1 chunk in acc1
  uint64_t* a1_empty = a1_full + 1;  // acc1 loaded by every epilogue warp
  uint64_t* g_full = a1_empty + 1;   // G written
  uint64_t* g_empty = g_full + 1;    // G consumed by FF2
  uint64_t* a2_full = g_empty + 1;
  uint64_t* a2_empty = a2_full + 1;
  uint64_t* stage_free = a2_empty + 1;  // every epilogue warp's row-epilogue stores have read G
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stage_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) report_status(status, kDevSmemMisaligned);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kFfWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    mbar_init(h_full, 1);
    mbar_init(h_empty, 1);
    mbar_init(a1_full, 1);
    mbar_init(a1_empty, kEpiWarps);
    mbar_init(g_full, kEpiWarps);
    mbar_init(g_empty, 1);
    mbar_init(a2_full, 1);
    mbar_init(a2_empty, kEpiWarps);
    mbar_init(stage_free, kEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kFfWarpW && lane == 0) {
    tma_prefetch(&tmW1);
    tma_prefetch(&tmW2);
  }
  if (warp == kFfWarpH && lane == 0) tma_prefetch(&tmH);
  if (warp == kFfWarpMma) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Register split, 256 x 200 + 128 x 104 <= 384 x 168 launch registers (the
  // launcher checks the compiled count before the first launch); each role
  // changes its own warpgroup's count at the top of its branch.
  if (warp >= kEpiWarps) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kFfRegsOther));

  if (warp == kFfWarpW) {
    // ---------------- weight tiles, in MMA order ----------------
    if (lane == 0) {
      uint32_t wc = 0;
      bool ok = true;
      auto load_w = [&](const CUtensorMap* m, int x, int y) {
        const int s = wc % kFfWStages;
        const uint32_t ph = (wc / kFfWStages) & 1;
        ++wc;
        if (!(ok = mbar_wait(&w_empty[s], ph ^ 1u, abort_flag, status))) return;
        mbar_arrive_expect_tx(&w_full[s], kFfWBytes);
        tma_load_2d(smem + kFfOffW + s * kFfWBytes, m, &w_full[s], x, y);
      };
      auto load_w1 = [&](int c) {
        for (int kb = 0; ok && kb < 4; ++kb) load_w(&tmW1, kb * kBK, c * kFfChunk);
      };
      auto load_w2 = [&](int c) {
        for (int kb = 0; ok && kb < 4; ++kb) load_w(&tmW2, c * kFfChunk + kb * kBK, 0);
      };
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        for (int c = 0; ok && c < kFfChunks; ++c) {
          load_w1(c);
          if (c > 0) load_w2(c - 1);
        }
        if (ok) load_w2(kFfChunks - 1);
      }
    }
  } else if (warp == kFfWarpH) {
    // ---------------- h tiles ----------------
    if (lane == 0) {
      int i = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++i) {
        if (!mbar_wait(h_empty, (i & 1) ^ 1u, abort_flag, status)) break;
        mbar_arrive_expect_tx(h_full, 4 * kFfTileBytes);
        for (int kb = 0; kb < 4; ++kb)
          tma_load_2d(smem + kFfOffH + kb * kFfTileBytes, &tmH, h_full, kb * kBK, tile * kBM);
      }
    }
  } else if (warp == kFfWarpMma) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t wc = 0;
      const uint32_t id = idesc_f16_f32(kBM, kFfChunk);
      auto w_tile = [&](uint32_t& sb) {
        const int s = wc % kFfWStages;
        if (!mbar_wait(&w_full[s], (wc / kFfWStages) & 1, abort_flag, status)) return false;
        tc_fence_after();
        sb = smem_u32(smem + kFfOffW + s * kFfWBytes);
        return true;
      };
      auto w_release = [&]() {
        mma_commit(&w_empty[wc % kFfWStages]);
        ++wc;
      };
      // g: chunk index over this CTA's tiles (phase g of the chunk barriers)
      auto ff1 = [&](int g) {
        if (!mbar_wait(a1_empty, (g & 1) ^ 1u, abort_flag, status)) return false;
        tc_fence_after();
        for (int kb = 0; kb < 4; ++kb) {
          uint32_t sb;
          if (!w_tile(sb)) return false;
          const uint32_t sa = smem_u32(smem + kFfOffH + kb * kFfTileBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16_ss(tmem, sdesc_sw128(sa + k * 32, 1024, 16), sdesc_sw128(sb + k * 32, 1024, 16), id,
                       (kb | k) != 0 ? 1u : 0u);
          w_release();
        }
        mma_commit(a1_full);
        return true;
      };
      auto ff2 = [&](int g, int c, int i) {
        if (c == 0) {
          if (!mbar_wait(a2_empty, (i & 1) ^ 1u, abort_flag, status)) return false;
        }
        if (!mbar_wait(g_full, g & 1, abort_flag, status)) return false;
        tc_fence_after();
        for (int kb = 0; kb < 4; ++kb) {
          uint32_t sb;
          if (!w_tile(sb)) return false;
          const uint32_t sa = smem_u32(smem + kFfOffG + kb * kFfTileBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_f16_ss(tmem + kFfChunk, sdesc_sw128(sa + k * 32, 1024, 16), sdesc_sw128(sb + k * 32, 1024, 16), id,
                       (c | kb | k) != 0 ? 1u : 0u);
          w_release();
        }
        mma_commit(g_empty);
        return true;
      };
      bool ok = true;
      int i = 0;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++i) {
        if (!(ok = mbar_wait(h_full, i & 1, abort_flag, status))) break;
        tc_fence_after();
        const int g0 = i * kFfChunks;
        for (int c = 0; ok && c < kFfChunks; ++c) {
          ok = ff1(g0 + c);
          if (ok && c == kFfChunks - 1) mma_commit(h_empty);  // h is free once this tile's FF1 completes
          if (ok && c > 0) ok = ff2(g0 + c - 1, c - 1, i);
        }
        if (ok) ok = ff2(g0 + kFfChunks - 1, kFfChunks - 1, i);
        if (ok) mma_commit(a2_full);
      }
    }
  } else if (warp < kEpiWarps) {
    // ---------------- epilogue warps ----------------
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kFfRegsEpi));
    EpiCtx x;
    x.lane = lane;
    x.q = warp & 3;  // TMEM lane quadrant this warp may access
    x.part = warp >> 2;
    x.c0 = x.part * kPartCols;
    x.row = x.q * 32 + lane;
    uint32_t* staging = reinterpret_cast<uint32_t*>(smem + kFfOffG);
    x.quad = staging + x.q * kParts * kStageWords;
    x.st.base = x.quad + x.part * kStageWords;
    x.st.lane = lane;
    x.st.phase = 0;
    x.st.last_f32 = false;
    x.bar_id = 1 + x.q;
    float* consts = reinterpret_cast<float*>(smem + kFfOffConst);
    x.consts = consts;
    x.id = x.part * 4 + x.q;
    epi.load_consts(consts, warp * 32 + lane, kEpiWarps * 32);
    copy_consts(consts + kFfB1, b1, 1024, warp * 32 + lane, kEpiWarps * 32);
    asm volatile("bar.sync 5, %0;" ::"n"(kEpiWarps * 32) : "memory");
    const uint32_t lane_off = static_cast<uint32_t>(x.q * 32) << 16;
    // this thread's row in G tile 2*part (+1 for the second 64 columns)
    uint8_t* grow = smem + kFfOffG + (2 * x.part) * kFfTileBytes + x.row * 128;
    int i = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++i) {
      const TileDesc t = epi.tile(tile);
      // The row epilogue reads this tile's fp32 residual (128 rows x 1 KB)
      // after the four GELU chunks: start bringing it into L2 now, four
      // 128-byte lines per thread, so that those reads do not wait for HBM.
      if (epi.resid && (warp * 32 + lane) / 2 < t.rows) {
        const char* rp = reinterpret_cast<const char*>(epi.resid + static_cast<size_t>(t.row0) * 256) +
                         (warp * 32 + lane) * 512;
#pragma unroll
        for (int k = 0; k < 4; ++k) prefetch_l2(rp + k * 128);
      }
      const int g0 = i * kFfChunks;
      for (int c = 0; ok && c < kFfChunks; ++c) {
        const int g = g0 + c;
        if (!(ok = mbar_wait(a1_full, g & 1, abort_flag, status))) break;
        tc_fence_after();
        uint32_t v[4][32];
#pragma unroll
        for (int b = 0; b < 4; ++b) tmem_ld32(tmem + lane_off + x.c0 + 32 * b, v[b]);
#pragma unroll
        for (int b = 0; b < 4; ++b) tmem_ld_wait(v[b]);
        // the chunk is in registers: FF1 of the next chunk may overwrite acc1
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(a1_empty);
        const float* bias = consts + kFfB1 + c * kFfChunk + x.c0;
        uint32_t w[4][16];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 bb = lds4(bias + 32 * b + 4 * j4);
            const float2 g0v = gelu_as2(
                __fadd2_rn(f2(__uint_as_float(v[b][4 * j4]), __uint_as_float(v[b][4 * j4 + 1])), f2(bb.x, bb.y)));
            const float2 g1v = gelu_as2(
                __fadd2_rn(f2(__uint_as_float(v[b][4 * j4 + 2]), __uint_as_float(v[b][4 * j4 + 3])), f2(bb.z, bb.w)));
            w[b][2 * j4] = pack_f16x2(g0v.x, g0v.y);
            w[b][2 * j4 + 1] = pack_f16x2(g1v.x, g1v.y);
          }
        }
        // G may be rewritten once FF2 of the previous chunk has read it
        if (!(ok = mbar_wait(g_empty, (g & 1) ^ 1u, abort_flag, status))) break;
        // 16-byte vector j of a 128-byte G row sits at j ^ (row & 7)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          uint8_t* dst = grow + (b >> 1) * kFfTileBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            *reinterpret_cast<uint4*>(dst + ((((b & 1) * 4 + k) ^ (x.row & 7)) << 4)) =
                make_uint4(w[b][4 * k], w[b][4 * k + 1], w[b][4 * k + 2], w[b][4 * k + 3]);
        }
        // the tensor core reads G through the async proxy
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(g_full);
      }
      if (!ok) break;
      if (!(ok = mbar_wait(a2_full, i & 1, abort_flag, status))) break;
      tc_fence_after();
      x.tm = tmem + lane_off + kFfChunk;
      x.next_tile = tile + static_cast<int>(gridDim.x) < n_tiles ? tile + static_cast<int>(gridDim.x) : -1;
      epi.run(t, x);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(a2_empty);
      // G held the staging buffers: the next tile's GELU rewrites it only
      // after every warp's stores have read their blocks
      x.st.drain();
      if (lane == 0) mbar_arrive(stage_free);
      ok = mbar_wait(stage_free, i & 1, abort_flag, status);
    }
    if (lane == 0) tma_store_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kFfWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <class Epi>
static cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const Epi& epi, int tiles, int* status,
                               cudaStream_t st) {
  static unsigned long long configured = 0;
  cudaError_t e = once_per_device(configured, [] {
    return cudaFuncSetAttribute(gemm_tc_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
  });
  if (e != cudaSuccess) return e;
  if (tiles <= 0) return cudaSuccess;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  count_launch();
  gemm_tc_kernel<Epi><<<grid, kGemmThreads, kGemmSmem, st>>>(a, b, epi, tiles, status);
  return cudaGetLastError();
}

static int dense_tiles(int M, int N) { return ((M + kBM - 1) / kBM) * (N / kBN); }

// fp16 [rows][cols] output map for 32 x 32 blocks (64-byte rows, 64-byte swizzle)
static cudaError_t out_map16(CUtensorMap* m, const void* base, int cols, uint64_t rows) {
  return make_map_2d(m, base, cols, rows, static_cast<uint64_t>(cols) * 2, 32, 32, MapElem::F16,
                     CU_TENSOR_MAP_SWIZZLE_64B);
}
// fp16 [rows][cols] output map for 32 x 64 blocks (128-byte rows, 128-byte swizzle)
static cudaError_t out_map16w(CUtensorMap* m, const void* base, int cols, uint64_t rows) {
  return make_map_2d(m, base, cols, rows, static_cast<uint64_t>(cols) * 2, 64, 32, MapElem::F16,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}
// fp32 [rows][cols] output map for 32 x 32 blocks (128-byte rows, 128-byte swizzle)
static cudaError_t out_map32(CUtensorMap* m, const void* base, int cols, uint64_t rows) {
  return make_map_2d(m, base, cols, rows, static_cast<uint64_t>(cols) * 4, 32, 32, MapElem::F32,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

static RowNormParams to_params(const RowNorm& n) {
  RowNormParams p{};
  p.norm = n.kind;
  p.gamma = n.gamma;
  p.gate_w = n.gate_w;
  p.gate_b = n.gate_b;
  p.gates = n.gates;
  p.xb16 = n.xb16;
  p.T = n.T;
  p.nb = n.nb;
  return p;
}

cudaError_t gemm_qkv(const __half* h16, const __half* w, const float* bias16, const float* cos, const float* sin,
                     __half* qkv, int M, int nb, int axis, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  EpiQKV ep;
  cudaError_t e = make_map_2d(&ta, h16, 256, M, 256 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w, 256, 1536, 256 * 2, kBK, kBN);
  if (e == cudaSuccess)
    e = make_map_2d(&ep.out_map, qkv, 1536, M, 1536 * 2, 64, 32, MapElem::F16, CU_TENSOR_MAP_SWIZZLE_128B);
  if (e != cudaSuccess) return e;
  ep.M = M;
  ep.n_tiles = 1536 / kBN;
  ep.kblocks = 256 / kBK;
  ep.ntd = make_fastdiv(ep.n_tiles, dense_tiles(M, 1536));
  ep.nbd = make_fastdiv(static_cast<uint32_t>(nb), static_cast<uint64_t>(M));
  ep.bias16 = bias16;
  ep.cos = cos;
  ep.sin = sin;
  ep.nb = nb;
  ep.axis = axis;
  return launch_gemm(ta, tb, ep, dense_tiles(M, 1536), status, st);
}

cudaError_t gemm_outproj_norm(const __half* scaled16, const __half* w, const float* bias, const float* resid,
                              const float* gamma, float* out, __half* h16, int M, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  EpiRow256 ep;
  cudaError_t e = make_map_2d(&ta, scaled16, 512, M, 512 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w, 512, 256, 512 * 2, kBK, kBN);
  if (e == cudaSuccess) e = out_map32(&ep.maps.out_map, out, 256, M);
  if (e == cudaSuccess) e = out_map16w(&ep.maps.h16_map, h16, 256, M);
  if (e != cudaSuccess) return e;
  ep.M = M;
  ep.n_tiles = 1;
  ep.kblocks = 512 / kBK;
  ep.ntd = make_fastdiv(ep.n_tiles, dense_tiles(M, 256));
  ep.bias = bias;
  ep.resid = resid;
  ep.np = RowNormParams{};
  ep.np.norm = 1;
  ep.np.gamma = gamma;
  return launch_gemm(ta, tb, ep, dense_tiles(M, 256), status, st);
}

cudaError_t gemm_ff1_gelu(const __half* h16, const __half* w1, const float* b1, __half* ff1, int M, int* status,
                          cudaStream_t st) {
  CUtensorMap ta, tb;
  EpiGelu ep;
  cudaError_t e = make_map_2d(&ta, h16, 256, M, 256 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w1, 256, 1024, 256 * 2, kBK, kBN);
  if (e == cudaSuccess) e = out_map16(&ep.out_map, ff1, 1024, M);
  if (e != cudaSuccess) return e;
  ep.M = M;
  ep.n_tiles = 1024 / kBN;
  ep.kblocks = 256 / kBK;
  ep.ntd = make_fastdiv(ep.n_tiles, dense_tiles(M, 1024));
  ep.bias = b1;
  ep.n = 1024;
  return launch_gemm(ta, tb, ep, dense_tiles(M, 1024), status, st);
}

cudaError_t gemm_ff2_resid(const __half* ff1, const __half* w2, const float* b2, const float* resid, float* x, int M,
                           const RowNorm& next, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  EpiRow256 ep;
  cudaError_t e = make_map_2d(&ta, ff1, 1024, M, 1024 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w2, 1024, 256, 1024 * 2, kBK, kBN);
  if (e == cudaSuccess) e = out_map32(&ep.maps.out_map, x, 256, M);
  if (e == cudaSuccess && next.h16) e = out_map16w(&ep.maps.h16_map, next.h16, 256, M);
  if (e != cudaSuccess) return e;
  ep.M = M;
  ep.n_tiles = 1;
  ep.kblocks = 1024 / kBK;
  ep.ntd = make_fastdiv(ep.n_tiles, dense_tiles(M, 256));
  ep.bias = b2;
  ep.resid = resid;
  ep.np = to_params(next);
  return launch_gemm(ta, tb, ep, dense_tiles(M, 256), status, st);
}

cudaError_t gemm_ff_fused(const __half* h16, const __half* w1, const float* b1, const __half* w2, const float* b2,
                          const float* resid, float* x, int M, const RowNorm& next, int* status, cudaStream_t st) {
  static unsigned long long configured = 0;
  cudaError_t e = once_per_device(configured, [] {
    cudaError_t r = cudaFuncSetAttribute(ff_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFfSmem);
    if (r != cudaSuccess) return r;
    // setmaxnreg.inc waits until the block's launch registers cover the split;
    // refuse to launch a build whose register count would not
    cudaFuncAttributes fa;
    r = cudaFuncGetAttributes(&fa, ff_fused_kernel);
    if (r != cudaSuccess) return r;
    if (fa.numRegs * kFfThreads < kEpiWarps * 32 * kFfRegsEpi + (kFfThreads - kEpiWarps * 32) * kFfRegsOther)
      return cudaErrorInvalidConfiguration;
    return cudaSuccess;
  });
  if (e != cudaSuccess) return e;
  CUtensorMap th, tw1, tw2;
  EpiRow256 ep;
  e = make_map_2d(&th, h16, 256, M, 256 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tw1, w1, 256, 1024, 256 * 2, kBK, kFfChunk);
  if (e == cudaSuccess) e = make_map_2d(&tw2, w2, 1024, 256, 1024 * 2, kBK, kFfChunk);
  if (e == cudaSuccess) e = out_map32(&ep.maps.out_map, x, 256, M);
  if (e == cudaSuccess && next.h16) e = out_map16w(&ep.maps.h16_map, next.h16, 256, M);
  if (e != cudaSuccess) return e;
  ep.M = M;
  ep.n_tiles = 1;
  ep.kblocks = 0;  // unused: the fused kernel walks its own K loops
  ep.ntd = make_fastdiv(1, dense_tiles(M, 256));
  ep.bias = b2;
  ep.resid = resid;
  ep.np = to_params(next);
  const int tiles = dense_tiles(M, 256);
  if (tiles <= 0) return cudaSuccess;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  count_launch();
  ff_fused_kernel<<<grid, kFfThreads, kFfSmem, st>>>(th, tw1, tw2, ep, b1, tiles, status);
  return cudaGetLastError();
}

cudaError_t gemm_bandsplit(const __half* xn, int xn_cols, const __half* wband, int wband_cols, const float* bias,
                           float* x, int T, int nb, const TileDesc* tiles, int n_tiles, const RowNorm& first,
                           int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  EpiBand ep;
  cudaError_t e = make_map_2d(&ta, xn, xn_cols, T, static_cast<uint64_t>(xn_cols) * 2, kBK, kBM);
  if (e == cudaSuccess)
    e = make_map_2d(&tb, wband, wband_cols, static_cast<uint64_t>(nb) * 256, static_cast<uint64_t>(wband_cols) * 2,
                    kBK, kBN);
  // token rows t*nb + band viewed as [T][nb][256]
  if (e == cudaSuccess)
    e = make_map_3d(&ep.maps.out_map, x, 256, nb, T, 256 * 4, static_cast<uint64_t>(nb) * 256 * 4, 32, 1, 32,
                    MapElem::F32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (e == cudaSuccess && first.h16)
    e = make_map_3d(&ep.maps.h16_map, first.h16, 256, nb, T, 256 * 2, static_cast<uint64_t>(nb) * 256 * 2, 64, 1,
                    32, MapElem::F16, CU_TENSOR_MAP_SWIZZLE_128B);
  if (e != cudaSuccess) return e;
  ep.table = tiles;
  ep.bias = bias;
  ep.nb = nb;
  ep.np = to_params(first);
  return launch_gemm(ta, tb, ep, n_tiles, status, st);
}

cudaError_t gemm_mask1(const __half* xb16, const __half* w1, const float* b1, __half* hidden, int T, int groups,
                       const TileDesc* tiles, int n_tiles, int* status, cudaStream_t st) {
  CUtensorMap ta, tb;
  EpiTanh ep;
  cudaError_t e = make_map_2d(&ta, xb16, 256, static_cast<uint64_t>(T) * kNumBands, 256 * 2, kBK, kBM);
  if (e == cudaSuccess) e = make_map_2d(&tb, w1, 256, static_cast<uint64_t>(groups) * 1024, 256 * 2, kBK, kBN);
  // hidden viewed as [groups][T][1024] so a tile's rows never spill into the next group
  if (e == cudaSuccess)
    e = make_map_3d(&ep.out_map, hidden, 1024, T, groups, 1024 * 2, static_cast<uint64_t>(T) * 1024 * 2, 64, 32, 1,
                    MapElem::F16, CU_TENSOR_MAP_SWIZZLE_128B);
  if (e != cudaSuccess) return e;
  ep.table = tiles;
  ep.bias = b1;
  return launch_gemm(ta, tb, ep, n_tiles, status, st);
}

cudaError_t gemm_mask2(const __half* hidden, const __half* w2, const float* b2, const int* band_f0,
                       const int* band_d, const int* band_o2, const float2* spec, float2* c2r, int T, int stems,
                       int n2tot, const TileDesc* tiles, int n_tiles, bool keep_dc_imag, int* status,
                       cudaStream_t st) {
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
  ep.keep_dc_imag = keep_dc_imag ? 1 : 0;
  return launch_gemm(ta, tb, ep, n_tiles, status, st);
}

}  // namespace lbrr
