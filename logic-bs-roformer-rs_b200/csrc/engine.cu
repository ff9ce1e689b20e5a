// Engine and C ABI (include/lbrr_gpu.h): weight validation and placement,
// per-length setup (RoPE tables, grouped-GEMM tile tables, cuFFT plans, ISTFT
// envelope), the chunk forward, the whole-song overlap-add across engines and
// the per-op entry points.
#include <cufft.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/lbrr_gpu.h"
#include "common.cuh"
#include "kernels.h"

using namespace lbrr;

thread_local long long lbrr::t_kernel_launches = 0;

// ---------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------
static thread_local std::string g_err;

static int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
#define CK(call)                                                                                   \
  do {                                                                                             \
    cudaError_t _e = (call);                                                                       \
    if (_e != cudaSuccess)                                                                         \
      return fail(LBRR_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(_e));              \
  } while (0)
#define CKFFT(call)                                                                                \
  do {                                                                                             \
    cufftResult _r = (call);                                                                       \
    if (_r != CUFFT_SUCCESS) return fail(LBRR_ERR_CUDA, std::string(#call) + ": cufft error " + std::to_string(_r)); \
  } while (0)

// ---------------------------------------------------------------------------
// fp16 packing contract (src/fp16.rs:4-37): RNE, NaN -> sign | 0x7c01.
// ---------------------------------------------------------------------------
static uint16_t f32_to_f16_bits(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  const uint16_t sign = static_cast<uint16_t>((b >> 16) & 0x8000u);
  const int exp = static_cast<int>((b >> 23) & 0xFFu);
  const uint32_t mant = b & 0x7FFFFFu;
  if (exp == 0xFF) return static_cast<uint16_t>(sign | 0x7C00u | (mant != 0 ? 1u : 0u));
  const int e = exp - 127 + 15;
  if (e >= 0x1F) return static_cast<uint16_t>(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return sign;
    const uint32_t m = mant | 0x800000u;
    const uint32_t shift = static_cast<uint32_t>(14 - e);
    const uint32_t half = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1);
    uint32_t hm = half;
    if (rem > halfway || (rem == halfway && (half & 1u))) hm += 1;
    return static_cast<uint16_t>(sign | hm);
  }
  uint32_t hm = (static_cast<uint32_t>(e) << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) hm += 1;
  return static_cast<uint16_t>(sign | hm);
}
static float f16_bits_to_f32(uint16_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t mant = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        mant <<= 1;
        ++e;
      } while (!(mant & 0x400u));
      bits = sign | (static_cast<uint32_t>(127 - 15 - e) << 23) | ((mant & 0x3FFu) << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (mant << 13);
  } else {
    bits = sign | ((exp - 15 + 127) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

extern "C" uint16_t lbrr_f32_to_f16_bits(float x) { return f32_to_f16_bits(x); }

// ---------------------------------------------------------------------------
// Model geometry
// ---------------------------------------------------------------------------
static const int kFreqs[kNumBands] = {2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,
                                      2,  2,  2,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  12, 12, 12, 12, 12, 12,
                                      12, 12, 24, 24, 24, 24, 24, 24, 24, 24, 48, 48, 48, 48, 48, 48, 48, 48, 128, 129};

struct BandGeom {
  int d[kNumBands], f0[kNumBands], offs[kNumBands + 1];
  int koff[kNumBands], kpad[kNumBands];  // xn / band-W column slots (multiples of 64)
  int n2pad[kNumBands], o2[kNumBands];   // permuted W2 rows per band (multiple of 16)
  int xn_cols, kpad_max, n2tot;
  BandGeom() {
    offs[0] = 0;
    int f = 0, ko = 0, o = 0;
    kpad_max = 0;
    for (int b = 0; b < kNumBands; ++b) {
      d[b] = 4 * kFreqs[b];
      f0[b] = f;
      f += kFreqs[b];
      offs[b + 1] = offs[b] + d[b];
      kpad[b] = (d[b] + 63) / 64 * 64;
      koff[b] = ko;
      ko += kpad[b];
      kpad_max = std::max(kpad_max, kpad[b]);
      n2pad[b] = (2 * d[b] + 15) / 16 * 16;
      o2[b] = o;
      o += n2pad[b];
    }
    xn_cols = ko;
    n2tot = o;
  }
};
static const BandGeom& geom() {
  static BandGeom g;
  return g;
}

// ---------------------------------------------------------------------------
// Engine
// ---------------------------------------------------------------------------
struct StepWeights {
  __half *wqkv, *wo, *w1, *w2;
  float *norm_g, *gate_w, *gate_b, *ff_g, *b1, *b2;
};

constexpr int kHostSlices = 8;  // slices of the stem download in lbrr_forward_chunk_host

// Threads kept by an engine for its host entry point: the copies between the
// caller's (pageable) buffers and pinned memory run on kHostWorkers threads,
// the calling thread being worker 0, without starting threads on every call.
constexpr int kHostWorkers = 4;
class HostPool {
 public:
  HostPool() {
    for (int w = 1; w < kHostWorkers; ++w) th_.emplace_back([this, w] { loop(w); });
  }
  ~HostPool() {
    {
      std::lock_guard<std::mutex> l(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
  }
  // f(w) for w = 0 .. kHostWorkers-1 (0 on the calling thread); returns once all are done
  void run(const std::function<void(int)>& f) {
    {
      std::lock_guard<std::mutex> l(m_);
      job_ = &f;
      pending_ = kHostWorkers - 1;
      ++gen_;
    }
    cv_.notify_all();
    f(0);
    std::unique_lock<std::mutex> l(m_);
    done_.wait(l, [&] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void loop(int w) {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void(int)>* f = nullptr;
      {
        std::unique_lock<std::mutex> l(m_);
        cv_.wait(l, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
        f = job_;
      }
      (*f)(w);
      {
        std::lock_guard<std::mutex> l(m_);
        --pending_;
      }
      done_.notify_one();
    }
  }
  std::vector<std::thread> th_;
  std::mutex m_;
  std::condition_variable cv_, done_;
  const std::function<void(int)>* job_ = nullptr;
  uint64_t gen_ = 0;
  int pending_ = 0;
  bool stop_ = false;
};

// Byte range [lo, hi) of worker w's share of n bytes (64-byte aligned cuts;
// the shares cover all n bytes whatever n mod kHostWorkers is).
static inline void host_share(size_t n, int w, size_t& lo, size_t& hi) {
  const size_t part = ((n + kHostWorkers - 1) / kHostWorkers + 63) / 64 * 64;
  lo = std::min(n, part * static_cast<size_t>(w));
  hi = std::min(n, lo + part);
}

struct lbrr_engine {
  int device = 0;
  cudaStream_t stream = nullptr;
  int64_t max_len = 0;
  int max_T = 0;
  bool weights_loaded = false;
  // weights
  void* warena = nullptr;
  size_t warena_bytes = 0;
  StepWeights steps[2 * kDepth];
  float *qkv_bias16 = nullptr, *out_bias = nullptr, *final_g = nullptr;
  __half* band_w = nullptr;
  float *band_b = nullptr, *band_g = nullptr;
  __half *mask_w1 = nullptr, *mask_w2 = nullptr;
  float *mask_b1 = nullptr, *mask_b2 = nullptr;
  int* band_tab = nullptr;  // [nb][8]: d, f0, koff, kpad, goff, o2, n2pad, 0
  int *band_f0 = nullptr, *band_d = nullptr, *band_o2 = nullptr;
  // per-length state
  int64_t cur_len = -1;
  int cur_T = -1;  // frames of one chunk
  int cur_B = 1;   // chunks batched along the frame axis (lbrr_forward_chunks)
  float *cos_t = nullptr, *sin_t = nullptr, *cos_f = nullptr, *sin_f = nullptr;
  TileDesc *tiles_band = nullptr, *tiles_m1 = nullptr, *tiles_m2 = nullptr;
  int n_band = 0, n_m1 = 0, n_m2 = 0;
  float* inv_env = nullptr;
  cufftHandle plan_r2c = 0, plan_c2r = 0;
  bool plans = false;
  // scratch
  void* sarena = nullptr;
  size_t sarena_bytes = 0;
  float *window = nullptr, *frames = nullptr, *x = nullptr, *gates = nullptr, *attn_out = nullptr, *pcm = nullptr;
  float2 *spec = nullptr, *c2r = nullptr;
  __half *xn = nullptr, *h16 = nullptr, *qkv = nullptr, *scaled = nullptr, *xb16 = nullptr,
         *hidden = nullptr;
  int* status = nullptr;
  // host staging for the end-to-end entry point
  float* pin_in = nullptr;
  float* pin_out = nullptr;
  float* dev_in = nullptr;
  float* dev_out = nullptr;
  // whole-song sharding (lbrr_separate_song): double-buffered pinned chunk
  // input and region output, the finished regions on the device (double-
  // buffered: a region's download runs on song_copy while the next chunk is
  // computed), the overlap strip this engine produces, and the strips it
  // receives (one per chunk)
  float* song_pin_in[2] = {nullptr, nullptr};
  float* song_pin_out[2] = {nullptr, nullptr};
  float* song_fin[2] = {nullptr, nullptr};
  cudaStream_t song_copy = nullptr;
  cudaEvent_t song_ev_reg[2] = {nullptr, nullptr};
  float* song_strip_out = nullptr;
  float* song_strip_in = nullptr;
  float* song_hann = nullptr;      // Hann fade table of the last Hann plan (song_hann_len samples)
  int64_t song_hann_len = 0;
  size_t song_strip_in_bytes = 0;
  cudaEvent_t song_ev_in[2] = {nullptr, nullptr};
  cudaEvent_t song_ev_out[2] = {nullptr, nullptr};
  // the chunk forward as a CUDA graph, for the last (input, output, length,
  // stream) seen twice in a row; replaying it saves the ~128 launch gaps
  cudaGraphExec_t graph = nullptr;
  const float* graph_x = nullptr;
  float* graph_out = nullptr;
  int64_t graph_len = -1;
  int graph_B = 0;
  cudaStream_t graph_stream = nullptr;
  int graph_seen = 0;
  // lbrr_forward_chunk_host with page-locked buffers: the forward up to the
  // mask estimator's first GEMM as a graph (for the last length seen twice in
  // a row), then per stem the second mask GEMM and the ISTFT, whose stems
  // download on host_copy while the next stem is computed
  cudaGraphExec_t head_graph = nullptr;
  int64_t head_len = -1;
  int head_seen = 0;
  cudaStream_t host_copy = nullptr;
  cudaEvent_t stem_ev[kStems] = {};
  // lbrr_forward_chunk_host: one event per downloaded slice of the stems, and
  // the host threads that copy them (started by the first call)
  cudaEvent_t host_ev[kHostSlices] = {};
  std::unique_ptr<HostPool> host_pool;
  float2* twiddles = nullptr;  // [2048] exp(+2 pi i k / 2048) for the in-house FFT
  bool pcm_valid = false;      // the last back end went through cuFFT and left "pcm"
  // options (lbrr_engine_set_option)
  bool keep_dc_imag = false;     // LBRR_OPT_DC_NYQUIST_IMAG
  int fft_backend = 0;           // LBRR_OPT_FFT_BACKEND
  int64_t song_fail_chunk = -1;  // LBRR_OPT_SONG_FAIL_CHUNK
  int64_t kernels_per_forward = 0;  // this library's launches in the last directly issued forward
  // host-side phase times of the last weight load and per-length setup (microseconds)
  int64_t us_read = 0, us_parse = 0, us_pack = 0, us_h2d = 0, us_setup = 0;
};

static int64_t us_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
}

// Called by the safetensors reader (safetensors.cpp) with the file-read and
// header-parse times of the load it is about to hand to lbrr_engine_load_weights.
extern "C" void lbrr_engine_note_file_times(lbrr_engine* e, int64_t us_read, int64_t us_parse) {
  if (!e) return;
  e->us_read = us_read;
  e->us_parse = us_parse;
}

namespace {
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Carver {
  size_t off = 0;
  template <class T>
  size_t take(size_t count) {
    off = align_up(off, 1024);
    const size_t o = off;
    off += count * sizeof(T);
    return o;
  }
};
}  // namespace

extern "C" const char* lbrr_last_error(void) { return g_err.c_str(); }
// Lets the host-only translation units (safetensors.cpp) report errors through
// the same thread-local message.
extern "C" int lbrr_set_error_for_host(int code, const char* msg) { return fail(code, msg ? msg : ""); }
extern "C" int lbrr_abi_version(void) { return 2; }

extern "C" int lbrr_host_alloc(size_t bytes, void** ptr) {
  if (!ptr) return fail(LBRR_ERR_INVALID, "lbrr_host_alloc: NULL ptr");
  *ptr = nullptr;
  if (bytes == 0) return fail(LBRR_ERR_INVALID, "lbrr_host_alloc: zero bytes");
  CK(cudaHostAlloc(ptr, bytes, cudaHostAllocPortable));
  return LBRR_OK;
}

extern "C" int lbrr_host_free(void* ptr) {
  if (!ptr) return LBRR_OK;
  CK(cudaFreeHost(ptr));
  return LBRR_OK;
}

extern "C" int lbrr_default_model(lbrr_model_desc* d, int32_t* freqs_out, int32_t capacity) {
  if (!d || !freqs_out || capacity < kNumBands) return fail(LBRR_ERR_INVALID, "lbrr_default_model: need 62 slots");
  for (int b = 0; b < kNumBands; ++b) freqs_out[b] = kFreqs[b];
  d->dim = kDim;
  d->depth = kDepth;
  d->heads = kHeads;
  d->dim_head = kDimHead;
  d->num_stems = kStems;
  d->mlp_expansion = 4;
  d->n_fft = kNfft;
  d->hop = kHop;
  d->sample_rate = 44100;
  d->num_bands = kNumBands;
  d->freqs_per_band = freqs_out;
  return LBRR_OK;
}

static int check_desc(const lbrr_model_desc* d) {
  if (!d) return LBRR_OK;  // NULL = the default model
  if (d->dim != kDim || d->depth != kDepth || d->heads != kHeads || d->dim_head != kDimHead ||
      d->num_stems != kStems || d->mlp_expansion != 4 || d->n_fft != kNfft || d->hop != kHop ||
      d->num_bands != kNumBands || !d->freqs_per_band)
    return fail(LBRR_ERR_INVALID, "unsupported model configuration (only the 62-band, 12-layer, dim-256 "
                                  "BS-RoFormer of logic_bs_roformer.yaml is built)");
  int sum = 0;
  for (int b = 0; b < kNumBands; ++b) {
    if (d->freqs_per_band[b] != kFreqs[b]) return fail(LBRR_ERR_INVALID, "unsupported freqs_per_band");
    sum += d->freqs_per_band[b];
  }
  if (sum != kBins) return fail(LBRR_ERR_INVALID, "freqs_per_band must sum to 1025");
  return LBRR_OK;
}

static int T_of(int64_t len) { return static_cast<int>(len / kHop + 1); }

// Placeholder base for laying out the weight arena before (or without) a device
// allocation; only differences from it are ever used.
static char* const kLayoutBase = reinterpret_cast<char*>(static_cast<uintptr_t>(1) << 30);

// Lay out the weight arena at base W (1024-aligned blocks) and point the
// engine's weight pointers into it; returns the arena size in bytes.
static size_t carve_weights(lbrr_engine* e, char* W) {
  const BandGeom& G = geom();
  Carver w;
  auto h16 = [&](size_t n) { return reinterpret_cast<__half*>(W + w.take<__half>(n)); };
  auto f32 = [&](size_t n) { return reinterpret_cast<float*>(W + w.take<float>(n)); };
  for (int k = 0; k < 2 * kDepth; ++k) {
    StepWeights& sw = e->steps[k];
    sw.wqkv = h16(1536 * 256);
    sw.wo = h16(256 * 512);
    sw.w1 = h16(1024 * 256);
    sw.w2 = h16(256 * 1024);
    sw.norm_g = f32(256);
    sw.gate_w = f32(8 * 256);
    sw.gate_b = f32(8);
    sw.ff_g = f32(256);
    sw.b1 = f32(1024);
    sw.b2 = f32(256);
  }
  e->qkv_bias16 = f32(1536);
  e->out_bias = f32(256);
  e->final_g = f32(256);
  e->band_w = h16(static_cast<size_t>(kNumBands) * 256 * G.kpad_max);
  e->band_b = f32(kNumBands * 256);
  e->band_g = f32(G.offs[kNumBands]);
  e->mask_w1 = h16(static_cast<size_t>(kStems) * kNumBands * 1024 * 256);
  e->mask_b1 = f32(static_cast<size_t>(kStems) * kNumBands * 1024);
  e->mask_w2 = h16(static_cast<size_t>(kStems) * G.n2tot * 1024);
  e->mask_b2 = f32(static_cast<size_t>(kStems) * G.n2tot);
  return align_up(w.off, 1024);
}

extern "C" int lbrr_engine_create(int device, const lbrr_model_desc* desc, int64_t max_len, lbrr_engine** out) {
  if (!out) return fail(LBRR_ERR_INVALID, "out is NULL");
  *out = nullptr;
  if (int rc = check_desc(desc)) return rc;
  if (max_len <= kNfft / 2 || max_len > (1ll << 26))
    return fail(LBRR_ERR_INVALID, "max_chunk_samples must be in (1024, 2^26]");
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(LBRR_ERR_INVALID, "device index out of range");
  DeviceGuard g(device);
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return fail(LBRR_ERR_INVALID, "this build targets sm_100a (B200); found sm_" +
                                                        std::to_string(prop.major) + std::to_string(prop.minor));
  lbrr_engine* e = new lbrr_engine();
  e->device = device;
  e->max_len = max_len;
  e->max_T = T_of(max_len);
  const BandGeom& G = geom();
  const size_t T = e->max_T, M = T * kNumBands;
  // ---- weights arena (sized first, pointers assigned after the allocation) ----
  e->warena_bytes = carve_weights(e, kLayoutBase);
  // ---- scratch arena ----
  Carver s;
  const size_t o_win = s.take<float>(kNfft), o_tw = s.take<float2>(2048), o_fr = s.take<float>(2 * T * kNfft),
               o_sp = s.take<float2>(2 * T * kBins);
  const size_t o_xn = s.take<__half>(T * G.xn_cols), o_x = s.take<float>(M * 256), o_h = s.take<__half>(M * 256);
  const size_t o_g = s.take<float>(M * 8), o_qkv = s.take<__half>(M * 1536), o_sc = s.take<__half>(M * 512);
  const size_t o_ao = s.take<float>(M * 256), o_xb = s.take<__half>(M * 256);
  const size_t o_hid = s.take<__half>(static_cast<size_t>(kStems) * M * 1024);
  const size_t o_c2r = s.take<float2>(static_cast<size_t>(2 * kStems) * T * kBins);
  const size_t o_pcm = s.take<float>(static_cast<size_t>(2 * kStems) * T * kNfft);
  const size_t o_st = s.take<int>(64);
  const size_t o_tab = s.take<int>(kNumBands * 8), o_f0 = s.take<int>(kNumBands), o_d = s.take<int>(kNumBands),
               o_o2 = s.take<int>(kNumBands);
  const size_t o_din = s.take<float>(2 * max_len), o_dout = s.take<float>(2 * kStems * max_len);
  e->sarena_bytes = align_up(s.off, 1024);

  auto cleanup = [&](int rc) {
    lbrr_engine_destroy(e);
    return rc;
  };
  cudaError_t ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
  if (ce == cudaSuccess) ce = cudaMalloc(&e->warena, e->warena_bytes);
  if (ce == cudaSuccess) ce = cudaMalloc(&e->sarena, e->sarena_bytes);
  if (ce == cudaSuccess) ce = cudaMemset(e->warena, 0, e->warena_bytes);
  if (ce == cudaSuccess) ce = cudaMemset(e->sarena, 0, e->sarena_bytes);
  if (ce == cudaSuccess) ce = cudaMallocHost(&e->pin_in, 2 * max_len * sizeof(float));
  if (ce == cudaSuccess) ce = cudaMallocHost(&e->pin_out, 2 * kStems * max_len * sizeof(float));
  if (ce != cudaSuccess) return cleanup(fail(LBRR_ERR_CUDA, std::string("engine allocation: ") + cudaGetErrorString(ce)));
  carve_weights(e, static_cast<char*>(e->warena));
  char* S = static_cast<char*>(e->sarena);
  e->band_tab = reinterpret_cast<int*>(S + o_tab);
  e->band_f0 = reinterpret_cast<int*>(S + o_f0);
  e->band_d = reinterpret_cast<int*>(S + o_d);
  e->band_o2 = reinterpret_cast<int*>(S + o_o2);
  e->window = reinterpret_cast<float*>(S + o_win);
  e->twiddles = reinterpret_cast<float2*>(S + o_tw);
  e->frames = reinterpret_cast<float*>(S + o_fr);
  e->spec = reinterpret_cast<float2*>(S + o_sp);
  e->xn = reinterpret_cast<__half*>(S + o_xn);
  e->x = reinterpret_cast<float*>(S + o_x);
  e->h16 = reinterpret_cast<__half*>(S + o_h);
  e->gates = reinterpret_cast<float*>(S + o_g);
  e->qkv = reinterpret_cast<__half*>(S + o_qkv);
  e->scaled = reinterpret_cast<__half*>(S + o_sc);
  e->attn_out = reinterpret_cast<float*>(S + o_ao);
  e->xb16 = reinterpret_cast<__half*>(S + o_xb);
  e->hidden = reinterpret_cast<__half*>(S + o_hid);
  e->c2r = reinterpret_cast<float2*>(S + o_c2r);
  e->pcm = reinterpret_cast<float*>(S + o_pcm);
  e->status = reinterpret_cast<int*>(S + o_st);
  e->dev_in = reinterpret_cast<float*>(S + o_din);
  e->dev_out = reinterpret_cast<float*>(S + o_dout);
  // constant tables: periodic Hann (f64 -> f32, src/stft.rs:25-29) and band geometry
  std::vector<float> win(kNfft);
  for (int i = 0; i < kNfft; ++i) win[i] = static_cast<float>(0.5 * (1.0 - std::cos(2.0 * M_PI * i / kNfft)));
  std::vector<int> tab(kNumBands * 8), f0(kNumBands), dd(kNumBands), o2(kNumBands);
  for (int b = 0; b < kNumBands; ++b) {
    int* r = &tab[b * 8];
    r[0] = G.d[b];
    r[1] = G.f0[b];
    r[2] = G.koff[b];
    r[3] = G.kpad[b];
    r[4] = G.offs[b];
    r[5] = G.o2[b];
    r[6] = G.n2pad[b];
    r[7] = 0;
    f0[b] = G.f0[b];
    dd[b] = G.d[b];
    o2[b] = G.o2[b];
  }
  std::vector<float2> tw(2048);
  for (int k = 0; k < 2048; ++k)
    tw[k] = make_float2(static_cast<float>(std::cos(2.0 * M_PI * k / 2048.0)),
                        static_cast<float>(std::sin(2.0 * M_PI * k / 2048.0)));
  ce = cudaMemcpy(e->window, win.data(), win.size() * 4, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMemcpy(e->twiddles, tw.data(), tw.size() * sizeof(float2), cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMemcpy(e->band_tab, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMemcpy(e->band_f0, f0.data(), f0.size() * 4, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMemcpy(e->band_d, dd.data(), dd.size() * 4, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMemcpy(e->band_o2, o2.data(), o2.size() * 4, cudaMemcpyHostToDevice);
  if (ce != cudaSuccess) return cleanup(fail(LBRR_ERR_CUDA, std::string("engine tables: ") + cudaGetErrorString(ce)));
  *out = e;
  return LBRR_OK;
}

extern "C" void lbrr_engine_destroy(lbrr_engine* e) {
  if (!e) return;
  DeviceGuard g(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  if (e->plans) {
    cufftDestroy(e->plan_r2c);
    cufftDestroy(e->plan_c2r);
  }
  cudaFree(e->cos_t);
  cudaFree(e->tiles_band);
  cudaFree(e->inv_env);
  cudaFree(e->warena);
  cudaFree(e->sarena);
  if (e->pin_in) cudaFreeHost(e->pin_in);
  if (e->pin_out) cudaFreeHost(e->pin_out);
  for (int i = 0; i < 2; ++i) {
    if (e->song_pin_in[i]) cudaFreeHost(e->song_pin_in[i]);
    if (e->song_pin_out[i]) cudaFreeHost(e->song_pin_out[i]);
    if (e->song_ev_in[i]) cudaEventDestroy(e->song_ev_in[i]);
    if (e->song_ev_out[i]) cudaEventDestroy(e->song_ev_out[i]);
    if (e->song_ev_reg[i]) cudaEventDestroy(e->song_ev_reg[i]);
    cudaFree(e->song_fin[i]);
  }
  if (e->song_copy) cudaStreamDestroy(e->song_copy);
  cudaFree(e->song_strip_out);
  cudaFree(e->song_strip_in);
  cudaFree(e->song_hann);
  if (e->graph) cudaGraphExecDestroy(e->graph);
  if (e->head_graph) cudaGraphExecDestroy(e->head_graph);
  for (auto& ev : e->stem_ev)
    if (ev) cudaEventDestroy(ev);
  if (e->host_copy) cudaStreamDestroy(e->host_copy);
  for (auto& ev : e->host_ev)
    if (ev) cudaEventDestroy(ev);
  e->host_pool.reset();
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

extern "C" int lbrr_engine_memory(const lbrr_engine* e, int64_t* wb, int64_t* sb) {
  if (!e) return fail(LBRR_ERR_INVALID, "engine is NULL");
  if (wb) *wb = static_cast<int64_t>(e->warena_bytes);
  if (sb) *sb = static_cast<int64_t>(e->sarena_bytes);
  return LBRR_OK;
}

// ---------------------------------------------------------------------------
// Weights
// ---------------------------------------------------------------------------
namespace {
struct ViewMap {
  std::map<std::string, const lbrr_weight_view*> m;
  std::map<std::string, int> used;
  std::string err;
  const float* take(const std::string& name, int64_t numel) {
    auto it = m.find(name);
    if (it == m.end()) {
      if (err.empty()) err = "missing tensor " + name;
      return nullptr;
    }
    if (used[name]++) {
      if (err.empty()) err = "duplicate key use: " + name;
      return nullptr;
    }
    if (it->second->numel != numel) {
      if (err.empty())
        err = name + ": len " + std::to_string(it->second->numel) + " != " + std::to_string(numel);
      return nullptr;
    }
    if (!it->second->data) {
      if (err.empty()) err = name + ": NULL data";
      return nullptr;
    }
    return it->second->data;
  }
};
void pack16(uint16_t* dst, const float* src, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = f32_to_f16_bits(src[i]);
}
}  // namespace

// Validate a checkpoint (every one of the 1989 keys exactly once with its exact
// size, shared biases bit-equal, analytic rotary freqs, no extra key;
// src/weights.rs:307-432) and build the packed host image of the weight arena
// whose pointers e holds relative to `base`.
static int build_weight_image(const lbrr_engine* e, const char* base, const lbrr_weight_view* views, size_t n,
                              std::vector<uint8_t>& host) {
  if (!views && n) return fail(LBRR_ERR_INVALID, "NULL views");
  const BandGeom& G = geom();
  ViewMap vm;
  for (size_t i = 0; i < n; ++i) {
    if (!views[i].name) return fail(LBRR_ERR_WEIGHTS, "weight view without a name");
    if (!vm.m.emplace(views[i].name, &views[i]).second)
      return fail(LBRR_ERR_WEIGHTS, std::string("duplicate tensor ") + views[i].name);
  }
  host.assign(e->warena_bytes, 0);
  auto hp = [&](const void* p) { return host.data() + (static_cast<const char*>(p) - base); };
  const float* sq = vm.take("linear_62_bias_0", 1536);
  const float* so = vm.take("linear_64_bias_0", 256);
  if (!vm.err.empty()) return fail(LBRR_ERR_WEIGHTS, vm.err);
  {
    float* qb = reinterpret_cast<float*>(hp(e->qkv_bias16));
    for (int i = 0; i < 1536; ++i) qb[i] = f16_bits_to_f32(f32_to_f16_bits(sq[i]));  // src/main.rs:5960-5962
    std::memcpy(hp(e->out_bias), so, 256 * 4);
  }
  for (int l = 0; l < kDepth; ++l) {
    for (int a = 0; a < 2; ++a) {
      const StepWeights& sw = e->steps[l * 2 + a];
      const std::string p = "layers." + std::to_string(l) + "." + std::to_string(a) + ".layers.0.0";
      const std::string fp = "layers." + std::to_string(l) + "." + std::to_string(a) + ".layers.0.1.net";
      const float* ng = vm.take(p + ".norm.gamma", 256);
      const float* wq = vm.take(p + ".to_qkv.weight", 1536 * 256);
      const float* wg = vm.take(p + ".to_gates.weight", 8 * 256);
      const float* bg = vm.take(p + ".to_gates.bias", 8);
      const float* wo = vm.take(p + ".to_out.0.weight", 256 * 512);
      const float* g0 = vm.take(fp + ".0.gamma", 256);
      const float* w1 = vm.take(fp + ".1.weight", 1024 * 256);
      const float* b1 = vm.take(fp + ".1.bias", 1024);
      const float* w2 = vm.take(fp + ".4.weight", 256 * 1024);
      const float* b2 = vm.take(fp + ".4.bias", 256);
      const float* qbias = vm.take(p + ".to_qkv.bias", 1536);
      const float* obias = vm.take(p + ".to_out.0.bias", 256);
      const float* freqs = vm.take(p + ".rotary_embed.freqs", 32);
      if (!vm.err.empty()) return fail(LBRR_ERR_WEIGHTS, vm.err);
      // shared biases must be byte-equal (src/weights.rs:362-372)
      if (std::memcmp(qbias, sq, 1536 * 4)) return fail(LBRR_ERR_WEIGHTS, p + ".to_qkv.bias != linear_62_bias_0");
      if (std::memcmp(obias, so, 256 * 4)) return fail(LBRR_ERR_WEIGHTS, p + ".to_out.0.bias != linear_64_bias_0");
      // rotary freqs analytic (src/weights.rs:375-382)
      for (int i = 0; i < 32; ++i) {
        const float want = 1.0f / std::pow(10000.0f, (2.0f * i) / 64.0f);
        if (!(std::fabs(freqs[i] - want) <= 1e-6f))
          return fail(LBRR_ERR_WEIGHTS, "rotary freqs[" + std::to_string(i) + "] != analytic in " + p);
      }
      pack16(reinterpret_cast<uint16_t*>(hp(sw.wqkv)), wq, 1536 * 256);
      pack16(reinterpret_cast<uint16_t*>(hp(sw.wo)), wo, 256 * 512);
      pack16(reinterpret_cast<uint16_t*>(hp(sw.w1)), w1, 1024 * 256);
      pack16(reinterpret_cast<uint16_t*>(hp(sw.w2)), w2, 256 * 1024);
      std::memcpy(hp(sw.norm_g), ng, 256 * 4);
      std::memcpy(hp(sw.gate_w), wg, 8 * 256 * 4);
      std::memcpy(hp(sw.gate_b), bg, 8 * 4);
      std::memcpy(hp(sw.ff_g), g0, 256 * 4);
      std::memcpy(hp(sw.b1), b1, 1024 * 4);
      std::memcpy(hp(sw.b2), b2, 256 * 4);
    }
  }
  const float* fg = vm.take("final_norm.gamma", 256);
  if (!vm.err.empty()) return fail(LBRR_ERR_WEIGHTS, vm.err);
  std::memcpy(hp(e->final_g), fg, 256 * 4);
  // band split: W [256][d_b] -> rows b*256+n, columns [0, d_b) of a kpad_max-wide slot
  for (int b = 0; b < kNumBands; ++b) {
    const std::string p = "band_split.to_features." + std::to_string(b);
    const int d = G.d[b];
    const float* gm = vm.take(p + ".0.gamma", d);
    const float* wb = vm.take(p + ".1.weight", 256 * d);
    const float* bb = vm.take(p + ".1.bias", 256);
    if (!vm.err.empty()) return fail(LBRR_ERR_WEIGHTS, vm.err);
    uint16_t* dst = reinterpret_cast<uint16_t*>(hp(e->band_w)) + static_cast<size_t>(b) * 256 * G.kpad_max;
    for (int nn = 0; nn < 256; ++nn) pack16(dst + static_cast<size_t>(nn) * G.kpad_max, wb + static_cast<size_t>(nn) * d, d);
    std::memcpy(reinterpret_cast<float*>(hp(e->band_b)) + b * 256, bb, 256 * 4);
    std::memcpy(reinterpret_cast<float*>(hp(e->band_g)) + G.offs[b], gm, d * 4);
  }
  // mask estimators: W1 [1024][256] per (stem, band); W2 rows interleaved (a_d, g_d)
  for (int s = 0; s < kStems; ++s) {
    for (int b = 0; b < kNumBands; ++b) {
      const std::string p = "mask_estimators." + std::to_string(s) + ".to_freqs." + std::to_string(b) + ".0";
      const int d = G.d[b];
      const float* w1 = vm.take(p + ".0.weight", 1024 * 256);
      const float* b1 = vm.take(p + ".0.bias", 1024);
      const float* w2 = vm.take(p + ".2.weight", static_cast<int64_t>(2 * d) * 1024);
      const float* b2 = vm.take(p + ".2.bias", 2 * d);
      if (!vm.err.empty()) return fail(LBRR_ERR_WEIGHTS, vm.err);
      const size_t grp = static_cast<size_t>(s) * kNumBands + b;
      pack16(reinterpret_cast<uint16_t*>(hp(e->mask_w1)) + grp * 1024 * 256, w1, 1024 * 256);
      std::memcpy(reinterpret_cast<float*>(hp(e->mask_b1)) + grp * 1024, b1, 1024 * 4);
      uint16_t* w2d = reinterpret_cast<uint16_t*>(hp(e->mask_w2)) + (static_cast<size_t>(s) * G.n2tot + G.o2[b]) * 1024;
      float* b2d = reinterpret_cast<float*>(hp(e->mask_b2)) + static_cast<size_t>(s) * G.n2tot + G.o2[b];
      for (int j = 0; j < G.n2pad[b]; ++j) {
        const int dd = j >> 1;
        if (dd < d) {
          const int src = (j & 1) ? d + dd : dd;
          pack16(w2d + static_cast<size_t>(j) * 1024, w2 + static_cast<size_t>(src) * 1024, 1024);
          b2d[j] = b2[src];
        }
      }
    }
  }
  // every checkpoint key consumed (src/weights.rs:428-432)
  for (auto& kv : vm.m)
    if (!vm.used.count(kv.first))
      return fail(LBRR_ERR_WEIGHTS, "unconsumed key " + kv.first);
  return LBRR_OK;
}

extern "C" int lbrr_engine_load_weights(lbrr_engine* e, const lbrr_weight_view* views, size_t n) {
  if (!e) return fail(LBRR_ERR_INVALID, "NULL engine");
  std::vector<uint8_t> host;
  e->us_read = e->us_parse = 0;
  auto t0 = std::chrono::steady_clock::now();
  if (int rc = build_weight_image(e, static_cast<const char*>(e->warena), views, n, host)) return rc;
  e->us_pack = us_since(t0);
  DeviceGuard g(e->device);
  t0 = std::chrono::steady_clock::now();
  CK(cudaMemcpy(e->warena, host.data(), host.size(), cudaMemcpyHostToDevice));
  e->us_h2d = us_since(t0);
  e->weights_loaded = true;
  return LBRR_OK;
}

extern "C" int lbrr_check_weights(const lbrr_weight_view* views, size_t n) {
  lbrr_engine layout;  // host-only: pointers laid out at a placeholder base, nothing allocated on a device
  layout.warena_bytes = carve_weights(&layout, kLayoutBase);
  std::vector<uint8_t> host;
  return build_weight_image(&layout, kLayoutBase, views, n, host);
}

// ---------------------------------------------------------------------------
// Per-length setup
// ---------------------------------------------------------------------------
static void rope_table(int P, std::vector<float>& c, std::vector<float>& s) {
  c.resize(static_cast<size_t>(P) * 32);
  s.resize(static_cast<size_t>(P) * 32);
  for (int p = 0; p < P; ++p)
    for (int i = 0; i < 32; ++i) {
      // angle in f64, rounded to f32, then cos/sin of that f32 (src/main.rs:7678-7681)
      const float a = static_cast<float>(p * (1.0 / std::pow(10000.0, 2.0 * i / 64.0)));
      c[p * 32 + i] = static_cast<float>(std::cos(static_cast<double>(a)));
      s[p * 32 + i] = static_cast<float>(std::sin(static_cast<double>(a)));
    }
}

static void drop_graph(lbrr_engine* e) {
  if (e->graph) cudaGraphExecDestroy(e->graph);
  e->graph = nullptr;
  e->graph_seen = 0;
  e->graph_len = -1;
  if (e->head_graph) cudaGraphExecDestroy(e->head_graph);
  e->head_graph = nullptr;
  e->head_seen = 0;
  e->head_len = -1;
}

// Frames of all chunks of the current forward (the row count of every
// frame-major buffer).
static int frames_all(const lbrr_engine* e) { return e->cur_T * e->cur_B; }

static int setup_length_impl(lbrr_engine* e, int64_t len, int B);
static int setup_length(lbrr_engine* e, int64_t len, int B = 1) {
  if (e->cur_len == len && e->cur_B == B) return LBRR_OK;
  const auto t0 = std::chrono::steady_clock::now();
  const int rc = setup_length_impl(e, len, B);
  e->us_setup = us_since(t0);
  return rc;
}

// Per-length tables for B chunks of len samples batched along the frame axis
// (B * T frames): the time-axis RoPE table repeats its T positions for every
// chunk, the grouped GEMMs' tile tables run over all B * T frames, the ISTFT
// envelope and the FFT plans are those of one chunk.
static int setup_length_impl(lbrr_engine* e, int64_t len, int B) {
  drop_graph(e);  // it refers to the per-length buffers released below
  const BandGeom& G = geom();
  const int T1 = T_of(len);
  const int T = T1 * B;  // frames of all chunks
  const int mt = (T + 127) / 128;
  // RoPE tables (time: T positions, freq: 62) -- one allocation for the tables,
  // tile tables follow in a second allocation, both released on the next change
  // the previous length's tables may still be read by queued work on any stream
  CK(cudaDeviceSynchronize());
  cudaFree(e->cos_t);
  cudaFree(e->tiles_band);
  cudaFree(e->inv_env);
  e->cos_t = nullptr;
  e->tiles_band = nullptr;
  e->inv_env = nullptr;
  std::vector<float> ct, st, cf, sf;
  {
    std::vector<float> c1, s1;
    rope_table(T1, c1, s1);
    for (int b = 0; b < B; ++b) {
      ct.insert(ct.end(), c1.begin(), c1.end());
      st.insert(st.end(), s1.begin(), s1.end());
    }
  }
  rope_table(kNumBands, cf, sf);
  float* tabs = nullptr;
  CK(cudaMalloc(&tabs, (2 * ct.size() + 2 * cf.size()) * sizeof(float)));
  e->cos_t = tabs;
  e->sin_t = tabs + ct.size();
  e->cos_f = tabs + 2 * ct.size();
  e->sin_f = tabs + 2 * ct.size() + cf.size();
  CK(cudaMemcpy(e->cos_t, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(e->sin_t, st.data(), st.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(e->cos_f, cf.data(), cf.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(e->sin_f, sf.data(), sf.size() * 4, cudaMemcpyHostToDevice));
  // grouped GEMM tile tables
  std::vector<TileDesc> tb, t1, t2;
  for (int b = 0; b < kNumBands; ++b)
    for (int m = 0; m < mt; ++m)
      tb.push_back({m * 128, G.koff[b], b * 256, G.kpad[b] / 64, 256, m * 128, std::min(128, T - m * 128), b});
  for (int s = 0; s < kStems; ++s)
    for (int b = 0; b < kNumBands; ++b)
      for (int m = 0; m < mt; ++m)
        for (int nt = 0; nt < 4; ++nt) {
          const int grp = s * kNumBands + b;
          t1.push_back({b * T + m * 128, 0, grp * 1024 + nt * 256, 4, 256, m * 128, std::min(128, T - m * 128),
                        grp * 4 + nt});
        }
  for (int s = 0; s < kStems; ++s)
    for (int b = 0; b < kNumBands; ++b)
      for (int m = 0; m < mt; ++m)
        for (int nt = 0; nt * 256 < G.n2pad[b]; ++nt) {
          const int grp = s * kNumBands + b;
          t2.push_back({grp * T + m * 128, 0, s * G.n2tot + G.o2[b] + nt * 256, 16,
                        std::min(256, G.n2pad[b] - nt * 256), m * 128, std::min(128, T - m * 128),
                        (s << 16) | (b << 8) | nt});
        }
  TileDesc* tiles = nullptr;
  CK(cudaMalloc(&tiles, (tb.size() + t1.size() + t2.size()) * sizeof(TileDesc)));
  e->tiles_band = tiles;
  e->tiles_m1 = tiles + tb.size();
  e->tiles_m2 = tiles + tb.size() + t1.size();
  e->n_band = static_cast<int>(tb.size());
  e->n_m1 = static_cast<int>(t1.size());
  e->n_m2 = static_cast<int>(t2.size());
  CK(cudaMemcpy(e->tiles_band, tb.data(), tb.size() * sizeof(TileDesc), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(e->tiles_m1, t1.data(), t1.size() * sizeof(TileDesc), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(e->tiles_m2, t2.data(), t2.size() * sizeof(TileDesc), cudaMemcpyHostToDevice));
  // ISTFT inverse window envelope over len + n_fft samples (benchmark::istft_inverse, src/benchmark.rs:129-142)
  {
    std::vector<float> win(kNfft), env(static_cast<size_t>(len) + kNfft, 0.f);
    for (int i = 0; i < kNfft; ++i) win[i] = static_cast<float>(0.5 * (1.0 - std::cos(2.0 * M_PI * i / kNfft)));
    for (int t = 0; t < T1; ++t)
      for (int nn = 0; nn < kNfft; ++nn) {
        const size_t p = static_cast<size_t>(t) * kHop + nn;
        if (p < env.size()) env[p] += win[nn] * win[nn];
      }
    for (auto& v : env) v = v > 1e-8f ? 1.0f / v : 0.f;
    CK(cudaMalloc(&e->inv_env, env.size() * sizeof(float)));
    CK(cudaMemcpy(e->inv_env, env.data(), env.size() * 4, cudaMemcpyHostToDevice));
  }
  // cuFFT plans (R2C batch 2T, src/stft.rs:36-45; C2R batch 12T), only for the
  // cuFFT back end or the reference's DC/Nyquist semantics
  const bool need_cufft = e->fft_backend == 1 || e->keep_dc_imag;
  if (!need_cufft && e->plans) {
    cufftDestroy(e->plan_r2c);
    cufftDestroy(e->plan_c2r);
    e->plans = false;
  }
  if (need_cufft && (e->cur_T != T1 || !e->plans)) {
    if (e->plans) {
      cufftDestroy(e->plan_r2c);
      cufftDestroy(e->plan_c2r);
      e->plans = false;
    }
    int n[1] = {kNfft};
    int inr[1] = {kNfft}, outc[1] = {kBins};
    CKFFT(cufftPlanMany(&e->plan_r2c, 1, n, inr, 1, kNfft, outc, 1, kBins, CUFFT_R2C, 2 * T1));
    CKFFT(cufftPlanMany(&e->plan_c2r, 1, n, outc, 1, kBins, inr, 1, kNfft, CUFFT_C2R, 2 * kStems * T1));
    e->plans = true;
  }
  e->cur_T = T1;
  e->cur_B = B;
  e->cur_len = len;
  return LBRR_OK;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
#define CKL(call)                                                                                  \
  do {                                                                                             \
    cudaError_t _e = (call);                                                                       \
    if (_e != cudaSuccess) return fail(LBRR_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(_e)); \
  } while (0)

// Pre-attention RMSNorm + gates of step k, fused into the producing GEMM epilogue.
static RowNorm attn_norm(lbrr_engine* e, int k) {
  RowNorm n;
  n.kind = 2;
  n.gamma = e->steps[k].norm_g;
  n.gate_w = e->steps[k].gate_w;
  n.gate_b = e->steps[k].gate_b;
  n.h16 = e->h16;
  n.gates = e->gates;
  return n;
}

static bool use_cufft_front(const lbrr_engine* e) { return e->fft_backend == 1; }
static bool use_cufft_back(const lbrr_engine* e) { return e->fft_backend == 1 || e->keep_dc_imag; }

static int run_front(lbrr_engine* e, const float* x, int64_t len, cudaStream_t st) {
  const BandGeom& G = geom();
  const int T = e->cur_T, Tall = frames_all(e);
  if (use_cufft_front(e)) {
    if (e->cur_B != 1) return fail(LBRR_ERR_STATE, "batched chunks need the in-house FFT");
    CKL(stft_frames(x, e->window, e->frames, static_cast<int>(len), T, st));
    CKFFT(cufftSetStream(e->plan_r2c, st));
    CKFFT(cufftExecR2C(e->plan_r2c, e->frames, reinterpret_cast<cufftComplex*>(e->spec)));
    CKL(band_norm(e->spec, e->band_g, e->band_tab, e->xn, G.xn_cols, T, kNumBands, st));
  } else {
    // framing + FFT + spectrum + band RMSNorm in one kernel
    CKL(stft_front(x, e->window, e->twiddles, e->spec, e->band_g, e->band_tab, e->xn, G.xn_cols,
                   static_cast<int>(len), T, kNumBands, e->cur_B, st));
  }
  // band split, fused with step 0's pre-attention RMSNorm + gates
  CKL(gemm_bandsplit(e->xn, G.xn_cols, e->band_w, G.kpad_max, e->band_b, e->x, Tall, kNumBands, e->tiles_band,
                     e->n_band, attn_norm(e, 0), e->status, st));
  return LBRR_OK;
}

// h16 + gates of step k come from the epilogue that produced x (band split or
// the previous step's FF2); after the last step that epilogue writes the final
// norm in band-major order instead.
static int run_step(lbrr_engine* e, int k, cudaStream_t st) {
  const int T = e->cur_T, Tall = frames_all(e), M = Tall * kNumBands, axis = k & 1;
  const StepWeights& w = e->steps[k];
  CKL(gemm_qkv(e->h16, w.wqkv, e->qkv_bias16, axis == 0 ? e->cos_t : e->cos_f, axis == 0 ? e->sin_t : e->sin_f,
               e->qkv, M, kNumBands, axis, e->status, st));
  CKL(attention_fwd(e->qkv, e->gates, e->scaled, T, kNumBands, axis, e->cur_B, e->status, st));
  CKL(gemm_outproj_norm(e->scaled, w.wo, e->out_bias, e->x, w.ff_g, e->attn_out, e->h16, M, e->status, st));
  RowNorm next;
  if (k + 1 < 2 * kDepth) {
    next = attn_norm(e, k + 1);
  } else {
    next.kind = 3;
    next.gamma = e->final_g;
    next.xb16 = e->xb16;
    next.T = Tall;
    next.nb = kNumBands;
  }
  // FF1 -> GELU -> FF2 + residual, the hidden activation kept on chip
  CKL(gemm_ff_fused(e->h16, w.w1, w.b1, w.w2, w.b2, e->attn_out, e->x, M, next, e->status, st));
  return LBRR_OK;
}

static int run_back(lbrr_engine* e, int64_t len, float* out, cudaStream_t st) {
  const BandGeom& G = geom();
  const int T = e->cur_T, Tall = frames_all(e);
  CKL(gemm_mask1(e->xb16, e->mask_w1, e->mask_b1, e->hidden, Tall, kStems * kNumBands, e->tiles_m1, e->n_m1,
                 e->status, st));
  CKL(gemm_mask2(e->hidden, e->mask_w2, e->mask_b2, e->band_f0, e->band_d, e->band_o2, e->spec, e->c2r, Tall, kStems,
                 G.n2tot, e->tiles_m2, e->n_m2, e->keep_dc_imag, e->status, st));
  if (use_cufft_back(e)) {
    if (e->cur_B != 1) return fail(LBRR_ERR_STATE, "batched chunks need the in-house FFT");
    CKFFT(cufftSetStream(e->plan_c2r, st));
    CKFFT(cufftExecC2R(e->plan_c2r, reinterpret_cast<cufftComplex*>(e->c2r), e->pcm));
    CKL(istft_ola(e->pcm, e->window, e->inv_env, out, static_cast<int>(len), T, 2 * kStems, st));
    e->pcm_valid = true;
  } else {
    // inverse FFT + window + overlap-add + envelope in one kernel
    CKL(istft_back(e->c2r, e->window, e->twiddles, e->inv_env, out, static_cast<int>(len), T, 2 * kStems, e->cur_B,
                   st));
    e->pcm_valid = false;
  }
  return LBRR_OK;
}

static int check_forward_args(lbrr_engine* e, const void* x, int64_t len, const void* out) {
  if (!e) return fail(LBRR_ERR_INVALID, "engine is NULL");
  if (!x || !out) return fail(LBRR_ERR_INVALID, "NULL buffer");
  if (!e->weights_loaded) return fail(LBRR_ERR_STATE, "weights not loaded");
  if (len <= kNfft / 2) return fail(LBRR_ERR_INVALID, "single-block input needs len > n_fft/2 (1024)");
  if (len > e->max_len) return fail(LBRR_ERR_INVALID, "len exceeds the engine's max_chunk_samples");
  return LBRR_OK;
}

static int run_forward(lbrr_engine* e, const float* x, int64_t len, float* out, cudaStream_t st) {
  const long long l0 = t_kernel_launches;
  if (int rc = run_front(e, x, len, st)) return rc;
  for (int k = 0; k < 2 * kDepth; ++k)
    if (int rc = run_step(e, k, st)) return rc;
  const int rc = run_back(e, len, out, st);
  e->kernels_per_forward = t_kernel_launches - l0;
  return rc;
}

// The forward up to the mask estimator's first GEMM (all stems), on x =
// e->dev_in: what precedes the per-stem back end of the page-locked host path.
static int run_head(lbrr_engine* e, int64_t len, cudaStream_t st) {
  if (int rc = run_front(e, e->dev_in, len, st)) return rc;
  for (int k = 0; k < 2 * kDepth; ++k)
    if (int rc = run_step(e, k, st)) return rc;
  CKL(gemm_mask1(e->xb16, e->mask_w1, e->mask_b1, e->hidden, frames_all(e), kStems * kNumBands, e->tiles_m1,
                 e->n_m1, e->status, st));
  return LBRR_OK;
}

// Per stem: the second mask GEMM over that stem's tiles (the tile table is
// stem-major), the ISTFT of its two channels into e->dev_out, and the
// download of those channels into outh on e->host_copy, which waits for the
// stem's event only, so stem s crosses PCIe while stem s+1 is computed.
static int run_tail_per_stem(lbrr_engine* e, int64_t len, float* outh, cudaStream_t st) {
  const BandGeom& G = geom();
  const int T = e->cur_T;
  if (e->cur_B != 1) return fail(LBRR_ERR_STATE, "the per-stem back end takes one chunk");
  const int per = e->n_m2 / kStems;
  const size_t chan = static_cast<size_t>(len);
  for (int s = 0; s < kStems; ++s) {
    CKL(gemm_mask2(e->hidden, e->mask_w2, e->mask_b2, e->band_f0, e->band_d, e->band_o2, e->spec, e->c2r, T, kStems,
                   G.n2tot, e->tiles_m2 + s * per, per, e->keep_dc_imag, e->status, st));
    CKL(istft_back(e->c2r + static_cast<size_t>(2 * s) * T * kBins, e->window, e->twiddles, e->inv_env,
                   e->dev_out + 2 * s * chan, static_cast<int>(len), T, 2, 1, st));
    CK(cudaEventRecord(e->stem_ev[s], st));
    CK(cudaStreamWaitEvent(e->host_copy, e->stem_ev[s], 0));
    CK(cudaMemcpyAsync(outh + 2 * s * chan, e->dev_out + 2 * s * chan, 2 * chan * sizeof(float),
                       cudaMemcpyDeviceToHost, e->host_copy));
  }
  e->pcm_valid = false;
  return LBRR_OK;
}

// The same launches captured into a graph on the caller's stream (not the
// legacy default stream, which cannot be captured).  Returns LBRR_OK with
// e->graph set, or an error after which the caller launches directly.
static int capture_forward(lbrr_engine* e, const float* x, int64_t len, float* out, cudaStream_t st) {
  cudaGraph_t graph = nullptr;
  if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    return LBRR_ERR_CUDA;
  }
  const int rc = run_forward(e, x, len, out, st);
  const cudaError_t ce = cudaStreamEndCapture(st, &graph);
  cudaGraphExec_t exec = nullptr;
  if (rc == LBRR_OK && ce == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
    e->graph = exec;
    e->graph_x = x;
    e->graph_out = out;
    e->graph_len = len;
    e->graph_stream = st;
  }
  if (graph) cudaGraphDestroy(graph);
  cudaGetLastError();
  return e->graph ? LBRR_OK : LBRR_ERR_CUDA;
}

// B chunks of len samples (x: B x [len][2], out: B x [6][2][len]) in one
// forward, replayed as a CUDA graph for the same (x, out, len, B, stream) on
// the second call in a row.
static int forward_device(lbrr_engine* e, const float* x, int64_t len, int B, float* out, cudaStream_t st) {
  if (int rc = setup_length(e, len, B)) return rc;
  const bool capturable = st != cudaStreamLegacy && st != cudaStreamPerThread && st != nullptr;
  if (capturable) {
    const bool same = e->graph_x == x && e->graph_out == out && e->graph_len == len && e->graph_B == B &&
                      e->graph_stream == st;
    if (e->graph && same) {
      CK(cudaGraphLaunch(e->graph, st));
      return LBRR_OK;
    }
    // capture on the second consecutive call with the same buffers: the first
    // one runs directly and performs every one-time setup outside a capture
    if (e->graph) cudaGraphExecDestroy(e->graph);
    e->graph = nullptr;
    if (same && e->graph_seen >= 1 && capture_forward(e, x, len, out, st) == LBRR_OK) {
      CK(cudaGraphLaunch(e->graph, st));
      return LBRR_OK;
    }
    e->graph_seen = same ? e->graph_seen + 1 : 1;
    e->graph_x = x;
    e->graph_out = out;
    e->graph_len = len;
    e->graph_B = B;
    e->graph_stream = st;
  }
  return run_forward(e, x, len, out, st);
}

extern "C" int lbrr_forward_chunk(lbrr_engine* e, const float* x, int64_t len, float* out, void* stream) {
  if (int rc = check_forward_args(e, x, len, out)) return rc;
  DeviceGuard g(e->device);
  return forward_device(e, x, len, 1, out, stream ? static_cast<cudaStream_t>(stream) : e->stream);
}

extern "C" int lbrr_forward_chunks(lbrr_engine* e, const float* x, int64_t len, int32_t n_chunks, float* out,
                                   void* stream) {
  if (int rc = check_forward_args(e, x, len, out)) return rc;
  if (n_chunks < 1) return fail(LBRR_ERR_INVALID, "n_chunks must be >= 1");
  if (static_cast<int64_t>(n_chunks) * T_of(len) > e->max_T)
    return fail(LBRR_ERR_INVALID, "n_chunks * (len / 512 + 1) frames exceed the engine's max_chunk_samples / 512 + 1");
  DeviceGuard g(e->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
  if (n_chunks == 1 || use_cufft_front(e) || use_cufft_back(e)) {
    // the cuFFT paths take one chunk per forward
    for (int c = 0; c < n_chunks; ++c)
      if (int rc = forward_device(e, x + 2 * c * len, len, 1, out + 2 * kStems * c * len, st)) return rc;
    return LBRR_OK;
  }
  return forward_device(e, x, len, n_chunks, out, st);
}

extern "C" int lbrr_forward_trunk(lbrr_engine* e, const float* x, int64_t len, int n_steps, float* x_out,
                                  void* stream) {
  if (int rc = check_forward_args(e, x, len, x_out)) return rc;
  if (n_steps < 0 || n_steps > 2 * kDepth) return fail(LBRR_ERR_INVALID, "n_steps must be in [0, 24]");
  DeviceGuard g(e->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
  if (int rc = setup_length(e, len)) return rc;
  if (int rc = run_front(e, x, len, st)) return rc;
  for (int k = 0; k < n_steps; ++k)
    if (int rc = run_step(e, k, st)) return rc;
  CK(cudaMemcpyAsync(x_out, e->x, static_cast<size_t>(frames_all(e)) * kNumBands * 256 * 4, cudaMemcpyDeviceToDevice,
                     st));
  return LBRR_OK;
}

extern "C" int lbrr_forward_back(lbrr_engine* e, int64_t len, float* stems_dev, void* stream) {
  if (!e || !stems_dev) return fail(LBRR_ERR_INVALID, "NULL argument");
  if (e->cur_len <= 0) return fail(LBRR_ERR_STATE, "no forward has run yet");
  if (len != e->cur_len) return fail(LBRR_ERR_STATE, "len differs from the last forward's");
  if (e->cur_B != 1) return fail(LBRR_ERR_STATE, "the last forward was a batch of chunks");
  DeviceGuard g(e->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
  return run_back(e, len, stems_dev, st);
}

static int check_status(int* status_dev, cudaStream_t st) {
  int h = 0;
  CK(cudaMemcpyAsync(&h, status_dev, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (h != 0) {
    cudaMemsetAsync(status_dev, 0, sizeof(int), st);
    cudaStreamSynchronize(st);
    return fail(LBRR_ERR_DEVICE, "kernel status " + std::to_string(h) +
                                     (h == kDevWaitTimeout ? " (pipeline wait timed out)" : "") +
                                     (h == kDevSmemMisaligned ? " (shared memory misaligned)" : ""));
  }
  return LBRR_OK;
}

extern "C" int lbrr_engine_read_buffer(lbrr_engine* e, const char* name, void* dst, int64_t bytes) {
  if (!e || !name || !dst || bytes < 0) return fail(LBRR_ERR_INVALID, "NULL argument");
  if (e->cur_T <= 0) return fail(LBRR_ERR_STATE, "no forward has run yet");
  DeviceGuard g(e->device);
  const size_t T = frames_all(e), M = T * kNumBands;
  const void* src = nullptr;
  size_t cap = 0;
  const std::string n(name);
  if (n == "spec") src = e->spec, cap = 2 * T * kBins * sizeof(float2);
  else if (n == "c2r") src = e->c2r, cap = 2 * kStems * T * kBins * sizeof(float2);
  else if (n == "pcm") {
    if (!e->pcm_valid)
      return fail(LBRR_ERR_STATE, "no \"pcm\" frames: the in-house back end fuses the inverse FFT with the "
                                  "overlap-add (select LBRR_OPT_FFT_BACKEND 1 to keep them)");
    src = e->pcm, cap = 2 * kStems * T * kNfft * sizeof(float);
  }
  else if (n == "x") src = e->x, cap = M * 256 * sizeof(float);
  else if (n == "xb16") src = e->xb16, cap = M * 256 * sizeof(__half);
  else if (n == "hidden") src = e->hidden, cap = kStems * M * 1024 * sizeof(__half);
  else return fail(LBRR_ERR_INVALID, "unknown buffer " + n);
  if (static_cast<size_t>(bytes) > cap) return fail(LBRR_ERR_INVALID, "read exceeds the buffer");
  CK(cudaStreamSynchronize(e->stream));
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpy(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToHost));
  return LBRR_OK;
}

extern "C" int lbrr_engine_sync(lbrr_engine* e) {
  if (!e) return fail(LBRR_ERR_INVALID, "engine is NULL");
  DeviceGuard g(e->device);
  CK(cudaStreamSynchronize(e->stream));
  return check_status(e->status, e->stream);
}

extern "C" int lbrr_engine_set_option(lbrr_engine* e, int option, int64_t value) {
  if (!e) return fail(LBRR_ERR_INVALID, "engine is NULL");
  switch (option) {
    case LBRR_OPT_DC_NYQUIST_IMAG:
      if (value != 0 && value != 1) return fail(LBRR_ERR_INVALID, "LBRR_OPT_DC_NYQUIST_IMAG takes 0 or 1");
      if (e->keep_dc_imag != (value == 1)) {
        DeviceGuard g(e->device);
        CK(cudaStreamSynchronize(e->stream));
        drop_graph(e);  // the captured launches carry the old setting
        e->keep_dc_imag = value == 1;
        e->cur_len = -1;  // the next forward redoes the per-length setup (cuFFT plans on demand)
      }
      return LBRR_OK;
    case LBRR_OPT_SONG_FAIL_CHUNK:
      if (value < -1) return fail(LBRR_ERR_INVALID, "LBRR_OPT_SONG_FAIL_CHUNK takes -1 or a chunk index");
      e->song_fail_chunk = value;
      return LBRR_OK;
    case LBRR_OPT_FFT_BACKEND:
      if (value != 0 && value != 1) return fail(LBRR_ERR_INVALID, "LBRR_OPT_FFT_BACKEND takes 0 or 1");
      if (e->fft_backend != value) {
        DeviceGuard g(e->device);
        CK(cudaStreamSynchronize(e->stream));
        drop_graph(e);
        e->fft_backend = static_cast<int>(value);
        e->cur_len = -1;  // the next forward redoes the per-length setup (cuFFT plans on demand)
      }
      return LBRR_OK;
    default:
      return fail(LBRR_ERR_INVALID, "unknown engine option " + std::to_string(option));
  }
}

extern "C" int lbrr_engine_get_option(const lbrr_engine* e, int option, int64_t* value) {
  if (!e || !value) return fail(LBRR_ERR_INVALID, "NULL argument");
  switch (option) {
    case LBRR_OPT_DC_NYQUIST_IMAG: *value = e->keep_dc_imag ? 1 : 0; return LBRR_OK;
    case LBRR_OPT_SONG_FAIL_CHUNK: *value = e->song_fail_chunk; return LBRR_OK;
    case LBRR_OPT_FFT_BACKEND: *value = e->fft_backend; return LBRR_OK;
    case LBRR_INFO_KERNELS_PER_FORWARD: *value = e->kernels_per_forward; return LBRR_OK;
    case LBRR_INFO_WEIGHTS_READ_US: *value = e->us_read; return LBRR_OK;
    case LBRR_INFO_WEIGHTS_PARSE_US: *value = e->us_parse; return LBRR_OK;
    case LBRR_INFO_WEIGHTS_PACK_US: *value = e->us_pack; return LBRR_OK;
    case LBRR_INFO_WEIGHTS_H2D_US: *value = e->us_h2d; return LBRR_OK;
    case LBRR_INFO_SETUP_US: *value = e->us_setup; return LBRR_OK;
    default: return fail(LBRR_ERR_INVALID, "unknown engine option " + std::to_string(option));
  }
}

// One CTA waits, through the bounded mbarrier wait every pipeline kernel uses,
// on a barrier whose phase nothing completes.  Nothing asynchronous is issued,
// so when the limit passes the CTA only records the timeout and returns.
__global__ void wait_probe_kernel(int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait(&bar, 0, &abort_flag, status, limit_ns);
    if (ok) report_status(status, kDevSmemMisaligned);  // cannot happen: nothing arrives
  }
  __syncthreads();
}

extern "C" int lbrr_engine_wait_probe(lbrr_engine* e, int64_t limit_ns) {
  if (!e) return fail(LBRR_ERR_INVALID, "engine is NULL");
  if (limit_ns < 1000000 || limit_ns > 10000000000ll)
    return fail(LBRR_ERR_INVALID, "limit_ns must be in [1 ms, 10 s]");
  DeviceGuard g(e->device);
  wait_probe_kernel<<<1, 32, 0, e->stream>>>(e->status, static_cast<unsigned long long>(limit_ns));
  CK(cudaGetLastError());
  return LBRR_OK;
}

// The stems leave the GPU in kHostSlices slices, each followed by an event;
// the engine's host threads copy every slice, a quarter each, from pinned
// memory into the caller's buffer as soon as it has arrived, so the host copy
// overlaps the rest of the download and the last slice's copy is short.  The
// input is staged into pinned memory by the same threads.
// Page-locked host memory (cudaHostAlloc / cudaHostRegister): checked at the
// first and the last byte of the range, the convention of CUDA host-copy
// callers (a range page-locked at both ends is taken to be one allocation).
static bool host_pinned(const void* p, size_t bytes) {
  auto pinned = [](const void* q) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
      cudaGetLastError();  // clear the sticky-free error of an unknown pointer
      return false;
    }
    return a.type == cudaMemoryTypeHost;
  };
  return bytes > 0 && pinned(p) && pinned(static_cast<const char*>(p) + bytes - 1);
}

extern "C" int lbrr_forward_chunk_host(lbrr_engine* e, const float* xh, int64_t len, float* outh) {
  if (int rc = check_forward_args(e, xh, len, outh)) return rc;
  DeviceGuard g(e->device);
  const size_t in_b = static_cast<size_t>(len) * 2 * sizeof(float);
  const size_t out_b = static_cast<size_t>(len) * 2 * kStems * sizeof(float);
  if (host_pinned(xh, in_b) && host_pinned(outh, out_b)) {
    // both buffers page-locked: the copy engines read and write them directly
    if (int rc = setup_length(e, len)) return rc;
    CK(cudaMemcpyAsync(e->dev_in, xh, in_b, cudaMemcpyHostToDevice, e->stream));
    if (use_cufft_back(e) || e->n_m2 % kStems != 0) {
      // the cuFFT back end inverts all channels in one plan: one download at the end
      if (int rc = lbrr_forward_chunk(e, e->dev_in, len, e->dev_out, e->stream)) return rc;
      CK(cudaMemcpyAsync(outh, e->dev_out, out_b, cudaMemcpyDeviceToHost, e->stream));
      CK(cudaStreamSynchronize(e->stream));
      return check_status(e->status, e->stream);
    }
    if (!e->host_copy) CK(cudaStreamCreateWithFlags(&e->host_copy, cudaStreamNonBlocking));
    for (auto& ev : e->stem_ev)
      if (!ev) CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    // the forward up to the first mask GEMM: replayed from a graph once the
    // same length comes twice in a row (the first call runs every one-time
    // setup outside a capture)
    if (!(e->head_graph && e->head_len == len)) {
      const bool same = e->head_len == len;
      if (e->head_graph) cudaGraphExecDestroy(e->head_graph);
      e->head_graph = nullptr;
      if (same && e->head_seen >= 1 &&
          cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        cudaGraph_t graph = nullptr;
        const int rc = run_head(e, len, e->stream);
        const cudaError_t ce = cudaStreamEndCapture(e->stream, &graph);
        cudaGraphExec_t exec = nullptr;
        if (rc == LBRR_OK && ce == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess)
          e->head_graph = exec;
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
      }
      e->head_seen = same ? e->head_seen + 1 : 1;
      e->head_len = len;
    }
    if (e->head_graph) {
      CK(cudaGraphLaunch(e->head_graph, e->stream));
    } else if (int rc = run_head(e, len, e->stream)) {
      return rc;
    }
    if (int rc = run_tail_per_stem(e, len, outh, e->stream)) return rc;
    CK(cudaStreamSynchronize(e->host_copy));
    return check_status(e->status, e->stream);
  }
  for (auto& ev : e->host_ev)
    if (!ev) CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  const bool threaded = out_b >= (4u << 20);
  if (threaded && !e->host_pool) e->host_pool = std::make_unique<HostPool>();
  if (threaded) {
    e->host_pool->run([&](int w) {
      size_t lo, hi;
      host_share(in_b, w, lo, hi);
      if (hi > lo)
        std::memcpy(reinterpret_cast<char*>(e->pin_in) + lo, reinterpret_cast<const char*>(xh) + lo, hi - lo);
    });
  } else {
    std::memcpy(e->pin_in, xh, in_b);
  }
  CK(cudaMemcpyAsync(e->dev_in, e->pin_in, in_b, cudaMemcpyHostToDevice, e->stream));
  if (int rc = lbrr_forward_chunk(e, e->dev_in, len, e->dev_out, e->stream)) return rc;
  const size_t slice = (out_b / kHostSlices + 255) / 256 * 256;
  int slices = 0;
  for (size_t o = 0; o < out_b; o += slice, ++slices) {
    const size_t n = std::min(slice, out_b - o);
    CK(cudaMemcpyAsync(reinterpret_cast<char*>(e->pin_out) + o, reinterpret_cast<const char*>(e->dev_out) + o, n,
                       cudaMemcpyDeviceToHost, e->stream));
    CK(cudaEventRecord(e->host_ev[slices], e->stream));
  }
  std::atomic<int> copy_err{0};
  auto copy_slices = [&](int w) {
    for (int i = 0; i < slices; ++i) {
      if (cudaEventSynchronize(e->host_ev[i]) != cudaSuccess) {
        copy_err.store(1);
        return;
      }
      const size_t o = static_cast<size_t>(i) * slice, n = std::min(slice, out_b - o);
      size_t lo = 0, hi = n;
      if (threaded) host_share(n, w, lo, hi);
      if (hi > lo)
        std::memcpy(reinterpret_cast<char*>(outh) + o + lo, reinterpret_cast<const char*>(e->pin_out) + o + lo,
                    hi - lo);
    }
  };
  if (threaded)
    e->host_pool->run(copy_slices);
  else
    copy_slices(0);
  if (int rc = check_status(e->status, e->stream)) return rc;
  if (copy_err.load()) return fail(LBRR_ERR_CUDA, "stem download");
  return LBRR_OK;
}

// ---------------------------------------------------------------------------
// Whole song
// ---------------------------------------------------------------------------
__global__ void ola_accumulate_kernel(const float* __restrict__ y, float* __restrict__ result,
                                      float* __restrict__ counter, long long out_len, long long s, int take, int c,
                                      int border, int is_first, int is_last, int chunk_stride, int channels,
                                      const float* __restrict__ hann) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= take) return;
  float wf = 1.0f;
  if (hann) {
    wf = hann[j];
  } else {
    if (j < border) wf = static_cast<float>(j) / static_cast<float>(border);
    const int j2 = c - 1 - j;
    if (j2 < border) wf = static_cast<float>(j2) / static_cast<float>(border);
  }
  if (is_first && j < border) wf = 1.0f;
  if (is_last && j + border >= c) wf = 1.0f;
  counter[s + j] += wf * wf;
  for (int sc = 0; sc < channels; ++sc) result[sc * out_len + s + j] += y[static_cast<long long>(sc) * chunk_stride + j] * wf;
}

__global__ void ola_finalize_kernel(const float* __restrict__ result, const float* __restrict__ counter,
                                    float* __restrict__ out, long long out_len, long long border, long long len,
                                    int channels) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= channels * len) return;
  const long long sc = i / len, k = i % len;
  const float c = counter[border + k];
  out[i] = result[sc * out_len + border + k] / fmaxf(c, 1e-8f);
}

namespace {
std::vector<int64_t> chunk_starts(int64_t len, int64_t chunk, int64_t step, int64_t border) {
  std::vector<int64_t> v;
  const int64_t needed = border + len;
  const int64_t last = std::max<int64_t>(0, (needed - chunk + step - 1) / step);
  for (int64_t i = 0; i <= last; ++i) v.push_back(i * step);
  return v;
}
}  // namespace

namespace {
std::vector<float> hann_window_host(int64_t C);
int ensure_song_hann(lbrr_engine* e, const std::vector<float>& w);
}  // namespace

// Plans whose chunks overlap by more than half (a sample in three or more
// chunks): every waveform is accumulated on engine 0 in chunk order.
static int separate_song_serial(lbrr_engine* const* engines, int n, const float* xh, int64_t len,
                                const lbrr_chunk_plan& P, float* outh) {
  const auto starts = chunk_starts(len, P.chunk, P.step, P.border);
  const int64_t needed = P.border + len;
  const int64_t right = starts.back() + P.chunk - needed;
  const int64_t C = P.chunk;
  // reflect pad (tools/bench_ref.py:39-45), interleaved
  std::vector<float> xp(static_cast<size_t>(P.border + len + right) * 2);
  for (int64_t i = 0; i < P.border + len + right; ++i) {
    int64_t src;
    if (len == 1) {
      src = 0;
    } else {
      const int64_t period = 2 * (len - 1);
      int64_t p = (i - P.border) % period;
      if (p < 0) p += period;
      src = p < len ? p : period - p;
    }
    xp[2 * i] = xh[2 * src];
    xp[2 * i + 1] = xh[2 * src + 1];
  }
  lbrr_engine* e0 = engines[0];
  const int channels = 2 * kStems;
  if (P.fade == LBRR_FADE_HANN) {
    DeviceGuard g(e0->device);
    if (int rc = ensure_song_hann(e0, hann_window_host(P.chunk))) return rc;
  }
  const size_t ybytes = static_cast<size_t>(channels) * C * sizeof(float);
  float *result = nullptr, *counter = nullptr, *stage = nullptr, *fin = nullptr;
  std::vector<cudaEvent_t> ev_done(n, nullptr), ev_used(n, nullptr);
  int rc = LBRR_OK;
  {
    DeviceGuard g(e0->device);
    CK(cudaMalloc(&result, static_cast<size_t>(channels) * needed * sizeof(float)));
    CK(cudaMalloc(&counter, static_cast<size_t>(needed) * sizeof(float)));
    CK(cudaMalloc(&stage, ybytes));
    CK(cudaMalloc(&fin, static_cast<size_t>(channels) * len * sizeof(float)));
    CK(cudaMemsetAsync(result, 0, static_cast<size_t>(channels) * needed * sizeof(float), e0->stream));
    CK(cudaMemsetAsync(counter, 0, static_cast<size_t>(needed) * sizeof(float), e0->stream));
  }
  for (int i = 0; rc == LBRR_OK && i < n; ++i) {
    // ev_done[i] is recorded on engine i's stream, ev_used[i] on the stitching
    // stream of engine 0: an event lives on the device whose streams record it
    {
      DeviceGuard g0(e0->device);
      if (cudaEventCreateWithFlags(&ev_used[i], cudaEventDisableTiming) != cudaSuccess)
        rc = fail(LBRR_ERR_CUDA, "event create");
    }
    DeviceGuard g(engines[i]->device);
    if (cudaEventCreateWithFlags(&ev_done[i], cudaEventDisableTiming) != cudaSuccess)
      rc = fail(LBRR_ERR_CUDA, "event create");
    if (i > 0 && engines[i]->device != e0->device) {
      // direct NVLink copies when peer access exists; otherwise cudaMemcpyPeerAsync
      // stages through host memory on its own
      int can = 0;
      cudaDeviceCanAccessPeer(&can, e0->device, engines[i]->device);
      if (can) {
        DeviceGuard g0(e0->device);
        const cudaError_t pe = cudaDeviceEnablePeerAccess(engines[i]->device, 0);
        if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled)
          rc = fail(LBRR_ERR_PEER, std::string("enable peer access: ") + cudaGetErrorString(pe));
        cudaGetLastError();
      }
    }
  }
  for (size_t ci = 0; rc == LBRR_OK && ci < starts.size(); ++ci) {
    lbrr_engine* e = engines[ci % n];
    const int slot = static_cast<int>(ci % n);
    const int64_t s = starts[ci];
    {
      DeviceGuard g(e->device);
      // the input staging slot and dev_out of this engine are free once the
      // previous chunk's waveform was consumed by the stitching stream
      if (cudaStreamWaitEvent(e->stream, ev_used[slot], 0) != cudaSuccess) { rc = fail(LBRR_ERR_CUDA, "stream wait"); break; }
      if (cudaStreamSynchronize(e->stream) != cudaSuccess) { rc = fail(LBRR_ERR_CUDA, "stream sync"); break; }
      std::memcpy(e->pin_in, xp.data() + 2 * s, static_cast<size_t>(C) * 2 * sizeof(float));
      if (cudaMemcpyAsync(e->dev_in, e->pin_in, static_cast<size_t>(C) * 2 * sizeof(float), cudaMemcpyHostToDevice,
                          e->stream) != cudaSuccess) { rc = fail(LBRR_ERR_CUDA, "H2D chunk"); break; }
      if (e->song_fail_chunk == static_cast<int64_t>(ci)) {  // host-side failure injection
        rc = fail(LBRR_ERR_STATE, "injected failure before the forward of chunk " + std::to_string(ci));
        break;
      }
      if ((rc = lbrr_forward_chunk(e, e->dev_in, C, e->dev_out, e->stream)) != LBRR_OK) break;
      if (cudaEventRecord(ev_done[slot], e->stream) != cudaSuccess) { rc = fail(LBRR_ERR_CUDA, "event record"); break; }
    }
    {
      DeviceGuard g(e0->device);
      if (cudaStreamWaitEvent(e0->stream, ev_done[slot], 0) != cudaSuccess) { rc = fail(LBRR_ERR_CUDA, "stream wait"); break; }
      const float* y = e->dev_out;
      if (e != e0) {
        if (cudaMemcpyPeerAsync(stage, e0->device, e->dev_out, e->device, ybytes, e0->stream) != cudaSuccess) {
          rc = fail(LBRR_ERR_PEER, "peer copy of a chunk waveform failed");
          break;
        }
        y = stage;
      }
      const int take = static_cast<int>(std::min<int64_t>(C, needed - s));
      ola_accumulate_kernel<<<(take + 255) / 256, 256, 0, e0->stream>>>(
          y, result, counter, needed, s, take, static_cast<int>(C), static_cast<int>(P.border), ci == 0,
          ci + 1 == starts.size(), static_cast<int>(C), channels, P.fade == LBRR_FADE_HANN ? e0->song_hann : nullptr);
      if (cudaGetLastError() != cudaSuccess) { rc = fail(LBRR_ERR_CUDA, "ola accumulate launch"); break; }
      if (cudaEventRecord(ev_used[slot], e0->stream) != cudaSuccess) { rc = fail(LBRR_ERR_CUDA, "event record"); break; }
    }
  }
  if (rc == LBRR_OK) {
    DeviceGuard g(e0->device);
    const long long total = static_cast<long long>(channels) * len;
    ola_finalize_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, e0->stream>>>(
        result, counter, fin, needed, P.border, len, channels);
    std::vector<float> cnt(static_cast<size_t>(len));
    cudaMemcpyAsync(cnt.data(), counter + P.border, static_cast<size_t>(len) * 4, cudaMemcpyDeviceToHost, e0->stream);
    cudaMemcpyAsync(outh, fin, static_cast<size_t>(total) * 4, cudaMemcpyDeviceToHost, e0->stream);
    for (int i = 0; i < n && rc == LBRR_OK; ++i) {
      DeviceGuard g2(engines[i]->device);
      rc = check_status(engines[i]->status, engines[i]->stream);
    }
    if (rc == LBRR_OK) {
      if (cudaStreamSynchronize(e0->stream) != cudaSuccess) rc = fail(LBRR_ERR_CUDA, "final sync");
      // demix counter must cover every output sample (src/main.rs:7776)
      for (int64_t i = 0; rc == LBRR_OK && i < len; ++i)
        if (!(cnt[i] > 1e-8f)) rc = fail(LBRR_ERR_STATE, "demix has uncovered output samples");
    }
  }
  for (int i = 0; i < n; ++i) {
    DeviceGuard g(engines[i]->device);
    cudaStreamSynchronize(engines[i]->stream);
    if (ev_done[i]) cudaEventDestroy(ev_done[i]);
  }
  {
    DeviceGuard g(e0->device);
    cudaStreamSynchronize(e0->stream);
    for (int i = 0; i < n; ++i)
      if (ev_used[i]) cudaEventDestroy(ev_used[i]);
  }
  {
    DeviceGuard g(e0->device);
    cudaFree(result);
    cudaFree(counter);
    cudaFree(stage);
    cudaFree(fin);
  }
  return rc;
}

// ---------------------------------------------------------------------------
// Per-op entry points
// ---------------------------------------------------------------------------
// Whole song, sharded (every sample in at most two chunks: 2 * step >= chunk)
// ---------------------------------------------------------------------------
// Chunk c (padded offset s_c) belongs to engine c % n.  That engine produces
// the song samples [s_c - border, s_{c+1} - border) (the first chunk from 0,
// the last to the end): its head, where chunk c-1 also contributes, and the
// part no other chunk covers.  The previous chunk's contribution to the head
// arrives as an overlap strip y*w | w*w of (chunk - step) samples, copied
// device to device (NVLink when the engines sit on different GPUs); nothing
// else crosses devices.  Each sample is then
//   (0 + y_{c-1} w_{c-1} + y_c w_c) / max(0 + w_{c-1}^2 + w_c^2, 1e-8)
// with every product and sum rounded on its own, in chunk order: the same
// fp32 operations, in the same order, as accumulating all chunks one after
// the other (tools/bench_ref.py:47-65; IEEE addition is commutative, so the
// two-term sums match exactly).  Each engine's host thread prepares its chunk
// inputs (reflect padding at the song edges), drives its GPU, and copies its
// finished regions into the caller's planar output.
namespace {
struct SongGeom {
  int64_t C, step, border, ov, len;
  int nc;
  const float* hann = nullptr;  // LBRR_FADE_HANN: [C] periodic Hann window on this engine's device
  __device__ float fade(int64_t rel, int c) const {
    if (hann) {
      // Hann-weighted chunks; the first chunk keeps its leading border, the last its trailing border
      if ((rel < border && c == 0) || (rel >= C - border && c == nc - 1)) return 1.0f;
      return hann[rel];
    }
    // linear fade of width border; the first chunk keeps its leading edge, the last its trailing edge
    if (rel < border && c != 0) return static_cast<float>(rel) / static_cast<float>(border);
    if (rel >= C - border && c != nc - 1) return static_cast<float>(C - 1 - rel) / static_cast<float>(border);
    return 1.0f;
  }
};

// Periodic Hann window of the chunk length, computed in double and rounded to
// fp32 (the song plan of BASELINE config 4).
std::vector<float> hann_window_host(int64_t C) {
  std::vector<float> w(static_cast<size_t>(C));
  for (int64_t i = 0; i < C; ++i)
    w[i] = static_cast<float>(0.5 * (1.0 - std::cos(2.0 * M_PI * static_cast<double>(i) / static_cast<double>(C))));
  return w;
}

// Overlap strip of chunk c: relative samples [step, C): 12 channels of y*w, then w*w.
__global__ void song_strip_kernel(const float* __restrict__ y, float* __restrict__ strip, SongGeom g, int c) {
  const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (j >= g.ov) return;
  const int64_t rel = g.step + j;
  const float w = g.fade(rel, c);
  for (int ch = 0; ch < 2 * kStems; ++ch) strip[ch * g.ov + j] = __fmul_rn(y[ch * g.C + rel], w);
  strip[2 * kStems * g.ov + j] = __fmul_rn(w, w);
}

// Finished song samples of chunk c: relative samples [r0, r0 + n), the first
// `head` of them also carrying the previous chunk's strip.
__global__ void song_region_kernel(const float* __restrict__ y, const float* __restrict__ strip_prev,
                                   float* __restrict__ fin, SongGeom g, int c, int64_t r0, int64_t n, int64_t head) {
  const int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const int64_t rel = r0 + j;
  const float w = g.fade(rel, c);
  float den = __fmul_rn(w, w);
  const bool both = rel < head;
  if (both) den = __fadd_rn(strip_prev[2 * kStems * g.ov + rel], den);
  den = fmaxf(den, 1e-8f);
  for (int ch = 0; ch < 2 * kStems; ++ch) {
    float num = __fmul_rn(y[ch * g.C + rel], w);
    if (both) num = __fadd_rn(strip_prev[ch * g.ov + rel], num);
    fin[ch * n + j] = __fdiv_rn(num, den);
  }
}

struct SongRun {
  std::atomic<int> abort{0};
  std::mutex mu;
  std::condition_variable cv;
  std::vector<int> strip_ready;      // chunk c's strip is recorded in strip_ev[c]
  std::vector<cudaEvent_t> strip_ev;  // created on the producing engine's device
  std::vector<int> rc;
  std::vector<std::string> msg;
  // caller buffers that are page-locked: interior chunks are uploaded from the
  // song itself, finished regions are downloaded straight into the output
  bool direct_in = false, direct_out = false;
};

// The Hann fade table on engine e's device (current device), uploaded once per chunk length.
int ensure_song_hann(lbrr_engine* e, const std::vector<float>& w) {
  const int64_t C = static_cast<int64_t>(w.size());
  if (e->song_hann && e->song_hann_len == C) return LBRR_OK;
  cudaFree(e->song_hann);
  e->song_hann = nullptr;
  e->song_hann_len = 0;
  CK(cudaMalloc(&e->song_hann, w.size() * sizeof(float)));
  CK(cudaMemcpy(e->song_hann, w.data(), w.size() * sizeof(float), cudaMemcpyHostToDevice));
  e->song_hann_len = C;
  return LBRR_OK;
}

int ensure_song_buffers(lbrr_engine* e, const SongGeom& g) {
  const size_t in_b = static_cast<size_t>(g.C) * 2 * sizeof(float);
  const size_t out_b = static_cast<size_t>(g.C) * 2 * kStems * sizeof(float);
  const size_t strip_b = static_cast<size_t>(2 * kStems + 1) * g.ov * sizeof(float);
  if (!e->song_fin[0]) {
    // sized for the largest chunk this engine takes
    const size_t max_in = static_cast<size_t>(e->max_len) * 2 * sizeof(float);
    const size_t max_out = static_cast<size_t>(e->max_len) * 2 * kStems * sizeof(float);
    const size_t max_strip = static_cast<size_t>(2 * kStems + 1) * (e->max_len / 2 + 1) * sizeof(float);
    for (int i = 0; i < 2; ++i) {
      CK(cudaMallocHost(&e->song_pin_in[i], max_in));
      CK(cudaMallocHost(&e->song_pin_out[i], max_out));
      CK(cudaEventCreateWithFlags(&e->song_ev_in[i], cudaEventDisableTiming));
      CK(cudaEventCreateWithFlags(&e->song_ev_out[i], cudaEventDisableTiming));
      CK(cudaEventCreateWithFlags(&e->song_ev_reg[i], cudaEventDisableTiming));
      CK(cudaMalloc(&e->song_fin[i], max_out));
    }
    CK(cudaStreamCreateWithFlags(&e->song_copy, cudaStreamNonBlocking));
    CK(cudaMalloc(&e->song_strip_out, max_strip));
  }
  (void)in_b;
  (void)out_b;
  const size_t need = strip_b * static_cast<size_t>(g.nc);
  if (e->song_strip_in_bytes < need) {
    cudaFree(e->song_strip_in);
    e->song_strip_in = nullptr;
    e->song_strip_in_bytes = 0;
    CK(cudaMalloc(&e->song_strip_in, need));
    e->song_strip_in_bytes = need;
  }
  return LBRR_OK;
}

void song_worker(lbrr_engine* const* engines, int n, int me, const float* xh, float* outh, SongGeom g,
                 const std::vector<int64_t>& starts, SongRun& run) {
  lbrr_engine* e = engines[me];
  DeviceGuard dg(e->device);
  if (g.hann) g.hann = e->song_hann;  // this engine's copy of the fade table
  const size_t strip_b = static_cast<size_t>(2 * kStems + 1) * g.ov * sizeof(float);
  auto bail = [&](int rc) {
    run.rc[me] = rc;
    run.msg[me] = lbrr_last_error();
    run.abort.store(1);
    run.cv.notify_all();
  };
  if (int rc = ensure_song_buffers(e, g)) return bail(rc);
  // deferred host copy of the previous region (slot, song offset, length)
  int pend_slot = -1;
  int64_t pend_o0 = 0, pend_n = 0;
  auto scatter = [&]() -> int {
    if (pend_slot < 0) return LBRR_OK;
    if (cudaEventSynchronize(e->song_ev_out[pend_slot]) != cudaSuccess) return fail(LBRR_ERR_CUDA, "region copy");
    const float* src = e->song_pin_out[pend_slot];
    for (int ch = 0; ch < 2 * kStems; ++ch)
      std::memcpy(outh + static_cast<size_t>(ch) * g.len + pend_o0, src + static_cast<size_t>(ch) * pend_n,
                  static_cast<size_t>(pend_n) * sizeof(float));
    pend_slot = -1;
    return LBRR_OK;
  };
  int k = 0;
  for (int c = me; c < g.nc; c += n, ++k) {
    if (run.abort.load()) return;
    const int slot = k & 1;
    const int64_t s = starts[c];
    // chunk input: padded samples [s, s + C), reflected outside the song
    const int64_t lo = std::max<int64_t>(s, g.border), hi = std::min<int64_t>(s + g.C, g.border + g.len);
    if (run.direct_in && lo == s && hi == s + g.C) {
      // wholly inside a page-locked song: one DMA, no staging
      if (cudaMemcpyAsync(e->dev_in, xh + 2 * (s - g.border), static_cast<size_t>(g.C) * 2 * sizeof(float),
                          cudaMemcpyHostToDevice, e->stream) != cudaSuccess)
        return bail(fail(LBRR_ERR_CUDA, "chunk upload"));
    } else {
      if (cudaEventSynchronize(e->song_ev_in[slot]) != cudaSuccess) return bail(fail(LBRR_ERR_CUDA, "input slot"));
      float* pin = e->song_pin_in[slot];
      if (hi > lo) std::memcpy(pin + 2 * (lo - s), xh + 2 * (lo - g.border), static_cast<size_t>(hi - lo) * 2 * sizeof(float));
      for (int64_t p = s; p < s + g.C; ++p) {
        if (p >= lo && p < hi) {
          p = hi - 1;
          continue;
        }
        int64_t src = 0;
        if (g.len > 1) {
          const int64_t period = 2 * (g.len - 1);
          int64_t q = (p - g.border) % period;
          if (q < 0) q += period;
          src = q < g.len ? q : period - q;
        }
        pin[2 * (p - s)] = xh[2 * src];
        pin[2 * (p - s) + 1] = xh[2 * src + 1];
      }
      if (cudaMemcpyAsync(e->dev_in, pin, static_cast<size_t>(g.C) * 2 * sizeof(float), cudaMemcpyHostToDevice,
                          e->stream) != cudaSuccess ||
          cudaEventRecord(e->song_ev_in[slot], e->stream) != cudaSuccess)
        return bail(fail(LBRR_ERR_CUDA, "chunk upload"));
    }
    if (e->song_fail_chunk == c)  // host-side failure injection (tests of the abort path)
      return bail(fail(LBRR_ERR_STATE, "injected failure before the forward of chunk " + std::to_string(c)));
    if (int rc = lbrr_forward_chunk(e, e->dev_in, g.C, e->dev_out, e->stream)) return bail(rc);
    const unsigned blocks_ov = static_cast<unsigned>((g.ov + 255) / 256);
    if (c + 1 < g.nc) {
      // strip for the next chunk's engine
      lbrr_engine* dst = engines[(c + 1) % n];
      float* dst_strip = dst->song_strip_in + static_cast<size_t>(c) * (strip_b / sizeof(float));
      song_strip_kernel<<<blocks_ov, 256, 0, e->stream>>>(e->dev_out, e->song_strip_out, g, c);
      cudaError_t ce = cudaGetLastError();
      if (ce == cudaSuccess)
        ce = cudaMemcpyPeerAsync(dst_strip, dst->device, e->song_strip_out, e->device, strip_b, e->stream);
      if (ce == cudaSuccess) ce = cudaEventRecord(run.strip_ev[c], e->stream);
      if (ce != cudaSuccess) return bail(fail(LBRR_ERR_PEER, std::string("overlap strip: ") + cudaGetErrorString(ce)));
      {
        std::lock_guard<std::mutex> lk(run.mu);
        run.strip_ready[c] = 1;
      }
      run.cv.notify_all();
    }
    // this chunk's finished samples
    const int64_t o0 = c == 0 ? 0 : s - g.border;
    const int64_t o1 = c + 1 < g.nc ? starts[c + 1] - g.border : g.len;
    const int64_t r0 = o0 + g.border - s, nreg = o1 - o0, head = c > 0 ? g.ov : 0;
    const float* strip_prev = nullptr;
    if (c > 0) {
      std::unique_lock<std::mutex> lk(run.mu);
      // the previous chunk's engine records its strip; a failed engine raises abort
      if (!run.cv.wait_for(lk, std::chrono::seconds(120), [&] { return run.strip_ready[c - 1] || run.abort.load(); }) ||
          run.abort.load())
        return run.abort.load() ? void() : bail(fail(LBRR_ERR_STATE, "overlap strip never arrived"));
      lk.unlock();
      if (cudaStreamWaitEvent(e->stream, run.strip_ev[c - 1], 0) != cudaSuccess)
        return bail(fail(LBRR_ERR_CUDA, "strip wait"));
      strip_prev = e->song_strip_in + static_cast<size_t>(c - 1) * (strip_b / sizeof(float));
    }
    if (nreg > 0) {
      // region buffer `slot` is free once its download two chunks ago is done
      if (cudaStreamWaitEvent(e->stream, e->song_ev_out[slot], 0) != cudaSuccess)
        return bail(fail(LBRR_ERR_CUDA, "region buffer wait"));
      song_region_kernel<<<static_cast<unsigned>((nreg + 255) / 256), 256, 0, e->stream>>>(
          e->dev_out, strip_prev, e->song_fin[slot], g, c, r0, nreg, head);
      if (cudaGetLastError() != cudaSuccess) return bail(fail(LBRR_ERR_CUDA, "region launch"));
    }
    // the host copy of the previous region overlaps this chunk's GPU work
    if (int rc = scatter()) return bail(rc);
    if (nreg > 0 && run.direct_out) {
      // page-locked output: the 12 channel rows of the region go straight to
      // their places in the caller's planar array (one 2-D copy)
      if (cudaEventRecord(e->song_ev_reg[slot], e->stream) != cudaSuccess ||
          cudaStreamWaitEvent(e->song_copy, e->song_ev_reg[slot], 0) != cudaSuccess ||
          cudaMemcpy2DAsync(outh + o0, static_cast<size_t>(g.len) * sizeof(float), e->song_fin[slot],
                            static_cast<size_t>(nreg) * sizeof(float), static_cast<size_t>(nreg) * sizeof(float),
                            2 * kStems, cudaMemcpyDeviceToHost, e->song_copy) != cudaSuccess ||
          cudaEventRecord(e->song_ev_out[slot], e->song_copy) != cudaSuccess)
        return bail(fail(LBRR_ERR_CUDA, "region download"));
    } else if (nreg > 0) {
      // the download runs on the copy stream, so the next chunk's forward on
      // the compute stream does not wait for it
      if (cudaEventRecord(e->song_ev_reg[slot], e->stream) != cudaSuccess ||
          cudaStreamWaitEvent(e->song_copy, e->song_ev_reg[slot], 0) != cudaSuccess ||
          cudaMemcpyAsync(e->song_pin_out[slot], e->song_fin[slot],
                          static_cast<size_t>(nreg) * 2 * kStems * sizeof(float), cudaMemcpyDeviceToHost,
                          e->song_copy) != cudaSuccess ||
          cudaEventRecord(e->song_ev_out[slot], e->song_copy) != cudaSuccess)
        return bail(fail(LBRR_ERR_CUDA, "region download"));
      pend_slot = slot;
      pend_o0 = o0;
      pend_n = nreg;
    }
  }
  if (int rc = scatter()) return bail(rc);
  if (run.direct_out && cudaStreamSynchronize(e->song_copy) != cudaSuccess)
    return bail(fail(LBRR_ERR_CUDA, "region download"));
  if (int rc = check_status(e->status, e->stream)) return bail(rc);
}
}  // namespace

extern "C" int lbrr_separate_song(lbrr_engine* const* engines, int n, const float* xh, int64_t len,
                                  const lbrr_chunk_plan* plan, float* outh) {
  if (!engines || n <= 0 || !xh || !outh) return fail(LBRR_ERR_INVALID, "NULL argument");
  if (len <= 0) return fail(LBRR_ERR_INVALID, "empty audio is unsupported");
  const lbrr_chunk_plan P = plan ? *plan : lbrr_chunk_plan{588800, 559360, 29440, LBRR_FADE_LINEAR};
  if (P.chunk <= kNfft / 2 || P.step <= 0 || P.step > P.chunk || P.border < 0 || 2 * P.border > P.chunk)
    return fail(LBRR_ERR_INVALID, "invalid chunk plan");
  if (P.fade != LBRR_FADE_LINEAR && P.fade != LBRR_FADE_HANN)
    return fail(LBRR_ERR_INVALID, "chunk plan fade must be LBRR_FADE_LINEAR or LBRR_FADE_HANN");
  if (P.fade == LBRR_FADE_LINEAR && P.border == 0 && P.step < P.chunk)
    return fail(LBRR_ERR_INVALID, "a linear fade needs border > 0 when chunks overlap");
  for (int i = 0; i < n; ++i) {
    if (!engines[i]) return fail(LBRR_ERR_INVALID, "NULL engine");
    if (!engines[i]->weights_loaded) return fail(LBRR_ERR_STATE, "weights not loaded");
    if (engines[i]->max_len < P.chunk) return fail(LBRR_ERR_INVALID, "engine scratch smaller than the chunk");
    for (int k = 0; k < i; ++k)
      if (engines[k] == engines[i]) return fail(LBRR_ERR_INVALID, "the same engine is listed twice");
  }
  if (2 * P.step < P.chunk) return separate_song_serial(engines, n, xh, len, P, outh);
  const auto starts = chunk_starts(len, P.chunk, P.step, P.border);
  SongGeom g;
  g.C = P.chunk;
  g.step = P.step;
  g.border = P.border;
  g.ov = P.chunk - P.step;
  g.len = len;
  g.nc = static_cast<int>(starts.size());
  const int workers = std::min<int>(n, g.nc);
  if (P.fade == LBRR_FADE_HANN) {
    const std::vector<float> w = hann_window_host(P.chunk);
    for (int i = 0; i < workers; ++i) {
      DeviceGuard dg(engines[i]->device);
      if (int rc = ensure_song_hann(engines[i], w)) return rc;
    }
    g.hann = engines[0]->song_hann;  // non-null marks the Hann plan; each worker uses its own copy
  }
  SongRun run;
  run.direct_in = host_pinned(xh, static_cast<size_t>(len) * 2 * sizeof(float));
  run.direct_out = host_pinned(outh, static_cast<size_t>(len) * 2 * kStems * sizeof(float));
  run.strip_ready.assign(g.nc, 0);
  run.strip_ev.assign(g.nc, nullptr);
  run.rc.assign(workers, LBRR_OK);
  run.msg.assign(workers, std::string());
  int rc = LBRR_OK;
  for (int c = 0; rc == LBRR_OK && c + 1 < g.nc; ++c) {
    DeviceGuard dg(engines[c % workers]->device);
    if (cudaEventCreateWithFlags(&run.strip_ev[c], cudaEventDisableTiming) != cudaSuccess)
      rc = fail(LBRR_ERR_CUDA, "event create");
  }
  if (rc == LBRR_OK) {
    // every engine's receive buffers exist before any strip is sent
    for (int i = 0; rc == LBRR_OK && i < workers; ++i) {
      DeviceGuard dg(engines[i]->device);
      rc = ensure_song_buffers(engines[i], g);
    }
  }
  if (rc == LBRR_OK) {
    std::vector<std::thread> th;
    for (int i = 0; i < workers; ++i)
      th.emplace_back(song_worker, engines, workers, i, xh, outh, g, std::cref(starts), std::ref(run));
    for (auto& t : th) t.join();
    for (int i = 0; i < workers && rc == LBRR_OK; ++i)
      if (run.rc[i] != LBRR_OK) rc = fail(run.rc[i], run.msg[i]);
    if (rc == LBRR_OK && run.abort.load()) rc = fail(LBRR_ERR_STATE, "song separation aborted");
  }
  for (int c = 0; c + 1 < g.nc; ++c)
    if (run.strip_ev[c]) {
      DeviceGuard dg(engines[c % workers]->device);
      cudaEventSynchronize(run.strip_ev[c]);
      cudaEventDestroy(run.strip_ev[c]);
    }
  return rc;
}

// ---------------------------------------------------------------------------
static int* op_status() {
  static std::mutex mu;
  static std::map<int, int*> per_dev;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = per_dev.find(dev);
  if (it != per_dev.end()) return it->second;
  int* p = nullptr;
  if (cudaMalloc(&p, 64 * sizeof(int)) != cudaSuccess) return nullptr;
  cudaMemset(p, 0, 64 * sizeof(int));
  cudaDeviceSynchronize();
  per_dev[dev] = p;
  return p;
}

#define OP_PROLOGUE                                                                                \
  int* status = op_status();                                                                       \
  if (!status) return fail(LBRR_ERR_CUDA, "op status allocation failed");                          \
  cudaStream_t st = static_cast<cudaStream_t>(stream);

extern "C" int lbrr_op_norm_gates(const float* x, const float* gamma, const float* gw, const float* gb, uint16_t* h16,
                                  float* gates, int64_t rows, void* stream) {
  if (!x || !gamma || !gw || !gb || !h16 || !gates || rows <= 0 || rows > (1ll << 30))
    return fail(LBRR_ERR_INVALID, "lbrr_op_norm_gates: bad arguments");
  OP_PROLOGUE
  (void)status;
  CK(norm_gates(x, gamma, gw, gb, reinterpret_cast<__half*>(h16), gates, static_cast<int>(rows), st));
  return LBRR_OK;
}

extern "C" int lbrr_op_qkv_rope(const uint16_t* h16, const uint16_t* w16, const float* bias16, const float* cos_tab,
                                const float* sin_tab, uint16_t* qkv, int64_t frames, int32_t bands, int32_t axis,
                                void* stream) {
  if (!h16 || !w16 || !bias16 || !cos_tab || !sin_tab || !qkv || frames <= 0 || bands <= 0 || (axis != 0 && axis != 1) ||
      frames * bands > (1ll << 30))
    return fail(LBRR_ERR_INVALID, "lbrr_op_qkv_rope: bad arguments");
  OP_PROLOGUE
  CK(gemm_qkv(reinterpret_cast<const __half*>(h16), reinterpret_cast<const __half*>(w16), bias16, cos_tab, sin_tab,
              reinterpret_cast<__half*>(qkv), static_cast<int>(frames * bands), bands, axis, status, st));
  return LBRR_OK;
}

extern "C" int lbrr_op_attention(const uint16_t* qkv, const float* gates, uint16_t* out, int64_t frames, int32_t bands,
                                 int32_t axis, void* stream) {
  if (!qkv || !gates || !out || frames <= 0 || bands <= 0 || (axis != 0 && axis != 1) || (axis == 1 && bands > 64) ||
      frames * bands > (1ll << 30))
    return fail(LBRR_ERR_INVALID, "lbrr_op_attention: bad arguments (freq axis needs bands <= 64)");
  OP_PROLOGUE
  CK(attention_fwd(reinterpret_cast<const __half*>(qkv), gates, reinterpret_cast<__half*>(out),
                   static_cast<int>(frames), bands, axis, 1, status, st));
  return LBRR_OK;
}

extern "C" int lbrr_op_outproj_norm(const uint16_t* scaled16, const uint16_t* w16, const float* bias,
                                    const float* resid, const float* gamma, float* attn_out, uint16_t* h16,
                                    int64_t rows, void* stream) {
  if (!scaled16 || !w16 || !bias || !resid || !gamma || !attn_out || !h16 || rows <= 0 || rows > (1ll << 30))
    return fail(LBRR_ERR_INVALID, "lbrr_op_outproj_norm: bad arguments");
  OP_PROLOGUE
  CK(gemm_outproj_norm(reinterpret_cast<const __half*>(scaled16), reinterpret_cast<const __half*>(w16), bias, resid,
                       gamma, attn_out, reinterpret_cast<__half*>(h16), static_cast<int>(rows), status, st));
  return LBRR_OK;
}

extern "C" int lbrr_op_ff1_gelu(const uint16_t* h16, const uint16_t* w16, const float* b1, uint16_t* ff1,
                                int64_t rows, void* stream) {
  if (!h16 || !w16 || !b1 || !ff1 || rows <= 0 || rows > (1ll << 30))
    return fail(LBRR_ERR_INVALID, "lbrr_op_ff1_gelu: bad arguments");
  OP_PROLOGUE
  CK(gemm_ff1_gelu(reinterpret_cast<const __half*>(h16), reinterpret_cast<const __half*>(w16), b1,
                   reinterpret_cast<__half*>(ff1), static_cast<int>(rows), status, st));
  return LBRR_OK;
}

extern "C" int lbrr_op_ff2_resid(const uint16_t* ff1, const uint16_t* w16, const float* b2, const float* resid,
                                 float* x, int64_t rows, void* stream) {
  if (!ff1 || !w16 || !b2 || !resid || !x || rows <= 0 || rows > (1ll << 30))
    return fail(LBRR_ERR_INVALID, "lbrr_op_ff2_resid: bad arguments");
  OP_PROLOGUE
  CK(gemm_ff2_resid(reinterpret_cast<const __half*>(ff1), reinterpret_cast<const __half*>(w16), b2, resid, x,
                    static_cast<int>(rows), RowNorm(), status, st));
  return LBRR_OK;
}

extern "C" int lbrr_op_feed_forward(const uint16_t* h16, const uint16_t* w1_16, const float* b1,
                                    const uint16_t* w2_16, const float* b2, const float* resid, float* x,
                                    int64_t rows, void* stream) {
  if (!h16 || !w1_16 || !b1 || !w2_16 || !b2 || !resid || !x || rows <= 0 || rows > (1ll << 30))
    return fail(LBRR_ERR_INVALID, "lbrr_op_feed_forward: bad arguments");
  OP_PROLOGUE
  CK(gemm_ff_fused(reinterpret_cast<const __half*>(h16), reinterpret_cast<const __half*>(w1_16), b1,
                   reinterpret_cast<const __half*>(w2_16), b2, resid, x, static_cast<int>(rows), RowNorm(), status,
                   st));
  return LBRR_OK;
}

extern "C" int lbrr_op_sync(void* stream) {
  int* status = op_status();
  if (!status) return fail(LBRR_ERR_CUDA, "op status allocation failed");
  return check_status(status, static_cast<cudaStream_t>(stream));
}
