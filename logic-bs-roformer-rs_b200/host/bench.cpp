// --bench / --dualbench / --kernel-regression of the host CLI.
//
// --bench times device-resident chunk forwards with CUDA events and writes the
// reference's schema-v1 report (schema_version, identity, shape, pipeline,
// backend, precision, timing_ms with the host sub-phases, memory_bytes,
// correctness per stem against a golden fixture, ola_vs_host, mfu;
// src/main.rs:7336-7347, src/benchmark.rs:57-160).  The FLOP count follows the
// input length (src/benchmark.rs:105-117).
//
// --kernel-regression runs the checkpoint-free checks: STFT -> C2R -> OLA
// impulses and silence through an identity mask (ola_regression,
// src/main.rs:7943-7965), one-hot mask estimators that make every masked
// spectrum slot identifiable (mask_layout_regression, :7967-8015), QKV + RoPE
// at the boundary frame counts of the RoPE/gate regression (:7911-7935), and
// the feed-forward at the FF1 regression's M list (:8017-8052), fused against
// unfused bit for bit.
#include "bench.h"

#include <cuda_runtime.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <complex>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <numeric>
#include <string>
#include <vector>

#include "../../include/lbrr_gpu.h"
#include "npz.h"
#include "synth.h"

extern "C" uint16_t lbrr_f32_to_f16_bits(float x);  // the library's fp16 packing contract

namespace lbrr_host {
namespace {

constexpr int kStems = 6;
constexpr int kSampleRate = 44100;

using Clock = std::chrono::steady_clock;
double ms_since(Clock::time_point t0) { return std::chrono::duration<double, std::milli>(Clock::now() - t0).count(); }

// ---- minimal JSON text builders ---------------------------------------------
std::string jstr(const std::string& s) {
  std::string o = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\') {
      o += '\\';
      o += c;
    } else if (static_cast<unsigned char>(c) < 0x20) {
      char b[8];
      std::snprintf(b, sizeof b, "\\u%04x", c);
      o += b;
    } else {
      o += c;
    }
  }
  return o + "\"";
}
std::string jnum(double v) {
  if (!std::isfinite(v)) return "null";
  char b[40];
  std::snprintf(b, sizeof b, "%.10g", v);
  return b;
}
std::string jint(long long v) { return std::to_string(v); }
std::string jbool(bool v) { return v ? "true" : "false"; }
using KV = std::vector<std::pair<std::string, std::string>>;
std::string jobj(const KV& kv) {
  std::string o = "{";
  for (size_t i = 0; i < kv.size(); ++i) o += (i ? ", " : "") + jstr(kv[i].first) + ": " + kv[i].second;
  return o + "}";
}
std::string jarr(const std::vector<std::string>& v) {
  std::string o = "[";
  for (size_t i = 0; i < v.size(); ++i) o += (i ? ", " : "") + v[i];
  return o + "]";
}

// ---- host metrics (src/benchmark.rs:57-95) ------------------------------------
struct Metric {
  bool finite = true, bit_equal = true;
  double rms = 0, snr = NAN, max_abs = 0;
  std::string json() const {
    return jobj({{"finite", jbool(finite)},
                 {"reference_rms", jnum(rms)},
                 {"snr_db", jnum(snr)},
                 {"max_abs_error", jnum(max_abs)},
                 {"bit_equal", jbool(bit_equal)}});
  }
};
Metric metric(const float* a, const float* r, size_t n) {
  Metric m;
  double sig = 0, noise = 0;
  for (size_t i = 0; i < n; ++i) {
    m.finite &= std::isfinite(a[i]) && std::isfinite(r[i]);
    m.bit_equal &= std::memcmp(&a[i], &r[i], 4) == 0;
    const double d = static_cast<double>(a[i]) - r[i];
    sig += static_cast<double>(r[i]) * r[i];
    noise += d * d;
    m.max_abs = std::max(m.max_abs, std::fabs(d));
  }
  m.rms = std::sqrt(sig / std::max<size_t>(1, n));
  if (m.finite && m.rms >= 1e-8) m.snr = 10.0 * std::log10(sig / std::max(noise, 1e-300));
  return m;
}

// In-place iterative radix-2 complex FFT in double precision (inverse,
// unnormalised: exp(+2 pi i k n / N)), N a power of two.
void host_ifft(std::vector<std::complex<double>>& a) {
  const size_t n = a.size();
  for (size_t i = 1, j = 0; i < n; ++i) {
    size_t bit = n >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) std::swap(a[i], a[j]);
  }
  for (size_t len = 2; len <= n; len <<= 1) {
    const double ang = 2.0 * M_PI / static_cast<double>(len);
    for (size_t i = 0; i < n; i += len)
      for (size_t k = 0; k < len / 2; ++k) {
        const std::complex<double> w(std::cos(ang * k), std::sin(ang * k));
        const std::complex<double> u = a[i + k], v = a[i + k + len / 2] * w;
        a[i + k] = u + v;
        a[i + k + len / 2] = u - v;
      }
  }
}

// Independent host ISTFT of the masked spectra (the C2R input, DC and Nyquist
// taken as real) in double precision: inverse real FFT, Hann window,
// overlap-add, division by the window-square envelope, crop -- the check the
// reference makes with benchmark::host_ola (src/benchmark.rs:143-175), here
// covering the in-house inverse FFT as well.
std::vector<float> host_istft(const std::vector<float>& c2r, int64_t len, int T) {
  std::vector<double> win(2048);
  for (int i = 0; i < 2048; ++i) win[i] = 0.5 * (1.0 - std::cos(2.0 * M_PI * i / 2048));
  const int64_t padded = len + 2048;
  std::vector<double> counter(padded, 0.0), result(static_cast<size_t>(12) * padded, 0.0);
  for (int t = 0; t < T; ++t)
    for (int n = 0; n < 2048; ++n) {
      const int64_t p = static_cast<int64_t>(t) * 512 + n;
      if (p < padded) counter[p] += win[n] * win[n];
    }
  std::vector<std::complex<double>> a(2048);
  for (int sc = 0; sc < 12; ++sc)
    for (int t = 0; t < T; ++t) {
      const float* X = c2r.data() + (static_cast<size_t>(sc) * T + t) * 1025 * 2;
      a[0] = X[0];
      a[1024] = X[2048];
      for (int k = 1; k < 1024; ++k) {
        a[k] = std::complex<double>(X[2 * k], X[2 * k + 1]);
        a[2048 - k] = std::conj(a[k]);
      }
      host_ifft(a);
      for (int n = 0; n < 2048; ++n) {
        const int64_t p = static_cast<int64_t>(t) * 512 + n;
        if (p < padded) result[sc * padded + p] += a[n].real() / 2048.0 * win[n];
      }
    }
  std::vector<float> out(static_cast<size_t>(12) * len);
  for (int sc = 0; sc < 12; ++sc)
    for (int64_t i = 0; i < len; ++i) {
      const int64_t p = i + 1024;
      out[sc * len + i] = counter[p] > 1e-8 ? static_cast<float>(result[sc * padded + p] / counter[p]) : 0.f;
    }
  return out;
}

uint64_t matrix_flops(int64_t t) {  // src/benchmark.rs:105-117
  const uint64_t T = static_cast<uint64_t>(t), m = 62 * T;
  const uint64_t trunk = 24 * (2 * m * 1536 * 256 + 2 * m * 256 * 512 + 2 * m * 1024 * 256 + 2 * m * 256 * 1024 +
                               2 * m * 8 * 256);
  const uint64_t attn = 12 * 4 * 62 * 8 * T * T * 64 + 12 * 4 * T * 8 * 62 * 62 * 64;
  const uint64_t mask = 6 * (2 * m * 1024 * 256 + 2 * T * 8200 * 1024);
  return trunk + attn + mask + 2 * T * 4100 * 256;
}

std::string run_cmd(const std::string& cmd) {
  std::string out;
  if (FILE* p = popen(cmd.c_str(), "r")) {
    char buf[256];
    while (std::fgets(buf, sizeof buf, p)) out += buf;
    pclose(p);
  }
  while (!out.empty() && (out.back() == '\n' || out.back() == ' ')) out.pop_back();
  return out;
}
// The OS SHA256 utility, as the reference does (src/benchmark.rs:176-200).
std::string sha256(const std::string& path) {
  if (path.empty()) return "null";
  std::string q = "'";
  for (char c : path) q += c == '\'' ? std::string("'\\''") : std::string(1, c);
  const std::string o = run_cmd("sha256sum " + q + "'" + " 2>/dev/null");
  if (o.size() < 64) return "null";
  return jstr(o.substr(0, 64));
}

std::string identity(const BenchArgs& a, const cudaDeviceProp& prop) {
  char exe[4096] = {0};
  const ssize_t n = readlink("/proc/self/exe", exe, sizeof exe - 1);
  int rt = 0;
  cudaRuntimeGetVersion(&rt);
  const std::string driver = run_cmd("nvidia-smi --query-gpu=driver_version --format=csv,noheader -i " +
                                     std::to_string(a.device) + " 2>/dev/null");
  std::string cfg = a.model_dir + "/logic_bs_roformer.yaml";
  if (FILE* f = std::fopen(cfg.c_str(), "rb")) {
    std::fclose(f);
  } else {
    cfg = a.model_dir + "/config.yaml";
  }
#ifdef LBRR_SOURCE_SHA256
  const std::string src = jstr(LBRR_SOURCE_SHA256);
#else
  const std::string src = "null";
#endif
  std::string fixture = "null";
  if (!a.reference.empty()) {
    const size_t s = a.reference.find_last_of('/');
    if (s != std::string::npos && s > 0) {
      const size_t s2 = a.reference.find_last_of('/', s - 1);
      fixture = jstr(a.reference.substr(s2 == std::string::npos ? 0 : s2 + 1, s - (s2 == std::string::npos ? 0 : s2 + 1)));
    }
  }
  return jobj({{"source_revision", "null"},
               {"source_sha256", src},
               {"source_hash_reason", jstr("SHA256 over the library, CLI and header sources, embedded at build time")},
               {"binary_sha256", n > 0 ? sha256(std::string(exe, n)) : "null"},
               {"library_abi", jint(lbrr_abi_version())},
               {"model_sha256", sha256(a.model_dir + "/model.safetensors")},
               {"config_sha256", sha256(cfg)},
               {"reference_sha256", a.reference.empty() ? "null" : sha256(a.reference)},
               {"fixture_id", fixture},
               {"device", jstr(prop.name)},
               {"sm", jstr(std::to_string(prop.major) + "." + std::to_string(prop.minor))},
               {"driver", driver.empty() ? "null" : jstr(driver)},
               {"cuda_runtime", jobj({{"version", jint(rt)}, {"library", jstr("libcudart (linked)")}})}});
}

struct Engine {
  lbrr_engine* e = nullptr;
  ~Engine() { lbrr_engine_destroy(e); }
};

int64_t info(lbrr_engine* e, int key) {
  int64_t v = 0;
  lbrr_engine_get_option(e, key, &v);
  return v;
}

int fail_msg(const char* what) {
  std::fprintf(stderr, "lbrr_b200: %s: %s\n", what, lbrr_last_error());
  return 1;
}

// Seeded synthetic stereo (interleaved): per channel eight sines and noise.
std::vector<float> synthetic_audio(int64_t L) {
  std::vector<float> x(static_cast<size_t>(2 * L));
  uint64_t st = 0x9E3779B97F4A7C15ull;
  auto uni = [&]() {
    st ^= st << 13;
    st ^= st >> 7;
    st ^= st << 17;
    return static_cast<double>(st >> 11) * (1.0 / 9007199254740992.0);
  };
  for (int ch = 0; ch < 2; ++ch) {
    double f[8], ph[8], amp[8];
    for (int k = 0; k < 8; ++k) {
      f[k] = 50.0 + uni() * 14950.0;
      ph[k] = uni() * 6.283185307179586;
      amp[k] = 0.05 + uni() * 0.1;
    }
    for (int64_t i = 0; i < L; ++i) {
      double v = (uni() - 0.5) * 0.1;
      for (int k = 0; k < 8; ++k) v += amp[k] * std::sin(6.283185307179586 * f[k] * i / 44100.0 + ph[k]);
      x[2 * i + ch] = static_cast<float>(0.25 * v);
    }
  }
  return x;
}

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() { cudaFree(p); }
};

}  // namespace

// ---------------------------------------------------------------------------
int run_bench(const BenchArgs& a) {
  if (a.stage != "waveform") {
    std::fprintf(stderr, "lbrr_b200: --bench-stage %s: this build fuses the overlap-add into the forward; only "
                         "'waveform' is measured\n", a.stage.c_str());
    return 2;
  }
  // ---- golden fixture (optional) or synthetic input ----
  std::vector<float> xi, ref_out;
  int64_t L = 588800;
  if (!a.reference.empty()) {
    std::map<std::string, NpyArray> z;
    std::string err;
    if (!read_npz_f32(a.reference, z, err)) {
      std::fprintf(stderr, "lbrr_b200: --bench-ref: %s\n", err.c_str());
      return 1;
    }
    auto it = z.find("inp"), ot = z.find("out");
    if (it == z.end() || ot == z.end()) {
      std::fprintf(stderr, "lbrr_b200: --bench-ref needs arrays 'inp' and 'out'\n");
      return 1;
    }
    const auto& is = it->second.shape;
    const auto& os = ot->second.shape;
    L = is.empty() ? 0 : is.back();
    const bool ishape = (is == std::vector<int64_t>{1, 2, L}) || (is == std::vector<int64_t>{2, L});
    const bool oshape = (os == std::vector<int64_t>{1, 6, 2, L}) || (os == std::vector<int64_t>{6, 2, L});
    if (!ishape || !oshape || L <= 1024 || L > 588800) {
      std::fprintf(stderr, "lbrr_b200: --bench-ref: inp must be [1,2,L] or [2,L] and out [1,6,2,L] or [6,2,L] "
                           "with 1024 < L <= 588800\n");
      return 1;
    }
    for (float v : it->second.data)
      if (!std::isfinite(v)) return std::fprintf(stderr, "lbrr_b200: fixture contains nonfinite values\n"), 1;
    xi.resize(static_cast<size_t>(2 * L));
    for (int64_t i = 0; i < L; ++i) {
      xi[2 * i] = it->second.data[i];
      xi[2 * i + 1] = it->second.data[L + i];
    }
    ref_out = ot->second.data;
  } else {
    xi = synthetic_audio(L);
  }
  const int T = static_cast<int>(L / 512 + 1);
  std::printf("bench: L=%lld T=%d bands=62 M=%d iters=%d pipeline=%s\n", static_cast<long long>(L), T, 62 * T, a.iters,
              a.stage.c_str());
  // ---- context + engine ----
  auto t0 = Clock::now();
  if (cudaSetDevice(a.device) != cudaSuccess || cudaFree(nullptr) != cudaSuccess) {
    std::fprintf(stderr, "lbrr_b200: device %d unavailable\n", a.device);
    return 1;
  }
  cudaDeviceProp prop;
  cudaGetDeviceProperties(&prop, a.device);
  lbrr_model_desc d;
  int32_t freqs[64];
  lbrr_default_model(&d, freqs, 64);
  Engine eng;
  if (lbrr_engine_create(a.device, &d, std::max<int64_t>(L, 588800), &eng.e) != LBRR_OK) return fail_msg("engine");
  const double context_ms = ms_since(t0);
  t0 = Clock::now();
  const std::string wpath = a.model_dir + "/model.safetensors";
  if (lbrr_engine_load_safetensors(eng.e, wpath.c_str()) != LBRR_OK) return fail_msg(wpath.c_str());
  const double weights_ms = ms_since(t0);
  // ---- buffers ----
  t0 = Clock::now();
  DevBuf dx, dy;
  cudaStream_t s = nullptr;
  if (cudaMalloc(&dx.p, xi.size() * 4) != cudaSuccess || cudaMalloc(&dy.p, static_cast<size_t>(12) * L * 4) != cudaSuccess ||
      cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMemcpy(dx.p, xi.data(), xi.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    std::fprintf(stderr, "lbrr_b200: bench buffers: %s\n", cudaGetErrorString(cudaGetLastError()));
    return 1;
  }
  std::unique_ptr<CUstream_st, void (*)(cudaStream_t)> sguard(s, [](cudaStream_t x) { cudaStreamDestroy(x); });
  const double alloc_ms = ms_since(t0);
  auto forward = [&]() { return lbrr_forward_chunk(eng.e, static_cast<float*>(dx.p), L, static_cast<float*>(dy.p), s); };
  // the first forward builds the per-length tables and FFT plans
  t0 = Clock::now();
  if (forward() != LBRR_OK || cudaStreamSynchronize(s) != cudaSuccess) return fail_msg("forward");
  const double prepare_ms = ms_since(t0);
  const double setup_ms = info(eng.e, LBRR_INFO_SETUP_US) / 1000.0;
  for (int i = 0; i < a.warmup; ++i)
    if (forward() != LBRR_OK) return fail_msg("forward");
  cudaStreamSynchronize(s);
  std::vector<cudaEvent_t> ev(2 * a.iters);
  for (auto& e : ev) cudaEventCreate(&e);
  t0 = Clock::now();
  for (int i = 0; i < a.iters; ++i) {
    cudaEventRecord(ev[2 * i], s);
    if (forward() != LBRR_OK) return fail_msg("forward");
    cudaEventRecord(ev[2 * i + 1], s);
  }
  cudaStreamSynchronize(s);
  const double host_ms = ms_since(t0);
  if (lbrr_engine_sync(eng.e) != LBRR_OK) return fail_msg("device status");
  std::vector<double> gpu_ms(a.iters);
  for (int i = 0; i < a.iters; ++i) {
    float t = 0;
    cudaEventElapsedTime(&t, ev[2 * i], ev[2 * i + 1]);
    gpu_ms[i] = t;
  }
  for (auto& e : ev) cudaEventDestroy(e);
  std::vector<double> sorted = gpu_ms;
  std::sort(sorted.begin(), sorted.end());
  const double median = sorted.size() % 2 ? sorted[sorted.size() / 2]
                                          : 0.5 * (sorted[sorted.size() / 2 - 1] + sorted[sorted.size() / 2]);
  const double avg = host_ms / a.iters;
  const double audio_ms = L * 1000.0 / kSampleRate;
  std::printf("BENCH warm aggregate: %.3f ms/iter over %d iters, RTF %.4f\n", avg, a.iters, avg / audio_ms);
  std::printf("BENCH CUDA Event: median %.3f ms, mean %.3f ms\n", median,
              std::accumulate(gpu_ms.begin(), gpu_ms.end(), 0.0) / a.iters);
  // ---- download, host OLA check, correctness ----
  t0 = Clock::now();
  std::vector<float> out(static_cast<size_t>(12) * L), c2r(static_cast<size_t>(12) * T * 1025 * 2);
  if (cudaMemcpy(out.data(), dy.p, out.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return fail_msg("download");
  if (lbrr_engine_read_buffer(eng.e, "c2r", c2r.data(), static_cast<int64_t>(c2r.size() * 4)) != LBRR_OK)
    return fail_msg("c2r tap");
  const std::vector<float> host = host_istft(c2r, L, T);
  const double download_ms = ms_since(t0);
  const Metric ola = metric(out.data(), host.data(), out.size());
  double peak = 0;
  for (float v : host) peak = std::max(peak, static_cast<double>(std::fabs(v)));
  // fp32 FFT + overlap-add against double precision: a few fp32 ulps of the waveform's scale
  if (!(ola.finite && ola.max_abs <= 2e-6 * std::max(1.0, peak))) {
    std::fprintf(stderr, "lbrr_b200: GPU ISTFT differs from the host ISTFT: max abs %.3g (peak %.3g)\n", ola.max_abs,
                 peak);
    return 1;
  }
  std::string correctness;
  if (!ref_out.empty()) {
    std::vector<std::string> stems;
    for (int st = 0; st < kStems; ++st)
      stems.push_back(metric(out.data() + static_cast<size_t>(st) * 2 * L, ref_out.data() + static_cast<size_t>(st) * 2 * L,
                             static_cast<size_t>(2 * L)).json());
    const Metric all = metric(out.data(), ref_out.data(), out.size());
    if (!all.finite) return std::fprintf(stderr, "lbrr_b200: nonfinite inference output\n"), 1;
    std::printf("BENCH final SNR vs reference: %.2f dB\n", std::isfinite(all.snr) ? all.snr : 300.0);
    correctness = jobj({{"finite", jbool(all.finite)},
                        {"shape", jarr({"1", "6", "2", jint(L)})},
                        {"stems", jarr(stems)},
                        {"overall", all.json()},
                        {"relative_to_b0", "null"},
                        {"relative_to_b0_reason", jstr("no B0 run in this build")},
                        {"tail_covered", "true"}});
  } else {
    bool finite = true;
    for (float v : out) finite &= std::isfinite(v);
    correctness = jobj({{"finite", jbool(finite)},
                        {"shape", jarr({"1", "6", "2", jint(L)})},
                        {"stems", "null"},
                        {"overall", "null"},
                        {"reason", jstr("no golden fixture (--bench-ref); synthetic input")},
                        {"tail_covered", "true"}});
  }
  if (!a.output.empty()) {
    std::FILE* f = std::fopen(a.output.c_str(), "wb");
    if (!f || std::fwrite(out.data(), 4, out.size(), f) != out.size() || std::fclose(f) != 0)
      return std::fprintf(stderr, "lbrr_b200: cannot write %s\n", a.output.c_str()), 1;
  }
  // ---- two chunks in flight: two engines on this GPU, one stream each ----
  double dual_ms = NAN;
  if (a.dual) {
    Engine e2;
    if (lbrr_engine_create(a.device, &d, std::max<int64_t>(L, 588800), &e2.e) != LBRR_OK ||
        lbrr_engine_load_safetensors(e2.e, wpath.c_str()) != LBRR_OK)
      return fail_msg("second engine");
    DevBuf dy2;
    cudaStream_t s2 = nullptr;
    if (cudaMalloc(&dy2.p, static_cast<size_t>(12) * L * 4) != cudaSuccess ||
        cudaStreamCreateWithFlags(&s2, cudaStreamNonBlocking) != cudaSuccess)
      return fail_msg("dual buffers");
    std::unique_ptr<CUstream_st, void (*)(cudaStream_t)> s2guard(s2, [](cudaStream_t x) { cudaStreamDestroy(x); });
    auto fwd2 = [&]() { return lbrr_forward_chunk(e2.e, static_cast<float*>(dx.p), L, static_cast<float*>(dy2.p), s2); };
    for (int i = 0; i < 3; ++i)
      if (forward() != LBRR_OK || fwd2() != LBRR_OK) return fail_msg("dual forward");
    cudaDeviceSynchronize();
    const int pairs = std::max(2, a.iters / 2);
    cudaEvent_t b0, b1, c1;
    cudaEventCreate(&b0);
    cudaEventCreate(&b1);
    cudaEventCreate(&c1);
    cudaEventRecord(b0, s);
    cudaStreamWaitEvent(s2, b0, 0);
    for (int i = 0; i < pairs; ++i)
      if (forward() != LBRR_OK || fwd2() != LBRR_OK) return fail_msg("dual forward");
    cudaEventRecord(c1, s2);
    cudaStreamWaitEvent(s, c1, 0);
    cudaEventRecord(b1, s);
    cudaEventSynchronize(b1);
    float t = 0;
    cudaEventElapsedTime(&t, b0, b1);
    dual_ms = t / (2.0 * pairs);
    cudaEventDestroy(b0);
    cudaEventDestroy(b1);
    cudaEventDestroy(c1);
    if (lbrr_engine_sync(e2.e) != LBRR_OK || lbrr_engine_sync(eng.e) != LBRR_OK) return fail_msg("dual status");
    std::printf("BENCH dual-stream frames: %.3f ms/iter\n", dual_ms);
  }
  // ---- report ----
  if (!a.json.empty()) {
    int64_t wb = 0, sb = 0;
    lbrr_engine_memory(eng.e, &wb, &sb);
    const uint64_t flops = matrix_flops(T);
    const bool b200 = std::strstr(prop.name, "B200") != nullptr;
    const double peak = b200 ? 2250.0 : NAN;  // nominal dense FP16/BF16 TFLOP/s
    std::vector<std::string> ev_json;
    for (double v : gpu_ms) ev_json.push_back(jnum(v));
    const std::string kernels = jstr(
        "hand-written sm_100a: tcgen05 GEMMs with fused epilogues, tcgen05 flash attention on both axes, "
        "STFT/norm/overlap-add bandwidth kernels; cuFFT R2C/C2R");
    std::string report = jobj({
        {"schema_version", "1"},
        {"identity", identity(a, prop)},
        {"shape", jobj({{"batch", "1"}, {"channels", "2"}, {"stems", "6"}, {"samples", jint(L)}, {"T", jint(T)},
                        {"bands", "62"}, {"sample_rate", jint(kSampleRate)}})},
        {"pipeline", jstr(a.stage)},
        {"backend", jobj({{"attention_time", jstr("attn_time_kernel (tcgen05, S/P/O in TMEM)")},
                          {"attention_freq", jstr("attn_freq_kernel (tcgen05, two sequences per tile)")},
                          {"ff1", jobj({{"requested", jstr("fused")}, {"selected", jstr("ff_fused_kernel")}})},
                          {"qk_rope", jstr("fused into the QKV GEMM epilogue")},
                          {"cublaslt", "false"},
                          {"cublaslt_version", "null"},
                          {"cublaslt_algorithms", "null"},
                          {"cudnn_version", "null"},
                          {"cudnn_plans", "null"},
                          {"kernels", kernels},
                          {"kernels_per_chunk", jint(info(eng.e, LBRR_INFO_KERNELS_PER_FORWARD))}})},
        {"precision", jobj({{"matrix_input", jstr("fp16")}, {"accumulation", jstr("fp32")}, {"residual", jstr("fp32")},
                            {"tf32", "false"}, {"input_resident_gpu", "true"}, {"output_resident_gpu", "true"},
                            {"output_kind", jstr(a.stage)}})},
        {"timing_ms", jobj({{"context_kernels", jnum(context_ms)},
                            {"weights_read", jnum(info(eng.e, LBRR_INFO_WEIGHTS_READ_US) / 1000.0)},
                            {"weights_parse", jnum(info(eng.e, LBRR_INFO_WEIGHTS_PARSE_US) / 1000.0)},
                            {"weights_pack_h2d", jnum(weights_ms)},
                            {"weights_conversion", jnum(info(eng.e, LBRR_INFO_WEIGHTS_PACK_US) / 1000.0)},
                            {"weights_h2d_and_alloc", jnum(info(eng.e, LBRR_INFO_WEIGHTS_H2D_US) / 1000.0)},
                            {"fft_plan", jnum(setup_ms)},
                            {"allocation_input_h2d", jnum(alloc_ms)},
                            {"prepare_algorithms", jnum(prepare_ms)},
                            {"warmup", jint(a.warmup)},
                            {"iterations", jint(a.iters)},
                            {"host_total", jnum(host_ms)},
                            {"host_per_iteration", jnum(avg)},
                            {"cuda_event", jarr(ev_json)},
                            {"cuda_event_median", jnum(median)},
                            {"dual_stream_per_chunk", jnum(dual_ms)},
                            {"download_and_host_ola_check", jnum(download_ms)},
                            {"process_before_hashes", jnum(ms_since(a.process_start))},
                            {"rtf", jnum(avg / audio_ms)}})},
        {"memory_bytes", jobj({{"weights", jint(wb)}, {"scratch", jint(sb)}, {"workspace", "0"},
                               {"tuning_temporary", "0"}, {"tracked_resident", jint(wb + sb)}, {"tuning_peak", "0"},
                               {"tracked_peak", jint(wb + sb)}, {"external_peak", "null"},
                               {"accounting", jstr("explicit device allocations of the engine (weight and scratch "
                                                   "arenas); cuFFT plan work areas and driver memory not tracked")}})},
        {"correctness", correctness},
        {"ola_vs_host", ola.json()},
        {"mfu", jobj({{"matrix_flops", jint(static_cast<long long>(flops))},
                      {"nominal_peak_tflops", jnum(peak)},
                      {"nominal_mfu", jnum(flops / (median * 1e9 * peak))},
                      {"reason", b200 ? "null" : jstr("no configured nominal dense FP16 peak for this device")}})},
    });
    std::FILE* f = std::fopen(a.json.c_str(), "w");
    if (!f || std::fprintf(f, "%s\n", report.c_str()) < 0 || std::fclose(f) != 0)
      return std::fprintf(stderr, "lbrr_b200: cannot write %s\n", a.json.c_str()), 1;
  }
  return 0;
}

// ---------------------------------------------------------------------------
// --kernel-regression
// ---------------------------------------------------------------------------
namespace {

float f16_bits_to_float(uint16_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400u));
      bits = sign | (static_cast<uint32_t>(112 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}
uint16_t to_f16(float x) { return lbrr_f32_to_f16_bits(x); }
float f16_round(float x) { return f16_bits_to_float(to_f16(x)); }

// Forward of `x` (interleaved) through `e`; returns planar stems [12][L].
bool run_forward(lbrr_engine* e, const std::vector<float>& x, std::vector<float>& y) {
  const int64_t L = static_cast<int64_t>(x.size() / 2);
  y.assign(static_cast<size_t>(12) * L, NAN);
  return lbrr_forward_chunk_host(e, x.data(), L, y.data()) == LBRR_OK;
}

bool ola_regression(lbrr_engine* e, Checkpoint& ck) {
  make_identity_masks(ck);
  const auto v = ck.views();
  if (lbrr_engine_load_weights(e, v.data(), v.size()) != LBRR_OK) return fail_msg("identity weights"), false;
  for (int64_t L : {1025, 18944, 132300, 588800}) {
    for (int silent = 0; silent < 2; ++silent) {
      std::vector<float> x(static_cast<size_t>(2 * L), 0.f), y;
      if (!silent) {
        x[0] = 0.5f;
        x[2 * (L - 1)] = 1.0f;
        x[2 * 31 + 1] = -0.25f;
        x[2 * (L - 1) + 1] = 0.125f;
      }
      if (!run_forward(e, x, y)) return fail_msg("forward"), false;
      double worst = 0;
      for (int sc = 0; sc < 12; ++sc)
        for (int64_t i = 0; i < L; ++i) {
          const float got = y[sc * L + i], want = x[2 * i + sc % 2];
          if (!std::isfinite(got)) worst = INFINITY;
          worst = std::max(worst, static_cast<double>(std::fabs(got - want)));
        }
      if (!(worst <= 1e-6)) {
        std::fprintf(stderr, "KERNEL_REGRESSION OLA L=%lld silent=%d: max error %.3g > 1e-6\n",
                     static_cast<long long>(L), silent, worst);
        return false;
      }
    }
    std::printf("KERNEL_REGRESSION STFT/OLA L=%lld impulse_channels=2 silence=true overwrite=true\n",
                static_cast<long long>(L));
  }
  return true;
}

bool mask_layout_regression(lbrr_engine* e, Checkpoint& ck) {
  for (int64_t L : {132300, 588800}) {
    const int T = static_cast<int>(L / 512 + 1);
    const std::vector<float> x = synthetic_audio(L);
    for (float offset : {0.0f, 0.5f}) {
      make_one_hot_masks(ck, offset);
      const auto v = ck.views();
      if (lbrr_engine_load_weights(e, v.data(), v.size()) != LBRR_OK) return fail_msg("one-hot weights"), false;
      std::vector<float> y;
      if (!run_forward(e, x, y)) return fail_msg("forward"), false;
      std::vector<uint16_t> hidden(static_cast<size_t>(372) * T * 1024);
      std::vector<float> spec(static_cast<size_t>(2) * T * 1025 * 2), c2r(static_cast<size_t>(12) * T * 1025 * 2);
      if (lbrr_engine_read_buffer(e, "hidden", hidden.data(), static_cast<int64_t>(hidden.size() * 2)) != LBRR_OK ||
          lbrr_engine_read_buffer(e, "spec", spec.data(), static_cast<int64_t>(spec.size() * 4)) != LBRR_OK ||
          lbrr_engine_read_buffer(e, "c2r", c2r.data(), static_cast<int64_t>(c2r.size() * 4)) != LBRR_OK)
        return fail_msg("taps"), false;
      long long bad = 0, checked = 0;
      for (int s = 0; s < 6; ++s)
        for (int b = 0; b < 62; ++b) {
          const int d = band_dim(b), f0 = band_offset(b) / 4;
          for (int t = 0; t < T; ++t) {
            const uint16_t* hrow = &hidden[(static_cast<size_t>(s * 62 + b) * T + t) * 1024];
            for (int k = 1; k < 1024; ++k) bad += hrow[k] != 0;  // tanh(0) = +0
            const float h0 = f16_bits_to_float(hrow[0]);
            for (int fi = 0; fi < d / 4; ++fi)
              for (int ch = 0; ch < 2; ++ch) {
                double m[2];
                for (int c = 0; c < 2; ++c) {
                  const int ja = fi * 4 + ch * 2 + c;
                  const float a = h0 + one_hot_bias(s, b, ja, offset);       // fp32 sum, as the epilogue
                  const float g = h0 + one_hot_bias(s, b, d + ja, offset);
                  m[c] = static_cast<double>(a) / (1.0 + std::exp(-static_cast<double>(g)));
                }
                const int f = f0 + fi;
                const size_t si = ((static_cast<size_t>(ch) * T + t) * 1025 + f) * 2;
                const double sr = spec[si], sim = spec[si + 1];
                double re = sr * m[0] - sim * m[1], im = sr * m[1] + sim * m[0];
                if (f == 0 || f == 1024) im = 0.0;  // the default keeps DC / Nyquist real
                const size_t di = ((static_cast<size_t>(s * 2 + ch) * T + t) * 1025 + f) * 2;
                const double bound = 2e-6 * std::hypot(sr, sim) * (std::fabs(m[0]) + std::fabs(m[1])) + 1e-30;
                const double gr = c2r[di], gi = c2r[di + 1];
                if (!std::isfinite(gr) || !std::isfinite(gi) || std::fabs(gr - re) > bound || std::fabs(gi - im) > bound)
                  ++bad;
                ++checked;
              }
          }
        }
      if (bad) {
        std::fprintf(stderr, "KERNEL_REGRESSION compact_mask T=%d offset=%g: %lld of %lld slots wrong\n", T, offset,
                     bad, checked);
        return false;
      }
    }
    std::printf("KERNEL_REGRESSION compact_mask T=%d bands=62 stems=6 all_slots_written=true\n", T);
  }
  return true;
}

// QKV + RoPE at the boundary frame counts of the RoPE/gate regression, against
// a host restatement (fp64 sums of the fp16 operands, fp16 rounding): at most
// one fp16 unit in the last place apart (the accumulation orders differ).
bool rope_regression() {
  std::vector<float> w(1536 * 256), bias(1536);
  for (size_t i = 0; i < w.size(); ++i) w[i] = f16_round(((static_cast<int>(i % 127)) - 63) / 2048.0f);
  for (int i = 0; i < 1536; ++i) bias[i] = f16_round(((i % 13) - 6) / 128.0f);
  std::vector<uint16_t> w16(w.size());
  for (size_t i = 0; i < w.size(); ++i) w16[i] = to_f16(w[i]);
  DevBuf dw, db, dh, dq, dc, ds;
  cudaMalloc(&dw.p, w16.size() * 2);
  cudaMalloc(&db.p, bias.size() * 4);
  cudaMemcpy(dw.p, w16.data(), w16.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(db.p, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice);
  for (int frames : {1, 37, 62, 63, 64, 65, 259, 1151}) {
    const int bands = 62, M = frames * bands;
    std::vector<float> h(static_cast<size_t>(M) * 256);
    for (size_t i = 0; i < h.size(); ++i) h[i] = f16_round(((static_cast<int>(i % 31)) - 15) / 32.0f);
    std::vector<uint16_t> h16(h.size());
    for (size_t i = 0; i < h.size(); ++i) h16[i] = to_f16(h[i]);
    cudaFree(dh.p);
    cudaFree(dq.p);
    dh.p = dq.p = nullptr;
    cudaMalloc(&dh.p, h16.size() * 2);
    cudaMalloc(&dq.p, static_cast<size_t>(M) * 1536 * 2);
    cudaMemcpy(dh.p, h16.data(), h16.size() * 2, cudaMemcpyHostToDevice);
    for (int axis = 0; axis < 2; ++axis) {
      const int P = axis == 0 ? frames : bands;
      std::vector<float> cs(static_cast<size_t>(P) * 32), sn(cs.size());
      for (int p = 0; p < P; ++p)
        for (int i = 0; i < 32; ++i) {
          const float ang = static_cast<float>(p * (1.0 / std::pow(10000.0, 2.0 * i / 64.0)));
          cs[p * 32 + i] = static_cast<float>(std::cos(static_cast<double>(ang)));
          sn[p * 32 + i] = static_cast<float>(std::sin(static_cast<double>(ang)));
        }
      cudaFree(dc.p);
      cudaFree(ds.p);
      dc.p = ds.p = nullptr;
      cudaMalloc(&dc.p, cs.size() * 4);
      cudaMalloc(&ds.p, sn.size() * 4);
      cudaMemcpy(dc.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(ds.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
      if (lbrr_op_qkv_rope(static_cast<uint16_t*>(dh.p), static_cast<uint16_t*>(dw.p), static_cast<float*>(db.p),
                           static_cast<float*>(dc.p), static_cast<float*>(ds.p), static_cast<uint16_t*>(dq.p), frames,
                           bands, axis, nullptr) != LBRR_OK ||
          lbrr_op_sync(nullptr) != LBRR_OK)
        return fail_msg("qkv rope"), false;
      std::vector<uint16_t> got(static_cast<size_t>(M) * 1536);
      cudaMemcpy(got.data(), dq.p, got.size() * 2, cudaMemcpyDeviceToHost);
      long long bad = 0;
      std::vector<double> acc(1536);
      // every row up to 4096 tokens; beyond, the first and last 512 rows and every 61st
      for (int r = 0; r < M; ++r) {
        if (M > 4096 && r >= 512 && r < M - 512 && r % 61) continue;
        for (int n = 0; n < 1536; ++n) {
          double a = 0;
          for (int k = 0; k < 256; ++k) a += static_cast<double>(h[static_cast<size_t>(r) * 256 + k]) * w[n * 256 + k];
          acc[n] = a + bias[n];
        }
        const int pos = axis == 0 ? r / bands : r % bands;
        for (int n = 0; n < 1536; ++n) {
          double want;
          if (n < 1024) {  // Q and K rotated pairwise
            const int dd = n & 63, i = dd >> 1, base = n - dd;
            const double e0 = acc[base + 2 * i], o0 = acc[base + 2 * i + 1];
            const double c = cs[pos * 32 + i], s2 = sn[pos * 32 + i];
            want = (dd & 1) ? o0 * c + e0 * s2 : e0 * c - o0 * s2;
          } else {
            want = acc[n];
          }
          const float wf = f16_round(static_cast<float>(want));
          const uint16_t wb = to_f16(wf), gb = got[static_cast<size_t>(r) * 1536 + n];
          const int diff = std::abs(static_cast<int>(wb & 0x7FFF) * ((wb & 0x8000) ? -1 : 1) -
                                    static_cast<int>(gb & 0x7FFF) * ((gb & 0x8000) ? -1 : 1));
          if (diff > 1) ++bad;
        }
      }
      if (bad) {
        std::fprintf(stderr, "KERNEL_REGRESSION RoPE T=%d axis=%d: %lld outputs more than 1 ulp off\n", frames, axis,
                     bad);
        return false;
      }
    }
    std::printf("KERNEL_REGRESSION QKV+RoPE T=%d axes=2 within_1ulp=true\n", frames);
  }
  return true;
}

// Feed-forward at the FF1 regression's M list: the fused kernel against FF1 ->
// fp16 buffer -> FF2, bit for bit, with median timings of both.
bool ff_regression(std::string& rows_json) {
  std::vector<float> w1(1024 * 256), b1(1024), w2(256 * 1024), b2(256);
  for (size_t i = 0; i < w1.size(); ++i) w1[i] = ((static_cast<int>(i % 19)) - 9) / 64.0f;
  for (int i = 0; i < 1024; ++i) b1[i] = ((i % 13) - 6) / 128.0f;
  for (size_t i = 0; i < w2.size(); ++i) w2[i] = ((static_cast<int>(i % 23)) - 11) / 256.0f;
  for (int i = 0; i < 256; ++i) b2[i] = ((i % 7) - 3) / 64.0f;
  std::vector<uint16_t> w1h(w1.size()), w2h(w2.size());
  for (size_t i = 0; i < w1.size(); ++i) w1h[i] = to_f16(w1[i]);
  for (size_t i = 0; i < w2.size(); ++i) w2h[i] = to_f16(w2[i]);
  DevBuf dw1, db1, dw2, db2;
  cudaMalloc(&dw1.p, w1h.size() * 2);
  cudaMalloc(&dw2.p, w2h.size() * 2);
  cudaMalloc(&db1.p, 1024 * 4);
  cudaMalloc(&db2.p, 256 * 4);
  cudaMemcpy(dw1.p, w1h.data(), w1h.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dw2.p, w2h.data(), w2h.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(db1.p, b1.data(), 1024 * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(db2.p, b2.data(), 256 * 4, cudaMemcpyHostToDevice);
  std::vector<std::string> rows;
  for (int m : {1, 37, 127, 129, 16058, 71362}) {
    std::vector<uint16_t> xh(static_cast<size_t>(m) * 256);
    std::vector<float> res(static_cast<size_t>(m) * 256);
    for (size_t i = 0; i < xh.size(); ++i) xh[i] = to_f16(((static_cast<int>(i % 31)) - 15) / 32.0f);
    for (size_t i = 0; i < res.size(); ++i) res[i] = ((static_cast<int>(i % 17)) - 8) / 16.0f;
    DevBuf dx, dr, df, dy1, dy2;
    cudaMalloc(&dx.p, xh.size() * 2);
    cudaMalloc(&dr.p, res.size() * 4);
    cudaMalloc(&df.p, static_cast<size_t>(m) * 1024 * 2);
    cudaMalloc(&dy1.p, res.size() * 4);
    cudaMalloc(&dy2.p, res.size() * 4);
    cudaMemcpy(dx.p, xh.data(), xh.size() * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(dr.p, res.data(), res.size() * 4, cudaMemcpyHostToDevice);
    auto unfused = [&]() {
      return lbrr_op_ff1_gelu(static_cast<uint16_t*>(dx.p), static_cast<uint16_t*>(dw1.p), static_cast<float*>(db1.p),
                              static_cast<uint16_t*>(df.p), m, nullptr) == LBRR_OK &&
             lbrr_op_ff2_resid(static_cast<uint16_t*>(df.p), static_cast<uint16_t*>(dw2.p), static_cast<float*>(db2.p),
                               static_cast<float*>(dr.p), static_cast<float*>(dy1.p), m, nullptr) == LBRR_OK;
    };
    auto fused = [&]() {
      return lbrr_op_feed_forward(static_cast<uint16_t*>(dx.p), static_cast<uint16_t*>(dw1.p),
                                  static_cast<float*>(db1.p), static_cast<uint16_t*>(dw2.p), static_cast<float*>(db2.p),
                                  static_cast<float*>(dr.p), static_cast<float*>(dy2.p), m, nullptr) == LBRR_OK;
    };
    for (int mode = 0; mode < 2; ++mode) {
      auto run = [&]() { return mode == 0 ? unfused() : fused(); };
      for (int i = 0; i < 3; ++i)
        if (!run()) return fail_msg("feed-forward"), false;
      cudaDeviceSynchronize();
      std::vector<double> groups;
      for (int g = 0; g < 3; ++g) {
        cudaEvent_t a0, a1;
        cudaEventCreate(&a0);
        cudaEventCreate(&a1);
        cudaEventRecord(a0, nullptr);
        for (int i = 0; i < 10; ++i) run();
        cudaEventRecord(a1, nullptr);
        cudaEventSynchronize(a1);
        float t = 0;
        cudaEventElapsedTime(&t, a0, a1);
        groups.push_back(t / 10.0);
        cudaEventDestroy(a0);
        cudaEventDestroy(a1);
      }
      if (lbrr_op_sync(nullptr) != LBRR_OK) return fail_msg("feed-forward status"), false;
      std::vector<double> s = groups;
      std::sort(s.begin(), s.end());
      bool equal = true;
      if (mode == 1) {
        std::vector<float> y1(res.size()), y2(res.size());
        cudaMemcpy(y1.data(), dy1.p, y1.size() * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(y2.data(), dy2.p, y2.size() * 4, cudaMemcpyDeviceToHost);
        equal = std::memcmp(y1.data(), y2.data(), y1.size() * 4) == 0;
        if (!equal) {
          std::fprintf(stderr, "KERNEL_REGRESSION FF M=%d: fused differs from FF1 -> FF2\n", m);
          return false;
        }
      }
      const char* name = mode == 0 ? "ff1_gelu+ff2_resid" : "ff_fused";
      std::printf("KERNEL_REGRESSION FF M=%d mode=%s median=%.5fms bit_equal=true\n", m, name, s[1]);
      rows.push_back(jobj({{"m", jint(m)}, {"n", "1024"}, {"k", "256"}, {"mode", jstr(name)}, {"median_ms", jnum(s[1])},
                           {"groups_ms", jarr({jnum(groups[0]), jnum(groups[1]), jnum(groups[2])})},
                           {"bit_equal", "true"}}));
    }
  }
  rows_json = jarr(rows);
  return true;
}

}  // namespace

int run_kernel_regression(const BenchArgs& a) {
  if (cudaSetDevice(a.device) != cudaSuccess) {
    std::fprintf(stderr, "lbrr_b200: device %d unavailable\n", a.device);
    return 1;
  }
  if (!rope_regression()) return 1;
  lbrr_model_desc d;
  int32_t freqs[64];
  lbrr_default_model(&d, freqs, 64);
  Engine eng;
  if (lbrr_engine_create(a.device, &d, 588800, &eng.e) != LBRR_OK) return fail_msg("engine");
  Checkpoint ck = synthetic_checkpoint(7);
  if (!ola_regression(eng.e, ck)) return 1;
  if (!mask_layout_regression(eng.e, ck)) return 1;
  std::string ff;
  if (!ff_regression(ff)) return 1;
  if (!a.json.empty()) {
    const std::string report = jobj({{"schema_version", "1"}, {"ff1", ff}, {"rope_gate_boundaries", jstr("within_1ulp")},
                                     {"stft_ola", jstr("impulses_1e-6")}, {"compact_mask", jstr("all_slots_written")}});
    std::FILE* f = std::fopen(a.json.c_str(), "w");
    if (!f || std::fprintf(f, "%s\n", report.c_str()) < 0 || std::fclose(f) != 0)
      return std::fprintf(stderr, "lbrr_b200: cannot write %s\n", a.json.c_str()), 1;
  }
  std::printf("KERNEL_REGRESSION_OK\n");
  return 0;
}

}  // namespace lbrr_host
