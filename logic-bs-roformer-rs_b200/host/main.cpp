// lbrr_b200: command-line front end over the engine's C ABI, mirroring the
// reference CLI's separation, dry-run, benchmark and model-inspection modes
// (argument parsing src/main.rs:70-141, separate() :7598-7819, --check-weights
// :332-365, --print-config).  WAV in (16/24-bit PCM, 32-bit float; mono is
// duplicated to stereo), one 32-bit float WAV per output target.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <sys/stat.h>
#include <vector>

#include "../../include/lbrr_gpu.h"
#include "bench.h"
#include "config.h"
#include "plan.h"
#include "wav.h"

using namespace lbrr_host;

namespace {

struct Args {
  std::string model_dir = "assets", input, outdir = "separated", mode, stems, bench_json, bench_ref, bench_output,
              bench_stage = "waveform";
  int device = 0, gpus = 1, warmup = 5, iters = 10;
  bool separate = false, dry_run = false, bench = false, dualbench = false, kernel_regression = false,
       print_config = false, check_weights = false;
};

void usage() {
  std::fprintf(stderr,
               "usage: lbrr_b200 [options] --input song.wav [--outdir DIR]          separation\n"
               "       lbrr_b200 --separate --model-dir DIR --input song.wav --outdir DIR [--gpus N] [--device D]\n"
               "       lbrr_b200 --dry-run --input song.wav [--mode vocals|stems] [--stems a,b]   plan only, no GPU\n"
               "       lbrr_b200 --bench --model-dir DIR [--warmup N --iters N --bench-stage waveform]\n"
               "                        [--bench-ref F.npz --bench-json F --bench-output F]   (--dualbench: 2 chunks in flight)\n"
               "       lbrr_b200 --kernel-regression [--bench-json F] [--device D]   checkpoint-free GPU checks\n"
               "       lbrr_b200 --print-config | --check-weights   (with --model-dir DIR)\n"
               "options: --mode stems|vocals, --stems all|names|indices, --device D (first GPU), --gpus N\n");
}

int parse_int(const char* s, const char* name, int lo, int& out) {
  char* end = nullptr;
  const long v = std::strtol(s, &end, 10);
  if (*end != '\0' || v < lo || v > 1 << 30) {
    std::fprintf(stderr, "lbrr_b200: bad %s %s\n", name, s);
    return 2;
  }
  out = static_cast<int>(v);
  return 0;
}

int parse_args(int argc, char** argv, Args& a) {
  for (int i = 1; i < argc; ++i) {
    const std::string s = argv[i];
    auto need = [&](const char* name) -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "lbrr_b200: missing value for %s\n", name);
        return nullptr;
      }
      return argv[++i];
    };
    const char* v = nullptr;
    if (s == "--model-dir") {
      if (!(v = need("--model-dir"))) return 2;
      a.model_dir = v;
    } else if (s == "--input") {
      if (!(v = need("--input"))) return 2;
      a.input = v;
    } else if (s == "--outdir") {
      if (!(v = need("--outdir"))) return 2;
      a.outdir = v;
    } else if (s == "--mode" || s == "--output-mode") {
      if (!(v = need("--mode"))) return 2;
      a.mode = v;
    } else if (s == "--stems" || s == "--tracks") {
      if (!(v = need("--stems"))) return 2;
      a.stems = v;
    } else if (s == "--device") {
      if (!(v = need("--device")) || parse_int(v, "--device", 0, a.device)) return 2;
    } else if (s == "--gpus") {
      if (!(v = need("--gpus")) || parse_int(v, "--gpus", 1, a.gpus)) return 2;
    } else if (s == "--warmup") {
      if (!(v = need("--warmup")) || parse_int(v, "--warmup", 0, a.warmup)) return 2;
    } else if (s == "--iters") {
      if (!(v = need("--iters")) || parse_int(v, "--iters", 1, a.iters)) return 2;
    } else if (s == "--bench-json") {
      if (!(v = need("--bench-json"))) return 2;
      a.bench_json = v;
    } else if (s == "--bench-ref") {
      if (!(v = need("--bench-ref"))) return 2;
      a.bench_ref = v;
    } else if (s == "--bench-output") {
      if (!(v = need("--bench-output"))) return 2;
      a.bench_output = v;
    } else if (s == "--bench-stage") {
      if (!(v = need("--bench-stage"))) return 2;
      a.bench_stage = v;
    } else if (s == "--dualbench") {
      a.dualbench = true;
    } else if (s == "--kernel-regression") {
      a.kernel_regression = true;
    } else if (s == "--separate") {
      a.separate = true;
    } else if (s == "--dry-run" || s == "--plan") {
      a.dry_run = true;
    } else if (s == "--bench") {
      a.bench = true;
    } else if (s == "--print-config") {
      a.print_config = true;
    } else if (s == "--check-weights") {
      a.check_weights = true;
    } else if (s == "-h" || s == "--help") {
      usage();
      std::exit(0);
    } else if (!s.empty() && s[0] != '-') {
      if (!a.input.empty()) {
        std::fprintf(stderr, "lbrr_b200: give either --input or a positional audio path, not both\n");
        return 2;
      }
      a.input = s;
    } else {
      std::fprintf(stderr, "lbrr_b200: unknown argument %s\n", s.c_str());
      return 2;
    }
  }
  return 0;
}

std::vector<std::string> names_of(const ModelConfig* cfg) {
  if (cfg && !cfg->instruments.empty()) return cfg->instruments;
  return std::vector<std::string>(kDefaultInstruments, kDefaultInstruments + 6);
}

// The engine runs exactly the geometry lbrr_default_model describes.
bool supported(const ModelConfig& c, std::string& why) {
  lbrr_model_desc d;
  int32_t freqs[64];
  lbrr_default_model(&d, freqs, 64);
  std::vector<int> want(freqs, freqs + d.num_bands);
  if (c.dim != d.dim || c.depth != d.depth || c.heads != d.heads || c.dim_head != d.dim_head ||
      c.num_stems != d.num_stems || c.mlp_expansion != d.mlp_expansion || c.stft_n_fft != d.n_fft ||
      c.stft_hop != d.hop || c.stft_win != d.n_fft || c.sample_rate != d.sample_rate || c.freqs_per_bands != want) {
    why = "this engine runs the 6-stem, 12-layer, dim-256, 62-band BS-RoFormer of logic_bs_roformer.yaml only";
    return false;
  }
  if (!c.use_shared_bias) {
    why = "the checkpoint layout needs use_shared_bias: true";
    return false;
  }
  if (static_cast<int>(c.instruments.size()) != c.num_stems) {
    why = "training.instruments must name num_stems stems";
    return false;
  }
  return true;
}

bool make_dirs(const std::string& path) {
  std::string cur;
  for (size_t i = 0; i <= path.size(); ++i) {
    if (i == path.size() || path[i] == '/') {
      if (!cur.empty() && cur != "." && mkdir(cur.c_str(), 0755) != 0) {
        struct stat st;
        if (stat(cur.c_str(), &st) != 0 || !S_ISDIR(st.st_mode)) return false;
      }
    }
    if (i < path.size()) cur += path[i];
  }
  return true;
}

int64_t chunk_count(int64_t len) {
  const int64_t C = 588800, STEP = 559360, BORDER = 29440, needed = BORDER + len;
  const int64_t last = std::max<int64_t>(0, (needed - C + STEP - 1) / STEP);
  return last + 1;
}

// Stereo input at 44.1 kHz: mono is duplicated, anything else needs a
// converter (the reference shells out to ffmpeg, which this build does not).
int prepare_input(const std::string& path, Wav& w) {
  std::string err;
  if (!read_wav(path, w, err)) {
    std::fprintf(stderr, "lbrr_b200: input: %s\n", err.c_str());
    return 2;
  }
  if (w.sample_rate != 44100 || w.channels > 2) {
    std::fprintf(stderr, "lbrr_b200: input: %s is %.1f kHz / %d ch; convert it to 44.1 kHz stereo first\n", path.c_str(),
                 w.sample_rate / 1000.0, w.channels);
    return 2;
  }
  if (w.channels == 1) {
    std::vector<float> st(w.samples.size() * 2);
    for (size_t i = 0; i < w.samples.size(); ++i) st[2 * i] = st[2 * i + 1] = w.samples[i];
    w.samples.swap(st);
    w.channels = 2;
  }
  if (w.samples.size() < 2) {
    std::fprintf(stderr, "lbrr_b200: input: %s has no samples\n", path.c_str());
    return 2;
  }
  return 0;
}

int print_config(const Args& a) {
  ModelConfig c;
  std::string err;
  if (!load_model_config(a.model_dir, c, err)) {
    std::fprintf(stderr, "lbrr_b200: %s\n", err.c_str());
    return 1;
  }
  std::string stems;
  for (const auto& s : c.instruments) stems += (stems.empty() ? "" : " ") + s;
  std::printf("model    : dim=%d depth=%d heads=%d dim_head=%d bands=%zu stems=[%s]\n", c.dim, c.depth, c.heads,
              c.dim_head, c.freqs_per_bands.size(), stems.c_str());
  std::printf("stft     : n_fft=%d hop=%d win=%d sample_rate=%d dim_freqs_in=%d\n", c.stft_n_fft, c.stft_hop,
              c.stft_win, c.sample_rate, c.dim_freqs_in);
  std::printf("ff       : mlp_expansion=%d shared_bias=%s chunk_size=%lld\n", c.mlp_expansion,
              c.use_shared_bias ? "true" : "false", c.chunk_size);
  std::string why;
  const bool ok = supported(c, why);
  std::printf("engine   : %s\n", ok ? "supported (sm_100a)" : ("not supported: " + why).c_str());
  return ok ? 0 : 1;
}

int check_weights(const Args& a) {
  ModelConfig c;
  std::string err, why;
  if (!load_model_config(a.model_dir, c, err)) {
    std::fprintf(stderr, "lbrr_b200: %s\n", err.c_str());
    return 1;
  }
  if (!supported(c, why)) {
    std::fprintf(stderr, "lbrr_b200: %s\n", why.c_str());
    return 1;
  }
  const std::string path = a.model_dir + "/model.safetensors";
  const auto t0 = std::chrono::steady_clock::now();
  if (lbrr_check_safetensors(path.c_str()) != LBRR_OK) {
    std::fprintf(stderr, "lbrr_b200: %s: %s\n", path.c_str(), lbrr_last_error());
    return 1;
  }
  const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  std::printf("weights OK: %d layers, %zu bands, %d stems; shared qkv bias len %d (%.0f ms)\n", c.depth,
              c.freqs_per_bands.size(), c.num_stems, 3 * c.heads * c.dim_head, ms);
  std::printf("all checkpoint keys consumed exactly once\n");
  return 0;
}

bool make_plan(const Args& a, const std::vector<std::string>& names, Plan& p) {
  std::string err;
  p.mode = Mode::Stems;
  if (!a.mode.empty() && !parse_mode(a.mode, p.mode, err)) {
    std::fprintf(stderr, "lbrr_b200: %s\n", err.c_str());
    return false;
  }
  if (!parse_stems(a.stems, names, p.stems, err)) {
    std::fprintf(stderr, "lbrr_b200: %s\n", err.c_str());
    return false;
  }
  return true;
}

int dry_run(const Args& a) {
  ModelConfig c;
  std::string err;
  const bool have_cfg = load_model_config(a.model_dir, c, err);
  const auto names = names_of(have_cfg ? &c : nullptr);
  Plan p;
  if (!make_plan(a, names, p)) return 2;
  Wav w;
  if (int rc = prepare_input(a.input, w)) return rc;
  const int64_t len = static_cast<int64_t>(w.samples.size() / 2);
  std::printf("input    : %s [44.1kHz stereo, %.1fs]\n", a.input.c_str(), len / 44100.0);
  std::printf("plan     : %s\n", plan_summary(p, names).c_str());
  std::printf("chunks   : %lld of 588800 samples (step 559360, border 29440)\n", static_cast<long long>(chunk_count(len)));
  std::printf("output   : %s/\n", a.outdir.c_str());
  return 0;
}

struct Engines {
  std::vector<lbrr_engine*> e;
  ~Engines() {
    for (auto* x : e) lbrr_engine_destroy(x);
  }
};

int open_engines(const Args& a, int count, Engines& out) {
  lbrr_model_desc d;
  int32_t freqs[64];
  lbrr_default_model(&d, freqs, 64);
  const std::string path = a.model_dir + "/model.safetensors";
  for (int g = 0; g < count; ++g) {
    lbrr_engine* e = nullptr;
    if (lbrr_engine_create(a.device + g, &d, 588800, &e) != LBRR_OK) {
      std::fprintf(stderr, "lbrr_b200: GPU %d: %s\n", a.device + g, lbrr_last_error());
      return 1;
    }
    out.e.push_back(e);
    if (lbrr_engine_load_safetensors(e, path.c_str()) != LBRR_OK) {
      std::fprintf(stderr, "lbrr_b200: %s: %s\n", path.c_str(), lbrr_last_error());
      return 1;
    }
  }
  return 0;
}

int separate(const Args& a) {
  const auto wall0 = std::chrono::steady_clock::now();
  ModelConfig c;
  std::string err, why;
  if (!load_model_config(a.model_dir, c, err)) {
    std::fprintf(stderr, "lbrr_b200: model: %s\n", err.c_str());
    return 1;
  }
  if (!supported(c, why)) {
    std::fprintf(stderr, "lbrr_b200: model: %s\n", why.c_str());
    return 1;
  }
  Plan p;
  if (!make_plan(a, c.instruments, p)) return 2;
  Wav w;
  if (int rc = prepare_input(a.input, w)) return rc;
  const int64_t len = static_cast<int64_t>(w.samples.size() / 2);
  std::string stems;
  for (const auto& s : c.instruments) stems += (stems.empty() ? "" : " ") + s;
  std::printf("input    : %s [44.1kHz stereo, %.1fs]\n", a.input.c_str(), len / 44100.0);
  std::printf("model    : dim=%d depth=%d bands=%zu stems=[%s]\n", c.dim, c.depth, c.freqs_per_bands.size(), stems.c_str());
  std::printf("plan     : %s\n", plan_summary(p, c.instruments).c_str());
  int ngpu = 0;
  if (cudaGetDeviceCount(&ngpu) != cudaSuccess || a.device + a.gpus > ngpu) {
    std::fprintf(stderr, "lbrr_b200: %d GPU(s) from device %d requested, %d present\n", a.gpus, a.device, ngpu);
    return 1;
  }
  Engines eng;
  if (int rc = open_engines(a, a.gpus, eng)) return rc;
  std::vector<float> out(static_cast<size_t>(2 * c.num_stems) * len);
  const auto g0 = std::chrono::steady_clock::now();
  lbrr_chunk_plan plan{588800, 559360, 29440, LBRR_FADE_LINEAR};
  if (lbrr_separate_song(eng.e.data(), static_cast<int>(eng.e.size()), w.samples.data(), len, &plan, out.data()) !=
      LBRR_OK) {
    std::fprintf(stderr, "lbrr_b200: separation: %s\n", lbrr_last_error());
    return 1;
  }
  const double gpu_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - g0).count();
  std::printf("gpu      : %d GPU(s), %lld chunks, wall %.3fs, RTF %.5f\n", a.gpus,
              static_cast<long long>(chunk_count(len)), gpu_s, gpu_s / (len / 44100.0));
  if (!make_dirs(a.outdir)) {
    std::fprintf(stderr, "lbrr_b200: outdir %s: cannot create\n", a.outdir.c_str());
    return 1;
  }
  std::string files;
  double bytes = 0;
  for (const auto& t : plan_targets(p, c.instruments)) {
    Wav o;
    o.sample_rate = w.sample_rate;
    o.channels = 2;
    o.samples.assign(static_cast<size_t>(len) * 2, 0.f);
    for (int ch = 0; ch < 2; ++ch)
      for (int s : t.sources) {
        const float* src = out.data() + static_cast<size_t>(2 * s + ch) * len;
        for (int64_t i = 0; i < len; ++i) o.samples[2 * i + ch] += src[i];
      }
    const std::string path = a.outdir + "/" + t.file;
    if (!write_wav_f32(path, o, err)) {
      std::fprintf(stderr, "lbrr_b200: %s\n", err.c_str());
      return 1;
    }
    bytes += 44.0 + 8.0 * len;
    files += (files.empty() ? "" : ", ") + t.file;
  }
  std::printf("output   : %zu tracks -> %s/ (%s, %.1f MB total)\n", plan_targets(p, c.instruments).size(),
              a.outdir.c_str(), files.c_str(), bytes / 1e6);
  std::printf("total    : %.1fs wall\n",
              std::chrono::duration<double>(std::chrono::steady_clock::now() - wall0).count());
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  const auto t_start = std::chrono::steady_clock::now();
  Args a;
  if (int rc = parse_args(argc, argv, a)) {
    usage();
    return rc;
  }
  if (a.print_config) return print_config(a);
  if (a.check_weights) return check_weights(a);
  if (a.bench || a.dualbench || a.kernel_regression) {
    BenchArgs b;
    b.model_dir = a.model_dir;
    b.reference = a.bench_ref;
    b.json = a.bench_json;
    b.output = a.bench_output;
    b.stage = a.bench_stage;
    b.device = a.device;
    b.warmup = a.warmup;
    b.iters = a.iters;
    b.dual = a.dualbench;
    b.process_start = t_start;
    if (a.kernel_regression) return run_kernel_regression(b);
    ModelConfig c;
    std::string err, why;
    if (!load_model_config(a.model_dir, c, err) || !supported(c, why)) {
      std::fprintf(stderr, "lbrr_b200: model: %s\n", err.empty() ? why.c_str() : err.c_str());
      return 1;
    }
    return run_bench(b);
  }
  if (a.input.empty()) {
    usage();
    return 2;
  }
  if (a.dry_run) return dry_run(a);
  return separate(a);
}
