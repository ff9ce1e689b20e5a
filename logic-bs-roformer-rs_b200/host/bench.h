// The CLI's measurement modes over the C ABI: --bench / --dualbench (the
// reference's bench_warm, src/main.rs:7254-7362, with its schema-v1 JSON
// report) and --kernel-regression (the checkpoint-free checks of
// src/main.rs:7909-8052, restated for this build's fused kernels).
#pragma once
#include <chrono>
#include <string>

namespace lbrr_host {

struct BenchArgs {
  std::string model_dir, reference, json, output, stage = "waveform";
  int device = 0, warmup = 5, iters = 10;
  bool dual = false;
  std::chrono::steady_clock::time_point process_start;
};

int run_bench(const BenchArgs& a);
int run_kernel_regression(const BenchArgs& a);

}  // namespace lbrr_host
