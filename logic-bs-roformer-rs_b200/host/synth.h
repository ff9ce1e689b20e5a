// Seeded synthetic checkpoint for the checkpoint-free modes of the host CLI
// (--kernel-regression): every tensor the loader consumes (src/weights.rs:
// 307-432, 1989 keys) with *.weight / *.bias ~ N(0, std), gammas 1, the shared
// QKV / out biases copied into the 24 per-layer keys and the analytic rotary
// frequencies, plus the mask-estimator overrides the regressions need.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "../../include/lbrr_gpu.h"

namespace lbrr_host {

struct Checkpoint {
  std::map<std::string, std::vector<float>> t;  // name -> fp32 data (row-major)
  std::vector<lbrr_weight_view> views() const;   // views into t (valid while t is unchanged)
};

extern const int kBandFreqs[62];
int band_dim(int b);     // 4 * freqs: complex x stereo
int band_offset(int b);  // prefix sum of band_dim

Checkpoint synthetic_checkpoint(uint64_t seed, float std = 0.02f);
std::string mask_key(int stem, int band, const char* leaf);  // leaf: "0.weight", "0.bias", "2.weight", "2.bias"

// Masks of exactly 1 + 0i for every stem, band, frame and channel: second mask
// layer zero, pre-GLU biases 1 (real parts) / 0 (imaginary parts), gate biases
// 100 (sigmoid = 1 in fp32).  The forward then reduces to STFT -> C2R -> OLA.
void make_identity_masks(Checkpoint& c);

// One-hot mask estimators (the reference's mask_layout_regression): hidden
// unit 0 = tanh(x[band][t][0] + stem / 32), all others 0; every pre-GLU column
// copies hidden unit 0 and adds its own bias, column * 3e-5 + stem / 16 + offset.
void make_one_hot_masks(Checkpoint& c, float offset);
float one_hot_bias(int stem, int band, int col, float offset);

}  // namespace lbrr_host
