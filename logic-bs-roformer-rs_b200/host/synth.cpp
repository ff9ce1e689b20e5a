#include "synth.h"

#include <cmath>

namespace lbrr_host {

const int kBandFreqs[62] = {2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,
                            2,  2,  2,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  12, 12, 12, 12, 12, 12,
                            12, 12, 24, 24, 24, 24, 24, 24, 24, 24, 48, 48, 48, 48, 48, 48, 48, 48, 128, 129};

int band_dim(int b) { return 4 * kBandFreqs[b]; }
int band_offset(int b) {
  int o = 0;
  for (int i = 0; i < b; ++i) o += band_dim(i);
  return o;
}

std::vector<lbrr_weight_view> Checkpoint::views() const {
  std::vector<lbrr_weight_view> v;
  v.reserve(t.size());
  for (const auto& kv : t)
    v.push_back(lbrr_weight_view{kv.first.c_str(), kv.second.data(), static_cast<int64_t>(kv.second.size())});
  return v;
}

std::string mask_key(int stem, int band, const char* leaf) {
  return "mask_estimators." + std::to_string(stem) + ".to_freqs." + std::to_string(band) + ".0." + leaf;
}

namespace {
struct Normal {
  uint64_t s;
  bool have = false;
  double spare = 0;
  double uni() {  // xorshift64*, 53-bit uniform in (0, 1)
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return ((s * 2685821657736338717ull) >> 11) * (1.0 / 9007199254740992.0) + 1e-300;
  }
  double next() {
    if (have) {
      have = false;
      return spare;
    }
    const double r = std::sqrt(-2.0 * std::log(uni())), a = 6.283185307179586 * uni();
    spare = r * std::sin(a);
    have = true;
    return r * std::cos(a);
  }
};
}  // namespace

Checkpoint synthetic_checkpoint(uint64_t seed, float std) {
  Checkpoint c;
  Normal g{seed * 0x9E3779B97F4A7C15ull + 1};
  auto rnd = [&](const std::string& k, size_t n) {
    std::vector<float> v(n);
    for (auto& x : v) x = static_cast<float>(g.next() * std);
    c.t[k] = std::move(v);
  };
  auto ones = [&](const std::string& k, size_t n) { c.t[k] = std::vector<float>(n, 1.0f); };
  rnd("linear_62_bias_0", 1536);
  rnd("linear_64_bias_0", 256);
  for (int l = 0; l < 12; ++l)
    for (int a = 0; a < 2; ++a) {
      const std::string p = "layers." + std::to_string(l) + "." + std::to_string(a) + ".layers.0.0";
      const std::string f = "layers." + std::to_string(l) + "." + std::to_string(a) + ".layers.0.1.net";
      ones(p + ".norm.gamma", 256);
      rnd(p + ".to_qkv.weight", 1536 * 256);
      rnd(p + ".to_gates.weight", 8 * 256);
      rnd(p + ".to_gates.bias", 8);
      rnd(p + ".to_out.0.weight", 256 * 512);
      ones(f + ".0.gamma", 256);
      rnd(f + ".1.weight", 1024 * 256);
      rnd(f + ".1.bias", 1024);
      rnd(f + ".4.weight", 256 * 1024);
      rnd(f + ".4.bias", 256);
      c.t[p + ".to_qkv.bias"] = c.t["linear_62_bias_0"];
      c.t[p + ".to_out.0.bias"] = c.t["linear_64_bias_0"];
      std::vector<float> fr(32);
      for (int i = 0; i < 32; ++i) fr[i] = 1.0f / std::pow(10000.0f, (2.0f * i) / 64.0f);
      c.t[p + ".rotary_embed.freqs"] = fr;
    }
  ones("final_norm.gamma", 256);
  for (int b = 0; b < 62; ++b) {
    const std::string p = "band_split.to_features." + std::to_string(b);
    const int d = band_dim(b);
    ones(p + ".0.gamma", d);
    rnd(p + ".1.weight", static_cast<size_t>(256) * d);
    rnd(p + ".1.bias", 256);
  }
  for (int s = 0; s < 6; ++s)
    for (int b = 0; b < 62; ++b) {
      const int d = band_dim(b);
      rnd(mask_key(s, b, "0.weight"), 1024 * 256);
      rnd(mask_key(s, b, "0.bias"), 1024);
      rnd(mask_key(s, b, "2.weight"), static_cast<size_t>(2 * d) * 1024);
      rnd(mask_key(s, b, "2.bias"), 2 * d);
    }
  return c;
}

void make_identity_masks(Checkpoint& c) {
  for (int s = 0; s < 6; ++s)
    for (int b = 0; b < 62; ++b) {
      const int d = band_dim(b);
      c.t[mask_key(s, b, "2.weight")].assign(static_cast<size_t>(2 * d) * 1024, 0.f);
      std::vector<float>& bias = c.t[mask_key(s, b, "2.bias")];
      bias.assign(2 * d, 100.0f);
      for (int j = 0; j < d; ++j) bias[j] = (j % 2 == 0) ? 1.0f : 0.0f;  // d = fi*4 + ch*2 + (re, im)
    }
}

float one_hot_bias(int stem, int band, int col, float offset) {
  return static_cast<float>((2.0 * band_offset(band) + col) * 0.00003 + stem / 16.0 + offset);
}

void make_one_hot_masks(Checkpoint& c, float offset) {
  for (int s = 0; s < 6; ++s)
    for (int b = 0; b < 62; ++b) {
      const int d = band_dim(b);
      std::vector<float>& w1 = c.t[mask_key(s, b, "0.weight")];
      w1.assign(1024 * 256, 0.f);
      w1[0] = 1.0f;
      std::vector<float>& b1 = c.t[mask_key(s, b, "0.bias")];
      b1.assign(1024, 0.f);
      b1[0] = s / 32.0f;
      std::vector<float>& w2 = c.t[mask_key(s, b, "2.weight")];
      w2.assign(static_cast<size_t>(2 * d) * 1024, 0.f);
      for (int j = 0; j < 2 * d; ++j) w2[static_cast<size_t>(j) * 1024] = 1.0f;
      std::vector<float>& b2 = c.t[mask_key(s, b, "2.bias")];
      b2.resize(2 * d);
      for (int j = 0; j < 2 * d; ++j) b2[j] = one_hot_bias(s, b, j, offset);
    }
}

}  // namespace lbrr_host
