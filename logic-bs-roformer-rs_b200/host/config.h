// Model configuration for the host CLI: the inference-relevant fields of the
// training YAML (assets/logic_bs_roformer.yaml), read with a small YAML subset
// parser (nested mappings by indentation, block sequences, inline [a, b]
// lists, scalars, `!!python/tuple` tags, `#` comments), the subset
// src/config.rs:1-6 documents.
#pragma once
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace lbrr_host {

struct YamlValue {
  enum Kind { Null, Scalar, List, Map } kind = Null;
  std::string text;                 // Scalar (quotes removed)
  std::vector<YamlValue> items;     // List
  std::map<std::string, YamlValue> map;  // Map
  const YamlValue* get(const std::string& key) const;
  bool as_long(long long& v) const;
  bool as_bool(bool& v) const;
};

// Returns false with a message (and line number) in `err` on malformed input.
bool parse_yaml(const std::string& text, YamlValue& root, std::string& err);

struct ModelConfig {
  int dim = 0, depth = 0, num_stems = 0, heads = 0, dim_head = 0;
  std::vector<int> freqs_per_bands;
  int dim_freqs_in = 0, stft_n_fft = 0, stft_hop = 0, stft_win = 0, mlp_expansion = 0;
  bool use_shared_bias = false;
  long long chunk_size = 0;
  int sample_rate = 0;
  std::vector<std::string> instruments;
};

// ModelConfig::parse of src/config.rs:92-133: required keys, freqs_per_bands
// summing to dim_freqs_in.
bool parse_model_config(const std::string& yaml_text, ModelConfig& cfg, std::string& err);

// Reads <model_dir>/logic_bs_roformer.yaml, else <model_dir>/config.yaml.
bool load_model_config(const std::string& model_dir, ModelConfig& cfg, std::string& err);

}  // namespace lbrr_host
