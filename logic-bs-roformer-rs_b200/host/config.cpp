#include "config.h"

#include <cctype>
#include <cstdlib>
#include <fstream>
#include <sstream>

namespace lbrr_host {

const YamlValue* YamlValue::get(const std::string& key) const {
  if (kind != Map) return nullptr;
  auto it = map.find(key);
  return it == map.end() ? nullptr : &it->second;
}

bool YamlValue::as_long(long long& v) const {
  if (kind != Scalar || text.empty()) return false;
  char* end = nullptr;
  const long long i = std::strtoll(text.c_str(), &end, 10);
  if (*end == '\0') {
    v = i;
    return true;
  }
  const double d = std::strtod(text.c_str(), &end);  // "1.0" and the like
  if (*end != '\0') return false;
  v = static_cast<long long>(d);
  return true;
}

bool YamlValue::as_bool(bool& v) const {
  if (kind != Scalar) return false;
  if (text == "true" || text == "True" || text == "TRUE") v = true;
  else if (text == "false" || text == "False" || text == "FALSE") v = false;
  else return false;
  return true;
}

namespace {
struct Line {
  int num, indent;
  std::string text;
};

std::string trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && std::isspace(static_cast<unsigned char>(s[a]))) ++a;
  while (b > a && std::isspace(static_cast<unsigned char>(s[b - 1]))) --b;
  return s.substr(a, b - a);
}

// `#` starts a comment at the line start or after whitespace, outside quotes.
std::string strip_comment(const std::string& s) {
  char q = 0;
  for (size_t i = 0; i < s.size(); ++i) {
    const char c = s[i];
    if (q) {
      if (c == q) q = 0;
    } else if (c == '\'' || c == '"') {
      q = c;
    } else if (c == '#' && (i == 0 || std::isspace(static_cast<unsigned char>(s[i - 1])))) {
      return s.substr(0, i);
    }
  }
  return s;
}

YamlValue scalar(std::string t) {
  t = trim(t);
  YamlValue v;
  if (t.rfind("!!", 0) == 0) {  // a tag before a scalar: drop it
    const size_t sp = t.find(' ');
    t = sp == std::string::npos ? std::string() : trim(t.substr(sp));
  }
  if (t.empty() || t == "~" || t == "null" || t == "Null" || t == "NULL") return v;
  if (t.size() >= 2 && ((t.front() == '\'' && t.back() == '\'') || (t.front() == '"' && t.back() == '"')))
    t = t.substr(1, t.size() - 2);
  v.kind = YamlValue::Scalar;
  v.text = t;
  return v;
}

bool inline_list(const std::string& t, YamlValue& out, std::string& err) {
  if (t.size() < 2 || t.back() != ']') {
    err = "unterminated inline list";
    return false;
  }
  out = YamlValue();
  out.kind = YamlValue::List;
  const std::string body = t.substr(1, t.size() - 2);
  std::string cur;
  char q = 0;
  for (char c : body) {
    if (q) {
      if (c == q) q = 0;
      cur += c;
    } else if (c == '\'' || c == '"') {
      q = c;
      cur += c;
    } else if (c == ',') {
      out.items.push_back(scalar(cur));
      cur.clear();
    } else {
      cur += c;
    }
  }
  if (!trim(cur).empty() || !out.items.empty()) out.items.push_back(scalar(cur));
  return true;
}

struct Parser {
  std::vector<Line> lines;
  size_t pos = 0;
  std::string err;

  bool value_of(const std::string& rest, int indent, YamlValue& out) {
    const std::string t = trim(rest);
    if (!t.empty() && t[0] == '[') return inline_list(t, out, err);
    const bool tag_only = t.rfind("!!", 0) == 0 && t.find(' ') == std::string::npos;
    if (!t.empty() && !tag_only) {
      out = scalar(t);
      return true;
    }
    // nested block: deeper lines, or a block sequence at the same indentation
    if (pos < lines.size() &&
        (lines[pos].indent > indent || (lines[pos].indent == indent && lines[pos].text.rfind("-", 0) == 0)))
      return block(lines[pos].indent, out);
    out = YamlValue();
    return true;
  }

  bool block(int indent, YamlValue& out) {
    out = YamlValue();
    if (pos >= lines.size()) return true;
    const bool seq = lines[pos].text == "-" || lines[pos].text.rfind("- ", 0) == 0;
    out.kind = seq ? YamlValue::List : YamlValue::Map;
    while (pos < lines.size() && lines[pos].indent == indent) {
      const Line& l = lines[pos];
      const bool is_item = l.text == "-" || l.text.rfind("- ", 0) == 0;
      // a sequence given as a key's value at the key's own indentation ends
      // where the parent mapping continues (and vice versa)
      if (is_item != seq) break;
      ++pos;
      if (seq) {
        YamlValue item;
        if (!value_of(l.text.size() > 1 ? l.text.substr(2) : std::string(), indent, item)) return false;
        out.items.push_back(std::move(item));
      } else {
        const size_t colon = l.text.find(':');
        if (colon == std::string::npos) {
          err = "line " + std::to_string(l.num) + ": expected key: value";
          return false;
        }
        const std::string key = scalar(l.text.substr(0, colon)).text;
        YamlValue v;
        if (!value_of(l.text.substr(colon + 1), indent, v)) return false;
        out.map[key] = std::move(v);
      }
    }
    if (pos < lines.size() && lines[pos].indent > indent) {
      err = "line " + std::to_string(lines[pos].num) + ": unexpected indentation";
      return false;
    }
    return true;
  }
};

bool req_int(const YamlValue* sec, const char* key, long long& v, std::string& err) {
  const YamlValue* x = sec ? sec->get(key) : nullptr;
  if (!x) {
    err = std::string("missing key ") + key;
    return false;
  }
  if (!x->as_long(v)) {
    err = std::string("key ") + key + " not numeric";
    return false;
  }
  return true;
}
}  // namespace

bool parse_yaml(const std::string& text, YamlValue& root, std::string& err) {
  Parser p;
  std::istringstream in(text);
  std::string raw;
  int num = 0;
  while (std::getline(in, raw)) {
    ++num;
    std::string s = strip_comment(raw);
    while (!s.empty() && std::isspace(static_cast<unsigned char>(s.back()))) s.pop_back();
    if (trim(s).empty()) continue;
    int indent = 0;
    while (indent < static_cast<int>(s.size()) && s[indent] == ' ') ++indent;
    p.lines.push_back(Line{num, indent, s.substr(indent)});
  }
  if (p.lines.empty()) {
    root = YamlValue();
    return true;
  }
  if (!p.block(p.lines[0].indent, root) || p.pos != p.lines.size()) {
    err = p.err.empty() ? "line " + std::to_string(p.lines[p.pos].num) + ": unexpected indentation" : p.err;
    return false;
  }
  return true;
}

bool parse_model_config(const std::string& yaml_text, ModelConfig& cfg, std::string& err) {
  YamlValue root;
  if (!parse_yaml(yaml_text, root, err)) return false;
  const YamlValue* audio = root.get("audio");
  const YamlValue* model = root.get("model");
  const YamlValue* training = root.get("training");
  if (!audio) return err = "missing audio section", false;
  if (!model) return err = "missing model section", false;
  if (!training) return err = "missing training section", false;
  long long v = 0;
  struct {
    const YamlValue* sec;
    const char* key;
    int* dst;
  } ints[] = {{model, "dim", &cfg.dim},
              {model, "depth", &cfg.depth},
              {model, "num_stems", &cfg.num_stems},
              {model, "heads", &cfg.heads},
              {model, "dim_head", &cfg.dim_head},
              {model, "dim_freqs_in", &cfg.dim_freqs_in},
              {model, "stft_n_fft", &cfg.stft_n_fft},
              {model, "stft_hop_length", &cfg.stft_hop},
              {model, "stft_win_length", &cfg.stft_win},
              {model, "mlp_expansion_factor", &cfg.mlp_expansion},
              {audio, "sample_rate", &cfg.sample_rate}};
  for (auto& f : ints) {
    if (!req_int(f.sec, f.key, v, err)) return false;
    *f.dst = static_cast<int>(v);
  }
  if (!req_int(audio, "chunk_size", cfg.chunk_size, err)) return false;
  const YamlValue* fb = model->get("freqs_per_bands");
  if (!fb || fb->kind != YamlValue::List) return err = "missing freqs_per_bands", false;
  cfg.freqs_per_bands.clear();
  for (const auto& it : fb->items) {
    if (!it.as_long(v)) return err = "freqs_per_bands entry not numeric", false;
    cfg.freqs_per_bands.push_back(static_cast<int>(v));
  }
  bool b = false;
  const YamlValue* sb = model->get("use_shared_bias");
  cfg.use_shared_bias = sb && sb->as_bool(b) ? b : false;
  const YamlValue* ins = training->get("instruments");
  if (!ins || ins->kind != YamlValue::List) return err = "missing instruments", false;
  cfg.instruments.clear();
  for (const auto& it : ins->items) {
    if (it.kind != YamlValue::Scalar) return err = "instrument name not a string", false;
    cfg.instruments.push_back(it.text);
  }
  long long sum = 0;
  for (int f : cfg.freqs_per_bands) sum += f;
  if (sum != cfg.dim_freqs_in) {
    err = "freqs_per_bands sum " + std::to_string(sum) + " != dim_freqs_in " + std::to_string(cfg.dim_freqs_in);
    return false;
  }
  return true;
}

bool load_model_config(const std::string& model_dir, ModelConfig& cfg, std::string& err) {
  for (const char* name : {"logic_bs_roformer.yaml", "config.yaml"}) {
    std::ifstream f(model_dir + "/" + name);
    if (!f) continue;
    std::stringstream ss;
    ss << f.rdbuf();
    if (!parse_model_config(ss.str(), cfg, err)) {
      err = model_dir + "/" + name + ": " + err;
      return false;
    }
    return true;
  }
  err = "no logic_bs_roformer.yaml or config.yaml in " + model_dir;
  return false;
}

}  // namespace lbrr_host
