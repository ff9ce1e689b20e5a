// Host-side .safetensors reader for lbrr_engine_load_safetensors: parses the
// JSON header (8-byte little-endian length, then {name: {dtype, shape,
// data_offsets}}), checks every tensor is F32 with a byte length matching its
// shape, and hands fp32 views to lbrr_engine_load_weights, which validates the
// key set.  Restates SafeTensors::open / f32_tensor / parse_header
// (src/weights.rs:25-120) without the Rust host.
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/lbrr_gpu.h"

namespace {

struct Meta {
  std::string name, dtype;
  std::vector<uint64_t> shape;
  uint64_t start = 0, end = 0;
};

struct Parser {
  const char* s;
  size_t n, i = 0;
  std::string err;
  void ws() {
    while (i < n && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool expect(char c) {
    ws();
    if (i < n && s[i] == c) {
      ++i;
      return true;
    }
    err = std::string("expected '") + c + "' at " + std::to_string(i);
    return false;
  }
  bool string(std::string& out) {
    ws();
    if (i >= n || s[i] != '"') {
      err = "expected string at " + std::to_string(i);
      return false;
    }
    ++i;
    out.clear();
    while (i < n && s[i] != '"') {
      if (s[i] == '\\' && i + 1 < n) {
        out.push_back(s[i + 1]);
        i += 2;
      } else {
        out.push_back(s[i++]);
      }
    }
    if (i >= n) {
      err = "unterminated string";
      return false;
    }
    ++i;
    return true;
  }
  bool number(double& v) {
    ws();
    size_t j = i;
    while (j < n && (std::strchr("+-.eE0123456789", s[j]) != nullptr)) ++j;
    if (j == i) {
      err = "expected number at " + std::to_string(i);
      return false;
    }
    v = std::strtod(std::string(s + i, j - i).c_str(), nullptr);
    i = j;
    return true;
  }
  // skip any JSON value
  bool skip() {
    ws();
    if (i >= n) return false;
    if (s[i] == '"') {
      std::string t;
      return string(t);
    }
    if (s[i] == '{' || s[i] == '[') {
      const char open = s[i], close = open == '{' ? '}' : ']';
      ++i;
      ws();
      if (i < n && s[i] == close) {
        ++i;
        return true;
      }
      for (;;) {
        if (open == '{') {
          std::string k;
          if (!string(k) || !expect(':')) return false;
        }
        if (!skip()) return false;
        ws();
        if (i < n && s[i] == ',') {
          ++i;
          continue;
        }
        return expect(close);
      }
    }
    if (!std::strncmp(s + i, "true", 4) || !std::strncmp(s + i, "null", 4)) {
      i += 4;
      return true;
    }
    if (!std::strncmp(s + i, "false", 5)) {
      i += 5;
      return true;
    }
    double d;
    return number(d);
  }
  bool u64_array(std::vector<uint64_t>& out) {
    if (!expect('[')) return false;
    out.clear();
    ws();
    if (i < n && s[i] == ']') {
      ++i;
      return true;
    }
    for (;;) {
      double d;
      if (!number(d)) return false;
      if (d < 0) {
        err = "negative size";
        return false;
      }
      out.push_back(static_cast<uint64_t>(d));
      ws();
      if (i < n && s[i] == ',') {
        ++i;
        continue;
      }
      return expect(']');
    }
  }
  bool header(std::vector<Meta>& metas) {
    if (!expect('{')) return false;
    ws();
    if (i < n && s[i] == '}') return true;
    for (;;) {
      Meta m;
      if (!string(m.name) || !expect(':')) return false;
      if (m.name == "__metadata__") {
        if (!skip()) return false;
      } else {
        if (!expect('{')) return false;
        for (;;) {
          std::string k;
          if (!string(k) || !expect(':')) return false;
          if (k == "dtype") {
            if (!string(m.dtype)) return false;
          } else if (k == "shape") {
            if (!u64_array(m.shape)) return false;
          } else if (k == "data_offsets") {
            std::vector<uint64_t> o;
            if (!u64_array(o)) return false;
            if (o.size() != 2) {
              err = m.name + ": offsets len != 2";
              return false;
            }
            m.start = o[0];
            m.end = o[1];
          } else if (!skip()) {
            return false;
          }
          ws();
          if (i < n && s[i] == ',') {
            ++i;
            continue;
          }
          if (!expect('}')) return false;
          break;
        }
        metas.push_back(std::move(m));
      }
      ws();
      if (i < n && s[i] == ',') {
        ++i;
        continue;
      }
      return expect('}');
    }
  }
};

}  // namespace

extern "C" const char* lbrr_last_error(void);
extern "C" int lbrr_set_error_for_host(int code, const char* msg);

namespace {
// Parse the file into fp32 buffers and name-keyed views (views point into bufs
// and metas, which the caller keeps alive).
int read_views(const char* path, std::vector<Meta>& metas, std::vector<std::vector<float>>& bufs,
               std::vector<lbrr_weight_view>& views, int64_t* us_read = nullptr, int64_t* us_parse = nullptr) {
  const auto t0 = std::chrono::steady_clock::now();
  FILE* f = std::fopen(path, "rb");
  if (!f) return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, (std::string("open ") + path).c_str());
  uint8_t lb[8];
  if (std::fread(lb, 1, 8, f) != 8) {
    std::fclose(f);
    return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, "short safetensors file");
  }
  uint64_t hlen = 0;
  for (int k = 7; k >= 0; --k) hlen = (hlen << 8) | lb[k];
  if (hlen > (64ull << 20)) {  // src/weights.rs:30-32
    std::fclose(f);
    return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, "safetensors header too large");
  }
  std::string header(hlen, '\0');
  if (std::fread(&header[0], 1, hlen, f) != hlen) {
    std::fclose(f);
    return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, "truncated safetensors header");
  }
  std::vector<uint8_t> data;
  {
    std::fseek(f, 0, SEEK_END);
    const long end = std::ftell(f);
    const long begin = static_cast<long>(8 + hlen);
    if (end < begin) {
      std::fclose(f);
      return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, "truncated safetensors data");
    }
    data.resize(static_cast<size_t>(end - begin));
    std::fseek(f, begin, SEEK_SET);
    if (!data.empty() && std::fread(data.data(), 1, data.size(), f) != data.size()) {
      std::fclose(f);
      return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, "short read of safetensors data");
    }
  }
  std::fclose(f);
  const auto t1 = std::chrono::steady_clock::now();
  Parser p{header.data(), header.size()};
  metas.clear();
  if (!p.header(metas)) return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, ("safetensors header: " + p.err).c_str());
  // copy each tensor into an aligned fp32 buffer (offsets are only byte-aligned)
  bufs.assign(metas.size(), std::vector<float>());
  views.assign(metas.size(), lbrr_weight_view{});
  for (size_t k = 0; k < metas.size(); ++k) {
    const Meta& m = metas[k];
    if (m.dtype != "F32")
      return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, (m.name + ": expected F32, got " + m.dtype).c_str());
    uint64_t numel = 1;
    for (uint64_t d : m.shape) numel *= d;
    if (m.end < m.start || m.end > data.size() || m.end - m.start != numel * 4)
      return lbrr_set_error_for_host(LBRR_ERR_WEIGHTS, (m.name + ": byte length mismatch").c_str());
    bufs[k].resize(numel);
    if (numel) std::memcpy(bufs[k].data(), data.data() + m.start, numel * 4);
    views[k].name = m.name.c_str();
    views[k].data = bufs[k].data();
    views[k].numel = static_cast<int64_t>(numel);
  }
  const auto t2 = std::chrono::steady_clock::now();
  if (us_read) *us_read = std::chrono::duration_cast<std::chrono::microseconds>(t1 - t0).count();
  if (us_parse) *us_parse = std::chrono::duration_cast<std::chrono::microseconds>(t2 - t1).count();
  return LBRR_OK;
}
}  // namespace

extern "C" void lbrr_engine_note_file_times(lbrr_engine* e, int64_t us_read, int64_t us_parse);

extern "C" int lbrr_engine_load_safetensors(lbrr_engine* e, const char* path) {
  if (!e || !path) return lbrr_set_error_for_host(LBRR_ERR_INVALID, "NULL engine or path");
  std::vector<Meta> metas;
  std::vector<std::vector<float>> bufs;
  std::vector<lbrr_weight_view> views;
  int64_t us_read = 0, us_parse = 0;
  if (int rc = read_views(path, metas, bufs, views, &us_read, &us_parse)) return rc;
  const int rc = lbrr_engine_load_weights(e, views.data(), views.size());
  if (rc == LBRR_OK) lbrr_engine_note_file_times(e, us_read, us_parse);
  return rc;
}

extern "C" int lbrr_check_safetensors(const char* path) {
  if (!path) return lbrr_set_error_for_host(LBRR_ERR_INVALID, "NULL path");
  std::vector<Meta> metas;
  std::vector<std::vector<float>> bufs;
  std::vector<lbrr_weight_view> views;
  if (int rc = read_views(path, metas, bufs, views)) return rc;
  return lbrr_check_weights(views.data(), views.size());
}
