#include "wav.h"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>

namespace lbrr_host {

namespace {
uint16_t le16(const uint8_t* p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }
uint32_t le32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}
void put16(uint8_t* p, uint16_t v) {
  p[0] = static_cast<uint8_t>(v);
  p[1] = static_cast<uint8_t>(v >> 8);
}
void put32(uint8_t* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = static_cast<uint8_t>(v >> (8 * i));
}
}  // namespace

bool read_wav(const std::string& path, Wav& out, std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    err = "read " + path + ": cannot open";
    return false;
  }
  std::vector<uint8_t> b((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  if (b.size() < 12 || std::memcmp(b.data(), "RIFF", 4) != 0 || std::memcmp(b.data() + 8, "WAVE", 4) != 0) {
    err = "not a RIFF/WAVE file";
    return false;
  }
  size_t pos = 12;
  bool have_fmt = false, have_data = false;
  uint16_t format = 3, bits = 0;
  uint16_t channels = 0;
  uint32_t rate = 0;
  const uint8_t* data = nullptr;
  size_t data_len = 0;
  while (b.size() - pos >= 8) {
    const uint8_t* id = b.data() + pos;
    const size_t size = le32(b.data() + pos + 4);
    pos += 8;
    if (size > b.size() - pos) {
      err = "truncated WAV chunk";
      return false;
    }
    if (std::memcmp(id, "fmt ", 4) == 0) {
      if (size < 16) {
        err = "short fmt chunk";
        return false;
      }
      const uint8_t* p = b.data() + pos;
      format = le16(p);
      channels = le16(p + 2);
      rate = le32(p + 4);
      bits = le16(p + 14);
      have_fmt = true;
    } else if (std::memcmp(id, "data", 4) == 0) {
      data = b.data() + pos;
      data_len = size;
      have_data = true;
    }
    pos += size;
  }
  if (!have_fmt) {
    err = "missing fmt chunk";
    return false;
  }
  if (!have_data) {
    err = "missing data chunk";
    return false;
  }
  if (channels == 0) {
    err = "WAV with zero channels";
    return false;
  }
  out.sample_rate = rate;
  out.channels = channels;
  out.samples.clear();
  if (format == 1 && bits == 16) {
    out.samples.resize(data_len / 2);
    for (size_t i = 0; i < out.samples.size(); ++i)
      out.samples[i] = static_cast<float>(static_cast<int16_t>(le16(data + 2 * i))) / 32768.0f;
  } else if (format == 1 && bits == 24) {
    out.samples.resize(data_len / 3);
    for (size_t i = 0; i < out.samples.size(); ++i) {
      const uint8_t* c = data + 3 * i;
      const int32_t v = static_cast<int32_t>((static_cast<uint32_t>(c[2]) << 24) | (static_cast<uint32_t>(c[1]) << 16) |
                                             (static_cast<uint32_t>(c[0]) << 8)) >> 8;
      out.samples[i] = static_cast<float>(v) / 8388608.0f;
    }
  } else if (format == 3 && bits == 32) {
    out.samples.resize(data_len / 4);
    std::memcpy(out.samples.data(), data, out.samples.size() * 4);  // little-endian host
  } else {
    err = "unsupported wav: format " + std::to_string(format) + ", " + std::to_string(bits) + " bits";
    return false;
  }
  return true;
}

bool write_wav_f32(const std::string& path, const Wav& wav, std::string& err) {
  if (wav.channels <= 0 || wav.channels > 65535 || wav.sample_rate == 0 ||
      wav.samples.size() % static_cast<size_t>(wav.channels) != 0) {
    err = "invalid WAV sample rate, channel count or incomplete frame";
    return false;
  }
  const uint64_t block_align = static_cast<uint64_t>(wav.channels) * 4;
  const uint64_t byte_rate = static_cast<uint64_t>(wav.sample_rate) * block_align;
  const uint64_t data_len = static_cast<uint64_t>(wav.samples.size()) * 4;
  if (block_align > 0xFFFF || byte_rate > 0xFFFFFFFFull || data_len + 36 > 0xFFFFFFFFull) {
    err = "WAV size fields overflow";
    return false;
  }
  uint8_t h[44];
  std::memcpy(h, "RIFF", 4);
  put32(h + 4, static_cast<uint32_t>(data_len + 36));
  std::memcpy(h + 8, "WAVEfmt ", 8);
  put32(h + 16, 16);
  put16(h + 20, 3);
  put16(h + 22, static_cast<uint16_t>(wav.channels));
  put32(h + 24, wav.sample_rate);
  put32(h + 28, static_cast<uint32_t>(byte_rate));
  put16(h + 32, static_cast<uint16_t>(block_align));
  put16(h + 34, 32);
  std::memcpy(h + 36, "data", 4);
  put32(h + 40, static_cast<uint32_t>(data_len));
  std::FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) {
    err = "write " + path + ": cannot create";
    return false;
  }
  bool ok = std::fwrite(h, 1, 44, f) == 44;
  if (ok && data_len) ok = std::fwrite(wav.samples.data(), 1, data_len, f) == data_len;
  ok = (std::fclose(f) == 0) && ok;
  if (!ok) err = "write " + path + ": I/O error";
  return ok;
}

}  // namespace lbrr_host
