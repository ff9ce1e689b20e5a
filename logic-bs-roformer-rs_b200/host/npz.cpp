#include "npz.h"

#include <cstring>
#include <fstream>
#include <sstream>

namespace lbrr_host {
namespace {

uint32_t u32(const uint8_t* p) { return p[0] | (p[1] << 8) | (p[2] << 16) | (static_cast<uint32_t>(p[3]) << 24); }
uint16_t u16(const uint8_t* p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }
uint64_t u64(const uint8_t* p) { return u32(p) | (static_cast<uint64_t>(u32(p + 4)) << 32); }

// One .npy payload: magic, version, header dict, raw data.
bool parse_npy(const uint8_t* p, uint64_t n, NpyArray& a, std::string& err) {
  if (n < 10 || std::memcmp(p, "\x93NUMPY", 6) != 0) return err = "not an .npy payload", false;
  const int major = p[6];
  uint64_t hl = 0, off = 0;
  if (major == 1) {
    hl = u16(p + 8);
    off = 10;
  } else if (major == 2 || major == 3) {
    if (n < 12) return err = "short .npy header", false;
    hl = u32(p + 8);
    off = 12;
  } else {
    return err = "unsupported .npy version", false;
  }
  if (off + hl > n) return err = "truncated .npy header", false;
  const std::string h(reinterpret_cast<const char*>(p + off), hl);
  if (h.find("'descr': '<f4'") == std::string::npos) return err = "array is not little-endian float32", false;
  if (h.find("'fortran_order': False") == std::string::npos) return err = "Fortran-order arrays unsupported", false;
  const size_t s0 = h.find("'shape': (");
  if (s0 == std::string::npos) return err = "no shape in .npy header", false;
  const size_t s1 = h.find(')', s0);
  std::stringstream ss(h.substr(s0 + 10, s1 - s0 - 10));
  std::string tok;
  a.shape.clear();
  uint64_t numel = 1;
  while (std::getline(ss, tok, ',')) {
    size_t i = tok.find_first_not_of(' ');
    if (i == std::string::npos) continue;
    const long long v = std::stoll(tok.substr(i));
    if (v < 0) return err = "negative dimension", false;
    a.shape.push_back(v);
    numel *= static_cast<uint64_t>(v);
  }
  if (off + hl + numel * 4 > n) return err = "truncated .npy data", false;
  a.data.resize(numel);
  if (numel) std::memcpy(a.data.data(), p + off + hl, numel * 4);
  return true;
}

}  // namespace

bool read_npz_f32(const std::string& path, std::map<std::string, NpyArray>& out, std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return err = "cannot open " + path, false;
  const std::vector<uint8_t> z((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  uint64_t pos = 0;
  while (pos + 30 <= z.size() && u32(&z[pos]) == 0x04034b50u) {
    const uint8_t* h = &z[pos];
    const uint16_t flags = u16(h + 6), method = u16(h + 8), nlen = u16(h + 26), xlen = u16(h + 28);
    uint64_t csize = u32(h + 18), usize = u32(h + 22);
    if (pos + 30 + nlen + xlen > z.size()) return err = path + ": truncated zip header", false;
    const std::string name(reinterpret_cast<const char*>(h + 30), nlen);
    const uint8_t* x = h + 30 + nlen;
    for (uint32_t k = 0; k + 4 <= xlen;) {  // zip64 extended sizes
      const uint16_t id = u16(x + k), sz = u16(x + k + 2);
      if (id == 0x0001) {
        uint32_t q = k + 4;
        if (usize == 0xFFFFFFFFu && q + 8 <= k + 4u + sz) usize = u64(x + q), q += 8;
        if (csize == 0xFFFFFFFFu && q + 8 <= k + 4u + sz) csize = u64(x + q);
      }
      k += 4 + sz;
    }
    if (method != 0) return err = path + ": compressed entry " + name + " (write the fixture with numpy.savez)", false;
    if ((flags & 8) && csize == 0) return err = path + ": streamed zip entry " + name + " unsupported", false;
    const uint64_t data = pos + 30 + nlen + xlen;
    if (data + csize > z.size()) return err = path + ": truncated entry " + name, false;
    std::string key = name;
    if (key.size() > 4 && key.compare(key.size() - 4, 4, ".npy") == 0) key.resize(key.size() - 4);
    NpyArray a;
    if (!parse_npy(&z[data], csize, a, err)) return err = path + ": " + name + ": " + err, false;
    out[key] = std::move(a);
    pos = data + csize;
    if (flags & 8) pos += (pos + 4 <= z.size() && u32(&z[pos]) == 0x08074b50u) ? 16 : 12;
  }
  if (out.empty()) return err = path + ": no arrays found", false;
  return true;
}

}  // namespace lbrr_host
