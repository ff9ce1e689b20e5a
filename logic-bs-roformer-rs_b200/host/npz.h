// Reader for .npz fixtures (the reference's --bench-ref golden: "inp" [1,2,L]
// or [2,L], "out" [1,6,2,L] or [6,2,L], src/main.rs:7258-7266, read there by
// src/npz.rs).  Supports what numpy.savez writes: a zip of stored (not
// deflated) entries, zip64 size fields, and little-endian float32 C-order .npy
// arrays.  numpy.savez_compressed fixtures are reported as unsupported.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace lbrr_host {

struct NpyArray {
  std::vector<int64_t> shape;
  std::vector<float> data;
};

bool read_npz_f32(const std::string& path, std::map<std::string, NpyArray>& out, std::string& err);

}  // namespace lbrr_host
