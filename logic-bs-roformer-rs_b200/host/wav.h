// WAV reading and writing for the host CLI: 16- and 24-bit PCM and 32-bit
// float in, 32-bit float out (the formats of src/audio.rs:12-145).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace lbrr_host {

struct Wav {
  uint32_t sample_rate = 0;
  int channels = 0;
  std::vector<float> samples;  // interleaved, frames * channels
};

// Parses RIFF/WAVE with `fmt ` and `data` chunks in any order (other chunks
// skipped).  PCM16 -> v/32768, PCM24 -> sign-extended v/8388608, float32 as is.
// Returns false with a message in `err` for anything else.
bool read_wav(const std::string& path, Wav& out, std::string& err);

// Writes a 44-byte-header IEEE-float WAV.  Rejects zero channels, a zero sample
// rate, an incomplete last frame and sizes that do not fit the 32-bit fields
// before creating the file.
bool write_wav_f32(const std::string& path, const Wav& wav, std::string& err);

}  // namespace lbrr_host
