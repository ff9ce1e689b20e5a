// Output plan of a separation (src/plan.rs): which files are written and
// from which stems.  `stems` mode writes `<index>_<name>.wav` per selected
// stem; `vocals` mode writes `vocals.wav` and `instrumental.wav`, the sum of
// every other stem.
#pragma once
#include <string>
#include <vector>

namespace lbrr_host {

enum class Mode { Stems, Vocals };

struct Target {
  std::string file;
  std::vector<int> sources;  // stems summed into this file (one for a plain stem)
};

struct Plan {
  Mode mode = Mode::Stems;
  std::vector<int> stems;  // selected stems in stems mode
};

extern const char* const kDefaultInstruments[6];

// "stems|stem|detailed|detail|6" or "vocals|vocal|inst|instrumental|karaoke|2".
bool parse_mode(const std::string& s, Mode& m, std::string& err);
// "all", or names / indices separated by commas, semicolons or spaces.
bool parse_stems(const std::string& spec, const std::vector<std::string>& names, std::vector<int>& out,
                 std::string& err);
// The stem whose name contains "vocal", else the fourth of six, else the first.
int vocals_index(const std::vector<std::string>& names);
std::vector<Target> plan_targets(const Plan& p, const std::vector<std::string>& names);
std::string plan_summary(const Plan& p, const std::vector<std::string>& names);

}  // namespace lbrr_host
