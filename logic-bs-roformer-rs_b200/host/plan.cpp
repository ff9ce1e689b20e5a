#include "plan.h"

#include <algorithm>
#include <cctype>
#include <cstdlib>

namespace lbrr_host {

const char* const kDefaultInstruments[6] = {"bass", "drums", "other", "vocals", "guitar", "piano"};

namespace {
std::string lower(std::string s) {
  for (char& c : s) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
  return s;
}
std::string trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && std::isspace(static_cast<unsigned char>(s[a]))) ++a;
  while (b > a && std::isspace(static_cast<unsigned char>(s[b - 1]))) --b;
  return s.substr(a, b - a);
}
}  // namespace

bool parse_mode(const std::string& s, Mode& m, std::string& err) {
  const std::string t = lower(trim(s));
  if (t == "stems" || t == "stem" || t == "detailed" || t == "detail" || t == "6") {
    m = Mode::Stems;
    return true;
  }
  if (t == "vocals" || t == "vocal" || t == "inst" || t == "instrumental" || t == "karaoke" || t == "2") {
    m = Mode::Vocals;
    return true;
  }
  err = "bad output mode \"" + t + "\": expected stems|vocals";
  return false;
}

bool parse_stems(const std::string& spec, const std::vector<std::string>& names, std::vector<int>& out,
                 std::string& err) {
  out.clear();
  const std::string s = trim(spec);
  if (s.empty() || lower(s) == "all") {
    for (int i = 0; i < static_cast<int>(names.size()); ++i) out.push_back(i);
    return true;
  }
  std::string part;
  auto flush = [&]() -> bool {
    const std::string p = trim(part);
    part.clear();
    if (p.empty()) return true;
    char* end = nullptr;
    long idx = std::strtol(p.c_str(), &end, 10);
    if (*end != '\0') {
      idx = -1;
      for (size_t i = 0; i < names.size(); ++i)
        if (lower(names[i]) == lower(p)) idx = static_cast<long>(i);
      if (idx < 0) {
        std::string all;
        for (size_t i = 0; i < names.size(); ++i) all += (i ? ", " : "") + names[i];
        err = "unknown stem \"" + p + "\": expected one of " + all + " or an index";
        return false;
      }
    }
    if (idx < 0 || idx >= static_cast<long>(names.size())) {
      err = "stem index " + std::to_string(idx) + " out of range (0.." + std::to_string(names.size()) + ")";
      return false;
    }
    if (std::find(out.begin(), out.end(), static_cast<int>(idx)) == out.end()) out.push_back(static_cast<int>(idx));
    return true;
  };
  for (char c : s) {
    if (c == ',' || c == ';' || c == ' ') {
      if (!flush()) return false;
    } else {
      part += c;
    }
  }
  if (!flush()) return false;
  if (out.empty()) {
    err = "no stems selected";
    return false;
  }
  std::sort(out.begin(), out.end());
  return true;
}

int vocals_index(const std::vector<std::string>& names) {
  for (size_t i = 0; i < names.size(); ++i)
    if (lower(names[i]).find("vocal") != std::string::npos) return static_cast<int>(i);
  return names.size() == 6 ? 3 : 0;
}

std::vector<Target> plan_targets(const Plan& p, const std::vector<std::string>& names) {
  std::vector<Target> out;
  if (p.mode == Mode::Stems) {
    std::vector<int> st;
    for (int i : p.stems)
      if (i >= 0 && i < static_cast<int>(names.size()) && std::find(st.begin(), st.end(), i) == st.end()) st.push_back(i);
    std::sort(st.begin(), st.end());
    for (int i : st) out.push_back(Target{std::to_string(i) + "_" + names[i] + ".wav", {i}});
  } else {
    const int v = vocals_index(names);
    out.push_back(Target{"vocals.wav", {v}});
    Target inst{"instrumental.wav", {}};
    for (int i = 0; i < static_cast<int>(names.size()); ++i)
      if (i != v) inst.sources.push_back(i);
    if (!inst.sources.empty()) out.push_back(inst);
  }
  return out;
}

std::string plan_summary(const Plan& p, const std::vector<std::string>& names) {
  std::string files;
  for (const auto& t : plan_targets(p, names)) files += (files.empty() ? "" : ", ") + t.file;
  return std::string(p.mode == Mode::Stems ? "detailed stems" : "vocals / instrumental") + " (" + files + ")";
}

}  // namespace lbrr_host
