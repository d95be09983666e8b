// Stand-in for the reference's tap writer (src/dump.h) used by the
// graph-level pin (test infrastructure): taps are kept in memory by name as
// contiguous f32 arrays instead of being written to dump files.
#pragma once
#include <map>
#include <string>
#include <vector>

namespace tp {
struct tap_writer {
    std::map<std::string, std::vector<float>> taps;
};
}  // namespace tp
