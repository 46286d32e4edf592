// Host construction of the wide solve's level programs (format in sbenv_dev.h).
#pragma once
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "sbenv_dev.h"

namespace sbenv {

struct HostWide {
    std::vector<uint8_t> blocks;      // the level blocks back to back (format in sbenv_dev.h)
    std::vector<uint32_t> lev_off;    // [nlev + 1] byte offset of each level's block
    int nlev = 0;
    int max_bytes = 0;                // largest level block
    int64_t segs = 0, chunks = 0;     // segments and chunks of all levels
    int64_t waits = 0;                // (row, count) acquires of all levels
    int64_t terms = 0, partial = 0;   // terms; segments that leave their row unfinished
    double sim_cycles = 0;            // modelled length of the sweep (cycles of one CTA)
};

// Per-row progress carried from one sweep's program to the next (the ready
// counts and stage numbers run on over both sweeps of a step).
struct WideFlags {
    std::vector<int> cnt;     // segments of the row so far
    std::vector<int> stage;   // stage of its last segment (very negative: none)
    std::vector<int> warp;    // warp of its last segment
    explicit WideFlags(int n = 0) : cnt(n, 0), stage(n, -(1 << 29)), warp(n, -1) {}
};

// Builds the level program of one triangular sweep for a wide-solve CTA.
//   terms[i]  (column, value) pairs of row i in the order in which the
//             reference's column push subtracts them from row i; every
//             segment of the program applies a contiguous run of them, so the
//             order (and so the rounding) of every row is the push order;
//   backward  U sweep: every row is finished by its diagonal (rows without
//             terms too); forward rows without terms are final from the start;
//   stage0    the stage index of the sweep's first level (the L sweep's levels
//             come first, then the U sweep's);
//   flags     the rows' progress before the sweep, updated.
// Returns "" or an error.
std::string build_wide(int n, const std::vector<std::vector<std::pair<int, double>>>& terms, bool backward,
                       int stage0, WideFlags& flags, HostWide& out);

}  // namespace sbenv
