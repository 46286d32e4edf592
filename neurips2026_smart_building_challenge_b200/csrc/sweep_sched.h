// Host construction of the solve kernel's sweep programs (format in sbenv_dev.h).
#pragma once
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "sbenv_dev.h"

namespace sbenv {

struct HostSweep {
    std::vector<uint8_t> bytes;             // all warps' streams back to back
    uint32_t warp_off[kSweepWarps] = {};    // stage index where warp w's stream starts
    uint32_t warp_stages[kSweepWarps] = {}; // stages in warp w's stream
    int ring_stages = 0;                    // ring depth the streams were laid out for
    // statistics of the schedule: terms, control records (bundles), term
    // records (blocks), waits, published rows and partial sums, row segments
    // (pieces), dense block records and the rows they finish
    int64_t terms = 0, bundles = 0, blocks = 0, prewaits = 0, publishes = 0, pieces = 0;
    int64_t dense_blocks = 0, block_rows = 0;
    double sim_cycles = 0;                  // modelled length of the sweep (cycles of one warp)
    int unpublished_row = -1;               // a row no warp waits for (its ready flag is never set)
};

// Builds the program of one triangular sweep.
//   terms[i]  (column, value) pairs of row i, in the order in which the
//             reference's column push subtracts them from row i;
//   backward  U sweep: every row is finished by a division by diag[i]
//             (rows without terms too); forward rows without terms are final
//             from the start and get no work;
//   ring_stages  depth of the kernel's per-warp ring (a bundle never wraps it).
// Returns "" or an error.
std::string build_sweep(int n, const std::vector<std::vector<std::pair<int, double>>>& terms, bool backward,
                        const std::vector<double>& diag, int ring_stages, HostSweep& out);

}  // namespace sbenv
