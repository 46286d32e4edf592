// Per-scenario random streams of one step, on a side stream concurrent with
// the pre/solve kernels (neither stream depends on temperatures):
//   * convection: Bernoulli cell picks, candidate draws, Fisher-Yates shuffle
//     and swaps (complete_port/csim/sb_convect.c:39-73), composed into one
//     permutation of the field that every env of the scenario applies;
//   * occupancy: the RandomizedArrivalDepartureOccupancy chains
//     (complete_port/csim/sb_occup.c:39-71), advanced for this step and, when
//     the step ends the episode, primed and advanced again for the restart
//     (complete_port/pufferlib_cpu_env.h:187-208, 239-256).
// All envs of a scenario step in lock step from identical seeds, so their
// streams are identical (the reference seeds every env alike); one warp per
// scenario runs them once.
#pragma once
#include "dev_util.cuh"

namespace sbenv {

struct RngOut {         // per scenario, rewritten every step
    double* V_step;     // [nz] occupancy after this step's advance (reward)
    double* V_prime;    // [nz] pre-episode interval of a restart (reset observation)
    double* V_zero;     // [nz] first interval of a restart (next step)
};

// Occupancy chains for one interval; every lane computes the same values.
__device__ inline void occ_advance(WarpMt& m, const ScnDev& s, int* st, int hour, int workday, double* V) {
    const int lane = threadIdx.x & 31;
    for (int z = 0; z < s.nz; z++) {
        int count = 0;
        int* sz = st + (size_t)z * s.assign;
        for (int a = 0; a < s.assign; a++) {
            int x = sz[a];
            if (!workday) x = 0;
            else if (x == 0) {
                if (hour >= s.ea && hour <= s.la && mt_sample(m) < s.p_arr) x = 1;
            } else if (hour < s.ed) {
                /* stays */
            } else if (hour >= s.ld) {
                x = 0;
            } else if (mt_sample(m) < s.p_dep) {
                x = 0;
            }
            __syncwarp();
            if (lane == 0) sz[a] = x;
            __syncwarp();
            count += x;
        }
        if (lane == 0) V[z] = (double)count;
    }
    __syncwarp();
}

__global__ void __launch_bounds__(32) k_rng(const StepCtx* __restrict__ ctx, int* scn_step, RngOut* outs,
                                              int reset_only) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int si = blockIdx.x;
    const ScnDev& s = ctx->scns[si];
    const GroupDev& g = ctx->groups[s.group];
    const int lane = threadIdx.x & 31;
    // shared memory: MT state 624 | next state 624 | tempered blocks 1248 |
    // perm, cand_off, pick cells, pick candidates (conv cells each) | room pick offsets
    const int ncells = g.cv_off[g.conv_nrooms];
    uint32_t* st = reinterpret_cast<uint32_t*>(smem);   // 624
    uint32_t* nx = st + 624;                             // 624
    uint32_t* tw = nx + 624;                             // 1248
    int* perm = reinterpret_cast<int*>(tw + 1248);       // [ncells]
    int* coff = perm + ncells;                           // [ncells + 1]: candidate list offsets
    int* left = coff + ncells + 1;                       // [ncells]: picked cells, all rooms
    int* right = left + ncells;                          // [ncells]: their candidate list entries
    int* roff = right + ncells;                          // [rooms + 1]: picks per room
    RngOut out = outs[si];
    WarpMt m;

    const int t = scn_step[si];
    const bool restart = reset_only || (t + 1 >= s.max_steps);
    if (!reset_only) {
        // ---------------- convection ----------------
        int npairs = 0;
        if (!(s.conv_p == 0.0 || s.conv_dist == 0)) {
            for (int x = lane; x <= ncells; x += 32) coff[x] = g.cand_off[x];
            for (int x = lane; x < ncells; x += 32) perm[x] = x;
            mt_load(m, s.conv_mt, st, nx, tw);   // its warp barriers order the loads above
            int total = 0;
            for (int rm = 0; rm < g.conv_nrooms; rm++) {
                const int base = g.cv_off[rm], cells = g.cv_off[rm + 1] - base;
                if (lane == 0) roff[rm] = total;
                int* L = left + total;
                int* Rr = right + total;
                int mcount = 0, j = 0;
                while (j < cells) {
                    mt_roll(m);
                    // each remaining cell costs two words unless it is picked: test 32 at once
                    const int jj = j + lane;
                    bool pick = false;
                    if (jj < cells) {
                        const uint32_t a = m.tw[m.pos + 2 * lane] >> 5;
                        const uint32_t b = m.tw[m.pos + 2 * lane + 1] >> 6;
                        const double u = (a * 67108864.0 + b) / 9007199254740992.0;
                        pick = !(u > s.conv_p);
                    }
                    const unsigned mask = __ballot_sync(0xffffffffu, pick);
                    if (mask == 0) {
                        const int adv = (cells - j) < 32 ? (cells - j) : 32;
                        m.pos += 2 * adv;
                        j += adv;
                        continue;
                    }
                    const int f = __ffs(mask) - 1;
                    m.pos += 2 * (f + 1);
                    const int gcell = base + j + f;
                    j += f + 1;
                    const int c0 = coff[gcell], c1 = coff[gcell + 1];
                    if (c1 <= c0) continue;
                    const uint32_t pick_i = mt_bounded(m, (uint32_t)(c1 - c0 - 1));
                    if (lane == 0) {
                        L[mcount] = gcell;
                        Rr[mcount] = c0 + (int)pick_i;   // resolved to a cell after all rooms
                    }
                    mcount++;
                }
                __syncwarp();
                for (int q = mcount - 1; q > 0; q--) {
                    const int u = (int)mt_bounded(m, (uint32_t)q);
                    if (lane == 0) {
                        int x = L[q]; L[q] = L[u]; L[u] = x;
                        x = Rr[q]; Rr[q] = Rr[u]; Rr[u] = x;
                    }
                    __syncwarp();
                }
                total += mcount;
            }
            if (lane == 0) roff[g.conv_nrooms] = total;
            mt_store(m, s.conv_mt);
            // candidate cells of all picks at once, then the swaps of every room
            // composed in order (rooms are disjoint: one lane per room)
            for (int q = lane; q < total; q += 32) right[q] = g.cand_idx[right[q]];
            __syncwarp();
            for (int rm = lane; rm < g.conv_nrooms; rm += 32)
                for (int q = roff[rm]; q < roff[rm + 1]; q++) {
                    const int ia = left[q], ib = right[q];
                    const int x = perm[ia]; perm[ia] = perm[ib]; perm[ib] = x;
                }
            __syncwarp();
            // emit the moved cells, compacted in ascending order
            for (int x0 = 0; x0 < ncells; x0 += 32) {
                const int x = x0 + lane;
                const bool moved = x < ncells && perm[x] != x;
                const unsigned mask = __ballot_sync(0xffffffffu, moved);
                if (moved) {
                    const int o = npairs + __popc(mask & ((1u << lane) - 1u));
                    s.conv_pairs[2 * o] = g.cv_pos[x];
                    s.conv_pairs[2 * o + 1] = g.cv_pos[perm[x]];
                }
                npairs += __popc(mask);
            }
        }
        if (lane == 0) *s.conv_npairs = npairs;
    }
    // ---------------- occupancy ----------------
    int* occ_st = reinterpret_cast<int*>(smem + (size_t)(624 + 624 + 1248) * 4);   // reuse: conv is done
    for (int x = lane; x < s.nz * s.assign; x += 32) occ_st[x] = s.occ_state0[x];
    __syncwarp();
    mt_load(m, s.occ_mt, st, nx, tw);
    if (!reset_only) {
        const int tn = t + 1;
        occ_advance(m, s, occ_st, (int)s.o_hour[tn], (int)s.o_wd[tn], out.V_step);
    }
    if (restart) {
        occ_advance(m, s, occ_st, s.hour_m1, s.wd_m1, out.V_prime);
        occ_advance(m, s, occ_st, (int)s.o_hour[0], (int)s.o_wd[0], out.V_zero);
    }
    mt_store(m, s.occ_mt);
    for (int x = lane; x < s.nz * s.assign; x += 32) s.occ_state0[x] = occ_st[x];
    if (lane == 0) scn_step[si] = restart ? 0 : t + 1;
    // launched as a programmatic dependent of the solve: complete only after it
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

}  // namespace sbenv
