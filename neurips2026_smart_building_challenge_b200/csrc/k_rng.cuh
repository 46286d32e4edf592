// The step's random inputs, produced one transition ahead of the step that
// consumes them, beside the thermal solve (none of them depends on
// temperatures):
//   * k_conv, one warp per scenario: the convection draws of one transition
//     (complete_port/csim/sb_convect.c:39-73) -- Bernoulli cell picks,
//     candidate draws, Fisher-Yates shuffle and swaps -- composed into one
//     permutation of the field that every env of the scenario applies. The
//     reference's envs of one scenario draw identical convection sequences
//     (same seed, one batch per step whatever the episode state), so one
//     stream serves them all.
//   * k_occ, one warp per occupancy stream: the
//     RandomizedArrivalDepartureOccupancy chains (complete_port/csim/
//     sb_occup.c:39-71) advanced for the transition and, when it ends the
//     episode, primed and advanced again for the restart
//     (complete_port/pufferlib_cpu_env.h:187-208, 239-256). A stream serves a
//     scenario while its envs step in lock step, else one env (desync,
//     random_start: the reference GPU backend's per-env chains,
//     gpu/sb_gpu_kernels.cuh:385-422). For random_start the stream also draws
//     each new episode's start day (gpu/smart_buildings.cu:1636-1657).
// Transition q (counted from puf_reset) is written to slot q & 1 and read by
// that step's k_post; k_occ's reset mode writes slot kResetSlot for puf_reset.
// In a step both run as programmatic dependents of the first solve (its
// heaviest class's launch when the first solve runs by class), on the SMs its
// slabs leave free once every slab is resident. Only CTA 0 of each waits for
// its primary (griddepcontrol.wait) before it exits, so the producer completes
// after the primary while its other CTAs free their SMs as soon as their work
// is done.
#pragma once
#include "dev_util.cuh"

namespace sbenv {

// SplitMix64's output function (Steele, Lea and Flood, OOPSLA 2014), the
// reference's per-env start-day stream.
SB_HD inline unsigned long long start_mix(unsigned long long x) {
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
}
// One start-day draw: the stream advances by the golden-ratio increment.
SB_HD inline int start_draw(unsigned long long& rng) {
    rng += 0x9e3779b97f4a7c15ULL;
    return (int)(start_mix(rng) % (unsigned long long)kStartDays);
}

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

// Priming interval of an episode that starts at calendar row off.
__device__ inline void occ_prime(WarpMt& m, const ScnDev& s, int* st, int off, double* V) {
    const int r = off < s.m1_rows ? off : 0;
    occ_advance(m, s, st, (int)s.o_hour_m1[r], (int)s.o_wd_m1[r], V);
}

// One transition's convection of one scenario (k_conv's body).
__device__ inline void conv_transition(const StepCtx* __restrict__ ctx, const ScnDev& s, const GroupDev& g,
                                       uint8_t* smem, int lane) {
    const int si = s.scn_index;
    for (int x = lane; x < 625; x += 32) s.conv_ckpt[x] = s.conv_mt[x];
    __syncwarp();
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
    const int slot = ctx->cseq[si] & 1;
    int32_t* pairs = s.conv_pairs + (size_t)slot * s.conv_stride;
    WarpMt m;
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
                pairs[2 * o] = g.cv_pos[x];
                pairs[2 * o + 1] = g.cv_pos[perm[x]];
            }
            npairs += __popc(mask);
        }
    }
    if (lane == 0) {
        s.conv_npairs[slot] = npairs;
        ctx->cseq[si] += 1;
    }
}

// restore = 1 (puf_reset): the stream goes back to its state before the last
// transition produced, which no step consumed. restore = 0: the next
// transition's swaps into slot cseq & 1, the state before it kept.
__global__ void __launch_bounds__(32) k_conv(const StepCtx* __restrict__ ctx, int restore) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int si = blockIdx.x;
    const ScnDev& s = ctx->scns[si];
    const GroupDev& g = ctx->groups[s.group];
    const int lane = threadIdx.x & 31;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (!restore) conv_transition(ctx, s, g, smem, lane);
    else if (*ctx->produced)
        for (int x = lane; x < 625; x += 32) s.conv_mt[x] = s.conv_ckpt[x];
    if (blockIdx.x == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// One warp per occupancy stream, kOccWarps streams per CTA. reset = 1: the
// puf_reset of the stream (start day, priming, first interval) into slot
// kResetSlot; the producer's episode state restarts from the consumer's
// (a transition produced ahead and not consumed is dropped). reset = 0: the
// stream's next transition into slot oseq & 1.
constexpr int kOccWarps = 4;
constexpr size_t kOccWarpSmem = 4 * (624 + 624 + 1248);   // MT blocks; occupant states follow
__device__ inline void occ_stream(const StepCtx* __restrict__ ctx, int u, int reset, uint8_t* smem);

__global__ void __launch_bounds__(32 * kOccWarps) k_occ(const StepCtx* __restrict__ ctx, int reset) {
    extern __shared__ __align__(128) uint8_t smem[];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int u = blockIdx.x * kOccWarps + (threadIdx.x >> 5);
    if (u < ctx->n_ostreams) occ_stream(ctx, u, reset, smem);
    if (blockIdx.x == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// One occupancy stream (one warp of k_occ).
__device__ inline void occ_stream(const StepCtx* __restrict__ ctx, int u, int reset, uint8_t* smem) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const ScnDev& s = ctx->scns[ctx->ostream_scn[u]];
    const size_t per_warp = kOccWarpSmem + 4 * (size_t)ctx->occ_stride;
    uint32_t* st = reinterpret_cast<uint32_t*>(smem + (size_t)w * per_warp);
    uint32_t* nx = st + 624;
    uint32_t* tw = nx + 624;
    int* ost = reinterpret_cast<int*>(tw + 1248);
    const int nocc = s.nz * s.assign;
    int* gst = ctx->occ_state + (size_t)u * ctx->occ_stride;
    uint32_t* gmt = ctx->occ_mt + (size_t)u * 625;
    uint32_t* cmt = ctx->ck_mt + (size_t)u * 625;
    int* cst = ctx->ck_state + (size_t)u * ctx->occ_stride;
    if (reset) {
        // undo the transition produced ahead (none before the first production)
        if (*ctx->produced) {
            for (int x = lane; x < 625; x += 32) gmt[x] = cmt[x];
            for (int x = lane; x < nocc; x += 32) gst[x] = cst[x];
        }
    } else {
        // keep the state before this production
        for (int x = lane; x < 625; x += 32) cmt[x] = gmt[x];
        for (int x = lane; x < nocc; x += 32) cst[x] = gst[x];
    }
    __syncwarp();
    for (int x = lane; x < nocc; x += 32) ost[x] = gst[x];
    WarpMt m;
    mt_load(m, gmt, st, nx, tw);
    const size_t vs = (size_t)ctx->n_ostreams * ctx->nz_max;
    if (reset) {
        // the consumer's state is final (puf_reset synchronises first)
        int len = s.max_steps;
        unsigned long long rng = 0ull;
        if (ctx->ostream_per_env) {
            len = ctx->Ist[(size_t)u * ctx->lay.ni + ctx->lay.eplen];
            rng = ctx->env_rng[u];
        }
        const int off = ctx->random_start ? kStepsPerDay * start_draw(rng) : 0;
        double* Vp = ctx->V_prime + kResetSlot * vs + (size_t)u * ctx->nz_max;
        double* Vz = ctx->V_zero + kResetSlot * vs + (size_t)u * ctx->nz_max;
        occ_prime(m, s, ost, off, Vp);
        occ_advance(m, s, ost, (int)s.o_hour[off], (int)s.o_wd[off], Vz);
        if (lane == 0) {
            ctx->new_off[kResetSlot * ctx->n_ostreams + u] = off;
            ctx->new_rng[kResetSlot * ctx->n_ostreams + u] = rng;
            ctx->ostep[u] = 0;
            ctx->oeplen[u] = len;
            ctx->ooff[u] = off;
            ctx->orng[u] = rng;
            ctx->oseq[u] = 0;
        }
    } else {
        const int slot = ctx->oseq[u] & 1;
        const int tn = ctx->ostep[u] + 1, off = ctx->ooff[u];
        occ_advance(m, s, ost, (int)s.o_hour[off + tn], (int)s.o_wd[off + tn],
                    ctx->V_step + slot * vs + (size_t)u * ctx->nz_max);
        if (tn >= ctx->oeplen[u]) {
            // the transition ends the episode: the restart's start day, priming
            // interval and first interval
            unsigned long long rng = ctx->orng[u];
            const int noff = ctx->random_start ? kStepsPerDay * start_draw(rng) : 0;
            occ_prime(m, s, ost, noff, ctx->V_prime + slot * vs + (size_t)u * ctx->nz_max);
            occ_advance(m, s, ost, (int)s.o_hour[noff], (int)s.o_wd[noff],
                        ctx->V_zero + slot * vs + (size_t)u * ctx->nz_max);
            if (lane == 0) {
                ctx->new_off[slot * ctx->n_ostreams + u] = noff;
                ctx->new_rng[slot * ctx->n_ostreams + u] = rng;
                ctx->ostep[u] = 0;
                ctx->oeplen[u] = s.max_steps;   // every later episode is whole
                ctx->ooff[u] = noff;
                ctx->orng[u] = rng;
            }
        } else if (lane == 0) {
            ctx->ostep[u] = tn;
        }
        if (lane == 0) {
            ctx->oseq[u] += 1;
            *ctx->produced = 1;
        }
    }
    mt_store(m, gmt);
    for (int x = lane; x < nocc; x += 32) gst[x] = ost[x];
}

}  // namespace sbenv
