// Fused thermal solve: forcing -> L sweep -> U sweep -> air-side dense system
// -> second L/U sweep -> interior mass + field update, for one slab of envs
// held in shared memory.
//
// Reference: complete_port/csim/sb_fdm.c:142-188 (one env) and sb_lu.c:38-63
// (the factor replay). The reference pushes each column of L/U into the rows
// below/above it; here every row pulls its terms in the same column order, so
// each row receives exactly the same sequence of subtractions and the result
// is bit-identical. The pull schedule is precomputed on the host
// (sweep_sched.cpp): every warp runs its own stream of bundles (four rows in
// lock step, one lane per env), streamed into a per-warp shared-memory ring
// with cp.async.bulk; before a bundle, the warp acquires the ready flags of
// the other warps' rows it reads.
#pragma once
#include "dev_util.cuh"

namespace sbenv {

struct SlabDesc {
    int group;
    int env0;   // first global env
    int nenv;   // envs in this slab (<= slab_envs)
    int pad;
};

constexpr uint32_t kSpinLimit = 1u << 22;

struct SolveShared {
    double* X;            // [B][stride]
    uint8_t* ring;        // [kSweepWarps][kRingBytes]
    uint64_t* bar;        // [kSweepWarps][kStages]
    uint8_t* ready;       // [n + 1] row ready flags (epoch of the sweep that finished the row)
    volatile int* abort;  // first error of this CTA
};

// Shared-memory bytes of a solve CTA besides the slab's field vectors.
__host__ __device__ constexpr size_t solve_smem_fixed(int n) {
    return (size_t)kSweepWarps * kRingBytes + (size_t)kSweepWarps * kStages * 8 + (((size_t)n + 1 + 15) & ~(size_t)15) +
           256;
}

// One triangular sweep. Every warp runs its own bundle stream; all threads of
// the CTA must call it. par: per-warp parity bits of the ring's mbarriers.
__device__ inline void run_sweep(const SolveShared& sh, const Sweep& sw, int B, int S, int n, uint32_t epoch,
                                 uint32_t& par) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int g = lane >> 3, e = lane & 7;
    const uint8_t* src = sw.stream + (size_t)sw.warp_off[w] * kStageBytes;
    const uint32_t nst = sw.warp_stages[w];
    uint8_t* ring = sh.ring + (size_t)w * kRingBytes;
    uint64_t* bar = sh.bar + w * kStages;
    // lanes of envs beyond the slab's capacity read env 0's field and never
    // store, so they touch no memory outside the field
    const bool owns = e < B;
    double* xe = sh.X + (size_t)(owns ? e : 0) * S;

    uint32_t issued = nst < (uint32_t)kStages ? nst : (uint32_t)kStages;
    uint32_t waited = 0, released = 0, p = 0, ro = 0;
    if (lane == 0) {
        fence_proxy_async();
        for (uint32_t k = 0; k < issued; k++) {
            mbar_expect_tx(&bar[k], kStageBytes);
            bulk_g2s(ring + k * kStageBytes, src + (size_t)k * kStageBytes, kStageBytes, &bar[k]);
        }
    }
    bool ok = true;
    // wait until the stream's bytes [0, end) are in the ring
    auto ensure = [&](uint32_t end) {
        while (end > waited * kStageBytes) {
            if (waited >= issued) { ok = false; break; }
            const uint32_t slot = waited % kStages;
            const uint32_t parity = ((par >> slot) & 1u) ^ ((waited / kStages) & 1u);
            if (!mbar_wait_bounded(&bar[slot], parity)) { ok = false; break; }
            waited++;
        }
    };
    // refill the slots of stages the warp has read completely; only stages
    // whose arrival was observed (a slot's mbarrier must not run two phases
    // ahead of its waiter, or the parity wait would never succeed)
    auto release = [&]() {
        const uint32_t upto = min(p / kStageBytes, waited);
        while (released < upto) {
            const uint32_t k = released + kStages;
            if (k < nst) {
                __syncwarp();
                if (lane == 0) {
                    const uint32_t slot = k % kStages;
                    fence_proxy_async();
                    mbar_expect_tx(&bar[slot], kStageBytes);
                    bulk_g2s(ring + slot * kStageBytes, src + (size_t)k * kStageBytes, kStageBytes, &bar[slot]);
                }
                issued = k + 1;
            }
            released++;
        }
    };

    for (;;) {
        int ab = 0;
        if (lane == 0) ab = *sh.abort;
        ab = __shfl_sync(full, ab, 0);
        ensure(p + sizeof(BundleHeader));
        if (!__all_sync(full, ok) || ab) break;
        const uint8_t* base = ring + ro;
        const uint4 hv = *reinterpret_cast<const uint4*>(base);
        const uint32_t flags = hv.z >> 16, nblk = hv.z & 0xFFFFu;
        if (flags & kBundleEnd) break;
        if (flags & kBundleSkip) {   // the next bundle starts at the ring's beginning
            p += kRingBytes - ro;
            ro = 0;
            ensure(p);   // observe the skipped stages before their slots are refilled
            release();
            continue;
        }
        const uint32_t row = ((g < 2 ? hv.x : hv.y) >> (16 * (g & 1))) & 0xFFFFu;
        const uint32_t fin = (hv.w >> (8 * g)) & 0xFFu;
        const uint32_t npre = (flags >> 8) & 0xFu;
        const uint32_t bsz = (uint32_t)bundle_bytes((int)npre, (flags & 0xF0u) != 0, (int)nblk);
        const bool bad = row > (uint32_t)n || (fin != kFinNever && fin > nblk) || (flags & 0x3000u) ||
                         npre > (uint32_t)kMaxPreItems || bsz > (uint32_t)kMaxBundleBytes ||
                         ro + bsz > (uint32_t)kRingBytes;
        if (__any_sync(full, bad)) { atomicCAS((int*)sh.abort, 0, kErrBadBundle); ok = false; break; }
        ensure(p + bsz);
        if (!__all_sync(full, ok)) break;
        // pre-waits: eight rows per item, one per lane; the warp barrier after
        // them orders every lane's later reads after all the acquires
        if (lane < 8 * (int)npre) {
            const uint32_t r = reinterpret_cast<const uint16_t*>(base + 16)[lane];
            if (r > (uint32_t)n) {
                atomicCAS((int*)sh.abort, 0, kErrBadBundle);
                ok = false;
            } else {
                uint32_t spins = 0;
                while (ld_acquire_u8(sh.ready + r) < epoch) {
                    if (++spins >= kSpinLimit) {
                        atomicCAS((int*)sh.abort, 0, kErrWaitTimeout);
                        ok = false;
                        break;
                    }
                    if ((spins & 1023u) == 0 && *sh.abort) { ok = false; break; }
                }
            }
        }
        __syncwarp();
        if (!__all_sync(full, ok)) break;
        uint32_t off = 16 + 16 * npre;
        const bool pub = (flags >> g) & 1u, div = (flags >> (4 + g)) & 1u;
        double d = 1.0;
        if (flags & 0xF0u) {
            d = reinterpret_cast<const double*>(base + off)[g];
            off += 32;
        }
        double acc = xe[row];
        bool final_written = false;
        auto finish = [&]() {
            if (div) acc = ddiv(acc, d);
            if (owns) xe[row] = acc;
            final_written = true;
            if (pub) {
                __syncwarp(0xFFu << (8 * g));
                if (e == 0) {
                    __threadfence_block();
                    st_release_u8(sh.ready + row, epoch);
                }
            }
        };
        if (fin == 0) finish();
        const uint8_t* bp = base + off;
        for (uint32_t b = 0; b < nblk; b++, bp += kTermBlockBytes) {
            const double2 v01 = *reinterpret_cast<const double2*>(bp + 32 * g);
            const double2 v23 = *reinterpret_cast<const double2*>(bp + 32 * g + 16);
            const uint2 cc = *reinterpret_cast<const uint2*>(bp + 128 + 8 * g);
            const double x0 = xe[cc.x & 0xFFFFu], x1 = xe[cc.x >> 16];
            const double x2 = xe[cc.y & 0xFFFFu], x3 = xe[cc.y >> 16];
            acc = dsub(acc, dmul(v01.x, x0));
            acc = dsub(acc, dmul(v01.y, x1));
            acc = dsub(acc, dmul(v23.x, x2));
            acc = dsub(acc, dmul(v23.y, x3));
            if (fin == b + 1) finish();
        }
        if (!final_written && owns) xe[row] = acc;
        __syncwarp();
        p += bsz;
        ro += bsz;
        if (ro == (uint32_t)kRingBytes) ro = 0;
        release();
    }
    if (!ok) atomicCAS((int*)sh.abort, 0, kErrRingTimeout);
    // every issued stage completes before the ring is reused
    for (; waited < issued; waited++) {
        const uint32_t slot = waited % kStages;
        mbar_wait_bounded(&bar[slot], ((par >> slot) & 1u) ^ ((waited / kStages) & 1u));
    }
    for (uint32_t s = 0; s < (uint32_t)kStages; s++) {
        const uint32_t used = issued > s ? (issued - s + kStages - 1) / kStages : 0;
        par ^= (used & 1u) << s;
    }
    __syncwarp();
}

// Dense k x k system M q = b per env with partial pivoting, the reference's
// elimination order (complete_port/csim/sb_fdm.c:9-38): first maximal |pivot|,
// rows with a zero multiplier untouched, a zero pivot column ends the solve.
// cap envs are processed at once; M rows have stride k+1 (conflict-free columns).
__device__ inline void dense_solve_chunk(double* base, int k, int cap, const int* live) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ld = k + 1;
    const size_t per_env = (size_t)k * ld + 3 * (size_t)k + 2;
    __shared__ int stop_col[16];
    if (tid < 16) stop_col[tid] = 0;
    __syncthreads();
    for (int c = 0; c < k; c++) {
        // (1) pivot search, row swap and multipliers: one warp per env
        for (int e = warp; e < cap; e += blockDim.x >> 5) {
            if (!live[e] || stop_col[e]) continue;
            double* M = base + e * per_env;
            double* b = M + (size_t)k * ld;
            double* f = b + k;
            const double diag = fabs(M[(size_t)c * ld + c]);
            double best = -1.0;
            int bidx = 1 << 30;
            for (int r = c + 1 + lane; r < k; r += 32) {
                const double v = fabs(M[(size_t)r * ld + c]);
                if (v > best) { best = v; bidx = r; }   // NaN never wins (as in the scan)
            }
            for (int o = 16; o > 0; o >>= 1) {
                const double ob = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
                if (ob > best || (ob == best && oi < bidx)) { best = ob; bidx = oi; }
            }
            // sequential scan semantics: the diagonal is the initial best; a later
            // row replaces it only if strictly larger (a NaN diagonal is never replaced)
            int piv = c;
            double pbest = diag;
            if (bidx < k && best > diag) { piv = bidx; pbest = best; }
            if (pbest == 0.0) {
                if (lane == 0) stop_col[e] = 1;
                __syncwarp();
                continue;
            }
            if (piv != c) {
                for (int j = c + lane; j < k; j += 32) {
                    const double t = M[(size_t)c * ld + j];
                    M[(size_t)c * ld + j] = M[(size_t)piv * ld + j];
                    M[(size_t)piv * ld + j] = t;
                }
                if (lane == 0) { const double t = b[c]; b[c] = b[piv]; b[piv] = t; }
            }
            __syncwarp();
            const double d = M[(size_t)c * ld + c];
            for (int r = c + 1 + lane; r < k; r += 32) f[r] = ddiv(M[(size_t)r * ld + c], d);
            __syncwarp();
        }
        __syncthreads();
        // (2) rank-1 update of the trailing rows (columns c+1..k-1) and of b
        const int rows = k - c - 1;
        if (rows > 0) {
            const int cols = k - c;   // column slot 0 updates b, slots 1.. the matrix
            const int per = rows * cols;
            for (int idx = tid; idx < cap * per; idx += blockDim.x) {
                const int e = idx / per, rem = idx % per;
                if (!live[e] || stop_col[e]) continue;
                const int r = c + 1 + rem / cols, jj = rem % cols;
                double* M = base + e * per_env;
                double* b = M + (size_t)k * ld;
                const double fr = b[k + r];
                if (fr == 0.0) continue;
                if (jj == 0) b[r] = dsub(b[r], dmul(fr, b[c]));
                else {
                    const int j = c + jj;
                    M[(size_t)r * ld + j] = dsub(M[(size_t)r * ld + j], dmul(fr, M[(size_t)c * ld + j]));
                }
            }
        }
        __syncthreads();
    }
    // (3) back substitution, one warp per env: products in parallel, the
    // subtraction chain in the reference's ascending-column order on lane 0
    for (int e = warp; e < cap; e += blockDim.x >> 5) {
        if (!live[e] || stop_col[e]) continue;
        double* M = base + e * per_env;
        double* b = M + (size_t)k * ld;
        double* prod = b + 2 * k;
        for (int r = k - 1; r >= 0; r--) {
            for (int j = r + 1 + lane; j < k; j += 32) prod[j] = dmul(M[(size_t)r * ld + j], b[j]);
            __syncwarp();
            if (lane == 0) {
                double s = b[r];
                for (int j = r + 1; j < k; j++) s = dsub(s, prod[j]);
                b[r] = ddiv(s, M[(size_t)r * ld + r]);
            }
            __syncwarp();
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kSolveThreads, 1)
k_solve(const StepCtx* __restrict__ ctx, const SlabDesc* __restrict__ slabs) {
    extern __shared__ __align__(128) uint8_t smem[];
    const SlabDesc sd = slabs[blockIdx.x];
    const GroupDev& g = ctx->groups[sd.group];
    const StateLayout& L = ctx->lay;
    const int B = g.slab_envs, S = g.stride, n = g.n, ncv = g.ncv, k = g.k;
    const int nenv = sd.nenv;
    const int tid = threadIdx.x;

    // shared memory: field [B][S] | rings | mbarriers | ready flags | misc
    SolveShared sh;
    sh.X = reinterpret_cast<double*>(smem);
    sh.ring = smem + (size_t)B * S * sizeof(double);
    sh.bar = reinterpret_cast<uint64_t*>(sh.ring + (size_t)kSweepWarps * kRingBytes);
    sh.ready = reinterpret_cast<uint8_t*>(sh.bar + kSweepWarps * kStages);
    int* misc = reinterpret_cast<int*>(sh.ready + ((n + 1 + 15) & ~15));
    sh.abort = misc;
    double* amb_e = reinterpret_cast<double*>(misc + 4);   // [8]
    int* active = reinterpret_cast<int*>(amb_e + 8);        // [8]
    if (tid < kSweepWarps * kStages) mbar_init(&sh.bar[tid], 1);
    if (tid == 0) misc[0] = 0;
    for (int i = tid; i <= n; i += blockDim.x) sh.ready[i] = i < n ? 0 : 0xFF;   // slot n: "no row"
    // padding slots (the zero column of padded terms) and envs the slab does not fill
    for (int e = 0; e < B; e++) {
        const int from = e < nenv ? n : 0;
        for (int i = from + tid; i < S; i += blockDim.x) sh.X[(size_t)e * S + i] = 0.0;
    }
    if (tid < nenv) {
        const int env = sd.env0 + tid;
        const ScnDev& sc = ctx->scns[ctx->envs[env].scn];
        const int step = ctx->Ist[(size_t)env * L.ni + L.step];
        amb_e[tid] = sc.amb[step];
        const double* D = ctx->Dst + (size_t)env * L.nd;
        int act = 0;
        for (int c = 0; c < k; c++)
            if (D[L.ag + c] != 0.0) { act = 1; break; }
        active[tid] = act;
    } else if (tid < 8) {
        active[tid] = 0;
    }
    mbar_fence_init();
    __syncthreads();
    uint32_t par = 0;   // ring mbarrier parities of this thread's warp

    // ---- forcing (sb_fdm.c:146-152), written in row order ----
    for (int idx = tid; idx < nenv * n; idx += blockDim.x) {
        const int e = idx / n, i = idx % n;
        const int env = sd.env0 + e, local = env - g.env0;
        const double* D = ctx->Dst + (size_t)env * L.nd;
        const int z = g.zone_of_row[i];
        const double q = z >= 0 ? D[L.qdiv + z] : 0.0;
        const double Ti = g.T[(size_t)local * ncv + i];
        const double Mi = g.M[(size_t)local * n + i];
        double b = dadd(dmul(g.cap[i], Ti), q);
        b = dadd(b, dmul(amb_e[e], g.dirx[i]));
        b = dadd(b, dmul(g.mc[i], Mi));
        sh.X[(size_t)e * S + i] = b;
    }
    __syncthreads();

    // ---- first solve ----
    run_sweep(sh, g.fwd, B, S, n, 1, par);
    __syncthreads();
    run_sweep(sh, g.bwd, B, S, n, 2, par);
    __syncthreads();
    if (*sh.abort) {   // uniform: read after the barrier
        if (tid == 0) set_error(ctx->status, *sh.abort);
        return;
    }

    // ---- air side (sb_fdm.c:155-181) ----
    double* pw = reinterpret_cast<double*>(sh.ring);   // [B][k], ring is idle between sweeps
    int any_active = 0;
    for (int e = 0; e < nenv; e++) any_active |= active[e];
    if (k > 0 && any_active) {
        for (int idx = tid; idx < nenv * k; idx += blockDim.x) {
            const int e = idx / k, i = idx % k;
            if (!active[e]) continue;
            const double* xe = sh.X + (size_t)e * S;
            double acc = 0.0;
            for (int p = g.sn_p[i]; p < g.sn_p[i + 1]; p++) acc = dadd(acc, dmul(g.sn_x[p], xe[g.sn_pos[p]]));
            const double* D = ctx->Dst + (size_t)(sd.env0 + e) * L.nd;
            pw[e * k + i] = dmul(D[L.ag + i], dsub(D[L.aT + i], acc));
        }
    }
    // y -> the field array (row positions); the second solve adds to it
    for (int idx = tid; idx < nenv * n; idx += blockDim.x) {
        const int e = idx / n, i = idx % n;
        const int local = sd.env0 + e - g.env0;
        g.T[(size_t)local * ncv + i] = sh.X[(size_t)e * S + i];
    }
    __syncthreads();
    if (k > 0 && any_active) {
        const int ld = k + 1;
        const size_t per_env = (size_t)k * ld + 3 * (size_t)k + 2;
        const int cap_all = (int)(((size_t)B * S) / per_env);
        const int cap = cap_all < 1 ? 1 : (cap_all > 16 ? 16 : cap_all);
        double* base = sh.X;
        __shared__ int live[16];
        for (int e0 = 0; e0 < nenv; e0 += cap) {
            const int ce = (nenv - e0) < cap ? (nenv - e0) : cap;
            if (tid < 16) live[tid] = (tid < ce) ? active[e0 + tid] : 0;
            __syncthreads();
            const int per = k * k;
            for (int idx = tid; idx < ce * per; idx += blockDim.x) {
                const int e = idx / per, rem = idx % per, i = rem / k, j = rem % k;
                if (!live[e]) continue;
                const double* D = ctx->Dst + (size_t)(sd.env0 + e0 + e) * L.nd;
                double* M = base + e * per_env;
                M[(size_t)i * ld + j] = dadd(i == j ? 1.0 : 0.0, dmul(D[L.ag + i], g.S[(size_t)i * k + j]));
            }
            for (int idx = tid; idx < ce * k; idx += blockDim.x) {
                const int e = idx / k, i = idx % k;
                if (live[e]) base[e * per_env + (size_t)k * ld + i] = pw[(e0 + e) * k + i];
            }
            __syncthreads();
            dense_solve_chunk(base, k, ce, live);
            for (int idx = tid; idx < ce * k; idx += blockDim.x) {
                const int e = idx / k, i = idx % k;
                if (live[e]) pw[(e0 + e) * k + i] = base[e * per_env + (size_t)k * ld + i];
            }
            __syncthreads();
        }
        // r = applied q, pulled per row in ascending column order; zero q skipped.
        // The dense workspace overlapped the field: padding slots and unused
        // envs are zeroed again (padded sweep terms read the zero slot).
        for (int idx = tid; idx < B * S; idx += blockDim.x) {
            const int e = idx / S, i = idx % S;
            double acc = 0.0;
            if (e < nenv && i < n && active[e]) {
                for (int p = g.ap_rp[i]; p < g.ap_rp[i + 1]; p++) {
                    const double qj = pw[e * k + g.ap_col[p]];
                    if (qj == 0.0) continue;
                    acc = dadd(acc, dmul(g.ap_x[p], qj));
                }
            }
            sh.X[(size_t)e * S + i] = acc;
        }
        __syncthreads();
        run_sweep(sh, g.fwd, B, S, n, 3, par);
        __syncthreads();
        run_sweep(sh, g.bwd, B, S, n, 4, par);
        __syncthreads();
        if (*sh.abort) {
            if (tid == 0) set_error(ctx->status, *sh.abort);
            return;
        }
    }

    // ---- interior mass + field (sb_fdm.c:183-187) ----
    for (int idx = tid; idx < nenv * n; idx += blockDim.x) {
        const int e = idx / n, i = idx % n;
        const int local = sd.env0 + e - g.env0;
        double y = g.T[(size_t)local * ncv + i];
        if (k > 0 && active[e]) y = dadd(y, sh.X[(size_t)e * S + i]);
        const double m = g.M[(size_t)local * n + i];
        g.M[(size_t)local * n + i] = dadd(dmul(m, g.ret[i]), dmul(g.gain[i], y));
        g.T[(size_t)local * ncv + i] = y;
    }
    for (int idx = tid; idx < nenv * (ncv - n); idx += blockDim.x) {
        const int e = idx / (ncv - n), i = n + idx % (ncv - n);
        const int local = sd.env0 + e - g.env0;
        g.T[(size_t)local * ncv + i] = amb_e[e];
    }
}

}  // namespace sbenv
