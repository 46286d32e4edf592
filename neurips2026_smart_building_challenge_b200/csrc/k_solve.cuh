// Fused thermal solve: forcing -> L sweep -> U sweep -> air-side dense system
// -> second L/U sweep -> interior mass + field update, for one slab of envs
// held in shared memory.
//
// Reference: complete_port/csim/sb_fdm.c:142-188 (one env) and sb_lu.c:38-63
// (the factor replay). The reference pushes each column of L/U into the rows
// below/above it; here every row pulls its terms in the same column order, so
// each row receives exactly the same sequence of subtractions and the result
// is bit-identical. The pull schedule is precomputed on the host
// (tables.cpp): phases of a level schedule, each phase a list of (row, run of
// terms) tasks, streamed into a shared-memory ring with cp.async.bulk.
#pragma once
#include "dev_util.cuh"

namespace sbenv {

struct SlabDesc {
    int group;
    int env0;   // first global env
    int nenv;   // envs in this slab (<= slab_envs)
    int pad;
};

struct SolveShared {
    double* X;          // [B][stride]
    uint8_t* ring;      // kRingSlots x kRingSlotBytes
    uint64_t* bar;      // kRingSlots
    int* flag;          // [0]: error seen in this CTA
    uint32_t chunk_seq; // chunks consumed by this CTA so far (mbarrier parity)
};

// One sweep over the schedule stream. All threads of the CTA participate.
__device__ inline void run_sweep(SolveShared& sh, const Sweep& sw, int B, int S, int nenv, int n,
                                 int* status) {
    const int tid = threadIdx.x;
    const int grp = tid / B, lane_env = tid % B;
    const int ngrp = blockDim.x / B;
    const uint32_t nch = sw.nchunks;
    uint32_t issue_off = 0;   // producer: byte offset of the next chunk to issue
    if (tid == 0) {
        fence_proxy_async();
        for (uint32_t c = 0; c < nch && c < (uint32_t)kRingSlots; c++) {
            const uint32_t seq = sh.chunk_seq + c;
            const int slot = seq % kRingSlots;
            const uint32_t bytes = sw.first_bytes[c];
            mbar_expect_tx(&sh.bar[slot], bytes);
            bulk_g2s(sh.ring + (size_t)slot * kRingSlotBytes, sw.stream + issue_off, bytes, &sh.bar[slot]);
            issue_off += bytes;
        }
    }
    for (uint32_t c = 0; c < nch; c++) {
        const uint32_t seq = sh.chunk_seq + c;
        const int slot = seq % kRingSlots;
        const uint32_t parity = (seq / kRingSlots) & 1u;
        if (!mbar_wait_bounded(&sh.bar[slot], parity)) sh.flag[0] = kErrRingTimeout;
        const uint8_t* base = sh.ring + (size_t)slot * kRingSlotBytes;
        const ChunkHeader hdr = *reinterpret_cast<const ChunkHeader*>(base);
        const bool ok = hdr.check == (hdr.ntask ^ (hdr.nval << 12) ^ 0x5B5B0000u) &&
                        16u + 10u * hdr.nval + 8u * hdr.ntask <= (uint32_t)kRingSlotBytes;
        if (!ok) sh.flag[0] = kErrBadChunk;
        if (ok && sh.flag[0] == 0) {
            const TaskRec* tasks = reinterpret_cast<const TaskRec*>(base + 16);
            const double* vals = reinterpret_cast<const double*>(base + 16 + 8 * hdr.ntask);
            const uint16_t* cols = reinterpret_cast<const uint16_t*>(vals + hdr.nval);
            double* xe = sh.X + (size_t)lane_env * S;
            for (uint32_t t = grp; t < hdr.ntask; t += ngrp) {
                const TaskRec r = tasks[t];
                const int nterm = (int)r.nterm_lo | ((int)(r.flags_hi & 0x0F) << 8);
                const uint32_t need = r.off + (uint32_t)nterm + ((r.flags_hi & 0x80) ? 1u : 0u);
                if (lane_env >= nenv || r.row >= n || need > hdr.nval) continue;
                double acc = xe[r.row];
                const double* v = vals + r.off;
                const uint16_t* cc = cols + r.off;
                int q = 0;
                for (; q + 4 <= nterm; q += 4) {
                    const double p0 = dmul(v[q], xe[cc[q]]);
                    const double p1 = dmul(v[q + 1], xe[cc[q + 1]]);
                    const double p2 = dmul(v[q + 2], xe[cc[q + 2]]);
                    const double p3 = dmul(v[q + 3], xe[cc[q + 3]]);
                    acc = dsub(acc, p0);
                    acc = dsub(acc, p1);
                    acc = dsub(acc, p2);
                    acc = dsub(acc, p3);
                }
                for (; q < nterm; q++) acc = dsub(acc, dmul(v[q], xe[cc[q]]));
                if (r.flags_hi & 0x80) acc = ddiv(acc, v[nterm]);
                xe[r.row] = acc;
            }
        }
        const uint32_t next_bytes = hdr.next_bytes;
        __syncthreads();
        if (sh.flag[0] != 0) {
            // error: drain the copies still in flight (bounded), then leave the sweep
            if (tid == 0)
                for (uint32_t d = c + 1; d < nch && d < c + kRingSlots; d++) {
                    const uint32_t sq = sh.chunk_seq + d;
                    mbar_wait_bounded(&sh.bar[sq % kRingSlots], (sq / kRingSlots) & 1u);
                }
            __syncthreads();
            break;
        }
        if (tid == 0 && c + kRingSlots < nch) {
            fence_proxy_async();
            mbar_expect_tx(&sh.bar[slot], next_bytes);
            bulk_g2s(sh.ring + (size_t)slot * kRingSlotBytes, sw.stream + issue_off, next_bytes, &sh.bar[slot]);
            issue_off += next_bytes;
        }
    }
    sh.chunk_seq += nch;
    if (tid == 0 && sh.flag[0] != 0) set_error(status, sh.flag[0]);
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

    SolveShared sh;
    sh.X = reinterpret_cast<double*>(smem);
    sh.ring = smem + (size_t)B * S * sizeof(double);
    sh.bar = reinterpret_cast<uint64_t*>(sh.ring + (size_t)kRingSlots * kRingSlotBytes);
    sh.flag = reinterpret_cast<int*>(sh.bar + kRingSlots);
    double* amb_e = reinterpret_cast<double*>(sh.flag + 4);   // [B]
    int* active = reinterpret_cast<int*>(amb_e + 8);           // [B]
    sh.chunk_seq = 0;
    if (tid < kRingSlots) mbar_init(&sh.bar[tid], 1);
    if (tid == 0) sh.flag[0] = 0;
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
    run_sweep(sh, g.fwd, B, S, nenv, n, ctx->status);
    run_sweep(sh, g.bwd, B, S, nenv, n, ctx->status);

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
        // r = applied q, pulled per row in ascending column order; zero q skipped
        for (int idx = tid; idx < nenv * n; idx += blockDim.x) {
            const int e = idx / n, i = idx % n;
            double acc = 0.0;
            if (active[e]) {
                for (int p = g.ap_rp[i]; p < g.ap_rp[i + 1]; p++) {
                    const double qj = pw[e * k + g.ap_col[p]];
                    if (qj == 0.0) continue;
                    acc = dadd(acc, dmul(g.ap_x[p], qj));
                }
            }
            sh.X[(size_t)e * S + i] = acc;
        }
        __syncthreads();
        run_sweep(sh, g.fwd, B, S, nenv, n, ctx->status);
        run_sweep(sh, g.bwd, B, S, nenv, n, ctx->status);
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
