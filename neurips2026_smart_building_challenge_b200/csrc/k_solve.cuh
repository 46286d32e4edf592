// Fused thermal solve: forcing -> L sweep -> U sweep -> air-side dense system
// -> second L/U sweep -> interior mass + field update, for one slab of envs
// held in shared memory.
//
// Reference: complete_port/csim/sb_fdm.c:142-188 (one env) and sb_lu.c:38-63
// (the factor replay). The reference pushes each column of L/U into the rows
// below/above it; here every row pulls its terms in the same column order, so
// each row receives exactly the same sequence of subtractions and the result
// is bit-identical. The pull schedule is precomputed on the host
// (sweep_sched.cpp): every warp runs its own program, streamed into a per-warp
// shared-memory ring with cp.async; its four lane groups (one lane per env)
// each work through their own rows, and control records acquire the ready
// flags of other warps' rows before rows that read them start.
#pragma once
#include "dev_util.cuh"

namespace sbenv {

struct SlabDesc {
    int group;
    int env0;   // first global env
    int nenv;   // envs in this slab (<= slab_envs)
    int pad;
};

constexpr uint32_t kSpinLimit = 1u << 22;   // polls of one ready flag (at most ~1 s with the sleeps)

struct SolveShared {
    double* X;            // [B][stride]
    uint8_t* ring;        // [kSweepWarps][ring_stages][kStageBytes]
    uint8_t* ready;       // [n + 1] row ready flags (epoch of the sweep that finished the row)
    volatile int* abort;  // first error of this CTA
};

// cp.async: 16 bytes global -> shared per lane; one commit group per stage
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// waits until at most `pending` of this thread's newest groups are in flight
__device__ __forceinline__ void cp_async_wait(uint32_t pending) {
    switch (pending) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
        case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
        case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
        case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
    }
}

// One triangular sweep. Every warp runs its own program, copied stage by
// stage (three records each) into its ring, 16 bytes per lane; all threads of
// the CTA must call it.
__device__ inline void run_sweep(const SolveShared& sh, const Sweep& sw, int B, int S, int n, uint32_t epoch) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int g = lane >> 3, e = lane & 7;
    const uint32_t R = sw.ring_stages;
    const uint32_t nst = sw.warp_stages[w];
    const bool copier = lane < kStageBytes / 16;
    const uint8_t* src = sw.stream + (size_t)sw.warp_off[w] * kStageBytes + 16 * lane;
    uint8_t* ring = sh.ring + (size_t)w * R * kStageBytes;
    // lanes of envs beyond the slab's capacity read env 0's field and never
    // store, so they touch no memory outside the field
    const bool owns = e < B;
    double* xe = sh.X + (size_t)(owns ? e : 0) * S;

    uint32_t issued = 0;
    for (; issued < nst && issued < R; issued++) {
        if (copier) cp_async16(ring + issued * kStageBytes + 16 * lane, src + (size_t)issued * kStageBytes);
        cp_async_commit();
    }
    bool ok = true, end = false, next_ctrl = true;
    uint32_t row = (uint32_t)n;   // this group's row (n: idle)
    double acc = 0.0;
    for (uint32_t s = 0; s < nst && !end; s++) {
        int ab = 0;
        if (lane == 0) ab = *sh.abort;
        ab = __shfl_sync(full, ab, 0);
        if (!__all_sync(full, ok) || ab) break;
        cp_async_wait(issued - 1 - s);
        __syncwarp();
        const uint8_t* stage = ring + (s % R) * kStageBytes;
        for (int q = 0; q < kRecordsPerStage && !end; q++) {
            const uint8_t* rec = stage + q * kRecordBytes;
            if (!next_ctrl) {
                // term record: four terms of this group's row
                const double2 v01 = *reinterpret_cast<const double2*>(rec + 32 * g);
                const double2 v23 = *reinterpret_cast<const double2*>(rec + 32 * g + 16);
                const uint2 cc = *reinterpret_cast<const uint2*>(rec + 128 + 8 * g);
                next_ctrl = (cc.x & kNextIsCtrl) != 0;
                const double x0 = xe[cc.x & kColMask], x1 = xe[cc.x >> 16];
                const double x2 = xe[cc.y & 0xFFFFu], x3 = xe[cc.y >> 16];
                acc = dsub(acc, dmul(v01.x, x0));
                acc = dsub(acc, dmul(v01.y, x1));
                acc = dsub(acc, dmul(v23.x, x2));
                acc = dsub(acc, dmul(v23.y, x3));
                continue;
            }
            // control record: end segments, wait, start rows (warp-uniform
            // control flow; per-group choices are predicates)
            const ControlRecord* c = reinterpret_cast<const ControlRecord*>(rec);
            const uint32_t gf = c->gflags[g];
            const uint32_t nw = c->nwait, newrow = c->row[g];
            const uint32_t cflags = c->flags;
            if (__any_sync(full, newrow > (uint32_t)n || nw > (uint32_t)kCtrlWaits)) {
                atomicCAS((int*)sh.abort, 0, kErrBadBundle);
                ok = false;
                break;
            }
            const bool ending = (gf & kGSwitch) && row < (uint32_t)n;
            if (__any_sync(full, ending && (gf & kGDivide))) {
                const double q = ddiv(acc, c->diag[g]);
                if (ending && (gf & kGDivide)) acc = q;
            }
            if (ending && owns) xe[row] = acc;   // final value, or the partial sum of a paused row
            const bool pub = ending && (gf & kGPublish);
            __syncwarp();
            if (__any_sync(full, pub) && pub && e == 0) {
                __threadfence_block();
                st_release_u8(sh.ready + row, epoch);
            }
            // waits: one row per lane; the warp barrier after them orders every
            // lane's later reads after all the acquires
            for (uint32_t i = lane; i < nw; i += 32) {
                const uint32_t r = c->wait[i];
                if (r > (uint32_t)n) {
                    atomicCAS((int*)sh.abort, 0, kErrBadBundle);
                    ok = false;
                    break;
                }
                // a few quick polls, then sleeps that leave the issue slots to
                // the warps doing work (bounded: kSpinLimit polls in all)
                uint32_t spins = 0, nap = 32;
                while (ld_acquire_u8(sh.ready + r) < epoch) {
                    if (++spins >= kSpinLimit) {
                        atomicCAS((int*)sh.abort, 0, kErrWaitTimeout);
                        ok = false;
                        break;
                    }
                    if ((spins & 255u) == 0 && *sh.abort) { ok = false; break; }
                    if (spins > 4) {
                        __nanosleep(nap);
                        nap = nap < 256 ? 2 * nap : 256;
                    }
                }
                if (!ok) break;
            }
            __syncwarp();
            if (!__all_sync(full, ok)) break;
            // new rows: slot n (idle) reads the zero column
            if (gf & kGSwitch) row = newrow;
            const double a0 = xe[row];
            acc = (gf & kGSwitch) ? a0 : acc;
            next_ctrl = (cflags & kCtrlNext) != 0;
            end = (cflags & kCtrlEnd) != 0;
        }
        if (!__all_sync(full, ok)) break;
        // refill the slot of stage s with stage s + R
        __syncwarp();
        if (!end && s + R < nst) {
            if (copier) cp_async16(ring + (s % R) * kStageBytes + 16 * lane, src + (size_t)(s + R) * kStageBytes);
            cp_async_commit();
            issued = s + R + 1;
        }
    }
    if (!ok || !end) atomicCAS((int*)sh.abort, 0, kErrBadBundle);
    // no copy may land after the sweep: the ring memory is reused
    cp_async_wait(0);
    __syncwarp();
}

// Dense k x k system M q = b of one env, solved by a team of warps with the
// reference's elimination (complete_port/csim/sb_fdm.c:9-38): partial
// pivoting on the first strictly largest |M[r][c]| below the diagonal (the
// diagonal wins ties, a NaN never wins), rows whose multiplier is 0 left
// untouched, a zero pivot column ends the solve with b as eliminated so far,
// then back substitution subtracting the products in ascending column order.
// Every element receives the reference's operations in the reference's order.
//
// Thread p of the team owns matrix row p for the whole solve. Row exchanges
// are virtual: each thread tracks the position its row currently holds in the
// reference's (physically swapped) matrix, so a swap moves no data.
//   M    column-major, k rows: element (r, j) at M[j * k + r]; column k is b
//   red  [2][team warps][2] doubles of scratch for the pivot reduction
//   z    [k] solution by position, then [1] diagonal scratch
__host__ __device__ constexpr size_t dense_env_doubles(int k) { return (size_t)k * (k + 1) + 16 + 2 * (size_t)k; }

__device__ inline void team_sync(int bar, int T) {
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(T) : "memory");
}

__device__ inline void dense_team(double* M, int k, int ttid, int T, int bar) {
    const int lane = ttid & 31, tw = ttid >> 5, W = T >> 5;
    double* red = M + (size_t)k * (k + 1);   // [2][W][2]
    double* z = red + 16;                     // [k]
    double* dg = z + k;                       // [k]: diagonal candidate per step parity slot
    const bool has_row = ttid < k;
    const int p = has_row ? ttid : 0;
    int mypos = ttid;
    bool stopped = false;
    for (int c = 0; c < k; c++) {
        // candidates below the diagonal: larger |value| wins, the lower position on
        // ties (key: position << 8 | row); a NaN never compares greater, so never wins
        double ba = -1.0;
        int key = 0x7FFFFFFF;
        if (has_row && mypos >= c) {
            const double v = M[(size_t)c * k + p];
            if (mypos == c) {
                dg[c & 1] = (double)p;   // the diagonal row: read by everyone after the barrier
            } else if (fabs(v) > -1.0) {
                ba = fabs(v);
                key = (mypos << 8) | p;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const double oa = __shfl_xor_sync(0xffffffffu, ba, o);
            const int ok = __shfl_xor_sync(0xffffffffu, key, o);
            if (oa > ba || (oa == ba && ok < key)) { ba = oa; key = ok; }
        }
        double* rb = red + (size_t)(c & 1) * W * 2;
        if (lane == 0) {
            rb[2 * tw] = ba;
            rb[2 * tw + 1] = int_in_double(key);
        }
        team_sync(bar, T);
        for (int q = 0; q < W; q++) {
            const double oa = rb[2 * q];
            const int ok = int_from_double(rb[2 * q + 1]);
            if (oa > ba || (oa == ba && ok < key)) { ba = oa; key = ok; }
        }
        // the reference: best = |diagonal|, replaced by a later row only if strictly larger
        const int drow = (int)dg[c & 1];
        const double dv = M[(size_t)c * k + drow];
        int piv = c, prow = drow;
        double pbest = fabs(dv);
        if (key != 0x7FFFFFFF && ba > pbest) { piv = key >> 8; prow = key & 0xFF; pbest = ba; }
        if (pbest == 0.0) { stopped = true; break; }
        const double d = M[(size_t)c * k + prow];
        if (mypos == c) mypos = piv;
        else if (mypos == piv) mypos = c;
        // eliminate below the pivot, eight columns at a time (all loads first)
        if (has_row && mypos > c) {
            const double fr = ddiv(M[(size_t)c * k + p], d);
            if (fr != 0.0) {
                int j = c + 1;
                for (; j + 8 <= k + 1; j += 8) {
                    double a[8], q[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        a[u] = M[(size_t)(j + u) * k + p];
                        q[u] = M[(size_t)(j + u) * k + prow];
                    }
#pragma unroll
                    for (int u = 0; u < 8; u++) M[(size_t)(j + u) * k + p] = dsub(a[u], dmul(fr, q[u]));
                }
                for (; j <= k; j++) M[(size_t)j * k + p] = dsub(M[(size_t)j * k + p], dmul(fr, M[(size_t)j * k + prow]));
            }
        }
    }
    // back substitution position by position (columns are not permuted): every
    // pending row forms its product with the newest z in place, the owner of
    // the position subtracts its products in ascending column order
    if (!stopped) {
        for (int pos = k - 1; pos >= 0; pos--) {
            if (has_row && mypos <= pos && pos + 1 < k)
                M[(size_t)(pos + 1) * k + p] = dmul(M[(size_t)(pos + 1) * k + p], z[pos + 1]);
            if (has_row && mypos == pos) {
                double s = M[(size_t)k * k + p];
                int j = pos + 1;
                for (; j + 8 <= k; j += 8) {
                    double q[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) q[u] = M[(size_t)(j + u) * k + p];
#pragma unroll
                    for (int u = 0; u < 8; u++) s = dsub(s, q[u]);
                }
                for (; j < k; j++) s = dsub(s, M[(size_t)j * k + p]);
                z[pos] = ddiv(s, M[(size_t)pos * k + p]);
            }
            team_sync(bar, T);
        }
    } else {
        // the reference leaves b as eliminated so far (in swapped order)
        if (has_row) z[mypos] = M[(size_t)k * k + p];
    }
    team_sync(bar, T);
}

__global__ void __launch_bounds__(kSolveThreads, 1)
k_solve(const StepCtx* __restrict__ ctx, const SlabDesc* __restrict__ slabs) {
    extern __shared__ __align__(128) uint8_t smem[];
    // a programmatic dependent (the random streams) may start once every CTA is resident
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const SlabDesc sd = slabs[blockIdx.x];
    const GroupDev& g = ctx->groups[sd.group];
    const StateLayout& L = ctx->lay;
    const int B = g.slab_envs, S = g.stride, n = g.n, ncv = g.ncv, k = g.k;
    const int nenv = sd.nenv;
    const int tid = threadIdx.x;

    // shared memory: field [B][S] | rings | ready flags | misc (solve_smem_bytes)
    const int R = (int)g.fwd.ring_stages;
    SolveShared sh;
    sh.X = reinterpret_cast<double*>(smem);
    sh.ring = smem + (size_t)B * S * sizeof(double);
    sh.ready = sh.ring + (size_t)kSweepWarps * R * kStageBytes;
    int* misc = reinterpret_cast<int*>(sh.ready + ((n + 1 + 15) & ~15));
    sh.abort = misc;
    double* amb_e = reinterpret_cast<double*>(misc + 4);   // [8]
    int* active = reinterpret_cast<int*>(amb_e + 8);        // [8]
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
    __syncthreads();

    // ---- forcing (sb_fdm.c:146-152), written in row order: one thread per
    // row for all envs of the slab, the row's coefficients loaded once ----
    const int local0 = sd.env0 - g.env0;
    for (int i = tid; i < n; i += blockDim.x) {
        const double cap = g.cap[i], dirx = g.dirx[i], mc = g.mc[i];
        const int z = g.zone_of_row[i];
        double Ti[kGroupLanes], Mi[kGroupLanes], qi[kGroupLanes];
#pragma unroll
        for (int e = 0; e < kGroupLanes; e++) {
            if (e >= nenv) break;
            Ti[e] = g.T[(size_t)(local0 + e) * ncv + i];
            Mi[e] = g.M[(size_t)(local0 + e) * n + i];
            qi[e] = z >= 0 ? ctx->Dst[(size_t)(sd.env0 + e) * L.nd + L.qdiv + z] : 0.0;
        }
#pragma unroll
        for (int e = 0; e < kGroupLanes; e++) {
            if (e >= nenv) break;
            double b = dadd(dmul(cap, Ti[e]), qi[e]);
            b = dadd(b, dmul(amb_e[e], dirx));
            b = dadd(b, dmul(mc, Mi[e]));
            sh.X[(size_t)e * S + i] = b;
        }
    }
    __syncthreads();

    // ---- first solve ----
    if (tid < kSweepWarps * 32) run_sweep(sh, g.fwd, B, S, n, 1);
    __syncthreads();
    if (tid < kSweepWarps * 32) run_sweep(sh, g.bwd, B, S, n, 2);
    __syncthreads();
    if (*sh.abort) {   // uniform: read after the barrier
        if (tid == 0) set_error(ctx->status, *sh.abort);
        return;
    }

    // ---- air side (sb_fdm.c:155-181) ----
    // between the sweeps the fields and the rings are free: the dense
    // workspace starts at the fields, the air-side vector pw sits at the end
    // of the rings (dense_workspace_doubles() is checked on the host)
    const size_t free_doubles = ((size_t)B * S * 8 + (size_t)kSweepWarps * R * kStageBytes) / 8;
    double* pw = sh.X + free_doubles - (size_t)B * k;   // [B][k]
    int any_active = 0;
    for (int e = 0; e < nenv; e++) any_active |= active[e];
    if (k > 0 && any_active) {
        // sensed temperature of each coupled VAV: one thread per VAV for all
        // envs, its terms fetched eight at a time, summed in order per env
        for (int i = tid; i < k; i += blockDim.x) {
            double acc[kGroupLanes];
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++) acc[e] = 0.0;
            const int p0 = g.sn_p[i], p1 = g.sn_p[i + 1];
            for (int p = p0; p < p1; p += 8) {
                double xv[8];
                int pos[8];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    xv[u] = p + u < p1 ? g.sn_x[p + u] : 0.0;
                    pos[u] = p + u < p1 ? g.sn_pos[p + u] : 0;
                }
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    if (p + u >= p1) break;
#pragma unroll
                    for (int e = 0; e < kGroupLanes; e++)
                        if (e < nenv) acc[e] = dadd(acc[e], dmul(xv[u], sh.X[(size_t)e * S + pos[u]]));
                }
            }
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++) {
                if (e >= nenv) break;
                if (!active[e]) continue;
                const double* D = ctx->Dst + (size_t)(sd.env0 + e) * L.nd;
                pw[e * k + i] = dmul(D[L.ag + i], dsub(D[L.aT + i], acc[e]));
            }
        }
    }
    // y -> the field array (row positions); the second solve adds to it
    for (int i = tid; i < n; i += blockDim.x) {
#pragma unroll
        for (int e = 0; e < kGroupLanes; e++)
            if (e < nenv) g.T[(size_t)(local0 + e) * ncv + i] = sh.X[(size_t)e * S + i];
    }
    __syncthreads();
    if (k > 0 && any_active) {
        // one team of warps per env (thread p owns row p), as many envs at once
        // as the free memory holds (at most 15: named barriers 1..15)
        const size_t per_env = dense_env_doubles(k);
        const int wpt = (k + 31) >> 5;                 // warps per team
        const int cap = dense_teams(n, k, B, R);       // >= 1 (host check)
        for (int e0 = 0; e0 < nenv; e0 += cap) {
            const int ce = (nenv - e0) < cap ? (nenv - e0) : cap;
            const int per = k * (k + 1);
            for (int idx = tid; idx < ce * per; idx += blockDim.x) {
                const int e = idx / per, rem = idx % per, j = rem / k, i = rem % k;   // column-major
                if (!active[e0 + e]) continue;
                const double* D = ctx->Dst + (size_t)(sd.env0 + e0 + e) * L.nd;
                sh.X[e * per_env + (size_t)j * k + i] =
                    j < k ? dadd(i == j ? 1.0 : 0.0, dmul(D[L.ag + i], g.S[(size_t)i * k + j])) : pw[(e0 + e) * k + i];
            }
            __syncthreads();
            const int team = (tid >> 5) / wpt;
            if (team < ce && active[e0 + team])
                dense_team(sh.X + team * per_env, k, tid - team * wpt * 32, wpt * 32, 1 + team);
            __syncthreads();
            for (int idx = tid; idx < ce * k; idx += blockDim.x) {
                const int e = idx / k, i = idx % k;
                if (active[e0 + e]) pw[(e0 + e) * k + i] = sh.X[e * per_env + (size_t)k * (k + 1) + 16 + i];
            }
            __syncthreads();
        }
        // r = applied q, pulled per row in ascending column order; zero q
        // skipped; one thread per row for all envs. The dense workspace
        // overlapped the field: padding slots and unused envs are zeroed again
        // (padded sweep terms read the zero slot).
        for (int i = tid; i < n; i += blockDim.x) {
            double acc[kGroupLanes];
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++) acc[e] = 0.0;
            const int p0 = g.ap_rp[i], p1 = g.ap_rp[i + 1];
            for (int p = p0; p < p1; p++) {
                const int col = g.ap_col[p];
                const double xv = g.ap_x[p];
#pragma unroll
                for (int e = 0; e < kGroupLanes; e++) {
                    if (e >= nenv) break;
                    const double qj = pw[e * k + col];
                    if (active[e] && qj != 0.0) acc[e] = dadd(acc[e], dmul(xv, qj));
                }
            }
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++)
                if (e < B) sh.X[(size_t)e * S + i] = e < nenv && active[e] ? acc[e] : 0.0;
        }
        for (int idx = tid; idx < B * (S - n); idx += blockDim.x)
            sh.X[(size_t)(idx / (S - n)) * S + n + idx % (S - n)] = 0.0;
        __syncthreads();
        if (tid < kSweepWarps * 32) run_sweep(sh, g.fwd, B, S, n, 3);
        __syncthreads();
        if (tid < kSweepWarps * 32) run_sweep(sh, g.bwd, B, S, n, 4);
        __syncthreads();
        if (*sh.abort) {
            if (tid == 0) set_error(ctx->status, *sh.abort);
            return;
        }
    }

    // ---- interior mass + field (sb_fdm.c:183-187): one thread per row ----
    for (int i = tid; i < n; i += blockDim.x) {
        const double ret = g.ret[i], gain = g.gain[i];
        double y[kGroupLanes], m[kGroupLanes];
#pragma unroll
        for (int e = 0; e < kGroupLanes; e++) {
            if (e >= nenv) break;
            y[e] = g.T[(size_t)(local0 + e) * ncv + i];
            m[e] = g.M[(size_t)(local0 + e) * n + i];
        }
#pragma unroll
        for (int e = 0; e < kGroupLanes; e++) {
            if (e >= nenv) break;
            double ye = y[e];
            if (k > 0 && active[e]) ye = dadd(ye, sh.X[(size_t)e * S + i]);
            g.M[(size_t)(local0 + e) * n + i] = dadd(dmul(m[e], ret), dmul(gain, ye));
            g.T[(size_t)(local0 + e) * ncv + i] = ye;
        }
    }
    for (int idx = tid; idx < nenv * (ncv - n); idx += blockDim.x) {
        const int e = idx / (ncv - n), i = n + idx % (ncv - n);
        const int local = sd.env0 + e - g.env0;
        g.T[(size_t)local * ncv + i] = amb_e[e];
    }
}

}  // namespace sbenv
