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
// with cp.async; before a bundle, the warp acquires the ready flags of the
// other warps' rows it reads.
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

// One triangular sweep. Every warp runs its own bundle stream, copied stage
// by stage into its ring (each lane copies 16 bytes of a stage); all threads
// of the CTA must call it.
__device__ inline void run_sweep(const SolveShared& sh, const Sweep& sw, int B, int S, int n, uint32_t epoch) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int g = lane >> 3, e = lane & 7;
    const uint32_t R = sw.ring_stages, ring_bytes = R * kStageBytes;
    const uint8_t* src = sw.stream + (size_t)sw.warp_off[w] * kStageBytes + 16 * lane;
    const uint32_t nst = sw.warp_stages[w];
    uint8_t* ring = sh.ring + (size_t)w * ring_bytes;
    // lanes of envs beyond the slab's capacity read env 0's field and never
    // store, so they touch no memory outside the field
    const bool owns = e < B;
    double* xe = sh.X + (size_t)(owns ? e : 0) * S;

    uint32_t issued = 0, waited = 0, released = 0, p = 0, ro = 0;
    for (; issued < nst && issued < R; issued++) {
        cp_async16(ring + issued * kStageBytes + 16 * lane, src + (size_t)issued * kStageBytes);
        cp_async_commit();
    }
    bool ok = true;
    // wait until the stream's bytes [0, end) are in the ring
    auto ensure = [&](uint32_t end) {
        if (end > waited * kStageBytes) {
            const uint32_t need = (end + kStageBytes - 1) / kStageBytes;   // stages [0, need)
            if (need > issued) { ok = false; return; }
            cp_async_wait(issued - need);
            __syncwarp();
            waited = need;
        }
    };
    // refill the slots of stages the warp has read completely
    auto release = [&]() {
        const uint32_t upto = min(p / kStageBytes, waited);
        if (released < upto) {
            __syncwarp();   // every lane's reads of those slots are done
            for (; released < upto; released++) {
                const uint32_t k = released + R;
                if (k < nst) {
                    cp_async16(ring + (k % R) * kStageBytes + 16 * lane, src + (size_t)k * kStageBytes);
                    cp_async_commit();
                    issued = k + 1;
                }
            }
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
            p += ring_bytes - ro;
            ro = 0;
            ensure(p);
            release();
            continue;
        }
        const uint32_t row = ((g < 2 ? hv.x : hv.y) >> (16 * (g & 1))) & 0xFFFFu;
        const uint32_t fin = (hv.w >> (8 * g)) & 0xFFu;
        const uint32_t npre = (flags >> 8) & 0xFu;
        const uint32_t bsz = (uint32_t)bundle_bytes((int)npre, (flags & 0xF0u) != 0, (int)nblk);
        const bool bad = row > (uint32_t)n || (fin != kFinNever && fin > nblk) || (flags & 0x3000u) ||
                         npre > (uint32_t)kMaxPreItems || bsz > (uint32_t)kMaxBundleBytes || ro + bsz > ring_bytes;
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
        if (ro == ring_bytes) ro = 0;
        release();
    }
    if (!ok) atomicCAS((int*)sh.abort, 0, kErrRingTimeout);
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
    run_sweep(sh, g.fwd, B, S, n, 1);
    __syncthreads();
    run_sweep(sh, g.bwd, B, S, n, 2);
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
        run_sweep(sh, g.fwd, B, S, n, 3);
        __syncthreads();
        run_sweep(sh, g.bwd, B, S, n, 4);
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
