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
// shared-memory ring by bulk copies; its four lane groups (one lane per env)
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

constexpr uint32_t kSpinLimit = 1u << 22;   // polls of one ready flag before the wait gives up (about a second)

struct SolveShared {
    double* X;            // [B][stride]
    uint8_t* ring;        // [kSweepWarps][ring_stages][kStageBytes]
    uint8_t* ready;       // [n + 1] row ready flags: 2 epoch final, 2 epoch - 1 outside terms applied
    uint64_t* bars;       // [kSweepWarps][kStagesMax] completion barriers of the ring stages
    volatile int* abort;  // first error of this CTA
    uint32_t spin_limit;  // polls of one ready flag (kSpinLimit unless a failure test lowers it)
};

// Waits (acquire) until every listed row's ready flag reaches its target:
// `fin` for a final row, fin - 1 for an entry with kWaitPartial. One row per
// lane; bounded, and left early once another warp has reported an error.
// Warp-uniform result: false if some lane gave up.
__device__ inline bool wait_rows(const SolveShared& sh, const uint16_t* list, uint32_t nw, uint32_t n, uint32_t fin) {
    const int lane = threadIdx.x & 31;
    bool ok = true;
    for (uint32_t i = lane; i < nw && ok; i += 32) {
        const uint32_t w = list[i];
        const uint32_t r = min(w & (uint32_t)kColMask, n);   // slot n is always ready
        const uint32_t need = (w & kWaitPartial) ? fin - 1 : fin;
        uint32_t spins = 0;
        while (ld_acquire_u8(sh.ready + r) < need) {
            if (++spins >= sh.spin_limit) {
                atomicCAS((int*)sh.abort, 0, kErrWaitTimeout);
                ok = false;
                break;
            }
            if ((spins & 1023u) == 0 && *sh.abort) { ok = false; break; }
            if (spins > 16) __nanosleep(32);
        }
    }
    return __all_sync(0xffffffffu, ok);
}

// The stage ring of one warp: its program is copied stage by stage (three
// records) into ring_stages slots by bulk copies that lane 0 issues, each
// completing on its slot's mbarrier. Stages are consumed in order; a slot is
// refilled with the stage ring_stages further on once its stage is consumed.
struct StageRing {
    uint8_t* ring;
    uint64_t* bar;
    const uint8_t* src;
    uint32_t R, nst;
    uint32_t head = 0, hslot = 0;               // first stage not consumed, its slot
    uint32_t landed = 0, lslot = 0, lpar = 0;   // stages < landed have arrived; slot and phase of `landed`

    __device__ void issue(uint32_t st, uint32_t slot) const {   // lane 0; the slot's earlier reads are complete
        mbar_expect_tx(bar + slot, kStageBytes);
        bulk_g2s(ring + (size_t)slot * kStageBytes, src + (size_t)st * kStageBytes, kStageBytes, bar + slot);
    }
    __device__ void start(int lane) {
        if (lane == 0) {
            for (uint32_t s = 0; s < R; s++) mbar_init(bar + s, 1);
            mbar_fence_init();
            for (uint32_t s = 0; s < R && s < nst; s++) issue(s, s);
        }
        __syncwarp();
    }
    // stage t has arrived (t < head + R); warp-uniform, false on timeout
    __device__ bool land(uint32_t t) {
        if (landed > t) return true;
        bool ok = true;
        while (landed <= t && ok) {
            ok = mbar_wait_bounded(bar + lslot, lpar);
            landed++;
            if (++lslot == R) { lslot = 0; lpar ^= 1u; }
        }
        return __all_sync(0xffffffffu, ok);
    }
    // stages < t (t <= head + R) are consumed: their slots are refilled. A
    // slot is refilled only after its copy has arrived, also for stages that
    // were skipped unread. Warp-uniform, false on timeout.
    __device__ bool consume(uint32_t t, int lane) {
        if (head >= t) return true;
        if (!land(t - 1)) return false;
        __syncwarp();   // every lane is done reading the slots
        for (; head < t; head++) {
            if (lane == 0 && head + R < nst) issue(head + R, hslot);
            if (++hslot == R) hslot = 0;
        }
        return true;
    }
    // no copy may land after the sweep (the ring memory is reused): wait for
    // the stages in flight, then retire the barriers
    __device__ bool finish(int lane) {
        const uint32_t end = min(head + R, nst);
        const bool ok = end == 0 || land(end - 1);
        __syncwarp();
        if (lane == 0)
            for (uint32_t s = 0; s < R; s++) mbar_inval(bar + s);
        __syncwarp();
        return ok;
    }
};

// L2 prefetch of [p, p + bytes) in 4 KB bulk requests spread over `workers`
// threads (the tail below a 16-byte multiple is left out).
__device__ __forceinline__ void prefetch_l2(const uint8_t* p, uint32_t bytes, uint32_t worker, uint32_t workers) {
    constexpr uint32_t kChunk = 4096;
    bytes &= ~15u;
    for (uint32_t off = worker * kChunk; off < bytes; off += workers * kChunk) {
        const uint32_t len = min(kChunk, bytes - off);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(len) : "memory");
    }
}

// L1 prefetch of the 128-byte lines of [p, p + bytes): one line per lane.
__device__ __forceinline__ void prefetch_lines(const uint8_t* p, uint32_t bytes, int lane) {
    const uintptr_t l0 = reinterpret_cast<uintptr_t>(p) >> 7;
    const uintptr_t l1 = (reinterpret_cast<uintptr_t>(p) + bytes - 1) >> 7;
    for (uintptr_t l = l0 + (uintptr_t)lane; l <= l1; l += 32) asm volatile("prefetch.global.L1 [%0];" ::"l"(l << 7));
}

// The rounds of one block (BW: the U sweep, rows descending, each finished
// by a division -- Recip: a multiplication by the stored reciprocal of the
// diagonal, the corrected and folded builds), after its header has been
// checked and its waits acquired.
template <bool BW, bool Recip>
__device__ __forceinline__ double block_finish(double a, double dg) {
    return BW ? (Recip ? dmul(a, dg) : ddiv(a, dg)) : a;
}
template <bool BW, bool Recip>
__device__ inline void block_rounds(const SolveShared& sh, const uint8_t* __restrict__ vals, uint32_t first,
                                    uint32_t size, uint64_t pubm, double* __restrict__ xe, bool owns, uint32_t fin) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31, e = lane & 7;
    const uint32_t g = (uint32_t)lane >> 3;
    constexpr int dir = BW ? -1 : 1;
    const double* __restrict__ xb = xe + (int)first;   // block row j at xb[dir * j]
    // this group's in-round terms (k < g at triangle index g(g-1)/2 + k)
    const uint32_t tri0 = g * (g - 1) / 2;
    const uint32_t o0 = 32 + 8 * min(tri0 + 0, 5u), o1 = 32 + 8 * min(tri0 + 1, 5u), o2 = 32 + 8 * min(tri0 + 2, 5u);
    const uint8_t* __restrict__ rp = vals;
    for (uint32_t c0 = 0; c0 < size; c0 += 4) {
        const uint32_t rbytes = (kRoundHead + 4 * c0) * 8;
        if (c0 + 4 < size) prefetch_lines(rp + rbytes, rbytes + 128, lane);   // the next round
        const bool mine = c0 + g < size;
        const int row = (int)first + dir * (int)(c0 + g);
        const double t0 = __ldg(reinterpret_cast<const double*>(rp + o0));
        const double t1 = __ldg(reinterpret_cast<const double*>(rp + o1));
        const double t2 = __ldg(reinterpret_cast<const double*>(rp + o2));
        const double dg = BW ? __ldg(reinterpret_cast<const double*>(rp + 8 * g)) : 1.0;
        // the row's partial sum, then its terms from the earlier rounds in order
        double a = xe[mine ? row : (int)first];
        const uint8_t* __restrict__ tv = rp + kRoundHead * 8 + 8 * c0 * g;
        for (uint32_t j = 0; j < c0; j += 4) {
            const double2 v01 = __ldg(reinterpret_cast<const double2*>(tv + 8 * j));
            const double2 v23 = __ldg(reinterpret_cast<const double2*>(tv + 8 * j + 16));
            const double x0 = xb[dir * (int)j], x1 = xb[dir * (int)(j + 1)];
            const double x2 = xb[dir * (int)(j + 2)], x3 = xb[dir * (int)(j + 3)];
            a = dsub(a, dmul(v01.x, x0));
            a = dsub(a, dmul(v01.y, x1));
            a = dsub(a, dmul(v23.x, x2));
            a = dsub(a, dmul(v23.y, x3));
        }
        // the four rows in turn: group k's row is final at stage k
        double xm;
        const double f0 = block_finish<BW, Recip>(a, dg);
        xm = f0;
        const double x0 = __shfl_sync(full, f0, e);
        if (g > 0) a = dsub(a, dmul(t0, x0));
        const double f1 = block_finish<BW, Recip>(a, dg);
        if (g == 1) xm = f1;
        const double x1 = __shfl_sync(full, f1, 8 | e);
        if (g > 1) a = dsub(a, dmul(t1, x1));
        const double f2 = block_finish<BW, Recip>(a, dg);
        if (g == 2) xm = f2;
        const double x2 = __shfl_sync(full, f2, 16 | e);
        if (g > 2) a = dsub(a, dmul(t2, x2));
        if (g == 3) xm = block_finish<BW, Recip>(a, dg);
        // the round's rows are final: store (later rounds read them), publish
        // those other warps read
        if (mine && owns) xe[row] = xm;
        __syncwarp();
        const uint32_t pb = (uint32_t)(pubm >> c0) & 0xFu;
        if (pb && mine && e == 0 && ((pb >> g) & 1u)) {
            __threadfence_block();
            st_release_u8(sh.ready + row, fin);
        }
        rp += rbytes;
    }
}

// One dense block record (format in sbenv_dev.h), the cursor at its header
// (stage rg.head, record hq); its values are read from global memory (the
// sweep's value region, sw_base + values) through L1, the next round's lines
// prefetched while the current one runs. Lane group g holds the block's rows
// i = g mod 4, one lane per env. Round c0: group g's row c0 + g loads its
// partial sum, pulls its terms from rows 0..c0-1 (final values in shared
// memory), then the round's four rows finish in turn, x_k from group k to all
// lanes by a shuffle (group 3's value is only stored). Returns false on an
// error (reported in sh.abort).
__device__ inline bool run_block(const SolveShared& sh, const StageRing& rg, uint32_t hq, const uint8_t* sw_base,
                                 uint32_t sw_bytes, double* __restrict__ xe, bool owns, uint32_t n, uint32_t fin,
                                 bool recip) {
    const int lane = threadIdx.x & 31;
    const BlockRecord* b = reinterpret_cast<const BlockRecord*>(rg.ring + (size_t)rg.hslot * kStageBytes + hq * kRecordBytes);
    const uint32_t first = b->first, size = b->size, bw = b->backward, nw = b->nwait, voff = b->values;
    const uint64_t pubm = b->publish;
    const uint32_t lastrow = bw ? first - (size - 1) : first + (size - 1);
    const uint32_t vbytes = (uint32_t)block_values((int)size) * 8u;
    if (size == 0 || size > (uint32_t)kMaxBlockRows || bw > 1 || first >= n || lastrow >= n || (voff & 15u) ||
        voff > sw_bytes || vbytes > sw_bytes - voff) {
        atomicCAS((int*)sh.abort, 0, kErrBadBundle);
        return false;
    }
    const uint8_t* __restrict__ vals = sw_base + voff;
    prefetch_lines(vals, min(vbytes, 2048u), lane);
    if (nw && !wait_rows(sh, b->wait, min(nw, (uint32_t)kCtrlWaits), n, fin)) return false;
    if (bw && recip) block_rounds<true, true>(sh, vals, first, size, pubm, xe, owns, fin);
    else if (bw) block_rounds<true, false>(sh, vals, first, size, pubm, xe, owns, fin);
    else block_rounds<false, false>(sh, vals, first, size, pubm, xe, owns, fin);
    return true;
}

// One triangular sweep. Every warp runs its own program from its stage ring;
// all threads of the CTA must call it. Term records: four terms per lane
// group. Control records: finish ending rows (divide, store, publish), wait
// for other warps' rows, load the new rows. Block records: run_block.
// Every branch on a record's contents is warp-uniform (record-level flags),
// so the warp never needs a vote on the hot path.
// stall_row >= 0 (failure test only): warp 0 first waits for that row, which
// no warp publishes, so the bounded wait runs out and the sweep aborts.
__device__ inline void run_sweep(const SolveShared& sh, const Sweep& sw, int B, int S, int n, uint32_t epoch,
                                 int stall_row = -1) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int g = lane >> 3, e = lane & 7;
    const uint32_t fin = 2 * epoch, un = (uint32_t)n;
    StageRing rg;
    rg.R = sw.ring_stages;
    rg.nst = sw.warp_stages[w];
    rg.src = sw.stream + (size_t)sw.warp_off[w] * kStageBytes;
    rg.ring = sh.ring + (size_t)w * rg.R * kStageBytes;
    rg.bar = sh.bars + (size_t)w * kStagesMax;
    // lanes of envs beyond the slab's capacity read env 0's field and never
    // store, so they touch no memory outside the field
    const bool owns = e < B;
    double* xe = sh.X + (size_t)(owns ? e : 0) * S;

    rg.start(lane);
    int err = rg.nst == 0 ? kErrBadBundle : (rg.land(0) ? kErrNone : kErrRingTimeout);
    if (stall_row >= 0 && w == 0 && err == kErrNone) {
        const uint16_t wr = (uint16_t)stall_row;
        if (!wait_rows(sh, &wr, 1, un, fin)) err = kErrWaitTimeout;
    }
    const uint8_t* rp = rg.ring;
    uint32_t q = 0;
    bool ctrl = true;
    uint32_t row = un;   // this group's row (n: idle, reads the zero slot)
    double acc = 0.0;
    while (err == kErrNone) {
        if (!ctrl) {
            // term record: four terms of this group's row
            const double2 v01 = *reinterpret_cast<const double2*>(rp + 32 * g);
            const double2 v23 = *reinterpret_cast<const double2*>(rp + 32 * g + 16);
            const uint2 cc = *reinterpret_cast<const uint2*>(rp + 128 + 8 * g);
            ctrl = (cc.x & kNextIsCtrl) != 0;
            const double x0 = xe[cc.x & kColMask], x1 = xe[cc.x >> 16];
            const double x2 = xe[cc.y & 0xFFFFu], x3 = xe[cc.y >> 16];
            acc = dsub(acc, dmul(v01.x, x0));
            acc = dsub(acc, dmul(v01.y, x1));
            acc = dsub(acc, dmul(v23.x, x2));
            acc = dsub(acc, dmul(v23.y, x3));
        } else {
            const ControlRecord* c = reinterpret_cast<const ControlRecord*>(rp);
            const uint32_t cf = c->flags;
            if (cf & kCtrlBlock) {
                if (!run_block(sh, rg, q, sw.stream, sw.total_bytes, xe, owns, un, fin, sw.recip != 0)) {
                    err = kErrBadBundle;
                    break;
                }
                ctrl = true;   // a block is followed by a control or block record
            } else {
                const uint32_t gf = c->gflags[g];
                const uint32_t newrow = min((uint32_t)c->row[g], un);
                const uint32_t nw = c->nwait;
                const bool ending = (gf & kGSwitch) && row < un;
                if (cf & kCtrlDivide) {
                    // the diagonal, or its reciprocal (corrected and folded builds)
                    const double dq = sw.recip ? dmul(acc, c->diag[g]) : ddiv(acc, c->diag[g]);
                    if (gf & kGDivide) acc = dq;
                }
                if (ending && owns) xe[row] = acc;   // final value, partial sum, or paused row
                if (cf & kCtrlPublish) {
                    __syncwarp();
                    if (ending && e == 0 && (gf & (kGPublish | kGPartial))) {
                        __threadfence_block();
                        st_release_u8(sh.ready + row, (gf & kGPublish) ? fin : fin - 1);
                    }
                }
                if (nw && !wait_rows(sh, c->wait, min(nw, (uint32_t)kCtrlWaits), un, fin)) { err = kErrWaitTimeout; break; }
                __syncwarp();   // stores of every group before any group's new loads
                if (gf & kGSwitch) {
                    row = newrow;
                    acc = xe[row];
                }
                if (cf & kCtrlEnd) break;
                ctrl = (cf & kCtrlNext) != 0;
            }
        }
        // next record
        if (++q == kRecordsPerStage) {
            if (!rg.consume(rg.head + 1, lane)) { err = kErrRingTimeout; break; }
            if (rg.head >= rg.nst) { err = kErrBadBundle; break; }
            if (!rg.land(rg.head)) { err = kErrRingTimeout; break; }
            q = 0;
            rp = rg.ring + (size_t)rg.hslot * kStageBytes;
        } else {
            rp += kRecordBytes;
        }
    }
    if (err != kErrNone) atomicCAS((int*)sh.abort, 0, err);
    if (!rg.finish(lane)) atomicCAS((int*)sh.abort, 0, kErrRingTimeout);
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
//
// One team barrier per column step c. Before it, every row publishes its
// column-c value: the diagonal row its value, each warp its best candidate
// below the diagonal, found by three warp reductions over the 64-bit pattern
// of |value| (monotonic for non-negative doubles; a NaN is no candidate) and
// the key position << 8 | row (lower position wins ties); then each row
// finishes the previous step's update of columns c + 1 .. k while the other
// warps reduce. After it, every thread picks the pivot from the published
// entries with no further dependent loads, forms its multiplier and updates
// column c + 1 first, which is the next step's candidate.
//   M    column-major, k rows: element (r, j) at M[j * k + r]; column k is b
//   red  [2 step parities][16] doubles: diagonal value and row, then per warp
//        {|value| pattern, key, value}
//   z    [k] solution by position
constexpr int kDenseRed = 32;
__host__ __device__ constexpr size_t dense_env_doubles(int k) { return (size_t)k * (k + 1) + kDenseRed + (size_t)k; }
__host__ __device__ constexpr size_t dense_smem_doubles(int k) { return dense_env_doubles(k); }
// Above kDenseHelperK rows every row owner has a helper thread (the second half
// of the team) that takes half of the row's deferred column updates.
constexpr int kDenseHelperK = 48;
__host__ __device__ constexpr int dense_threads(int k) {
    return (k > kDenseHelperK ? 64 : 32) * ((k + 31) / 32);
}

__device__ inline void team_sync(int bar, int T) {
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(T) : "memory");
}

// M[j][p] -= f * M[j][pr] for columns j0 .. j1 (eight at a time, loads first);
// Fused: one fused multiply-add per element (the corrected and folded builds)
// instead of the reference's multiply then subtract
template <bool Fused>
__device__ __forceinline__ double dense_axpy(double a, double f, double q) {
    return Fused ? __fma_rn(-f, q, a) : dsub(a, dmul(f, q));
}
template <bool Fused>
__device__ __forceinline__ void dense_update(double* M, int k, int p, int pr, double f, int j0, int j1) {
    int j = j0;
    for (; j + 8 <= j1 + 1; j += 8) {
        double a[8], q[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            a[u] = M[(size_t)(j + u) * k + p];
            q[u] = M[(size_t)(j + u) * k + pr];
        }
#pragma unroll
        for (int u = 0; u < 8; u++) M[(size_t)(j + u) * k + p] = dense_axpy<Fused>(a[u], f, q[u]);
    }
    for (; j <= j1; j++) M[(size_t)j * k + p] = dense_axpy<Fused>(M[(size_t)j * k + p], f, M[(size_t)j * k + pr]);
}

// Tolerant: the corrected and folded builds (1e-9 contract) -- fused
// multiply-add updates and the column-oriented back substitution; otherwise
// the reference's operations in the reference's order.
template <bool Tolerant>
__device__ inline void dense_team(double* M, int k, int ttid, int T, int bar) {
    const unsigned full = 0xffffffffu;
    const int Tr = 32 * ((k + 31) / 32);   // row owners; threads Tr .. T-1 (if any) are their helpers
    const bool helped = T > Tr, helper = ttid >= Tr;
    const int rid = helper ? ttid - Tr : ttid;
    const int lane = rid & 31, tw = rid >> 5, W = Tr >> 5;
    double* red = M + (size_t)k * (k + 1);
    double* z = red + kDenseRed;
    const bool has_row = rid < k;
    const int p = has_row ? rid : 0;
    int mypos = rid;
    bool stopped = false;
    double cv = has_row && !helper ? M[p] : 0.0;   // the owner's value of its row in the current column
    double fr = 0.0;                    // the previous step's multiplier (0: nothing pending)
    int prow = 0;                       // the previous step's pivot row
    for (int c = 0; c < k; c++) {
        double* sl = red + (c & 1) * 16;
        if (!helper) {   // publish: the diagonal, and the warp's best candidate below it
        const double av = fabs(cv);
        const uint64_t pat = (has_row && mypos > c && av == av) ? (uint64_t)__double_as_longlong(av) + 1ull : 0ull;
        if (has_row && mypos == c) {
            sl[0] = cv;
            sl[1] = (double)p;
        }
        const unsigned hi = (unsigned)(pat >> 32);
        const unsigned mhi = __reduce_max_sync(full, hi);
        const unsigned mlo = __reduce_max_sync(full, hi == mhi ? (unsigned)pat : 0u);
        const bool top = pat != 0ull && hi == mhi && (unsigned)pat == mlo;
        const unsigned key = top ? ((unsigned)mypos << 8) | (unsigned)p : 0xFFFFFFFFu;
        const unsigned mkey = __reduce_min_sync(full, key);
        if (lane == 0) {
            sl[2 + 3 * tw] = __longlong_as_double((long long)(((uint64_t)mhi << 32) | mlo));
            sl[3 + 3 * tw] = (double)mkey;
        }
        if (top && key == mkey) sl[4 + 3 * tw] = cv;
        }
        // the rest of the previous step's update (columns c + 1 .. k), split
        // between the owner and its helper when there is one
        if (fr != 0.0) {
            const int mid = helped ? c + 1 + (k - c) / 2 : k + 1;
            if (!helper) dense_update<Tolerant>(M, k, p, prow, fr, c + 1, mid - 1);
            else dense_update<Tolerant>(M, k, p, prow, fr, mid, k);
        }
        team_sync(bar, T);
        // the pivot: the best candidate if strictly larger than the diagonal
        const double dv = sl[0];
        const int drow = (int)sl[1];
        uint64_t bp = 0ull;
        unsigned bk = 0xFFFFFFFFu;
        double bv = 0.0;
        for (int q = 0; q < W; q++) {
            const uint64_t qp = (uint64_t)__double_as_longlong(sl[2 + 3 * q]);
            const unsigned qk = (unsigned)sl[3 + 3 * q];
            const double qv = sl[4 + 3 * q];
            if (qp > bp || (qp == bp && qk < bk)) { bp = qp; bk = qk; bv = qv; }
        }
        int piv = c, pr = drow;
        double d = dv;
        if (bp != 0ull && fabs(bv) > fabs(dv)) { piv = (int)(bk >> 8); pr = (int)(bk & 0xFFu); d = bv; }
        if (fabs(d) == 0.0) { stopped = true; break; }
        if (mypos == c) mypos = piv;
        else if (mypos == piv) mypos = c;
        // this step's multiplier; column c + 1 now (the next candidate), the rest later
        fr = 0.0;
        if (helper) {   // the same multiplier from the same value (written before this step's barrier)
            if (has_row && mypos > c) {
                const double f = ddiv(M[(size_t)c * k + p], d);
                if (f != 0.0) {
                    fr = f;
                    prow = pr;
                }
            }
        } else if (has_row && mypos > c) {
            const double f = ddiv(cv, d);
            double* mc = M + (size_t)(c + 1) * k;
            if (f != 0.0) {
                fr = f;
                prow = pr;
                cv = dense_axpy<Tolerant>(mc[p], f, mc[pr]);
                mc[p] = cv;
            } else {
                cv = mc[p];
            }
        }
    }
    // back substitution position by position (columns are not permuted)
    if (!stopped && Tolerant) {
        // the corrected and folded builds (1e-9 contract): column-oriented --
        // every pending row subtracts its product with the newest z from its
        // running sum at once, so the sums are formed in descending column
        // order (the reference's ascending order only changes the rounding)
        // and each position costs one division and one barrier
        double s = !helper && has_row ? M[(size_t)k * k + p] : 0.0;
        for (int pos = k - 1; pos >= 0; pos--) {
            if (!helper && has_row && mypos == pos) z[pos] = ddiv(s, M[(size_t)pos * k + p]);
            team_sync(bar, T);
            if (!helper && has_row && mypos < pos) s = dsub(s, dmul(M[(size_t)pos * k + p], z[pos]));
        }
    } else if (!stopped) {
        // every pending row forms its product with the newest z in place, the
        // owner of the position subtracts its products in ascending column order
        for (int pos = k - 1; pos >= 0; pos--) {
            if (!helper && has_row && mypos <= pos && pos + 1 < k)
                M[(size_t)(pos + 1) * k + p] = dmul(M[(size_t)(pos + 1) * k + p], z[pos + 1]);
            if (!helper && has_row && mypos == pos) {
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
        if (!helper && has_row) z[mypos] = M[(size_t)k * k + p];
    }
    team_sync(bar, T);
}

// Air-side dense solve of every env, one CTA per env (heaviest groups first):
// M = I + diag(g) S (sb_fdm.c:160-170) in shared memory, column-major with
// the right side ctx->airq as column k, solved by dense_team; the solution
// replaces the right side in ctx->airq. Envs whose VAV gains are all zero
// (or whose building couples no VAV) have no air side and return at once.
// One launch per class of equal k (heaviest class first), each sized for its k;
// the classes after the first are programmatic dependents of the one before,
// so they share the SMs, and each CTA waits for the previous class to complete
// before it exits: the last class completes after all of them.
__device__ inline void dense_env(const StepCtx* __restrict__ ctx, int env) {
    extern __shared__ __align__(16) double dsm[];
    const ScnDev& sc = ctx->scns[ctx->envs[env].scn];
    const GroupDev& g = ctx->groups[sc.group];
    const StateLayout& L = ctx->lay;
    const int k = g.k, tid = threadIdx.x;
    if (k == 0) return;
    const double* D = ctx->Dst + (size_t)env * L.nd;
    int any = 0;
    for (int i = tid; i < k; i += blockDim.x) any |= D[L.ag + i] != 0.0;
    if (!__syncthreads_or(any)) return;
    double* q = ctx->airq + (size_t)env * ctx->k_max;
    const int per = k * (k + 1);
    for (int idx = tid; idx < per; idx += blockDim.x) {
        const int j = idx / k, i = idx % k;
        dsm[idx] = j < k ? dadd(i == j ? 1.0 : 0.0, dmul(D[L.ag + i], g.St[idx])) : q[i];
    }
    __syncthreads();
    const int T = dense_threads(k);
    if (tid < T) {
        if (g.corr || g.fold) dense_team<true>(dsm, k, tid, T, 1);
        else dense_team<false>(dsm, k, tid, T, 1);
    }
    __syncthreads();
    for (int i = tid; i < k; i += blockDim.x) q[i] = dsm[per + kDenseRed + i];
}

__global__ void __launch_bounds__(2 * kMaxK) k_dense(const StepCtx* __restrict__ ctx, int first) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    dense_env(ctx, ctx->dense_order[first + blockIdx.x]);
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Test entry of the dense solver: n systems of size k, Mt [n][k][k] the
// matrices transposed (column-major), b [n][k]; the solutions to out [n][k].
// One CTA per system, dense_threads(k) threads, the path of k_dense (tolerant:
// the corrected and folded builds' solver).
__global__ void __launch_bounds__(2 * kMaxK) k_dense_check(int k, const double* __restrict__ Mt,
                                                       const double* __restrict__ b, double* __restrict__ out,
                                                       int tolerant) {
    extern __shared__ __align__(16) double dsm[];
    const size_t sys = blockIdx.x;
    const double* A = Mt + sys * k * k;
    const int T = dense_threads(k), tid = threadIdx.x;
    const int per = k * (k + 1);
    for (int idx = tid; idx < per; idx += blockDim.x) dsm[idx] = idx < k * k ? A[idx] : b[sys * k + idx - k * k];
    __syncthreads();
    if (tid < T) {
        if (tolerant) dense_team<true>(dsm, k, tid, T, 1);
        else dense_team<false>(dsm, k, tid, T, 1);
    }
    __syncthreads();
    for (int i = tid; i < k; i += blockDim.x) out[sys * k + i] = dsm[per + kDenseRed + i];
}

// Phase 0: forcing, first L/U solve, sensed air-side right side (to
// ctx->airq), y to the field. Phase 1 (after k_dense): applied heat of the
// dense solution, second L/U solve, interior mass and field.
template <int Phase>
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
    // the group's first slab pulls its sweep programs into L2 ahead of every
    // slab's ring copies (the programs are shared by all slabs of the group)
    if (sd.env0 == g.env0) {
        prefetch_l2(g.fwd.stream, g.fwd.total_bytes, tid, blockDim.x);
        prefetch_l2(g.bwd.stream, g.bwd.total_bytes, tid, blockDim.x);
        // and the tables the phase reads after its sweeps
        if (Phase == 0 && g.fold) {
            prefetch_l2(reinterpret_cast<const uint8_t*>(g.rs_x), (uint32_t)g.rs_nnz * 8u, tid, blockDim.x);
            prefetch_l2(reinterpret_cast<const uint8_t*>(g.rs_pos), (uint32_t)g.rs_nnz * 4u, tid, blockDim.x);
        } else if (Phase == 0) {
            prefetch_l2(reinterpret_cast<const uint8_t*>(g.sn_x), (uint32_t)g.sn_nnz * 8u, tid, blockDim.x);
            prefetch_l2(reinterpret_cast<const uint8_t*>(g.sn_pos), (uint32_t)g.sn_nnz * 4u, tid, blockDim.x);
        } else {
            if (g.fold) {
                prefetch_l2(reinterpret_cast<const uint8_t*>(g.zr_x), (uint32_t)g.zr_nnz * 8u, tid, blockDim.x);
                prefetch_l2(reinterpret_cast<const uint8_t*>(g.zr_col), (uint32_t)g.zr_nnz * 4u, tid, blockDim.x);
            }
            prefetch_l2(reinterpret_cast<const uint8_t*>(g.ret), (uint32_t)g.n * 8u, tid, blockDim.x);
            prefetch_l2(reinterpret_cast<const uint8_t*>(g.gain), (uint32_t)g.n * 8u, tid, blockDim.x);
        }
    }

    // shared memory: field [B][S] | rings | ready flags | misc (solve_smem_bytes)
    const int R = (int)g.fwd.ring_stages;
    SolveShared sh;
    sh.X = reinterpret_cast<double*>(smem);
    sh.ring = smem + (size_t)B * S * sizeof(double);
    sh.ready = sh.ring + (size_t)kSweepWarps * R * kStageBytes;
    sh.bars = reinterpret_cast<uint64_t*>(sh.ready + ((n + 1 + 15) & ~15));
    int* misc = reinterpret_cast<int*>(sh.bars + kSweepWarps * kStagesMax);
    sh.abort = misc;
    double* amb_e = reinterpret_cast<double*>(misc + 4);   // [8]
    int* active = reinterpret_cast<int*>(amb_e + 8);        // [8]
    if (tid == 0) misc[0] = 0;
    const int stall = ctx->test_ctl[0] ? g.stall_row : -1;
    sh.spin_limit = ctx->test_ctl[1] > 0 ? (uint32_t)ctx->test_ctl[1] : kSpinLimit;
    for (int i = tid; i <= n; i += blockDim.x) sh.ready[i] = i < n ? 0 : 0xFF;   // slot n: "no row"
    // padding slots (the zero column of padded terms) and envs the slab does not fill
    for (int e = 0; e < B; e++) {
        const int from = e < nenv ? n : 0;
        for (int i = from + tid; i < S; i += blockDim.x) sh.X[(size_t)e * S + i] = 0.0;
    }
    if (tid < nenv) {
        const int env = sd.env0 + tid;
        const ScnDev& sc = ctx->scns[ctx->envs[env].scn];
        const int cal = ctx->Ist[(size_t)env * L.ni + L.cal];   // calendar row of this step
        amb_e[tid] = sc.amb[cal];
        const double* D = ctx->Dst + (size_t)env * L.nd;
        int act = 0;
        for (int c = 0; c < k; c++)
            if (D[L.ag + c] != 0.0) { act = 1; break; }
        active[tid] = act;
    } else if (tid < 8) {
        active[tid] = 0;
    }
    __syncthreads();

    int any_active = 0;
    for (int e = 0; e < nenv; e++) any_active |= active[e];
    if (Phase == 0) {
        // ---- forcing (sb_fdm.c:146-152), written in row order: one thread per
        // row for all envs of the slab, the row's coefficients loaded once ----
        const int local0 = sd.env0 - g.env0;
        // the envs' per-zone heat staged in the (not yet used) ring memory, so
        // the row loop below has no dependent global load
        double* qz = reinterpret_cast<double*>(sh.ring);   // [nenv][nz]
        const bool qstaged = (size_t)nenv * g.nz * sizeof(double) <= (size_t)kSweepWarps * R * kStageBytes;
        if (qstaged)
            for (int t = tid; t < nenv * g.nz; t += blockDim.x) {
                const int e = t / g.nz, z = t - e * g.nz;
                qz[t] = ctx->Dst[(size_t)(sd.env0 + e) * L.nd + L.qdiv + z];
            }
        __syncthreads();
        for (int i = tid; i < n; i += blockDim.x) {
            const double cap = g.cap[i], dirx = g.dirx[i], mc = g.mc[i];
            const int z = g.zone_of_row[i];
            double Ti[kGroupLanes], Mi[kGroupLanes], qi[kGroupLanes];
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++) {
                if (e >= nenv) break;
                Ti[e] = g.T[(size_t)(local0 + e) * ncv + i];
                Mi[e] = g.M[(size_t)(local0 + e) * n + i];
            }
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++) {
                if (e >= nenv) break;
                qi[e] = z < 0 ? 0.0 : qstaged ? qz[e * g.nz + z] : ctx->Dst[(size_t)(sd.env0 + e) * L.nd + L.qdiv + z];
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

        // ---- first solve (the folded build: its forward half only) ----
        if (tid < kSweepWarps * 32) run_sweep(sh, g.fwd, B, S, n, 1, stall);
        __syncthreads();
        if (!g.fold) {
            if (tid < kSweepWarps * 32) run_sweep(sh, g.bwd, B, S, n, 2);
            __syncthreads();
        }
        if (*sh.abort) {   // uniform: read after the barrier
            if (tid == 0) set_error(ctx->status, *sh.abort);
            return;
        }

        // ---- folded air side: sensed = R z, one warp per sensor, its terms
        // spread over the lanes, a warp reduction per env ----
        if (g.fold && k > 0 && any_active) {
            const int lane = tid & 31;
            for (int r = tid >> 5; r < k; r += (int)(blockDim.x >> 5)) {
                double acc[kGroupLanes];
#pragma unroll
                for (int e = 0; e < kGroupLanes; e++) acc[e] = 0.0;
                const int p1 = g.rs_p[r + 1];
                for (int p = g.rs_p[r] + lane; p < p1; p += 32) {
                    const double xv = g.rs_x[p];
                    const int pos = g.rs_pos[p];
#pragma unroll
                    for (int e = 0; e < kGroupLanes; e++)
                        if (e < nenv) acc[e] = fma(xv, sh.X[(size_t)e * S + pos], acc[e]);
                }
#pragma unroll
                for (int e = 0; e < kGroupLanes; e++) {
                    double v = acc[e];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    acc[e] = v;
                }
                if (lane == 0) {
#pragma unroll
                    for (int e = 0; e < kGroupLanes; e++) {
                        if (e >= nenv) break;
                        if (!active[e]) continue;
                        const double* D = ctx->Dst + (size_t)(sd.env0 + e) * L.nd;
                        ctx->airq[(size_t)(sd.env0 + e) * ctx->k_max + r] = dmul(D[L.ag + r], dsub(D[L.aT + r], acc[e]));
                    }
                }
            }
        }
        // ---- air side (sb_fdm.c:155-181): the sensed right side to ctx->airq ----
        if (!g.fold && k > 0 && any_active) {
            // the sensed terms staged in the (now idle) ring memory when they fit
            const size_t ring_bytes = (size_t)kSweepWarps * R * kStageBytes;
            const bool staged = (size_t)g.sn_nnz * 12 <= ring_bytes;
            const double* snx = g.sn_x;
            const int32_t* snp = g.sn_pos;
            if (staged) {
                double* sx = reinterpret_cast<double*>(sh.ring);
                int32_t* sp = reinterpret_cast<int32_t*>(sh.ring + (size_t)g.sn_nnz * 8);
                block_copy(sx, g.sn_x, g.sn_nnz);
                block_copy(sp, g.sn_pos, g.sn_nnz);
                snx = sx;
                snp = sp;
            }
            __syncthreads();
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
                        xv[u] = p + u < p1 ? snx[p + u] : 0.0;
                        pos[u] = p + u < p1 ? snp[p + u] : 0;
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
                    ctx->airq[(size_t)(sd.env0 + e) * ctx->k_max + i] = dmul(D[L.ag + i], dsub(D[L.aT + i], acc[e]));
                }
            }
        }
        // y (folded build: z) -> the field array (row positions); phase 1 adds to it
        for (int i = tid; i < n; i += blockDim.x) {
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++)
                if (e < nenv) g.T[(size_t)(local0 + e) * ncv + i] = sh.X[(size_t)e * S + i];
        }
        return;
    }   // Phase 0

    const int local0 = sd.env0 - g.env0;
    // ---- folded build: the U sweep from z + Z q (z from phase 0 in the field
    // array, q k_dense's solution staged in the idle ring memory) ----
    if (g.fold) {
        double* qs = reinterpret_cast<double*>(sh.ring);   // [nenv][k]
        const bool air = k > 0 && any_active;
        const bool qstaged = (size_t)nenv * k * sizeof(double) <= (size_t)kSweepWarps * R * kStageBytes;
        if (air && qstaged)
            for (int t = tid; t < nenv * k; t += blockDim.x) {
                const int e = t / k, c = t - e * k;
                qs[t] = ctx->airq[(size_t)(sd.env0 + e) * ctx->k_max + c];
            }
        __syncthreads();
        const double* q = qstaged ? qs : ctx->airq;
        const size_t qstride = qstaged ? (size_t)k : (size_t)ctx->k_max;
        const size_t qbase = qstaged ? 0 : (size_t)sd.env0 * ctx->k_max;
        for (int i = tid; i < n; i += blockDim.x) {
            double acc[kGroupLanes];
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++)
                acc[e] = e < nenv ? g.T[(size_t)(local0 + e) * ncv + i] : 0.0;
            if (air) {
                const int p0 = g.zr_p[i], p1 = g.zr_p[i + 1];
                for (int p = p0; p < p1; p++) {
                    const int col = g.zr_col[p];
                    const double xv = g.zr_x[p];
#pragma unroll
                    for (int e = 0; e < kGroupLanes; e++) {
                        if (e >= nenv) break;
                        if (active[e]) acc[e] = fma(xv, q[qbase + (size_t)e * qstride + col], acc[e]);
                    }
                }
            }
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++)
                if (e < B) sh.X[(size_t)e * S + i] = acc[e];
        }
        __syncthreads();
        if (tid < kSweepWarps * 32) run_sweep(sh, g.bwd, B, S, n, 1);
        __syncthreads();
        if (*sh.abort) {
            if (tid == 0) set_error(ctx->status, *sh.abort);
            return;
        }
    }
    // ---- second solve: r = applied q (k_dense's solution), pulled per row in
    // ascending column order, zero q skipped; one thread per row for all envs ----
    if (!g.fold && k > 0 && any_active) {
        // the slab's dense solutions staged in the (not yet used) ring memory
        double* qs = reinterpret_cast<double*>(sh.ring);   // [nenv][k]
        const bool qstaged = (size_t)nenv * k * sizeof(double) <= (size_t)kSweepWarps * R * kStageBytes;
        if (qstaged)
            for (int t = tid; t < nenv * k; t += blockDim.x) {
                const int e = t / k, c = t - e * k;
                qs[t] = ctx->airq[(size_t)(sd.env0 + e) * ctx->k_max + c];
            }
        __syncthreads();
        const double* q = qstaged ? qs : ctx->airq;
        const size_t qstride = qstaged ? (size_t)k : (size_t)ctx->k_max;
        const size_t qbase = qstaged ? 0 : (size_t)sd.env0 * ctx->k_max;
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
                    const double qj = q[qbase + (size_t)e * qstride + col];
                    if (active[e] && qj != 0.0) acc[e] = dadd(acc[e], dmul(xv, qj));
                }
            }
#pragma unroll
            for (int e = 0; e < kGroupLanes; e++)
                if (e < B) sh.X[(size_t)e * S + i] = e < nenv && active[e] ? acc[e] : 0.0;
        }
        __syncthreads();
        if (tid < kSweepWarps * 32) run_sweep(sh, g.fwd, B, S, n, 1);
        __syncthreads();
        if (tid < kSweepWarps * 32) run_sweep(sh, g.bwd, B, S, n, 2);
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
            if (g.fold) ye = sh.X[(size_t)e * S + i];
            else if (k > 0 && active[e]) ye = dadd(ye, sh.X[(size_t)e * S + i]);
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
