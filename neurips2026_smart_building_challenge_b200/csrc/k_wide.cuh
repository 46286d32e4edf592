// Wide solve, phase 0: forcing, first L/U sweep pair (the folded build: its
// L sweep), the air side's sensed right side (folded: R z), y (folded: z) to
// the field -- the work of k_solve<0>, for a tile of up to 32 envs of one
// group per CTA, lane l of every solver warp working for env l of the tile.
//
// Reference: complete_port/csim/sb_fdm.c:142-181 (one env) and sb_lu.c:38-63
// (the factor replay). The tile's vectors live in a global scratch array
// X [n + 1][32] (the 32 envs of one row in 256 contiguous bytes, row n always
// zero) that stays in L1/L2, instead of a shared-memory slab of at most eight
// envs. The sweeps are level programs (wide_sched.cpp): each row receives its
// terms in the reference's push order, so the exact build (Tol = false: a
// rounded product and a rounded subtraction per term, the division by the
// diagonal) is bit-identical to the reference; the corrected and folded
// builds (Tol = true) use fused multiply-adds and the diagonal's reciprocal.
// A producer warp streams the level blocks into a shared-memory ring; the
// solver warps synchronise only through the rows' ready counts.
#pragma once
#include "dev_util.cuh"
#include "k_solve.cuh"   // prefetch_l2

namespace sbenv {

constexpr int kWideThreads = (kWideWarps + 1) * 32;   // the solver warps and the producer warp
constexpr uint32_t kWideSpin = 1u << 22;                // polls of one ready count before the wait gives up
constexpr int kWideRun = 8;                             // rows of one forcing / write-back run of a warp

// Shared memory of a wide-solve CTA: the stage ring, its full and empty
// mbarriers, the rows' ready counts and the abort word.
SB_HD constexpr size_t wide_smem_bytes(int n) {
    return (size_t)kWideStages * kWideStageBytes + 2 * kWideStages * 8 + (((size_t)n + 1) * 2 + 15) / 16 * 16 + 16;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u16(const uint16_t* p) {
    uint16_t v;
    asm volatile("ld.acquire.cta.shared::cta.u16 %0, [%1];" : "=h"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u16(uint16_t* p, uint32_t v) {
    asm volatile("st.release.cta.shared::cta.u16 [%0], %1;" ::"r"(smem_u32(p)), "h"((uint16_t)v) : "memory");
}

struct WideShared {
    uint8_t* slots;     // [kWideStages][kWideStageBytes]
    uint64_t* full;     // [kWideStages] the stage's copy has landed
    uint64_t* empty;    // [kWideStages] every solver warp is done with the stage
    uint16_t* ready;    // [n + 1] the rows' ready counts
    volatile int* abort;
    uint32_t spin;      // polls of one ready count (kWideSpin unless a failure test lowers it)
    bool stall;         // failure test: solver warp 0 waits for a count no row reaches
};

// Bounded mbarrier wait that also gives up once another warp has aborted.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort) {
    for (uint32_t it = 0; it < (1u << 22); it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 255u && *abort) return false;
    }
    return false;
}

// The level block of stage t: the L sweep's levels, then the U sweep's.
__device__ __forceinline__ void stage_src(const GroupDev& g, int t, const uint8_t*& src, uint32_t& bytes) {
    const WideSweep& s = t < g.wfwd.nlev ? g.wfwd : g.wbwd;
    const int lv = t < g.wfwd.nlev ? t : t - g.wfwd.nlev;
    const uint32_t off = __ldg(s.lev_off + lv);
    bytes = __ldg(s.lev_off + lv + 1) - off;
    src = s.blocks + off;
}

// Producer (lane 0 of the last warp): stage t into slot t % kWideStages once
// every solver warp has released stage t - kWideStages. Before it returns,
// every copy it issued has landed (bounded waits).
__device__ void wide_produce(const GroupDev& g, const WideShared& sh, int total) {
    int issued = 0;
    for (int t = 0; t < total && !*sh.abort; t++) {
        const int slot = t % kWideStages;
        if (t >= kWideStages && !mbar_wait_or_abort(sh.empty + slot, (uint32_t)(t / kWideStages - 1) & 1u, sh.abort)) {
            atomicCAS((int*)sh.abort, 0, kErrRingTimeout);
            break;
        }
        const uint8_t* src;
        uint32_t bytes;
        stage_src(g, t, src, bytes);
        fence_proxy_async();
        mbar_expect_tx(sh.full + slot, bytes);
        bulk_g2s(sh.slots + (size_t)slot * kWideStageBytes, src, bytes, sh.full + slot);
        issued = t + 1;
    }
    for (int t = max(0, issued - kWideStages); t < issued; t++)
        mbar_wait_bounded(sh.full + t % kWideStages, (uint32_t)(t / kWideStages) & 1u);
}

// One solver warp's part of one level: acquire the listed rows, then run the
// segments in order, publishing each row's count after its segment. Xl = the
// tile's X + lane; wdiag the U rows' diagonal (exact) or its reciprocal
// (tolerant). Warp-uniform; false if a wait gave up.
template <bool Tol>
__device__ __forceinline__ bool wide_level(const uint8_t* blk, const WideShared& sh, double* Xl,
                                           const double* __restrict__ wdiag, int warp, int lane, bool stall) {
    const char* xb = reinterpret_cast<const char*>(Xl);
    const int32_t* hdr = reinterpret_cast<const int32_t*>(blk);
    const int a = hdr[warp], b = hdr[warp + 1], nseg = hdr[kWideWarps];
    const int w0 = hdr[kWideWarps + 1 + warp], w1 = hdr[kWideWarps + 2 + warp], nwait = hdr[2 * kWideWarps + 1];
    const uint32_t* waits = reinterpret_cast<const uint32_t*>(blk + kWideHdrBytes);
    const uint8_t* segb = blk + kWideHdrBytes + (size_t)((nwait + 3) & ~3) * 4;
    const uint4* segs = reinterpret_cast<const uint4*>(segb);
    const WideChunk* chunks = reinterpret_cast<const WideChunk*>(segb + (size_t)nseg * sizeof(WideSeg));
    bool ok = true;
    // failure test: lane 0 also waits for row 0 to reach a count no row reaches
    const int first = stall ? w0 - 1 : w0;
    for (int i = first + lane; i < w1 && ok; i += 32) {
        const uint32_t e = i < w0 ? 0xFFFFu : waits[i];
        const uint16_t* f = sh.ready + (e >> 16);
        const uint32_t need = e & 0xFFFFu;
        uint32_t spins = 0;
        while (ld_acquire_u16(f) < need) {
            if (++spins >= sh.spin || ((spins & 1023u) == 0 && *sh.abort)) {
                atomicCAS((int*)sh.abort, 0, kErrWaitTimeout);
                ok = false;
                break;
            }
            if (spins > 16) __nanosleep(32);
        }
    }
    if (!__all_sync(0xffffffffu, ok)) return false;
    __threadfence_block();   // what the acquiring lanes saw, for every lane of the warp
    for (int q = a; q < b; q++) {
        const uint4 sg = segs[q];
        double acc = Xl[(size_t)sg.x * kWideEnvs];
        const WideChunk* ch = chunks + sg.y;
        // the source values of up to kWideGroup chunks are loaded together,
        // then those chunks' terms applied in order
        for (uint32_t c0 = 0; c0 < sg.z; c0 += kWideGroup) {
            const uint32_t m = min((uint32_t)kWideGroup, sg.z - c0);
            double x[kWideGroup][4];
#pragma unroll
            for (int j = 0; j < kWideGroup; j++) {
                if ((uint32_t)j < m) {
                    const uint4 o = *reinterpret_cast<const uint4*>(ch[c0 + j].off);
                    x[j][0] = *reinterpret_cast<const double*>(xb + o.x);
                    x[j][1] = *reinterpret_cast<const double*>(xb + o.y);
                    x[j][2] = *reinterpret_cast<const double*>(xb + o.z);
                    x[j][3] = *reinterpret_cast<const double*>(xb + o.w);
                }
            }
#pragma unroll
            for (int j = 0; j < kWideGroup; j++) {
                if ((uint32_t)j < m) {
                    const double2 v01 = reinterpret_cast<const double2*>(ch[c0 + j].v)[0];
                    const double2 v23 = reinterpret_cast<const double2*>(ch[c0 + j].v)[1];
                    if (Tol) {
                        acc = fma(-v01.x, x[j][0], acc);
                        acc = fma(-v01.y, x[j][1], acc);
                        acc = fma(-v23.x, x[j][2], acc);
                        acc = fma(-v23.y, x[j][3], acc);
                    } else {
                        acc = dsub(acc, dmul(v01.x, x[j][0]));
                        acc = dsub(acc, dmul(v01.y, x[j][1]));
                        acc = dsub(acc, dmul(v23.x, x[j][2]));
                        acc = dsub(acc, dmul(v23.y, x[j][3]));
                    }
                }
            }
        }
        if (sg.w & 1u) acc = Tol ? dmul(acc, __ldg(wdiag + sg.x)) : ddiv(acc, __ldg(wdiag + sg.x));
        Xl[(size_t)sg.x * kWideEnvs] = acc;
        __syncwarp();   // every lane's store precedes the release below
        if (lane == 0) st_release_u16(sh.ready + sg.x, sg.w >> 16);
    }
    return true;
}

// The solver warps' sweeps: stage after stage from the ring, each released
// to the producer once the warp is done with it.
template <bool Tol>
__device__ void wide_solve(const GroupDev& g, const WideShared& sh, int total, double* Xl, int warp, int lane) {
    for (int t = 0; t < total; t++) {
        const int slot = t % kWideStages;
        bool ok = !*sh.abort && mbar_wait_or_abort(sh.full + slot, (uint32_t)(t / kWideStages) & 1u, sh.abort);
        ok = __all_sync(0xffffffffu, ok);
        if (ok)
            ok = wide_level<Tol>(sh.slots + (size_t)slot * kWideStageBytes, sh, Xl, g.wdiag, warp, lane,
                                 sh.stall && warp == 0 && t == 0);
        __syncwarp();
        if (lane == 0) {
            if (!ok) atomicCAS((int*)sh.abort, 0, kErrRingTimeout);
            mbar_arrive(sh.empty + slot);
        }
        if (!ok) return;
    }
}

template <bool Tol>
__global__ void __launch_bounds__(kWideThreads, kWideCtas)
k_wide0(const StepCtx* __restrict__ ctx, const WideTile* __restrict__ tiles) {
    // a programmatic dependent (the random streams) may start once every CTA is resident
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const WideTile wt = tiles[blockIdx.x];
    const GroupDev& g = ctx->groups[wt.group];
    const StateLayout& L = ctx->lay;
    const int n = g.n, ncv = g.ncv, k = g.k;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool solver = warp < kWideWarps;
    const bool live = lane < wt.nenv;
    // lanes past the tile's envs compute on env0's inputs and write nothing
    const int env = wt.env0 + (live ? lane : 0);
    const int local = env - g.env0;
    double* Xl = g.X + (size_t)wt.tile * (n + 1) * kWideEnvs + lane;
    extern __shared__ __align__(128) uint8_t wsm[];
    WideShared sh;
    sh.slots = wsm;
    sh.full = reinterpret_cast<uint64_t*>(wsm + (size_t)kWideStages * kWideStageBytes);
    sh.empty = sh.full + kWideStages;
    sh.ready = reinterpret_cast<uint16_t*>(sh.empty + kWideStages);
    sh.abort = reinterpret_cast<volatile int*>(wsm + wide_smem_bytes(n) - 16);
    sh.stall = ctx->test_ctl[0] != 0;
    sh.spin = ctx->test_ctl[1] > 0 ? (uint32_t)ctx->test_ctl[1] : kWideSpin;
    const int total = g.wfwd.nlev + (g.fold ? 0 : g.wbwd.nlev);
    if (tid == 0) {
        *sh.abort = 0;
        for (int s = 0; s < kWideStages; s++) {
            mbar_init(sh.full + s, 1);
            mbar_init(sh.empty + s, kWideWarps);
        }
        mbar_fence_init();
    }
    for (int i = tid; i <= n; i += blockDim.x) sh.ready[i] = 0;
    // the group's first tile pulls the level programs into L2 for the others
    if (wt.tile == 0) {
        prefetch_l2(g.wfwd.blocks, g.wfwd.lev_off[g.wfwd.nlev], tid, blockDim.x);
        if (!g.fold) prefetch_l2(g.wbwd.blocks, g.wbwd.lev_off[g.wbwd.nlev], tid, blockDim.x);
    }
    const ScnDev& sc = ctx->scns[ctx->envs[env].scn];
    const double amb = sc.amb[ctx->Ist[(size_t)env * L.ni + L.cal]];   // this step's calendar row
    const double* D = ctx->Dst + (size_t)env * L.nd;
    const double* Tg = g.T + (size_t)local * ncv;
    const double* Mg = g.M + (size_t)local * n;

    // ---- forcing (sb_fdm.c:146-152): runs of kWideRun rows per solver warp,
    // all their loads in flight together; a lane's loads of one run share
    // sectors of its env's field and mass ----
    for (int i0 = warp * kWideRun; solver && i0 < n; i0 += kWideWarps * kWideRun) {
        double Ti[kWideRun], Mi[kWideRun], qi[kWideRun];
#pragma unroll
        for (int j = 0; j < kWideRun; j++) {
            const int i = min(i0 + j, n - 1);
            const int z = __ldg(g.zone_of_row + i);
            Ti[j] = Tg[i];
            Mi[j] = Mg[i];
            qi[j] = z < 0 ? 0.0 : D[L.qdiv + z];
        }
#pragma unroll
        for (int j = 0; j < kWideRun; j++) {
            const int i = i0 + j;
            if (i >= n) break;
            double b = dadd(dmul(__ldg(g.cap + i), Ti[j]), qi[j]);
            b = dadd(b, dmul(amb, __ldg(g.dirx + i)));
            b = dadd(b, dmul(__ldg(g.mc + i), Mi[j]));
            Xl[(size_t)i * kWideEnvs] = b;
        }
    }
    __syncthreads();

    // ---- first solve (the folded build: its forward half only): the
    // producer warp streams the level blocks, the solver warps run them ----
    if (solver) wide_solve<Tol>(g, sh, total, Xl, warp, lane);
    else if (lane == 0) wide_produce(g, sh, total);
    __syncthreads();
    const int err = *sh.abort;
    if (tid == 0)
        for (int s = 0; s < kWideStages; s++) {
            mbar_inval(sh.full + s);
            mbar_inval(sh.empty + s);
        }
    if (err) {   // uniform
        if (tid == 0) set_error(ctx->status, err);
        return;
    }

    // ---- air side: the sensed right side (sb_fdm.c:155-181) or, folded, R z;
    // one solver warp per coupled VAV ----
    if (k > 0) {
        int act = 0;
        for (int c = 0; c < k; c++)
            if (D[L.ag + c] != 0.0) { act = 1; break; }
        const int32_t* rp = g.fold ? g.rs_p : g.sn_p;
        const int32_t* rpos = g.fold ? g.rs_pos : g.sn_pos;
        const double* rx = g.fold ? g.rs_x : g.sn_x;
        for (int r = warp; solver && r < k; r += kWideWarps) {
            double acc = 0.0;
            const int p1 = __ldg(rp + r + 1);
            // four terms' loads in flight, then their products summed in order
            for (int p0 = __ldg(rp + r); p0 < p1; p0 += 4) {
                double xv[4], cv[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int p = min(p0 + u, p1 - 1);
                    xv[u] = Xl[(size_t)__ldg(rpos + p) * kWideEnvs];
                    cv[u] = __ldg(rx + p);
                }
#pragma unroll
                for (int u = 0; u < 4; u++)
                    if (p0 + u < p1) acc = Tol ? fma(cv[u], xv[u], acc) : dadd(acc, dmul(cv[u], xv[u]));
            }
            if (live && act) ctx->airq[(size_t)env * ctx->k_max + r] = dmul(D[L.ag + r], dsub(D[L.aT + r], acc));
        }
    }
    // ---- y (folded build: z) -> the field array (row positions); phase 1
    // adds to it ----
    if (live && solver) {
        double* Tw = g.T + (size_t)local * ncv;
        for (int i0 = warp * kWideRun; i0 < n; i0 += kWideWarps * kWideRun) {
            double y[kWideRun];
#pragma unroll
            for (int j = 0; j < kWideRun; j++) y[j] = Xl[(size_t)min(i0 + j, n - 1) * kWideEnvs];
#pragma unroll
            for (int j = 0; j < kWideRun; j++)
                if (i0 + j < n) Tw[i0 + j] = y[j];
        }
    }
}

}  // namespace sbenv
