// Corrected air side: the second phase of the solve without a second
// triangular solve. The reference core solves A y2 = applied q and adds y2 to
// the first solution (complete_port/csim/sb_fdm.c:171-181); since A is fixed
// per building, y2 = W q with W = A^-1 applied, the n x k response the core
// already forms at setup to build S (sb_fdm.c:103-114). This kernel adds W q
// to y for every env, then updates the interior mass and the field
// (sb_fdm.c:183-187): a streaming pass over the field and the mass, bound by
// HBM, in place of a latency-bound pair of triangular sweeps. The sums run in
// a different order from the reference's solve, so the build agrees with it
// within the north star's 1e-9 per-step tolerance, not bit for bit.
//
// One CTA per tile of kCorrRows rows x kCorrEnvs envs of one group. The
// tile's W block is stored on the host as [k][kCorrRows] (rows past n zero)
// and lands in shared memory with one bulk copy; the envs' dense solutions
// sit beside it as [k][kCorrEnvs]. Warp w forms, for its eight envs
// 8 (w & 3) .. +7 and its rows lane + 32 i (i < kCorrRowsPerLane) of row
// half w >> 2, sixteen outputs per thread: per column two W values and eight
// broadcast solution values feed sixteen fused multiply-adds.
#pragma once
#include "dev_util.cuh"

namespace sbenv {

struct CorrTile {
    int group;
    int row0;    // first row of the tile
    int env0;    // first global env
    int nenv;    // envs in the tile (<= kCorrEnvs)
    long long w; // offset (doubles) of the tile's W block in its group's array
};
constexpr int kCorrRows = 128;
constexpr int kCorrEnvs = 32;
constexpr int kCorrThreads = 256;
constexpr int kCorrRowsPerLane = kCorrRows / 64;   // two row halves of 64 rows
constexpr int kCorrEnvsPerThread = kCorrEnvs / 4;  // four env groups of 8
__host__ __device__ constexpr size_t corr_smem_bytes(int k) {
    return sizeof(double) * ((size_t)k * kCorrRows + (size_t)k * kCorrEnvs + kCorrEnvs) + 16 + 4 * kCorrEnvs;
}

__global__ void __launch_bounds__(kCorrThreads) k_correct(const StepCtx* __restrict__ ctx,
                                                          const CorrTile* __restrict__ tiles) {
    extern __shared__ __align__(128) double csm[];
    const CorrTile t = tiles[blockIdx.x];
    const GroupDev& g = ctx->groups[t.group];
    const StateLayout& L = ctx->lay;
    const int k = g.k, n = g.n, ncv = g.ncv, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    double* Wt = csm;                                   // [k][kCorrRows]
    double* Q = Wt + (size_t)k * kCorrRows;             // [k][kCorrEnvs]
    double* amb = Q + (size_t)k * kCorrEnvs;            // [kCorrEnvs]
    uint64_t* bar = reinterpret_cast<uint64_t*>(amb + kCorrEnvs);
    const uint32_t wbytes = (uint32_t)(k * kCorrRows * sizeof(double));
    if (tid == 0 && k > 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
        mbar_expect_tx(bar, wbytes);
        bulk_g2s(Wt, g.W + t.w, wbytes, bar);
    }
    // this thread's field values (y of the first solve) and interior masses,
    // loaded while the W block lands
    const int e0 = 8 * (w & 3), rbase = 64 * (w >> 2) + lane;
    double acc[kCorrRowsPerLane][kCorrEnvsPerThread], mas[kCorrRowsPerLane][kCorrEnvsPerThread];
#pragma unroll
    for (int i = 0; i < kCorrRowsPerLane; i++)
#pragma unroll
        for (int j = 0; j < kCorrEnvsPerThread; j++) {
            const int r = t.row0 + rbase + 32 * i, e = e0 + j;
            const bool in = r < n && e < t.nenv;
            const size_t local = (size_t)(t.env0 + (in ? e : 0) - g.env0);
            acc[i][j] = in ? g.T[local * ncv + r] : 0.0;
            mas[i][j] = in ? g.M[local * n + r] : 0.0;
        }
    // the envs' dense solutions (zero for an env whose air side is off this
    // step: its right side was never formed) and calendar ambient; every load
    // of the prologue is independent of the others, so they are all in flight
    // together with the W block and the field values above
    int* act = reinterpret_cast<int*>(bar + 1);         // [kCorrEnvs]
    if (tid < kCorrEnvs) act[tid] = 0;
    __syncthreads();
    for (int idx = tid; idx < t.nenv * k; idx += kCorrThreads) {
        const int e = idx / k, c = idx - e * k;
        if (ctx->Dst[(size_t)(t.env0 + e) * L.nd + L.ag + c] != 0.0) act[e] = 1;
    }
    if (tid < t.nenv) {
        const int env = t.env0 + tid;
        const ScnDev& sc = ctx->scns[ctx->envs[env].scn];
        amb[tid] = sc.amb[ctx->Ist[(size_t)env * L.ni + L.cal]];
    }
    __syncthreads();
    for (int idx = tid; idx < k * kCorrEnvs; idx += kCorrThreads) {
        const int c = idx / kCorrEnvs, e = idx - c * kCorrEnvs;
        Q[idx] = (e < t.nenv && act[e]) ? ctx->airq[(size_t)(t.env0 + e) * ctx->k_max + c] : 0.0;
    }
    __syncthreads();
    bool landed = true;
    if (k > 0) landed = mbar_wait_bounded(bar, 0);
    if (!__syncthreads_and(landed)) {
        if (tid == 0) set_error(ctx->status, kErrRingTimeout);
        return;
    }
    for (int c = 0; c < k; c++) {
        double wv[kCorrRowsPerLane];
#pragma unroll
        for (int i = 0; i < kCorrRowsPerLane; i++) wv[i] = Wt[(size_t)c * kCorrRows + rbase + 32 * i];
        const double2* qv = reinterpret_cast<const double2*>(Q + (size_t)c * kCorrEnvs + e0);
        double qe[kCorrEnvsPerThread];
#pragma unroll
        for (int j = 0; j < kCorrEnvsPerThread / 2; j++) {
            const double2 v = qv[j];
            qe[2 * j] = v.x;
            qe[2 * j + 1] = v.y;
        }
#pragma unroll
        for (int i = 0; i < kCorrRowsPerLane; i++)
#pragma unroll
            for (int j = 0; j < kCorrEnvsPerThread; j++) acc[i][j] = fma(wv[i], qe[j], acc[i][j]);
    }
    // interior mass and field (sb_fdm.c:183-187)
#pragma unroll
    for (int i = 0; i < kCorrRowsPerLane; i++) {
        const int r = t.row0 + rbase + 32 * i;
        if (r >= n) continue;
        const double ret = g.ret[r], gain = g.gain[r];
#pragma unroll
        for (int j = 0; j < kCorrEnvsPerThread; j++) {
            const int e = e0 + j;
            if (e >= t.nenv) break;
            const size_t local = (size_t)(t.env0 + e - g.env0);
            g.M[local * n + r] = dadd(dmul(mas[i][j], ret), dmul(gain, acc[i][j]));
            g.T[local * ncv + r] = acc[i][j];
        }
    }
    // cells outside the solve take the ambient (the tiles of the first rows)
    if (t.row0 == 0 && ncv > n)
        for (int e = w; e < t.nenv; e += kCorrThreads / 32)
            for (int i = n + lane; i < ncv; i += 32) g.T[(size_t)(t.env0 + e - g.env0) * ncv + i] = amb[e];
    if (tid == 0 && k > 0) mbar_inval(bar);
}

}  // namespace sbenv
