// Device helpers: exact-order fp64 arithmetic, mbarrier + bulk-copy PTX, and a
// warp-cooperative MT19937 matching numpy's RandomState stream.
#pragma once
#include <cstdint>

#include "sbenv_dev.h"

namespace sbenv {

// Every parity-critical operation is written with the _rn intrinsics, which the
// compiler never contracts into FMA; the library is also built with -fmad=false.
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double ddiv(double a, double b) { return __ddiv_rn(a, b); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait: returns false if the phase never completed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    for (uint32_t it = 0; it < (1u << 22); it++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// Plain (non-multicast) bulk copy global -> this CTA's shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// An int carried in the low word of a double (scratch exchange through shared memory).
__device__ __forceinline__ double int_in_double(int v) { return __hiloint2double(0, v); }
__device__ __forceinline__ int int_from_double(double d) { return __double2loint(d); }

// Row ready flags of the solve sweeps (shared memory, CTA scope).
__device__ __forceinline__ uint32_t ld_acquire_u8(const uint8_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u8 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u8(uint8_t* p, uint32_t v) {
    asm volatile("st.release.cta.shared::cta.u8 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// Block-wide copy of n elements, eight loads in flight per thread before the stores.
template <class T>
__device__ inline void block_copy(T* __restrict__ dst, const T* __restrict__ src, int n) {
    const int nt = (int)blockDim.x;
    int base = 0;
    for (; base + 8 * nt <= n; base += 8 * nt) {
        T v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = src[base + u * nt + (int)threadIdx.x];
#pragma unroll
        for (int u = 0; u < 8; u++) dst[base + u * nt + (int)threadIdx.x] = v[u];
    }
    for (int i = base + (int)threadIdx.x; i < n; i += nt) dst[i] = src[i];
}

// Block-wide gather dst[t] = src[idx[t]], eight loads in flight per thread.
__device__ inline void block_gather(double* __restrict__ dst, const double* __restrict__ src,
                                    const int32_t* __restrict__ idx, int n) {
    const int nt = (int)blockDim.x;
    int base = 0;
    for (; base + 8 * nt <= n; base += 8 * nt) {
        int ix[8];
        double v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) ix[u] = idx[base + u * nt + (int)threadIdx.x];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = src[ix[u]];
#pragma unroll
        for (int u = 0; u < 8; u++) dst[base + u * nt + (int)threadIdx.x] = v[u];
    }
    for (int i = base + (int)threadIdx.x; i < n; i += nt) dst[i] = src[idx[i]];
}

__device__ __forceinline__ void set_error(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------------------
// MT19937 (Matsumoto & Nishimura) in numpy RandomState's conventions:
// random_sample = ((w1 >> 5) * 2^26 + (w2 >> 6)) / 2^53 from two consecutive
// tempered words; randint(0, hi+1) by masked rejection. One warp runs the
// stream in lock step: every lane holds the same position and sees the same
// words, and the 624-word regeneration is shared across the lanes.
// ---------------------------------------------------------------------------
struct WarpMt {
    uint32_t* st;   // 624 raw state words of the current block (shared memory)
    uint32_t* nx;   // 624 raw state words of the next block
    uint32_t* tw;   // 2 x 624 tempered words: current block, next block
    int pos;        // absolute index into tw (0..1247); words < 624 are the current block
};

__device__ __forceinline__ uint32_t mt_temper(uint32_t y) {
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

__device__ __forceinline__ uint32_t mt_mix(uint32_t si, uint32_t si1, uint32_t sm) {
    const uint32_t x = (si & 0x80000000u) | (si1 & 0x7fffffffu);
    return sm ^ (x >> 1) ^ ((x & 1u) ? 0x9908b0dfu : 0u);
}

// In-place regeneration of the 624-word state. The sequential recurrence
// new[i] = f(old[i], old[i+1], new-or-old[i+397 mod 624]) reads only old words
// for i < 227, words of the first range for 227 <= i < 454 and of the second
// for i >= 454 (with new[0] for i = 623): three ranges, each computed by the
// whole warp from values read before any of it is written.
__device__ inline void mt_twist_warp(uint32_t* st) {
    const int lane = threadIdx.x & 31;
    uint32_t v[8];
    // [0, 227): st[i + 397] is still old
#pragma unroll
    for (int q = 0; q < 8; q++) {
        const int i = lane + 32 * q;
        v[q] = i < 227 ? mt_mix(st[i], st[i + 1], st[i + 397]) : 0u;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 8; q++) {
        const int i = lane + 32 * q;
        if (i < 227) st[i] = v[q];
    }
    __syncwarp();
    // [227, 454): st[i - 227] is new
#pragma unroll
    for (int q = 0; q < 8; q++) {
        const int i = 227 + lane + 32 * q;
        v[q] = i < 454 ? mt_mix(st[i], st[i + 1], st[i - 227]) : 0u;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 8; q++) {
        const int i = 227 + lane + 32 * q;
        if (i < 454) st[i] = v[q];
    }
    __syncwarp();
    // [454, 624): st[i - 227] is new, and so is st[0] for i = 623
#pragma unroll
    for (int q = 0; q < 6; q++) {
        const int i = 454 + lane + 32 * q;
        v[q] = i < 624 ? mt_mix(st[i], st[(i + 1) % 624], st[i - 227]) : 0u;
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 6; q++) {
        const int i = 454 + lane + 32 * q;
        if (i < 624) st[i] = v[q];
    }
    __syncwarp();
}

// Tempered current block from st, raw and tempered next block from a copy.
__device__ inline void mt_prepare_blocks(WarpMt& m) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < 624; i += 32) {
        m.tw[i] = mt_temper(m.st[i]);
        m.nx[i] = m.st[i];
    }
    __syncwarp();
    mt_twist_warp(m.nx);
    for (int i = lane; i < 624; i += 32) m.tw[624 + i] = mt_temper(m.nx[i]);
    __syncwarp();
}

// Loads a stream (624 raw words + position). A stream whose position is 624
// (fresh seed or block fully used) starts with a regeneration, as the
// sequential generator would.
__device__ inline void mt_load(WarpMt& m, const uint32_t* g, uint32_t* st, uint32_t* nx, uint32_t* tw) {
    const int lane = threadIdx.x & 31;
    m.st = st;
    m.nx = nx;
    m.tw = tw;
    for (int i = lane; i < 624; i += 32) st[i] = g[i];
    const int p = (int)g[624];
    __syncwarp();
    if (p >= 624) {
        mt_twist_warp(st);
        m.pos = 0;
    } else {
        m.pos = p;   // the raw state is the twisted block the position indexes into
    }
    mt_prepare_blocks(m);
}

// Advances to the next block once the current one is used up: the next block
// becomes current (raw and tempered), and one regeneration makes the new next.
__device__ inline void mt_roll(WarpMt& m) {
    if (m.pos < 624) return;
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < 624; i += 32) {
        m.st[i] = m.nx[i];
        m.tw[i] = m.tw[624 + i];
    }
    __syncwarp();
    mt_twist_warp(m.nx);
    for (int i = lane; i < 624; i += 32) m.tw[624 + i] = mt_temper(m.nx[i]);
    __syncwarp();
    m.pos -= 624;
}

__device__ __forceinline__ uint32_t mt_word(WarpMt& m) {
    mt_roll(m);
    return m.tw[m.pos++];
}

__device__ __forceinline__ double mt_sample(WarpMt& m) {
    const uint32_t a = mt_word(m) >> 5;
    const uint32_t b = mt_word(m) >> 6;
    return (a * 67108864.0 + b) / 9007199254740992.0;
}

__device__ __forceinline__ uint32_t mt_bounded(WarpMt& m, uint32_t hi) {
    if (hi == 0) return 0;
    uint32_t mask = hi;
    mask |= mask >> 1; mask |= mask >> 2; mask |= mask >> 4; mask |= mask >> 8; mask |= mask >> 16;
    uint32_t v = mt_word(m) & mask;
    while (v > hi) v = mt_word(m) & mask;
    return v;
}

// Stores the stream back: raw words of the current block + position. A
// warp-parallel scan may have read ahead into the next block (position up to
// 1247); the stored position must index the block the state words describe,
// so such a stream is rolled forward first.
__device__ inline void mt_store(WarpMt& m, uint32_t* g) {
    if (m.pos > 624) mt_roll(m);
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < 624; i += 32) g[i] = m.st[i];
    if (lane == 0) g[624] = (uint32_t)m.pos;
    __syncwarp();
}

}  // namespace sbenv
