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
    uint32_t* st;   // 624 raw state words (shared memory)
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

// In-place regeneration of the 624-word state. Processing 32-word chunks in
// increasing index order, reading each chunk before writing it, reproduces the
// sequential recurrence: s[i] uses the old s[i+1] and the new s[i-227].
__device__ inline void mt_twist_warp(uint32_t* st) {
    const int lane = threadIdx.x & 31;
    for (int base = 0; base < 624; base += 32) {
        const int i = base + lane;
        uint32_t nv = 0;
        if (i < 624) {
            const uint32_t x = (st[i] & 0x80000000u) | (st[(i + 1) % 624] & 0x7fffffffu);
            uint32_t xa = x >> 1;
            if (x & 1u) xa ^= 0x9908b0dfu;
            nv = st[(i + 397) % 624] ^ xa;
        }
        __syncwarp();
        if (i < 624) st[i] = nv;
        __syncwarp();
    }
}

__device__ inline void mt_fill_block(uint32_t* st, uint32_t* dst) {
    mt_twist_warp(st);
    for (int i = threadIdx.x & 31; i < 624; i += 32) dst[i] = mt_temper(st[i]);
    __syncwarp();
}

// Loads a stream (624 raw words + position) and prepares the current and next
// tempered blocks. A stream whose position is 624 (fresh seed or block fully
// used) starts with a regeneration, as the sequential generator would.
__device__ inline void mt_load(WarpMt& m, const uint32_t* g, uint32_t* st, uint32_t* tw) {
    const int lane = threadIdx.x & 31;
    m.st = st;
    m.tw = tw;
    for (int i = lane; i < 624; i += 32) st[i] = g[i];
    const int p = (int)g[624];
    __syncwarp();
    if (p >= 624) {
        mt_fill_block(st, tw);
        m.pos = 0;
    } else {
        // the raw state is the twisted block the position indexes into
        for (int i = lane; i < 624; i += 32) tw[i] = mt_temper(st[i]);
        __syncwarp();
        m.pos = p;
    }
    // next block from a copy of the state (the stored state stays the current block)
    for (int i = lane; i < 624; i += 32) tw[624 + i] = st[i];
    __syncwarp();
    mt_twist_warp(tw + 624);
    for (int i = lane; i < 624; i += 32) tw[624 + i] = mt_temper(tw[624 + i]);
    __syncwarp();
}

// Advances to the next block once the current one is used up: the next block
// becomes current, and its raw state (st twisted once more) is kept in st.
__device__ inline void mt_roll(WarpMt& m) {
    if (m.pos < 624) return;
    const int lane = threadIdx.x & 31;
    mt_twist_warp(m.st);   // st now holds the raw words of the block that becomes current
    for (int i = lane; i < 624; i += 32) m.tw[i] = m.tw[624 + i];
    __syncwarp();
    // new next block: twist a scratch copy of st (scratch = next-block area)
    for (int i = lane; i < 624; i += 32) m.tw[624 + i] = m.st[i];
    __syncwarp();
    mt_twist_warp(m.tw + 624);
    for (int i = lane; i < 624; i += 32) m.tw[624 + i] = mt_temper(m.tw[624 + i]);
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
