// Action sampler of the policy-in-loop rollout: the
// trainer's mixed heads of the reference (patches/pufferlib_core.diff:2490-2580,
// Beta draws :1015-1040, head activity :828-834; config/smart_buildings.ini
// beta_floor / beta_conc_max), one thread per (env, head).
//
// Logit layout, as the trainer's: two blocks [2][n][kMaskWidth] (the second
// block at raw + n * kMaskWidth). Block 0 holds, per env, the 256 continuous
// heads' u then the 16 discrete heads' class logits (off, on); block 1 holds
// the continuous heads' v (its discrete columns are unused).
//
// Continuous head h (mask[env][h] != 0): alpha = softplus(u) + floor, beta =
// softplus(v) + floor, both scaled by cap / (alpha + beta) when alpha + beta
// exceeds the cap (the mean is kept); x ~ Beta(alpha, beta) = G1 / (G1 + G2),
// clamped into [kXLo, kXHi]; action 2x - 1.
// Discrete head d: classes whose mask entry is 0 are excluded; the drawn class
// index (0.0 / 1.0) is the action (the env runs a discrete actuator iff its
// action is 1.0).
// A head with no unmasked entry is padding: action 0.0, no draw.
// Logits pass through finite_or_clamp: NaN -> 0, clamped into [-1e6, 1e6].
//
// Random numbers: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011), counter = (head, env, call, draw
// block), key = seed; normals by Box-Muller. Gamma: Marsaglia and Tsang, "A
// simple method for generating gamma variables" (ACM TOMS 2000), with the
// acceptance test written in 1 - t and log1p(cz) so it keeps its precision
// when t is near 1; shape k < 1 draws G(k + 1) U^(1/k). At most kGammaTries
// proposals (the acceptance rate is above 0.95 for shapes >= 1); after that
// the draw returns d, the scale of the proposal's mode.
#pragma once
#include <cstdint>

#include "sbenv_dev.h"

namespace sbenv {

constexpr int kGammaTries = 64;
constexpr float kXLo = 1.0e-6f, kXHi = 1.0f - 1.0e-6f;

struct Philox {
    uint32_t c[4];
    uint32_t k[2];
    uint32_t out[4];
    int used = 4;

    __device__ static inline void round(uint32_t* x, const uint32_t* key) {
        const uint32_t m0 = 0xD2511F53u, m1 = 0xCD9E8D57u;
        const uint32_t hi0 = __umulhi(m0, x[0]), lo0 = m0 * x[0];
        const uint32_t hi1 = __umulhi(m1, x[2]), lo1 = m1 * x[2];
        const uint32_t y0 = hi1 ^ x[1] ^ key[0], y2 = hi0 ^ x[3] ^ key[1];
        x[0] = y0;
        x[1] = lo1;
        x[2] = y2;
        x[3] = lo0;
    }
    __device__ inline void block() {
        uint32_t x[4] = {c[0], c[1], c[2], c[3]};
        uint32_t key[2] = {k[0], k[1]};
#pragma unroll
        for (int r = 0; r < 10; r++) {
            round(x, key);
            key[0] += 0x9E3779B9u;
            key[1] += 0xBB67AE85u;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) out[i] = x[i];
        c[3]++;   // the next block of this stream
        used = 0;
    }
    __device__ inline uint32_t next() {
        if (used == 4) block();
        return out[used++];
    }
    // uniform in (0, 1]
    __device__ inline float uniform() { return ((float)(next() >> 8) + 1.0f) * (1.0f / 16777216.0f); }
    __device__ inline float normal() {
        const float u1 = uniform(), u2 = uniform();
        return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
};

__device__ inline float gamma_draw(Philox& rng, float k) {
    const float kk = k < 1.0f ? k + 1.0f : k;
    const float d = kk - 1.0f / 3.0f, c = rsqrtf(9.0f * d);
    float t = 1.0f;
    for (int tries = 0;; tries++) {
        if (tries == kGammaTries) { t = 1.0f; break; }
        const float z = rng.normal();
        const float cz = c * z;
        if (cz <= -1.0f) continue;
        const float v = 1.0f + cz;
        t = v * v * v;
        const float u = rng.uniform();
        if (u < 1.0f - 0.0331f * z * z * z * z) break;
        const float one_minus_t = -cz * (3.0f + cz * (3.0f + cz));
        if (logf(u) < 0.5f * z * z + d * (one_minus_t + 3.0f * log1pf(cz))) break;
    }
    const float scale = k < 1.0f ? d * powf(rng.uniform(), 1.0f / k) : d;
    return scale * t;
}

__device__ inline float finite_or_clamp(float x) {
    if (x != x) return 0.0f;
    return fminf(1.0e6f, fmaxf(-1.0e6f, x));
}

// softplus(u) + floor without overflow: max(u, 0) + log1p(exp(-|u|))
__device__ inline float concentration(float u, float floor_c) {
    return fmaxf(u, 0.0f) + log1pf(expf(-fabsf(u))) + floor_c;
}

// call: device word counting the draws (read here, advanced by the caller),
// so a captured graph draws fresh numbers on every replay
__global__ void __launch_bounds__(256) k_beta_actions(const float* __restrict__ raw,
                                                      const uint8_t* __restrict__ mask,
                                                      float* __restrict__ actions, int n, float floor_c,
                                                      float cap, uint64_t seed,
                                                      const unsigned long long* __restrict__ call_dev) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * kAct) return;
    const uint64_t call = *call_dev;
    const int env = i / kAct, head = i % kAct;
    const float* row = raw + (size_t)env * kMaskWidth;
    const float* row2 = raw + ((size_t)n + env) * kMaskWidth;
    const uint8_t* m = mask ? mask + (size_t)env * kMaskWidth : nullptr;
    Philox rng;
    rng.c[0] = (uint32_t)head;
    rng.c[1] = (uint32_t)env;
    rng.c[2] = (uint32_t)call;
    rng.c[3] = (uint32_t)(call >> 32) << 16;
    rng.k[0] = (uint32_t)seed;
    rng.k[1] = (uint32_t)(seed >> 32);
    if (head >= kCont) {
        const int off = kCont + 2 * (head - kCont);
        const bool on0 = !m || m[off] != 0, on1 = !m || m[off + 1] != 0;
        if (!on0 && !on1) { actions[i] = 0.0f; return; }
        if (!on0 || !on1) { actions[i] = on1 ? 1.0f : 0.0f; return; }
        // P(class 1) = 1 / (1 + exp(l0 - l1))
        const float p1 = 1.0f / (1.0f + expf(finite_or_clamp(row[off]) - finite_or_clamp(row[off + 1])));
        actions[i] = rng.uniform() <= p1 ? 1.0f : 0.0f;
        return;
    }
    if (m && m[head] == 0) { actions[i] = 0.0f; return; }
    float a = concentration(finite_or_clamp(row[head]), floor_c);
    float b = concentration(finite_or_clamp(row2[head]), floor_c);
    if (cap > 0.0f && a + b > cap) {   // keep the mean, cap the concentration
        const float s = cap / (a + b);
        a *= s;
        b *= s;
    }
    const float g1 = gamma_draw(rng, a), g2 = gamma_draw(rng, b);
    const float x = fminf(kXHi, fmaxf(kXLo, g1 / (g1 + g2)));
    actions[i] = 2.0f * x - 1.0f;
}

}  // namespace sbenv
