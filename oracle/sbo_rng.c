/* TEST INFRASTRUCTURE: MT19937 matching numpy's legacy RandomState stream,
 * restated from the published algorithm (Matsumoto & Nishimura 1998) and
 * numpy's random_sample / bounded-integer conventions, as the reference uses
 * them (complete_port/csim/sb_rng.c:9-54):
 *   seed      init_genrand: s[0] = seed, s[i] = 1812433253*(s[i-1]^(s[i-1]>>30)) + i
 *   sample    (a>>5) * 2^26 + (b>>6), divided by 2^53, from two consecutive words
 *   bounded   mask = smallest 2^m - 1 >= hi; draw (word & mask) until <= hi */
#include "sbo_internal.h"

void sbo_mt_seed(SboMt* m, uint32_t seed) {
    m->s[0] = seed;
    for (int i = 1; i < 624; i++) m->s[i] = 1812433253u * (m->s[i - 1] ^ (m->s[i - 1] >> 30)) + (uint32_t)i;
    m->pos = 624;
}

static void mt_twist(SboMt* m) {
    for (int i = 0; i < 624; i++) {
        uint32_t x = (m->s[i] & 0x80000000u) | (m->s[(i + 1) % 624] & 0x7fffffffu);
        uint32_t xa = x >> 1;
        if (x & 1u) xa ^= 0x9908b0dfu;
        m->s[i] = m->s[(i + 397) % 624] ^ xa;
    }
    m->pos = 0;
}

uint32_t sbo_mt_next(SboMt* m) {
    if (m->pos >= 624) mt_twist(m);
    uint32_t y = m->s[m->pos++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

double sbo_mt_sample(SboMt* m) {
    uint32_t a = sbo_mt_next(m) >> 5;
    uint32_t b = sbo_mt_next(m) >> 6;
    return (a * 67108864.0 + b) / 9007199254740992.0;
}

uint32_t sbo_mt_bounded(SboMt* m, uint32_t hi) {
    if (hi == 0) return 0;
    uint32_t mask = hi;
    mask |= mask >> 1; mask |= mask >> 2; mask |= mask >> 4; mask |= mask >> 8; mask |= mask >> 16;
    uint32_t v;
    do { v = sbo_mt_next(m) & mask; } while (v > hi);
    return v;
}
