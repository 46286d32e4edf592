/* Oracle driver ABI -- TEST INFRASTRUCTURE ONLY.
 *
 * Two shared libraries export this same ABI:
 *   liboracle.so        this repository's C restatement of the reference's CPU
 *                       core (oracle/sbo_*.c), self-contained;
 *   _ref/libcsimref.so  the reference's own C core (complete_port/csim sources,
 *                       compiled unmodified from the reference tree by
 *                       oracle/Makefile) behind ref_driver.c.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * either library, and only as the checker or the timed CPU baseline; the
 * product path (libsbenv.so) never links or calls them.
 *
 * One SboEnv is one environment of the reference CPU env
 * (complete_port/pufferlib_cpu_env.h:187-257): reset primes the occupancy
 * chains and writes the reset observation; step clamps and decodes the packed
 * [cont 256][disc 16] action, advances the simulator, writes the observation,
 * advances occupancy, computes the reward and auto-resets at max_steps. */
#ifndef SBO_H
#define SBO_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SBO_OBS 1024
#define SBO_CONT 256
#define SBO_DISC 16
#define SBO_NACT (SBO_CONT + SBO_DISC)
#define SBO_DAY_STEPS 288

/* The env's start-day stream: SplitMix64's output function (Steele, Lea and
 * Flood, OOPSLA 2014) over a golden-ratio increment. */
static inline unsigned long long sbo_start_mix(unsigned long long x) {
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
}
static inline int sbo_start_draw(unsigned long long* rng) {
    *rng += 0x9e3779b97f4a7c15ULL;
    return (int)(sbo_start_mix(*rng) % 7ULL);
}

typedef struct SboEnv SboEnv;

/* max_steps <= 0: the blob's episode length (obs_meta[3], else occ_hour rows - 1). */
SboEnv* sbo_create(const char* blob_path, int max_steps);
void sbo_destroy(SboEnv* e);
/* out[10] = {n_cvs, n_solved, k, n_zones, n_vav, n_ahu, n_action, n_cont, n_disc, obs_len} */
void sbo_dims(const SboEnv* e, int* out);
void sbo_reset(SboEnv* e, float* obs);
/* act: SBO_NACT floats; obs: SBO_OBS floats. parts12: the 12 diagnostic values
 * the reference reward writes (may be NULL). log8: {productivity, energy cost,
 * carbon, mean zone deviation K, worst zone deviation K, out-of-band fraction,
 * electricity kWh, gas kWh} of this step (may be NULL; a library that cannot
 * form an entry writes NaN there). */
void sbo_step(SboEnv* e, const float* act, float* obs, float* reward, float* terminal,
              double* reward_f64, double* parts12, double* log8);
void sbo_get_temp(const SboEnv* e, double* out);  /* n_cvs, cell order */
void sbo_get_mass(const SboEnv* e, double* out);  /* n_solved, solved order */
int sbo_step_index(const SboEnv* e);               /* steps in the current episode */
/* Re-seeds the occupancy and convection generators from the blob (tests that
 * compare two passes of one env need identical random streams). */
void sbo_reseed(SboEnv* e);
/* Episode options of the reference GPU backend (gpu/smart_buildings.cu:1636-1657,
 * 2806-2816, 1936-2050), which its CPU env lacks: the first episode's length
 * (desync; <= 0 keeps the blob's), and random starts -- at every reset the
 * SplitMix64 stream start_rng draws a day d in 0..6 and the episode runs from
 * calendar row d * 288 (priming with that row's occ_hour_m1 entry when the
 * blob has one per row). Call before the first reset. */
void sbo_set_episode(SboEnv* e, int first_len, unsigned long long start_rng, int random_start);
/* Calendar offset of the current episode. */
int sbo_episode_offset(const SboEnv* e);
/* Inspection (restatement only): out = [air_g k][air_T k][per-cell zone heat nz]
 * [flow factor sum, reheat W, boiler T, boiler return, pump head] of the last step. */
int sbo_debug(const SboEnv* e, double* out);
/* Visible state after the last step (the snapshot fields); -1 where not exported. */
int sbo_visible(const SboEnv* e, double* out);

#ifdef __cplusplus
}
#endif
#endif /* SBO_H */
