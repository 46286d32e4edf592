/* TEST INFRASTRUCTURE: drives the reference's own C core (complete_port/csim,
 * compiled unmodified from the reference tree) behind the oracle ABI in sbo.h.
 *
 * The call sequence is the reference CPU env's, complete_port/pufferlib_cpu_env.h:
 *   reset :187-208  sb_sim_reset, sb_occup_prime, obs(0), sb_occup_advance(0)
 *   step  :211-257  clamp cont to [-1,1], sb_decode_native, sb_sim_apply_native,
 *                   sb_sim_step, obs(step), sb_occup_advance(step),
 *                   sb_reward(step), terminal at max_steps + auto-reset.
 * The reference's ctypes bridge (csim/sb_bridge.c) is not used: its decode
 * line reads and increments the same index in one expression. */
#include "sbo.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "sb_baked.h"
#include "sb_convect.h"
#include "sb_fdm.h"
#include "sb_obs.h"
#include "sb_occup.h"
#include "sb_reward.h"
#include "sb_sim.h"

struct SboEnv {
    SbBlob blob;
    SbFdm fdm;
    SbConv conv;
    SbOccup occ;
    SbSim sim;
    const uint8_t* is_disc;
    int n_act, n_cont, n_disc, obs_len, step, max_steps;
    int cur_len, off, random_start, m1_rows;
    unsigned long long start_rng;
    const int64_t* hour_m1;
    const uint8_t* wd_m1;
    double cont[SBO_CONT], disc[SBO_DISC], native[SBO_NACT], parts[12];
};

SboEnv* sbo_create(const char* path, int max_steps) {
    SboEnv* e = (SboEnv*)calloc(1, sizeof(SboEnv));
    if (!e) return NULL;
    if (sb_open(&e->blob, path) != 0) { free(e); return NULL; }
    if (sb_fdm_init(&e->fdm, &e->blob) || sb_conv_init(&e->conv, &e->blob) ||
        sb_occup_init(&e->occ, &e->blob) || sb_sim_init(&e->sim, &e->blob, &e->fdm, &e->conv, &e->occ)) {
        sb_close(&e->blob);
        free(e);
        return NULL;
    }
    e->is_disc = sb_u8(&e->blob, "act_is_discrete");
    e->n_act = e->sim.n_action;
    for (int i = 0; i < e->n_act; i++) {
        if (e->is_disc[i]) e->n_disc++; else e->n_cont++;
    }
    e->obs_len = e->sim.n_dev + e->sim.n_aux;
    if (e->n_cont > SBO_CONT || e->n_disc > SBO_DISC || e->obs_len > SBO_OBS) {
        sbo_destroy(e);
        return NULL;
    }
    if (max_steps <= 0) {
        const SbSection* m = sb_find(&e->blob, "obs_meta");
        if (m && m->count > 3) max_steps = (int)sb_f64(&e->blob, "obs_meta")[3];
        if (max_steps <= 0) {
            const SbSection* o = sb_find(&e->blob, "occ_hour");
            max_steps = (o && o->count > 1) ? (int)o->count - 1 : 8640;
        }
    }
    e->max_steps = max_steps;
    e->cur_len = max_steps;
    /* the priming hour per calendar row, where the blob carries it for random starts */
    e->hour_m1 = sb_i64(&e->blob, "occ_hour_m1");
    e->wd_m1 = sb_u8(&e->blob, "occ_workday_m1");
    {
        const SbSection* h = sb_find(&e->blob, "occ_hour_m1");
        const SbSection* w = sb_find(&e->blob, "occ_workday_m1");
        e->m1_rows = (h && w && e->hour_m1 && e->wd_m1) ? (int)(h->count < w->count ? h->count : w->count) : 0;
    }
    return e;
}

void sbo_set_episode(SboEnv* e, int first_len, unsigned long long start_rng, int random_start) {
    e->cur_len = first_len > 0 ? first_len : e->max_steps;
    e->start_rng = start_rng;
    e->random_start = random_start;
}

int sbo_episode_offset(const SboEnv* e) { return e->off; }

void sbo_destroy(SboEnv* e) {
    if (!e) return;
    sb_sim_free(&e->sim);
    sb_occup_free(&e->occ);
    sb_conv_free(&e->conv);
    sb_fdm_free(&e->fdm);
    sb_close(&e->blob);
    free(e);
}

void sbo_dims(const SboEnv* e, int* out) {
    out[0] = e->sim.n_cvs; out[1] = e->sim.n_solved; out[2] = e->sim.k;
    out[3] = e->sim.n_zones; out[4] = e->sim.n_vav; out[5] = e->sim.n_ahu;
    out[6] = e->n_act; out[7] = e->n_cont; out[8] = e->n_disc; out[9] = e->obs_len;
}

static void write_obs(SboEnv* e, int j, float* obs) {
    sb_obs(&e->sim, e->occ.V, j, obs);
    for (int i = e->obs_len; i < SBO_OBS; i++) obs[i] = 0.0f;
}

void sbo_reset(SboEnv* e, float* obs) {
    e->off = e->random_start ? SBO_DAY_STEPS * sbo_start_draw(&e->start_rng) : 0;
    sb_sim_reset(&e->sim, &e->blob);
    e->sim.step_index = e->off;   /* the calendar row the simulator reads */
    if (e->off < e->m1_rows) {
        e->occ.hour_m1 = (int)e->hour_m1[e->off];
        e->occ.workday_m1 = e->wd_m1[e->off];
    }
    sb_occup_prime(&e->occ);
    e->step = 0;
    for (int i = 0; i < e->n_act; i++) e->native[i] = 0.0;
    write_obs(e, e->off, obs);
    sb_occup_advance(&e->occ, e->off);
}

void sbo_step(SboEnv* e, const float* act, float* obs, float* reward, float* terminal,
              double* reward_f64, double* parts12, double* log8) {
    SbSim* s = &e->sim;
    for (int i = 0; i < e->n_cont; i++) {
        double a = (double)act[i];
        if (a > 1.0) a = 1.0;
        else if (a < -1.0) a = -1.0;
        e->cont[i] = a;
    }
    for (int i = 0; i < e->n_disc; i++) e->disc[i] = (double)act[SBO_CONT + i];
    sb_decode_native(e->n_act, e->is_disc, sb_f64(&e->blob, "act_min_native"),
                     sb_f64(&e->blob, "act_max_native"), sb_f64(&e->blob, "act_min_norm"),
                     sb_f64(&e->blob, "act_max_norm"), e->cont, e->disc, e->native);
    sb_sim_apply_native(s, e->native);
    sb_sim_step(s, e->occ.V);
    e->step += 1;
    const int j = e->off + e->step;   /* calendar row */
    write_obs(e, j, obs);
    sb_occup_advance(&e->occ, j);
    double rew = sb_reward(s, e->occ.V, j, e->parts);
    if (reward) *reward = (float)rew;
    if (reward_f64) *reward_f64 = rew;
    if (parts12) memcpy(parts12, e->parts, sizeof(e->parts));
    if (log8) {
        /* sb_reward leaves the post-step zone means in s->avg_temp */
        const int kv = j;
        const double hsp = s->sched_heat_sp[kv], csp = s->sched_cool_sp[kv];
        double dsum = 0.0, dmax = 0.0;
        int oob = 0;
        for (int z = 0; z < s->n_zones; z++) {
            double dev = s->avg_temp[z] - csp;
            if (hsp - s->avg_temp[z] > dev) dev = hsp - s->avg_temp[z];
            if (dev < 0.0) dev = 0.0;
            dsum += dev;
            if (dev > dmax) dmax = dev;
            if (dev > 0.0) oob++;
        }
        const double elec_rate = e->parts[5] + fabs(e->parts[6]) + e->parts[7];
        log8[0] = e->parts[0];
        log8[1] = e->parts[1];
        log8[2] = e->parts[2];
        log8[3] = s->n_zones > 0 ? dsum / s->n_zones : 0.0;
        log8[4] = dmax;
        log8[5] = s->n_zones > 0 ? (double)oob / s->n_zones : 0.0;
        log8[6] = fabs(elec_rate) * s->dt_sec / 3.6e6;
        log8[7] = NAN;  /* the gas rate is internal to sb_reward */
    }
    const int done = e->step >= e->cur_len;
    if (terminal) *terminal = done ? 1.0f : 0.0f;
    if (done) {
        e->cur_len = e->max_steps;   /* every later episode is whole */
        sbo_reset(e, obs);
    }
}

void sbo_get_temp(const SboEnv* e, double* out) {
    memcpy(out, e->fdm.temp, sizeof(double) * (size_t)e->sim.n_cvs);
}

void sbo_get_mass(const SboEnv* e, double* out) {
    memcpy(out, e->fdm.mass_temp, sizeof(double) * (size_t)e->sim.n_solved);
}

int sbo_step_index(const SboEnv* e) { return e->step; }

void sbo_reseed(SboEnv* e) {
    sb_rng_seed(&e->occ.rng, (uint32_t)sb_i64_1(&e->blob, "occ_seed", 17321));
    sb_rng_seed(&e->conv.rng, e->conv.seed);
}

int sbo_debug(const SboEnv* e, double* out) { (void)e; (void)out; return -1; }
int sbo_visible(const SboEnv* e, double* out) { (void)e; (void)out; return -1; }
