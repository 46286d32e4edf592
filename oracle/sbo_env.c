/* TEST INFRASTRUCTURE: the oracle ABI (sbo.h) over the C restatement.
 * Reset/step order restates the reference CPU env,
 * complete_port/pufferlib_cpu_env.h:187-257. */
#include <stdlib.h>
#include <string.h>

#include "sbo.h"
#include "sbo_internal.h"

struct SboEnv {
    SboScn scn;
    SboState st;
    int cur_len;                 /* this episode's length (desync cuts the first) */
    int off;                     /* this episode's calendar offset */
    int random_start;
    unsigned long long start_rng;
};

SboEnv* sbo_create(const char* path, int max_steps) {
    SboEnv* e = (SboEnv*)calloc(1, sizeof(SboEnv));
    if (!e) return NULL;
    if (sbo_scn_load(&e->scn, path, max_steps) != 0 || e->scn.n_cont > SBO_CONT ||
        e->scn.n_disc > SBO_DISC || e->scn.n_dev + e->scn.n_aux > SBO_OBS) {
        sbo_scn_free(&e->scn);
        free(e);
        return NULL;
    }
    sbo_state_alloc(&e->st, &e->scn);
    e->cur_len = e->scn.max_steps;
    return e;
}

void sbo_set_episode(SboEnv* e, int first_len, unsigned long long start_rng, int random_start) {
    e->cur_len = first_len > 0 ? first_len : e->scn.max_steps;
    e->start_rng = start_rng;
    e->random_start = random_start;
}

int sbo_episode_offset(const SboEnv* e) { return e->off; }

void sbo_destroy(SboEnv* e) {
    if (!e) return;
    sbo_state_free(&e->st);
    sbo_scn_free(&e->scn);
    free(e);
}

void sbo_dims(const SboEnv* e, int* out) {
    const SboScn* s = &e->scn;
    out[0] = s->ncv; out[1] = s->n; out[2] = s->k; out[3] = s->nz; out[4] = s->nv; out[5] = s->na;
    out[6] = s->nact; out[7] = s->n_cont; out[8] = s->n_disc; out[9] = s->n_dev + s->n_aux;
}

static void write_obs(SboEnv* e, int j, float* obs) {
    sbo_observe(&e->st, &e->scn, j, obs);
    for (int i = e->scn.n_dev + e->scn.n_aux; i < SBO_OBS; i++) obs[i] = 0.0f;
}

void sbo_reset(SboEnv* e, float* obs) {
    const SboScn* s = &e->scn;
    e->off = e->random_start ? SBO_DAY_STEPS * sbo_start_draw(&e->start_rng) : 0;
    const int off = e->off;
    sbo_sim_reset(&e->st, s);
    e->st.step_index = off;
    if (off > 0 && off < s->m1_rows)   /* prime [ts_off-1, ts_off) */
        sbo_occ_advance(&e->st, s, (int)s->o_hour_m1[off], (int)s->o_wd_m1[off]);
    else
        sbo_occ_advance(&e->st, s, s->hour_m1, s->wd_m1);
    e->st.step = 0;
    memset(e->st.native, 0, sizeof(e->st.native));
    write_obs(e, off, obs);
    sbo_occ_advance(&e->st, s, (int)s->o_hour[off], (int)s->o_wd[off]);
}

void sbo_step(SboEnv* e, const float* act, float* obs, float* reward, float* terminal,
              double* reward_f64, double* parts12, double* log8) {
    SboScn* s = &e->scn;
    SboState* st = &e->st;
    sbo_decode(s, act, st->native);
    sbo_apply_native(st, s, st->native);
    sbo_sim_step(st, s);
    st->step += 1;
    const int j = e->off + st->step;   /* calendar row */
    write_obs(e, j, obs);
    sbo_occ_advance(st, s, (int)s->o_hour[j], (int)s->o_wd[j]);
    const double rew = sbo_reward(st, s, j, parts12, log8);
    if (reward) *reward = (float)rew;
    if (reward_f64) *reward_f64 = rew;
    const int done = st->step >= e->cur_len;
    if (terminal) *terminal = done ? 1.0f : 0.0f;
    if (done) {
        e->cur_len = s->max_steps;   /* every later episode is whole */
        sbo_reset(e, obs);
    }
}

void sbo_get_temp(const SboEnv* e, double* out) {
    memcpy(out, e->st.temp, sizeof(double) * (size_t)e->scn.ncv);
}

void sbo_get_mass(const SboEnv* e, double* out) {
    memcpy(out, e->st.mass, sizeof(double) * (size_t)e->scn.n);
}

int sbo_step_index(const SboEnv* e) { return e->st.step; }

void sbo_reseed(SboEnv* e) {
    sbo_mt_seed(&e->st.orng, e->scn.occ_seed);
    sbo_mt_seed(&e->st.crng, e->scn.conv_seed);
}

int sbo_debug(const SboEnv* e, double* out) {
    const SboScn* s = &e->scn;
    const SboState* st = &e->st;
    int o = 0;
    for (int i = 0; i < s->k; i++) out[o++] = st->ag[i];
    for (int i = 0; i < s->k; i++) out[o++] = st->aT[i];
    for (int z = 0; z < s->nz; z++) out[o++] = st->qpre[z];
    out[o++] = st->ff_sum; out[o++] = st->reheat_w; out[o++] = st->b_cur; out[o++] = st->b_ret;
    out[o++] = st->pump_head;
    return o;
}

/* One env's visible state after the last step, in the layout of the library's
 * snapshot staging: field [ncv] in cell order, zone means, occupancy, zone flow
 * setpoint and flow [nz each], VAV heating / cooling setpoints, damper, reheat
 * [nv each], AHU supply temperature, flow, run [na each], native actions [nact],
 * then step, boiler setpoint, boiler return. Returns the number of doubles. */
int sbo_visible(const SboEnv* e, double* out) {
    const SboScn* s = &e->scn;
    const SboState* st = &e->st;
    int o = 0;
    for (int c = 0; c < s->ncv; c++) out[o++] = st->temp[c];
    for (int z = 0; z < s->nz; z++) out[o++] = st->zavg[z];
    for (int z = 0; z < s->nz; z++) out[o++] = st->V[z];
    for (int z = 0; z < s->nz; z++) out[o++] = st->zfsp[z];
    for (int z = 0; z < s->nz; z++) out[o++] = st->zfact[z];
    for (int v = 0; v < s->nv; v++) out[o++] = st->v_hsp[v];
    for (int v = 0; v < s->nv; v++) out[o++] = st->v_csp[v];
    for (int v = 0; v < s->nv; v++) out[o++] = st->v_damp[v];
    for (int v = 0; v < s->nv; v++) out[o++] = st->v_reh[v];
    for (int a = 0; a < s->na; a++) out[o++] = st->ahu_sat[a];
    for (int a = 0; a < s->na; a++) out[o++] = st->ahu_flow[a];
    for (int a = 0; a < s->na; a++) out[o++] = (double)st->ahu_run[a];
    for (int i = 0; i < s->nact; i++) out[o++] = st->native[i];
    out[o++] = (double)e->st.step;
    out[o++] = st->b_sp;
    out[o++] = st->b_ret;
    return o;
}
