/* TEST INFRASTRUCTURE: C restatement of the reference CPU simulator
 * (complete_port/csim). Each function cites the reference lines whose
 * arithmetic it repeats; the order of every floating-point operation is kept
 * so results are bit-identical (no FMA: built with -ffp-contract=off). */
#include "sbo_internal.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define RHO_AIR 1.2
#define CP_AIR 1006.0
#define RHO_W 1000.0
#define CP_W 4180.0
#define GRAV 9.8
#define PA_PER_BAR 100000.0
enum { M_OFF = 0, M_HEAT = 1, M_COOL = 2, M_PASSIVE = 3 };

#define GETF(name) ((const double*)sbo_blob_get(&s->blob, name, 0))
#define GETL(name) ((const int64_t*)sbo_blob_get(&s->blob, name, 2))
#define GETI(name) ((const int32_t*)sbo_blob_get(&s->blob, name, 3))
#define GETB(name) ((const uint8_t*)sbo_blob_get(&s->blob, name, 5))

static double clampd(double v, double lo, double hi) { return v < lo ? lo : (v > hi ? hi : v); }
static int cnt(const SboScn* s, const char* name) {
    const SboSec* x = sbo_blob_find(&s->blob, name);
    return x ? (int)x->count : 0;
}

/* x = A^-1 b by replay of the stored L/U (complete_port/csim/sb_lu.c:38-63):
 * w = b[inv(perm_r)], unit-L column push, U column push with divide, x = w[perm_c]. */
static void lu_apply(const SboScn* s, const double* b, double* x, double* w) {
    const int n = s->n;
    for (int i = 0; i < n; i++) w[i] = b[s->ir[i]];
    for (int j = 0; j < n; j++) {
        const double yj = w[j];
        for (int q = s->Lp[j]; q < s->Lp[j + 1]; q++)
            if (q != s->Ldg[j]) w[s->Li[q]] -= s->Lx[q] * yj;
    }
    for (int j = n - 1; j >= 0; j--) {
        const double zj = w[j] / s->Ux[s->Udg[j]];
        w[j] = zj;
        for (int q = s->Up[j]; q < s->Up[j + 1]; q++)
            if (q != s->Udg[j]) w[s->Ui[q]] -= s->Ux[q] * zj;
    }
    for (int t = 0; t < n; t++) x[t] = w[s->pc[t]];
}

int sbo_scn_load(SboScn* s, const char* path, int max_steps) {
    memset(s, 0, sizeof(*s));
    if (sbo_blob_open(&s->blob, path) != 0) return -1;
    const int64_t* grid = GETL("grid");
    const int64_t* snshape = GETL("sensed_shape");
    if (!grid) return -1;
    s->nr = (int)grid[0];
    s->nc = (int)grid[1];
    s->ncv = s->nr * s->nc;
    s->n = cnt(s, "solved");
    s->k = snshape ? (int)snshape[0] : 0;
    s->solved = GETL("solved");
    s->cap = GETF("capacitance_rate");
    s->dir = GETF("dirichlet_conductance");
    s->mc = GETF("mass_coupling");
    s->mret = GETF("mass_retained");
    s->mgain = GETF("mass_gained");
    s->horiz = GETF("horizontal");
    s->vert = GETF("vertical");
    s->cond = GETF("solver_conductivity");
    s->af0 = GETF("ambient_face_areas_0");
    s->af1 = GETF("ambient_face_areas_1");
    s->temp_init = GETF("temp_init");
    s->mass_init = GETF("mass_temp_init");
    s->Lp = GETI("lu_L_indptr"); s->Li = GETI("lu_L_indices"); s->Lx = GETF("lu_L_data");
    s->Up = GETI("lu_U_indptr"); s->Ui = GETI("lu_U_indices"); s->Ux = GETF("lu_U_data");
    const int32_t* pr = GETI("lu_perm_r");
    const int32_t* pcc = GETI("lu_perm_c");
    if (!s->solved || !s->Lp || !s->Up || !pr || !pcc || !s->temp_init || !s->mass_init) return -1;
    const int n = s->n, k = s->k;
    /* diagonal positions and permutations (sb_lu.c:5-34) */
    s->Ldg = (int*)malloc(sizeof(int) * n);
    s->Udg = (int*)malloc(sizeof(int) * n);
    s->ir = (int*)malloc(sizeof(int) * n);
    s->pc = (int*)malloc(sizeof(int) * n);
    for (int j = 0; j < n; j++) {
        s->Ldg[j] = s->Udg[j] = -1;
        for (int q = s->Lp[j]; q < s->Lp[j + 1]; q++) if (s->Li[q] == j) { s->Ldg[j] = q; break; }
        for (int q = s->Up[j]; q < s->Up[j + 1]; q++) if (s->Ui[q] == j) { s->Udg[j] = q; break; }
        if (s->Ldg[j] < 0 || s->Udg[j] < 0) return -1;
    }
    for (int i = 0; i < n; i++) s->ir[pr[i]] = i;
    for (int j = 0; j < n; j++) s->pc[j] = pcc[j];

    s->ap_p = GETI("applied_indptr"); s->ap_i = GETI("applied_indices"); s->ap_x = GETF("applied_data");
    s->sn_p = GETI("sensed_indptr"); s->sn_i = GETI("sensed_indices"); s->sn_x = GETF("sensed_data");
    s->as_p = GETI("air_side_sensed_indptr"); s->as_i = GETI("air_side_sensed_indices");
    s->as_x = GETF("air_side_sensed_data");
    if (!s->ap_p || !s->sn_p || !s->as_p) return -1;

    /* S = sensed A^-1 applied, one column per coupled VAV (sb_fdm.c:103-114) */
    s->S = (double*)malloc(sizeof(double) * (size_t)(k ? k * k : 1));
    {
        double* r = (double*)malloc(sizeof(double) * n);
        double* yr = (double*)malloc(sizeof(double) * n);
        double* w = (double*)malloc(sizeof(double) * n);
        for (int j = 0; j < k; j++) {
            for (int t = 0; t < n; t++) r[t] = 0.0;
            for (int q = s->ap_p[j]; q < s->ap_p[j + 1]; q++) r[s->ap_i[q]] = s->ap_x[q];
            lu_apply(s, r, yr, w);
            for (int i = 0; i < k; i++) {
                double acc = 0.0;
                for (int q = s->sn_p[i]; q < s->sn_p[i + 1]; q++) acc += s->sn_x[q] * yr[s->sn_i[q]];
                s->S[i * k + j] = acc;
            }
        }
        free(r); free(yr); free(w);
    }

    /* simulator tables and scalar defaults (sb_sim.c:23-97) */
    s->na = cnt(s, "ahu_const") / 9;
    s->nv = cnt(s, "vav_zone_offsets") - 1;
    s->nz = cnt(s, "zone_area");
    s->nact = cnt(s, "act_owner_kind");
    s->vz_off = GETI("vav_zone_offsets"); s->vz_idx = GETI("vav_zone_idx"); s->v_ahu = GETI("vav_ahu_idx");
    s->coupled = GETI("coupled_vav_idx"); s->proom = GETI("phys_room_idx");
    s->room_off = GETI("room_offsets"); s->room_cells = GETI("room_cells");
    s->zarea = GETF("zone_area"); s->ahu_c = GETF("ahu_const"); s->vav_c = GETF("vav_const");
    s->a_kind = GETB("act_owner_kind"); s->a_idx = GETI("act_owner_index"); s->a_act = GETB("act_actuator");
    s->a_disc = GETB("act_is_discrete");
    s->a_mn = GETF("act_min_native"); s->a_mx = GETF("act_max_native");
    s->a_mnr = GETF("act_min_norm"); s->a_mxr = GETF("act_max_norm");
    s->s_comf = GETF("sched_comfort"); s->s_heat = GETF("sched_heat_sp"); s->s_cool = GETF("sched_cool_sp");
    s->amb = GETF("weather_ambient");
    s->internal_w = sbo_blob_f64_1(&s->blob, "internal_gain_w_per_m2", 0.0);
    s->standby = sbo_blob_f64_1(&s->blob, "internal_gain_standby_fraction", 1.0);
    s->occ_w = sbo_blob_f64_1(&s->blob, "occupant_sensible_heat_w", 0.0);
    s->h = sbo_blob_f64_1(&s->blob, "convection_coefficient", 8.8);
    {
        const double* op = GETF("occ_params");
        s->dt = op ? op[5] : 300.0;
        const double cvm = sbo_blob_f64_1(&s->blob, "cv_size_cm", 20.0) / 100.0;
        s->cv_area = cvm * cvm;
        if (!op) return -1;
        s->assign = (int)op[0];
        s->ea = (int)op[1]; s->la = (int)op[2]; s->ed = (int)op[3]; s->ld = (int)op[4];
        /* p = 1 / ((end - start) * 3600 / step / 2)  (sb_occup.c:14-16) */
        s->p_arr = 1.0 / ((s->la - s->ea) * 3600.0 / op[5] / 2.0);
        s->p_dep = 1.0 / ((s->ld - s->ed) * 3600.0 / op[5] / 2.0);
    }
    s->header_res = sbo_blob_f64_1(&s->blob, "hws_header_resistance", 0.0);
    s->is_boiler = (int)sbo_blob_f64_1(&s->blob, "hws_is_boiler", 1.0);
    {
        const double* bc = GETF("boiler_const");
        for (int i = 0; i < 10; i++) s->boiler[i] = bc ? bc[i] : 0.0;
        const double* pcst = GETF("pump_const");
        s->pump_head0 = pcst ? pcst[0] : 0.0;
        s->pump_eff = pcst ? pcst[1] : 1.0;
    }
    s->zv_off = GETI("zone_vav_offsets"); s->zv_idx = GETI("zone_vav_idx");
    s->r_hour = GETL("rew_hour"); s->r_month = GETL("rew_month"); s->r_wd = GETB("rew_workday");
    s->f_kind = GETB("f_dev_kind"); s->f_idx = GETI("f_dev_idx"); s->f_id = GETB("f_obs_id");
    s->f_mean = GETF("f_norm_mean"); s->f_var = GETF("f_norm_var"); s->aux = GETF("aux_time");
    s->n_dev = (int)sbo_blob_i64_1(&s->blob, "n_dev", 0);
    s->n_aux = (int)sbo_blob_i64_1(&s->blob, "n_aux", 0);
    s->rw = GETF("reward_scalars");
    s->e_wd = GETF("elec_weekday_price"); s->e_we = GETF("elec_weekend_price");
    s->e_c = GETF("elec_carbon_rate"); s->g_p = GETF("gas_month_price");
    s->g_c = sbo_blob_f64_1(&s->blob, "gas_carbon_rate", 0.0);
    s->o_hour = GETL("occ_hour");
    s->o_wd = GETB("occ_workday");
    s->hour_m1 = (int)sbo_blob_i64_1(&s->blob, "occ_hour_m1", 0);
    {
        const uint8_t* wm = GETB("occ_workday_m1");
        s->wd_m1 = wm ? wm[0] : 0;
    }
    s->o_hour_m1 = GETL("occ_hour_m1");
    s->o_wd_m1 = GETB("occ_workday_m1");
    s->m1_rows = (s->o_hour_m1 && s->o_wd_m1) ? cnt(s, "occ_hour_m1") : 0;
    if (s->o_wd_m1 && cnt(s, "occ_workday_m1") < s->m1_rows) s->m1_rows = cnt(s, "occ_workday_m1");
    s->occ_seed = (uint32_t)sbo_blob_i64_1(&s->blob, "occ_seed", 17321);
    /* convection (sb_convect.c:6-30) */
    s->conv_p = sbo_blob_f64_1(&s->blob, "conv_p", 0.0);
    s->conv_dist = (int)sbo_blob_f64_1(&s->blob, "conv_distance", -1.0);
    s->conv_seed = (uint32_t)sbo_blob_i64_1(&s->blob, "conv_seed", 0);
    s->cv_off = GETI("conv_room_offsets"); s->cv_cells = GETI("conv_room_cells");
    s->cand_off = GETI("conv_cand_offsets"); s->cand_idx = GETI("conv_cand_idx");
    if (!s->cv_off || !s->cv_cells || !s->cand_off || !s->cand_idx || !s->o_hour || !s->o_wd) return -1;
    s->conv_nrooms = cnt(s, "conv_room_offsets") - 1;
    for (int r = 0; r < s->conv_nrooms; r++) {
        int m = s->cv_off[r + 1] - s->cv_off[r];
        if (m > s->conv_maxroom) s->conv_maxroom = m;
    }
    for (int i = 0; i < s->nact; i++) {
        if (s->a_disc[i]) s->n_disc++; else s->n_cont++;
    }
    if (max_steps <= 0) {
        const SboSec* m = sbo_blob_find(&s->blob, "obs_meta");
        if (m && m->count > 3) max_steps = (int)GETF("obs_meta")[3];
        if (max_steps <= 0) max_steps = cnt(s, "occ_hour") > 1 ? cnt(s, "occ_hour") - 1 : 8640;
    }
    s->max_steps = max_steps;
    return 0;
}

void sbo_scn_free(SboScn* s) {
    free(s->Ldg); free(s->Udg); free(s->ir); free(s->pc); free(s->S);
    sbo_blob_close(&s->blob);
    memset(s, 0, sizeof(*s));
}

#define DALLOC(p, m) ((p) = (double*)calloc((size_t)((m) > 0 ? (m) : 1), sizeof(double)))
#define IALLOC(p, m) ((p) = (int*)calloc((size_t)((m) > 0 ? (m) : 1), sizeof(int)))

int sbo_state_alloc(SboState* e, const SboScn* s) {
    memset(e, 0, sizeof(*e));
    const int n = s->n, k = s->k, na = s->na, nv = s->nv, nz = s->nz;
    DALLOC(e->temp, s->ncv); DALLOC(e->mass, n); DALLOC(e->inq, s->ncv);
    DALLOC(e->work, n); DALLOC(e->y, n); DALLOC(e->yr, n); DALLOC(e->rhs, n);
    DALLOC(e->pw, k); DALLOC(e->qv, k); DALLOC(e->mat, k * k);
    IALLOC(e->ahu_run, na); IALLOC(e->ahu_creq, na);
    DALLOC(e->ahu_rec, na); DALLOC(e->ahu_sat, na); DALLOC(e->ahu_fan, na); DALLOC(e->ahu_flow, na);
    DALLOC(e->ahu_ws, na); DALLOC(e->ahu_at, na); DALLOC(e->ahu_sv, na); DALLOC(e->demand, na);
    DALLOC(e->v_damp, nv); DALLOC(e->v_reh, nv); DALLOC(e->v_ratio, nv); DALLOC(e->v_hsp, nv);
    DALLOC(e->v_csp, nv); DALLOC(e->v_dcmd, nv); DALLOC(e->v_rcmd, nv); DALLOC(e->v_sense, nv);
    DALLOC(e->v_area, nv);
    IALLOC(e->v_mode, nv); IALLOC(e->v_prev, nv); IALLOC(e->v_dset, nv); IALLOC(e->v_rset, nv);
    DALLOC(e->zavg, nz); DALLOC(e->zq, nz); DALLOC(e->smean, k); DALLOC(e->ag, k); DALLOC(e->aT, k);
    DALLOC(e->coil, k); DALLOC(e->zfsp, nz); DALLOC(e->zfact, nz);
    IALLOC(e->ostate, nz * s->assign); DALLOC(e->V, nz);
    IALLOC(e->cl, s->conv_maxroom); IALLOC(e->cr, s->conv_maxroom);
    DALLOC(e->qpre, nz);
    memcpy(e->temp, s->temp_init, sizeof(double) * (size_t)s->ncv);
    memcpy(e->mass, s->mass_init, sizeof(double) * (size_t)n);
    e->pump_head = s->pump_head0;   /* set once at init, never by reset (sb_sim.c:71-75) */
    sbo_mt_seed(&e->orng, s->occ_seed);
    sbo_mt_seed(&e->crng, s->conv_seed);
    return 0;
}

void sbo_state_free(SboState* e) {
    void* ptrs[] = {e->temp, e->mass, e->inq, e->work, e->y, e->yr, e->rhs, e->pw, e->qv, e->mat,
                    e->ahu_run, e->ahu_creq, e->ahu_rec, e->ahu_sat, e->ahu_fan, e->ahu_flow, e->ahu_ws,
                    e->ahu_at, e->ahu_sv, e->demand, e->v_damp, e->v_reh, e->v_ratio, e->v_hsp, e->v_csp,
                    e->v_dcmd, e->v_rcmd, e->v_sense, e->v_area, e->v_mode, e->v_prev, e->v_dset, e->v_rset,
                    e->zavg, e->zq, e->smean, e->ag, e->aT, e->coil, e->zfsp, e->zfact, e->ostate, e->V,
                    e->cl, e->cr, e->qpre};
    for (size_t i = 0; i < sizeof(ptrs) / sizeof(ptrs[0]); i++) free(ptrs[i]);
    memset(e, 0, sizeof(*e));
}

/* zone means of the field over each physical room's cells, in stored order (sb_sim.c:149-160) */
static void zone_means(SboState* e, const SboScn* s) {
    for (int z = 0; z < s->nz; z++) {
        const int rm = s->proom[z];
        const int a = s->room_off[rm], b = s->room_off[rm + 1];
        double sum = 0.0;
        for (int t = a; t < b; t++) sum += e->temp[s->room_cells[2 * t] * s->nc + s->room_cells[2 * t + 1]];
        e->zavg[z] = sum / (double)(b - a);
    }
}

/* area-weighted VAV sensing temperature (sb_sim.c:163-175) */
static void vav_sense_all(SboState* e, const SboScn* s) {
    for (int v = 0; v < s->nv; v++) {
        double area = 0.0, wt = 0.0;
        for (int t = s->vz_off[v]; t < s->vz_off[v + 1]; t++) {
            const int z = s->vz_idx[t];
            area += s->zarea[z];
            wt += e->zavg[z] * s->zarea[z];
        }
        e->v_area[v] = area;
        e->v_sense[v] = area > 0.0 ? wt / area : 0.0;
    }
}

/* sb_sim.c:177-218 */
void sbo_sim_reset(SboState* e, const SboScn* s) {
    for (int a = 0; a < s->na; a++) {
        const double* c = &s->ahu_c[a * 9];
        e->ahu_run[a] = (int)c[8];
        e->ahu_rec[a] = c[0];
        e->ahu_sat[a] = c[6];
        e->ahu_fan[a] = c[7];
        e->ahu_flow[a] = 0.0;
        e->ahu_creq[a] = 0;
    }
    for (int v = 0; v < s->nv; v++) {
        const double* c = &s->vav_c[v * 9];
        e->v_damp[v] = c[7];
        e->v_reh[v] = c[8];
        e->v_ratio[v] = 1.0;
        e->v_hsp[v] = c[5];
        e->v_csp[v] = c[6];
        e->v_mode[v] = M_OFF;
        e->v_prev[v] = e->v_dset[v] = e->v_rset[v] = 0;
        e->v_dcmd[v] = e->v_rcmd[v] = 0.0;
    }
    e->ff_sum = 0.0;
    e->hws_req = 0;
    e->hws_run = e->pump_run = 1;
    e->b_sp = s->boiler[0];
    e->b_ret = s->boiler[1];
    e->b_cur = s->boiler[0];
    e->b_step = 0.0;
    e->step_index = 0;
    memcpy(e->temp, s->temp_init, sizeof(double) * (size_t)s->ncv);
    memcpy(e->mass, s->mass_init, sizeof(double) * (size_t)s->n);
    memset(e->inq, 0, sizeof(double) * (size_t)s->ncv);
    zone_means(e, s);
    vav_sense_all(e, s);
}

/* clamp (pufferlib_cpu_env.h:218-227) + sb_decode_native (sb_sim.c:557-576) */
void sbo_decode(const SboScn* s, const float* act, double* native) {
    int ci = 0, di = 0;
    for (int i = 0; i < s->nact; i++) {
        if (s->a_disc[i]) {
            const double dv = (double)act[256 + di++];
            const double merged = dv == 1.0 ? 1.0 : -1.0;
            native[i] = (merged - s->a_mnr[i]) / (s->a_mxr[i] - s->a_mnr[i]) * (s->a_mx[i] - s->a_mn[i]) + s->a_mn[i];
        } else {
            double a = (double)act[ci++];
            a = a > 1.0 ? 1.0 : (a < -1.0 ? -1.0 : a);
            const float m = (float)a;
            const float span_in = (float)(s->a_mxr[i] - s->a_mnr[i]);
            const float span_out = (float)(s->a_mx[i] - s->a_mn[i]);
            const float r = (m - (float)s->a_mnr[i]) / span_in * span_out + (float)s->a_mn[i];
            native[i] = (double)r;
        }
    }
}

/* sb_sim.c:220-244 */
void sbo_apply_native(SboState* e, const SboScn* s, const double* native) {
    for (int i = 0; i < s->nact; i++) {
        const double val = native[i];
        const int idx = s->a_idx[i], act = s->a_act[i];
        if (s->a_kind[i] == 0) {
            if (act == 0) e->ahu_sat[idx] = val;
            else if (act == 1) e->ahu_fan[idx] = val;
            else if (act == 2) e->ahu_rec[idx] = clampd(val, 0.0, s->ahu_c[idx * 9 + 3]);
            else e->ahu_run[idx] = val == 1.0 ? 1 : 0;
        } else if (s->a_kind[i] == 1) {
            if (act == 0) { e->v_dcmd[idx] = clampd(val, 0.0, 1.0); e->v_dset[idx] = 1; }
            else { e->v_rcmd[idx] = clampd(val, 0.0, 1.0); e->v_rset[idx] = 1; }
        } else {
            if (act == 0) e->b_sp = val;
            else if (act == 1) e->pump_head = val / (GRAV * RHO_W / PA_PER_BAR);
            else { const int on = val == 1.0 ? 1 : 0; e->hws_run = on; e->pump_run = on; }
        }
    }
}

/* device formulas (sb_sim.c:246-314) */
static double ahu_static_p(const SboState* e, const SboScn* s, int a) {
    if (e->ahu_run[a] != 1) return 0.0;
    const double sp = e->ahu_fan[a], mn = s->ahu_c[a * 9 + 2];
    return sp > mn ? sp : mn;
}
static double vav_unrestr(const SboState* e, const SboScn* s, int v) {
    const double* c = &s->vav_c[v * 9];
    const double d = e->v_damp[v] * c[0] * sqrt(ahu_static_p(e, s, s->v_ahu[v]) / c[4]);
    return d > 0.00001 ? d : 0.00001;
}
static double vav_demand(const SboState* e, const SboScn* s, int v) { return vav_unrestr(e, s, v) * e->v_ratio[v]; }
static double pump_dp(const SboState* e) { return e->pump_run != 1 ? 0.0 : GRAV * RHO_W * e->pump_head / PA_PER_BAR; }
static double water_flow(const SboState* e, const SboScn* s) {
    const double ff = e->ff_sum;
    return ff * sqrt(pump_dp(e) / (1.0 + ff * ff * s->header_res)) / 3600.0;
}
static double reheat_w(const SboState* e, const SboScn* s, int v, double sat, double iwt) {
    const double air_cap = CP_AIR * RHO_AIR * vav_demand(e, s, v);
    double eff;
    if (air_cap <= 0.0) {
        eff = 0.0;
    } else {
        double wf = 0.0;
        if (e->ff_sum != 0.0) wf = water_flow(e, s) * (e->v_reh[v] * s->vav_c[v * 9 + 1] / e->ff_sum);
        eff = CP_W * RHO_W * wf / air_cap;
        if (eff > 1.0) eff = 1.0;
        if (iwt - sat > 0.0) {
            const double head = s->vav_c[v * 9 + 3] - sat;
            if (head <= 0.0) eff = 0.0;
            else {
                const double hr = head / (iwt - sat);
                eff = eff < hr ? eff : hr;
            }
        }
    }
    return eff * CP_AIR * RHO_AIR * vav_demand(e, s, v) * (iwt - sat);
}

/* thermostat with hysteresis (sb_sim.c:316-339) */
static void mode_default(SboState* e, int v, double zt, double hsp, double csp) {
    const double mid = 0.5 * (csp - hsp) + hsp;
    if (zt < hsp) e->v_mode[v] = M_HEAT;
    else if (zt > csp) e->v_mode[v] = M_COOL;
    else if (zt < mid && e->v_mode[v] == M_HEAT) e->v_mode[v] = M_HEAT;
    else if (zt > mid && e->v_mode[v] == M_COOL) e->v_mode[v] = M_COOL;
    else e->v_mode[v] = M_OFF;
}
static int mode_update(SboState* e, const SboScn* s, int v, double zt, int kk, int comfort) {
    const double hsp = s->s_heat[kk], csp = s->s_cool[kk];
    if (comfort) mode_default(e, v, zt, hsp, csp);
    else if (e->v_prev[v] && s->s_comf[kk - 1] != 0.0) e->v_mode[v] = M_PASSIVE;
    else if (e->v_mode[v] == M_PASSIVE && zt > hsp && zt < csp) e->v_mode[v] = M_PASSIVE;
    else mode_default(e, v, zt, hsp, csp);
    e->v_prev[v] = 1;
    return e->v_mode[v];
}

/* sb_sim_step_pre (sb_sim.c:341-457) */
static void step_pre(SboState* e, const SboScn* s) {
    const int kk = e->step_index;
    const double ambient = s->amb[kk];
    const int comfort = s->s_comf[kk] != 0.0;
    e->hws_req = s->nv;
    zone_means(e, s);
    for (int a = 0; a < s->na; a++) { e->ahu_ws[a] = 0.0; e->ahu_at[a] = 0.0; }
    for (int v = 0; v < s->nv; v++) {
        double area = 0.0, wt = 0.0;
        for (int t = s->vz_off[v]; t < s->vz_off[v + 1]; t++) {
            const int z = s->vz_idx[t];
            area += s->zarea[z];
            wt += e->zavg[z] * s->zarea[z];
        }
        e->v_area[v] = area;
        if (area <= 0.0) { e->v_sense[v] = 0.0; continue; }
        const double sensing = wt / area;
        e->v_sense[v] = sensing;
        /* vav_update_settings (sb_sim.c:341-355) */
        const double* c = &s->vav_c[v * 9];
        e->v_hsp[v] = s->s_heat[kk];
        e->v_csp[v] = s->s_cool[kk];
        const int mode = mode_update(e, s, v, sensing, kk, comfort);
        double damper, reheat;
        if (mode == M_HEAT) { damper = 1.0; reheat = 1.0; }
        else if (mode == M_COOL) { damper = 1.0; reheat = 0.0; }
        else { damper = c[2]; reheat = 0.0; }
        if (e->v_dset[v]) damper = e->v_dcmd[v];
        if (e->v_rset[v]) reheat = e->v_rcmd[v];
        e->v_damp[v] = damper > c[2] ? damper : c[2];
        e->v_reh[v] = reheat;
        const int a = s->v_ahu[v];
        e->ahu_ws[a] += sensing * area;
        e->ahu_at[a] += area;
    }
    for (int a = 0; a < s->na; a++) {
        double recirc;
        if (e->ahu_at[a] > 0.0) recirc = e->ahu_ws[a] / e->ahu_at[a];
        else {
            double mean = 0.0;
            for (int p = 0; p < s->ncv; p++) mean += e->temp[p];
            recirc = mean / (double)s->ncv;
        }
        const double mixed = e->ahu_rec[a] * recirc + (1.0 - e->ahu_rec[a]) * ambient;
        e->ahu_sv[a] = (mixed > e->ahu_sat[a] && e->ahu_run[a] == 1) ? e->ahu_sat[a] : mixed;
    }
    for (int a = 0; a < s->na; a++) { e->ahu_flow[a] = 0.0; e->ahu_creq[a] = 0; }
    e->ff_sum = 0.0;
    for (int v = 0; v < s->nv; v++) e->ff_sum += e->v_reh[v] * s->vav_c[v * 9 + 1];
    for (int a = 0; a < s->na; a++) e->demand[a] = 0.0;
    for (int v = 0; v < s->nv; v++) e->demand[s->v_ahu[v]] += vav_unrestr(e, s, v);
    for (int v = 0; v < s->nv; v++) {
        const int a = s->v_ahu[v];
        const double d = e->demand[a];
        if (d > 0.0) {
            const double r = s->ahu_c[a * 9 + 1] / d;
            e->v_ratio[v] = r < 1.0 ? r : 1.0;
        } else {
            e->v_ratio[v] = 1.0;
        }
    }
    for (int z = 0; z < s->nz; z++) e->zq[z] = 0.0;
    e->reheat_w = 0.0;
    for (int col = 0; col < s->k; col++) {
        const int v = s->coupled[col];
        if (e->v_area[v] <= 0.0) { e->ag[col] = 0.0; e->aT[col] = 0.0; continue; }
        const int a = s->v_ahu[v];
        const double sat = e->ahu_sv[a];
        e->aT[col] = sat;
        const double rw = reheat_w(e, s, v, sat, e->b_cur);
        e->reheat_w += rw;
        e->coil[col] = sat;
        const double fd = vav_demand(e, s, v);
        if (e->v_damp[v] > 0.0 && s->vav_c[v * 9] > 0.0) {
            e->ag[col] = fd * RHO_AIR * CP_AIR;
            for (int t = s->vz_off[v]; t < s->vz_off[v + 1]; t++) {
                const int z = s->vz_idx[t];
                e->zq[z] += rw * s->zarea[z] / e->v_area[v];
            }
        } else {
            e->ag[col] = 0.0;
        }
        if (fd > 0.0) {
            e->ahu_flow[a] += fd;
            const double mf = s->ahu_c[a * 9 + 1];
            if (e->ahu_flow[a] > mf) e->ahu_flow[a] = mf;
            e->ahu_creq[a] += 1;
        }
    }
    if (s->internal_w > 0.0) {
        const double frac = comfort ? 1.0 : s->standby;
        const double wpc = s->internal_w * s->cv_area * frac;
        for (int z = 0; z < s->nz; z++) {
            const int rm = s->proom[z];
            e->zq[z] += wpc * (double)(s->room_off[rm + 1] - s->room_off[rm]);
        }
    }
    if (s->occ_w > 0.0)
        for (int z = 0; z < s->nz; z++) e->zq[z] += e->V[z] * s->occ_w;
    for (int z = 0; z < s->nz; z++) {
        const int rm = s->proom[z];
        const int a = s->room_off[rm], b = s->room_off[rm + 1];
        const double q = e->zq[z] / (double)(b - a);
        e->qpre[z] = q;
        for (int t = a; t < b; t++) e->inq[s->room_cells[2 * t] * s->nc + s->room_cells[2 * t + 1]] = q;
    }
}

/* partial-pivot Gaussian elimination on a row-major k x k system (sb_fdm.c:9-38) */
static void gauss_solve(int k, double* M, double* b) {
    for (int c = 0; c < k; c++) {
        int piv = c;
        double best = fabs(M[c * k + c]);
        for (int r = c + 1; r < k; r++) {
            const double v = fabs(M[r * k + c]);
            if (v > best) { best = v; piv = r; }
        }
        if (best == 0.0) return;
        if (piv != c) {
            for (int j = c; j < k; j++) { double t = M[c * k + j]; M[c * k + j] = M[piv * k + j]; M[piv * k + j] = t; }
            double t = b[c]; b[c] = b[piv]; b[piv] = t;
        }
        const double d = M[c * k + c];
        for (int r = c + 1; r < k; r++) {
            const double f = M[r * k + c] / d;
            if (f == 0.0) continue;
            for (int j = c; j < k; j++) M[r * k + j] -= f * M[c * k + j];
            b[r] -= f * b[c];
        }
    }
    for (int r = k - 1; r >= 0; r--) {
        double acc = b[r];
        for (int j = r + 1; j < k; j++) acc -= M[r * k + j] * b[j];
        b[r] = acc / M[r * k + r];
    }
}

/* sb_fdm_step (sb_fdm.c:126-188) */
static void fdm_step(SboState* e, const SboScn* s, double ambient) {
    const int n = s->n, k = s->k;
    for (int t = 0; t < n; t++) {
        const int64_t p = s->solved[t];
        double ex = 0.0;
        if (s->af0[p] > 0.0) ex += s->h * s->af0[p] / (1.0 + s->h * 0.5 * s->horiz[p] / s->cond[p]);
        if (s->af1[p] > 0.0) ex += s->h * s->af1[p] / (1.0 + s->h * 0.5 * s->vert[p] / s->cond[p]);
        e->rhs[t] = s->cap[t] * e->temp[p] + e->inq[p] + ambient * (s->dir[t] + ex) + s->mc[t] * e->mass[t];
    }
    lu_apply(s, e->rhs, e->y, e->work);
    int active = 0;
    for (int i = 0; i < k; i++) if (e->ag[i] != 0.0) { active = 1; break; }
    if (k > 0 && active) {
        for (int i = 0; i < k; i++) {
            double acc = 0.0;
            for (int q = s->sn_p[i]; q < s->sn_p[i + 1]; q++) acc += s->sn_x[q] * e->y[s->sn_i[q]];
            e->pw[i] = e->ag[i] * (e->aT[i] - acc);
        }
        for (int i = 0; i < k; i++)
            for (int j = 0; j < k; j++) e->mat[i * k + j] = (i == j ? 1.0 : 0.0) + e->ag[i] * s->S[i * k + j];
        gauss_solve(k, e->mat, e->pw);
        for (int t = 0; t < n; t++) e->rhs[t] = 0.0;
        for (int j = 0; j < k; j++) {
            const double qj = e->pw[j];
            if (qj == 0.0) continue;
            for (int q = s->ap_p[j]; q < s->ap_p[j + 1]; q++) e->rhs[s->ap_i[q]] += s->ap_x[q] * qj;
        }
        lu_apply(s, e->rhs, e->yr, e->work);
        for (int t = 0; t < n; t++) e->y[t] += e->yr[t];
    }
    for (int t = 0; t < n; t++) e->mass[t] = e->mass[t] * s->mret[t] + s->mgain[t] * e->y[t];
    for (int p = 0; p < s->ncv; p++) e->temp[p] = ambient;
    for (int t = 0; t < n; t++) e->temp[s->solved[t]] = e->y[t];
}

/* stochastic convection swaps (sb_convect.c:39-73) */
static void convect(SboState* e, const SboScn* s) {
    if (s->conv_p == 0.0 || s->conv_dist == 0) return;
    for (int rm = 0; rm < s->conv_nrooms; rm++) {
        const int base = s->cv_off[rm], cells = s->cv_off[rm + 1] - base;
        if (cells <= 0) continue;
        int m = 0;
        for (int j = 0; j < cells; j++) {
            if (sbo_mt_sample(&e->crng) > s->conv_p) continue;
            const int g = base + j;
            const int c0 = s->cand_off[g], c1 = s->cand_off[g + 1];
            if (c1 <= c0) continue;
            e->cl[m] = g;
            e->cr[m] = s->cand_idx[c0 + (int)sbo_mt_bounded(&e->crng, (uint32_t)(c1 - c0 - 1))];
            m++;
        }
        for (int t = m - 1; t > 0; t--) {
            const int u = (int)sbo_mt_bounded(&e->crng, (uint32_t)t);
            int x = e->cl[t]; e->cl[t] = e->cl[u]; e->cl[u] = x;
            x = e->cr[t]; e->cr[t] = e->cr[u]; e->cr[u] = x;
        }
        for (int t = 0; t < m; t++) {
            const int ia = s->cv_cells[2 * e->cl[t]] * s->nc + s->cv_cells[2 * e->cl[t] + 1];
            const int ib = s->cv_cells[2 * e->cr[t]] * s->nc + s->cv_cells[2 * e->cr[t] + 1];
            const double held = e->temp[ia];
            e->temp[ia] = e->temp[ib];
            e->temp[ib] = held;
        }
    }
}

/* sb_sim_step_post (sb_sim.c:459-521) */
static void step_post(SboState* e, const SboScn* s) {
    if (s->k > 0) {
        /* sensed means + post-step applied heat: kept for fidelity although
         * nothing observable reads them before the next step rewrites them */
        for (int c = 0; c < s->k; c++) e->smean[c] = 0.0;
        for (int p = 0; p < s->ncv; p++) {
            const double tp = e->temp[p];
            if (tp == 0.0) continue;
            for (int q = s->as_p[p]; q < s->as_p[p + 1]; q++) e->smean[s->as_i[q]] += s->as_x[q] * tp;
        }
        for (int col = 0; col < s->k; col++) {
            const int v = s->coupled[col];
            if (e->v_area[v] <= 0.0) continue;
            const double q = e->ag[col] * (e->aT[col] - e->smean[col]);
            for (int t = s->vz_off[v]; t < s->vz_off[v + 1]; t++) {
                const int z = s->vz_idx[t];
                e->zq[z] += q * s->zarea[z] / e->v_area[v];
            }
        }
        for (int z = 0; z < s->nz; z++) {
            const int rm = s->proom[z];
            const int a = s->room_off[rm], b = s->room_off[rm + 1];
            const double q = e->zq[z] / (double)(b - a);
            for (int t = a; t < b; t++) e->inq[s->room_cells[2 * t] * s->nc + s->room_cells[2 * t + 1]] = q;
        }
    }
    convect(e, s);
    const double wcap = CP_W * RHO_W * water_flow(e, s);
    if (wcap > 0.0 && s->k > 0) {
        const double supply = e->b_cur;
        double rt = supply - e->reheat_w / wcap;
        double at = e->coil[0];
        for (int c = 1; c < s->k; c++) {
            if (e->reheat_w >= 0.0) { if (e->coil[c] < at) at = e->coil[c]; }
            else { if (e->coil[c] > at) at = e->coil[c]; }
        }
        const double lo = supply < at ? supply : at, hi = supply > at ? supply : at;
        if (rt < lo) rt = lo;
        if (rt > hi) rt = hi;
        e->b_ret = rt;
    }
    const double begin = e->b_cur, sp = e->b_sp, dtm = s->dt / 60.0;
    if (sp > begin) {
        const double v = begin + s->boiler[2] * dtm;
        e->b_cur = v < sp ? v : sp;
    } else if (sp < begin) {
        const double v = begin - s->boiler[3] * dtm;
        e->b_cur = v > sp ? v : sp;
    } else {
        e->b_cur = sp;
    }
    e->b_step = e->b_cur - begin;
    e->step_index += 1;
}

/* sb_sim_step (sb_sim.c:526-531) */
void sbo_sim_step(SboState* e, const SboScn* s) {
    step_pre(e, s);
    fdm_step(e, s, s->amb[e->step_index]);
    step_post(e, s);
}

/* sb_obs (sb_obs.c:11-64) */
static double obs_field(const SboState* e, const SboScn* s, int kind, int idx, int id, int j) {
    if (kind == 0) {
        switch (id) {
            case 0: return (double)e->ahu_creq[idx];
            case 1: return ahu_static_p(e, s, idx);
            case 2: return e->ahu_run[idx] == 1 ? e->ahu_flow[idx] : 0.0;
            case 3: return e->ahu_sat[idx];
            case 4: return (double)e->ahu_run[idx];
            case 5: return e->ahu_flow[idx] / s->ahu_c[idx * 9 + 1];
            case 6: return (1.0 - e->ahu_rec[idx]) * e->ahu_flow[idx];
            case 7: return (double)e->ahu_run[idx];
            case 8: return e->ahu_rec[idx];
            default: return s->amb[j];
        }
    }
    if (kind == 1) {
        switch (id) {
            case 0: return e->v_reh[idx];
            case 1: return e->v_damp[idx];
            case 2: return s->vav_c[idx * 9];
            case 3: return e->v_csp[idx];
            case 4: return e->v_hsp[idx];
            default: return e->v_sense[idx];
        }
    }
    switch (id) {
        case 0: case 2: return pump_dp(e);
        case 1: return e->b_cur;
        case 3: case 5: return (double)e->hws_run;
        case 4: return (double)e->hws_req;
        default: return e->b_sp;
    }
}

void sbo_observe(SboState* e, const SboScn* s, int j, float* out) {
    for (int i = 0; i < s->n_dev; i++) {
        const double v = obs_field(e, s, s->f_kind[i], s->f_idx[i], s->f_id[i], j);
        const double var = s->f_var[i];
        const float v32 = (float)v;
        out[i] = (float)(var > 0.0 ? ((double)v32 - s->f_mean[i]) / sqrt(var) : 0.0);
    }
    const double* aux = &s->aux[(size_t)j * (s->n_aux - 1)];
    for (int q = 0; q < s->n_aux - 1; q++) out[s->n_dev + q] = (float)aux[q];
    double occ = 0.0;
    for (int z = 0; z < s->nz; z++) occ += e->V[z];
    out[s->n_dev + s->n_aux - 1] = (float)(int)occ;
}

/* RandomizedArrivalDepartureOccupancy chains (sb_occup.c:39-71) */
void sbo_occ_advance(SboState* e, const SboScn* s, int hour, int workday) {
    for (int z = 0; z < s->nz; z++) {
        int count = 0;
        int* st = &e->ostate[(size_t)z * s->assign];
        for (int a = 0; a < s->assign; a++) {
            if (!workday) st[a] = 0;
            else if (st[a] == 0) {
                if (hour >= s->ea && hour <= s->la && sbo_mt_sample(&e->orng) < s->p_arr) st[a] = 1;
            } else if (hour < s->ed) {
                /* stays at work */
            } else if (hour >= s->ld) {
                st[a] = 0;
            } else if (sbo_mt_sample(&e->orng) < s->p_dep) {
                st[a] = 0;
            }
            if (st[a]) count++;
        }
        e->V[z] = (double)count;
    }
}

/* sb_reward (sb_reward.c:12-155) plus the per-step log terms */
double sbo_reward(SboState* e, const SboScn* s, int kv, double* parts12, double* log8) {
    const int nz = s->nz;
    const double dt = s->dt, inv_hour = 1.0 / 3600.0;
    zone_means(e, s);
    for (int z = 0; z < nz; z++) {
        double fsp = 0.0, fact = 0.0;
        for (int t = s->zv_off[z]; t < s->zv_off[z + 1]; t++) {
            const int v = s->zv_idx[t];
            const double va = e->v_area[v];
            if (va <= 0.0) continue;
            const double share = s->zarea[z] / va;
            fsp += s->vav_c[v * 9] * share;
            fact += vav_demand(e, s, v) * share;
        }
        e->zfsp[z] = fsp;
        e->zfact[z] = fact;
    }
    const double ambient = s->amb[kv];
    const int hour = (int)s->r_hour[kv], month = (int)s->r_month[kv], wd = (int)s->r_wd[kv];
    double cooling = 0.0, intake = 0.0, exhaust = 0.0;
    for (int a = 0; a < s->na; a++) { e->ahu_ws[a] = 0.0; e->ahu_at[a] = 0.0; }
    for (int v = 0; v < s->nv; v++) {
        double area = 0.0, wt = 0.0;
        for (int t = s->vz_off[v]; t < s->vz_off[v + 1]; t++) {
            const int z = s->vz_idx[t];
            area += s->zarea[z];
            wt += e->zavg[z] * s->zarea[z];
        }
        if (area > 0.0) {
            const int a = s->v_ahu[v];
            e->ahu_ws[a] += (wt / area) * area;
            e->ahu_at[a] += area;
        }
    }
    double tmean = 0.0;
    for (int p = 0; p < s->ncv; p++) tmean += e->temp[p];
    tmean /= (double)s->ncv;
    for (int a = 0; a < s->na; a++) {
        const double recirc = e->ahu_at[a] > 0.0 ? e->ahu_ws[a] / e->ahu_at[a] : tmean;
        const double st = ahu_static_p(e, s, a);
        const double fe = s->ahu_c[a * 9 + 5];
        const double flow = e->ahu_run[a] == 1 ? e->ahu_flow[a] : 0.0;
        intake += flow * st / fe;
        exhaust += flow * (1.0 - e->ahu_rec[a]) * st / fe;
        const double mixed = e->ahu_rec[a] * recirc + (1.0 - e->ahu_rec[a]) * ambient;
        const double sat = (mixed > e->ahu_sat[a] && e->ahu_run[a] == 1) ? e->ahu_sat[a] : mixed;
        cooling += flow * RHO_AIR * CP_AIR * (sat - mixed) / s->ahu_c[a * 9 + 4];
    }
    const double blower = intake + exhaust;
    const double tf = water_flow(e, s);
    /* boiler gas rate (sb_reward.c:12-29) */
    double gas_rate;
    {
        const double* c = s->boiler;
        const double rwt = e->b_ret;
        const double supply = e->b_sp > rwt ? e->b_sp : rwt;
        const double flow = CP_W * RHO_W * tf * (supply - rwt);
        double diss = 0.0;
        if (supply >= ambient) {
            const double num = c[5] * 2.0 * 3.14159265358979323846 * (supply - ambient);
            const double r2 = c[6] + c[9];
            const double cond = log(r2 / c[6]) / c[8];
            const double conv = 1.0 / c[4] / r2;
            diss = num / (cond + conv);
        }
        double tank = 0.0;
        if (dt > 0.0) tank = CP_W * RHO_W * c[7] * e->b_step / dt;
        const double tot = flow + diss + tank;
        gas_rate = tot > 0.0 ? tot : 0.0;
    }
    const double pump_e = tf * RHO_W * GRAV * e->pump_head / s->pump_eff;
    const double max_pph = s->rw[0], min_pph = s->rw[1], ref = s->rw[2];
    double total_occ = 0.0, cum = 0.0, dsum = 0.0, dmax = 0.0;
    int oob = 0;
    for (int z = 0; z < nz; z++) {
        const double occ = e->V[z];
        total_occ += occ;
        const double zt = e->zavg[z];
        const double hsp = s->s_heat[kv], csp = s->s_cool[kv];
        double dev = zt - csp;
        if (hsp - zt > dev) dev = hsp - zt;
        if (dev < 0.0) dev = 0.0;
        dsum += dev;
        if (dev > dmax) dmax = dev;
        if (dev > 0.0) oob++;
        const double shortfall = dev <= ref ? dev / ref : 1.0 + ((dev - ref) / ref) * ((dev - ref) / ref);
        cum += max_pph * (1.0 - shortfall) * occ * dt * inv_hour;
    }
    const double max_prod = max_pph * total_occ * dt * inv_hour;
    const double min_prod = min_pph * total_occ * dt * inv_hour;
    const double npr = (total_occ > 0.0 && (max_prod - min_prod) != 0.0)
                           ? (cum - min_prod) / (max_prod - min_prod) - 1.0 : 0.0;
    const double elec_rate = blower + fabs(cooling) + pump_e;
    const double price = wd ? s->e_wd[hour] : s->e_we[hour];
    const double crate = s->e_c[hour];
    const double elec_cost = price * fabs(elec_rate) * dt;
    const double elec_cost_max = price * s->rw[3] * dt;
    const double elec_carb = crate * fabs(elec_rate) * dt;
    const double elec_carb_max = crate * s->rw[3] * dt;
    const double gprice = s->g_p[month - 1];
    const double g = gas_rate > 0.0 ? gas_rate : 0.0;
    const double gas_cost = gprice * g * dt;
    const double gas_cost_max = gprice * s->rw[4] * dt;
    const double gas_carb = s->g_c * g * dt;
    const double gas_carb_max = s->g_c * s->rw[4] * dt;
    const double den_e = elec_cost_max + gas_cost_max;
    const double nec = den_e > 0.0 ? (elec_cost + gas_cost) / den_e : 0.0;
    const double den_c = elec_carb_max + gas_carb_max;
    const double ncar = den_c > 0.0 ? (elec_carb + gas_carb) / den_c : 0.0;
    if (parts12) {
        parts12[0] = npr; parts12[1] = nec; parts12[2] = ncar;
        parts12[3] = elec_cost; parts12[4] = gas_cost;
        parts12[5] = blower; parts12[6] = cooling; parts12[7] = pump_e;
        parts12[8] = price; parts12[9] = dt; parts12[10] = (double)hour; parts12[11] = (double)wd;
    }
    if (log8) {
        log8[0] = npr; log8[1] = nec; log8[2] = ncar;
        log8[3] = nz > 0 ? dsum / nz : 0.0;
        log8[4] = dmax;
        log8[5] = nz > 0 ? (double)oob / nz : 0.0;
        log8[6] = fabs(elec_rate) * dt / 3.6e6;
        log8[7] = g * dt / 3.6e6;
    }
    const double pw = s->rw[5], ew = s->rw[6], cw = s->rw[7];
    return (npr * pw - nec * ew - ncar * cw) / (pw + ew + cw);
}
