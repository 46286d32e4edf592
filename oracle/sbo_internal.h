/* TEST INFRASTRUCTURE: internal types of this repository's C restatement of the
 * reference CPU simulator (complete_port/csim). Nothing here is product code.
 *
 * Layout: SboScn holds the read-only scenario tables of one blob; SboState
 * holds everything an environment mutates. The arithmetic of every function
 * follows the cited reference lines operation for operation (same order, no
 * FMA) so the restatement is bit-identical to the reference and can pin the
 * device path. */
#ifndef SBO_INTERNAL_H
#define SBO_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

/* ---- blob (SBB1) ---- */
typedef struct {
    const char* name;
    uint32_t dtype, ndim;
    uint64_t count, off;
} SboSec;

typedef struct {
    uint8_t* map;
    size_t size;
    int nsec;
    SboSec* sec;
} SboBlob;

int sbo_blob_open(SboBlob* b, const char* path);
void sbo_blob_close(SboBlob* b);
const SboSec* sbo_blob_find(const SboBlob* b, const char* name);
const void* sbo_blob_get(const SboBlob* b, const char* name, uint32_t dtype);
double sbo_blob_f64_1(const SboBlob* b, const char* name, double dflt);
int64_t sbo_blob_i64_1(const SboBlob* b, const char* name, int64_t dflt);

/* ---- MT19937, numpy RandomState stream ---- */
typedef struct { uint32_t s[624]; int pos; } SboMt;
void sbo_mt_seed(SboMt* m, uint32_t seed);
uint32_t sbo_mt_next(SboMt* m);
double sbo_mt_sample(SboMt* m);                 /* random_sample: 53-bit double */
uint32_t sbo_mt_bounded(SboMt* m, uint32_t hi); /* randint(0, hi + 1), masked rejection */

/* ---- scenario tables ---- */
typedef struct {
    SboBlob blob;
    int nr, nc, ncv, n, k, na, nv, nz, nact, n_cont, n_disc, n_dev, n_aux, max_steps;
    const int64_t* solved;
    const double *cap, *dir, *mc, *mret, *mgain, *horiz, *vert, *cond, *af0, *af1;
    const double *temp_init, *mass_init;
    /* factor replay */
    const int32_t *Lp, *Li, *Up, *Ui;
    const double *Lx, *Ux;
    int *Ldg, *Udg, *ir, *pc;
    /* air side */
    const int32_t *ap_p, *ap_i, *sn_p, *sn_i, *as_p, *as_i;
    const double *ap_x, *sn_x, *as_x;
    double* S;  /* k x k sensed response */
    /* HVAC / topology */
    const int32_t *vz_off, *vz_idx, *v_ahu, *coupled, *zv_off, *zv_idx, *proom, *room_off, *room_cells;
    const double *zarea, *ahu_c, *vav_c;
    const uint8_t *a_kind, *a_act, *a_disc;
    const int32_t* a_idx;
    const double *a_mn, *a_mx, *a_mnr, *a_mxr;
    const double *s_comf, *s_heat, *s_cool, *amb;
    double internal_w, standby, occ_w, cv_area, h, dt;
    double header_res, pump_head0, pump_eff, boiler[10];
    int is_boiler;
    /* observation / reward */
    const uint8_t *f_kind, *f_id;
    const int32_t* f_idx;
    const double *f_mean, *f_var, *aux;
    const double *rw, *e_wd, *e_we, *e_c, *g_p;
    double g_c;
    const int64_t *r_hour, *r_month;
    const uint8_t* r_wd;
    /* occupancy */
    int assign, ea, la, ed, ld, hour_m1, wd_m1;
    const int64_t* o_hour_m1;   /* priming hour per calendar row (m1_rows entries) */
    const uint8_t* o_wd_m1;
    int m1_rows;
    double p_arr, p_dep;
    const int64_t* o_hour;
    const uint8_t* o_wd;
    uint32_t occ_seed;
    /* convection */
    double conv_p;
    int conv_dist, conv_nrooms, conv_maxroom;
    uint32_t conv_seed;
    const int32_t *cv_off, *cv_cells, *cand_off, *cand_idx;
} SboScn;

/* ---- mutable environment state ---- */
typedef struct {
    double *temp, *mass, *inq;                 /* field (ncv), interior mass (n), applied heat (ncv) */
    double *work, *y, *yr, *rhs, *pw, *qv, *mat; /* solve scratch */
    int *ahu_run, *ahu_creq;
    double *ahu_rec, *ahu_sat, *ahu_fan, *ahu_flow, *ahu_ws, *ahu_at, *ahu_sv;
    double *v_damp, *v_reh, *v_ratio, *v_hsp, *v_csp, *v_dcmd, *v_rcmd, *v_sense, *v_area;
    int *v_mode, *v_prev, *v_dset, *v_rset;
    double *zavg, *zq, *smean, *ag, *aT, *coil, *zfsp, *zfact, *demand;
    double ff_sum, reheat_w, pump_head, b_sp, b_ret, b_cur, b_step;
    int hws_req, hws_run, pump_run, step_index;
    /* occupancy */
    SboMt orng;
    int* ostate;
    double* V;
    /* convection */
    SboMt crng;
    int *cl, *cr;
    /* env wrapper */
    int step;
    double parts[12];
    double* qpre;   /* applied heat per zone cell after the pre stage (inspection) */
    double native[272];
} SboState;

int sbo_scn_load(SboScn* s, const char* path, int max_steps);
void sbo_scn_free(SboScn* s);
int sbo_state_alloc(SboState* e, const SboScn* s);
void sbo_state_free(SboState* e);

void sbo_sim_reset(SboState* e, const SboScn* s);
void sbo_decode(const SboScn* s, const float* act, double* native);
void sbo_apply_native(SboState* e, const SboScn* s, const double* native);
void sbo_sim_step(SboState* e, const SboScn* s);
void sbo_observe(SboState* e, const SboScn* s, int j, float* out);
void sbo_occ_advance(SboState* e, const SboScn* s, int hour, int workday);
double sbo_reward(SboState* e, const SboScn* s, int kv, double* parts12, double* log8);

#endif /* SBO_INTERNAL_H */
