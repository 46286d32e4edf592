/* Synthetic scenario generator: writes SBB1 blobs that the reference's C core
 * (complete_port/csim) and this library's device env both load.
 *
 * The reference bakes its blobs from the organisers' Python simulator and
 * scipy's SuperLU (complete_port/pysim/bake_scenario.py:42-205,
 * complete_port/pysim/bake_env.py:21-396). Neither the simulator nor the
 * shipped blobs are available, so this generator writes every section the C
 * core reads from seeded synthetic buildings: recursive rectangular room
 * partitions on a control-volume grid, face conductances, interior mass,
 * VAV/AHU/boiler constants, calendars, AR(1) weather, tariffs, observation
 * normalisers, and the nested-dissection LDL^T factors of the thermal matrix
 * (stored as the SuperLU-style CSC L/U + row/column permutations that
 * complete_port/csim/sb_lu.c:5-34 replays).
 *
 * Plain C ABI: no allocation is handed to the caller. */
#ifndef SBGEN_H
#define SBGEN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int rows, cols;            /* control-volume grid */
    int n_rooms;               /* physical zones (one VAV each) */
    int n_ahu;                 /* air handlers; zones split into contiguous blocks */
    int notch_rows, notch_cols;/* exterior (unsolved) corner cut-out, 0 = none */
    int dense_walls;           /* 1: extra partition faces inside rooms */
    int n_steps;               /* episode length; tables hold n_steps + 1 rows */
    int start_doy;             /* day of year of the first step (0 = Jan 1, a Sunday) */
    int start_hour;
    int zone_assignment;       /* occupants per zone */
    int conv_distance;
    double cv_size_cm;
    double dt_sec;
    double t_mean_c, t_amp_k;  /* outdoor dry bulb = mean + amp*sin(2pi(h-9)/24) + AR(1) */
    double ar_phi, ar_sigma_k; /* AR(1) coefficient and stationary std */
    double conv_p;
    uint64_t layout_seed;      /* geometry, conductances, HVAC constants */
    uint64_t climate_seed;     /* weather noise */
    int64_t occ_seed, conv_seed;
    int random_start_days;     /* 0, or 7: calendar tables 6 * 288 rows longer than the
                                  episode, the priming hour per row and
                                  random_start_offsets (for the env's random_start) */
} SbGenParams;

/* Fills `out` with the parameters of one BASELINE configuration scenario.
 * config 1: the single 64x48 / 41-zone building;
 * config 2: index 0..29 = layout (index / 5) x climate (index % 5) of the
 *           960-env mix (six layouts of 41-81 zones, 1-4 AHUs);
 * config 3: the 128x96 / 81-zone / 4-AHU building (dense walls).
 * Returns 0, or -1 for an unknown config/index. */
int sbgen_preset(int config, int index, SbGenParams* out);

/* Generates the scenario and writes it to `path`. Returns 0 on success; on
 * failure writes a one-line reason into err (if non-NULL) and returns -1. */
int sbgen_write(const char* path, const SbGenParams* p, char* err, int errlen);

/* Summary numbers of the factor the generator produced for `p` (for reports):
 * n (solved cells), nnz of L and of U including diagonals. Returns 0 or -1. */
int sbgen_factor_stats(const SbGenParams* p, int64_t* n, int64_t* nnz_l, int64_t* nnz_u);

#ifdef __cplusplus
}
#endif
#endif /* SBGEN_H */
