// Host-side construction of the device tables from SBB1 blobs.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "sbb.h"
#include "sbenv_dev.h"
#include "sweep_sched.h"

namespace sbenv {

struct HostGroup {
    int n = 0, ncv = 0, k = 0, nz = 0, nv = 0, na = 0;
    int rows = 0, cols = 0;   // the thermal grid
    int64_t nnzL = 0, nnzU = 0;
    std::vector<double> cap, dirx, mc, ret, gain;   // row order
    std::vector<int32_t> zone_of_row;
    HostSweep fwd, bwd;                   // built by build_sweeps once the ring depth is known
    std::vector<std::vector<std::pair<int, double>>> lt, ut;   // sweep terms in push order
    std::vector<double> udiag;
    std::vector<int32_t> sn_p, sn_pos, ap_rp, ap_col;
    std::vector<double> sn_x, ap_x, S;
    std::vector<int32_t> room_off, room_pos, cell_of_pos, pos_of_cell;
    std::vector<int32_t> cv_off, cv_pos, cand_off, cand_idx;
    int conv_maxroom = 0;
    std::vector<int32_t> row_of_solved;   // solved index t -> row position
    // air-side response W = A^-1 applied in row order, [n][k] (the columns the
    // reference core computes to form S); the corrected build adds W q to y
    std::vector<double> W;
    // folded air side (build_fold): Z = L^-1 applied by row, R = sensed U^-1 by sensor
    std::vector<int32_t> zr_p, zr_col, rs_p, rs_pos;
    std::vector<double> zr_x, rs_x;
};

struct HostScn {
    std::string path, name;
    int group = -1;
    int na = 0, nv = 0, nz = 0, k = 0, nact = 0, n_cont = 0, n_disc = 0, n_dev = 0, n_aux = 0, max_steps = 0;
    int assign = 0, ea = 0, la = 0, ed = 0, ld = 0, hour_m1 = 0, wd_m1 = 0, tmean_needed = 0, conv_dist = 0;
    double p_arr = 0, p_dep = 0, dt = 300, internal_w = 0, standby = 1, occ_w = 0, cv_area = 0, header_res = 0;
    double pump_eff = 1, pump_head0 = 0, gas_carbon = 0, conv_p = 0, boiler_cond = 0;
    double boiler[10] = {0};
    uint32_t occ_seed = 0, conv_seed = 0;
    std::vector<double> amb, s_comf, s_heat, s_cool, aux;
    std::vector<int64_t> o_hour, r_hour, r_month;
    std::vector<uint8_t> o_wd, r_wd;
    std::vector<double> ahu_c, vav_c, zarea;
    std::vector<int32_t> vz_off, vz_idx, v_ahu, coupled, zv_off, zv_idx, proom, room_ncell;
    std::vector<int32_t> zc_off, zc_col, ac_off, ac_col, av_off, av_idx;   // per-zone / per-AHU ascending lists
    std::vector<uint8_t> a_kind, a_act, a_disc;
    std::vector<int32_t> a_idx, a_slot;
    std::vector<double> a_mn, a_mx, a_mnr, a_mxr;
    std::vector<uint8_t> f_kind, f_id;
    std::vector<int32_t> f_idx;
    std::vector<double> f_mean, f_var;
    std::vector<double> rw, e_wd, e_we, e_c, g_p;
    std::vector<double> temp_init, mass_init;   // extended row order / row order
    std::vector<int64_t> o_hour_m1;             // priming hour per calendar row (or one entry)
    std::vector<uint8_t> o_wd_m1;
    int obs_len() const { return n_dev + n_aux; }
};

// Builds the solver/geometry tables of a group from its first blob.
std::string build_group(const sbb::Reader& b, HostGroup& g);
// Deepest per-warp ring (stages, at most kStagesMax) that a slab of B envs of an
// n-cell field leaves room for within smem_cap bytes; 0 if not even kStagesMin.
int solve_ring_stages(int n, int B, size_t smem_cap);
// Builds the group's L and U sweep programs for a per-warp ring of ring_stages.
// tolerant (the corrected and folded builds): the L sweep's terms of every row
// ordered by the depth of their source rows instead of the reference's push
// order, and the U sweep's diagonal entries hold 1 / diagonal (multiplied,
// not divided); the exact build keeps the reference's order and divisions
std::string build_sweeps(HostGroup& g, int ring_stages, bool tolerant = false);
// Builds the folded air side's Z = L^-1 applied and R = sensed U^-1 (row order).
std::string build_fold(HostGroup& g);
// Builds the per-scenario tables (needs the group's position maps).
// random_start: the blob must carry the seven start offsets (d * 288) and
// calendar tables 6 * 288 rows longer than the episode
// (complete_port/gpu/smart_buildings.cu:2460-2495).
std::string build_scenario(const sbb::Reader& b, const HostGroup& g, int max_steps_kw, bool random_start,
                           HostScn& s);
// True when b can share a's group: every geometry / solver section identical.
bool same_geometry(const sbb::Reader& a, const sbb::Reader& b);

// The reference's S computation (complete_port/csim/sb_fdm.c:103-114) as a
// host helper, exposed for tests: x = A^-1 b by factor replay in solved order.
void lu_replay(const sbb::Reader& b, const std::vector<double>& rhs, std::vector<double>& x);

}  // namespace sbenv
