// Host-side construction of the device tables (declarations in tables.h).
// Built with -ffp-contract=off: the setup arithmetic (exposure, the sensed
// response S, log of the boiler geometry) must round exactly like the
// reference C core's.
#include "tables.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <numeric>
#include <set>

namespace sbenv {

namespace {

#define NEED(ptr, name)                                     \
    do {                                                    \
        if (!(ptr)) return std::string("missing or mistyped section ") + (name); \
    } while (0)

template <class T> std::vector<T> vec(const T* p, uint64_t n) { return p ? std::vector<T>(p, p + n) : std::vector<T>(); }

struct Factor {
    int n;
    const int32_t *Lp, *Li, *Up, *Ui, *pr, *pcc;
    const double *Lx, *Ux;
    std::vector<int> Ldg, Udg, ir;
};

std::string load_factor(const sbb::Reader& b, Factor& F) {
    F.n = (int)b.count("solved");
    F.Lp = b.i32("lu_L_indptr"); F.Li = b.i32("lu_L_indices"); F.Lx = b.f64("lu_L_data");
    F.Up = b.i32("lu_U_indptr"); F.Ui = b.i32("lu_U_indices"); F.Ux = b.f64("lu_U_data");
    F.pr = b.i32("lu_perm_r"); F.pcc = b.i32("lu_perm_c");
    NEED(F.Lp, "lu_L_indptr"); NEED(F.Li, "lu_L_indices"); NEED(F.Lx, "lu_L_data");
    NEED(F.Up, "lu_U_indptr"); NEED(F.Ui, "lu_U_indices"); NEED(F.Ux, "lu_U_data");
    NEED(F.pr, "lu_perm_r"); NEED(F.pcc, "lu_perm_c");
    const int n = F.n;
    if (b.count("lu_L_indptr") != (uint64_t)n + 1 || b.count("lu_U_indptr") != (uint64_t)n + 1 ||
        b.count("lu_perm_r") != (uint64_t)n || b.count("lu_perm_c") != (uint64_t)n)
        return "factor sections do not match the solved-cell count";
    if ((uint64_t)F.Lp[n] > b.count("lu_L_indices") || (uint64_t)F.Up[n] > b.count("lu_U_indices"))
        return "factor index arrays shorter than their indptr";
    F.Ldg.assign(n, -1);
    F.Udg.assign(n, -1);
    for (int j = 0; j < n; j++) {
        for (int q = F.Lp[j]; q < F.Lp[j + 1]; q++) {
            if (F.Li[q] < j || F.Li[q] >= n) return "L has an entry above the diagonal or out of range";
            if (F.Li[q] == j && F.Ldg[j] < 0) F.Ldg[j] = q;
        }
        for (int q = F.Up[j]; q < F.Up[j + 1]; q++) {
            if (F.Ui[q] > j || F.Ui[q] < 0) return "U has an entry below the diagonal or out of range";
            if (F.Ui[q] == j && F.Udg[j] < 0) F.Udg[j] = q;
        }
        if (F.Ldg[j] < 0 || F.Udg[j] < 0) return "factor column without a diagonal entry";
    }
    F.ir.assign(n, -1);
    for (int i = 0; i < n; i++) {
        if (F.pr[i] < 0 || F.pr[i] >= n || F.ir[F.pr[i]] >= 0) return "lu_perm_r is not a permutation";
        F.ir[F.pr[i]] = i;
    }
    return "";
}

void replay(const Factor& F, const std::vector<double>& b, std::vector<double>& x) {
    // complete_port/csim/sb_lu.c:38-63, in the same order
    const int n = F.n;
    std::vector<double> w(n);
    for (int i = 0; i < n; i++) w[i] = b[F.ir[i]];
    for (int j = 0; j < n; j++) {
        const double yj = w[j];
        for (int q = F.Lp[j]; q < F.Lp[j + 1]; q++)
            if (q != F.Ldg[j]) w[F.Li[q]] -= F.Lx[q] * yj;
    }
    for (int j = n - 1; j >= 0; j--) {
        const double zj = w[j] / F.Ux[F.Udg[j]];
        w[j] = zj;
        for (int q = F.Up[j]; q < F.Up[j + 1]; q++)
            if (q != F.Udg[j]) w[F.Ui[q]] -= F.Ux[q] * zj;
    }
    x.resize(n);
    for (int t = 0; t < n; t++) x[t] = w[F.pcc[t]];
}

const char* kGeometry[] = {
    "grid", "solved", "capacitance_rate", "dirichlet_conductance", "mass_coupling", "mass_retained",
    "mass_gained", "horizontal", "vertical", "solver_conductivity", "ambient_face_areas_0",
    "ambient_face_areas_1", "convection_coefficient", "lu_L_indptr", "lu_L_indices", "lu_L_data",
    "lu_U_indptr", "lu_U_indices", "lu_U_data", "lu_perm_r", "lu_perm_c", "applied_indptr",
    "applied_indices", "applied_data", "sensed_shape", "sensed_indptr", "sensed_indices", "sensed_data",
    "room_offsets", "room_cells", "phys_room_idx", "conv_room_offsets", "conv_room_cells",
    "conv_cand_offsets", "conv_cand_idx", "zone_area", nullptr};

}  // namespace

void lu_replay(const sbb::Reader& b, const std::vector<double>& rhs, std::vector<double>& x) {
    Factor F;
    if (!load_factor(b, F).empty()) { x.clear(); return; }
    replay(F, rhs, x);
}

bool same_geometry(const sbb::Reader& a, const sbb::Reader& b) {
    for (int i = 0; kGeometry[i]; i++) {
        const sbb::Section* sa = a.find(kGeometry[i]);
        const sbb::Section* sb = b.find(kGeometry[i]);
        if (!sa || !sb) {
            if (sa != sb) return false;
            continue;
        }
        if (sa->dtype != sb->dtype || sa->count != sb->count) return false;
        if (memcmp(a.data(sa), b.data(sb), sa->count * sbb::dtype_size(sa->dtype)) != 0) return false;
    }
    return true;
}

std::string build_group(const sbb::Reader& b, HostGroup& g) {
    const int64_t* grid = b.i64("grid");
    NEED(grid, "grid");
    const int nr = (int)grid[0], nc = (int)grid[1];
    g.ncv = nr * nc;
    g.rows = nr;
    g.cols = nc;
    const int64_t* solved = b.i64("solved");
    NEED(solved, "solved");
    Factor F;
    std::string e = load_factor(b, F);
    if (!e.empty()) return e;
    const int n = F.n;
    g.n = n;
    if (n > 65535) return "more than 65535 solved cells (16-bit schedule indices)";
    for (int t = 0; t < n; t++)
        if (solved[t] < 0 || solved[t] >= g.ncv) return "solved cell index out of range";
    for (int i = 0; i < n; i++)
        if (F.pcc[F.ir[i]] != i)
            return "perm_c o inv(perm_r) is not the identity (row-pivoted factors are not supported)";
    g.nnzL = F.Lp[n];
    g.nnzU = F.Up[n];
    g.row_of_solved.assign(n, 0);
    for (int i = 0; i < n; i++) g.row_of_solved[F.ir[i]] = i;
    // positions
    g.pos_of_cell.assign(g.ncv, -1);
    for (int t = 0; t < n; t++) {
        if (g.pos_of_cell[solved[t]] >= 0) return "a cell is solved twice";
        g.pos_of_cell[solved[t]] = g.row_of_solved[t];
    }
    int nxt = n;
    for (int p = 0; p < g.ncv; p++)
        if (g.pos_of_cell[p] < 0) g.pos_of_cell[p] = nxt++;
    g.cell_of_pos.assign(g.ncv, 0);
    for (int p = 0; p < g.ncv; p++) g.cell_of_pos[g.pos_of_cell[p]] = p;

    // coefficients in row order; exposure exactly as complete_port/csim/sb_fdm.c:126-140
    const double* cap = b.f64("capacitance_rate");
    const double* dir = b.f64("dirichlet_conductance");
    const double* mc = b.f64("mass_coupling");
    const double* mr = b.f64("mass_retained");
    const double* mg = b.f64("mass_gained");
    const double* hor = b.f64("horizontal");
    const double* ver = b.f64("vertical");
    const double* cond = b.f64("solver_conductivity");
    const double* af0 = b.f64("ambient_face_areas_0");
    const double* af1 = b.f64("ambient_face_areas_1");
    NEED(cap, "capacitance_rate"); NEED(dir, "dirichlet_conductance"); NEED(mc, "mass_coupling");
    NEED(mr, "mass_retained"); NEED(mg, "mass_gained"); NEED(hor, "horizontal"); NEED(ver, "vertical");
    NEED(cond, "solver_conductivity"); NEED(af0, "ambient_face_areas_0"); NEED(af1, "ambient_face_areas_1");
    const double h = b.f64_1("convection_coefficient", 8.8);
    g.cap.resize(n); g.dirx.resize(n); g.mc.resize(n); g.ret.resize(n); g.gain.resize(n);
    for (int i = 0; i < n; i++) {
        const int t = F.ir[i];
        const int64_t p = solved[t];
        double ex = 0.0;
        if (af0[p] > 0.0) ex += h * af0[p] / (1.0 + h * 0.5 * hor[p] / cond[p]);
        if (af1[p] > 0.0) ex += h * af1[p] / (1.0 + h * 0.5 * ver[p] / cond[p]);
        g.cap[i] = cap[t];
        g.dirx[i] = dir[t] + ex;
        g.mc[i] = mc[t];
        g.ret[i] = mr[t];
        g.gain[i] = mg[t];
    }
    // rooms
    const int32_t* room_off = b.i32("room_offsets");
    const int32_t* room_cells = b.i32("room_cells");
    const int32_t* proom = b.i32("phys_room_idx");
    NEED(room_off, "room_offsets"); NEED(room_cells, "room_cells"); NEED(proom, "phys_room_idx");
    const int nrooms = (int)b.count("room_offsets") - 1;
    g.room_off = vec(room_off, (uint64_t)nrooms + 1);
    if ((uint64_t)2 * room_off[nrooms] > b.count("room_cells")) return "room_cells shorter than room_offsets";
    if (room_off[nrooms] > g.ncv) return "more room cells than grid cells";
    g.room_pos.resize(room_off[nrooms]);
    for (int t = 0; t < room_off[nrooms]; t++) {
        const int r = room_cells[2 * t], c = room_cells[2 * t + 1];
        if (r < 0 || r >= nr || c < 0 || c >= nc) return "room cell out of the grid";
        g.room_pos[t] = g.pos_of_cell[r * nc + c];
    }
    g.nz = (int)b.count("zone_area");
    std::vector<int> cell_zone(g.ncv, -1);
    for (int z = 0; z < g.nz; z++) {
        const int rm = proom[z];
        if (rm < 0 || rm >= nrooms) return "phys_room_idx out of range";
        if (room_off[rm + 1] - room_off[rm] <= 0) return "a physical zone has no cells";
        for (int t = room_off[rm]; t < room_off[rm + 1]; t++)
            cell_zone[room_cells[2 * t] * nc + room_cells[2 * t + 1]] = z;
    }
    g.zone_of_row.resize(n);
    for (int i = 0; i < n; i++) g.zone_of_row[i] = cell_zone[solved[F.ir[i]]];

    // sweeps: L rows pull columns ascending, U rows pull columns descending
    std::vector<std::vector<std::pair<int, double>>>& lt = g.lt;
    std::vector<std::vector<std::pair<int, double>>>& ut = g.ut;
    std::vector<double>& udiag = g.udiag;
    lt.assign(n, {});
    ut.assign(n, {});
    udiag.assign(n, 0.0);
    for (int j = 0; j < n; j++)
        for (int q = F.Lp[j]; q < F.Lp[j + 1]; q++)
            if (q != F.Ldg[j]) lt[F.Li[q]].push_back({j, F.Lx[q]});
    for (int j = n - 1; j >= 0; j--) {
        udiag[j] = F.Ux[F.Udg[j]];
        for (int q = F.Up[j]; q < F.Up[j + 1]; q++)
            if (q != F.Udg[j]) ut[F.Ui[q]].push_back({j, F.Ux[q]});
    }
    for (int i = 0; i < n; i++)
        for (size_t a = 0; a < ut[i].size(); a++)
            if (ut[i][a].first == i) return "U has a duplicate diagonal";
    if (n >= 0xFFFF) return "more than 65534 solved cells";

    // air side
    const int64_t* shp = b.i64("sensed_shape");
    g.k = shp ? (int)shp[0] : 0;
    const int k = g.k;
    if (k > kMaxK) return "more than 128 coupled VAVs";
    if (k > 0) {
        const int32_t* sp = b.i32("sensed_indptr");
        const int32_t* si = b.i32("sensed_indices");
        const double* sx = b.f64("sensed_data");
        const int32_t* ap = b.i32("applied_indptr");
        const int32_t* ai = b.i32("applied_indices");
        const double* ax = b.f64("applied_data");
        NEED(sp, "sensed_indptr"); NEED(si, "sensed_indices"); NEED(sx, "sensed_data");
        NEED(ap, "applied_indptr"); NEED(ai, "applied_indices"); NEED(ax, "applied_data");
        g.sn_p = vec(sp, (uint64_t)k + 1);
        g.sn_pos.resize(sp[k]);
        g.sn_x = vec(sx, (uint64_t)sp[k]);
        for (int q = 0; q < sp[k]; q++) {
            if (si[q] < 0 || si[q] >= n) return "sensed index out of range";
            g.sn_pos[q] = g.row_of_solved[si[q]];
        }
        std::vector<std::vector<std::pair<int, double>>> rows(n);
        for (int j = 0; j < k; j++)
            for (int q = ap[j]; q < ap[j + 1]; q++) {
                if (ai[q] < 0 || ai[q] >= n) return "applied index out of range";
                rows[g.row_of_solved[ai[q]]].push_back({j, ax[q]});
            }
        g.ap_rp.assign(n + 1, 0);
        for (int i = 0; i < n; i++) {
            for (auto& e2 : rows[i]) { g.ap_col.push_back(e2.first); g.ap_x.push_back(e2.second); }
            g.ap_rp[i + 1] = (int32_t)g.ap_col.size();
        }
        // S = sensed A^-1 applied (complete_port/csim/sb_fdm.c:103-114); the
        // columns A^-1 applied are kept in row order as W
        g.S.assign((size_t)k * k, 0.0);
        g.W.assign((size_t)n * k, 0.0);
        std::vector<double> r(n), yr;
        for (int j = 0; j < k; j++) {
            std::fill(r.begin(), r.end(), 0.0);
            for (int q = ap[j]; q < ap[j + 1]; q++) r[ai[q]] = ax[q];
            replay(F, r, yr);
            for (int t = 0; t < n; t++) g.W[(size_t)g.row_of_solved[t] * k + j] = yr[t];
            for (int i = 0; i < k; i++) {
                double acc = 0.0;
                for (int q = sp[i]; q < sp[i + 1]; q++) acc += sx[q] * yr[si[q]];
                g.S[(size_t)i * k + j] = acc;
            }
        }
    } else {
        g.sn_p.assign(1, 0);
        g.ap_rp.assign(n + 1, 0);
    }
    // convection
    const int32_t* coff = b.i32("conv_room_offsets");
    const int32_t* ccell = b.i32("conv_room_cells");
    const int32_t* cno = b.i32("conv_cand_offsets");
    const int32_t* cni = b.i32("conv_cand_idx");
    NEED(coff, "conv_room_offsets"); NEED(ccell, "conv_room_cells");
    NEED(cno, "conv_cand_offsets"); NEED(cni, "conv_cand_idx");
    const int ncr = (int)b.count("conv_room_offsets") - 1;
    g.cv_off = vec(coff, (uint64_t)ncr + 1);
    const int ncc = coff[ncr];
    if ((uint64_t)ncc + 1 > b.count("conv_cand_offsets")) return "conv_cand_offsets too short";
    g.cv_pos.resize(ncc);
    for (int x = 0; x < ncc; x++) {
        const int r = ccell[2 * x], c = ccell[2 * x + 1];
        if (r < 0 || r >= nr || c < 0 || c >= nc) return "convection cell out of the grid";
        g.cv_pos[x] = g.pos_of_cell[r * nc + c];
    }
    g.cand_off = vec(cno, (uint64_t)ncc + 1);
    g.cand_idx = vec(cni, (uint64_t)cno[ncc]);
    for (int32_t c : g.cand_idx)
        if (c < 0 || c >= ncc) return "convection candidate out of range";
    for (int rm = 0; rm < ncr; rm++) g.conv_maxroom = std::max(g.conv_maxroom, coff[rm + 1] - coff[rm]);
    if (g.conv_maxroom > kMaxConvRoom) return "a convection room has more than 8192 cells";
    return "";
}

std::string build_scenario(const sbb::Reader& b, const HostGroup& g, int max_steps_kw, bool random_start,
                           HostScn& s) {
    s.path = b.path();
    {
        const size_t sl = s.path.find_last_of('/');
        s.name = sl == std::string::npos ? s.path : s.path.substr(sl + 1);
        const size_t dot = s.name.rfind(".sbb");
        if (dot != std::string::npos) s.name = s.name.substr(0, dot);
    }
    const int64_t* solved = b.i64("solved");
    const int n = g.n;
    s.k = g.k;
    s.na = (int)(b.count("ahu_const") / 9);
    s.nv = (int)b.count("vav_zone_offsets") - 1;
    s.nz = (int)b.count("zone_area");
    s.nact = (int)b.count("act_owner_kind");
    if (s.na < 1 || s.na > kMaxAhu) return "AHU count outside 1..16";
    if (s.nv < 0 || s.nz < 1) return "missing VAV/zone tables";
    s.ahu_c = vec(b.f64("ahu_const"), (uint64_t)s.na * 9);
    s.vav_c = vec(b.f64("vav_const"), (uint64_t)s.nv * 9);
    s.zarea = vec(b.f64("zone_area"), (uint64_t)s.nz);
    s.vz_off = vec(b.i32("vav_zone_offsets"), (uint64_t)s.nv + 1);
    if ((int)s.vav_c.size() != s.nv * 9 || s.vz_off.empty()) return "missing vav_const / vav_zone_offsets";
    s.vz_idx = vec(b.i32("vav_zone_idx"), (uint64_t)s.vz_off[s.nv]);
    s.v_ahu = vec(b.i32("vav_ahu_idx"), (uint64_t)s.nv);
    s.coupled = vec(b.i32("coupled_vav_idx"), (uint64_t)s.k);
    s.zv_off = vec(b.i32("zone_vav_offsets"), (uint64_t)s.nz + 1);
    if (s.zv_off.empty()) return "missing zone_vav_offsets";
    s.zv_idx = vec(b.i32("zone_vav_idx"), (uint64_t)s.zv_off[s.nz]);
    s.proom = vec(b.i32("phys_room_idx"), (uint64_t)s.nz);
    if ((int)s.v_ahu.size() != s.nv || (int)s.coupled.size() != s.k || (int)s.proom.size() != s.nz)
        return "VAV/zone topology sections missing";
    for (int v = 0; v < s.nv; v++)
        if (s.v_ahu[v] < 0 || s.v_ahu[v] >= s.na) return "vav_ahu_idx out of range";
    for (int c : s.coupled)
        if (c < 0 || c >= s.nv) return "coupled_vav_idx out of range";
    for (int z : s.vz_idx)
        if (z < 0 || z >= s.nz) return "vav_zone_idx out of range";
    // per-zone coupled columns, per-AHU coupled columns and VAVs, ascending: the
    // device accumulates each zone's and each AHU's sums on one thread in the
    // order of the reference's single loops (sb_sim.c:367-392, :408-436)
    {
        std::vector<std::vector<int32_t>> zl(s.nz), al(s.na), vl(s.na);
        for (int col = 0; col < s.k; col++) {
            const int v = s.coupled[col];
            for (int t = s.vz_off[v]; t < s.vz_off[v + 1]; t++) zl[s.vz_idx[t]].push_back(col);
            al[s.v_ahu[v]].push_back(col);
        }
        for (int v = 0; v < s.nv; v++) vl[s.v_ahu[v]].push_back(v);
        auto flat = [](const std::vector<std::vector<int32_t>>& ls, std::vector<int32_t>& off, std::vector<int32_t>& idx) {
            off.assign(1, 0);
            idx.clear();
            for (const auto& l : ls) {
                idx.insert(idx.end(), l.begin(), l.end());
                off.push_back((int32_t)idx.size());
            }
        };
        flat(zl, s.zc_off, s.zc_col);
        flat(al, s.ac_off, s.ac_col);
        flat(vl, s.av_off, s.av_idx);
    }
    s.room_ncell.resize(s.nz);
    for (int z = 0; z < s.nz; z++) s.room_ncell[z] = g.room_off[s.proom[z] + 1] - g.room_off[s.proom[z]];
    // static: does some AHU see no VAV area (then the field mean feeds its recirculation)?
    {
        std::vector<double> at(s.na, 0.0);
        for (int v = 0; v < s.nv; v++) {
            double area = 0.0;
            for (int t = s.vz_off[v]; t < s.vz_off[v + 1]; t++) area += s.zarea[s.vz_idx[t]];
            if (area > 0.0) at[s.v_ahu[v]] += area;
        }
        for (int a = 0; a < s.na; a++)
            if (!(at[a] > 0.0)) s.tmean_needed = 1;
    }
    // actions (complete_port/csim/sb_sim.c:220-244, :557-576)
    s.a_kind = vec(b.u8("act_owner_kind"), (uint64_t)s.nact);
    s.a_idx = vec(b.i32("act_owner_index"), (uint64_t)s.nact);
    s.a_act = vec(b.u8("act_actuator"), (uint64_t)s.nact);
    s.a_disc = vec(b.u8("act_is_discrete"), (uint64_t)s.nact);
    s.a_mn = vec(b.f64("act_min_native"), (uint64_t)s.nact);
    s.a_mx = vec(b.f64("act_max_native"), (uint64_t)s.nact);
    s.a_mnr = vec(b.f64("act_min_norm"), (uint64_t)s.nact);
    s.a_mxr = vec(b.f64("act_max_norm"), (uint64_t)s.nact);
    if ((int)s.a_mxr.size() != s.nact || (int)s.a_idx.size() != s.nact || (int)s.a_disc.size() != s.nact)
        return "action tables missing";
    {
        std::set<std::tuple<int, int, int>> targets;
        int nc2 = 0, nd2 = 0;
        s.a_slot.resize(s.nact);
        for (int i = 0; i < s.nact; i++) {
            s.a_slot[i] = s.a_disc[i] ? nd2++ : nc2++;
            const int kind = s.a_kind[i], idx = s.a_idx[i], act = s.a_act[i];
            if (kind == 0 && (idx < 0 || idx >= s.na)) return "action owner AHU out of range";
            if (kind == 1 && (idx < 0 || idx >= s.nv)) return "action owner VAV out of range";
            const int tgt = kind == 0 ? std::min(act, 3) : kind == 1 ? std::min(act, 1) : std::min(act, 2);
            if (!targets.insert({kind, kind == 2 ? 0 : idx, tgt}).second)
                return "two actions drive the same actuator";
        }
        s.n_cont = nc2;
        s.n_disc = nd2;
        if (s.n_cont > kCont || s.n_disc > kDisc) return "more than 256 continuous or 16 discrete actions";
    }
    // observation
    s.n_dev = (int)b.i64_1("n_dev", 0);
    s.n_aux = (int)b.i64_1("n_aux", 0);
    if (s.n_aux < 1 || s.obs_len() > kObs) return "observation layout outside 1..1024 fields";
    s.f_kind = vec(b.u8("f_dev_kind"), (uint64_t)s.n_dev);
    s.f_idx = vec(b.i32("f_dev_idx"), (uint64_t)s.n_dev);
    s.f_id = vec(b.u8("f_obs_id"), (uint64_t)s.n_dev);
    s.f_mean = vec(b.f64("f_norm_mean"), (uint64_t)s.n_dev);
    s.f_var = vec(b.f64("f_norm_var"), (uint64_t)s.n_dev);
    if ((int)s.f_var.size() != s.n_dev || (int)s.f_idx.size() != s.n_dev) return "observation tables missing";
    for (int i = 0; i < s.n_dev; i++) {
        const int kd = s.f_kind[i], ix = s.f_idx[i];
        if ((kd == 0 && (ix < 0 || ix >= s.na)) || (kd == 1 && (ix < 0 || ix >= s.nv)))
            return "observation field owner out of range";
    }
    // episode length (smart_buildings.cu:835-843; env.max_steps only shortens it)
    int ep = 0;
    {
        const double* om = b.f64("obs_meta");
        if (om && b.count("obs_meta") > 3) ep = (int)om[3];
        if (ep <= 0) ep = b.count("occ_hour") > 1 ? (int)b.count("occ_hour") - 1 : 8640;
        if (max_steps_kw > 0 && max_steps_kw < ep) ep = max_steps_kw;
    }
    s.max_steps = ep;
    // calendar rows the episodes read: random starts begin up to six days in
    const uint64_t rows = (uint64_t)ep + 1 + (random_start ? (uint64_t)6 * kStepsPerDay : 0);
    if (random_start) {
        const int64_t* off = b.i64("random_start_offsets");
        const double* op5 = b.f64("occ_params");
        if (!off || b.count("random_start_offsets") != (uint64_t)kStartDays || !op5 || b.count("occ_params") < 6 ||
            op5[5] != 300.0)
            return "random_start needs a seven-day random-start blob with five-minute steps";
        for (int d = 0; d < kStartDays; d++)
            if (off[d] != (int64_t)d * kStepsPerDay) return "random_start_offsets malformed";
        if (b.count("occ_hour_m1") < rows || b.count("occ_workday_m1") < rows)
            return "random_start section occ_hour_m1 / occ_workday_m1 too short";
    }
    auto need_rows = [&](const char* nm) { return b.count(nm) >= rows; };
    for (const char* nm : {"weather_ambient", "sched_comfort", "sched_heat_sp", "sched_cool_sp", "occ_hour",
                           "occ_workday", "rew_hour", "rew_month", "rew_workday"})
        if (!need_rows(nm)) return std::string("section ") + nm + " shorter than the episode";
    if (b.count("aux_time") < rows * (uint64_t)(s.n_aux - 1)) return "aux_time shorter than the episode";
    s.amb = vec(b.f64("weather_ambient"), rows);
    s.s_comf = vec(b.f64("sched_comfort"), rows);
    s.s_heat = vec(b.f64("sched_heat_sp"), rows);
    s.s_cool = vec(b.f64("sched_cool_sp"), rows);
    s.aux = vec(b.f64("aux_time"), rows * (uint64_t)(s.n_aux - 1));
    s.o_hour = vec(b.i64("occ_hour"), rows);
    s.o_wd = vec(b.u8("occ_workday"), rows);
    s.r_hour = vec(b.i64("rew_hour"), rows);
    s.r_month = vec(b.i64("rew_month"), rows);
    s.r_wd = vec(b.u8("rew_workday"), rows);
    if (s.amb.empty() || s.o_hour.empty() || s.r_month.empty()) return "schedule sections mistyped";
    for (uint64_t q = 0; q < rows; q++) {
        if (s.r_hour[q] < 0 || s.r_hour[q] > 23 || s.r_month[q] < 1 || s.r_month[q] > 12)
            return "reward calendar out of range";
    }
    // simulator scalars (complete_port/csim/sb_sim.c:52-75)
    s.internal_w = b.f64_1("internal_gain_w_per_m2", 0.0);
    s.standby = b.f64_1("internal_gain_standby_fraction", 1.0);
    s.occ_w = b.f64_1("occupant_sensible_heat_w", 0.0);
    const double* op = b.f64("occ_params");
    NEED(op, "occ_params");
    s.dt = op[5];
    {
        const double cvm = b.f64_1("cv_size_cm", 20.0) / 100.0;
        s.cv_area = cvm * cvm;
    }
    s.header_res = b.f64_1("hws_header_resistance", 0.0);
    {
        const double* bc = b.f64("boiler_const");
        for (int i = 0; i < 10; i++) s.boiler[i] = bc ? bc[i] : 0.0;
        const double r2 = s.boiler[6] + s.boiler[9];
        s.boiler_cond = std::log(r2 / s.boiler[6]) / s.boiler[8];
        const double* pc = b.f64("pump_const");
        s.pump_head0 = pc ? pc[0] : 0.0;
        s.pump_eff = pc ? pc[1] : 1.0;
    }
    // occupancy (complete_port/csim/sb_occup.c:6-30)
    s.assign = (int)op[0];
    s.ea = (int)op[1]; s.la = (int)op[2]; s.ed = (int)op[3]; s.ld = (int)op[4];
    s.p_arr = 1.0 / ((s.la - s.ea) * 3600.0 / op[5] / 2.0);
    s.p_dep = 1.0 / ((s.ld - s.ed) * 3600.0 / op[5] / 2.0);
    s.hour_m1 = (int)b.i64_1("occ_hour_m1", 0);
    {
        const uint8_t* wm = b.u8("occ_workday_m1");
        s.wd_m1 = wm ? wm[0] : 0;
    }
    if (random_start) {
        s.o_hour_m1 = vec(b.i64("occ_hour_m1"), rows);
        s.o_wd_m1 = vec(b.u8("occ_workday_m1"), rows);
    } else {
        s.o_hour_m1.assign(1, s.hour_m1);
        s.o_wd_m1.assign(1, (uint8_t)s.wd_m1);
    }
    s.occ_seed = (uint32_t)b.i64_1("occ_seed", 17321);
    // convection
    s.conv_p = b.f64_1("conv_p", 0.0);
    s.conv_dist = (int)b.f64_1("conv_distance", -1.0);
    s.conv_seed = (uint32_t)b.i64_1("conv_seed", 0);
    // reward
    s.rw = vec(b.f64("reward_scalars"), 8);
    s.e_wd = vec(b.f64("elec_weekday_price"), 24);
    s.e_we = vec(b.f64("elec_weekend_price"), 24);
    s.e_c = vec(b.f64("elec_carbon_rate"), 24);
    s.g_p = vec(b.f64("gas_month_price"), 12);
    if (s.rw.size() != 8 || s.e_wd.size() != 24 || s.e_we.size() != 24 || s.e_c.size() != 24 || s.g_p.size() != 12)
        return "reward tables missing";
    s.gas_carbon = b.f64_1("gas_carbon_rate", 0.0);
    // initial state in the device orders
    const double* ti = b.f64("temp_init");
    const double* mi = b.f64("mass_temp_init");
    NEED(ti, "temp_init"); NEED(mi, "mass_temp_init");
    s.temp_init.resize(g.ncv);
    for (int q = 0; q < g.ncv; q++) s.temp_init[q] = ti[g.cell_of_pos[q]];
    s.mass_init.resize(n);
    for (int t = 0; t < n; t++) s.mass_init[g.row_of_solved[t]] = mi[t];
    (void)solved;
    return "";
}

int solve_ring_stages(int n, int B, size_t smem_cap) {
    const size_t kStatic = 512;   // the solve kernel's static shared memory, with margin
    for (int r = kStagesMax; r >= kStagesMin; r--)
        if (solve_smem_bytes(n, B, r) + kStatic <= smem_cap) return r;
    return 0;
}

// The terms of every row sorted by the depth of their source row in the
// sweep's dependency graph (rows with no terms: depth 0; a row: one more than
// its deepest source), stable otherwise: a row can then start with the terms
// whose sources finish first. Changes the summation order, so only for the
// builds held to a tolerance.
static std::vector<std::vector<std::pair<int, double>>> terms_by_depth(
    const std::vector<std::vector<std::pair<int, double>>>& t, bool backward) {
    const int n = (int)t.size();
    std::vector<int> depth(n, 0);
    for (int p = 0; p < n; p++) {
        const int i = backward ? n - 1 - p : p;
        int d = 0;
        for (const auto& x : t[i]) d = std::max(d, depth[x.first] + 1);
        depth[i] = d;
    }
    auto out = t;
    for (auto& r : out)
        std::stable_sort(r.begin(), r.end(), [&](const std::pair<int, double>& a, const std::pair<int, double>& b) {
            return depth[a.first] < depth[b.first];
        });
    return out;
}

std::string build_sweeps(HostGroup& g, int ring_stages, bool tolerant) {
    // the corrected and folded builds: the L sweep's terms by source depth, and
    // U rows finished with a multiplication by the diagonal's reciprocal
    // (rounded once, here) instead of a division
    std::string e = build_sweep(g.n, tolerant ? terms_by_depth(g.lt, false) : g.lt, false, g.udiag, ring_stages, g.fwd);
    if (e.empty()) {
        std::vector<double> d = g.udiag;
        if (tolerant)
            for (double& x : d) x = 1.0 / x;
        e = build_sweep(g.n, g.ut, true, d, ring_stages, g.bwd);
    }
    return e;
}

// Folded air side (the reference GPU backend's fast path,
// complete_port/gpu/smart_buildings.cu:686-826 and sb_gpu_lusolve.cuh:190-259):
// with z = L^-1 b the first solve's forward half, the sensed values are
// sensed . U^-1 z = R z with R = sensed U^-1 (k x n, row r = U^-T sensed_r),
// and the corrected field is U^-1 (z + Z q) with Z = L^-1 applied (n x k), so
// one L sweep and one U sweep replace the exact build's two pairs. Both
// matrices are formed here in row order from the same sweep terms the device
// replays; exact zeros are dropped.
std::string build_fold(HostGroup& g) {
    const int n = g.n, k = g.k;
    g.zr_p.assign(n + 1, 0);
    g.zr_col.clear();
    g.zr_x.clear();
    g.rs_p.assign(k + 1, 0);
    g.rs_pos.clear();
    g.rs_x.clear();
    if (k == 0) return "";
    // Z, column by column (forward substitution with the L sweep's terms)
    std::vector<std::vector<std::pair<int32_t, double>>> zrows(n);
    std::vector<double> a(n);
    for (int c = 0; c < k; c++) {
        std::fill(a.begin(), a.end(), 0.0);
        for (int i = 0; i < n; i++)
            for (int q = g.ap_rp[i]; q < g.ap_rp[i + 1]; q++)
                if (g.ap_col[q] == c) a[i] += g.ap_x[q];
        for (int i = 0; i < n; i++) {
            double v = a[i];
            for (const auto& t : g.lt[i]) v -= t.second * a[t.first];
            a[i] = v;
            if (v != 0.0) zrows[i].push_back({c, v});
        }
    }
    for (int i = 0; i < n; i++) {
        for (const auto& t : zrows[i]) {
            g.zr_col.push_back(t.first);
            g.zr_x.push_back(t.second);
        }
        g.zr_p[i + 1] = (int32_t)g.zr_col.size();
    }
    // R, sensor by sensor (forward substitution with U^T, pushed over U's rows)
    std::vector<double> w(n);
    for (int r = 0; r < k; r++) {
        std::fill(w.begin(), w.end(), 0.0);
        for (int q = g.sn_p[r]; q < g.sn_p[r + 1]; q++) w[g.sn_pos[q]] += g.sn_x[q];
        for (int i = 0; i < n; i++) {
            if (w[i] == 0.0) continue;
            const double ri = w[i] / g.udiag[i];
            w[i] = ri;
            for (const auto& t : g.ut[i]) w[t.first] -= t.second * ri;
        }
        for (int i = 0; i < n; i++)
            if (w[i] != 0.0) {
                g.rs_pos.push_back(i);
                g.rs_x.push_back(w[i]);
            }
        g.rs_p[r + 1] = (int32_t)g.rs_pos.size();
    }
    return "";
}

}  // namespace sbenv
