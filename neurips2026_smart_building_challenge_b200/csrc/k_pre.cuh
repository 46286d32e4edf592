// Pre-solve stage of one env step: action decode, actuator routing, zone
// sensing, thermostats, VAV/AHU air flows, reheat, and the per-zone applied
// heat the forcing needs. One CTA per env; order-dependent sums run on one
// thread in the reference's order, independent per-VAV work runs in parallel.
//
// Reference: complete_port/pufferlib_cpu_env.h:218-234 (clamp + decode),
// complete_port/csim/sb_sim.c:220-244 (apply), :246-355 (device models,
// thermostat), :357-457 (sb_sim_step_pre).
#pragma once
#include "dev_util.cuh"

namespace sbenv {

constexpr double RHO_AIR = 1.2;
constexpr double CP_AIR = 1006.0;
constexpr double RHO_W = 1000.0;
constexpr double CP_W = 4180.0;
constexpr double GRAV = 9.8;
constexpr double PA_PER_BAR = 100000.0;
enum { M_OFF = 0, M_HEAT = 1, M_COOL = 2, M_PASSIVE = 3 };

struct EnvView {   // one env's state blocks
    double* D;
    int32_t* I;
    const StateLayout* L;
    __device__ double& d(int off, int i = 0) const { return D[off + i]; }
    __device__ int32_t& iv(int off, int i = 0) const { return I[off + i]; }
};

__device__ __forceinline__ double ahu_static_p(const EnvView& v, const ScnDev& s, int a) {
    if (v.iv(v.L->ahu_run, a) != 1) return 0.0;
    const double sp = v.d(v.L->ahu_fan, a), mn = s.ahu_c[a * 9 + 2];
    return sp > mn ? sp : mn;
}
__device__ __forceinline__ double vav_unrestricted(const EnvView& v, const ScnDev& s, int vv) {
    const double* vc = &s.vav_c[vv * 9];
    const double stat = ahu_static_p(v, s, s.v_ahu[vv]);
    const double d = dmul(dmul(v.d(v.L->v_damp, vv), vc[0]), sqrt(ddiv(stat, vc[4])));
    return d > 0.00001 ? d : 0.00001;
}
__device__ __forceinline__ double pump_dp(const EnvView& v) {
    if (v.iv(v.L->pump_run) != 1) return 0.0;
    return ddiv(dmul(GRAV * RHO_W, v.d(v.L->pump_head)), PA_PER_BAR);
}
__device__ __forceinline__ double water_flow(const EnvView& v, const ScnDev& s) {
    const double ff = v.d(v.L->ff_sum);
    const double den = dadd(1.0, dmul(dmul(ff, ff), s.header_res));
    return ddiv(dmul(ff, sqrt(ddiv(pump_dp(v), den))), 3600.0);
}
// reheat_energy (sb_sim.c:289-314); vd = vav_flow_demand of this VAV
__device__ inline double reheat_energy(const EnvView& v, const ScnDev& s, int vv, double sat, double iwt,
                                       double vd) {
    const double air_cap = dmul(CP_AIR * RHO_AIR, vd);
    double eff;
    if (air_cap <= 0.0) {
        eff = 0.0;
    } else {
        const double ffs = v.d(v.L->ff_sum);
        double wf = 0.0;
        if (ffs != 0.0) wf = dmul(water_flow(v, s), ddiv(dmul(v.d(v.L->v_reh, vv), s.vav_c[vv * 9 + 1]), ffs));
        eff = ddiv(dmul(CP_W * RHO_W, wf), air_cap);
        if (eff > 1.0) eff = 1.0;
        const double gap = dsub(iwt, sat);
        if (gap > 0.0) {
            const double head = dsub(s.vav_c[vv * 9 + 3], sat);
            if (head <= 0.0) eff = 0.0;
            else {
                const double hr = ddiv(head, gap);
                eff = eff < hr ? eff : hr;
            }
        }
    }
    return dmul(dmul(dmul(dmul(eff, CP_AIR), RHO_AIR), vd), dsub(iwt, sat));
}

// Native value of action i from the framework's actions of one env
// (pufferlib_cpu_env.h:218-234, sb_sim.c:557-576): continuous slots clamped to
// [-1, 1] and mapped in float, discrete slots (+1 iff the action is 1.0) in double.
__device__ inline double decode_native(const ScnDev& s, int i, const float* act) {
    const int slot = s.a_slot[i];   // position in the packed continuous / discrete block
    if (s.a_disc[i]) {
        const double dv = (double)act[kCont + slot];
        const double merged = dv == 1.0 ? 1.0 : -1.0;
        return dadd(dmul(ddiv(dsub(merged, s.a_mnr[i]), dsub(s.a_mxr[i], s.a_mnr[i])), dsub(s.a_mx[i], s.a_mn[i])),
                    s.a_mn[i]);
    }
    double a = (double)act[slot];
    a = a > 1.0 ? 1.0 : (a < -1.0 ? -1.0 : a);
    const float m = (float)a;
    const float span_in = (float)dsub(s.a_mxr[i], s.a_mnr[i]);
    const float span_out = (float)dsub(s.a_mx[i], s.a_mn[i]);
    const float r =
        __fadd_rn(__fmul_rn(__fdiv_rn(__fsub_rn(m, (float)s.a_mnr[i]), span_in), span_out), (float)s.a_mn[i]);
    return (double)r;
}

// Field-averaged zone temperatures (sb_sim.c:149-160) from an extended-order
// field in global memory: one thread per zone, cells fetched eight at a time,
// summed in the reference's order.
__device__ inline void zone_means(const GroupDev& g, const ScnDev& s, const double* T, double* zavg) {
    for (int z = threadIdx.x; z < s.nz; z += blockDim.x) {
        const int rm = s.proom[z];
        const int a = g.room_off[rm], b = g.room_off[rm + 1];
        double sum = 0.0;
        for (int t = a; t < b; t += 8) {
            double tv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) tv[u] = t + u < b ? T[g.room_pos[t + u]] : 0.0;
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (t + u < b) sum = dadd(sum, tv[u]);
        }
        zavg[z] = ddiv(sum, (double)(b - a));
    }
}

// VAV area + sensing (sb_sim.c:163-175), one thread per VAV.
__device__ inline void vav_sensing(const ScnDev& s, const double* zavg, double* area_out, double* sense_out) {
    for (int v = threadIdx.x; v < s.nv; v += blockDim.x) {
        double area = 0.0, wt = 0.0;
        for (int t = s.vz_off[v]; t < s.vz_off[v + 1]; t++) {
            const int z = s.vz_idx[t];
            area = dadd(area, s.zarea[z]);
            wt = dadd(wt, dmul(zavg[z], s.zarea[z]));
        }
        area_out[v] = area;
        sense_out[v] = area > 0.0 ? ddiv(wt, area) : 0.0;
    }
}

__device__ __forceinline__ void mode_default(int& mode, double zt, double hsp, double csp) {
    const double mid = dadd(dmul(0.5, dsub(csp, hsp)), hsp);
    if (zt < hsp) mode = M_HEAT;
    else if (zt > csp) mode = M_COOL;
    else if (zt < mid && mode == M_HEAT) mode = M_HEAT;
    else if (zt > mid && mode == M_COOL) mode = M_COOL;
    else mode = M_OFF;
}

// One CTA per env: env blockIdx.x (first < 0) or dense_order[first + blockIdx.x]
// (one class's envs)
__global__ void __launch_bounds__(128) k_pre(const StepCtx* __restrict__ ctx, int first) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int env = first < 0 ? (int)blockIdx.x : ctx->dense_order[first + blockIdx.x];
    const EnvIndex ei = ctx->envs[env];
    const GroupDev& g = ctx->groups[ei.group];
    const ScnDev& s = ctx->scns[ei.scn];
    const StateLayout& L = ctx->lay;
    const int tid = threadIdx.x;
    const int na = s.na, nv = s.nv, nz = s.nz, k = s.k;
    // the env's state blocks are worked on in shared memory (the ordered loops
    // below read and update them element by element) and written back at the end
    double* Dg = ctx->Dst + (size_t)env * L.nd;
    int32_t* Ig = ctx->Ist + (size_t)env * L.ni;
    double* Ds = reinterpret_cast<double*>(smem);          // [nd]
    int32_t* Is = reinterpret_cast<int32_t*>(Ds + L.nd);   // [ni]
    block_copy(Ds, Dg, L.nd);
    block_copy(Is, Ig, L.ni);
    EnvView v{Ds, Is, &ctx->lay};
    double* zavg = reinterpret_cast<double*>(Is + L.ni);   // [nz] (ni is a multiple of 4)
    double* zq = zavg + nz;                           // [nz]
    double* unr = zq + nz;                            // [nv]
    double* sv = unr + nv;                            // [na] supply air temperature
    double* demand = sv + na;                         // [na]
    double* rw = demand + na;                         // [k]
    double* fdv = rw + k;                             // [k]

    __syncthreads();
    const int kk = v.iv(L.cal);   // calendar row of this step
    const double ambient = s.amb[kk];
    const int comfort = s.s_comf[kk] != 0.0;

    // ---- decode + apply (pufferlib_cpu_env.h:218-234, sb_sim.c:557-576, :220-244) ----
    // Actuator targets are unique per blob (checked on the host), so actions apply in parallel.
    const float* act = ctx->actions + (size_t)env * kAct;
    for (int i = tid; i < s.nact; i += blockDim.x) {
        const double val = decode_native(s, i, act);
        const int idx = s.a_idx[i], ac = s.a_act[i];
        if (s.a_kind[i] == 0) {
            if (ac == 0) v.d(L.ahu_sat, idx) = val;
            else if (ac == 1) v.d(L.ahu_fan, idx) = val;
            else if (ac == 2) {
                const double hi = s.ahu_c[idx * 9 + 3];
                v.d(L.ahu_rec, idx) = val < 0.0 ? 0.0 : (val > hi ? hi : val);
            } else v.iv(L.ahu_run, idx) = val == 1.0 ? 1 : 0;
        } else if (s.a_kind[i] == 1) {
            const double c01 = val < 0.0 ? 0.0 : (val > 1.0 ? 1.0 : val);
            if (ac == 0) { v.d(L.v_dcmd, idx) = c01; v.iv(L.v_dset, idx) = 1; }
            else { v.d(L.v_rcmd, idx) = c01; v.iv(L.v_rset, idx) = 1; }
        } else {
            if (ac == 0) v.d(L.b_sp) = val;
            else if (ac == 1) v.d(L.pump_head) = ddiv(val, ddiv(GRAV * RHO_W, PA_PER_BAR));
            else { const int on = val == 1.0 ? 1 : 0; v.iv(L.hws_run) = on; v.iv(L.pump_run) = on; }
        }
    }
    // ---- zone means of the field: the previous k_post (or the reset) computed
    // them from this same field (sb_sim.c:149-160) and left them in the state ----
    const double* Tg = g.T + (size_t)(env - g.env0) * g.ncv;
    __syncthreads();
    if (tid == 0) v.iv(L.hws_req) = nv;
    for (int z = tid; z < nz; z += blockDim.x) zavg[z] = v.d(L.zavg, z);
    __syncthreads();
    // ---- VAV sensing, thermostat, damper/reheat (sb_sim.c:368-384, :316-355) ----
    for (int vv = tid; vv < nv; vv += blockDim.x) {
        double area = 0.0, wt = 0.0;
        for (int t = s.vz_off[vv]; t < s.vz_off[vv + 1]; t++) {
            const int z = s.vz_idx[t];
            area = dadd(area, s.zarea[z]);
            wt = dadd(wt, dmul(zavg[z], s.zarea[z]));
        }
        v.d(L.v_area, vv) = area;
        if (area <= 0.0) { v.d(L.v_sense, vv) = 0.0; continue; }
        const double sensing = ddiv(wt, area);
        v.d(L.v_sense, vv) = sensing;
        const double* c = &s.vav_c[vv * 9];
        const double hsp = s.s_heat[kk], csp = s.s_cool[kk];
        v.d(L.v_hsp, vv) = hsp;
        v.d(L.v_csp, vv) = csp;
        int mode = v.iv(L.v_mode, vv);
        if (comfort) mode_default(mode, sensing, hsp, csp);
        else if (v.iv(L.v_prev, vv) && s.s_comf[kk - 1] != 0.0) mode = M_PASSIVE;
        else if (mode == M_PASSIVE && sensing > hsp && sensing < csp) mode = M_PASSIVE;
        else mode_default(mode, sensing, hsp, csp);
        v.iv(L.v_mode, vv) = mode;
        v.iv(L.v_prev, vv) = 1;
        double damper, reheat;
        if (mode == M_HEAT) { damper = 1.0; reheat = 1.0; }
        else if (mode == M_COOL) { damper = 1.0; reheat = 0.0; }
        else { damper = c[2]; reheat = 0.0; }
        if (v.iv(L.v_dset, vv)) damper = v.d(L.v_dcmd, vv);
        if (v.iv(L.v_rset, vv)) reheat = v.d(L.v_rcmd, vv);
        v.d(L.v_damp, vv) = damper > c[2] ? damper : c[2];
        v.d(L.v_reh, vv) = reheat;
    }
    __syncthreads();
    // ---- ordered accumulations (sb_sim.c:367-392) ----
    if (!s.tmean_needed) {
        // every AHU sees VAV area (checked on the host): one thread per AHU sums
        // its VAVs in ascending order, one thread the reheat flow factor
        if (tid < na) {
            const int a = tid;
            double ws = 0.0, at = 0.0;
            for (int q = s.av_off[a]; q < s.av_off[a + 1]; q++) {
                const int vv = s.av_idx[q];
                const double area = v.d(L.v_area, vv);
                if (area <= 0.0) continue;
                ws = dadd(ws, dmul(v.d(L.v_sense, vv), area));
                at = dadd(at, area);
            }
            const double recirc = ddiv(ws, at);
            const double rec = v.d(L.ahu_rec, a);
            const double mixed = dadd(dmul(rec, recirc), dmul(dsub(1.0, rec), ambient));
            sv[a] = (mixed > v.d(L.ahu_sat, a) && v.iv(L.ahu_run, a) == 1) ? v.d(L.ahu_sat, a) : mixed;
            v.d(L.ahu_flow, a) = 0.0;
            v.iv(L.ahu_creq, a) = 0;
        }
        if (tid == 64) {
            double ff = 0.0;
            for (int vv = 0; vv < nv; vv++) ff = dadd(ff, dmul(v.d(L.v_reh, vv), s.vav_c[vv * 9 + 1]));
            v.d(L.ff_sum) = ff;
        }
    } else if (tid == 0) {
        double ws[kMaxAhu], at[kMaxAhu];
        for (int a = 0; a < na; a++) { ws[a] = 0.0; at[a] = 0.0; }
        for (int vv = 0; vv < nv; vv++) {
            const double area = v.d(L.v_area, vv);
            if (area <= 0.0) continue;
            const int a = s.v_ahu[vv];
            ws[a] = dadd(ws[a], dmul(v.d(L.v_sense, vv), area));
            at[a] = dadd(at[a], area);
        }
        double tmean = 0.0;
        if (s.tmean_needed) {
            for (int p = 0; p < g.ncv; p++) tmean = dadd(tmean, Tg[g.pos_of_cell[p]]);
            tmean = ddiv(tmean, (double)g.ncv);
        }
        for (int a = 0; a < na; a++) {
            const double recirc = at[a] > 0.0 ? ddiv(ws[a], at[a]) : tmean;
            const double rec = v.d(L.ahu_rec, a);
            const double mixed = dadd(dmul(rec, recirc), dmul(dsub(1.0, rec), ambient));
            sv[a] = (mixed > v.d(L.ahu_sat, a) && v.iv(L.ahu_run, a) == 1) ? v.d(L.ahu_sat, a) : mixed;
            v.d(L.ahu_flow, a) = 0.0;
            v.iv(L.ahu_creq, a) = 0;
            demand[a] = 0.0;
        }
        double ff = 0.0;
        for (int vv = 0; vv < nv; vv++) ff = dadd(ff, dmul(v.d(L.v_reh, vv), s.vav_c[vv * 9 + 1]));
        v.d(L.ff_sum) = ff;
    }
    __syncthreads();
    for (int vv = tid; vv < nv; vv += blockDim.x) unr[vv] = vav_unrestricted(v, s, vv);
    __syncthreads();
    if (tid < na) {   // each AHU's demand over its VAVs, ascending
        double d = 0.0;
        for (int q = s.av_off[tid]; q < s.av_off[tid + 1]; q++) d = dadd(d, unr[s.av_idx[q]]);
        demand[tid] = d;
    }
    __syncthreads();
    for (int vv = tid; vv < nv; vv += blockDim.x) {
        const int a = s.v_ahu[vv];
        const double d = demand[a];
        if (d > 0.0) {
            const double r = ddiv(s.ahu_c[a * 9 + 1], d);
            v.d(L.v_ratio, vv) = r < 1.0 ? r : 1.0;
        } else {
            v.d(L.v_ratio, vv) = 1.0;
        }
    }
    for (int z = tid; z < nz; z += blockDim.x) zq[z] = 0.0;
    __syncthreads();
    // ---- coupled columns (sb_sim.c:408-436): per-column values in parallel ----
    const double b_cur = v.d(L.b_cur);
    for (int col = tid; col < k; col += blockDim.x) {
        const int vv = s.coupled[col];
        if (v.d(L.v_area, vv) <= 0.0) {
            v.d(L.ag, col) = 0.0;
            v.d(L.aT, col) = 0.0;
            rw[col] = 0.0;
            fdv[col] = 0.0;
            continue;
        }
        const double sat = sv[s.v_ahu[vv]];
        v.d(L.aT, col) = sat;
        v.d(L.coil, col) = sat;
        const double vd = dmul(unr[vv], v.d(L.v_ratio, vv));
        rw[col] = reheat_energy(v, s, vv, sat, b_cur, vd);
        fdv[col] = vd;
        const bool flows = v.d(L.v_damp, vv) > 0.0 && s.vav_c[vv * 9] > 0.0;
        v.d(L.ag, col) = flows ? dmul(dmul(vd, RHO_AIR), CP_AIR) : 0.0;
    }
    __syncthreads();
    // ... and their order-dependent sums: each zone's heat over its columns,
    // each AHU's flow over its columns, the reheat total over all columns, each
    // on one thread in ascending column order
    for (int z = tid; z < nz; z += blockDim.x) {
        double q = zq[z];
        for (int e = s.zc_off[z]; e < s.zc_off[z + 1]; e++) {
            const int col = s.zc_col[e];
            const int vv = s.coupled[col];
            const double area = v.d(L.v_area, vv);
            if (area <= 0.0 || !(v.d(L.v_damp, vv) > 0.0 && s.vav_c[vv * 9] > 0.0)) continue;
            q = dadd(q, ddiv(dmul(rw[col], s.zarea[z]), area));
        }
        zq[z] = q;
    }
    const int last = (int)blockDim.x - 1;
    if (tid == last) {
        double rsum = 0.0;
        for (int col = 0; col < k; col++)
            if (v.d(L.v_area, s.coupled[col]) > 0.0) rsum = dadd(rsum, rw[col]);
        v.d(L.reheat_w) = rsum;
    }
    if (tid < last && tid >= last - na) {
        const int a = last - 1 - tid;
        const double mf = s.ahu_c[a * 9 + 1];
        double f = v.d(L.ahu_flow, a);
        int creq = v.iv(L.ahu_creq, a);
        for (int e = s.ac_off[a]; e < s.ac_off[a + 1]; e++) {
            const int col = s.ac_col[e];
            if (v.d(L.v_area, s.coupled[col]) <= 0.0) continue;
            const double fd = fdv[col];
            if (fd > 0.0) {
                f = dadd(f, fd);
                if (f > mf) f = mf;
                creq += 1;
            }
        }
        v.d(L.ahu_flow, a) = f;
        v.iv(L.ahu_creq, a) = creq;
    }
    __syncthreads();
    // ---- internal + occupant gains, per-cell applied heat (sb_sim.c:438-455) ----
    const double* Vin = v.D + L.V;
    const double frac = comfort ? 1.0 : s.standby;
    const double wpc = dmul(dmul(s.internal_w, s.cv_area), frac);
    for (int z = tid; z < nz; z += blockDim.x) {
        double q = zq[z];
        const double cells = (double)s.room_ncell[z];
        if (s.internal_w > 0.0) q = dadd(q, dmul(wpc, cells));
        if (s.occ_w > 0.0) q = dadd(q, dmul(Vin[z], s.occ_w));
        v.d(L.qdiv, z) = ddiv(q, cells);
    }
    __syncthreads();
    for (int i = tid; i < L.nd; i += blockDim.x) Dg[i] = Ds[i];
    for (int i = tid; i < L.ni; i += blockDim.x) Ig[i] = Is[i];
}

}  // namespace sbenv
