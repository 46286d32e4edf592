// Post-solve stage of one env step: convection permutation, boiler return and
// setpoint ramp, observation, reward, episode bookkeeping and the in-step
// restart at the episode length. One CTA per env.
//
// Reference: complete_port/csim/sb_sim.c:459-521 (post step), sb_obs.c:11-64,
// sb_reward.c:12-155, complete_port/pufferlib_cpu_env.h:236-256 (observation,
// occupancy, reward, terminal and restart order), complete_port/gpu/
// smart_buildings.cu:1936-2050 (device episode log and live sums).
#pragma once
#include "../../include/sbenv.h"
#include "k_pre.cuh"

namespace sbenv {

__device__ inline double obs_field(const EnvView& v, const ScnDev& s, int kind, int idx, int id, int j) {
    const StateLayout& L = *v.L;
    if (kind == 0) {
        switch (id) {
            case 0: return (double)v.iv(L.ahu_creq, idx);
            case 1: return ahu_static_p(v, s, idx);
            case 2: return v.iv(L.ahu_run, idx) == 1 ? v.d(L.ahu_flow, idx) : 0.0;
            case 3: return v.d(L.ahu_sat, idx);
            case 4: return (double)v.iv(L.ahu_run, idx);
            case 5: return ddiv(v.d(L.ahu_flow, idx), s.ahu_c[idx * 9 + 1]);
            case 6: return dmul(dsub(1.0, v.d(L.ahu_rec, idx)), v.d(L.ahu_flow, idx));
            case 7: return (double)v.iv(L.ahu_run, idx);
            case 8: return v.d(L.ahu_rec, idx);
            default: return s.amb[j];
        }
    }
    if (kind == 1) {
        switch (id) {
            case 0: return v.d(L.v_reh, idx);
            case 1: return v.d(L.v_damp, idx);
            case 2: return s.vav_c[idx * 9];
            case 3: return v.d(L.v_csp, idx);
            case 4: return v.d(L.v_hsp, idx);
            default: return v.d(L.v_sense, idx);
        }
    }
    switch (id) {
        case 0: case 2: return pump_dp(v);
        case 1: return v.d(L.b_cur);
        case 3: case 5: return (double)v.iv(L.hws_run);
        case 4: return (double)v.iv(L.hws_req);
        default: return v.d(L.b_sp);
    }
}

// Observation at calendar index j with occupancy V (sb_obs.c:49-64). Only the
// first n_dev + n_aux floats are written; the zero tail is set at reset.
__device__ inline void write_obs(const EnvView& v, const ScnDev& s, int j, const double* V, float* out) {
    const int tid = threadIdx.x;
    for (int i = tid; i < s.n_dev; i += blockDim.x) {
        const double val = obs_field(v, s, s.f_kind[i], s.f_idx[i], s.f_id[i], j);
        const double var = s.f_var[i];
        const float v32 = (float)val;
        out[i] = (float)(var > 0.0 ? ddiv(dsub((double)v32, s.f_mean[i]), sqrt(var)) : 0.0);
    }
    const double* aux = s.aux + (size_t)j * (s.n_aux - 1);
    for (int q = tid; q < s.n_aux - 1; q += blockDim.x) out[s.n_dev + q] = (float)aux[q];
    if (tid < 32) {   // warp 0: the zones' occupancy loaded 32 at a time, summed in order on lane 0
        double occ = 0.0;
        for (int base = 0; base < s.nz; base += 128) {
            double vz[4];
#pragma unroll
            for (int c = 0; c < 4; c++) vz[c] = base + 32 * c + tid < s.nz ? V[base + 32 * c + tid] : 0.0;
#pragma unroll
            for (int c = 0; c < 4; c++)
                for (int q = 0; q < 32 && base + 32 * c + q < s.nz; q++)
                    occ = dadd(occ, __shfl_sync(0xffffffffu, vz[c], q));
        }
        if (tid == 0) out[s.n_dev + s.n_aux - 1] = (float)(int)occ;
    }
}

// Reset of one env's simulator state (sb_sim.c:177-218); the caller syncs.
__device__ inline void reset_state(const EnvView& v, const ScnDev& s) {
    const StateLayout& L = *v.L;
    for (int a = threadIdx.x; a < s.na; a += blockDim.x) {
        const double* c = &s.ahu_c[a * 9];
        v.iv(L.ahu_run, a) = (int)c[8];
        v.d(L.ahu_rec, a) = c[0];
        v.d(L.ahu_sat, a) = c[6];
        v.d(L.ahu_fan, a) = c[7];
        v.d(L.ahu_flow, a) = 0.0;
        v.iv(L.ahu_creq, a) = 0;
    }
    for (int vv = threadIdx.x; vv < s.nv; vv += blockDim.x) {
        const double* c = &s.vav_c[vv * 9];
        v.d(L.v_damp, vv) = c[7];
        v.d(L.v_reh, vv) = c[8];
        v.d(L.v_ratio, vv) = 1.0;
        v.d(L.v_hsp, vv) = c[5];
        v.d(L.v_csp, vv) = c[6];
        v.iv(L.v_mode, vv) = M_OFF;
        v.iv(L.v_prev, vv) = 0;
        v.iv(L.v_dset, vv) = 0;
        v.iv(L.v_rset, vv) = 0;
        v.d(L.v_dcmd, vv) = 0.0;
        v.d(L.v_rcmd, vv) = 0.0;
    }
    if (threadIdx.x == 0) {
        v.d(L.ff_sum) = 0.0;
        v.iv(L.hws_req) = 0;
        v.iv(L.hws_run) = 1;
        v.iv(L.pump_run) = 1;
        v.d(L.b_sp) = s.boiler[0];
        v.d(L.b_ret) = s.boiler[1];
        v.d(L.b_cur) = s.boiler[0];
        v.d(L.b_step) = 0.0;
        v.iv(L.step) = 0;
    }
}

// The consumer's side of a restart's random-start draw: the env's episode
// offset, its Env record and the start-day statistics (smart_buildings.cu:1643-1657).
__device__ inline void take_start(const StepCtx* ctx, int env, int scn, const EnvView& v, int off,
                                  unsigned long long rng) {
    const StateLayout& L = ctx->lay;
    v.iv(L.off) = off;
    v.iv(L.cal) = off;
    Env* er = reinterpret_cast<Env*>(ctx->env_records) + env;
    er->start_offset = off;
    er->start_day = off / kStepsPerDay;
    if (ctx->random_start) {
        ctx->env_rng[env] = rng;
        er->start_rng = rng;
        atomicAdd(&ctx->start_draws[((size_t)scn * 2 + (er->start_draws == 0 ? 0 : 1)) * kStartDays + off / kStepsPerDay],
                  1.0);
        er->start_draws += 1;
    }
}

// Shared-memory layout of k_post / k_reset: staging, zone scratch. Kept small
// (the state and the field stay in global memory) so that seven 128-thread
// CTAs fit on an SM and every env's CTA is resident in one wave.
struct PostShared {
    double *stage, *zavg, *zterm, *zdev, *vws, *varea;
    double* ahu;   // [3][kMaxAhu] per-AHU reward terms: intake, exhaust, cooling
    double* sc;    // [kPostScalars] reward scalars handed to the final thread
};
constexpr int kPostScalars = 10;   // [0..7] reward scalars, [8] the done flag
__host__ __device__ constexpr size_t post_smem_doubles(int ncv, int nz, int nv) {
    return (size_t)ncv + 3 * (size_t)nz + 2 * (size_t)nv + 3 * kMaxAhu + kPostScalars;
}
__device__ inline PostShared post_shared(uint8_t* smem, int ncv, int nz, int nv) {
    PostShared p;
    p.stage = reinterpret_cast<double*>(smem);
    p.zavg = p.stage + ncv;
    p.zterm = p.zavg + nz;
    p.zdev = p.zterm + nz;
    p.vws = p.zdev + nz;
    p.varea = p.vws + nv;
    p.ahu = p.varea + nv;
    p.sc = p.ahu + 3 * kMaxAhu;
    return p;
}

// Restart one env in place: state, field, interior mass, sensing, reset
// observation with the primed occupancy (pufferlib_cpu_env.h:187-208), at the
// new episode's calendar offset off (random_start; else 0).
__device__ inline void restart_env(const StepCtx* ctx, int env, const GroupDev& g, const ScnDev& s,
                                   const EnvView& v, PostShared& p, const double* Vprime, const double* Vzero,
                                   int off, unsigned long long rng) {
    const StateLayout& L = ctx->lay;
    const int local = env - g.env0;
    reset_state(v, s);
    if (threadIdx.x == 0) take_start(ctx, env, ctx->envs[env].scn, v, off, rng);
    double* Tg = g.T + (size_t)local * g.ncv;
    double* Mg = g.M + (size_t)local * g.n;
    block_copy(Tg, s.temp_init, g.ncv);
    block_copy(Mg, s.mass_init, g.n);
    __syncthreads();
    zone_means(g, s, s.temp_init, p.zavg);
    __syncthreads();
    vav_sensing(s, p.zavg, v.D + L.v_area, v.D + L.v_sense);
    for (int z = threadIdx.x; z < s.nz; z += blockDim.x) v.d(L.zavg, z) = p.zavg[z];
    __syncthreads();
    float* o = ctx->obs + (size_t)env * kObs;
    write_obs(v, s, off, Vprime, o);
    for (int z = threadIdx.x; z < s.nz; z += blockDim.x) v.d(L.V, z) = Vzero[z];
    __syncthreads();
}

// One CTA per env: env blockIdx.x (first < 0) or dense_order[first + blockIdx.x]
// (one class's envs)
__global__ void __launch_bounds__(128) k_post(const StepCtx* __restrict__ ctx, int first) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int env = first < 0 ? (int)blockIdx.x : ctx->dense_order[first + blockIdx.x];
    const EnvIndex ei = ctx->envs[env];
    const GroupDev& g = ctx->groups[ei.group];
    const ScnDev& s = ctx->scns[ei.scn];
    const StateLayout& L = ctx->lay;
    const int tid = threadIdx.x;
    const int nz = s.nz, nv = s.nv, na = s.na, k = s.k;
    PostShared p = post_shared(smem, g.ncv, nz, nv);
    EnvView v{ctx->Dst + (size_t)env * L.nd, ctx->Ist + (size_t)env * L.ni, &ctx->lay};
    const int local = env - g.env0;
    double* Tg = g.T + (size_t)local * g.ncv;

    // this transition's random inputs (produced one step ahead): slot tseq & 1
    const int slot = v.iv(L.tseq) & 1;
    const size_t vslot = ((size_t)slot * ctx->n_ostreams + ei.ostream) * ctx->nz_max;
    // ---- convection (sb_sim.c:489): apply this step's permutation to the
    // field in global memory, the moved values staged first ----
    const int npairs = s.conv_npairs[slot];
    const int32_t* pairs = s.conv_pairs + (size_t)slot * s.conv_stride;
    for (int q = tid; q < npairs; q += blockDim.x) p.stage[q] = Tg[pairs[2 * q + 1]];
    __syncthreads();
    for (int q = tid; q < npairs; q += blockDim.x) Tg[pairs[2 * q]] = p.stage[q];
    // ---- boiler return and setpoint ramp (sb_sim.c:491-521) ----
    const int kk = v.iv(L.step);
    const int cal = v.iv(L.cal);
    if (tid == 0) {
        const double wcap = dmul(CP_W * RHO_W, water_flow(v, s));
        if (wcap > 0.0 && k > 0) {
            const double supply = v.d(L.b_cur);
            const double rsum = v.d(L.reheat_w);
            double rt = dsub(supply, ddiv(rsum, wcap));
            double at = v.d(L.coil, 0);
            for (int c = 1; c < k; c++) {
                const double cc = v.d(L.coil, c);
                if (rsum >= 0.0) { if (cc < at) at = cc; }
                else { if (cc > at) at = cc; }
            }
            const double lo = supply < at ? supply : at, hi = supply > at ? supply : at;
            if (rt < lo) rt = lo;
            if (rt > hi) rt = hi;
            v.d(L.b_ret) = rt;
        }
        const double begin = v.d(L.b_cur), sp = v.d(L.b_sp), dtm = ddiv(s.dt, 60.0);
        double cur;
        if (sp > begin) {
            const double x = dadd(begin, dmul(s.boiler[2], dtm));
            cur = x < sp ? x : sp;
        } else if (sp < begin) {
            const double x = dsub(begin, dmul(s.boiler[3], dtm));
            cur = x > sp ? x : sp;
        } else {
            cur = sp;
        }
        v.d(L.b_cur) = cur;
        v.d(L.b_step) = dsub(cur, begin);
        v.iv(L.step) = kk + 1;
        v.iv(L.cal) = cal + 1;
        v.iv(L.tseq) += 1;
    }
    __syncthreads();
    const int j = kk + 1;     // episode step after this transition
    const int jc = cal + 1;   // its calendar row: observation and reward index
    const double* Vin = v.D + L.V;
    const double* Vst = ctx->V_step + vslot;

    // ---- observation at ts_j with the interval that just ran (pufferlib_cpu_env.h:237-239) ----
    float* o = ctx->obs + (size_t)env * kObs;
    write_obs(v, s, jc, Vin, o);

    // ---- reward (sb_reward.c:31-155) ----
    // zone means (sb_sim.c:149-160): the field copied into room order (p.stage
    // is free after the convection), then one thread per zone sums its cells
    block_gather(p.stage, Tg, g.room_pos, g.room_cells);
    __syncthreads();
    for (int z = tid; z < nz; z += blockDim.x) {
        const int rm = s.proom[z];
        const int a = g.room_off[rm], b = g.room_off[rm + 1];
        const double* r = p.stage + a;
        double sum = 0.0;
        int t = 0;
        for (; t + 8 <= b - a; t += 8) {
            double tv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) tv[u] = r[t + u];
#pragma unroll
            for (int u = 0; u < 8; u++) sum = dadd(sum, tv[u]);
        }
        for (; t < b - a; t++) sum = dadd(sum, r[t]);
        p.zavg[z] = ddiv(sum, (double)(b - a));
    }
    __syncthreads();
    const double hsp = s.s_heat[jc], csp = s.s_cool[jc];
    const double dt = s.dt, inv_hour = 1.0 / 3600.0;
    const double max_pph = s.rw[0], min_pph = s.rw[1], ref = s.rw[2];
    for (int z = tid; z < nz; z += blockDim.x) {
        const double zt = p.zavg[z];
        v.d(L.zavg, z) = zt;   // the next k_pre's zone means (the field is unchanged until then)
        {   // zone flow setpoint and actual flow (sb_reward.c:44-56; snapshots show them)
            double fsp = 0.0, fact = 0.0;
            for (int t = s.zv_off[z]; t < s.zv_off[z + 1]; t++) {
                const int vv = s.zv_idx[t];
                const double va = v.d(L.v_area, vv);
                if (va <= 0.0) continue;
                const double share = ddiv(s.zarea[z], va);
                fsp = dadd(fsp, dmul(s.vav_c[vv * 9], share));
                fact = dadd(fact, dmul(dmul(vav_unrestricted(v, s, vv), v.d(L.v_ratio, vv)), share));
            }
            v.d(L.zfsp, z) = fsp;
            v.d(L.zfact, z) = fact;
        }
        double dev = dsub(zt, csp);
        if (dsub(hsp, zt) > dev) dev = dsub(hsp, zt);
        if (dev < 0.0) dev = 0.0;
        const double sf = dev <= ref ? ddiv(dev, ref)
                                     : dadd(1.0, dmul(ddiv(dsub(dev, ref), ref), ddiv(dsub(dev, ref), ref)));
        p.zdev[z] = dev;
        p.zterm[z] = dmul(dmul(dmul(dmul(max_pph, dsub(1.0, sf)), Vst[z]), dt), inv_hour);
    }
    for (int vv = tid; vv < nv; vv += blockDim.x) {
        double area = 0.0, wt = 0.0;
        for (int t = s.vz_off[vv]; t < s.vz_off[vv + 1]; t++) {
            const int z = s.vz_idx[t];
            area = dadd(area, s.zarea[z]);
            wt = dadd(wt, dmul(p.zavg[z], s.zarea[z]));
        }
        p.varea[vv] = area;
        p.vws[vv] = area > 0.0 ? dmul(ddiv(wt, area), area) : 0.0;
    }
    if (tid == 0 && s.tmean_needed) {   // the field mean, for an AHU without VAV area
        double tmean = 0.0;
        for (int q = 0; q < g.ncv; q++) tmean = dadd(tmean, Tg[g.pos_of_cell[q]]);
        p.sc[0] = ddiv(tmean, (double)g.ncv);
    }
    __syncthreads();
    // the reward's independent terms in parallel: per AHU (its VAVs in ascending
    // order), boiler and pump, and the two zone sums; the final thread adds them
    // up in the reference's order
    const double ambient = s.amb[jc];
    if (tid < na) {
        const int a = tid;
        double ws = 0.0, at = 0.0;
        for (int q = s.av_off[a]; q < s.av_off[a + 1]; q++) {
            const int vv = s.av_idx[q];
            if (p.varea[vv] > 0.0) {
                ws = dadd(ws, p.vws[vv]);
                at = dadd(at, p.varea[vv]);
            }
        }
        const double recirc = at > 0.0 ? ddiv(ws, at) : p.sc[0];
        const double st = ahu_static_p(v, s, a);
        const double fe = s.ahu_c[a * 9 + 5];
        const double flow = v.iv(L.ahu_run, a) == 1 ? v.d(L.ahu_flow, a) : 0.0;
        const double rec = v.d(L.ahu_rec, a);
        p.ahu[a] = ddiv(dmul(flow, st), fe);
        p.ahu[kMaxAhu + a] = ddiv(dmul(dmul(flow, dsub(1.0, rec)), st), fe);
        const double mixed = dadd(dmul(rec, recirc), dmul(dsub(1.0, rec), ambient));
        const double sat = (mixed > v.d(L.ahu_sat, a) && v.iv(L.ahu_run, a) == 1) ? v.d(L.ahu_sat, a) : mixed;
        p.ahu[2 * kMaxAhu + a] = ddiv(dmul(dmul(dmul(flow, RHO_AIR), CP_AIR), dsub(sat, mixed)), s.ahu_c[a * 9 + 4]);
    }
    if (tid == 32) {
        const double tf = water_flow(v, s);
        // boiler gas rate (sb_reward.c:12-29); log(r2/c6)/c8 precomputed on the host
        double gas_rate;
        {
            const double* c = s.boiler;
            const double rwt = v.d(L.b_ret);
            const double bsp = v.d(L.b_sp);
            const double supply = bsp > rwt ? bsp : rwt;
            const double flow = dmul(dmul(CP_W * RHO_W, tf), dsub(supply, rwt));
            double diss = 0.0;
            if (supply >= ambient) {
                const double num = dmul(dmul(dmul(c[5], 2.0), 3.14159265358979323846), dsub(supply, ambient));
                const double r2 = dadd(c[6], c[9]);
                const double conv = ddiv(ddiv(1.0, c[4]), r2);
                diss = ddiv(num, dadd(s.boiler_cond, conv));
            }
            double tank = 0.0;
            if (dt > 0.0) tank = ddiv(dmul(dmul(CP_W * RHO_W, c[7]), v.d(L.b_step)), dt);
            const double tot = dadd(dadd(flow, diss), tank);
            gas_rate = tot > 0.0 ? tot : 0.0;
        }
        p.sc[1] = gas_rate;
        p.sc[2] = ddiv(dmul(dmul(dmul(tf, RHO_W), GRAV), v.d(L.pump_head)), s.pump_eff);
    }
    if (tid == 64) {
        double total_occ = 0.0, cum = 0.0;
        for (int z = 0; z < nz; z++) {
            total_occ = dadd(total_occ, Vst[z]);
            cum = dadd(cum, p.zterm[z]);
        }
        p.sc[3] = total_occ;
        p.sc[4] = cum;
    }
    if (tid == 96) {
        double dsum = 0.0, dmax = 0.0;
        int oob = 0;
        for (int z = 0; z < nz; z++) {
            const double dev = p.zdev[z];
            dsum = dadd(dsum, dev);
            if (dev > dmax) dmax = dev;
            if (dev > 0.0) oob++;
        }
        p.sc[5] = dsum;
        p.sc[6] = dmax;
        p.sc[7] = (double)oob;
    }
    __syncthreads();
    if (tid == 0) {
        const int hour = (int)s.r_hour[jc], month = (int)s.r_month[jc], wd = (int)s.r_wd[jc];
        double intake = 0.0, exhaust = 0.0, cooling = 0.0;
        for (int a = 0; a < na; a++) {
            intake = dadd(intake, p.ahu[a]);
            exhaust = dadd(exhaust, p.ahu[kMaxAhu + a]);
            cooling = dadd(cooling, p.ahu[2 * kMaxAhu + a]);
        }
        const double blower = dadd(intake, exhaust);
        const double gas_rate = p.sc[1], pump_e = p.sc[2], total_occ = p.sc[3], cum = p.sc[4];
        const double dsum = p.sc[5], dmax = p.sc[6];
        const int oob = (int)p.sc[7];
        const double max_prod = dmul(dmul(dmul(max_pph, total_occ), dt), inv_hour);
        const double min_prod = dmul(dmul(dmul(min_pph, total_occ), dt), inv_hour);
        const double npr = (total_occ > 0.0 && dsub(max_prod, min_prod) != 0.0)
                               ? dsub(ddiv(dsub(cum, min_prod), dsub(max_prod, min_prod)), 1.0) : 0.0;
        const double elec_rate = dadd(dadd(blower, fabs(cooling)), pump_e);
        const double price = wd ? s.e_wd[hour] : s.e_we[hour];
        const double crate = s.e_c[hour];
        const double elec_cost = dmul(dmul(price, fabs(elec_rate)), dt);
        const double elec_cost_max = dmul(dmul(price, s.rw[3]), dt);
        const double elec_carb = dmul(dmul(crate, fabs(elec_rate)), dt);
        const double elec_carb_max = dmul(dmul(crate, s.rw[3]), dt);
        const double gprice = s.g_p[month - 1];
        const double gg = gas_rate > 0.0 ? gas_rate : 0.0;
        const double gas_cost = dmul(dmul(gprice, gg), dt);
        const double gas_cost_max = dmul(dmul(gprice, s.rw[4]), dt);
        const double gas_carb = dmul(dmul(s.gas_carbon, gg), dt);
        const double gas_carb_max = dmul(dmul(s.gas_carbon, s.rw[4]), dt);
        const double den_e = dadd(elec_cost_max, gas_cost_max);
        const double nec = den_e > 0.0 ? ddiv(dadd(elec_cost, gas_cost), den_e) : 0.0;
        const double den_c = dadd(elec_carb_max, gas_carb_max);
        const double ncar = den_c > 0.0 ? ddiv(dadd(elec_carb, gas_carb), den_c) : 0.0;
        const double pw = s.rw[5], ew = s.rw[6], cw = s.rw[7];
        const double rew = ddiv(dsub(dsub(dmul(npr, pw), dmul(nec, ew)), dmul(ncar, cw)), dadd(dadd(pw, ew), cw));
        double parts[kParts];
        parts[0] = npr;
        parts[1] = nec;
        parts[2] = ncar;
        parts[3] = nz > 0 ? ddiv(dsum, (double)nz) : 0.0;
        parts[4] = dmax;
        parts[5] = nz > 0 ? ddiv((double)oob, (double)nz) : 0.0;
        parts[6] = ddiv(dmul(fabs(elec_rate), dt), 3.6e6);
        parts[7] = ddiv(dmul(gg, dt), 3.6e6);

        // ---- finalize (smart_buildings.cu:1936-2050) ----
        const float r = (float)rew;
        if (ctx->rnorm) {   // rew_norm / rew_center: the learning signal only; logs keep r
            const float* rn = ctx->rnorm + 2 * (size_t)ei.scn;
            const float z = (r - rn[0]) * rn[1];
            ctx->rewards[env] = z;
            if (ctx->znclip) {
                const float az = fabsf(z);
                if (az > 1.0f) atomicAdd(&ctx->znclip[0], 1.0);
                if (az > 3.0f) atomicAdd(&ctx->znclip[1], 1.0);
                if (az > 5.0f) atomicAdd(&ctx->znclip[2], 1.0);
            }
        } else {
            ctx->rewards[env] = r * ctx->reward_scale;
        }
        ctx->rew_f64[env] = rew;
        for (int q = 0; q < kParts; q++) ctx->parts_out[(size_t)env * kParts + q] = parts[q];
        Env* er = reinterpret_cast<Env*>(ctx->env_records) + env;
        er->step = j;
        const bool done = j >= v.iv(L.eplen);
        ctx->terminals[env] = done ? 1.0f : 0.0f;
        er->ep_ret += r;
        ctx->epret_d[env] += rew;
        for (int q = 0; q < kParts; q++) er->ep_part[q] += (float)parts[q];
        if ((float)parts[4] > er->ep_worst) er->ep_worst = (float)parts[4];
        atomicAdd(&ctx->live[0], 1.0);
        atomicAdd(&ctx->live[1], (double)r);
        for (int q = 0; q < kParts; q++) atomicAdd(&ctx->live[2 + q], parts[q]);
        double* ls = ctx->live_scn + (size_t)ei.scn * 4;
        atomicAdd(&ls[0], (double)r);
        atomicAdd(&ls[1], parts[3]);
        atomicAdd(&ls[2], 1.0);
        atomicAdd(&ls[3], (double)r * (double)r);
        if (done) {
            // only whole episodes enter the log: a first episode cut short by
            // desync is a truncation
            const float st = (float)j;
            if (j >= s.max_steps) {
                const float mean = er->ep_ret / st;
                const double mean_d = ctx->epret_d[env] / (double)j;
                atomicAdd(&ctx->ep_scn[(size_t)ei.scn * 2], mean_d);
                atomicAdd(&ctx->ep_scn[(size_t)ei.scn * 2 + 1], 1.0);
                if (ctx->random_start) {
                    double* es = ctx->ep_start + ((size_t)ei.scn * kStartDays + v.iv(L.off) / kStepsPerDay) * 7;
                    atomicAdd(&es[0], 1.0);
                    atomicAdd(&es[1], mean_d);
                    for (int q = 0; q < 3; q++) atomicAdd(&es[2 + q], (double)(er->ep_part[q] / st));
                    atomicAdd(&es[5], (double)er->ep_part[6]);
                    atomicAdd(&es[6], (double)er->ep_part[7]);
                }
                er->log.perf += mean;
                er->log.score += mean;
                er->log.episode_return += er->ep_ret;
                er->log.episode_length += st;
                er->log.productivity += er->ep_part[0] / st;
                er->log.energy_cost_norm += er->ep_part[1] / st;
                er->log.carbon_norm += er->ep_part[2] / st;
                er->log.comfort_dev_K += er->ep_part[3] / st;
                er->log.worst_dev_K += er->ep_worst;
                er->log.out_of_band_frac += er->ep_part[5] / st;
                er->log.elec_kwh += er->ep_part[6];
                er->log.gas_kwh += er->ep_part[7];
                er->log.n += 1.0f;
            }
            er->max_steps = s.max_steps;   // every later episode has the scenario's full length
            v.iv(L.eplen) = s.max_steps;
            er->ep_ret = 0.0f;
            ctx->epret_d[env] = 0.0;
            for (int q = 0; q < kParts; q++) er->ep_part[q] = 0.0f;
            er->ep_worst = 0.0f;
            er->step = 0;
        }
        p.sc[8] = done ? 1.0 : 0.0;
    }
    __syncthreads();
    const bool done = p.sc[8] != 0.0;
    if (done) {
        const size_t so = (size_t)slot * ctx->n_ostreams + ei.ostream;
        restart_env(ctx, env, g, s, v, p, ctx->V_prime + vslot, ctx->V_zero + vslot, ctx->new_off[so],
                    ctx->new_rng[so]);
    } else {
        for (int z = tid; z < nz; z += blockDim.x) v.d(L.V, z) = Vst[z];
    }
}

// One env's visible state packed for a snapshot file (the reference's SBS1
// writer, complete_port/gpu/smart_buildings.cu:2205-2290), in doubles:
// field [ncv] in cell order, zone means, occupancy, zone flow setpoint and
// actual [nz each], VAV heating / cooling setpoints, damper, reheat [nv each],
// AHU supply temperature, flow, run [na each], native actions [nact], then
// step, boiler setpoint, boiler return.
__host__ __device__ constexpr size_t snap_doubles(int ncv, int nz, int nv, int na, int nact) {
    return (size_t)ncv + 4 * (size_t)nz + 4 * (size_t)nv + 3 * (size_t)na + (size_t)nact + 3;
}
__global__ void __launch_bounds__(128) k_snapshot(const StepCtx* __restrict__ ctx, int env, double* __restrict__ out) {
    const EnvIndex ei = ctx->envs[env];
    const GroupDev& g = ctx->groups[ei.group];
    const ScnDev& s = ctx->scns[ei.scn];
    const StateLayout& L = ctx->lay;
    EnvView v{ctx->Dst + (size_t)env * L.nd, ctx->Ist + (size_t)env * L.ni, &ctx->lay};
    const int tid = threadIdx.x, nz = s.nz, nv = s.nv, na = s.na;
    const double* Tg = g.T + (size_t)(env - g.env0) * g.ncv;
    double* o = out;
    for (int c = tid; c < g.ncv; c += blockDim.x) o[c] = Tg[g.pos_of_cell[c]];
    o += g.ncv;
    for (int z = tid; z < nz; z += blockDim.x) {
        o[z] = v.d(L.zavg, z);
        o[nz + z] = v.d(L.V, z);
        o[2 * nz + z] = v.d(L.zfsp, z);
        o[3 * nz + z] = v.d(L.zfact, z);
    }
    o += 4 * nz;
    for (int q = tid; q < nv; q += blockDim.x) {
        o[q] = v.d(L.v_hsp, q);
        o[nv + q] = v.d(L.v_csp, q);
        o[2 * nv + q] = v.d(L.v_damp, q);
        o[3 * nv + q] = v.d(L.v_reh, q);
    }
    o += 4 * nv;
    for (int a = tid; a < na; a += blockDim.x) {
        o[a] = v.d(L.ahu_sat, a);
        o[na + a] = v.d(L.ahu_flow, a);
        o[2 * na + a] = (double)v.iv(L.ahu_run, a);
    }
    o += 3 * na;
    const float* act = ctx->actions + (size_t)env * kAct;
    for (int i = tid; i < s.nact; i += blockDim.x) o[i] = decode_native(s, i, act);
    o += s.nact;
    if (tid == 0) {
        o[0] = (double)v.iv(L.step);
        o[1] = v.d(L.b_sp);
        o[2] = v.d(L.b_ret);
    }
}

// Explicit restart of every env (puf_reset), after k_occ ran in reset mode.
__global__ void __launch_bounds__(128) k_reset(const StepCtx* __restrict__ ctx) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int env = blockIdx.x;
    const EnvIndex ei = ctx->envs[env];
    const GroupDev& g = ctx->groups[ei.group];
    const ScnDev& s = ctx->scns[ei.scn];
    const StateLayout& L = ctx->lay;
    EnvView v{ctx->Dst + (size_t)env * L.nd, ctx->Ist + (size_t)env * L.ni, &ctx->lay};
    PostShared p = post_shared(smem, g.ncv, s.nz, s.nv);
    float* o = ctx->obs + (size_t)env * kObs;
    for (int i = threadIdx.x; i < kObs; i += blockDim.x) o[i] = 0.0f;
    if (threadIdx.x == 0) {
        Env* er = reinterpret_cast<Env*>(ctx->env_records) + env;
        er->step = 0;
        er->ep_ret = 0.0f;
        er->ep_worst = 0.0f;
        for (int q = 0; q < kParts; q++) er->ep_part[q] = 0.0f;
        ctx->epret_d[env] = 0.0;
        v.iv(L.tseq) = 0;
    }
    __syncthreads();
    const size_t so = (size_t)kResetSlot * ctx->n_ostreams + ei.ostream;
    const size_t vslot = so * ctx->nz_max;
    restart_env(ctx, env, g, s, v, p, ctx->V_prime + vslot, ctx->V_zero + vslot, ctx->new_off[so], ctx->new_rng[so]);
}

}  // namespace sbenv
