// Sweep programs for the solve kernel: a static list schedule of the
// triangular factor's rows over the warps (and their four lane groups) of one
// solve CTA.
//
// The reference solves L y = b, U z = y by column push
// (complete_port/csim/sb_lu.c:38-63): column j, once final, is subtracted from
// every row below (L) or above (U) it. Here every row pulls its terms itself,
// in exactly the order the push would deliver them, so the rounding sequence
// of each row is unchanged. Rows are spread over the warps and lane groups by
// simulating the sweep with a simple cost model; the model decides only
// speed, never results. A lane group starts a run of a row's terms ("segment")
// only at a control record, and only with terms whose columns are final by
// then: rows finished earlier by this warp, or rows of other warps covered by
// the record's waits (a wait for a row also covers every row it depends on).
//
// Deadlock freedom: a control record waits only for rows finished at control
// records created earlier in the simulation (smaller sequence number), and
// every warp runs its records in creation order. The unfinished control
// record with the smallest sequence number therefore always finds its waits
// satisfied and its warp at it; term records never wait.
#include "sweep_sched.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>

namespace sbenv {

namespace {

// Cost model of one warp, in cycles. Only used to order the work.
constexpr double kCCtrl = 100;  // a control record: finishes, waits, new rows
constexpr double kCBlk = 40;    // a term record
constexpr double kC2 = 80;      // release store until another warp's acquire sees it
constexpr double kSlack = 150;  // a row may be picked this long before its next input is ready
constexpr int kMinSeg = 16;      // shortest segment worth a control record (unless the row ends sooner)
constexpr double kCritical = 0.9;    // rows within this fraction of the top priority start at any length
constexpr int kUnsched = std::numeric_limits<int>::max();

inline bool test(const uint64_t* s, int i) { return (s[i >> 6] >> (i & 63)) & 1u; }
inline void set(uint64_t* s, int i) { s[i >> 6] |= uint64_t(1) << (i & 63); }
inline void orr(uint64_t* d, const uint64_t* s, int w) {
    for (int k = 0; k < w; k++) d[k] |= s[k];
}

struct Group {
    int row = -1;     // -1: idle
    int q = 0, qend = 0;
};

struct WarpProg {
    double T = 0;
    Group g[kBundleRows];
    std::vector<uint8_t> rec;   // records, kRecordBytes each
    int last = -1;              // index of the last record
    bool last_ctrl = false;
    bool ended = false;
    bool idle = false;          // found nothing to do at T in the current state
};

}  // namespace

std::string build_sweep(int n, const std::vector<std::vector<std::pair<int, double>>>& terms, bool backward,
                        const std::vector<double>& diag, int ring_stages, HostSweep& out) {
    out = HostSweep();
    if (n <= 0 || n >= (int)kColMask) return "factor too large for the sweep format";
    if (ring_stages < kStagesMin || ring_stages > kStagesMax) return "unsupported ring depth";
    out.ring_stages = ring_stages;
    const int W = kSweepWarps;
    std::vector<int> nt(n);
    std::vector<char> need(n);
    int remaining = 0;
    for (int i = 0; i < n; i++) {
        nt[i] = (int)terms[i].size();
        need[i] = backward || nt[i] > 0;
        remaining += need[i];
        out.terms += nt[i];
        for (auto& t : terms[i])
            if (t.first < 0 || t.first >= n || (backward ? t.first <= i : t.first >= i))
                return "triangular term outside its triangle";
    }

    // priority: longest modelled path from the row to the end of the sweep
    std::vector<std::vector<int>> dependents(n);
    for (int i = 0; i < n; i++)
        for (auto& t : terms[i]) dependents[t.first].push_back(i);
    std::vector<double> prio(n, 0.0);
    for (int s = 0; s < n; s++) {
        const int i = backward ? s : n - 1 - s;   // dependents first
        double best = 0.0;
        for (int d : dependents[i]) best = std::max(best, prio[d]);
        prio[i] = best + kC2 + kCCtrl + kCBlk * std::ceil(nt[i] / (double)kTermSteps);
    }

    // closure[i]: rows that are final whenever row i is (i and, recursively,
    // the rows of its terms)
    const int WD = (n + 1 + 63) / 64;
    std::vector<uint64_t> clo((size_t)n * WD, 0);
    for (int s = 0; s < n; s++) {
        const int i = backward ? n - 1 - s : s;
        uint64_t* ci = clo.data() + (size_t)i * WD;
        set(ci, i);
        for (auto& tm : terms[i]) orr(ci, clo.data() + (size_t)tm.first * WD, WD);
    }

    // ---- home warps: subtrees of the dependency forest (parent = the nearest
    // row that reads the row) are spread over the warps so that most reads
    // stay inside one warp; rows above those subtrees go to any warp ----
    std::vector<int> parent(n, -1);
    for (int i = 0; i < n; i++)
        for (int d : dependents[i])
            if (parent[i] < 0 || (backward ? d > parent[i] : d < parent[i])) parent[i] = d;
    std::vector<double> subw(n, 0.0);
    std::vector<std::vector<int>> children(n);
    double total_w = 0.0;
    for (int s = 0; s < n; s++) {
        const int i = backward ? n - 1 - s : s;   // children before parents
        subw[i] += 1.0 + nt[i];
        total_w += 1.0 + nt[i];
        if (parent[i] >= 0) {
            subw[parent[i]] += subw[i];
            children[parent[i]].push_back(i);
        }
    }
    std::vector<int> home(n, -1), pool;
    for (int i = 0; i < n; i++)
        if (parent[i] < 0) pool.push_back(i);
    for (;;) {
        auto it = std::max_element(pool.begin(), pool.end(), [&](int a, int b) { return subw[a] < subw[b]; });
        if (it == pool.end() || subw[*it] <= total_w / (2.0 * W) || children[*it].empty()) break;
        const int r = *it;
        pool.erase(it);
        for (int c : children[r]) pool.push_back(c);
    }
    std::sort(pool.begin(), pool.end(), [&](int a, int b) { return subw[a] != subw[b] ? subw[a] > subw[b] : a < b; });
    {
        std::vector<double> load(W, 0.0);
        std::vector<int> stack;
        for (int r : pool) {
            const int w = (int)(std::min_element(load.begin(), load.end()) - load.begin());
            load[w] += subw[r];
            stack.assign(1, r);
            while (!stack.empty()) {
                const int v = stack.back();
                stack.pop_back();
                home[v] = w;
                for (int c : children[v]) stack.push_back(c);
            }
        }
    }

    // ---- list-scheduling simulation ----
    std::vector<double> done(n, std::numeric_limits<double>::infinity());
    std::vector<int> fseq(n, kUnsched), owner(n, -1), prog(n, 0);
    std::vector<char> in_use(n, 0), waited(n, 0);
    std::vector<int> open;
    std::vector<uint64_t> K((size_t)W * WD, 0);   // per warp: rows it knows final
    for (int w = 0; w < W; w++) set(K.data() + (size_t)w * WD, n);
    for (int i = 0; i < n; i++) {
        if (need[i]) open.push_back(i);
        else {
            done[i] = 0.0;
            fseq[i] = -1;
            for (int w = 0; w < W; w++) set(K.data() + (size_t)w * WD, i);
        }
    }
    std::vector<WarpProg> wp(W);
    std::vector<int> cand;
    std::vector<uint64_t> Kb(WD);
    int seq = 0;
    int64_t guard = 0;

    auto new_record = [&](WarpProg& P, bool ctrl) -> uint8_t* {
        if (P.last >= 0) {   // tell the previous record what follows
            uint8_t* prev = P.rec.data() + (size_t)P.last * kRecordBytes;
            if (ctrl) {
                if (P.last_ctrl) reinterpret_cast<ControlRecord*>(prev)->flags |= kCtrlNext;
                else
                    for (int g = 0; g < kBundleRows; g++) reinterpret_cast<TermRecord*>(prev)->col[g][0] |= kNextIsCtrl;
            }
        }
        P.rec.resize(P.rec.size() + kRecordBytes, 0);
        P.last++;
        P.last_ctrl = ctrl;
        return P.rec.data() + (size_t)P.last * kRecordBytes;
    };
    auto may_take = [&](int w, int r) {
        return (owner[r] == -1 || owner[r] == w) && (home[r] == -1 || home[r] == w) && !in_use[r];
    };

    while (true) {
        if (++guard > 256LL * n + 100000) return "sweep schedule did not converge";
        // the warp with the earliest time (busy before idle on ties); done when all ended
        int w = -1;
        for (int q = 0; q < W; q++) {
            if (wp[q].ended) continue;
            if (w < 0 || wp[q].T < wp[w].T || (wp[q].T == wp[w].T && wp[w].idle && !wp[q].idle)) w = q;
        }
        if (w < 0) break;
        WarpProg& P = wp[w];
        const double t = P.T;
        uint64_t* Kw = K.data() + (size_t)w * WD;

        // (a) segments that ended: rows final or paused
        ControlRecord cr;
        memset(&cr, 0, sizeof(cr));
        for (int g = 0; g < kBundleRows; g++) cr.row[g] = (uint16_t)n;
        bool any = false;
        for (int g = 0; g < kBundleRows; g++) {
            Group& G = P.g[g];
            if (G.row < 0 || G.q < G.qend) continue;
            const int r = G.row;
            prog[r] = G.q;
            in_use[r] = 0;
            cr.gflags[g] = kGSwitch;
            if (G.q == nt[r]) {
                cr.gflags[g] |= kGFinal;
                if (backward) {
                    cr.gflags[g] |= kGDivide;
                    cr.diag[g] = diag[r];
                }
                done[r] = t + kCCtrl;
                fseq[r] = seq;
                set(Kw, r);
                remaining--;
            }
            G.row = -1;
            any = true;
        }
        if (any)
            open.erase(std::remove_if(open.begin(), open.end(), [&](int r) { return fseq[r] != kUnsched; }),
                       open.end());

        // (b) new segments for the free groups, most urgent rows first
        cand.clear();
        double next_event = std::numeric_limits<double>::infinity();
        for (int r : open) {
            if (!may_take(w, r)) continue;
            if (prog[r] < nt[r]) {
                const int c = terms[r][prog[r]].first;
                if (!test(Kw, c)) {
                    if (fseq[c] == kUnsched) continue;
                    if (done[c] + kC2 - kSlack > t) { next_event = std::min(next_event, done[c] + kC2 - kSlack); continue; }
                }
            }
            cand.push_back(r);
        }
        std::sort(cand.begin(), cand.end(), [&](int a, int b) {
            if (prio[a] != prio[b]) return prio[a] > prio[b];
            return backward ? a > b : a < b;
        });
        double top_prio = 0.0;
        for (int r : open) top_prio = std::max(top_prio, prio[r]);
        std::copy(Kw, Kw + WD, Kb.begin());
        std::vector<int> waits;
        double ready = t;
        size_t ci = 0;
        for (int g = 0; g < kBundleRows && ci < cand.size(); g++) {
            if (P.g[g].row >= 0) continue;
            while (ci < cand.size()) {
                const int r = cand[ci++];
                int q = prog[r];
                double rdy = ready;
                std::vector<int> wnew;
                while (q < nt[r]) {
                    const int c = terms[r][q].first;
                    if (!test(Kb.data(), c)) {
                        if (!(fseq[c] < seq && done[c] + kC2 <= t + kSlack) ||
                            (int)(waits.size() + wnew.size()) >= kCtrlWaits)
                            break;
                        int top = c;
                        while (parent[top] >= 0 && fseq[parent[top]] < seq && done[parent[top]] + kC2 <= t + kSlack)
                            top = parent[top];
                        wnew.push_back(top);
                        rdy = std::max(rdy, done[top] + kC2);
                        orr(Kb.data(), clo.data() + (size_t)top * WD, WD);
                    }
                    q++;
                }
                if (q == prog[r] && q < nt[r]) continue;   // not a single term ready after all
                if (q < nt[r] && q - prog[r] < kMinSeg && prio[r] < kCritical * top_prio) {
                    // too short a run for an off-critical row: its waits are not kept
                    std::copy(Kw, Kw + WD, Kb.begin());
                    for (int x : waits) orr(Kb.data(), clo.data() + (size_t)x * WD, WD);
                    continue;
                }
                for (int x : wnew) waits.push_back(x);
                ready = rdy;
                P.g[g] = Group{r, prog[r], q};
                in_use[r] = 1;
                owner[r] = w;
                cr.gflags[g] |= kGSwitch;
                cr.row[g] = (uint16_t)r;
                any = true;
                out.pieces++;
                break;
            }
        }
        if (any || !waits.empty()) {
            cr.nwait = (uint8_t)waits.size();
            for (size_t i = 0; i < waits.size(); i++) {
                cr.wait[i] = (uint16_t)waits[i];
                waited[waits[i]] = 1;
            }
            out.prewaits += (int64_t)waits.size();
            std::copy(Kb.begin(), Kb.end(), Kw);
            memcpy(new_record(P, true), &cr, sizeof(cr));
            P.T = std::max(t, ready) + kCCtrl;
            out.sim_cycles = std::max(out.sim_cycles, P.T);
            seq++;
            for (auto& x : wp) x.idle = false;
        }
        // (c) run term records until the first active segment ends
        int nb = std::numeric_limits<int>::max();
        bool active = false;
        for (int g = 0; g < kBundleRows; g++)
            if (P.g[g].row >= 0) {
                active = true;
                nb = std::min(nb, (P.g[g].qend - P.g[g].q + kTermSteps - 1) / kTermSteps);
            }
        if (active) {
            for (int b = 0; b < nb; b++) {
                TermRecord tr;
                for (int g = 0; g < kBundleRows; g++)
                    for (int s = 0; s < kTermSteps; s++) {
                        Group& G = P.g[g];
                        if (G.row >= 0 && G.q < G.qend) {
                            const auto& tm = terms[G.row][G.q++];
                            tr.val[g][s] = tm.second;
                            tr.col[g][s] = (uint16_t)tm.first;
                        } else {   // padding: 0 * x[n] (the zero slot) leaves the row unchanged
                            tr.val[g][s] = 0.0;
                            tr.col[g][s] = (uint16_t)n;
                        }
                    }
                memcpy(new_record(P, false), &tr, sizeof(tr));
                out.blocks++;
            }
            P.T += nb * kCBlk;
            out.sim_cycles = std::max(out.sim_cycles, P.T);
            continue;
        }
        // (d) nothing running: end, or wait for the next event
        bool future = false;
        for (int r : open)
            if ((owner[r] == -1 || owner[r] == w) && (home[r] == -1 || home[r] == w)) { future = true; break; }
        if (!future) {
            ControlRecord end;
            memset(&end, 0, sizeof(end));
            for (int g = 0; g < kBundleRows; g++) end.row[g] = (uint16_t)n;
            end.flags = kCtrlEnd;
            memcpy(new_record(P, true), &end, sizeof(end));
            P.ended = true;
            continue;
        }
        bool other_now = false;
        for (int q = 0; q < W; q++) {
            if (q == w || wp[q].ended) continue;
            if (wp[q].T > t) next_event = std::min(next_event, wp[q].T);
            other_now |= (wp[q].T == t && !wp[q].idle);
        }
        if (any) continue;   // the control record moved time on
        if (other_now) { P.idle = true; continue; }
        if (!std::isfinite(next_event)) return "sweep schedule deadlocked";
        P.T = next_event;
        P.idle = false;
    }
    if (remaining != 0) return "sweep schedule left rows unfinished";

    // ---- serialise; a row another warp waits for is published where it
    // finishes (a control record finishes the row its group was given before) ----
    for (int w = 0; w < W; w++) {
        WarpProg& P = wp[w];
        // the row a group finishes at a control record is the row it was given earlier
        int cur[kBundleRows];
        for (int g = 0; g < kBundleRows; g++) cur[g] = -1;
        bool ctrl = true;
        for (int i = 0; i <= P.last; i++) {
            uint8_t* r = P.rec.data() + (size_t)i * kRecordBytes;
            out.bundles += ctrl ? 1 : 0;
            if (ctrl) {
                ControlRecord* c = reinterpret_cast<ControlRecord*>(r);
                for (int g = 0; g < kBundleRows; g++) {
                    if (!(c->gflags[g] & kGSwitch)) continue;
                    if ((c->gflags[g] & kGFinal) && cur[g] >= 0 && waited[cur[g]]) {
                        c->gflags[g] |= kGPublish;
                        out.publishes++;
                    }
                    cur[g] = c->row[g] < n ? c->row[g] : -1;
                }
                ctrl = (c->flags & kCtrlNext) != 0;
            } else {
                ctrl = (reinterpret_cast<TermRecord*>(r)->col[0][0] & kNextIsCtrl) != 0;
            }
        }
        const size_t stages = (P.rec.size() + kStageBytes - 1) / kStageBytes;
        P.rec.resize(stages * kStageBytes, 0);
        out.warp_off[w] = (uint32_t)(out.bytes.size() / kStageBytes);
        out.warp_stages[w] = (uint32_t)stages;
        out.bytes.insert(out.bytes.end(), P.rec.begin(), P.rec.end());
    }
    return "";
}

}  // namespace sbenv
