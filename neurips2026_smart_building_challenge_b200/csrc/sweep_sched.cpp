// Sweep programs for the solve kernel: a static list schedule of the
// triangular factor's rows over the warps (and their four lane groups) of one
// solve CTA.
//
// The reference solves L y = b, U z = y by column push
// (complete_port/csim/sb_lu.c:38-63): column j, once final, is subtracted from
// every row below (L) or above (U) it. Here every row pulls its terms itself,
// in exactly the order the push would deliver them, so the rounding sequence
// of each row is unchanged. Rows are spread over the warps and lane groups by
// simulating the sweep with a cost model of the kernel; the model decides only
// speed, never results. A lane group starts a run of a row's terms ("segment")
// only at a control record, and only with terms whose columns are final by
// then: rows finished earlier by this warp, or rows of other warps covered by
// the record's waits (a wait for a row also covers every row it depends on).
//
// Dense blocks (runs of consecutive rows, in sweep order, whose terms among
// themselves form a full triangle: the separators of the nested-dissection
// order) are finished by one warp in a block record, four rows per round
// (each pulls its terms from the earlier rounds, then the four finish in
// turn); their rows' other ("outside") terms run before as ordinary segments.
//
// Deadlock freedom: a record waits only for rows (or rows' outside terms)
// finished at records created earlier in the simulation (smaller sequence
// number), and every warp runs its records in creation order. The unfinished
// record with the smallest sequence number therefore always finds its waits
// satisfied and its warp at it; term records never wait.
#include "sweep_sched.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>

namespace sbenv {

namespace {

// Cost model of one warp, in SM cycles (measured with clock64 traces of the
// kernel on B200). Only used to order the work.
constexpr double kCCtrl = 500;    // a control record: finish rows, waits, start rows
constexpr double kCBlk = 250;     // a term record
constexpr double kC2 = 800;       // release store until the waiting warp has seen it
constexpr double kCBRound = 1800; // one round (four rows) of a block record ...
constexpr double kCBRow = 17;     // ... plus this per row of the earlier rounds
constexpr double kSlack = 150;    // a row may be picked this long before its next input is ready
constexpr int kMinSeg = 16;       // shortest segment worth a control record (unless the row ends sooner)
constexpr double kCritical = 0.9; // rows within this fraction of the top priority start at any length
constexpr int kMinBlock = 16;     // shortest run of rows solved as a dense block
constexpr int kUnsched = std::numeric_limits<int>::max();
constexpr double kInf = std::numeric_limits<double>::infinity();

inline bool test(const uint64_t* s, int i) { return (s[i >> 6] >> (i & 63)) & 1u; }
inline void set(uint64_t* s, int i) { s[i >> 6] |= uint64_t(1) << (i & 63); }
inline void orr(uint64_t* d, const uint64_t* s, int w) {
    for (int k = 0; k < w; k++) d[k] |= s[k];
}

// modelled length of the round of a block of s rows that starts at row c0
inline double block_round(int s, int c0) { (void)s; return kCBRound + kCBRow * c0; }

struct Group {
    int row = -1;     // -1: idle
    int q = 0, qend = 0;
};

struct WarpProg {
    double T = 0;
    Group g[kBundleRows];
    std::vector<uint8_t> rec;   // records, kRecordBytes each
    int last = -1;              // index of the last header record (term, control or block)
    int last_kind = 0;          // 0 term, 1 control or block
    bool ended = false;
    bool idle = false;          // found nothing to do at T in the current state
    double wake = 0;            // when idle: the earliest time it could start something
};

struct Block {
    std::vector<int> rows;      // in sweep order
    int outside_left = 0;       // rows whose outside terms are not finished yet
    bool scheduled = false;
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
    for (int i = 0; i < n; i++) {
        nt[i] = (int)terms[i].size();
        out.terms += nt[i];
        for (auto& t : terms[i])
            if (t.first < 0 || t.first >= n || (backward ? t.first <= i : t.first >= i))
                return "triangular term outside its triangle";
    }
    auto row_at = [&](int p) { return backward ? n - 1 - p : p; };   // sweep order

    // ---- dense blocks: the row at sweep position p joins the block started at
    // position s0 if its last p - s0 terms are the rows s0 .. p-1 in order ----
    std::vector<int> blk(n, -1), nout(nt);
    std::vector<Block> blocks;
    const int max_block = kMaxBlockRows;
    {
        int s0 = 0;
        for (int p = 1; p <= n; p++) {
            bool extend = p < n && p - s0 < max_block;
            if (extend) {
                const int r = row_at(p), m = p - s0;
                extend = nt[r] >= m;
                for (int a = 0; extend && a < m; a++) extend = terms[r][nt[r] - m + a].first == row_at(s0 + a);
            }
            if (extend) continue;
            if (p - s0 >= kMinBlock) {
                Block B;
                for (int x = s0; x < p; x++) {
                    const int r = row_at(x);
                    blk[r] = (int)blocks.size();
                    nout[r] = nt[r] - (x - s0);
                    B.rows.push_back(r);
                }
                blocks.push_back(B);
            }
            s0 = p;
        }
    }
    out.dense_blocks = (int64_t)blocks.size();

    // priority: longest modelled path from the row to the end of the sweep
    std::vector<std::vector<int>> dependents(n);
    for (int i = 0; i < n; i++)
        for (auto& t : terms[i]) dependents[t.first].push_back(i);
    std::vector<double> prio(n, 0.0);
    for (int s = 0; s < n; s++) {
        const int i = row_at(n - 1 - s);   // dependents first
        double best = 0.0;
        for (int d : dependents[i]) best = std::max(best, prio[d]);
        prio[i] = best + (blk[i] >= 0 ? kCBRound / 4 + kCBlk * std::ceil(nout[i] / (double)kTermSteps)
                                      : kC2 + kCCtrl + kCBlk * std::ceil(nt[i] / (double)kTermSteps));
    }

    // clo[i]: rows that are final whenever row i is; oclo[i]: rows that are
    // final whenever row i's outside terms are applied
    const int WD = (n + 1 + 63) / 64;
    std::vector<uint64_t> clo((size_t)n * WD, 0), oclo((size_t)n * WD, 0);
    for (int s = 0; s < n; s++) {
        const int i = row_at(s);
        uint64_t* ci = clo.data() + (size_t)i * WD;
        uint64_t* oi = oclo.data() + (size_t)i * WD;
        for (int a = 0; a < nout[i]; a++) orr(oi, clo.data() + (size_t)terms[i][a].first * WD, WD);
        orr(ci, oi, WD);
        set(ci, i);
        for (int a = nout[i]; a < nt[i]; a++) orr(ci, clo.data() + (size_t)terms[i][a].first * WD, WD);
    }

    // ---- home warps: subtrees of the dependency forest (parent = the nearest
    // row that reads the row) are spread over the warps so that most reads
    // stay inside one warp; rows above those subtrees and block rows' outside
    // terms go to any warp ----
    std::vector<int> parent(n, -1);
    for (int i = 0; i < n; i++)
        for (int d : dependents[i])
            if (parent[i] < 0 || (backward ? d > parent[i] : d < parent[i])) parent[i] = d;
    std::vector<double> subw(n, 0.0);
    std::vector<std::vector<int>> children(n);
    double total_w = 0.0;
    for (int s = 0; s < n; s++) {
        const int i = row_at(s);   // children before parents
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
    for (int i = 0; i < n; i++)
        if (blk[i] >= 0) home[i] = -1;

    // ---- list-scheduling simulation ----
    // fseq/done: the record finishing a row; oseq/odone: the record finishing a
    // block row's outside terms (oend: its warp)
    std::vector<double> done(n, kInf), odone(n, kInf);
    std::vector<int> fseq(n, kUnsched), oseq(n, kUnsched), oend(n, -1), owner(n, -1), prog(n, 0);
    std::vector<char> in_use(n, 0), waited(n, 0), owaited(n, 0);
    std::vector<int> open;
    std::vector<uint64_t> K((size_t)W * WD, 0);   // per warp: rows it knows final
    for (int w = 0; w < W; w++) set(K.data() + (size_t)w * WD, n);
    int remaining = 0;
    for (int i = 0; i < n; i++) {
        if (blk[i] >= 0) {
            remaining++;
            if (nout[i] > 0) {
                open.push_back(i);
                blocks[blk[i]].outside_left++;
            } else {   // no outside terms: the right side is the partial sum
                odone[i] = 0.0;
                oseq[i] = -1;
            }
        } else if (backward || nt[i] > 0) {   // backward rows always need their division
            remaining++;
            open.push_back(i);
        } else {
            done[i] = 0.0;
            fseq[i] = -1;
            for (int w = 0; w < W; w++) set(K.data() + (size_t)w * WD, i);
        }
    }
    auto lim = [&](int r) { return blk[r] >= 0 ? nout[r] : nt[r]; };   // terms a row's segments cover
    std::vector<WarpProg> wp(W);
    std::vector<double> block_vals;   // all blocks' values (region after the programs)
    std::vector<int> cand;
    std::vector<uint64_t> Kb(WD), Ksave;
    int seq = 0;
    int64_t guard = 0;

    auto new_record = [&](WarpProg& P, int kind) -> uint8_t* {
        if (P.last >= 0 && kind != 0) {   // tell the previous record that a control/block record follows
            uint8_t* prev = P.rec.data() + (size_t)P.last * kRecordBytes;
            if (P.last_kind == 0)
                for (int g = 0; g < kBundleRows; g++) reinterpret_cast<TermRecord*>(prev)->col[g][0] |= kNextIsCtrl;
            else
                reinterpret_cast<ControlRecord*>(prev)->flags |= kCtrlNext;
        }
        P.rec.resize(P.rec.size() + kRecordBytes, 0);
        P.last = (int)(P.rec.size() / kRecordBytes) - 1;
        P.last_kind = kind;
        return P.rec.data() + (size_t)P.last * kRecordBytes;
    };
    auto may_take = [&](int w, int r) {
        return (owner[r] == -1 || owner[r] == w) && (home[r] == -1 || home[r] == w) && !in_use[r];
    };
    // a wait for final row c (the highest final ancestor that covers it) or
    // for block row c's outside terms; returns when the warp sees it
    auto add_wait = [&](std::vector<int>& waits, int c, bool partial, double t) -> double {
        if (partial) {
            waits.push_back(c | kWaitPartial);
            owaited[c] = 1;
            orr(Kb.data(), oclo.data() + (size_t)c * WD, WD);
            return odone[c] + kC2;
        }
        int top = c;
        while (parent[top] >= 0 && fseq[parent[top]] < seq && done[parent[top]] + kC2 <= t + kSlack) top = parent[top];
        waits.push_back(top);
        waited[top] = 1;
        orr(Kb.data(), clo.data() + (size_t)top * WD, WD);
        return done[top] + kC2;
    };
    // a block whose rows' outside terms are all applied and visible to warp w
    // by time t (through records created before now)
    auto block_ready = [&](int b, int w, double t) {
        const Block& B = blocks[b];
        if (B.scheduled || B.outside_left > 0) return false;
        for (int r : B.rows)
            if (oseq[r] >= seq || (oend[r] != w && oend[r] >= 0 && odone[r] + kC2 > t + kSlack)) return false;
        return true;
    };

    while (true) {
        if (++guard > 256LL * n + 100000) return "sweep schedule did not converge";
        int w = -1;
        for (int q = 0; q < W; q++) {
            if (wp[q].ended) continue;
            if (w < 0 || wp[q].T < wp[w].T || (wp[q].T == wp[w].T && wp[w].idle && !wp[q].idle)) w = q;
        }
        if (w < 0) break;
        WarpProg& P = wp[w];
        const double t = P.T;
        uint64_t* Kw = K.data() + (size_t)w * WD;

        // (a) segments that ended: rows final, outside terms applied, or paused
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
            if (blk[r] < 0 && G.q == nt[r]) {
                cr.gflags[g] |= kGFinal;
                if (backward) {
                    cr.gflags[g] |= kGDivide;
                    cr.diag[g] = diag[r];
                }
                done[r] = t + kCCtrl;
                fseq[r] = seq;
                set(Kw, r);
                remaining--;
            } else if (blk[r] >= 0 && G.q == nout[r]) {
                cr.gflags[g] |= kGPartial;   // dropped below unless another warp's block reads it
                odone[r] = t + kCCtrl;
                oseq[r] = seq;
                oend[r] = w;
                blocks[blk[r]].outside_left--;
            }
            G.row = -1;
            any = true;
        }
        if (any)
            open.erase(std::remove_if(open.begin(), open.end(),
                                      [&](int r) { return fseq[r] != kUnsched || oseq[r] != kUnsched; }),
                       open.end());
        std::copy(Kw, Kw + WD, Kb.begin());
        std::vector<int> waits;
        double ready = t;

        // rows this warp could start now, most urgent first
        cand.clear();
        double next_event = kInf;
        for (int r : open) {
            if (!may_take(w, r)) continue;
            if (prog[r] < lim(r)) {
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
        double top_open = 0.0;   // the most urgent row this warp may take (started or not)
        for (int r : open)
            if (may_take(w, r)) top_open = std::max(top_open, prio[r]);

        // (b) the most urgent ready block, if it beats every row this warp can start now
        int pick_block = -1;
        for (size_t b = 0; b < blocks.size(); b++)
            if (block_ready((int)b, w, t) && (pick_block < 0 || prio[blocks[b].rows[0]] > prio[blocks[pick_block].rows[0]]))
                pick_block = (int)b;
        bool groups_idle = true;
        for (int g = 0; g < kBundleRows; g++) groups_idle &= P.g[g].row < 0;
        const bool block_first = pick_block >= 0 && (cand.empty() || prio[blocks[pick_block].rows[0]] >= prio[cand[0]]);
        if (block_first && groups_idle && !any) {
            Block& B = blocks[pick_block];
            B.scheduled = true;
            const int s = (int)B.rows.size();
            for (int r : B.rows)
                if (oend[r] != w && oend[r] >= 0 && !test(Kb.data(), r)) ready = std::max(ready, add_wait(waits, r, true, t));
            while ((int)waits.size() > kCtrlWaits) {   // waits beyond one record's go to wait-only control records
                ControlRecord wr;
                memset(&wr, 0, sizeof(wr));
                for (int g = 0; g < kBundleRows; g++) wr.row[g] = (uint16_t)n;
                wr.nwait = (uint8_t)kCtrlWaits;
                for (int i = 0; i < kCtrlWaits; i++) wr.wait[i] = (uint16_t)waits[waits.size() - kCtrlWaits + i];
                waits.resize(waits.size() - kCtrlWaits);
                memcpy(new_record(P, 1), &wr, sizeof(wr));
                ready += kCCtrl;
                out.prewaits += kCtrlWaits;
            }
            BlockRecord br;
            memset(&br, 0, sizeof(br));
            br.first = (uint16_t)B.rows[0];
            br.size = (uint16_t)s;
            br.backward = backward ? 1 : 0;
            br.nwait = (uint8_t)waits.size();
            br.flags = kCtrlBlock;
            for (size_t i = 0; i < waits.size(); i++) br.wait[i] = (uint16_t)waits[i];
            // values round by round (layout in sbenv_dev.h) into the sweep's
            // value region; v(i, j) is row i's in-block term from row j
            auto v = [&](int i, int j) { return terms[B.rows[i]][nout[B.rows[i]] + j]; };
            for (int i = 1; i < s; i++)
                for (int j = 0; j < i; j++)
                    if (v(i, j).first != B.rows[j]) return "dense block term out of order";
            br.values = (uint32_t)(block_vals.size() * 8);   // region-relative until serialised
            for (int c0 = 0; c0 < s; c0 += 4) {
                for (int k = 0; k < 4; k++) block_vals.push_back(backward && c0 + k < s ? diag[B.rows[c0 + k]] : 0.0);
                for (int r = 1; r < 4; r++)
                    for (int k = 0; k < r; k++) block_vals.push_back(c0 + r < s ? v(c0 + r, c0 + k).second : 0.0);
                block_vals.push_back(0.0);
                block_vals.push_back(0.0);
                for (int q = 0; q < 4; q++)
                    for (int j = 0; j < c0; j++) block_vals.push_back(c0 + q < s ? v(c0 + q, j).second : 0.0);
            }
            memcpy(new_record(P, 1), &br, sizeof(br));
            double tj = std::max(t, ready) + kCCtrl;
            for (int j = 0; j < s; j++) {
                const int r = B.rows[j];
                if (j % 4 == 0) tj += block_round(s, j);
                done[r] = tj;
                fseq[r] = seq;
                owner[r] = w;
                set(Kb.data(), r);
                orr(Kb.data(), clo.data() + (size_t)r * WD, WD);
                remaining--;
            }
            out.prewaits += (int64_t)waits.size();
            std::copy(Kb.begin(), Kb.end(), Kw);
            P.T = tj;
            out.sim_cycles = std::max(out.sim_cycles, P.T);
            seq++;
            for (auto& x : wp) x.idle = false;
            continue;
        }

        // (c) new segments for the free groups, most urgent rows first (none
        // while a more urgent block waits for this warp's groups to drain)
        if (block_first) cand.clear();
        bool others_busy = false;   // another warp may still change the state
        for (int q = 0; q < W; q++)
            if (q != w && !wp[q].ended && (wp[q].T > t || !wp[q].idle)) others_busy = true;
        for (int pass = 0; pass < 2; pass++) {
            // pass 1 only when the warp would otherwise wait for nothing: short segments allowed
            const bool strict = pass == 0;
            bool started = false;
            double short_event = kInf;
            size_t ci = 0;
            for (int g = 0; g < kBundleRows && ci < cand.size(); g++) {
                if (P.g[g].row >= 0) continue;
                while (ci < cand.size()) {
                    const int r = cand[ci++];
                    if (in_use[r]) continue;
                    int q = prog[r];
                    double rdy = ready;
                    const size_t w0 = waits.size();
                    Ksave.assign(Kb.begin(), Kb.end());
                    int stop = -1;
                    while (q < lim(r)) {
                        const int c = terms[r][q].first;
                        if (!test(Kb.data(), c)) {
                            if (!(fseq[c] < seq && done[c] + kC2 <= t + kSlack) || (int)waits.size() >= kCtrlWaits) {
                                stop = c;
                                break;
                            }
                            rdy = std::max(rdy, add_wait(waits, c, false, t));
                        }
                        q++;
                    }
                    const bool ends = q == lim(r);
                    if (q == prog[r] && !ends) continue;   // not a single term ready after all
                    if (strict && !ends && q - prog[r] < kMinSeg && prio[r] < kCritical * top_open) {
                        // too short a run for an off-critical row: its waits are not kept
                        std::copy(Ksave.begin(), Ksave.end(), Kb.begin());
                        waits.resize(w0);
                        if (stop >= 0 && fseq[stop] != kUnsched) short_event = std::min(short_event, done[stop] + kC2 - kSlack);
                        continue;
                    }
                    ready = rdy;
                    P.g[g] = Group{r, prog[r], q};
                    in_use[r] = 1;
                    owner[r] = w;
                    cr.gflags[g] |= kGSwitch;
                    cr.row[g] = (uint16_t)r;
                    started = true;
                    out.pieces++;
                    break;
                }
            }
            next_event = std::min(next_event, short_event);
            any |= started;
            if (started || !strict || others_busy || std::isfinite(next_event) || cand.empty()) break;
            ci = 0;   // nothing else will happen: take a short segment after all
        }
        if (any || !waits.empty()) {
            cr.nwait = (uint8_t)waits.size();
            for (size_t i = 0; i < waits.size(); i++) cr.wait[i] = (uint16_t)waits[i];
            out.prewaits += (int64_t)waits.size();
            std::copy(Kb.begin(), Kb.end(), Kw);
            memcpy(new_record(P, 1), &cr, sizeof(cr));
            P.T = std::max(t, ready) + kCCtrl;
            out.sim_cycles = std::max(out.sim_cycles, P.T);
            seq++;
            for (auto& x : wp) x.idle = false;
        }
        // (d) run term records until the first active segment ends
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
                memcpy(new_record(P, 0), &tr, sizeof(tr));
                out.blocks++;
            }
            P.T += nb * kCBlk;
            out.sim_cycles = std::max(out.sim_cycles, P.T);
            continue;
        }
        if (any) continue;   // the control record moved time on
        // (e) nothing running: end, or wait for the next event
        bool future = false;
        for (int r : open)
            if ((owner[r] == -1 || owner[r] == w) && (home[r] == -1 || home[r] == w)) { future = true; break; }
        for (const Block& B : blocks) future |= !B.scheduled;
        if (!future) {
            ControlRecord end;
            memset(&end, 0, sizeof(end));
            for (int g = 0; g < kBundleRows; g++) end.row[g] = (uint16_t)n;
            end.flags = kCtrlEnd;
            memcpy(new_record(P, 1), &end, sizeof(end));
            P.ended = true;
            continue;
        }
        for (const Block& B : blocks) {   // block rows' outside terms becoming visible
            if (B.scheduled || B.outside_left > 0) continue;
            for (int r : B.rows)
                if (oend[r] != w && oend[r] >= 0 && odone[r] + kC2 - kSlack > t)
                    next_event = std::min(next_event, odone[r] + kC2 - kSlack);
        }
        bool other_now = false;
        for (int q = 0; q < W; q++) {
            if (q == w || wp[q].ended) continue;
            if (wp[q].T > t) next_event = std::min(next_event, wp[q].T);
            if (wp[q].T == t && wp[q].idle) next_event = std::min(next_event, wp[q].wake);
            other_now |= (wp[q].T == t && !wp[q].idle);
        }
        if (other_now) {
            P.idle = true;
            P.wake = next_event;
            continue;
        }
        if (!std::isfinite(next_event)) return "sweep schedule deadlocked";
        P.T = next_event;
        P.idle = false;
    }
    if (remaining != 0) return "sweep schedule left rows unfinished";

    for (int r = 0; r < n && out.unpublished_row < 0; r++)
        if (!waited[r] && !owaited[r]) out.unpublished_row = r;
    // ---- publish bits and record summaries, then stage padding. A control
    // record finishes the row its group was given before; a block publishes
    // the rows another warp waits for.
    for (int w = 0; w < W; w++) {
        WarpProg& P = wp[w];
        int cur[kBundleRows];
        for (int g = 0; g < kBundleRows; g++) cur[g] = -1;
        bool ctrl = true;   // a program starts with a control record
        const int nrec = (int)(P.rec.size() / kRecordBytes);
        for (int i = 0; i < nrec; i++) {
            uint8_t* r = P.rec.data() + (size_t)i * kRecordBytes;
            if (!ctrl) {
                ctrl = (reinterpret_cast<TermRecord*>(r)->col[0][0] & kNextIsCtrl) != 0;
                continue;
            }
            ControlRecord* c = reinterpret_cast<ControlRecord*>(r);
            if (c->flags & kCtrlBlock) {
                BlockRecord* b = reinterpret_cast<BlockRecord*>(r);
                for (int j = 0; j < b->size; j++) {
                    const int row = backward ? b->first - j : b->first + j;
                    if (waited[row]) {
                        b->publish |= uint64_t(1) << j;
                        out.publishes++;
                    }
                }
                out.block_rows += b->size;
                ctrl = (b->flags & kCtrlNext) != 0;
                continue;
            }
            out.bundles++;
            for (int g = 0; g < kBundleRows; g++) {
                if (!(c->gflags[g] & kGSwitch)) continue;
                if (cur[g] >= 0) {
                    if ((c->gflags[g] & kGFinal) && waited[cur[g]]) c->gflags[g] |= kGPublish;
                    if ((c->gflags[g] & kGPartial) && !owaited[cur[g]]) c->gflags[g] &= (uint8_t)~kGPartial;
                }
                if (c->gflags[g] & (kGPublish | kGPartial)) {
                    c->flags |= kCtrlPublish;
                    out.publishes++;
                }
                if (c->gflags[g] & kGDivide) c->flags |= kCtrlDivide;
                cur[g] = c->row[g] < n ? c->row[g] : -1;
            }
            ctrl = (c->flags & kCtrlNext) != 0;
        }
        const size_t stages = (P.rec.size() + kStageBytes - 1) / kStageBytes;
        P.rec.resize(stages * kStageBytes, 0);
        out.warp_off[w] = (uint32_t)(out.bytes.size() / kStageBytes);
        out.warp_stages[w] = (uint32_t)stages;
        out.bytes.insert(out.bytes.end(), P.rec.begin(), P.rec.end());
    }
    // the value region after the programs; block records point into it
    const uint32_t region = (uint32_t)out.bytes.size();
    if ((uint64_t)region + block_vals.size() * 8 > 0xFFFFFFF0ull) return "sweep buffer too large";
    for (int w = 0; w < W; w++) {
        uint8_t* base = out.bytes.data() + (size_t)out.warp_off[w] * kStageBytes;
        const int nrec = (int)(out.warp_stages[w] * kRecordsPerStage);
        bool ctrl = true;
        for (int i = 0; i < nrec; i++) {
            uint8_t* r = base + (size_t)i * kRecordBytes;
            if (!ctrl) {
                ctrl = (reinterpret_cast<TermRecord*>(r)->col[0][0] & kNextIsCtrl) != 0;
                continue;
            }
            ControlRecord* c = reinterpret_cast<ControlRecord*>(r);
            if (c->flags & kCtrlBlock) reinterpret_cast<BlockRecord*>(r)->values += region;
            else if (c->flags & kCtrlEnd) break;
            ctrl = (c->flags & kCtrlNext) != 0;
        }
    }
    const size_t at = out.bytes.size();
    out.bytes.resize(at + block_vals.size() * 8);
    if (!block_vals.empty()) memcpy(out.bytes.data() + at, block_vals.data(), block_vals.size() * 8);
    return "";
}

}  // namespace sbenv
