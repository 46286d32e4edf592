// Sweep programs for the solve kernel: a static list schedule of the
// triangular factor's rows over the warps of one solve CTA.
//
// The reference solves L y = b, U z = y by column push
// (complete_port/csim/sb_lu.c:38-63): column j, once final, is subtracted from
// every row below (L) or above (U) it. Here every row pulls its terms itself,
// in exactly the order the push would deliver them, so the rounding sequence
// of each row is unchanged. Rows are spread over the warps by simulating the
// sweep with a simple cost model; the model decides only speed, never
// results: a bundle reads another warp's row only after waiting for the ready
// flag of that row or of a row whose completion implies it.
//
// Deadlock freedom: a bundle waits only for rows whose final piece lies in a
// bundle created earlier in the simulation (smaller sequence number), and
// every warp runs its bundles in creation order. The unfinished bundle with
// the smallest sequence number therefore always has its inputs done and its
// warp at it.
#include "sweep_sched.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>

namespace sbenv {

namespace {

// Cost model of one warp, in cycles. Only used to order the work.
constexpr double kC0 = 120;    // bundle start: stage waits, header, pre-waits, row loads
constexpr double kCBlk = 60;   // one TermBlock (four terms of four rows)
constexpr double kCEnd = 30;   // bundle end: stores, warp barrier
constexpr double kC2 = 80;     // release store until another warp's acquire sees it
constexpr double kCPub = 30;   // publishing a row
constexpr double kSlack = 150; // a row may be picked this long before its next input is ready
constexpr int kPartnerPool = 16;   // bundle partners are chosen among this many top rows
constexpr int kMaxPre = 8 * kMaxPreItems;
constexpr int kMaxBlk = (kMaxBundleBytes - bundle_bytes(kMaxPreItems, true, 0)) / kTermBlockBytes;
constexpr int kUnsched = std::numeric_limits<int>::max();
static_assert(kMaxBlk >= 1, "a bundle must hold one term block");

struct Piece {
    int row = -1, q0 = 0, q1 = 0;
    bool fin = false;
    int fin_blk = kFinNever;
};

struct Bundle {
    int nblk = 0;
    Piece p[kBundleRows];
    std::vector<int> pre;   // rows the warp waits for before the bundle
};

inline bool test(const uint64_t* s, int i) { return (s[i >> 6] >> (i & 63)) & 1u; }
inline void set(uint64_t* s, int i) { s[i >> 6] |= uint64_t(1) << (i & 63); }
inline void orr(uint64_t* d, const uint64_t* s, int w) {
    for (int k = 0; k < w; k++) d[k] |= s[k];
}

}  // namespace

std::string build_sweep(int n, const std::vector<std::vector<std::pair<int, double>>>& terms, bool backward,
                        const std::vector<double>& diag, int ring_stages, HostSweep& out) {
    out = HostSweep();
    if (n <= 0 || n >= 0xFFFF) return "factor too large for the sweep format";
    if (ring_stages < kStagesMin || ring_stages > kStagesMax) return "unsupported ring depth";
    out.ring_stages = ring_stages;
    const size_t ring_bytes = (size_t)ring_stages * kStageBytes;
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
        prio[i] = best + kC2 + kC0 + kCBlk * std::ceil(nt[i] / (double)kTermSteps);
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
    std::vector<double> free_t(W, 0.0);
    std::vector<std::vector<Bundle>> wb(W);
    std::vector<int> cand;
    std::vector<uint64_t> Kb(WD);
    std::vector<char> waited(n, 0);
    int seq = 0;
    int64_t guard = 0;
    // idle[w]: w found no work at free_t[w] in the current state (reset whenever
    // a bundle is created); among warps free at the same time, busy ones go first
    std::vector<char> idle(W, 0);
    while (remaining > 0) {
        if (++guard > 64LL * n + 100000) return "sweep schedule did not converge";
        int w = 0;
        for (int q = 1; q < W; q++)
            if (free_t[q] < free_t[w] || (free_t[q] == free_t[w] && idle[w] && !idle[q])) w = q;
        const double t = free_t[w];
        uint64_t* Kw = K.data() + (size_t)w * WD;
        cand.clear();
        double next_event = std::numeric_limits<double>::infinity();
        for (int r : open) {
            if (owner[r] != -1 && owner[r] != w) continue;
            if (home[r] != -1 && home[r] != w) continue;
            if (prog[r] < nt[r]) {
                const int c = terms[r][prog[r]].first;
                if (!test(Kw, c)) {
                    if (fseq[c] == kUnsched) continue;
                    if (done[c] + kC2 - kSlack > t) { next_event = std::min(next_event, done[c] + kC2 - kSlack); continue; }
                }
            }
            cand.push_back(r);
        }
        if (cand.empty()) {
            bool other_now = false;
            for (int q = 0; q < W; q++) {
                if (q != w && free_t[q] > t) next_event = std::min(next_event, free_t[q]);
                other_now |= (q != w && free_t[q] == t && !idle[q]);
            }
            if (other_now) { idle[w] = 1; continue; }
            if (!std::isfinite(next_event)) return "sweep schedule deadlocked";
            free_t[w] = next_event;
            idle[w] = 0;
            continue;
        }
        std::fill(idle.begin(), idle.end(), 0);
        // the most urgent row, then partners of similar remaining length among
        // the next most urgent ones (lock-step rows pad to the longest)
        const int pool_n = std::min<int>(kPartnerPool, (int)cand.size());
        std::partial_sort(cand.begin(), cand.begin() + pool_n, cand.end(), [&](int a, int b) {
            if (prio[a] != prio[b]) return prio[a] > prio[b];
            return backward ? a > b : a < b;
        });
        const int take = std::min<int>(kBundleRows, pool_n);
        {
            const int len0 = std::min(nt[cand[0]] - prog[cand[0]], kMaxBlk * kTermSteps);
            std::stable_sort(cand.begin() + 1, cand.begin() + pool_n, [&](int a, int b) {
                const int la = std::min(nt[a] - prog[a], kMaxBlk * kTermSteps);
                const int lb = std::min(nt[b] - prog[b], kMaxBlk * kTermSteps);
                return std::abs(la - len0) < std::abs(lb - len0);
            });
        }
        // the bundle starts once the first inputs of its rows are ready
        double T0 = t;
        for (int g = 0; g < take; g++) {
            const int r = cand[g];
            if (prog[r] < nt[r]) {
                const int c = terms[r][prog[r]].first;
                if (!test(Kw, c)) T0 = std::max(T0, done[c] + kC2);
            }
        }
        // every group takes the terms whose inputs are ready at T0: known to the
        // warp, or covered by a pre-wait (the highest row above the input that is
        // also ready, so that one flag covers as much as possible)
        Bundle B;
        std::copy(Kw, Kw + WD, Kb.begin());
        int steps_max = 0, ng = 0;
        for (int g = 0; g < take; g++) {
            const int r = cand[g];
            int q = prog[r];
            int steps = 0;
            while (q < nt[r] && steps < kMaxBlk * kTermSteps) {
                const int c = terms[r][q].first;
                if (!test(Kb.data(), c)) {
                    if (!(fseq[c] < seq && done[c] + kC2 <= T0) || (int)B.pre.size() >= kMaxPre) break;
                    int top = c;
                    while (parent[top] >= 0 && fseq[parent[top]] < seq && done[parent[top]] + kC2 <= T0)
                        top = parent[top];
                    B.pre.push_back(top);
                    orr(Kb.data(), clo.data() + (size_t)top * WD, WD);
                }
                q++;
                steps++;
            }
            const bool fin = q == nt[r];
            if (steps == 0 && !fin) continue;   // nothing ready for this row after all
            Piece& p = B.p[ng++];
            p.row = r;
            p.q0 = prog[r];
            p.q1 = q;
            p.fin = fin;
            p.fin_blk = fin ? (steps + kTermSteps - 1) / kTermSteps : kFinNever;
            steps_max = std::max(steps_max, steps);
        }
        B.nblk = (steps_max + kTermSteps - 1) / kTermSteps;
        for (int top : B.pre) waited[top] = 1;
        std::copy(Kb.begin(), Kb.end(), Kw);
        const double tstart = T0 + kC0;
        for (int g = 0; g < ng; g++) {
            Piece& p = B.p[g];
            owner[p.row] = w;
            prog[p.row] = p.q1;
            out.pieces++;
            if (p.fin) {
                done[p.row] = tstart + p.fin_blk * kCBlk + kCPub;
                fseq[p.row] = seq;
                set(Kw, p.row);
                remaining--;
            }
        }
        out.prewaits += (int64_t)B.pre.size();
        open.erase(std::remove_if(open.begin(), open.end(), [&](int r) { return fseq[r] != kUnsched; }),
                   open.end());
        free_t[w] = tstart + B.nblk * kCBlk + kCEnd;
        out.sim_cycles = std::max(out.sim_cycles, free_t[w]);
        wb[w].push_back(std::move(B));
        seq++;
    }

    // ---- serialise ----
    std::vector<uint8_t> stream;
    auto put = [&](const void* src, size_t sz) {
        const size_t at = stream.size();
        stream.resize(at + sz);
        memcpy(stream.data() + at, src, sz);
    };
    for (int w = 0; w < W; w++) {
        stream.clear();
        for (const Bundle& B : wb[w]) {
            BundleHeader h;
            memset(&h, 0, sizeof(h));
            h.nblk = (uint16_t)B.nblk;
            double dg[kBundleRows] = {1.0, 1.0, 1.0, 1.0};
            const int npre = ((int)B.pre.size() + 7) / 8;
            for (int g = 0; g < kBundleRows; g++) {
                const Piece& p = B.p[g];
                h.row[g] = (uint16_t)(p.row < 0 ? n : p.row);
                h.fin[g] = p.row >= 0 && p.fin ? (uint8_t)p.fin_blk : kFinNever;
                if (p.row >= 0 && p.fin && waited[p.row]) { h.flags |= (uint16_t)(1u << g); out.publishes++; }
                if (p.row >= 0 && p.fin && backward) {
                    h.flags |= (uint16_t)(1u << (4 + g));
                    dg[g] = diag[p.row];
                }
            }
            h.flags |= (uint16_t)(npre << 8);
            const size_t bytes = (size_t)bundle_bytes(npre, (h.flags & 0xF0) != 0, B.nblk);
            if (bytes > (size_t)kMaxBundleBytes) return "sweep bundle too large";
            const size_t ro = stream.size() % ring_bytes;
            if (ro + bytes > ring_bytes) {   // continue at the start of the ring
                BundleHeader skip;
                memset(&skip, 0, sizeof(skip));
                skip.flags = kBundleSkip;
                for (int g = 0; g < kBundleRows; g++) skip.fin[g] = kFinNever;
                put(&skip, sizeof(skip));
                stream.resize(stream.size() + (ring_bytes - ro - sizeof(skip)), 0);
            }
            put(&h, sizeof(h));
            for (int it = 0; it < npre; it++) {
                uint16_t rows8[8];
                for (int k = 0; k < 8; k++) {
                    const size_t at = (size_t)it * 8 + k;
                    rows8[k] = (uint16_t)(at < B.pre.size() ? B.pre[at] : n);
                }
                put(rows8, sizeof(rows8));
            }
            if (h.flags & 0xF0) put(dg, sizeof(dg));
            for (int b = 0; b < B.nblk; b++) {
                double val[kBundleRows][kTermSteps];
                uint16_t col[kBundleRows][kTermSteps];
                for (int g = 0; g < kBundleRows; g++)
                    for (int s = 0; s < kTermSteps; s++) {
                        const Piece& p = B.p[g];
                        const int a = b * kTermSteps + s;
                        if (p.row >= 0 && a < p.q1 - p.q0) {
                            const auto& tm = terms[p.row][p.q0 + a];
                            val[g][s] = tm.second;
                            col[g][s] = (uint16_t)tm.first;
                        } else {   // padding: 0 * x[n] (the zero slot) leaves the row unchanged
                            val[g][s] = 0.0;
                            col[g][s] = (uint16_t)n;
                        }
                    }
                uint8_t blk[kTermBlockBytes];
                memcpy(blk, val, sizeof(val));
                memcpy(blk + sizeof(val), col, sizeof(col));
                put(blk, sizeof(blk));
                out.blocks++;
            }
            out.bundles++;
        }
        BundleHeader end;
        memset(&end, 0, sizeof(end));
        end.flags = kBundleEnd;
        for (int g = 0; g < kBundleRows; g++) end.fin[g] = kFinNever;
        put(&end, sizeof(end));
        stream.resize((stream.size() + kStageBytes - 1) / kStageBytes * kStageBytes, 0);
        out.warp_off[w] = (uint32_t)(out.bytes.size() / kStageBytes);
        out.warp_stages[w] = (uint32_t)(stream.size() / kStageBytes);
        out.bytes.insert(out.bytes.end(), stream.begin(), stream.end());
    }
    return "";
}

}  // namespace sbenv
