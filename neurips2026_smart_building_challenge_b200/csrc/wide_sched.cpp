// Level programs for the wide solve kernel (k_wide.cuh): a static schedule of
// one triangular sweep over the solver warps of a CTA, in levels.
//
// The reference solves L y = b, U z = y by column push
// (complete_port/csim/sb_lu.c:38-63): column j, once final, is subtracted from
// every row below (L) or above (U) it, so row i receives its terms in
// ascending (L) or descending (U) column order. Here every row pulls its
// terms itself, in runs ("segments") that follow exactly that order, so the
// rounding sequence of every row is the reference's.
//
// A segment may read rows finished before its level (any warp) and rows that
// its own warp finished earlier in the same level: a thread sees its own
// stores, so a chain of dependent rows -- a nested-dissection separator, each
// row reading all the earlier ones -- runs on one warp inside one level. Level
// l places, in this order:
//  (a) the finishing segment of every row whose remaining terms all read rows
//      final before level l, spread over the warps longest first;
//  (b) in sweep order, every row whose unfinished sources were all placed in
//      this level on one warp, appended to that warp behind them, while the
//      warp's load stays within the level's longest or a chain allowance;
//  (c) partial segments: the longest run of a waiting row's next terms whose
//      source rows are final before level l, on warps whose load stays within
//      the level's longest, the rows that finish soonest first. (c) moves the
//      outside terms of the separators' rows -- up to a few hundred per row --
//      off the chains.
// The warps do not meet at a barrier between levels: each waits only for the
// rows it reads (see the wait lists in sbenv_dev.h), so the levels fix the
// order of each warp's work and the grouping of the program into stages. The
// cost model counts one memory round trip per kWideGroup chunks of a segment,
// the kernel's real unit of latency. Every level's program is one contiguous
// block of at most kWideStageBytes; a level is closed when the next segment
// would not fit.
#include "wide_sched.h"

#include <algorithm>
#include <cstring>

namespace sbenv {

namespace {

// Cost model of one warp, in SM cycles; only used to place work.
constexpr double kCSeg = 100;       // a segment: its row's store and publication
constexpr double kCGroup = 600;     // kWideGroup chunks: one round trip of their source loads
constexpr double kCTerm = 8;        // a term (the dependent subtraction chain)
constexpr double kCBar = 300;       // a level: the start of its stage
constexpr double kChainCap = 4000;  // a warp's load a chain may reach in any level
constexpr int kMinPartial = 8;      // shortest partial segment

}  // namespace

std::string build_wide(int n, const std::vector<std::vector<std::pair<int, double>>>& terms, bool backward,
                       int stage0, WideFlags& flags, HostWide& out) {
    out = HostWide();
    if ((int)terms.size() != n) return "wide program: term lists do not match the row count";
    if ((int)flags.cnt.size() != n) return "wide program: progress state does not match the row count";
    if (n >= 0xFFFF) return "wide program: more than 65534 solved cells";
    for (int i = 0; i < n; i++)
        for (const auto& t : terms[i])
            if (t.first < 0 || t.first >= n || (backward ? t.first <= i : t.first >= i))
                return "wide program: a term outside the triangle";
    // dependency level of every row (rows without terms: 0 in L; U rows always
    // need their diagonal)
    std::vector<int> lev(n, 0);
    for (int p = 0; p < n; p++) {
        const int i = backward ? n - 1 - p : p;
        int d = 0;
        for (const auto& t : terms[i]) d = std::max(d, lev[t.first]);
        lev[i] = (terms[i].empty() && !backward) ? 0 : d + 1;
        out.terms += (int64_t)terms[i].size();
    }
    constexpr int kNever = 0x7FFFFFFF;
    const int max_chunks = (kWideStageBytes - kWideHdrBytes - 64 - (int)sizeof(WideSeg)) / (int)sizeof(WideChunk);
    std::vector<int> fin(n, kNever);    // level at which the row is finished (0: from the start)
    std::vector<int> fwarp(n, -1);      // the warp that finished it
    std::vector<int> prog(n, 0);        // terms applied so far
    std::vector<int> waiting;
    for (int i = 0; i < n; i++) {
        if (lev[i] == 0) fin[i] = 0;
        else waiting.push_back(i);
    }
    struct Item { int row, from, to, w; };
    struct Cand { int row, from, to; };
    std::vector<Item> items;
    std::vector<Cand> fins, parts;
    std::vector<double> load(kWideWarps);
    std::vector<uint8_t> placed(n, 0);
    std::vector<int> wmark((size_t)kWideWarps * n, 0);   // (warp, row) already counted in the level
    std::vector<int> need(n, 0);
    std::vector<int> touched;
    auto chunks_of = [](int from, int to) { return (to - from + 3) / 4; };
    auto cost = [&](int from, int to) {
        const int c = chunks_of(from, to);
        return kCSeg + kCGroup * ((c + kWideGroup - 1) / kWideGroup) + kCTerm * 4.0 * c;
    };
    auto least = [&]() { return (int)(std::min_element(load.begin(), load.end()) - load.begin()); };
    out.lev_off.push_back(0);
    for (int level = 1; !waiting.empty(); level++) {
        if (level > 4 * n + 4) return "wide program: no progress";
        const int stage = stage0 + level - 1;
        fins.clear();
        parts.clear();
        items.clear();
        std::fill(load.begin(), load.end(), 0.0);
        // bytes of the level block so far; the waits are counted as segments
        // are placed, from the progress before the level (an upper bound: a
        // source finished earlier in the level by the same warp needs none)
        int bytes = kWideHdrBytes + 16;
        auto new_waits = [&](int r, int from, int to, int w, bool mark) {
            int c = 0;
            auto one = [&](int q) {
                if (flags.cnt[q] <= 0 || flags.warp[q] == w || flags.stage[q] <= stage - kWideStages) return;
                int& m = wmark[(size_t)w * n + q];
                if (m == stage + 1) return;
                m = stage + 1;
                c++;
            };
            std::vector<int> undo;
            auto probe = [&](int q) {   // counts without marking
                const int before = c;
                one(q);
                if (c != before && !mark) undo.push_back(q);
            };
            probe(r);
            for (int a = from; a < to; a++) probe(terms[r][a].first);
            for (int q : undo) wmark[(size_t)w * n + q] = 0;
            return c;
        };
        auto fits = [&](int r, int from, int to, int w) {
            return bytes + 4 * new_waits(r, from, to, w, false) + (int)sizeof(WideSeg) +
                       (int)sizeof(WideChunk) * chunks_of(from, to) <= kWideStageBytes;
        };
        auto place = [&](int r, int from, int to, int w, bool last) {
            items.push_back({r, from, to, w});
            load[w] += cost(from, to);
            bytes += 4 * new_waits(r, from, to, w, true) + (int)sizeof(WideSeg) +
                     (int)sizeof(WideChunk) * chunks_of(from, to);
            prog[r] = to;
            placed[r] = 1;
            if (last) {
                fin[r] = level;
                fwarp[r] = w;
            }
        };
        for (int r : waiting) {
            const auto& t = terms[r];
            int q = prog[r];
            while (q < (int)t.size() && fin[t[q].first] < level) q++;
            if (q == (int)t.size()) fins.push_back({r, prog[r], q});
            else if (q - prog[r] >= kMinPartial) parts.push_back({r, prog[r], q});
        }
        // (a) rows ready at the level, longest first
        std::stable_sort(fins.begin(), fins.end(), [&](const Cand& a, const Cand& b) {
            return a.to - a.from > b.to - b.from;
        });
        for (const Cand& c : fins) {
            const int w = least();
            // a row too long for one stage: its first run goes out as a partial segment
            if (chunks_of(c.from, c.to) > max_chunks) {
                const int to = c.from + 4 * (max_chunks / 2);
                if (fits(c.row, c.from, to, w)) place(c.row, c.from, to, w, false);
                continue;
            }
            if (fits(c.row, c.from, c.to, w)) place(c.row, c.from, c.to, w, true);
        }
        double span = *std::max_element(load.begin(), load.end());
        // (b) chains behind rows placed in this level, in sweep order
        for (int p = 0; p < n; p++) {
            const int r = backward ? n - 1 - p : p;
            if (fin[r] != kNever || placed[r]) continue;
            const auto& t = terms[r];
            int w = -1;
            bool ok = true;
            for (int a = prog[r]; a < (int)t.size() && ok; a++) {
                const int s = t[a].first;
                if (fin[s] < level) continue;
                if (fin[s] != level || (w >= 0 && fwarp[s] != w)) ok = false;
                else w = fwarp[s];
            }
            if (!ok || w < 0) continue;
            if (chunks_of(prog[r], (int)t.size()) > max_chunks) continue;
            if (load[w] + cost(prog[r], (int)t.size()) > std::max(span, kChainCap)) continue;
            if (!fits(r, prog[r], (int)t.size(), w)) continue;
            place(r, prog[r], (int)t.size(), w, true);
        }
        span = *std::max_element(load.begin(), load.end());
        // (c) partial segments within the level's span
        std::stable_sort(parts.begin(), parts.end(), [&](const Cand& a, const Cand& b) {
            if (lev[a.row] != lev[b.row]) return lev[a.row] < lev[b.row];
            return a.to - a.from > b.to - b.from;
        });
        for (const Cand& c : parts) {
            if (placed[c.row]) continue;
            const int to = std::min(c.to, c.from + 4 * (max_chunks / 2));
            const int w = least();
            if (load[w] + cost(c.from, to) > span || !fits(c.row, c.from, to, w)) continue;
            place(c.row, c.from, to, w, false);
            out.partial++;
        }
        if (items.empty()) return "wide program: a level places no segment";
        out.sim_cycles += span + kCBar;
        for (const Item& it : items) placed[it.row] = 0;
        waiting.erase(std::remove_if(waiting.begin(), waiting.end(), [&](int r) { return fin[r] == level; }),
                      waiting.end());
        // emit the level block: header (first segment and first wait of each
        // warp, relative), the waits, then the segments warp by warp, then
        // their chunks in the same order
        std::vector<int32_t> hdr(2 * (kWideWarps + 1), 0);
        std::vector<uint32_t> waits;
        std::vector<WideSeg> segs;
        std::vector<WideChunk> chunks;
        for (int w = 0; w < kWideWarps; w++) {
            hdr[w] = (int32_t)segs.size();
            hdr[kWideWarps + 1 + w] = (int32_t)waits.size();
            touched.clear();
            auto want = [&](int r, int count) {   // count `count` of row r made by another warp recently?
                if (count <= 0 || flags.warp[r] == w || flags.stage[r] <= stage - kWideStages) return;
                if (need[r] == 0) touched.push_back(r);
                need[r] = std::max(need[r], count);
            };
            for (const Item& it : items) {
                if (it.w != w) continue;
                // its own row's previous segment, then the sources (complete in
                // this sweep: their last segment so far)
                want(it.row, flags.cnt[it.row]);
                for (int a = it.from; a < it.to; a++) want(terms[it.row][a].first, flags.cnt[terms[it.row][a].first]);
                WideSeg s;
                s.row = (uint32_t)it.row;
                s.chunk0 = (uint32_t)chunks.size();
                s.nchunk = (uint32_t)chunks_of(it.from, it.to);
                flags.cnt[it.row]++;
                flags.stage[it.row] = stage;
                flags.warp[it.row] = w;
                if (flags.cnt[it.row] > 0xFFFF) return "wide program: too many segments of one row";
                s.fin = ((backward && it.to == (int)terms[it.row].size()) ? 1u : 0u) |
                        ((uint32_t)flags.cnt[it.row] << 16);
                for (int a = it.from; a < it.to; a += 4) {
                    WideChunk ch;
                    for (int u = 0; u < 4; u++) {
                        const bool in = a + u < it.to;
                        ch.v[u] = in ? terms[it.row][a + u].second : 0.0;
                        ch.off[u] = (uint32_t)((in ? terms[it.row][a + u].first : n) * kWideEnvs * 8);
                    }
                    chunks.push_back(ch);
                }
                segs.push_back(s);
            }
            std::sort(touched.begin(), touched.end());
            for (int r : touched) {
                waits.push_back(((uint32_t)r << 16) | (uint32_t)need[r]);
                need[r] = 0;
            }
        }
        hdr[kWideWarps] = (int32_t)segs.size();
        hdr[2 * kWideWarps + 1] = (int32_t)waits.size();
        out.waits += (int64_t)waits.size();
        while (waits.size() % 4) waits.push_back(0xFFFFFFFFu);   // padding (never read)
        const size_t nb = kWideHdrBytes + waits.size() * 4 + segs.size() * sizeof(WideSeg) +
                          chunks.size() * sizeof(WideChunk);
        if (nb > (size_t)kWideStageBytes) return "wide program: a level exceeds its stage";
        const size_t base = out.blocks.size();
        out.blocks.resize(base + nb, 0);
        uint8_t* dst = out.blocks.data() + base;
        memcpy(dst, hdr.data(), hdr.size() * sizeof(int32_t));
        memcpy(dst + kWideHdrBytes, waits.data(), waits.size() * 4);
        memcpy(dst + kWideHdrBytes + waits.size() * 4, segs.data(), segs.size() * sizeof(WideSeg));
        memcpy(dst + kWideHdrBytes + waits.size() * 4 + segs.size() * sizeof(WideSeg), chunks.data(),
               chunks.size() * sizeof(WideChunk));
        out.lev_off.push_back((uint32_t)out.blocks.size());
        out.max_bytes = std::max(out.max_bytes, (int)nb);
        out.segs += (int64_t)segs.size();
        out.chunks += (int64_t)chunks.size();
        out.nlev = level;
    }
    return "";
}

}  // namespace sbenv
