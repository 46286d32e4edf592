// Device-side table and state descriptors shared by the host builder
// (tables.cpp, sweep_sched.cpp, env.cu) and the kernels (k_*.cuh).
//
// Terminology (the reference's domain):
//   scenario  one SBB1 blob = one building x one weather/calendar;
//   group     scenarios whose geometry and thermal factors are byte-identical,
//             so they share one set of device solver tables;
//   slab      the envs of one group that one solve CTA holds in shared memory;
//   row order the row index space of the factored matrix B = Pr A Pc: solved
//             cell t sits at row position i with t = inv(perm_r)[i]. The field
//             of every env is kept in "extended row order": positions [0, n)
//             are the solved cells in row order, [n, ncv) the unsolved cells.
#pragma once
#include <cstdint>

#ifdef __CUDACC__
#define SB_HD __host__ __device__
#else
#define SB_HD
#endif

namespace sbenv {

constexpr int kObs = 1024;             // OBS_SIZE (complete_port/gpu/smart_buildings.cu:33)
constexpr int kCont = 256;             // SB_CONT
constexpr int kDisc = 16;              // SB_DISC
constexpr int kAct = kCont + kDisc;    // NUM_ATNS
constexpr int kMaskWidth = kCont + 2 * kDisc;
constexpr int kParts = 8;              // per-step log terms (smart_buildings.cu:101-115)
constexpr int kSolveThreads = 512;
constexpr int kMaxK = 128;             // coupled VAVs (dense air-side system in shared memory)
constexpr int kMaxAhu = 16;
constexpr int kMaxConvRoom = 8192;     // cells of one convection room

// Error codes written to the device status word (first error wins).
enum : int {
    kErrNone = 0,
    kErrRingTimeout = 1,   // a schedule stage never arrived (bounded mbarrier wait)
    kErrBadChunk = 2,      // reserved
    kErrConvOverflow = 3,  // convection swap list exceeded its buffer
    kErrDenseSingular = 4, // reserved: the reference tolerates a zero pivot, so do we
    kErrWaitTimeout = 5,   // a row's ready flag never arrived (bounded spin)
    kErrBadBundle = 6      // a sweep bundle header failed its consistency check
};

// Solve schedule ("sweep program"), built on the host (sweep_sched.cpp).
//
// Each of the kSweepWarps warps of a solve CTA runs its own program. The warp
// is four lane groups (kGroupLanes lanes each, one per env of the slab); each
// group works through its own sequence of rows, and the groups advance in
// lock step, four terms per group per term record. Every term subtracts
// val * x[col] from the group's accumulator, in the order the reference's
// column push would deliver it (bit-exact). Control records switch groups to
// new rows: they finish the ending rows (backward sweep: divide by the
// diagonal; publish with a release store of the sweep's epoch where another
// warp reads them), then wait (acquire) for the rows of other warps that the
// new rows read, then load the new rows' accumulators.
//
// A block record solves a dense block of up to kMaxBlockRows consecutive rows
// (in sweep order) whose terms among themselves form a full triangle (the
// separators of the nested-dissection order): the whole warp works on it,
// lane group q holding the block's rows i = q mod 4, one lane per env. The
// block is solved in rounds of four rows c0..c0+3 (left-looking): each of
// the round's rows first pulls its terms from the rows of the earlier rounds
// (final in shared memory), then the four rows finish one after another
// inside the round, each handing its value to the others by a shuffle; so
// every row receives its in-block terms in the push order. The rows' terms
// from outside the block are applied before, as ordinary segments; the end of
// such a segment publishes a "partial" flag where another warp runs the
// block. Ready flags: a finished row holds 2 epoch, a row whose outside terms
// are applied 2 epoch - 1. The block's values sit after all warps' programs
// in the sweep's buffer (read through L1, not the stage ring), round after
// round: 4 diagonals (U; zero in L), the 6 in-round terms (c0+1,c0) (c0+2,c0)
// (c0+2,c0+1) (c0+3,c0) (c0+3,c0+1) (c0+3,c0+2), 2 zeros, then for each row
// c0+q (q = 0..3) its terms (c0+q, 0..c0-1) (zeros for rows past the block).
//
// A program is a sequence of kRecordBytes records, kRecordsPerStage to a ring stage;
// it starts with a control record, and a control record with kCtrlEnd ends it.
constexpr int kSweepWarps = kSolveThreads / 32;   // warps that run sweep programs
constexpr int kGroupLanes = 8;           // envs per lane group (slab_envs <= 8)
constexpr int kBundleRows = 4;           // lane groups per warp
constexpr int kTermSteps = 4;            // terms per group per term record
constexpr int kRecordBytes = 160;
constexpr int kRecordsPerStage = 9;
constexpr int kStageBytes = kRecordBytes * kRecordsPerStage;   // one copy into a warp's ring
constexpr int kStagesMin = 2;            // ring depth per warp (stages), chosen per group
constexpr int kStagesMax = 3;
constexpr int kCtrlWaits = 56;           // wait rows per control record
constexpr int kMaxBlockRows = 48;        // rows of a dense block record (12 register slots per lane group)
constexpr uint16_t kWaitPartial = 0x8000; // wait entry: the row's outside terms only
constexpr uint16_t kNextIsCtrl = 0x8000; // TermRecord.col[g][0]: a control record follows
constexpr uint16_t kColMask = 0x7FFF;
// ControlRecord.gflags bits
constexpr uint8_t kGSwitch = 1;          // the group ends its segment and starts row[g]
constexpr uint8_t kGFinal = 2;           // the ending segment completes its row
constexpr uint8_t kGDivide = 4;          // ... and divides it by diag[g] (backward sweep)
constexpr uint8_t kGPublish = 8;         // ... and publishes it
constexpr uint8_t kGPartial = 16;        // the ending segment completes the row's outside terms: publish them
// ControlRecord.flags bits (warp-uniform summaries of the record)
constexpr uint8_t kCtrlNext = 1;         // the next record is a control or block record
constexpr uint8_t kCtrlEnd = 2;          // the program ends after this record
constexpr uint8_t kCtrlBlock = 4;        // a BlockRecord (its values follow it)
constexpr uint8_t kCtrlDivide = 8;       // some group has kGDivide
constexpr uint8_t kCtrlPublish = 16;     // some group has kGPublish or kGPartial

struct TermRecord {
    double val[kBundleRows][kTermSteps];
    uint16_t col[kBundleRows][kTermSteps];   // column; n = the always-zero padding slot
};
struct ControlRecord {
    uint16_t row[kBundleRows];   // new row of a switching group (n: the group idles)
    uint8_t gflags[kBundleRows];
    uint8_t nwait;
    uint8_t flags;
    uint16_t pad;
    double diag[kBundleRows];
    uint16_t wait[kCtrlWaits];   // rows to acquire before the new rows start
};
struct BlockRecord {
    uint16_t first;              // the block's first row
    uint16_t size;               // rows (1..kMaxBlockRows)
    uint8_t backward;            // 0: rows first, first+1, ..; 1: first, first-1, .. (divides)
    uint8_t pad0[7];
    uint8_t nwait;               // at ControlRecord.nwait's offset
    uint8_t flags;               // at ControlRecord.flags' offset: kCtrlBlock | kCtrlNext
    uint16_t pad1;
    uint64_t publish;            // bit i: publish row i when it is final
    uint32_t values;             // byte offset of the block's values from the start of the sweep's buffer
    uint8_t pad2[20];
    uint16_t wait[kCtrlWaits];   // rows to acquire first (kWaitPartial: outside terms only)
};
static_assert(sizeof(TermRecord) == kRecordBytes && sizeof(ControlRecord) == kRecordBytes &&
                  sizeof(BlockRecord) == kRecordBytes, "record size");
constexpr int kRoundHead = 12;           // doubles of a block round before its rows' terms
// Doubles of a block's values (all rounds).
SB_HD constexpr int block_values(int size) {
    int v = 0;
    for (int c0 = 0; c0 < size; c0 += 4) v += kRoundHead + 4 * c0;
    return v;
}


// Shared memory of a solve CTA: the slab's fields [B][stride] | the warps'
// rings [kSweepWarps][ring_stages][kStageBytes] | ready flags [n + 1] |
// ring stage barriers [kSweepWarps][kStagesMax] | misc.
SB_HD constexpr int slab_stride(int n) { return ((n + 15) & ~15) + 2; }   // >= n + 1: slot n is zero
// Doubles free between the sweeps (fields and rings): the air-side dense
// systems and pw [B][k] live there.
SB_HD constexpr size_t dense_free_doubles(int n, int B, int ring_stages) {
    return ((size_t)B * slab_stride(n) * 8 + (size_t)kSweepWarps * ring_stages * kStageBytes) / 8;
}
// Envs whose dense systems the solve kernel holds at once: one team of
// ceil(k/32) warps each, within the free memory, at most 15 (named barriers).
SB_HD constexpr int dense_teams(int n, int k, int B, int ring_stages) {
    const size_t per_env = (size_t)k * (k + 1) + 16 + 2 * (size_t)k;
    const size_t fr = dense_free_doubles(n, B, ring_stages);
    const int by_mem = fr > (size_t)B * k ? (int)((fr - (size_t)B * k) / per_env) : 0;
    const int by_warps = kSolveThreads / 32 / ((k + 31) / 32);
    const int c = by_mem < by_warps ? by_mem : by_warps;
    return c > 15 ? 15 : c;
}
SB_HD constexpr size_t solve_smem_bytes(int n, int B, int ring_stages) {
    return (size_t)B * slab_stride(n) * 8 + (size_t)kSweepWarps * ring_stages * kStageBytes +
           (((size_t)n + 1 + 15) & ~(size_t)15) + (size_t)kSweepWarps * kStagesMax * 8 + 256;
}

// One triangular sweep: per-warp byte streams, each a whole number of stages.
struct Sweep {
    const uint8_t* stream;                 // all warps' streams back to back, then the block value region
    uint32_t total_bytes;                  // the whole buffer
    uint32_t warp_off[kSweepWarps];        // stage index where warp w's stream starts
    uint32_t warp_stages[kSweepWarps];     // stages in warp w's stream
    uint32_t ring_stages;                  // ring depth the streams were laid out for
    uint32_t recip;                        // 1: U-sweep records hold 1 / diagonal (multiply, not divide)
};

// Wide solve (level programs, built on the host by build_wide,
// wide_sched.cpp): one CTA holds a tile of up to kWideEnvs envs of one group;
// lane l of each of its kWideWarps solver warps works for env l. The tile's
// vectors live in a global scratch array X [n + 1][kWideEnvs] (row n always
// zero), cached in L1/L2 rather than held in shared memory, so that an SM is
// not limited to the eight envs whose fields fit in its shared memory. A
// sweep is a sequence of levels; in each level every solver warp runs its
// list of segments. A segment applies a contiguous run of one row's terms, in
// the reference's push order, to the row's value in X and, when it is the
// row's last, finishes the row (U sweep: the diagonal).
//
// Synchronisation: each row has a ready count in shared memory, the number
// of its segments completed so far (over both sweeps); a warp publishes it
// after each segment. A segment reads rows that are complete before its
// level or finished earlier by its own warp. A level's program is one block
// of at most kWideStageBytes that a producer warp streams, by one bulk copy,
// into a ring of kWideStages shared-memory stages; a stage is refilled only
// after every solver warp has released it, so when a warp works on stage t
// every warp has finished stage t - kWideStages. Each warp's list in a level
// starts with the (row, count) pairs it must acquire: the rows it reads (and
// its own row's previous segment) produced by another warp less than
// kWideStages stages earlier. Block layout: a header of two int32 tables --
// warp w's segments are [seg[w], seg[w + 1]) and its waits [wait[w],
// wait[w + 1]) -- padded to kWideHdrBytes, the waits (uint32 row << 16 |
// count, padded to 16 bytes), the segments (chunk0 relative to the block's
// first chunk), then the chunks.
// Ring and occupancy of the wide solve (compile-time; the level programs are
// built for the same values). Measured on B200 (config 4, corrected build):
// two stages of 16 KB and one CTA per SM leave the most L1 to the tiles'
// vectors (phase 0 1.30 ms against 1.69 ms with four stages and two CTAs per
// SM, 1.75 ms with 8 KB stages); four chunks' loads in flight per warp beat
// three and six.
#ifndef SB_WIDE_STAGES
#define SB_WIDE_STAGES 2
#endif
#ifndef SB_WIDE_STAGE_BYTES
#define SB_WIDE_STAGE_BYTES 16384
#endif
#ifndef SB_WIDE_GROUP
#define SB_WIDE_GROUP 4
#endif
#ifndef SB_WIDE_CTAS
#define SB_WIDE_CTAS 1
#endif
#ifndef SB_WIDE_WARPS
#define SB_WIDE_WARPS 16
#endif
constexpr int kWideWarps = SB_WIDE_WARPS;
constexpr int kWideEnvs = 32;
constexpr int kWideStageBytes = SB_WIDE_STAGE_BYTES;
constexpr int kWideStages = SB_WIDE_STAGES;
constexpr int kWideHdrBytes = (8 * (kWideWarps + 1) + 15) / 16 * 16;
constexpr int kWideGroup = SB_WIDE_GROUP;   // chunks whose source loads a solver warp issues together
constexpr int kWideCtas = SB_WIDE_CTAS;     // wide-solve CTAs per SM (register and shared-memory budget)
static_assert(kWideHdrBytes >= 8 * (kWideWarps + 1) && kWideHdrBytes % 16 == 0, "level header");
struct WideSeg {
    uint32_t row;      // the row whose value the segment updates
    uint32_t chunk0;   // its first chunk (relative to the level block's chunks)
    uint32_t nchunk;   // chunks (terms / 4, rounded up)
    uint32_t fin;      // bit 0: the segment finishes a U row (diagonal); bits 16-31: the row's ready count after it
};
struct WideChunk {
    double v[4];       // term values (padding: 0)
    uint32_t off[4];   // byte offset of the term's source row in X (row * kWideEnvs * 8; padding: row n)
};
static_assert(sizeof(WideChunk) == 48 && sizeof(WideSeg) == 16, "wide record sizes");
struct WideSweep {
    const uint8_t* blocks;     // the level blocks back to back
    const uint32_t* lev_off;   // [nlev + 1] byte offset of level l's block
    int nlev;
};
struct WideTile {
    int group;
    int env0;   // first global env
    int nenv;   // envs in the tile (<= kWideEnvs)
    int tile;   // index of the tile in its group (its scratch block)
};

// Geometry + solver tables of one group and the state of its envs.
struct GroupDev {
    int n, ncv, k, nz, nv, na;
    int stride;        // shared-memory vector stride (doubles) of one env in a slab
    int slab_envs;     // envs per solve CTA
    int n_env;         // envs in the group
    int env0;          // first global env index
    int sigma_identity;
    // row-order coefficient tables
    const double *cap, *dirx, *mc, *ret, *gain;
    const int32_t* zone_of_row;   // -1: no applied heat on this cell
    Sweep fwd, bwd;
    // air side in row positions
    const int32_t *sn_p, *sn_pos;   // sensed CSR, k rows
    int sn_nnz, ap_nnz;             // sensed / applied term counts
    const double* sn_x;
    const int32_t *ap_rp, *ap_col;  // applied by row position, coupled columns ascending
    const double* ap_x;
    const double* S;                // k x k sensed response
    const double* St;               // its transpose (column j of S contiguous)
    // rooms: cells of each room in extended positions
    const int32_t *room_off, *room_pos;
    int room_cells;                 // room_off[rooms]: cells in rooms, at most ncv
    const int32_t* cell_of_pos;     // extended position -> cell index (field mean order)
    const int32_t* pos_of_cell;
    // convection (room-local candidate lists in convection-cell numbering)
    const int32_t *cv_off, *cv_pos, *cand_off, *cand_idx;
    int conv_nrooms, conv_maxroom;
    // folded air side (fold = 1): phase 0 runs the L sweep only and reads the
    // sensed values as R z; phase 1 starts the U sweep from z + Z q
    int fold;
    // corrected air side (corr = 1): phase 0 is the exact build's first solve
    // (y and the sensed right side), and k_correct forms y + W q with the
    // precomputed response W = A^-1 applied ([n][k], row order) instead of a
    // second triangular solve
    int corr;
    const double* W;                // row tiles of k_correct, each [k][kCorrRows]
    int stall_row;                  // a row of the L sweep no warp publishes (failure test)
    int zr_nnz, rs_nnz;
    const int32_t *zr_p, *zr_col;   // Z = L^-1 applied, CSR by row position (coupled columns)
    const double* zr_x;
    const int32_t *rs_p, *rs_pos;   // R = sensed U^-1, CSR by sensor (row positions)
    const double* rs_x;
    // wide solve: level programs, the U diagonal (exact build) or its
    // reciprocal (corrected and folded builds) by row, and the scratch
    // vectors of the group's tiles, [tiles][n + 1][kWideEnvs]
    WideSweep wfwd, wbwd;
    const double* wdiag;
    double* X;
    // per-env state
    double* T;     // [n_env][ncv] extended row order (between the phases of the
                   // folded build: z = L^-1 b in the solved rows)
    double* M;     // [n_env][n] interior mass, row order
};

// Per-scenario (blob) tables. Everything that may differ between weathers of
// one building lives here.
struct ScnDev {
    int group;
    int env0, n_env;           // global env range
    int na, nv, nz, k, nact, n_cont, n_disc, n_dev, n_aux, max_steps;
    int assign, ea, la, ed, ld, hour_m1, wd_m1;
    int tmean_needed;          // some AHU serves no VAV area: the field mean is used
    double p_arr, p_dep, dt, internal_w, standby, occ_w, cv_area, header_res, pump_eff;
    double pump_head0, gas_carbon, conv_p;
    int conv_dist;
    double boiler[10];
    double boiler_cond;        // log(r2/c6)/c8, evaluated once on the host
    const double *amb, *s_comf, *s_heat, *s_cool, *aux;
    const int64_t *o_hour, *r_hour, *r_month;
    const uint8_t *o_wd, *r_wd;
    const double *ahu_c, *vav_c, *zarea;
    const int32_t *vz_off, *vz_idx, *v_ahu, *coupled, *zv_off, *zv_idx, *proom, *room_ncell;
    // ascending lists: coupled columns per zone (zc), coupled columns per AHU
    // (ac), VAVs per AHU (av) -- one thread per zone / AHU accumulates in the
    // reference's loop order
    const int32_t *zc_off, *zc_col, *ac_off, *ac_col, *av_off, *av_idx;
    const uint8_t *a_kind, *a_act, *a_disc;
    const int32_t *a_idx, *a_slot;
    const double *a_mn, *a_mx, *a_mnr, *a_mxr;
    const uint8_t *f_kind, *f_id;
    const int32_t* f_idx;
    const double *f_mean, *f_var;
    const double *rw, *e_wd, *e_we, *e_c, *g_p;
    const double *temp_init, *mass_init;   // extended row order / row order
    // occupancy priming calendar: the hour / workday of the interval before
    // calendar row r (m1_rows entries; one entry unless the blob carries them
    // per row for random starts)
    const int64_t* o_hour_m1;
    const uint8_t* o_wd_m1;
    int m1_rows;
    // convection stream (per scenario): MT19937 raw state + position, and its
    // swap lists of the next two transitions (slot q & 1 for transition q)
    uint32_t* conv_mt;   // 625 words: 624 state + position
    uint32_t* conv_ckpt; // 625 words: the state before the last transition produced
    int32_t* conv_pairs; // [2][conv_stride]: (dst, src) extended positions
    int* conv_npairs;    // [2]
    int conv_stride;     // 2 * ncv + 2
    int scn_index;
};

// Per-env HVAC state. Offsets into one env's double and int blocks.
struct StateLayout {
    int nd, ni;   // doubles / ints per env
    int ahu_rec, ahu_sat, ahu_fan, ahu_flow;
    int v_damp, v_reh, v_ratio, v_hsp, v_csp, v_dcmd, v_rcmd, v_sense, v_area;
    int qdiv, ag, aT, coil, V;   // step transients / occupancy
    int zavg;                    // zone means of the field as the last step (or reset) left it
    int zfsp, zfact;             // zone flow setpoint / actual of the last reward (snapshots)
    int ff_sum, pump_head, b_sp, b_ret, b_cur, b_step, reheat_w;
    int ahu_run, ahu_creq, v_mode, v_prev, v_dset, v_rset;
    int hws_req, hws_run, pump_run, step, gen, active;
    int cal;       // calendar row of the current step (episode offset + step)
    int off;       // calendar offset of the current episode
    int eplen;     // length of the current episode
    int tseq;      // transitions since the last puf_reset (slot parity)
};

struct EnvIndex {   // global env -> its group and scenario
    int group, scn, local;   // local: index inside the group
    int ostream;             // the env's occupancy stream (its scenario's, or its own)
};

// Random inputs are produced one transition ahead of their consumer (k_conv /
// k_occ on their own streams, beside the whole step): transition q (counted
// from puf_reset) uses slot q & 1; slot 2 holds what puf_reset consumes.
constexpr int kRngSlots = 3;
constexpr int kResetSlot = 2;
constexpr int kStartDays = 7;
constexpr int kStepsPerDay = 288;

// Everything one step launch needs; copied to device memory once.
struct StepCtx {
    const GroupDev* groups;
    const ScnDev* scns;
    const EnvIndex* envs;
    int n_env, n_groups, n_scns;
    StateLayout lay;
    double* Dst;          // [n_env][lay.nd]
    int32_t* Ist;         // [n_env][lay.ni]
    // framework buffers (device memory owned by the caller)
    const float* actions; // [n_env][kAct]
    float* obs;           // [n_env][kObs]
    float* rewards;       // [n_env]
    float* terminals;     // [n_env]
    float reward_scale;
    void* env_records;    // Env[n_env] (managed memory, layout in include/sbenv.h)
    // episode statistics
    double* rew_f64;      // [n_env] last step's reward in double
    double* parts_out;    // [n_env][kParts] last step's log terms
    double* epret_d;      // [n_env] running episode return in double
    double* live;         // [2 + kParts] step-level sums: count, reward, parts
    double* live_scn;     // [n_scns][4]: reward, mean deviation, count, reward^2
    double* ep_scn;       // [n_scns][2]: completed-episode mean rewards, count
    int* status;          // device error word
    // occupancy streams: one per scenario while its envs step in lock step,
    // one per env with desync or random_start (complete_port/csim/sb_occup.c;
    // the reference GPU backend keeps one per env, gpu/sb_gpu_kernels.cuh:385-422)
    int n_ostreams, ostream_per_env, random_start;
    const int* ostream_scn;     // [n_ostreams] the stream's scenario
    uint32_t* occ_mt;           // [n_ostreams][625] MT19937 state + position
    int* occ_state;             // [n_ostreams][occ_stride] occupant states
    int occ_stride;
    int* ostep;                 // [n_ostreams] producer: step in the current episode
    int* oeplen;                // [n_ostreams] producer: current episode's length
    int* ooff;                  // [n_ostreams] producer: current episode's calendar offset
    int* oseq;                  // [n_ostreams] transitions produced since puf_reset
    unsigned long long* orng;   // [n_ostreams] producer: random-start stream
    // each stream's MT state and occupant states before its last production
    // (a transition produced ahead and never consumed is undone by puf_reset;
    // the episode counters restart from the consumer's then)
    uint32_t* ck_mt;            // [n_ostreams][625]
    int* ck_state;              // [n_ostreams][occ_stride]
    int* produced;              // 1 once a transition was produced since creation
    int* cseq;                  // [n_scns] convection transitions produced since creation
    // producer outputs, [kRngSlots][n_ostreams]...: occupancy after the
    // transition (reward), of the priming interval (reset observation), of
    // the new episode's first interval, and the new episode's offset and
    // random-start stream state
    double* V_step;             // [slot][n_ostreams][nz_max]
    double* V_prime;
    double* V_zero;
    int* new_off;               // [slot][n_ostreams]
    unsigned long long* new_rng;// [slot][n_ostreams]
    int nz_max;
    unsigned long long* env_rng;// [n_env] the consumer's random-start stream state
    double* start_draws;        // [n_scns][2][kStartDays] start days drawn (first draw, later)
    double* ep_start;           // [n_scns][kStartDays][7] whole episodes by start day
    int full_len_max;           // longest episode length (calendar rows needed)
    // learning-reward normalisation (rew_norm / rew_center): per scenario
    // (mean, inv_std); null: rewards scaled by reward_scale
    const float* rnorm;
    double* znclip;             // [3] rewards beyond 1 / 3 / 5 (rew_norm only)
    // failure test (sb_test_stall): {1: warp 0 of every slab waits at the start
    // of the L sweep for a row no warp publishes, spin limit (0: the default)}
    const int* test_ctl;
    // air side: per env the dense system's right side (k_solve phase 0), then
    // its solution (k_dense), read by k_solve phase 1
    double* airq;           // [n_env][k_max]
    int k_max;
    const int* dense_order; // [n_env] envs by descending k (k_dense's CTA order)
};

}  // namespace sbenv
