/* Batched Smart Buildings HVAC environment on B200 -- C ABI.
 *
 * Drop-in for the reference's PufferLib 5.0 GPU env backend
 * (complete_port/gpu/smart_buildings.cu:3307-3323, PUF_BACKEND PUF_GPU with
 * PUF_HAS_LIVE_LOG and PUF_HAS_MASK_INIT, smart_buildings.cu:94-95,65): the same
 * entry points, argument meanings, buffer layouts and episode semantics. The
 * whole step runs on the device on the stream bound with puf_bind_stream; the
 * host only enqueues kernels, so puf_step can be captured in a CUDA graph.
 *
 * Buffer layout (the trainer owns these device buffers; the env writes them in place):
 *   observations  float [n][SB_OBS]   real fields first, zero tail
 *   actions       float [n][SB_NUM_ATNS] = [SB_CONT continuous in [-1,1]][SB_DISC run bits]
 *   rewards       float [n]
 *   terminals     float [n]            1.0 on the step that ends an episode
 * (complete_port/gpu/smart_buildings.cu:33-71, complete_port/pufferlib_cpu_env.h:50-80)
 *
 * Errors: the reference abort()s on a bad configuration
 * (complete_port/pufferlib_cpu_env.h:316-358). Here puf_vec_create returns
 * NULL and every call records a one-line reason readable with sb_last_error();
 * device-side faults the kernels detect (a bounded wait that expired, a corrupt
 * schedule chunk) are latched in a device status word reported by
 * sb_device_status(). Nothing traps and no wait is unbounded. */
#ifndef SBENV_H
#define SBENV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_OBS 1024
#define SB_CONT 256
#define SB_DISC 16
#define SB_NUM_ATNS (SB_CONT + SB_DISC)
#define SB_MASK_WIDTH (SB_CONT + 2 * SB_DISC)
#define SB_NPARTS_ENV 8

typedef float obs_t;
typedef struct CUstream_st* sb_stream_t; /* == cudaStream_t */

/* Per-env episode log (complete_port/gpu/smart_buildings.cu:101-115). Fields are
 * sums over completed episodes; the trainer divides by n. */
typedef struct Log {
    float perf;
    float score;
    float episode_return;
    float episode_length;
    float comfort_dev_K;
    float worst_dev_K;
    float out_of_band_frac;
    float productivity;
    float energy_cost_norm;
    float carbon_norm;
    float elec_kwh;
    float gas_kwh;
    float n;
} Log;

/* PufferLib's per-agent buffer record (pufferenv.h of PufferLib 5.0, which is
 * not vendored): the five pointers the env fills. A translation unit that has
 * PufferLib's own Agent defines SB_HAVE_AGENT before including this header;
 * the layout below must then be the same as PufferLib's. */
#ifndef SB_HAVE_AGENT
typedef struct Agent {
    float* observations;
    float* actions;
    float* rewards;
    float* terminals;
    unsigned char* action_mask;
} Agent;
#endif

/* One environment record; an array of n of them is returned by puf_vec_create
 * in managed memory. The members and their order are the reference GPU
 * backend's (complete_port/gpu/smart_buildings.cu:116-143, non-entity build),
 * so a trainer indexing envs[i] with the reference's struct reads the same
 * fields; `scenario` is an addition after them. agents[0] points into the
 * caller's buffers (env i's slices); cont / disc / native are NULL (the device
 * step keeps its decoded actions on the device). The step writes log / ep_* /
 * step / max_steps / start_* on the device; the host reads them only after
 * synchronising. */
typedef struct Env {
    Agent agents[1];
    Log log;
    float ep_ret;
    float ep_part[SB_NPARTS_ENV];
    float ep_worst;
    int num_agents;
    int tag;
    int boundary_reached;
    int step;
    int max_steps;            /* this episode's length (desync: the first one is cut) */
    int start_offset;         /* calendar row of this episode's first step (random_start) */
    int start_day;            /* start_offset / 288 */
    unsigned long long start_rng;   /* the env's random-start stream (SplitMix64) */
    unsigned int start_draws; /* start days drawn so far */
    int n_act, n_cont, n_disc;
    int loaded;
    unsigned int rng;
    int seed;
    double* cont;
    double* disc;
    double* native;
    int env_id;
    int scenario;             /* addition: the env's scenario index */
} Env;

/* PufferLib's keyword dictionary, minimal layout: a key with a numeric value
 * and/or a string value. dict_find returns NULL for a missing key. */
typedef struct DictItem {
    const char* key;
    double value;
    const char* str;
} DictItem;
typedef struct Dict {
    DictItem* items;
    int size;
    int capacity;
} Dict;

Dict* sb_dict_new(int capacity);
void sb_dict_free(Dict* d);
DictItem* dict_find(Dict* d, const char* key);
void dict_set(Dict* d, const char* key, double value);
void dict_set_str(Dict* d, const char* key, const char* value);

/* ---- the PufferLib GPU-backend entry points ---- */

/* n envs over the scenarios named by kwargs "blob" (one .sbb path) or
 * "blob_dir" (every *.sbb in the directory; env SB_BLOB_DIR as fallback),
 * spread round-robin by building (smart_buildings.cu:2497-2560). Other keys:
 * groups (scenario count, 0 = n/32), max_steps (0 = the blob's episode
 * length), merge_weathers (share one solver group across weathers of a
 * building, default 1), reward_scale (default 1), solve_exact (1, default:
 * the reference core's two triangular solves per step, bit for bit; 0: one L
 * and one U sweep per step, agreeing with the reference within 1e-9 relative
 * per step -- the air-side correction added as W q with W = A^-1 applied
 * precomputed per building (default), or with fold = 1 folded into the sweep
 * pair as the reference's GPU backend does).
 * Episode options of the reference's GPU backend (smart_buildings.cu:2583-2608,
 * 2806-2816, 1636-1657, 1936-2050): desync (1: env i's first episode ends at a
 * step in [1, episode length] drawn from i; later episodes are whole, the cut
 * first ones stay out of the log), random_start (1: every episode starts at a
 * calendar offset of d * 288 steps, d in 0..6 drawn per env and episode from a
 * SplitMix64 stream seeded by random_start_seed and the env index; needs
 * blobs with random_start_offsets and tables 6 * 288 rows longer than the
 * episode; desync is then ignored), rew_norm (1: the reward buffer holds
 * (r - mean) * inv_std per scenario, the statistics moved by 0.1 towards each
 * puf_live_log window, starting at mean 0 and variance 0.217) and rew_center
 * (1: (r - mean) only, the mean moved by center_beta, default 0.01; rew_norm
 * wins when both are set). env_offset: the global index of this batch's first
 * env when a batch is sharded over several GPUs (the per-env draws follow the
 * global index; default 0). overlap (scheduling only, results unchanged):
 * with several classes of equal air-side size k, 1 runs each class's dense
 * systems and then its phase-1 work (the correction or the second solve) on a
 * stream of its own, 2 its first solve too, 0 every part on one stream in
 * turn; default -1: 2 when the first solve's slabs are more than one wave of
 * the GPU's SMs, else 1. wide (scheduling only, results unchanged): 1 runs
 * the first solve on tiles of 32 envs whose vectors stay in L1/L2 (level
 * programs streamed to 16 solver warps, per-row ready counts), 0 on slabs of
 * up to 8 envs held in shared memory (per-warp programs, ready flags);
 * default -1: 1 when the slabs would be three or more waves of the GPU's SMs.
 * Returns NULL on error. */
Env* puf_vec_create(int n, Dict* kwargs, obs_t* observations, float* actions, float* rewards,
                    float* terminals);
void puf_bind_stream(sb_stream_t stream);
void puf_init(Env* env, Dict* kwargs);
/* Restarts every env: state from the blob, occupancy primed, reset observation
 * written; clears the device status word (sb_device_status). */
void puf_reset(Env* envs);
/* One batched step of every env (device only, graph-capturable). With the
 * environment variable SB_SNAPSHOT=<file> set it also writes a snapshot of env
 * SB_SNAP_ENV (default 0) every SB_SNAP_EVERY-th call (default 1) that is not
 * being captured, synchronising the stream, as the reference does
 * (smart_buildings.cu:3015-3026); puf_live_log then writes one as well. */
void puf_step(Env* envs);
void puf_render(Env* env);
void puf_close(Env* env);
void puf_log(Log* log, Dict* out);
/* Step-level metrics since the previous call, per scenario as scenario/<name>/... */
void puf_live_log(Env* envs, Dict* out);
/* Fills the trainer's [nagents][width] action mask (device pointer): active
 * continuous heads and active discrete categories 1, padding 0. */
void puf_mask_init(unsigned char* mask, int width, int nagents);

/* ---- additions for hosts without PufferLib (no counterpart in the reference) ---- */

/* Last error text of this thread ("" if none). */
const char* sb_last_error(void);
/* Device status word: 0, or the first kernel-detected error code since the
 * last puf_reset: 1 a sweep program stage never arrived (bounded mbarrier
 * wait expired), 3 a convection swap list overflow, 5 a row's ready flag never
 * arrived within the bounded wait, 6 a malformed or truncated sweep program.
 * The kernel that detects one leaves its sweep and returns; the env's state
 * for that step is then meaningless until puf_reset. Synchronises the bound
 * stream. */
int sb_device_status(void);
/* Failure test of the bounded waits (no counterpart in the reference): on = 1
 * makes warp 0 of every solve CTA wait, at the start of its L sweep, for a
 * row of the sweep program that no warp publishes (wide tiles: for a ready
 * count that no row reaches), polling at most spin_limit times (0: the
 * production limit, 2^22 polls, about a second), so the wait runs out, the
 * CTA's other warps and its program producer leave their waits, and the next
 * puf_step reports code 5 without a fault or a hang; on = 0 turns it off (and
 * restores the limit). Synchronises. 0 or -1. */
int sb_test_stall(int on, unsigned int spin_limit);
/* Shape of the loaded batch: out[8] = {n_env, n_scenarios, n_groups, obs_len_max,
 * n_cont_max, n_disc_max, first-solve CTAs (slabs, or 32-env tiles with the wide
 * solve), kernels_per_step}. */
void sb_shape(int* out);
/* Per-env observation length / scenario index (host arrays of n). */
void sb_env_info(int* obs_len, int* scenario);
/* Copies one env's temperature field (cell order, n_cvs doubles) to host memory. */
int sb_get_temp(int env, double* out, int n_cvs);
/* Copies one env's interior-mass temperatures (solved-cell order) to host memory. */
int sb_get_mass(int env, double* out, int n_solved);
/* Copies the last step's per-env reward (double) and log terms [n][8] to host memory. */
int sb_get_reward_f64(double* reward, double* parts);
/* Episode options as set up at creation: per env the first episode's length
 * (desync) and the initial random-start stream state (the value before the
 * first draw), host arrays of n (either may be NULL). Returns 0 or -1. */
int sb_episode_options(int* first_len, unsigned long long* start_rng);
/* Policy-in-loop rollouts: actions drawn from a
 * policy's logits, as the reference trainer's mixed heads do
 * (patches/pufferlib_core.diff:2490-2580; beta_floor / beta_conc_max of
 * config/smart_buildings.ini). raw: two device f32 blocks [2][n][288] (the
 * second at raw + n * 288): block 0 = the 256 continuous heads' u, then the 16
 * discrete heads' class logits (off, on); block 1 = the continuous heads' v.
 * Continuous head: alpha = softplus(u) + floor_c, beta = softplus(v) + floor_c,
 * both scaled down so that alpha + beta <= cap (cap <= 0: no cap; else cap must
 * exceed 2 floor_c), action 2x - 1 with x ~ Beta(alpha, beta). Discrete head:
 * the drawn class index (0.0 / 1.0). mask: device u8 [n][288] as puf_mask_init
 * writes it, or NULL for all heads active; a head with no unmasked entry gets
 * action 0.0, a masked class is never drawn. Draws come from Philox4x32-10
 * streams keyed by seed and counted by *call (a device u64 the caller advances
 * between draws, so a captured graph draws fresh numbers on every replay).
 * actions: device f32 [n][272], as puf_vec_create's actions. Enqueued on the
 * bound stream (capturable). 0 ok, -1 bad arguments / launch error. */
int sb_beta_actions(const float* raw, const unsigned char* mask, float* actions, int n, float floor_c, float cap,
                    unsigned long long seed, const unsigned long long* call);
/* Verification entry: solves n dense k x k systems (row-major m [n][k][k], right
 * sides b [n][k]) with the air-side solver of k_dense (partial pivoting in the
 * reference's order); solutions to out [n][k]. Host pointers; synchronous. */
int sb_dense_check(int k, int n, const double* m_rowmajor, const double* b, double* out);
/* sb_dense_check with the solver of the corrected and folded builds when
 * tolerant != 0: the same pivoting, fused multiply-add row updates and a
 * column-oriented back substitution (every pending row subtracts its product
 * with the newest solution value at once, so the sums are formed in descending
 * column order); the solutions agree with the reference's to rounding.
 * tolerant = 0 is sb_dense_check. */
int sb_dense_check_mode(int k, int n, const double* m_rowmajor, const double* b, double* out, int tolerant);
/* The same dense solves as sb_dense_check, on device buffers and without
 * allocating anything: for callers that cannot call cudaMalloc, such as a host
 * program whose device memory is owned by another allocator or code that runs
 * where allocation is not allowed. It has no counterpart in the reference.
 * m_rowmajor [n][k][k], b [n][k] and out [n][k] are device pointers the caller
 * owns. The column-major working copy goes to one fixed device array of 2^19
 * doubles (4 MiB, held by every GPU that loads the library): n * k * k above
 * that is rejected with -1 and a message, as are k outside 1..128 and null
 * pointers. The first call on a device (of this entry point or of
 * sb_dense_check) looks up that array's device address and sets the kernel's
 * shared-memory limit for the largest k, under a lock, so host threads may make
 * it at the same time; make it before any stream capture. Enqueued on the bound
 * stream (the default stream without an env batch) and asynchronous; every call
 * shares the array, so calls that overlap on the GPU (other streams, other
 * threads) race. Nothing in the array needs to start at zero: each call
 * overwrites the part it reads. 0 ok, -1 error (sb_last_error). */
int sb_dense_solve_noalloc(int k, int n, const double* m_rowmajor, const double* b, double* out);
/* Snapshot of one env's visible state to a file, the reference's headless
 * viewer feed (SBS1, smart_buildings.cu:2205-2290), after the last step:
 * "SBS1", i32[12] {1, step in the episode, episode length, env index in its
 * solver group, zones, VAVs, AHUs, grid rows, grid columns, cells, actions, 0},
 * f64[12] {reward, episode return, boiler setpoint, boiler return, the 8 reward
 * terms}, char[512] scenario path, f32 field[cells] (K, cell order), f64 zone
 * means / occupancy / flow setpoint / flow [zones each], f64 VAV heating and
 * cooling setpoints / damper / reheat [VAVs each], f64 AHU supply temperature /
 * flow [AHUs each], i32 AHU run [AHUs], f64 native actions [actions], all
 * little-endian. Written to <path>.tmp, then renamed. Synchronises the bound
 * stream (not capturable). 0 ok, 1 error (sb_last_error). */
int sb_snapshot_write(int env, const char* path);
/* Number of hot-path kernel launches one puf_step enqueues. */
int sb_kernels_per_step(void);
/* Measurement: runs one step with CUDA events around each kernel on the bound
 * streams (not for graph capture). ms[7] = {-1, k_pre, solve, k_post, solve
 * phase 0, k_dense, solve phase 1}; solve = phase 0 + k_dense + phase 1; the
 * random inputs of the next transition (k_conv, k_occ) run beside phase 1,
 * inside its interval, and have no time of their own (ms[0] = -1). */
int sb_step_timed(float* ms);
/* Algorithmic bytes one solve launch must move for the loaded batch: per env the
 * field and interior mass read and written plus the per-zone heat and air-side
 * vectors; per solver group the factor and coupling tables once. */
int sb_solve_bytes(double* per_launch);
/* fp64 operations one solve launch performs for the loaded batch (the
 * triangular solves' multiply / subtract / divide, forcing, coupling products,
 * the dense systems' elimination, the mass / field update). */
int sb_solve_flops(double* per_launch);
/* Measured fp64 issue rate of the current GPU in TFLOP/s: a plain timed kernel
 * of independent fused multiply-add chains over every SM (changes no setting). */
int sb_fp64_peak(double* tflops);
/* Per-scenario episode statistics since creation or the last clear, out
 * [n_scenarios][6] = {reward sum, mean-deviation sum, steps, reward^2 sum,
 * sum of whole-episode mean rewards, whole episodes}; clear != 0 zeroes the
 * sums (puf_live_log reads and clears the same sums). Returns the scenario
 * count, -1 on error. Synchronises the bound stream. */
int sb_scenario_stats(double* out, int clear);
/* Inspection: one env's last pre-stage results, out = [air conductance k][supply
 * air temperature k][applied heat per zone cell nz][flow factor sum, reheat W,
 * boiler temperature, boiler return, pump head]. Returns the count or -1. */
int sb_debug_state(int env, double* out, int cap);
/* Host-only: the solve kernel's program for one sweep of a blob's factor
 * (sweep 0 = L, 1 = U), laid out for per-warp rings of ring_stages 512-byte
 * stages (4..8; 0 = the depth a full slab leaves on a B200): the
 * sb_sweep_warps() warps' programs back to back; warp_stages[] receives each
 * program's stage count. Returns 0, 1 if cap is too small (*used then holds the size), -1 on
 * error. No counterpart in the reference (its CPU core has no schedule). */
int sb_solve_schedule(const char* blob_path, int sweep, int ring_stages, uint8_t* out, size_t cap, size_t* used,
                      uint32_t* warp_stages);
/* Warps of a solve CTA that run sweep programs (streams per sweep). */
int sb_sweep_warps(void);
/* Host-only: statistics of that program, out[10] = {terms, control records,
 * term records, row segments, waits, published rows and partial sums,
 * modelled cycles, stream bytes, dense block records, rows they finish}. */
int sb_sweep_stats(const char* blob_path, int sweep, int ring_stages, double* out);
/* Host-only: the wide solve's level program of the blob's L (sweep 0) or U
 * (sweep 1) sweep; the U program's stages and ready counts continue the L
 * program's. info[8] receives {levels, segments, chunks, partial segments,
 * terms, modelled cycles, bytes of all level blocks, largest level block};
 * with lev_off (levels + 1 uint32: each level block's byte offset) and blocks
 * (the level blocks: two int32 tables of sb_wide_warps() + 1 entries --
 * first segment and first wait of each warp -- padded to 144 bytes, the
 * waits (uint32 row << 16 | count, padded to 16 bytes), 16-byte segments
 * {row, first chunk, chunks, finish | count << 16}, 48-byte chunks {four
 * f64 values, four uint32 byte offsets}) both non-null the program is copied
 * out and 0 returned, else 1; -1 on error. No counterpart in the reference
 * (its CPU core has no schedule). */
int sb_wide_schedule(const char* blob_path, int sweep, int64_t* info, uint32_t* lev_off, uint8_t* blocks);
/* Solver warps of a wide-solve CTA (level program columns). */
int sb_wide_warps(void);
/* The wide solve's build constants: out[6] = {solver warps, ring stages, stage
 * bytes, level header bytes, chunks whose loads a warp issues together, CTAs
 * per SM}. No counterpart in the reference. */
void sb_wide_config(int* out);

#ifdef __cplusplus
}
#endif
#endif /* SBENV_H */
