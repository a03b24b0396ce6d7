/*
 * tthrml.h — C ABI of the B200 block-Gibbs sweep library (libtthrml_b200.so).
 *
 * The reference (tt-thrml) runs one fused device kernel per sampling group per
 * sweep with the signature
 *     (global_state, *rng_slices) -> new_global_state
 * (tt_thrml/compiler.py:3-4, 436-450; tt_thrml/executor.py:187-212, 240-275),
 * launched through `tt_runtime.submit` (tt_thrml/executor.py:269).  This
 * library replaces that kernel: one call per sampling group per sweep, in
 * place on device memory, on the caller's CUDA stream.  The state gains a
 * chain axis the reference does not have: every state buffer here is
 * chain-innermost, `state[row][chain]`, row = the reference's flat
 * block-ordered node index (tt_thrml/compiler.py:117-153).
 *
 * Conventions
 *   - Every entry point returns TTHRML_OK (0) or a negative error code and
 *     never aborts, traps or throws.  `tthrml_last_error()` returns the
 *     message of the calling thread's last failure.
 *   - All pointers named `*_dev` or documented as device memory must be
 *     device pointers valid on the current CUDA device; host pointers are
 *     named `*_host`.
 *   - `stream` is a cudaStream_t passed as `void*` (NULL = legacy default).
 *   - Run control: when `ctl` (a device tthrml_run_ctl) is given, kernels use
 *     sweep index `sweep + ctl->sweep` and Philox seed `ctl->seed`, so one
 *     captured CUDA graph of n sweeps serves every position of every run.
 *   - RNG: with `variates == NULL` the kernels draw from an on-device
 *     counter-based Philox4x32-10 stream keyed by `seed`, counter
 *     (chain/4, row, sweep, salt) -- or (chain, row/4, sweep, salt) for the
 *     dense and 2-D lattice kernels, as documented at each entry point.
 *     With `variates != NULL` they consume
 *     caller-provided variates exactly like the reference's uploaded RNG
 *     slices (tt_thrml/rng.py:132-222): spin threshold logits, categorical
 *     Gumbel noise, gaussian standard normals.
 */
#ifndef TTHRML_H_
#define TTHRML_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTHRML_ABI_VERSION 1

/* status codes */
#define TTHRML_OK 0
#define TTHRML_ERR_ARG -1     /* invalid argument (sizes, alignment, NULL) */
#define TTHRML_ERR_CUDA -2    /* a CUDA runtime call failed */
#define TTHRML_ERR_UNSUPPORTED -3

/* parameter families (tt_thrml/core.py:15-18) */
#define TTHRML_SPIN 0
#define TTHRML_CATEGORICAL 1
#define TTHRML_GAUSSIAN 2

/* contribution kinds (tt_thrml/compiler.py:82-114) */
#define TTHRML_KIND_LINEAR 0    /* "default" or "linear" */
#define TTHRML_KIND_PRECISION 1 /* "precision" (reciprocal of inverse_weights) */

/* state element types */
#define TTHRML_STATE_F32 0 /* float32: spin ±1.0, categorical index, gaussian value */
#define TTHRML_STATE_I8 1  /* int8:    spin ±1, categorical index (no gaussian) */
#define TTHRML_STATE_BITS 2 /* spin only: row = n_chains bits in uint32 words,
                               bit c set = chain c is -1 (n_chains % 32 == 0) */

#define TTHRML_MAX_CAT_SOURCES 4
#define TTHRML_MAX_CATEGORIES 64

/* Device-resident run control read by graph-captured kernels. */
typedef struct tthrml_run_ctl {
  uint32_t sweep;  /* added to the kernel's sweep argument */
  uint32_t reserved;
  uint64_t seed;   /* Philox seed, replaces the kernel's seed argument */
} tthrml_run_ctl;

/*
 * One lowered interaction of one block, in ragged-ELL form: the terms of
 * target node i are t in [row_ptr[i], row_ptr[i+1]).  A dense reference
 * table (n_nodes, n_terms) is the special case row_ptr[i] = i*n_terms.
 * Mirrors FusedInteractionSpec (tt_thrml/core.py:43-57) as built by
 * _build_interaction_spec (tt_thrml/compiler.py:156-217).
 */
typedef struct tthrml_interaction {
  const int64_t* row_ptr;   /* device, [n_nodes + 1] */
  const float* weights;     /* device, [nnz][w_inner]: weights x active mask */
  const int32_t* sources;   /* device, [n_sources][nnz]: flat state rows */
  int64_t nnz;              /* terms in this interaction (row_ptr[n_nodes]) */
  int32_t n_sources;        /* gathered sources per term */
  int32_t n_categorical;    /* trailing sources that select a weight slice */
  int32_t kind;             /* TTHRML_KIND_* */
  int32_t w_inner;          /* q_target (categorical target, else 1) x prod(cat_q) */
  int32_t cat_q[TTHRML_MAX_CAT_SOURCES]; /* categories of each categorical source */
} tthrml_interaction;

/*
 * One block of a sampling group.  Mirrors FusedBlockSpec
 * (tt_thrml/core.py:60-70).
 */
typedef struct tthrml_block {
  int32_t family;           /* TTHRML_SPIN / _CATEGORICAL / _GAUSSIAN */
  int32_t n_categories;     /* categorical q (<= TTHRML_MAX_CATEGORIES), else 1 */
  int32_t n_interactions;
  int32_t reserved;
  int64_t n_nodes;
  int64_t row_start;        /* first flat state row of the block */
  const tthrml_interaction* interactions; /* device array [n_interactions] */
  const float* variates;    /* device, [n_sweeps][n_nodes][qv][n_chains] or NULL
                               (qv = n_categories for categorical, else 1) */
  int64_t variates_sweeps;  /* sweeps held by `variates` */
} tthrml_block;

/*
 * Generic group step (any mix of spin / categorical / gaussian blocks).
 * Every block of the group reads the pre-group state and the group commits
 * together (tt_thrml/compiler.py:436-450).  When `in_place` is 0 the new
 * values go to `scratch` ([sum n_nodes][n_chains] elements of the state
 * type) and a second kernel commits them; `in_place` = 1 is allowed only
 * when no block of the group reads a row of the group.
 * Reference: _sample_block and helpers, tt_thrml/compiler.py:274-385.
 */
typedef struct tthrml_group {
  const tthrml_block* blocks; /* device array [n_blocks] */
  int32_t n_blocks;
  int32_t state_dtype;        /* TTHRML_STATE_* */
  int64_t group_rows;         /* sum of the blocks' n_nodes */
  int64_t n_chains;           /* chains held by this state (row length) */
  int64_t chain_offset;       /* global index of chain 0 (multiple of 4) */
  void* state;                /* device, [total_rows][n_chains] */
  void* scratch;              /* device, [group_rows][n_chains] or NULL */
  int32_t in_place;
  int32_t use_variates;       /* 1: read blocks[].variates; 0: Philox */
  uint64_t seed;
  uint32_t sweep;             /* sweep index (ctl->sweep is added when ctl is set) */
  uint32_t reserved;
  const tthrml_run_ctl* ctl;  /* device run control or NULL (CUDA-graph replay) */
} tthrml_group;

int tthrml_group_step(const tthrml_group* group_host, void* stream);

/*
 * Allocation-free tthrml_group_step.  It has no counterpart in the reference.
 *
 * tthrml_group_step wants a caller buffer for `scratch` whenever a group
 * reads its own rows.  Callers that cannot provide one, such as a plugin or
 * FFI host that owns every buffer it passes and has no device allocator to
 * lend, or a running control loop that must not call cudaMalloc (it can
 * synchronise the whole device), use this entry point instead: `scratch` in
 * the descriptor is ignored and the staging area is a device array inside
 * this library of TTHRML_STATIC_SCRATCH_BYTES.  A device reserves the array
 * when the library's generic group kernels are first used on it (lazy module
 * loading, the CUDA 12 default) and keeps it until the process exits.  Groups
 * that stage more than that (group_rows * n_chains * element size) are
 * rejected with TTHRML_ERR_ARG before anything is launched; groups with
 * `in_place` set stage nothing and are never rejected for their size.  No
 * memory is allocated and no allocating routine is called.
 *
 * The array's device address belongs to the CUDA context that loaded the
 * library's module.  Every call made outside stream capture looks it up in
 * the current context (cudaGetSymbolAddress); a call made while its stream is
 * being captured uses the address its context's last uncaptured call found,
 * so the first call in each context (including the new context after a
 * cudaDeviceReset) must come before any stream capture.  Every call shares
 * the one array and the array keeps the last call's contents; nothing has to
 * start at zero because the step writes every scratch element before it reads
 * it back.  Calls whose kernels overlap on the GPU race on the array:
 * serialise them (one stream, or events) per device.
 */
#define TTHRML_STATIC_SCRATCH_BYTES (16u << 20)
int tthrml_group_step_static_scratch(const tthrml_group* group_host, void* stream);

/*
 * Sparse spin block (pairwise spin couplings + bias) on int8 ±1 state:
 * gamma = bias + sum_e w_e * s[col_e], s = +1 where 2*gamma > logit(u).
 * Reference: _accumulate_gamma + _sample_spin_block
 * (tt_thrml/compiler.py:303-324) for a block whose interactions are one
 * bias (no source) and one pair interaction (one spin source).
 * Writes the block's rows in place; the caller guarantees the block reads
 * none of its own rows (a proper colouring).
 * Requires n_chains % 32 == 0 and chain_offset % 4 == 0.
 */
int tthrml_spin_csr_step(const int64_t* row_ptr_dev, /* [n_rows + 1] */
                         const int32_t* cols_dev,    /* [nnz] flat rows */
                         const float* vals_dev,      /* [nnz] */
                         const float* bias_dev,      /* [n_rows] or NULL */
                         int64_t row_start, int64_t n_rows,
                         int8_t* state_dev, int64_t n_chains, int64_t chain_offset,
                         const float* variates_dev,  /* [variates_sweeps][n_rows][n_chains] logits, or NULL */
                         int64_t variates_sweeps,
                         uint64_t seed, uint32_t sweep,
                         const tthrml_run_ctl* ctl_dev, /* device run control, or NULL */
                         void* stream);

/*
 * The same block update on bit-packed state (TTHRML_STATE_BITS):
 * state_dev is [rows][n_chains/32] uint32, bit c of a row = 1 when chain c
 * is -1.  Same arguments, arithmetic and Philox stream as
 * tthrml_spin_csr_step, so both layouts produce identical samples.
 * Requires n_chains % 256 == 0 and chain_offset % 4 == 0.
 */
int tthrml_spin_bits_step(const int64_t* row_ptr_dev, const int32_t* cols_dev, const float* vals_dev,
                          const float* bias_dev, int64_t row_start, int64_t n_rows,
                          uint32_t* state_dev, int64_t n_chains, int64_t chain_offset,
                          const float* variates_dev, int64_t variates_sweeps,
                          uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl_dev,
                          void* stream);

/*
 * tthrml_spin_bits_step with the block's rows processed in the order given
 * by row_order_dev (int32 [n_rows], a permutation of 0..n_rows-1, e.g. rows
 * sorted by degree so that the rows handled side by side need equally many
 * neighbour terms).  The order changes only which rows run together, not
 * any sample: every row's field, draw and Philox counter are its own.
 */
int tthrml_spin_bits_step_ordered(const int64_t* row_ptr_dev, const int32_t* cols_dev, const float* vals_dev,
                                  const float* bias_dev, int64_t row_start, int64_t n_rows, uint32_t* state_dev,
                                  int64_t n_chains, int64_t chain_offset, const float* variates_dev,
                                  int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                                  const tthrml_run_ctl* ctl_dev, const int32_t* row_order_dev, void* stream);

/*
 * Checkerboard colour block of a q-state Potts model on a periodic X x Y x Z
 * lattice (q <= 8; one q x q matrix per axis).  Replaces the group kernel of
 * the categorical block (tt_thrml/compiler.py:289-344) for lattice programs:
 * the neighbour gather is computed from the site coordinates instead of read
 * from tables.  state_dev: int8 [rows][n_chains] categories; colour-c site
 * (x, y, z) sits at row target_row0 + L/2 with L = (z*Y + y)*X + x, its
 * neighbours at source_row0 + L'/2.  J: float [3][q][q] (axis, target
 * category, neighbour category); bias: float [X*Y*Z/2][q] per target row.
 * theta_k = ((b_k + (Jx[k][s_x-] + Jx[k][s_x+])) + (Jy..)) + (Jz..), each sum
 * rounded in float32.  variates: [variates_sweeps][X*Y*Z/2][q][n_chains]
 * Gumbels (argmax(theta + g)) or NULL (Philox: one uniform per update from
 * counter (chain/4, row, sweep, "CAT"), inverse-CDF draw, identical to the
 * generic kernel).  Requires even X, Y, Z, n_chains % 4 == 0, chain_offset %
 * 4 == 0 and 16-byte aligned buffers.
 */
int tthrml_potts3d_step(int8_t* state_dev, int64_t n_chains, int32_t X, int32_t Y, int32_t Z, int32_t colour,
                        int64_t target_row0, int64_t source_row0, const float* J_dev, const float* bias_dev,
                        int32_t q, int64_t chain_offset, const float* variates_dev, int64_t variates_sweeps,
                        uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl_dev, void* stream);

/*
 * The per-site bias weights e^(b_k - max b) of a q = 8 Potts block, computed
 * once (they do not change between sweeps): bias and bias_weights are float32
 * [n_sites][8], 16-byte aligned.  tthrml_potts3d_step_weights is
 * tthrml_potts3d_step reading these weights instead of recomputing them per
 * site and sweep (the same values, so the same samples; the raw bias is still
 * read when a chain's weights underflow).
 */
int tthrml_potts3d_bias_weights(const float* bias_dev, int64_t n_sites, int32_t q, float* bias_weights_dev,
                                void* stream);
int tthrml_potts3d_step_weights(int8_t* state_dev, int64_t n_chains, int32_t X, int32_t Y, int32_t Z,
                                int32_t colour, int64_t target_row0, int64_t source_row0, const float* J_dev,
                                const float* bias_dev, int32_t q, int64_t chain_offset, const float* variates_dev,
                                int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                                const tthrml_run_ctl* ctl_dev, const float* bias_weights_dev, void* stream);

/*
 * One checkerboard half-sweep of a single-chain 2-D Ising lattice (uniform
 * couplings) on split-colour int8 state.  Replaces the spin group kernel
 * (tt_thrml/compiler.py:303-324) for lattice programs, where neighbours follow
 * from the site position.  colour_state / other_state: int8 +-1 arrays
 * [rows_local][width/2] of the updated colour and of the other colour; local
 * row i is lattice row (global_row0 + i) mod height; site (Y, x) of colour
 * (x + Y) % 2 is column x/2.  Rows [row_lo, row_hi) are updated; their up and
 * down neighbours are local rows i-1 and i+1 (halo rows of a strip), or wrap
 * around when wrap_rows is set (rows_local == height, the whole lattice).
 * The decision uses the 4 neighbour signs (left, right, up, down; bit set =
 * -1) as an index into thresholds[16] (Philox: "up" iff the 23-bit draw m <
 * threshold) or fields[16] (variates: "up" iff 2 * field > logit, variates
 * [variates_sweeps][height * width/2] per colour block).  Philox draws are
 * split uniforms: with flat row f = block_row0 + Y*width/2 + x/2, the top 16
 * bits of m are half f % 2 of word (f / 2) % 4 of counter (chain, f / 8,
 * sweep, "LSPI"), the low 7 bits word 0 >> 25 of (chain, f, sweep, "LREF"),
 * read only when the top bits equal the threshold's.  trace (NULL to
 * skip): int64 [trace_len][2]; entry `sweep` receives the sum of the new
 * spins of local rows [count_lo, count_hi) and, for colour 1, the bond sum
 * sum_i s_i (s_left + s_right + s_up + s_down) over them.  Requires width %
 * 32 == 0, even height and 16-byte aligned buffers.
 */
int tthrml_ising2d_halfsweep(int8_t* colour_state, const int8_t* other_state, int64_t width, int64_t rows_local,
                             int32_t wrap_rows, int64_t row_lo, int64_t row_hi, int64_t global_row0, int64_t height,
                             int32_t colour, int64_t block_row0, const uint32_t* thresholds_dev,
                             const float* fields_dev, const float* variates_dev, int64_t variates_sweeps,
                             int64_t chain, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl_dev,
                             int64_t count_lo, int64_t count_hi, int64_t* trace_dev, int64_t trace_len,
                             void* stream);

/*
 * Persistent multi-sweep update of a small periodic 2-D Ising lattice with
 * many chains (uniform couplings): every CTA keeps the lattice of 8 chains in
 * shared memory (height * width bytes) and runs n_half_sweeps checkerboard
 * half-sweeps from colour0 (sweep index sweep0 + (colour0 + t) / 2 for
 * half-sweep t), then writes the state back.  state_dev: bit-packed uint32
 * [rows][n_chains/32] (bit set = -1) with colour c's site (Y, x) at row
 * row0_colour_c + Y*width/2 + x/2.  Decision as tthrml_ising2d_halfsweep
 * (16-entry threshold table over the left/right/up/down sign pattern);
 * split-uniform Philox draws: top 16 bits half chain % 2 of word (chain / 2)
 * % 4 of counter (chain / 8, row, sweep, "LSPI"), low 7 bits word 0 >> 25 of
 * (chain, row, sweep, "LREF").  obs_dev (NULL: none): float64 [n_obs][n_chains],
 * sample i = per-chain sum of the spins of the colours in obs_colours (bit
 * mask) after half-sweep obs_first + i * obs_every.  A thrml schedule with
 * its magnetisation observable is one launch.  Requires n_chains % 32 == 0,
 * chain_offset % 8 == 0, even dimensions.  Half-sweeps are separated by a
 * bounded split-phase barrier in shared memory: on expiry *error_dev, when
 * not NULL, receives a non-zero code and the remaining half-sweeps are
 * skipped.
 */
int tthrml_ising2d_resident(uint32_t* state_dev, int64_t n_chains, int32_t height, int32_t width,
                            int64_t row0_colour0, int64_t row0_colour1, const uint32_t* thresholds_dev,
                            uint64_t seed, uint32_t sweep0, int32_t colour0, int64_t n_half_sweeps,
                            double* obs_dev, int64_t obs_first, int64_t obs_every, int64_t n_obs,
                            int32_t obs_colours, int64_t chain_offset, const tthrml_run_ctl* ctl_dev,
                            int32_t* error_dev, void* stream);

/*
 * tthrml_ising2d_resident for count-symmetric threshold tables (the kernel
 * reads thresholds[2^n - 1] for n = 0..4), bit-sliced over 4 sites x 8 chains
 * per 32-bit word.  Random bits ("planes8"): bit 22 - b of the 23-bit draw of
 * chain c at flat row f is bit 8 (f % 4) + c % 8 of word b % 4 of counter
 * (c / 8, f / 4, sweep, "LPL0" + b / 4).  Requires width % 8 == 0 and block
 * rows % 4 == 0.
 */
int tthrml_ising2d_resident_planes(uint32_t* state_dev, int64_t n_chains, int32_t height, int32_t width,
                                   int64_t row0_colour0, int64_t row0_colour1, const uint32_t* thresholds_dev,
                                   uint64_t seed, uint32_t sweep0, int32_t colour0, int64_t n_half_sweeps,
                                   double* obs_dev, int64_t obs_first, int64_t obs_every, int64_t n_obs,
                                   int32_t obs_colours, int64_t chain_offset, const tthrml_run_ctl* ctl_dev,
                                   int32_t* error_dev, void* stream);

/*
 * Halo export of a strip-decomposed lattice (tthrml_ising2d_halfsweep_x):
 * while a half-sweep computes local rows [up_row0, up_row0 + rows) it also
 * stores them at `up` (the up neighbour's mailbox, peer memory), rows
 * [down_row0, down_row0 + rows) at `down`, in parity slot
 * ((sweep / sweeps_per_period) + 1) % 2 (slot_bytes apart).  rows = 0: none.
 */
typedef struct tthrml_halo_export {
  int8_t* up;
  int8_t* down;
  int64_t up_row0;
  int64_t down_row0;
  int64_t rows;
  int64_t slot_bytes;
  uint32_t sweeps_per_period;
  uint32_t reserved;
} tthrml_halo_export;

/* tthrml_ising2d_halfsweep with the fused halo export (export_host may be NULL). */
int tthrml_ising2d_halfsweep_x(int8_t* colour_state, const int8_t* other_state, int64_t width, int64_t rows_local,
                               int32_t wrap_rows, int64_t row_lo, int64_t row_hi, int64_t global_row0,
                               int64_t height, int32_t colour, int64_t block_row0, const uint32_t* thresholds_dev,
                               const float* fields_dev, const float* variates_dev, int64_t variates_sweeps,
                               int64_t chain, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl_dev,
                               int64_t count_lo, int64_t count_hi, int64_t* trace_dev, int64_t trace_len,
                               const tthrml_halo_export* export_host, void* stream);

/*
 * tthrml_ising2d_halfsweep_planes on bit-packed rows: colour_state and
 * other_state are uint32 [rows_local][width/64], word w of a row holding the
 * row's sites 32w .. 32w + 31 (site s at bit 8 (s % 4) + s / 4, bit set = -1);
 * the same draws and decisions as tthrml_ising2d_halfsweep_planes.  The halo
 * export stores words (slot_bytes >= rows * width/16).  Requires width % 64 ==
 * 0 and block_row0 % 32 == 0.
 */
int tthrml_ising2d_halfsweep_bits(uint32_t* colour_state, const uint32_t* other_state, int64_t width,
                                  int64_t rows_local, int32_t wrap_rows, int64_t row_lo, int64_t row_hi,
                                  int64_t global_row0, int64_t height, int32_t colour, int64_t block_row0,
                                  const uint32_t* thresholds_dev, int64_t chain, uint64_t seed, uint32_t sweep,
                                  const tthrml_run_ctl* ctl_dev, int64_t count_lo, int64_t count_hi,
                                  int64_t* trace_dev, int64_t trace_len, const tthrml_halo_export* export_host,
                                  void* stream);

/*
 * tthrml_ising2d_halfsweep_x for count-symmetric threshold tables (thresholds
 * equal for patterns with the same number of -1 neighbours; the kernel reads
 * thresholds[2^n - 1] for n = 0..4), Philox mode, bit-sliced over 32 sites.
 * Random bits ("planes"): bit 22 - b of the 23-bit draw of flat row f is bit
 * 8 (f % 4) + (f % 32) / 4 of word b % 4 of counter (chain, f / 32, sweep,
 * "LPL0" + b / 4).  Requires width % 64 == 0 and block_row0 % 32 == 0.
 * Replaces the same reference group call as tthrml_ising2d_halfsweep
 * (tt_thrml/compiler.py:436-450) for uniform lattices.
 */
int tthrml_ising2d_halfsweep_planes(int8_t* colour_state, const int8_t* other_state, int64_t width,
                                    int64_t rows_local, int32_t wrap_rows, int64_t row_lo, int64_t row_hi,
                                    int64_t global_row0, int64_t height, int32_t colour, int64_t block_row0,
                                    const uint32_t* thresholds_dev, int64_t chain, uint64_t seed, uint32_t sweep,
                                    const tthrml_run_ctl* ctl_dev, int64_t count_lo, int64_t count_hi,
                                    int64_t* trace_dev, int64_t trace_len, const tthrml_halo_export* export_host,
                                    void* stream);

/*
 * Peer memory for the halo mailboxes: tthrml_ipc_malloc allocates zeroed
 * device memory and writes its 64-byte CUDA IPC handle to `handle_host`;
 * another process opens it with tthrml_ipc_open (peer access enabled on
 * demand) and releases it with tthrml_ipc_close; tthrml_free frees the
 * owner's allocation.
 */
int tthrml_ipc_malloc(int64_t bytes, void** ptr_out, void* handle_host);
int tthrml_ipc_open(const void* handle_host, void** ptr_out);
int tthrml_ipc_close(void* ptr);
int tthrml_free(void* ptr);
/* cudaMemcpyAsync with the kind inferred from the addresses (host, device or
 * a peer's IPC mapping), ordered on `stream`. */
int tthrml_memcpy(void* dst, const void* src, int64_t bytes, void* stream);

/*
 * End of an exchange period: publishes the period number p =
 * (sweep + ctl->sweep) / sweeps_per_period + 1 in the two neighbours' flags
 * (system-scope release after a system fence).
 */
int tthrml_halo_signal(uint32_t* up_flag_dev, uint32_t* down_flag_dev, uint32_t sweeps_per_period, uint32_t sweep,
                       const tthrml_run_ctl* ctl_dev, void* stream);

/*
 * Start of exchange period p (computed as above; p = 1 imports nothing):
 * waits until both own flags (from up, from down) reach p - 1 -- a bounded
 * wait of about one second; on expiry *error_dev is set to 1 and nothing is
 * copied -- then copies the mailbox slot (p - 1) % 2 ([2 directions][2
 * colours][rows][width/2]) into local rows [top_row0, +rows) (from up) and
 * [bottom_row0, +rows) (from down) of both colours.
 */
int tthrml_halo_import(int8_t* colour0_dev, int8_t* colour1_dev, int64_t width, int64_t rows, int64_t top_row0,
                       int64_t bottom_row0, const int8_t* mailbox_dev, const uint32_t* flags_dev,
                       uint32_t sweeps_per_period, uint32_t sweep, const tthrml_run_ctl* ctl_dev, int32_t* error_dev,
                       void* stream);

/*
 * Dense bipartite block update on the tensor cores (tcgen05, bf16 operands,
 * fp32 accumulation in TMEM).  Replaces the group kernel of a block whose
 * interaction with another block is a dense weight matrix (the RBM case:
 * per-node weight rows over every source unit, tt_thrml/compiler.py:173-176,
 * 303-365):
 *   field[m][n] = sum_k source_state[m][k] * weights_nk[n][k] + bias[n]
 * source_state: bf16 [n_chains][n_sources] (chain-major), weights_nk: bf16
 * [n_units][n_sources]; the target block's new state is written to out_state
 * as `out_pieces` bf16 pieces per value (bf16 [n_chains][out_pieces *
 * n_units]; piece p, at column p * n_units + unit, is the bf16 rounding of
 * the value minus pieces 0..p-1, so 3 pieces hold a float32 exactly and a
 * source operand built from them with the weights repeated along K gives the
 * float32 field) and, when out_state_f32 is not NULL, to float32.
 * family TTHRML_SPIN draws +1 with probability sigmoid(2*field) (variates:
 * 2*field > logit); TTHRML_GAUSSIAN draws field*var + sqrt(var)*xi with
 * var = 1/(precision + 1e-6).  Philox counters run along the unit axis of a
 * chain: spins of units 4j..4j+3 take the four words of
 * (chain_offset + chain, (row0 + unit) / 4, sweep, "DSPI"); gaussian units
 * of flat rows 4j..4j+3 (row = row0 + unit) the counter (chain_offset +
 * chain, j, sweep, "DGAU") through Box-Muller: words 2p, 2p+1 give
 * r = sqrt(-2 ln u0), theta = 2 pi u1, row 4j+2p takes r cos theta and row
 * 4j+2p+1 r sin theta.  variates: [variates_sweeps][n_units][n_chains]
 * or NULL.
 * Requires n_chains % 128 == 0, n_units % 256 == 0, n_sources % 64 == 0 and
 * 16-byte aligned buffers.  Waits inside the kernel are bounded: a device
 * error word (*error, zero on entry) receives a non-zero code if one expired.
 */
int tthrml_dense_field_sample(const void* source_state, const void* weights_nk, int64_t n_chains,
                              int64_t n_units, int64_t n_sources, const float* bias, int32_t family,
                              float precision, void* out_state, float* out_state_f32, int32_t out_pieces,
                              int64_t row0,
                              int64_t chain_offset, const float* variates, int64_t variates_sweeps,
                              uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, int32_t* error,
                              void* stream);

/*
 * tthrml_dense_field_sample with the spin decisions settled from the exact
 * field (the same group call, tt_thrml/compiler.py:173-176, 303-365).  The
 * tensor cores' float32 sum of a K-term field can be off by ~1e-5 at K =
 * 4096; a spin decided within 1e-5 of its threshold (u * (1 + e^(-2 field))
 * against 1, or 2 field - logit in variates mode) is recorded in `ties` and
 * decided again by a second kernel on the same stream from bias[n] +
 * sum_k source_state[m][k] * weights_nk[n][k] summed in double, with the
 * same Philox word or uploaded logit.  ties: uint32 [4 + 2 * ties_capacity],
 * 16-byte aligned, zero before its first use and owned by one stream; words
 * 0-1 are zero again after each call, word 2 counts the near decisions that
 * did not fit (they keep their float32 decision), then (chain, unit) pairs.
 * 1 <= ties_capacity < 2^31.  Gaussian blocks ignore the list.  Other
 * arguments and requirements as tthrml_dense_field_sample.
 */
int tthrml_dense_field_sample_ties(const void* source_state, const void* weights_nk, int64_t n_chains,
                                   int64_t n_units, int64_t n_sources, const float* bias, int32_t family,
                                   float precision, void* out_state, float* out_state_f32, int32_t out_pieces,
                                   int64_t row0, int64_t chain_offset, const float* variates,
                                   int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                                   const tthrml_run_ctl* ctl, int32_t* error, uint32_t* ties,
                                   int64_t ties_capacity, void* stream);

/*
 * Adds `delta` to ctl->sweep on `stream` (the last node of a captured
 * multi-sweep CUDA graph, so each replay continues the run).
 */
int tthrml_ctl_advance(tthrml_run_ctl* ctl_dev, uint32_t delta, void* stream);

/*
 * Read-back helper: copies rows [row_start, row_start+n_rows) of a
 * chain-innermost state into a chain-major buffer out[chain][row] decoded
 * like _global_chunk_to_block_state (tt_thrml/executor.py:433-438):
 *   out_kind 0: uint8 bool   (spin: value > 0)
 *   out_kind 1: int32        (categorical: rounded index)
 *   out_kind 2: float32      (gaussian / raw)
 */
int tthrml_decode_rows(const void* state_dev, int32_t state_dtype, int64_t n_chains,
                       int64_t row_start, int64_t n_rows, int32_t out_kind,
                       void* out_dev, void* stream);

/*
 * Inverse of tthrml_decode_rows for load_state
 * (tt_thrml/executor.py:104-136): in_dev is chain-major [n_chains][n_rows]
 * values of type in_dtype (TTHRML_STATE_F32 or TTHRML_STATE_I8; bool data
 * passes as I8).  With as_spin set a value v is stored as +1 if v > 0 else
 * -1 (tt_thrml/executor.py:132-133); otherwise it is stored as is
 * (categorical index, gaussian value).
 */
int tthrml_encode_rows(const void* in_dev, int32_t in_dtype, int32_t as_spin, int64_t n_rows,
                       int32_t state_dtype, int64_t n_chains, int64_t row_start, void* state_dev,
                       void* stream);

/*
 * Per-chain sum of rows [row_start, row_start+n_rows): out[chain] (float64,
 * accumulated with atomics onto the existing value).  Magnetisation of spin
 * blocks; the observable of the lattice configurations.
 */
int tthrml_sum_rows(const void* state_dev, int32_t state_dtype, int64_t n_chains,
                    int64_t row_start, int64_t n_rows, double* out_dev, void* stream);

/*
 * Device-side moment accumulation (the reference's MomentAccumulatorObserver
 * with the state left on the device, tt_thrml/executor.py:389-409): for each
 * moment m, acc[m][chain] += product over k < order of value(rows[m][k],
 * chain), stopping at the first row < 0.  value: spins +-1, or 1 / 0 when
 * spin_as_bool is set (the reference's boolean spin state, spin rows flagged
 * in spin_rows[m][k]; every row of a bit-packed state is a spin); other rows
 * as stored.  rows / spin_rows: device [n_moments][order]; acc: device
 * float64 [n_moments][n_chains].  n_moments <= 65535.
 */
int tthrml_moments_accumulate(const void* state_dev, int32_t state_dtype, int64_t n_chains,
                              const int64_t* rows_dev, const uint8_t* spin_rows_dev, int32_t order,
                              int64_t n_moments, int32_t spin_as_bool, double* acc_dev, void* stream);

/* Host-only: greedy graph colouring in node order (smallest free colour).
 * Returns the number of colours in *n_colours.  No device work. */
int tthrml_greedy_colouring(int64_t n_nodes, const int64_t* row_ptr_host,
                            const int32_t* cols_host, int32_t* colour_host,
                            int32_t* n_colours);

/* Makes `device` current for this library's CUDA runtime on the calling
 * thread (the library links its own runtime; callers that switch devices
 * call this before launching on another device). */
int tthrml_set_device(int32_t device);

const char* tthrml_last_error(void);
int tthrml_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* TTHRML_H_ */
