/*
 * hello_b200.h - C ABI of the B200-native HELLO hot path (libhello_b200.so).
 *
 * Plain pointers and sizes only.  Every array argument is a CUDA device
 * pointer on the current device unless stated otherwise; `stream` is a
 * cudaStream_t (NULL = legacy default stream).  Functions return 0 on success
 * and a nonzero HB_* code on failure; hb_last_error() then holds a message
 * (per calling thread).  No entry point allocates device memory: callers
 * provide scratch through `workspace`, sized by the matching *_workspace()
 * query for the same shapes on the same device, 256-byte aligned (as returned
 * by cudaMalloc or a caching allocator).  Calls that report device
 * status (scans, pair costs, the PDHG solve) synchronise `stream` before
 * returning.
 *
 * Paths in the citations are inside the reference project (WenzhouXia/hello-ot).
 */
#ifndef HELLO_B200_H
#define HELLO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HB_ABI_VERSION 2

enum {
    HB_OK = 0,
    HB_BAD_ARGUMENT = 1,   /* shapes, k, scale, cost type, null pointers */
    HB_BAD_INPUT = 2,      /* index data out of range (pair costs, PDHG support) */
    HB_WORKSPACE = 3,      /* workspace smaller than the *_workspace() size */
    HB_CUDA = 4,           /* a CUDA runtime call failed */
    HB_TENSOR_MAP = 5,     /* TMA descriptor could not be built */
    HB_LAUNCH = 6,         /* a kernel launch failed */
    HB_DEVICE_TIMEOUT = 7  /* a bounded device-side wait gave up */
};

int hb_abi_version(void);
const char* hb_last_error(void);

/* Instrumentation (no counterpart in the reference, which has no kernel timers,
 * docs/generic_scan.md:68-70).  hb_kernel_launch_count: kernels launched by this
 * library in this process so far.  hb_set_kernel_timing(1) makes the calling
 * thread's next calls bracket their main kernels with CUDA events;
 * hb_last_kernel_times then returns their device times in ms (scans: pass 1,
 * pass 2; pair costs: the pair kernel; PDHG: one iteration block average). */
unsigned long long hb_kernel_launch_count(void);
void hb_set_kernel_timing(int enable);
int hb_last_kernel_times(double* ms, int capacity);

/* ---------------------------------------------------------------------------
 * ℓ2² (bilinear) full-space pricing scan, bidirectional top-k + certificate.
 *
 * Replaces ScanExtension.fused_bidir_topk_stats_raw
 * (src/hello_ot/kernels/generic_scan.py:577-597) and the kernels behind it,
 * raw_scan_tiled (src/hello_ot/_native/generic_scan/pricing_small.cu:298-304)
 * and pricing.scan (pricing.cu:203-212); also ScanExtension.raw_lowrank_stats_only
 * (generic_scan.py:502-510) when k == 0.
 *
 * x: q x d, y: n x d, fp32 row-major.  x_cost = a (|x|^2), y_cost = b,
 * x_bias = f - a, y_bias = g - b (fp64).  For every pair
 *   dot = fp32(dot_scale * <x_i, y_j>), cost = (a_i + b_j) - dot,
 *   score = (dot + x_bias_i) + y_bias_j                      (fp64)
 * row_vals/row_idx (q x k): best k (score, j) of each x row; col_vals/col_idx
 * (n x k): best k (score, i) of each y row; descending, lower index on ties,
 * missing slots (-inf, -1).  k in 0..32 (0: certificate only, outputs unused).
 * stats5 (device, 5 doubles): [sum max(s,0)^2, sum cost^2, max s+, max |cost|,
 * count s>0] over all q*n pairs; written when compute_stats != 0.
 * precision: 1 = one TF32 tensor-core product, 3 = 3-term split hi*hi + hi*lo + lo*hi
 * on fp16 halves of the clouds scaled by powers of two (fp32-class dots; feature
 * magnitudes must be finite and below 2^75, else HB_BAD_INPUT),
 * optionally OR one of HB_L2SQ_ONE_PASS / HB_L2SQ_TWO_PASS.  A one-pass scan
 * (k <= 8) keeps row lists in registers and column lists in the workspace; a
 * two-pass scan runs the row pass again with the clouds' roles exchanged.  Both
 * give the same lists bit for bit (the certificate sums differ in summation
 * order only).  Without a flag the scan picks one pass when k <= 8 and the
 * tensor-core work per pair dominates the list upkeep (d >= 128), else two.
 * The one-pass kernel runs either one CTA per rectangle of the pair space or
 * CTA pairs (clusters of two sharing each column tile through a cta_group::2
 * MMA); OR HB_L2SQ_CTA_PAIRS or HB_L2SQ_SINGLE_CTA to force either (same lists).
 * OR HB_L2SQ_EXACT for the fp64 re-check: the lists are then the exact top-k of
 * score = (dot_scale <x_i, y_j> + x_bias_i) + y_bias_j with the dot in fp64 from the
 * fp32 features (values reported in that arithmetic): each list's candidates are
 * re-scored in fp64, and a list whose runner-up lies within a rigorous bound of the
 * approximate dot's error of its k-th exact score is recomputed in fp64 against every
 * column (index sets equal the exact fp64 top-k wherever the k-th/(k+1)-th gap exceeds
 * the fp64 rounding of the scores).  The certificate sums stay fp32-class.
 * min_groups: column groups (0 = automatic).
 * ------------------------------------------------------------------------- */
#define HB_L2SQ_TWO_PASS 0x10
#define HB_L2SQ_ONE_PASS 0x20
#define HB_L2SQ_CTA_PAIRS 0x100
#define HB_L2SQ_SINGLE_CTA 0x200
#define HB_L2SQ_EXACT 0x400
size_t hb_l2sq_scan_workspace(int64_t q, int64_t n, int64_t d, int k, int precision, int min_groups);
int hb_l2sq_scan(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* x_cost,
                 const double* y_cost, const double* x_bias, const double* y_bias, int k, double dot_scale,
                 int compute_stats, int precision, int min_groups, double* row_vals, int32_t* row_idx,
                 double* col_vals, int32_t* col_idx, double* stats5, void* workspace, size_t workspace_bytes,
                 void* stream);
/* Lists the calling thread's last HB_L2SQ_EXACT scan recomputed against every column
 * (out2[0]: row lists, out2[1]: column lists; zeros after a scan without the flag).
 * Instrumentation of the fp64 re-check; no counterpart in the reference. */
int hb_l2sq_last_rescans(int64_t* out2);

/* ---------------------------------------------------------------------------
 * Cost perturbation of the norm costs (the _ex entry points below).
 *
 * Replaces the sigma > 0 arguments of the reference's fused norm kernels:
 * NoiseParams / sigma_noise (src/hello_ot/_native/generic_scan/cost.cu:350-423,
 * norm_cost_scan_kernel.cu:48-...), with the coefficients of
 * src/hello_ot/costs/metric_perturbation.py:19-33 (_index_hash_parameters).
 * The perturbed cost is c_ij + noise(source, target) in fp64; mode 1
 * (index_hash) noise is sigma * fp32 hash of the two global indices, mode 0
 * (rank2) fp32(sigma) * (__sinf(...) / 2 + 1/2).  query_index / database_index
 * (device, int64) hold the global index of each x row / y row (for pair costs:
 * of each source row / target row); row_is_source tells whether the x rows
 * are the sources.  sigma == 0 (or a null pointer) means no perturbation.
 * ------------------------------------------------------------------------- */
typedef struct hb_perturbation {
    double sigma;
    int64_t seed;
    int32_t mode;          /* 0 rank2, 1 index_hash */
    int32_t row_is_source; /* 1: x rows are sources */
    const int64_t* query_index;
    const int64_t* database_index;
    int64_t coefficients[6]; /* index_hash: (source, target, offset) for prime 2003, then for 2011 */
} hb_perturbation;

/* ---------------------------------------------------------------------------
 * ℓ2² directional top-k (one side only: the initial dual-assignment scan).
 *
 * Replaces ScanExtension.initialization_directional_topk_raw and its alias
 * fused_directional_topk_raw (src/hello_ot/kernels/generic_scan.py:512-518,
 * 560-575) and the kernel behind them, raw_initial
 * (src/hello_ot/_native/generic_scan/cost.cu:248-348).
 *
 * For every x row the best k (score, j), score = (fp32(dot_scale <x_i, y_j>)
 * + x_bias_i) + y_bias_j in fp64, descending, lower index on ties, missing
 * slots (-inf, -1); k in 1..32.  Same kernel and arithmetic as the row side of
 * hb_l2sq_scan, without the column lists and the certificate.
 * ------------------------------------------------------------------------- */
size_t hb_l2sq_topk_workspace(int64_t q, int64_t n, int64_t d, int k, int precision);
int hb_l2sq_topk(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* x_bias,
                 const double* y_bias, int k, double dot_scale, int precision, double* row_vals, int32_t* row_idx,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * ℓ1 / ℓ∞ / ℓ2 directional top-k (the initial c-transform scan).
 *
 * Replaces ScanExtension.fused_gcost_topk (src/hello_ot/kernels/generic_scan.py:520-531)
 * -> directional(minimum=True) (:219-306) and its kernels, queue_kernel
 * (src/hello_ot/_native/generic_scan/initial.cu:34-107).
 *
 * For every x row the best k (score, j) with score = g_j - c_ij (fp64, c_ij the
 * fp32 distance), descending, lower index on ties, missing slots (-inf, -1);
 * the reference reports the values negated (c_ij - g_j ascending), which the
 * host layer does.  stats2 (device, 2 doubles, when compute_stats != 0):
 * [sum c^2, max |c|] over all q*n pairs.  k in 1..32.
 * ------------------------------------------------------------------------- */
size_t hb_norm_topk_workspace(int64_t q, int64_t n, int k);
int hb_norm_topk(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* g, int cost_type,
                 int k, int compute_stats, double* row_vals, int32_t* row_idx, double* stats2, void* workspace,
                 size_t workspace_bytes, void* stream);
int hb_norm_topk_ex(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* g, int cost_type,
                    int k, int compute_stats, double* row_vals, int32_t* row_idx, double* stats2, void* workspace,
                    size_t workspace_bytes, void* stream, const hb_perturbation* perturbation);

/* ---------------------------------------------------------------------------
 * ℓ1 / ℓ∞ / ℓ2 full-space pricing scan (CUDA cores), bidirectional top-k +
 * certificate.  cost_type: 0 l1, 1 linf, 2 l2.
 *
 * Replaces ScanExtension.fused_gcost_bidir_certificate and
 * ScanExtension.fused_gcost_certificate (src/hello_ot/kernels/generic_scan.py:533-558)
 * with their unperturbed generic_scan.bidirectional / certificate_only paths
 * (generic_scan.py:328-465; kernels cost.cu:10-85, pricing_small.cu:70-160).
 *
 * score = (g_j - c_ij) + f_i with c_ij the fp32 distance (features summed in
 * index order, ℓ2 via fma then sqrtf).  Outputs and k as for hb_l2sq_scan.
 * For 1 <= k <= 8 the scan makes one pass over the pairs (column lists kept
 * per row group in the workspace); cost_type | HB_NORM_TWO_PASS forces a
 * second pass with the clouds' roles exchanged instead.  Both give the same
 * lists bit for bit.  The workspace size covers both.
 * ------------------------------------------------------------------------- */
#define HB_NORM_TWO_PASS 0x10
size_t hb_norm_scan_workspace(int64_t q, int64_t n, int k);
int hb_norm_scan(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* f, const double* g,
                 int cost_type, int k, int compute_stats, double* row_vals, int32_t* row_idx, double* col_vals,
                 int32_t* col_idx, double* stats5, void* workspace, size_t workspace_bytes, void* stream);
int hb_norm_scan_ex(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* f, const double* g,
                    int cost_type, int k, int compute_stats, double* row_vals, int32_t* row_idx, double* col_vals,
                    int32_t* col_idx, double* stats5, void* workspace, size_t workspace_bytes, void* stream,
                    const hb_perturbation* perturbation);

/* ---------------------------------------------------------------------------
 * Allocation-free variant of hb_norm_scan (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory themselves: a host runtime
 * reached through an FFI that has no CUDA allocator binding, a caller running
 * under a fixed memory budget that forbids new device allocations, or one that
 * must not grow the process footprint in the middle of a solve.  It takes no
 * workspace: its scratch is a static device array of
 * HB_NORM_NOALLOC_SCRATCH_BYTES inside libhello_b200.so, which every GPU that
 * loads the library holds until the process exits.  Problems whose scratch
 * (hb_norm_scan_workspace(q, n, k)) exceeds that size are rejected with
 * HB_WORKSPACE and a message; use hb_norm_scan for them.  It calls no
 * cudaMalloc/cudaFree or other allocating routine.  Every call looks up the
 * array's device address on the current device (nothing is cached, so a device
 * reset is harmless); the first call on a device also loads the library's
 * module there and should come before any stream capture.  All calls on a
 * device share the one array, so calls that overlap
 * on the GPU (other streams, other host threads) race; serialise them.
 * Arguments and results as hb_norm_scan; the stream is synchronised.
 * ------------------------------------------------------------------------- */
#define HB_NORM_NOALLOC_SCRATCH_BYTES (16u << 20)
int hb_norm_scan_noalloc(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* f,
                         const double* g, int cost_type, int k, int compute_stats, double* row_vals, int32_t* row_idx,
                         double* col_vals, int32_t* col_idx, double* stats5, void* stream);

/* ---------------------------------------------------------------------------
 * Merge of top-k lists: for each of `rows` rows, the best k (score, index)
 * entries over `parts` lists of `width` entries (vals/idx laid out
 * [parts][rows][width], index -1 = empty), same order and tie rule as the scans.
 * Replaces the cross-tile merges of the reference (generic_scan.py:131-147
 * _merge, pricing.cu:164-180 reduce_columns, pricing_small.cu:270-277
 * merge_raw_tile) and merges per-GPU column lists of a row-sharded scan.
 * ------------------------------------------------------------------------- */
int hb_merge_topk(const double* vals, const int32_t* idx, int parts, int64_t rows, int width, int k,
                  double* out_vals, int32_t* out_idx, void* stream);

/* ---------------------------------------------------------------------------
 * Active-support pair costs (SDDMM), fp64 output in input order.
 * cost_type 3 (bilinear): out_e = (a_r + b_c) - dot_scale <x_r, y_c>, replacing
 *   _cost_pairs_lowrank_batched (src/hello_ot/costs/pairs.py:221-440).
 * cost_type 0/1/2 (ℓ1/ℓ∞/ℓ2): replacing fused_gcost_pairs
 *   (src/hello_ot/_native/norm_cost_scan/norm_cost_scan_kernel.cu:249-275)
 *   without perturbation; a and b are ignored (may be NULL).
 * rows/cols: int64 indices into x (nx rows) and y (ny rows).  An index out of
 * range gives HB_BAD_INPUT (its output is NaN).
 * ------------------------------------------------------------------------- */
size_t hb_pair_costs_workspace(void);
int hb_pair_costs(int cost_type, const float* x, const float* y, int64_t nx, int64_t ny, int64_t d,
                  const double* a, const double* b, double dot_scale, const int64_t* rows, const int64_t* cols,
                  int64_t count, double* out, void* workspace, size_t workspace_bytes, void* stream);
int hb_pair_costs_ex(int cost_type, const float* x, const float* y, int64_t nx, int64_t ny, int64_t d,
                     const double* a, const double* b, double dot_scale, const int64_t* rows, const int64_t* cols,
                     int64_t count, double* out, void* workspace, size_t workspace_bytes, void* stream,
                     const hb_perturbation* perturbation);

/* ---------------------------------------------------------------------------
 * Restricted-OT Halpern-PDHG (balanced transport LP on the active support).
 *
 * Replaces RestrictedOTPDLP.solve_restricted / _solve_once
 * (src/hello_ot/_internal/lp/restricted_ot_pdlp.py:39-100,
 * cpp_restricted_ot.py:40-72 -> src/hello_ot/_native/cpp/solver.cpp:39-381)
 * and, behind backend="native", the cuPDLPx loop (cupdlpx/solver.cu:581-700).
 * One call is one _solve_once: the NUMERICAL_DIVERGENCE retry with scalar
 * rescaling is the caller's (restricted_ot_pdlp.py:76-100).
 *
 * rows/cols/costs: E edges (int64, int64, fp64); masses: n source masses
 * followed by m target masses; x0 (E) and y0 (n+m) warm starts or NULL.
 * x_out (E), y_out (n+m): unscaled primal and dual.
 * trace (host memory, may be NULL): one hb_pdlp_trace_row per evaluation.
 * ------------------------------------------------------------------------- */
typedef struct hb_pdlp_controls {
    int32_t evaluation_frequency;  /* iterations between evaluations (200 in the reference) */
    int32_t scalar_rescaling;      /* 1: bound/objective scalar rescaling (the retry mode) */
    int64_t iteration_limit;
    double time_limit_seconds;
    double tol_objective, tol_primal, tol_dual;
    double initial_primal_weight;  /* > 0 overrides the initial norm-ratio weight */
    int32_t atomic_sums;           /* node-sum order, one of HB_PDLP_SUMS_*:
                                      ORDERED (0): each node sums its edges in the reference's order,
                                        bit-reproducible and bit-identical to the reference;
                                      ATOMIC (1): atomics in the edge pass (fastest on large random
                                        supports; the order, so the last bits, vary run to run);
                                      TREE (2): as ORDERED, except that a side whose mean degree is
                                        >= 64 (a dense support, e.g. a coarsest level) sums each node
                                        in a fixed lane-strided tree: bit-reproducible run to run,
                                        not the reference's order, several times faster there */
    int32_t termination_norm;      /* norm of the termination test, one of HB_PDLP_NORM_*:
                                      L2 (0): solver.cpp's, ||Ax - b||_2 / (1 + ||b||_2) and
                                        ||(A^T y - c)_+||_2 / (1 + ||c||_2);
                                      LINF (1): cuPDLPx's termination_norm = "linf"
                                        (cupdlpx/utils.cu:1027-1041): the same residuals in the
                                        max norm over (1 + ||b||_inf), (1 + ||c||_inf); restarts and
                                        the primal weight stay on the L2 residuals */
} hb_pdlp_controls;

enum { HB_PDLP_SUMS_ORDERED = 0, HB_PDLP_SUMS_ATOMIC = 1, HB_PDLP_SUMS_TREE = 2 };
enum { HB_PDLP_NORM_L2 = 0, HB_PDLP_NORM_LINF = 1 };

enum { HB_PDLP_OPTIMAL = 1, HB_PDLP_ITERATION_LIMIT = 2, HB_PDLP_NUMERICAL_DIVERGENCE = 3, HB_PDLP_TIME_LIMIT = 4 };

typedef struct hb_pdlp_info {
    int64_t iterations, restarts;
    int32_t termination, pad;
    double primal_objective, dual_objective;
    /* residuals in the termination norm, and the norms of c and b they are relative to */
    double abs_primal_residual, rel_primal_residual, abs_dual_residual, rel_dual_residual, rel_gap;
    double primal_weight, cost_norm, mass_norm;
    double setup_seconds, iteration_seconds;
    /* the L2 residuals (the restart and weight rules use these in either norm) */
    double l2_abs_primal_residual, l2_rel_primal_residual, l2_abs_dual_residual, l2_rel_dual_residual;
} hb_pdlp_info;

typedef struct hb_pdlp_trace_row {
    double iteration, primal_objective, dual_objective, rel_primal, rel_dual, rel_gap, primal_weight;
} hb_pdlp_trace_row;

size_t hb_restricted_ot_workspace(int64_t n, int64_t m, int64_t e);
int hb_restricted_ot_solve(const int64_t* rows, const int64_t* cols, const double* costs, int64_t e,
                           const double* masses, int64_t n, int64_t m, const double* x0, const double* y0,
                           const hb_pdlp_controls* controls, double* x_out, double* y_out, hb_pdlp_info* info,
                           hb_pdlp_trace_row* trace, int32_t trace_capacity, int32_t* trace_length,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Active-support maintenance: new candidate pairs.
 *
 * Replaces ActiveSupport.filter_new_candidate_pairs
 * (src/hello_ot/restricted_ot/active_support.py:483-506).
 *
 * Candidate keys rows[i] * n_target + cols[i] are sorted and made unique; a key
 * present among the n_active support keys (active_sorted != 0: already sorted
 * ascending) is dropped.  new_rows / new_cols (capacity n_candidates) receive
 * the remaining pairs in ascending key order, *new_count (host) their number.
 * A candidate index outside [0, n_source) x [0, n_target) is HB_BAD_INPUT.
 * ------------------------------------------------------------------------- */
size_t hb_filter_new_pairs_workspace(int64_t n_active, int64_t n_candidates);
int hb_filter_new_pairs(const int64_t* active_keys, int64_t n_active, int32_t active_sorted, const int32_t* rows,
                        const int32_t* cols, int64_t n_candidates, int64_t n_source, int64_t n_target,
                        int32_t* new_rows, int32_t* new_cols, int64_t* new_count, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Budgeted pruning: positions to remove from the active support.
 *
 * Replaces DualGapCleaning.select_indices_to_remove in protect-new mode with
 * ActiveSupport.pruning_values (src/hello_ot/refinement/budgeted_pruning.py:27-57,
 * 119-201; src/hello_ot/restricted_ot/active_support.py:401-421).
 *
 * An edge is removable when creation_iteration != current_inner_iter, != -1
 * (structural) and |x_prev| <= 1e-15.  Reduced cost = costs - (duals[row] +
 * duals[n_source + col]) in fp64, non-finite -> -inf.  *removable_count (host)
 * receives the number of removable edges; when it is >= num_to_remove,
 * positions receives the num_to_remove removable positions with the largest
 * reduced costs, descending, equal values by ascending position.
 * ------------------------------------------------------------------------- */
size_t hb_prune_select_workspace(int64_t n_edges);
int hb_prune_select(const int32_t* rows, const int32_t* cols, const double* costs, const double* x_prev,
                    const int32_t* creation_iteration, int64_t n_edges, const double* duals, int64_t n_source,
                    int64_t n_target, int32_t current_inner_iter, int64_t num_to_remove, int32_t* positions,
                    int64_t* removable_count, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* HELLO_B200_H */
