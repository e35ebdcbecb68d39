// Internal host-side interface between the kernel files and abi.cu.
#pragma once
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

namespace hb {

struct Perturb;  // cost perturbation parameters (perturb.cuh)

// Instrumentation: a process-wide count of kernel launches issued by this
// library, and optional CUDA-event timing of the main kernels of a call.
void count_launches(int n);
// Error reporting of the C ABI for entry points defined outside abi.cu:
// abi_fail records the message for hb_last_error and returns code;
// abi_finish synchronises the stream and maps a CUDA error to HB_CUDA.
int abi_fail(int code, const std::string& msg);
int abi_finish(cudaStream_t st, const char* what);
void timing_mark(cudaStream_t st);  // no-op unless timing is enabled on this thread

// ℓ2² scan (scan_l2sq.cu).  `precision` carries the public pass flags and, internally,
// L2SQ_ROWS_ONLY: row lists only (no column lists, no certificate; the cost vectors
// and column outputs may be null), the directional top-k.
constexpr int L2SQ_ROWS_ONLY = 0x40;
size_t l2sq_bytes(int64_t q, int64_t n, int64_t d, int k, int precision, int min_groups);
int l2sq_scan(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* nx, const double* ny,
              const double* qb, const double* dbb, int k, double dot_scale, int want_stats, int precision,
              int min_groups, double* rv, int* ri, double* cv, int* ci, double* stats5, void* ws, size_t ws_bytes,
              int* status_out, cudaStream_t st, std::string& err, int* rescans_out = nullptr);

// norm scans (scan_norm.cu).  f == nullptr: no query bias (the score is g - c
// exactly); rows_only: no column lists (cv/ci unused).
size_t norm_bytes(int64_t q, int64_t n, int k);
int norm_scan(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* f, const double* g,
              int kind, int k, int want_stats, double* rv, int* ri, double* cv, int* ci, double* stats5, void* ws,
              size_t ws_bytes, cudaStream_t st, std::string& err, bool rows_only = false,
              const struct Perturb* pert = nullptr);

// fp64 re-check of the ℓ2² lists (exact.cu).  exact_bounds writes the per-row error
// bounds of both clouds (y_err padded with zeros to n_pad); exact_finish re-scores one
// side's K-wide approximate lists in fp64, writes the exact top k_out and rescans the
// lists whose runner-up lies within the bound of the k-th exact score.
struct ExactSide {
    const float* qf;       // the lists' own rows (x for row lists, y for column lists)
    const float* dbf;      // the other cloud
    int64_t nq, ndb;
    const double* qbias;   // bias of the lists' own rows
    const double* dbias;   // bias of the other cloud
    const double* lv;      // [nq][K] approximate lists and their runner-ups
    const int* li;
    const double* run;
    const float* qerr;     // [nq] error bound of each list's approximate scores
    double* ov;            // [nq][k_out] exact top-k
    int* oi;
    int* flags;            // [nq] scratch: lists to rescan
    int* nflag;            // [1] scratch
    bool swap;             // the lists' rows are y: score (dot + dbias) + qbias
};
cudaError_t exact_bounds(const float* x, const float* y, int64_t q, int64_t n, int d, int64_t n_pad, int precision,
                         const int* exps, double dot_scale, float* norms_x, float* norms_y, unsigned* maxes,
                         float* x_err, float* y_err, int sms, cudaStream_t st);
cudaError_t exact_finish(int K, const ExactSide& side, int d, double dot_scale, int k_out, int sms, cudaStream_t st);

// partial top-k merge (scan_l2sq.cu): lists of `width` entries, bucket K >= width;
// pr / run_out: the partial lists' runner-ups in, the merged list's runner-up out (optional)
cudaError_t merge_lists(int K, const double* pv, const int* pi, int parts, int64_t rows, int width, int k_out,
                        double* ov, int* oi, cudaStream_t st, const double* pr = nullptr, double* run_out = nullptr);
cudaError_t merge_any(int K, const double* pv, const int* pi, int parts, int64_t rows, int k_out, double* ov, int* oi,
                      cudaStream_t st, const double* pr = nullptr, double* run_out = nullptr);

// pair costs (pairs.cu)
int pair_costs(int kind, const float* x, const float* y, int64_t nx, int64_t ny, int64_t d, const double* a,
               const double* b, double scale, const int64_t* rows, const int64_t* cols, int64_t count, double* out,
               int* status, cudaStream_t st, std::string& err, const Perturb* pert = nullptr);

// restricted-OT PDHG (pdlp.cu)
struct PdlpControls {
    int frequency;
    double time_limit;
    int64_t iteration_limit;
    double tol_objective, tol_primal, tol_dual;
    int rescale;
    double weight0;  // > 0: initial primal weight instead of the norm ratio
    int atomic;      // node sums by atomics in the edge pass (order varies run to run)
    int tree;        // high-degree sides summed by a fixed lane tree (not the reference's order)
    int linf = 0;    // termination test in the max norm (cuPDLPx termination_norm = "linf")
};
struct PdlpResult {
    int64_t iterations, restarts;
    int reason;  // 1 OPTIMAL, 2 ITERATION_LIMIT, 3 NUMERICAL_DIVERGENCE, 4 TIME_LIMIT
    double pobj, dobj, ap, rp, ad, rd, gap, weight, cost_norm, mass_norm;  // termination norm
    double ap2, rp2, ad2, rd2;  // L2 residuals
    double setup_seconds, iteration_seconds;
};
struct TraceRow { double iteration, pobj, dobj, rp, rd, gap, weight; };
size_t pdlp_bytes(int64_t n, int64_t m, int64_t e);
int pdlp_solve(const int64_t* rows, const int64_t* cols, const double* costs, int64_t e, const double* masses,
               int64_t n, int64_t m, const double* x0, const double* y0, const PdlpControls& ctl, double* x_out,
               double* y_out, PdlpResult* res, TraceRow* trace, int trace_cap, int* trace_len, void* ws,
               size_t ws_bytes, cudaStream_t st, std::string& err);

}  // namespace hb
