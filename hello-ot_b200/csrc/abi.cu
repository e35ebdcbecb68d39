// extern "C" entry points of libhello_b200.so (declared in include/hello_b200.h).
// Argument validation, workspace sizing, stream synchronisation and the
// translation of device status words into HB_* codes live here.
#include <cmath>
#include <cstdio>
#include <string>

#include "../../include/hello_b200.h"
#include "common.cuh"
#include "perturb.cuh"
#include "scan_common.cuh"

#include "internal.h"

#include <atomic>
#include <vector>

namespace {
thread_local std::string g_error;
thread_local int64_t g_rescans[2] = {0, 0};  // row and column lists the last exact l2sq scan rescanned
std::atomic<unsigned long long> g_launches{0};

// Per-thread event timing of the kernels of the last call.
struct Timing {
    bool on = false;
    std::vector<cudaEvent_t> events;
    int used = 0;
    std::vector<double> last_ms;
};
thread_local Timing g_timing;

int fail(int code, const std::string& msg) {
    g_error = msg;
    return code;
}

// Called after the call's stream has been synchronised: turn the marks into
// per-interval device times (marks are placed in pairs around kernels).
void collect_timing() {
    Timing& t = g_timing;
    if (t.used == 0) return;  // a call without timed kernels keeps the previous times
    t.last_ms.clear();
    for (int i = 0; i + 1 < t.used; i += 2) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, t.events[i], t.events[i + 1]);
        t.last_ms.push_back(ms);
    }
    t.used = 0;
}
// Synchronise the stream, then map the scan's device status word.
int finish(cudaStream_t st, const int* status_dev, const char* what) {
    int status = 0;
    if (status_dev) {
        cudaError_t e = cudaMemcpyAsync(&status, status_dev, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) return fail(HB_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    }
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(HB_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    collect_timing();
    if (status & hb::kErrWaitTimeout) return fail(HB_DEVICE_TIMEOUT, std::string(what) + ": a device-side wait timed out");
    if (status & hb::kErrBadInput) return fail(HB_BAD_INPUT, std::string(what) + ": index out of range");
    g_error.clear();
    return HB_OK;
}

bool valid_k(int k) { return k >= 0 && k <= 32; }

}  // namespace

namespace hb {
int abi_fail(int code, const std::string& msg) { return fail(code, msg); }
int abi_finish(cudaStream_t st, const char* what) { return finish(st, nullptr, what); }
void count_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }
void timing_mark(cudaStream_t st) {
    Timing& t = g_timing;
    if (!t.on) return;
    if (t.used == (int)t.events.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return;
        t.events.push_back(e);
    }
    cudaEventRecord(t.events[t.used++], st);
}
}  // namespace hb

extern "C" {

int hb_abi_version(void) { return HB_ABI_VERSION; }

const char* hb_last_error(void) { return g_error.c_str(); }

unsigned long long hb_kernel_launch_count(void) { return g_launches.load(); }

void hb_set_kernel_timing(int enable) {
    g_timing.on = enable != 0;
    g_timing.used = 0;
}

int hb_last_kernel_times(double* ms, int capacity) {
    const int n = (int)g_timing.last_ms.size();
    for (int i = 0; i < n && i < capacity; ++i) ms[i] = g_timing.last_ms[i];
    return n;
}

}  // extern "C"

// hb_perturbation -> the kernels' parameters; false (with the message set) when invalid.
static bool make_perturb(const hb_perturbation* in, hb::Perturb* out, bool pairs) {
    *out = hb::Perturb{};
    if (!in || in->sigma == 0.0) return true;
    if (!std::isfinite(in->sigma) || in->sigma < 0.0 || (in->mode != 0 && in->mode != 1)) {
        fail(HB_BAD_ARGUMENT, "perturbation: sigma must be finite and >= 0, mode 0 (rank2) or 1 (index_hash)");
        return false;
    }
    if (!in->query_index || !in->database_index) {
        fail(HB_BAD_ARGUMENT, "perturbation: global indices are required when sigma > 0");
        return false;
    }
    if (pairs && !in->row_is_source) {
        fail(HB_BAD_ARGUMENT, "perturbation: pair costs take source rows (row_is_source = 1)");
        return false;
    }
    out->sigma = in->sigma;
    out->seed_term = (float)((double)in->seed * 0.001);
    out->mode = in->mode;
    out->row_is_source = in->row_is_source != 0;
    const int64_t* c = in->coefficients;
    out->a0 = (float)c[0]; out->b0 = (float)c[1]; out->o0 = (float)c[2];
    out->a1 = (float)c[3]; out->b1 = (float)c[4]; out->o1 = (float)c[5];
    out->row_index = in->query_index;
    out->col_index = in->database_index;
    return true;
}

extern "C" {

size_t hb_l2sq_scan_workspace(int64_t q, int64_t n, int64_t d, int k, int precision, int min_groups) {
    if (q < 1 || n < 1 || d < 1 || !valid_k(k)) return 0;
    return hb::l2sq_bytes(q, n, d, k, precision, min_groups);
}

int hb_l2sq_scan(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* x_cost,
                 const double* y_cost, const double* x_bias, const double* y_bias, int k, double dot_scale,
                 int compute_stats, int precision, int min_groups, double* row_vals, int32_t* row_idx,
                 double* col_vals, int32_t* col_idx, double* stats5, void* workspace, size_t workspace_bytes,
                 void* stream) {
    if (!x || !y || !x_cost || !y_cost || !x_bias || !y_bias || !workspace)
        return fail(HB_BAD_ARGUMENT, "null input or workspace pointer");
    if (q < 1 || n < 1 || d < 1 || q >= INT32_MAX || n >= INT32_MAX || d >= INT32_MAX)
        return fail(HB_BAD_ARGUMENT, "q, n, d must be in [1, 2^31)");
    if (!valid_k(k)) return fail(HB_BAD_ARGUMENT, "k must be in 0..32");
    if (dot_scale != 1.0 && dot_scale != 2.0) return fail(HB_BAD_ARGUMENT, "dot_scale must be exactly 1 or 2");
    {
        const int base =
            precision & ~(HB_L2SQ_TWO_PASS | HB_L2SQ_ONE_PASS | HB_L2SQ_CTA_PAIRS | HB_L2SQ_SINGLE_CTA | HB_L2SQ_EXACT);
        if (base != 1 && base != 3)
            return fail(HB_BAD_ARGUMENT, "precision must be 1 (tf32) or 3 (fp32-class split), optionally | a pass flag");
        if ((precision & HB_L2SQ_TWO_PASS) && (precision & HB_L2SQ_ONE_PASS))
            return fail(HB_BAD_ARGUMENT, "HB_L2SQ_ONE_PASS and HB_L2SQ_TWO_PASS are exclusive");
        if ((precision & HB_L2SQ_CTA_PAIRS) && (precision & HB_L2SQ_SINGLE_CTA))
            return fail(HB_BAD_ARGUMENT, "HB_L2SQ_CTA_PAIRS and HB_L2SQ_SINGLE_CTA are exclusive");
        if ((precision & HB_L2SQ_ONE_PASS) && (k < 1 || k > 8))
            return fail(HB_BAD_ARGUMENT, "a one-pass scan needs 1 <= k <= 8");
    }
    if (k > 0 && (!row_vals || !row_idx || !col_vals || !col_idx)) return fail(HB_BAD_ARGUMENT, "null output pointer");
    if (compute_stats && !stats5) return fail(HB_BAD_ARGUMENT, "null stats pointer");
    if (workspace_bytes < hb::l2sq_bytes(q, n, d, k, precision, min_groups))
        return fail(HB_WORKSPACE, "workspace smaller than hb_l2sq_scan_workspace()");
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(HB_BAD_ARGUMENT, "workspace must be 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::string err;
    int status_host = 0;
    int rescans[2] = {0, 0};
    int rc = hb::l2sq_scan(x, y, q, n, d, x_cost, y_cost, x_bias, y_bias, k, dot_scale, compute_stats, precision,
                           min_groups, row_vals, row_idx, col_vals, col_idx, stats5, workspace, workspace_bytes,
                           &status_host, st, err, rescans);
    if (rc) return fail(rc == 3 ? HB_WORKSPACE : rc == 5 ? HB_TENSOR_MAP : HB_LAUNCH, err);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(HB_CUDA, std::string("l2sq scan: ") + cudaGetErrorString(e));
    collect_timing();
    if (status_host & hb::kErrWaitTimeout) return fail(HB_DEVICE_TIMEOUT, "l2sq scan: a device-side wait timed out");
    if (status_host & hb::kErrBadInput)
        return fail(HB_BAD_INPUT, "l2sq scan: a feature magnitude of 2^75 or more (or a non-finite one)");
    g_rescans[0] = rescans[0];
    g_rescans[1] = rescans[1];
    g_error.clear();
    return HB_OK;
}

int hb_l2sq_last_rescans(int64_t* out2) {
    if (!out2) return fail(HB_BAD_ARGUMENT, "null output pointer");
    out2[0] = g_rescans[0];
    out2[1] = g_rescans[1];
    return HB_OK;
}

size_t hb_norm_scan_workspace(int64_t q, int64_t n, int k) {
    if (q < 1 || n < 1 || !valid_k(k)) return 0;
    return hb::norm_bytes(q, n, k);
}

int hb_norm_scan(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* f, const double* g,
                 int cost_type, int k, int compute_stats, double* row_vals, int32_t* row_idx, double* col_vals,
                 int32_t* col_idx, double* stats5, void* workspace, size_t workspace_bytes, void* stream) {
    return hb_norm_scan_ex(x, y, q, n, d, f, g, cost_type, k, compute_stats, row_vals, row_idx, col_vals, col_idx,
                           stats5, workspace, workspace_bytes, stream, nullptr);
}

int hb_norm_scan_ex(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* f, const double* g,
                    int cost_type, int k, int compute_stats, double* row_vals, int32_t* row_idx, double* col_vals,
                    int32_t* col_idx, double* stats5, void* workspace, size_t workspace_bytes, void* stream,
                    const hb_perturbation* perturbation) {
    hb::Perturb pert;
    if (!make_perturb(perturbation, &pert, false)) return HB_BAD_ARGUMENT;
    if (!x || !y || !f || !g || !workspace) return fail(HB_BAD_ARGUMENT, "null input or workspace pointer");
    if (q < 1 || n < 1 || d < 1 || q >= INT32_MAX || n >= INT32_MAX || d >= INT32_MAX)
        return fail(HB_BAD_ARGUMENT, "q, n, d must be in [1, 2^31)");
    if ((cost_type & ~HB_NORM_TWO_PASS) < 0 || (cost_type & ~HB_NORM_TWO_PASS) > 2)
        return fail(HB_BAD_ARGUMENT, "cost_type must be 0 (l1), 1 (linf) or 2 (l2), optionally | HB_NORM_TWO_PASS");
    if (!valid_k(k)) return fail(HB_BAD_ARGUMENT, "k must be in 0..32");
    if (k > 0 && (!row_vals || !row_idx || !col_vals || !col_idx)) return fail(HB_BAD_ARGUMENT, "null output pointer");
    if (compute_stats && !stats5) return fail(HB_BAD_ARGUMENT, "null stats pointer");
    if (workspace_bytes < hb::norm_bytes(q, n, k)) return fail(HB_WORKSPACE, "workspace smaller than hb_norm_scan_workspace()");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::string err;
    int rc = hb::norm_scan(x, y, q, n, d, f, g, cost_type, k, compute_stats, row_vals, row_idx, col_vals, col_idx,
                           stats5, workspace, workspace_bytes, st, err, false, &pert);
    if (rc) return fail(rc == 3 ? HB_WORKSPACE : HB_LAUNCH, err);
    return finish(st, nullptr, "norm scan");
}

size_t hb_l2sq_topk_workspace(int64_t q, int64_t n, int64_t d, int k, int precision) {
    if (q < 1 || n < 1 || d < 1 || k < 1 || k > 32) return 0;
    return hb::l2sq_bytes(q, n, d, k, (precision & 0xF) | hb::L2SQ_ROWS_ONLY, 0);
}

int hb_l2sq_topk(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* x_bias,
                 const double* y_bias, int k, double dot_scale, int precision, double* row_vals, int32_t* row_idx,
                 void* workspace, size_t workspace_bytes, void* stream) {
    if (!x || !y || !x_bias || !y_bias || !workspace) return fail(HB_BAD_ARGUMENT, "null input or workspace pointer");
    if (!row_vals || !row_idx) return fail(HB_BAD_ARGUMENT, "null output pointer");
    if (q < 1 || n < 1 || d < 1 || q >= INT32_MAX || n >= INT32_MAX || d >= INT32_MAX)
        return fail(HB_BAD_ARGUMENT, "q, n, d must be in [1, 2^31)");
    if (k < 1 || k > 32) return fail(HB_BAD_ARGUMENT, "k must be in 1..32");
    if (dot_scale != 1.0 && dot_scale != 2.0) return fail(HB_BAD_ARGUMENT, "dot_scale must be exactly 1 or 2");
    if (precision != 1 && precision != 3) return fail(HB_BAD_ARGUMENT, "precision must be 1 (tf32) or 3 (fp32-class split)");
    const int flags = precision | hb::L2SQ_ROWS_ONLY;
    if (workspace_bytes < hb::l2sq_bytes(q, n, d, k, flags, 0))
        return fail(HB_WORKSPACE, "workspace smaller than hb_l2sq_topk_workspace()");
    if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(HB_BAD_ARGUMENT, "workspace must be 256-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::string err;
    int status_host = 0;
    int rc = hb::l2sq_scan(x, y, q, n, d, nullptr, nullptr, x_bias, y_bias, k, dot_scale, 0, flags, 0, row_vals,
                           row_idx, nullptr, nullptr, nullptr, workspace, workspace_bytes, &status_host, st, err);
    if (rc) return fail(rc == 3 ? HB_WORKSPACE : rc == 5 ? HB_TENSOR_MAP : HB_LAUNCH, err);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(HB_CUDA, std::string("l2sq top-k: ") + cudaGetErrorString(e));
    collect_timing();
    if (status_host & hb::kErrWaitTimeout) return fail(HB_DEVICE_TIMEOUT, "l2sq top-k: a device-side wait timed out");
    if (status_host & hb::kErrBadInput)
        return fail(HB_BAD_INPUT, "l2sq top-k: a feature magnitude of 2^75 or more (or a non-finite one)");
    g_error.clear();
    return HB_OK;
}

// The norm top-k workspace is the norm scan's plus 64 bytes for the five certificate slots.
size_t hb_norm_topk_workspace(int64_t q, int64_t n, int k) {
    if (q < 1 || n < 1 || k < 1 || k > 32) return 0;
    return ((hb::norm_bytes(q, n, k) + 7) & ~size_t(7)) + 64;
}

int hb_norm_topk(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* g, int cost_type,
                 int k, int compute_stats, double* row_vals, int32_t* row_idx, double* stats2, void* workspace,
                 size_t workspace_bytes, void* stream) {
    return hb_norm_topk_ex(x, y, q, n, d, g, cost_type, k, compute_stats, row_vals, row_idx, stats2, workspace,
                           workspace_bytes, stream, nullptr);
}

int hb_norm_topk_ex(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* g, int cost_type,
                    int k, int compute_stats, double* row_vals, int32_t* row_idx, double* stats2, void* workspace,
                    size_t workspace_bytes, void* stream, const hb_perturbation* perturbation) {
    hb::Perturb pert;
    if (!make_perturb(perturbation, &pert, false)) return HB_BAD_ARGUMENT;
    if (!x || !y || !g || !workspace) return fail(HB_BAD_ARGUMENT, "null input or workspace pointer");
    if (!row_vals || !row_idx) return fail(HB_BAD_ARGUMENT, "null output pointer");
    if (q < 1 || n < 1 || d < 1 || q >= INT32_MAX || n >= INT32_MAX || d >= INT32_MAX)
        return fail(HB_BAD_ARGUMENT, "q, n, d must be in [1, 2^31)");
    if (cost_type < 0 || cost_type > 2) return fail(HB_BAD_ARGUMENT, "cost_type must be 0 (l1), 1 (linf) or 2 (l2)");
    if (k < 1 || k > 32) return fail(HB_BAD_ARGUMENT, "k must be in 1..32");
    if (compute_stats && !stats2) return fail(HB_BAD_ARGUMENT, "null stats pointer");
    if (workspace_bytes < hb_norm_topk_workspace(q, n, k))
        return fail(HB_WORKSPACE, "workspace smaller than hb_norm_topk_workspace()");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::string err;
    // the five certificate slots sit after the scan's scratch; [1] and [3] are the cost terms
    double* stats5 = compute_stats ? reinterpret_cast<double*>(static_cast<char*>(workspace) +
                                                              ((hb::norm_bytes(q, n, k) + 7) & ~size_t(7)))
                                   : nullptr;
    int rc = hb::norm_scan(x, y, q, n, d, nullptr, g, cost_type, k, compute_stats, row_vals, row_idx, nullptr, nullptr,
                           stats5, workspace, workspace_bytes, st, err, true, &pert);
    if (rc) return fail(rc == 3 ? HB_WORKSPACE : HB_LAUNCH, err);
    if (compute_stats) {
        cudaError_t e = cudaMemcpyAsync(stats2, stats5 + 1, sizeof(double), cudaMemcpyDeviceToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(stats2 + 1, stats5 + 3, sizeof(double), cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return fail(HB_CUDA, std::string("norm top-k: ") + cudaGetErrorString(e));
    }
    return finish(st, nullptr, "norm top-k");
}

int hb_merge_topk(const double* vals, const int32_t* idx, int parts, int64_t rows, int width, int k,
                  double* out_vals, int32_t* out_idx, void* stream) {
    if (!vals || !idx || !out_vals || !out_idx) return fail(HB_BAD_ARGUMENT, "null pointer");
    if (parts < 1 || rows < 0 || width < 1 || width > 32 || k < 1 || k > 32)
        return fail(HB_BAD_ARGUMENT, "merge needs parts >= 1, 1 <= width, k <= 32");
    if (rows == 0) { g_error.clear(); return HB_OK; }
    const int K = hb::bucket_of(width > k ? width : k);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = hb::merge_lists(K, vals, idx, parts, rows, width, k, out_vals, out_idx, st);
    if (e != cudaSuccess) return fail(HB_LAUNCH, std::string("merge: ") + cudaGetErrorString(e));
    return finish(st, nullptr, "merge");
}

size_t hb_pair_costs_workspace(void) { return 256; }

int hb_pair_costs(int cost_type, const float* x, const float* y, int64_t nx, int64_t ny, int64_t d,
                  const double* a, const double* b, double dot_scale, const int64_t* rows, const int64_t* cols,
                  int64_t count, double* out, void* workspace, size_t workspace_bytes, void* stream) {
    return hb_pair_costs_ex(cost_type, x, y, nx, ny, d, a, b, dot_scale, rows, cols, count, out, workspace,
                            workspace_bytes, stream, nullptr);
}

int hb_pair_costs_ex(int cost_type, const float* x, const float* y, int64_t nx, int64_t ny, int64_t d,
                     const double* a, const double* b, double dot_scale, const int64_t* rows, const int64_t* cols,
                     int64_t count, double* out, void* workspace, size_t workspace_bytes, void* stream,
                     const hb_perturbation* perturbation) {
    hb::Perturb pert;
    if (!make_perturb(perturbation, &pert, true)) return HB_BAD_ARGUMENT;
    if (cost_type < 0 || cost_type > 3) return fail(HB_BAD_ARGUMENT, "cost_type must be 0..3");
    if (count < 0 || d < 1 || d >= INT32_MAX || nx < 1 || ny < 1) return fail(HB_BAD_ARGUMENT, "invalid sizes");
    if (count == 0) { g_error.clear(); return HB_OK; }
    if (!x || !y || !rows || !cols || !out || !workspace) return fail(HB_BAD_ARGUMENT, "null pointer");
    if (cost_type == 3 && (!a || !b)) return fail(HB_BAD_ARGUMENT, "bilinear pair costs need a and b");
    if (cost_type == 3 && dot_scale != 1.0 && dot_scale != 2.0)
        return fail(HB_BAD_ARGUMENT, "dot_scale must be exactly 1 or 2");
    if (workspace_bytes < hb_pair_costs_workspace()) return fail(HB_WORKSPACE, "workspace smaller than 256 bytes");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* status = static_cast<int*>(workspace);
    cudaMemsetAsync(status, 0, sizeof(int), st);
    std::string err;
    int rc = hb::pair_costs(cost_type, x, y, nx, ny, d, a, b, dot_scale, rows, cols, count, out, status, st, err,
                            &pert);
    if (rc) return fail(rc == 2 ? HB_BAD_ARGUMENT : HB_LAUNCH, err);
    return finish(st, status, "pair costs");
}

size_t hb_restricted_ot_workspace(int64_t n, int64_t m, int64_t e) {
    if (n < 1 || m < 1 || e < 1) return 0;
    return hb::pdlp_bytes(n, m, e);
}

int hb_restricted_ot_solve(const int64_t* rows, const int64_t* cols, const double* costs, int64_t e,
                           const double* masses, int64_t n, int64_t m, const double* x0, const double* y0,
                           const hb_pdlp_controls* controls, double* x_out, double* y_out, hb_pdlp_info* info,
                           hb_pdlp_trace_row* trace, int32_t trace_capacity, int32_t* trace_length,
                           void* workspace, size_t workspace_bytes, void* stream) {
    if (!rows || !cols || !costs || !masses || !controls || !x_out || !y_out || !info || !workspace)
        return fail(HB_BAD_ARGUMENT, "null pointer");
    if (workspace_bytes < hb::pdlp_bytes(n, m, e))
        return fail(HB_WORKSPACE, "workspace smaller than hb_restricted_ot_workspace()");
    hb::PdlpControls ctl;
    ctl.frequency = controls->evaluation_frequency;
    ctl.time_limit = controls->time_limit_seconds;
    ctl.iteration_limit = controls->iteration_limit;
    ctl.tol_objective = controls->tol_objective;
    ctl.tol_primal = controls->tol_primal;
    ctl.tol_dual = controls->tol_dual;
    ctl.rescale = controls->scalar_rescaling;
    ctl.weight0 = controls->initial_primal_weight;
    if (controls->atomic_sums < HB_PDLP_SUMS_ORDERED || controls->atomic_sums > HB_PDLP_SUMS_TREE)
        return fail(HB_BAD_ARGUMENT, "atomic_sums must be one of HB_PDLP_SUMS_ORDERED, _ATOMIC, _TREE");
    ctl.atomic = controls->atomic_sums == HB_PDLP_SUMS_ATOMIC;
    ctl.tree = controls->atomic_sums == HB_PDLP_SUMS_TREE;
    if (controls->termination_norm != HB_PDLP_NORM_L2 && controls->termination_norm != HB_PDLP_NORM_LINF)
        return fail(HB_BAD_ARGUMENT, "termination_norm must be HB_PDLP_NORM_L2 or HB_PDLP_NORM_LINF");
    ctl.linf = controls->termination_norm == HB_PDLP_NORM_LINF;
    hb::PdlpResult r{};
    static_assert(sizeof(hb::TraceRow) == sizeof(hb_pdlp_trace_row), "trace row layout");
    int tlen = 0;
    std::string err;
    int rc = hb::pdlp_solve(rows, cols, costs, e, masses, n, m, x0, y0, ctl, x_out, y_out, &r,
                            reinterpret_cast<hb::TraceRow*>(trace), trace ? trace_capacity : 0, &tlen, workspace,
                            workspace_bytes, static_cast<cudaStream_t>(stream), err);
    if (rc) return fail(rc == 2 ? HB_BAD_INPUT : rc == 3 ? HB_WORKSPACE : HB_CUDA, err);
    collect_timing();  // the solve synchronised its stream before returning
    info->iterations = r.iterations;
    info->restarts = r.restarts;
    info->termination = r.reason;
    info->pad = 0;
    info->primal_objective = r.pobj;
    info->dual_objective = r.dobj;
    info->abs_primal_residual = r.ap;
    info->rel_primal_residual = r.rp;
    info->abs_dual_residual = r.ad;
    info->rel_dual_residual = r.rd;
    info->rel_gap = r.gap;
    info->primal_weight = r.weight;
    info->cost_norm = r.cost_norm;
    info->mass_norm = r.mass_norm;
    info->setup_seconds = r.setup_seconds;
    info->iteration_seconds = r.iteration_seconds;
    info->l2_abs_primal_residual = r.ap2;
    info->l2_rel_primal_residual = r.rp2;
    info->l2_abs_dual_residual = r.ad2;
    info->l2_rel_dual_residual = r.rd2;
    if (trace_length) *trace_length = tlen;
    g_error.clear();
    return HB_OK;
}

}  // extern "C"
