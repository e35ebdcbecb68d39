// Active-support maintenance: the new candidate pairs of a scan that are not
// already in the support (sorted, unique), on the GPU.
//
// Replaces ActiveSupport.filter_new_candidate_pairs
// (src/hello_ot/restricted_ot/active_support.py:483-506): candidate keys
// row * n_target + col are sorted and made unique, and a key is new when a
// binary search does not find it among the sorted support keys.  Integer work,
// HBM- and sort-bound: CUB radix sorts (only the key bits that can be set),
// one flag pass, one compaction.
//
// Budgeted pruning: the removal positions of DualGapCleaning in protect-new
// mode (src/hello_ot/refinement/budgeted_pruning.py:27-57, 119-175, with the
// reduced costs of ActiveSupport.pruning_values, active_support.py:401-421):
// among old (not created this iteration, not structural) zero-flow edges, the
// num_to_remove with the largest reduced cost c - u_row - v_col, ties by
// position (stable), non-finite reduced costs counting as -inf.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_select.cuh>

#include <string>

#include "../../include/hello_b200.h"
#include "internal.h"
#include "scan_common.cuh"

namespace hb {
namespace support {

__global__ void make_keys(const int32_t* __restrict__ rows, const int32_t* __restrict__ cols, int64_t count,
                          int64_t n_target, int64_t n_source, int64_t* __restrict__ keys, int* status) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
        const int64_t r = rows[i], c = cols[i];
        if (r < 0 || r >= n_source || c < 0 || c >= n_target) {
            atomicOr(status, 1);
            keys[i] = 0;
        } else {
            keys[i] = r * n_target + c;
        }
    }
}

// keep[i]: first of its run of equal sorted keys and absent from the sorted support
__global__ void flag_new(const int64_t* __restrict__ keys, int64_t count, const int64_t* __restrict__ active,
                         int64_t n_active, unsigned char* __restrict__ keep) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
        const int64_t k = keys[i];
        bool fresh = i == 0 || keys[i - 1] != k;
        if (fresh && n_active > 0) {
            int64_t lo = 0, hi = n_active;  // first active key >= k
            while (lo < hi) {
                const int64_t mid = (lo + hi) >> 1;
                if (active[mid] < k) lo = mid + 1; else hi = mid;
            }
            fresh = !(lo < n_active && active[lo] == k);
        }
        keep[i] = fresh ? 1 : 0;
    }
}

__global__ void split_keys(const int64_t* __restrict__ keys, const int64_t* __restrict__ count, int64_t n_target,
                           int32_t* __restrict__ rows, int32_t* __restrict__ cols) {
    const int64_t n = *count, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t k = keys[i];
        rows[i] = (int32_t)(k / n_target);
        cols[i] = (int32_t)(k % n_target);
    }
}

constexpr double POSITIVE_SUPPORT_TOLERANCE = 1e-15;  // support_budget.py:7

// removable[i] = old, not structural, zero flow; rc[i] = its reduced cost (canonical zero)
__global__ void prune_values(const int32_t* __restrict__ rows, const int32_t* __restrict__ cols,
                             const double* __restrict__ costs, const double* __restrict__ x,
                             const int32_t* __restrict__ created, int64_t e, const double* __restrict__ duals,
                             int n_source, int n_target, int current_iter, unsigned char* __restrict__ removable,
                             double* __restrict__ rc, int* status) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e; i += stride) {
        const int r = rows[i], c = cols[i];
        if (r < 0 || r >= n_source || c < 0 || c >= n_target) {
            atomicOr(status, 1);
            removable[i] = 0;
            continue;
        }
        double v = costs[i] - (duals[r] + duals[n_source + c]);
        v = isfinite(v) ? v + 0.0 : -INFINITY;  // + 0.0 turns -0.0 into +0.0: equal keys sort by position
        rc[i] = v;
        const int it = created[i];
        removable[i] = (it != current_iter && it != -1 && !(fabs(x[i]) > POSITIVE_SUPPORT_TOLERANCE)) ? 1 : 0;
    }
}

__global__ void iota32(int32_t* v, int64_t e) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x)
        v[i] = (int32_t)i;
}

__global__ void gather_keys(const int32_t* __restrict__ idx, const int64_t* __restrict__ count,
                            const double* __restrict__ rc, double* __restrict__ keys) {
    const int64_t n = *count;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        keys[i] = rc[idx[i]];
}

int key_bits(int64_t max_key) {
    int b = 1;
    while (b < 63 && (int64_t(1) << b) <= max_key) ++b;
    return b;
}

}  // namespace support

struct SupportLayout {
    int64_t *ckeys = nullptr, *csorted = nullptr, *asorted = nullptr, *newkeys = nullptr, *count = nullptr;
    unsigned char* keep = nullptr;
    void* cub = nullptr;
    size_t cub_bytes = 0, bytes = 0;
    int* status = nullptr;
    bool ok = true;
};

SupportLayout support_layout(void* base, size_t size, int64_t n_active, int64_t n_cand) {
    SupportLayout L;
    Arena ar{static_cast<char*>(base), size, 0};
    auto chk = [&](const void* p) { if (base && !p) L.ok = false; };
    L.ckeys = ar.take<int64_t>(n_cand > 0 ? n_cand : 1); chk(L.ckeys);
    L.csorted = ar.take<int64_t>(n_cand > 0 ? n_cand : 1); chk(L.csorted);
    L.asorted = ar.take<int64_t>(n_active > 0 ? n_active : 1); chk(L.asorted);
    L.newkeys = ar.take<int64_t>(n_cand > 0 ? n_cand : 1); chk(L.newkeys);
    L.keep = ar.take<unsigned char>(n_cand > 0 ? n_cand : 1); chk(L.keep);
    L.count = ar.take<int64_t>(1); chk(L.count);
    L.status = ar.take<int>(1); chk(L.status);
    size_t a = 0, b = 0, c = 0;
    const int64_t big = n_cand > n_active ? n_cand : n_active;
    cub::DeviceRadixSort::SortKeys(nullptr, a, (const int64_t*)nullptr, (int64_t*)nullptr, (int64_t)(big > 0 ? big : 1));
    cub::DeviceSelect::Flagged(nullptr, b, (const int64_t*)nullptr, (const unsigned char*)nullptr, (int64_t*)nullptr,
                               (int64_t*)nullptr, (int64_t)(n_cand > 0 ? n_cand : 1));
    c = a > b ? a : b;
    L.cub_bytes = c;
    L.cub = ar.take<char>(c > 0 ? c : 1); chk(L.cub);
    L.bytes = ar.used + 256;
    return L;
}

size_t support_bytes(int64_t n_active, int64_t n_cand) { return support_layout(nullptr, 0, n_active, n_cand).bytes; }

struct PruneLayout {
    unsigned char* removable = nullptr;
    double *rc = nullptr, *keys = nullptr, *keys_sorted = nullptr;
    int32_t *iota = nullptr, *idx = nullptr, *idx_sorted = nullptr;
    int64_t* count = nullptr;
    int* status = nullptr;
    void* cub = nullptr;
    size_t cub_bytes = 0, bytes = 0;
    bool ok = true;
};

PruneLayout prune_layout(void* base, size_t size, int64_t e) {
    PruneLayout L;
    Arena ar{static_cast<char*>(base), size, 0};
    auto chk = [&](const void* p) { if (base && !p) L.ok = false; };
    const int64_t n = e > 0 ? e : 1;
    L.removable = ar.take<unsigned char>(n); chk(L.removable);
    L.rc = ar.take<double>(n); chk(L.rc);
    L.keys = ar.take<double>(n); chk(L.keys);
    L.keys_sorted = ar.take<double>(n); chk(L.keys_sorted);
    L.iota = ar.take<int32_t>(n); chk(L.iota);
    L.idx = ar.take<int32_t>(n); chk(L.idx);
    L.idx_sorted = ar.take<int32_t>(n); chk(L.idx_sorted);
    L.count = ar.take<int64_t>(1); chk(L.count);
    L.status = ar.take<int>(1); chk(L.status);
    size_t a = 0, b = 0;
    cub::DeviceSelect::Flagged(nullptr, a, (const int32_t*)nullptr, (const unsigned char*)nullptr, (int32_t*)nullptr,
                               (int64_t*)nullptr, (int64_t)n);
    cub::DeviceRadixSort::SortPairsDescending(nullptr, b, (const double*)nullptr, (double*)nullptr,
                                              (const int32_t*)nullptr, (int32_t*)nullptr, (int64_t)n);
    L.cub_bytes = a > b ? a : b;
    L.cub = ar.take<char>(L.cub_bytes > 0 ? L.cub_bytes : 1); chk(L.cub);
    L.bytes = ar.used + 256;
    return L;
}

size_t prune_bytes(int64_t e) { return prune_layout(nullptr, 0, e).bytes; }

// Returns 0 with *removable_count and, when it is >= num_to_remove, the first
// num_to_remove positions in out (selection order); 2 = index out of range,
// 3 = workspace, 6 = CUDA.
int select_prune_positions(const int32_t* rows, const int32_t* cols, const double* costs, const double* x,
                           const int32_t* created, int64_t e, const double* duals, int64_t n_source, int64_t n_target,
                           int current_iter, int64_t num_to_remove, int32_t* out, int64_t* removable_count,
                           void* ws, size_t ws_bytes, cudaStream_t st, std::string& err) {
    *removable_count = 0;
    if (e == 0) return 0;
    PruneLayout L = prune_layout(ws, ws_bytes, e);
    if (!L.ok) { err = "workspace too small for the pruning selection"; return 3; }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int blocks = sms * 8;
    cudaError_t rc = cudaMemsetAsync(L.status, 0, sizeof(int), st);
    support::prune_values<<<blocks, 256, 0, st>>>(rows, cols, costs, x, created, e, duals, (int)n_source, (int)n_target,
                                                  current_iter, L.removable, L.rc, L.status);
    support::iota32<<<blocks, 256, 0, st>>>(L.iota, e);
    count_launches(2);
    size_t cb = L.cub_bytes;
    if (rc == cudaSuccess) rc = cub::DeviceSelect::Flagged(L.cub, cb, L.iota, L.removable, L.idx, L.count, e, st);
    count_launches(1);
    int64_t nrem = 0;
    int status = 0;
    if (rc == cudaSuccess) rc = cudaMemcpyAsync(&nrem, L.count, sizeof(int64_t), cudaMemcpyDeviceToHost, st);
    if (rc == cudaSuccess) rc = cudaMemcpyAsync(&status, L.status, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (rc == cudaSuccess) rc = cudaStreamSynchronize(st);
    if (rc != cudaSuccess) { err = std::string("pruning selection: ") + cudaGetErrorString(rc); return 6; }
    if (status) { err = "support row or column outside the dual vector"; return 2; }
    *removable_count = nrem;
    if (nrem < num_to_remove || num_to_remove <= 0) return 0;
    support::gather_keys<<<blocks, 256, 0, st>>>(L.idx, L.count, L.rc, L.keys);
    count_launches(1);
    cb = L.cub_bytes;  // stable: equal reduced costs keep their (ascending) positions
    rc = cub::DeviceRadixSort::SortPairsDescending(L.cub, cb, L.keys, L.keys_sorted, L.idx, L.idx_sorted, nrem, 0, 64, st);
    count_launches(1);
    if (rc == cudaSuccess)
        rc = cudaMemcpyAsync(out, L.idx_sorted, sizeof(int32_t) * num_to_remove, cudaMemcpyDeviceToDevice, st);
    if (rc != cudaSuccess) { err = std::string("pruning selection: ") + cudaGetErrorString(rc); return 6; }
    return 0;
}

// Returns 0 and *new_count; 2 = an index out of range (status), 3 = workspace, 6 = CUDA.
int filter_new_pairs(const int64_t* active_keys, int64_t n_active, int active_sorted, const int32_t* rows,
                     const int32_t* cols, int64_t n_cand, int64_t n_source, int64_t n_target, int32_t* new_rows,
                     int32_t* new_cols, int64_t* new_count, void* ws, size_t ws_bytes, cudaStream_t st,
                     std::string& err) {
    *new_count = 0;
    if (n_cand == 0) return 0;
    SupportLayout L = support_layout(ws, ws_bytes, n_active, n_cand);
    if (!L.ok) { err = "workspace too small for the support filter"; return 3; }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int blocks = sms * 8;
    const int bits = support::key_bits(n_source * n_target - 1);
    cudaError_t e = cudaMemsetAsync(L.status, 0, sizeof(int), st);
    support::make_keys<<<blocks, 256, 0, st>>>(rows, cols, n_cand, n_target, n_source, L.ckeys, L.status);
    count_launches(1);
    size_t cb = L.cub_bytes;
    if (e == cudaSuccess)
        e = cub::DeviceRadixSort::SortKeys(L.cub, cb, L.ckeys, L.csorted, n_cand, 0, bits, st);
    const int64_t* active = active_keys;
    if (e == cudaSuccess && n_active > 0 && !active_sorted) {
        cb = L.cub_bytes;
        e = cub::DeviceRadixSort::SortKeys(L.cub, cb, active_keys, L.asorted, n_active, 0, bits, st);
        active = L.asorted;
    }
    count_launches(active_sorted ? 1 : 2);
    if (e != cudaSuccess) { err = std::string("support sort: ") + cudaGetErrorString(e); return 6; }
    support::flag_new<<<blocks, 256, 0, st>>>(L.csorted, n_cand, active, n_active, L.keep);
    count_launches(1);
    cb = L.cub_bytes;
    e = cub::DeviceSelect::Flagged(L.cub, cb, L.csorted, L.keep, L.newkeys, L.count, n_cand, st);
    count_launches(1);
    if (e != cudaSuccess) { err = std::string("support select: ") + cudaGetErrorString(e); return 6; }
    support::split_keys<<<blocks, 256, 0, st>>>(L.newkeys, L.count, n_target, new_rows, new_cols);
    count_launches(1);
    int status = 0;
    e = cudaMemcpyAsync(new_count, L.count, sizeof(int64_t), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&status, L.status, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { err = std::string("support filter: ") + cudaGetErrorString(e); return 6; }
    if (status) { err = "candidate row or column out of range"; return 2; }
    return 0;
}

}  // namespace hb

extern "C" size_t hb_prune_select_workspace(int64_t n_edges) {
    if (n_edges < 0) return 0;
    return hb::prune_bytes(n_edges);
}

extern "C" int hb_prune_select(const int32_t* rows, const int32_t* cols, const double* costs, const double* x_prev,
                               const int32_t* creation_iteration, int64_t n_edges, const double* duals,
                               int64_t n_source, int64_t n_target, int32_t current_inner_iter, int64_t num_to_remove,
                               int32_t* positions, int64_t* removable_count, void* workspace, size_t workspace_bytes,
                               void* stream) {
    if (!removable_count || (n_edges > 0 && (!rows || !cols || !costs || !x_prev || !creation_iteration || !duals ||
                                             !workspace)) || (num_to_remove > 0 && !positions))
        return hb::abi_fail(HB_BAD_ARGUMENT, "null pointer");
    if (n_edges < 0 || n_edges > INT32_MAX || n_source < 1 || n_target < 1 || n_source + n_target > INT32_MAX ||
        num_to_remove < 0)
        return hb::abi_fail(HB_BAD_ARGUMENT, "sizes out of range");
    if (workspace_bytes < hb::prune_bytes(n_edges))
        return hb::abi_fail(HB_WORKSPACE, "workspace smaller than hb_prune_select_workspace()");
    std::string err;
    int rc = hb::select_prune_positions(rows, cols, costs, x_prev, creation_iteration, n_edges, duals, n_source,
                                        n_target, current_inner_iter, num_to_remove, positions, removable_count,
                                        workspace, workspace_bytes, static_cast<cudaStream_t>(stream), err);
    if (rc) return hb::abi_fail(rc == 2 ? HB_BAD_INPUT : rc == 3 ? HB_WORKSPACE : HB_CUDA, err);
    return hb::abi_finish(static_cast<cudaStream_t>(stream), "pruning selection");
}

extern "C" size_t hb_filter_new_pairs_workspace(int64_t n_active, int64_t n_candidates) {
    if (n_active < 0 || n_candidates < 0) return 0;
    return hb::support_bytes(n_active, n_candidates);
}

extern "C" int hb_filter_new_pairs(const int64_t* active_keys, int64_t n_active, int32_t active_sorted,
                                   const int32_t* rows, const int32_t* cols, int64_t n_candidates, int64_t n_source,
                                   int64_t n_target, int32_t* new_rows, int32_t* new_cols, int64_t* new_count,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    if (!new_count || (n_active > 0 && !active_keys) ||
        (n_candidates > 0 && (!rows || !cols || !new_rows || !new_cols || !workspace)))
        return hb::abi_fail(HB_BAD_ARGUMENT, "null pointer");
    if (n_active < 0 || n_candidates < 0 || n_source < 1 || n_target < 1 || n_source > INT32_MAX ||
        n_target > INT32_MAX)
        return hb::abi_fail(HB_BAD_ARGUMENT, "sizes out of range");
    if (workspace_bytes < hb::support_bytes(n_active, n_candidates))
        return hb::abi_fail(HB_WORKSPACE, "workspace smaller than hb_filter_new_pairs_workspace()");
    std::string err;
    int rc = hb::filter_new_pairs(active_keys, n_active, active_sorted, rows, cols, n_candidates, n_source, n_target,
                                  new_rows, new_cols, new_count, workspace, workspace_bytes,
                                  static_cast<cudaStream_t>(stream), err);
    if (rc) return hb::abi_fail(rc == 2 ? HB_BAD_INPUT : rc == 3 ? HB_WORKSPACE : HB_CUDA, err);
    return hb::abi_finish(static_cast<cudaStream_t>(stream), "support filter");
}
