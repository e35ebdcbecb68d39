// Pieces shared by the ℓ2² (tensor-core) and norm (CUDA-core) pricing scans:
// work decomposition, partial top-k merge, certificate finalisation and the
// workspace layout.
//
// A scan pass covers q query rows x n database columns.  Query rows are cut
// into row blocks, database columns into column tiles; a *unit* is one row
// block times one contiguous group of column tiles.  Each unit keeps the row
// top-k of its rows in registers while it sweeps its column group and writes
// one partial k-list per row; merge_partials reduces the C partial lists of a
// row in column-group order.  Column top-k comes from a second pass with the
// roles of the two clouds exchanged (see scan_plan()).
#pragma once
#include "common.cuh"

namespace hb {

struct ScanPlan {
    int rb;      // row blocks
    int ct;      // column tiles
    int groups;  // column groups (C)
    int tpg;     // column tiles per group
    int units;   // rb * groups
    int grid;    // CTAs launched (persistent)
};

// Column groups: enough units to fill the GPU and, for wide features, few
// enough distinct row blocks in flight that their feature slabs stay in L2.
inline ScanPlan scan_plan(int64_t q, int64_t n, int bm, int bn, int ctas_per_sm, int sms, int min_groups) {
    ScanPlan p{};
    p.rb = (int)((q + bm - 1) / bm);
    p.ct = (int)((n + bn - 1) / bn);
    const int slots = sms * ctas_per_sm;
    int groups = min_groups < 1 ? 1 : min_groups;
    while ((int64_t)p.rb * groups < 2 * slots && groups < p.ct) groups *= 2;
    if (groups > p.ct) groups = p.ct;
    p.tpg = (p.ct + groups - 1) / groups;
    p.groups = (p.ct + p.tpg - 1) / p.tpg;
    p.units = p.rb * p.groups;
    p.grid = p.units < slots ? p.units : slots;
    return p;
}

// Merge the `parts` partial lists of each row (rows x width per part, parts
// stored part-major, width <= K) into the first `k_out` entries of the final
// list.  Slots with index INT32_MAX or negative are empty; empty output slots
// come out as (-inf, -1).  Thread per row.  With `run_out`, also the row's
// runner-up: the largest score offered to any of its lists (pr: the partial
// lists' runner-ups, parts x rows) that is not among the k_out entries.
template <int K>
__global__ void merge_partials(const double* __restrict__ pv, const int* __restrict__ pi, int parts, int64_t rows,
                               int width, int k_out, double* __restrict__ out_v, int* __restrict__ out_i,
                               const double* __restrict__ pr, double* __restrict__ run_out) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    TopK<K> top;
    top.reset();
    double run = -INFINITY;
    for (int c = 0; c < parts; ++c) {
        const double* v = pv + ((int64_t)c * rows + r) * width;
        const int* ix = pi + ((int64_t)c * rows + r) * width;
        for (int s = 0; s < width; ++s) {
            const int id = ix[s];
            if (id != INT32_MAX && id >= 0) top.offer_track(v[s], id, run);
        }
        if (pr) run = fmax(run, pr[(int64_t)c * rows + r]);
    }
#pragma unroll
    for (int s = 0; s < K; ++s) {
        if (s < k_out) {
            out_v[r * k_out + s] = top.v[s];
            out_i[r * k_out + s] = top.i[s] == INT32_MAX ? -1 : top.i[s];
        } else if (top.i[s] != INT32_MAX) {
            run = fmax(run, top.v[s]);
        }
    }
    if (run_out) run_out[r] = run;
}

// Sum the per-CTA certificate partials in CTA order (deterministic for a
// given grid): [sum s+^2, sum c^2, max s+, max |c|, #s>0].
static __global__ void finalize_stats(const double* __restrict__ cta, int ctas, double* __restrict__ out5) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    double a[5] = {0, 0, 0, 0, 0};
    for (int b = 0; b < ctas; ++b) {
        a[0] += cta[b * 5 + 0];
        a[1] += cta[b * 5 + 1];
        a[2] = fmax(a[2], cta[b * 5 + 2]);
        a[3] = fmax(a[3], cta[b * 5 + 3]);
        a[4] += cta[b * 5 + 4];
    }
    for (int j = 0; j < 5; ++j) out5[j] = a[j];
}

// Bytes of scratch a bucket-K pass needs for its partial lists.
inline size_t partial_bytes(int64_t rows, int parts, int K) {
    return (size_t)parts * rows * K * (sizeof(double) + sizeof(int));
}

// Simple bump allocator over a caller-provided workspace.
struct Arena {
    char* base;
    size_t size, used;
    template <class T>
    T* take(size_t count) {
        size_t off = (used + 255) & ~size_t(255);
        size_t bytes = count * sizeof(T);
        if (base == nullptr) { used = off + bytes; return nullptr; }  // sizing pass
        if (off + bytes > size) return nullptr;
        used = off + bytes;
        return reinterpret_cast<T*>(base + off);
    }
};

inline int bucket_of(int k) {
    int b = 1;
    while (b < k) b <<= 1;
    return b;
}

}  // namespace hb
