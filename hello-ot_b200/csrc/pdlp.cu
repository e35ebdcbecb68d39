// Restricted-OT Halpern-PDHG on the GPU, matrix-free over the active support.
//
// Restates the reference's restricted-OT PDLP
// (src/hello_ot/_native/cpp/solver.cpp:39-381, the same algorithm as
// src/hello_ot/_internal/lp/torch_restricted_ot.py:105-390) and replaces the
// cuPDLPx CSR SpMV + update kernels used behind backend="native"
// (src/hello_ot/_native/cupdlpx/cupdlpx/solver.cu:581-700, utils.cu:87-385).
//
// Layout in HBM: edges sorted by (source row, original index), so a source
// row's edges are contiguous; a target's incident edges are kept as a list of
// positions in that order, sorted by original edge index, and (for the fused
// passes) the per-edge state is kept a second time in that target order.  Per
// iteration one fused launch runs on sparse supports: a warp per 32 nodes of either
// side applies the per-edge update (primal step, reflection, Halpern averaging) to
// its nodes' contiguous edges in its own copy of the state, sums each node's
// reflected primal and updates the node's dual; both copies see the same
// operations, so they stay equal.  Dense sides (a coarsest level's complete
// support) and atomic node sums use an edge pass plus node passes instead.  Each
// node's incident sum is accumulated sequentially in the reference's edge order
// and this file is compiled without fma contraction, so with the same step sizes
// one block of iterations reproduces the reference arithmetic bit for bit.
//
// Control (evaluation every `frequency` iterations, adaptive restarts, PID
// primal weight, termination) runs on the host exactly as solver.cpp:157-312;
// the host reads a handful of reduced scalars once per evaluation.
#include <cub/device/device_radix_sort.cuh>

#include <chrono>
#include <cmath>
#include <limits>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "scan_common.cuh"

namespace hb {
namespace pdlp {

constexpr int RED_BLOCKS = 1184;  // reduction partial slots (8 per SM on a B200)
constexpr int RED_THREADS = 256;
// Iteration blocks of up to STEP_CAP iterations run as one CUDA graph whose
// kernels read their per-iteration parameters from D.steps.
constexpr int STEP_CAP = 8192;

struct Step {
    double primal_step, dual_step, halpern;
    int checkpoint, major;
    int parity;  // fused passes: the node-scale buffer the iteration reads (it writes the other)
    int pad;
};

struct Dev {
    int n, m, nodes;
    int64_t e;
    int* e_row;     // source of each sorted edge
    int* e_col;     // target of each sorted edge
    int* e_orig;    // original index of each sorted edge
    int* s_off;     // [n+1] source offsets into the sorted edges
    int* t_off;     // [m+1] target offsets into t_pos
    int* t_pos;     // sorted-edge positions of each target's edges, by original index
    double *cost, *cs, *ax, *x, *px, *rx, *dx;  // per sorted edge
    double *mass, *scale, *bs, *ns, *ay, *y, *py, *dy, *td;
    double* sd;     // [n] source dual / node scale, the value every edge of the row uses
    double *ssum, *tsum;  // [n], [m] node sums of the reflected primal (atomic mode; zero between passes)
    // fused passes: the edge state also in target order (by target, then original index) and
    // the node scales double-buffered (sdb[b] / tdb[b]; buffer 0 is sd / td)
    double *tx, *tax, *tcs;
    int *t_row, *t_col;
    double *sdb[2], *tdb[2];
    unsigned char *e_lane, *t_lane;  // fused passes: the own endpoint's place in its tile (node % 256), both orders
    int* fp_part;   // fused passes: tile runs of the blocks, sources then targets ([2][FP_MAX_RUNS + 1])
    double* red;    // [RED_BLOCKS][8]
    Step* steps;    // [frequency] the current block's per-iteration parameters
    double* scal;   // [16] reduced scalars
    int* status;
};

__device__ __forceinline__ double max0(double v) { return v < 0.0 ? 0.0 : v; }  // std::max(v, 0.0)

// Sequential (lane-order) sum over a warp's values; identical on every lane.
__device__ __forceinline__ double ordered_warp_sum(double acc, double v, int count) {
    for (int l = 0; l < count; ++l) acc += __shfl_sync(0xffffffffu, v, l);
    return acc;
}

// ------------------------------------------------------------------ setup
__global__ void iota_kernel(int* v, int64_t e) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x)
        v[i] = (int)i;
}

__global__ void check_convert(const int64_t* rows, const int64_t* cols, int64_t e, int n, int m, int* r32, int* c32,
                              int* status) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = rows[i], c = cols[i];
        if (r < 0 || r >= n || c < 0 || c >= m) { atomicOr(status, kErrBadInput); r32[i] = 0; c32[i] = 0; }
        else { r32[i] = (int)r; c32[i] = (int)c; }
    }
}

// offsets[k] = first position whose key is >= k (keys sorted ascending)
__global__ void offsets_kernel(const int* keys, int64_t e, int nkeys, int* off) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k <= nkeys; k += (int64_t)gridDim.x * blockDim.x) {
        int64_t lo = 0, hi = e;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (keys[mid] < k) lo = mid + 1; else hi = mid;
        }
        off[k] = (int)lo;
    }
}

__global__ void gather_edges(const int* order, const int* c32, const double* costs, const double* x0, int64_t e,
                             int* e_col, double* cost, double* x0s, int* inv) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < e; p += (int64_t)gridDim.x * blockDim.x) {
        const int o = order[p];
        e_col[p] = c32[o];
        cost[p] = costs[o];
        x0s[p] = x0 ? x0[o] : 0.0;
        inv[o] = (int)p;
    }
}

__global__ void map_positions(const int* t_orig, const int* inv, int64_t e, int* t_pos) {
    for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < e; s += (int64_t)gridDim.x * blockDim.x)
        t_pos[s] = inv[t_orig[s]];
}

// Block-partial sums of squares of two vectors (a over na, b over nb).
__global__ void sumsq2_kernel(const double* a, int64_t na, const double* b, int64_t nb, double* red) {
    __shared__ double sh[2][RED_THREADS];
    double sa = 0, sb = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na; i += (int64_t)gridDim.x * blockDim.x) sa += a[i] * a[i];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nb; i += (int64_t)gridDim.x * blockDim.x) sb += b[i] * b[i];
    sh[0][threadIdx.x] = sa; sh[1][threadIdx.x] = sb;
    __syncthreads();
    for (int w = RED_THREADS / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) { sh[0][threadIdx.x] += sh[0][threadIdx.x + w]; sh[1][threadIdx.x] += sh[1][threadIdx.x + w]; }
        __syncthreads();
    }
    if (threadIdx.x == 0) { red[blockIdx.x * 8 + 0] = sh[0][0]; red[blockIdx.x * 8 + 1] = sh[1][0]; }
}

// Block-partial maxima of |a| (over na) and |b| (over nb) into red[b][0..1].
__global__ void maxabs2_kernel(const double* a, int64_t na, const double* b, int64_t nb, double* red) {
    __shared__ double sh[2][RED_THREADS];
    double ma = 0, mb = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na; i += (int64_t)gridDim.x * blockDim.x) ma = fmax(ma, fabs(a[i]));
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nb; i += (int64_t)gridDim.x * blockDim.x) mb = fmax(mb, fabs(b[i]));
    sh[0][threadIdx.x] = ma; sh[1][threadIdx.x] = mb;
    __syncthreads();
    for (int w = RED_THREADS / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            sh[0][threadIdx.x] = fmax(sh[0][threadIdx.x], sh[0][threadIdx.x + w]);
            sh[1][threadIdx.x] = fmax(sh[1][threadIdx.x], sh[1][threadIdx.x + w]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) { red[blockIdx.x * 8 + 0] = sh[0][0]; red[blockIdx.x * 8 + 1] = sh[1][0]; }
}

// Maximum of the block partials: scal[base + j] = max_b red[b][first + j], j < cnt.
__global__ void finish_red_max(const double* red, int blocks, int first, int cnt, double* scal, int base) {
    if (threadIdx.x == 0) {
        for (int j = 0; j < cnt; ++j) {
            double s = 0;
            for (int b = 0; b < blocks; ++b) s = fmax(s, red[b * 8 + first + j]);
            scal[base + j] = s;
        }
    }
}

// Fixed-order sum of the block partials: scal[base + j] = sum_b red[b][j], j < cnt.
__global__ void finish_red(const double* red, int blocks, int cnt, double* scal, int base) {
    if (threadIdx.x == 0) {
        for (int j = 0; j < cnt; ++j) {
            double s = 0;
            for (int b = 0; b < blocks; ++b) s += red[b * 8 + j];
            scal[base + j] = s;
        }
    }
}

__global__ void degree_scale(const int* s_off, const int* t_off, int n, int m, double* scale) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n + m; i += gridDim.x * blockDim.x) {
        const int deg = i < n ? s_off[i + 1] - s_off[i] : t_off[i - n + 1] - t_off[i - n];
        scale[i] = sqrt((double)(deg > 1 ? deg : 1));
    }
}

// solver.cpp:96-109
__global__ void init_state(Dev D, const double* masses, const double* y0, const double* x0s, double bound,
                           double objective, double variable) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < D.e; p += stride) {
        D.cs[p] = D.cost[p] * objective / variable;
        const double a = max0(x0s[p]) * variable * bound;
        D.ax[p] = a; D.x[p] = a; D.px[p] = a;
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < D.nodes; i += stride) {
        D.mass[i] = masses[i];
        D.bs[i] = masses[i] * bound / D.scale[i];
        D.ns[i] = variable * D.scale[i];
        const double a = (y0 ? y0[i] : 0.0) * D.scale[i] * objective;
        D.ay[i] = a; D.y[i] = a; D.py[i] = a;
        if (i >= D.n) D.td[i - D.n] = a / D.ns[i];
        else D.sd[i] = a / D.ns[i];
    }
}

// ------------------------------------------------------------------ iteration


// One PDHG iteration runs as three kernels (solver.cpp:255-281) when the node sums are
// accumulated with atomics or a side is dense (otherwise the fused passes below, one launch):
//  edge_pass   : thread per edge, primal update, reflection, Halpern averaging
//                (coalesced over the source-sorted edges, perfectly balanced);
//  source_pass : warp per 32 source rows (coalesced staging), ordered sum of
//                each row's reflected primal and the source dual update;
//  target_pass : thread per target, ordered gather-sum and the target dual update.
// Each node sums its edges sequentially in the reference's edge order.
template <bool ATOMIC>
__global__ void __launch_bounds__(256) edge_pass(Dev D, int it) {
    const Step s = D.steps[it];
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int lane = threadIdx.x & 31;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < D.e; base += stride) {  // block-uniform
        const int64_t p = base + threadIdx.x;
        const bool live = p < D.e;
        double r = 0.0;
        int row = -1;
        if (live) {
            row = D.e_row[p];
            const int col = D.e_col[p];
            const double at = D.sd[row] + D.td[col];
            const double xv = D.x[p];
            const double pxv = max0(xv - s.primal_step * (D.cs[p] - at));
            r = 2.0 * pxv - xv;
            if (s.checkpoint) D.dx[p] = r - xv;
            D.x[p] = s.halpern * r + (1.0 - s.halpern) * D.ax[p];
            if (s.major) D.px[p] = pxv;
            if (ATOMIC) atomicAdd(D.tsum + col, r);
            else D.rx[p] = r;
        }
        if (ATOMIC) {
            // the warp's edges are sorted by source: suffix sums within each run of one
            // source (a lane adds lane+off only inside its run), then one atomic per run
            double v = r;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const double vo = __shfl_down_sync(0xffffffffu, v, off);
                const int ro = __shfl_down_sync(0xffffffffu, row, off);
                if (lane + off < 32 && ro == row) v += vo;
            }
            const int prev = __shfl_up_sync(0xffffffffu, row, 1);
            if (live && (lane == 0 || prev != row)) atomicAdd(D.ssum + row, v);
        }
    }
}

// Sums of the segments [off[v], off[v+1]) of `vals` for the 32 consecutive nodes
// v = v0 + lane of a warp, each in index order.  The warp's whole range is staged
// through shared memory in coalesced chunks; every lane then adds its own
// node's values of the chunk.  All lanes take the same loop (warp-uniform).
constexpr int SEG_CHUNK = 256;
__device__ __forceinline__ double warp_segment_sum(const double* __restrict__ vals, const int* __restrict__ off,
                                                   int v0, int nodes, double* stage) {
    const int lane = threadIdx.x & 31, v = v0 + lane;
    const int w0 = off[v0], w1 = off[min(v0 + 32, nodes)];
    const int b0 = v < nodes ? off[v] : w1, b1 = v < nodes ? off[v + 1] : w1;
    double sum = 0.0;
    for (int c0 = w0; c0 < w1; c0 += SEG_CHUNK) {
        const int c1 = min(w1, c0 + SEG_CHUNK);
        for (int i = c0 + lane; i < c1; i += 32) stage[i - c0] = __ldg(vals + i);
        __syncwarp();
        const int lo = max(b0, c0), hi = min(b1, c1);
        for (int q = lo; q < hi; ++q) sum += stage[q - c0];
        __syncwarp();
    }
    return sum;
}

template <bool ATOMIC>
__global__ void __launch_bounds__(256) source_pass(Dev D, int it) {
    const Step s = D.steps[it];
    __shared__ double stage[ATOMIC ? 1 : 8][ATOMIC ? 1 : SEG_CHUNK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int v0 = (blockIdx.x * 8 + warp) * 32;
    if (v0 >= D.n) return;  // warp-uniform
    double sum;
    if (ATOMIC) {
        const int i = v0 + lane;
        sum = i < D.n ? D.ssum[i] : 0.0;
        if (i < D.n) D.ssum[i] = 0.0;
    } else {
        sum = warp_segment_sum(D.rx, D.s_off, v0, D.n, stage[warp]);
    }
    const int i = v0 + lane;
    if (i >= D.n) return;
    const double yv = D.y[i];
    const double pyv = yv - s.dual_step * (sum / D.ns[i] - D.bs[i]);
    const double refl = 2.0 * pyv - yv;
    if (s.checkpoint) D.dy[i] = refl - yv;
    const double ynew = s.halpern * refl + (1.0 - s.halpern) * D.ay[i];
    D.y[i] = ynew;
    D.sd[i] = ynew / D.ns[i];
    if (s.major) D.py[i] = pyv;
}

template <bool ATOMIC>
__global__ void __launch_bounds__(256) target_pass(Dev D, int it) {
    const Step s = D.steps[it];
    const int stride = gridDim.x * blockDim.x;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < D.m; j += stride) {
        const int b0 = ATOMIC ? 0 : D.t_off[j], b1 = ATOMIC ? 0 : D.t_off[j + 1];
        double sum = 0.0;
        if (ATOMIC) { sum = D.tsum[j]; D.tsum[j] = 0.0; }
        int sl = b0;
        for (; sl + 4 <= b1; sl += 4) {  // four independent gathers in flight, summed in order
            const double r0 = D.rx[D.t_pos[sl]], r1 = D.rx[D.t_pos[sl + 1]];
            const double r2 = D.rx[D.t_pos[sl + 2]], r3 = D.rx[D.t_pos[sl + 3]];
            sum += r0; sum += r1; sum += r2; sum += r3;
        }
        for (; sl < b1; ++sl) sum += D.rx[D.t_pos[sl]];
        const int i = D.n + j;
        const double yv = D.y[i];
        const double pyv = yv - s.dual_step * (sum / D.ns[i] - D.bs[i]);
        const double refl = 2.0 * pyv - yv;
        if (s.checkpoint) D.dy[i] = refl - yv;
        const double ynew = s.halpern * refl + (1.0 - s.halpern) * D.ay[i];
        D.y[i] = ynew;
        if (s.major) D.py[i] = pyv;
        D.td[j] = ynew / D.ns[i];
    }
}

// Wide variants for high-degree nodes (mean degree >= WIDE_DEGREE, e.g. the complete
// support of a coarsest level): one warp per node.  The warp stages the node's
// reflected primal values (contiguous for sources, gathered through t_pos for
// targets) into shared memory in chunks of SEG_CHUNK, and lane 0 adds them in edge
// order, so the sums are the same as the thread-per-node passes'.
constexpr int WIDE_DEGREE = 64;

__device__ __forceinline__ void dual_update(const Dev& D, const Step& s, int i, double sum) {
    const double yv = D.y[i];
    const double pyv = yv - s.dual_step * (sum / D.ns[i] - D.bs[i]);
    const double refl = 2.0 * pyv - yv;
    if (s.checkpoint) D.dy[i] = refl - yv;
    const double ynew = s.halpern * refl + (1.0 - s.halpern) * D.ay[i];
    D.y[i] = ynew;
    if (s.major) D.py[i] = pyv;
    if (i < D.n) D.sd[i] = ynew / D.ns[i];
    else D.td[i - D.n] = ynew / D.ns[i];
}

// Blocks [0, src_blocks) take sources, the next tgt_blocks blocks take targets: the two
// sides only read the edge pass's output, so one launch runs both side by side.
// TREE: every lane adds its own strided values in order, then a fixed butterfly over
// the lanes (a deterministic order, not the reference's; no serial chain).
constexpr int WIDE_CHUNK = 512;
template <bool TREE>
__global__ void __launch_bounds__(256) node_pass_wide(Dev D, int it, int src_blocks) {
    __shared__ double stage[TREE ? 1 : 8][TREE ? 1 : WIDE_CHUNK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool target = (int)blockIdx.x >= src_blocks;  // block-uniform
    const int v = ((int)blockIdx.x - (target ? src_blocks : 0)) * 8 + warp;
    if (v >= (target ? D.m : D.n)) return;  // warp-uniform
    const int* off = target ? D.t_off : D.s_off;
    const int b0 = off[v], b1 = off[v + 1];
    double* st = stage[TREE ? 0 : warp];
    double sum = 0.0;
    for (int c0 = b0; c0 < b1; c0 += WIDE_CHUNK) {
        const int c1 = min(b1, c0 + WIDE_CHUNK);
        // all of a lane's loads of the chunk in flight at once (positions, then values)
        constexpr int PER_LANE = WIDE_CHUNK / 32;
        int pos[PER_LANE];
#pragma unroll
        for (int u = 0; u < PER_LANE; ++u) {
            const int q = c0 + u * 32 + lane;
            pos[u] = q < c1 ? (target ? __ldg(D.t_pos + q) : q) : -1;
        }
        double val[PER_LANE];
#pragma unroll
        for (int u = 0; u < PER_LANE; ++u) val[u] = pos[u] >= 0 ? __ldg(D.rx + pos[u]) : 0.0;
        if (TREE) {
#pragma unroll
            for (int u = 0; u < PER_LANE; ++u) sum += val[u];
            continue;
        }
#pragma unroll
        for (int u = 0; u < PER_LANE; ++u) st[u * 32 + lane] = val[u];
        __syncwarp();
        if (lane == 0) {
            const int len = c1 - c0;
#pragma unroll 8
            for (int q = 0; q < len; ++q) sum += st[q];
        }
        __syncwarp();
    }
    if (TREE) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    if (lane == 0) dual_update(D, D.steps[it], target ? D.n + v : v, sum);
}

// Complete supports stored row-major (edge p = i * m + j after the source sort, e.g. a
// coarsest level's dense transport), summation "tree": the target sums read the reflected
// primal as a matrix, a block per 32 targets, warp w adding rows w, w + 32, ... of its lane's
// column (32 consecutive columns: coalesced), then warp 0 adding the 32 partials in warp order.
// A fixed order (not the reference's), like the lane tree of node_pass_wide, without its
// stride-m gathers.
__global__ void __launch_bounds__(1024) dense_target_pass(Dev D, int it) {
    __shared__ double part[32][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * 32 + lane;
    double acc = 0.0;
    if (j < D.m) {
        const double* col = D.rx + j;
        for (int i = warp; i < D.n; i += 32) acc += __ldg(col + (int64_t)i * D.m);
    }
    part[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && j < D.m) {
        double sum = 0.0;
        for (int w = 0; w < 32; ++w) sum += part[w][lane];
        dual_update(D, D.steps[it], D.n + j, sum);
    }
}

// flag = 1 unless every sorted edge p has target p % m (the row-major complete layout).
__global__ void check_rowmajor(Dev D, int* flag) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < D.e; p += (int64_t)gridDim.x * blockDim.x)
        if (D.e_col[p] != (int)(p % D.m)) atomicOr(flag, 1);
}

// Fused passes (the default for sparse supports): one launch per iteration.  The edge state
// is kept twice, in source order (x, ax, cs) and in target order (tx, tax, tcs), so each side
// reads its nodes' edges contiguously.  Tiles are C::TN consecutive nodes of one side (node v
// at place v % C::TN, owned by thread v % C::TN; 256 per tile, or 64 on small supports so
// that every block has a tile).  A persistent block of FP_THREADS threads owns a run of
// consecutive tiles of one side, the runs balanced by edges, and streams the run's edge
// state through a ring of C::ST shared-memory stages of C::CH edges, filled by bulk copies
// (cp.async.bulk issued by one thread, completion on one mbarrier per stage).  Per stage:
// the threads apply the per-edge update (primal step, reflection, Halpern averaging: the
// operations of edge_pass, so both copies stay equal bit for bit) to the stage's edges,
// thread-strided, write the new primal and stage the reflected primal; after one barrier
// the stage is refilled, the node scales of the next stage's edges are gathered (from L2;
// they arrive while the block works on), and each thread adds its node's reflected primals
// in edge order (the reference's order), updating its node's dual when its tile's edges
// end.  The edge updates read the node scales of buffer `parity` and the dual updates write
// the other buffer, so the source and target sides run side by side in one launch.  The
// source side also writes px / dx, which the evaluation and restart kernels read.
constexpr int FP_THREADS = 256;    // threads per block
constexpr int FP_MAX_RUNS = 4096;  // blocks per side, at most

template <int CH_, int ST_, int BPS_, bool CG_ = false, int TN_ = 256>
struct FpCfg {
    static constexpr int TN = TN_;    // nodes per tile (divides 256: the lane byte is node % 256)
    static constexpr int CH = CH_;    // edges per stage
    static constexpr int ST = ST_;    // stages
    static constexpr int BPS = BPS_;  // blocks per SM
    static constexpr bool CG = CG_;   // node-scale gathers cached in L2 only
    static constexpr int PER = CH / FP_THREADS;  // edges per thread in one stage
};

template <class C>
struct FpStage {  // 16-byte-aligned starts, each array rounded so the next stays aligned
    double x[C::CH + 4], ax[C::CH + 4], cs[C::CH + 4];
    int o[C::CH + 4];
    unsigned char ln[C::CH + 16];
};
template <class C>
struct alignas(16) FpShared {
    FpStage<C> st[C::ST];
    double rs[2][C::CH];  // reflected primals of the last two stages
    uint64_t bar[C::ST];
    int abort_flag;
};

template <class C, bool TGT>
__device__ __forceinline__ void fp_side(const Dev& D, const Step& s, int tb, int te, FpShared<C>& sh) {
    constexpr int CH = C::CH, ST = C::ST, PER = C::PER;
    const int t = threadIdx.x, nodes = TGT ? D.m : D.n;
    const int* off = TGT ? D.t_off : D.s_off;
    double* X = TGT ? D.tx : D.x;
    const double* AX = TGT ? D.tax : D.ax;
    const double* CS = TGT ? D.tcs : D.cs;
    const int* O = TGT ? D.t_row : D.e_col;                 // the other endpoint of each edge
    const unsigned char* LN = TGT ? D.t_lane : D.e_lane;    // the own endpoint's place in its tile
    const double* ownb = (TGT ? D.tdb : D.sdb)[s.parity];
    const double* other = TGT ? D.sdb[s.parity] : D.tdb[s.parity];
    constexpr int TN = C::TN;
    auto tile_end = [&](int tl) { return off[min(tl * TN + TN, nodes)]; };
    const int E0 = off[tb * TN], E1 = tile_end(te - 1);
    const int nch = (E1 - E0 + CH - 1) / CH;
    auto issue = [&](int k) {  // one thread: the bulk copies of chunk k into stage k % ST
        const int c0 = E0 + k * CH, c1 = min(E1, c0 + CH);
        const int d0 = c0 & ~1, d1 = (c1 + 1) & ~1, i0 = c0 & ~3, i1 = (c1 + 3) & ~3, b0 = c0 & ~15,
                  b1 = (c1 + 15) & ~15;
        FpStage<C>& S = sh.st[k % ST];
        uint64_t* bar = &sh.bar[k % ST];
        const uint32_t nd = (uint32_t)(d1 - d0) * 8u, ni = (uint32_t)(i1 - i0) * 4u, nb = (uint32_t)(b1 - b0);
        mbar_arrive_expect_tx(bar, 3u * nd + ni + nb);
        bulk_load_1d(S.x, X + d0, nd, bar);
        bulk_load_1d(S.ax, AX + d0, nd, bar);
        bulk_load_1d(S.cs, CS + d0, nd, bar);
        bulk_load_1d(S.o, O + i0, ni, bar);
        bulk_load_1d(S.ln, LN + b0, nb, bar);
    };
    if (t == 0)
        for (int k = 0; k < ST && k < nch; ++k) issue(k);
    // gather cursor: tile gt holds the first edge of the stage being gathered; gT1 / gT2 are
    // the ends of tiles gt and gt + 1 (the run's end past the run)
    int gt = tb, gT1 = tile_end(tb), gT2 = tb + 1 < te ? tile_end(tb + 1) : E1;
    double o[PER], m[PER];  // the other and own node scales of the stage's edges
    auto gather = [&](int k) {  // false: the stage's copies never completed
        if (!mbar_wait(&sh.bar[k % ST], (uint32_t)((k / ST) & 1), &sh.abort_flag, D.status)) return false;
        const FpStage<C>& S = sh.st[k % ST];
        const int c0 = E0 + k * CH, c1 = min(E1, c0 + CH), i0 = c0 & ~3, lb0 = c0 & ~15;
        while (gT1 <= c0 && gt + 1 < te) {  // block-uniform
            ++gt;
            gT1 = gT2;
            gT2 = gt + 1 < te ? tile_end(gt + 1) : E1;
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int q = c0 + j * FP_THREADS + t;
            o[j] = m[j] = 0.0;
            if (q < c1) {
                int tl = q < gT1 ? gt : gt + 1;
                if (q >= gT2) {  // past tile gt + 1 (tiles of few edges): the last tile starting at or before q
                    int lo = gt + 2, hi = te - 1;
                    while (lo < hi) {
                        const int mid = (lo + hi + 1) >> 1;
                        if (off[mid * TN] <= q) lo = mid; else hi = mid - 1;
                    }
                    tl = lo;
                }
                if (C::CG) {
                    o[j] = __ldcg(other + S.o[q - i0]);
                    m[j] = __ldcg(ownb + tl * TN + (S.ln[q - lb0] & (TN - 1)));
                } else {
                    o[j] = __ldg(other + S.o[q - i0]);
                    m[j] = __ldg(ownb + tl * TN + (S.ln[q - lb0] & (TN - 1)));
                }
            }
        }
        return true;
    };
    auto drain = [&](int k) {  // after a failed wait: a bounded wait for the copies in flight
        for (int j = k + 1; j < nch && j < k + ST; ++j)
            for (int u = 0; u < 64 && !mbar_try_wait(&sh.bar[j % ST], (uint32_t)((j / ST) & 1)); ++u) {
            }
    };
    // sum cursor: this thread's node of tile `tile`, its edge range, its state; the next
    // tile's offsets are loaded one tile ahead
    // threads t >= TN own no node (v = nodes: empty segment, no dual update)
    auto node_of = [&](int tl) { return t < TN ? min(tl * TN + t, nodes) : nodes; };
    int tile = tb, v = node_of(tb);
    int T1 = gT1;
    int b0 = v < nodes ? off[v] : T1, b1 = v < nodes ? off[v + 1] : T1;
    int nT1 = 0, nb0 = 0, nb1 = 0;
    auto prefetch_next = [&]() {
        if (tile + 1 >= te) return;
        const int nv = node_of(tile + 1);
        nT1 = tile_end(tile + 1);
        nb0 = nv < nodes ? off[nv] : nT1;
        nb1 = nv < nodes ? off[nv + 1] : nT1;
    };
    prefetch_next();
    double yv, nsv, bsv, ayv;
    auto node_state = [&]() {
        const int i = (TGT ? D.n : 0) + (v < nodes ? v : 0);
        yv = D.y[i]; nsv = D.ns[i]; bsv = D.bs[i]; ayv = D.ay[i];
    };
    node_state();
    double sum = 0.0;
    auto finish_tile = [&]() {  // the dual update of this thread's node; false past the run
        if (v < nodes) {
            const int i = TGT ? D.n + v : v;
            const double pyv = yv - s.dual_step * (sum / nsv - bsv);
            const double refl = 2.0 * pyv - yv;
            if (s.checkpoint) D.dy[i] = refl - yv;
            const double ynew = s.halpern * refl + (1.0 - s.halpern) * ayv;
            D.y[i] = ynew;
            if (s.major) D.py[i] = pyv;
            (TGT ? D.tdb : D.sdb)[s.parity ^ 1][v] = ynew / nsv;
        }
        sum = 0.0;
        if (++tile >= te) return false;
        v = node_of(tile);
        T1 = nT1; b0 = nb0; b1 = nb1;
        prefetch_next();
        node_state();
        return true;
    };
    bool more = true;
    if (nch > 0 && !gather(0)) { drain(0); return; }
    for (int k = 0; k < nch; ++k) {
        const FpStage<C>& S = sh.st[k % ST];
        const int c0 = E0 + k * CH, c1 = min(E1, c0 + CH), d0 = c0 & ~1;
        double* rs = sh.rs[k & 1];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int q = c0 + j * FP_THREADS + t;
            if (q >= c1) continue;
            const double xv = S.x[q - d0];
            const double at = TGT ? o[j] + m[j] : m[j] + o[j];  // sd[row] + td[col]
            const double pxv = max0(xv - s.primal_step * (S.cs[q - d0] - at));
            const double r = 2.0 * pxv - xv;
            if (!TGT) {
                if (s.checkpoint) D.dx[q] = r - xv;
                if (s.major) D.px[q] = pxv;
            }
            X[q] = s.halpern * r + (1.0 - s.halpern) * S.ax[q - d0];
            rs[q - c0] = r;
        }
        __syncthreads();  // stage k is consumed; rs[k & 1] is complete
        if (t == 0 && k + ST < nch) issue(k + ST);
        if (k + 1 < nch && !gather(k + 1)) { drain(k + 1); return; }
        for (;;) {  // this thread's nodes with edges in the stage
            const int l0 = max(b0, c0), h0 = min(b1, c1);
            int q = l0;
            for (; q + 4 <= h0; q += 4) {  // loads side by side, adds in edge order
                const double r0 = rs[q - c0], r1 = rs[q + 1 - c0], r2 = rs[q + 2 - c0], r3 = rs[q + 3 - c0];
                sum += r0; sum += r1; sum += r2; sum += r3;
            }
            for (; q < h0; ++q) sum += rs[q - c0];
            if (T1 > c1) break;  // the tile goes on into the next stage
            if (!(more = finish_tile())) break;
        }
    }
    while (more) more = finish_tile();  // tiles without edges after the last stage
}

// Blocks [0, runs) take source runs, [runs, 2 runs) target runs; run r of a side covers the
// tiles [part[r], part[r + 1]).
template <class C>
__global__ void __launch_bounds__(FP_THREADS, C::BPS) fused_pass(Dev D, int it, int runs) {
    extern __shared__ __align__(128) unsigned char fp_smem[];
    FpShared<C>& sh = *reinterpret_cast<FpShared<C>*>(fp_smem);
    const bool target = (int)blockIdx.x >= runs;
    const int r = target ? (int)blockIdx.x - runs : (int)blockIdx.x;
    const int* part = D.fp_part + (target ? FP_MAX_RUNS + 1 : 0);
    const int tb = part[r], te = part[r + 1];
    if (tb >= te) return;  // block-uniform
    if (threadIdx.x == 0) {
        sh.abort_flag = 0;
        for (int j = 0; j < C::ST; ++j) mbar_init(&sh.bar[j], 1);
        fence_barrier_init();
    }
    __syncthreads();
    const Step s = D.steps[it];
    if (target) fp_side<C, true>(D, s, tb, te, sh);
    else fp_side<C, false>(D, s, tb, te, sh);
}

// Tile runs balanced by edges: part[r] = the first tile whose first edge is at or after
// r * E / runs, part[runs] = all tiles; sources at fp_part, targets at fp_part + FP_MAX_RUNS + 1.
__global__ void fp_partition(Dev D, int runs, int tn) {
    for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < 2 * (runs + 1); u += gridDim.x * blockDim.x) {
        const bool target = u > runs;
        const int r = target ? u - runs - 1 : u;
        const int nodes = target ? D.m : D.n;
        const int* off = target ? D.t_off : D.s_off;
        const int tiles = (nodes + tn - 1) / tn;
        int res = tiles;
        if (r < runs) {
            const int64_t want = D.e * (int64_t)r / runs;
            int lo = 0, hi = tiles;  // first tile with off[tn tile] >= want
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (off[mid * tn] < want) lo = mid + 1; else hi = mid;
            }
            res = lo;
        }
        D.fp_part[(target ? FP_MAX_RUNS + 1 : 0) + r] = res;
    }
}

// The target-order copy of the edge state: structure (once), cost and primal (at the
// start and after every restart, from the source-order state).
__global__ void target_copy(Dev D, int structure) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < D.e; q += stride) {
        const int p = D.t_pos[q];
        if (structure) {
            D.t_row[q] = D.e_row[p]; D.t_col[q] = D.e_col[p]; D.tcs[q] = D.cs[p];
            D.t_lane[q] = (unsigned char)(D.e_col[p] & 255);
            D.e_lane[q] = (unsigned char)(D.e_row[q] & 255);
        }
        D.tx[q] = D.x[p];
        D.tax[q] = D.ax[p];
    }
}

// ------------------------------------------------------------------ reductions
template <int CNT>
__device__ __forceinline__ void block_store(double (&v)[CNT], double* red) {
    __shared__ double sh[CNT][RED_THREADS];
#pragma unroll
    for (int j = 0; j < CNT; ++j) sh[j][threadIdx.x] = v[j];
    __syncthreads();
    for (int w = RED_THREADS / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w)
#pragma unroll
            for (int j = 0; j < CNT; ++j) sh[j][threadIdx.x] += sh[j][threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0)
#pragma unroll
        for (int j = 0; j < CNT; ++j) red[blockIdx.x * 8 + j] = sh[j][0];
}

// Residuals of the unscaled problem (solver.cpp:115-136):
// [0] sum of squared marginal errors, [1] sum of squared dual violations,
// [2] primal objective, [3] dual objective; with `linf`, also [4] the largest |marginal
// error| and [5] the largest dual violation (the max-norm termination test).
__global__ void __launch_bounds__(RED_THREADS) evaluate_kernel(Dev D, double vb, double objective, int linf) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    double v[4] = {0, 0, 0, 0};
    double mx[2] = {0, 0};
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < D.nodes; i += warps) {
        const bool src = i < D.n;
        const int b0 = src ? D.s_off[i] : D.t_off[i - D.n], b1 = src ? D.s_off[i + 1] : D.t_off[i - D.n + 1];
        double sum = 0.0;
        for (int base = b0; base < b1; base += 32) {
            const int sl = base + lane;
            const double r = sl < b1 ? D.px[src ? sl : D.t_pos[sl]] / vb : 0.0;
            sum = ordered_warp_sum(sum, r, min(32, b1 - base));
        }
        if (lane == 0) {
            const double delta = sum - D.mass[i];
            v[0] += delta * delta;
            v[3] += D.mass[i] * (D.py[i] / (D.scale[i] * objective));
            mx[0] = fmax(mx[0], fabs(delta));
        }
    }
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < D.e; p += stride) {
        const int r = D.e_row[p], c = D.n + D.e_col[p];
        const double score = D.py[r] / (D.scale[r] * objective) + D.py[c] / (D.scale[c] * objective) - D.cost[p];
        const double viol = max0(score);
        v[1] += viol * viol;
        v[2] += D.cost[p] * (D.px[p] / vb);
        mx[1] = fmax(mx[1], viol);
    }
    block_store<4>(v, D.red);
    if (linf) {  // block maxima into red[b][4..5] (block_store's last barrier is behind every thread)
        __shared__ double shm[2][RED_THREADS];
        shm[0][threadIdx.x] = mx[0]; shm[1][threadIdx.x] = mx[1];
        __syncthreads();
        for (int w = RED_THREADS / 2; w > 0; w >>= 1) {
            if (threadIdx.x < w) {
                shm[0][threadIdx.x] = fmax(shm[0][threadIdx.x], shm[0][threadIdx.x + w]);
                shm[1][threadIdx.x] = fmax(shm[1][threadIdx.x], shm[1][threadIdx.x + w]);
            }
            __syncthreads();
        }
        if (threadIdx.x == 0) { D.red[blockIdx.x * 8 + 4] = shm[0][0]; D.red[blockIdx.x * 8 + 5] = shm[1][0]; }
    }
}

// Restart distances: [0] |px - ax|^2, [1] |py - ay|^2 (solver.cpp:203-213).
__global__ void __launch_bounds__(RED_THREADS) restart_dist_kernel(Dev D) {
    double v[2] = {0, 0};
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < D.e; p += stride) {
        const double t = D.px[p] - D.ax[p];
        v[0] += t * t;
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < D.nodes; i += stride) {
        const double t = D.py[i] - D.ay[i];
        v[1] += t * t;
    }
    block_store<2>(v, D.red);
}

// Restart to the last PDHG iterate (solver.cpp:238-242); the node scales go to buffer
// `parity` (the one the next iteration reads), the target-order copy follows (fused passes).
__global__ void restart_kernel(Dev D, int parity, int fused) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < D.e; p += stride) {
        const double v = D.px[p];
        D.ax[p] = v; D.x[p] = v;
        if (fused) {
            const double t = D.px[D.t_pos[p]];
            D.tax[p] = t; D.tx[p] = t;
        }
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < D.nodes; i += stride) {
        const double v = D.py[i];
        D.ay[i] = v; D.y[i] = v;
        if (i >= D.n) D.tdb[parity][i - D.n] = v / D.ns[i];
        else D.sdb[parity][i] = v / D.ns[i];
    }
}

// Fixed-point error terms (solver.cpp:286-294): [0] |dx|^2, [1] |dy|^2,
// [2] interaction sum (dy_r/ns_r + dy_c/ns_c) dx.
__global__ void __launch_bounds__(RED_THREADS) fixed_point_kernel(Dev D) {
    double v[3] = {0, 0, 0};
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < D.e; p += stride) {
        const int r = D.e_row[p], c = D.n + D.e_col[p];
        const double dxv = D.dx[p];
        v[0] += dxv * dxv;
        v[2] += (D.dy[r] / D.ns[r] + D.dy[c] / D.ns[c]) * dxv;
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < D.nodes; i += stride) v[1] += D.dy[i] * D.dy[i];
    block_store<3>(v, D.red);
}

__global__ void output_kernel(Dev D, double vb, double objective, double* x_out, double* y_out) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < D.e; p += stride)
        x_out[D.e_orig[p]] = D.px[p] / vb;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < D.nodes; i += stride)
        y_out[i] = D.py[i] / (D.scale[i] * objective);
}

}  // namespace pdlp

// ------------------------------------------------------------------ host
struct PdlpLayout {
    pdlp::Dev D{};
    int *r32 = nullptr, *c32 = nullptr, *iota = nullptr, *keys_out = nullptr, *t_orig = nullptr, *t_keys = nullptr,
        *inv = nullptr;
    double* x0s = nullptr;
    void* cub = nullptr;
    size_t cub_bytes = 0;
    size_t bytes = 0;
    bool ok = true;
};

PdlpLayout pdlp_layout(void* base, size_t size, int64_t n, int64_t m, int64_t e) {
    PdlpLayout L;
    const int64_t nodes = n + m;
    // arrays start on 256-byte boundaries of the device address space (the fused passes
    // bulk-copy edge arrays from 16-byte-aligned starts); the edge arrays the fused passes
    // stream hold e rounded up to 4 elements, as the copies read whole 4-element groups
    char* b = static_cast<char*>(base);
    if (b) {
        const uintptr_t a = (reinterpret_cast<uintptr_t>(b) + 255) & ~uintptr_t(255);
        const size_t skip = a - reinterpret_cast<uintptr_t>(b);
        size = size > skip ? size - skip : 0;
        b = reinterpret_cast<char*>(a);
    }
    Arena ar{b, size, 0};
    const int64_t e4 = (e + 3) & ~int64_t(3);
    auto take_i = [&](int*& p, size_t c) { p = ar.take<int>(c); if (base && !p) L.ok = false; };
    auto take_d = [&](double*& p, size_t c) { p = ar.take<double>(c); if (base && !p) L.ok = false; };
    pdlp::Dev& D = L.D;
    take_i(D.e_row, e); take_i(D.e_col, e4); take_i(D.e_orig, e); take_i(D.s_off, n + 1); take_i(D.t_off, m + 1);
    take_i(D.t_pos, e);
    take_d(D.cost, e); take_d(D.cs, e4); take_d(D.ax, e4); take_d(D.x, e4); take_d(D.px, e); take_d(D.rx, e);
    take_d(D.dx, e);
    take_d(D.mass, nodes); take_d(D.scale, nodes); take_d(D.bs, nodes); take_d(D.ns, nodes); take_d(D.ay, nodes);
    take_d(D.y, nodes); take_d(D.py, nodes); take_d(D.dy, nodes); take_d(D.td, m); take_d(D.sd, n); take_d(D.ssum, n); take_d(D.tsum, m);
    take_d(D.tx, e4); take_d(D.tax, e4); take_d(D.tcs, e4); take_i(D.t_row, e4); take_i(D.t_col, e);
    take_i(D.fp_part, 2 * (pdlp::FP_MAX_RUNS + 1));
    D.e_lane = ar.take<unsigned char>((size_t)((e + 15) & ~int64_t(15)));
    D.t_lane = ar.take<unsigned char>((size_t)((e + 15) & ~int64_t(15)));
    if (base && (!D.e_lane || !D.t_lane)) L.ok = false;
    D.sdb[0] = D.sd; D.tdb[0] = D.td;
    take_d(D.sdb[1], n); take_d(D.tdb[1], m);
    take_d(D.red, (size_t)pdlp::RED_BLOCKS * 8); take_d(D.scal, 16);
    D.steps = ar.take<pdlp::Step>((size_t)pdlp::STEP_CAP);
    if (base && !D.steps) L.ok = false;
    take_i(D.status, 1);
    take_i(L.r32, e); take_i(L.c32, e); take_i(L.iota, e); take_i(L.keys_out, e); take_i(L.t_orig, e);
    take_i(L.t_keys, e); take_i(L.inv, e);
    take_d(L.x0s, e);
    size_t cub_bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, cub_bytes, (const int*)nullptr, (int*)nullptr, (const int*)nullptr,
                                    (int*)nullptr, (int)e);
    L.cub_bytes = cub_bytes;
    L.cub = ar.take<char>(cub_bytes > 0 ? cub_bytes : 1);
    if (base && !L.cub) L.ok = false;
    L.bytes = ar.used + 256;
    return L;
}

size_t pdlp_bytes(int64_t n, int64_t m, int64_t e) { return pdlp_layout(nullptr, 0, n, m, e).bytes; }

#define HB_LAUNCHED(n) count_launches(n)

int pdlp_solve(const int64_t* rows, const int64_t* cols, const double* costs, int64_t e, const double* masses,
               int64_t n, int64_t m, const double* x0, const double* y0, const PdlpControls& ctl, double* x_out,
               double* y_out, PdlpResult* res, TraceRow* trace, int trace_cap, int* trace_len, void* ws,
               size_t ws_bytes, cudaStream_t st, std::string& err) {
    using Clock = std::chrono::steady_clock;
    const auto started = Clock::now();
    if (n < 1 || m < 1 || e < 1 || e > INT32_MAX - 1024 || n + m > INT32_MAX - 1 || ctl.frequency < 1 ||
        ctl.iteration_limit < 1 || !(ctl.time_limit > 0)) {
        err = "invalid restricted OT dimensions or runtime limits";
        return 2;
    }
    PdlpLayout L = pdlp_layout(ws, ws_bytes, n, m, e);
    if (!L.ok) { err = "workspace too small for the restricted OT solve"; return 3; }
    pdlp::Dev D = L.D;
    D.n = (int)n; D.m = (int)m; D.nodes = (int)(n + m); D.e = e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int gb = sms * 8;
    auto fail = [&](const char* what) {
        cudaError_t ce = cudaGetLastError();
        err = std::string(what) + (ce != cudaSuccess ? std::string(": ") + cudaGetErrorString(ce) : std::string());
        return 6;
    };
    cudaMemsetAsync(D.status, 0, sizeof(int), st);
    cudaMemsetAsync(D.ssum, 0, sizeof(double) * n, st);
    cudaMemsetAsync(D.tsum, 0, sizeof(double) * m, st);
    // --- incidence structure (solver.cpp:74-90): sort by source, then by target
    pdlp::check_convert<<<gb, 256, 0, st>>>(rows, cols, e, (int)n, (int)m, L.r32, L.c32, D.status);
    HB_LAUNCHED(1);
    pdlp::iota_kernel<<<gb, 256, 0, st>>>(L.iota, e);
    HB_LAUNCHED(1);
    size_t cb = L.cub_bytes;
    if (cub::DeviceRadixSort::SortPairs(L.cub, cb, L.r32, D.e_row, L.iota, D.e_orig, (int)e, 0, 32, st) != cudaSuccess)
        return fail("source sort");
    HB_LAUNCHED(1);
    cb = L.cub_bytes;
    if (cub::DeviceRadixSort::SortPairs(L.cub, cb, L.c32, L.t_keys, L.iota, L.t_orig, (int)e, 0, 32, st) != cudaSuccess)
        return fail("target sort");
    HB_LAUNCHED(1);
    pdlp::offsets_kernel<<<(unsigned)((n + 256) / 256), 256, 0, st>>>(D.e_row, e, (int)n, D.s_off);
    HB_LAUNCHED(1);
    pdlp::offsets_kernel<<<(unsigned)((m + 256) / 256), 256, 0, st>>>(L.t_keys, e, (int)m, D.t_off);
    HB_LAUNCHED(1);
    pdlp::gather_edges<<<gb, 256, 0, st>>>(D.e_orig, L.c32, costs, x0, e, D.e_col, D.cost, L.x0s, L.inv);
    HB_LAUNCHED(1);
    pdlp::map_positions<<<gb, 256, 0, st>>>(L.t_orig, L.inv, e, D.t_pos);
    HB_LAUNCHED(1);
    pdlp::degree_scale<<<gb, 256, 0, st>>>(D.s_off, D.t_off, (int)n, (int)m, D.scale);
    HB_LAUNCHED(1);
    // --- norms and scaling (solver.cpp:91-110)
    double h[16];
    pdlp::sumsq2_kernel<<<pdlp::RED_BLOCKS, pdlp::RED_THREADS, 0, st>>>(masses, n + m, costs, e, D.red);
    HB_LAUNCHED(1);
    pdlp::finish_red<<<1, 32, 0, st>>>(D.red, pdlp::RED_BLOCKS, 2, D.scal, 0);
    HB_LAUNCHED(1);
    if (ctl.linf) {  // max norms of b and c for the max-norm termination test (cupdlpx/solver.cu:920-954)
        pdlp::maxabs2_kernel<<<pdlp::RED_BLOCKS, pdlp::RED_THREADS, 0, st>>>(masses, n + m, costs, e, D.red);
        pdlp::finish_red_max<<<1, 32, 0, st>>>(D.red, pdlp::RED_BLOCKS, 0, 2, D.scal, 14);
        HB_LAUNCHED(2);
    }
    if (cudaGetLastError() != cudaSuccess) return fail("setup");
    cudaMemcpyAsync(h, D.scal, 16 * sizeof(double), cudaMemcpyDeviceToHost, st);
    int status = 0;
    cudaMemcpyAsync(&status, D.status, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return fail("setup sync");
    if (status & kErrBadInput) { err = "active-support endpoint index is out of bounds"; return 2; }
    const double mass_norm = std::sqrt(h[0]), cost_norm = std::sqrt(h[1]);
    const double mass_inf = ctl.linf ? h[14] : 0.0, cost_inf = ctl.linf ? h[15] : 0.0;
    const double bound = ctl.rescale ? 1.0 / std::max(1.0, mass_norm) : 1.0;
    const double objective = ctl.rescale ? 1.0 / std::max(1.0, cost_norm) : 1.0;
    const double variable = std::sqrt(2.0);
    const double vb = variable * bound;
    pdlp::init_state<<<gb, 256, 0, st>>>(D, masses, y0, L.x0s, bound, objective, variable);
    HB_LAUNCHED(1);
    double weight = 1.0;
    if (!ctl.rescale) {
        pdlp::sumsq2_kernel<<<pdlp::RED_BLOCKS, pdlp::RED_THREADS, 0, st>>>(D.cs, e, D.bs, n + m, D.red);
        HB_LAUNCHED(1);
        pdlp::finish_red<<<1, 32, 0, st>>>(D.red, pdlp::RED_BLOCKS, 2, D.scal, 0);
        HB_LAUNCHED(1);
        cudaMemcpyAsync(h, D.scal, 2 * sizeof(double), cudaMemcpyDeviceToHost, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail("weight sync");
        weight = std::max(std::sqrt(h[0]) / std::max(std::sqrt(h[1]), 1e-16), 1e-16);
    }
    if (ctl.weight0 > 0) weight = ctl.weight0;
    const double setup_seconds = std::chrono::duration<double>(Clock::now() - started).count();
    const auto iter_started = Clock::now();
    // --- control loop (solver.cpp:157-312)
    const double inf = std::numeric_limits<double>::infinity();
    double best_weight = weight, error_sum = 0.0, best_balance = inf, initial_error = inf, last_trial = inf,
           fixed = inf;
    int64_t count = 0, inner = 0, restarts = 0;
    int reason = 0;
    double pobj = 0, dobj = 0, ap = 0, rp = 0, ad = 0, rd = 0, gap = 0;
    double tap = 0, trp = 0, tad = 0, trd = 0;  // residuals of the termination test
    bool restart = false;
    int tlen = 0;
    const int F = ctl.frequency;
    const bool wide_sources = e >= (int64_t)pdlp::WIDE_DEGREE * n, wide_targets = e >= (int64_t)pdlp::WIDE_DEGREE * m;
    // fused passes (one launch per iteration) unless node sums are atomic or a side is dense
    const bool fused = !ctl.atomic && !wide_sources && !wide_targets;
    // complete row-major support in tree mode: the coalesced target pass
    bool dense_rm = false;
    if (!fused && !ctl.atomic && ctl.tree && wide_targets && e == n * m) {
        int* flag = reinterpret_cast<int*>(D.red);  // reduction scratch, free before the iterations
        cudaMemsetAsync(flag, 0, sizeof(int), st);
        pdlp::check_rowmajor<<<gb, 256, 0, st>>>(D, flag);
        HB_LAUNCHED(1);
        int hflag = 1;
        cudaMemcpyAsync(&hflag, flag, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail("layout check");
        dense_rm = hflag == 0;
    }
    const int per_iter = fused ? 1 : dense_rm ? 3 : (!ctl.atomic && wide_sources && wide_targets) ? 2 : 3;  // kernels per iteration
    // fused passes: persistent blocks (one wave at the kernel's occupancy), half of them per side;
    // stages of 512 edges, two per block (a third stage measured slower, 489 against 394 us per
    // iteration at E = 21M, also with the grid sized to its occupancy), node-scale gathers cached
    // in L2 only
    using FpBig = pdlp::FpCfg<512, 2, 4, true, 256>;
    using FpSmall = pdlp::FpCfg<512, 2, 4, true, 64>;
    // 64-node tiles below about four 256-node tiles per block and side (19.3 against 29.6 us per
    // iteration at n = m = 32768, equal at 131072 and 262144, 256-node tiles 7% faster at 2^20)
    const bool small_tiles = std::max(n, m) < (int64_t)4 * 256 * sms * FpBig::BPS / 2;
    const int fp_tn = small_tiles ? FpSmall::TN : FpBig::TN;
    void (*fp_kernel)(pdlp::Dev, int, int) = small_tiles ? pdlp::fused_pass<FpSmall> : pdlp::fused_pass<FpBig>;
    const size_t fp_bytes = small_tiles ? sizeof(pdlp::FpShared<FpSmall>) : sizeof(pdlp::FpShared<FpBig>);
    using FpDefault = FpBig;
    int fp_per_sm = FpDefault::BPS;  // resident blocks per SM: one wave of persistent blocks
    int runs = 1;
    int parity = 0;  // fused passes: the node-scale buffer the next iteration reads
    if (fused) {
        if (cudaFuncSetAttribute(fp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fp_bytes) != cudaSuccess)
            return fail("fused pass shared memory");
        int occ = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fp_kernel, pdlp::FP_THREADS, fp_bytes) == cudaSuccess &&
            occ > 0)
            fp_per_sm = occ;
        runs = std::max(1, std::min(sms * fp_per_sm / 2, pdlp::FP_MAX_RUNS));
        pdlp::target_copy<<<gb, 256, 0, st>>>(D, 1);
        pdlp::fp_partition<<<(2 * runs + 257) / 256, 256, 0, st>>>(D, runs, fp_tn);
        HB_LAUNCHED(2);
    }
    // One iteration: the three kernels reading D.steps[it].
    auto launch_iteration = [&](cudaStream_t s_, int it, bool counted) {
        if (fused) {
            fp_kernel<<<(unsigned)(2 * runs), pdlp::FP_THREADS, fp_bytes, s_>>>(D, it, runs);
        } else if (ctl.atomic) {
            pdlp::edge_pass<true><<<gb, 256, 0, s_>>>(D, it);
            pdlp::source_pass<true><<<(unsigned)((n + 255) / 256), 256, 0, s_>>>(D, it);
            pdlp::target_pass<true><<<(unsigned)((m + 255) / 256), 256, 0, s_>>>(D, it);
        } else {
            pdlp::edge_pass<false><<<gb, 256, 0, s_>>>(D, it);
            const int sb = wide_sources ? (n + 7) / 8 : 0, tb = wide_targets && !dense_rm ? (m + 7) / 8 : 0;
            if (dense_rm) pdlp::dense_target_pass<<<(unsigned)((m + 31) / 32), 1024, 0, s_>>>(D, it);
            if (sb + tb > 0) {
                if (ctl.tree) pdlp::node_pass_wide<true><<<(unsigned)(sb + tb), 256, 0, s_>>>(D, it, sb);
                else pdlp::node_pass_wide<false><<<(unsigned)(sb + tb), 256, 0, s_>>>(D, it, sb);
            }
            if (!wide_sources) pdlp::source_pass<false><<<(unsigned)((n + 255) / 256), 256, 0, s_>>>(D, it);
            if (!wide_targets) pdlp::target_pass<false><<<(unsigned)((m + 255) / 256), 256, 0, s_>>>(D, it);
        }
        if (counted) HB_LAUNCHED(per_iter);
    };
    // A block of F iterations as one graph (captured on a private stream, launched on st):
    // the fixed-point reductions run after iteration 0 (used when the block starts with a
    // restart; their result is ignored otherwise) and after the last (major) iteration.
    struct Graph {
        cudaStream_t cs = nullptr;
        cudaGraph_t g = nullptr;
        cudaGraphExec_t exec = nullptr;
        ~Graph() {
            if (exec) cudaGraphExecDestroy(exec);
            if (g) cudaGraphDestroy(g);
            if (cs) cudaStreamDestroy(cs);
        }
    } graph;
    std::vector<pdlp::Step> hsteps((size_t)std::min(F, pdlp::STEP_CAP));
    if (F <= pdlp::STEP_CAP && cudaStreamCreateWithFlags(&graph.cs, cudaStreamNonBlocking) == cudaSuccess &&
        cudaStreamBeginCapture(graph.cs, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        for (int t = 0; t < F; ++t) {
            launch_iteration(graph.cs, t, false);  // captured, not launched
            if (t == 0 || t == F - 1) {
                pdlp::fixed_point_kernel<<<pdlp::RED_BLOCKS, pdlp::RED_THREADS, 0, graph.cs>>>(D);
                pdlp::finish_red<<<1, 32, 0, graph.cs>>>(D.red, pdlp::RED_BLOCKS, 3, D.scal, t == F - 1 ? 9 : 5);
            }
        }
        const bool captured = cudaStreamEndCapture(graph.cs, &graph.g) == cudaSuccess && graph.g;
        if (!captured || cudaGraphInstantiate(&graph.exec, graph.g, 0) != cudaSuccess) graph.exec = nullptr;
        cudaGetLastError();  // a failed capture leaves the direct launches below
    }
    for (;;) {
        pdlp::evaluate_kernel<<<pdlp::RED_BLOCKS, pdlp::RED_THREADS, 0, st>>>(D, vb, objective, ctl.linf ? 1 : 0);
        HB_LAUNCHED(1);
        pdlp::finish_red<<<1, 32, 0, st>>>(D.red, pdlp::RED_BLOCKS, 4, D.scal, 0);
        HB_LAUNCHED(1);
        if (ctl.linf) {
            pdlp::finish_red_max<<<1, 32, 0, st>>>(D.red, pdlp::RED_BLOCKS, 4, 2, D.scal, 12);
            HB_LAUNCHED(1);
        }
        if (cudaGetLastError() != cudaSuccess) return fail("evaluate");
        cudaMemcpyAsync(h, D.scal, 16 * sizeof(double), cudaMemcpyDeviceToHost, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail("evaluate sync");
        if (count > 0) {
            // fixed-point errors of the block just run (solver.cpp:304-306), with that block's weight
            auto fpe = [&](int b) {
                const double sq = h[b] * weight + h[b + 1] / weight + 2.0 * 0.998 * h[b + 2];
                return std::sqrt(std::max(0.0, sq));
            };
            fixed = fpe(9);
            if (restart) initial_error = F == 1 ? fixed : fpe(5);
        }
        ap = std::sqrt(h[0]);
        ad = std::sqrt(h[1]);
        pobj = h[2];
        dobj = h[3];
        rp = ap / (1.0 + mass_norm);
        rd = ad / (1.0 + cost_norm);
        gap = std::abs(pobj - dobj) / (1.0 + std::abs(pobj) + std::abs(dobj));
        // the termination test's residuals: L2 (solver.cpp), or the max norm (cuPDLPx "linf")
        tap = ctl.linf ? h[12] : ap;
        tad = ctl.linf ? h[13] : ad;
        trp = ctl.linf ? tap / (1.0 + mass_inf) : rp;
        trd = ctl.linf ? tad / (1.0 + cost_inf) : rd;
        if (trace && tlen < trace_cap) trace[tlen++] = {(double)count, pobj, dobj, trp, trd, gap, weight};
        const bool finite = std::isfinite(pobj) && std::isfinite(dobj) && std::isfinite(ap) && std::isfinite(rp) &&
                            std::isfinite(ad) && std::isfinite(rd) && std::isfinite(gap) && std::isfinite(trp) &&
                            std::isfinite(trd);
        if (!finite || !std::isfinite(weight)) reason = 3;
        else if (trp < ctl.tol_primal && trd < ctl.tol_dual && gap < ctl.tol_objective) reason = 1;
        else if (count >= ctl.iteration_limit) reason = 2;
        else if (std::chrono::duration<double>(Clock::now() - started).count() >= ctl.time_limit) reason = 4;
        if (reason) break;
        restart = false;
        if (count == F) restart = true;
        else if (count > F)
            restart = inner >= 0.36 * count || fixed <= 0.2 * initial_error ||
                      (fixed <= 0.5 * initial_error && fixed > last_trial);
        last_trial = fixed;
        if (restart) {
            pdlp::restart_dist_kernel<<<pdlp::RED_BLOCKS, pdlp::RED_THREADS, 0, st>>>(D);
            HB_LAUNCHED(1);
            pdlp::finish_red<<<1, 32, 0, st>>>(D.red, pdlp::RED_BLOCKS, 2, D.scal, 0);
            HB_LAUNCHED(1);
            cudaMemcpyAsync(h, D.scal, 2 * sizeof(double), cudaMemcpyDeviceToHost, st);
            if (cudaStreamSynchronize(st) != cudaSuccess) return fail("restart sync");
            const double pd = std::sqrt(h[0]), dd = std::sqrt(h[1]);
            const double ratio = rd / std::max(rp, 1e-300);
            if (pd > 1e-16 && pd < 1e12 && dd > 1e-16 && dd < 1e12 && ratio > 1e-8 && ratio < 1e8) {
                const double error = std::log(dd) - std::log(pd) - std::log(weight);
                error_sum = 0.3 * error_sum + error;
                weight *= std::exp(0.99 * error + 0.01 * error_sum);
            } else {
                weight = best_weight;
                error_sum = 0;
            }
            if (rp > 0 && rd > 0) {
                const double balance = std::abs(std::log10(rd / rp));
                if (balance < best_balance) { best_balance = balance; best_weight = weight; }
            }
            inner = 0;
            last_trial = inf;
            ++restarts;
            pdlp::restart_kernel<<<gb, 256, 0, st>>>(D, parity, fused ? 1 : 0);
            HB_LAUNCHED(1);
        }
        const double primal_step = 0.998 / weight, dual_step = 0.998 * weight;
        const bool first_block = count == 0;
        auto step_of = [&](int t) {
            pdlp::Step s;
            s.primal_step = primal_step;
            s.dual_step = dual_step;
            s.halpern = double(inner + t + 1) / double(inner + t + 2);
            s.major = ((count + t + 1) % F) == 0;
            s.checkpoint = s.major || (t == 0 && restart);
            s.parity = fused ? ((parity + t) & 1) : 0;
            s.pad = 0;
            return s;
        };
        if (first_block) timing_mark(st);
        if (graph.exec) {
            for (int t = 0; t < F; ++t) hsteps[t] = step_of(t);
            if (cudaMemcpyAsync(D.steps, hsteps.data(), sizeof(pdlp::Step) * F, cudaMemcpyHostToDevice, st) !=
                    cudaSuccess || cudaGraphLaunch(graph.exec, st) != cudaSuccess)
                return fail("iteration block");
            HB_LAUNCHED(per_iter * F + (F == 1 ? 2 : 4));
        } else {
            for (int t = 0; t < F; ++t) {
                hsteps[0] = step_of(t);
                cudaMemcpyAsync(D.steps, hsteps.data(), sizeof(pdlp::Step), cudaMemcpyHostToDevice, st);
                launch_iteration(st, 0, true);
                if (hsteps[0].checkpoint) {
                    pdlp::fixed_point_kernel<<<pdlp::RED_BLOCKS, pdlp::RED_THREADS, 0, st>>>(D);
                    // scal[5..7]: terms at the restart iteration, scal[9..11]: at the major iteration
                    pdlp::finish_red<<<1, 32, 0, st>>>(D.red, pdlp::RED_BLOCKS, 3, D.scal, hsteps[0].major ? 9 : 5);
                    HB_LAUNCHED(2);
                }
            }
        }
        count += F;
        inner += F;
        if (fused) parity ^= (F & 1);
        if (first_block) timing_mark(st);
        if (cudaGetLastError() != cudaSuccess) return fail("iteration");
    }
    pdlp::output_kernel<<<gb, 256, 0, st>>>(D, vb, objective, x_out, y_out);
    HB_LAUNCHED(1);
    if (cudaStreamSynchronize(st) != cudaSuccess) return fail("output");
    res->iterations = count;
    res->restarts = restarts;
    res->reason = reason;
    res->pobj = pobj; res->dobj = dobj; res->ap = tap; res->rp = trp; res->ad = tad; res->rd = trd; res->gap = gap;
    res->ap2 = ap; res->rp2 = rp; res->ad2 = ad; res->rd2 = rd;
    res->weight = weight;
    res->cost_norm = ctl.linf ? cost_inf : cost_norm;
    res->mass_norm = ctl.linf ? mass_inf : mass_norm;
    res->setup_seconds = setup_seconds;
    res->iteration_seconds = std::chrono::duration<double>(Clock::now() - iter_started).count();
    if (trace_len) *trace_len = tlen;
    return 0;
}

}  // namespace hb
