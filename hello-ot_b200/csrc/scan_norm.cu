// ℓ1 / ℓ∞ / ℓ2 full-space pricing scan on the CUDA cores (sm_100a).
//
// Replaces the reference's direct-norm tiles + selection
// (src/hello_ot/_native/generic_scan/cost.cu:10-85 direct_norm_kernel,
// pricing_small.cu:70-160 scan_kernel, matrix_selection.cuh) with one fused
// persistent kernel per pass: no cost tile reaches HBM.
//
// Distances are accumulated in fp32 over the feature index in increasing
// order (ℓ2 with an fma per term, then sqrtf), so every distance equals the
// sequential fp32 model of the oracle bit for bit.  Score and certificate in
// fp64 as in the reference: score = (g_j - c_ij) + f_i (pricing_small.cu:112).
//
// Tile 128 rows x 128 columns, 256 threads: each thread accumulates an 8x8
// register block from k-major shared-memory slabs; the distance tile is then
// handed through shared memory to a row-per-thread epilogue (two threads per
// row, one per half of the columns) that keeps the row top-k in registers.
#include <algorithm>
#include <string>
#include <type_traits>

#include "../../include/hello_b200.h"
#include "common.cuh"
#include "internal.h"
#include "perturb.cuh"
#include "scan_common.cuh"

namespace hb {
namespace norm {

constexpr int BM = 128, BN = 128, BKS = 8, THREADS = 256;

// Slab position of tile row r: rows ty, ty+16, ty+32, ty+48 of the thread with
// distance-block row ty fill the 16-byte chunk ty, rows ty+64..ty+112 the chunk
// 16 + ty, so a thread reads its 8 values with two 16-byte loads (likewise for
// columns) and the 8 lanes of a load phase read 8 consecutive chunks (no bank
// conflict).
__device__ __forceinline__ int slab_pos(int r) { return (r & 64) | ((r & 15) << 2) | ((r >> 4) & 3); }

struct Smem {
    float xs[2][BKS][BM];  // k-major slabs, rows at slab_pos
    float ys[2][BKS][BN];
    float dist[BM][BN + 1];
    double dbias[BN];      // the tile's column biases
    double rbx[BM];        // the tile's row biases (one-pass column epilogue)
    float cthr[BN];        // the tile's column thresholds (one pass)
    float2 rnz[BM], cnz[BN];  // perturbation: noise inputs of the tile's rows and columns
    double red[8 * 5];
};

struct Params {
    const float* x;  // query features (q x d)
    const float* y;  // database features (n x d)
    int q, n, d;
    bool vec;        // d % 4 == 0 and both feature bases 16-byte aligned
    int groups, tpg, ct, units;
    const double* q_bias;
    const double* d_bias;
    double* part_v;  // [groups*2][q][K]
    int* part_i;
    double* cta_stats;
    // one pass: CTA b owns row group b / groups (rbg row blocks) x column group b % groups
    int rb, rbg;
    int* ckey;      // [ct * BN] column screening thresholds (ordered-int image of fp32)
    double* cval;   // [row groups * 2][n][K] column lists (per row group and row half)
    int* cidx;
    int* progress;  // [grid] tiles started by each CTA
    Perturb pert;   // cost perturbation (sigma == 0: none)
};

template <int KIND>
__device__ __forceinline__ float accumulate(float acc, float a, float b) {
    const float z = a - b;
    if (KIND == 0) return acc + fabsf(z);
    if (KIND == 1) return fmaxf(acc, fabsf(z));
    return fmaf(z, z, acc);
}

// 128 rows x 8 features, stored k-major.  Warp w covers features (w >> 2) * 4..+3
// of 32 rows; lane (a = lane & 7, b = lane >> 3) takes row a + 8 (w & 1) +
// 16 (b + 4 ((w >> 1) & 1)), whose slab position lands in bank 4 a + b, so each
// of the four shared-memory stores is conflict-free.  vec: d % 4 == 0 and a
// 16-byte aligned base, read with one 16-byte load per row.
__device__ __forceinline__ void load_slab(const float* __restrict__ src, int rows_total, int d, int r0, int k0,
                                          float (*dst)[BM], bool vec) {
    const int t = threadIdx.x, w = t >> 5, lane = t & 31;
    const int r = (lane & 7) + 8 * (w & 1) + 16 * ((lane >> 3) + 4 * ((w >> 1) & 1));
    const int kb = (w >> 2) * 4;
    const int gr = r0 + r, pos = slab_pos(r), k = k0 + kb;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (gr < rows_total) {
        const float* row = src + (int64_t)gr * d;
        if (vec) {
            if (k < d) {
                const float4 f = *reinterpret_cast<const float4*>(row + k);
                v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = k + j < d ? row[k + j] : 0.0f;
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[kb + j][pos] = v[j];
}

// Order-preserving integer image of an fp32 value (atomicMax on thresholds).
__device__ __forceinline__ int order_key(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float order_value(int key) { return __int_as_float(key >= 0 ? key : key ^ 0x7FFFFFFF); }

// One pass: a column group's CTAs (one per row group) stream the same column
// tiles; each stays within PACE tiles of the slowest so the tiles one of them
// reads are still in L2 for the others.  The wait is bounded (PACE_SPINS
// sleeps, then it proceeds): no CTA depends on another making progress.
constexpr int PACE = 2, PACE_SPINS = 64;
__device__ __forceinline__ void pace(const Params& p, int t) {
    volatile int* prog = p.progress;
    prog[blockIdx.x] = t;
    const int g = blockIdx.x % p.groups, gr = gridDim.x / p.groups;
    for (int spin = 0; spin < PACE_SPINS; ++spin) {
        int slow = INT32_MAX;
        for (int r = 0; r < gr; ++r) slow = min(slow, prog[r * p.groups + g]);
        if (t - slow <= PACE) return;
        __nanosleep(500);
    }
}

// ONE (one pass, K <= 8): after the row epilogue, thread (column c, row half h)
// screens the 64 rows of its half against the column's threshold and inserts
// the candidates into the column's list for (row group, h) in HBM; a full list
// raises the shared threshold.  Scores are the row epilogue's: (g - c) + f.
template <int KIND, int K, bool STATS, bool SWAP, bool ONE>
__global__ void __launch_bounds__(THREADS, 2) scan_kernel(const Params p) {
    extern __shared__ uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    constexpr int KK = K > 0 ? K : 1;
    const int t = threadIdx.x;
    const int ty = t >> 4, tx = t & 15;           // distance block: rows ty+16i, cols tx+16j
    const int er = t & (BM - 1), half = t >> 7;   // epilogue: row er, columns half*64..+63
    double acc[5] = {0, 0, 0, 0, 0};
    TopK<KK> top;
    int u0 = blockIdx.x, ustep = gridDim.x, uend = p.units;
    if (ONE) {
        const int rg = blockIdx.x / p.groups, g = blockIdx.x % p.groups;
        const int rb0 = rg * p.rbg, rb1 = min(p.rb, rb0 + p.rbg);
        u0 = rb0 * p.groups + g; ustep = p.groups; uend = rb1 > rb0 ? rb1 * p.groups : 0;
    }
    const int64_t list_base = ONE ? (int64_t)((blockIdx.x / p.groups) * 2 + half) * p.n : 0;
    const bool perturbed = p.pert.sigma != 0.0;
    // the cost of tile entry (rl, cl) in fp64, with the perturbation noise when it is on
    auto pcost = [&](int rl, int cl) -> double {
        const double c = (double)s.dist[rl][cl];
        return perturbed ? c + noise_of(p.pert, s.rnz[rl], s.cnz[cl]) : c;
    };
    int tile = 0;
    for (int u = u0; u < uend; u += ustep) {
        const int rb = u / p.groups, g = u % p.groups;
        const int ct1 = min(p.ct, (g + 1) * p.tpg);
        const int row = rb * BM + er;
        const bool rvalid = row < p.q;
        // no query bias: add -0.0, the exact identity (keeps g - c bit for bit, signed zeros included)
        const double rbias = rvalid && p.q_bias ? p.q_bias[row] : -0.0;
        top.reset();
        for (int ct = g * p.tpg; ct < ct1; ++ct, ++tile) {
            const int c0 = ct * BN;
            if (ONE && t == 0) pace(p, tile);
            float dist[8][8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) dist[i][j] = 0.0f;
            const int nslab = (p.d + BKS - 1) / BKS;
            load_slab(p.x, p.q, p.d, rb * BM, 0, s.xs[0], p.vec);
            load_slab(p.y, p.n, p.d, c0, 0, s.ys[0], p.vec);
            __syncthreads();
            for (int sl = 0; sl < nslab; ++sl) {
                const int cur = sl & 1;
                if (sl + 1 < nslab) {
                    load_slab(p.x, p.q, p.d, rb * BM, (sl + 1) * BKS, s.xs[cur ^ 1], p.vec);
                    load_slab(p.y, p.n, p.d, c0, (sl + 1) * BKS, s.ys[cur ^ 1], p.vec);
                }
                // the slab's features below d, in increasing order (the slab rows past d
                // hold zeros and are not read); not unrolled: unrolling hoists the slab
                // loads and spills the 8x8 block
                const int kend = min(BKS, p.d - sl * BKS);
#pragma unroll 1
                for (int k = 0; k < kend; ++k) {
                    const float4 xa = *reinterpret_cast<const float4*>(&s.xs[cur][k][ty * 4]);
                    const float4 xb = *reinterpret_cast<const float4*>(&s.xs[cur][k][64 + ty * 4]);
                    const float4 ya = *reinterpret_cast<const float4*>(&s.ys[cur][k][tx * 4]);
                    const float4 yb = *reinterpret_cast<const float4*>(&s.ys[cur][k][64 + tx * 4]);
                    const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                    const float yv[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i)
#pragma unroll
                        for (int j = 0; j < 8; ++j) dist[i][j] = accumulate<KIND>(dist[i][j], xv[i], yv[j]);
                }
                __syncthreads();
            }
            // hand the tile to the row-per-thread epilogue
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    s.dist[ty + 16 * i][tx + 16 * j] = KIND == 2 ? sqrtf(dist[i][j]) : dist[i][j];
            const int ncols = min(BN, p.n - c0);
            if (t < BN) {
                s.dbias[t] = t < ncols ? p.d_bias[c0 + t] : 0.0;
                if (ONE) {
                    s.rbx[t] = rbias;  // thread t < BM owns row t (half 0)
                    s.cthr[t] = t < ncols ? order_value(p.ckey[c0 + t]) : INFINITY;
                }
                if (perturbed) {
                    s.cnz[t] = t < ncols ? noise_input(p.pert, p.pert.col_index[c0 + t]) : make_float2(0.f, 0.f);
                    s.rnz[t] = rvalid ? noise_input(p.pert, p.pert.row_index[row]) : make_float2(0.f, 0.f);
                }
            }
            __syncthreads();
            if (rvalid) {
                const int cb0 = half * 64;
                const int live = min(64, ncols - cb0);  // valid columns of this half
                const double tv = top.v[KK - 1];
                uint64_t mask = 0;
                double num4[4] = {0, 0, 0, 0}, den4[4] = {0, 0, 0, 0};
                double mpos = 0.0, mcost = 0.0;
                int cnt = 0;
                // phase 1: scores, certificate terms and the candidate mask, in chunks of 16
                // columns with constant mask bits; FULL (all 64 columns valid) drops the
                // column checks.  The mask screens with sc >= the list's k-th score, a
                // superset of the columns that beat it: phase 2's offer() decides exactly.
                auto phase1 = [&](auto full) {
                    constexpr bool FULL = decltype(full)::value;
#pragma unroll 1
                    for (int jb = 0; jb < 64; jb += 16) {
                        uint32_t m16 = 0;
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            const int j = jb + u;
                            const bool ok = FULL || j < live;
                            const double cost = pcost(er, cb0 + j);
                            const double cbias = s.dbias[cb0 + j];
                            const double sc = SWAP ? ((rbias - cost) + cbias) : ((cbias - cost) + rbias);
                            if (STATS && ok) {
                                den4[u & 3] = fma(cost, cost, den4[u & 3]);
                                mcost = fmax(mcost, fabs(cost));
                                if (sc > 0.0) {
                                    num4[u & 3] = fma(sc, sc, num4[u & 3]);
                                    mpos = fmax(mpos, sc);
                                    ++cnt;
                                }
                            }
                            if (K > 0 && ok && sc >= tv) m16 |= 1u << u;
                        }
                        mask |= (uint64_t)m16 << jb;
                    }
                };
                if (live == 64) phase1(std::true_type{});
                else phase1(std::false_type{});
                if (STATS) {
                    acc[0] += (num4[0] + num4[1]) + (num4[2] + num4[3]);
                    acc[1] += (den4[0] + den4[1]) + (den4[2] + den4[3]);
                    acc[2] = fmax(acc[2], mpos);
                    acc[3] = fmax(acc[3], mcost);
                    acc[4] += (double)cnt;
                }
                // phase 2: insert the masked columns (rare once the list has filled)
                while (K > 0 && mask) {
                    const int j = __ffsll(mask) - 1;
                    mask &= mask - 1;
                    const double cost = pcost(er, cb0 + j);
                    const double cbias = s.dbias[cb0 + j];
                    const double sc = SWAP ? ((rbias - cost) + cbias) : ((cbias - cost) + rbias);
                    top.offer(sc, c0 + cb0 + j);
                }
            }
            if (ONE && K > 0) {  // column side: thread (column er, row half `half`)
                const int c = er, r0 = half * 64;
                const int rlive = min(64, p.q - rb * BM - r0);  // valid rows of this half
                if (c < ncols && rlive > 0) {
                    const double cb = s.dbias[c];
                    const double thr = (double)s.cthr[c];
                    uint64_t cmask = 0;
                    auto screen = [&](auto full) {
                        constexpr bool FULL = decltype(full)::value;
#pragma unroll 1
                        for (int rbk = 0; rbk < 64; rbk += 16) {
                            uint32_t m16 = 0;
#pragma unroll
                            for (int u = 0; u < 16; ++u) {
                                const int r = rbk + u;
                                const double sc = (cb - pcost(r0 + r, c)) + s.rbx[r0 + r];
                                if ((FULL || r < rlive) && sc >= thr) m16 |= 1u << u;
                            }
                            cmask |= (uint64_t)m16 << rbk;
                        }
                    };
                    if (rlive == 64) screen(std::true_type{});
                    else screen(std::false_type{});
                    if (cmask) {
                        const int64_t base = (list_base + c0 + c) * KK;
                        TopK<KK> cl;
#pragma unroll
                        for (int q2 = 0; q2 < KK; ++q2) { cl.v[q2] = p.cval[base + q2]; cl.i[q2] = p.cidx[base + q2]; }
                        while (cmask) {
                            const int r = __ffsll(cmask) - 1;
                            cmask &= cmask - 1;
                            cl.offer((cb - pcost(r0 + r, c)) + s.rbx[r0 + r], rb * BM + r0 + r);
                        }
#pragma unroll
                        for (int q2 = 0; q2 < KK; ++q2) { p.cval[base + q2] = cl.v[q2]; p.cidx[base + q2] = cl.i[q2]; }
                        if (cl.i[KK - 1] != INT32_MAX)
                            atomicMax(p.ckey + c0 + c, order_key(__double2float_rd(cl.v[KK - 1])));
                    }
                }
            }
            __syncthreads();
        }
        if (K > 0 && rvalid) {
            const int part = g * 2 + half;
            double* pv = p.part_v + ((int64_t)part * p.q + row) * KK;
            int* pi = p.part_i + ((int64_t)part * p.q + row) * KK;
#pragma unroll
            for (int j = 0; j < KK; ++j) { pv[j] = top.v[j]; pi[j] = top.i[j]; }
        }
    }
    if (ONE && t == 0) *(volatile int*)(p.progress + blockIdx.x) = INT32_MAX;  // done: never wait for this CTA
    if (STATS) {
        const int lane = t & 31, w = t >> 5;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const double o0 = __shfl_down_sync(0xffffffffu, acc[0], off);
            const double o1 = __shfl_down_sync(0xffffffffu, acc[1], off);
            const double o2 = __shfl_down_sync(0xffffffffu, acc[2], off);
            const double o3 = __shfl_down_sync(0xffffffffu, acc[3], off);
            const double o4 = __shfl_down_sync(0xffffffffu, acc[4], off);
            acc[0] += o0; acc[1] += o1; acc[2] = fmax(acc[2], o2); acc[3] = fmax(acc[3], o3); acc[4] += o4;
        }
        if (lane == 0)
            for (int j = 0; j < 5; ++j) s.red[w * 5 + j] = acc[j];
        __syncthreads();
        if (t == 0) {
            double a[5] = {0, 0, 0, 0, 0};
            for (int ww = 0; ww < THREADS / 32; ++ww) {
                a[0] += s.red[ww * 5 + 0]; a[1] += s.red[ww * 5 + 1];
                a[2] = fmax(a[2], s.red[ww * 5 + 2]); a[3] = fmax(a[3], s.red[ww * 5 + 3]);
                a[4] += s.red[ww * 5 + 4];
            }
            for (int j = 0; j < 5; ++j) p.cta_stats[blockIdx.x * 5 + j] = a[j];
        }
    }
}

}  // namespace norm

namespace {

template <int KIND, int K, bool STATS, bool SWAP, bool ONE = false>
cudaError_t norm_launch(const norm::Params& p, int grid, cudaStream_t st) {
    auto fn = norm::scan_kernel<KIND, K, STATS, SWAP, ONE>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(norm::Smem));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    timing_mark(st);
    fn<<<grid, norm::THREADS, sizeof(norm::Smem), st>>>(p);
    timing_mark(st);
    count_launches(1);
    return cudaGetLastError();
}

template <int KIND, bool STATS, bool SWAP>
cudaError_t norm_k(int K, const norm::Params& p, int grid, cudaStream_t st) {
    switch (K) {
        case 0: return norm_launch<KIND, 0, STATS, SWAP>(p, grid, st);
        case 1: return norm_launch<KIND, 1, STATS, SWAP>(p, grid, st);
        case 2: return norm_launch<KIND, 2, STATS, SWAP>(p, grid, st);
        case 4: return norm_launch<KIND, 4, STATS, SWAP>(p, grid, st);
        case 8: return norm_launch<KIND, 8, STATS, SWAP>(p, grid, st);
        case 16: return norm_launch<KIND, 16, STATS, SWAP>(p, grid, st);
        case 32: return norm_launch<KIND, 32, STATS, SWAP>(p, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

template <int KIND, bool STATS>
cudaError_t norm_one_k(int K, const norm::Params& p, int grid, cudaStream_t st) {
    switch (K) {
        case 1: return norm_launch<KIND, 1, STATS, false, true>(p, grid, st);
        case 2: return norm_launch<KIND, 2, STATS, false, true>(p, grid, st);
        case 4: return norm_launch<KIND, 4, STATS, false, true>(p, grid, st);
        case 8: return norm_launch<KIND, 8, STATS, false, true>(p, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

template <bool STATS>
cudaError_t norm_one(int kind, int K, const norm::Params& p, int grid, cudaStream_t st) {
    switch (kind) {
        case 0: return norm_one_k<0, STATS>(K, p, grid, st);
        case 1: return norm_one_k<1, STATS>(K, p, grid, st);
        case 2: return norm_one_k<2, STATS>(K, p, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

__global__ void init_norm_columns(double* cval, int* cidx, int* ckey, int64_t lists, int64_t nkeys, int K) {
    const int64_t total = lists * K > nkeys ? lists * K : nkeys;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        if (e < lists * K) { cval[e] = -INFINITY; cidx[e] = INT32_MAX; }
        if (e < nkeys) ckey[e] = norm::order_key(-INFINITY);
    }
}

template <bool STATS, bool SWAP>
cudaError_t norm_kind(int kind, int K, const norm::Params& p, int grid, cudaStream_t st) {
    switch (kind) {
        case 0: return norm_k<0, STATS, SWAP>(K, p, grid, st);
        case 1: return norm_k<1, STATS, SWAP>(K, p, grid, st);
        case 2: return norm_k<2, STATS, SWAP>(K, p, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace

struct NormLayout {
    double *pv1 = nullptr, *pv2 = nullptr, *cta = nullptr;
    int *pi1 = nullptr, *pi2 = nullptr;
    ScanPlan p1{}, p2{};
    // one pass (1 <= K <= 8): rectangles of gr row groups x gc column groups
    bool one = false;
    int gr = 0, rbg = 0, gc = 0, tpg = 0, rb = 0, ct = 0, grid = 0;
    double* cval = nullptr;
    int *cidx = nullptr, *ckey = nullptr, *progress = nullptr;
    size_t bytes = 0;
    bool ok = true;
};

constexpr int NORM_ONE_PASS_ROW_GROUPS = 8;

NormLayout norm_layout(void* base, size_t size, int64_t q, int64_t n, int k, bool one) {
    NormLayout L;
    const int sms = sm_count();
    const int K = k > 0 ? bucket_of(k) : 0;
    Arena ar{static_cast<char*>(base), size, 0};
    auto fail_if = [&](const void* ptr) { if (base && !ptr) L.ok = false; };
    L.one = one && K >= 1 && K <= 8;
    if (L.one) {
        L.rb = (int)((q + norm::BM - 1) / norm::BM);
        L.ct = (int)((n + norm::BN - 1) / norm::BN);
        L.gr = std::min(NORM_ONE_PASS_ROW_GROUPS, L.rb);
        L.rbg = (L.rb + L.gr - 1) / L.gr;
        L.gr = (L.rb + L.rbg - 1) / L.rbg;
        const int gc = std::min(L.ct, std::max(1, 2 * sms / L.gr));  // two CTAs per SM
        L.tpg = (L.ct + gc - 1) / gc;
        L.gc = (L.ct + L.tpg - 1) / L.tpg;
        L.grid = L.gr * L.gc;
        const size_t lists = (size_t)L.gr * 2 * n;
        L.pv1 = ar.take<double>((size_t)L.gc * 2 * q * K); fail_if(L.pv1);
        L.pi1 = ar.take<int>((size_t)L.gc * 2 * q * K); fail_if(L.pi1);
        L.cval = ar.take<double>(lists * K); fail_if(L.cval);
        L.cidx = ar.take<int>(lists * K); fail_if(L.cidx);
        L.ckey = ar.take<int>((size_t)L.ct * norm::BN); fail_if(L.ckey);
        L.progress = ar.take<int>((size_t)L.grid); fail_if(L.progress);
        L.cta = ar.take<double>((size_t)L.grid * 5); fail_if(L.cta);
    } else {
        L.p1 = scan_plan(q, n, norm::BM, norm::BN, 2, sms, 1);
        L.p2 = scan_plan(n, q, norm::BM, norm::BN, 2, sms, 1);
        if (K > 0) {
            L.pv1 = ar.take<double>((size_t)L.p1.groups * 2 * q * K); fail_if(L.pv1);
            L.pi1 = ar.take<int>((size_t)L.p1.groups * 2 * q * K); fail_if(L.pi1);
            L.pv2 = ar.take<double>((size_t)L.p2.groups * 2 * n * K); fail_if(L.pv2);
            L.pi2 = ar.take<int>((size_t)L.p2.groups * 2 * n * K); fail_if(L.pi2);
        }
        L.cta = ar.take<double>((size_t)(L.p1.grid > L.p2.grid ? L.p1.grid : L.p2.grid) * 5); fail_if(L.cta);
    }
    L.bytes = ar.used + 256;
    return L;
}

// One workspace size serves both modes.
size_t norm_bytes(int64_t q, int64_t n, int k) {
    return std::max(norm_layout(nullptr, 0, q, n, k, false).bytes, norm_layout(nullptr, 0, q, n, k, true).bytes);
}

int norm_scan(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* f, const double* g,
              int kind, int k, int want_stats, double* rv, int* ri, double* cv, int* ci, double* stats5, void* ws,
              size_t ws_bytes, cudaStream_t st, std::string& err, bool rows_only, const Perturb* pert) {
    const bool two_pass = (kind & HB_NORM_TWO_PASS) != 0;
    kind &= 0xF;
    const int K = k > 0 ? bucket_of(k) : 0;
    NormLayout L = norm_layout(ws, ws_bytes, q, n, k, !rows_only && !two_pass);
    if (!L.ok) { err = "workspace too small for the norm scan"; return 3; }
    norm::Params p{};
    p.x = x; p.y = y; p.q = (int)q; p.n = (int)n; p.d = (int)d;
    p.vec = d % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
    p.q_bias = f; p.d_bias = g;
    p.part_v = L.pv1; p.part_i = L.pi1; p.cta_stats = L.cta;
    if (pert && pert->sigma != 0.0) p.pert = *pert;
    cudaError_t e;
    if (L.one) {
        const int blocks = sm_count() * 8;
        init_norm_columns<<<blocks, 256, 0, st>>>(L.cval, L.cidx, L.ckey, (int64_t)L.gr * 2 * n,
                                                  (int64_t)L.ct * norm::BN, K);
        count_launches(1);
        e = cudaMemsetAsync(L.progress, 0, sizeof(int) * L.grid, st);
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
        p.groups = L.gc; p.tpg = L.tpg; p.ct = L.ct; p.units = L.rb * L.gc;
        p.rb = L.rb; p.rbg = L.rbg;
        p.ckey = L.ckey; p.cval = L.cval; p.cidx = L.cidx; p.progress = L.progress;
        e = want_stats ? norm_one<true>(kind, K, p, L.grid, st) : norm_one<false>(kind, K, p, L.grid, st);
        if (e != cudaSuccess) { err = std::string("norm scan: ") + cudaGetErrorString(e); return 6; }
        if (want_stats) { finalize_stats<<<1, 32, 0, st>>>(L.cta, L.grid, stats5); count_launches(1); }
        e = merge_any(K, L.pv1, L.pi1, L.gc * 2, q, k, rv, ri, st);
        if (e == cudaSuccess) e = merge_any(K, L.cval, L.cidx, L.gr * 2, n, k, cv, ci, st);
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
        return 0;
    }
    p.groups = L.p1.groups; p.tpg = L.p1.tpg; p.ct = L.p1.ct; p.units = L.p1.units;
    e = want_stats ? norm_kind<true, false>(kind, K, p, L.p1.grid, st)
                   : norm_kind<false, false>(kind, K, p, L.p1.grid, st);
    if (e != cudaSuccess) { err = std::string("norm pass 1: ") + cudaGetErrorString(e); return 6; }
    if (want_stats) { finalize_stats<<<1, 32, 0, st>>>(L.cta, L.p1.grid, stats5); count_launches(1); }
    if (K > 0) {
        e = merge_any(K, L.pv1, L.pi1, L.p1.groups * 2, q, k, rv, ri, st);
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
    }
    if (K > 0 && !rows_only) {
        norm::Params p2 = p;
        p2.x = y; p2.y = x; p2.q = (int)n; p2.n = (int)q;
        p2.groups = L.p2.groups; p2.tpg = L.p2.tpg; p2.ct = L.p2.ct; p2.units = L.p2.units;
        p2.q_bias = g; p2.d_bias = f;
        p2.part_v = L.pv2; p2.part_i = L.pi2;
        std::swap(p2.pert.row_index, p2.pert.col_index);  // rows are the targets now
        p2.pert.row_is_source = !p.pert.row_is_source;
        e = norm_kind<false, true>(kind, K, p2, L.p2.grid, st);
        if (e != cudaSuccess) { err = std::string("norm pass 2: ") + cudaGetErrorString(e); return 6; }
        e = merge_any(K, L.pv2, L.pi2, L.p2.groups * 2, n, k, cv, ci, st);
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
    }
    return 0;
}

}  // namespace hb

// ---------------------------------------------------------------------------
// Allocation-free norm scan.  The scratch (partial top-k lists and per-CTA
// certificate partials) lives in this file-scope device array instead of a
// caller-provided workspace; every GPU that loads the library holds it until
// the process exits.  In host code `g_norm_scratch` is only a host-side stand-in
// for the symbol, so every call looks up its device address on the current
// device and passes that to the kernels.  The address is not cached: after a
// cudaDeviceReset the module is loaded again and the array may move.
static __device__ __align__(256) unsigned char g_norm_scratch[HB_NORM_NOALLOC_SCRATCH_BYTES];

namespace {
// Device address of g_norm_scratch on the current device.
cudaError_t norm_scratch_address(void** out) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_norm_scratch);
    if (e != cudaSuccess) return e;
    *out = ptr;
    return cudaSuccess;
}
}  // namespace

extern "C" int hb_norm_scan_noalloc(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* f,
                                    const double* g, int cost_type, int k, int compute_stats, double* row_vals,
                                    int32_t* row_idx, double* col_vals, int32_t* col_idx, double* stats5,
                                    void* stream) {
    using namespace hb;
    if (!x || !y || !f || !g) return abi_fail(HB_BAD_ARGUMENT, "null input pointer");
    if (q < 1 || n < 1 || d < 1 || q >= INT32_MAX || n >= INT32_MAX || d >= INT32_MAX)
        return abi_fail(HB_BAD_ARGUMENT, "q, n, d must be in [1, 2^31)");
    if ((cost_type & ~HB_NORM_TWO_PASS) < 0 || (cost_type & ~HB_NORM_TWO_PASS) > 2)
        return abi_fail(HB_BAD_ARGUMENT, "cost_type must be 0 (l1), 1 (linf) or 2 (l2), optionally | HB_NORM_TWO_PASS");
    if (k < 0 || k > 32) return abi_fail(HB_BAD_ARGUMENT, "k must be in 0..32");
    if (k > 0 && (!row_vals || !row_idx || !col_vals || !col_idx)) return abi_fail(HB_BAD_ARGUMENT, "null output pointer");
    if (compute_stats && !stats5) return abi_fail(HB_BAD_ARGUMENT, "null stats pointer");
    const size_t need = norm_bytes(q, n, k);
    if (need > (size_t)HB_NORM_NOALLOC_SCRATCH_BYTES)
        return abi_fail(HB_WORKSPACE, "hb_norm_scan_noalloc: this problem needs " + std::to_string(need) +
                                          " bytes of scratch but the static buffer holds " +
                                          std::to_string((size_t)HB_NORM_NOALLOC_SCRATCH_BYTES) +
                                          "; use hb_norm_scan with a workspace");
    void* scratch = nullptr;
    cudaError_t e = norm_scratch_address(&scratch);
    if (e != cudaSuccess)
        return abi_fail(HB_CUDA, std::string("hb_norm_scan_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::string err;
    int rc = norm_scan(x, y, q, n, d, f, g, cost_type, k, compute_stats, row_vals, row_idx, col_vals, col_idx, stats5,
                       scratch, (size_t)HB_NORM_NOALLOC_SCRATCH_BYTES, st, err);
    if (rc) return abi_fail(rc == 3 ? HB_WORKSPACE : HB_LAUNCH, err);
    return abi_finish(st, "norm scan (no alloc)");
}

