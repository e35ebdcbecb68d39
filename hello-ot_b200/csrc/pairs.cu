// Active-support pair costs (SDDMM): one cost per (row, col) edge.
//
// ℓ2²: c_e = (a_r + b_c) - s<x_r, y_c>   replaces the CSR-blocked
//      torch.sparse.sampled_addmm of src/hello_ot/costs/pairs.py:221-440
// ℓ1 / ℓ∞ / ℓ2: fp64 accumulation of (double)y - (double)x per feature,
//      replaces gcost_sparse_pairs_kernel,
//      src/hello_ot/_native/norm_cost_scan/norm_cost_scan_kernel.cu:234-245
//
// All arithmetic is fp64 on the fp32 features (products of two fp32 values are
// exact in fp64).  A group of G lanes serves one edge and reads the two
// feature rows with 128-bit loads when the rows are 16-byte aligned; the
// group reduces with a fixed xor-shuffle tree, so results are deterministic.
// Each warp takes one contiguous block of edges, so the source row of edges
// grouped by source (the reference's CSR-blocked order) is read from HBM once
// and then from L1.  HBM-bound: every edge gathers its database row once.
#include <string>

#include "common.cuh"
#include "internal.h"
#include "perturb.cuh"

namespace hb {
namespace pairs {

template <int KIND>
__device__ __forceinline__ double step(double acc, float a, float b) {
    if (KIND == 3) return fma((double)a, (double)b, acc);
    const double z = (double)b - (double)a;
    if (KIND == 0) return acc + fabs(z);
    if (KIND == 1) return fmax(acc, fabs(z));
    return fma(z, z, acc);
}

template <int KIND>
__device__ __forceinline__ double combine(double a, double b) {
    return KIND == 1 ? fmax(a, b) : a + b;
}

template <int KIND, int G, bool VEC>
__global__ void __launch_bounds__(256) pair_kernel(const float* __restrict__ x, const float* __restrict__ y, int64_t nx,
                                                   int64_t ny, int d, const double* __restrict__ a,
                                                   const double* __restrict__ b, double scale,
                                                   const int64_t* __restrict__ rows, const int64_t* __restrict__ cols,
                                                   int64_t count, double* __restrict__ out, int* status,
                                                   const Perturb pert) {
    // warp-uniform loop: each warp walks its own contiguous block of edges,
    // 32/G consecutive edges per step
    const int lane = threadIdx.x & 31, sub = lane & (G - 1);
    const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    constexpr int EPW = 32 / G;
    const int64_t per_warp = ((count + warps - 1) / warps + EPW - 1) / EPW * EPW;
    const int64_t e_end = min(count, (warp_id + 1) * per_warp);
    for (int64_t eb = warp_id * per_warp; eb < e_end; eb += EPW) {
        const int64_t e = eb + lane / G;
        const bool live = e < e_end;
        const int64_t r = live ? rows[e] : 0, c = live ? cols[e] : 0;
        const bool ok = live && r >= 0 && r < nx && c >= 0 && c < ny;
        double acc = 0.0;
        if (ok) {
            const float* xr = x + r * d;
            const float* yc = y + c * d;
            if (VEC) {
                const float4* x4 = reinterpret_cast<const float4*>(xr);
                const float4* y4 = reinterpret_cast<const float4*>(yc);
                for (int k = sub; k < d / 4; k += G) {
                    const float4 u = __ldg(x4 + k), v = __ldg(y4 + k);
                    acc = step<KIND>(acc, u.x, v.x);
                    acc = step<KIND>(acc, u.y, v.y);
                    acc = step<KIND>(acc, u.z, v.z);
                    acc = step<KIND>(acc, u.w, v.w);
                }
            } else {
                for (int k = sub; k < d; k += G) acc = step<KIND>(acc, __ldg(xr + k), __ldg(yc + k));
            }
        }
#pragma unroll
        for (int off = G / 2; off > 0; off >>= 1) acc = combine<KIND>(acc, __shfl_xor_sync(0xffffffffu, acc, off, G));
        if (sub == 0 && live) {
            if (!ok) {
                atomicOr(status, kErrBadInput);
                out[e] = __longlong_as_double(0x7ff8000000000000LL);
            } else if (KIND == 3) {
                out[e] = (a[r] + b[c]) - scale * acc;
            } else {
                const double dist = KIND == 2 ? sqrt(acc) : acc;
                // perturbed norm costs: the noise of (source row, target column) added in fp64
                out[e] = pert.sigma != 0.0 ? dist + noise_of(pert, noise_input(pert, pert.row_index[r]),
                                                                noise_input(pert, pert.col_index[c]))
                                           : dist;
            }
        }
    }
}

// d = 128 NV with 16-byte-aligned rows: a warp per edge, lane l holding the float4 chunks
// l + 32 v (v < NV) of the source row converted to fp64 in registers while consecutive edges
// share the source row (the reference's source-grouped order), so each edge converts only
// its target row.  The same chunks, order and reduction tree as pair_kernel<KIND, 32, true>:
// the results are identical.
template <int KIND, int NV>
__global__ void __launch_bounds__(256, NV <= 1 ? 4 : NV == 2 ? 3 : 2) pair_kernel_rows(const float* __restrict__ x, const float* __restrict__ y,
                                                        int64_t nx, int64_t ny, int d, const double* __restrict__ a,
                                                        const double* __restrict__ b, double scale,
                                                        const int64_t* __restrict__ rows,
                                                        const int64_t* __restrict__ cols, int64_t count,
                                                        double* __restrict__ out, int* status, const Perturb pert) {
    const int lane = threadIdx.x & 31;
    const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t per_warp = (count + warps - 1) / warps;
    const int64_t e_end = min(count, (warp_id + 1) * per_warp);
    // one edge ahead: the next edge's indices, target row chunks and (when it starts a new
    // source row) source row chunks are loaded before this edge's arithmetic
    double xd[NV * 4];
    float4 yv[NV], yn[NV], xn[NV];
    int64_t e = warp_id * per_warp;
    int64_t r = 0, c = 0, held = -1;
    bool ok = false, fresh = false;  // fresh: xn holds this edge's source row (a new one)
    auto fetch = [&](int64_t ee, int64_t prev, int64_t& rr, int64_t& cc, bool& okk, bool& fr) {
        rr = rows[ee];
        cc = cols[ee];
        okk = rr >= 0 && rr < nx && cc >= 0 && cc < ny;
        fr = okk && rr != prev;
        if (okk) {
            const float4* y4 = reinterpret_cast<const float4*>(y + cc * d);
#pragma unroll
            for (int v = 0; v < NV; ++v) yn[v] = __ldg(y4 + lane + 32 * v);
        }
        if (fr) {
            const float4* x4 = reinterpret_cast<const float4*>(x + rr * d);
#pragma unroll
            for (int v = 0; v < NV; ++v) xn[v] = __ldg(x4 + lane + 32 * v);
        }
    };
    if (e < e_end) fetch(e, held, r, c, ok, fresh);
    for (; e < e_end; ++e) {  // warp-uniform
        if (fresh) {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                xd[4 * v] = xn[v].x; xd[4 * v + 1] = xn[v].y; xd[4 * v + 2] = xn[v].z; xd[4 * v + 3] = xn[v].w;
            }
            held = r;
        }
#pragma unroll
        for (int v = 0; v < NV; ++v) yv[v] = yn[v];
        const int64_t rc = r, cc = c;
        const bool okc = ok;
        if (e + 1 < e_end) fetch(e + 1, held, r, c, ok, fresh);
        double acc = 0.0;
        if (okc) {
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const float yy[4] = {yv[v].x, yv[v].y, yv[v].z, yv[v].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const double xa = xd[4 * v + j], yb = (double)yy[j];
                    if (KIND == 3) {
                        acc = fma(xa, yb, acc);
                    } else {
                        const double z = yb - xa;
                        acc = KIND == 0 ? acc + fabs(z) : KIND == 1 ? fmax(acc, fabs(z)) : fma(z, z, acc);
                    }
                }
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc = combine<KIND>(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        if (lane == 0) {
            if (!okc) {
                atomicOr(status, kErrBadInput);
                out[e] = __longlong_as_double(0x7ff8000000000000LL);
            } else if (KIND == 3) {
                out[e] = (a[rc] + b[cc]) - scale * acc;
            } else {
                const double dist = KIND == 2 ? sqrt(acc) : acc;
                out[e] = pert.sigma != 0.0 ? dist + noise_of(pert, noise_input(pert, pert.row_index[rc]),
                                                                noise_input(pert, pert.col_index[cc]))
                                           : dist;
            }
        }
    }
}

template <int KIND, int G>
void launch_g(bool vec, const float* x, const float* y, int64_t nx, int64_t ny, int d, const double* a,
              const double* b, double s, const int64_t* rows, const int64_t* cols, int64_t count, double* out,
              int* status, int blocks, cudaStream_t st, const Perturb& pert) {
    timing_mark(st);
    if (vec)
        pair_kernel<KIND, G, true><<<blocks, 256, 0, st>>>(x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, pert);
    else
        pair_kernel<KIND, G, false><<<blocks, 256, 0, st>>>(x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, pert);
    timing_mark(st);
    count_launches(1);
}

template <int KIND>
void launch_kind(const float* x, const float* y, int64_t nx, int64_t ny, int d, const double* a, const double* b,
                 double s, const int64_t* rows, const int64_t* cols, int64_t count, double* out, int* status,
                 cudaStream_t st, int sms, const Perturb& pert) {
    const bool vec = (d % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) % 16 == 0);
    const int chunks = vec ? d / 4 : d;  // loads per edge
    const int g = chunks <= 1 ? 1 : chunks <= 2 ? 2 : chunks <= 4 ? 4 : chunks <= 8 ? 8 : chunks <= 16 ? 16 : 32;
    int64_t want = (count * g + 255) / 256;
    const int64_t cap = (int64_t)sms * 16;
    const int blocks = (int)(want < 1 ? 1 : (want > cap ? cap : want));
    if (vec && (d == 128 || d == 256 || d == 512)) {
        timing_mark(st);
        if (d == 128)
            pair_kernel_rows<KIND, 1><<<blocks, 256, 0, st>>>(x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, pert);
        else if (d == 256)
            pair_kernel_rows<KIND, 2><<<blocks, 256, 0, st>>>(x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, pert);
        else
            pair_kernel_rows<KIND, 4><<<blocks, 256, 0, st>>>(x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, pert);
        timing_mark(st);
        count_launches(1);
        return;
    }
    switch (g) {
        case 1: launch_g<KIND, 1>(vec, x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, blocks, st, pert); break;
        case 2: launch_g<KIND, 2>(vec, x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, blocks, st, pert); break;
        case 4: launch_g<KIND, 4>(vec, x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, blocks, st, pert); break;
        case 8: launch_g<KIND, 8>(vec, x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, blocks, st, pert); break;
        case 16: launch_g<KIND, 16>(vec, x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, blocks, st, pert); break;
        default: launch_g<KIND, 32>(vec, x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, blocks, st, pert); break;
    }
}

}  // namespace pairs

int pair_costs(int kind, const float* x, const float* y, int64_t nx, int64_t ny, int64_t d, const double* a,
               const double* b, double scale, const int64_t* rows, const int64_t* cols, int64_t count, double* out,
               int* status, cudaStream_t st, std::string& err, const Perturb* pert_in) {
    if (count == 0) return 0;
    Perturb pert;
    if (pert_in && pert_in->sigma != 0.0 && kind != 3) pert = *pert_in;  // the l2^2 kind is never perturbed here
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    switch (kind) {
        case 0: pairs::launch_kind<0>(x, y, nx, ny, (int)d, a, b, scale, rows, cols, count, out, status, st, sms, pert); break;
        case 1: pairs::launch_kind<1>(x, y, nx, ny, (int)d, a, b, scale, rows, cols, count, out, status, st, sms, pert); break;
        case 2: pairs::launch_kind<2>(x, y, nx, ny, (int)d, a, b, scale, rows, cols, count, out, status, st, sms, pert); break;
        case 3: pairs::launch_kind<3>(x, y, nx, ny, (int)d, a, b, scale, rows, cols, count, out, status, st, sms, pert); break;
        default: err = "unknown pair cost kind"; return 2;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
    return 0;
}

}  // namespace hb
