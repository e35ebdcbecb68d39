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
// and then from L1.  For d = 128, 256, 512 (pair_kernel_ring) a warp serves one
// edge at a time from a ring of target rows in shared memory, filled ahead by
// bulk copies, with the source row held in registers.  HBM-bound: every edge
// gathers its database row once.
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

// d = 128 NV with 16-byte-aligned rows, target rows through a shared-memory ring: each
// warp keeps RING edges' target rows in flight as bulk copies (cp.async.bulk of the d-float
// row, issued by lane 0, one mbarrier per slot), so a warp's loads need no registers; the
// source row is held in registers as fp64 while the run of one source row lasts.  Same
// chunks, order and reduction tree as pair_kernel<KIND, 32, true>: the results are identical.
constexpr int RING = 4;  // slots per warp (deeper rings cost resident warps and measured slower)
template <int NV>
constexpr size_t ring_smem() { return (size_t)8 * RING * (NV * 512 + 8) + 16; }

template <int KIND, int NV>
__global__ void __launch_bounds__(256) pair_kernel_ring(const float* __restrict__ x, const float* __restrict__ y,
                                                        int64_t nx, int64_t ny, int d, const double* __restrict__ a,
                                                        const double* __restrict__ b, double scale,
                                                        const int64_t* __restrict__ rows,
                                                        const int64_t* __restrict__ cols, int64_t count,
                                                        double* __restrict__ out, int* status, const Perturb pert) {
    extern __shared__ __align__(128) unsigned char ring_buf[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float4* slots = reinterpret_cast<float4*>(ring_buf) + (size_t)warp * RING * 32 * NV;
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring_buf + (size_t)8 * RING * NV * 512) + warp * RING;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(ring_buf + (size_t)8 * RING * (NV * 512 + 8));
    if (threadIdx.x == 0) *abort_flag = 0;
    if (lane == 0) {
        for (int j = 0; j < RING; ++j) mbar_init(&bars[j], 1);
        fence_barrier_init();
    }
    __syncthreads();
    const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t per_warp = (count + warps - 1) / warps;
    const int64_t e0 = warp_id * per_warp, e1 = min(count, e0 + per_warp);
    const uint32_t row_bytes = (uint32_t)d * 4u;
    auto issue = [&](int64_t e) {  // lane 0: edge e's target row into slot (e - e0) % RING
        const int slot = (int)((e - e0) % RING);
        const int64_t c = cols[e], r = rows[e];
        if (r >= 0 && r < nx && c >= 0 && c < ny) {
            mbar_arrive_expect_tx(&bars[slot], row_bytes);
            bulk_load_1d(slots + slot * 32 * NV, y + c * d, row_bytes, &bars[slot]);
        } else {
            mbar_arrive(&bars[slot]);  // nothing to copy: the phase completes at once
        }
    };
    if (lane == 0)
        for (int64_t e = e0; e < e1 && e < e0 + RING; ++e) issue(e);
    int64_t held = -1;
    double xd[NV * 4];
    for (int64_t e = e0; e < e1; ++e) {  // warp-uniform
        const int slot = (int)((e - e0) % RING);
        const uint32_t par = (uint32_t)(((e - e0) / RING) & 1);
        const int64_t r = rows[e], c = cols[e];
        const bool ok = r >= 0 && r < nx && c >= 0 && c < ny;
        if (!mbar_wait(&bars[slot], par, abort_flag, status)) {
            // a copy never completed: give the copies in flight a bounded time, then leave
            for (int64_t f = e + 1; f < e1 && f < e + RING; ++f)
                for (int t = 0; t < 64 && !mbar_try_wait(&bars[(f - e0) % RING], (uint32_t)(((f - e0) / RING) & 1));
                     ++t) {
                }
            return;
        }
        double acc = 0.0;
        if (ok) {
            if (r != held) {
                const float4* x4 = reinterpret_cast<const float4*>(x + r * d);
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    const float4 u = __ldg(x4 + lane + 32 * v);
                    xd[4 * v] = u.x; xd[4 * v + 1] = u.y; xd[4 * v + 2] = u.z; xd[4 * v + 3] = u.w;
                }
                held = r;
            }
            const float4* yr = slots + slot * 32 * NV;
#pragma unroll
            for (int v = 0; v < NV; ++v) {
                const float4 yv = yr[lane + 32 * v];
                const float yy[4] = {yv.x, yv.y, yv.z, yv.w};
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
        __syncwarp();  // every lane is done with the slot
        if (lane == 0 && e + RING < e1) issue(e + RING);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc = combine<KIND>(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        if (lane == 0) {
            if (!ok) {
                atomicOr(status, kErrBadInput);
                out[e] = __longlong_as_double(0x7ff8000000000000LL);
            } else if (KIND == 3) {
                out[e] = (a[r] + b[c]) - scale * acc;
            } else {
                const double dist = KIND == 2 ? sqrt(acc) : acc;
                out[e] = pert.sigma != 0.0 ? dist + noise_of(pert, noise_input(pert, pert.row_index[r]),
                                                                noise_input(pert, pert.col_index[c]))
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
        const size_t sm = d == 128 ? ring_smem<1>() : d == 256 ? ring_smem<2>() : ring_smem<4>();
        auto kern = d == 128 ? pair_kernel_ring<KIND, 1> : d == 256 ? pair_kernel_ring<KIND, 2> : pair_kernel_ring<KIND, 4>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        int per = 4;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, 256, sm);
        const int64_t cap2 = (int64_t)sms * (per > 0 ? per : 1);
        const int nb = (int)(want < 1 ? 1 : (want > cap2 ? cap2 : want));
        timing_mark(st);
        kern<<<nb, 256, sm, st>>>(x, y, nx, ny, d, a, b, s, rows, cols, count, out, status, pert);
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
