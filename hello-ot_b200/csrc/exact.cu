// fp64 re-check of the ℓ2² scan's top-k lists (HB_L2SQ_EXACT).
//
// The tensor-core scan ranks pairs by an approximate score: its dot product is
// fp32-class (3-term fp16 split, fp32 accumulation) or one TF32 product.  The
// reference ranks by fp32 SGEMM dots; both are approximations of the exact
// score (s<x_i, y_j> + qb_i) + dbb_j.  This file turns the scan's lists into the
// exact fp64 top-k of every row and column:
//
//   bounds   per row i a rigorous bound E_i of |approximate - exact| over all
//            columns (and per column over all rows), from the rows' l2 / l1
//            norms, the other cloud's largest norms and the split's error model;
//   scan     screens drop a pair only when its approximate score is more than
//            2E below the list's last approximate score, every list holds two
//            entries more than the bucket, and each list records its runner-up:
//            the largest approximate score offered and not kept;
//   recheck  a warp per list recomputes the candidates' dots in fp64 from the
//            fp32 features and re-ranks them.  The list is exact when
//            runner-up + E < the k-th exact score: every pair outside it then
//            scores below the k-th (a dropped pair is below the last kept
//            approximate score - 2E, hence below every kept pair's exact score);
//   rescan   a list that fails the test (a near tie within the bound) is
//            recomputed from scratch: block per list, fp64 scores against every
//            column.
//
// Error model of the 3-term split (x' = x 2^e, hi = fp16(x'), lo = fp16(x' - hi),
// x' = hi + lo + dx with |dx| <= 2^-22 |x'| + 2^-25): each product term pair
// differs from x'y' by at most 3 2^-22 |x'y'| + 2^-25 (|x'| + |y'|) (to first
// order); the three exact fp16 products are summed in fp32 over 3 dp16 terms.
// Per pair, in real units:
//   |err| <= s [c1 sum|x_k y_k| + 2^-25 (2^-ex sum|y_k| + 2^-ey sum|x_k|)]
//   c1 = 3 2^-22 + (3 dp16 + 2) 2^-24
// and the bound used doubles the accumulation and floor terms (the accumulation
// order inside an MMA is not documented), applies Cauchy-Schwarz
// (sum|x_k y_k| <= |x|_2 |y|_2) and maximises over the other cloud.  TF32
// (one product, operands truncated to 10 fraction bits): c1 = 2 2^-10 + 2^-20 +
// (dp + 2) 2^-24, no floor term.  A slack of 2^-48 s |x|_2 max|y|_2 covers the fp64
// rounding of the scores themselves.
#include <algorithm>
#include <cmath>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace hb {
namespace exact {

// l2 and l1 norm of every row (rounded up to fp32), and the largest of each over
// the cloud (bit patterns of non-negative floats: integer order is value order).
__global__ void row_norms(const float* __restrict__ x, int64_t rows, int d, float* __restrict__ n2,
                          float* __restrict__ n1, unsigned* __restrict__ max2, unsigned* __restrict__ max1) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    unsigned m2 = 0, m1 = 0;
    const double grow = 1.0 + (double)d * 0x1p-52;  // fp64 summation error of d terms
    for (int64_t r = warp; r < rows; r += nwarps) {
        const float* row = x + r * d;
        double sq = 0.0, ab = 0.0;
        for (int c = lane; c < d; c += 32) {
            const double v = (double)row[c];
            sq = fma(v, v, sq);
            ab += fabs(v);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, off);
            ab += __shfl_xor_sync(0xffffffffu, ab, off);
        }
        const float l2 = __double2float_ru(__dsqrt_ru(sq * grow));
        const float l1 = __double2float_ru(ab * grow);
        if (lane == 0) { n2[r] = l2; n1[r] = l1; }
        m2 = max(m2, __float_as_uint(l2));
        m1 = max(m1, __float_as_uint(l1));
    }
    if (lane == 0) {
        if (m2) atomicMax(max2, m2);
        if (m1) atomicMax(max1, m1);
    }
}

// E of every row against the other cloud; rows_pad >= rows entries are written
// (zeros beyond rows).  other: the other cloud's largest l2 / l1 norms; exps: the
// clouds' power-of-two scales (3-term split) or null (TF32).
__global__ void row_bounds(const float* __restrict__ n2, const float* __restrict__ n1, int64_t rows,
                           int64_t rows_pad, const unsigned* __restrict__ other_max2,
                           const unsigned* __restrict__ other_max1, const int* __restrict__ exps, int self_slot,
                           double c1, double scale, float* __restrict__ err) {
    const double o2 = (double)__uint_as_float(*other_max2), o1 = (double)__uint_as_float(*other_max1);
    double fs = 0.0, fo = 0.0;
    if (exps) {  // floor terms, doubled: 2^-24 2^-e per side
        fs = ldexp(1.0, -24 - exps[self_slot]);
        fo = ldexp(1.0, -24 - exps[1 - self_slot]);
    }
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows_pad;
         r += (int64_t)gridDim.x * blockDim.x) {
        if (r >= rows) { err[r] = 0.0f; continue; }
        const double a2 = (double)n2[r], a1 = (double)n1[r];
        const double e = scale * ((c1 + 0x1p-48) * a2 * o2 + fs * o1 + fo * a1) * (1.0 + 0x1p-20);
        err[r] = __double2float_ru(e);
    }
}

// fp64 dot of two fp32 rows (products exact, fp64 sums), warp-wide: every lane returns
// the same value (fixed xor-butterfly order).
__device__ __forceinline__ double warp_dot(const float* __restrict__ a, const float* __restrict__ b, int d,
                                           int lane) {
    double acc = 0.0;
    for (int c = lane; c < d; c += 32) acc = fma((double)a[c], (double)b[c], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    return acc;
}

// Warp per list: exact scores of the K candidates, the exact top k_out, and the test
// runner-up + E < k-th exact score (with a relative fp64 slack); lists that fail it are
// appended to `flags`.  SWAP: the queries are the y rows (score (dot + dbias) + qbias).
template <int K, bool SWAP>
__global__ void recheck(const float* __restrict__ qf, const float* __restrict__ dbf, int64_t nq, int d, double scale,
                        const double* __restrict__ qbias, const double* __restrict__ dbias,
                        const int* __restrict__ li, const double* __restrict__ run, const float* __restrict__ qerr,
                        int k_out, double* __restrict__ ov, int* __restrict__ oi, int* __restrict__ flags,
                        int* __restrict__ nflag) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < nq; r += nwarps) {
        const float* qrow = qf + r * d;
        const double qb = qbias[r];
        TopK<K> top;
        top.reset();
        for (int s = 0; s < K; ++s) {
            const int j = li[r * K + s];
            if (j < 0 || j == INT32_MAX) continue;
            const double dot = scale * warp_dot(qrow, dbf + (int64_t)j * d, d, lane);
            const double sc = SWAP ? ((dot + dbias[j]) + qb) : ((dot + qb) + dbias[j]);
            top.offer(sc, j);
        }
        if (lane == 0) {
            double sk = -INFINITY;  // the k-th exact score (compile-time slot indices keep top in registers)
#pragma unroll
            for (int s = 0; s < K; ++s)
                if (s == k_out - 1 && top.i[s] != INT32_MAX) sk = top.v[s];
            const double ru = run[r];
            bool ok = ru == -INFINITY;
            if (!ok && sk > -INFINITY) {
                const double slack = 0x1p-50 * (fabs(ru) + fabs(sk) + 2.0 * fabs(qb));
                ok = ru + (double)qerr[r] * (1.0 + 0x1p-10) + slack < sk;
            }
#pragma unroll
            for (int s = 0; s < K; ++s)
                if (s < k_out) {
                    ov[r * k_out + s] = top.v[s];
                    oi[r * k_out + s] = top.i[s] == INT32_MAX ? -1 : top.i[s];
                }
            if (!ok) flags[atomicAdd(nflag, 1)] = (int)r;
        }
    }
}

// Block per flagged list: exact fp64 scores against every database row, exact top k_out.
// WARP: a warp per database row (coalesced row reads, features >= 64), else a thread per
// database row.
template <int K, bool SWAP, bool WARP>
__global__ void __launch_bounds__(256) rescan(const float* __restrict__ qf, const float* __restrict__ dbf, int64_t ndb,
                                              int d, double scale, const double* __restrict__ qbias,
                                              const double* __restrict__ dbias, const int* __restrict__ flags,
                                              const int* __restrict__ nflag, int k_out, double* __restrict__ ov,
                                              int* __restrict__ oi) {
    __shared__ double sv[8][K];
    __shared__ int si[8][K];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int count = *nflag;
    for (int f = blockIdx.x; f < count; f += gridDim.x) {
        const int64_t r = flags[f];
        const float* qrow = qf + r * d;
        const double qb = qbias[r];
        TopK<K> top;
        top.reset();
        if constexpr (WARP) {  // every lane holds the same score, so every lane's list is the warp's
            for (int64_t j = warp; j < ndb; j += 8) {
                const double dot = scale * warp_dot(qrow, dbf + j * d, d, lane);
                top.offer(SWAP ? ((dot + dbias[j]) + qb) : ((dot + qb) + dbias[j]), (int)j);
            }
        } else {
            for (int64_t j = threadIdx.x; j < ndb; j += blockDim.x) {
                const float* row = dbf + j * d;
                double acc = 0.0;
                for (int c = 0; c < d; ++c) acc = fma((double)qrow[c], (double)row[c], acc);
                const double dot = scale * acc;
                top.offer(SWAP ? ((dot + dbias[j]) + qb) : ((dot + qb) + dbias[j]), (int)j);
            }
            // warp merge by shuffles into lane 0
            for (int src = 1; src < 32; ++src)
#pragma unroll
                for (int s = 0; s < K; ++s) {
                    const double v = __shfl_sync(0xffffffffu, top.v[s], src);
                    const int i = __shfl_sync(0xffffffffu, top.i[s], src);
                    if (lane == 0 && i != INT32_MAX) top.offer(v, i);
                }
        }
        if (lane == 0)
#pragma unroll
            for (int s = 0; s < K; ++s) { sv[warp][s] = top.v[s]; si[warp][s] = top.i[s]; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
                for (int s = 0; s < K; ++s)
                    if (si[w][s] != INT32_MAX) top.offer(sv[w][s], si[w][s]);
#pragma unroll
            for (int s = 0; s < K; ++s)
                if (s < k_out) {
                    ov[r * k_out + s] = top.v[s];
                    oi[r * k_out + s] = top.i[s] == INT32_MAX ? -1 : top.i[s];
                }
        }
        __syncthreads();
    }
}

template <int K, bool SWAP>
void launch_rescan(const ExactSide& side, int d, double scale, int k_out, int sms, cudaStream_t st) {
    if (d >= 64)
        rescan<K, SWAP, true><<<sms * 2, 256, 0, st>>>(side.qf, side.dbf, side.ndb, d, scale, side.qbias, side.dbias,
                                                       side.flags, side.nflag, k_out, side.ov, side.oi);
    else
        rescan<K, SWAP, false><<<sms * 2, 256, 0, st>>>(side.qf, side.dbf, side.ndb, d, scale, side.qbias,
                                                        side.dbias, side.flags, side.nflag, k_out, side.ov, side.oi);
}

template <int K>
cudaError_t finish_k(const ExactSide& side, int d, double scale, int k_out, int sms, cudaStream_t st) {
    const unsigned blocks = (unsigned)std::min<int64_t>((side.nq + 7) / 8, (int64_t)sms * 16);
    if (side.swap) {
        recheck<K, true><<<blocks, 256, 0, st>>>(side.qf, side.dbf, side.nq, d, scale, side.qbias, side.dbias, side.li,
                                                 side.run, side.qerr, k_out, side.ov, side.oi, side.flags, side.nflag);
        launch_rescan<K, true>(side, d, scale, k_out, sms, st);
    } else {
        recheck<K, false><<<blocks, 256, 0, st>>>(side.qf, side.dbf, side.nq, d, scale, side.qbias, side.dbias,
                                                  side.li, side.run, side.qerr, k_out, side.ov, side.oi, side.flags,
                                                  side.nflag);
        launch_rescan<K, false>(side, d, scale, k_out, sms, st);
    }
    count_launches(2);
    return cudaGetLastError();
}

}  // namespace exact

cudaError_t exact_bounds(const float* x, const float* y, int64_t q, int64_t n, int d, int64_t n_pad, int precision,
                         const int* exps, double dot_scale, float* norms_x, float* norms_y, unsigned* maxes,
                         float* x_err, float* y_err, int sms, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(maxes, 0, 4 * sizeof(unsigned), st);
    if (e != cudaSuccess) return e;
    const unsigned nb = (unsigned)sms * 8;
    exact::row_norms<<<nb, 256, 0, st>>>(x, q, d, norms_x, norms_x + q, maxes + 0, maxes + 1);
    exact::row_norms<<<nb, 256, 0, st>>>(y, n, d, norms_y, norms_y + n, maxes + 2, maxes + 3);
    double c1;
    if (precision == 3) {
        const double dp16 = (double)((d + 7) / 8 * 8);
        c1 = 3.0 * 0x1p-22 + 2.0 * (3.0 * dp16 + 2.0) * 0x1p-24;
    } else {
        const double dp = (double)((d + 3) / 4 * 4);
        c1 = 2.0 * 0x1p-10 + 0x1p-20 + 2.0 * (dp + 2.0) * 0x1p-24;
        exps = nullptr;
    }
    exact::row_bounds<<<nb, 256, 0, st>>>(norms_x, norms_x + q, q, q, maxes + 2, maxes + 3, exps, 0, c1, dot_scale,
                                          x_err);
    exact::row_bounds<<<nb, 256, 0, st>>>(norms_y, norms_y + n, n, n_pad, maxes + 0, maxes + 1, exps, 1, c1,
                                          dot_scale, y_err);
    count_launches(4);
    return cudaGetLastError();
}

cudaError_t exact_finish(int K, const ExactSide& side, int d, double dot_scale, int k_out, int sms, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(side.nflag, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
    switch (K) {
        case 1: return exact::finish_k<1>(side, d, dot_scale, k_out, sms, st);
        case 2: return exact::finish_k<2>(side, d, dot_scale, k_out, sms, st);
        case 3: return exact::finish_k<3>(side, d, dot_scale, k_out, sms, st);
        case 4: return exact::finish_k<4>(side, d, dot_scale, k_out, sms, st);
        case 6: return exact::finish_k<6>(side, d, dot_scale, k_out, sms, st);
        case 8: return exact::finish_k<8>(side, d, dot_scale, k_out, sms, st);
        case 10: return exact::finish_k<10>(side, d, dot_scale, k_out, sms, st);
        case 16: return exact::finish_k<16>(side, d, dot_scale, k_out, sms, st);
        case 18: return exact::finish_k<18>(side, d, dot_scale, k_out, sms, st);
        case 32: return exact::finish_k<32>(side, d, dot_scale, k_out, sms, st);
        case 34: return exact::finish_k<34>(side, d, dot_scale, k_out, sms, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace hb
