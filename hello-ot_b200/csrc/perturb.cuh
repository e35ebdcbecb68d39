// Cost perturbation of the norm costs: c'_ij = c_ij + noise(source_i, target_j)
// in fp64, with the reference's two noise families
// (src/hello_ot/_native/generic_scan/cost.cu:350-423 sigma_noise, the same
// formulas as src/hello_ot/costs/metric_perturbation.py:19-92):
//
//   index_hash (mode 1): for each prime p in (2003, 2011), with s = source mod p,
//     t = target mod p as fp32 and seed-derived integer coefficients (a, b, o):
//     x = ((a s + b t) + s t) + o,  h = x - p floor(x * fp32(1/p))
//     value = ((h_2003 + 2003 h_2011) + 0.5) * fp32(1/(2003*2011))
//     noise = sigma * (double)value
//   rank2 (mode 0): z = fma(target, 78.233, source * 12.9898) + seed_term,
//     noise = fp32(sigma) * ((__sinf(z) * 0.5) + 0.5) (fp32), as the reference's
//     fused kernels compute it.
//
// Every fp32 step is rounded individually (no contraction) so the index-hash
// noise equals the reference's NumPy / Torch / CUDA values bit for bit.
#pragma once
#include <cstdint>

namespace hb {

struct Perturb {
    double sigma = 0.0;     // 0: no perturbation
    float seed_term = 0.f;  // (float)(seed * 0.001)
    int mode = 1;           // 0 rank2, 1 index_hash
    int row_is_source = 1;  // the scan's rows are the sources
    float a0 = 0.f, b0 = 0.f, o0 = 0.f, a1 = 0.f, b1 = 0.f, o1 = 0.f;  // index-hash coefficients
    const int64_t* row_index = nullptr;  // global index of each row of the call
    const int64_t* col_index = nullptr;  // global index of each column
};

// Per-index inputs of the noise: index-hash residues (mod 2003, mod 2011) as
// fp32, or the index itself as fp32 (rank2, in .x).
__device__ __forceinline__ float2 noise_input(const Perturb& p, int64_t idx) {
    if (p.mode == 0) return make_float2((float)idx, 0.f);
    return make_float2((float)(idx % 2003), (float)(idx % 2011));
}

__device__ __forceinline__ float hash_step(float a, float b, float o, float s, float t, float prime, float recip) {
    const float x = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(a, s), __fmul_rn(b, t)), __fmul_rn(s, t)), o);
    return __fsub_rn(x, __fmul_rn(prime, floorf(__fmul_rn(x, recip))));
}

// Noise of the pair (row input r, column input c); the source / target roles
// follow row_is_source.
__device__ __forceinline__ double noise_of(const Perturb& p, float2 r, float2 c) {
    const float2 src = p.row_is_source ? r : c, tgt = p.row_is_source ? c : r;
    if (p.mode == 0) {
        const float z = __fadd_rn(fmaf(tgt.x, 78.233f, __fmul_rn(src.x, 12.9898f)), p.seed_term);
        return (double)__fmul_rn((float)p.sigma, __fadd_rn(__fmul_rn(__sinf(z), 0.5f), 0.5f));
    }
    const float h0 = hash_step(p.a0, p.b0, p.o0, src.x, tgt.x, 2003.0f, (float)(1.0 / 2003.0));
    const float h1 = hash_step(p.a1, p.b1, p.o1, src.y, tgt.y, 2011.0f, (float)(1.0 / 2011.0));
    const float v = __fmul_rn(__fadd_rn(__fadd_rn(h0, __fmul_rn(2003.0f, h1)), 0.5f), (float)(1.0 / 4028033.0));
    return __dmul_rn(p.sigma, (double)v);
}

}  // namespace hb
