// ℓ2² (bilinear) full-space pricing scan on the sm_100a tensor cores.
//
// Replaces the reference's SGEMM-tile + selection kernels
// (src/hello_ot/_native/generic_scan/pricing_small.cu:230-304, pricing.cu,
// matrix_selection.cuh) with one fused persistent kernel per pass:
//
//   TMA (64B-swizzled slabs of fp16 halves, or of fp32 features in the TF32
//   mode; local HBM only, no multicast load)
//     -> tcgen05.mma kind::f16 (kind::tf32), 128x256 tile (256x256 over a CTA
//        pair with cta_group::2), fp32 accumulator in TMEM
//        (two accumulators: the MMA of tile t+1 overlaps the epilogue of t)
//     -> epilogue warps: tcgen05.ld, score, certificate sums, row top-k in
//        registers and (one-pass mode) column top-k in per-warp HBM lists.
//   No cost tile is ever written to HBM.
//
// Score arithmetic follows the reference raw path (matrix_selection.cuh:20-26):
//   dot = fp32(s * <x,y>);  cost = (a_i + b_j) - dot;  score = (dot + qb_i) + dbb_j
// in fp64.  <x,y> is computed either with one TF32 product ("tf32", kind::tf32 on
// the fp32 features) or as the 3-term split hi*hi + hi*lo + lo*hi on fp16 halves
// (kind::f16): each cloud is scaled by one power of two 2^e so that its largest
// |x| lies in [2^14, 2^15), hi = fp16(x 2^e), lo = fp16(x 2^e - hi) (22 bits of
// every element kept, products exact, fp32 accumulation), and the epilogue
// multiplies the accumulated dot by 2^-(e_x + e_y), exactly: an fp32-class dot
// (each product within 3 2^-22 |x||y|) at the fp16 tensor-core rate and with
// 4 bytes per element of operand traffic.
//
// Warp roles: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, 4 or 8
// epilogue warps (thread = tile row = TMEM lane).
//
// Column top-k.  One-pass mode (k <= 8): each CTA owns a fixed rectangle of
// the pair space (a row group x a column group); every epilogue warp keeps, in
// HBM, the top-k list of each of its columns over the rows it sees (one list
// per row group and TMEM lane quarter, so each list has exactly one writer).
// Pairs are screened in fp32 against a per-column threshold shared by all of
// the column's lists (the largest k-th score among them); chunks with a
// candidate are transposed through shared memory and each lane inserts its
// column's candidates with exact fp64 scores.  A merge combines the lists.
// Two-pass mode: a second pass with the clouds' roles exchanged computes the
// column lists as row lists (same products, same order, same scores).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "../../include/hello_b200.h"
#include "common.cuh"
#include "internal.h"
#include "scan_common.cuh"

namespace hb {
namespace l2sq {

// K slab of 16 fp32 (64-byte rows, 64-byte swizzle).  A stage holds the query
// and database tiles and, for the 3-term split, their low parts, so all three
// products of a slab come from one fetch: [A | A_lo | B | B_lo] = 8+8+16+16 KB.
constexpr int BM = 128, BN = 256, BK = 16;
constexpr int A_BYTES = BM * BK * 4, B_BYTES = BN * BK * 4;
constexpr int OFF_ALO = A_BYTES, OFF_B = 2 * A_BYTES, OFF_BLO = 2 * A_BYTES + B_BYTES;
constexpr int STAGE_BYTES = 2 * (A_BYTES + B_BYTES);
// CTA pairs (one pass, cta_group::2): each CTA of a pair stages its own 128 query
// rows and half (128 columns) of the database tile; one M = 256 x N = 256 MMA
// issued by the even CTA covers both, and each CTA's TMEM receives its 128 rows.
constexpr int BNH = BN / 2;
constexpr int BH_BYTES = BNH * BK * 4;
constexpr int P_OFF_ALO = A_BYTES, P_OFF_B = 2 * A_BYTES, P_OFF_BLO = 2 * A_BYTES + BH_BYTES;
constexpr int PAIR_STAGE_BYTES = 2 * (A_BYTES + BH_BYTES);
constexpr int EPI_FIRST = 64;  // warps 0-1: TMA producer, MMA issuer; then EW epilogue warps
constexpr int MAX_EW = 8;
// Epilogue warps per CTA: 8 (two per TMEM lane quarter, each on half the
// columns) when the row list is small enough for the register budget, else 4.
template <int K>
struct Epi {
    static constexpr int EW = K <= 10 ? 8 : 4;
    static constexpr int THREADS = EPI_FIRST + 32 * EW;
};
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t IDESC = idesc_tf32(BM, BN);
constexpr uint32_t IDESC_PAIR = idesc_tf32(2 * BM, BN);
constexpr uint32_t IDESC_F16 = idesc_f16(BM, BN);
constexpr uint32_t IDESC_F16_PAIR = idesc_f16(2 * BM, BN);
// fp16 operands: 32 halves per 64-byte slab row (the same bytes as 16 fp32), K = 16 per MMA
constexpr int BK16 = 32;

struct Params {
    CUtensorMap qmap[2];  // query operand: [0] features (read as tf32 = hi part), [1] low parts
    CUtensorMap dmap[2];  // database operand
    int terms;            // 1: x*y (TF32, fp32 operands); 3: hi*hi + hi*lo + lo*hi (fp16 halves)
    int kslabs;
    const int* exps;      // terms == 3: the clouds' power-of-two scales e_query, e_database
    int q, n;
    int groups, tpg, ct, units;
    const double* q_cost;  // a_i  (certificate only)
    const double* d_cost;  // b_j, padded to whole column tiles (null: no cost terms in this pass)
    const double* q_bias;  // query-side bias
    const double* d_bias;  // database-side bias, padded to whole column tiles
    float scale;
    double* part_v;
    int* part_i;
    double* cta_stats;
    int* status;
    // one-pass mode: CTA b owns row group b / groups (rbg row blocks) x column group b % groups
    int rb, rbg;
    int* progress;  // [grid] tiles started by each CTA (pacing of a column group's CTAs)
    int* ckey;     // [ct * BN] screening threshold of each column (ordered-int fp32 image), see below
    double* cval;  // [row groups * 4][n][K]
    int* cidx;
    // fp64 re-check (HB_L2SQ_EXACT; null pointers: off).  row_err: bound E of the error of each
    // query row's approximate scores (over all columns); col_err (one pass): each column's,
    // padded to whole tiles.  Screens drop a pair only when its approximate score is more
    // than 2E below the list's k-th, and every list records its runner-up (the largest
    // approximate score offered to it and not kept): part_run per partial row list,
    // crun per column list ([row groups * 4][n]).
    const float* row_err;
    const float* col_err;
    double* part_run;
    double* crun;
};

// Column vectors of a tile (bias, cost, threshold) are bulk-copied by the
// producer into a ring of CS slots, ahead of the tile's epilogue.
template <int NST, int NCS, bool ONE, int STB>
struct __align__(1024) SmemT {
    static constexpr int STAGES = NST, CS = NCS;
    uint8_t stage[NST][STB];
    double cbias[NCS][BN];                     // the tile's column biases
    double ccost[NCS][BN];                     // the tile's column costs (cost terms)
    int ckey[ONE ? NCS : 1][ONE ? BN : 4];     // the tile's column thresholds (one pass)
    __align__(16) float cerr[ONE ? NCS : 1][ONE ? BN : 4];  // the tile's column error bounds (one pass, exact)
    // per epilogue warp, its column slice (EW x BN/(EW/4) = 4 BN entries in all), fp32
    // constants read once per pair: x = bias, y = the column's screening threshold (one
    // pass; threshold less the rounding margin), z = column cost (cost terms), w unused
    __align__(16) float colx[4 * BN];  // bias
    __align__(16) float coly[4 * BN];  // column screening threshold (one pass)
    __align__(16) float colz[4 * BN];  // column cost (cost terms)
    float trans[ONE ? MAX_EW * 32 * 33 : 1];   // per warp: 32 x 32 chunk, transposed
    double rbx[ONE ? MAX_EW * 32 : 1];         // per warp: the chunk rows' biases
    double red[MAX_EW * 5];
    uint64_t full[NST], empty[NST], tfull[2], tempty[2], cfull[NCS], cempty[NCS];
    uint32_t tmem_base;
    int abort;
};
template <bool ONE, bool PAIR = false>
using Smem = SmemT<PAIR ? 4 : (ONE ? 3 : 4), 4, ONE, PAIR ? PAIR_STAGE_BYTES : STAGE_BYTES>;
template <bool ONE, bool PAIR = false>
constexpr size_t smem_bytes() { return sizeof(Smem<ONE, PAIR>) + 1024; }
static_assert(smem_bytes<false>() <= 227 * 1024 && smem_bytes<true>() <= 227 * 1024 &&
              smem_bytes<true, true>() <= 227 * 1024, "dynamic shared memory above the 227 KB a CTA may use");

// Tile schedule of a CTA: units u = rb * groups + g in [u0, uend) by ustep.
struct Sched {
    int u0, ustep, uend;
};
// With CTA pairs a unit's row block index counts pairs of row blocks: the CTA of
// rank r of the pair takes row block 2 * (u / groups) + r.
template <bool ONE, bool PAIR = false>
__device__ __forceinline__ Sched schedule(const Params& p) {
    if (!ONE) return {(int)blockIdx.x, (int)gridDim.x, p.units};
    const int cl = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int rg = cl / p.groups, g = cl % p.groups;
    const int rb0 = rg * p.rbg, rb1 = min(p.rb, rb0 + p.rbg);
    return {rb0 * p.groups + g, p.groups, rb1 > rb0 ? rb1 * p.groups : 0};
}

// One pass: the CTAs of a column group (one per row group) stream the same
// column tiles.  Each keeps within PACE tiles of the slowest of them, so a tile
// one of them brings from HBM is still in L2 for the others; unpaced they
// drift apart and every one of them reads the whole target cloud from HBM.
// The wait is bounded (PACE_SPINS sleeps, then it proceeds): no CTA ever
// depends on another one making progress.
constexpr int PACE = 2, PACE_SPINS = 64;

template <bool PAIR = false>
__device__ __forceinline__ void pace(const Params& p, int t) {
    volatile int* prog = p.progress;
    prog[blockIdx.x] = t;
    constexpr int W = PAIR ? 2 : 1;  // CTAs per rectangle
    const int cl = blockIdx.x / W;
    const int g = cl % p.groups, gr = (gridDim.x / W) / p.groups;
    for (int spin = 0; spin < PACE_SPINS; ++spin) {
        int slow = INT32_MAX;
        for (int r = 0; r < gr; ++r)
            for (int w = 0; w < W; ++w) slow = min(slow, prog[(r * p.groups + g) * W + w]);
        if (t - slow <= PACE) return;
        __nanosleep(500);
    }
}

// CTA pairs: both CTAs load their own A rows and B half into their own shared
// memory; the completions of both count on the even CTA's full barrier, which
// the even CTA's producer arms with the bytes of both.
template <bool ONE, bool PAIR = false>
__device__ __forceinline__ void producer(const Params& p, Smem<ONE, PAIR>& s) {
    constexpr int STAGES = Smem<ONE, PAIR>::STAGES, CSLOTS = Smem<ONE, PAIR>::CS;
    uint32_t stage = 0, phase = 0;
    const int rank = PAIR ? (int)cluster_rank() : 0;
    const uint32_t bytes = PAIR ? (p.terms == 3 ? PAIR_STAGE_BYTES : A_BYTES + BH_BYTES)
                                : (p.terms == 3 ? STAGE_BYTES : A_BYTES + B_BYTES);
    const uint32_t cbytes = BN * 8 + (p.d_cost ? BN * 8 : 0) + (ONE ? BN * 4 : 0) + (ONE && p.col_err ? BN * 4 : 0);
    const int kw = p.terms == 3 ? BK16 : BK;  // elements per 64-byte slab row
    uint32_t t = 0;
    const Sched sc = schedule<ONE, PAIR>(p);
    for (int u = sc.u0; u < sc.uend; u += sc.ustep) {
        const int rb = PAIR ? 2 * (u / p.groups) + rank : u / p.groups, g = u % p.groups;
        const int ct1 = min(p.ct, (g + 1) * p.tpg);
        for (int ct = g * p.tpg; ct < ct1; ++ct, ++t) {
            if (ONE) pace<PAIR>(p, (int)t);
            // the tile's column vectors (the slot was released CSLOTS tiles ago)
            const uint32_t cs = t % CSLOTS;
            if (!mbar_wait(&s.cempty[cs], ((t / CSLOTS) & 1) ^ 1, &s.abort, p.status)) return;
            mbar_arrive_expect_tx(&s.cfull[cs], cbytes);
            bulk_load_1d(s.cbias[cs], p.d_bias + (size_t)ct * BN, BN * 8, &s.cfull[cs]);
            if (p.d_cost) bulk_load_1d(s.ccost[cs], p.d_cost + (size_t)ct * BN, BN * 8, &s.cfull[cs]);
            if (ONE) bulk_load_1d(s.ckey[cs], p.ckey + (size_t)ct * BN, BN * 4, &s.cfull[cs]);
            if (ONE && p.col_err) bulk_load_1d(s.cerr[cs], p.col_err + (size_t)ct * BN, BN * 4, &s.cfull[cs]);
            for (int ks = 0; ks < p.kslabs; ++ks) {
                if (!mbar_wait(&s.empty[stage], phase ^ 1, &s.abort, p.status)) return;
                uint8_t* a = s.stage[stage];
                if constexpr (PAIR) {
                    const uint32_t fb = peer_smem(&s.full[stage], 0);
                    if (rank == 0) mbar_arrive_expect_tx(&s.full[stage], 2 * bytes);
                    tma_load_2d_pair(a, &p.qmap[0], fb, ks * kw, rb * BM);
                    tma_load_2d_pair(a + P_OFF_B, &p.dmap[0], fb, ks * kw, ct * BN + rank * BNH);
                    if (p.terms == 3) {
                        tma_load_2d_pair(a + P_OFF_ALO, &p.qmap[1], fb, ks * kw, rb * BM);
                        tma_load_2d_pair(a + P_OFF_BLO, &p.dmap[1], fb, ks * kw, ct * BN + rank * BNH);
                    }
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                    continue;
                }
                mbar_arrive_expect_tx(&s.full[stage], bytes);
                tma_load_2d(a, &p.qmap[0], &s.full[stage], ks * kw, rb * BM);
                tma_load_2d(a + OFF_B, &p.dmap[0], &s.full[stage], ks * kw, ct * BN);
                if (p.terms == 3) {
                    tma_load_2d(a + OFF_ALO, &p.qmap[1], &s.full[stage], ks * kw, rb * BM);
                    tma_load_2d(a + OFF_BLO, &p.dmap[1], &s.full[stage], ks * kw, ct * BN);
                }
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
        }
    }
    if (ONE) *(volatile int*)(p.progress + blockIdx.x) = INT32_MAX;  // done: never wait for this CTA
}

// Products per K step of 8: pass 1 (query = x): x*y, x*lo(y), lo(x)*y; pass 2
// (query = y) issues the same three products with the operands exchanged and
// in the same order, so both passes accumulate bit-identical dots.
// CTA pairs: issued by the even CTA only (M = 256 over both CTAs' A tiles); the
// commits arrive on the barriers of both CTAs.
template <bool SWAP, bool ONE, bool PAIR = false>
__device__ __forceinline__ void mma_issuer(const Params& p, Smem<ONE, PAIR>& s, uint32_t tmem) {
    constexpr int STAGES = Smem<ONE, PAIR>::STAGES;
    constexpr int OA_LO = PAIR ? P_OFF_ALO : OFF_ALO, OB = PAIR ? P_OFF_B : OFF_B, OB_LO = PAIR ? P_OFF_BLO : OFF_BLO;
    constexpr uint32_t ID = PAIR ? IDESC_PAIR : IDESC;
    constexpr uint32_t ID16 = PAIR ? IDESC_F16_PAIR : IDESC_F16;
    const bool f16 = p.terms == 3;  // fp16 halves (kind::f16), else fp32 features (kind::tf32)
    auto mma = [f16](uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
        if constexpr (PAIR) {
            if (f16) mma_f16_pair(d, a, b, ID16, acc);
            else mma_tf32_pair(d, a, b, ID, acc);
        } else {
            if (f16) mma_f16(d, a, b, ID16, acc);
            else mma_tf32(d, a, b, ID, acc);
        }
    };
    auto commit = [](uint64_t* bar) {
        if constexpr (PAIR) mma_commit_pair(bar);
        else mma_commit(bar);
    };
    uint32_t stage = 0, phase = 0, t = 0;
    const Sched sc = schedule<ONE, PAIR>(p);
    for (int u = sc.u0; u < sc.uend; u += sc.ustep) {
        const int g = u % p.groups;
        const int ct1 = min(p.ct, (g + 1) * p.tpg);
        for (int ct = g * p.tpg; ct < ct1; ++ct, ++t) {
            const uint32_t acc = t & 1, aph = (t >> 1) & 1;
            if (!mbar_wait(&s.tempty[acc], aph ^ 1, &s.abort, p.status)) return;
            tc_fence_after();
            const uint32_t d = tmem + acc * BN;
            uint32_t accumulate = 0;
            for (int ks = 0; ks < p.kslabs; ++ks) {
                if (!mbar_wait(&s.full[stage], phase, &s.abort, p.status)) return;
                tc_fence_after();
                const uint32_t a0 = smem_u32(s.stage[stage]);
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const uint32_t o = kk * 32;
                    const uint64_t ah = smem_desc_sw64(a0 + o), bh = smem_desc_sw64(a0 + OB + o);
                    mma(d, ah, bh, accumulate);
                    accumulate = 1;
                    if (p.terms == 3) {
                        const uint64_t al = smem_desc_sw64(a0 + OA_LO + o), bl = smem_desc_sw64(a0 + OB_LO + o);
                        if (!SWAP) { mma(d, ah, bl, 1); mma(d, al, bh, 1); }
                        else { mma(d, al, bh, 1); mma(d, ah, bl, 1); }
                    }
                }
                commit(&s.empty[stage]);
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
            commit(&s.tfull[acc]);
        }
    }
}

// Certificate terms computed by a pass (bit mask): score terms (sum s+^2,
// max s+, count) and cost terms (sum c^2, max |c|).  The row pass takes the
// score terms and the column pass the cost terms.
enum : int { kScoreStats = 1, kCostStats = 2 };

// Phase 1 of one 32-column chunk, branch-free and in fp32: fp32 score / cost
// of every pair (within 2^-22 (|dot| + |a| + |b| + |biases|) of the fp64
// values for the same dot), certificate partials (fp32 over 8 terms, then
// fp64), and the candidate masks: columns whose fp32 score reaches the row's
// screening threshold (its k-th score rounded down, less the rounding margin,
// screen_threshold) and, one pass, the column's screening threshold.
// FULL: all 32 columns are valid for the whole warp (no per-column masking).
// Two adjacent columns per instruction where the arithmetic allows it (fma / add
// .rn.f32x2: each lane of the pair rounds like the scalar instruction).
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 upk2(uint64_t r) {
    float2 f;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(r));
    return f;
}
__device__ __forceinline__ uint64_t add_x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma_x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

template <int K, int SM, bool SWAP, bool FULL, bool ONE>
__device__ __forceinline__ uint32_t chunk_phase1(const float (&v)[32], float scale, const float* cx, const float* cy,
                                                 const float* cz, float rbias_f, float rcost_f, int live, float thr,
                                                 uint32_t& cmask, double (&acc)[5]) {
    uint32_t mask = 0, cm = 0;
    uint64_t num2[2] = {0, 0}, den2[2] = {0, 0};  // partial sums of columns j & 3 = (0, 1) and (2, 3)
    float mpos = 0.0f, mcost = 0.0f;
    int cnt = 0;
    const uint64_t sc2 = pk2(scale, scale), nsc2 = pk2(-scale, -scale);
    const uint64_t rb2 = pk2(rbias_f, rbias_f), rc2 = pk2(rcost_f, rcost_f);
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        const bool ok0 = FULL || j < live, ok1 = FULL || j + 1 < live;
        const uint64_t v2 = pk2(v[j], v[j + 1]);
        // scale * v is exact (scale is a power of two), so each fma rounds like the add it replaces
        if (K > 0 || (SM & kScoreStats)) {
            const uint64_t cx2 = *reinterpret_cast<const uint64_t*>(cx + j);  // broadcast
            const uint64_t sf2 = SWAP ? add_x2(fma_x2(sc2, v2, cx2), rb2) : add_x2(fma_x2(sc2, v2, rb2), cx2);
            const float2 sf = upk2(sf2);
            if (SM & kScoreStats) {
                const bool pos0 = ok0 && sf.x > 0.0f, pos1 = ok1 && sf.y > 0.0f;
                num2[(j >> 1) & 1] = fma_x2(sf2, pk2(pos0 ? sf.x : 0.0f, pos1 ? sf.y : 0.0f), num2[(j >> 1) & 1]);
                mpos = fmaxf(mpos, FULL ? sf.x : (ok0 ? sf.x : 0.0f));
                mpos = fmaxf(mpos, FULL ? sf.y : (ok1 ? sf.y : 0.0f));
                cnt += (pos0 ? 1 : 0) + (pos1 ? 1 : 0);
            }
            if (K > 0) {
                mask |= ((ok0 && sf.x >= thr) ? (1u << j) : 0u) | ((ok1 && sf.y >= thr) ? (2u << j) : 0u);
                if (ONE) {
                    const float2 cyy = *reinterpret_cast<const float2*>(cy + j);
                    cm |= ((ok0 && sf.x >= cyy.x) ? (1u << j) : 0u) | ((ok1 && sf.y >= cyy.y) ? (2u << j) : 0u);
                }
            }
        }
        if (SM & kCostStats) {
            const uint64_t cz2 = *reinterpret_cast<const uint64_t*>(cz + j);
            const uint64_t cf2 = fma_x2(nsc2, v2, add_x2(rc2, cz2));
            const float2 cf = upk2(cf2);
            const uint64_t m2 = FULL ? cf2 : pk2(ok0 ? cf.x : 0.0f, ok1 ? cf.y : 0.0f);
            den2[(j >> 1) & 1] = fma_x2(cf2, m2, den2[(j >> 1) & 1]);
            mcost = fmaxf(mcost, ok0 ? fabsf(cf.x) : 0.0f);
            mcost = fmaxf(mcost, ok1 ? fabsf(cf.y) : 0.0f);
        }
    }
    const float2 n01 = upk2(num2[0]), n23 = upk2(num2[1]), d01 = upk2(den2[0]), d23 = upk2(den2[1]);
    const float num4[4] = {n01.x, n01.y, n23.x, n23.y}, den4[4] = {d01.x, d01.y, d23.x, d23.y};
    if (SM & kScoreStats) {
        acc[0] += ((double)num4[0] + (double)num4[1]) + ((double)num4[2] + (double)num4[3]);
        acc[2] = fmax(acc[2], (double)mpos);
        acc[4] += (double)cnt;
    }
    if (SM & kCostStats) {
        acc[1] += ((double)den4[0] + (double)den4[1]) + ((double)den4[2] + (double)den4[3]);
        acc[3] = fmax(acc[3], (double)mcost);
    }
    cmask = cm;
    return mask;
}

// Screening threshold with the rounding margin folded in: a pair whose exact score
// reaches t has an fp32 score of at least t - (2^-21 |t| + 2^-20 (|cbias| + |rbias|));
// b = 2^-20 (|cbias| + |rbias|) bounded over the tile; inflated by 2^-20 for the fp32
// evaluation of the margin itself and rounded down.
__device__ __forceinline__ float screen_threshold(float t, float b) {
    if (!(t > -INFINITY) || !(t < INFINITY)) return t;
    const float m = fmaf(fabsf(t), 0x1p-21f, b) * (1.0f + 0x1p-20f);
    return __fsub_rd(t, m);
}

// Column thresholds.  Every full column list's k-th score is a lower bound on
// the k-th best score of that column over all rows, so the largest of them is
// too: a pair below it is in no final column list and need not be offered.
// Lists of all row groups raise one shared threshold per column (atomicMax on
// an order-preserving integer image of the fp32 value, rounded down); a stale
// read only screens less.  The threshold array (4 bytes per column) stays in L2.
__device__ __forceinline__ int order_key(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float order_value(int key) { return __int_as_float(key >= 0 ? key : key ^ 0x7FFFFFFF); }

// One-pass column update of a 32 x 32 chunk (all lanes of the warp), in two
// steps so the chunk's registers are free during the list insertions:
// column_stage transposes the fp32 dots (and the rows' biases) through shared
// memory; column_update then has lane c insert the candidate rows of column c
// (the bits c of the rows' masks) into that column's list with exact fp64
// scores (dot + qb_row) + dbb_col.  The list is read from and written back to
// HBM only when the lane has a candidate, and a full list raises the column
// threshold.
// A column list (K scores, K indices) in HBM, moved with 16-byte accesses where the
// list size allows (an even size for the scores, a multiple of four for the indices).
template <int KK>
__device__ __forceinline__ void load_list(const Params& p, int64_t base, TopK<KK>& ct) {
    if constexpr (KK % 2 == 0) {
#pragma unroll
        for (int t = 0; t < KK; t += 2) {
            const double2 w = *reinterpret_cast<const double2*>(p.cval + base + t);
            ct.v[t] = w.x; ct.v[t + 1] = w.y;
        }
    } else {
#pragma unroll
        for (int t = 0; t < KK; ++t) ct.v[t] = p.cval[base + t];
    }
    if constexpr (KK % 4 == 0) {
#pragma unroll
        for (int t = 0; t < KK; t += 4) {
            const int4 w = *reinterpret_cast<const int4*>(p.cidx + base + t);
            ct.i[t] = w.x; ct.i[t + 1] = w.y; ct.i[t + 2] = w.z; ct.i[t + 3] = w.w;
        }
    } else {
#pragma unroll
        for (int t = 0; t < KK; ++t) ct.i[t] = p.cidx[base + t];
    }
}
template <int KK>
__device__ __forceinline__ void store_list(const Params& p, int64_t base, const TopK<KK>& ct) {
    if constexpr (KK % 2 == 0) {
#pragma unroll
        for (int t = 0; t < KK; t += 2)
            *reinterpret_cast<double2*>(p.cval + base + t) = make_double2(ct.v[t], ct.v[t + 1]);
    } else {
#pragma unroll
        for (int t = 0; t < KK; ++t) p.cval[base + t] = ct.v[t];
    }
    if constexpr (KK % 4 == 0) {
#pragma unroll
        for (int t = 0; t < KK; t += 4)
            *reinterpret_cast<int4*>(p.cidx + base + t) = make_int4(ct.i[t], ct.i[t + 1], ct.i[t + 2], ct.i[t + 3]);
    } else {
#pragma unroll
        for (int t = 0; t < KK; ++t) p.cidx[base + t] = ct.i[t];
    }
}

template <class S>
__device__ __forceinline__ void column_stage(S& s, const float (&v)[32], int ew, int lane, double rbias) {
    float* T = s.trans + ew * 32 * 33;
#pragma unroll
    for (int j = 0; j < 32; ++j) T[lane * 33 + j] = v[j];
    s.rbx[ew * 32 + lane] = rbias;
    __syncwarp();
}

template <int K, class S>
__device__ __forceinline__ void column_update(const Params& p, S& s, uint32_t cmask, int ew, int lane,
                                              int row0, int col0, double cbias, int64_t list_base, float scale) {
    constexpr int KK = K > 0 ? K : 1;
    const float* T = s.trans + ew * 32 * 33;
    const double* RB = s.rbx + ew * 32;
    // rows with a candidate (few once the lists have filled); lane c collects the
    // rows whose candidate mask has bit c
    uint32_t rows = __ballot_sync(0xffffffffu, cmask != 0u), mine = 0;
    while (rows) {
        const int r = __ffs(rows) - 1;
        rows &= rows - 1;
        const uint32_t m = __shfl_sync(0xffffffffu, cmask, r);
        mine |= ((m >> lane) & 1u) << r;
    }
    if (mine) {
        const int64_t base = (list_base + col0 + lane) * KK;
        TopK<KK> ct;
        load_list<KK>(p, base, ct);
        double run = p.crun ? p.crun[list_base + col0 + lane] : -INFINITY;
        while (mine) {
            const int r = __ffs(mine) - 1;
            mine &= mine - 1;
            const double dot = (double)(scale * T[r * 33 + lane]);
            ct.offer_track((dot + RB[r]) + cbias, row0 + r, run);
        }
        store_list<KK>(p, base, ct);
        if (p.crun) p.crun[list_base + col0 + lane] = run;
        if (ct.i[KK - 1] != INT32_MAX) atomicMax(p.ckey + col0 + lane, order_key(__double2float_rd(ct.v[KK - 1])));
    }
    __syncwarp();
}

// Epilogue.  Thread = one tile row (TMEM lane) in one column slice.  Per 32
// columns: phase 1 (above), then phase 2 inserts the masked columns into the
// row's k-list with exact fp64 scores (rare once the list has filled), so
// reported scores follow the reference arithmetic (dot + qb) + dbb in fp64.
template <int K, int SM, bool SWAP, bool ONE, bool PAIR = false>
__device__ __forceinline__ void epilogue(const Params& p, Smem<ONE, PAIR>& s, uint32_t tmem, double (&acc)[5]) {
    constexpr int KK = K > 0 ? K : 1;
    constexpr int EW = Epi<K>::EW;
    constexpr int SLICES = EW / 4;
    constexpr int SLICE = BN / SLICES;
    constexpr int CSLOTS = Smem<ONE, PAIR>::CS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = PAIR ? (int)cluster_rank() : 0;
    const int ew = warp - EPI_FIRST / 32;
    const int quarter = warp & 3;           // TMEM lanes this warp may read
    const int slice = ew / 4;
    const int r = quarter * 32 + lane;      // tile row owned by this thread
    float* wcx = s.colx + ew * SLICE;
    float* wcy = s.coly + ew * SLICE;
    float* wcz = s.colz + ew * SLICE;
    // one-pass: this warp's column lists (row group of the CTA [and its rank in the
    // pair], TMEM lane quarter)
    const int rgl = PAIR ? (int)(blockIdx.x >> 1) / p.groups * 2 + rank : (int)blockIdx.x / p.groups;
    const int64_t list_base = ONE ? (int64_t)(rgl * 4 + quarter) * p.n : 0;
    // CTA pairs: the accumulator is released on the even CTA's barrier
    const uint32_t tempty_peer = PAIR ? peer_smem(&s.tempty[0], 0) : 0u;
    // dot = dot_scale * 2^-(e_x + e_y) * (accumulated dot of the scaled halves): exact
    const float scale = p.terms == 3 ? ldexpf(p.scale, -(p.exps[0] + p.exps[1])) : p.scale;
    TopK<KK> top;
    uint32_t t = 0;
    const Sched sched = schedule<ONE, PAIR>(p);
    for (int u = sched.u0; u < sched.uend; u += sched.ustep) {
        const int rb = PAIR ? 2 * (u / p.groups) + rank : u / p.groups, g = u % p.groups;
        const int ct1 = min(p.ct, (g + 1) * p.tpg);
        const int row = rb * BM + r;
        const bool rvalid = row < p.q;
        const double rbias = rvalid ? p.q_bias[row] : 0.0;
        const float rbias_f = (float)rbias;
        const float rmarg_f = 0x1p-20f * fabsf(rbias_f);
        const float rbmax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(rbias_f))));
        const float rcost_f = ((SM & kCostStats) && rvalid) ? (float)p.q_cost[row] : 0.0f;
        const float rband = (p.row_err && rvalid) ? 2.0f * p.row_err[row] : 0.0f;  // 2E: the re-check band
        double run = -INFINITY;
        top.reset();
        for (int ct = g * p.tpg; ct < ct1; ++ct, ++t) {
            const uint32_t buf = t & 1, aph = (t >> 1) & 1;
            const int c0 = ct * BN + slice * SLICE;
            const int ncols = min(SLICE, p.n - c0);  // may be <= 0 for the last tile's upper slice
            const uint32_t cs = t % CSLOTS;
            if (!mbar_wait(&s.cfull[cs], (t / CSLOTS) & 1, &s.abort, p.status)) return;
            const double* wbias = s.cbias[cs] + slice * SLICE;  // exact column biases of the slice
            __syncwarp();  // the warp is done reading the previous tile's constants
            unsigned cbm = 0u;
            for (int c = lane; c < SLICE; c += 32) {
                const bool ok = c < ncols;
                const float bf = ok ? (float)wbias[c] : 0.0f;
                float cf = 0.0f, th = 0.0f;
                if constexpr ((SM & kCostStats) != 0) cf = ok ? (float)s.ccost[cs][slice * SLICE + c] : 0.0f;
                if constexpr (ONE) {
                    th = ok ? order_value(s.ckey[cs][slice * SLICE + c]) : INFINITY;
                    if (p.col_err && ok) th = __fsub_rd(th, 2.0f * s.cerr[cs][slice * SLICE + c]);
                    th = screen_threshold(th, 0x1p-20f * (fabsf(bf) + rbmax));
                }
                cbm = max(cbm, __float_as_uint(fabsf(bf)));
                wcx[c] = bf; wcy[c] = th; wcz[c] = cf;
            }
            const float cbmax = __uint_as_float(__reduce_max_sync(0xffffffffu, cbm));
            __syncwarp();
            if (!mbar_wait(&s.tfull[buf], aph, &s.abort, p.status)) return;
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + buf * BN + slice * SLICE;
            for (int ch = 0; ch < SLICE / 32 && ch * 32 < ncols; ++ch) {
                float v[32];
                tmem_ld32(taddr + ch * 32, v);
                tmem_wait_ld(v);
                const int cb = ch * 32;
                const int live = rvalid ? min(32, ncols - cb) : 0;  // valid columns of this chunk
                const float thr = top.i[KK - 1] == INT32_MAX ? -INFINITY
                                  : screen_threshold(__fsub_rd(__double2float_rd(top.v[KK - 1]), rband),
                                                     0x1p-20f * cbmax + rmarg_f);
                uint32_t mask, cmask;
                if (__all_sync(0xffffffffu, live == 32))
                    mask = chunk_phase1<K, SM, SWAP, true, ONE>(v, scale, wcx + cb, wcy + cb, wcz + cb, rbias_f, rcost_f,
                                                                live, thr, cmask, acc);
                else
                    mask = chunk_phase1<K, SM, SWAP, false, ONE>(v, scale, wcx + cb, wcy + cb, wcz + cb, rbias_f, rcost_f,
                                                                 live, thr, cmask, acc);
                const bool colwork = ONE && K > 0 && __any_sync(0xffffffffu, cmask != 0u);
                if (colwork) column_stage(s, v, ew, lane, rbias);
                // phase 2: exact fp64 scores of the masked columns into the row list
                while (K > 0 && mask) {
                    const int j = __ffs(mask) - 1;
                    mask &= mask - 1;
                    float vj = 0.0f;
#pragma unroll
                    for (int t2 = 0; t2 < 32; ++t2) vj = t2 == j ? v[t2] : vj;
                    const double dot = (double)(scale * vj);
                    const double cbias = wbias[cb + j];
                    const double sc = SWAP ? ((dot + cbias) + rbias) : ((dot + rbias) + cbias);
                    top.offer_track(sc, c0 + cb + j, run);
                }
                if (colwork)
                    column_update<K>(p, s, cmask, ew, lane, rb * BM + quarter * 32, c0 + cb, wbias[cb + lane],
                                     list_base, scale);
            }
            tc_fence_before();
            if (PAIR && rank != 0) mbar_arrive_remote(tempty_peer + buf * (uint32_t)sizeof(uint64_t));
            else mbar_arrive(&s.tempty[buf]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.cempty[cs]);  // the warp is done with the tile's column slot
        }
        if (K > 0 && rvalid) {
            const int part = g * SLICES + slice;
            double* pv = p.part_v + ((int64_t)part * p.q + row) * KK;
            int* pi = p.part_i + ((int64_t)part * p.q + row) * KK;
#pragma unroll
            for (int j = 0; j < KK; ++j) { pv[j] = top.v[j]; pi[j] = top.i[j]; }
            if (p.part_run) p.part_run[(int64_t)part * p.q + row] = run;
        }
    }
}

// CTA pairs (PAIR, launched as clusters of 2): TMEM is allocated in both CTAs by
// their warp 1 with cta_group::2; the two CTAs synchronise (cluster barrier) after
// the barrier initialisation and before the TMEM release, and every role of both
// returns to the end of the kernel, also after an aborted wait, so both always
// reach both cluster barriers.
template <int K, int SM, bool SWAP, bool ONE, bool PAIR = false>
__global__ void __launch_bounds__(Epi<K>::THREADS, 1) scan_kernel(const __grid_constant__ Params p) {
    constexpr int EW = Epi<K>::EW;
    using S = Smem<ONE, PAIR>;
    constexpr int STAGES = S::STAGES;
    extern __shared__ uint8_t smem_raw[];
    S& s = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) { mbar_init(&s.full[i], 1); mbar_init(&s.empty[i], 1); }
        for (int i = 0; i < 2; ++i) { mbar_init(&s.tfull[i], 1); mbar_init(&s.tempty[i], 32 * EW * (PAIR ? 2 : 1)); }
        for (int i = 0; i < S::CS; ++i) { mbar_init(&s.cfull[i], 1); mbar_init(&s.cempty[i], EW); }
        s.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.qmap[0]); prefetch_tmap(&p.qmap[1]);
        prefetch_tmap(&p.dmap[0]); prefetch_tmap(&p.dmap[1]);
    }
    if (warp == 1) {
        if constexpr (PAIR) { tmem_alloc_pair(&s.tmem_base, TMEM_COLS); tmem_relinquish_pair(); }
        else { tmem_alloc(&s.tmem_base, TMEM_COLS); tmem_relinquish(); }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;
    if (warp == 0) {
        if (lane == 0) producer<ONE, PAIR>(p, s);
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) mma_issuer<SWAP, ONE, PAIR>(p, s, tmem);
    } else {
        double acc[5] = {0, 0, 0, 0, 0};
        epilogue<K, SM, SWAP, ONE, PAIR>(p, s, tmem, acc);
        if (SM) {  // warp totals in a fixed shuffle order
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
                for (int j = 0; j < 5; ++j) s.red[(warp - EPI_FIRST / 32) * 5 + j] = acc[j];
        }
    }
    tc_fence_before();
    __syncthreads();  // every role returns here, also after an aborted wait
    if constexpr (PAIR) cluster_sync();  // the pair is done with each other's barriers and TMEM
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem, TMEM_COLS);
        else tmem_dealloc(tmem, TMEM_COLS);
    }
    if (SM && threadIdx.x == EPI_FIRST) {
        double a[5] = {0, 0, 0, 0, 0};
        for (int w = 0; w < EW; ++w) {
            a[0] += s.red[w * 5 + 0]; a[1] += s.red[w * 5 + 1];
            a[2] = fmax(a[2], s.red[w * 5 + 2]); a[3] = fmax(a[3], s.red[w * 5 + 3]);
            a[4] += s.red[w * 5 + 4];
        }
        for (int j = 0; j < 5; ++j) p.cta_stats[blockIdx.x * 5 + j] = a[j];
    }
}

// Column vectors padded with zeros to whole column tiles (bulk copies read
// whole tiles): dst[i] = i < n ? src[i] : 0 for up to four vectors.
struct PadJob {
    const double* src[4];
    double* dst[4];
    int64_t n[4], npad[4];
};
__global__ void pad_columns(const PadJob job) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int v = 0; v < 4; ++v) {
        if (!job.dst[v]) continue;
        for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < job.npad[v]; e += stride)
            job.dst[v][e] = e < job.n[v] ? job.src[v][e] : 0.0;
    }
}

// Empty one-pass column lists: (-inf, no index), thresholds -inf, runner-ups -inf.
__global__ void init_columns(double* cval, int* cidx, int* ckey, int64_t lists, int64_t n, int K, double* crun) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t total = lists * K > n ? lists * K : n;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        if (e < lists * K) { cval[e] = -INFINITY; cidx[e] = INT32_MAX; }
        if (crun && e < lists) crun[e] = -INFINITY;
        if (e < n) ckey[e] = order_key(-INFINITY);
    }
}

// Largest |x| of a cloud (rows x d contiguous fp32) as its bit pattern (atomicMax on
// non-negative floats orders like the values); *out must start at 0.
__global__ void absmax_kernel(const float* __restrict__ x, int64_t total, unsigned* out) {
    unsigned m = 0;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x)
        m = max(m, __float_as_uint(fabsf(x[e])));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0 && m) atomicMax(out, m);
}

// The cloud's power-of-two scale: max |x| 2^e in [2^14, 2^15), e clamped to [-60, 60] so
// that 2^-(e_x + e_y) stays a normal fp32 number (clouds below 2^-46 lose low bits to
// fp16 subnormals).  A largest |x| of 2^75 or more (or a non-finite one) cannot be
// represented and is reported as bad input.
__device__ __forceinline__ int cloud_exponent(unsigned bits, int* status) {
    if (bits == 0u) return 0;  // an all-zero cloud
    const float m = __uint_as_float(bits);
    if (!(m < 0x1p75f)) { atomicOr(status, kErrBadInput); return 0; }  // too large, infinite or NaN
    int ex = 0;
    frexpf(m, &ex);  // m = f 2^ex, f in [0.5, 1)
    return max(-60, min(60, 15 - ex));
}

// fp16 halves of a cloud, rows padded to dp16 (a multiple of 8) with zeros:
// hi = fp16(x 2^e), lo = fp16(x 2^e - hi); block 0 also records e.
__global__ void prep_f16(const float* __restrict__ x, int64_t rows, int d, int dp16, const unsigned* amax,
                         int* exp_out, int* status, __half* __restrict__ hi, __half* __restrict__ lo) {
    const int e = cloud_exponent(*amax, status);
    if (blockIdx.x == 0 && threadIdx.x == 0) *exp_out = e;
    const int64_t total = rows * dp16;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / dp16;
        const int c = (int)(i - r * dp16);
        const float v = c < d ? ldexpf(x[r * d + c], e) : 0.0f;
        const __half h = __float2half_rn(v);
        hi[i] = h;
        lo[i] = __float2half_rn(v - __half2float(h));
    }
}

// One-product (TF32) mode: copy fp32 features into a TMA-legal layout (row stride a
// multiple of 16 B, zero padded) when d is not a multiple of 4.
__global__ void prep_kernel(const float* __restrict__ x, int64_t rows, int d, int dp, float* __restrict__ xpad) {
    const int64_t total = rows * dp;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / dp;
        const int c = (int)(e - r * dp);
        xpad[e] = c < d ? x[r * d + c] : 0.0f;
    }
}

}  // namespace l2sq

// ------------------------------------------------------------------ host side
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(ptr);
    }
    return fn;
}

// 2-D map of a row-major [rows][dp] operand read in 64-byte slab rows (16 fp32 or
// 32 fp16 elements) with the 64-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int dp, int box_rows, bool f16 = false) {
    EncodeTiled enc = encode_fn();
    if (!enc) return false;
    const size_t es = f16 ? 2 : 4;
    cuuint64_t dims[2] = {(cuuint64_t)dp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)dp * es};
    cuuint32_t box[2] = {(cuuint32_t)(f16 ? l2sq::BK16 : l2sq::BK), (cuuint32_t)box_rows};  // 64-byte rows
    cuuint32_t estr[2] = {1, 1};
    return enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base),
               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int K, int SM, bool SWAP, bool ONE = false, bool PAIR = false>
cudaError_t launch_pass(const l2sq::Params& p, int grid, cudaStream_t st) {
    auto fn = l2sq::scan_kernel<K, SM, SWAP, ONE, PAIR>;
    constexpr size_t smem = l2sq::smem_bytes<ONE, PAIR>();
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    timing_mark(st);
    if constexpr (PAIR) {  // clusters of two CTAs (grid is even)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(l2sq::Epi<K>::THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, fn, p);
        timing_mark(st);
        count_launches(1);
        return e != cudaSuccess ? e : cudaGetLastError();
    }
    fn<<<grid, l2sq::Epi<K>::THREADS, smem, st>>>(p);
    timing_mark(st);
    count_launches(1);
    return cudaGetLastError();
}

// Clusters of two CTAs of the paired one-pass kernel that fit on the device at once.
int pair_clusters() {
    static int cached = -1;
    if (cached >= 0) return cached;
    auto fn = l2sq::scan_kernel<8, l2sq::kScoreStats | l2sq::kCostStats, false, true, true>;
    constexpr size_t smem = l2sq::smem_bytes<true, true>();
    int n = 0;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2);
        cfg.blockDim = dim3(l2sq::Epi<8>::THREADS);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();  // clear a failed query
    cached = n;
    return n;
}

template <int SM, bool SWAP>
cudaError_t launch_k(int K, const l2sq::Params& p, int grid, cudaStream_t st) {
    switch (K) {
        case 1: return launch_pass<1, SM, SWAP>(p, grid, st);
        case 2: return launch_pass<2, SM, SWAP>(p, grid, st);
        case 4: return launch_pass<4, SM, SWAP>(p, grid, st);
        case 8: return launch_pass<8, SM, SWAP>(p, grid, st);
        case 16: return launch_pass<16, SM, SWAP>(p, grid, st);
        case 32: return launch_pass<32, SM, SWAP>(p, grid, st);
        // list sizes of the fp64 re-check (bucket + EXACT_EXTRA)
        case 3: return launch_pass<3, SM, SWAP>(p, grid, st);
        case 6: return launch_pass<6, SM, SWAP>(p, grid, st);
        case 10: return launch_pass<10, SM, SWAP>(p, grid, st);
        case 18: return launch_pass<18, SM, SWAP>(p, grid, st);
        case 34: return launch_pass<34, SM, SWAP>(p, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

template <int SM, bool PAIR = false>
cudaError_t launch_one(int K, const l2sq::Params& p, int grid, cudaStream_t st) {
    switch (K) {
        case 1: return launch_pass<1, SM, false, true, PAIR>(p, grid, st);
        case 2: return launch_pass<2, SM, false, true, PAIR>(p, grid, st);
        case 4: return launch_pass<4, SM, false, true, PAIR>(p, grid, st);
        case 8: return launch_pass<8, SM, false, true, PAIR>(p, grid, st);
        case 3: return launch_pass<3, SM, false, true, PAIR>(p, grid, st);
        case 6: return launch_pass<6, SM, false, true, PAIR>(p, grid, st);
        case 10: return launch_pass<10, SM, false, true, PAIR>(p, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

int device_sms() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace

template <int K>
cudaError_t launch_merge(const double* pv, const int* pi, int parts, int64_t rows, int width, int k_out, double* ov,
                         int* oi, cudaStream_t st, const double* pr, double* run_out) {
    merge_partials<K><<<(unsigned)((rows + 127) / 128), 128, 0, st>>>(pv, pi, parts, rows, width, k_out, ov, oi, pr,
                                                                       run_out);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t merge_any(int K, const double* pv, const int* pi, int parts, int64_t rows, int k_out, double* ov, int* oi,
                      cudaStream_t st, const double* pr, double* run_out) {
    return merge_lists(K, pv, pi, parts, rows, K, k_out, ov, oi, st, pr, run_out);
}

cudaError_t merge_lists(int K, const double* pv, const int* pi, int parts, int64_t rows, int width, int k_out,
                        double* ov, int* oi, cudaStream_t st, const double* pr, double* run_out) {
    switch (K) {
        case 1: return launch_merge<1>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 2: return launch_merge<2>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 4: return launch_merge<4>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 8: return launch_merge<8>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 16: return launch_merge<16>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 32: return launch_merge<32>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        // list sizes of the fp64 re-check (bucket + EXACT_EXTRA)
        case 3: return launch_merge<3>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 6: return launch_merge<6>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 10: return launch_merge<10>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 18: return launch_merge<18>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        case 34: return launch_merge<34>(pv, pi, parts, rows, width, k_out, ov, oi, st, pr, run_out);
        default: return cudaErrorInvalidValue;
    }
}

// Column slices per tile (= row partial lists per unit) of the bucket-K kernel.
inline int l2sq_slices(int K) { return (K <= 10 ? 8 : 4) / 4; }
// The fp64 re-check keeps EXACT_EXTRA more entries than the bucket in every list: the
// re-scored candidates then include the bucket's next entries, so a list needs a full
// rescan only when EXACT_EXTRA + 1 approximate scores fall within the error band of the
// k-th (a near tie of the k-th and the (k+1)-th alone is settled by the re-score).
constexpr int EXACT_EXTRA = 2;
inline int list_size(int K, bool exact) { return exact ? K + EXACT_EXTRA : K; }

// One-pass rectangle plan: GR row groups x GC column groups, one CTA each.
// Few row groups keep the number of column partial lists (4 GR per column)
// and their insertions small; each row group re-reads its column groups'
// features once per row block, which costs HBM bandwidth (not the bound).
constexpr int ONE_PASS_ROW_GROUPS = 8;
// Automatic choice: the one-pass epilogue costs about the same per pair at any
// d (list upkeep), the tensor-core work grows with d, and the column lists see
// more rows (fewer insertions) as q grows.
// CTA pairs for the one-pass kernel: forced by HB_L2SQ_CTA_PAIRS or HB_L2SQ_SINGLE_CTA,
// else chosen for wide features (needs clusters of two to fit on the device).  Measured
// on one B200, same data, alternating runs: d = 2048 (131072^2) 50.8 Gpairs/s paired
// against 46.9 single; d = 256 (1048576^2) 304.9 against 309.5, where the 1 kW power cap
// sets the clock and the halved column-tile traffic buys nothing.
constexpr int64_t PAIRS_MIN_D = 1024;
inline bool use_pairs(int precision, int64_t d) {
    if (precision & HB_L2SQ_SINGLE_CTA) return false;
    if (!(precision & HB_L2SQ_CTA_PAIRS) && d < PAIRS_MIN_D) return false;
    return pair_clusters() > 0;
}
inline bool use_one_pass(int K, int precision, int64_t q, int64_t d) {
    if (K < 1 || K > 8 || (precision & (HB_L2SQ_TWO_PASS | L2SQ_ROWS_ONLY))) return false;
    if (precision & HB_L2SQ_ONE_PASS) return true;
    (void)q;
    return d >= 128;
}

// CTA pairs: a rectangle is a cluster of two CTAs whose units are pairs of row
// blocks (rb counts them); half as many row groups keep the same number of column
// lists per column (4 x 2 ranks x 4 quarters), and each column tile is read by
// half as many rectangles.
struct OnePlan {
    int rb, ct, gr, rbg, gc, tpg, grid;
    bool pair;
    int lists_per_col() const { return gr * (pair ? 2 : 1) * 4; }
};
inline OnePlan one_plan(int64_t q, int64_t n, int sms, int min_groups, bool pair = false, int clusters = 0) {
    OnePlan o{};
    o.pair = pair;
    const int rows_per_unit = l2sq::BM * (pair ? 2 : 1);
    o.rb = (int)((q + rows_per_unit - 1) / rows_per_unit);
    o.ct = (int)((n + l2sq::BN - 1) / l2sq::BN);
    o.gr = std::min(ONE_PASS_ROW_GROUPS / (pair ? 2 : 1), o.rb);
    o.rbg = (o.rb + o.gr - 1) / o.gr;
    o.gr = (o.rb + o.rbg - 1) / o.rbg;
    const int slots = pair ? clusters : sms;  // rectangles that run at once
    int gc = std::max(1, std::max(slots / o.gr, min_groups));
    gc = std::min(gc, o.ct);
    o.tpg = (o.ct + gc - 1) / gc;
    o.gc = (o.ct + o.tpg - 1) / o.tpg;
    o.grid = o.gr * o.gc * (pair ? 2 : 1);
    return o;
}

// Scratch layout of one ℓ2² scan call.  With base == nullptr only sizes it.
struct L2sqLayout {
    float *xpad = nullptr, *ypad = nullptr;
    __half *xh = nullptr, *xl = nullptr, *yh = nullptr, *yl = nullptr;  // 3-term split: fp16 halves
    unsigned* amax = nullptr;  // [2] largest |x|, |y| (bit patterns)
    int* exps = nullptr;       // [2] the clouds' power-of-two scales
    double *pv1 = nullptr, *pv2 = nullptr, *cta = nullptr;
    int *pi1 = nullptr, *pi2 = nullptr, *status = nullptr;
    int* ckey = nullptr;  // one-pass column lists and thresholds
    int* progress = nullptr;
    double *ybp = nullptr, *ycp = nullptr, *xbp = nullptr, *xcp = nullptr;  // padded column vectors
    double* cval = nullptr;
    int* cidx = nullptr;
    // fp64 re-check (HB_L2SQ_EXACT): error bounds, runner-ups, list-size approximate lists, flags
    bool exact = false;
    float *xnorm = nullptr, *ynorm = nullptr, *xerr = nullptr, *yerr = nullptr;
    unsigned* nmax = nullptr;
    double *prun1 = nullptr, *prun2 = nullptr, *crun = nullptr, *run1 = nullptr, *run2 = nullptr;
    double *tv1 = nullptr, *tv2 = nullptr;
    int *ti1 = nullptr, *ti2 = nullptr, *flag1 = nullptr, *flag2 = nullptr, *nflag = nullptr;
    ScanPlan p1{}, p2{};
    OnePlan one{};
    bool one_pass = false;
    size_t bytes = 0;
    bool ok = true;
};

L2sqLayout l2sq_layout(void* base, size_t size, int64_t q, int64_t n, int64_t d, int k, int precision, int min_groups) {
    L2sqLayout L;
    const int sms = device_sms();
    const int K = k > 0 ? bucket_of(k) : 0;
    const int prec = precision & 0xF;
    const int dp = (int)((d + 3) / 4 * 4);
    const int dp16 = (int)((d + 7) / 8 * 8);
    const bool pad = prec != 3 && dp != d;
    Arena ar{static_cast<char*>(base), size, 0};
    auto need = [&](bool cond, auto*& ptr, size_t count) {
        using T = std::remove_pointer_t<std::remove_reference_t<decltype(ptr)>>;
        if (!cond) return;
        ptr = ar.take<T>(count);
        if (base && !ptr) L.ok = false;
    };
    need(pad, L.xpad, (size_t)q * dp);
    need(pad, L.ypad, (size_t)n * dp);
    need(prec == 3, L.xh, (size_t)q * dp16);
    need(prec == 3, L.xl, (size_t)q * dp16);
    need(prec == 3, L.yh, (size_t)n * dp16);
    need(prec == 3, L.yl, (size_t)n * dp16);
    need(prec == 3, L.amax, 2);
    need(prec == 3, L.exps, 2);
    const size_t npad = (size_t)(n + l2sq::BN - 1) / l2sq::BN * l2sq::BN;
    const size_t qpad = (size_t)(q + l2sq::BN - 1) / l2sq::BN * l2sq::BN;
    L.one_pass = use_one_pass(K, precision, q, d);
    const bool rows_only = (precision & L2SQ_ROWS_ONLY) != 0;
    L.exact = (precision & HB_L2SQ_EXACT) && K > 0 && !rows_only;
    const int LK = list_size(K, L.exact);  // entries per list
    const int slices = K > 0 ? l2sq_slices(LK) : 1;
    need(L.exact, L.xnorm, (size_t)2 * q);
    need(L.exact, L.ynorm, (size_t)2 * n);
    need(L.exact, L.xerr, (size_t)q);
    need(L.exact, L.yerr, npad > qpad ? npad : qpad);
    need(L.exact, L.nmax, 4);
    need(L.exact, L.run1, (size_t)q);
    need(L.exact, L.run2, (size_t)n);
    need(L.exact, L.tv1, (size_t)q * LK);
    need(L.exact, L.ti1, (size_t)q * LK);
    need(L.exact, L.tv2, (size_t)n * LK);
    need(L.exact, L.ti2, (size_t)n * LK);
    need(L.exact, L.flag1, (size_t)q);
    need(L.exact, L.flag2, (size_t)n);
    need(L.exact, L.nflag, 2);
    need(true, L.ybp, npad);
    need(!rows_only, L.ycp, npad);
    need(!L.one_pass && !rows_only && K > 0, L.xbp, qpad);
    need(!L.one_pass && !rows_only && K > 0, L.xcp, qpad);
    if (L.one_pass) {
        const bool pair = use_pairs(precision, d);
        L.one = one_plan(q, n, sms, min_groups, pair, pair ? pair_clusters() : 0);
        const size_t lists = (size_t)L.one.lists_per_col() * n;
        need(true, L.pv1, (size_t)L.one.gc * slices * q * LK);
        need(true, L.pi1, (size_t)L.one.gc * slices * q * LK);
        need(true, L.cval, lists * LK);
        need(true, L.cidx, lists * LK);
        need(true, L.ckey, npad);
        need(true, L.progress, (size_t)L.one.grid);
        need(true, L.cta, (size_t)L.one.grid * 5);
        need(L.exact, L.prun1, (size_t)L.one.gc * slices * q);
        need(L.exact, L.crun, lists);
    } else {
        // features wider than ~1k keep more column groups so the row-block slabs in flight fit in L2
        const int wide = (int)(d / 1024) + 1;
        L.p1 = scan_plan(q, n, l2sq::BM, l2sq::BN, 1, sms, min_groups > 0 ? min_groups : wide);
        L.p2 = scan_plan(n, q, l2sq::BM, l2sq::BN, 1, sms, min_groups > 0 ? min_groups : wide);
        need(K > 0, L.pv1, (size_t)L.p1.groups * slices * q * LK);
        need(K > 0, L.pi1, (size_t)L.p1.groups * slices * q * LK);
        need(K > 0 && !rows_only, L.pv2, (size_t)L.p2.groups * slices * n * LK);
        need(K > 0 && !rows_only, L.pi2, (size_t)L.p2.groups * slices * n * LK);
        need(true, L.cta, (size_t)(L.p1.grid + L.p2.grid) * 5);
        need(L.exact, L.prun1, (size_t)L.p1.groups * slices * q);
        need(L.exact, L.prun2, (size_t)L.p2.groups * slices * n);
    }
    need(true, L.status, 1);
    L.bytes = ar.used + 256;
    return L;
}

size_t l2sq_bytes(int64_t q, int64_t n, int64_t d, int k, int precision, int min_groups) {
    return l2sq_layout(nullptr, 0, q, n, d, k, precision, min_groups).bytes;
}

int l2sq_scan(const float* x, const float* y, int64_t q, int64_t n, int64_t d, const double* nx, const double* ny,
              const double* qb, const double* dbb, int k, double dot_scale, int want_stats, int precision,
              int min_groups, double* rv, int* ri, double* cv, int* ci, double* stats5, void* ws, size_t ws_bytes,
              int* status_out, cudaStream_t st, std::string& err, int* rescans_out) {
    L2sqLayout L = l2sq_layout(ws, ws_bytes, q, n, d, k, precision, min_groups);
    if (!L.ok) { err = "workspace too small for the l2sq scan"; return 3; }
    const int K = k > 0 ? bucket_of(k) : 0;
    const int LK = list_size(K, L.exact);  // entries per list (the kernels' K)
    const int prec = precision & 0xF;
    const bool rows_only = (precision & L2SQ_ROWS_ONLY) != 0;
    if (rows_only) want_stats = 0;
    const int dp = (int)((d + 3) / 4 * 4);
    const int dp16 = (int)((d + 7) / 8 * 8);
    cudaError_t e = cudaMemsetAsync(L.status, 0, sizeof(int), st);
    if (e != cudaSuccess) { err = cudaGetErrorString(e); return 4; }
    const float* xs = x;
    const float* ys = y;
    const int prep_blocks = device_sms() * 8;
    if (prec == 3) {  // fp16 halves of both clouds, each scaled by its power of two
        e = cudaMemsetAsync(L.amax, 0, 2 * sizeof(unsigned), st);
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 4; }
        l2sq::absmax_kernel<<<prep_blocks, 256, 0, st>>>(x, q * d, L.amax);
        l2sq::absmax_kernel<<<prep_blocks, 256, 0, st>>>(y, n * d, L.amax + 1);
        l2sq::prep_f16<<<prep_blocks, 256, 0, st>>>(x, q, (int)d, dp16, L.amax, L.exps, L.status, L.xh, L.xl);
        l2sq::prep_f16<<<prep_blocks, 256, 0, st>>>(y, n, (int)d, dp16, L.amax + 1, L.exps + 1, L.status, L.yh, L.yl);
        count_launches(4);
    } else if (L.xpad) {
        l2sq::prep_kernel<<<prep_blocks, 256, 0, st>>>(x, q, (int)d, dp, L.xpad);
        l2sq::prep_kernel<<<prep_blocks, 256, 0, st>>>(y, n, (int)d, dp, L.ypad);
        count_launches(2);
        xs = L.xpad; ys = L.ypad;
    }
    const int64_t npad = (n + l2sq::BN - 1) / l2sq::BN * l2sq::BN;
    const int64_t qpad = (q + l2sq::BN - 1) / l2sq::BN * l2sq::BN;
    if (L.exact) {  // error bounds of both clouds' approximate scores (y's padded to whole tiles)
        e = exact_bounds(x, y, q, n, (int)d, npad, prec, prec == 3 ? L.exps : nullptr, dot_scale, L.xnorm, L.ynorm,
                         L.nmax, L.xerr, L.yerr, device_sms(), st);
        if (e != cudaSuccess) { err = std::string("l2sq exact bounds: ") + cudaGetErrorString(e); return 6; }
    }
    {
        l2sq::PadJob job{};
        job.src[0] = dbb; job.dst[0] = L.ybp; job.n[0] = n; job.npad[0] = npad;
        job.src[1] = ny; job.dst[1] = L.ycp; job.n[1] = n; job.npad[1] = npad;
        job.src[2] = qb; job.dst[2] = L.xbp; job.n[2] = q; job.npad[2] = qpad;
        job.src[3] = nx; job.dst[3] = L.xcp; job.n[3] = q; job.npad[3] = qpad;
        l2sq::pad_columns<<<prep_blocks, 256, 0, st>>>(job);
        count_launches(1);
    }
    l2sq::Params p;
    std::memset(&p, 0, sizeof(p));
    const bool pair = L.one_pass && L.one.pair;
    const int brows = pair ? l2sq::BNH : l2sq::BN;  // database box: half a column tile per CTA of a pair
    bool maps;
    if (prec == 3) {
        maps = make_map(&p.qmap[0], L.xh, q, dp16, l2sq::BM, true) && make_map(&p.dmap[0], L.yh, n, dp16, brows, true) &&
               make_map(&p.qmap[1], L.xl, q, dp16, l2sq::BM, true) && make_map(&p.dmap[1], L.yl, n, dp16, brows, true);
    } else {
        maps = make_map(&p.qmap[0], xs, q, dp, l2sq::BM) && make_map(&p.dmap[0], ys, n, dp, brows);
        p.qmap[1] = p.qmap[0]; p.dmap[1] = p.dmap[0];
    }
    if (!maps) { err = "cuTensorMapEncodeTiled failed (alignment or driver entry point)"; return 5; }
    p.terms = prec == 3 ? 3 : 1;
    p.kslabs = prec == 3 ? (dp16 + l2sq::BK16 - 1) / l2sq::BK16 : (dp + l2sq::BK - 1) / l2sq::BK;
    p.exps = L.exps;
    p.scale = (float)dot_scale;
    p.status = L.status;
    p.cta_stats = L.cta;
    p.q = (int)q; p.n = (int)n;
    p.q_cost = nx; p.d_cost = L.ycp; p.q_bias = qb; p.d_bias = L.ybp;
    p.part_v = L.pv1; p.part_i = L.pi1;
    if (L.exact) { p.row_err = L.xerr; p.part_run = L.prun1; }
    // the exact lists of one side: list-size approximate lists with runner-ups re-scored in fp64
    auto finish_side = [&](bool cols) -> cudaError_t {
        ExactSide sd{};
        sd.qf = cols ? y : x; sd.dbf = cols ? x : y;
        sd.nq = cols ? n : q; sd.ndb = cols ? q : n;
        sd.qbias = cols ? dbb : qb; sd.dbias = cols ? qb : dbb;
        sd.lv = cols ? L.tv2 : L.tv1; sd.li = cols ? L.ti2 : L.ti1; sd.run = cols ? L.run2 : L.run1;
        sd.qerr = cols ? L.yerr : L.xerr;
        sd.ov = cols ? cv : rv; sd.oi = cols ? ci : ri;
        sd.flags = cols ? L.flag2 : L.flag1; sd.nflag = L.nflag + (cols ? 1 : 0);
        sd.swap = cols;
        return exact_finish(LK, sd, (int)d, dot_scale, k, device_sms(), st);
    };
    if (L.one_pass) {
        // one pass: row lists in registers, column lists per (row group, lane quarter) in HBM
        const OnePlan& o = L.one;
        const int64_t lists = (int64_t)o.lists_per_col() * n;
        l2sq::init_columns<<<prep_blocks, 256, 0, st>>>(L.cval, L.cidx, L.ckey, lists, npad, LK, L.crun);
        count_launches(1);
        p.groups = o.gc; p.tpg = o.tpg; p.ct = o.ct; p.units = o.rb * o.gc;
        p.rb = o.rb; p.rbg = o.rbg;
        p.ckey = L.ckey; p.cval = L.cval; p.cidx = L.cidx;
        p.progress = L.progress;
        if (L.exact) { p.col_err = L.yerr; p.crun = L.crun; }
        e = cudaMemsetAsync(L.progress, 0, sizeof(int) * o.grid, st);
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 4; }
        if (!want_stats) p.d_cost = nullptr;  // the cost vector is staged only for the cost terms
        if (o.pair)
            e = want_stats ? launch_one<l2sq::kScoreStats | l2sq::kCostStats, true>(LK, p, o.grid, st)
                           : launch_one<0, true>(LK, p, o.grid, st);
        else
            e = want_stats ? launch_one<l2sq::kScoreStats | l2sq::kCostStats>(LK, p, o.grid, st)
                           : launch_one<0>(LK, p, o.grid, st);
        if (e != cudaSuccess) { err = std::string("l2sq scan: ") + cudaGetErrorString(e); return 6; }
        if (L.exact) {
            e = merge_any(LK, L.pv1, L.pi1, o.gc * l2sq_slices(LK), q, LK, L.tv1, L.ti1, st, L.prun1, L.run1);
            if (e == cudaSuccess)
                e = merge_any(LK, L.cval, L.cidx, o.lists_per_col(), n, LK, L.tv2, L.ti2, st, L.crun, L.run2);
            if (e == cudaSuccess) e = finish_side(false);
            if (e == cudaSuccess) e = finish_side(true);
        } else {
            e = merge_any(K, L.pv1, L.pi1, o.gc * l2sq_slices(K), q, k, rv, ri, st);
            if (e == cudaSuccess) e = merge_any(K, L.cval, L.cidx, o.lists_per_col(), n, k, cv, ci, st);
        }
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
        if (want_stats) {
            finalize_stats<<<1, 32, 0, st>>>(L.cta, o.grid, stats5);
            count_launches(1);
        }
        if (status_out) cudaMemcpyAsync(status_out, L.status, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (rescans_out && L.exact) cudaMemcpyAsync(rescans_out, L.nflag, 2 * sizeof(int), cudaMemcpyDeviceToHost, st);
        return 0;
    }
    // pass 1: x rows are the queries (row top-k + certificate)
    p.groups = L.p1.groups; p.tpg = L.p1.tpg; p.ct = L.p1.ct; p.units = L.p1.units;
    if (K != 0) p.d_cost = nullptr;  // cost terms are in pass 2 (a certificate-only pass takes all terms)
    // certificate: score terms in the row pass, cost terms in the column pass
    // (a certificate-only call has no column pass and takes all terms here)
    if (K == 0) e = launch_pass<0, l2sq::kScoreStats | l2sq::kCostStats, false>(p, L.p1.grid, st);
    else e = want_stats ? launch_k<l2sq::kScoreStats, false>(LK, p, L.p1.grid, st)
                        : launch_k<0, false>(LK, p, L.p1.grid, st);
    if (e != cudaSuccess) { err = std::string("l2sq pass 1: ") + cudaGetErrorString(e); return 6; }
    if (K > 0) {
        e = L.exact ? merge_any(LK, L.pv1, L.pi1, L.p1.groups * l2sq_slices(LK), q, LK, L.tv1, L.ti1, st, L.prun1, L.run1)
                    : merge_any(K, L.pv1, L.pi1, L.p1.groups * l2sq_slices(K), q, k, rv, ri, st);
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
    }
    if (K > 0 && !rows_only) {
        // pass 2: y rows are the queries, same products in the same order;
        // the maps are rebuilt because a map fixes its box height (A 128 rows, B 256 rows)
        l2sq::Params p2 = p;
        bool maps2;
        if (prec == 3) {
            maps2 = make_map(&p2.qmap[0], L.yh, n, dp16, l2sq::BM, true) &&
                    make_map(&p2.dmap[0], L.xh, q, dp16, l2sq::BN, true) &&
                    make_map(&p2.qmap[1], L.yl, n, dp16, l2sq::BM, true) &&
                    make_map(&p2.dmap[1], L.xl, q, dp16, l2sq::BN, true);
        } else {
            maps2 = make_map(&p2.qmap[0], ys, n, dp, l2sq::BM) && make_map(&p2.dmap[0], xs, q, dp, l2sq::BN);
            p2.qmap[1] = p2.qmap[0]; p2.dmap[1] = p2.dmap[0];
        }
        if (!maps2) { err = "cuTensorMapEncodeTiled failed (alignment or driver entry point)"; return 5; }
        p2.q = (int)n; p2.n = (int)q;
        p2.groups = L.p2.groups; p2.tpg = L.p2.tpg; p2.ct = L.p2.ct; p2.units = L.p2.units;
        p2.q_cost = ny; p2.d_cost = want_stats ? L.xcp : nullptr; p2.q_bias = dbb; p2.d_bias = L.xbp;
        p2.part_v = L.pv2; p2.part_i = L.pi2;
        if (L.exact) { p2.row_err = L.yerr; p2.part_run = L.prun2; }
        p2.cta_stats = L.cta + (size_t)L.p1.grid * 5;
        e = want_stats ? launch_k<l2sq::kCostStats, true>(LK, p2, L.p2.grid, st) : launch_k<0, true>(LK, p2, L.p2.grid, st);
        if (e != cudaSuccess) { err = std::string("l2sq pass 2: ") + cudaGetErrorString(e); return 6; }
        e = L.exact ? merge_any(LK, L.pv2, L.pi2, L.p2.groups * l2sq_slices(LK), n, LK, L.tv2, L.ti2, st, L.prun2, L.run2)
                    : merge_any(K, L.pv2, L.pi2, L.p2.groups * l2sq_slices(K), n, k, cv, ci, st);
        if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
        if (L.exact) {
            e = finish_side(false);
            if (e == cudaSuccess) e = finish_side(true);
            if (e != cudaSuccess) { err = cudaGetErrorString(e); return 6; }
        }
    }
    if (want_stats) {  // per-CTA partials of both passes, unused terms are zero
        finalize_stats<<<1, 32, 0, st>>>(L.cta, L.p1.grid + (K > 0 ? L.p2.grid : 0), stats5);
        count_launches(1);
    }
    if (status_out) cudaMemcpyAsync(status_out, L.status, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (rescans_out && L.exact) cudaMemcpyAsync(rescans_out, L.nflag, 2 * sizeof(int), cudaMemcpyDeviceToHost, st);
    return 0;
}

}  // namespace hb
