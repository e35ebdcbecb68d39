/*
 * CPU oracle for the HELLO hot path: pricing scan, active-support pair costs
 * and the restricted-OT Halpern-PDHG.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the hello-ot_b200
 * package, its CUDA library or its C ABI) may call, link or load this file.
 * It is used by tests/, by __graft_entry__.smoke() as the checker, and by
 * bench.py's cpu_baseline / reference legs.
 *
 * Every function restates the reference algorithm in plain C; the reference
 * file:line each one follows is cited beside it (paths inside the reference
 * project, src/hello_ot/ abbreviated to h/).  Build: `make -C oracle`.
 * The restatement is pinned against the reference's own C++ backend compiled
 * from its sources into oracle/_ref (see oracle/Makefile and
 * tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_NO_INDEX INT64_MAX

/* Candidate order of every top-k in the reference: larger score first, the
 * lower index wins an exact tie, NaN never enters.  h/_native/generic_scan/
 * pricing_small.cu:37-50 (IEEE order keys on sm_100 are equivalent to the
 * plain comparison below: +0 == -0, NaN compares false). */
static inline int orc_better(double a, int64_t ai, double b, int64_t bi) {
    return a > b || (a == b && ai < bi);
}

/* Sorted insertion into a k-slot list, pricing_small.cu:51-59. */
static inline void orc_insert(double* v, int64_t* ix, int k, double a, int64_t ai) {
    if (!orc_better(a, ai, v[k - 1], ix[k - 1])) return;
    int p = k - 1;
    while (p > 0 && orc_better(a, ai, v[p - 1], ix[p - 1])) {
        v[p] = v[p - 1];
        ix[p] = ix[p - 1];
        --p;
    }
    v[p] = a;
    ix[p] = ai;
}

typedef struct {
    int kind;      /* 0 l1, 1 linf, 2 l2, 3 raw bilinear (l2^2 lowered) */
    int exact;     /* 1: fp64 arithmetic on the fp32 inputs; 0: sequential fp32 model */
    const float* x;
    const float* y;
    int64_t d;
    const double* rowb; /* raw: query bias f - a;  norms: f */
    const double* colb; /* raw: db bias g - b;     norms: g */
    const double* nx;   /* raw only: a = |x|^2 */
    const double* ny;   /* raw only: b = |y|^2 */
    double scale;       /* raw only: dot_scale in {1, 2} */
} orc_scan_ctx;

/* Score and cost of one pair.
 * raw:   dot = s<x,y>;  cost = (a_i + b_j) - dot;  score = (dot + qb_i) + dbb_j
 *        h/_native/generic_scan/matrix_selection.cuh:20-26 (RAW branch) with
 *        the SGEMM alpha applied in fp32, pricing_small.cu:241-256.
 * norms: score = (g_j - c_ij) + f_i, pricing_small.cu:112;
 *        c = sum|x-y| / max|x-y| / sqrt(sum (x-y)^2), pricing_small.cu:62-67;
 *        the fp32 model (exact == 0) accumulates in feature order, ℓ2 with one
 *        fma per term. */
static inline void orc_pair(const orc_scan_ctx* c, int64_t i, int64_t j, double* score, double* cost) {
    const float* xi = c->x + i * c->d;
    const float* yj = c->y + j * c->d;
    if (c->kind == 3) {
        double dot;
        if (c->exact) {
            double acc = 0.0;
            for (int64_t k = 0; k < c->d; ++k) acc += (double)xi[k] * (double)yj[k];
            dot = c->scale * acc;
        } else {
            float acc = 0.0f;
            for (int64_t k = 0; k < c->d; ++k) acc = acc + xi[k] * yj[k];
            dot = (double)((float)c->scale * acc);
        }
        *cost = (c->nx[i] + c->ny[j]) - dot;
        *score = (dot + c->rowb[i]) + c->colb[j];
        return;
    }
    double dist;
    if (c->exact) {
        double acc = 0.0;
        for (int64_t k = 0; k < c->d; ++k) {
            double z = (double)yj[k] - (double)xi[k];
            if (c->kind == 0) acc += fabs(z);
            else if (c->kind == 1) acc = fmax(acc, fabs(z));
            else acc += z * z;
        }
        dist = c->kind == 2 ? sqrt(acc) : acc;
    } else {
        float acc = 0.0f;
        for (int64_t k = 0; k < c->d; ++k) {
            float z = xi[k] - yj[k];
            if (c->kind == 0) acc = acc + fabsf(z);
            else if (c->kind == 1) acc = fmaxf(acc, fabsf(z));
            else acc = fmaf(z, z, acc);
        }
        dist = c->kind == 2 ? (double)sqrtf(acc) : (double)acc;
    }
    *cost = dist;
    *score = (c->colb[j] - dist) + c->rowb[i];
}

/* Bidirectional pricing scan: per query row its rk best (score, column),
 * per database column its ck best (score, row), and the five certificate
 * sums over all q*n pairs [sum max(s,0)^2, sum c^2, max s+, max |c|, #s>0]
 * (pricing_small.cu:70-160; certificate formula h/kernels/bilinear_topk.py:440).
 * Missing slots are (-inf, -1).  rk or ck may be 0 to skip a direction. */
int orc_scan(int kind, int exact, const float* x, const float* y, int64_t q, int64_t n, int64_t d,
             const double* rowb, const double* colb, const double* nx, const double* ny, double scale,
             int rk, int ck, double* rv, int64_t* ri, double* cv, int64_t* ci, double* stats5,
             int threads) {
    if (q < 1 || n < 1 || d < 1 || rk < 0 || ck < 0 || kind < 0 || kind > 3) return 1;
    orc_scan_ctx c = {kind, exact, x, y, d, rowb, colb, nx, ny, scale};
    double* part = (double*)calloc((size_t)q * 5, sizeof(double));
    if (!part) return 2;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t i = 0; i < q; ++i) {
        double* v = rk ? rv + i * rk : NULL;
        int64_t* ix = rk ? ri + i * rk : NULL;
        for (int s = 0; s < rk; ++s) { v[s] = -INFINITY; ix[s] = ORC_NO_INDEX; }
        double num = 0, den = 0, mp = 0, mc = 0, cnt = 0;
        for (int64_t j = 0; j < n; ++j) {
            double sc, co;
            orc_pair(&c, i, j, &sc, &co);
            den += co * co;
            mc = fmax(mc, fabs(co));
            if (sc > 0) { num += sc * sc; mp = fmax(mp, sc); cnt += 1; }
            if (rk) orc_insert(v, ix, rk, sc, j);
        }
        for (int s = 0; s < rk; ++s) if (ix[s] == ORC_NO_INDEX) ix[s] = -1;
        part[i * 5 + 0] = num; part[i * 5 + 1] = den; part[i * 5 + 2] = mp;
        part[i * 5 + 3] = mc; part[i * 5 + 4] = cnt;
    }
    if (ck) {
#pragma omp parallel for schedule(dynamic, 16)
        for (int64_t j = 0; j < n; ++j) {
            double* v = cv + j * ck;
            int64_t* ix = ci + j * ck;
            for (int s = 0; s < ck; ++s) { v[s] = -INFINITY; ix[s] = ORC_NO_INDEX; }
            for (int64_t i = 0; i < q; ++i) {
                double sc, co;
                orc_pair(&c, i, j, &sc, &co);
                orc_insert(v, ix, ck, sc, i);
            }
            for (int s = 0; s < ck; ++s) if (ix[s] == ORC_NO_INDEX) ix[s] = -1;
        }
    }
    double acc[5] = {0, 0, 0, 0, 0};
    for (int64_t i = 0; i < q; ++i) {
        acc[0] += part[i * 5 + 0]; acc[1] += part[i * 5 + 1];
        acc[2] = fmax(acc[2], part[i * 5 + 2]); acc[3] = fmax(acc[3], part[i * 5 + 3]);
        acc[4] += part[i * 5 + 4];
    }
    memcpy(stats5, acc, sizeof(acc));
    free(part);
    return 0;
}

/* Exact score of selected pairs (used by parity tests to check a GPU
 * candidate list entry by entry). */
int orc_pair_scores(int kind, const float* x, const float* y, int64_t d, const double* rowb,
                    const double* colb, const double* nx, const double* ny, double scale,
                    const int64_t* rows, const int64_t* cols, int64_t count, double* score,
                    double* cost, int threads) {
    orc_scan_ctx c = {kind, 1, x, y, d, rowb, colb, nx, ny, scale};
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < count; ++e) {
        double s, co;
        orc_pair(&c, rows[e], cols[e], &s, &co);
        score[e] = s;
        if (cost) cost[e] = co;
    }
    return 0;
}

/* Active-support pair costs (the SDDMM).
 * kind 3: c_e = (a_r + b_c) - s<x_r, y_c>, h/costs/pairs.py:394-406, evaluated
 *         here in fp64 from the fp32 features.
 * kinds 0-2: fp64 accumulation of (double)y - (double)x per dimension,
 *         h/_native/norm_cost_scan/norm_cost_scan_kernel.cu:136-198,234-245. */
int orc_pair_costs(int kind, const float* x, const float* y, int64_t d, const double* a,
                   const double* b, double scale, const int64_t* rows, const int64_t* cols,
                   int64_t count, double* out, int threads) {
    if (kind < 0 || kind > 3 || d < 1) return 1;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < count; ++e) {
        const float* xr = x + rows[e] * d;
        const float* yc = y + cols[e] * d;
        double acc = 0.0;
        if (kind == 3) {
            for (int64_t k = 0; k < d; ++k) acc += (double)xr[k] * (double)yc[k];
            out[e] = (a[rows[e]] + b[cols[e]]) - scale * acc;
        } else {
            for (int64_t k = 0; k < d; ++k) {
                double z = (double)yc[k] - (double)xr[k];
                if (kind == 0) acc += fabs(z);
                else if (kind == 1) acc = fmax(acc, fabs(z));
                else acc += z * z;
            }
            out[e] = kind == 2 ? sqrt(acc) : acc;
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------------
 * Restricted-OT Halpern-PDHG, restating h/_native/cpp/solver.cpp:39-381 with a
 * team of one thread (same operation order, so with the reference's
 * num_threads=1 the two agree bit for bit).  Termination codes:
 * 1 OPTIMAL, 2 ITERATION_LIMIT, 3 NUMERICAL_DIVERGENCE.
 * ------------------------------------------------------------------------- */
typedef struct {
    int64_t iterations;
    int64_t restarts;
    int32_t reason;
    int32_t pad;
    double pobj, dobj, ap, rp, ad, rd, gap, weight, cost_norm, mass_norm;
} orc_pdlp_info;

static double orc_max0(double v) { return v < 0.0 ? 0.0 : v; } /* std::max(v, 0.0) */
static double orc_norm(const double* v, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += v[i] * v[i];
    return sqrt(s);
}

int orc_pdlp(const int64_t* rows, const int64_t* cols, const double* c, int64_t e, const double* b,
             int64_t n, int64_t nodes, const double* x0, const double* y0, int frequency,
             int64_t iteration_limit, double tol_objective, double tol_primal, double tol_dual,
             int rescale, double* x_out, double* y_out, orc_pdlp_info* info) {
    const int64_t m = nodes - n;
    if (n < 1 || m < 1 || e < 1 || frequency < 1 || iteration_limit < 1) return 1;
    for (int64_t j = 0; j < e; ++j)
        if (rows[j] < 0 || rows[j] >= n || cols[j] < 0 || cols[j] >= m) return 2;
    int64_t* offsets = (int64_t*)calloc(nodes + 1, sizeof(int64_t));
    int64_t* cursor = (int64_t*)malloc((nodes + 1) * sizeof(int64_t));
    int64_t* edge_ids = (int64_t*)malloc(2 * e * sizeof(int64_t));
    double* work = (double*)malloc(sizeof(double) * (8 * e + 9 * nodes + m));
    if (!offsets || !cursor || !edge_ids || !work) return 3;
    double *cs = work, *ax = cs + e, *x = ax + e, *px = x + e, *rx = px + e, *dx = rx + e;
    double *scale = dx + e, *bs = scale + nodes, *ns = bs + nodes, *ay = ns + nodes, *y = ay + nodes;
    double *py = y + nodes, *dy = py + nodes, *td = dy + nodes;
    /* incidence lists, solver.cpp:76-90 */
    for (int64_t j = 0; j < e; ++j) { ++offsets[rows[j] + 1]; ++offsets[n + cols[j] + 1]; }
    for (int64_t i = 0; i < nodes; ++i) {
        int64_t deg = offsets[i + 1] > 1 ? offsets[i + 1] : 1;
        scale[i] = sqrt((double)deg);
    }
    for (int64_t i = 0; i < nodes; ++i) offsets[i + 1] += offsets[i];
    memcpy(cursor, offsets, (nodes + 1) * sizeof(int64_t));
    for (int64_t j = 0; j < e; ++j) { edge_ids[cursor[rows[j]]++] = j; edge_ids[cursor[n + cols[j]]++] = j; }
    /* scaling, solver.cpp:91-110 */
    const double mass_norm = orc_norm(b, nodes), cost_norm = orc_norm(c, e);
    const double bound = rescale ? 1.0 / (mass_norm > 1.0 ? mass_norm : 1.0) : 1.0;
    const double objective = rescale ? 1.0 / (cost_norm > 1.0 ? cost_norm : 1.0) : 1.0;
    const double variable = sqrt(2.0);
    for (int64_t j = 0; j < e; ++j) {
        cs[j] = c[j] * objective / variable;
        ax[j] = orc_max0(x0[j]) * variable * bound;
    }
    for (int64_t i = 0; i < nodes; ++i) {
        bs[i] = b[i] * bound / scale[i];
        ns[i] = variable * scale[i];
        ay[i] = y0[i] * scale[i] * objective;
    }
    memcpy(x, ax, e * sizeof(double)); memcpy(px, ax, e * sizeof(double));
    memcpy(y, ay, nodes * sizeof(double)); memcpy(py, ay, nodes * sizeof(double));
    for (int64_t j = 0; j < m; ++j) td[j] = y[n + j] / ns[n + j];
    double weight;
    if (rescale) weight = 1.0;
    else {
        double bsn = orc_norm(bs, nodes);
        weight = orc_norm(cs, e) / (bsn > 1e-16 ? bsn : 1e-16);
        if (weight < 1e-16) weight = 1e-16;
    }
    double best_weight = weight, error_sum = 0.0;
    double best_balance = INFINITY, initial_error = INFINITY, last_trial = INFINITY, fixed = INFINITY;
    int64_t count = 0, inner = 0, restarts = 0;
    int reason = 0, restart = 0;
    double pobj = 0, dobj = 0, ap = 0, rp = 0, ad = 0, rd = 0, gap = 0;
    for (;;) {
        if (count % frequency == 0) {
            /* residuals of the unscaled problem, solver.cpp:115-136,174-186 */
            double primal_sq = 0, dual_sq = 0;
            pobj = dobj = 0;
            for (int64_t i = 0; i < nodes; ++i) {
                double sum = 0;
                for (int64_t k = offsets[i]; k < offsets[i + 1]; ++k) sum += px[edge_ids[k]] / (variable * bound);
                double delta = sum - b[i];
                primal_sq += delta * delta;
                dobj += b[i] * (py[i] / (scale[i] * objective));
            }
            for (int64_t j = 0; j < e; ++j) {
                double score = py[rows[j]] / (scale[rows[j]] * objective)
                             + py[n + cols[j]] / (scale[n + cols[j]] * objective) - c[j];
                double v = orc_max0(score);
                dual_sq += v * v;
                pobj += c[j] * (px[j] / (variable * bound));
            }
            ap = sqrt(primal_sq);
            ad = sqrt(dual_sq);
            rp = ap / (1.0 + mass_norm);
            rd = ad / (1.0 + cost_norm);
            gap = fabs(pobj - dobj) / (1.0 + fabs(pobj) + fabs(dobj));
            if (!(isfinite(pobj) && isfinite(dobj) && isfinite(ap) && isfinite(rp) && isfinite(ad)
                  && isfinite(rd) && isfinite(gap)) || !isfinite(weight)) reason = 3;
            else if (rp < tol_primal && rd < tol_dual && gap < tol_objective) reason = 1;
            else if (count >= iteration_limit) reason = 2;
            if (reason) break;
            /* adaptive restart rule, solver.cpp:189-198 */
            restart = 0;
            if (count == frequency) restart = 1;
            else if (count > frequency)
                restart = inner >= 0.36 * count || fixed <= 0.2 * initial_error
                       || (fixed <= 0.5 * initial_error && fixed > last_trial);
            last_trial = fixed;
            if (restart) {
                /* primal-weight PID update, solver.cpp:201-246 */
                double pd = 0, dd = 0;
                for (int64_t j = 0; j < e; ++j) { double t = px[j] - ax[j]; pd += t * t; }
                for (int64_t i = 0; i < nodes; ++i) { double t = py[i] - ay[i]; dd += t * t; }
                pd = sqrt(pd);
                dd = sqrt(dd);
                double ratio = rd / (rp > 1e-300 ? rp : 1e-300);
                if (pd > 1e-16 && pd < 1e12 && dd > 1e-16 && dd < 1e12 && ratio > 1e-8 && ratio < 1e8) {
                    double err = log(dd) - log(pd) - log(weight);
                    error_sum = 0.3 * error_sum + err;
                    weight *= exp(0.99 * err + 0.01 * error_sum);
                } else {
                    weight = best_weight;
                    error_sum = 0;
                }
                if (rp > 0 && rd > 0) {
                    double balance = fabs(log10(rd / rp));
                    if (balance < best_balance) { best_balance = balance; best_weight = weight; }
                }
                inner = 0;
                last_trial = INFINITY;
                ++restarts;
                for (int64_t j = 0; j < e; ++j) ax[j] = x[j] = px[j];
                for (int64_t i = 0; i < nodes; ++i) {
                    ay[i] = y[i] = py[i];
                    if (i >= n) td[i - n] = y[i] / ns[i];
                }
            }
        }
        /* one fused PDHG iteration, solver.cpp:249-311 */
        const double primal_step = 0.998 / weight;
        const double dual_step = 0.998 * weight;
        const double halpern = (double)(inner + 1) / (double)(inner + 2);
        const int major = ((count + 1) % frequency) == 0;
        const int is_restart = (count % frequency == 0) && restart;
        const int checkpoint = major || is_restart;
        for (int64_t i = 0; i < n; ++i) {
            const double sdual = y[i] / ns[i];
            double sum = 0.0;
            for (int64_t k = offsets[i]; k < offsets[i + 1]; ++k) {
                int64_t j = edge_ids[k];
                double at = sdual + td[cols[j]];
                px[j] = orc_max0(x[j] - primal_step * (cs[j] - at));
                rx[j] = 2.0 * px[j] - x[j];
                if (checkpoint) dx[j] = rx[j] - x[j];
                x[j] = halpern * rx[j] + (1.0 - halpern) * ax[j];
                sum += rx[j];
            }
            py[i] = y[i] - dual_step * (sum / ns[i] - bs[i]);
            const double refl = 2.0 * py[i] - y[i];
            if (checkpoint) dy[i] = refl - y[i];
            y[i] = halpern * refl + (1.0 - halpern) * ay[i];
        }
        for (int64_t i = n; i < nodes; ++i) {
            double sum = 0.0;
            for (int64_t k = offsets[i]; k < offsets[i + 1]; ++k) sum += rx[edge_ids[k]];
            py[i] = y[i] - dual_step * (sum / ns[i] - bs[i]);
            const double refl = 2.0 * py[i] - y[i];
            if (checkpoint) dy[i] = refl - y[i];
            y[i] = halpern * refl + (1.0 - halpern) * ay[i];
            td[i - n] = y[i] / ns[i];
        }
        if (checkpoint) {
            double movement = 0, dual_movement = 0, interaction = 0;
            for (int64_t j = 0; j < e; ++j) {
                movement += dx[j] * dx[j];
                interaction += (dy[rows[j]] / ns[rows[j]] + dy[n + cols[j]] / ns[n + cols[j]]) * dx[j];
            }
            for (int64_t i = 0; i < nodes; ++i) dual_movement += dy[i] * dy[i];
            double squared = movement * weight + dual_movement / weight + 2.0 * 0.998 * interaction;
            fixed = sqrt(squared > 0.0 ? squared : 0.0);
            if (is_restart) initial_error = fixed;
        }
        ++count;
        ++inner;
    }
    for (int64_t j = 0; j < e; ++j) x_out[j] = px[j] / (variable * bound);
    for (int64_t i = 0; i < nodes; ++i) y_out[i] = py[i] / (scale[i] * objective);
    info->iterations = count;
    info->restarts = restarts;
    info->reason = reason;
    info->pobj = pobj; info->dobj = dobj; info->ap = ap; info->rp = rp; info->ad = ad;
    info->rd = rd; info->gap = gap; info->weight = weight;
    info->cost_norm = cost_norm; info->mass_norm = mass_norm;
    free(offsets); free(cursor); free(edge_ids); free(work);
    return 0;
}
