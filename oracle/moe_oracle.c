/*
 * moe_oracle.c -- CPU restatement of momij's 2-bit MoE expert path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker + timed CPU baseline); see
 * moe_oracle.h for the semantics and the reference file:line each function
 * follows.  Parity against MLX gather_qmm itself is unpinned (MLX absent).
 *
 * All accumulation is float64; results are rounded (round-to-nearest-even)
 * to the activation dtype exactly where the reference's MLX path holds an
 * activation-dtype array: gather_qmm outputs, the SwiGLU output and the
 * combined output.
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- 16-bit float formats ------------------------------------------------ */

static void fmt_params(int dtype, int* mant, int* expb) {
    if (dtype == ORACLE_F16) { *mant = 10; *expb = 5; }
    else { *mant = 7; *expb = 8; }
}

double oracle_half_to_double(uint16_t h, int dtype) {
    int mant, expb;
    fmt_params(dtype, &mant, &expb);
    int bias = (1 << (expb - 1)) - 1;
    int sign = (h >> 15) & 1;
    int e = (h >> mant) & ((1 << expb) - 1);
    int m = h & ((1 << mant) - 1);
    double v;
    if (e == 0) v = ldexp((double)m, 1 - bias - mant);
    else if (e == (1 << expb) - 1) v = m ? NAN : INFINITY;
    else v = ldexp((double)(m | (1 << mant)), e - bias - mant);
    return sign ? -v : v;
}

/* Round a double straight to the 16-bit format (no double rounding through
 * float), ties to even, with subnormals and overflow to infinity. */
uint16_t oracle_double_to_half(double d, int dtype) {
    int mant, expb;
    fmt_params(dtype, &mant, &expb);
    int bias = (1 << (expb - 1)) - 1;
    int emin = 1 - bias, emax = bias;
    uint16_t sign = signbit(d) ? 0x8000 : 0;
    uint16_t inf = (uint16_t)(((1 << expb) - 1) << mant);
    if (isnan(d)) return (uint16_t)(sign | inf | (1 << (mant - 1)));
    double a = fabs(d);
    if (isinf(a)) return sign | inf;
    if (a == 0.0) return sign;
    int e;
    frexp(a, &e);
    e -= 1; /* a in [2^e, 2^(e+1)) */
    if (e < emin) e = emin;
    double quantum = ldexp(1.0, e - mant);
    double r = nearbyint(a / quantum); /* default rounding mode: ties to even */
    double v = r * quantum;
    if (v >= ldexp(1.0, emax + 1)) return sign | inf;
    if (v < ldexp(1.0, emin)) return (uint16_t)(sign | (uint16_t)r); /* subnormal */
    int ve;
    frexp(v, &ve);
    ve -= 1;
    int mbits = (int)(ldexp(v, mant - ve)) - (1 << mant);
    return (uint16_t)(sign | ((ve + bias) << mant) | mbits);
}

static inline double h2d(uint16_t h, int dt) { return oracle_half_to_double(h, dt); }
static inline uint16_t d2h(double d, int dt) { return oracle_double_to_half(d, dt); }

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---- router (SeedlessMetal.swift:2720-2791, MapleMoE.swift:49-55) --------
 * Selection restates maple_route_top8's reduction tree (:2764-2775): per
 * round, positions 0..W-1 (W = 256, the kernel's threadgroup; the next power
 * of two for E > 256) hold the candidates, and at stage s = W/2 .. 1 position
 * t < s takes the candidate of t + s only if its value is strictly greater
 * (float comparison: signed zeros are equal, NaN never replaces and is never
 * replaced).  Positions >= E and experts already selected take no further
 * part (the kernel marks them -inf, which only matters when fewer than K
 * finite logits remain).  Scores: softmax gates exp(l - max) / Z over all
 * experts, then the selected gates divided by their sum in k order
 * (:2755-2790). */

static int route_tree_width(int E) {
    int W = 256;
    while (W < E) W <<= 1;
    return W;
}

int oracle_route(const float* logits, int M, int E, int K, int32_t* inds, float* scores) {
    if (M < 0 || E <= 0 || K <= 0 || K > E) return -1;
    const int W = route_tree_width(E);
    float* red = (float*)malloc(sizeof(float) * W);
    int* ri = (int*)malloc(sizeof(int) * W);
    unsigned char* live = (unsigned char*)malloc((size_t)W);
    unsigned char* used = (unsigned char*)malloc((size_t)W);
    double* sel = (double*)malloc(sizeof(double) * K);
    for (int m = 0; m < M; ++m) {
        const float* lg = logits + (size_t)m * E;
        double mx = -INFINITY;
        for (int e = 0; e < E; ++e) if (lg[e] > mx) mx = lg[e];
        double Z = 0.0;
        for (int e = 0; e < E; ++e) Z += exp((double)lg[e] - mx);
        memset(used, 0, (size_t)W);
        double ss = 0.0;
        for (int k = 0; k < K; ++k) {
            for (int t = 0; t < W; ++t) {
                red[t] = t < E ? lg[t] : -INFINITY;
                ri[t] = t;
                live[t] = t < E && !used[t];
            }
            for (int st = W / 2; st > 0; st >>= 1)
                for (int t = 0; t < st; ++t)
                    if (live[t + st] && (!live[t] || red[t + st] > red[t])) {
                        red[t] = red[t + st];
                        ri[t] = ri[t + st];
                        live[t] = 1;
                    }
            const int bi = ri[0];
            used[bi] = 1;
            inds[(size_t)m * K + k] = bi;
            sel[k] = exp((double)lg[bi] - mx) / Z;
            ss += sel[k];
        }
        for (int k = 0; k < K; ++k) scores[(size_t)m * K + k] = (float)(sel[k] / ss);
    }
    free(red);
    free(ri);
    free(live);
    free(used);
    free(sel);
    return 0;
}

int oracle_permute(const int32_t* inds, const float* scores, int M, int K, int E,
                   int32_t* offsets, int32_t* pair, float* weight) {
    if (M < 0 || K <= 0 || E <= 0) return -1;
    size_t P = (size_t)M * K;
    for (int e = 0; e <= E; ++e) offsets[e] = 0;
    for (size_t i = 0; i < P; ++i) {
        if (inds[i] < 0 || inds[i] >= E) return -2;
        offsets[inds[i] + 1]++;
    }
    for (int e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
    int32_t* fill = (int32_t*)malloc(sizeof(int32_t) * (size_t)E);
    for (int e = 0; e < E; ++e) fill[e] = offsets[e];
    for (size_t i = 0; i < P; ++i) {
        int32_t pos = fill[inds[i]]++;
        pair[pos] = (int32_t)i;
        weight[pos] = scores[i];
    }
    free(fill);
    return 0;
}

/* ---- gather-qmv (SeedlessMetal.swift:2145-2221) -------------------------- */

int oracle_gqmm2(const uint16_t* x, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                 const int32_t* inds, uint16_t* out, int M, int Ktop, int Kdim, int N, int E,
                 int gs, int lhs_per_expert, int dtype) {
    if (M < 0 || Ktop <= 0 || N <= 0 || Kdim <= 0 || gs <= 0 || gs % 16 != 0 || Kdim % gs != 0)
        return -1;
    const int MK = M * Ktop;
    for (int mk = 0; mk < MK; ++mk)
        if (inds[mk] < 0 || inds[mk] >= E) return -2;
    const int words = Kdim / 16, groups = Kdim / gs;
    const int xrows = lhs_per_expert ? MK : M;
    double* xd = (double*)malloc(sizeof(double) * (size_t)xrows * Kdim);
    double* xs = (double*)malloc(sizeof(double) * (size_t)xrows * groups);
    for (int r = 0; r < xrows; ++r) {
        for (int k = 0; k < Kdim; ++k) xd[(size_t)r * Kdim + k] = h2d(x[(size_t)r * Kdim + k], dtype);
        for (int g = 0; g < groups; ++g) {
            double t = 0.0;
            for (int k = g * gs; k < (g + 1) * gs; ++k) t += xd[(size_t)r * Kdim + k];
            xs[(size_t)r * groups + g] = t;
        }
    }
    long long total = (long long)MK * N;
#pragma omp parallel for schedule(static)
    for (long long idx = 0; idx < total; ++idx) {
        int mk = (int)(idx / N), n = (int)(idx % N);
        int e = inds[mk];
        int xr = lhs_per_expert ? mk : mk / Ktop;
        const double* xv = xd + (size_t)xr * Kdim;
        const double* sx = xs + (size_t)xr * groups;
        const uint32_t* wr = w + ((size_t)e * N + n) * words;
        const uint16_t* sr = s + ((size_t)e * N + n) * groups;
        const uint16_t* br = b + ((size_t)e * N + n) * groups;
        double acc = 0.0;
        for (int g = 0; g < groups; ++g) {
            double sq = 0.0;
            for (int k = g * gs; k < (g + 1) * gs; ++k) {
                uint32_t q = (wr[k >> 4] >> (2 * (k & 15))) & 3u;
                sq += (double)q * xv[k];
            }
            acc += h2d(sr[g], dtype) * sq + h2d(br[g], dtype) * sx[g];
        }
        out[(size_t)mk * N + n] = d2h(acc, dtype);
    }
    free(xd);
    free(xs);
    return 0;
}

/* ---- SwiGLU / combine ---------------------------------------------------- */

void oracle_clamped_swiglu(const uint16_t* ug, uint16_t* act, int rows, int I, float clamp,
                           int dtype) {
    for (int r = 0; r < rows; ++r) {
        for (int j = 0; j < I; ++j) {
            double up = h2d(ug[(size_t)r * 2 * I + j], dtype);
            double gate = h2d(ug[(size_t)r * 2 * I + I + j], dtype);
            if (gate > clamp) gate = clamp;
            if (up > clamp) up = clamp;
            if (up < -clamp) up = -clamp;
            double silu = gate / (1.0 + exp(-gate));
            act[(size_t)r * I + j] = d2h(silu * up, dtype);
        }
    }
}

static double combine_one(const uint16_t* down, const float* scores, int m, int Ktop, int H,
                          int h, int dtype) {
    double acc = 0.0;
    for (int k = 0; k < Ktop; ++k) {
        size_t mk = (size_t)m * Ktop + k;
        acc += h2d(down[mk * H + h], dtype) * (double)scores[mk];
    }
    return acc;
}

void oracle_score_reduce(const uint16_t* down, const float* scores, uint16_t* y, int M, int Ktop,
                         int H, int dtype) {
    for (int m = 0; m < M; ++m)
        for (int h = 0; h < H; ++h)
            y[(size_t)m * H + h] = d2h(combine_one(down, scores, m, Ktop, H, h, dtype), dtype);
}

void oracle_score_resid(const uint16_t* down, const float* scores, uint16_t* hbuf, int M,
                        int Ktop, int H, int dtype) {
    for (int m = 0; m < M; ++m)
        for (int h = 0; h < H; ++h) {
            double acc = combine_one(down, scores, m, Ktop, H, h, dtype);
            double delta = h2d(d2h(acc, dtype), dtype);
            size_t off = (size_t)m * H + h;
            hbuf[off] = d2h(h2d(hbuf[off], dtype) + delta, dtype);
        }
}

int oracle_expert_ffn(const uint16_t* x, const uint32_t* w_ug, const uint16_t* s_ug,
                      const uint16_t* b_ug, const uint32_t* w_dn, const uint16_t* s_dn,
                      const uint16_t* b_dn, const int32_t* inds, const float* scores, uint16_t* y,
                      uint16_t* resid_h, int M, int H, int I, int E, int Ktop, int gs, float clamp,
                      int dtype, uint16_t* ug, uint16_t* act, uint16_t* down) {
    int rc = oracle_gqmm2(x, w_ug, s_ug, b_ug, inds, ug, M, Ktop, H, 2 * I, E, gs, 0, dtype);
    if (rc) return rc;
    oracle_clamped_swiglu(ug, act, M * Ktop, I, clamp, dtype);
    rc = oracle_gqmm2(act, w_dn, s_dn, b_dn, inds, down, M, Ktop, I, H, E, gs, 1, dtype);
    if (rc) return rc;
    if (resid_h) oracle_score_resid(down, scores, resid_h, M, Ktop, H, dtype);
    else oracle_score_reduce(down, scores, y, M, Ktop, H, dtype);
    return 0;
}
