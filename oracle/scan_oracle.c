/*
 * CPU oracle for the diagonal selective scan -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is a plain-C restatement of the reference's scan algorithm. It is
 * compiled into oracle/_build/libscan_oracle.so and loaded only by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg, always as the
 * checker and never as the product. The product path (the CUDA library under
 * mamba-metal-scan_b200/csrc) never links or calls it.
 *
 * Algorithm followed (reference = Anamaya1729/mamba-metal-scan):
 *   forward   mamba_metal/scan.py:13-15 (recurrence), :105-126 (ssm_fwd loop,
 *             checkpoint every K steps and at T), :320-333 (selective_scan_ref)
 *   backward  mamba_metal/scan.py:26-34 (adjoint formulas), :173-248 (ssm_bwd:
 *             chunks last to first, g_t = dy_t*C_t + dA_{t+1}*g_{t+1}, dx, ddt,
 *             dAneg, dB = sum_d, dC = sum_d)
 *
 * Differences from the reference kernel that do not change the mathematics:
 *   - h is kept for the whole sequence of one (b, d) instead of being
 *     recomputed per chunk from checkpoints (the oracle trades memory for
 *     clarity);
 *   - dA_t * h_{t-1} is formed directly instead of as h_t - b_t;
 *   - dB, dC and dAneg are summed in a fixed order (no atomics), so the oracle
 *     is deterministic.
 *
 * Parity is pinned by tests/test_oracle.py against golden vectors produced by
 * running the reference's own selective_scan_ref (forward + autograd backward)
 * in float32 and float64 (tests/golden/make_golden.py).
 *
 * Two precisions are built from the same source: REAL=double (the float64
 * arbiter) and REAL=float (an fp32 restatement of the reference's arithmetic
 * order: dA = exp(-dt*Aneg), b = (dt*B)*x, h = dA*h + b, y = sum_n C*h).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_OK 0
#define ORACLE_EINVAL 1
#define ORACLE_ENOMEM 2

#define DEFINE_ORACLE(REAL, SUF, EXP)                                           \
/* y (B,T,D); ckpt (B, ceil(T/K), D, N) or NULL; scan.py:105-126 */             \
int oracle_fwd_##SUF(const REAL *x, const REAL *dt, const REAL *aneg,           \
                     const REAL *Bm, const REAL *Cm, REAL *y, REAL *ckpt,       \
                     int Bt, int T, int D, int N, int K)                        \
{                                                                               \
    if (Bt < 0 || T < 0 || D < 0 || N <= 0 || K <= 0) return ORACLE_EINVAL;     \
    const int nchunk = (T + K - 1) / K;                                         \
    int err = 0;                                                                \
    _Pragma("omp parallel for schedule(static) reduction(|:err)")               \
    for (long bd = 0; bd < (long)Bt * D; ++bd) {                                \
        const int b = (int)(bd / D), d = (int)(bd % D);                         \
        REAL *h = (REAL *)calloc((size_t)N, sizeof(REAL));                      \
        if (!h) { err |= 1; continue; }                                         \
        for (int t = 0; t < T; ++t) {                                           \
            const size_t xt = ((size_t)b * T + t) * D + d;                      \
            const size_t st = ((size_t)b * T + t) * N;                          \
            const REAL dtv = dt[xt];                                            \
            REAL yv = 0;                                                        \
            for (int n = 0; n < N; ++n) {                                       \
                const REAL da = EXP(-dtv * aneg[(size_t)d * N + n]);            \
                const REAL bv = dtv * Bm[st + n] * x[xt];                       \
                h[n] = da * h[n] + bv;                                          \
                yv += Cm[st + n] * h[n];                                        \
            }                                                                   \
            y[xt] = yv;                                                         \
            const int tn = t + 1;                                               \
            if (ckpt && (tn % K == 0 || tn == T)) {                             \
                const int c = (tn % K == 0) ? tn / K - 1 : nchunk - 1;          \
                REAL *o = ckpt + (((size_t)b * nchunk + c) * D + d) * N;        \
                memcpy(o, h, (size_t)N * sizeof(REAL));                         \
            }                                                                   \
        }                                                                       \
        free(h);                                                                \
    }                                                                           \
    return err ? ORACLE_ENOMEM : ORACLE_OK;                                     \
}                                                                               \
                                                                                \
/* dx, ddt (B,T,D); dAneg (D,N); dB, dC (B,T,N); scan.py:26-34, 173-260.        \
 * Every output is fully written (no accumulation into caller memory). */      \
int oracle_bwd_##SUF(const REAL *x, const REAL *dt, const REAL *aneg,           \
                     const REAL *Bm, const REAL *Cm, const REAL *dy,            \
                     REAL *dx, REAL *ddt, REAL *dAneg, REAL *dB, REAL *dC,      \
                     int Bt, int T, int D, int N)                               \
{                                                                               \
    if (Bt < 0 || T < 0 || D < 0 || N <= 0) return ORACLE_EINVAL;               \
    const size_t DN = (size_t)D * N;                                            \
    REAL *dA_b = (REAL *)calloc((size_t)(Bt > 0 ? Bt : 1) * DN, sizeof(REAL));  \
    if (!dA_b) return ORACLE_ENOMEM;                                            \
    int err = 0;                                                                \
    /* one batch row per task: dB/dC are summed over d in ascending order */    \
    _Pragma("omp parallel for schedule(dynamic) reduction(|:err)")              \
    for (int b = 0; b < Bt; ++b) {                                              \
        REAL *hs = (REAL *)malloc(((size_t)T + 1) * N * sizeof(REAL));          \
        REAL *g = (REAL *)malloc((size_t)N * sizeof(REAL));                     \
        if (!hs || !g) { free(hs); free(g); err |= 1; continue; }               \
        REAL *dBb = dB + (size_t)b * T * N, *dCb = dC + (size_t)b * T * N;      \
        memset(dBb, 0, (size_t)T * N * sizeof(REAL));                           \
        memset(dCb, 0, (size_t)T * N * sizeof(REAL));                           \
        for (int d = 0; d < D; ++d) {                                           \
            const REAL *an = aneg + (size_t)d * N;                              \
            /* hs[t+1] = h_t, hs[0] = h_{-1} = 0 */                             \
            memset(hs, 0, (size_t)N * sizeof(REAL));                            \
            for (int t = 0; t < T; ++t) {                                       \
                const size_t xt = ((size_t)b * T + t) * D + d;                  \
                const size_t st = ((size_t)b * T + t) * N;                      \
                const REAL dtv = dt[xt];                                        \
                for (int n = 0; n < N; ++n)                                     \
                    hs[(size_t)(t + 1) * N + n] =                               \
                        EXP(-dtv * an[n]) * hs[(size_t)t * N + n]               \
                        + dtv * Bm[st + n] * x[xt];                             \
            }                                                                   \
            for (int n = 0; n < N; ++n) g[n] = 0;                               \
            REAL *dAd = dA_b + (size_t)b * DN + (size_t)d * N;                  \
            for (int t = T - 1; t >= 0; --t) {                                  \
                const size_t xt = ((size_t)b * T + t) * D + d;                  \
                const size_t st = ((size_t)b * T + t) * N;                      \
                const REAL dtv = dt[xt], xv = x[xt], dyv = dy[xt];              \
                const REAL dtn = (t + 1 < T) ? dt[xt + D] : 0;                  \
                REAL dxv = 0, ddtv = 0;                                         \
                for (int n = 0; n < N; ++n) {                                   \
                    const REAL danext = (t + 1 < T) ? EXP(-dtn * an[n]) : 0;    \
                    g[n] = dyv * Cm[st + n] + danext * g[n];                    \
                    /* dA_t * h_{t-1}: the part of h_t that came from the past */\
                    const REAL hm = EXP(-dtv * an[n]) * hs[(size_t)t * N + n];  \
                    const REAL gB = g[n] * Bm[st + n];                          \
                    dxv += dtv * gB;                                            \
                    ddtv += xv * gB - an[n] * g[n] * hm;                        \
                    dAd[n] += -dtv * g[n] * hm;                                 \
                    dBb[(size_t)t * N + n] += g[n] * dtv * xv;                  \
                    dCb[(size_t)t * N + n] += dyv * hs[(size_t)(t + 1) * N + n];\
                }                                                               \
                dx[xt] = dxv;                                                   \
                ddt[xt] = ddtv;                                                 \
            }                                                                   \
        }                                                                       \
        free(hs);                                                               \
        free(g);                                                                \
    }                                                                           \
    /* dAneg = sum over b (ascending), scan.py:34 */                            \
    for (size_t i = 0; i < DN; ++i) {                                           \
        REAL s = 0;                                                             \
        for (int b = 0; b < Bt; ++b) s += dA_b[(size_t)b * DN + i];             \
        dAneg[i] = s;                                                           \
    }                                                                           \
    free(dA_b);                                                                 \
    return err ? ORACLE_ENOMEM : ORACLE_OK;                                     \
}

DEFINE_ORACLE(double, f64, exp)
DEFINE_ORACLE(float, f32, expf)

/* Number of OpenMP threads the oracle will use (1 when built without it). */
int oracle_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
