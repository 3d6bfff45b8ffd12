// Backward selective scan for sm_100a.
//
// Math (reference mamba_metal/scan.py:26-34, kernel ssm_bwd at :132-261):
//     g_t    = dy_t*C_t + dA_{t+1}*g_{t+1}
//     dx_t   = dt_t * sum_n g_tn*B_tn
//     ddt_t  = x_t * sum_n g_tn*B_tn - sum_n Aneg_n*g_tn*(dA_tn*h_{t-1,n})
//     dAneg  = -sum_{b,t} dt_t*g_tn*(dA_tn*h_{t-1,n})
//     dB_tn  = sum_d g_tdn*dt_td*x_td          dC_tn = sum_d dy_td*h_tdn
//
// Decomposition is the forward's: a thread owns 4 states of one (b, d)
// channel, G lanes share a channel, a CTA covers DPB = 256/G channels of one
// batch row and walks the whole sequence from the last chunk to the first.
//
// Recompute with two exps per element and no (B,K,D,N) scratch:
//   * a chunk (K steps between the forward's checkpoints) is cut into
//     segments of SEG = GRP*SLOTS steps; the state entering a segment is the
//     checkpoint or, in chunks longer than SEG, a segment-start state that a
//     pre-pass stored in the workspace;
//   * a segment is recomputed once, keeping only the state that enters each
//     GRP-step group (SLOTS float4 per thread in shared memory);
//   * the walk takes the groups last to first; each group is rebuilt from its
//     slot (GRP exps per state) and its decays and states stay in registers for
//     the group's backward steps: dA_t for dA_t*h_{t-1} and, carried one step,
//     dA_{t+1} for the adjoint.
//
// Memory: every pass reads GRP-step tiles (x, dt, dy, B, C of the CTA's
// channels) that cp.async stages in natural layout three groups ahead, along
// the exact order the passes consume them (WorkCursor). One group ahead of its
// use, a tile is rewritten in shared memory into the layouts the inner loops
// read with the fewest instructions: x, dt, dy as per-channel runs of 4 steps
// (one 16-byte load per 4 steps) and B, C in the lane-specific state orders
// described next.
//
// Arithmetic: the 4 states of a thread are two float2 pairs driven by the
// packed FFMA2/FMUL2 instructions of sm_100.
//
// Reductions, all deterministic (fixed order, no atomics):
//   * sum over n (dx, ddt): per-lane partials in shared memory, finished once
//     per group by one thread per (t, d), which also writes dx/ddt coalesced;
//   * sum over d (dB, dC): a transposed butterfly across a warp's channels.
//     Each lane holds its 4 states in the order state(r) = r XOR tau, where tau
//     is made of the lane's two highest channel bits; then at the first two
//     butterfly levels every lane keeps registers {0,1} and then {0}, so only
//     the last level (dB vs dC) needs selects. The CTA's warps are summed in
//     shared memory once per group into one partial per CTA, and
//     reduce_kernel adds the CTAs of a batch row;
//   * dAneg: per-thread register sums over the whole walk, one partial per
//     batch row; reduce_kernel adds the rows.
#include "mms_common.cuh"
#include "mms_kernels.h"
#include "mms_stage.cuh"

namespace mms {

#ifndef MMS_BWD_GRP
#define MMS_BWD_GRP 8
#endif
#ifndef MMS_BWD_MINB
#define MMS_BWD_MINB 2
#endif
#ifndef MMS_BWD_CP
#define MMS_BWD_CP 1
#endif
#ifndef MMS_BWD_W8
#define MMS_BWD_W8 1
#endif
#ifndef MMS_BWD_K8_MINB
#define MMS_BWD_K8_MINB 2
#endif

constexpr int BWD_THREADS = 256;
constexpr int BWD_WARPS = BWD_THREADS / 32;
constexpr int GRP = MMS_BWD_GRP;          // steps rebuilt per group
constexpr int SLOTS = 64 / GRP;           // groups per segment
constexpr int SEG = GRP * SLOTS;          // steps per segment (64)
constexpr int NAT_BUFS = 3;               // natural-layout tiles (cp.async targets)
constexpr int DER_BUFS = 2;               // rewritten tiles (in use, being prepared)
constexpr float MMS_LN2 = 0.6931471805599453f;

template <int G>
struct BwdShape {
    static constexpr int DPB = BWD_THREADS / G;            // channels per CTA
    static constexpr int NPAD = 4 * G;
    static constexpr int NROWF = 3 * DPB + 2 * NPAD;       // natural row: x, dt, dy, B, C
    static constexpr int NATF = GRP * NROWF;
    static constexpr int NPERM = G <= 8 ? 4 : 2;           // distinct tau values
    static constexpr int QF = GRP * DPB;                   // one array in 4-step runs
    static constexpr int PF = GRP * NPERM * NPAD;          // B or C in NPERM orders
    static constexpr int DERF = 3 * QF + 2 * PF;
    static constexpr int NV2 = 2 * NPAD;                   // dB|dC values per step per warp
    static constexpr size_t SLOTF = (size_t)SLOTS * BWD_THREADS * 4;
    static constexpr size_t SDF = (size_t)GRP * BWD_WARPS * NV2;   // one of two buffers
    static constexpr size_t CKF = (size_t)DPB * NPAD;            // entry-state slab of a group
    static constexpr size_t SMEM_K8 =
        sizeof(float) * ((size_t)NAT_BUFS * (NATF + CKF) + (size_t)DER_BUFS * DERF + 2 * SDF);
    static constexpr size_t SMEM = SMEM_K8 + sizeof(float) * SLOTF;
};

// The order in which one CTA consumes GRP-step groups of its batch row:
// chunks last to first; in each chunk an optional pre-pass (P) that stores
// segment-start states, then per segment (last to first) the recompute (R,
// groups forward, all but the last) and the walk (W, groups backward).
struct WorkCursor {
    int c, phase, sg, j;       // phase 0 = P, 1 = R, 2 = W; c < 0 when done
    int t0c, t1c, nseg, u0, u1, ngrp;
    int T, K, clo;             // chunks clo .. (start) are this CTA's

    __device__ void start(int T_, int K_, int chi, int clo_) {
        T = T_; K = K_; clo = clo_;
        enter_chunk(chi);
    }
    __device__ void enter_chunk(int c_) {
        c = c_ < clo ? -1 : c_;
        if (c < 0) return;
        t0c = c * K;
        t1c = min(t0c + K, T);
        nseg = (t1c - t0c + SEG - 1) / SEG;
        if (nseg > 1) { phase = 0; j = 0; } else { enter_segment(0); }
    }
    __device__ void enter_segment(int sg_) {
        sg = sg_;
        u0 = t0c + sg * SEG;
        u1 = min(u0 + SEG, t1c);
        ngrp = (u1 - u0 + GRP - 1) / GRP;
        if (ngrp > 1) { phase = 1; j = 0; } else { phase = 2; j = ngrp - 1; }
    }
    __device__ void advance() {
        if (phase == 0) {
            if (++j < (nseg - 1) * SLOTS) return;
            enter_segment(nseg - 1);
        } else if (phase == 1) {
            if (++j < ngrp - 1) return;
            phase = 2;
            j = ngrp - 1;
        } else {
            if (--j >= 0) return;
            if (sg > 0) enter_segment(sg - 1);
            else enter_chunk(c - 1);
        }
    }
    __device__ bool done() const { return c < 0; }
    __device__ int tstart() const { return phase == 0 ? t0c + j * GRP : u0 + j * GRP; }
    __device__ int nvalid() const { return phase == 0 ? GRP : min(GRP, u1 - (u0 + j * GRP)); }
};

__device__ __forceinline__ float2 shfl2(float2 v, int m) {
    return f2(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m));
}

// Rewrite a natural tile into the compute layouts (see the file comment); x,
// dt, dy are widened from their storage type E to fp32 here.
template <int G, typename E = float>
__device__ __forceinline__ void rewrite_tile(const float *nat, float *der, int tid, const Proj &pj)
{
    using S = BwdShape<G>;
    constexpr int DPB = S::DPB, NPAD = S::NPAD, QF = S::QF, PF = S::PF;
    constexpr int CHF = TileRow<3, DPB, E>::CHF;           // floats of x, dt, dy per step
    constexpr int NROWF = CHF + 2 * NPAD;                  // staged row (floats)
    constexpr int RSTR = NROWF * 4 / (int)sizeof(E);       // the same in elements of E
    constexpr int NQ = GRP / 4;
    for (int e = tid; e < 3 * NQ * DPB; e += BWD_THREADS) {
        const int a = e / (NQ * DPB), rem = e % (NQ * DPB);
        const int q = rem / DPB, cc = rem % DPB;
        const E *src = reinterpret_cast<const E *>(nat + (4 * q) * NROWF) + a * DPB + cc;
        float4 v4 = make_float4(to_f(src[0]), to_f(src[RSTR]), to_f(src[2 * RSTR]),
                                to_f(src[3 * RSTR]));
        if (pj.on && a == 1)
            v4 = make_float4(fmaf(pj.range, sigmoid_fast(v4.x), pj.lo), fmaf(pj.range, sigmoid_fast(v4.y), pj.lo),
                             fmaf(pj.range, sigmoid_fast(v4.z), pj.lo), fmaf(pj.range, sigmoid_fast(v4.w), pj.lo));
        *reinterpret_cast<float4 *>(der + a * QF + (q * DPB + cc) * 4) = v4;
    }
    constexpr int NQ4 = NPAD / 4;
    for (int e = tid; e < 2 * GRP * S::NPERM * NQ4; e += BWD_THREADS) {
        const int q4 = e % NQ4;
        const int pi = (e / NQ4) % S::NPERM;
        const int i = (e / (NQ4 * S::NPERM)) % GRP;
        const int a = e / (NQ4 * S::NPERM * GRP);
        const int tau = S::NPERM == 4 ? pi : 2 * pi;
        const float *src = nat + i * NROWF + CHF + a * NPAD + 4 * q4;
        *reinterpret_cast<float4 *>(der + 3 * QF + a * PF + (i * S::NPERM + pi) * NPAD + 4 * q4) =
            make_float4(src[0 ^ tau], src[1 ^ tau], src[2 ^ tau], src[3 ^ tau]);
    }
}

// Per-thread view of a rewritten tile.
template <int G>
struct TileView {
    using S = BwdShape<G>;
    const float *qx, *qdt, *qdy, *pB, *pC;
    __device__ TileView(const float *der, int c, int g, int pidx) {
        qx = der + c * 4;
        qdt = der + S::QF + c * 4;
        qdy = der + 2 * S::QF + c * 4;
        pB = der + 3 * S::QF + pidx * S::NPAD + 4 * g;
        pC = pB + S::PF;
    }
    // 4 consecutive steps [4q, 4q+4) of the thread's channel
    __device__ float4 x4(int q) const { return *reinterpret_cast<const float4 *>(qx + q * S::DPB * 4); }
    __device__ float4 dt4(int q) const { return *reinterpret_cast<const float4 *>(qdt + q * S::DPB * 4); }
    __device__ float4 dy4(int q) const { return *reinterpret_cast<const float4 *>(qdy + q * S::DPB * 4); }
    // the thread's 4 states of step i in its own state order
    __device__ float4 B(int i) const { return *reinterpret_cast<const float4 *>(pB + i * S::NPERM * S::NPAD); }
    __device__ float4 C(int i) const { return *reinterpret_cast<const float4 *>(pC + i * S::NPERM * S::NPAD); }
};

// h <- recurrence over the GRP steps of a tile (padding steps are zeros).
template <int G>
__device__ __forceinline__ void advance_tile(float2 (&h)[2], const float2 (&an2)[2],
                                             const TileView<G> &v)
{
#pragma unroll
    for (int q = 0; q < GRP / 4; ++q) {
        const float4 x4 = v.x4(q), d4 = v.dt4(q);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float dtv = comp(d4, k), bx = dtv * comp(x4, k);
            const float4 Bv = v.B(4 * q + k);
            const float2 md = f2(-dtv, -dtv), bx2 = f2(bx, bx);
            h[0] = fma2(ex2x2(mul2(md, an2[0])), h[0], mul2(bx2, lo(Bv)));
            h[1] = fma2(ex2x2(mul2(md, an2[1])), h[1], mul2(bx2, hi(Bv)));
        }
    }
}

// Per-thread constants shared by both backward kernels.
template <int G>
struct Lane {
    using S = BwdShape<G>;
    int tid, lane, warp, g, c, d0, d, b, tau, pidx, u3, sd_pos;
    bool act, sd_writer;
    bool n_ddt;          // after the sum over the channel's lanes this lane holds ddt (else dx)
    bool n_writer;       // ... and stores it
    float2 an2[2];                                  // Aneg * log2(e) in lane state order

    __device__ Lane(const float *aneg, int D, int N, const Proj &pj) {
        tid = threadIdx.x;
        lane = tid & 31;
        warp = tid >> 5;
        g = tid & (G - 1);
        c = tid / G;
        d0 = blockIdx.x * S::DPB;
        d = d0 + c;
        b = blockIdx.y;
        act = d < D && (4 * g < N);
        // Lane-specific state order: register r holds state 4g + (r ^ tau).
        const int u1 = (lane >> 4) & 1;
        const int u2 = G <= 8 ? (lane >> 3) & 1 : 0;
        tau = 2 * u1 + u2;
        pidx = S::NPERM == 4 ? tau : u1;
        u3 = G <= 4 ? (lane >> 2) & 1 : 0;          // dB (0) / dC (1) kept at the last level
        // Output position of this lane's dB/dC value after the butterfly
        // (G <= 4: kind u3, state tau; G >= 8 writes several values).
        sd_pos = (G <= 4 ? u3 * S::NPAD : 0) + 4 * g + tau;
        sd_writer = G >= 4 || (lane & (G == 2 ? 2 : 3)) == 0;
        n_ddt = G > 1 && (g & (G / 2)) != 0;
        n_writer = d < D && (G == 1 || (g & (G / 2 - 1)) == 0);
        an2[0] = f2(0.f, 0.f);
        an2[1] = f2(0.f, 0.f);
        if (act) {
            const float *ap = aneg + (size_t)d * N + 4 * g;
            float a[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                a[r] = __ldg(ap + (r ^ tau));
                if (pj.on) a[r] = softplus(a[r]);
            }
            an2[0] = f2(a[0] * MMS_LOG2E, a[1] * MMS_LOG2E);
            an2[1] = f2(a[2] * MMS_LOG2E, a[3] * MMS_LOG2E);
        }
    }
    // The 4 states of channel d, group g, in lane order, from a (D, N) plane.
    __device__ void load_state(float2 (&h)[2], const float *plane_base, int N) const {
        float hh[4] = {0.f, 0.f, 0.f, 0.f};
        if (act) {
            const float *p = plane_base + (size_t)d * N + 4 * g;
#pragma unroll
            for (int r = 0; r < 4; ++r) hh[r] = __ldg(p + (r ^ tau));
        }
        h[0] = f2(hh[0], hh[1]);
        h[1] = f2(hh[2], hh[3]);
    }
};

// Carried across the backward walk.
struct Adjoint {
    float2 gad[2];      // adjoint g of the most recent (later) step
    float2 anx[2];      // dA of the step after it; zero past the end of the sequence
    float2 dac[2];      // sum_t dt*g*dA*h_{t-1}
};

// Rebuild one group from the state entering it, then walk it backwards:
// dx/ddt are finished with shuffles across the channel's lanes and stored
// (dxo/ddto point at this lane's channel at step t0), per-warp dB/dC sums go to sd.
#ifndef MMS_WALK_KEEP_A
#define MMS_WALK_KEEP_A 0
#endif

template <int G, bool FULL, typename E = float>
__device__ __forceinline__ void walk_group(const TileView<G> &v, const float2 (&hb)[2],
                                           const Lane<G> &L, Adjoint &A, int nv,
                                           E *dxo, E *ddto, int D, float *sd,
                                           const Proj &pj)
{
    E *outp = L.n_ddt ? ddto : dxo;
    using S = BwdShape<G>;
    constexpr int NPAD = S::NPAD, NV2 = S::NV2;
    // Rebuild: the states of the group's steps (and, when kept, their decays).
    float2 hv[GRP][2];
#if MMS_WALK_KEEP_A
    float2 av[GRP][2];
#endif
#pragma unroll
    for (int q = 0; q < GRP / 4; ++q) {
        const float4 x4 = v.x4(q), d4 = v.dt4(q);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = 4 * q + k;
            const float dtv = comp(d4, k), bx = dtv * comp(x4, k);
            const float4 Bv = v.B(i);
            const float2 md = f2(-dtv, -dtv), bx2 = f2(bx, bx);
            const float2 a0 = ex2x2(mul2(md, L.an2[0]));
            const float2 a1 = ex2x2(mul2(md, L.an2[1]));
#if MMS_WALK_KEEP_A
            av[i][0] = a0;
            av[i][1] = a1;
#endif
            hv[i][0] = fma2(a0, i ? hv[i > 0 ? i - 1 : 0][0] : hb[0], mul2(bx2, lo(Bv)));
            hv[i][1] = fma2(a1, i ? hv[i > 0 ? i - 1 : 0][1] : hb[1], mul2(bx2, hi(Bv)));
        }
    }
    // Walk: acar carries dA of the step after the current one.
    float2 acar[2] = {A.anx[0], A.anx[1]};
#pragma unroll
    for (int q = GRP / 4 - 1; q >= 0; --q) {
        const float4 x4 = v.x4(q), d4 = v.dt4(q), y4 = v.dy4(q);
#pragma unroll
        for (int k = 3; k >= 0; --k) {
            const int i = 4 * q + k;
            if (!FULL && i >= nv) continue;           // uniform
            const float dtv = comp(d4, k), xv = comp(x4, k), dyv = comp(y4, k);
            const float4 Bv = v.B(i), Cv = v.C(i);
            const float2 dy2 = f2(dyv, dyv), dt2 = f2(dtv, dtv);
            const float dxv = dtv * xv;
            const float2 dxv2 = f2(dxv, dxv);
#if !MMS_WALK_KEEP_A
            const float2 md = f2(-dtv, -dtv);
#endif
            float2 p1 = f2(0.f, 0.f), p2 = f2(0.f, 0.f), vb[2], vc[2];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
#if MMS_WALK_KEEP_A
                const float2 ai = av[i][p];
#else
                const float2 am = mul2(md, L.an2[p]);
                const float2 ai = f2(ex2_fresh(am.x), ex2_fresh(am.y));
#endif
                const float2 cp = p ? hi(Cv) : lo(Cv);
                const float2 bp = p ? hi(Bv) : lo(Bv);
                A.gad[p] = fma2(acar[p], A.gad[p], mul2(dy2, cp));
                acar[p] = ai;
                const float2 hp = i ? hv[i > 0 ? i - 1 : 0][p] : hb[p];
                const float2 u = mul2(A.gad[p], mul2(ai, hp));
                p1 = fma2(A.gad[p], bp, p1);
                p2 = fma2(L.an2[p], u, p2);
                A.dac[p] = fma2(dt2, u, A.dac[p]);
                vb[p] = mul2(A.gad[p], dxv2);
                vc[p] = mul2(dy2, hv[i][p]);
            }
            {   // dx = dt*sum_n g*B, ddt = x*sum_n g*B - sum_n Aneg*u (an2 carries log2 e)
                const float s1 = p1.x + p1.y, s2 = p2.x + p2.y;
                float vn[2] = {dtv * s1, fmaf(xv, s1, -MMS_LN2 * s2)};
                if constexpr (G > 1) {
                    int fn;
                    transposed_reduce<2, G / 2, 1>(vn, L.lane, fn);
                    // prologue: d(logit) = ddt * d dt / d logit = ddt * (dt-lo)(lo+range-dt)/range
                    if (pj.on && L.n_ddt) vn[0] *= dt_slope(pj, dtv);
                    if (L.n_writer) outp[(size_t)i * D] = from_f<E>(vn[0]);
                } else if (L.n_writer) {
                    if (pj.on) vn[1] *= dt_slope(pj, dtv);
                    dxo[(size_t)i * D] = from_f<E>(vn[0]);
                    ddto[(size_t)i * D] = from_f<E>(vn[1]);
                }
            }
            // dB|dC butterfly across the warp's channels
            vb[0] = add2(vb[0], shfl2(vb[1], 16));
            vc[0] = add2(vc[0], shfl2(vc[1], 16));
            float *r = sd + (i * BWD_WARPS + L.warp) * NV2;
            if constexpr (G == 16) {
                r[4 * L.g + L.tau] = vb[0].x;
                r[4 * L.g + (L.tau ^ 1)] = vb[0].y;
                r[NPAD + 4 * L.g + L.tau] = vc[0].x;
                r[NPAD + 4 * L.g + (L.tau ^ 1)] = vc[0].y;
            } else {
                const float2 s2 = add2(f2(vb[0].x, vc[0].x),
                                       f2(__shfl_xor_sync(0xffffffffu, vb[0].y, 8),
                                          __shfl_xor_sync(0xffffffffu, vc[0].y, 8)));
                if constexpr (G == 8) {
                    r[4 * L.g + L.tau] = s2.x;
                    r[NPAD + 4 * L.g + L.tau] = s2.y;
                } else {
                    const float send = L.u3 ? s2.x : s2.y;
                    float keep = L.u3 ? s2.y : s2.x;
                    keep += __shfl_xor_sync(0xffffffffu, send, 4);
                    if constexpr (G <= 2) keep += __shfl_xor_sync(0xffffffffu, keep, 2);
                    if constexpr (G == 1) keep += __shfl_xor_sync(0xffffffffu, keep, 1);
                    if (L.sd_writer) r[L.sd_pos] = keep;
                }
            }
        }
    }
    A.anx[0] = acar[0];
    A.anx[1] = acar[1];
}

// After a barrier: this CTA's partial of dB, dC for a walked group (the sum
// over the CTA's warps of the per-warp butterfly results in sd).
template <int G>
__device__ __forceinline__ void flush_group(const float *sd, int tid, int t0, int nv, int N,
                                            float *pbc)
{
    using S = BwdShape<G>;
    constexpr int NPAD = S::NPAD, NV2 = S::NV2;
    for (int p = tid; p < GRP * NV2; p += BWD_THREADS) {
        const int i = p / NV2, jj = p % NV2;
        if (i >= nv) break;
        const int kind = jj / NPAD, n = jj % NPAD;
        const float *rr = sd + i * BWD_WARPS * NV2 + jj;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < BWD_WARPS; ++w) sum += rr[w * NV2];
        if (n < N) pbc[(size_t)(t0 + i) * 2 * N + kind * N + n] = sum;
    }
}

// Adjoint entering the CTA's last step: zero at the end of the sequence;
// otherwise the carry the segment combine left for time segment `sg`, which is
// the whole dA_{t+1} * g_{t+1} term (so the decay multiplying it is 1).
template <int G>
__device__ __forceinline__ void init_adjoint(Adjoint &A, const Lane<G> &L, const float *seg_e,
                                             int sg, int nsg, int D, int N)
{
#pragma unroll
    for (int p = 0; p < 2; ++p) A.gad[p] = A.anx[p] = A.dac[p] = f2(0.f, 0.f);
    if (sg + 1 < nsg) {
        L.load_state(A.gad, seg_e + ((size_t)L.b * nsg + sg) * D * N, N);
        A.anx[0] = A.anx[1] = f2(1.f, 1.f);
    }
}

template <int G>
__device__ __forceinline__ void store_dacc(const Lane<G> &L, const Adjoint &A, float *part_a,
                                           int D, int N)
{
    if (!L.act) return;
    float *pa = part_a + (((size_t)L.b * gridDim.z + blockIdx.z) * D + L.d) * N + 4 * L.g;
    pa[0 ^ L.tau] = -A.dac[0].x;
    pa[1 ^ L.tau] = -A.dac[0].y;
    pa[2 ^ L.tau] = -A.dac[1].x;
    pa[3 ^ L.tau] = -A.dac[1].y;
}

// General backward: any checkpoint stride K (see the file comment).
template <int G, bool VEC, bool PROJ>
__global__ void __launch_bounds__(BWD_THREADS, MMS_BWD_MINB)
bwd_kernel(const float *__restrict__ x, const float *__restrict__ dt,
           const float *__restrict__ aneg, const float *__restrict__ Bm,
           const float *__restrict__ Cm, const float *__restrict__ dy,
           const float *__restrict__ ckpt, float *__restrict__ dx,
           float *__restrict__ ddt, float *__restrict__ part_bc,
           float *__restrict__ part_a, float *subck, const float *__restrict__ seg_e,
           int T, int D, int N, int K, int nblk, int nsegk, int cps, Proj pj_in)
{
    Proj pj = pj_in;                 // the prologue is compiled in only where it is used
    pj.on = PROJ;
    using S = BwdShape<G>;
    constexpr int DPB = S::DPB, NPAD = S::NPAD;
    extern __shared__ __align__(16) float smem[];
    float *nat = smem;                                               // [NAT_BUFS][NATF]
    float *der = nat + NAT_BUFS * S::NATF;                           // [DER_BUFS][DERF]
    float *sd = der + DER_BUFS * S::DERF;                            // [2][GRP][WARPS][NV2]
    float4 *slots = reinterpret_cast<float4 *>(sd + 2 * S::SDF);     // [SLOTS][THREADS]

    const Lane<G> L(aneg, D, N, pj);
    const int tid = L.tid;
    const int nchunk = (T + K - 1) / K;
    const size_t plane = (size_t)D * N;
    const size_t chan = (size_t)L.d * N + 4 * L.g;
    const size_t rowD = (size_t)L.b * T * D;
    const float *xb = x + rowD, *dtb = dt + rowD, *dyb = dy + rowD;
    const float *Bb = Bm + (size_t)L.b * T * N, *Cb = Cm + (size_t)L.b * T * N;
    float *pbc = part_bc + ((size_t)L.b * nblk + blockIdx.x) * T * 2 * N;

    // time segment blockIdx.z: chunks [sg*cps, min((sg+1)*cps, nchunk))
    const int sg = blockIdx.z, nsg = gridDim.z;
    float *subb = subck + ((size_t)L.b * nsg + sg) * nsegk * plane;   // this CTA's slab
    WorkCursor cur, pre;
    cur.start(T, K, min((sg + 1) * cps, nchunk) - 1, sg * cps);
    pre = cur;
#pragma unroll
    for (int s = 0; s < NAT_BUFS; ++s) {
        if (!pre.done()) {
            stage_tile<3, 2, DPB, NPAD, GRP, BWD_THREADS, VEC>(
                nat + s * S::NATF, xb, dtb, dyb, Bb, Cb, pre.tstart(), pre.nvalid(), L.d0, D, N, tid);
            pre.advance();
        }
        cp_commit();
    }
    cp_wait<NAT_BUFS - 1>();
    __syncthreads();
    rewrite_tile<G>(nat, der, tid, pj);

    Adjoint A;
    init_adjoint<G>(A, L, seg_e, sg, nsg, D, N);
    float2 hs[2];
    int cur_chunk = -1, cur_seg = -1;
    int nw = 0, pend_t0 = 0, pend_nv = 0;            // walked groups; the one awaiting its flush

    for (int it = 0; !cur.done(); ++it, cur.advance()) {
        cp_wait<NAT_BUFS - 2>();                      // this thread's copies of item it+1
        __syncthreads();                              // everyone's copies; item it rewritten
        if (pend_nv) {                                // dB|dC of the previous walked group
            flush_group<G>(sd + ((nw - 1) & 1) * S::SDF, tid, pend_t0, pend_nv, N, pbc);
            pend_nv = 0;
        }
        {
            WorkCursor nxt = cur;
            nxt.advance();
            if (!nxt.done())
                rewrite_tile<G>(nat + ((it + 1) % NAT_BUFS) * S::NATF,
                                der + ((it + 1) % DER_BUFS) * S::DERF, tid, pj);
        }
        if (!pre.done()) {                            // item it+3 into item it's natural tile
            stage_tile<3, 2, DPB, NPAD, GRP, BWD_THREADS, VEC>(
                nat + ((it + NAT_BUFS) % NAT_BUFS) * S::NATF, xb, dtb, dyb, Bb, Cb,
                pre.tstart(), pre.nvalid(), L.d0, D, N, tid);
            pre.advance();
        }
        cp_commit();
        const float *dtile = der + (it % DER_BUFS) * S::DERF;
        const TileView<G> v(dtile, L.c, L.g, L.pidx);

        if (cur.c != cur_chunk) {                     // first group of a chunk
            cur_chunk = cur.c;
            cur_seg = -1;
            if (cur.phase == 0) {
                if (cur.c > 0) L.load_state(hs, ckpt + ((size_t)L.b * nchunk + cur.c - 1) * plane, N);
                else hs[0] = hs[1] = f2(0.f, 0.f);
            }
        }
        if (cur.phase == 0) {                         // pre-pass: segment-start states
            advance_tile<G>(hs, L.an2, v);
            if ((cur.j + 1) % SLOTS == 0 && L.act) {
                const int q = (cur.j + 1) / SLOTS;
                *reinterpret_cast<float4 *>(subb + (size_t)q * plane + chan) =
                    make_float4(hs[0].x, hs[0].y, hs[1].x, hs[1].y);
            }
            continue;
        }
        if (cur.sg != cur_seg) {                      // first group of a segment
            cur_seg = cur.sg;
            if (cur.sg > 0) {
                // written by this same thread in the pre-pass: coherent plain load
                float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
                if (L.act) w = *reinterpret_cast<const float4 *>(
                    subb + (size_t)cur.sg * plane + chan);
                hs[0] = lo(w);
                hs[1] = hi(w);
            } else if (cur.c > 0) {
                L.load_state(hs, ckpt + ((size_t)L.b * nchunk + cur.c - 1) * plane, N);
            } else {
                hs[0] = hs[1] = f2(0.f, 0.f);
            }
        }
        if (cur.phase == 1) {                         // recompute: keep group-entry states
            slots[cur.j * BWD_THREADS + tid] = make_float4(hs[0].x, hs[0].y, hs[1].x, hs[1].y);
            advance_tile<G>(hs, L.an2, v);
            continue;
        }

        // ---- walk one group backwards
        const int nv = cur.nvalid();
        const int t0 = cur.tstart();
        float2 hb[2];
        if (cur.j == cur.ngrp - 1) {
            hb[0] = hs[0];
            hb[1] = hs[1];
        } else {
            const float4 w = slots[cur.j * BWD_THREADS + tid];
            hb[0] = lo(w);
            hb[1] = hi(w);
        }
        float *dxo = dx + rowD + (size_t)t0 * D + L.d, *ddto = ddt + rowD + (size_t)t0 * D + L.d;
        float *sdb = sd + (nw & 1) * S::SDF;
        if (nv == GRP) walk_group<G, true>(v, hb, L, A, nv, dxo, ddto, D, sdb, pj);
        else walk_group<G, false>(v, hb, L, A, nv, dxo, ddto, D, sdb, pj);
        ++nw;
        pend_t0 = t0;
        pend_nv = nv;
    }
    cp_wait<0>();
    __syncthreads();
    if (pend_nv) flush_group<G>(sd + ((nw - 1) & 1) * S::SDF, tid, pend_t0, pend_nv, N, pbc);
    store_dacc<G>(L, A, part_a, D, N);
}

// Backward for checkpoint stride K == GRP: every chunk is one group whose
// entry state is the forward's checkpoint, so there is no recompute pass and
// no slot storage; groups are simply chunks nchunk-1 .. 0.
// E: storage type of x, dt, dy, dx, ddt (float or bf16).
template <int G, bool VEC, bool PROJ, typename E>
__global__ void __launch_bounds__(BWD_THREADS, MMS_BWD_K8_MINB)
bwd_kernel_k8(const E *__restrict__ x, const E *__restrict__ dt,
              const float *__restrict__ aneg, const float *__restrict__ Bm,
              const float *__restrict__ Cm, const E *__restrict__ dy,
              const float *__restrict__ ckpt, E *__restrict__ dx,
              E *__restrict__ ddt, float *__restrict__ part_bc,
              float *__restrict__ part_a, const float *__restrict__ seg_e,
              int T, int D, int N, int nblk, int cps, Proj pj_in)
{
    Proj pj = pj_in;                 // the prologue is compiled in only where it is used
    pj.on = PROJ;
    using S = BwdShape<G>;
    constexpr int DPB = S::DPB, NPAD = S::NPAD;
    extern __shared__ __align__(16) float smem[];
    float *nat = smem;
    float *der = nat + NAT_BUFS * S::NATF;
    float *sd = der + DER_BUFS * S::DERF;               // [2][GRP][WARPS][NV2]
    float *cks = sd + 2 * S::SDF;                      // [NAT_BUFS][DPB][NPAD] entry states

    const Lane<G> L(aneg, D, N, pj);
    const int tid = L.tid;
    const int nchunk = (T + GRP - 1) / GRP;
    const size_t plane = (size_t)D * N;
    const size_t rowD = (size_t)L.b * T * D;
    const E *xb = x + rowD, *dtb = dt + rowD, *dyb = dy + rowD;
    const float *Bb = Bm + (size_t)L.b * T * N, *Cb = Cm + (size_t)L.b * T * N;
    const float *ckb = ckpt + (size_t)L.b * nchunk * plane;
    float *pbc = part_bc + ((size_t)L.b * nblk + blockIdx.x) * T * 2 * N;

    // Stage group c: its inputs and the checkpoint it starts from (zeros for c == 0).
    auto stage = [&](int buf, int c) {
        stage_tile<3, 2, DPB, NPAD, GRP, BWD_THREADS, VEC, E>(
            nat + buf * S::NATF, xb, dtb, dyb, Bb, Cb, c * GRP, min(GRP, T - c * GRP),
            L.d0, D, N, tid);
        constexpr int QN = NPAD / 4;
        for (int k = tid; k < DPB * QN; k += BWD_THREADS) {
            const int cc = k / QN, q = k % QN;
            const bool ok = c >= 1 && L.d0 + cc < D && 4 * q < N;
            const float *src = ok ? ckb + (size_t)(c - 1) * plane + (size_t)(L.d0 + cc) * N + 4 * q
                                  : ckb;
            cp16(cks + buf * S::CKF + cc * NPAD + 4 * q, src, ok);
        }
    };
    // The lane's 4 entry states (lane order) from a staged slab.
    auto entry = [&](float2 (&h)[2], int buf) {
        const float *p = cks + buf * S::CKF + L.c * NPAD + 4 * L.g;
        h[0] = f2(p[0 ^ L.tau], p[1 ^ L.tau]);
        h[1] = f2(p[2 ^ L.tau], p[3 ^ L.tau]);
    };

    // time segment blockIdx.z: groups chi .. clo, last to first
    const int sg = blockIdx.z, nsg = gridDim.z;
    const int clo = sg * cps, chi = min((sg + 1) * cps, nchunk) - 1;
    const int ngrp = chi - clo + 1;
#pragma unroll
    for (int s = 0; s < NAT_BUFS; ++s) {
        if (chi - s >= clo) stage(s, chi - s);
        cp_commit();
    }
    cp_wait<NAT_BUFS - 1>();
    __syncthreads();
    rewrite_tile<G, E>(nat, der, tid, pj);
    float2 hnext[2];                                   // state entering the current group
    entry(hnext, 0);

    Adjoint A;
    init_adjoint<G>(A, L, seg_e, sg, nsg, D, N);

    for (int it = 0; it < ngrp; ++it) {
        const int c = chi - it;
        cp_wait<NAT_BUFS - 2>();
        __syncthreads();
        if (it > 0)                                    // dB|dC of the group walked last
            flush_group<G>(sd + ((it - 1) & 1) * S::SDF, tid, (c + 1) * GRP,
                           min(GRP, T - (c + 1) * GRP), N, pbc);
        const float2 hb[2] = {hnext[0], hnext[1]};
        if (c - 1 >= clo) {                            // group it+1: rewrite, take its entry state
            const int nb = (it + 1) % NAT_BUFS;
            rewrite_tile<G, E>(nat + nb * S::NATF, der + ((it + 1) % DER_BUFS) * S::DERF, tid, pj);
            entry(hnext, nb);
        }
        if (c - NAT_BUFS >= clo) stage((it + NAT_BUFS) % NAT_BUFS, c - NAT_BUFS);
        cp_commit();

        const float *dtile = der + (it % DER_BUFS) * S::DERF;
        const TileView<G> v(dtile, L.c, L.g, L.pidx);
        const int t0 = c * GRP;
        const int nv = min(GRP, T - t0);
        E *dxo = dx + rowD + (size_t)t0 * D + L.d, *ddto = ddt + rowD + (size_t)t0 * D + L.d;
        float *sdb = sd + (it & 1) * S::SDF;
        if (nv == GRP) walk_group<G, true, E>(v, hb, L, A, nv, dxo, ddto, D, sdb, pj);
        else walk_group<G, false, E>(v, hb, L, A, nv, dxo, ddto, D, sdb, pj);
    }
    cp_wait<0>();
    __syncthreads();
    flush_group<G>(sd + ((ngrp - 1) & 1) * S::SDF, tid, clo * GRP, min(GRP, T - clo * GRP), N, pbc);
    store_dacc<G>(L, A, part_a, D, N);
}

// The backward's two fixed-order reductions in one launch. Blocks
// [0, nb_bc): dB|dC = sum over the nblk CTA partials of each batch row.
// The other blocks: dAneg = sum over the (batch row, time segment) partials;
// with the prologue, the gradient of the raw A is dAneg * softplus'(A) =
// dAneg * sigmoid(A). A thread takes 4 consecutive outputs (float4): with
// N % 4 == 0 no quad straddles dB and dC and every quad is 16-byte aligned.
// Each output is summed in the same order as one scalar loop would.
__global__ void reduce_kernel(const float *__restrict__ part_bc, float *__restrict__ dB,
                              float *__restrict__ dC, int Bt, int T, int N, int nblk, int nb_bc,
                              const float *__restrict__ part_a, float *__restrict__ daneg,
                              int rows, size_t DN, const float *__restrict__ a_raw, int proj)
{
    if ((int)blockIdx.x < nb_bc) {
        const size_t per_b = (size_t)T * 2 * N;
        const size_t quads = (size_t)Bt * per_b / 4;
        for (size_t qi = (size_t)blockIdx.x * blockDim.x + threadIdx.x; qi < quads;
             qi += (size_t)nb_bc * blockDim.x) {
            const size_t idx = 4 * qi;
            const size_t b = idx / per_b, r = idx - b * per_b;
            const float *p = part_bc + b * nblk * per_b + r;
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k = 0; k < nblk; ++k) {
                const float4 v = ld4(p + (size_t)k * per_b);
                sum.x += v.x;
                sum.y += v.y;
                sum.z += v.z;
                sum.w += v.w;
            }
            const size_t t = r / (2 * N);
            const int j = (int)(r - t * 2 * N);
            st4(j < N ? dB + (b * T + t) * N + j : dC + (b * T + t) * N + (j - N), sum);
        }
        return;
    }
    const size_t nb_a = gridDim.x - nb_bc;
    for (size_t qi = (size_t)(blockIdx.x - nb_bc) * blockDim.x + threadIdx.x; qi < DN / 4;
         qi += nb_a * blockDim.x) {
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < rows; ++r) {
            const float4 v = ld4(part_a + (size_t)r * DN + 4 * qi);
            sum.x += v.x;
            sum.y += v.y;
            sum.z += v.z;
            sum.w += v.w;
        }
        if (proj) {
            const float4 a = ld4(a_raw + 4 * qi);
            sum.x *= 1.f / (1.f + expf(-a.x));
            sum.y *= 1.f / (1.f + expf(-a.y));
            sum.z *= 1.f / (1.f + expf(-a.z));
            sum.w *= 1.f / (1.f + expf(-a.w));
        }
        st4(daneg + 4 * qi, sum);
    }
}

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

BwdWorkspace bwd_workspace_layout(int Bt, int T, int D, int N, int K)
{
    BwdWorkspace w{};
    const int G = groups_for(N);
    const int dpb = BWD_THREADS / G;
    w.nblk = (D + dpb - 1) / dpb;
    const int kk = K < T ? K : T;
    w.nseg = (kk + SEG - 1) / SEG;
    w.plan = seg_plan(Bt, T, D, N, K, true);
    const size_t planes = (size_t)Bt * w.plan.S * D * N * sizeof(float);
    size_t off = 0;
    w.part_bc = off;
    off = align256(off + (size_t)Bt * w.nblk * T * 2 * N * sizeof(float));
    w.part_a = off;
    off = align256(off + planes);
    w.subck = off;
    if (w.nseg > 1) off = align256(off + planes * w.nseg);
    w.seg_e = w.seg_p = off;
    if (w.plan.S > 1) {
        off = align256(off + planes);
        w.seg_p = off;
        off = align256(off + planes);
    }
    w.total = off;
    return w;
}

template <int G, bool VEC, bool PROJ, typename E = float>
static cudaError_t launch_bwd_gvp(const BwdArgs &a, const BwdWorkspace &w, cudaStream_t stream)
{
    using S = BwdShape<G>;
    cudaError_t e;
    char *ws = static_cast<char *>(a.workspace);
    float *part_bc = reinterpret_cast<float *>(ws + w.part_bc);
    float *part_a = reinterpret_cast<float *>(ws + w.part_a);
    float *subck = reinterpret_cast<float *>(ws + w.subck);
    float *seg_e = reinterpret_cast<float *>(ws + w.seg_e);
    float *seg_p = reinterpret_cast<float *>(ws + w.seg_p);
    const SegPlan sp = w.plan;
    if (sp.S > 1) {
        // local adjoint carries of segments 1..S-1, then the chain (last to first)
        SegLocalArgs la{a.dy, a.dt, a.aneg, a.C, seg_e, seg_p, a.Bt, a.T, a.D, a.N,
                        sp.cps * a.K, 1, sp.S - 1, sp.S, 1, 0, 0, a.proj, a.bf16};
        if ((e = launch_seg_local(la, true, stream)) != cudaSuccess) return e;
        if ((e = launch_seg_combine_bwd(seg_e, seg_p, a.Bt, sp.S, (size_t)a.D * a.N, stream)) !=
            cudaSuccess)
            return e;
    }
    dim3 grid(w.nblk, a.Bt, sp.S);
    int nblk = w.nblk;                                 // CTAs along D that wrote dB|dC partials
    if (G >= 4 && MMS_BWD_CP && bwd_cp_applies(a)) {
        e = launch_bwd_cp(a, part_bc, part_a, seg_e, sp, stream, &nblk);
    } else if (G == 4 && bwd_w8_applies(a.N, a.K) && (MMS_BWD_W8 || a.bf16)) {
        e = launch_bwd_w8(a, part_bc, part_a, seg_e, w.nblk, sp, stream);
    } else if (a.K == GRP) {
        e = smem_opt_in<bwd_kernel_k8<G, VEC, PROJ, E>>(S::SMEM_K8);
        if (e != cudaSuccess) return e;
        auto cE = [](const float *p) { return reinterpret_cast<const E *>(p); };
        auto mE = [](float *p) { return reinterpret_cast<E *>(p); };
        bwd_kernel_k8<G, VEC, PROJ, E><<<grid, BWD_THREADS, S::SMEM_K8, stream>>>(
            cE(a.x), cE(a.dt), a.aneg, a.B, a.C, cE(a.dy), a.ckpt, mE(a.dx), mE(a.ddt), part_bc,
            part_a, seg_e, a.T, a.D, a.N, w.nblk, sp.cps, a.proj);
    } else if constexpr (sizeof(E) != 4) {
        return cudaErrorInvalidValue;                  // bf16 storage: stride 8 only
    } else {
        e = smem_opt_in<bwd_kernel<G, VEC, PROJ>>(S::SMEM);
        if (e != cudaSuccess) return e;
        bwd_kernel<G, VEC, PROJ><<<grid, BWD_THREADS, S::SMEM, stream>>>(
            a.x, a.dt, a.aneg, a.B, a.C, a.dy, a.ckpt, a.dx, a.ddt, part_bc, part_a, subck, seg_e,
            a.T, a.D, a.N, a.K, w.nblk, w.nseg, sp.cps, a.proj);
    }
    if (e != cudaSuccess) return e;                    // a launcher's own failure
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    auto blocks = [](size_t quads) {
        const size_t b = (quads + 255) / 256;
        return (int)(b < (size_t)N_SM * 16 ? b : (size_t)N_SM * 16);
    };
    const int nb_bc = blocks((size_t)a.Bt * a.T * 2 * a.N / 4);
    const size_t dn = (size_t)a.D * a.N;
    const int nb_a = blocks(dn / 4);
    reduce_kernel<<<nb_bc + nb_a, 256, 0, stream>>>(part_bc, a.dB, a.dC, a.Bt, a.T, a.N, nblk,
                                                    nb_bc, part_a, a.daneg, a.Bt * sp.S, dn,
                                                    a.aneg, a.proj.on);
    return cudaGetLastError();
}

template <int G, bool VEC>
static cudaError_t launch_bwd_gv(const BwdArgs &a, const BwdWorkspace &w, cudaStream_t stream)
{
    return a.proj.on ? launch_bwd_gvp<G, VEC, true>(a, w, stream)
                     : launch_bwd_gvp<G, VEC, false>(a, w, stream);
}

template <int G>
static cudaError_t launch_bwd_g(const BwdArgs &a, const BwdWorkspace &w, cudaStream_t stream)
{
    return vec_ok(a.D, a.x, a.dt, a.dy) ? launch_bwd_gv<G, true>(a, w, stream)
                                        : launch_bwd_gv<G, false>(a, w, stream);
}

cudaError_t launch_bwd(const BwdArgs &a, cudaStream_t stream)
{
    const BwdWorkspace w = bwd_workspace_layout(a.Bt, a.T, a.D, a.N, a.K);
    if (a.bf16) {
        // bf16 channel arrays: the stride-8 backwards (channel-pair for
        // 8 < N <= 64, else 4-state), 16-byte aligned arrays
        if (a.K != GRP || a.D % 8 != 0 || a.proj.on || !vec_ok(a.D, a.x, a.dt, a.dy) ||
            !vec_ok(a.D, a.dx, a.ddt))
            return cudaErrorInvalidValue;
        using BF = __nv_bfloat16;
        switch (groups_for(a.N)) {
        case 1: return launch_bwd_gvp<1, true, false, BF>(a, w, stream);
        case 2: return launch_bwd_gvp<2, true, false, BF>(a, w, stream);
        case 4: return launch_bwd_gvp<4, true, false, BF>(a, w, stream);
        case 8: return launch_bwd_gvp<8, true, false, BF>(a, w, stream);
        case 16: return launch_bwd_gvp<16, true, false, BF>(a, w, stream);
        default: return cudaErrorInvalidValue;
        }
    }
    switch (groups_for(a.N)) {
    case 1: return launch_bwd_g<1>(a, w, stream);
    case 2: return launch_bwd_g<2>(a, w, stream);
    case 4: return launch_bwd_g<4>(a, w, stream);
    case 8: return launch_bwd_g<8>(a, w, stream);
    case 16: return launch_bwd_g<16>(a, w, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace mms
