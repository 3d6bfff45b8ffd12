// Backward selective scan on channel pairs (8 < N <= 64, checkpoint stride K =
// 8m with 1 <= m <= 8).
//
// Same mathematics as mms_bwd.cu (reference mamba_metal/scan.py:26-34, kernel
// ssm_bwd at :132-261):
//     g_t = dy_t*C_t + r_{t+1},   r_t = dA_t*g_t,   u_t = r_t*h_{t-1}
//     dx_t = dt_t*sum_n g*B,  ddt_t = x_t*sum_n g*B - sum_n Aneg*u,
//     dAneg = -sum_{b,t} dt*u,  dB_t = sum_d g*dt*x,  dC_t = sum_d dy*h_t
// with u_t = g_t*dA_t*h_{t-1} taken from the stored h_{t-1}, so h is never
// run backwards.
//
// Decomposition, chosen from the measured per-SM rates of this GPU (FP32 128
// lanes/clk with packed FFMA2 no faster than FFMA, MUFU ex2 16/clk, warp
// shuffles about 20/clk): a thread owns two adjacent channels x SPT states.
//   * dB and dC are sums over channels. Holding two channels, a thread adds
//     them before any cross-lane work; the warp then reduces over its channel
//     pairs. At N = 16 (4 lanes per pair, 8 pairs per warp) that is 7
//     shuffles for dB|dC and 3 for dx / ddt per 8 state-steps, 1.25 shuffles
//     per state-step instead of 2 with one channel per thread.
//   * The 8 decays of a sub-chunk stay in registers from the rebuild to the
//     walk, so every state-step costs one MUFU ex2 (at K = 8).
// Lane layout: NQ lanes share a channel pair (NQ = N / SPT rounded up to a
// power of two); q = the low log2(NQ) lane bits picks states SPT*q ..
// SPT*q + SPT-1, the higher lane bits the channel pair within the warp. The
// thread keeps its states in the order SPT*q + (m XOR tau), tau from lane
// bits 4 and 3 that are pair bits, so the butterfly levels of the dB|dC
// reduction over those bits are select-free; B and C are rewritten once per
// sub-chunk into the lane orders in shared memory. The lowest pair bit left,
// if any, reduces by kind (dB on one lane, dC on its partner).
//   SPT = 4 (the default; about 250 registers) on NQ = 4, 8, 16 lanes for
//     N <= 16, 32, 64, in 128-thread CTAs (2 per SM), at N > 32 in 256-thread
//     CTAs (1 per SM, MMS_BWD_CP_WIDE): the same CTA slots, with 32 instead
//     of 16 channels per CTA, which halves the per-CTA dB|dC partials
//     (config 3b backward 3290 -> 3174 us);
//   SPT = 2 (256-thread CTAs at 128 registers, 2 per SM: twice the warps) on
//     NQ = 8, 16 lanes for N <= 16, 32, built when MMS_BWD_CP2_MAXN is set.
//     It measures slower (config 1 at K = 8: 443 against 346 us, N = 32:
//     897 against 670 us): per state-step it loads, shuffles and selects
//     more than the extra warps hide.
// The 128-thread CTAs cover 256 / groups_for(N) channels, the general
// backward's block, the 256-thread ones twice that; either fits its
// workspace.
//
// Time: a CTA walks its checkpoint chunks last to first in 8-step
// sub-chunks. A sub-chunk is rebuilt from the state entering it (all 8
// decays kept, states of steps 4..7 kept), walked over steps 7..5, its steps
// 0..3 recomputed from the entry state with the kept decays (no ex2), and
// walked over steps 4..0. For K > 8 the states entering sub-chunks 1..m-1 of
// a chunk come from a forward pre-pass over the chunk into shared-memory
// slots.
//
// Staging: one item per sub-chunk visit (pre-pass or walk), in the order the
// CTA consumes them, by six TMA tile loads (x, dt, dy boxes of the CTA's
// channels x 8 steps, B and C boxes, and the channels x SPT*NQ checkpoint
// slab the chunk starts from, read at chunk -1 as zeros for the first chunk)
// issued by one thread two items ahead, completing on per-stage mbarriers,
// three stages.
// Out-of-range steps, channels and states arrive as zeros, which makes them
// no-ops (dt = 0 gives dA = 1 and no input; dy = C = 0 give no adjoint).
//
// Reductions (deterministic, no float atomics): dx / ddt are finished by the
// lane exchange above; dB / dC per warp go to shared memory and the CTA's
// warps are summed into one partial per CTA and step (reduce_kernel
// adds the CTAs); dAneg accumulates in registers over the walk into one
// partial per (batch row, time segment).
//
// Waits: every thread polls the stage's mbarrier at most `wait_limit` times.
// If any thread's wait runs out, the CTA leaves together (the decision is a
// __syncthreads_or), after thread 0 has waited (again bounded) for the copies
// it still has in flight, and a device flag reports the timeout
// (mms_device_status). `skip_item` >= 0 withholds that item's copies in every
// CTA: a test hook that makes the wait run out without any fault.
#include <string.h>

#include "mms_common.cuh"
#include "mms_kernels.h"
#include "mms_stage.cuh"
#include "mms_tma.cuh"

namespace mms {

namespace {

constexpr int CP_SUB = 8;                     // steps per sub-chunk
constexpr int CP_NAT = 3;                     // TMA stages
constexpr int CP_MAXM = 8;                    // sub-chunks per chunk (K <= 64)
constexpr float CP_LN2 = 0.6931471805599453f;

// Geometry: NQ lanes share a channel pair, each lane holding SPT states of
// both channels, in CTAs of THREADS threads: 2 * THREADS / NQ channels.
template <int NQ_, int SPT_, int THREADS_ = 512 / SPT_>
struct CpGeo {
    static constexpr int NQ = NQ_, SPT = SPT_;
    static_assert((SPT == 4 && (NQ == 4 || NQ == 8 || NQ == 16)) || (SPT == 2 && (NQ == 8 || NQ == 16)),
                  "4 states on 4, 8 or 16 lanes, or 2 states on 8 or 16 lanes");
    static constexpr int THREADS = THREADS_;
    static_assert(THREADS == 512 / SPT || (SPT == 4 && THREADS == 256), "128 or 256 threads at 4 states");
    static constexpr int MINB = THREADS * SPT == 1024 ? 1 : 2;  // CTAs per SM the registers allow
    static constexpr int WARPS = THREADS / 32;
    static constexpr int LOGQ = NQ == 4 ? 2 : NQ == 8 ? 3 : 4;
    static constexpr int DPB = 2 * THREADS / NQ;            // channels per CTA
    static constexpr int NP = SPT * NQ;                     // states, padded
    static constexpr int PPW = 32 / NQ;                     // channel pairs per warp
    static constexpr int HALVES = SPT / 2;                  // float4 of duplicated B per step
    static constexpr int TAUS = SPT == 2 || NQ == 16 ? 2 : 4;   // state orders in use
    static constexpr int DUP_STEP = HALVES * TAUS * NQ * 4; // duplicated B (or C) per step
    static constexpr int DUP = 2 * CP_SUB * DUP_STEP;       // both arrays
    static constexpr int SD = CP_SUB * WARPS * 2 * NP;      // per-warp dB|dC sums
    static constexpr int SLOT = THREADS * 2 * SPT;          // one entry state per thread
};

// Stage layout (floats from the stage start, every region 128-byte aligned):
// x, dt, dy [8][DPB] of E, B, C [8][NP], entry slab [DPB][NP].
template <typename E, typename G>
struct CpTile {
    static constexpr int ARR = CP_SUB * G::DPB * (int)sizeof(E) / 4;
    static constexpr int BC = 3 * ARR;
    static constexpr int CK = BC + 2 * CP_SUB * G::NP;
    static constexpr int F = CK + G::DPB * G::NP;
    static constexpr uint32_t BYTES = 4u * F;
    // `bufs`: 2 with one barrier per item (double-buffered rows and sums), else 1
    static size_t smem(int m, int bufs) {
        return sizeof(float) * ((size_t)CP_NAT * F + bufs * (G::DUP + G::SD) + (size_t)(m - 1) * G::SLOT) + 64;
    }
};

__device__ unsigned int g_cp_timeout;

__device__ __forceinline__ bool cp_wait_bar(uint32_t bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try(bar, parity)) return true;
    return false;
}

struct CpMaps {
    CUtensorMap x, dt, dy, B, C, ck;
};

__device__ __forceinline__ float2 shfl2(float2 v, int m) {
    return f2(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m));
}

__device__ __forceinline__ float2 ld_pair(const float *p) { return *reinterpret_cast<const float2 *>(p); }
// bf16 to fp32 is exact: the bf16 bits are the top half of the fp32 word
// (integer shift and mask, no conversion instruction).
__device__ __forceinline__ float2 ld_pair(const __nv_bfloat16 *p) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
    return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Per-thread constants. Every float2 of a thread pairs its two channels
// (channel 0, channel 1) for one state, so the per-channel step inputs (dt,
// x, dy and dt*x) are natural pairs loaded by one 8-byte read, and the packed
// FFMA2 / FMUL2 instructions take two elements per issue; B and C, which are
// per state, come pre-duplicated from shared memory.
template <typename G>
struct CpLane {
    int lane, q, tau, ti, pr;     // ti: index of the order tau among the orders in use
    int d0c;                      // channel 0 of the pair
    bool dv0, dv1;
    float2 nan[G::SPT];           // -Aneg*log2(e) of state s(m), (channel 0, channel 1)
    __device__ CpLane(const float *aneg, int D, int N, bool proj) {
        const int tid = threadIdx.x;
        lane = tid & 31;
        q = lane & (G::NQ - 1);
        if constexpr (G::SPT == 4) {
            tau = (((lane >> 4) & 1) << 1) | (G::NQ <= 8 ? (lane >> 3) & 1 : 0);
            ti = G::NQ == 16 ? tau >> 1 : tau;
        } else {
            tau = ti = (lane >> 4) & 1;
        }
        pr = (tid >> 5) * G::PPW + (lane >> G::LOGQ);
        d0c = blockIdx.x * G::DPB + 2 * pr;
        dv0 = d0c < D;
        dv1 = d0c + 1 < D;
#pragma unroll
        for (int m = 0; m < G::SPT; ++m) {
            const int s = state(m);
            float a0 = dv0 && s < N ? __ldg(aneg + (size_t)d0c * N + s) : 0.f;
            float a1 = dv1 && s < N ? __ldg(aneg + (size_t)(d0c + 1) * N + s) : 0.f;
            if (proj) {
                a0 = dv0 && s < N ? softplus(a0) : 0.f;
                a1 = dv1 && s < N ? softplus(a1) : 0.f;
            }
            nan[m] = f2(-a0 * MMS_LOG2E, -a1 * MMS_LOG2E);
        }
    }
    __device__ int state(int m) const { return G::SPT * q + (m ^ tau); }
};

// One thread's state values: [position m] = (channel 0, channel 1) of state s(m).
template <int SPT>
struct St {
    float2 v[SPT];
};

// The duplicated B (or C) of one step for one lane: (B_s(m), B_s(m)) at m.
template <int SPT>
struct DupV;
template <>
struct DupV<4> {
    float4 a, b;
    __device__ float2 operator[](int m) const { return m == 0 ? lo(a) : m == 1 ? hi(a) : m == 2 ? lo(b) : hi(b); }
};
template <>
struct DupV<2> {
    float4 a;
    __device__ float2 operator[](int m) const { return m == 0 ? lo(a) : hi(a); }
};

// B and C of the 8 steps duplicated per state, in the lane state orders:
// [a (B, C)][t][half][ti][q][4] holds (B_s(2h), B_s(2h), B_s(2h+1),
// B_s(2h+1)) of lane (q, tau) at half h; a warp's 16-byte reads of one half
// touch consecutive 16-byte pieces (no bank conflicts).
template <typename E, typename G>
struct CpView {
    using Q = CpTile<E, G>;
    const E *x, *dt, *dy;        // channel pair of this lane, step stride DPB
    const float *B, *C;          // this lane's duplicated rows, step stride DUP_STEP
    const float *ck;             // entry slab [DPB][NP]
    __device__ CpView(const float *st, const float *dup, const CpLane<G> &L) {
        x = reinterpret_cast<const E *>(st) + 2 * L.pr;
        dt = reinterpret_cast<const E *>(st + Q::ARR) + 2 * L.pr;
        dy = reinterpret_cast<const E *>(st + 2 * Q::ARR) + 2 * L.pr;
        B = dup + (L.ti * G::NQ + L.q) * 4;
        C = B + CP_SUB * G::DUP_STEP;
        ck = st + Q::CK;
    }
    __device__ float2 xs(int t) const { return ld_pair(x + t * G::DPB); }
    __device__ float2 dts(int t) const { return ld_pair(dt + t * G::DPB); }
    __device__ float2 dys(int t) const { return ld_pair(dy + t * G::DPB); }
    static __device__ DupV<G::SPT> dupv(const float *p) {
        const float4 *v = reinterpret_cast<const float4 *>(p);
        if constexpr (G::SPT == 4) return {v[0], v[G::TAUS * G::NQ]};
        else return {v[0]};
    }
    __device__ DupV<G::SPT> Bs(int t) const { return dupv(B + t * G::DUP_STEP); }
    __device__ DupV<G::SPT> Cs(int t) const { return dupv(C + t * G::DUP_STEP); }
    // the chunk's entry state from the checkpoint slab
    __device__ void entry(St<G::SPT> &h, const CpLane<G> &L) const {
        const float *r0 = ck + (2 * L.pr) * G::NP, *r1 = r0 + G::NP;
#pragma unroll
        for (int m = 0; m < G::SPT; ++m) h.v[m] = f2(r0[L.state(m)], r1[L.state(m)]);
    }
};

// h <- one step; the step's dA returned in dA.
template <typename E, typename G>
__device__ __forceinline__ void cp_advance(St<G::SPT> &h, St<G::SPT> &dA, const CpView<E, G> &v,
                                           const CpLane<G> &L, int t) {
    const float2 dt2 = v.dts(t);
    const float2 bx2 = mul2(dt2, v.xs(t));
    const DupV<G::SPT> Bv = v.Bs(t);
#pragma unroll
    for (int m = 0; m < G::SPT; ++m) {
        dA.v[m] = ex2x2(mul2(dt2, L.nan[m]));
        h.v[m] = fma2(dA.v[m], h.v[m], mul2(bx2, Bv[m]));
    }
}

// h <- one step with a known dA (no ex2).
template <typename E, typename G>
__device__ __forceinline__ void cp_replay(St<G::SPT> &h, const St<G::SPT> &dA, const CpView<E, G> &v, int t) {
    const float2 bx2 = mul2(v.dts(t), v.xs(t));
    const DupV<G::SPT> Bv = v.Bs(t);
#pragma unroll
    for (int m = 0; m < G::SPT; ++m) h.v[m] = fma2(dA.v[m], h.v[m], mul2(bx2, Bv[m]));
}

// One backward step t: hc = h_t, hp = h_{t-1}, dA = dA_t; r carries
// dA_{t+1}*g_{t+1} in and dA_t*g_t out.
template <typename E, typename G, bool PROJ>
__device__ __forceinline__ void cp_walk_step(const CpView<E, G> &v, const CpLane<G> &L,
                                             const St<G::SPT> &hc, const St<G::SPT> &hp,
                                             const St<G::SPT> &dA, St<G::SPT> &r, St<G::SPT> &dac,
                                             int t, int nv, E *outp, int D, float *sd, int warp,
                                             const Proj &pj)
{
    constexpr int SPT = G::SPT, NQ = G::NQ;
    const float2 dt2 = v.dts(t), x2 = v.xs(t), dy2 = v.dys(t);
    const float2 bx2 = mul2(dt2, x2);
    const DupV<SPT> Bv = v.Bs(t), Cv = v.Cs(t);
    float2 sB, sA, P[SPT];                // P[m] = (sum over the pair of g*dt*x, of dy*h_t)
#pragma unroll
    for (int m = 0; m < SPT; ++m) {
        const float2 g = fma2(dy2, Cv[m], r.v[m]);
        const float2 rn = mul2(dA.v[m], g);
        const float2 u = mul2(rn, hp.v[m]);
        sB = m ? fma2(g, Bv[m], sB) : mul2(g, Bv[m]);
        sA = m ? fma2(L.nan[m], u, sA) : mul2(L.nan[m], u);
        dac.v[m] = fma2(dt2, u, dac.v[m]);
        const float2 pb = mul2(g, bx2), pc = mul2(dy2, hc.v[m]);
        P[m] = f2(pb.x + pb.y, pc.x + pc.y);
        r.v[m] = rn;
    }
    {   // dx = dt*sum gB, ddt = x*sum gB + ln2*sum nan*u, over the pair's NQ state lanes
        const float2 pdx = mul2(dt2, sB);
        const float2 pddt = fma2(x2, sB, mul2(f2(CP_LN2, CP_LN2), sA));
        const bool b0 = L.lane & 1, b1 = (L.lane >> 1) & 1;
        float kx = b0 ? pdx.y : pdx.x, kd = b0 ? pddt.y : pddt.x;
        kx += __shfl_xor_sync(0xffffffffu, b0 ? pdx.x : pdx.y, 1);
        kd += __shfl_xor_sync(0xffffffffu, b0 ? pddt.x : pddt.y, 1);
        float kv = b1 ? kd : kx;
        kv += __shfl_xor_sync(0xffffffffu, b1 ? kx : kd, 2);
        if constexpr (NQ >= 8) kv += __shfl_xor_sync(0xffffffffu, kv, 4);
        if constexpr (NQ >= 16) kv += __shfl_xor_sync(0xffffffffu, kv, 8);
        // this lane ends with channel b0, kind b1 (0 dx, 1 ddt); outp points at
        // its own output array and channel; lanes with q < 4 store
        if (PROJ && b1) {
            const float dtv = b0 ? dt2.y : dt2.x;
            kv *= dt_slope(pj, dtv);
        }
        if (t < nv && (NQ == 4 || L.q < 4) && (b0 ? L.dv1 : L.dv0)) outp[(size_t)t * D] = from_f<E>(kv);
    }
    // dB | dC over the warp's channel pairs: the pair bits among lane bits 4
    // and 3 select-free (the states' order tau), the lowest pair bit by kind
    // where one is left
    float *row = sd + (t * G::WARPS + warp) * 2 * G::NP;
    if constexpr (SPT == 4) {
        P[0] = add2(P[0], shfl2(P[2], 16));
        P[1] = add2(P[1], shfl2(P[3], 16));
        if constexpr (NQ <= 8) P[0] = add2(P[0], shfl2(P[1], 8));
    } else {
        P[0] = add2(P[0], shfl2(P[1], 16));
    }
    constexpr int KIND_BIT = SPT == 4 && NQ == 4 ? 2 : SPT == 2 && NQ == 8 ? 3 : -1;
    if constexpr (KIND_BIT >= 0) {
        const int kb = (L.lane >> KIND_BIT) & 1;
        float kk = kb ? P[0].y : P[0].x;
        kk += __shfl_xor_sync(0xffffffffu, kb ? P[0].x : P[0].y, 1 << KIND_BIT);
        row[kb * G::NP + L.state(0)] = kk;
    } else {
        row[L.state(0)] = P[0].x;
        row[G::NP + L.state(0)] = P[0].y;
        if constexpr (SPT == 4 && NQ == 16) {
            row[L.state(1)] = P[1].x;
            row[G::NP + L.state(1)] = P[1].y;
        }
    }
}

// The state entering sub-chunk j of a chunk: the checkpoint slab (j == 0) or
// the pre-pass slot (j > 0).
template <typename E, typename G>
__device__ __forceinline__ void cp_entry(St<G::SPT> &h, const CpView<E, G> &v, const CpLane<G> &L, int j,
                                         const float *slot_in)
{
    if (j == 0) {
        v.entry(h, L);
    } else {
        const float4 *sl = reinterpret_cast<const float4 *>(slot_in);
#pragma unroll
        for (int k = 0; k < G::SPT / 2; ++k) {
            const float4 a = sl[k];
            h.v[2 * k] = lo(a);
            h.v[2 * k + 1] = hi(a);
        }
    }
}

// Rebuild and walk a sub-chunk (nv valid steps) from its entry state and
// carry r. All 8 decays are kept; of the states only h_4..h_7, and h_{-1}..h_3
// are recomputed from the entry state with the kept decays (no ex2) when the
// walk reaches them, which keeps the live registers low.
template <typename E, typename G, bool PROJ>
__device__ __forceinline__ void cp_walk(const CpView<E, G> &v, const CpLane<G> &L, int j,
                                        const float *slot_in, St<G::SPT> &r, St<G::SPT> &dac, int nv,
                                        E *outp, int D, float *sd, int warp, const Proj &pj)
{
    using S = St<G::SPT>;
    S dA[CP_SUB], hk[4];                  // hk[t - 4] = h_t
    {
        S h;
        cp_entry<E, G>(h, v, L, j, slot_in);
#pragma unroll
        for (int t = 0; t < CP_SUB; ++t) {
            cp_advance<E, G>(h, dA[t], v, L, t);
            if (t >= 4) hk[t - 4] = h;
        }
    }
#pragma unroll
    for (int t = CP_SUB - 1; t >= 5; --t)
        cp_walk_step<E, G, PROJ>(v, L, hk[t - 4], hk[t - 5], dA[t], r, dac, t, nv, outp, D, sd, warp, pj);
    S hl[5];                              // hl[t + 1] = h_t for t = -1 .. 3
    cp_entry<E, G>(hl[0], v, L, j, slot_in);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        hl[t + 1] = hl[t];
        cp_replay<E, G>(hl[t + 1], dA[t], v, t);
    }
    cp_walk_step<E, G, PROJ>(v, L, hk[0], hl[4], dA[4], r, dac, 4, nv, outp, D, sd, warp, pj);
#pragma unroll
    for (int t = 3; t >= 0; --t)
        cp_walk_step<E, G, PROJ>(v, L, hl[t + 1], hl[t], dA[t], r, dac, t, nv, outp, D, sd, warp, pj);
}

// The item sequence of one CTA: chunks chi down to clo; in a chunk with mv
// valid sub-chunks, a pre-pass over sub-chunks 0..mv-2, then walks of
// mv-1..0 (2*mv - 1 items). A cursor steps through it without divisions.
struct CpCursor {
    int c, k, mvc;              // chunk, item within the chunk, its valid sub-chunks
    int M;
    __device__ CpCursor(int chi, int M_, int T, int K, int nchunk) : c(chi), k(0), M(M_) {
        mvc = chi == nchunk - 1 ? min(M, (T - chi * K + CP_SUB - 1) / CP_SUB) : M;
    }
    __device__ bool walk() const { return k >= mvc - 1; }
    __device__ int j() const { return k >= mvc - 1 ? 2 * mvc - 2 - k : k; }
    __device__ void next() {
        if (++k == 2 * mvc - 1) {
            --c;
            k = 0;
            mvc = M;
        }
    }
};

template <typename E, typename G, bool PROJ, bool ONEBAR>
__global__ void __launch_bounds__(G::THREADS, G::MINB)
bwd_kernel_cp(const float *__restrict__ aneg, E *__restrict__ dx, E *__restrict__ ddt,
              float *__restrict__ part_bc, float *__restrict__ part_a,
              const float *__restrict__ seg_e, int T, int D, int N, int M, int nblk, int cps,
              const __grid_constant__ CpMaps maps, Proj pj_in, uint32_t wait_limit, int skip_item)
{
    Proj pj = pj_in;
    pj.on = PROJ;
    constexpr int SPT = G::SPT, NQ = G::NQ, THREADS = G::THREADS;
    using Q = CpTile<E, G>;
    using S = St<SPT>;
    extern __shared__ __align__(128) float smem[];
    float *stages = smem;                                  // [CP_NAT][Q::F]
    constexpr int BUFS = ONEBAR ? 2 : 1;
    float *dup = stages + CP_NAT * Q::F;                   // [BUFS][G::DUP] B, C duplicated
    float *sd = dup + BUFS * G::DUP;                       // [BUFS][8][WARPS][2 NP]
    float *slots = sd + BUFS * G::SD;                      // [M-1][THREADS][2 SPT]
    const uint32_t bars = smem_u32(slots + (size_t)(M - 1) * G::SLOT);

    const CpLane<G> L(aneg, D, N, PROJ);
    const int tid = threadIdx.x, brow = blockIdx.y;
    const int K = M * CP_SUB;
    const int nchunk = (T + K - 1) / K;
    const size_t plane = (size_t)D * N;
    const size_t rowD = (size_t)brow * T * D;
    const int d0 = blockIdx.x * G::DPB;
    float *pbc = part_bc + ((size_t)brow * nblk + blockIdx.x) * T * 2 * N;

    const int sg = blockIdx.z, nsg = gridDim.z;
    const int clo = sg * cps, chi = min((sg + 1) * cps, nchunk) - 1;
    const int first_items = 2 * CpCursor(chi, M, T, K, nchunk).mvc - 1;
    const int total = first_items + (chi - clo) * (2 * M - 1);

    // thread 0: TMA loads of the item at cursor `at`, number i, into stage i % 3
    auto issue = [&](const CpCursor &at, int i, int buf) {
        if (i == skip_item) return;
        const uint32_t bar = bars + 8 * buf, dst = smem_u32(stages + buf * Q::F);
        const int t0 = (at.c * M + at.j()) * CP_SUB;
        mbar_expect(bar, Q::BYTES);
        tma3(dst, &maps.x, d0, t0, brow, bar);
        tma3(dst + 4 * Q::ARR, &maps.dt, d0, t0, brow, bar);
        tma3(dst + 8 * Q::ARR, &maps.dy, d0, t0, brow, bar);
        tma3(dst + 4 * Q::BC, &maps.B, 0, t0, brow, bar);
        tma3(dst + 4 * (Q::BC + CP_SUB * G::NP), &maps.C, 0, t0, brow, bar);
        tma4(dst + 4 * Q::CK, &maps.ck, 0, d0, at.c - 1, brow, bar);
    };

    S r, dac;
#pragma unroll
    for (int m = 0; m < SPT; ++m) r.v[m] = dac.v[m] = f2(0.f, 0.f);
    if (sg + 1 < nsg) {                                    // adjoint carry from the later segments
        const float *src = seg_e + ((size_t)brow * nsg + sg) * plane + (size_t)L.d0c * N;
#pragma unroll
        for (int m = 0; m < SPT; ++m) {
            const int s = L.state(m);
            r.v[m] = f2(L.dv0 && s < N ? src[s] : 0.f, L.dv1 && s < N ? src[N + s] : 0.f);
        }
    }

    CpCursor ahead(chi, M, T, K, nchunk);                  // thread 0: the next item to issue
    if (tid == 0) {
        for (int s = 0; s < CP_NAT; ++s) mbar_init(bars + 8 * s, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        for (int i = 0; i < 2 && i < total; ++i) {
            issue(ahead, i, i);
            ahead.next();
        }
    }
    __syncthreads();

    // this thread's share of the dB|dC flush: rows fr, fr + RPP, ... of a
    // walked sub-chunk, column fj of the warps' sums
    constexpr int COLS = 2 * G::NP, RPP = THREADS / COLS;
    const int fr = tid / COLS, fj = tid % COLS;
    const bool fvalid = fj % G::NP < N;
    float *pbc_col = pbc + (fj / G::NP) * N + fj % G::NP;
    auto flush = [&](const float *sdp, int t0p, int nvp) {
#pragma unroll
        for (int h = 0; h < CP_SUB / RPP; ++h) {
            const int i = fr + RPP * h;
            if (i < nvp && fvalid) {
                const float *q = sdp + i * G::WARPS * COLS + fj;
                float a = q[0] + q[COLS];
#pragma unroll
                for (int w = 2; w < G::WARPS; w += 2) a += q[w * COLS] + q[(w + 1) * COLS];
                pbc_col[(size_t)(t0p + i) * 2 * N] = a;
            }
        }
    };
    // this thread's share of the B, C duplication: combination pc = (half,
    // order, quad) of a step, rows pat, pat + GRP, ... of the 16 (array, step) rows
    constexpr int CMB = G::HALVES * G::TAUS * NQ, GRP = THREADS / CMB;
    const int pc = tid % CMB, pat = tid / CMB;
    const int pq = pc % NQ, pti = (pc / NQ) % G::TAUS, ph = pc / (NQ * G::TAUS);
    const int ptau = SPT == 4 && NQ == 16 ? pti << 1 : pti;
    const int ps0 = SPT * pq + ((2 * ph) ^ ptau), ps1 = SPT * pq + ((2 * ph + 1) ^ ptau);

    CpCursor cur(chi, M, T, K, nchunk);
    int pend_t0 = -1, pend_nv = 0;
    const float *pend_sd = sd;
    int buf = 0;
    uint32_t parity = 0;
    // ONEBAR: one barrier per item. The duplicated B / C rows and the
    // per-warp dB|dC sums alternate between two buffers by item parity, so a
    // thread can write item i's rows while others still read item i-1's, and
    // flush item i-1's sums while others already walk item i; the barrier
    // orders every buffer's reuse two items apart, and frees the stage of
    // item i-1 for the copies of item i+2. Otherwise (one buffer each) a
    // second barrier separates the rewrite and the flush from the walk.
    auto prepare = [&](const float *st, float *dupi) {
        // B, C of the 8 steps duplicated per state in the lane orders
#pragma unroll
        for (int k = 0; k < 2 * CP_SUB / GRP; ++k) {
            const int at = pat + GRP * k;                  // array at / 8, step at % 8
            const float *src = st + Q::BC + at * G::NP;
            const float b0 = src[ps0], b1 = src[ps1];
            *reinterpret_cast<float4 *>(dupi + at * G::DUP_STEP + 4 * pc) = make_float4(b0, b0, b1, b1);
        }
        if constexpr (PROJ) {                              // dt from its logit, in place (fp32)
            float *dts = const_cast<float *>(st) + Q::ARR;
            for (int e = tid; e < CP_SUB * G::DPB; e += THREADS)
                dts[e] = fmaf(pj.range, sigmoid_fast(dts[e]), pj.lo);
        }
    };
    for (int i = 0; i < total; ++i) {
        const bool ok = cp_wait_bar(bars + 8 * buf, parity, wait_limit);
        float *st = stages + buf * Q::F;
        const int par = ONEBAR ? (i & 1) : 0;
        float *dupi = dup + par * G::DUP;
        if (ONEBAR && ok) prepare(st, dupi);
        if (__syncthreads_or(!ok)) {
            // a stage never arrived: leave together, after the copies still in flight
            if (tid == 0) {
                for (int k = i; k < min(i + CP_NAT - 1, total); ++k)
                    if (k != skip_item) cp_wait_bar(bars + 8 * (k % CP_NAT), (k / CP_NAT) & 1, wait_limit);
                atomicOr(&g_cp_timeout, 1u);
            }
            return;
        }
        if (tid == 0 && i + 2 < total) {
            fence_async_smem();                            // stage (i+2)%3 was read before the barrier
            issue(ahead, i + 2, buf == 0 ? 2 : buf - 1);
            ahead.next();
        }
        if (pend_t0 >= 0) {
            flush(pend_sd, pend_t0, pend_nv);
            pend_t0 = -1;
        }
        if constexpr (!ONEBAR) {
            prepare(st, dupi);
            __syncthreads();
        }
        const int c = cur.c, j = cur.j();
        const bool walk = cur.walk();

        const CpView<E, G> v(st, dupi, L);
        const int u = c * M + j;                           // sub-chunk index in the sequence
        const int t0 = u * CP_SUB;
        const int nv = min(CP_SUB, T - t0);
        const float *slot_in = slots + (size_t)(j - 1) * G::SLOT + tid * 2 * SPT;
        if (!walk) {
            // pre-pass: the state entering sub-chunk j+1 into slot j
            S h, dA;
            cp_entry<E, G>(h, v, L, j, slot_in);
#pragma unroll
            for (int t = 0; t < CP_SUB; ++t) cp_advance<E, G>(h, dA, v, L, t);
            float4 *sl = reinterpret_cast<float4 *>(slots + (size_t)j * G::SLOT + tid * 2 * SPT);
#pragma unroll
            for (int k = 0; k < SPT / 2; ++k)
                sl[k] = make_float4(h.v[2 * k].x, h.v[2 * k].y, h.v[2 * k + 1].x, h.v[2 * k + 1].y);
        } else {
            // this lane's output after the dx / ddt exchange: array (lane bit 1), channel (bit 0)
            E *outp = ((L.lane >> 1) & 1 ? ddt : dx) + rowD + (size_t)t0 * D + L.d0c + (L.lane & 1);
            float *sdi = sd + par * G::SD;
            cp_walk<E, G, PROJ>(v, L, j, slot_in, r, dac, nv, outp, D, sdi, tid >> 5, pj);
            pend_t0 = t0;
            pend_nv = nv;
            pend_sd = sdi;
        }
        cur.next();
        if (++buf == CP_NAT) {
            buf = 0;
            parity ^= 1u;
        }
    }
    __syncthreads();
    if (pend_t0 >= 0) flush(pend_sd, pend_t0, pend_nv);
    float *pa = part_a + ((size_t)brow * nsg + sg) * plane + (size_t)L.d0c * N;
#pragma unroll
    for (int m = 0; m < SPT; ++m) {
        const int s = L.state(m);
        if (s < N) {
            if (L.dv0) pa[s] = -dac.v[m].x;
            if (L.dv1) pa[N + s] = -dac.v[m].y;
        }
    }
}

template <typename G>
bool build_cp_maps(const BwdArgs &a, CpMaps *m)
{
    const auto fn = tma_encoder();
    if (!fn || !tma_context()) return false;
    const cuuint64_t dX[3] = {(cuuint64_t)a.D, (cuuint64_t)a.T, (cuuint64_t)a.Bt};
    const cuuint32_t bX[3] = {G::DPB, CP_SUB, 1};
    const cuuint64_t dB[3] = {(cuuint64_t)a.N, (cuuint64_t)a.T, (cuuint64_t)a.Bt};
    const cuuint32_t bB[3] = {G::NP, CP_SUB, 1};
    const int nchunk = (a.T + a.K - 1) / a.K;
    const cuuint64_t dK[4] = {(cuuint64_t)a.N, (cuuint64_t)a.D, (cuuint64_t)nchunk, (cuuint64_t)a.Bt};
    const cuuint32_t bK[4] = {G::NP, G::DPB, 1, 1};
    const int ex = a.bf16 ? 2 : 4;
    return tma_encode(fn, &m->x, a.x, 3, dX, bX, ex) && tma_encode(fn, &m->dt, a.dt, 3, dX, bX, ex) &&
           tma_encode(fn, &m->dy, a.dy, 3, dX, bX, ex) && tma_encode(fn, &m->B, a.B, 3, dB, bB) &&
           tma_encode(fn, &m->C, a.C, 3, dB, bB) && tma_encode(fn, &m->ck, a.ckpt, 4, dK, bK);
}

// One barrier per item where the double buffers still leave the CTAs per SM
// that the registers allow (228 KB of shared memory, 1 KB of it reserved per
// CTA), except at 8 lanes per pair (d_state 20..32), which measured 1.5 %
// slower with it.
template <typename E, typename G>
bool cp_onebar(int M)
{
    return G::NQ != 8 && CpTile<E, G>::smem(M, 2) + 1024 <= 228 * 1024 / G::MINB;
}

template <typename E, typename G, bool PROJ, bool ONEBAR>
cudaError_t launch_cpb(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                       int nblk, SegPlan sp, const CpMaps &maps, cudaStream_t stream)
{
    using Q = CpTile<E, G>;
    const int M = a.K / CP_SUB;
    const int bufs = ONEBAR ? 2 : 1;
    cudaError_t e = smem_opt_in<bwd_kernel_cp<E, G, PROJ, ONEBAR>>(Q::smem(CP_MAXM, bufs));
    if (e != cudaSuccess) return e;                        // one opt-in size for every M
    const uint32_t limit = tma_wait_limit();
    const int skip = tma_skip_item();
    dim3 grid(nblk, a.Bt, sp.S);                           // nblk = ceil(D / DPB)
    bwd_kernel_cp<E, G, PROJ, ONEBAR><<<grid, G::THREADS, Q::smem(M, bufs), stream>>>(
        a.aneg, reinterpret_cast<E *>(a.dx), reinterpret_cast<E *>(a.ddt), part_bc, part_a, seg_e,
        a.T, a.D, a.N, M, nblk, sp.cps, maps, a.proj, limit, skip);
    return cudaGetLastError();
}

template <typename E, typename G, bool PROJ>
cudaError_t launch_cp(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                      int nblk, SegPlan sp, cudaStream_t stream)
{
    CpMaps maps;
    memset(&maps, 0, sizeof(maps));
    if (!build_cp_maps<G>(a, &maps)) return cudaErrorInvalidValue;
    return cp_onebar<E, G>(a.K / CP_SUB)
               ? launch_cpb<E, G, PROJ, true>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream)
               : launch_cpb<E, G, PROJ, false>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream);
}

template <typename G>
cudaError_t launch_cp_g(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                        int nblk, SegPlan sp, cudaStream_t stream)
{
    if (a.bf16) return launch_cp<__nv_bfloat16, G, false>(a, part_bc, part_a, seg_e, nblk, sp, stream);
    return a.proj.on ? launch_cp<float, G, true>(a, part_bc, part_a, seg_e, nblk, sp, stream)
                     : launch_cp<float, G, false>(a, part_bc, part_a, seg_e, nblk, sp, stream);
}

}  // namespace

bool bwd_cp_applies(const BwdArgs &a)
{
    if (!cp_shape(a.N, a.K)) return false;
    // bf16 and fp32 run the same kernel on a shape (fp32 arrays that bf16
    // could share are aligned), so bf16 storage only rounds the fp32 results
    if (a.bf16 && (a.D % 8 != 0 || a.proj.on)) return false;
    return vec_ok(a.D, a.x, a.dt, a.dy);
}

int cp_channels_per_cta(int N)
{
    const int G = groups_for(N);
    if (G != 4 && G != 8 && G != 16) return 0;
    return (MMS_BWD_CP_WIDE & G ? 512 : 256) / G;
}

cudaError_t launch_bwd_cp(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                          SegPlan sp, cudaStream_t stream, int *nblk_used)
{
    const int G = groups_for(a.N);
    const int dpb = cp_channels_per_cta(a.N);
    if (dpb == 0) return cudaErrorInvalidValue;
    const int nblk = (a.D + dpb - 1) / dpb;
    *nblk_used = nblk;
#if MMS_BWD_CP2_MAXN > 0
    if (cp_two_states(a.N) && !(MMS_BWD_CP_WIDE & G)) {    // same channels per CTA as 128-thread 4-state
        switch (G) {
        case 4: return launch_cp_g<CpGeo<8, 2>>(a, part_bc, part_a, seg_e, nblk, sp, stream);
        case 8: return launch_cp_g<CpGeo<16, 2>>(a, part_bc, part_a, seg_e, nblk, sp, stream);
        default: return cudaErrorInvalidValue;
        }
    }
#endif
    constexpr int T4 = MMS_BWD_CP_WIDE & 4 ? 256 : 128, T8 = MMS_BWD_CP_WIDE & 8 ? 256 : 128,
                  T16 = MMS_BWD_CP_WIDE & 16 ? 256 : 128;
    switch (G) {
    case 4: return launch_cp_g<CpGeo<4, 4, T4>>(a, part_bc, part_a, seg_e, nblk, sp, stream);
    case 8: return launch_cp_g<CpGeo<8, 4, T8>>(a, part_bc, part_a, seg_e, nblk, sp, stream);
    case 16: return launch_cp_g<CpGeo<16, 4, T16>>(a, part_bc, part_a, seg_e, nblk, sp, stream);
    default: return cudaErrorInvalidValue;
    }
}

int cp_take_timeout()
{
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_cp_timeout, sizeof(v)) != cudaSuccess) return -1;
    if (v) {
        const unsigned int z = 0;
        cudaMemcpyToSymbol(g_cp_timeout, &z, sizeof(z));
    }
    return v ? 1 : 0;
}

}  // namespace mms
