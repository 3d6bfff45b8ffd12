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
// shuffles about 20/clk): a thread owns two adjacent channels x four states.
//   * dB and dC are sums over channels. Holding two channels, a thread adds
//     them with FMAs before any cross-lane work, and the warp then reduces 8
//     values over its 8 channel pairs (7 shuffles); with dx / ddt (3 shuffles
//     over the channel's 4 state lanes) that is 1.25 shuffles per state-step
//     instead of 2 with one channel per thread.
//   * The 8 decays of a sub-chunk stay in registers from the rebuild to the
//     walk, so every state-step costs one MUFU ex2 (at K = 8).
// Lane layout: NQ = N/4 (rounded up to 4, 8 or 16) lanes share a channel
// pair; q = the low log2(NQ) lane bits picks states 4q..4q+3, the higher
// lane bits the channel pair within the warp. The thread keeps its states in
// the order 4q + (m XOR tau), tau = lane bits 4,3 (bit 4 only for NQ = 16),
// so the butterfly levels of the dB|dC reduction over the pair bits among
// lane bits 4 and 3 are select-free; B and C are rewritten once per
// sub-chunk into the lane orders in shared memory. The dB|dC reduction has
// log2(32/NQ) levels (3, 2, 1) and dx / ddt log2(NQ) (2, 3, 4).
//
// Time: a CTA (128 threads, 256/NQ channels of one batch row, 2 per SM) walks its
// checkpoint chunks last to first in 8-step sub-chunks. A sub-chunk is
// rebuilt from the state entering it (all 8 decays kept, states of steps 4..7
// kept), walked over steps 7..5, its steps 0..3 recomputed from the entry
// state with the kept decays (no ex2), and walked over steps 4..0. For K > 8
// the states entering sub-chunks 1..m-1 of a chunk come from a forward
// pre-pass over the chunk into shared-memory slots.
//
// Staging: one item per sub-chunk visit (pre-pass or walk), in the order the
// CTA consumes them, by six TMA tile loads (x, dt, dy boxes of the CTA's
// channels x 8 steps, B and C boxes, and the channels x 4*NQ checkpoint slab the chunk starts
// from, read at chunk -1 as zeros for the first chunk) issued by one thread
// two items ahead, completing on per-stage mbarriers, three stages.
// Out-of-range steps, channels and states arrive as zeros, which makes them
// no-ops (dt = 0 gives dA = 1 and no input; dy = C = 0 give no adjoint).
//
// Reductions (deterministic, no float atomics): dx / ddt are finished by the
// lane exchange above; dB / dC per warp go to shared memory and the CTA's
// four warps are summed into one partial per CTA and step (reduce_kernel
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

#ifndef MMS_BWD_CP_MINB
#define MMS_BWD_CP_MINB 2
#endif
// K = 8 runs the 8-state kernel (mms_bwd_w8.cu) unless this is set.
#ifndef MMS_BWD_CP_K8
#define MMS_BWD_CP_K8 0
#endif

namespace mms {

namespace {

constexpr int CP_THREADS = 128;
constexpr int CP_WARPS = CP_THREADS / 32;
constexpr int CP_SUB = 8;                     // steps per sub-chunk
constexpr int CP_NAT = 3;                     // TMA stages
constexpr int CP_MAXM = 8;                    // sub-chunks per chunk (K <= 64)
constexpr float CP_LN2 = 0.6931471805599453f;

// Geometry for NQ lanes per channel pair (4 states each).
template <int NQ>
struct CpGeo {
    static_assert(NQ == 4 || NQ == 8 || NQ == 16, "4, 8 or 16 lanes per channel pair");
    static constexpr int LOGQ = NQ == 4 ? 2 : NQ == 8 ? 3 : 4;
    static constexpr int DPB = 2 * CP_THREADS / NQ;        // channels per CTA
    static constexpr int NP = 4 * NQ;                       // states, padded
    static constexpr int PPW = 32 / NQ;                     // channel pairs per warp
    static constexpr int TAUS = NQ == 16 ? 2 : 4;           // state orders in use
    static constexpr int DUP_STEP = 2 * TAUS * NQ * 4;      // duplicated B (or C) per step
    static constexpr int DUP = 2 * CP_SUB * DUP_STEP;       // both arrays
    static constexpr int SD = CP_SUB * CP_WARPS * 2 * NP;   // per-warp dB|dC sums
};

// Stage layout (floats from the stage start, every region 128-byte aligned):
// x, dt, dy [8][DPB] of E, B, C [8][NP], entry slab [DPB][NP].
template <typename E, int NQ>
struct CpTile {
    using G = CpGeo<NQ>;
    static constexpr int ARR = CP_SUB * G::DPB * (int)sizeof(E) / 4;
    static constexpr int BC = 3 * ARR;
    static constexpr int CK = BC + 2 * CP_SUB * G::NP;
    static constexpr int F = CK + G::DPB * G::NP;
    static constexpr uint32_t BYTES = 4u * F;
};

struct CpSmem {
    static constexpr int SLOT = CP_THREADS * 8;             // one entry state per thread
    template <typename E, int NQ>
    static size_t bytes(int m) {
        using G = CpGeo<NQ>;
        return sizeof(float) * ((size_t)CP_NAT * CpTile<E, NQ>::F + G::DUP + G::SD +
                                (size_t)(m - 1) * SLOT) + 64;
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
__device__ __forceinline__ float2 ld_pair(const __nv_bfloat16 *p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
}

// Per-thread constants. Every float2 of a thread pairs its two channels
// (channel 0, channel 1) for one state, so the per-channel step inputs (dt,
// x, dy and dt*x) are natural pairs loaded by one 8-byte read, and the packed
// FFMA2 / FMUL2 instructions take two elements per issue; B and C, which are
// per state, come pre-duplicated from shared memory.
template <int NQ>
struct CpLane {
    int lane, q, tau, ti, pr;     // ti: index of the order tau among the orders in use
    int d0c;                      // channel 0 of the pair
    bool dv0, dv1;
    float2 nan[4];                // -Aneg*log2(e) of state s(m), (channel 0, channel 1)
    __device__ CpLane(const float *aneg, int D, int N, bool proj) {
        using G = CpGeo<NQ>;
        const int tid = threadIdx.x;
        lane = tid & 31;
        q = lane & (NQ - 1);
        tau = (((lane >> 4) & 1) << 1) | (NQ <= 8 ? (lane >> 3) & 1 : 0);
        ti = NQ == 16 ? tau >> 1 : tau;
        pr = (tid >> 5) * G::PPW + (lane >> G::LOGQ);
        d0c = blockIdx.x * G::DPB + 2 * pr;
        dv0 = d0c < D;
        dv1 = d0c + 1 < D;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
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
    __device__ int state(int m) const { return 4 * q + (m ^ tau); }
};

// One thread's 8 state values: [position m] = (channel 0, channel 1) of state s(m).
struct St8 {
    float2 v[4];
};

// B and C of the 8 steps duplicated per state, in the lane state orders:
// [a (B, C)][t][half][ti][q][4] holds (B_s(2h), B_s(2h), B_s(2h+1),
// B_s(2h+1)) of lane (q, tau) at half h; a warp's 16-byte reads of one half
// touch consecutive 16-byte pieces (no bank conflicts).
template <typename E, int NQ>
struct CpView {
    using G = CpGeo<NQ>;
    const E *x, *dt, *dy;        // channel pair of this lane, step stride DPB
    const float *B, *C;          // this lane's duplicated rows, step stride DUP_STEP
    const float *ck;             // entry slab [DPB][NP]
    __device__ CpView(const float *st, const float *dup, const CpLane<NQ> &L) {
        x = reinterpret_cast<const E *>(st) + 2 * L.pr;
        dt = reinterpret_cast<const E *>(st + CpTile<E, NQ>::ARR) + 2 * L.pr;
        dy = reinterpret_cast<const E *>(st + 2 * CpTile<E, NQ>::ARR) + 2 * L.pr;
        B = dup + (L.ti * NQ + L.q) * 4;
        C = B + CP_SUB * G::DUP_STEP;
        ck = st + CpTile<E, NQ>::CK;
    }
    __device__ float2 xs(int t) const { return ld_pair(x + t * G::DPB); }
    __device__ float2 dts(int t) const { return ld_pair(dt + t * G::DPB); }
    __device__ float2 dys(int t) const { return ld_pair(dy + t * G::DPB); }
    // (B_s(2h), B_s(2h), B_s(2h+1), B_s(2h+1))
    __device__ float4 Bs(int t, int h) const {
        return *reinterpret_cast<const float4 *>(B + t * G::DUP_STEP + h * 4 * G::TAUS * NQ);
    }
    __device__ float4 Cs(int t, int h) const {
        return *reinterpret_cast<const float4 *>(C + t * G::DUP_STEP + h * 4 * G::TAUS * NQ);
    }
    // the chunk's entry state from the checkpoint slab
    __device__ void entry(St8 &h, const CpLane<NQ> &L) const {
        const float *r0 = ck + (2 * L.pr) * G::NP, *r1 = r0 + G::NP;
#pragma unroll
        for (int m = 0; m < 4; ++m) h.v[m] = f2(r0[L.state(m)], r1[L.state(m)]);
    }
};

__device__ __forceinline__ float2 dup_of(const float4 &lo4, const float4 &hi4, int m) {
    return m == 0 ? lo(lo4) : m == 1 ? hi(lo4) : m == 2 ? lo(hi4) : hi(hi4);
}

// h <- one step; the step's dA returned in dA.
template <typename E, int NQ>
__device__ __forceinline__ void cp_advance(St8 &h, St8 &dA, const CpView<E, NQ> &v, const CpLane<NQ> &L,
                                           int t) {
    const float2 dt2 = v.dts(t);
    const float2 bx2 = mul2(dt2, v.xs(t));
    const float4 B0 = v.Bs(t, 0), B1 = v.Bs(t, 1);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        dA.v[m] = ex2x2(mul2(dt2, L.nan[m]));
        h.v[m] = fma2(dA.v[m], h.v[m], mul2(bx2, dup_of(B0, B1, m)));
    }
}

// h <- one step with a known dA (no ex2).
template <typename E, int NQ>
__device__ __forceinline__ void cp_replay(St8 &h, const St8 &dA, const CpView<E, NQ> &v, int t) {
    const float2 bx2 = mul2(v.dts(t), v.xs(t));
    const float4 B0 = v.Bs(t, 0), B1 = v.Bs(t, 1);
#pragma unroll
    for (int m = 0; m < 4; ++m) h.v[m] = fma2(dA.v[m], h.v[m], mul2(bx2, dup_of(B0, B1, m)));
}

// One backward step t: hc = h_t, hp = h_{t-1}, dA = dA_t; r carries
// dA_{t+1}*g_{t+1} in and dA_t*g_t out.
template <typename E, int NQ, bool PROJ>
__device__ __forceinline__ void cp_walk_step(const CpView<E, NQ> &v, const CpLane<NQ> &L, const St8 &hc,
                                             const St8 &hp, const St8 &dA, St8 &r, St8 &dac, int t,
                                             int nv, E *outp, int D, float *sd, int warp,
                                             const Proj &pj)
{
    using G = CpGeo<NQ>;
    const float2 dt2 = v.dts(t), x2 = v.xs(t), dy2 = v.dys(t);
    const float2 bx2 = mul2(dt2, x2);
    const float4 B0 = v.Bs(t, 0), B1 = v.Bs(t, 1), C0 = v.Cs(t, 0), C1 = v.Cs(t, 1);
    float2 sB, sA, P[4];                  // P[m] = (sum over the pair of g*dt*x, of dy*h_t)
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float2 g = fma2(dy2, dup_of(C0, C1, m), r.v[m]);
        const float2 rn = mul2(dA.v[m], g);
        const float2 u = mul2(rn, hp.v[m]);
        sB = m ? fma2(g, dup_of(B0, B1, m), sB) : mul2(g, dup_of(B0, B1, m));
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
            kv *= (dtv - pj.lo) * (pj.lo + pj.range - dtv) / pj.range;
        }
        if (t < nv && (NQ == 4 || L.q < 4) && (b0 ? L.dv1 : L.dv0)) outp[(size_t)t * D] = from_f<E>(kv);
    }
    // dB | dC over the warp's channel pairs: lane bit 4 (and 3 for NQ <= 8)
    // select-free, then lane bit 2 by kind for NQ = 4
    P[0] = add2(P[0], shfl2(P[2], 16));
    P[1] = add2(P[1], shfl2(P[3], 16));
    float *row = sd + (t * CP_WARPS + warp) * 2 * G::NP;
    if constexpr (NQ <= 8) P[0] = add2(P[0], shfl2(P[1], 8));
    if constexpr (NQ == 4) {
        const int kb = (L.lane >> 2) & 1;
        float kk = kb ? P[0].y : P[0].x;
        kk += __shfl_xor_sync(0xffffffffu, kb ? P[0].x : P[0].y, 4);
        row[kb * G::NP + L.state(0)] = kk;
    } else {
        row[L.state(0)] = P[0].x;
        row[G::NP + L.state(0)] = P[0].y;
        if constexpr (NQ == 16) {
            row[L.state(1)] = P[1].x;
            row[G::NP + L.state(1)] = P[1].y;
        }
    }
}

// The state entering sub-chunk j of a chunk: the checkpoint slab (j == 0) or
// the pre-pass slot (j > 0).
template <typename E, int NQ>
__device__ __forceinline__ void cp_entry(St8 &h, const CpView<E, NQ> &v, const CpLane<NQ> &L, int j,
                                         const float *slot_in)
{
    if (j == 0) {
        v.entry(h, L);
    } else {
        const float4 a0 = reinterpret_cast<const float4 *>(slot_in)[0];
        const float4 a1 = reinterpret_cast<const float4 *>(slot_in)[1];
        h.v[0] = lo(a0);
        h.v[1] = hi(a0);
        h.v[2] = lo(a1);
        h.v[3] = hi(a1);
    }
}

// Rebuild and walk a sub-chunk (nv valid steps) from its entry state and
// carry r. All 8 decays are kept; of the states only h_4..h_7, and h_{-1}..h_3
// are recomputed from the entry state with the kept decays (no ex2) when the
// walk reaches them, which keeps the live registers low.
template <typename E, int NQ, bool PROJ>
__device__ __forceinline__ void cp_walk(const CpView<E, NQ> &v, const CpLane<NQ> &L, int j,
                                        const float *slot_in, St8 &r, St8 &dac, int nv, E *outp,
                                        int D, float *sd, int warp, const Proj &pj)
{
    St8 dA[CP_SUB], hk[4];                // hk[t - 4] = h_t
    {
        St8 h;
        cp_entry<E, NQ>(h, v, L, j, slot_in);
#pragma unroll
        for (int t = 0; t < CP_SUB; ++t) {
            cp_advance<E, NQ>(h, dA[t], v, L, t);
            if (t >= 4) hk[t - 4] = h;
        }
    }
#pragma unroll
    for (int t = CP_SUB - 1; t >= 5; --t)
        cp_walk_step<E, NQ, PROJ>(v, L, hk[t - 4], hk[t - 5], dA[t], r, dac, t, nv, outp, D, sd, warp, pj);
    St8 hl[5];                            // hl[t + 1] = h_t for t = -1 .. 3
    cp_entry<E, NQ>(hl[0], v, L, j, slot_in);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        hl[t + 1] = hl[t];
        cp_replay<E, NQ>(hl[t + 1], dA[t], v, t);
    }
    cp_walk_step<E, NQ, PROJ>(v, L, hk[0], hl[4], dA[4], r, dac, 4, nv, outp, D, sd, warp, pj);
#pragma unroll
    for (int t = 3; t >= 0; --t)
        cp_walk_step<E, NQ, PROJ>(v, L, hl[t + 1], hl[t], dA[t], r, dac, t, nv, outp, D, sd, warp, pj);
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

template <typename E, int NQ, bool PROJ>
__global__ void __launch_bounds__(CP_THREADS, MMS_BWD_CP_MINB)
bwd_kernel_cp(const float *__restrict__ aneg, E *__restrict__ dx, E *__restrict__ ddt,
              float *__restrict__ part_bc, float *__restrict__ part_a,
              const float *__restrict__ seg_e, int T, int D, int N, int M, int nblk, int cps,
              const __grid_constant__ CpMaps maps, Proj pj_in, uint32_t wait_limit, int skip_item)
{
    Proj pj = pj_in;
    pj.on = PROJ;
    using G = CpGeo<NQ>;
    using Q = CpTile<E, NQ>;
    extern __shared__ __align__(128) float smem[];
    float *stages = smem;                                  // [CP_NAT][Q::F]
    float *dup = stages + CP_NAT * Q::F;                   // B, C duplicated (G::DUP)
    float *sd = dup + G::DUP;                              // [8][4 warps][2 NP]
    float *slots = sd + G::SD;                             // [M-1][128][8]
    const uint32_t bars = smem_u32(slots + (size_t)(M - 1) * CpSmem::SLOT);

    const CpLane<NQ> L(aneg, D, N, PROJ);
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

    St8 r, dac;
#pragma unroll
    for (int m = 0; m < 4; ++m) r.v[m] = dac.v[m] = f2(0.f, 0.f);
    if (sg + 1 < nsg) {                                    // adjoint carry from the later segments
        const float *src = seg_e + ((size_t)brow * nsg + sg) * plane + (size_t)L.d0c * N;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
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
    // walked sub-chunk, column fj of the four warps' sums
    constexpr int COLS = 2 * G::NP, RPP = CP_THREADS / COLS;
    const int fr = tid / COLS, fj = tid % COLS;
    const bool fvalid = fj % G::NP < N;
    float *pbc_col = pbc + (fj / G::NP) * N + fj % G::NP;
    auto flush = [&](int t0p, int nvp) {
#pragma unroll
        for (int h = 0; h < CP_SUB / RPP; ++h) {
            const int i = fr + RPP * h;
            if (i < nvp && fvalid) {
                const float *q = sd + i * CP_WARPS * COLS + fj;
                pbc_col[(size_t)(t0p + i) * 2 * N] = (q[0] + q[COLS]) + (q[2 * COLS] + q[3 * COLS]);
            }
        }
    };
    // this thread's share of the B, C duplication: combination pc = (half,
    // order, quad) of a step, rows pat, pat + GRP, ... of the 16 (array, step) rows
    constexpr int CMB = 2 * G::TAUS * NQ, GRP = CP_THREADS / CMB;
    const int pc = tid % CMB, pat = tid / CMB;
    const int pq = pc % NQ, pti = (pc / NQ) % G::TAUS, ph = pc / (NQ * G::TAUS);
    const int ptau = NQ == 16 ? pti << 1 : pti;
    const int ps0 = 4 * pq + ((2 * ph) ^ ptau), ps1 = 4 * pq + ((2 * ph + 1) ^ ptau);

    CpCursor cur(chi, M, T, K, nchunk);
    int pend_t0 = -1, pend_nv = 0;
    int buf = 0;
    uint32_t parity = 0;
    for (int i = 0; i < total; ++i) {
        const bool ok = cp_wait_bar(bars + 8 * buf, parity, wait_limit);
        if (__syncthreads_or(!ok)) {
            // a stage never arrived: leave together, after the copies still in flight
            if (tid == 0) {
                for (int k = i; k < min(i + CP_NAT - 1, total); ++k)
                    if (k != skip_item) cp_wait_bar(bars + 8 * (k % CP_NAT), (k / CP_NAT) & 1, wait_limit);
                atomicOr(&g_cp_timeout, 1u);
            }
            return;
        }
        const int c = cur.c, j = cur.j();
        const bool walk = cur.walk();
        float *st = stages + buf * Q::F;
        if (pend_t0 >= 0) {
            flush(pend_t0, pend_nv);
            pend_t0 = -1;
        }
        // B, C of the 8 steps duplicated per state in the lane orders
#pragma unroll
        for (int k = 0; k < 2 * CP_SUB / GRP; ++k) {
            const int at = pat + GRP * k;                  // array at / 8, step at % 8
            const float *src = st + Q::BC + at * G::NP;
            const float b0 = src[ps0], b1 = src[ps1];
            *reinterpret_cast<float4 *>(dup + at * G::DUP_STEP + 4 * pc) = make_float4(b0, b0, b1, b1);
        }
        if constexpr (PROJ) {                              // dt from its logit, in place (fp32)
            float *dts = st + Q::ARR;
            for (int e = tid; e < CP_SUB * G::DPB; e += CP_THREADS)
                dts[e] = fmaf(pj.range, sigmoid_fast(dts[e]), pj.lo);
        }
        if (tid == 0 && i + 2 < total) {
            fence_async_smem();                            // stage (i+2)%3 was read before the barrier
            issue(ahead, i + 2, buf == 0 ? 2 : buf - 1);
            ahead.next();
        }
        __syncthreads();

        const CpView<E, NQ> v(st, dup, L);
        const int u = c * M + j;                           // sub-chunk index in the sequence
        const int t0 = u * CP_SUB;
        const int nv = min(CP_SUB, T - t0);
        const float *slot_in = slots + (size_t)(j - 1) * CpSmem::SLOT + tid * 8;
        if (!walk) {
            // pre-pass: the state entering sub-chunk j+1 into slot j
            St8 h, dA;
            cp_entry<E, NQ>(h, v, L, j, slot_in);
#pragma unroll
            for (int t = 0; t < CP_SUB; ++t) cp_advance<E, NQ>(h, dA, v, L, t);
            float4 *sl = reinterpret_cast<float4 *>(slots + (size_t)j * CpSmem::SLOT + tid * 8);
            sl[0] = make_float4(h.v[0].x, h.v[0].y, h.v[1].x, h.v[1].y);
            sl[1] = make_float4(h.v[2].x, h.v[2].y, h.v[3].x, h.v[3].y);
        } else {
            // this lane's output after the dx / ddt exchange: array (lane bit 1), channel (bit 0)
            E *outp = ((L.lane >> 1) & 1 ? ddt : dx) + rowD + (size_t)t0 * D + L.d0c + (L.lane & 1);
            cp_walk<E, NQ, PROJ>(v, L, j, slot_in, r, dac, nv, outp, D, sd, tid >> 5, pj);
            pend_t0 = t0;
            pend_nv = nv;
        }
        cur.next();
        if (++buf == CP_NAT) {
            buf = 0;
            parity ^= 1u;
        }
    }
    __syncthreads();
    if (pend_t0 >= 0) flush(pend_t0, pend_nv);
    float *pa = part_a + ((size_t)brow * nsg + sg) * plane + (size_t)L.d0c * N;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int s = L.state(m);
        if (s < N) {
            if (L.dv0) pa[s] = -dac.v[m].x;
            if (L.dv1) pa[N + s] = -dac.v[m].y;
        }
    }
}

template <int NQ>
bool build_cp_maps(const BwdArgs &a, CpMaps *m)
{
    using G = CpGeo<NQ>;
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

template <typename E, int NQ, bool PROJ>
cudaError_t launch_cp(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                      int nblk, SegPlan sp, cudaStream_t stream)
{
    CpMaps maps;
    memset(&maps, 0, sizeof(maps));
    if (!build_cp_maps<NQ>(a, &maps)) return cudaErrorInvalidValue;
    const int M = a.K / CP_SUB;
    const size_t smem = CpSmem::bytes<E, NQ>(CP_MAXM);     // one opt-in size for every M
    cudaError_t e = smem_opt_in<bwd_kernel_cp<E, NQ, PROJ>>(smem);
    if (e != cudaSuccess) return e;
    const uint32_t limit = tma_wait_limit();
    const int skip = tma_skip_item();
    dim3 grid((a.D + CpGeo<NQ>::DPB - 1) / CpGeo<NQ>::DPB, a.Bt, sp.S);
    bwd_kernel_cp<E, NQ, PROJ><<<grid, CP_THREADS, CpSmem::bytes<E, NQ>(M), stream>>>(
        a.aneg, reinterpret_cast<E *>(a.dx), reinterpret_cast<E *>(a.ddt), part_bc, part_a, seg_e,
        a.T, a.D, a.N, M, nblk, sp.cps, maps, a.proj, limit, skip);
    return cudaGetLastError();
}

template <int NQ>
cudaError_t launch_cp_n(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                        int nblk, SegPlan sp, cudaStream_t stream)
{
    if (a.bf16) return launch_cp<__nv_bfloat16, NQ, false>(a, part_bc, part_a, seg_e, nblk, sp, stream);
    return a.proj.on ? launch_cp<float, NQ, true>(a, part_bc, part_a, seg_e, nblk, sp, stream)
                     : launch_cp<float, NQ, false>(a, part_bc, part_a, seg_e, nblk, sp, stream);
}

}  // namespace

bool bwd_cp_applies(const BwdArgs &a)
{
    if (!cp_shape(a.N, a.K)) return false;
    // stride 8 at 8 < N <= 16 runs the 8-state kernel (mms_bwd_w8.cu), bf16
    // always and fp32 unless MMS_BWD_CP_K8: bf16 and fp32 run the same kernel
    // on a shape, so bf16 storage only rounds the fp32 results
    if (w8_shape(a.N, a.K) && (!MMS_BWD_CP_K8 || a.bf16)) return false;
    if (a.bf16 && (a.D % 8 != 0 || a.proj.on)) return false;
    return vec_ok(a.D, a.x, a.dt, a.dy);
}

cudaError_t launch_bwd_cp(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                          int nblk, SegPlan sp, cudaStream_t stream)
{
    switch (groups_for(a.N)) {
    case 4: return launch_cp_n<4>(a, part_bc, part_a, seg_e, nblk, sp, stream);
    case 8: return launch_cp_n<8>(a, part_bc, part_a, seg_e, nblk, sp, stream);
    case 16: return launch_cp_n<16>(a, part_bc, part_a, seg_e, nblk, sp, stream);
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
