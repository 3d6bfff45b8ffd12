// Backward selective scan on channel pairs (8 < N <= 16, checkpoint stride K =
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
// Lane layout: q = lane bits 0-1 picks states 4q..4q+3, lane bits 2-4 the
// channel pair within the warp. The thread keeps its states in the order
// 4q + (m XOR tau), tau = lane bits 4,3, so the first two butterfly levels of
// the dB|dC reduction (over lane bits 4 and 3) are select-free; B and C are
// rewritten once per sub-chunk into the four orders in shared memory.
//
// Time: a CTA (128 threads, 64 channels of one batch row, 3 per SM) walks its
// checkpoint chunks last to first in 8-step sub-chunks. A sub-chunk is
// rebuilt from the state entering it (all 8 decays kept, states of steps 4..7
// kept), walked over steps 7..5, its steps 0..3 recomputed from the entry
// state with the kept decays (no ex2), and walked over steps 4..0. For K > 8
// the states entering sub-chunks 1..m-1 of a chunk come from a forward
// pre-pass over the chunk into shared-memory slots.
//
// Staging: one item per sub-chunk visit (pre-pass or walk), in the order the
// CTA consumes them, by six TMA tile loads (x, dt, dy boxes of 64 channels x
// 8 steps, B and C boxes, and the 64 x 16 checkpoint slab the chunk starts
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
constexpr int CP_DPB = 64;                    // channels per CTA
constexpr int CP_SUB = 8;                     // steps per sub-chunk
constexpr int CP_NAT = 3;                     // TMA stages
constexpr int CP_MAXM = 8;                    // sub-chunks per chunk (K <= 64)
constexpr float CP_LN2 = 0.6931471805599453f;

// Stage layout (floats from the stage start, every region 128-byte aligned):
// x, dt, dy [8][64] of E, B, C [8][16], entry slab [64][16].
template <typename E>
struct CpTile {
    static constexpr int ARR = CP_SUB * CP_DPB * (int)sizeof(E) / 4;
    static constexpr int BC = 3 * ARR;
    static constexpr int CK = BC + 2 * CP_SUB * 16;
    static constexpr int F = CK + CP_DPB * 16;
    static constexpr uint32_t BYTES = 4u * F;
};

struct CpSmem {
    static constexpr int SD = CP_SUB * CP_WARPS * 32;       // per-warp dB|dC sums
    static constexpr int SLOT = CP_THREADS * 8;             // one entry state per thread
    template <typename E>
    static size_t bytes(int m) {
        return sizeof(float) * ((size_t)CP_NAT * CpTile<E>::F + 2 * CP_SUB * 64 + SD + (size_t)(m - 1) * SLOT) + 64;
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

// Per-thread constants. The arithmetic is scalar: packed FFMA2 / FMUL2 add no
// FP32 throughput on this GPU (measured 122.6 vs 123.8 lanes per clock per
// SM) and their register-pair operands cost moves.
struct CpLane {
    int lane, q, tau, pr;
    int d0c;                      // channel 0 of the pair
    bool dv0, dv1;
    float nan[4][2];              // -Aneg*log2(e) of state s(m), [m][channel]
    __device__ CpLane(const float *aneg, int D, int N, bool proj) {
        const int tid = threadIdx.x;
        lane = tid & 31;
        q = lane & 3;
        tau = (((lane >> 4) & 1) << 1) | ((lane >> 3) & 1);
        pr = (tid >> 5) * 8 + (lane >> 2);
        d0c = blockIdx.x * CP_DPB + 2 * pr;
        dv0 = d0c < D;
        dv1 = d0c + 1 < D;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int s = state(m);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const bool ok = (c ? dv1 : dv0) && s < N;
                float a = ok ? __ldg(aneg + (size_t)(d0c + c) * N + s) : 0.f;
                if (proj) a = ok ? softplus(a) : 0.f;
                nan[m][c] = -a * MMS_LOG2E;
            }
        }
    }
    __device__ int state(int m) const { return 4 * q + (m ^ tau); }
};

// One thread's 8 state values: [position m (state s(m))][channel].
struct St8 {
    float v[4][2];
};

// B and C rows of the 8 steps in the four lane state orders,
// [a (B, C)][t][tau][16]: (B_s(0), .., B_s(3)) of lane (q, tau) at [..][tau][4q].
constexpr int CP_PERM = 2 * CP_SUB * 4 * 16;

template <typename E>
struct CpView {
    const E *x, *dt, *dy;        // channel pair of this lane, step stride CP_DPB
    const float *B, *C;          // this lane's permuted rows, step stride 64
    const float *ck;             // entry slab [64][16]
    __device__ CpView(const float *st, const float *perm, const CpLane &L) {
        x = reinterpret_cast<const E *>(st) + 2 * L.pr;
        dt = reinterpret_cast<const E *>(st + CpTile<E>::ARR) + 2 * L.pr;
        dy = reinterpret_cast<const E *>(st + 2 * CpTile<E>::ARR) + 2 * L.pr;
        B = perm + L.tau * 16 + 4 * L.q;
        C = B + CP_SUB * 64;
        ck = st + CpTile<E>::CK;
    }
    __device__ float2 xs(int t) const { return ld_pair(x + t * CP_DPB); }
    __device__ float2 dts(int t) const { return ld_pair(dt + t * CP_DPB); }
    __device__ float2 dys(int t) const { return ld_pair(dy + t * CP_DPB); }
    __device__ float4 Bs(int t) const { return *reinterpret_cast<const float4 *>(B + t * 64); }
    __device__ float4 Cs(int t) const { return *reinterpret_cast<const float4 *>(C + t * 64); }
    // the chunk's entry state from the checkpoint slab
    __device__ void entry(St8 &h, const CpLane &L) const {
        const float *r0 = ck + (2 * L.pr) * 16, *r1 = r0 + 16;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            h.v[m][0] = r0[L.state(m)];
            h.v[m][1] = r1[L.state(m)];
        }
    }
};

__device__ __forceinline__ float cpt(const float2 &v, int c) { return c ? v.y : v.x; }

// h <- one step; the step's dA returned in dA.
template <typename E>
__device__ __forceinline__ void cp_advance(St8 &h, St8 &dA, const CpView<E> &v, const CpLane &L, int t) {
    const float2 dt2 = v.dts(t), x2 = v.xs(t);
    const float4 Bv = v.Bs(t);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const float dtc = cpt(dt2, c), bx = dtc * cpt(x2, c);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            dA.v[m][c] = ex2(dtc * L.nan[m][c]);
            h.v[m][c] = fmaf(dA.v[m][c], h.v[m][c], bx * comp(Bv, m));
        }
    }
}

// One backward step t: hc = h_t, hp = h_{t-1}, dA = dA_t; r carries
// dA_{t+1}*g_{t+1} in and dA_t*g_t out.
template <typename E, bool PROJ>
__device__ __forceinline__ void cp_walk_step(const CpView<E> &v, const CpLane &L, const St8 &hc,
                                             const St8 &hp, const St8 &dA, St8 &r, St8 &dac, int t,
                                             int nv, E *outp, int D, float *sd, int warp,
                                             const Proj &pj)
{
    const float2 dt2 = v.dts(t), x2 = v.xs(t), dy2 = v.dys(t);
    const float4 Bv = v.Bs(t), Cv = v.Cs(t);
    float sB[2], sA[2], vb[4], vc[4];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const float dtc = cpt(dt2, c), dyc = cpt(dy2, c), bx = dtc * cpt(x2, c);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const float g = fmaf(dyc, comp(Cv, m), r.v[m][c]);
            const float rn = dA.v[m][c] * g;
            const float u = rn * hp.v[m][c];
            sB[c] = m ? fmaf(g, comp(Bv, m), sB[c]) : g * comp(Bv, m);
            sA[c] = m ? fmaf(L.nan[m][c], u, sA[c]) : L.nan[m][c] * u;
            dac.v[m][c] = fmaf(dtc, u, dac.v[m][c]);
            vb[m] = c ? fmaf(bx, g, vb[m]) : bx * g;
            vc[m] = c ? fmaf(dyc, hc.v[m][c], vc[m]) : dyc * hc.v[m][c];
            r.v[m][c] = rn;
        }
    }
    {   // dx = dt*sum gB, ddt = x*sum gB + ln2*sum nan*u, over the pair's 4 state lanes
        const float dx0 = dt2.x * sB[0], dx1 = dt2.y * sB[1];
        const float dd0 = fmaf(x2.x, sB[0], CP_LN2 * sA[0]), dd1 = fmaf(x2.y, sB[1], CP_LN2 * sA[1]);
        const bool b0 = L.lane & 1, b1 = (L.lane >> 1) & 1;
        float kx = b0 ? dx1 : dx0, kd = b0 ? dd1 : dd0;
        kx += __shfl_xor_sync(0xffffffffu, b0 ? dx0 : dx1, 1);
        kd += __shfl_xor_sync(0xffffffffu, b0 ? dd0 : dd1, 1);
        float kv = b1 ? kd : kx;
        kv += __shfl_xor_sync(0xffffffffu, b1 ? kx : kd, 2);
        // this lane ends with channel b0, kind b1 (0 dx, 1 ddt); outp points at
        // its own output array and channel
        if (PROJ && b1) {
            const float dtv = b0 ? dt2.y : dt2.x;
            kv *= (dtv - pj.lo) * (pj.lo + pj.range - dtv) / pj.range;
        }
        if (t < nv && (b0 ? L.dv1 : L.dv0)) outp[(size_t)t * D] = from_f<E>(kv);
    }
    // dB | dC over the warp's 8 channel pairs: lane bits 4, 3 select-free, bit 2 by kind
    vb[0] += __shfl_xor_sync(0xffffffffu, vb[2], 16);
    vb[1] += __shfl_xor_sync(0xffffffffu, vb[3], 16);
    vc[0] += __shfl_xor_sync(0xffffffffu, vc[2], 16);
    vc[1] += __shfl_xor_sync(0xffffffffu, vc[3], 16);
    vb[0] += __shfl_xor_sync(0xffffffffu, vb[1], 8);
    vc[0] += __shfl_xor_sync(0xffffffffu, vc[1], 8);
    const int kb = (L.lane >> 2) & 1;
    float kk = kb ? vc[0] : vb[0];
    kk += __shfl_xor_sync(0xffffffffu, kb ? vb[0] : vc[0], 4);
    sd[(t * CP_WARPS + warp) * 32 + kb * 16 + L.state(0)] = kk;
}

// The state entering sub-chunk j of a chunk: the checkpoint slab (j == 0) or
// the pre-pass slot (j > 0).
template <typename E>
__device__ __forceinline__ void cp_entry(St8 &h, const CpView<E> &v, const CpLane &L, int j,
                                         const float *slot_in)
{
    if (j == 0) {
        v.entry(h, L);
    } else {
        const float4 a0 = reinterpret_cast<const float4 *>(slot_in)[0];
        const float4 a1 = reinterpret_cast<const float4 *>(slot_in)[1];
        h.v[0][0] = a0.x; h.v[0][1] = a0.y; h.v[1][0] = a0.z; h.v[1][1] = a0.w;
        h.v[2][0] = a1.x; h.v[2][1] = a1.y; h.v[3][0] = a1.z; h.v[3][1] = a1.w;
    }
}

// h <- one step with a known dA (no ex2).
template <typename E>
__device__ __forceinline__ void cp_replay(St8 &h, const St8 &dA, const CpView<E> &v, int t) {
    const float2 dt2 = v.dts(t), x2 = v.xs(t);
    const float4 Bv = v.Bs(t);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const float bx = cpt(dt2, c) * cpt(x2, c);
#pragma unroll
        for (int m = 0; m < 4; ++m) h.v[m][c] = fmaf(dA.v[m][c], h.v[m][c], bx * comp(Bv, m));
    }
}

// Rebuild and walk a sub-chunk (nv valid steps) from its entry state and
// carry r. All 8 decays are kept; of the states only h_4..h_7, and h_{-1}..h_3
// are recomputed from the entry state with the kept decays (no ex2) when the
// walk reaches them, which keeps the live registers low.
template <typename E, bool PROJ>
__device__ __forceinline__ void cp_walk(const CpView<E> &v, const CpLane &L, int j,
                                        const float *slot_in, St8 &r, St8 &dac, int nv, E *outp,
                                        int D, float *sd, int warp, const Proj &pj)
{
    St8 dA[CP_SUB], hk[4];                // hk[t - 4] = h_t
    {
        St8 h;
        cp_entry<E>(h, v, L, j, slot_in);
#pragma unroll
        for (int t = 0; t < CP_SUB; ++t) {
            cp_advance<E>(h, dA[t], v, L, t);
            if (t >= 4) hk[t - 4] = h;
        }
    }
#pragma unroll
    for (int t = CP_SUB - 1; t >= 5; --t)
        cp_walk_step<E, PROJ>(v, L, hk[t - 4], hk[t - 5], dA[t], r, dac, t, nv, outp, D, sd, warp, pj);
    St8 hl[5];                            // hl[t + 1] = h_t for t = -1 .. 3
    cp_entry<E>(hl[0], v, L, j, slot_in);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        hl[t + 1] = hl[t];
        cp_replay<E>(hl[t + 1], dA[t], v, t);
    }
    cp_walk_step<E, PROJ>(v, L, hk[0], hl[4], dA[4], r, dac, 4, nv, outp, D, sd, warp, pj);
#pragma unroll
    for (int t = 3; t >= 0; --t)
        cp_walk_step<E, PROJ>(v, L, hl[t + 1], hl[t], dA[t], r, dac, t, nv, outp, D, sd, warp, pj);
}

// The item sequence of one CTA: chunks chi down to clo; in a chunk with mv
// valid sub-chunks, a pre-pass over sub-chunks 0..mv-2, then walks of mv-1..0.
struct CpItems {
    int chi, M, mv_first, first_items, per_chunk, total;
    __device__ CpItems(int clo, int chi_, int M_, int T, int K, int nchunk) : chi(chi_), M(M_) {
        const int steps_last = T - chi * K;                       // valid steps of chunk chi
        mv_first = chi == nchunk - 1 ? min(M, (steps_last + CP_SUB - 1) / CP_SUB) : M;
        first_items = 2 * mv_first - 1;
        per_chunk = 2 * M - 1;
        total = first_items + (chi - clo) * per_chunk;
    }
    // item i -> chunk, sub-chunk within it, walk?
    __device__ void at(int i, int &c, int &j, bool &walk) const {
        int mvc, k;
        if (i < first_items) {
            c = chi;
            k = i;
            mvc = mv_first;
        } else {
            const int e = i - first_items;
            c = chi - 1 - e / per_chunk;
            k = e % per_chunk;
            mvc = M;
        }
        walk = k >= mvc - 1;
        j = walk ? 2 * mvc - 2 - k : k;
    }
};

template <typename E, bool PROJ>
__global__ void __launch_bounds__(CP_THREADS, MMS_BWD_CP_MINB)
bwd_kernel_cp(const float *__restrict__ aneg, E *__restrict__ dx, E *__restrict__ ddt,
              float *__restrict__ part_bc, float *__restrict__ part_a,
              const float *__restrict__ seg_e, int T, int D, int N, int M, int nblk, int cps,
              const __grid_constant__ CpMaps maps, Proj pj_in, uint32_t wait_limit, int skip_item)
{
    Proj pj = pj_in;
    pj.on = PROJ;
    using Q = CpTile<E>;
    extern __shared__ __align__(128) float smem[];
    float *stages = smem;                                  // [CP_NAT][Q::F]
    float *perm = stages + CP_NAT * Q::F;                  // B, C in the lane orders (CP_PERM)
    float *sd = perm + CP_PERM;                            // [8][4][32]
    float *slots = sd + CpSmem::SD;                        // [M-1][128][8]
    const uint32_t bars = smem_u32(slots + (size_t)(M - 1) * CpSmem::SLOT);

    const CpLane L(aneg, D, N, PROJ);
    const int tid = threadIdx.x, brow = blockIdx.y;
    const int K = M * CP_SUB;
    const int nchunk = (T + K - 1) / K;
    const size_t plane = (size_t)D * N;
    const size_t rowD = (size_t)brow * T * D;
    const int d0 = blockIdx.x * CP_DPB;
    float *pbc = part_bc + ((size_t)brow * nblk + blockIdx.x) * T * 2 * N;

    const int sg = blockIdx.z, nsg = gridDim.z;
    const int clo = sg * cps, chi = min((sg + 1) * cps, nchunk) - 1;
    const CpItems items(clo, chi, M, T, K, nchunk);

    auto issue = [&](int i) {                              // thread 0: TMA loads of item i
        if (i >= items.total || i == skip_item) return;
        int c, j;
        bool walk;
        items.at(i, c, j, walk);
        const int buf = i % CP_NAT;
        const uint32_t bar = bars + 8 * buf, dst = smem_u32(stages + buf * Q::F);
        const int t0 = (c * M + j) * CP_SUB;
        mbar_expect(bar, Q::BYTES);
        tma3(dst, &maps.x, d0, t0, brow, bar);
        tma3(dst + 4 * Q::ARR, &maps.dt, d0, t0, brow, bar);
        tma3(dst + 8 * Q::ARR, &maps.dy, d0, t0, brow, bar);
        tma3(dst + 4 * Q::BC, &maps.B, 0, t0, brow, bar);
        tma3(dst + 4 * (Q::BC + CP_SUB * 16), &maps.C, 0, t0, brow, bar);
        tma4(dst + 4 * Q::CK, &maps.ck, 0, d0, c - 1, brow, bar);
    };

    St8 r, dac;
#pragma unroll
    for (int m = 0; m < 4; ++m) r.v[m][0] = r.v[m][1] = dac.v[m][0] = dac.v[m][1] = 0.f;
    if (sg + 1 < nsg) {                                    // adjoint carry from the later segments
        const float *src = seg_e + ((size_t)brow * nsg + sg) * plane + (size_t)L.d0c * N;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int s = L.state(m);
            r.v[m][0] = L.dv0 && s < N ? src[s] : 0.f;
            r.v[m][1] = L.dv1 && s < N ? src[N + s] : 0.f;
        }
    }

    if (tid == 0) {
        for (int s = 0; s < CP_NAT; ++s) mbar_init(bars + 8 * s, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        issue(0);
        issue(1);
    }
    __syncthreads();

    // dB|dC partial of the walked sub-chunk starting at step t0p (nvp steps)
    auto flush = [&](int t0p, int nvp) {
        for (int p = tid; p < CP_SUB * 32; p += CP_THREADS) {
            const int i = p >> 5, j = p & 31;
            const int kind = j >> 4, n = j & 15;
            if (i < nvp && n < N) {
                const float *s = sd + i * CP_WARPS * 32 + j;
                pbc[(size_t)(t0p + i) * 2 * N + kind * N + n] = (s[0] + s[32]) + (s[64] + s[96]);
            }
        }
    };

    int pend_t0 = -1, pend_nv = 0;
    for (int i = 0; i < items.total; ++i) {
        const int buf = i % CP_NAT;
        const bool ok = cp_wait_bar(bars + 8 * buf, (i / CP_NAT) & 1, wait_limit);
        if (__syncthreads_or(!ok)) {
            // a stage never arrived: leave together, after the copies still in flight
            if (tid == 0) {
                for (int k = i; k < min(i + CP_NAT - 1, items.total); ++k)
                    if (k != skip_item) cp_wait_bar(bars + 8 * (k % CP_NAT), (k / CP_NAT) & 1, wait_limit);
                atomicOr(&g_cp_timeout, 1u);
            }
            return;
        }
        int c, j;
        bool walk;
        items.at(i, c, j, walk);
        float *st = stages + buf * Q::F;
        if (pend_t0 >= 0) {
            flush(pend_t0, pend_nv);
            pend_t0 = -1;
        }
        // B, C of the 8 steps in the four lane state orders: perm[a][t][tau][16]
        for (int e = tid; e < 2 * CP_SUB * 4 * 4; e += CP_THREADS) {
            const int qq = e & 3, ta = (e >> 2) & 3, t = (e >> 4) & 7, a = e >> 7;
            const float *src = st + Q::BC + (a * CP_SUB + t) * 16 + 4 * qq;
            *reinterpret_cast<float4 *>(perm + ((a * CP_SUB + t) * 4 + ta) * 16 + 4 * qq) =
                make_float4(src[0 ^ ta], src[1 ^ ta], src[2 ^ ta], src[3 ^ ta]);
        }
        if constexpr (PROJ) {                              // dt from its logit, in place (fp32)
            float *dts = st + Q::ARR;
            for (int e = tid; e < CP_SUB * CP_DPB; e += CP_THREADS)
                dts[e] = fmaf(pj.range, sigmoid_fast(dts[e]), pj.lo);
        }
        if (tid == 0 && i + 2 < items.total) {
            fence_async_smem();                            // stage (i+2)%3 was read before the barrier
            issue(i + 2);
        }
        __syncthreads();

        const CpView<E> v(st, perm, L);
        const int u = c * M + j;                           // sub-chunk index in the sequence
        const int t0 = u * CP_SUB;
        const int nv = min(CP_SUB, T - t0);
        const float *slot_in = slots + (size_t)(j - 1) * CpSmem::SLOT + tid * 8;
        if (!walk) {
            // pre-pass: the state entering sub-chunk j+1 into slot j
            St8 h, dA;
            cp_entry<E>(h, v, L, j, slot_in);
#pragma unroll
            for (int t = 0; t < CP_SUB; ++t) cp_advance<E>(h, dA, v, L, t);
            float4 *sl = reinterpret_cast<float4 *>(slots + (size_t)j * CpSmem::SLOT + tid * 8);
            sl[0] = make_float4(h.v[0][0], h.v[0][1], h.v[1][0], h.v[1][1]);
            sl[1] = make_float4(h.v[2][0], h.v[2][1], h.v[3][0], h.v[3][1]);
        } else {
            // this lane's output after the dx / ddt exchange: array (lane bit 1), channel (bit 0)
            E *outp = ((L.lane >> 1) & 1 ? ddt : dx) + rowD + (size_t)t0 * D + L.d0c + (L.lane & 1);
            cp_walk<E, PROJ>(v, L, j, slot_in, r, dac, nv, outp, D, sd, tid >> 5, pj);
            pend_t0 = t0;
            pend_nv = nv;
        }
    }
    __syncthreads();
    if (pend_t0 >= 0) flush(pend_t0, pend_nv);
    float *pa = part_a + ((size_t)brow * nsg + sg) * plane + (size_t)L.d0c * N;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int s = L.state(m);
        if (s < N) {
            if (L.dv0) pa[s] = -dac.v[m][0];
            if (L.dv1) pa[N + s] = -dac.v[m][1];
        }
    }
}

bool build_cp_maps(const BwdArgs &a, CpMaps *m)
{
    const auto fn = tma_encoder();
    if (!fn || !tma_context()) return false;
    const cuuint64_t dX[3] = {(cuuint64_t)a.D, (cuuint64_t)a.T, (cuuint64_t)a.Bt};
    const cuuint32_t bX[3] = {CP_DPB, CP_SUB, 1};
    const cuuint64_t dB[3] = {(cuuint64_t)a.N, (cuuint64_t)a.T, (cuuint64_t)a.Bt};
    const cuuint32_t bB[3] = {16, CP_SUB, 1};
    const int nchunk = (a.T + a.K - 1) / a.K;
    const cuuint64_t dK[4] = {(cuuint64_t)a.N, (cuuint64_t)a.D, (cuuint64_t)nchunk, (cuuint64_t)a.Bt};
    const cuuint32_t bK[4] = {16, CP_DPB, 1, 1};
    const int ex = a.bf16 ? 2 : 4;
    return tma_encode(fn, &m->x, a.x, 3, dX, bX, ex) && tma_encode(fn, &m->dt, a.dt, 3, dX, bX, ex) &&
           tma_encode(fn, &m->dy, a.dy, 3, dX, bX, ex) && tma_encode(fn, &m->B, a.B, 3, dB, bB) &&
           tma_encode(fn, &m->C, a.C, 3, dB, bB) && tma_encode(fn, &m->ck, a.ckpt, 4, dK, bK);
}

template <typename E, bool PROJ>
cudaError_t launch_cp(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                      int nblk, SegPlan sp, const CpMaps &maps, cudaStream_t stream)
{
    const int M = a.K / CP_SUB;
    const size_t smem = CpSmem::bytes<E>(CP_MAXM);         // one opt-in size for every M
    cudaError_t e = smem_opt_in<bwd_kernel_cp<E, PROJ>>(smem);
    if (e != cudaSuccess) return e;
    const uint32_t limit = tma_wait_limit();
    const int skip = tma_skip_item();
    dim3 grid((a.D + CP_DPB - 1) / CP_DPB, a.Bt, sp.S);
    bwd_kernel_cp<E, PROJ><<<grid, CP_THREADS, CpSmem::bytes<E>(M), stream>>>(
        a.aneg, reinterpret_cast<E *>(a.dx), reinterpret_cast<E *>(a.ddt), part_bc, part_a, seg_e,
        a.T, a.D, a.N, M, nblk, sp.cps, maps, a.proj, limit, skip);
    return cudaGetLastError();
}

}  // namespace

bool bwd_cp_applies(const BwdArgs &a)
{
    if (!cp_shape(a.N, a.K) || (a.K == CP_SUB && !MMS_BWD_CP_K8)) return false;

    if (a.bf16) return false;              // bf16 stays on the 8-state kernel (mms_bwd_w8.cu)
    return vec_ok(a.D, a.x, a.dt, a.dy);
}

cudaError_t launch_bwd_cp(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                          int nblk, SegPlan sp, cudaStream_t stream)
{
    CpMaps maps;
    memset(&maps, 0, sizeof(maps));
    if (!build_cp_maps(a, &maps)) return cudaErrorInvalidValue;
    return a.proj.on ? launch_cp<float, true>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream)
                     : launch_cp<float, false>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream);
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
