// Backward selective scan, 8 states per lane (8 < N <= 16, checkpoint stride 8).
//
// The channel-pair kernel (mms_bwd_cp.cu) runs these shapes when the channel
// arrays are 16-byte aligned (it measured 5-6 % faster); this one runs them
// otherwise, on cp.async staging, and for every such shape in a build with
// MMS_BWD_CP_K8=0, where its TMA staging is used.
//
// Same mathematics as mms_bwd.cu (reference mamba_metal/scan.py:26-34, kernel
// ssm_bwd at :132-261); a different decomposition for the d_state 12/16 case:
// two lanes share a channel and each holds 8 of its 16 states. Compared with
// four lanes of 4 states, every per-step cost that does not depend on the
// state count (x/dt/dy loads and products, the dx/ddt sum over the channel's
// lanes, loop and address work) is spread over 8 states instead of 4, and
// the dx/ddt sum needs one shuffle level instead of two.
//
// A CTA of 128 threads covers 64 channels of one batch row and walks its
// checkpoint chunks (8 steps each) last to first. Per chunk:
//   * the chunk's inputs and its entry checkpoint arrive by cp.async two
//     chunks ahead; after a barrier they are rewritten once into the layouts
//     the walk reads (x, dt, dy as 4-step runs per channel; B and C in the 8
//     lane-specific state orders below); a second barrier publishes them;
//   * the chunk is walked as two 4-step groups, later one first. A group's
//     states are rebuilt from the state entering it and kept in registers
//     (4 steps x 8 states). The later group starts 4 steps into the chunk, so
//     the first 4 steps are advanced once more to reach it (1.5 rebuilds per
//     step instead of 1 in exchange for half the registers).
// Reductions (deterministic, no atomics):
//   * dx, ddt: the two lanes of a channel exchange one value (transposed
//     pair); the lane with the first half stores dx, the other ddt;
//   * dB, dC over the warp's 16 channels: a transposed butterfly over lane
//     bits 4, 3, 2 (where the lane's state order r XOR tau, tau = lane bits
//     2..4, makes every level select-free) and a last transposed level over
//     lane bit 1 (dB vs dC). Each lane ends with one value; the CTA's four
//     warps are summed per step into one partial per CTA (reduce_kernel
//     adds the CTAs);
//   * dAneg: register sums over the walk, one partial per (batch row, time
//     segment).
#include <string.h>

#include "mms_common.cuh"
#include "mms_kernels.h"
#include "mms_stage.cuh"
#include "mms_tma.cuh"

#ifndef MMS_W8_TREE
#define MMS_W8_TREE 1
#endif

namespace mms {

namespace {

constexpr int W8_THREADS = 128;
constexpr int W8_WARPS = W8_THREADS / 32;
constexpr int W8_DPB = W8_THREADS / 2;          // channels per CTA
constexpr int W8_CH = 8;                        // steps per chunk (the checkpoint stride)
constexpr int W8_NAT = 3;                       // natural-layout stages
constexpr float W8_LN2 = 0.6931471805599453f;

// Set when a wait on a TMA completion barrier gave up (see w8_wait);
// read and cleared by mms_device_status().
__device__ unsigned int g_w8_timeout;

// Bounded wait for a stage's copies: at most `limit` polls (each may suspend
// briefly in hardware). A wait that runs out makes the CTA leave (see the
// kernel), so a lost copy turns into an error status instead of a hung GPU.
__device__ __forceinline__ bool w8_wait(uint32_t bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try(bar, parity)) return true;
    return false;
}
// The six tensor maps of the TMA staging path.
struct W8Maps {
    CUtensorMap x, dt, dy, B, C, ck;
};

struct W8Shape {
    static constexpr int NROWF = 3 * W8_DPB + 2 * 16;          // x, dt, dy, B, C per step
    static constexpr int NATF = W8_CH * NROWF;
    static constexpr int CKF = W8_DPB * 16;                    // entry-state slab
    static constexpr int STAGEF = NATF + CKF;
    static constexpr int QF = W8_CH * W8_DPB;                  // one array as 4-step runs
    static constexpr int PF = W8_CH * 8 * 16;                  // B or C in 8 state orders
    static constexpr int DERF = 3 * QF + 2 * PF;
    static constexpr int SDF = W8_CH * W8_WARPS * 32;          // per-warp dB|dC sums
    static constexpr size_t SMEM = sizeof(float) * ((size_t)W8_NAT * STAGEF + DERF + SDF);
    // TMA layout of a stage (array-major, every region 128-byte aligned):
    // x, dt, dy [CH][DPB], B, C [CH][16], entry slab [DPB][16]; same size.
    static constexpr int T_ARR = W8_CH * W8_DPB;               // floats per channel array
    static constexpr int T_BC = 3 * T_ARR;
    static constexpr int T_CK = T_BC + 2 * W8_CH * 16;
    static constexpr uint32_t T_BYTES = 4u * (T_CK + W8_DPB * 16);
    static constexpr size_t SMEM_TMA = SMEM + 64;             // + the stage barriers
};
static_assert(W8Shape::T_CK + W8_DPB * 16 == W8Shape::STAGEF, "stage layouts differ in size");

// TMA stage for channel arrays of storage type E (float or bf16): x, dt, dy
// take ARR floats each, then B, C [CH][16] and the entry slab [DPB][16] (fp32);
// BYTES is what one stage's six loads bring.
template <typename E>
struct W8Tile {
    static constexpr int ARR = W8_CH * W8_DPB * (int)sizeof(E) / 4;
    static constexpr int BC = 3 * ARR;
    static constexpr int CK = BC + 2 * W8_CH * 16;
    static constexpr uint32_t BYTES = 4u * (CK + W8_DPB * 16);
};
static_assert(W8Tile<float>::BYTES == W8Shape::T_BYTES, "fp32 TMA stage is the full stage");

__device__ __forceinline__ float2 shfl2x(float2 v, int m) {
    return f2(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m));
}

// The rewrite: staged tile -> 4-step runs and permuted B/C (fp32 from here
// on, whatever the storage type E of x, dt, dy). TMA selects the stage
// layout: array-major (TMA) or one interleaved row per step (cp.async, fp32).
template <bool TMA, typename E>
__device__ __forceinline__ void w8_rewrite(const float *nat, float *der, int tid, const Proj &pj)
{
    static_assert(TMA || sizeof(E) == 4, "bf16 stages come by TMA");
    constexpr int DPB = W8_DPB, NROWF = W8Shape::NROWF, QF = W8Shape::QF, PF = W8Shape::PF;
    constexpr int AROW = TMA ? DPB : NROWF;                      // step stride, channel arrays (E)
    constexpr int AOFF = TMA ? W8_CH * DPB : DPB;                // array stride (E)
    constexpr int BROW = TMA ? 16 : NROWF;                       // step stride, B and C
    constexpr int BOFF = TMA ? W8Tile<E>::BC : 3 * DPB;          // floats
    constexpr int BARR = TMA ? W8_CH * 16 : 16;                  // B -> C
    // x, dt, dy: der[a][q][c][k] = arr_a[4q + k][c]
    for (int e = tid; e < 3 * 2 * DPB; e += W8_THREADS) {
        const int a = e / (2 * DPB), q = (e / DPB) & 1, cc = e % DPB;
        const E *src = reinterpret_cast<const E *>(nat) + (4 * q) * AROW + a * AOFF + cc;
        float4 v4 = make_float4(to_f(src[0]), to_f(src[AROW]), to_f(src[2 * AROW]),
                                to_f(src[3 * AROW]));
        if (pj.on && a == 1)        // prologue: dt from its logit
            v4 = make_float4(fmaf(pj.range, sigmoid_fast(v4.x), pj.lo), fmaf(pj.range, sigmoid_fast(v4.y), pj.lo),
                             fmaf(pj.range, sigmoid_fast(v4.z), pj.lo), fmaf(pj.range, sigmoid_fast(v4.w), pj.lo));
        *reinterpret_cast<float4 *>(der + a * QF + (q * DPB + cc) * 4) = v4;
    }
    // B, C: der[3QF + a*PF + (i*8 + tau)*16 + 8h + r] = arr_a[i][8h + (r ^ tau)]
    for (int e = tid; e < 2 * W8_CH * 8 * 4; e += W8_THREADS) {
        const int q4 = e & 3;                       // float4 within the 16 outputs
        const int tau = (e >> 2) & 7;
        const int i = (e >> 5) & 7;
        const int a = e >> 8;
        const int h = q4 >> 1, r0 = (q4 & 1) * 4;
        const float *src = nat + i * BROW + BOFF + a * BARR + 8 * h;
        *reinterpret_cast<float4 *>(der + 3 * QF + a * PF + (i * 8 + tau) * 16 + 4 * q4) =
            make_float4(src[(r0 + 0) ^ tau], src[(r0 + 1) ^ tau], src[(r0 + 2) ^ tau],
                        src[(r0 + 3) ^ tau]);
    }
}

struct W8Lane {
    int tid, lane, warp, h, c, d0, d, b, tau, kbit;
    bool dval;
    float2 an2[4];                 // Aneg * log2(e), lane state order
    __device__ W8Lane(const float *aneg, int D, int N, const Proj &pj) {
        tid = threadIdx.x;
        lane = tid & 31;
        warp = tid >> 5;
        h = tid & 1;
        c = tid >> 1;
        d0 = blockIdx.x * W8_DPB;
        d = d0 + c;
        b = blockIdx.y;
        tau = (lane >> 2) & 7;
        kbit = (lane >> 1) & 1;
        dval = d < D;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            float v0 = 0.f, v1 = 0.f;
            const int s0 = 8 * h + ((2 * p) ^ tau), s1 = 8 * h + ((2 * p + 1) ^ tau);
            if (dval && s0 < N) v0 = __ldg(aneg + (size_t)d * N + s0);
            if (dval && s1 < N) v1 = __ldg(aneg + (size_t)d * N + s1);
            if (pj.on) {
                v0 = dval && s0 < N ? softplus(v0) : 0.f;
                v1 = dval && s1 < N ? softplus(v1) : 0.f;
            }
            v0 *= MMS_LOG2E;
            v1 *= MMS_LOG2E;
            an2[p] = f2(v0, v1);
        }
    }
    // the lane's 8 states (lane order) from a row of n floats (states >= n read as 0)
    __device__ void load8(float2 (&v)[4], const float *row, int n) const {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int s0 = 8 * h + ((2 * p) ^ tau), s1 = 8 * h + ((2 * p + 1) ^ tau);
            v[p] = f2(s0 < n ? row[s0] : 0.f, s1 < n ? row[s1] : 0.f);
        }
    }
};

struct W8View {
    const float *qx, *qdt, *qdy, *pB, *pC;
    __device__ W8View(const float *der, const W8Lane &L) {
        qx = der + L.c * 4;
        qdt = der + W8Shape::QF + L.c * 4;
        qdy = der + 2 * W8Shape::QF + L.c * 4;
        pB = der + 3 * W8Shape::QF + L.tau * 16 + 8 * L.h;
        pC = pB + W8Shape::PF;
    }
    __device__ float4 x4(int q) const { return *reinterpret_cast<const float4 *>(qx + q * W8_DPB * 4); }
    __device__ float4 dt4(int q) const { return *reinterpret_cast<const float4 *>(qdt + q * W8_DPB * 4); }
    __device__ float4 dy4(int q) const { return *reinterpret_cast<const float4 *>(qdy + q * W8_DPB * 4); }
    __device__ float4 B(int i, int half) const {
        return *reinterpret_cast<const float4 *>(pB + i * 8 * 16 + 4 * half);
    }
    __device__ float4 C(int i, int half) const {
        return *reinterpret_cast<const float4 *>(pC + i * 8 * 16 + 4 * half);
    }
};

__device__ __forceinline__ float2 pick(const float4 &a, const float4 &b, int p) {
    return p == 0 ? lo(a) : p == 1 ? hi(a) : p == 2 ? lo(b) : hi(b);
}

// h <- 4 steps (quad q of the chunk) from h, states not kept.
__device__ __forceinline__ void w8_advance(float2 (&h)[4], const W8Lane &L, const W8View &v, int q)
{
    const float4 x4 = v.x4(q), d4 = v.dt4(q);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = 4 * q + k;
        const float dtv = comp(d4, k), bx = dtv * comp(x4, k);
        const float4 B0 = v.B(i, 0), B1 = v.B(i, 1);
        const float2 md = f2(-dtv, -dtv), bx2 = f2(bx, bx);
#pragma unroll
        for (int p = 0; p < 4; ++p)
            h[p] = fma2(ex2x2(mul2(md, L.an2[p])), h[p], mul2(bx2, pick(B0, B1, p)));
    }
}

struct W8Adj {
    float2 gad[4], anx[4], dac[4];
};

// Rebuild quad q from hb, then walk it backwards; dx / ddt go to outq (E).
template <bool FULL, typename E>
__device__ __forceinline__ void w8_walk(const W8View &v, const float2 (&hb)[4], const W8Lane &L,
                                        W8Adj &A, int q, int nv, E *outq, int D, float *sd,
                                        const Proj &pj)
{
    float2 hv[4][4];
    {
        const float4 x4 = v.x4(q), d4 = v.dt4(q);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = 4 * q + k;
            const float dtv = comp(d4, k), bx = dtv * comp(x4, k);
            const float4 B0 = v.B(i, 0), B1 = v.B(i, 1);
            const float2 md = f2(-dtv, -dtv), bx2 = f2(bx, bx);
#pragma unroll
            for (int p = 0; p < 4; ++p)
                hv[k][p] = fma2(ex2x2(mul2(md, L.an2[p])), k ? hv[k > 0 ? k - 1 : 0][p] : hb[p],
                                mul2(bx2, pick(B0, B1, p)));
        }
    }
    const float4 x4 = v.x4(q), d4 = v.dt4(q), y4 = v.dy4(q);
#pragma unroll
    for (int k = 3; k >= 0; --k) {
        const int i = 4 * q + k;
        if (!FULL && i >= nv) continue;                       // uniform
        const float dtv = comp(d4, k), xv = comp(x4, k), dyv = comp(y4, k);
        const float4 B0 = v.B(i, 0), B1 = v.B(i, 1), C0 = v.C(i, 0), C1 = v.C(i, 1);
        const float2 dy2 = f2(dyv, dyv), dt2 = f2(dtv, dtv), md = f2(-dtv, -dtv);
        const float dxv = dtv * xv;
        const float2 dxv2 = f2(dxv, dxv);
        float2 p1[2] = {f2(0.f, 0.f), f2(0.f, 0.f)}, p2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
        float2 vb[4], vc[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const float2 am = mul2(md, L.an2[p]);
            const float2 ai = f2(ex2_fresh(am.x), ex2_fresh(am.y));
            A.gad[p] = fma2(A.anx[p], A.gad[p], mul2(dy2, pick(C0, C1, p)));
            A.anx[p] = ai;
            const float2 hp = k ? hv[k > 0 ? k - 1 : 0][p] : hb[p];
            const float2 u = mul2(A.gad[p], mul2(ai, hp));
            // two partial sums each (MMS_W8_TREE) instead of one serial chain
            p1[MMS_W8_TREE ? p & 1 : 0] = fma2(A.gad[p], pick(B0, B1, p), p1[MMS_W8_TREE ? p & 1 : 0]);
            p2[MMS_W8_TREE ? p & 1 : 0] = fma2(L.an2[p], u, p2[MMS_W8_TREE ? p & 1 : 0]);
            A.dac[p] = fma2(dt2, u, A.dac[p]);
            vb[p] = mul2(A.gad[p], dxv2);
            vc[p] = mul2(dy2, hv[k][p]);
        }
        {   // dx = dt*sum_n g*B, ddt = x*sum_n g*B - sum_n Aneg*u over both lanes of the channel
            const float2 q1 = add2(p1[0], p1[1]), q2 = add2(p2[0], p2[1]);
            const float s1 = q1.x + q1.y, s2 = q2.x + q2.y;
            const float v0 = dtv * s1, v1 = fmaf(xv, s1, -W8_LN2 * s2);
            float keep = L.h ? v1 : v0;
            keep += __shfl_xor_sync(0xffffffffu, L.h ? v0 : v1, 1);
            // prologue: d(logit) = ddt * d dt / d logit = ddt * (dt-lo)(lo+range-dt)/range
            if (pj.on && L.h) keep *= dt_slope(pj, dtv);
            if (L.dval) outq[(size_t)k * D] = from_f<E>(keep);
        }
        // dB|dC over the warp's 16 channels
        vb[0] = add2(vb[0], shfl2x(vb[2], 16));
        vb[1] = add2(vb[1], shfl2x(vb[3], 16));
        vc[0] = add2(vc[0], shfl2x(vc[2], 16));
        vc[1] = add2(vc[1], shfl2x(vc[3], 16));
        vb[0] = add2(vb[0], shfl2x(vb[1], 8));
        vc[0] = add2(vc[0], shfl2x(vc[1], 8));
        const float2 bc = add2(f2(vb[0].x, vc[0].x),
                               f2(__shfl_xor_sync(0xffffffffu, vb[0].y, 4),
                                  __shfl_xor_sync(0xffffffffu, vc[0].y, 4)));
        float keep = L.kbit ? bc.y : bc.x;
        keep += __shfl_xor_sync(0xffffffffu, L.kbit ? bc.x : bc.y, 2);
        sd[(i * W8_WARPS + L.warp) * 32 + L.kbit * 16 + 8 * L.h + L.tau] = keep;
    }
}

#ifndef MMS_BWD_W8_MINB
#define MMS_BWD_W8_MINB 4
#endif

// VEC: 16-byte cp.async staging (D % 4 == 0, aligned arrays). TMA: the
// stages are filled by TMA tile loads from the tensor maps in `maps` (one
// thread issues 6 loads per chunk; out-of-range steps, channels, states and
// the chunk-0 entry state arrive as zeros) and complete on per-stage
// mbarriers. E: storage type of x, dt, dy, dx, ddt (float, or bf16 with TMA).
template <bool VEC, bool TMA, bool PROJ, typename E>
__global__ void __launch_bounds__(W8_THREADS, MMS_BWD_W8_MINB)
bwd_kernel_w8(const E *__restrict__ x, const E *__restrict__ dt,
              const float *__restrict__ aneg, const float *__restrict__ Bm,
              const float *__restrict__ Cm, const E *__restrict__ dy,
              const float *__restrict__ ckpt, E *__restrict__ dx,
              E *__restrict__ ddt, float *__restrict__ part_bc,
              float *__restrict__ part_a, const float *__restrict__ seg_e,
              int T, int D, int N, int nblk, int cps, const __grid_constant__ W8Maps maps,
              Proj pj_in, uint32_t wait_limit, int skip_item)
{
    // the prologue is compiled in only where it is used
    Proj pj = pj_in;
    pj.on = PROJ;
    constexpr int DPB = W8_DPB;
    extern __shared__ __align__(128) float smem[];
    float *nat = smem;                                     // [W8_NAT][STAGEF]
    float *der = nat + W8_NAT * W8Shape::STAGEF;           // [DERF]
    float *sd = der + W8Shape::DERF;                       // [CH][WARPS][32]
    const uint32_t bars = smem_u32(sd + W8Shape::SDF);     // TMA: W8_NAT stage barriers

    const W8Lane L(aneg, D, N, pj);
    const int tid = L.tid;
    const int nchunk = (T + W8_CH - 1) / W8_CH;
    const size_t plane = (size_t)D * N;
    const size_t rowD = (size_t)L.b * T * D;
    const E *xb = x + rowD, *dtb = dt + rowD, *dyb = dy + rowD;
    const float *Bb = Bm + (size_t)L.b * T * N, *Cb = Cm + (size_t)L.b * T * N;
    const float *ckb = ckpt + (size_t)L.b * nchunk * plane;
    float *pbc = part_bc + ((size_t)L.b * nblk + blockIdx.x) * T * 2 * N;

    // inputs of chunk c and the checkpoint it starts from (zeros for c == 0)
    const int sg = blockIdx.z, nsg = gridDim.z;
    const int clo = sg * cps, chi = min((sg + 1) * cps, nchunk) - 1;
    const int nch = chi - clo + 1;

    // inputs of chunk c (item chi - c of this CTA) and the checkpoint it starts
    // from (zeros for c == 0); the test hook withholds item skip_item
    auto stage = [&](int buf, int c) {
        float *st = nat + buf * W8Shape::STAGEF;
        if constexpr (TMA) {
            if (tid == 0 && chi - c != skip_item) {
                const uint32_t bar = bars + 8 * buf, dst = smem_u32(st);
                using Q = W8Tile<E>;
                mbar_expect(bar, Q::BYTES);
                const int t0 = c * W8_CH;
                tma3(dst, &maps.x, L.d0, t0, L.b, bar);
                tma3(dst + 4 * Q::ARR, &maps.dt, L.d0, t0, L.b, bar);
                tma3(dst + 8 * Q::ARR, &maps.dy, L.d0, t0, L.b, bar);
                tma3(dst + 4 * Q::BC, &maps.B, 0, t0, L.b, bar);
                tma3(dst + 4 * (Q::BC + W8_CH * 16), &maps.C, 0, t0, L.b, bar);
                tma4(dst + 4 * Q::CK, &maps.ck, 0, L.d0, c - 1, L.b, bar);
            }
            return;
        }
        stage_tile<3, 2, DPB, 16, W8_CH, W8_THREADS, VEC>(st, xb, dtb, dyb, Bb, Cb, c * W8_CH,
                                                          min(W8_CH, T - c * W8_CH), L.d0, D, N, tid);
        float *cks = st + W8Shape::NATF;
        for (int k = tid; k < DPB * 4; k += W8_THREADS) {
            const int cc = k >> 2, q = k & 3;
            const bool ok = c >= 1 && L.d0 + cc < D && 4 * q < N;
            const float *src = ok ? ckb + (size_t)(c - 1) * plane + (size_t)(L.d0 + cc) * N + 4 * q : ckb;
            cp16(cks + cc * 16 + 4 * q, src, ok);
        }
    };

    W8Adj A;
#pragma unroll
    for (int p = 0; p < 4; ++p) A.gad[p] = A.anx[p] = A.dac[p] = f2(0.f, 0.f);
    if (sg + 1 < nsg) {                                    // carry from the later segments
        if (L.dval) L.load8(A.gad, seg_e + ((size_t)L.b * nsg + sg) * plane + (size_t)L.d * N, N);
#pragma unroll
        for (int p = 0; p < 4; ++p) A.anx[p] = f2(1.f, 1.f);
    }

    if constexpr (TMA) {
        if (tid == 0) {
            for (int s2 = 0; s2 < W8_NAT; ++s2) mbar_init(bars + 8 * s2, 1);
            asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        }
        __syncthreads();
    }
    stage(0, chi);
    cp_commit();
    if (nch > 1) stage(1, chi - 1);
    cp_commit();

    for (int it = 0; it < nch; ++it) {
        const int c = chi - it;
        if constexpr (TMA) {
            const bool ok = w8_wait(bars + 8 * (it % W8_NAT), (it / W8_NAT) & 1, wait_limit);
            if (__syncthreads_or(!ok)) {
                // a stage never arrived: leave together, after the copies still in flight
                if (tid == 0) {
                    for (int k = it; k < min(it + 2, nch); ++k)
                        if (k != skip_item) w8_wait(bars + 8 * (k % W8_NAT), (k / W8_NAT) & 1, wait_limit);
                    atomicOr(&g_w8_timeout, 1u);
                }
                return;
            }
        } else {
            cp_wait<1>();
            __syncthreads();                               // chunk c staged; chunk c+1 walked
        }
        if (it > 0) {                                      // dB|dC partial of chunk c+1
            const int t0p = (c + 1) * W8_CH, nvp = min(W8_CH, T - t0p);
            for (int p = tid; p < W8_CH * 32; p += W8_THREADS) {
                const int i = p >> 5, j = p & 31;
                const int kind = j >> 4, n = j & 15;
                if (i < nvp && n < N) {
                    const float *r = sd + i * W8_WARPS * 32 + j;
                    pbc[(size_t)(t0p + i) * 2 * N + kind * N + n] = (r[0] + r[32]) + (r[64] + r[96]);
                }
            }
        }
        const float *st = nat + (it % W8_NAT) * W8Shape::STAGEF;
        w8_rewrite<TMA, E>(st, der, tid, pj);
        float2 hA[4];
        L.load8(hA, st + (TMA ? W8Tile<E>::CK : W8Shape::NATF) + L.c * 16, 16);
        if (c - 2 >= clo) {
            // the stage's previous chunk was read before the barrier above
            if (TMA && tid == 0) fence_async_smem();
            stage((it + 2) % W8_NAT, c - 2);
        }
        cp_commit();
        __syncthreads();                                   // der ready, sd free

        const W8View v(der, L);
        const int t0 = c * W8_CH;
        const int nv = min(W8_CH, T - t0);
        E *outb = (L.h ? ddt : dx) + rowD + (size_t)t0 * D + L.d;
        // later group (steps 4..7) from the state after step 3, then the first group
        if (nv > 4) {
            float2 h4[4] = {hA[0], hA[1], hA[2], hA[3]};
            w8_advance(h4, L, v, 0);
            if (nv == W8_CH) w8_walk<true, E>(v, h4, L, A, 1, nv, outb + (size_t)4 * D, D, sd, pj);
            else w8_walk<false, E>(v, h4, L, A, 1, nv, outb + (size_t)4 * D, D, sd, pj);
            w8_walk<true, E>(v, hA, L, A, 0, nv, outb, D, sd, pj);
        } else {
            w8_walk<false, E>(v, hA, L, A, 0, nv, outb, D, sd, pj);
        }
    }
    cp_wait<0>();
    __syncthreads();
    {
        const int t0p = clo * W8_CH, nvp = min(W8_CH, T - t0p);
        for (int p = tid; p < W8_CH * 32; p += W8_THREADS) {
            const int i = p >> 5, j = p & 31;
            const int kind = j >> 4, n = j & 15;
            if (i < nvp && n < N) {
                const float *r = sd + i * W8_WARPS * 32 + j;
                pbc[(size_t)(t0p + i) * 2 * N + kind * N + n] = (r[0] + r[32]) + (r[64] + r[96]);
            }
        }
    }
    if (L.dval) {
        float *pa = part_a + (((size_t)L.b * nsg + sg) * D + L.d) * N;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int s0 = 8 * L.h + ((2 * p) ^ L.tau), s1 = 8 * L.h + ((2 * p + 1) ^ L.tau);
            if (s0 < N) pa[s0] = -A.dac[p].x;
            if (s1 < N) pa[s1] = -A.dac[p].y;
        }
    }
}

}  // namespace

bool bwd_w8_applies(int N, int K) { return K == W8_CH && w8_shape(N, K); }

#ifndef MMS_BWD_TMA
#define MMS_BWD_TMA 1
#endif

namespace {

bool build_maps(const BwdArgs &a, W8Maps *m)
{
    const auto fn = tma_encoder();
    if (!fn || !tma_context()) return false;
    const cuuint64_t dX[3] = {(cuuint64_t)a.D, (cuuint64_t)a.T, (cuuint64_t)a.Bt};
    const cuuint32_t bX[3] = {W8_DPB, W8_CH, 1};
    const cuuint64_t dB[3] = {(cuuint64_t)a.N, (cuuint64_t)a.T, (cuuint64_t)a.Bt};
    const cuuint32_t bB[3] = {16, W8_CH, 1};
    const int nchunk = (a.T + W8_CH - 1) / W8_CH;
    const cuuint64_t dK[4] = {(cuuint64_t)a.N, (cuuint64_t)a.D, (cuuint64_t)nchunk, (cuuint64_t)a.Bt};
    const cuuint32_t bK[4] = {16, W8_DPB, 1, 1};
    const int ex = a.bf16 ? 2 : 4;
    return tma_encode(fn, &m->x, a.x, 3, dX, bX, ex) && tma_encode(fn, &m->dt, a.dt, 3, dX, bX, ex) &&
           tma_encode(fn, &m->dy, a.dy, 3, dX, bX, ex) && tma_encode(fn, &m->B, a.B, 3, dB, bB) &&
           tma_encode(fn, &m->C, a.C, 3, dB, bB) && tma_encode(fn, &m->ck, a.ckpt, 4, dK, bK);
}

template <bool VEC, bool TMA, bool PROJ, typename E = float>
cudaError_t launch_w8p(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                       int nblk, SegPlan sp, const W8Maps &maps, cudaStream_t stream)
{
    const size_t smem = TMA ? W8Shape::SMEM_TMA : W8Shape::SMEM;
    cudaError_t e = smem_opt_in<bwd_kernel_w8<VEC, TMA, PROJ, E>>(smem);
    if (e != cudaSuccess) return e;
    dim3 grid((a.D + W8_DPB - 1) / W8_DPB, a.Bt, sp.S);
    auto cE = [](const float *p) { return reinterpret_cast<const E *>(p); };
    auto mE = [](float *p) { return reinterpret_cast<E *>(p); };
    bwd_kernel_w8<VEC, TMA, PROJ, E><<<grid, W8_THREADS, smem, stream>>>(
        cE(a.x), cE(a.dt), a.aneg, a.B, a.C, cE(a.dy), a.ckpt, mE(a.dx), mE(a.ddt), part_bc, part_a,
        seg_e, a.T, a.D, a.N, nblk, sp.cps, maps, a.proj, tma_wait_limit(), tma_skip_item());
    return cudaGetLastError();
}

template <bool VEC, bool TMA>
cudaError_t launch_w8(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                      int nblk, SegPlan sp, const W8Maps &maps, cudaStream_t stream)
{
    return a.proj.on ? launch_w8p<VEC, TMA, true>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream)
                     : launch_w8p<VEC, TMA, false>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream);
}

}  // namespace

cudaError_t launch_bwd_w8(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                          int nblk, SegPlan sp, cudaStream_t stream)
{
    W8Maps maps;
    memset(&maps, 0, sizeof(maps));
    if (a.bf16) {
        // bf16 channel arrays: TMA staging only (D % 8 == 0, aligned arrays)
        if (a.D % 8 != 0 || a.proj.on || !vec_ok(a.D, a.x, a.dt, a.dy) ||
            !vec_ok(a.D, a.dx, a.ddt) || !build_maps(a, &maps))
            return cudaErrorInvalidValue;
        return launch_w8p<true, true, false, __nv_bfloat16>(a, part_bc, part_a, seg_e, nblk, sp,
                                                             maps, stream);
    }
    if (!vec_ok(a.D, a.x, a.dt, a.dy))
        return launch_w8<false, false>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream);
    if (MMS_BWD_TMA && build_maps(a, &maps))
        return launch_w8<true, true>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream);
    return launch_w8<true, false>(a, part_bc, part_a, seg_e, nblk, sp, maps, stream);
}

int w8_take_timeout()
{
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_w8_timeout, sizeof(v)) != cudaSuccess) return -1;
    if (v) {
        const unsigned int z = 0;
        cudaMemcpyToSymbol(g_w8_timeout, &z, sizeof(z));
    }
    return v ? 1 : 0;
}

}  // namespace mms
