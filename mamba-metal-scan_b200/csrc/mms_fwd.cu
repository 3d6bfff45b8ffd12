// Forward selective scan for sm_100a.
//
// Math (reference mamba_metal/scan.py:13-15, kernel ssm_fwd at :78-127):
//     dA = exp(-dt*Aneg);  h_t = dA*h_{t-1} + dt*B_t*x_t;  y_t = sum_n C_tn*h_tn
// with h checkpointed at the end of every K-step chunk and at t = T-1.
//
// Work decomposition: one thread owns 4 consecutive states (a "state group")
// of one (b, d) channel; G = ceil(N/4) rounded up to a power of two lanes
// share a channel, so a warp covers 32/G channels and a CTA of FWD_WARPS
// warps covers FWD_WARPS*32/G consecutive channels of one batch row. Compared
// with one thread per (b, d), this gives G times more threads in flight (the
// (b,d) count alone cannot fill 148 SMs) and keeps only 4 states, 4 decay
// rates in registers.
//
// y_t needs the sum over the G lanes of a channel. Instead of reducing every
// step, each lane keeps its partial for G consecutive steps and one
// transposed butterfly (G-1 shuffles) leaves lane g holding the full y for
// step t0+g, which it stores.
#include "mms_common.cuh"
#include "mms_kernels.h"

namespace mms {

constexpr int FWD_WARPS = 4;

template <int G>
__global__ void __launch_bounds__(FWD_WARPS * 32)
fwd_kernel(const float *__restrict__ x, const float *__restrict__ dt,
           const float *__restrict__ aneg, const float *__restrict__ Bm,
           const float *__restrict__ Cm, float *__restrict__ y,
           float *__restrict__ ckpt, int T, int D, int N, int K)
{
    constexpr int DPW = 32 / G;                      // channels per warp
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane & (G - 1);
    const int d = (blockIdx.x * FWD_WARPS + warp) * DPW + lane / G;
    const int b = blockIdx.y;
    const bool dval = d < D;
    const bool act = dval && (4 * g < N);           // masked groups hold zeros
    const int nchunk = (T + K - 1) / K;

    // Decay rates pre-scaled by log2(e): dA = 2^(-dt * an).
    float an[4] = {0.f, 0.f, 0.f, 0.f};
    if (act) {
        const float4 a4 = ld4(aneg + (size_t)d * N + 4 * g);
        an[0] = a4.x * MMS_LOG2E; an[1] = a4.y * MMS_LOG2E;
        an[2] = a4.z * MMS_LOG2E; an[3] = a4.w * MMS_LOG2E;
    }
    float h[4] = {0.f, 0.f, 0.f, 0.f};

    const float *xb = x + (size_t)b * T * D + d;
    const float *dtb = dt + (size_t)b * T * D + d;
    const float *Bb = Bm + (size_t)b * T * N + 4 * g;
    const float *Cb = Cm + (size_t)b * T * N + 4 * g;
    float *yb = y + (size_t)b * T * D + d;
    float *ckb = ckpt + (size_t)b * nchunk * D * N + (size_t)d * N + 4 * g;

    int next_ck = min(K, T) - 1;                     // step whose state is checkpointed next
    int chunk = 0;

    for (int t0 = 0; t0 < T; t0 += G) {
        float yp[G];
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int t = t0 + j;
            const bool tv = t < T;
            float dtv = 0.f, xv = 0.f;
            float4 Bv = make_float4(0.f, 0.f, 0.f, 0.f), Cv = Bv;
            if (tv && dval) {
                dtv = __ldg(dtb + (size_t)t * D);
                xv = __ldg(xb + (size_t)t * D);
            }
            if (tv && act) {
                Bv = ld4(Bb + (size_t)t * N);
                Cv = ld4(Cb + (size_t)t * N);
            }
            // Padding steps (t >= T) have dt = 0: dA = 1, b = 0, h unchanged.
            const float ml = -dtv;
            const float bx = dtv * xv;
            float acc = 0.f;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const float a = ex2(ml * an[s]);
                h[s] = fmaf(a, h[s], bx * comp(Bv, s));
                acc = fmaf(comp(Cv, s), h[s], acc);
            }
            yp[j] = acc;
            if (t == next_ck) {                       // uniform across the CTA
                if (act) st4(ckb + (size_t)chunk * D * N, make_float4(h[0], h[1], h[2], h[3]));
                ++chunk;
                next_ck = min(next_ck + K, T - 1);
            }
        }
        int first = 0;
        if constexpr (G > 1) transposed_reduce<G, G / 2, 1>(yp, lane, first);
        const int t = t0 + first;
        if (dval && t < T) yb[(size_t)t * D] = yp[0];
    }
}

template <int G>
static cudaError_t launch_fwd_g(const FwdArgs &a, cudaStream_t stream)
{
    constexpr int DPB = FWD_WARPS * 32 / G;          // channels per CTA
    dim3 grid((a.D + DPB - 1) / DPB, a.Bt);
    fwd_kernel<G><<<grid, FWD_WARPS * 32, 0, stream>>>(
        a.x, a.dt, a.aneg, a.B, a.C, a.y, a.ckpt, a.T, a.D, a.N, a.K);
    return cudaGetLastError();
}

cudaError_t launch_fwd(const FwdArgs &a, cudaStream_t stream)
{
    switch (groups_for(a.N)) {
    case 1: return launch_fwd_g<1>(a, stream);
    case 2: return launch_fwd_g<2>(a, stream);
    case 4: return launch_fwd_g<4>(a, stream);
    case 8: return launch_fwd_g<8>(a, stream);
    case 16: return launch_fwd_g<16>(a, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace mms
