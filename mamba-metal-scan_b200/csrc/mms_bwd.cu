// Backward selective scan for sm_100a.
//
// Math (reference mamba_metal/scan.py:26-34, kernel ssm_bwd at :132-261):
//     g_t    = dy_t*C_t + dA_{t+1}*g_{t+1}
//     dx_t   = dt_t * sum_n g_tn*B_tn
//     ddt_t  = x_t * sum_n g_tn*B_tn - sum_n Aneg_n*g_tn*(dA_tn*h_{t-1,n})
//     dAneg  = -sum_{b,t} dt_t*g_tn*(dA_tn*h_{t-1,n})
//     dB_tn  = sum_d g_tdn*dt_td*x_td          dC_tn = sum_d dy_td*h_tdn
//
// Work decomposition is the forward's: a thread owns 4 states of one (b, d)
// channel, G lanes share a channel, a CTA covers BWD_WARPS*32/G channels of
// one batch row and walks the whole sequence from the last chunk to the first.
//
// Recompute without a (B,K,D,N) scratch and with two exps per element:
//   * a chunk (K steps, bounded by the forward's checkpoints) is split into
//     segments of SEG = GRP*SLOTS steps; the state entering each segment comes
//     from the checkpoint or, for chunks longer than SEG, from a pre-pass that
//     stores segment-start states in the workspace;
//   * a segment is recomputed once, keeping only the state entering every
//     GRP-step group (SLOTS float4 per thread in shared memory);
//   * the walk visits groups last to first; each group is rebuilt from its
//     slot with GRP exps per state, and those decays and states stay in
//     registers for the group's backward steps (dA_t for dA_t*h_{t-1} and,
//     carried one step, dA_{t+1} for the adjoint).
//
// Reductions, all deterministic (fixed order, no atomics):
//   * sum over n (dx, ddt): transposed butterfly across the channel's G lanes;
//   * sum over d (dB, dC): transposed butterfly across a warp's channels, then
//     the CTA's warps in shared memory once per group, written as one partial
//     per CTA; reduce_bc_kernel sums the CTAs of a batch row;
//   * dAneg: per-thread register accumulation over the whole walk, one partial
//     per batch row; reduce_a_kernel sums the rows.
#include "mms_common.cuh"
#include "mms_kernels.h"

namespace mms {

constexpr int BWD_WARPS = 8;
constexpr int BWD_THREADS = BWD_WARPS * 32;
constexpr int GRP = 4;                    // steps rebuilt per group
constexpr int SLOTS = 16;                 // groups per segment
constexpr int SEG = GRP * SLOTS;          // steps per segment

template <int G>
constexpr int log2_const() { return G <= 1 ? 0 : 1 + log2_const<G / 2>(); }

template <int G>
struct BwdShape {
    static constexpr int DPW = 32 / G;                 // channels per warp
    static constexpr int DPB = BWD_WARPS * DPW;        // channels per CTA
    static constexpr int NPAD = 4 * G;
    static constexpr int NV2 = 2 * NPAD;               // dB|dC values per step per warp
    static constexpr int LEV_D = log2_const<DPW>();    // butterfly levels across channels
    static constexpr int NLEFT_D = (8 >> LEV_D) > 0 ? (8 >> LEV_D) : 1;
    static constexpr int DUP_D = G >= 4 ? 0 : (3 & ~(G - 1));   // lanes holding copies
    static constexpr size_t SMEM = (size_t)SLOTS * BWD_THREADS * sizeof(float4)
                                 + (size_t)2 * GRP * BWD_WARPS * NV2 * sizeof(float);
};

// h <- recurrence over steps [tb, te), nothing stored.
__device__ __forceinline__ void advance(float (&h)[4], const float (&an2)[4],
                                        const float *dtp, const float *xp, const float *Bp,
                                        int tb, int te, int D, int N, bool dval, bool act)
{
#pragma unroll 4
    for (int t = tb; t < te; ++t) {
        float dtv = 0.f, xv = 0.f;
        float4 Bv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (dval) {
            dtv = __ldg(dtp + (size_t)t * D);
            xv = __ldg(xp + (size_t)t * D);
        }
        if (act) Bv = ld4(Bp + (size_t)t * N);
        const float ml = -dtv, bx = dtv * xv;
#pragma unroll
        for (int s = 0; s < 4; ++s)
            h[s] = fmaf(ex2(ml * an2[s]), h[s], bx * comp(Bv, s));
    }
}

template <int G>
__global__ void __launch_bounds__(BWD_THREADS, 2)
bwd_kernel(const float *__restrict__ x, const float *__restrict__ dt,
           const float *__restrict__ aneg, const float *__restrict__ Bm,
           const float *__restrict__ Cm, const float *__restrict__ dy,
           const float *__restrict__ ckpt, float *__restrict__ dx,
           float *__restrict__ ddt, float *__restrict__ part_bc,
           float *__restrict__ part_a, float *subck,
           int T, int D, int N, int K, int nblk, int nsegk)
{
    using S = BwdShape<G>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float4 *slots = reinterpret_cast<float4 *>(smem_raw);                  // [SLOTS][threads]
    float *red = reinterpret_cast<float *>(slots + SLOTS * BWD_THREADS);  // [2][GRP][warps][NV2]

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int g = lane & (G - 1);
    const int d = (blockIdx.x * BWD_WARPS + warp) * S::DPW + lane / G;
    const int b = blockIdx.y;
    const bool dval = d < D;
    const bool act = dval && (4 * g < N);
    const int nchunk = (T + K - 1) / K;

    float an[4] = {0.f, 0.f, 0.f, 0.f}, an2[4];
    if (act) {
        const float4 a4 = ld4(aneg + (size_t)d * N + 4 * g);
        an[0] = a4.x; an[1] = a4.y; an[2] = a4.z; an[3] = a4.w;
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) an2[s] = an[s] * MMS_LOG2E;

    const size_t rowD = (size_t)b * T * D + d;
    const float *xp = x + rowD, *dtp = dt + rowD, *dyp = dy + rowD;
    float *dxp = dx + rowD, *ddtp = ddt + rowD;
    const float *Bp = Bm + (size_t)b * T * N + 4 * g;
    const float *Cp = Cm + (size_t)b * T * N + 4 * g;
    const size_t chan = (size_t)d * N + 4 * g;          // (d, 4g) inside a (D, N) plane
    const size_t plane = (size_t)D * N;
    float *pbc = part_bc + ((size_t)b * nblk + blockIdx.x) * T * (2 * N);

    float gad[4] = {0.f, 0.f, 0.f, 0.f};    // adjoint g, carried across steps
    float anx[4] = {0.f, 0.f, 0.f, 0.f};    // dA_{t+1}; zero past the end
    float dac[4] = {0.f, 0.f, 0.f, 0.f};    // sum_t dt*g*dA*h_{t-1}
    int buf = 0;

    for (int c = nchunk - 1; c >= 0; --c) {
        const int t0 = c * K, t1 = min(t0 + K, T);
        const int nseg = (t1 - t0 + SEG - 1) / SEG;
        float hc[4] = {0.f, 0.f, 0.f, 0.f};
        if (c > 0 && act) {
            const float4 v = ld4(ckpt + ((size_t)b * nchunk + (c - 1)) * plane + chan);
            hc[0] = v.x; hc[1] = v.y; hc[2] = v.z; hc[3] = v.w;
        }
        if (nseg > 1) {                      // segment-start states of a long chunk
            float hq[4] = {hc[0], hc[1], hc[2], hc[3]};
            for (int q = 1; q < nseg; ++q) {
                advance(hq, an2, dtp, xp, Bp, t0 + (q - 1) * SEG, t0 + q * SEG, D, N, dval, act);
                if (act) st4(subck + ((size_t)b * nsegk + q) * plane + chan,
                             make_float4(hq[0], hq[1], hq[2], hq[3]));
            }
        }
        for (int sg = nseg - 1; sg >= 0; --sg) {
            const int u0 = t0 + sg * SEG, u1 = min(u0 + SEG, t1);
            const int ngrp = (u1 - u0 + GRP - 1) / GRP;
            float hs[4] = {hc[0], hc[1], hc[2], hc[3]};
            if (sg > 0) {
                // written above by this same thread: coherent plain load
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (act) v = *reinterpret_cast<const float4 *>(
                    subck + ((size_t)b * nsegk + sg) * plane + chan);
                hs[0] = v.x; hs[1] = v.y; hs[2] = v.z; hs[3] = v.w;
            }
            // Recompute the segment, keeping the state that enters each group.
            for (int j = 0; j < ngrp; ++j) {
                slots[j * BWD_THREADS + tid] = make_float4(hs[0], hs[1], hs[2], hs[3]);
                if (j + 1 < ngrp)
                    advance(hs, an2, dtp, xp, Bp, u0 + j * GRP, u0 + (j + 1) * GRP, D, N, dval, act);
            }
            // Walk the groups backwards.
            for (int j = ngrp - 1; j >= 0; --j) {
                const int v0 = u0 + j * GRP;
                const int nv = min(GRP, u1 - v0);
                const float4 hb4 = slots[j * BWD_THREADS + tid];
                const float hb[4] = {hb4.x, hb4.y, hb4.z, hb4.w};
                float av[GRP][4], hv[GRP][4], dtv[GRP], xv[GRP], dyv[GRP];
                float4 Bv[GRP], Cv[GRP];
#pragma unroll
                for (int i = 0; i < GRP; ++i) {
                    const int t = v0 + i;
                    dtv[i] = 0.f; xv[i] = 0.f; dyv[i] = 0.f;
                    Bv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    Cv[i] = Bv[i];
                    if (i < nv && dval) {
                        dtv[i] = __ldg(dtp + (size_t)t * D);
                        xv[i] = __ldg(xp + (size_t)t * D);
                        dyv[i] = __ldg(dyp + (size_t)t * D);
                    }
                    if (i < nv && act) {
                        Bv[i] = ld4(Bp + (size_t)t * N);
                        Cv[i] = ld4(Cp + (size_t)t * N);
                    }
                    const float ml = -dtv[i], bx = dtv[i] * xv[i];
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        av[i][s] = ex2(ml * an2[s]);
                        hv[i][s] = fmaf(av[i][s], i ? hv[i - 1][s] : hb[s], bx * comp(Bv[i], s));
                    }
                }
#pragma unroll
                for (int i = GRP - 1; i >= 0; --i) {
                    if (i < nv) {
                        const int t = v0 + i;
                        const float dxv = dtv[i] * xv[i];
                        float p1 = 0.f, p2 = 0.f, vbc[8];
#pragma unroll
                        for (int s = 0; s < 4; ++s) {
                            float a1 = anx[s];
                            if (i + 1 < GRP && i + 1 < nv) a1 = av[i + 1 < GRP ? i + 1 : i][s];
                            gad[s] = fmaf(a1, gad[s], dyv[i] * comp(Cv[i], s));
                            const float hp = i ? hv[i > 0 ? i - 1 : 0][s] : hb[s];
                            const float u = gad[s] * (av[i][s] * hp);
                            p1 = fmaf(gad[s], comp(Bv[i], s), p1);
                            p2 = fmaf(an[s], u, p2);
                            dac[s] = fmaf(dtv[i], u, dac[s]);
                            vbc[s] = gad[s] * dxv;
                            vbc[4 + s] = dyv[i] * hv[i][s];
                        }
                        // dx, ddt: sum over the channel's lanes
                        float vn[2] = {dtv[i] * p1, fmaf(xv[i], p1, -p2)};
                        if constexpr (G == 1) {
                            if (dval) { dxp[(size_t)t * D] = vn[0]; ddtp[(size_t)t * D] = vn[1]; }
                        } else {
                            int fn;
                            transposed_reduce<2, G / 2, 1>(vn, lane, fn);
                            if (dval && (g & (G / 2 - 1)) == 0) {
                                if (fn == 0) dxp[(size_t)t * D] = vn[0];
                                else ddtp[(size_t)t * D] = vn[0];
                            }
                        }
                        // dB, dC: sum over the warp's channels
                        int fb;
                        transposed_reduce<8, 16, G>(vbc, lane, fb);
                        if ((lane & S::DUP_D) == 0) {
                            float *r = red + ((buf * GRP + i) * BWD_WARPS + warp) * S::NV2;
#pragma unroll
                            for (int k = 0; k < S::NLEFT_D; ++k) {
                                const int idx = fb + k;
                                r[idx < 4 ? 4 * g + idx : S::NPAD + 4 * g + idx - 4] = vbc[k];
                            }
                        }
                    }
                }
#pragma unroll
                for (int s = 0; s < 4; ++s) anx[s] = av[0][s];
                __syncthreads();
                // This CTA's share of dB|dC for the group's steps.
                const int twoN = 2 * N;
                for (int o = tid; o < nv * twoN; o += BWD_THREADS) {
                    const int i = o / twoN, jj = o - i * twoN;
                    const int pos = jj < N ? jj : S::NPAD + jj - N;
                    const float *r = red + (buf * GRP + i) * BWD_WARPS * S::NV2 + pos;
                    float sum = 0.f;
#pragma unroll
                    for (int w = 0; w < BWD_WARPS; ++w) sum += r[w * S::NV2];
                    pbc[(size_t)(v0 + i) * twoN + jj] = sum;
                }
                buf ^= 1;
            }
        }
    }
    if (act) {
        float *pa = part_a + (size_t)b * plane + chan;
        st4(pa, make_float4(-dac[0], -dac[1], -dac[2], -dac[3]));
    }
}

// dB|dC = sum over the nblk CTA partials of each batch row (fixed order).
__global__ void reduce_bc_kernel(const float *__restrict__ part, float *__restrict__ dB,
                                 float *__restrict__ dC, int Bt, int T, int N, int nblk)
{
    const size_t per_b = (size_t)T * 2 * N;
    const size_t total = (size_t)Bt * per_b;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t b = idx / per_b, r = idx - b * per_b;
        const float *p = part + b * nblk * per_b + r;
        float s = 0.f;
        for (int k = 0; k < nblk; ++k) s += p[(size_t)k * per_b];
        const size_t t = r / (2 * N);
        const int j = (int)(r - t * 2 * N);
        if (j < N) dB[(b * T + t) * N + j] = s;
        else dC[(b * T + t) * N + (j - N)] = s;
    }
}

// dAneg = sum over batch rows (fixed order).
__global__ void reduce_a_kernel(const float *__restrict__ part, float *__restrict__ daneg,
                                int Bt, size_t DN)
{
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < DN;
         idx += (size_t)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int b = 0; b < Bt; ++b) s += part[(size_t)b * DN + idx];
        daneg[idx] = s;
    }
}

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

static int dpb_for(int G)
{
    return BWD_WARPS * 32 / G;
}

BwdWorkspace bwd_workspace_layout(int Bt, int T, int D, int N, int K)
{
    BwdWorkspace w{};
    const int G = groups_for(N);
    const int dpb = dpb_for(G);
    w.nblk = (D + dpb - 1) / dpb;
    const int kk = K < T ? K : T;
    w.nseg = (kk + SEG - 1) / SEG;
    size_t off = 0;
    w.part_bc = off;
    off = align256(off + (size_t)Bt * w.nblk * T * 2 * N * sizeof(float));
    w.part_a = off;
    off = align256(off + (size_t)Bt * D * N * sizeof(float));
    w.subck = off;
    if (w.nseg > 1) off = align256(off + (size_t)Bt * w.nseg * D * N * sizeof(float));
    w.total = off;
    return w;
}

template <int G>
static cudaError_t launch_bwd_g(const BwdArgs &a, const BwdWorkspace &w, cudaStream_t stream)
{
    using S = BwdShape<G>;
    cudaError_t e = cudaFuncSetAttribute(bwd_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)S::SMEM);
    if (e != cudaSuccess) return e;
    char *ws = static_cast<char *>(a.workspace);
    float *part_bc = reinterpret_cast<float *>(ws + w.part_bc);
    float *part_a = reinterpret_cast<float *>(ws + w.part_a);
    float *subck = reinterpret_cast<float *>(ws + w.subck);
    dim3 grid(w.nblk, a.Bt);
    bwd_kernel<G><<<grid, BWD_THREADS, S::SMEM, stream>>>(
        a.x, a.dt, a.aneg, a.B, a.C, a.dy, a.ckpt, a.dx, a.ddt, part_bc, part_a, subck,
        a.T, a.D, a.N, a.K, w.nblk, w.nseg);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t nbc = (size_t)a.Bt * a.T * 2 * a.N;
    const int rb = (int)((nbc + 255) / 256 < 148 * 16 ? (nbc + 255) / 256 : 148 * 16);
    reduce_bc_kernel<<<rb, 256, 0, stream>>>(part_bc, a.dB, a.dC, a.Bt, a.T, a.N, w.nblk);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t dn = (size_t)a.D * a.N;
    const int ra = (int)((dn + 255) / 256 < 148 * 16 ? (dn + 255) / 256 : 148 * 16);
    reduce_a_kernel<<<ra, 256, 0, stream>>>(part_a, a.daneg, a.Bt, dn);
    return cudaGetLastError();
}

cudaError_t launch_bwd(const BwdArgs &a, cudaStream_t stream)
{
    const BwdWorkspace w = bwd_workspace_layout(a.Bt, a.T, a.D, a.N, a.K);
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
