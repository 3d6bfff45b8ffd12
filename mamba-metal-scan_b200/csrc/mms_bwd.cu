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
// Memory: every pass reads its time steps from shared-memory tiles of one
// group (x, dt, dy, B, C for the CTA's channels) staged by cp.async two tiles
// ahead along the exact order the passes consume them (WorkCursor).
//
// Reductions, all deterministic (fixed order, no atomics):
//   * sum over n (dx, ddt): per-lane partials in shared memory, finished once
//     per group by one thread per (t, d), which also writes dx/ddt coalesced;
//   * sum over d (dB, dC): transposed butterfly across a warp's channels, the
//     CTA's warps summed in shared memory once per group and written as one
//     partial per CTA; reduce_bc_kernel adds the CTAs of a batch row;
//   * dAneg: per-thread register sums over the whole walk, one partial per
//     batch row; reduce_a_kernel adds the rows.
#include "mms_common.cuh"
#include "mms_kernels.h"
#include "mms_stage.cuh"

namespace mms {

constexpr int BWD_THREADS = 256;
constexpr int BWD_WARPS = BWD_THREADS / 32;
constexpr int GRP = 8;                    // steps rebuilt per group
constexpr int SLOTS = 8;                  // groups per segment
constexpr int SEG = GRP * SLOTS;          // steps per segment
constexpr int BWD_STAGES = 3;

template <int G>
constexpr int log2_const() { return G <= 1 ? 0 : 1 + log2_const<G / 2>(); }

template <int G>
struct BwdShape {
    static constexpr int DPB = BWD_THREADS / G;            // channels per CTA
    static constexpr int DPW = 32 / G;                     // channels per warp
    static constexpr int NPAD = 4 * G;
    static constexpr int ROWF = 3 * DPB + 2 * NPAD;        // x, dt, dy, B, C per step
    static constexpr int NV2 = 2 * NPAD;                   // dB|dC values per step per warp
    static constexpr int LEV_D = log2_const<DPW>();
    static constexpr int NLEFT_D = (8 >> LEV_D) > 0 ? (8 >> LEV_D) : 1;
    static constexpr int DUP_D = G >= 4 ? 0 : (3 & ~(G - 1));   // lanes holding copies
    static constexpr size_t TILES = (size_t)BWD_STAGES * GRP * ROWF;       // floats
    static constexpr size_t SLOTF = (size_t)SLOTS * BWD_THREADS * 4;       // floats
    static constexpr size_t SNF = (size_t)GRP * DPB * G * 2;               // floats
    static constexpr size_t SDF = (size_t)GRP * BWD_WARPS * NV2;           // floats
    static constexpr size_t SMEM = sizeof(float) * (TILES + SLOTF + SNF + SDF);
};

// The order in which one CTA consumes GRP-step groups of its batch row:
// chunks last to first; in each chunk an optional pre-pass (P) that stores
// segment-start states, then per segment (last to first) the recompute (R,
// groups forward, all but the last) and the walk (W, groups backward).
struct WorkCursor {
    int c, phase, sg, j;       // phase 0 = P, 1 = R, 2 = W; c < 0 when done
    int t0c, t1c, nseg, u0, u1, ngrp;
    int T, K;

    __device__ void start(int T_, int K_) {
        T = T_; K = K_;
        enter_chunk((T + K - 1) / K - 1);
    }
    __device__ void enter_chunk(int c_) {
        c = c_;
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

// h <- recurrence over the GRP steps of a staged tile (padding steps are zeros).
template <int DPB, int NPAD, int ROWF>
__device__ __forceinline__ void advance_tile(float (&h)[4], const float (&an2)[4],
                                             const float *tile, int c, int g)
{
#pragma unroll
    for (int i = 0; i < GRP; ++i) {
        const float *row = tile + i * ROWF;
        const float xv = row[c], dtv = row[DPB + c];
        const float4 Bv = *reinterpret_cast<const float4 *>(row + 3 * DPB + 4 * g);
        const float ml = -dtv, bx = dtv * xv;
#pragma unroll
        for (int s = 0; s < 4; ++s) h[s] = fmaf(ex2(ml * an2[s]), h[s], bx * comp(Bv, s));
    }
}

template <int G, bool VEC>
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
    constexpr int DPB = S::DPB, NPAD = S::NPAD, ROWF = S::ROWF, NV2 = S::NV2;
    extern __shared__ __align__(16) float smem[];
    float *tiles = smem;                                             // [STAGES][GRP][ROWF]
    float4 *slots = reinterpret_cast<float4 *>(smem + S::TILES);    // [SLOTS][THREADS]
    float *sn = smem + S::TILES + S::SLOTF;                          // [GRP][DPB][G][2]
    float *sd = sn + S::SNF;                                         // [GRP][WARPS][NV2]

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int g = tid & (G - 1);
    const int c = tid / G;
    const int d0 = blockIdx.x * DPB;
    const int d = d0 + c;
    const int b = blockIdx.y;
    const bool act = d < D && (4 * g < N);
    const int nchunk = (T + K - 1) / K;
    const int twoN = 2 * N;

    float an[4] = {0.f, 0.f, 0.f, 0.f}, an2[4];
    if (act) {
        const float4 a4 = ld4(aneg + (size_t)d * N + 4 * g);
        an[0] = a4.x; an[1] = a4.y; an[2] = a4.z; an[3] = a4.w;
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) an2[s] = an[s] * MMS_LOG2E;

    const size_t plane = (size_t)D * N;
    const size_t chan = (size_t)d * N + 4 * g;
    const float *xb = x + (size_t)b * T * D, *dtb = dt + (size_t)b * T * D;
    const float *dyb = dy + (size_t)b * T * D;
    const float *Bb = Bm + (size_t)b * T * N, *Cb = Cm + (size_t)b * T * N;
    float *dxb = dx + (size_t)b * T * D;
    float *ddtb = ddt + (size_t)b * T * D;
    float *pbc = part_bc + ((size_t)b * nblk + blockIdx.x) * T * twoN;

    WorkCursor cur, pre;
    cur.start(T, K);
    pre = cur;
#pragma unroll
    for (int s = 0; s < BWD_STAGES - 1; ++s) {
        if (!pre.done()) {
            stage_tile<3, 2, DPB, NPAD, GRP, BWD_THREADS, VEC>(
                tiles + s * GRP * ROWF, xb, dtb, dyb, Bb, Cb, pre.tstart(), pre.nvalid(), d0, D, N, tid);
            pre.advance();
        }
        cp_commit();
    }

    float gad[4] = {0.f, 0.f, 0.f, 0.f};    // adjoint g, carried across steps
    float anx[4] = {0.f, 0.f, 0.f, 0.f};    // dA_{t+1}; zero past the end
    float dac[4] = {0.f, 0.f, 0.f, 0.f};    // sum_t dt*g*dA*h_{t-1}
    float hc[4], hq[4], hs[4];
    int cur_chunk = -1, cur_seg = -1;

    for (int it = 0; !cur.done(); ++it, cur.advance()) {
        cp_wait<BWD_STAGES - 2>();
        __syncthreads();
        if (!pre.done()) {
            stage_tile<3, 2, DPB, NPAD, GRP, BWD_THREADS, VEC>(
                tiles + ((it + BWD_STAGES - 1) % BWD_STAGES) * GRP * ROWF, xb, dtb, dyb, Bb, Cb,
                pre.tstart(), pre.nvalid(), d0, D, N, tid);
            pre.advance();
        }
        cp_commit();
        const float *tile = tiles + (it % BWD_STAGES) * GRP * ROWF;

        if (cur.c != cur_chunk) {                      // first group of a chunk
            cur_chunk = cur.c;
            cur_seg = -1;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (cur.c > 0 && act) v = ld4(ckpt + ((size_t)b * nchunk + (cur.c - 1)) * plane + chan);
            hc[0] = v.x; hc[1] = v.y; hc[2] = v.z; hc[3] = v.w;
#pragma unroll
            for (int s = 0; s < 4; ++s) hq[s] = hc[s];
        }
        if (cur.phase == 0) {                          // pre-pass: segment-start states
            advance_tile<DPB, NPAD, ROWF>(hq, an2, tile, c, g);
            if ((cur.j + 1) % SLOTS == 0 && act) {
                const int q = (cur.j + 1) / SLOTS;
                *reinterpret_cast<float4 *>(subck + ((size_t)b * nsegk + q) * plane + chan) =
                    make_float4(hq[0], hq[1], hq[2], hq[3]);
            }
            continue;
        }
        if (cur.sg != cur_seg) {                       // first group of a segment
            cur_seg = cur.sg;
            if (cur.sg == 0) {
#pragma unroll
                for (int s = 0; s < 4; ++s) hs[s] = hc[s];
            } else {
                // written by this same thread in the pre-pass: coherent plain load
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (act) v = *reinterpret_cast<const float4 *>(
                    subck + ((size_t)b * nsegk + cur.sg) * plane + chan);
                hs[0] = v.x; hs[1] = v.y; hs[2] = v.z; hs[3] = v.w;
            }
        }
        if (cur.phase == 1) {                          // recompute: keep group-entry states
            slots[cur.j * BWD_THREADS + tid] = make_float4(hs[0], hs[1], hs[2], hs[3]);
            advance_tile<DPB, NPAD, ROWF>(hs, an2, tile, c, g);
            continue;
        }

        // ---- walk one group backwards
        const int j = cur.j;
        const int nv = cur.nvalid();
        const int t0 = cur.tstart();
        float hb[4];
        if (j == cur.ngrp - 1) {
#pragma unroll
            for (int s = 0; s < 4; ++s) hb[s] = hs[s];
        } else {
            const float4 v = slots[j * BWD_THREADS + tid];
            hb[0] = v.x; hb[1] = v.y; hb[2] = v.z; hb[3] = v.w;
        }
        float av[GRP][4], hv[GRP][4];
#pragma unroll
        for (int i = 0; i < GRP; ++i) {
            const float *row = tile + i * ROWF;
            const float xv = row[c], dtv = row[DPB + c];
            const float4 Bv = *reinterpret_cast<const float4 *>(row + 3 * DPB + 4 * g);
            const float ml = -dtv, bx = dtv * xv;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                av[i][s] = ex2(ml * an2[s]);
                hv[i][s] = fmaf(av[i][s], i ? hv[i > 0 ? i - 1 : 0][s] : hb[s], bx * comp(Bv, s));
            }
        }
#pragma unroll
        for (int i = GRP - 1; i >= 0; --i) {
            if (i < nv) {                               // uniform
                const float *row = tile + i * ROWF;
                const float xv = row[c], dtv = row[DPB + c], dyv = row[2 * DPB + c];
                const float4 Bv = *reinterpret_cast<const float4 *>(row + 3 * DPB + 4 * g);
                const float4 Cv = *reinterpret_cast<const float4 *>(row + 3 * DPB + NPAD + 4 * g);
                const float dxv = dtv * xv;
                float p1 = 0.f, p2 = 0.f, vbc[8];
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    float a1 = anx[s];
                    if (i + 1 < GRP) {
                        if (i + 1 < nv) a1 = av[i + 1 < GRP ? i + 1 : i][s];
                    }
                    gad[s] = fmaf(a1, gad[s], dyv * comp(Cv, s));
                    const float hp = i ? hv[i > 0 ? i - 1 : 0][s] : hb[s];
                    const float u = gad[s] * (av[i][s] * hp);
                    p1 = fmaf(gad[s], comp(Bv, s), p1);
                    p2 = fmaf(an[s], u, p2);
                    dac[s] = fmaf(dtv, u, dac[s]);
                    vbc[s] = gad[s] * dxv;
                    vbc[4 + s] = dyv * hv[i][s];
                }
                *reinterpret_cast<float2 *>(sn + ((i * DPB + c) * G + g) * 2) = make_float2(p1, p2);
                int fb;
                transposed_reduce<8, 16, G>(vbc, lane, fb);
                if ((lane & S::DUP_D) == 0) {
                    float *r = sd + (i * BWD_WARPS + warp) * NV2;
#pragma unroll
                    for (int k2 = 0; k2 < S::NLEFT_D; ++k2) {
                        const int idx = fb + k2;
                        r[idx < 4 ? 4 * g + idx : NPAD + 4 * g + idx - 4] = vbc[k2];
                    }
                }
            }
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) anx[s] = av[0][s];
        __syncthreads();
        // dx, ddt: finish the sums over n, one thread per (t, d), coalesced stores
        for (int p = tid; p < nv * DPB; p += BWD_THREADS) {
            const int i = p / DPB, cc = p % DPB;
            const float *src = sn + (size_t)p * G * 2;
            float s1 = 0.f, s2 = 0.f;
#pragma unroll
            for (int q = 0; q < G; ++q) { s1 += src[2 * q]; s2 += src[2 * q + 1]; }
            const float *row = tile + i * ROWF;
            if (d0 + cc < D) {
                const size_t o = (size_t)(t0 + i) * D + d0 + cc;
                dxb[o] = row[DPB + cc] * s1;
                ddtb[o] = fmaf(row[cc], s1, -s2);
            }
        }
        // dB, dC: this CTA's partial for the group's steps
        for (int p = tid; p < nv * twoN; p += BWD_THREADS) {
            const int i = p / twoN, jj = p - i * twoN;
            const int pos = jj < N ? jj : NPAD + jj - N;
            const float *r = sd + i * BWD_WARPS * NV2 + pos;
            float sum = 0.f;
#pragma unroll
            for (int w = 0; w < BWD_WARPS; ++w) sum += r[w * NV2];
            pbc[(size_t)(t0 + i) * twoN + jj] = sum;
        }
    }
    cp_wait<0>();
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

BwdWorkspace bwd_workspace_layout(int Bt, int T, int D, int N, int K)
{
    BwdWorkspace w{};
    const int G = groups_for(N);
    const int dpb = BWD_THREADS / G;
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

template <int G, bool VEC>
static cudaError_t launch_bwd_gv(const BwdArgs &a, const BwdWorkspace &w, cudaStream_t stream)
{
    using S = BwdShape<G>;
    cudaError_t e = cudaFuncSetAttribute(bwd_kernel<G, VEC>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM);
    if (e != cudaSuccess) return e;
    char *ws = static_cast<char *>(a.workspace);
    float *part_bc = reinterpret_cast<float *>(ws + w.part_bc);
    float *part_a = reinterpret_cast<float *>(ws + w.part_a);
    float *subck = reinterpret_cast<float *>(ws + w.subck);
    dim3 grid(w.nblk, a.Bt);
    bwd_kernel<G, VEC><<<grid, BWD_THREADS, S::SMEM, stream>>>(
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

template <int G>
static cudaError_t launch_bwd_g(const BwdArgs &a, const BwdWorkspace &w, cudaStream_t stream)
{
    return vec_ok(a.D, a.x, a.dt, a.dy) ? launch_bwd_gv<G, true>(a, w, stream)
                                        : launch_bwd_gv<G, false>(a, w, stream);
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
