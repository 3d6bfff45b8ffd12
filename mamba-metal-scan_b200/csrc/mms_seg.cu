// Time-segment passes for long sequences with few channels (sm_100a).
//
// When batch rows x channel blocks leave SMs idle, the scan also splits the
// sequence into S segments (seg_plan in mms_kernels.h) and each segment runs
// in its own CTAs. A segment needs what enters it from the rest of the
// sequence: the state h from the earlier segments (forward) or the adjoint
// carry from the later ones (backward). Both are affine chains over the
// segments, so they come from two small passes:
//
//   local    every segment that feeds another is scanned from a zero start;
//            the result is its end value v_s and its decay product
//            P_s = exp(-Aneg * sum_{t in s} dt_t)  (the product of its dA);
//   combine  one thread per (b, d, n) chains the S values in order:
//            forward   h_in(s+1) = P_s * h_in(s) + v_s       (h_in(0) = 0)
//            backward  E(s)      = v_s + P_s * E(s+1)        (E(S) = 0)
//            where v_s = dA_{t0(s)} * g^local_{t0(s)} and E(s+1) is what the
//            walk of segment s adds to g at its last step.
//
// The local pass costs one more exp per element of the segments it scans,
// which pays only while the unsplit kernels would leave most SMs idle.
//
// Forward: v_s goes to checkpoint slot (s+1)*cps-1 (the segment's last
// chunk), P_s to slot (s+1)*cps-2; the combine overwrites slot (s+1)*cps-1
// with the true state there, which is the checkpoint the forward proper then
// leaves in place. So the forward needs no memory beyond ckpt. Backward: v_s
// and P_s live in the caller's workspace.
#include "mms_common.cuh"
#include "mms_kernels.h"
#include "mms_stage.cuh"

namespace mms {

// The local pass is bound by MUFU: one ex2 per state-step against 3 FP32
// lanes. MMS_SEGL_POLY moves a share of its exponentials to the FMA-pipe
// polynomial (ex2_poly2): 0 none, 1 the first state pair on every other step
// (25 %), 2 the first state pair on every step (50 %).
#ifndef MMS_SEGL_POLY
#define MMS_SEGL_POLY 1
#endif

constexpr int SEGL_THREADS = 256;
constexpr int SEGL_STAGES = 3;
constexpr int SEGL_TT = 16;

template <int G>
struct SegLocalShape {
    static constexpr int DPB = SEGL_THREADS / G;
    static constexpr int NPAD = 4 * G;
    static constexpr int ROWF = 2 * DPB + NPAD;          // u, dt, row floats per step
    static constexpr size_t SMEM = sizeof(float) * (size_t)SEGL_STAGES * SEGL_TT * ROWF;
};

// One CTA: DPB channels of batch row blockIdx.z, segment s_first + blockIdx.y.
// Forward: v <- dA*v + dt*x*B over the segment, ascending.
// Backward: g <- dA_next*g + dy*C, descending; v = dA_{t0} * g_{t0} at the end.
// E: storage type of u and dt (float or bf16; row is always fp32).
template <int G, bool BWD, bool VEC, bool PROJ, typename E>
__global__ void __launch_bounds__(SEGL_THREADS, 2)
seg_local_kernel(const E *__restrict__ u, const E *__restrict__ dt,
                 const float *__restrict__ aneg, const float *__restrict__ row,
                 float *__restrict__ vout, float *__restrict__ pout,
                 int T, int D, int N, int L, int s_first, int bplanes, int splanes,
                 int voff, int poff, Proj pj_in)
{
    Proj pj = pj_in;                 // the prologue is compiled in only where it is used
    pj.on = PROJ;
    static_assert(!PROJ || sizeof(E) == 4, "the prologue takes fp32 arrays");
    using S = SegLocalShape<G>;
    constexpr int DPB = S::DPB, NPAD = S::NPAD, TT = SEGL_TT;
    constexpr int CHF = TileRow<2, DPB, E>::CHF;           // floats of u, dt per step
    constexpr int ROWF = CHF + NPAD;                       // <= S::ROWF
    extern __shared__ __align__(16) float smem[];
    const int tid = threadIdx.x;
    const int g = tid & (G - 1);
    const int c = tid / G;
    const int d0 = blockIdx.x * DPB;
    const int d = d0 + c;
    const int s = s_first + blockIdx.y;
    const int b = blockIdx.z;
    const bool act = d < D && 4 * g < N;
    const int tb = s * L;
    const int te = min(T, tb + L);
    const int ntiles = (te - tb + TT - 1) / TT;

    float2 nan2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
    if (act) {
        float4 a4 = ld4(aneg + (size_t)d * N + 4 * g);
        if (pj.on) a4 = make_float4(softplus(a4.x), softplus(a4.y), softplus(a4.z), softplus(a4.w));
        nan2[0] = f2(-a4.x * MMS_LOG2E, -a4.y * MMS_LOG2E);
        nan2[1] = f2(-a4.z * MMS_LOG2E, -a4.w * MMS_LOG2E);
    }
    const E *ub = u + (size_t)b * T * D, *dtb = dt + (size_t)b * T * D;
    const float *rb = row + (size_t)b * T * N;
    // k-th tile in processing order (descending for the backward)
    auto tstart = [&](int k) { return BWD ? tb + (ntiles - 1 - k) * TT : tb + k * TT; };
    auto stage = [&](int buf, int k) {
        const int t0 = tstart(k);
        stage_tile<2, 1, DPB, NPAD, TT, SEGL_THREADS, VEC, E>(smem + buf * TT * ROWF, ub, dtb, dtb,
                                                           rb, rb, t0, min(TT, te - t0), d0, D,
                                                           N, tid);
    };
#pragma unroll
    for (int st = 0; st < SEGL_STAGES - 1; ++st) {
        if (st < ntiles) stage(st, st);
        cp_commit();
    }

    float2 v[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
    float2 anx[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};    // backward: dA of the later step
    float sdt = 0.f;
    for (int k = 0; k < ntiles; ++k) {
        cp_wait<SEGL_STAGES - 2>();
        __syncthreads();
        const int kn = k + SEGL_STAGES - 1;
        if (kn < ntiles) stage(kn % SEGL_STAGES, kn);
        cp_commit();
        float *tile = smem + (k % SEGL_STAGES) * TT * ROWF;
        const int tk = tstart(k);
        if constexpr (PROJ) {
            // dt from its logit once per element (the channel's G lanes, one
            // warp, share its column); rows past the segment's end were staged
            // as zeros and keep dt = 0 (dA = 1, no input) rather than mapped
            for (int j = g; j < TT; j += G) {
                float *p = tile + j * ROWF + DPB + c;
                *p = tk + j < te ? fmaf(pj.range, sigmoid_fast(*p), pj.lo) : 0.f;
            }
            __syncwarp();
        }
#pragma unroll
        for (int jj = 0; jj < TT; ++jj) {
            // rows past the segment's end were staged as zeros: dA = 1, no input
            const int j = BWD ? TT - 1 - jj : jj;
            const float *r = tile + j * ROWF;
            const E *re = reinterpret_cast<const E *>(r);
            const float uv = to_f(re[c]);
            const float dtv = to_f(re[DPB + c]);
            const float4 R = *reinterpret_cast<const float4 *>(r + CHF + 4 * g);
            const float2 dt2 = f2(dtv, dtv);
            // a share of the exponentials on the FMA pipe (see MMS_SEGL_POLY)
            const bool poly0 = MMS_SEGL_POLY >= 2 || (MMS_SEGL_POLY == 1 && (jj & 1) == 0);
            const float2 a0 = poly0 ? ex2_poly2(mul2(dt2, nan2[0])) : ex2x2(mul2(dt2, nan2[0]));
            const float2 a1 = ex2x2(mul2(dt2, nan2[1]));
            sdt += dtv;
            if constexpr (!BWD) {
                const float bx = dtv * uv;
                const float2 bx2 = f2(bx, bx);
                v[0] = fma2(a0, v[0], mul2(bx2, lo(R)));
                v[1] = fma2(a1, v[1], mul2(bx2, hi(R)));
            } else {
                const float2 dy2 = f2(uv, uv);
                v[0] = fma2(anx[0], v[0], mul2(dy2, lo(R)));
                v[1] = fma2(anx[1], v[1], mul2(dy2, hi(R)));
                anx[0] = a0;
                anx[1] = a1;
            }
        }
    }
    if constexpr (BWD) {
        v[0] = mul2(anx[0], v[0]);
        v[1] = mul2(anx[1], v[1]);
    }
    if (act) {
        const float2 sd2 = f2(sdt, sdt);
        const float2 p0 = ex2x2(mul2(sd2, nan2[0])), p1 = ex2x2(mul2(sd2, nan2[1]));
        const size_t DN = (size_t)D * N, e = (size_t)d * N + 4 * g;
        const size_t pl = (size_t)b * bplanes + (size_t)s * splanes;
        st4(vout + (pl + voff) * DN + e, make_float4(v[0].x, v[0].y, v[1].x, v[1].y));
        st4(pout + (pl + poff) * DN + e, make_float4(p0.x, p0.y, p1.x, p1.y));
    }
}

__global__ void seg_combine_fwd_kernel(float *__restrict__ ckpt, int Bt, int nchunk, int S,
                                       int cps, size_t DN)
{
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < (size_t)Bt * DN;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t b = idx / DN, e = idx - b * DN;
        float *base = ckpt + b * (size_t)nchunk * DN + e;
        float h = 0.f;
        for (int s = 0; s + 1 < S; ++s) {
            float *hv = base + (size_t)((s + 1) * cps - 1) * DN;
            const float p = base[(size_t)((s + 1) * cps - 2) * DN];
            h = fmaf(p, h, *hv);
            *hv = h;
        }
    }
}

__global__ void seg_combine_bwd_kernel(float *__restrict__ E, const float *__restrict__ P, int Bt,
                                       int S, size_t DN)
{
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < (size_t)Bt * DN;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t b = idx / DN, e = idx - b * DN;
        float *eb = E + b * (size_t)S * DN + e;
        const float *pb = P + b * (size_t)S * DN + e;
        float carry = 0.f;                              // E(s+1)
        for (int s = S - 1; s >= 1; --s) {
            const float local = eb[(size_t)s * DN];
            const float p = pb[(size_t)s * DN];
            eb[(size_t)s * DN] = carry;                 // carry into segment s
            carry = fmaf(p, carry, local);              // E(s)
        }
        eb[0] = carry;
    }
}

template <int G, bool BWD, bool VEC, bool PROJ, typename E = float>
static cudaError_t launch_local_gvp(const SegLocalArgs &a, cudaStream_t stream)
{
    using S = SegLocalShape<G>;
    cudaError_t e = smem_opt_in<seg_local_kernel<G, BWD, VEC, PROJ, E>>(S::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((a.D + S::DPB - 1) / S::DPB, a.nseg, a.Bt);
    seg_local_kernel<G, BWD, VEC, PROJ, E><<<grid, SEGL_THREADS, S::SMEM, stream>>>(
        reinterpret_cast<const E *>(a.u), reinterpret_cast<const E *>(a.dt), a.aneg, a.row, a.vout, a.pout, a.T, a.D, a.N, a.L, a.s_first, a.bplanes,
        a.splanes, a.voff, a.poff, a.proj);
    return cudaGetLastError();
}

template <int G, bool BWD, bool VEC>
static cudaError_t launch_local_gv(const SegLocalArgs &a, cudaStream_t stream)
{
    return a.proj.on ? launch_local_gvp<G, BWD, VEC, true>(a, stream)
                     : launch_local_gvp<G, BWD, VEC, false>(a, stream);
}

template <int G>
static cudaError_t launch_local_g(const SegLocalArgs &a, bool backward, cudaStream_t stream)
{
    const bool v = vec_ok(a.D, a.u, a.dt);
    if (backward) return v ? launch_local_gv<G, true, true>(a, stream)
                           : launch_local_gv<G, true, false>(a, stream);
    return v ? launch_local_gv<G, false, true>(a, stream) : launch_local_gv<G, false, false>(a, stream);
}

template <int G>
static cudaError_t launch_local_bf16(const SegLocalArgs &a, bool backward, cudaStream_t stream)
{
    return backward ? launch_local_gvp<G, true, true, false, __nv_bfloat16>(a, stream)
                    : launch_local_gvp<G, false, true, false, __nv_bfloat16>(a, stream);
}

cudaError_t launch_seg_local(const SegLocalArgs &a, bool backward, cudaStream_t stream)
{
    if (a.bf16) {
        // bf16 u, dt: 16-byte staging (D % 8 == 0, aligned), no prologue
        if (!vec_ok(a.D, a.u, a.dt) || a.D % 8 != 0 || a.proj.on) return cudaErrorInvalidValue;
        switch (groups_for(a.N)) {
        case 1: return launch_local_bf16<1>(a, backward, stream);
        case 2: return launch_local_bf16<2>(a, backward, stream);
        case 4: return launch_local_bf16<4>(a, backward, stream);
        case 8: return launch_local_bf16<8>(a, backward, stream);
        case 16: return launch_local_bf16<16>(a, backward, stream);
        default: return cudaErrorInvalidValue;
        }
    }
    switch (groups_for(a.N)) {
    case 1: return launch_local_g<1>(a, backward, stream);
    case 2: return launch_local_g<2>(a, backward, stream);
    case 4: return launch_local_g<4>(a, backward, stream);
    case 8: return launch_local_g<8>(a, backward, stream);
    case 16: return launch_local_g<16>(a, backward, stream);
    default: return cudaErrorInvalidValue;
    }
}

static int combine_blocks(size_t n)
{
    const size_t b = (n + 255) / 256;
    return (int)(b < (size_t)N_SM * 8 ? b : (size_t)N_SM * 8);
}

cudaError_t launch_seg_combine_fwd(float *ckpt, int Bt, int nchunk, int S, int cps, size_t DN,
                                   cudaStream_t stream)
{
    seg_combine_fwd_kernel<<<combine_blocks((size_t)Bt * DN), 256, 0, stream>>>(ckpt, Bt, nchunk,
                                                                                S, cps, DN);
    return cudaGetLastError();
}

cudaError_t launch_seg_combine_bwd(float *E, const float *P, int Bt, int S, size_t DN,
                                   cudaStream_t stream)
{
    seg_combine_bwd_kernel<<<combine_blocks((size_t)Bt * DN), 256, 0, stream>>>(E, P, Bt, S, DN);
    return cudaGetLastError();
}

}  // namespace mms
