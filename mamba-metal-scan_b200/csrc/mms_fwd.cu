// Forward selective scan for sm_100a.
//
// Math (reference mamba_metal/scan.py:13-15, kernel ssm_fwd at :78-127):
//     dA = exp(-dt*Aneg);  h_t = dA*h_{t-1} + dt*B_t*x_t;  y_t = sum_n C_tn*h_tn
// with h checkpointed at the end of every K-step chunk and at t = T-1.
//
// Decomposition: a thread owns 4 consecutive states of one (b, d) channel and
// G = (N/4 rounded up to a power of two) lanes share a channel, so a CTA of
// FWD_THREADS threads covers DPB = FWD_THREADS/G consecutive channels of one
// batch row and walks the whole sequence. One thread per (b, d), as in the
// reference, would leave most of the 148 SMs idle; G lanes per channel give G
// times the threads and keep only 4 states and 4 decay rates per thread.
//
// Memory: x, dt, B, C arrive in shared memory as time tiles of TT steps,
// staged by cp.async FWD_STAGES-1 tiles ahead of the compute, so the serial
// recurrence never waits on DRAM. y_t needs the sum over the channel's G
// lanes: each lane stores its partial in shared memory and, once per tile,
// every thread finishes some (t, d) sums and writes y with coalesced stores.
#include <string.h>

#include "mms_common.cuh"
#include "mms_kernels.h"
#include "mms_stage.cuh"
#include "mms_tma.cuh"

namespace mms {

constexpr int FWD_THREADS = 256;
constexpr int FWD_STAGES = 3;

// Where lane g's y partial of row p (= step * DPB + channel) sits in the
// [TT*DPB][G] partial buffer. For G >= 8 a row spans 2 or 4 float4 quads;
// quad (g >> 2) is stored at quad (g >> 2) ^ f(p), so the reduction's float4
// reads of consecutive rows touch every bank group (rows at 32- or 64-byte
// stride would otherwise put 8 or 16 lanes on the same banks). The reduction
// reads the quads in logical order, so sums are unchanged.
template <int G>
__device__ __forceinline__ int ys_at(int p, int g)
{
    if constexpr (G == 16) return p * 16 + 4 * ((g >> 2) ^ ((p >> 1) & 3)) + (g & 3);
    else if constexpr (G == 8) return p * 8 + 4 * ((g >> 2) ^ ((p >> 2) & 1)) + (g & 3);
    else return p * G + g;
}

template <int G>
struct FwdShape {
    static constexpr int DPB = FWD_THREADS / G;            // channels per CTA
    static constexpr int NPAD = 4 * G;
    static constexpr int TT = G == 1 ? 8 : 16;             // steps per tile
    static constexpr int ROWF = 2 * DPB + 2 * NPAD;        // x, dt, B, C floats per step
    static constexpr size_t SMEM = sizeof(float) * ((size_t)FWD_STAGES * TT * ROWF
                                                    + (size_t)TT * DPB * G);
};

// E: storage type of x, dt and y (float or bf16; bf16 rows are staged in
// 16-byte pieces, VEC).
template <int G, bool VEC, bool PROJ, typename E>
__global__ void __launch_bounds__(FWD_THREADS, 2)
fwd_kernel(const E *__restrict__ x, const E *__restrict__ dt,
           const float *__restrict__ aneg, const float *__restrict__ Bm,
           const float *__restrict__ Cm, E *__restrict__ y,
           float *__restrict__ ckpt, int T, int D, int N, int K, int L, int cps, Proj pj_in)
{
    Proj pj = pj_in;                 // the prologue is compiled in only where it is used
    pj.on = PROJ;
    static_assert(!PROJ || sizeof(E) == 4, "the prologue takes fp32 arrays");
    using S = FwdShape<G>;
    constexpr int DPB = S::DPB, NPAD = S::NPAD, TT = S::TT, ROWF = S::ROWF;
    constexpr int CHF = TileRow<2, DPB, E>::CHF;           // floats of x, dt per staged step
    constexpr int RROW = CHF + 2 * NPAD;                   // staged step (floats), <= ROWF
    extern __shared__ __align__(128) float smem[];
    float *tiles = smem;                                   // [STAGES][TT][ROWF]
    float *ys = smem + FWD_STAGES * TT * ROWF;             // [TT][DPB][G] partial y

    const int tid = threadIdx.x;
    const int g = tid & (G - 1);
    const int c = tid / G;                                 // channel within the CTA
    const int d0 = blockIdx.x * DPB;
    const int d = d0 + c;
    const int b = blockIdx.y;
    const bool act = d < D && 4 * g < N;
    const int nchunk = (T + K - 1) / K;
    // Time segment blockIdx.z of gridDim.z covers steps [tb, te) = chunks
    // [sg*cps, (sg+1)*cps); a single segment is the whole sequence.
    const int sg = blockIdx.z, nsg = gridDim.z;
    const int tb = sg * L, te = min(T, tb + L);

    // -Aneg * log2(e) as two packed pairs: dA = 2^(dt * nan2).
    float2 nan2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
    if (act) {
        float4 a4 = ld4(aneg + (size_t)d * N + 4 * g);
        if (pj.on) a4 = make_float4(softplus(a4.x), softplus(a4.y), softplus(a4.z), softplus(a4.w));
        nan2[0] = f2(-a4.x * MMS_LOG2E, -a4.y * MMS_LOG2E);
        nan2[1] = f2(-a4.z * MMS_LOG2E, -a4.w * MMS_LOG2E);
    }

    const E *xb = x + (size_t)b * T * D, *dtb = dt + (size_t)b * T * D;
    const float *Bb = Bm + (size_t)b * T * N, *Cb = Cm + (size_t)b * T * N;
    float *ckb = ckpt + (size_t)b * nchunk * D * N + (size_t)d * N + 4 * g;
    E *yb = y + (size_t)b * T * D;

    // The state entering the segment: the checkpoint the segment combine left
    // at the end of the previous segment (zero for the first).
    float2 h[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
    if (sg > 0 && act) {
        const float4 w = *reinterpret_cast<const float4 *>(ckb + (size_t)(sg * cps - 1) * D * N);
        h[0] = lo(w);
        h[1] = hi(w);
    }
    // that boundary checkpoint is final; the segment's own last one is left alone
    const int ck_keep = sg + 1 < nsg ? (sg + 1) * cps - 1 : -1;

    const int ntiles = (te - tb + TT - 1) / TT;
#pragma unroll
    for (int s = 0; s < FWD_STAGES - 1; ++s) {
        if (s < ntiles)
            stage_tile<2, 2, DPB, NPAD, TT, FWD_THREADS, VEC, E>(tiles + s * TT * ROWF, xb, dtb, dtb, Bb, Cb,
                                                              tb + s * TT, min(TT, te - tb - s * TT),
                                                              d0, D, N, tid);
        cp_commit();
    }

    int next_ck = min(tb + K, T) - 1;                      // step whose state is checkpointed next
    int chunk = sg * cps;
    for (int k = 0; k < ntiles; ++k) {
        cp_wait<FWD_STAGES - 2>();
        __syncthreads();
        const int kn = k + FWD_STAGES - 1;
        if (kn < ntiles)
            stage_tile<2, 2, DPB, NPAD, TT, FWD_THREADS, VEC, E>(
                tiles + (kn % FWD_STAGES) * TT * ROWF, xb, dtb, dtb, Bb, Cb, tb + kn * TT,
                min(TT, te - tb - kn * TT), d0, D, N, tid);
        cp_commit();

        float *tile = tiles + (k % FWD_STAGES) * TT * ROWF;
        const int t0 = tb + k * TT;
        if constexpr (PROJ) {
            // dt from its logit once per element: the channel's G lanes (one
            // warp) share its column of the tile
            for (int j = g; j < TT; j += G) {
                float *p = tile + j * RROW + DPB + c;
                *p = fmaf(pj.range, sigmoid_fast(*p), pj.lo);
            }
            __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < TT; ++j) {
            const float *row = tile + j * RROW;
            const E *re = reinterpret_cast<const E *>(row);
            // Steps past T were staged as zeros: dt = 0 gives dA = 1, b = 0.
            const float xv = to_f(re[c]);
            const float dtv = to_f(re[DPB + c]);
            const float4 Bv = *reinterpret_cast<const float4 *>(row + CHF + 4 * g);
            const float4 Cv = *reinterpret_cast<const float4 *>(row + CHF + NPAD + 4 * g);
            const float bx = dtv * xv;
            const float2 dt2 = f2(dtv, dtv), bx2 = f2(bx, bx);
            h[0] = fma2(ex2x2(mul2(dt2, nan2[0])), h[0], mul2(bx2, lo(Bv)));
            h[1] = fma2(ex2x2(mul2(dt2, nan2[1])), h[1], mul2(bx2, hi(Bv)));
            const float2 acc = fma2(hi(Cv), h[1], mul2(lo(Cv), h[0]));
            ys[ys_at<G>(j * DPB + c, g)] = acc.x + acc.y;
            if (t0 + j == next_ck && t0 + j < te) {        // uniform across the CTA
                if (act && chunk != ck_keep)
                    st4(ckb + (size_t)chunk * D * N, make_float4(h[0].x, h[0].y, h[1].x, h[1].y));
                ++chunk;
                next_ck = min(next_ck + K, T - 1);
            }
        }
        __syncthreads();
        // y = sum of the G lane partials; consecutive threads take consecutive channels.
        for (int p = tid; p < TT * DPB; p += FWD_THREADS) {
            const int j = p / DPB, cc = p % DPB;
            float sum = 0.f;
            if constexpr (G >= 4) {
#pragma unroll
                for (int q = 0; q < G; q += 4) {
                    const float4 v = *reinterpret_cast<const float4 *>(ys + ys_at<G>(p, q));
                    sum += (v.x + v.y) + (v.z + v.w);
                }
            } else {
                const float *src = ys + (size_t)p * G;
#pragma unroll
                for (int q = 0; q < G; ++q) sum += src[q];
            }
            if (t0 + j < te && d0 + cc < D) yb[(size_t)(t0 + j) * D + d0 + cc] = from_f<E>(sum);
        }
    }
}


// ---------------------------------------------------------------------------
// Whole-state variant for 8 < N <= 16: one thread per (b, d) channel holds all
// 16 states. y_t is then a sum inside the thread (no cross-lane reduction),
// B_t and C_t are broadcast loads, and each step offers 16 independent ex2.
// Used when there are enough channels to fill the GPU (B*D >= S16_MIN_CHANNELS);
// otherwise the G-lane kernel above gives more threads.
//
// Output (BULK): y rows and checkpoints are written to shared memory and
// leave for HBM on the bulk-copy engine, one tile later, so the 226 MB of y +
// checkpoint writes at config 1 do not occupy the warps' load/store issue.
// Per tile of 16 steps: y rows [16][128] and up to two checkpoint slabs of
// 128 channels x N (each a contiguous block of ckpt), double buffered; a
// third checkpoint in one tile (only the t = T-1 one can be) is stored
// directly. With TMA staging the slabs are sent by TMA tile stores from a
// swizzled layout (see fwd_kernel_s16), otherwise by plain bulk copies.
#ifndef MMS_FWD_ACC
#define MMS_FWD_ACC 4
#endif
constexpr int S16_DPB = 128;                                 // channels per CTA
// Lanes per channel: 1 (a thread holds all 16 states) or 2 (8 states each:
// twice the warps per SM for the same shared memory; the two halves of y
// meet by one shuffle). Two measured slower: config 1 118.6 against
// 111.6 us, config 4 897 against 834 us.
#ifndef MMS_S16_LPC
#define MMS_S16_LPC 1
#endif
constexpr int S16_LPC = MMS_S16_LPC;
static_assert(S16_LPC == 1 || S16_LPC == 2, "1 or 2 lanes per channel");
constexpr int S16_THREADS = S16_DPB * S16_LPC;
constexpr int S16_NP = 8 / S16_LPC;                          // state pairs per thread
#ifndef MMS_S16_TT
#define MMS_S16_TT 16
#endif
#ifndef MMS_S16_MINB
#define MMS_S16_MINB 2
#endif
#ifndef MMS_S16_UNROLL
#define MMS_S16_UNROLL 4
#endif
constexpr int S16_UNROLL = MMS_S16_UNROLL;                   // steps unrolled in the tile loop

// How many of the 8 state pairs of the whole-state forward take their decays
// from the FMA-pipe polynomial (ex2_poly2) instead of MUFU ex2: one ex2 per
// state and step is the kernel's MUFU load (16 per SM per clock, the binding
// pipe), while its FP32 work is 4 lanes per state and step out of 128 per SM
// per clock, so a share of the exponentials on the FMA pipe balances the two.
#ifndef MMS_FWD_POLY_PAIRS
#define MMS_FWD_POLY_PAIRS 1
#endif
// The thread's decays 2^(dt * nan2) of step j. One lane per channel: its
// pairs 0 .. MMS_FWD_POLY_PAIRS-1 take the polynomial; two lanes: those
// pairs of each lane on even steps, the same share of the channel's
// exponentials. `p` and `j & 1` are constants after the step loop's
// unrolling, so each pair is compiled to one of the two paths.
__device__ __forceinline__ void fwd_decays(float2 (&dA)[S16_NP], float dtv, const float2 (&nan2)[S16_NP],
                                           int j) {
    const float2 dt2 = f2(dtv, dtv);
#pragma unroll
    for (int p = 0; p < S16_NP; ++p) {
        const bool poly = p < MMS_FWD_POLY_PAIRS && (S16_LPC == 1 || (j & 1) == 0);
        dA[p] = poly ? ex2_poly2(mul2(dt2, nan2[p])) : ex2x2(mul2(dt2, nan2[p]));
    }
}
constexpr int S16_TT = MMS_S16_TT;                           // steps per staged tile
constexpr int S16_MIN_CHANNELS = 148 * S16_DPB;

struct S16Shape {
    static constexpr int DPB = S16_DPB;
    static constexpr int ROWF = 2 * DPB + 2 * 16;            // x, dt, B, C floats per step
    static constexpr size_t TILEF = (size_t)FWD_STAGES * S16_TT * ROWF;
    static constexpr size_t YF = (size_t)2 * S16_TT * DPB;   // [2][TT][DPB]
    static constexpr size_t CKF = (size_t)2 * 2 * DPB * 16;  // [2][2][DPB*N]
    static constexpr size_t SMEM = sizeof(float) * TILEF;
    static constexpr size_t SMEM_BULK = sizeof(float) * (TILEF + YF + CKF);
    // + 1 KB to align the checkpoint slabs for their swizzled TMA stores,
    // + the stage barriers
    static constexpr size_t SMEM_TMA = SMEM_BULK + 1024 + 64;
    static constexpr uint32_t TILE_BYTES = sizeof(float) * S16_TT * ROWF;
};

// TMA tile of channel-array storage type E: x and dt take XF floats each,
// then B and C (fp32) [TT][16] each; BYTES is what one tile's four loads bring.
template <typename E>
struct S16Tile {
    static constexpr int XF = S16_TT * S16_DPB * (int)sizeof(E) / 4;
    static constexpr uint32_t BYTES = 4u * (2 * XF + 2 * S16_TT * 16);
};
static_assert(S16Tile<float>::BYTES == S16Shape::TILE_BYTES, "fp32 TMA tile is the full tile");

// Tensor maps of the TMA staging path: x, dt (D, T, Bt) with 128 x 16 boxes,
// B, C (N, T, Bt) with 16 x 16 boxes; for the stores, y (D, T, Bt) with
// 128 x 16 boxes and ckpt (N, D, nchunk, Bt) with 16 x 128 boxes in the
// 64-byte swizzled shared layout.
struct FwdMaps {
    CUtensorMap x, dt, B, C, y, ck;
};

// Set when a wait on a forward TMA stage gave up; read by mms_device_status().
__device__ unsigned int g_fwd_timeout;

// Bounded wait for a tile's copies (at most `limit` polls); a wait that runs
// out makes the CTA leave (see the kernel) instead of hanging the GPU.
__device__ __forceinline__ bool fwd_wait(uint32_t bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try(bar, parity)) return true;
    return false;
}

// TMA: tiles arrive by TMA tile loads (one thread, 4 per tile) that complete
// on per-stage mbarriers, in an array-major layout [x TTxDPB][dt TTxDPB]
// [B TTx16][C TTx16]; out-of-range steps, channels and states load as zeros,
// like the cp.async path's zero fill.
// E: storage type of x, dt and y (float, or bf16 with TMA staging only).
template <bool VEC, bool BULK, bool TMA, bool PROJ, bool SEG, typename E>
__global__ void __launch_bounds__(S16_THREADS, MMS_S16_MINB)
fwd_kernel_s16(const E *__restrict__ x, const E *__restrict__ dt,
               const float *__restrict__ aneg, const float *__restrict__ Bm,
               const float *__restrict__ Cm, E *__restrict__ y,
               float *__restrict__ ckpt, int T, int D, int N, int K, int L, int cps,
               const __grid_constant__ FwdMaps maps, Proj pj_in, uint32_t wait_limit,
               int skip_item)
{
    Proj pj = pj_in;                                       // the prologue only where used
    pj.on = PROJ;
    static_assert(sizeof(E) == 4 || (TMA && BULK), "bf16 arrays take the TMA / bulk path");
    constexpr int DPB = S16Shape::DPB, ROWF = S16Shape::ROWF, TT = S16_TT;
    constexpr int XF = S16Tile<E>::XF;
    // where step j of a tile keeps x, dt (elements of E from their region's
    // start), B, C (floats); region offsets in floats from the tile start
    constexpr int XROW = TMA ? DPB : ROWF, XOFF = 0;
    constexpr int DOFF = TMA ? XF : DPB;
    constexpr int BROW = TMA ? 16 : ROWF, BOFF = TMA ? 2 * XF : 2 * DPB;
    constexpr int COFF = TMA ? 2 * XF + TT * 16 : 2 * DPB + 16;
    extern __shared__ __align__(128) float smem[];
    float *tiles = smem;                                   // [STAGES][TT][ROWF]
    float *ys = smem + S16Shape::TILEF;                    // BULK: [2][TT][DPB] of E
    E *yse = reinterpret_cast<E *>(ys);
    // BULK: [2][2] checkpoint slabs. cp.async path: [DPB][N] rows, sent by bulk
    // copies. TMA path: [DPB][16] rows in the 64-byte swizzled layout (state
    // quad q of channel c at quad q ^ ((c >> 1) & 3), so a warp's 16-byte
    // stores of 32 channels hit all banks), 1024-byte aligned, sent by TMA
    // tile stores that undo the swizzle.
    float *cks = ys + S16Shape::YF;
    if constexpr (TMA) cks += ((1024u - (smem_u32(cks) & 1023u)) & 1023u) / 4u;
    constexpr int CKROW = TMA ? 16 : 0;                    // TMA slab row (floats); else N
    const uint32_t bars = smem_u32(cks + S16Shape::CKF);   // TMA: FWD_STAGES barriers

    const int tid = threadIdx.x;
    const int c = tid / S16_LPC, hf = tid % S16_LPC;       // channel in the CTA, its half
    constexpr int NQ = S16_NP / 2;                         // state quads per thread
    const int q0 = hf * NQ;                                // the thread's first quad
    const int d0 = blockIdx.x * DPB;
    const int d = d0 + c;
    const int b = blockIdx.y;
    const bool dval = d < D;
    const int dcnt = min(DPB, D - d0);
    const int nchunk = (T + K - 1) / K;
    // Time segment blockIdx.z of gridDim.z: steps [tb, te) = chunks
    // [sg*cps, (sg+1)*cps); a single segment is the whole sequence.
    // (SEG false: one segment, compiled without the segment bookkeeping)
    const int sg = SEG ? (int)blockIdx.z : 0, nsg = SEG ? (int)gridDim.z : 1;
    const int tb = SEG ? sg * L : 0, te = SEG ? min(T, tb + L) : T;
    // the combine left the checkpoint at this segment's end; it is not rewritten
    const int ck_keep = SEG && sg + 1 < nsg ? (sg + 1) * cps - 1 : -1;

    // -Aneg * log2(e) for the thread's states (zero past N): dA = 2^(dt * nan2).
    float2 nan2[S16_NP], h[S16_NP];
#pragma unroll
    for (int p = 0; p < S16_NP; ++p) {
        float a0 = 0.f, a1 = 0.f;
        const int s = 4 * q0 + 2 * p;                      // the pair's first state
        if (dval && s < N) {
            float2 v = *reinterpret_cast<const float2 *>(aneg + (size_t)d * N + s);
            if (pj.on) v = f2(softplus(v.x), softplus(v.y));
            a0 = -v.x * MMS_LOG2E;
            a1 = -v.y * MMS_LOG2E;
        }
        nan2[p] = f2(a0, a1);
        h[p] = f2(0.f, 0.f);
    }

    const E *xb = x + (size_t)b * T * D, *dtb = dt + (size_t)b * T * D;
    const float *Bb = Bm + (size_t)b * T * N, *Cb = Cm + (size_t)b * T * N;
    float *ckb = ckpt + (size_t)b * nchunk * D * N + (size_t)d * N;
    E *yb = y + (size_t)b * T * D + d;
    if (SEG && sg > 0 && dval) {                           // state entering the segment
        const float *src = ckb + (size_t)(sg * cps - 1) * D * N;
#pragma unroll
        for (int q = 0; q < NQ; ++q)
            if (4 * (q0 + q) < N) {
                const float4 w = *reinterpret_cast<const float4 *>(src + 4 * (q0 + q));
                h[2 * q] = lo(w);
                h[2 * q + 1] = hi(w);
            }
    }

    // BULK: send tile kp's y rows and its (up to two) checkpoint slabs.
    auto send = [&](int kp, int nck, int ck0, int ck1) {
        const int t0p = tb + kp * TT, rows = min(TT, te - t0p);
        const E *ysrc = yse + (kp & 1) * TT * DPB;
        if (TMA && (!SEG || rows == TT)) {
            // one tile store; rows past T and channels past D are not written
            tma_store3(&maps.y, smem_u32(ysrc), d0, t0p, b);
        } else {
            // a segment's last rows stop at te, inside the tensor: row by row
            for (int r = 0; r < rows; ++r)
                bulk_store(y + ((size_t)b * T + t0p + r) * D + d0, ysrc + r * DPB,
                           dcnt * (uint32_t)sizeof(E));
        }
        for (int i = 0; i < nck; ++i) {
            if constexpr (TMA)
                tma_store4(&maps.ck, smem_u32(cks + ((kp & 1) * 2 + i) * DPB * CKROW), 0, d0,
                           i ? ck1 : ck0, b);
            else
                bulk_store(ckpt + ((size_t)b * nchunk + (i ? ck1 : ck0)) * D * N + (size_t)d0 * N,
                           cks + ((kp & 1) * 2 + i) * DPB * N, (uint32_t)dcnt * N * 4u);
        }
        bulk_commit();
    };

    // stage tile kt into buffer buf
    auto stage = [&](int buf, int kt) {
        float *tile = tiles + buf * TT * ROWF;
        if constexpr (TMA) {
            if (tid == 0 && kt != skip_item) {             // the test hook withholds one tile
                const uint32_t bar = bars + 8 * buf, dst = smem_u32(tile);
                mbar_expect(bar, S16Tile<E>::BYTES);
                tma3(dst, &maps.x, d0, tb + kt * TT, b, bar);
                tma3(dst + 4 * DOFF, &maps.dt, d0, tb + kt * TT, b, bar);
                tma3(dst + 4 * BOFF, &maps.B, 0, tb + kt * TT, b, bar);
                tma3(dst + 4 * COFF, &maps.C, 0, tb + kt * TT, b, bar);
            }
        } else {
            stage_tile<2, 2, DPB, 16, TT, S16_THREADS, VEC>(tile, xb, dtb, dtb, Bb, Cb, tb + kt * TT,
                                                    min(TT, te - tb - kt * TT), d0, D, N, tid);
        }
    };

    // Rows past te (TMA: the next segment's steps; cp.async: zeros) move the
    // state on, but nothing past te is stored.
    const int ntiles = (te - tb + TT - 1) / TT;
    if constexpr (TMA) {
        if (tid == 0) {
            for (int s = 0; s < FWD_STAGES; ++s) mbar_init(bars + 8 * s, 1);
            asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        }
        __syncthreads();
    }
#pragma unroll
    for (int s = 0; s < FWD_STAGES - 1; ++s) {
        if (s < ntiles) stage(s, s);
        cp_commit();
    }

    int next_ck = min(tb + K, T) - 1;
    int chunk = sg * cps;
    int nck = 0, ck0 = 0, ck1 = 0;                         // checkpoints of the current tile
    int pnck = 0, pck0 = 0, pck1 = 0;                      // ... of the previous tile
    for (int k = 0; k < ntiles; ++k) {
        if constexpr (BULK) {
            if (k > 0) fence_async_smem();                 // tile k-1's y / checkpoints
            if (tid == 0) bulk_wait_read<0>();             // tile k-2's copies have left set k&1
        }
        if constexpr (TMA) {
            const bool ok = fwd_wait(bars + 8 * (k % FWD_STAGES), (k / FWD_STAGES) & 1, wait_limit);
            if (__syncthreads_or(!ok)) {
                // a tile never arrived: leave together, after the loads still in
                // flight and the bulk stores already issued
                if (tid == 0) {
                    for (int j = k; j < min(k + FWD_STAGES - 1, ntiles); ++j)
                        if (j != skip_item)
                            fwd_wait(bars + 8 * (j % FWD_STAGES), (j / FWD_STAGES) & 1, wait_limit);
                    if constexpr (BULK) bulk_wait<0>();
                    atomicOr(&g_fwd_timeout, 1u);
                }
                return;
            }
        } else {
            cp_wait<FWD_STAGES - 2>();
            __syncthreads();
        }
        if constexpr (BULK) {
            if (k > 0 && tid == 0) send(k - 1, pnck, pck0, pck1);
        }
        const int kn = k + FWD_STAGES - 1;
        if (kn < ntiles) {
            // the buffer's previous tile (k-1) was read before the barrier above
            if (TMA && tid == 0) fence_async_smem();
            stage(kn % FWD_STAGES, kn);
        }
        cp_commit();

        const float *tile = tiles + (k % FWD_STAGES) * TT * ROWF;
        const E *tx = reinterpret_cast<const E *>(tile + XOFF);
        const E *tdt = reinterpret_cast<const E *>(tile + DOFF);
        E *yrow = yse + (k & 1) * TT * DPB + c;
        const int t0 = tb + k * TT;
        nck = 0;
#pragma unroll S16_UNROLL
        for (int j = 0; j < TT; ++j) {
            // Steps past T were staged as zeros: dt = 0 gives dA = 1, b = 0.
            const float xv = to_f(tx[j * XROW + c]);
            float dtv = to_f(tdt[j * XROW + c]);
            if (pj.on) dtv = fmaf(pj.range, sigmoid_fast(dtv), pj.lo);
            float2 dAc[S16_NP];
            fwd_decays(dAc, dtv, nan2, j);
            const float4 *bp = reinterpret_cast<const float4 *>(tile + BOFF + j * BROW) + q0;
            const float4 *cp = reinterpret_cast<const float4 *>(tile + COFF + j * BROW) + q0;
            const float bx = dtv * xv;
            const float2 bx2 = f2(bx, bx);
            // y = sum_n C*h over MMS_FWD_ACC independent partial sums (shorter chains)
            float2 acc[MMS_FWD_ACC];
#pragma unroll
            for (int q = 0; q < MMS_FWD_ACC; ++q) acc[q] = f2(0.f, 0.f);
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
                const float4 Bv = bp[q], Cv = cp[q];
                h[2 * q] = fma2(dAc[2 * q], h[2 * q], mul2(bx2, lo(Bv)));
                h[2 * q + 1] = fma2(dAc[2 * q + 1], h[2 * q + 1], mul2(bx2, hi(Bv)));
                acc[(2 * q) % MMS_FWD_ACC] = fma2(lo(Cv), h[2 * q], acc[(2 * q) % MMS_FWD_ACC]);
                acc[(2 * q + 1) % MMS_FWD_ACC] = fma2(hi(Cv), h[2 * q + 1], acc[(2 * q + 1) % MMS_FWD_ACC]);
            }
#pragma unroll
            for (int q = 1; q < MMS_FWD_ACC; ++q) acc[0] = add2(acc[0], acc[q]);
            float yv = acc[0].x + acc[0].y;
            if constexpr (S16_LPC == 2) yv += __shfl_xor_sync(0xffffffffu, yv, 1);
            const int t = t0 + j;
            if constexpr (BULK) {
                if (hf == 0) yrow[j * DPB] = from_f<E>(yv);
            } else if (hf == 0 && dval && t < te) {
                yb[(size_t)t * D] = from_f<E>(yv);
            }
            if (t == next_ck && (!SEG || t < te)) {        // uniform across the CTA
                float *o = ckb + (size_t)chunk * D * N;
                const bool keep = SEG && chunk == ck_keep;
                int swz = 0;                               // quad index XOR (TMA slabs)
                if (BULK && nck < 2 && !keep) {
                    if constexpr (TMA) {
                        o = cks + ((k & 1) * 2 + nck) * DPB * CKROW + c * CKROW;
                        swz = (c >> 1) & 3;
                    } else {
                        o = cks + ((k & 1) * 2 + nck) * DPB * N + c * N;
                    }
                    if (nck == 0) ck0 = chunk; else ck1 = chunk;
                    ++nck;
                }
                if (dval && !keep) {
#pragma unroll
                    for (int q = 0; q < NQ; ++q)
                        if (4 * (q0 + q) < N)
                            st4(o + 4 * ((q0 + q) ^ swz), make_float4(h[2 * q].x, h[2 * q].y,
                                                                      h[2 * q + 1].x, h[2 * q + 1].y));
                }
                ++chunk;
                next_ck = min(next_ck + K, T - 1);
            }
        }
        pnck = nck;
        pck0 = ck0;
        pck1 = ck1;
    }
    if constexpr (BULK) {
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            send(ntiles - 1, pnck, pck0, pck1);
            bulk_wait<0>();
        }
    }
}

// Time segments for the whole-state forward: its CTAs hold 128 channels and
// run 2 per SM, so segments are cut when batch rows x 128-channel blocks
// leave SMs without a CTA, aiming at one full wave.
static SegPlan seg_plan_s16(int Bt, int T, int D, int K)
{
    const long long base = (long long)Bt * ((D + S16_DPB - 1) / S16_DPB);
    const int nchunk = (T + K - 1) / K;
    SegPlan p{1, nchunk};
    if (base >= N_SM) return p;
    const long long want = ((long long)MMS_S16_MINB * N_SM) / base;
    long long cps = (nchunk + want - 1) / want;
    if (cps < 2) cps = 2;                           // P_s is kept in chunk cps-2
    if (cps * K < 64) cps = (64 + K - 1) / K;
    const long long S = (nchunk + cps - 1) / cps;
    if (S < 2) return p;
    p.S = (int)S;
    p.cps = (int)cps;
    return p;
}

template <bool VEC, bool BULK, bool TMA, bool PROJ, bool SEG, typename E>
static cudaError_t launch_fwd_s16_q(const FwdArgs &a, const FwdMaps &maps, SegPlan sp,
                                    cudaStream_t stream)
{
    const size_t smem = TMA ? S16Shape::SMEM_TMA : BULK ? S16Shape::SMEM_BULK : S16Shape::SMEM;
    cudaError_t e = smem_opt_in<fwd_kernel_s16<VEC, BULK, TMA, PROJ, SEG, E>>(smem);
    if (e != cudaSuccess) return e;
    dim3 grid((a.D + S16Shape::DPB - 1) / S16Shape::DPB, a.Bt, sp.S);
    fwd_kernel_s16<VEC, BULK, TMA, PROJ, SEG, E><<<grid, S16_THREADS, smem, stream>>>(
        reinterpret_cast<const E *>(a.x), reinterpret_cast<const E *>(a.dt), a.aneg, a.B, a.C,
        reinterpret_cast<E *>(a.y), a.ckpt, a.T, a.D, a.N, a.K, sp.cps * a.K, sp.cps, maps,
        a.proj, tma_wait_limit(), tma_skip_item());
    return cudaGetLastError();
}

template <bool VEC, bool BULK, bool TMA, bool PROJ, typename E = float>
static cudaError_t launch_fwd_s16_p(const FwdArgs &a, const FwdMaps &maps, SegPlan sp,
                                    cudaStream_t stream)
{
    if (sp.S > 1) return launch_fwd_s16_q<VEC, BULK, TMA, PROJ, true, E>(a, maps, sp, stream);
    return launch_fwd_s16_q<VEC, BULK, TMA, PROJ, false, E>(a, maps, sp, stream);
}

// local end states and decay products of segments 0..S-2, then the chain
static cudaError_t fwd_s16_segments(const FwdArgs &a, SegPlan sp, cudaStream_t stream)
{
    if (sp.S <= 1) return cudaSuccess;
    const int nchunk = (a.T + a.K - 1) / a.K;
    SegLocalArgs la{a.x, a.dt, a.aneg, a.B, a.ckpt, a.ckpt, a.Bt, a.T, a.D, a.N, sp.cps * a.K,
                    0, sp.S - 1, nchunk, sp.cps, sp.cps - 1, sp.cps - 2, a.proj, a.bf16};
    cudaError_t e = launch_seg_local(la, false, stream);
    if (e != cudaSuccess) return e;
    return launch_seg_combine_fwd(a.ckpt, a.Bt, nchunk, sp.S, sp.cps, (size_t)a.D * a.N, stream);
}

template <bool VEC, bool BULK, bool TMA>
static cudaError_t launch_fwd_s16_vb(const FwdArgs &a, const FwdMaps &maps, cudaStream_t stream)
{
    const SegPlan sp = seg_plan_s16(a.Bt, a.T, a.D, a.K);
    const cudaError_t e = fwd_s16_segments(a, sp, stream);
    if (e != cudaSuccess) return e;
    return a.proj.on ? launch_fwd_s16_p<VEC, BULK, TMA, true>(a, maps, sp, stream)
                     : launch_fwd_s16_p<VEC, BULK, TMA, false>(a, maps, sp, stream);
}

#ifndef MMS_FWD_BULK
#define MMS_FWD_BULK 1
#endif
#ifndef MMS_FWD_TMA
#define MMS_FWD_TMA 1
#endif

static bool fwd_maps(const FwdArgs &a, FwdMaps *m)
{
    const auto fn = tma_encoder();
    if (!fn || !tma_context()) return false;
    const cuuint64_t dX[3] = {(cuuint64_t)a.D, (cuuint64_t)a.T, (cuuint64_t)a.Bt};
    const cuuint32_t bX[3] = {S16_DPB, S16_TT, 1};
    const cuuint64_t dB[3] = {(cuuint64_t)a.N, (cuuint64_t)a.T, (cuuint64_t)a.Bt};
    const cuuint32_t bB[3] = {16, S16_TT, 1};
    const int ex = a.bf16 ? 2 : 4;
    const int nchunk = (a.T + a.K - 1) / a.K;
    const cuuint64_t dK[4] = {(cuuint64_t)a.N, (cuuint64_t)a.D, (cuuint64_t)nchunk, (cuuint64_t)a.Bt};
    const cuuint32_t bK[4] = {16, S16_DPB, 1, 1};
    return tma_encode(fn, &m->ck, a.ckpt, 4, dK, bK, 4, CU_TENSOR_MAP_SWIZZLE_64B) &&
           tma_encode(fn, &m->y, a.y, 3, dX, bX, ex) &&
           tma_encode(fn, &m->x, a.x, 3, dX, bX, ex) && tma_encode(fn, &m->dt, a.dt, 3, dX, bX, ex) &&
           tma_encode(fn, &m->B, a.B, 3, dB, bB) && tma_encode(fn, &m->C, a.C, 3, dB, bB);
}

static cudaError_t launch_fwd_s16(const FwdArgs &a, cudaStream_t stream)
{
    // The bulk-store path needs 16-byte aligned y rows (D % 4 == 0, aligned y)
    // and suits strides K >= 8 (at most two checkpoints per 16-step tile); the
    // TMA-staged variant of it also needs the tensor maps to encode.
    FwdMaps maps;
    memset(&maps, 0, sizeof(maps));
    if (!vec_ok(a.D, a.x, a.dt)) return launch_fwd_s16_vb<false, false, false>(a, maps, stream);
    if (MMS_FWD_BULK && a.K >= 8 && vec_ok(a.D, a.y, a.y)) {
        if (MMS_FWD_TMA && fwd_maps(a, &maps))
            return launch_fwd_s16_vb<true, true, true>(a, maps, stream);
        return launch_fwd_s16_vb<true, true, false>(a, maps, stream);
    }
    return launch_fwd_s16_vb<true, false, false>(a, maps, stream);
}

int fwd_take_timeout()
{
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_fwd_timeout, sizeof(v)) != cudaSuccess) return -1;
    if (v) {
        const unsigned int z = 0;
        cudaMemcpyToSymbol(g_fwd_timeout, &z, sizeof(z));
    }
    return v ? 1 : 0;
}

template <int G, bool VEC, bool PROJ, typename E = float>
static cudaError_t launch_fwd_gvp(const FwdArgs &a, cudaStream_t stream)
{
    using S = FwdShape<G>;
    cudaError_t e = smem_opt_in<fwd_kernel<G, VEC, PROJ, E>>(S::SMEM);
    if (e != cudaSuccess) return e;
    const SegPlan sp = seg_plan(a.Bt, a.T, a.D, a.N, a.K, false);
    const int nchunk = (a.T + a.K - 1) / a.K;
    const int L = sp.cps * a.K;
    if (sp.S > 1) {
        // local end states and decay products of segments 0..S-2, then the chain
        SegLocalArgs la{a.x, a.dt, a.aneg, a.B, a.ckpt, a.ckpt, a.Bt, a.T, a.D, a.N, L, 0,
                        sp.S - 1, nchunk, sp.cps, sp.cps - 1, sp.cps - 2, a.proj, a.bf16};
        if ((e = launch_seg_local(la, false, stream)) != cudaSuccess) return e;
        if ((e = launch_seg_combine_fwd(a.ckpt, a.Bt, nchunk, sp.S, sp.cps, (size_t)a.D * a.N,
                                        stream)) != cudaSuccess)
            return e;
    }
    dim3 grid((a.D + S::DPB - 1) / S::DPB, a.Bt, sp.S);
    fwd_kernel<G, VEC, PROJ, E><<<grid, FWD_THREADS, S::SMEM, stream>>>(
        reinterpret_cast<const E *>(a.x), reinterpret_cast<const E *>(a.dt), a.aneg, a.B, a.C,
        reinterpret_cast<E *>(a.y), a.ckpt, a.T, a.D, a.N, a.K, L, sp.cps, a.proj);
    return cudaGetLastError();
}

template <int G, bool VEC>
static cudaError_t launch_fwd_gv(const FwdArgs &a, cudaStream_t stream)
{
    return a.proj.on ? launch_fwd_gvp<G, VEC, true>(a, stream) : launch_fwd_gvp<G, VEC, false>(a, stream);
}

template <int G>
static cudaError_t launch_fwd_g(const FwdArgs &a, cudaStream_t stream)
{
    return vec_ok(a.D, a.x, a.dt) ? launch_fwd_gv<G, true>(a, stream)
                                  : launch_fwd_gv<G, false>(a, stream);
}

// bf16 channel arrays (D % 8 == 0, 16-byte aligned x, dt, y): for 8 < N <= 16
// and K >= 8 the whole-state kernel with TMA staging and bulk y stores (by the
// fp32 rule: enough channels, or both kernels segmented), else the G-lane
// kernel with 16-byte cp.async staging.
static cudaError_t launch_fwd_bf16(const FwdArgs &a, cudaStream_t stream)
{
    using BF = __nv_bfloat16;
    if (a.D % 8 != 0 || a.proj.on || !vec_ok(a.D, a.x, a.dt) || !vec_ok(a.D, a.y, a.y))
        return cudaErrorInvalidValue;
    if (groups_for(a.N) == 4 && a.K >= 8 &&
        ((long long)a.Bt * a.D >= S16_MIN_CHANNELS ||
         (seg_plan_s16(a.Bt, a.T, a.D, a.K).S > 1 && seg_plan(a.Bt, a.T, a.D, a.N, a.K, false).S > 1))) {
        FwdMaps maps;
        memset(&maps, 0, sizeof(maps));
        if (!fwd_maps(a, &maps)) return cudaErrorInvalidValue;
        const SegPlan sp = seg_plan_s16(a.Bt, a.T, a.D, a.K);
        const cudaError_t e = fwd_s16_segments(a, sp, stream);
        if (e != cudaSuccess) return e;
        return launch_fwd_s16_p<true, true, true, false, BF>(a, maps, sp, stream);
    }
    switch (groups_for(a.N)) {
    case 1: return launch_fwd_gvp<1, true, false, BF>(a, stream);
    case 2: return launch_fwd_gvp<2, true, false, BF>(a, stream);
    case 4: return launch_fwd_gvp<4, true, false, BF>(a, stream);
    case 8: return launch_fwd_gvp<8, true, false, BF>(a, stream);
    case 16: return launch_fwd_gvp<16, true, false, BF>(a, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_fwd(const FwdArgs &a, cudaStream_t stream)
{
    if (a.bf16) return launch_fwd_bf16(a, stream);
    // Whole-state kernel: with enough channels to fill the GPU, or when both
    // kernels would need time segments (few channels, long sequences; then it
    // needs 16-byte rows for its TMA / bulk path). In between, the G-lane
    // kernel fills the GPU without segments and runs 7-15 % faster than the
    // segmented whole-state one (B4 T4096 D4096: 569 vs 615 us).
    if (groups_for(a.N) == 4 &&
        ((long long)a.Bt * a.D >= S16_MIN_CHANNELS ||
         (seg_plan_s16(a.Bt, a.T, a.D, a.K).S > 1 && seg_plan(a.Bt, a.T, a.D, a.N, a.K, false).S > 1 &&
          a.K >= 8 && vec_ok(a.D, a.x, a.dt) && vec_ok(a.D, a.y, a.y))))
        return launch_fwd_s16(a, stream);
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
