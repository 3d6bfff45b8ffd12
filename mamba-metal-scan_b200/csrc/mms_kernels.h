// Internal launcher interface between the C ABI (mms_api.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>

namespace mms {

// The fused _proj prologue (reference mamba_metal/model.py:191-201): when
// `on`, the dt argument holds logits z and the aneg argument holds the raw
// parameter A, and the kernels use
//     dt = lo + range * sigmoid(z),     Aneg = softplus(A),
// returning gradients with respect to z and A.
struct Proj {
    int on;
    float lo, range;
    float inv_range;            // 1 / range
};

// The prologue's d dt / d logit = range * s * (1 - s) with s the sigmoid,
// written from dt = lo + range * s.
__device__ __forceinline__ float dt_slope(const Proj &pj, float dtv) {
    return (dtv - pj.lo) * (pj.lo + pj.range - dtv) * pj.inv_range;
}

// bf16 != 0: the (B, T, D) channel arrays (x, dt, y; dy, dx, ddt) hold bf16
// values (the pointers are passed through as float * and reinterpreted by
// the launchers); everything else stays fp32.
struct FwdArgs {
    const float *x, *dt, *aneg, *B, *C;
    float *y, *ckpt;
    int Bt, T, D, N, K;
    Proj proj;
    int bf16;
};

struct BwdArgs {
    const float *x, *dt, *aneg, *B, *C, *dy, *ckpt;
    float *dx, *ddt, *daneg, *dB, *dC;
    void *workspace;
    int Bt, T, D, N, K;
    Proj proj;
    int bf16;
};

struct StepArgs {
    const float *x, *dt, *aneg, *B, *C;
    float *h, *y;
    int Bt, D, N;
};

// Opt a kernel into `bytes` of dynamic shared memory once per device: the
// setting persists, and repeating it on every launch costs a driver call.
// KERNEL is the kernel's address, so every kernel has its own flags.
template <auto KERNEL>
inline cudaError_t smem_opt_in(size_t bytes)
{
    static std::atomic<unsigned long long> done{0};         // one bit per device (< 64)
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(KERNEL, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_release);
    return e;
}

// Lanes per channel: ceil(N/4) rounded up to a power of two (N in [4, 64]).
inline int groups_for(int N)
{
    const int q = (N + 3) / 4;
    int g = 1;
    while (g < q) g <<= 1;
    return g;
}

// Time segments. A CTA of the G-lane kernels covers 256/G channels of one batch
// row; when batch rows x channel blocks cannot fill the 148 SMs (long
// sequences with few channels per GPU), the sequence is also cut into S
// segments of `cps` checkpoint chunks (L = cps*K steps) that run in parallel.
// A segment's entry state (forward) or adjoint carry (backward) comes from a
// local pass over the other segments plus a sequential combine over S:
//     state entering s+1 = P_s * (state entering s) + h_s
// with h_s the segment's end state from a zero start and
// P_s = prod over the segment of exp(-dt*Aneg) = exp(-Aneg * sum dt).
// The forward and backward use the same plan (it depends on the shape only).
constexpr int N_SM = 148;

struct SegPlan {
    int S;      // segments (1: no split)
    int cps;    // checkpoint chunks per segment
};

// Stride 8 at 8 < N <= 16 on the channel-pair backward (1) or on the
// 8-state one (0). The channel-pair kernel measured 5-6 % faster at configs
// 1, 3a and 4 and 9-17 % on config 4's 2- and 4-way d_inner shards (6 %
// slower on its 8-way shard).
#ifndef MMS_BWD_CP_K8
#define MMS_BWD_CP_K8 1
#endif
// The channel-pair backward with 2 states per thread (256-thread CTAs) up to
// this N (at most 32), else 4 states per thread (128-thread CTAs).
#ifndef MMS_BWD_CP2_MAXN
#define MMS_BWD_CP2_MAXN 0
#endif

// The shapes of the 8-state backward (mms_bwd_w8.cu): 8 < N <= 16, K == 8.
// With MMS_BWD_CP_K8 it runs them only where the channel-pair kernel cannot
// (channel arrays not 16-byte aligned).
inline bool w8_shape(int N, int K) { return groups_for(N) == 4 && N > 8 && K == 8; }
inline bool w8_first(int N, int K) { return w8_shape(N, K) && !MMS_BWD_CP_K8; }
// The shapes of the channel-pair backward (mms_bwd_cp.cu): 8 < N <= 64,
// K a multiple of 8 up to 64, except those the 8-state kernel takes first.
inline bool cp_shape(int N, int K) { return N > 8 && N <= 64 && K % 8 == 0 && K <= 64 && !w8_first(N, K); }
inline bool cp_two_states(int N) { return N <= MMS_BWD_CP2_MAXN && N <= 32; }
// The lane widths (groups_for(N): bit 4, 8, 16) at which the channel-pair
// backward runs 256-thread CTAs (1 per SM) instead of 128-thread CTAs (2 per
// SM): the same CTA slots, twice the channels per CTA, half the per-CTA
// dB|dC partials. Default: 16 (32 < N <= 64).
#ifndef MMS_BWD_CP_WIDE
#define MMS_BWD_CP_WIDE 16
#endif

// Bounded waits of the TMA-staged kernels: polls of one stage's completion
// barrier before a kernel gives up (default 2^22), and a staged item whose
// copies are withheld (-1: none). Both are test hooks set through
// mms_debug_set_wait (mms_api.cu); launchers read them at launch.
uint32_t tma_wait_limit();
int tma_skip_item();

// `backward`: the plan of the backward, else of the G-lane forward. The two
// may differ: a backward segment starts from the forward's checkpoint at its
// first chunk, whatever segments the forward ran.
inline SegPlan seg_plan(int Bt, int T, int D, int N, int K, bool backward)
{
    const int dpb = 256 / groups_for(N);
    const long long base = (long long)Bt * ((D + dpb - 1) / dpb);
    const int nchunk = (T + K - 1) / K;
    SegPlan p{1, nchunk};
    // Segments for one whole wave of the backward: the 8-state kernel runs 4
    // CTAs per SM, the channel-pair and 4-state kernels 2. More segments than
    // one wave holds only add local-pass work. The forward at stride 8 and
    // 8 < N <= 16 plans for 4 per SM whichever backward runs (measured at
    // config 3a: 378 us against 469 us with the 2-per-SM plan).
    const bool s8 = groups_for(N) == 4 && N > 8 && K == 8;
    const long long per_sm = backward ? (w8_first(N, K) ? 4 : 2) : (s8 ? 4 : 2);
    // Splitting costs a local pass over S-1 segments (about 40 % more work for
    // a fwd+bwd step), which pays only when the batch rows x channel blocks
    // leave SMs idle: below one CTA per SM, and for the 8-state backward (4
    // per SM) below half a wave (measured at B4 T4096 D4096: 1528 us split in
    // two against 1735 us unsplit; the forward there loses by splitting).
    const long long min_base = backward && per_sm == 4 ? 2 * N_SM : N_SM;
    if (base >= min_base) return p;
    const long long want = (per_sm * N_SM) / base;
    long long cps = (nchunk + want - 1) / want;
    if (cps < 2) cps = 2;                           // the forward keeps P_s in chunk cps-2
    if (cps * K < 64) cps = (64 + K - 1) / K;       // at least 64 steps per segment
    const long long S = (nchunk + cps - 1) / cps;
    if (S < 2) return p;
    p.S = (int)S;
    p.cps = (int)cps;
    return p;
}

// 16-byte staging of (T, D) channel arrays is possible when every row starts
// 16-byte aligned: D % 4 == 0 and 16-byte aligned base pointers.
inline bool vec_ok(int D, const void *p0, const void *p1, const void *p2 = nullptr)
{
    auto al = [](const void *p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return D % 4 == 0 && al(p0) && al(p1) && al(p2);
}

// Workspace layout of the backward (byte offsets from the workspace base,
// every region 256-byte aligned).
struct BwdWorkspace {
    size_t part_bc;    // (Bt, nblk, T, 2N) per-CTA partial sums of dB|dC over its channels
    size_t part_a;     // (Bt*S, D, N) per-(batch row, time segment) partial sums of dAneg
    size_t subck;      // (Bt*S, nseg, D, N) segment-start states inside long chunks
    size_t seg_e;      // (Bt, S, D, N) adjoint carries of the time segments (S > 1)
    size_t seg_p;      // (Bt, S, D, N) decay products of the time segments (S > 1)
    size_t total;
    int nblk;          // CTAs along D
    int nseg;          // segments per chunk (1 when K <= segment length)
    SegPlan plan;      // time segments
};

BwdWorkspace bwd_workspace_layout(int Bt, int T, int D, int N, int K);

// Segment passes (mms_seg.cu). `u` is x (forward) or dy (backward), `row` is
// B (forward) or C (backward); segments s_first .. s_first+nseg-1 are scanned
// from a zero start and their end value / decay product stored at
// (b*bplanes + s*splanes + off) * D*N in vout / pout.
struct SegLocalArgs {
    const float *u, *dt, *aneg, *row;
    float *vout, *pout;
    int Bt, T, D, N, L, s_first, nseg, bplanes, splanes, voff, poff;
    Proj proj;
    int bf16;          // u and dt hold bf16
};
cudaError_t launch_seg_local(const SegLocalArgs &a, bool backward, cudaStream_t stream);

// Backward with 8 states per lane (mms_bwd_w8.cu) for 8 < N <= 16 and K == 8
// where the channel-pair backward does not run (see w8_first); same
// workspace regions as the general backward.
bool bwd_w8_applies(int N, int K);
cudaError_t launch_bwd_w8(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                          int nblk, SegPlan sp, cudaStream_t stream);
// 1 if a TMA-stage wait timed out since the last call (and clears it), 0 if
// not, -1 if the flag could not be read.
int w8_take_timeout();

// Backward on channel pairs (mms_bwd_cp.cu) for cp_shape() with TMA-ready
// arrays (D % 4 == 0 and 16-byte aligned; bf16: D % 8 == 0, no prologue);
// same workspace regions as the general backward. Its CTAs cover
// cp_channels_per_cta(N) channels, at least the general kernel's 256 /
// groups_for(N), so its per-CTA dB|dC partials fit the workspace;
// *nblk_used receives how many CTAs along D wrote them.
bool bwd_cp_applies(const BwdArgs &a);
int cp_channels_per_cta(int N);
cudaError_t launch_bwd_cp(const BwdArgs &a, float *part_bc, float *part_a, const float *seg_e,
                          SegPlan sp, cudaStream_t stream, int *nblk_used);
int cp_take_timeout();

// Gate epilogue out = (y + D_skip) * silu(z) (mms_gate.cu); rows = Bt * T.
size_t gate_workspace_bytes(long long rows, int D);
cudaError_t launch_gate_fwd(const float *y, const float *z, long long ldz, const float *dskip,
                            float *out, long long rows, int D, cudaStream_t stream);
cudaError_t launch_gate_bwd(const float *dout, const float *y, const float *z, long long ldz,
                            const float *dskip, float *dy, float *dz, float *dd, void *workspace,
                            long long rows, int D, cudaStream_t stream);
int fwd_take_timeout();
// forward: chain the segment end states through the checkpoint slots
cudaError_t launch_seg_combine_fwd(float *ckpt, int Bt, int nchunk, int S, int cps, size_t DN,
                                   cudaStream_t stream);
// backward: chain the adjoint carries in place; afterwards E[b, s] is the carry into segment s
cudaError_t launch_seg_combine_bwd(float *E, const float *P, int Bt, int S, size_t DN,
                                   cudaStream_t stream);

cudaError_t launch_fwd(const FwdArgs &a, cudaStream_t stream);
cudaError_t launch_bwd(const BwdArgs &a, cudaStream_t stream);
cudaError_t launch_step(const StepArgs &a, cudaStream_t stream);

}  // namespace mms
