// Internal launcher interface between the C ABI (mms_api.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mms {

struct FwdArgs {
    const float *x, *dt, *aneg, *B, *C;
    float *y, *ckpt;
    int Bt, T, D, N, K;
};

struct BwdArgs {
    const float *x, *dt, *aneg, *B, *C, *dy, *ckpt;
    float *dx, *ddt, *daneg, *dB, *dC;
    void *workspace;
    int Bt, T, D, N, K;
};

struct StepArgs {
    const float *x, *dt, *aneg, *B, *C;
    float *h, *y;
    int Bt, D, N;
};

// Lanes per channel: ceil(N/4) rounded up to a power of two (N in [4, 64]).
inline int groups_for(int N)
{
    const int q = (N + 3) / 4;
    int g = 1;
    while (g < q) g <<= 1;
    return g;
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
    size_t part_a;     // (Bt, D, N) per-batch-row partial sums of dAneg
    size_t subck;      // (Bt, nseg, D, N) segment-start states inside long chunks
    size_t total;
    int nblk;          // CTAs along D
    int nseg;          // segments per chunk (1 when K <= segment length)
};

BwdWorkspace bwd_workspace_layout(int Bt, int T, int D, int N, int K);

cudaError_t launch_fwd(const FwdArgs &a, cudaStream_t stream);
cudaError_t launch_bwd(const BwdArgs &a, cudaStream_t stream);
cudaError_t launch_step(const StepArgs &a, cudaStream_t stream);

}  // namespace mms
