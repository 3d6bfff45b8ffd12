// Pipe-throughput probes: how many operations of one kind an SM completes per
// clock, measured on the SM's own cycle counter.
//
// The scan's roofline is the slower of HBM bytes and its exp2 count at the
// MUFU rate; this measures that rate (and the FP32, packed-FP32, shuffle and
// FMA-pipe exp2 rates the kernels trade it against) on the GPU in use, so
// the roofline does not rest on a datasheet figure.
//
// Each thread runs PROBE_CHAINS independent dependency chains of one
// operation for `iters` rounds between two clock64() reads taken after a
// barrier; every CTA records its cycle count and its SM. Operations per SM
// per clock = (operations of the CTAs on that SM) / (longest CTA on it); the
// host takes the median over SMs. All CTAs of the grid are resident at once
// (4 CTAs of 256 threads per SM, few registers).
#include <stdint.h>

#include "mms_common.cuh"
#include "mms_scan.h"

namespace mms {
namespace {

constexpr int PROBE_THREADS = 256;
constexpr int PROBE_CHAINS = 8;

__device__ __forceinline__ unsigned smid() {
    unsigned s;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(s));
    return s;
}

template <int KIND>
__device__ __forceinline__ void probe_round(float (&v)[PROBE_CHAINS], int i) {
#pragma unroll
    for (int k = 0; k < PROBE_CHAINS; ++k) {
        if constexpr (KIND == MMS_PROBE_EX2) {
            v[k] = ex2_fresh(-v[k]);                              // stays in [1/2, 1]
        } else if constexpr (KIND == MMS_PROBE_FFMA) {
            v[k] = fmaf(v[k], 0.999f, 1e-4f);
        } else if constexpr (KIND == MMS_PROBE_SHFL) {
            v[k] = __shfl_xor_sync(0xffffffffu, v[k], 1 << ((k + i) % 5)) + 1.f;
        } else if constexpr (KIND == MMS_PROBE_EX2_POLY) {
            v[k] = ex2_poly(-v[k]);
        }
    }
}

template <int KIND>
__global__ void __launch_bounds__(PROBE_THREADS)
probe_kernel(float *sink, long long *cycles, unsigned *sm, int iters)
{
    float v[PROBE_CHAINS];
#pragma unroll
    for (int k = 0; k < PROBE_CHAINS; ++k) v[k] = 0.5f + 0.01f * (float)((threadIdx.x + k) & 15);
    __syncthreads();
    const long long c0 = clock64();
    if constexpr (KIND == MMS_PROBE_FFMA2 || KIND == MMS_PROBE_EX2_POLY2) {
        float2 w[PROBE_CHAINS / 2];
#pragma unroll
        for (int k = 0; k < PROBE_CHAINS / 2; ++k) w[k] = f2(v[2 * k], v[2 * k + 1]);
        for (int i = 0; i < iters; ++i) {
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int k = 0; k < PROBE_CHAINS / 2; ++k) {
                    if constexpr (KIND == MMS_PROBE_FFMA2)
                        w[k] = fma2(w[k], f2(0.999f, 0.999f), f2(1e-4f, 1e-4f));
                    else
                        w[k] = ex2_poly2(f2(-w[k].x, -w[k].y));
                }
        }
#pragma unroll
        for (int k = 0; k < PROBE_CHAINS / 2; ++k) {
            v[2 * k] = w[k].x;
            v[2 * k + 1] = w[k].y;
        }
    } else {
        for (int i = 0; i < iters; ++i) {
            probe_round<KIND>(v, i);
            probe_round<KIND>(v, i + 1);
        }
    }
    __syncthreads();
    const long long c1 = clock64();
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < PROBE_CHAINS; ++k) s += v[k];
    if (s == -1.f) sink[threadIdx.x] = s;                        // keeps the chains live
    if (threadIdx.x == 0) {
        cycles[blockIdx.x] = c1 - c0;
        sm[blockIdx.x] = smid();
    }
}

// y[i] = 2^x[i] by MUFU ex2.approx.ftz (kind 0), the FMA-pipe polynomial
// (kind 1) or its packed-pair form (kind 2, pairs (x[2j], x[2j+1])).
__global__ void exp2_kernel(const float *__restrict__ x, float *__restrict__ y, long long n, int kind)
{
    const long long i = 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= n) return;
    const float a = x[i], b = i + 1 < n ? x[i + 1] : 0.f;
    float2 r;
    if (kind == 0) r = f2(ex2_fresh(a), ex2_fresh(b));
    else if (kind == 1) r = f2(ex2_poly(a), ex2_poly(b));
    else r = ex2_poly2(f2(a, b));
    y[i] = r.x;
    if (i + 1 < n) y[i + 1] = r.y;
}

}  // namespace
}  // namespace mms

extern "C" int mms_probe_exp2(const float *x, float *y, long long n, int kind, void *stream)
{
    if (!x || !y || n < 0 || kind < 0 || kind > 2) return MMS_ERR_INVALID_ARG;
    if (n == 0) return MMS_OK;
    const long long threads = (n + 1) / 2;
    mms::exp2_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, y, n, kind);
    return cudaGetLastError() == cudaSuccess ? MMS_OK : MMS_ERR_CUDA;
}

extern "C" int mms_probe_pipe(int kind, int iters, int blocks, float *sink, long long *cycles,
                              unsigned *sm, void *stream)
{
    using namespace mms;
    if (iters < 1 || blocks < 1 || !sink || !cycles || !sm) return MMS_ERR_INVALID_ARG;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (kind) {
    case MMS_PROBE_EX2: probe_kernel<MMS_PROBE_EX2><<<blocks, PROBE_THREADS, 0, s>>>(sink, cycles, sm, iters); break;
    case MMS_PROBE_FFMA: probe_kernel<MMS_PROBE_FFMA><<<blocks, PROBE_THREADS, 0, s>>>(sink, cycles, sm, iters); break;
    case MMS_PROBE_FFMA2: probe_kernel<MMS_PROBE_FFMA2><<<blocks, PROBE_THREADS, 0, s>>>(sink, cycles, sm, iters); break;
    case MMS_PROBE_SHFL: probe_kernel<MMS_PROBE_SHFL><<<blocks, PROBE_THREADS, 0, s>>>(sink, cycles, sm, iters); break;
    case MMS_PROBE_EX2_POLY: probe_kernel<MMS_PROBE_EX2_POLY><<<blocks, PROBE_THREADS, 0, s>>>(sink, cycles, sm, iters); break;
    case MMS_PROBE_EX2_POLY2: probe_kernel<MMS_PROBE_EX2_POLY2><<<blocks, PROBE_THREADS, 0, s>>>(sink, cycles, sm, iters); break;
    default: return MMS_ERR_INVALID_ARG;
    }
    return cudaGetLastError() == cudaSuccess ? MMS_OK : MMS_ERR_CUDA;
}

// Operations one probe launch performs per CTA (thread-level operations; a
// packed FFMA2 counts as two FMAs, an exp2 pair as two exp2).
extern "C" long long mms_probe_ops_per_cta(int kind, int iters)
{
    if (iters < 1) return 0;
    switch (kind) {
    case MMS_PROBE_EX2:
    case MMS_PROBE_FFMA:
    case MMS_PROBE_SHFL:
    case MMS_PROBE_EX2_POLY:
    case MMS_PROBE_FFMA2:
    case MMS_PROBE_EX2_POLY2:
        return 2LL * iters * mms::PROBE_CHAINS * mms::PROBE_THREADS;
    default: return 0;
    }
}
