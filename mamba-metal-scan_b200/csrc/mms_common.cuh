// Shared device helpers for the sm_100a selective-scan kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MMS_LOG2E 1.4426950408889634f

namespace mms {

// 2^x on the MUFU pipe (ex2.approx.ftz.f32). The scan feeds it -dt*Aneg*log2(e),
// which is <= 0, so the result lies in [0, 1]; flushing denormal results to
// zero only affects states that have already decayed below 1e-38.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Same, but never merged with an identical ex2 elsewhere: used where a decay
// is deliberately recomputed instead of being kept in a register.
__device__ __forceinline__ float ex2_fresh(float x) {
    float y;
    asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x on the FMA pipe, for moving a share of the scan's exponentials off
// MUFU. Cody and Waite's argument reduction, 2^x = 2^j * 2^f with j = round(x)
// and f = x - j in [-1/2, 1/2] (both exact in fp32), and 2^f ~ p(f) =
// 1 + f*q(f), q of degree 4 with coefficients from the minimax fit in
// csrc/exp2_fit.py (max relative error of the fp32 evaluation 1.7e-7, about
// 1.4 ulp; ex2.approx.ftz is of the same order). j is read from the low
// mantissa bits of x + 1.5*2^23 and added to p's exponent field. x is clamped
// to [-125, 125], so results below 2^-125 are not flushed to zero like
// ex2.approx.ftz does, and arguments above 125 saturate instead of
// overflowing; the scan's decays have x = -dt*Aneg*log2(e) <= 0.
constexpr float EXP2_RND = 12582912.f;                 // 1.5 * 2^23
constexpr float EXP2_C1 = 0x1.62e42ap-1f, EXP2_C2 = 0x1.ebf9bcp-3f, EXP2_C3 = 0x1.c6b752p-5f,
                EXP2_C4 = 0x1.3cea7cp-7f, EXP2_C5 = 0x1.5bb9f8p-10f;

__device__ __forceinline__ float ex2_poly(float x) {
    x = fminf(fmaxf(x, -125.f), 125.f);
    const float t = x + EXP2_RND;
    const float f = x - (t - EXP2_RND);
    float p = fmaf(EXP2_C5, f, EXP2_C4);
    p = fmaf(p, f, EXP2_C3);
    p = fmaf(p, f, EXP2_C2);
    p = fmaf(p, f, EXP2_C1);
    p = fmaf(p, f, 1.f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// sigmoid(z) = 1 / (1 + 2^(-z*log2 e)); saturates to 0 / 1 for large |z|.
// The reciprocal is MUFU's (rcp.approx, about 1 ulp; 1/inf = 0, so a large
// negative z gives 0).
__device__ __forceinline__ float sigmoid_fast(float z) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + ex2(-z * MMS_LOG2E)));
    return r;
}

// softplus(a) = log(1 + e^a), = a once e^a dwarfs 1 in fp32.
__device__ __forceinline__ float softplus(float a) {
    return a > 20.f ? a : log1pf(expf(a));
}

// Storage element of the (B, T, D) channel arrays: float, or bf16 for the
// bf16 entry points (the arithmetic is fp32 either way).
__device__ __forceinline__ float to_f(float v) { return v; }
// bf16 to fp32 is exact: the bf16 bits become the top half of the fp32 word.
__device__ __forceinline__ float to_f(__nv_bfloat16 v) {
    return __uint_as_float((uint32_t)__bfloat16_as_ushort(v) << 16);
}
template <typename E>
__device__ __forceinline__ E from_f(float v) {
    if constexpr (sizeof(E) == 4) return v;
    else return __float2bfloat16_rn(v);
}

__device__ __forceinline__ float4 ld4(const float *p) {
    return __ldg(reinterpret_cast<const float4 *>(p));
}

__device__ __forceinline__ void st4(float *p, float4 v) {
    *reinterpret_cast<float4 *>(p) = v;
}

__device__ __forceinline__ float comp(const float4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Packed fp32 pairs: sm_100's FFMA2/FMUL2/FADD2 do two lanes of work per issue.
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 ex2x2(float2 v) { return f2(ex2(v.x), ex2(v.y)); }

// ex2_poly on a pair, the polynomial on packed FFMA2 (same results as two
// ex2_poly calls: every packed operation rounds each lane as the scalar one).
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
    x = f2(fminf(fmaxf(x.x, -125.f), 125.f), fminf(fmaxf(x.y, -125.f), 125.f));
    const float2 t = add2(x, f2(EXP2_RND, EXP2_RND));
    const float2 j = add2(t, f2(-EXP2_RND, -EXP2_RND));
    const float2 f = fma2(j, f2(-1.f, -1.f), x);
    float2 p = fma2(f2(EXP2_C5, EXP2_C5), f, f2(EXP2_C4, EXP2_C4));
    p = fma2(p, f, f2(EXP2_C3, EXP2_C3));
    p = fma2(p, f, f2(EXP2_C2, EXP2_C2));
    p = fma2(p, f, f2(EXP2_C1, EXP2_C1));
    p = fma2(p, f, f2(1.f, 1.f));
    return f2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
              __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}
__device__ __forceinline__ float2 lo(float4 v) { return f2(v.x, v.y); }
__device__ __forceinline__ float2 hi(float4 v) { return f2(v.z, v.w); }

// Transposed butterfly reduction over the lanes selected by lane-bit masks
// MASK_HI, MASK_HI/2, ..., MASK_LO (powers of two). Each lane starts with NV
// values v[0..NV); lanes that differ only in those bits hold partials of the
// same NV sums. At each level a lane keeps half of its values (the upper half
// if its mask bit is set) and adds the partner's copy of that half, so the
// work per lane is NV-1 shuffles instead of NV*levels. When a lane is down to
// one value the remaining levels are plain xor-reductions.
//
// On return v[0..nleft) hold complete sums; `first` is the index of v[0] in
// the original numbering. nleft = max(1, NV >> levels).
template <int NV, int MASK_HI, int MASK_LO>
__device__ __forceinline__ void transposed_reduce(float (&v)[NV], int lane, int &first) {
    first = 0;
    int cur = NV;
#pragma unroll
    for (int m = MASK_HI; m >= MASK_LO && m > 0; m >>= 1) {
        if (cur > 1) {
            const int half = cur >> 1;
            const bool upper = (lane & m) != 0;
#pragma unroll
            for (int i = 0; i < NV / 2; ++i) {
                if (i < half) {
                    const float send = upper ? v[i] : v[i + half];
                    const float keep = upper ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
                }
            }
            if (upper) first += half;
            cur = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
        }
    }
}

}  // namespace mms
