// Asynchronous global->shared staging of time tiles (cp.async, sm_80+ ISA,
// also the cheapest per-thread async copy on sm_100a). Every copy carries a
// source size, so rows past T, channels past D and states past N arrive as
// zeros and the compute loops need no bounds checks.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mms {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte copy; zero-fills the destination when !valid (src is then not read).
__device__ __forceinline__ void cp16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)),
                 "l"(src), "r"(valid ? 16 : 0));
}

// 4-byte copy; zero-fills the destination when !valid.
__device__ __forceinline__ void cp4(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_u32(dst)),
                 "l"(src), "r"(valid ? 4 : 0));
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }

template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Asynchronous shared -> global copy on the bulk-copy (TMA) engine, no tensor
// map: both addresses 16-byte aligned, bytes a multiple of 16. The issuing
// thread continues at once; smem written by ordinary stores must be published
// to the async proxy first (fence_async_smem by the writers, then a barrier).
__device__ __forceinline__ void bulk_store(void *gdst, const void *ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n"
                 ::"l"(gdst), "r"(smem_u32(ssrc)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// Wait until at most N committed groups are still reading their smem sources.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
// Wait until at most N committed groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait() { asm volatile("cp.async.bulk.wait_group %0;\n" ::"n"(N) : "memory"); }
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// Copy `rows` consecutive time steps [t0, t0+rows) of NARR channel arrays
// (each (T, D) row-major, already offset to the batch row) and of NBC state
// arrays (each (T, N), fp32) into a tile laid out per step as
//     [arr0[DPB] arr1[DPB] ... arr{NARR-1}[DPB] bc0[NPAD] bc1[NPAD] ...]
// (ROWF floats per step). The channel arrays keep their storage type E
// (float, or bf16 whose NARR*DPB elements then take NARR*DPB/2 floats of the
// row). Steps >= nvalid, channels >= D - d0 and states >= N are zero-filled.
// VEC selects 16-byte copies for the channel arrays, which needs every row
// 16-byte aligned (D a multiple of 16/sizeof(E), aligned arrays; checked by
// the host); bf16 arrays are always staged that way.
//
// The arrays are passed as separate pointers (a2 unused when NARR == 2) and
// picked by value, so no pointer table lands in local memory.
template <int NARR, int DPB, typename E>
struct TileRow {
    static constexpr int CHF = NARR * DPB * (int)sizeof(E) / 4;   // floats of the channel arrays
};

template <int NARR, int NBC, int DPB, int NPAD, int ROWS, int NTHREADS, bool VEC, typename E = float>
__device__ __forceinline__ void stage_tile(float *tile, const E *a0, const E *a1, const E *a2,
                                           const float *b0, const float *b1,
                                           int t0, int nvalid, int d0, int D, int N, int tid)
{
    static_assert(VEC || sizeof(E) == 4, "bf16 channel arrays are staged in 16-byte pieces");
    auto arr = [&](int a) { return a == 0 ? a0 : (a == 1 || NARR == 2) ? a1 : a2; };
    auto bc = [&](int a) { return a == 0 || NBC == 1 ? b0 : b1; };
    constexpr int CHF = TileRow<NARR, DPB, E>::CHF;
    constexpr int ROWF = CHF + NBC * NPAD;
    const int dleft = D - d0;
    if constexpr (VEC) {
        constexpr int EPV = 16 / (int)sizeof(E);         // elements per 16-byte copy
        constexpr int QD = DPB / EPV;                    // copies per channel row
        constexpr int TOT = NARR * ROWS * QD;
        for (int k = tid; k < TOT; k += NTHREADS) {
            const int a = k / (ROWS * QD);
            const int r = (k / QD) % ROWS;
            const int q = k % QD;
            const bool ok = r < nvalid && EPV * q < dleft;
            const E *src = ok ? arr(a) + (size_t)(t0 + r) * D + d0 + EPV * q : arr(a);
            cp16(reinterpret_cast<E *>(tile + r * ROWF) + a * DPB + EPV * q, src, ok);
        }
    } else {
        constexpr int TOT = NARR * ROWS * DPB;
        for (int k = tid; k < TOT; k += NTHREADS) {
            const int a = k / (ROWS * DPB);
            const int r = (k / DPB) % ROWS;
            const int q = k % DPB;
            const bool ok = r < nvalid && q < dleft;
            const float *src = ok ? arr(a) + (size_t)(t0 + r) * D + d0 + q : arr(a);
            cp4(tile + r * ROWF + a * DPB + q, src, ok);
        }
    }
    constexpr int QN = NPAD / 4;
    constexpr int TOTN = NBC * ROWS * QN;
    for (int k = tid; k < TOTN; k += NTHREADS) {
        const int a = k / (ROWS * QN);
        const int r = (k / QN) % ROWS;
        const int q = k % QN;
        const bool ok = r < nvalid && 4 * q < N;
        const float *src = ok ? bc(a) + (size_t)(t0 + r) * N + 4 * q : bc(a);
        cp16(tile + r * ROWF + CHF + a * NPAD + 4 * q, src, ok);
    }
}

}  // namespace mms
