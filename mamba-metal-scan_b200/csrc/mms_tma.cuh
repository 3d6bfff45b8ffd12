// TMA (Tensor Memory Accelerator) staging helpers for sm_100a.
//
// Device side: mbarrier completion barriers and tile loads from a tensor map
// into this CTA's shared memory (never with cluster multicast). Host side:
// fp32 tile maps encoded through the driver entry point, so the library has
// no link-time dependency on libcuda.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace mms {

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// TMA tile loads (no multicast) that complete on an mbarrier.
__device__ __forceinline__ void tma3(uint32_t dst, const CUtensorMap *m, int c0, int c1, int c2,
                                     uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4}], [%5];\n"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tma4(uint32_t dst, const CUtensorMap *m, int c0, int c1, int c2,
                                     int c3, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4, %5}], [%6];\n"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
                   "r"(bar)
                 : "memory");
}

// TMA tile store of a 4-D box from this CTA's shared memory to global memory,
// tracked by the bulk-group commit / wait of bulk_store. Every coordinate is
// non-negative; elements of the box outside the tensor are not written.
__device__ __forceinline__ void tma_store3(const CUtensorMap *m, uint32_t src, int c0, int c1,
                                           int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group"
                 " [%0, {%1, %2, %3}], [%4];\n"
                 ::"l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(src)
                 : "memory");
}
__device__ __forceinline__ void tma_store4(const CUtensorMap *m, uint32_t src, int c0, int c1,
                                           int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group"
                 " [%0, {%1, %2, %3, %4}], [%5];\n"
                 ::"l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(src)
                 : "memory");
}

inline PFN_cuTensorMapEncodeTiled_v12000 tma_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// cuTensorMapEncodeTiled fails (on every map) when the calling thread has no
// current CUDA context, which is the case on a thread that has made no CUDA
// runtime call yet (PyTorch's autograd worker, for one). Make the current
// device's primary context current first; cheap when it already is.
inline bool tma_context()
{
    int dev = 0;
    return cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess;
}

// Tile map over a row-major array of fp32 (elem 4) or bf16 (elem 2) whose
// innermost `rank` dims are `dim` (dim[0] contiguous), box `box`;
// out-of-range elements load as zeros. `swz` is the shared-memory layout of a
// box (CU_TENSOR_MAP_SWIZZLE_64B: the 16-byte piece j of 64-byte row r sits
// at piece j ^ ((r >> 1) & 3), on a 1024-byte aligned box).
inline bool tma_encode(PFN_cuTensorMapEncodeTiled_v12000 fn, CUtensorMap *m, const void *base, int rank,
            const cuuint64_t *dim, const cuuint32_t *box, int elem = 4,
            CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_NONE)
{
    cuuint64_t stride[4];
    cuuint64_t s = (cuuint64_t)elem;
    for (int i = 0; i + 1 < rank; ++i) {
        s *= dim[i];
        stride[i] = s;
    }
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUtensorMapDataType ty = elem == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    return fn(m, ty, rank, const_cast<void *>(base), dim, stride, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace mms
