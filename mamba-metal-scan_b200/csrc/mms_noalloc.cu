// mms_bwd_noalloc: the backward scan for callers that cannot allocate device
// memory at run time.
//
// mms_bwd() needs a caller-provided workspace (per-CTA partial sums of dB/dC,
// per-row partials of dAneg, segment-start states of long chunks). Some
// callers cannot get one: a plugin living inside a host framework that has
// reserved all device memory up front and forbids further cudaMalloc, or a
// latency-critical path where cudaMalloc's implicit device-wide
// synchronisation is not acceptable. For them this entry point uses a scratch
// array compiled into the library instead: MMS_NOALLOC_SCRATCH_BYTES (16 MiB)
// of static device memory that every GPU which loads the library keeps until
// the process exits. Shapes whose workspace would exceed it are rejected.
//
// Host code cannot use the array's name as a device address (it names a
// host-side stand-in), so the device address is looked up once per device
// with cudaGetSymbolAddress, with that device current, on the first call made
// on it; make that first call before any stream capture.
//
// Every call shares the one array and it keeps whatever the last call left
// there. The backward writes every workspace word it later reads, so nothing
// needs clearing; but calls that overlap on the GPU (different streams, or
// different host threads without ordering) race on the array and must be
// serialised by the caller.
#include <mutex>

#include "mms_kernels.h"
#include "mms_scan.h"

namespace {

constexpr size_t kScratchBytes = MMS_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_lock;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of g_scratch on the current device, looked up once per device.
cudaError_t scratch_address(void **out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> guard(g_lock);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int mms_bwd_noalloc(const float *x, const float *dt, const float *aneg,
                               const float *B, const float *C, const float *dy,
                               const float *ckpt, float *dx, float *ddt, float *daneg,
                               float *dB, float *dC, int Bt, int T, int D, int N, int K,
                               void *stream)
{
    const size_t need = mms_bwd_workspace_size(Bt, T, D, N, K);
    if (need == 0) {
        // mms_bwd_workspace_size() answers 0 only for invalid shapes: let
        // mms_bwd report which one, without touching the GPU.
        return mms_bwd(x, dt, aneg, B, C, dy, ckpt, dx, ddt, daneg, dB, dC, nullptr, 0, Bt, T,
                       D, N, K, stream);
    }
    if (need > kScratchBytes) return MMS_ERR_TOO_LARGE;
    void *ws = nullptr;
    if (scratch_address(&ws) != cudaSuccess) return MMS_ERR_CUDA;
    return mms_bwd(x, dt, aneg, B, C, dy, ckpt, dx, ddt, daneg, dB, dC, ws, kScratchBytes, Bt, T,
                   D, N, K, stream);
}
