// C ABI of libmms_scan.so (declared in include/mms_scan.h).
//
// Argument checking happens here, before anything is launched, so that a bad
// call returns an MMS_* status instead of reaching a kernel. The checks mirror
// the reference's host-side validation (mamba_metal/scan.py:274-276 for
// d_state, :355-365 for shapes) plus what raw pointers add: alignment and
// NULL checks.
#include <stdint.h>

#include <atomic>

#include "mms_kernels.h"
#include "mms_scan.h"

namespace {

// The CUDA error behind the calling thread's last MMS_ERR_CUDA (mms_last_cuda_error).
thread_local cudaError_t g_last_cuda = cudaSuccess;

int status_of(cudaError_t e)
{
    if (e == cudaSuccess) return MMS_OK;
    g_last_cuda = e;
    return MMS_ERR_CUDA;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int check_shape(int Bt, int T, int D, int N, int K)
{
    if (N < 4 || N > 64 || N % 4 != 0) return MMS_ERR_UNSUPPORTED_N;
    if (Bt < 1 || T < 1 || D < 1 || K < 1) return MMS_ERR_INVALID_ARG;
    if (Bt > 65535) return MMS_ERR_INVALID_ARG;            // grid.y
    return MMS_OK;
}

int fwd_impl(const float *x, const float *dt, const float *aneg, const float *B, const float *C,
             float *y, float *ckpt, int Bt, int T, int D, int N, int K, void *stream,
             mms::Proj proj)
{
    int rc = check_shape(Bt, T, D, N, K);
    if (rc) return rc;
    if (!x || !dt || !aneg || !B || !C || !y || !ckpt) return MMS_ERR_INVALID_ARG;
    if (!aligned(aneg, 16) || !aligned(B, 16) || !aligned(C, 16) || !aligned(ckpt, 16) ||
        !aligned(x, 4) || !aligned(dt, 4) || !aligned(y, 4))
        return MMS_ERR_MISALIGNED;
    mms::FwdArgs a{x, dt, aneg, B, C, y, ckpt, Bt, T, D, N, K, proj, 0};
    return status_of(mms::launch_fwd(a, static_cast<cudaStream_t>(stream)));
}

int bwd_impl(const float *x, const float *dt, const float *aneg, const float *B, const float *C,
             const float *dy, const float *ckpt, float *dx, float *ddt, float *daneg, float *dB,
             float *dC, void *workspace, size_t workspace_bytes, int Bt, int T, int D, int N,
             int K, void *stream, mms::Proj proj)
{
    int rc = check_shape(Bt, T, D, N, K);
    if (rc) return rc;
    if (!x || !dt || !aneg || !B || !C || !dy || !ckpt || !dx || !ddt || !daneg || !dB || !dC)
        return MMS_ERR_INVALID_ARG;
    if (!aligned(aneg, 16) || !aligned(B, 16) || !aligned(C, 16) || !aligned(ckpt, 16) ||
        !aligned(daneg, 16) || !aligned(dB, 16) || !aligned(dC, 16) || !aligned(x, 4) ||
        !aligned(dt, 4) || !aligned(dy, 4) || !aligned(dx, 4) || !aligned(ddt, 4))
        return MMS_ERR_MISALIGNED;
    const size_t need = mms::bwd_workspace_layout(Bt, T, D, N, K).total;
    if (!workspace || workspace_bytes < need) return MMS_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return MMS_ERR_MISALIGNED;
    mms::BwdArgs a{x, dt, aneg, B, C, dy, ckpt, dx, ddt, daneg, dB, dC, workspace,
                   Bt, T, D, N, K, proj, 0};
    return status_of(mms::launch_bwd(a, static_cast<cudaStream_t>(stream)));
}

// Shapes the bf16 entry points cover: bf16 rows staged in 16-byte pieces
// (D % 8 == 0); the backward at checkpoint stride 8 (its 8-step kernels).
int check_bf16(int D, int K, bool backward)
{
    if (D % 8 != 0 || (backward && K != 8)) return MMS_ERR_UNSUPPORTED_BF16;
    return MMS_OK;
}

// pointers carried through the float-typed launcher structs
const float *fp(const uint16_t *p) { return reinterpret_cast<const float *>(p); }
float *fp(uint16_t *p) { return reinterpret_cast<float *>(p); }

// dt = dt_min + (dt_max - dt_min) * sigmoid(logit) needs finite bounds in order.
bool proj_ok(float dt_min, float dt_max)
{
    return dt_min == dt_min && dt_max == dt_max && dt_min > -3.0e38f && dt_max < 3.0e38f &&
           dt_max > dt_min;
}

std::atomic<uint32_t> g_wait_limit{0};
std::atomic<int> g_skip_item{-1};

}  // namespace

namespace mms {
uint32_t tma_wait_limit()
{
    const uint32_t v = g_wait_limit.load(std::memory_order_relaxed);
    return v ? v : (1u << 22);
}
int tma_skip_item() { return g_skip_item.load(std::memory_order_relaxed); }
}  // namespace mms

extern "C" {

int mms_abi_version(void) { return MMS_ABI_VERSION; }

const char *mms_status_string(int status)
{
    switch (status) {
    case MMS_OK: return "ok";
    case MMS_ERR_INVALID_ARG: return "invalid argument (size out of range or NULL pointer)";
    case MMS_ERR_UNSUPPORTED_N: return "unsupported d_state: N must be a multiple of 4 in [4, 64]";
    case MMS_ERR_WORKSPACE: return "workspace missing or smaller than mms_bwd_workspace_size()";
    case MMS_ERR_MISALIGNED: return "misaligned pointer (B, C, Aneg, ckpt, dB, dC, dAneg need 16 bytes)";
    case MMS_ERR_CUDA: return "CUDA call failed (mms_last_cuda_error() names the CUDA error)";
    case MMS_ERR_TIMEOUT: return "a kernel timed out waiting for its staged copies (results invalid)";
    case MMS_ERR_UNSUPPORTED_BF16:
        return "bf16 scan needs D % 8 == 0 (and K == 8 for the backward)";
    case MMS_ERR_TOO_LARGE:
        return "shape needs more workspace than mms_bwd_noalloc's static scratch "
               "(MMS_NOALLOC_SCRATCH_BYTES = 16 MiB); use mms_bwd with a caller workspace";
    default: return "unknown status";
    }
}

int mms_fwd(const float *x, const float *dt, const float *aneg, const float *B, const float *C,
            float *y, float *ckpt, int Bt, int T, int D, int N, int K, void *stream)
{
    return fwd_impl(x, dt, aneg, B, C, y, ckpt, Bt, T, D, N, K, stream, mms::Proj{0, 0.f, 0.f, 0.f});
}

int mms_fwd_proj(const float *x, const float *dt_logit, const float *a_param, const float *B,
                 const float *C, float dt_min, float dt_max, float *y, float *ckpt, int Bt, int T,
                 int D, int N, int K, void *stream)
{
    if (!proj_ok(dt_min, dt_max)) return MMS_ERR_INVALID_ARG;
    return fwd_impl(x, dt_logit, a_param, B, C, y, ckpt, Bt, T, D, N, K, stream,
                    mms::Proj{1, dt_min, dt_max - dt_min, 1.f / (dt_max - dt_min)});
}

size_t mms_bwd_workspace_size(int Bt, int T, int D, int N, int K)
{
    if (check_shape(Bt, T, D, N, K)) return 0;
    return mms::bwd_workspace_layout(Bt, T, D, N, K).total;
}

int mms_bwd(const float *x, const float *dt, const float *aneg, const float *B, const float *C,
            const float *dy, const float *ckpt, float *dx, float *ddt, float *daneg, float *dB,
            float *dC, void *workspace, size_t workspace_bytes, int Bt, int T, int D, int N, int K,
            void *stream)
{
    return bwd_impl(x, dt, aneg, B, C, dy, ckpt, dx, ddt, daneg, dB, dC, workspace, workspace_bytes,
                    Bt, T, D, N, K, stream, mms::Proj{0, 0.f, 0.f, 0.f});
}

int mms_bwd_proj(const float *x, const float *dt_logit, const float *a_param, const float *B,
                 const float *C, const float *dy, const float *ckpt, float dt_min, float dt_max,
                 float *dx, float *d_dt_logit, float *d_a_param, float *dB, float *dC,
                 void *workspace, size_t workspace_bytes, int Bt, int T, int D, int N, int K,
                 void *stream)
{
    if (!proj_ok(dt_min, dt_max)) return MMS_ERR_INVALID_ARG;
    return bwd_impl(x, dt_logit, a_param, B, C, dy, ckpt, dx, d_dt_logit, d_a_param, dB, dC,
                    workspace, workspace_bytes, Bt, T, D, N, K, stream,
                    mms::Proj{1, dt_min, dt_max - dt_min, 1.f / (dt_max - dt_min)});
}

int mms_step(const float *x, const float *dt, const float *aneg, const float *B, const float *C,
             float *h, float *y, int Bt, int D, int N, void *stream)
{
    int rc = check_shape(Bt, 1, D, N, 1);
    if (rc) return rc;
    if ((long long)Bt * D * N > (1LL << 40)) return MMS_ERR_INVALID_ARG;
    if (!x || !dt || !aneg || !B || !C || !h || !y) return MMS_ERR_INVALID_ARG;
    if (!aligned(aneg, 16) || !aligned(B, 16) || !aligned(C, 16) || !aligned(h, 16) ||
        !aligned(x, 4) || !aligned(dt, 4) || !aligned(y, 4))
        return MMS_ERR_MISALIGNED;
    mms::StepArgs a{x, dt, aneg, B, C, h, y, Bt, D, N};
    return status_of(mms::launch_step(a, static_cast<cudaStream_t>(stream)));
}

size_t mms_gate_workspace_size(int Bt, int T, int D)
{
    if (Bt < 1 || T < 1 || D < 1) return 0;
    return mms::gate_workspace_bytes((long long)Bt * T, D);
}

int mms_gate_fwd(const float *y, const float *z, long long ldz, const float *d_skip, float *out,
                 int Bt, int T, int D, void *stream)
{
    if (Bt < 1 || T < 1 || D < 1 || ldz < D || !y || !z || !d_skip || !out)
        return MMS_ERR_INVALID_ARG;
    if (!aligned(y, 4) || !aligned(z, 4) || !aligned(d_skip, 4) || !aligned(out, 4))
        return MMS_ERR_MISALIGNED;
    return status_of(mms::launch_gate_fwd(y, z, ldz, d_skip, out, (long long)Bt * T, D,
                                static_cast<cudaStream_t>(stream)));
}

int mms_gate_bwd(const float *dout, const float *y, const float *z, long long ldz,
                 const float *d_skip, float *dy, float *dz, float *d_dskip, void *workspace,
                 size_t workspace_bytes, int Bt, int T, int D, void *stream)
{
    if (Bt < 1 || T < 1 || D < 1 || ldz < D || !dout || !y || !z || !d_skip || !dy || !dz ||
        !d_dskip)
        return MMS_ERR_INVALID_ARG;
    if (!aligned(dout, 4) || !aligned(y, 4) || !aligned(z, 4) || !aligned(d_skip, 4) ||
        !aligned(dy, 4) || !aligned(dz, 4) || !aligned(d_dskip, 4))
        return MMS_ERR_MISALIGNED;
    if (!workspace || workspace_bytes < mms::gate_workspace_bytes((long long)Bt * T, D))
        return MMS_ERR_WORKSPACE;
    if (!aligned(workspace, 16)) return MMS_ERR_MISALIGNED;
    return status_of(mms::launch_gate_bwd(dout, y, z, ldz, d_skip, dy, dz, d_dskip, workspace,
                                (long long)Bt * T, D, static_cast<cudaStream_t>(stream)));
}

int mms_fwd_bf16(const uint16_t *x, const uint16_t *dt, const float *aneg, const float *B,
                 const float *C, uint16_t *y, float *ckpt, int Bt, int T, int D, int N, int K,
                 void *stream)
{
    int rc = check_shape(Bt, T, D, N, K);
    if (rc) return rc;
    if ((rc = check_bf16(D, K, false))) return rc;
    if (!x || !dt || !aneg || !B || !C || !y || !ckpt) return MMS_ERR_INVALID_ARG;
    if (!aligned(aneg, 16) || !aligned(B, 16) || !aligned(C, 16) || !aligned(ckpt, 16) ||
        !aligned(x, 16) || !aligned(dt, 16) || !aligned(y, 16))
        return MMS_ERR_MISALIGNED;
    mms::FwdArgs a{fp(x), fp(dt), aneg, B, C, fp(y), ckpt, Bt, T, D, N, K, mms::Proj{0, 0.f, 0.f, 0.f}, 1};
    return status_of(mms::launch_fwd(a, static_cast<cudaStream_t>(stream)));
}

int mms_bwd_bf16(const uint16_t *x, const uint16_t *dt, const float *aneg, const float *B,
                 const float *C, const uint16_t *dy, const float *ckpt, uint16_t *dx, uint16_t *ddt,
                 float *daneg, float *dB, float *dC, void *workspace, size_t workspace_bytes,
                 int Bt, int T, int D, int N, int K, void *stream)
{
    int rc = check_shape(Bt, T, D, N, K);
    if (rc) return rc;
    if ((rc = check_bf16(D, K, true))) return rc;
    if (!x || !dt || !aneg || !B || !C || !dy || !ckpt || !dx || !ddt || !daneg || !dB || !dC)
        return MMS_ERR_INVALID_ARG;
    if (!aligned(aneg, 16) || !aligned(B, 16) || !aligned(C, 16) || !aligned(ckpt, 16) ||
        !aligned(daneg, 16) || !aligned(dB, 16) || !aligned(dC, 16) || !aligned(x, 16) ||
        !aligned(dt, 16) || !aligned(dy, 16) || !aligned(dx, 16) || !aligned(ddt, 16))
        return MMS_ERR_MISALIGNED;
    const size_t need = mms::bwd_workspace_layout(Bt, T, D, N, K).total;
    if (!workspace || workspace_bytes < need) return MMS_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return MMS_ERR_MISALIGNED;
    mms::BwdArgs a{fp(x), fp(dt), aneg, B, C, fp(dy), ckpt, fp(dx), fp(ddt), daneg, dB, dC,
                   workspace, Bt, T, D, N, K, mms::Proj{0, 0.f, 0.f, 0.f}, 1};
    return status_of(mms::launch_bwd(a, static_cast<cudaStream_t>(stream)));
}

int mms_device_status(void)
{
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return status_of(e);
    const int t = mms::w8_take_timeout(), f = mms::fwd_take_timeout(), c = mms::cp_take_timeout();
    if (t < 0 || f < 0 || c < 0) return status_of(cudaGetLastError());
    return t || f || c ? MMS_ERR_TIMEOUT : MMS_OK;
}

const char *mms_last_cuda_error(void) { return cudaGetErrorString(g_last_cuda); }

int mms_debug_set_wait(unsigned int polls, int skip_item)
{
    if (skip_item < -1) return MMS_ERR_INVALID_ARG;
    g_wait_limit.store(polls, std::memory_order_relaxed);
    g_skip_item.store(skip_item, std::memory_order_relaxed);
    return MMS_OK;
}

}  // extern "C"
