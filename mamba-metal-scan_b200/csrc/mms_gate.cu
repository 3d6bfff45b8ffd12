// Gate epilogue of the Mamba block, fused into one kernel each way (sm_100a).
//
// The reference block ends with PyTorch ops on the scan output y
// (mamba_metal/model.py:255-256):
//     out = (y + D_skip) * silu(z),       silu(z) = z * sigmoid(z)
// which run as separate elementwise passes over (B, T, D) tensors forward and
// more of them backward. Here:
//   forward   one pass: read y, z, write out                (12 bytes/element)
//   backward  one pass: read dout, y, z, write dy, dz       (20 bytes/element)
//             dy = dout * silu(z)
//             dz = dout * (y + D) * sigmoid(z) * (1 + z * (1 - sigmoid(z)))
//             dD = sum over (b, t) of dy, as fixed-order partial sums over
//                  row blocks (workspace) and a second pass over the blocks.
// z may be a strided view (row stride ldz >= D), as the block's z is the
// second half of in_proj's output. Both are bound by HBM. A thread owns 4 consecutive channels (float4 when
// D % 4 == 0 and the pointers are 16-byte aligned) and walks rows; a warp
// covers 128 consecutive channels of a row, so every access is coalesced.
#include "mms_common.cuh"
#include "mms_kernels.h"

namespace mms {

namespace {

constexpr int GATE_THREADS = 256;
constexpr int GATE_ROWS = 8;           // rows (b, t) per backward block, at least
constexpr int GATE_BWD_WAVE = 5;       // backward blocks resident per SM (48 registers a thread)

// Rows per backward block: as few as fill one wave of GATE_BWD_WAVE blocks
// per SM across the grid's channel blocks (a thread keeps 3 arrays x 4 rows
// of loads in flight, enough to stream HBM at that occupancy), at least
// GATE_ROWS, and enough that the blocks fit grid.y.
long long rows_per_block(long long rows, int D)
{
    const long long gx = ((D + 3) / 4 + GATE_THREADS - 1) / GATE_THREADS;
    long long by = (long long)N_SM * GATE_BWD_WAVE / gx;
    if (by < 1) by = 1;
    long long r = (rows + by - 1) / by;
    if (r < GATE_ROWS) r = GATE_ROWS;
    const long long lim = (rows + 65534) / 65535;
    return r > lim ? r : lim;
}

__device__ __forceinline__ float silu_of(float z, float &sig) {
    sig = sigmoid_fast(z);
    return z * sig;
}

template <bool VEC>
__global__ void __launch_bounds__(GATE_THREADS)
gate_fwd_kernel(const float *__restrict__ y, const float *__restrict__ z,
                const float *__restrict__ dskip, float *__restrict__ out, long long rows, int D,
                long long ldz)
{
    const int nq = (D + 3) / 4;                            // channel quads per row
    const long long total = rows * nq;
    for (long long i = (long long)blockIdx.x * GATE_THREADS + threadIdx.x; i < total;
         i += (long long)gridDim.x * GATE_THREADS) {
        const long long r = i / nq;
        const int d = (int)(i - r * nq) * 4;
        const size_t o = (size_t)r * D + d, oz = (size_t)r * ldz + d;
        if (VEC) {
            const float4 yv = ld4(y + o), zv = ld4(z + oz), dv = ld4(dskip + d);
            float s;
            float4 w;
            w.x = (yv.x + dv.x) * silu_of(zv.x, s);
            w.y = (yv.y + dv.y) * silu_of(zv.y, s);
            w.z = (yv.z + dv.z) * silu_of(zv.z, s);
            w.w = (yv.w + dv.w) * silu_of(zv.w, s);
            st4(out + o, w);
        } else {
            for (int k = 0; k < 4 && d + k < D; ++k) {
                float s;
                out[o + k] = (y[o + k] + dskip[d + k]) * silu_of(z[oz + k], s);
            }
        }
    }
}

// grid: (ceil(nq / 256), ceil(rows / rpb)); each thread: 4 channels x rpb
// rows, writing its dD partial for row block blockIdx.y.
template <bool VEC>
__global__ void __launch_bounds__(GATE_THREADS)
gate_bwd_kernel(const float *__restrict__ dout, const float *__restrict__ y,
                const float *__restrict__ z, const float *__restrict__ dskip,
                float *__restrict__ dy, float *__restrict__ dz, float *__restrict__ part,
                long long rows, int D, long long rpb, long long ldz)
{
    const int nq = (D + 3) / 4;
    const int q = blockIdx.x * GATE_THREADS + threadIdx.x;
    if (q >= nq) return;
    const int d = 4 * q;
    const long long r0 = (long long)blockIdx.y * rpb;
    const long long r1 = r0 + rpb < rows ? r0 + rpb : rows;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float dv[4];
    for (int k = 0; k < 4; ++k) dv[k] = d + k < D ? dskip[d + k] : 0.f;
#pragma unroll 4
    for (long long r = r0; r < r1; ++r) {
        const size_t o = (size_t)r * D + d, ozz = (size_t)r * ldz + d;
        float g[4], yy[4], zz[4];
        if (VEC) {
            const float4 a = ld4(dout + o), b = ld4(y + o), c = ld4(z + ozz);
            g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w;
            yy[0] = b.x; yy[1] = b.y; yy[2] = b.z; yy[3] = b.w;
            zz[0] = c.x; zz[1] = c.y; zz[2] = c.z; zz[3] = c.w;
        } else {
            for (int k = 0; k < 4; ++k) {
                const bool ok = d + k < D;
                g[k] = ok ? dout[o + k] : 0.f;
                yy[k] = ok ? y[o + k] : 0.f;
                zz[k] = ok ? z[ozz + k] : 0.f;
            }
        }
        float oy[4], oz[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float s;
            const float sl = silu_of(zz[k], s);
            oy[k] = g[k] * sl;
            oz[k] = g[k] * (yy[k] + dv[k]) * (s * (1.f + zz[k] * (1.f - s)));
            acc[k] += oy[k];
        }
        if (VEC) {
            st4(dy + o, make_float4(oy[0], oy[1], oy[2], oy[3]));
            st4(dz + o, make_float4(oz[0], oz[1], oz[2], oz[3]));
        } else {
            for (int k = 0; k < 4 && d + k < D; ++k) {
                dy[o + k] = oy[k];
                dz[o + k] = oz[k];
            }
        }
    }
    float *pp = part + (size_t)blockIdx.y * D + d;
    for (int k = 0; k < 4 && d + k < D; ++k) pp[k] = acc[k];
}

__global__ void gate_reduce_kernel(const float *__restrict__ part, float *__restrict__ dd,
                                   int nblk, int D)
{
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < D; d += gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int k = 0; k < nblk; ++k) s += part[(size_t)k * D + d];
        dd[d] = s;
    }
}

int grid_for(long long work)
{
    const long long b = (work + GATE_THREADS - 1) / GATE_THREADS;
    return (int)(b < (long long)N_SM * 16 ? b : (long long)N_SM * 16);
}

}  // namespace

size_t gate_workspace_bytes(long long rows, int D)
{
    const long long rpb = rows_per_block(rows, D);
    const long long nblk = (rows + rpb - 1) / rpb;
    return (size_t)nblk * D * sizeof(float);
}

cudaError_t launch_gate_fwd(const float *y, const float *z, long long ldz, const float *dskip,
                            float *out, long long rows, int D, cudaStream_t stream)
{
    const long long work = rows * ((D + 3) / 4);
    if (vec_ok(D, y, z, out) && vec_ok(D, dskip, dskip) && ldz % 4 == 0)
        gate_fwd_kernel<true><<<grid_for(work), GATE_THREADS, 0, stream>>>(y, z, dskip, out, rows, D,
                                                                            ldz);
    else
        gate_fwd_kernel<false><<<grid_for(work), GATE_THREADS, 0, stream>>>(y, z, dskip, out, rows,
                                                                             D, ldz);
    return cudaGetLastError();
}

cudaError_t launch_gate_bwd(const float *dout, const float *y, const float *z, long long ldz,
                            const float *dskip, float *dy, float *dz, float *dd, void *workspace,
                            long long rows, int D, cudaStream_t stream)
{
    float *part = static_cast<float *>(workspace);
    const int nq = (D + 3) / 4;
    const long long rpb = rows_per_block(rows, D);
    const long long nblk = (rows + rpb - 1) / rpb;
    dim3 grid((nq + GATE_THREADS - 1) / GATE_THREADS, (unsigned)nblk);
    if (vec_ok(D, dout, y, z) && vec_ok(D, dy, dz, dskip) && ldz % 4 == 0)
        gate_bwd_kernel<true><<<grid, GATE_THREADS, 0, stream>>>(dout, y, z, dskip, dy, dz, part,
                                                                  rows, D, rpb, ldz);
    else
        gate_bwd_kernel<false><<<grid, GATE_THREADS, 0, stream>>>(dout, y, z, dskip, dy, dz, part,
                                                                   rows, D, rpb, ldz);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    gate_reduce_kernel<<<(D + 255) / 256, 256, 0, stream>>>(part, dd, (int)nblk, D);
    return cudaGetLastError();
}

}  // namespace mms
