/*
 * mms_scan.h -- C ABI of the B200 (sm_100a) selective-scan library
 * (libmms_scan.so, built from mamba-metal-scan_b200/csrc).
 *
 * The scan (reference: Anamaya1729/mamba-metal-scan, mamba_metal/scan.py:13-34):
 *
 *     dA[t,d,n] = exp(-dt[t,d] * Aneg[d,n])
 *     h[t,d,n]  = dA[t,d,n] * h[t-1,d,n] + dt[t,d] * B[t,n] * x[t,d]     h[-1] = 0
 *     y[t,d]    = sum_n C[t,n] * h[t,d,n]
 *
 * Layouts (all float32, C-contiguous, device pointers):
 *     x, dt, y, dy, dx, ddt   (Bt, T, D)
 *     Aneg, dAneg             (D, N)
 *     B, C, dB, dC            (Bt, T, N)
 *     ckpt                    (Bt, ceil(T/K), D, N): h at the end of every K-step
 *                             chunk; the last one is h at t = T-1.
 *
 * Conventions shared by every entry point:
 *   - The caller owns all memory. The library never allocates device memory;
 *     the backward's scratch is a caller-provided workspace whose size comes
 *     from mms_bwd_workspace_size().
 *   - Every output is fully written (no accumulation into caller memory, no
 *     pre-zeroing needed).
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = the legacy default
 *     stream) and runs asynchronously; nothing synchronises.
 *   - The return value is an MMS_* status. Argument errors are detected before
 *     anything is launched. Results are deterministic: no floating-point
 *     atomics anywhere, fixed reduction order.
 *   - Supported shapes: N a multiple of 4 with 4 <= N <= 64, K >= 1,
 *     Bt, D >= 1, T >= 1. B, C, Aneg, ckpt, dB, dC, dAneg must be 16-byte
 *     aligned (row strides are then 16-byte multiples because N % 4 == 0);
 *     x, dt, y, dy, dx, ddt need 4-byte alignment.
 *   - Stateless and reentrant, calls on different streams may overlap, with
 *     two exceptions: mms_bwd_noalloc() shares one static scratch array
 *     between all its calls (overlapping calls race), and the test hook
 *     mms_debug_set_wait() changes a process-wide setting.
 */
#ifndef MMS_SCAN_H
#define MMS_SCAN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MMS_OK 0
#define MMS_ERR_INVALID_ARG 1      /* a size, stride or pointer is out of range        */
#define MMS_ERR_UNSUPPORTED_N 2    /* N is not a multiple of 4 in [4, 64]              */
#define MMS_ERR_WORKSPACE 3        /* workspace NULL or smaller than required           */
#define MMS_ERR_MISALIGNED 4       /* a pointer violates the alignment rules above      */
#define MMS_ERR_CUDA 5             /* a kernel launch failed (see cudaGetLastError)      */
#define MMS_ERR_TOO_LARGE 6        /* mms_bwd_noalloc: the shape needs more scratch than
                                      MMS_NOALLOC_SCRATCH_BYTES                          */
#define MMS_ERR_TIMEOUT 7          /* a kernel gave up waiting for its own staged copies
                                      (reported by mms_device_status)                    */
#define MMS_ERR_UNSUPPORTED_BF16 8 /* the bf16 entry points need D % 8 == 0, and K == 8
                                      for the backward                                   */

/* Version of the ABI in this header (major * 100 + minor). */
#define MMS_ABI_VERSION 105
int mms_abi_version(void);

/* Human-readable text for an MMS_* status. Never NULL. */
const char *mms_status_string(int status);

/* The CUDA runtime's text for the error behind the calling thread's most
 * recent MMS_ERR_CUDA ("no error" if there was none). Never NULL. */
const char *mms_last_cuda_error(void);

/*
 * Forward scan: writes y and ckpt.
 * Replaces the reference's `lib.ssm_fwd(x, dt, aneg, b_in, c_in, y, ckpt,
 * bt, t_len, d, chunk, ...)` launch (mamba_metal/scan.py:376-378; kernel
 * ssm_fwd at scan.py:78-127), including the checkpoint layout (:120-125).
 */
int mms_fwd(const float *x, const float *dt, const float *aneg,
            const float *B, const float *C,
            float *y, float *ckpt,
            int Bt, int T, int D, int N, int K, void *stream);

/*
 * Forward scan with the model's _proj prologue fused in (reference
 * mamba_metal/model.py:191-201, which computes these with PyTorch ops before
 * calling the scan):
 *     dt   = dt_min + (dt_max - dt_min) * sigmoid(dt_logit)      (Bt, T, D)
 *     Aneg = softplus(a_param)                                    (D, N)
 * Otherwise exactly mms_fwd(). Needs finite dt_min < dt_max.
 * No counterpart in the reference.
 */
int mms_fwd_proj(const float *x, const float *dt_logit, const float *a_param,
                 const float *B, const float *C, float dt_min, float dt_max,
                 float *y, float *ckpt,
                 int Bt, int T, int D, int N, int K, void *stream);

/*
 * Bytes of device workspace mms_bwd() needs for this shape.
 * Replaces the reference's process-global (B, K, D, N) scratch buffer
 * (`_get_scratch`, mamba_metal/scan.py:293-308), which the caller now owns.
 */
size_t mms_bwd_workspace_size(int Bt, int T, int D, int N, int K);

/*
 * Backward scan: from dy and the forward's ckpt, writes dx, ddt, dAneg, dB, dC.
 * Replaces the reference's `lib.ssm_bwd(x, dt, aneg, b_in, c_in, dy, dx, ddt,
 * dAneg, dB, dC, ckpt, scratch, bt, t_len, d, chunk, ...)` launch
 * (mamba_metal/scan.py:406-410; kernel ssm_bwd at scan.py:132-261). Unlike the
 * reference, dAneg/dB/dC need no zero-fill: they are written, not accumulated.
 * `workspace` must hold mms_bwd_workspace_size() bytes, 256-byte aligned.
 */
int mms_bwd(const float *x, const float *dt, const float *aneg,
            const float *B, const float *C, const float *dy, const float *ckpt,
            float *dx, float *ddt, float *daneg, float *dB, float *dC,
            void *workspace, size_t workspace_bytes,
            int Bt, int T, int D, int N, int K, void *stream);

/*
 * Backward of mms_fwd_proj(): gradients with respect to x, dt_logit, a_param,
 * B and C (d_dt_logit = ddt * dsigmoid, d_a_param = dAneg * sigmoid(a_param)).
 * Same workspace as mms_bwd() (mms_bwd_workspace_size), ckpt from
 * mms_fwd_proj(). No counterpart in the reference.
 */
int mms_bwd_proj(const float *x, const float *dt_logit, const float *a_param,
                 const float *B, const float *C, const float *dy, const float *ckpt,
                 float dt_min, float dt_max,
                 float *dx, float *d_dt_logit, float *d_a_param, float *dB, float *dC,
                 void *workspace, size_t workspace_bytes,
                 int Bt, int T, int D, int N, int K, void *stream);

/*
 * Backward scan that allocates nothing, for callers that cannot allocate
 * device memory at run time (a plugin inside a host framework that has
 * reserved all GPU memory and forbids further cudaMalloc, or a latency-bound
 * path that cannot afford cudaMalloc's implicit device synchronisation).
 * No counterpart in the reference: it is mms_bwd() with its workspace taken
 * from MMS_NOALLOC_SCRATCH_BYTES of static device memory compiled into the
 * library, held by every GPU that loads the library until the process exits.
 *  - Shapes with mms_bwd_workspace_size() > MMS_NOALLOC_SCRATCH_BYTES return
 *    MMS_ERR_TOO_LARGE (nothing is launched).
 *  - The first call on a device looks the scratch address up (cudaGetSymbolAddress,
 *    with that device current); make that first call before any stream capture.
 *    The address is kept for the life of the process and is valid while the
 *    device's primary context lives: after cudaDeviceReset() (or anything
 *    else that destroys that context) do not call mms_bwd_noalloc again in the
 *    same process.
 *  - All calls share the one scratch array: calls that overlap on the GPU
 *    (other streams, unordered host threads) race and must be serialised.
 *    Nothing in it needs clearing between calls.
 * Other arguments, outputs and status codes are those of mms_bwd().
 */
#define MMS_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int mms_bwd_noalloc(const float *x, const float *dt, const float *aneg,
                    const float *B, const float *C, const float *dy, const float *ckpt,
                    float *dx, float *ddt, float *daneg, float *dB, float *dC,
                    int Bt, int T, int D, int N, int K, void *stream);

/*
 * One recurrent (decode) step on a cached state, in place:
 *     h[b,d,n] = exp(-dt[b,d] * Aneg[d,n]) * h[b,d,n] + dt[b,d] * B[b,n] * x[b,d]
 *     y[b,d]   = sum_n C[b,n] * h[b,d,n]            (with the updated h)
 * Layouts: x, dt, y (Bt, D); B, C (Bt, N); Aneg (D, N); h (Bt, D, N), which
 * is the layout of ckpt's last chunk, so the forward's final checkpoint can
 * be the cache. h must not overlap any other argument. Alignment and N rules
 * as above (h: 16 bytes).
 * Replaces the reference's per-token torch ops on cache["h"]
 * (mamba_metal/model.py:228-241), which have no kernel of their own there.
 */
int mms_step(const float *x, const float *dt, const float *aneg,
             const float *B, const float *C, float *h, float *y,
             int Bt, int D, int N, void *stream);

/*
 * Gate epilogue of the Mamba block, one kernel each way (reference
 * mamba_metal/model.py:255-256 runs it as separate PyTorch ops):
 *     out = (y + d_skip) * silu(z),   silu(z) = z * sigmoid(z)
 * y, out, dout, dy, dz are (Bt, T, D) contiguous; z is (Bt, T, D) with row
 * stride ldz >= D elements (the block's z is a half of in_proj's output);
 * d_skip, d_dskip are (D,).
 * mms_gate_bwd writes dy = dout * silu(z), dz = dout * (y + d_skip) * silu'(z)
 * and d_dskip = sum over (Bt, T) of dy (fixed order, through a caller
 * workspace of mms_gate_workspace_size() bytes, 16-byte aligned).
 * No counterpart in the reference.
 */
size_t mms_gate_workspace_size(int Bt, int T, int D);
int mms_gate_fwd(const float *y, const float *z, long long ldz, const float *d_skip,
                 float *out, int Bt, int T, int D, void *stream);
int mms_gate_bwd(const float *dout, const float *y, const float *z, long long ldz,
                 const float *d_skip, float *dy, float *dz, float *d_dskip,
                 void *workspace, size_t workspace_bytes,
                 int Bt, int T, int D, void *stream);

/*
 * The scan with bf16 storage for the (Bt, T, D) channel arrays: x, dt and y
 * (forward), dy, dx and ddt (backward) hold bf16 bit patterns (uint16_t);
 * Aneg, dAneg, B, C, dB, dC and ckpt stay float32, and every sum, product
 * and exponential is computed in float32 as in mms_fwd / mms_bwd. Outputs
 * are rounded to bf16 once, at the store. Halves the bytes of the six
 * arrays that dominate the traffic.
 * Shapes: every N of mms_fwd / mms_bwd; D % 8 == 0, and K == 8 for the
 * backward (any K for the forward); otherwise MMS_ERR_UNSUPPORTED_BF16. The
 * bf16 arrays must be 16-byte aligned. Workspace as mms_bwd (same size
 * function).
 * No counterpart in the reference, which is float32-only
 * (mamba_metal/scan.py:350-354).
 */
int mms_fwd_bf16(const uint16_t *x, const uint16_t *dt, const float *aneg,
                 const float *B, const float *C, uint16_t *y, float *ckpt,
                 int Bt, int T, int D, int N, int K, void *stream);
int mms_bwd_bf16(const uint16_t *x, const uint16_t *dt, const float *aneg,
                 const float *B, const float *C, const uint16_t *dy, const float *ckpt,
                 uint16_t *dx, uint16_t *ddt, float *daneg, float *dB, float *dC,
                 void *workspace, size_t workspace_bytes,
                 int Bt, int T, int D, int N, int K, void *stream);

/*
 * Device-side status of the kernels launched so far, for failure detection.
 * The backward's TMA staging waits on completion barriers with a bounded
 * poll; a wait that runs out records a flag instead of hanging the GPU (the
 * results of that call are then wrong). Returns MMS_ERR_TIMEOUT if the flag
 * was set since the previous call (and clears it), MMS_ERR_CUDA if it cannot
 * be read, else MMS_OK. Synchronises the device.
 * No counterpart in the reference (its Metal launches cannot time out).
 */
int mms_device_status(void);

/*
 * Test hook for the failure detection above, process-wide, read by every
 * later launch of the TMA-staged backward: `polls` is how often a thread
 * polls a stage's completion barrier before the kernel gives up (0 restores
 * the default, 2^22); `skip_item` >= 0 makes every CTA withhold the copies of
 * its staged item number `skip_item` (-1: none), so that its wait runs out
 * without any fault: the CTAs leave together after their other copies have
 * landed, the outputs of that call are invalid, and mms_device_status()
 * reports MMS_ERR_TIMEOUT. Not for concurrent use with production calls.
 * No counterpart in the reference.
 */
int mms_debug_set_wait(unsigned int polls, int skip_item);

/*
 * Pipe-throughput probe, for the roofline the benchmark reports (the scan is
 * bound by HBM bytes or by its exp2 count at the MUFU rate; this measures
 * that rate on the GPU in use). Launches `blocks` CTAs of 256 threads, each
 * thread running 8 independent chains of one operation for 2*iters rounds;
 * per CTA it writes the elapsed SM clock cycles to cycles[cta] and the SM it
 * ran on to sm[cta]. Operations per CTA: mms_probe_ops_per_cta(kind, iters)
 * (thread-level; a packed FFMA2 counts as two FMAs). Keep blocks <= 4 per SM
 * so every CTA is resident at once. `sink` needs 256 floats (never written in
 * practice). No counterpart in the reference.
 */
#define MMS_PROBE_EX2 0        /* ex2.approx.ftz.f32 (MUFU)                        */
#define MMS_PROBE_FFMA 1       /* fp32 fused multiply-add                          */
#define MMS_PROBE_FFMA2 2      /* packed fp32 pair FMA (two lanes per instruction)  */
#define MMS_PROBE_SHFL 3       /* warp shuffle (plus one fp32 add)                  */
#define MMS_PROBE_EX2_POLY 4   /* the library's FMA-pipe exp2 polynomial            */
#define MMS_PROBE_EX2_POLY2 5  /* the same on packed pairs                          */
int mms_probe_pipe(int kind, int iters, int blocks, float *sink, long long *cycles,
                   unsigned *sm, void *stream);
long long mms_probe_ops_per_cta(int kind, int iters);

/*
 * y[i] = 2^x[i] for n floats (device pointers) by one of the library's exp2
 * paths: kind 0 MUFU ex2.approx.ftz, 1 the FMA-pipe polynomial the forward
 * uses for a share of its decays, 2 the same on packed pairs. For the
 * accuracy tests of the polynomial. No counterpart in the reference.
 */
int mms_probe_exp2(const float *x, float *y, long long n, int kind, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MMS_SCAN_H */
