/*
 * fpa.h -- C ABI of the B200-native First Passage Attention (FPA) operator.
 *
 * FPA is causal softmax attention with the first-passage bias
 *     b_ts = beta_h * min(0, min_{s<u<=t} phi_u - psi_s),   b_tt = 0,
 * whose backward pass takes the gradient of phi through the soft minimum -tau*log sum_{s<u<=t} exp(-phi_u/tau).
 *
 * The library (libfpa_b200.so) is plain C at its boundary: device pointers, element strides, sizes and a
 * cudaStream_t (passed as void*). It never allocates or frees device memory and never synchronises the stream;
 * callers allocate the outputs and a workspace of the size the *_workspace_bytes queries return. All entry points
 * are asynchronous on the given stream and reentrant.
 *
 * The entry points replace the reference implementation's device launches (yliu-fort/first-passage-attention):
 *   fpa_fwd  <- kernel.py:398-412 (`_forward`: `_block_stats` -> `_stats`, then `_fwd`)
 *   fpa_bwd  <- kernel.py:424-451 (`_FirstPassageAttention.backward`: `_bwd_delta`, `_bwd_kv`,
 *               `_bwd_dphi_diag`, `_bwd_q`, `_bwd_dphi`, and the host-side `dbeta.sum((0, 2))`)
 * The argument checks mirror kernel.py:469-488 (see fpa_status_string for the messages).
 */
#ifndef FPA_B200_H
#define FPA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FPA_ABI_VERSION 1

#if defined(__GNUC__)
#define FPA_API __attribute__((visibility("default")))
#else
#define FPA_API
#endif

/* Element type of q, k, v, o, do, dq, dk, dv (kernel.py:471: all fp16 or all fp32). phi, psi, beta, lse, dphi,
 * dpsi and dbeta are always float32. */
enum FpaDtype { FPA_DTYPE_F16 = 0, FPA_DTYPE_F32 = 1 };

/* Which kernels to run. AUTO picks the tensor-core (tcgen05) kernels for fp16 with D <= 128 and the FFMA kernels
   for fp32 and for D = 256. */
enum FpaPath { FPA_PATH_AUTO = 0, FPA_PATH_SIMT = 1, FPA_PATH_TENSOR = 2 };

enum FpaStatus {
  FPA_OK = 0,
  FPA_ERR_INVALID_ARGUMENT = 1, /* shapes, dtypes, null pointers, tau <= 0 (kernel.py:469-486) */
  FPA_ERR_UNSUPPORTED = 2,      /* a valid request that the selected kernels do not cover (e.g. layout for TMA) */
  FPA_ERR_CUDA = 3,             /* a CUDA runtime or driver call failed (launch error, attribute, tensor map) */
  FPA_ERR_TIMEOUT = 4,          /* a bounded device-side wait expired; reported through fpa_workspace_status */
  FPA_ERR_WORKSPACE = 5         /* workspace pointer null, misaligned (256 B) or smaller than required */
};

/* Forward: o = softmax(q k^T / sqrt(D) + bias, causal) v, and lse_t = log2 sum_s exp2(scaled logits), the row
 * statistic the backward pass needs. q, k, v, o: [B, H, T, D] with arbitrary element strides (stride[3] must be 1
 * for the tensor-core path); phi, psi, lse: [B, H, T] contiguous float32; beta: [H] float32. */
typedef struct FpaFwdArgs {
  int32_t dtype;            /* FpaDtype */
  int32_t path;             /* FpaPath */
  int32_t B, H, T, D;       /* D in {16, 32, 64, 128, 256} (kernel.py:476: a power of two >= 16); B, H <= 65535; B*H*T < 2^31 */
  float tau;                /* soft-min temperature, > 0 (enters only the backward pass) */
  const void* q; int64_t q_stride[4];
  const void* k; int64_t k_stride[4];
  const void* v; int64_t v_stride[4];
  const float* phi;         /* [B, H, T] */
  const float* psi;         /* [B, H, T] */
  const float* beta;        /* [H] */
  void* o; int64_t o_stride[4];
  float* lse;               /* [B, H, T], base-2 log-sum-exp of the log2e-scaled logits */
  void* workspace;          /* fpa_fwd_workspace_bytes(...) bytes, 256-byte aligned */
  size_t workspace_bytes;
  int32_t kernels_launched; /* out: number of kernels this call launched */
  int32_t path_taken;       /* out: FPA_PATH_SIMT or FPA_PATH_TENSOR */
} FpaFwdArgs;

/* Backward of sum(o * do): dq, dk, dv in the input dtype ([B, H, T, D], arbitrary strides), dphi and dpsi
 * [B, H, T] float32 contiguous, dbeta [H] float32 summed over the batch (kernel.py:450). Deterministic: repeated
 * calls on the same inputs give bit-identical results (no floating-point atomics). */
typedef struct FpaBwdArgs {
  int32_t dtype;
  int32_t path;
  int32_t B, H, T, D;
  float tau;
  const void* q; int64_t q_stride[4];
  const void* k; int64_t k_stride[4];
  const void* v; int64_t v_stride[4];
  const void* o; int64_t o_stride[4];
  const void* dout; int64_t dout_stride[4];
  const float* lse;         /* as written by fpa_fwd */
  const float* phi;
  const float* psi;
  const float* beta;
  void* dq; int64_t dq_stride[4];
  void* dk; int64_t dk_stride[4];
  void* dv; int64_t dv_stride[4];
  float* dphi;              /* [B, H, T] */
  float* dpsi;              /* [B, H, T] */
  float* dbeta;             /* [H] */
  void* workspace;          /* fpa_bwd_workspace_bytes(...) bytes, 256-byte aligned */
  size_t workspace_bytes;
  int32_t kernels_launched; /* out */
  int32_t path_taken;       /* out */
} FpaBwdArgs;

/* The layer's field (kernel.py:502-509). proj is the fp32 output of the Field's projection, [B, T, 3H] with element
 * strides proj_stride = {b, t, column}: per head h, delta = column h, g = column H + h, hh = column 2H + h. Forward:
 * w_t = sum_{u<=t} delta_u, phi = w + g, psi = w + hh, written to phi, psi [B, H, T] contiguous float32. Backward:
 * from dphi, dpsi [B, H, T] contiguous float32 it writes dproj (same layout as proj, strides dproj_stride):
 * d delta_t = sum_{u>=t} (dphi_u + dpsi_u), dg = dphi, dhh = dpsi. Deterministic (fixed summation order). */
typedef struct FpaFieldArgs {
  int32_t B, T, H;
  const float* proj; int64_t proj_stride[3];
  float* phi;               /* out (forward) */
  float* psi;               /* out (forward) */
  const float* dphi;        /* in (backward) */
  const float* dpsi;        /* in (backward) */
  float* dproj; int64_t dproj_stride[3]; /* out (backward) */
} FpaFieldArgs;

/* ABI version of the loaded library (FPA_ABI_VERSION). */
FPA_API int fpa_abi_version(void);

/* sizeof(FpaFwdArgs) for which == 0, sizeof(FpaBwdArgs) for 1, sizeof(FpaFieldArgs) for 2; lets bindings check their
 * struct mirrors. */
FPA_API size_t fpa_struct_size(int which);

/* Workspace sizes in bytes for a call with these sizes (0 for invalid sizes). Call them with the device that will run
 * the call current: on the tensor-core path, a forward whose grid is too small to fill that device's SMs also gets
 * room for the partial outputs of its key-range split (each query tile's key tiles cut into chunks that run on
 * separate CTAs and are then joined). fpa_fwd also accepts a workspace without that room and then runs unsplit. */
FPA_API size_t fpa_fwd_workspace_bytes(int dtype, int B, int H, int T, int D, int path);
FPA_API size_t fpa_bwd_workspace_bytes(int dtype, int B, int H, int T, int D, int path);

/* Forward pass (replaces kernel.py:398-412). Returns an FpaStatus. */
FPA_API int fpa_fwd(FpaFwdArgs* args, void* stream);

/* Backward pass (replaces kernel.py:424-451). Returns an FpaStatus. */
FPA_API int fpa_bwd(FpaBwdArgs* args, void* stream);

/* Field forward and backward (replace the PyTorch ops of kernel.py:504-509: the fp32 projection's split into
 * delta, g, h, the cumsum and the two additions, and their autograd backward). Return an FpaStatus. */
FPA_API int fpa_field_fwd(const FpaFieldArgs* args, void* stream);
FPA_API int fpa_field_bwd(const FpaFieldArgs* args, void* stream);

/* Synchronises `stream`, then reads and clears the device status word at the head of a workspace that a previous
 * fpa_fwd / fpa_bwd call used: FPA_OK, or FPA_ERR_TIMEOUT if a bounded device-side wait expired in that call. */
FPA_API int fpa_workspace_status(void* workspace, void* stream);

/* Human-readable text for an FpaStatus, or the message of the last argument error on this thread. */
FPA_API const char* fpa_status_string(int status);

/* The message of the last error raised on the calling thread (empty string when none). */
FPA_API const char* fpa_last_error(void);

/* Kernel timing for profiling. While enabled, every kernel that fpa_fwd / fpa_bwd launch is bracketed by CUDA
 * events recorded on the call's stream (this adds event records to the stream; leave it off for production).
 * fpa_profile returns the previous setting. fpa_profile_report synchronises on the recorded events, writes one
 * line "<kernel> <launches> <total ms>" per kernel into buf (NUL-terminated, truncated to len), clears the records
 * and returns the number of kernels (or -1 on a CUDA error). No counterpart in the reference (its benchmark times
 * whole calls, bench.py:11-23). */
FPA_API int fpa_profile(int enable);
FPA_API int fpa_profile_report(char* buf, size_t len);

/* Failure-path self-test of the bounded device-side waits. Launches one warp on `stream` that waits, through the
 * same bounded mbarrier wait every tensor-core kernel uses, on an mbarrier nothing ever arrives on, with a limit of
 * limit_ns nanoseconds (0 < limit_ns <= 1e9); the wait runs out, records FPA_ERR_TIMEOUT and its site id in the
 * status word of `workspace` (256 bytes, 256-byte aligned) and the kernel returns. fpa_workspace_status then
 * reports FPA_ERR_TIMEOUT. It faults and hangs nothing; the context stays usable. No counterpart in the reference
 * (whose Triton kernels have no bounded waits). */
FPA_API int fpa_selftest_wait_timeout(void* workspace, unsigned long long limit_ns, void* stream);

/* Size of the scratch array built into the library for fpa_fwd_noalloc (8 MiB per GPU that loads the library). */
#define FPA_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)

/* Forward pass for callers that cannot allocate device memory (a plugin host that hands over only the input and
 * output buffers, a runtime whose device memory is fully reserved, code that must not allocate after start-up).
 * This entry point has no counterpart in the reference. It runs the same kernels as fpa_fwd, but their scratch
 * lives in a device array that is part of the library image (FPA_NOALLOC_SCRATCH_BYTES) instead of a caller
 * workspace: args->workspace and args->workspace_bytes are ignored and overwritten. It calls no allocator. A call
 * whose scratch need, the least workspace fpa_fwd accepts for its sizes (fpa_fwd_workspace_bytes without the room
 * for the key-range split, which runs only when the rest of the array covers it), exceeds FPA_NOALLOC_SCRATCH_BYTES
 * returns FPA_ERR_WORKSPACE with a message and launches nothing (the need grows with B*H*ceil(T/128)*128, about 28
 * bytes per padded query position on the tensor-core path). The array's address is looked up in the current CUDA
 * context on every call made outside stream capture; CUDA creates the array on the first lookup in a context
 * (modules load lazily), so a caller that must not allocate later makes that first lookup at start-up with the
 * set-up call fpa_fwd_noalloc(NULL, stream), which launches nothing, and before any stream capture. All calls
 * share the one array: calls whose kernels overlap on the GPU race and must be serialised by the caller. */
FPA_API int fpa_fwd_noalloc(FpaFwdArgs* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FPA_B200_H */
