/*
 * zb_ssd.h — C ABI of the B200 (sm_100a) SSD chunked-scan library (libzenith_ssd.so).
 *
 * The library replaces the reference's pure-PyTorch scan
 *     ssd(x, q, k, kp, xp, adt, gamma, beta, chunk_size)          zenith/mamba3.py:30-56
 * which Mamba3 calls through its injectable `scan` attribute      zenith/mamba3.py:77,118
 * and whose backward the reference leaves to PyTorch autograd.  Layouts are the caller's:
 *     x, xp, y, dy          [B, T, H, P]
 *     q, k, kp              [B, T, G, N]   (G == H in the reference; head h uses group h/(H/G))
 *     adt, gamma, beta      [B, T, H]
 *     states (initial/final, dinitial/dfinal)   [B, H, P, N] contiguous, fp32 (fp64 for fp64 inputs)
 * Every tensor is passed as a base pointer plus element strides over (b, t, h); the innermost
 * dimension (P or N) must be contiguous.  No torch types cross this boundary and no C++
 * exception leaves it: every entry point returns a zb_status code.
 *
 * Threading/streams: calls are asynchronous on the given cudaStream_t (NULL = legacy default
 * stream).  Calls that share a workspace must be ordered (same stream).  Kernels never spin
 * without a bound: a chained state hand-off that waits longer than about one second sets
 * *status (device memory) to ZB_ERR_TIMEOUT and the kernel returns; zb_ssd_check_status()
 * reads it back.
 */
#ifndef ZB_SSD_H
#define ZB_SSD_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ZB_API __attribute__((visibility("default")))
#else
#define ZB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  ZB_OK = 0,
  ZB_ERR_SHAPE = 1,        /* T % chunk_size != 0, H % G != 0, non-positive sizes */
  ZB_ERR_DTYPE = 2,        /* unsupported dtype combination */
  ZB_ERR_LAYOUT = 3,       /* innermost stride != 1 or a required pointer is NULL */
  ZB_ERR_CUDA = 4,         /* a CUDA runtime call failed (see zb_last_cuda_error) */
  ZB_ERR_TIMEOUT = 5,      /* a kernel gave up waiting for the preceding chunk's state */
  ZB_ERR_WORKSPACE = 6,    /* workspace or saved-states buffer too small / misaligned */
  ZB_ERR_UNSUPPORTED = 7,  /* sizes beyond what the kernels handle (e.g. P > 256) */
  ZB_ERR_SCRATCH_LIMIT = 8, /* zb_ssd_fwd_noalloc: the call needs more scratch than ZB_NOALLOC_SCRATCH_BYTES */
  ZB_ERR_INDEX = 9          /* zb_xent: a label outside [0, V) that is not ignore_index */
} zb_status;

typedef enum { ZB_F32 = 0, ZB_BF16 = 1, ZB_F16 = 2, ZB_F64 = 3 } zb_dtype;

/* A [B, T, H(or G), D] tensor (or [B, T, H] for the per-token scalars).  The library sizes every
   operand from zb_ssd_args' B, T, H, G, P, N and never sees a tensor's own extent: each view must
   address that many elements of memory on the current CUDA device (the device the calls launch on,
   on the stream they are given). */
typedef struct {
  void* ptr;
  int64_t sb, st, sh; /* element strides of the batch, token and head dimensions */
} zb_view;

/* flags */
#define ZB_FLAG_STATE_ONLY 1  /* forward: only the final state (no y);  backward: only dinitial_state */
#define ZB_FLAG_SHIFTED 2     /* xp and kp are x and k one token later (xp[t] = x[t-1], zero at t = 0), as
                                 Mamba3.forward builds them (zenith/mamba3.py:115-116): the kernels read x and k
                                 at t - 1 and the xp / kp views are ignored.  No segmentation. */

typedef struct {
  int64_t B, T, H, G, P, N;
  int64_t chunk_size;  /* the caller's chunk size: T % chunk_size == 0 is enforced (mamba3.py:33) */
  int32_t dtype;       /* zb_dtype of x, q, k, kp, xp, y, dy and of their gradients */
  int32_t scalar_dtype;/* zb_dtype of adt, gamma, beta and of their gradients */
  int32_t flags;
  int32_t reserved;
  /* forward inputs (also read by the backward) */
  zb_view x, q, k, kp, xp, adt, gamma, beta;
  /* forward output */
  zb_view y;
  const void* initial_state; /* optional [B,H,P,N]; NULL = zero state (the reference)       */
  void* final_state;         /* optional [B,H,P,N] output                                   */
  /* saved chunk states: written by the forward, read by the backward of the same call
     arguments.  Size from zb_ssd_states_bytes(); NULL in a forward that will not be
     differentiated. */
  void* states;
  /* backward inputs / outputs */
  zb_view dy;
  const void* dfinal_state;  /* optional gradient w.r.t. final_state                        */
  zb_view dx, dq, dk, dkp, dxp, dadt, dgamma, dbeta;
  void* dinitial_state;      /* optional [B,H,P,N] output                                   */
  /* scratch: zb_ssd_workspace_bytes(args, backward) bytes, 256-byte aligned */
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;           /* device int32; 0 = fine.  Never cleared by the library.      */
} zb_ssd_args;

/* Library version (major*10000 + minor*100 + patch). */
ZB_API int zb_version(void);

/* Human-readable name of a status code. */
ZB_API const char* zb_strerror(int status);

/* Text of the last CUDA error seen by this thread inside the library ("" if none). */
ZB_API const char* zb_last_cuda_error(void);

/* Bytes of the saved chunk-state buffer for these sizes/dtypes (0 if the arguments are invalid).
 * Replaces the autograd-saved `states` list of zenith/mamba3.py:49-54. */
ZB_API size_t zb_ssd_states_bytes(const zb_ssd_args* args);

/* Bytes of scratch memory the forward (backward = 0) or backward (backward = 1) needs. */
ZB_API size_t zb_ssd_workspace_bytes(const zb_ssd_args* args, int backward);

/* Forward scan: y = ssd(x, q, k, kp, xp, adt, gamma, beta, chunk_size)
 * (zenith/mamba3.py:30-56), plus the optional initial/final state.
 * Writes the saved chunk states when args->states != NULL. */
ZB_API int zb_ssd_fwd(const zb_ssd_args* args, void* stream);

/* Backward scan: all eight input gradients of the forward (the autograd of
 * zenith/mamba3.py:30-56), plus dinitial_state when requested.  Reads args->states written by
 * zb_ssd_fwd with the same arguments.  dq/dk/dkp are summed over the heads of a group. */
ZB_API int zb_ssd_bwd(const zb_ssd_args* args, void* stream);

/* Recurrent form for decode: advance a state through args->T tokens in order,
 *     h = e^{adt} h + gamma x k^T + beta xp kp^T ,   y = h q      (tests/test_mamba3.py:10-21)
 * from initial_state (NULL = zero) to final_state (required; may be the same buffer, updated in
 * place), writing y.  Uses x, q, k, kp, xp, adt, gamma, beta, y, initial_state, final_state of
 * args (chunk_size, states and workspace are ignored).  fp32 / bf16 / fp16 vectors with fp32
 * scalars, P <= 128, N <= 128; states fp32.  Not differentiated. */
ZB_API int zb_ssd_decode(const zb_ssd_args* args, void* stream);

/* Context-parallel combine of per-rank boundary states (no reference counterpart; the
 * reference is single-device): given the state entering this rank's range `s_prev`,
 * the total decay exp(sum adt) of the previous rank's range `decay_prev` [B*H], and that
 * rank's locally computed final state `f_prev`, write s_next = decay_prev * s_prev + f_prev.
 * All [B,H,P,N] fp32 contiguous. Also used in reverse for the state gradient. */
ZB_API int zb_ssd_state_combine(const float* s_prev, const float* decay_prev, const float* f_prev,
                         float* s_next, int64_t BH, int64_t PN, void* stream);

/* Per (b, h): exp(sum_t adt[b, t, h]) over the whole sequence, fp32 [B*H]. */
ZB_API int zb_ssd_total_decay(const zb_ssd_args* args, float* out, void* stream);

/* Copy the device status word to the host (synchronises `stream`) and report it. */
ZB_API int zb_ssd_check_status(const int32_t* status, void* stream);

/* Which kernel family a call with these arguments uses: 0 = SIMT (fp32/fp64 FMA path),
 * 1 = tensor-core (tcgen05) path.  `states_saved` says whether the forward saves states for a
 * backward.  No reference counterpart (diagnostic); -1 on invalid arguments. */
ZB_API int zb_ssd_kernel_family(const zb_ssd_args* args, int states_saved);

/* Number of kernels this library has launched in this process (all devices, all threads).
 * No reference counterpart: lets a benchmark count the GPU launches of a timed region. */
ZB_API uint64_t zb_launch_count(void);

/* Diagnostic, no reference counterpart: runs one of the library's bounded device-side waits on its
 * own so that a test can watch it give up.  which = 0: the chained hand-off wait on `*flag` (device
 * int; it ends when the flag becomes 1, another nonzero value, or *status is nonzero); which = 1:
 * a wait on a fresh mbarrier that never completes (`flag` unused).  After about one second the
 * wait records ZB_ERR_TIMEOUT in *status (device int32, left alone if already nonzero) and returns.
 * result (device int32[2]): [0] what the wait returned (flag: 1 ready, 2 aborted; mbarrier: 1
 * completed, 0 gave up), [1] microseconds it took.  One thread, one launch; nothing faults. */
ZB_API int zb_wait_probe(const int* flag, int32_t* status, int32_t* result, int which, void* stream);

/* Size of the fixed device scratch array behind zb_ssd_fwd_noalloc (32 MiB per GPU). */
#define ZB_NOALLOC_SCRATCH_BYTES (32u << 20)

/* Forward scan that allocates nothing.  This entry point has no counterpart in the reference.
 *
 * It is for callers that cannot obtain device memory for a call: a serving runtime that
 * reserves all device memory up front and hands out no scratch, or a foreign-language binding
 * that can pass tensors it was given but has no CUDA allocator of its own.  The caller passes
 * the inputs and outputs exactly as for zb_ssd_fwd; `workspace` and `workspace_bytes` are
 * ignored.  Scratch comes from one file-scope device array of ZB_NOALLOC_SCRATCH_BYTES that
 * every GPU which loads the library holds until the process exits.
 *
 * - The first call on a device looks the array up for that device (cudaGetSymbolAddress);
 *   make that first call before any stream capture on the device.
 * - A call whose scratch need (zb_ssd_workspace_bytes(args, 0)) exceeds
 *   ZB_NOALLOC_SCRATCH_BYTES returns ZB_ERR_SCRATCH_LIMIT and launches nothing.
 * - All calls on a device share the array: calls that overlap on the GPU (different streams
 *   without ordering) race and give wrong results.  Order them on one stream.
 * - No cudaMalloc, cudaFree or allocating library routine is called. */
ZB_API int zb_ssd_fwd_noalloc(const zb_ssd_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ZB_SSD_H */
