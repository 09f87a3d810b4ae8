/*
 * coalibi.h -- C ABI of the sm_100a (B200) Co-ALiBi attention library
 * (libcoalibi_sm100.so).
 *
 * Co-ALiBi attention, per batch b, query head h, query row i and key j:
 *   p_ij = sm_scale * q_i . k_j          (masked where causal and j > i)
 *   s_ij = sigmoid(p_ij), z_ij = sum_{t >= j} s_it
 *   o_i  = softmax_j(p_ij - slope_h * z_ij) @ V
 *
 * All tensors are device pointers to contiguous row-major arrays:
 *   q, o, dout, dq     [B, Hq,  Sq,  D]
 *   k, v, dk, dv       [B, Hkv, Skv, D]      (Hq % Hkv == 0; q head h reads kv head h / (Hq/Hkv))
 *   lse, rowsig        [B, Hq,  Sq]  float32
 *   slopes             [Hq]          float32, float16 or bfloat16 (slopes_dtype)
 * with D in {64, 128}, dtype float16 or bfloat16, every pointer 16-byte aligned.
 *
 * The library never allocates device memory, never synchronises and only
 * enqueues work on the stream it is given (a cudaStream_t passed as void*; NULL
 * means the legacy default stream), which must belong to the device that holds
 * the tensors (else COALIBI_ERR_DEVICE).  Each call makes that device current
 * while it runs and puts the calling thread's previous CUDA context (possibly
 * none) back before it returns.  Calls are reentrant and thread-safe across
 * streams and devices.  Each function returns COALIBI_OK or an error code;
 * coalibi_strerror() names it.  Kernel-side failures (a bounded wait that timed
 * out) are reported asynchronously through the optional device status word.
 *
 * The forward and backward kernels are launched with programmatic stream
 * serialization: one may start its set-up while the kernel before it on the
 * stream is still finishing, but it waits for that kernel to complete before
 * it touches global memory, so stream order holds for every read and write.
 */
#ifndef COALIBI_H_
#define COALIBI_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define COALIBI_ABI_VERSION 1

enum coalibi_dtype {
  COALIBI_F16 = 0,
  COALIBI_BF16 = 1,
  COALIBI_F32 = 2 /* only valid for slopes_dtype */
};

enum coalibi_error {
  COALIBI_OK = 0,
  COALIBI_ERR_NULL_POINTER = 1,
  COALIBI_ERR_HEAD_DIM = 2,     /* D not in {64, 128} */
  COALIBI_ERR_DTYPE = 3,        /* dtype not float16 / bfloat16 */
  COALIBI_ERR_SHAPE = 4,        /* non-positive sizes, Hq % Hkv != 0, or too large */
  COALIBI_ERR_ALIGNMENT = 5,    /* a pointer is not 16-byte aligned */
  COALIBI_ERR_LAUNCH = 6,       /* CUDA launch / attribute error */
  COALIBI_ERR_TENSOR_MAP = 7,   /* cuTensorMapEncodeTiled failed or unavailable */
  COALIBI_ERR_WORKSPACE = 8,    /* workspace missing or smaller than coalibi_bwd_workspace_bytes() */
  COALIBI_ERR_DEVICE = 9,       /* device is not sm_100, or the stream is on another device */
  COALIBI_ERR_TIMEOUT = 10      /* device status only: a bounded wait expired */
};

/* Forward.  Replaces the Triton launch in co_alibi_attn/co_alibi_attn.py:44-57
 * (CoALIBIAttention.forward) and the kernel co_alibi_attn/co_alibi_fwd_kernel.py:29-127.
 * Writes o, lse = m + log(l + 1e-9) (natural log) and rowsig = sum_j sigmoid(p_ij),
 * the two float32 side outputs the backward consumes. */
typedef struct CoalibiFwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* slopes;
  void* o;
  float* lse;
  float* rowsig;
  int B, Hq, Hkv, Sq, Skv, D;
  int dtype;        /* enum coalibi_dtype of q, k, v, o */
  int slopes_dtype; /* enum coalibi_dtype of slopes */
  int causal;       /* nonzero: top-left aligned causal mask (key j > query i masked) */
  float sm_scale;
  int* status;      /* optional device int; a kernel-side error code is CAS'ed in */
  unsigned int timeout_ms; /* bound on every in-kernel wait; 0 = default (2000 ms) */
} CoalibiFwdArgs;

int coalibi_fwd(const CoalibiFwdArgs* args, void* stream);

/* Forward for few query rows (Sq <= COALIBI_DECODE_MAX_SQ, e.g. one new token
 * against a long key/value sequence): the same arguments, mask semantics and
 * results (o, lse, rowsig) as coalibi_fwd, for the shapes the reference forward
 * launches with a nearly empty query block (co_alibi_attn/co_alibi_attn.py:44-57).
 * The keys are split into chunks (one per warp of the partial kernel) and merged
 * exactly: the sigmoid totals of the chunks to the right shift each chunk's
 * logits.  workspace: device scratch of at least coalibi_fwd_decode_workspace_bytes()
 * bytes, 16-byte aligned; contents on entry do not matter.  Sq above the limit
 * returns COALIBI_ERR_SHAPE. */
#define COALIBI_DECODE_MAX_SQ 16
size_t coalibi_fwd_decode_workspace_bytes(int B, int Hq, int Hkv, int Sq, int Skv, int D);
int coalibi_fwd_decode(const CoalibiFwdArgs* args, void* workspace, size_t workspace_bytes, void* stream);

/* Backward.  Replaces co_alibi_attn/co_alibi_attn.py:73-135 (CoALIBIAttention.backward,
 * including the dk/dv partial-buffer reduction at :132-133 and, for GQA, the group
 * sum autograd performs through repeat_interleave at :145-146) and the kernel
 * co_alibi_attn/co_alibi_bwd_kernel.py:19-146.  dk and dv have Hkv heads.
 * workspace: device scratch, 256-byte aligned, its contents on entry irrelevant.
 * The size picks the algorithm: with at least the "stored" size (what
 * coalibi_bwd_workspace_size() returns while that stays below 24 GiB) the first
 * kernel also writes P and dS as 16-bit 128 x 128 tiles -- 4 bytes per visible
 * score, 4.3 GB at B8 H16 S4096 causal, half the reference's dk/dv partial
 * buffers -- and dK, dV come from a streaming GEMM over them; with less, down to
 * coalibi_bwd_workspace_min_bytes() (8 bytes per row per 32 keys), the second
 * kernel recomputes P and dS instead.  Both agree with the reference within the
 * same tolerances; less than the minimum returns COALIBI_ERR_WORKSPACE. */
typedef struct CoalibiBwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;
  const float* rowsig;
  const void* slopes;
  void* dq;
  void* dk;
  void* dv;
  void* workspace;
  size_t workspace_bytes;
  int B, Hq, Hkv, Sq, Skv, D;
  int dtype;
  int slopes_dtype;
  int causal;
  float sm_scale;
  int* status;
  unsigned int timeout_ms;
} CoalibiBwdArgs;

/* Workspace size to allocate for this call's problem and mask (args->B, Hq, Hkv,
 * Sq, Skv, D, causal; the pointers are not read): the stored layout while its
 * P / dS scratch stays below 24 GiB, else the recompute layout. */
size_t coalibi_bwd_workspace_size(const CoalibiBwdArgs* args);

/* A size that serves either mask of the problem (the larger of the two
 * coalibi_bwd_workspace_size values). */
size_t coalibi_bwd_workspace_bytes(int B, int Hq, int Hkv, int Sq, int Skv, int D);

/* The smallest workspace coalibi_bwd accepts for the problem (the recompute layout). */
size_t coalibi_bwd_workspace_min_bytes(int B, int Hq, int Hkv, int Sq, int Skv, int D);

int coalibi_bwd(const CoalibiBwdArgs* args, void* stream);

/* Backward of one key shard of longer rows (sequence / context parallelism, which
 * the reference does not have): the keys of this call are a contiguous piece of
 * each row's keys.  Same arguments as coalibi_bwd, read this way: o, lse and dout
 * are those of the whole row (so delta and P are global); rowsig is the sigmoid
 * total of this call's keys plus that of every key right of them; dA_carry_in
 * [B * Hq * Sq] float32 is sum_t P_it (dP_it - delta_i) over the keys left of them.
 * dq, dk and dv are this shard pair's contributions (sum them over the shards). */
int coalibi_bwd_carry(const CoalibiBwdArgs* args, const float* dA_carry_in, void* stream);

/* Profiling aid with no counterpart in the reference: launch only the backward
 * kernels selected by phase_mask (bit 0: delta = rowsum(dO * O) pre-pass, bit 1:
 * pass A -> dq and, in the workspace, P / dS tiles or the per-32-key carries,
 * bit 2: pass B -> dk, dv).
 * Phases read what earlier phases wrote into the workspace, so they must run in
 * order on one stream; coalibi_bwd(args, s) == coalibi_bwd_phases(args, 7, s). */
int coalibi_bwd_phases(const CoalibiBwdArgs* args, int phase_mask, void* stream);

/* Size of the static device scratch used by coalibi_bwd_noalloc (64 MiB). */
#define COALIBI_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)

/* Backward that allocates nothing and needs no workspace: same arguments and
 * results as coalibi_bwd, with args->workspace / workspace_bytes ignored.  It has
 * no counterpart in the reference.  It is for callers that cannot allocate device
 * memory at the call -- a plugin host or FFI caller that owns only the tensors
 * it passes, or code that must avoid cudaMalloc there because it can synchronise
 * the device.  Its scratch is one file-scope device array of
 * COALIBI_NOALLOC_SCRATCH_BYTES per GPU, held until the process exits; the
 * backward runs the stored path when its scratch fits there, else the recompute
 * path; problems needing more (coalibi_bwd_workspace_min_bytes() > that) return
 * COALIBI_ERR_WORKSPACE without launching.  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress); make it before any stream capture.  The address
 * is not looked up again, so it is stale after cudaDeviceReset on that device.
 * All calls on a device share the array, so calls that overlap on the GPU race:
 * serialise them. */
int coalibi_bwd_noalloc(const CoalibiBwdArgs* args, void* stream);

/* Self-test of the kernels' bounded waits, with no counterpart in the reference:
 * enqueues one CTA whose warps wait on mbarriers that nothing ever arrives on.
 * Every such wait in this library gives up after its timeout, raises the CTA's
 * abort flag and records COALIBI_ERR_TIMEOUT in the device word *status (if it
 * still holds 0), so the kernel ends after about timeout_ms (0: the default of
 * 2000) and the CUDA context stays usable.  Returns the launch result; read
 * *status after synchronising the stream. */
int coalibi_selftest_wait_timeout(unsigned int timeout_ms, int* status, void* stream);

/* The launch configuration this library picks for a problem, as one line of
 * text: the counterpart of the reference's COALIBI_VERBOSE=1 print of the
 * configuration its autotuner chose (co_alibi_attn/co_alibi_attn.py:58-63 for the
 * forward, :125-130 for the backward).  which: 0 forward (coalibi_fwd), 1 decode
 * forward (coalibi_fwd_decode), 2 backward (coalibi_bwd, with the workspace of
 * coalibi_bwd_workspace_size); causal: the mask; device: the CUDA device index (for
 * its SM count).  Writes a NUL-terminated description into buf, truncated to
 * buf_len bytes.  Launches nothing and changes no CUDA state. */
int coalibi_describe_launch(int which, int B, int Hq, int Hkv, int Sq, int Skv, int D, int causal, int device,
                            char* buf, size_t buf_len);

/* Static name of an error code. */
const char* coalibi_strerror(int code);

/* COALIBI_ABI_VERSION of the loaded library. */
int coalibi_abi_version(void);

/* Detail (driver/runtime result and arguments) of the last failing call made by
 * the calling thread; "" if none.  No counterpart in the reference. */
const char* coalibi_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* COALIBI_H_ */
