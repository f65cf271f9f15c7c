/*
 * tops_gla.h -- C ABI of the B200-native Gated Linear Attention library (libtops_gla.so).
 *
 * This is the drop-in boundary for the GLA operators of the reference package
 * `tops` (primatrix/pallas-kernel).  The reference has no FFI: its boundary is the
 * Python module `tops.ops.gla` (tops/ops/gla/__init__.py:1-34) whose functions
 * launch Pallas-TPU kernels in-process.  Each entry point below replaces one of
 * those functions (cited per declaration); the Python package
 * `pallas-kernel_b200/tops` binds them with ctypes and keeps the reference's
 * Python signatures, and a JAX custom-call binding targets the same symbols.
 *
 * Conventions
 *  - All tensor pointers are DEVICE pointers to dense row-major (contiguous)
 *    arrays.  Layout is [B, T, H, D] for token tensors (FLA convention) and
 *    [N, H, K, V] for recurrent states; per-chunk states are [NT, H, K, V] with
 *    chunks in sequence order (== the reference's [B, NT, H, K, V] or, for
 *    variable-length input, [1, NT_total, H, K, V]).
 *  - `dtype` is the storage type of q, k, v, o, do, dq, dk, dv (TOPS_F32, TOPS_BF16
 *    or TOPS_F16).  Gates g/gk/gv, their gradients, states (h0, ht, dht, dh0) and
 *    every per-chunk intermediate (g_cumsum, A, h, dh, dA) are fp32, as in the
 *    reference (tops/ops/gla/chunk.py:1226-1231 casts to fp32;
 *    tops/ops/gla/fused_recurrent.py:261-263 returns fp32 o/ht).
 *  - Variable-length input: B == 1, `cu_seqlens` = device int32 [N+1] and
 *    `chunk_offsets` = device int32 [N+1] from tops_gla_num_chunks() (the
 *    reference computes the same map on the host: tops/utils.py:70-89).
 *    Segments need not be multiples of chunk_size (ragged chunks behave as the
 *    reference's per-segment zero padding, tops/ops/gla/chunk.py:751-793).
 *  - Every function is stream-ordered on `stream` (a cudaStream_t; NULL = legacy
 *    default stream), allocates no device memory, and returns TOPS_OK (0) or a
 *    negative status; tops_gla_last_error() gives the message (thread-local).
 *    Nothing aborts, traps or waits without a bound.
 */
#ifndef TOPS_GLA_H_
#define TOPS_GLA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TOPS_GLA_ABI_VERSION 1

#if defined(__GNUC__) || defined(__clang__)
#define TOPS_API __attribute__((visibility("default")))
#else
#define TOPS_API
#endif

enum tops_dtype { TOPS_F32 = 0, TOPS_BF16 = 1, TOPS_F16 = 2 };

enum tops_status {
  TOPS_OK = 0,
  TOPS_ERR_INVALID = -1,      /* bad shape / null pointer / inconsistent arguments */
  TOPS_ERR_UNSUPPORTED = -2,  /* valid request this build cannot serve (e.g. no sm_100 device) */
  TOPS_ERR_CUDA = -3,         /* a CUDA runtime call failed */
  TOPS_ERR_WORKSPACE = -4,    /* workspace missing or smaller than *_workspace_size() */
  TOPS_ERR_TIMEOUT = -5,      /* a bounded device-side wait gave up */
  TOPS_ERR_NCCL = -6          /* an NCCL call failed */
};

/* Problem description shared by every chunked entry point. */
typedef struct tops_gla_shape {
  int32_t B, T, H, K, V;       /* q,k: [B,T,H,K]  v: [B,T,H,V] */
  int32_t N;                   /* number of sequences: B, or len(cu_seqlens)-1 */
  int32_t NT;                  /* total chunks over all sequences (tops_gla_num_chunks) */
  int32_t chunk_size;          /* power of two; the reference API default is 16 */
  int32_t dtype;               /* enum tops_dtype of q/k/v/o/do/dq/dk/dv */
  float scale;                 /* attention scale (reference default K^-0.5) */
  const int32_t* cu_seqlens;   /* device [N+1] or NULL */
  const int32_t* chunk_offsets;/* device [N+1] or NULL (required iff cu_seqlens) */
} tops_gla_shape;

/* ---- host helpers ------------------------------------------------------- */

/* Number of chunks of a problem: B*ceil(T/C) or sum_n ceil(len_n/C) when
 * `cu_seqlens_host` ([N+1], host memory) is given.  If `chunk_offsets_host` is not
 * NULL it receives the [N+1] prefix (to be copied to the device by the caller).
 * Replaces tops/utils.py:70-89 (prepare_chunk_indices).  Returns -1 on bad input. */
TOPS_API int32_t tops_gla_num_chunks(int32_t B, int32_t T, int32_t chunk_size, const int32_t* cu_seqlens_host,
                            int32_t N, int32_t* chunk_offsets_host);

TOPS_API const char* tops_gla_last_error(void);
/* Number of kernels (and device memsets) this library has launched in the process. */
TOPS_API uint64_t tops_gla_launch_count(void);
/* Per-launch timing for benchmarks: when enabled, every kernel launch is bracketed by
 * CUDA events on its stream; tops_gla_timing_collect() waits for them, writes up to
 * `max_entries` (name, milliseconds) pairs and clears the record.  Returns the number
 * of launches recorded.  Off by default (no events, no overhead). */
TOPS_API void tops_gla_timing_enable(int32_t on);
TOPS_API int32_t tops_gla_timing_collect(char* names, int32_t name_stride, float* ms, int32_t max_entries);
TOPS_API int32_t tops_gla_abi_version(void);
/* First error code recorded by a device-side bounded wait since the last call
 * (0 = none, 1 = an mbarrier wait timed out, 3 = a peer-memory exchange gave up waiting for
 * a rank); reading clears it.  Synchronizes. */
TOPS_API int32_t tops_gla_device_error(void);
/* Check of the failure path: launches one thread that waits on an mbarrier nothing will
 * complete, so its bounded wait runs out (about 2 s) and records code 1 for
 * tops_gla_device_error(); the kernel then returns and the context stays usable.
 * Returns the launch status. */
TOPS_API int tops_gla_selftest_wait_timeout(void* stream);
/* 1 when the current device can run the tcgen05 (sm_100a) kernels. */
TOPS_API int32_t tops_gla_has_tcgen05(void);

/* ---- public operators ---------------------------------------------------- */

typedef struct tops_gla_chunk_fwd_args {
  tops_gla_shape s;
  const void* q; const void* k; const void* v;
  const float* g;              /* [B,T,H,K] log-space gates, NULL = no decay (zero gates, as the
                                  reference substitutes; on the tensor-core path they are a zeroed
                                  region of the workspace, which *_workspace_size then includes) */
  const float* h0;             /* [N,H,K,V] or NULL */
  void* o;                     /* out [B,T,H,V] (dtype); NULL = final state only (ht required) */
  float* ht;                   /* out [N,H,K,V] or NULL (output_final_state=False) */
  /* Optional saved intermediates for the backward (reference chunk_gla_fwd
   * returns (g_cumsum, A, h, ht, o), tops/ops/gla/chunk.py:1083-1179).  NULL = not
   * returned.  Their layout follows `chunk_size`. */
  float* g_cumsum;             /* [B,T,H,K] */
  float* A;                    /* [B,T,H,C] */
  float* h;                    /* [NT,H,K,V] */
  void* workspace; size_t workspace_bytes;
  /* Opaque block receiving what the backward reuses when the forward runs on the
   * tensor-core path (bf16 or fp16, K in {64, 128, 256}, V = 64 or a multiple of 128); size from
   * tops_gla_chunk_saved_size(), NULL = do not save.  Pass it to the backward. */
  void* saved; size_t saved_bytes;
} tops_gla_chunk_fwd_args;

/* Chunked GLA forward: o = chunk_gla(q,k,v,g,scale,h0)[0], ht = final state.
 * Replaces tops.ops.gla.chunk_gla / chunk_gla_fwd (tops/ops/gla/chunk.py:1187,1083)
 * and fused_chunk_gla (tops/ops/gla/fused_chunk.py:4).  With o == NULL only the
 * final state is computed (the state scan without the output GEMM): the first pass
 * of a sequence-parallel forward, whose span states are exchanged between ranks. */
TOPS_API int tops_gla_chunk_fwd(const tops_gla_chunk_fwd_args* a, void* stream);
TOPS_API size_t tops_gla_chunk_fwd_workspace_size(const tops_gla_chunk_fwd_args* a);
/* Bytes of the forward's saved block for this problem; 0 when the problem runs on
 * the CUDA-core path (which saves into the g_cumsum / A / h arguments instead). */
TOPS_API size_t tops_gla_chunk_saved_size(const tops_gla_shape* s);

typedef struct tops_gla_chunk_bwd_args {
  tops_gla_shape s;
  const void* q; const void* k; const void* v;
  const float* g;              /* raw gates or NULL */
  const float* h0;             /* [N,H,K,V] or NULL */
  const void* do_;             /* [B,T,H,V] (dtype) */
  const float* dht;            /* [N,H,K,V] or NULL */
  const float* g_cumsum;       /* optional saved fwd intermediates (NULL = recompute) */
  const float* A;
  const float* h;
  void* dq; void* dk; void* dv;/* out (dtype); all four gradients NULL = dh0 only */
  float* dg;                   /* out [B,T,H,K] fp32 */
  float* dh0;                  /* out [N,H,K,V] or NULL */
  void* workspace; size_t workspace_bytes;
  const void* saved; size_t saved_bytes;  /* block written by the forward, or NULL */
} tops_gla_chunk_bwd_args;

/* Chunked GLA backward -> dq, dk, dv, dg, dh0.
 * Replaces tops.ops.gla.chunk_gla_bwd (tops/ops/gla/chunk.py:815) and
 * chunk_gla_bwd_with_pl (tops/ops/gla/chunk.py:980).  With dq, dk, dv and dg all
 * NULL only dh0 is computed (the reverse state scan): the first pass of a
 * sequence-parallel backward. */
TOPS_API int tops_gla_chunk_bwd(const tops_gla_chunk_bwd_args* a, void* stream);

/* Chunked GLA forward that allocates nothing and needs no workspace.  No counterpart
 * in the reference (whose JAX ops get their memory from XLA): it exists for callers
 * that cannot call cudaMalloc or pass a scratch buffer -- e.g. a host framework that
 * plans all device memory up front and gives an operator only its inputs and
 * outputs, or a serving loop that must not call the allocator.  Same arguments and
 * results as tops_gla_chunk_fwd; a->workspace is ignored.  Scratch comes from a
 * fixed array of TOPS_GLA_NOALLOC_SCRATCH_BYTES inside the library's device image,
 * one per GPU that loads the library, held until the process exits.  Problems whose
 * scratch (tops_gla_chunk_fwd_workspace_size) exceeds it are rejected with
 * TOPS_ERR_WORKSPACE.  CUDA loads the library's device image on a GPU lazily, so the
 * first call on a device (unless another of this library's kernels ran there before)
 * loads it and thereby reserves the 16 MiB: a host that must not allocate after
 * start-up makes one warm-up call per device at start-up, before any stream capture.
 * Every call looks up the array's address on the current device (a host-side symbol
 * lookup), so a cudaDeviceReset or another context does not leave a stale address.
 * All calls on a device share the one array and it keeps the last call's contents:
 * calls whose kernels may overlap on the GPU (different streams, no ordering between
 * them) race and give wrong results; order them on one stream or with events. */
#define TOPS_GLA_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
TOPS_API int tops_gla_chunk_fwd_noalloc(const tops_gla_chunk_fwd_args* a, void* stream);
TOPS_API size_t tops_gla_chunk_bwd_workspace_size(const tops_gla_chunk_bwd_args* a);

typedef struct tops_gla_recurrent_args {
  int32_t B, T, H, K, V, N;
  int32_t dtype;               /* storage type of q, k, v */
  float scale;
  int32_t reverse;             /* iterate t = T-1 .. 0 */
  const int32_t* cu_seqlens;   /* device [N+1] or NULL (then N == B) */
  const void* q; const void* k; const void* v;
  const float* gk;             /* [B,T,H,K] or NULL */
  const float* gv;             /* [B,T,H,V] or NULL */
  const float* h0;             /* [N,H,K,V] or NULL */
  float* o;                    /* out [B,T,H,V] fp32 */
  float* ht;                   /* out [N,H,K,V] or NULL */
  void* workspace; size_t workspace_bytes;
} tops_gla_recurrent_args;

/* Token-by-token recurrence (decode).  Replaces tops.ops.gla.fused_recurrent_gla
 * (tops/ops/gla/fused_recurrent.py:438 -> :379 -> :235, kernel :139). */
TOPS_API int tops_gla_recurrent_fwd(const tops_gla_recurrent_args* a, void* stream);
TOPS_API size_t tops_gla_recurrent_fwd_workspace_size(const tops_gla_recurrent_args* a);

typedef struct tops_gla_recurrent_bwd_args {
  tops_gla_recurrent_args f;   /* forward inputs (f.o / f.ht unused) */
  const float* o;              /* forward output [B,T,H,V] fp32; required when f.gv is given
                                  (as in the reference, fused_recurrent.py:934) */
  const void* do_;             /* [B,T,H,V] (dtype) */
  const float* dht;            /* [N,H,K,V] or NULL */
  float* dq; float* dk; float* dv;   /* out fp32 */
  float* dgk;                  /* out [B,T,H,K] or NULL (needs gk) */
  float* dgv;                  /* out [B,T,H,V] or NULL (needs gv) */
  float* dh0;                  /* out [N,H,K,V] or NULL */
} tops_gla_recurrent_bwd_args;

/* Backward of the recurrence.  Replaces tops.ops.gla.fused_recurrent_gla_bwd
 * (tops/ops/gla/fused_recurrent.py:879; kernel :495; gate grads :798-876). */
TOPS_API int tops_gla_recurrent_bwd(const tops_gla_recurrent_bwd_args* a, void* stream);
TOPS_API size_t tops_gla_recurrent_bwd_workspace_size(const tops_gla_recurrent_bwd_args* a);

/* ---- chunk sub-functions (exported by tops.ops.gla, __init__.py:2-14) ------ */

/* g_cumsum = scale * chunk-local inclusive cumsum of g (suffix sums when reverse != 0).
 * tops/ops/gla/chunk.py:110 (chunk_local_cumsum_vector; kernel :55). */
TOPS_API int tops_gla_chunk_local_cumsum(const tops_gla_shape* s, const float* g, float* g_cumsum, int32_t reverse,
                                         float scale, void* stream);

/* h[c] = state at the start of chunk c; ht = final state.  tops/ops/common/chunk_h.py:137,277. */
TOPS_API int tops_gla_chunk_fwd_h(const tops_gla_shape* s, const void* k, const void* v, const float* g_cumsum,
                         const float* h0, float* h, float* ht, void* stream);

/* Reverse scan: dh[c] = dL/d(state at the end of chunk c); dh0.  tops/ops/common/chunk_h.py:399,605. */
TOPS_API int tops_gla_chunk_bwd_dh(const tops_gla_shape* s, const void* q, const float* g_cumsum, const void* do_,
                          const float* dht, float* dh, float* dh0, void* stream);

/* A = intra-chunk gated attention [B,T,H,C]; the full C x C block when causal == 0
 * (as the exported reference sub-function returns it), lower-triangular when causal != 0
 * (as chunk_gla_fwd uses it).  tops/ops/gla/chunk.py:386 (kernel :350, ref :300). */
TOPS_API int tops_gla_chunk_fwd_intra(const tops_gla_shape* s, const void* q, const void* k, const float* g_cumsum,
                                      int32_t causal, float* A, void* stream);

/* o = scale (q e^G) h + tril(A) v.  tops/ops/gla/chunk.py:1387 (kernel :1259, ref :441). */
TOPS_API int tops_gla_chunk_fwd_o(const tops_gla_shape* s, const void* q, const void* v, const float* g_cumsum,
                         const float* A, const float* h, void* o, void* stream);

/* dA = tril(scale do v^T).  tops/ops/gla/chunk.py:504 (chunk_gla_bwd_dA_ref). */
TOPS_API int tops_gla_chunk_bwd_dA(const tops_gla_shape* s, const void* v, const void* do_, float* dA, void* stream);

/* dv = tril(A)^T do + (k e^{G_last-G}) dh.  tops/ops/gla/chunk.py:547 (chunk_gla_bwd_dv_ref). */
TOPS_API int tops_gla_chunk_bwd_dv(const tops_gla_shape* s, const void* k, const float* g_cumsum, const float* A,
                          const void* do_, const float* dh, float* dv, void* stream);

/* Intra-chunk dq, dk from dA.  tops/ops/gla/chunk.py:603 (chunk_gla_bwd_dqk_intra_ref). */
TOPS_API int tops_gla_chunk_bwd_dqk_intra(const tops_gla_shape* s, const void* q, const void* k, const float* g_cumsum,
                                 const float* dA, float* dq, float* dk, void* stream);

/* Inter-chunk dq, dk (added to dq_in/dk_in) and dg.  tops/ops/gla/chunk.py:656 (chunk_gla_bwd_dqkg_ref).
 * dq_out/dk_out have storage type `out_dtype` (enum tops_dtype); dg is fp32. */
TOPS_API int tops_gla_chunk_bwd_dqkg(const tops_gla_shape* s, const void* q, const void* k, const void* v,
                            const float* h, const float* g_cumsum, const void* do_, const float* dh,
                            const float* dq_in, const float* dk_in, void* dq_out, void* dk_out,
                            int32_t out_dtype, float* dg, void* stream);

/* ---- sequence-parallel state hand-off (no reference counterpart: the reference
 *      has no multi-device code; BASELINE config 4 asks for it) ------------- */

/* D[n,h,k] = exp(sum over the sequence of g[.,h,k]): the total decay of a span. */
TOPS_API int tops_gla_span_decay(const tops_gla_shape* s, const float* g, float* decay, void* stream);

/* out = decay (broadcast over V) * h_in + s_local, all [N,H,K,V] fp32 (decay [N,H,K]).
 * out may alias s_local. */
TOPS_API int tops_gla_state_combine(int32_t N, int32_t H, int32_t K, int32_t V, const float* decay, const float* h_in,
                           const float* s_local, float* out, void* stream);

/* ---- sequence-parallel forward / backward in two phases ---
 * No reference counterpart (the reference has no multi-device code); the math is the
 * linear decomposition of its chunked scan (tops/ops/common/chunk_h.py:372-386).  Each rank
 * holds one contiguous span of a long sequence (fixed length, tensor-core path: bf16 or fp16,
 * K in {64, 128, 256}, V = 64 or a multiple of 128).  The scan is linear in the span's incoming state, so the
 * first phase does all the work that does not depend on it and returns the span's own
 * final state from a zero state (local_state [N,H,K,V] fp32) and its total decay
 * (decay [N,H,K] fp32, exp of the span's gate sums); the host exchanges these between ranks
 * (tops_gla_state_exchange, or any all-gather + prefix) and the second phase finishes from
 * the span's incoming state.  Per rank the two phases cost what one tops_gla_chunk_fwd
 * (tops_gla_chunk_bwd) costs, plus one small combine kernel.
 *  - the saved block (a->saved, tops_gla_chunk_span_saved_size bytes) is written by
 *    fwd_span_begin and read by fwd_span_finish and both backward phases;
 *  - fwd_span_finish: a->h0 = the span's incoming state (NULL = zero), a->o out, a->ht
 *    (optional) = the span's final state;
 *  - bwd_span_begin: local_dh0 = gradient w.r.t. the span's incoming state of the span's
 *    own loss (a zero final-state gradient); a->workspace (tops_gla_chunk_bwd_span_
 *    workspace_size bytes) holds state between the two backward calls: pass the same one;
 *  - bwd_span_finish: a->dht = the gradient w.r.t. the span's final state from the later
 *    spans (NULL = zero), outputs dq, dk, dv, dg and (optional) dh0.
 * Other problems get TOPS_ERR_UNSUPPORTED; use tops_gla_chunk_fwd with o == NULL and
 * tops_gla_chunk_bwd with NULL gradients for them. */
TOPS_API size_t tops_gla_chunk_span_saved_size(const tops_gla_shape* s);
TOPS_API int tops_gla_chunk_fwd_span_begin(const tops_gla_chunk_fwd_args* a, float* local_state, float* decay,
                                           void* stream);
TOPS_API int tops_gla_chunk_fwd_span_finish(const tops_gla_chunk_fwd_args* a, void* stream);
TOPS_API size_t tops_gla_chunk_bwd_span_workspace_size(const tops_gla_chunk_bwd_args* a);
TOPS_API int tops_gla_chunk_bwd_span_begin(const tops_gla_chunk_bwd_args* a, float* local_dh0, void* stream);
TOPS_API int tops_gla_chunk_bwd_span_finish(const tops_gla_chunk_bwd_args* a, void* stream);

/* ---- sequence-parallel state exchange over NCCL ---------
 * Every rank holds one contiguous span of a long sequence.  Forward (backward = 0):
 * local_state = the span's final state from a zero state S [N,H,K,V] (tops_gla_chunk_fwd
 * with o == NULL), decay = exp(sum of the span's gates) D [N,H,K] (tops_gla_span_decay),
 * boundary = the sequence's initial state h0 or NULL; out = this rank's incoming state
 * (prefix H_0 = h0, H_{r+1} = D_r H_r + S_r), total = the whole sequence's final state
 * (optional).  Backward (backward = 1): local_state = the gradient w.r.t. this span's
 * incoming state from its own loss (tops_gla_chunk_bwd with NULL gradients and dht = NULL),
 * boundary = dht or NULL; out = the final-state gradient this rank's backward must use
 * (suffix G_{R-1} = dht, G_{r-1} = D_r G_r + L_r).  One ncclAllGather on `stream`, then one
 * kernel; all fp32.  The reference has no multi-device code (its scan is
 * tops/ops/common/chunk_h.py:372-386; this is its exact linear decomposition).  `comm` is an
 * ncclComm_t; NCCL is loaded at run time (libnccl.so.2), TOPS_ERR_UNSUPPORTED without it. */
typedef struct tops_gla_exchange_args {
  void* comm;
  int32_t rank, world;
  int32_t N, H, K, V;
  int32_t backward;
  const float* local_state;
  const float* decay;
  const float* boundary;
  float* out;
  float* total;
  void* workspace; size_t workspace_bytes;
} tops_gla_exchange_args;
TOPS_API size_t tops_gla_state_exchange_workspace_size(const tops_gla_exchange_args* a);
TOPS_API int tops_gla_state_exchange(const tops_gla_exchange_args* a, void* stream);
/* Communicator helpers for hosts without their own: id is NCCL's 128-byte unique id
 * (created on one rank, broadcast by the host, passed to every rank). */
TOPS_API int tops_gla_nccl_get_unique_id(void* id);
TOPS_API int tops_gla_nccl_comm_init(void** comm, int32_t world, const void* id, int32_t rank);
TOPS_API int tops_gla_nccl_comm_destroy(void* comm);
/* Failure handling.  A lost peer is best detected on the host before an exchange is
 * launched (the Python host checks a heartbeat of every rank first); these cover what
 * happens after a launch.  comm_abort: ncclCommAbort (ends the communicator's in-flight
 * work without waiting for peers; the handle is freed, do not destroy it afterwards).
 * comm_check: TOPS_OK, or TOPS_ERR_NCCL with NCCL's asynchronous error.  exchange_wait:
 * waits on the host, at most timeout_ms, for the work enqueued on `stream` so far (the
 * exchange) while polling the communicator's asynchronous error; on an error or at the
 * deadline it aborts the communicator and returns TOPS_ERR_NCCL / TOPS_ERR_TIMEOUT instead of
 * blocking.  No reference counterpart (the reference has no multi-device code). */
TOPS_API int tops_gla_nccl_comm_abort(void* comm);
TOPS_API int tops_gla_nccl_comm_check(void* comm);
TOPS_API int tops_gla_state_exchange_wait(void* comm, void* stream, int32_t timeout_ms);

/* The same exchange through peer memory instead of NCCL: one process per GPU, every rank's
 * receive region mapped into every process (CUDA IPC; NVLink / NVSwitch peer access).
 * p2p_exchange runs two kernels on `stream`: this rank's packed (state | decay) is stored
 * straight into its slot of every rank's region and, once all of it is written, an epoch flag
 * into every region; then the prefix (forward: out = this rank's incoming state, total = the
 * whole sequence's final state) or suffix (backward: out = this rank's final-state gradient)
 * of tops_gla_state_exchange, computed from this rank's own region after every rank's flag
 * for the epoch has arrived.  The results are bit-identical to tops_gla_state_exchange.  The
 * wait is bounded: after timeout_ms it records device error 3 and leaves `out` unwritten.
 * The epoch lives in the region (device memory), so the two kernels can be captured in a CUDA
 * graph and replayed.  Every rank must run the same sequence of exchanges on one region.
 * regions: device array [world] of every rank's region as mapped in this process (this
 * rank's own included); own_region: this rank's.  At most 64 ranks.
 * region_size: bytes of one region (a 4 KB control block and two slots per rank);
 * p2p_alloc / p2p_free: a zeroed region from cudaMalloc (IPC needs a whole allocation);
 * ipc_handle / ipc_open / ipc_close: cudaIpcGetMemHandle / cudaIpcOpenMemHandle (peer
 * access enabled) / cudaIpcCloseMemHandle, handle = TOPS_GLA_IPC_HANDLE_BYTES bytes.
 * No reference counterpart (the reference has no multi-device code). */
#define TOPS_GLA_IPC_HANDLE_BYTES 64
typedef struct tops_gla_p2p_args {
  int32_t rank, world;
  int32_t N, H, K, V;
  int32_t backward;
  const float* local_state;
  const float* decay;
  const float* boundary;
  float* out;
  float* total;
  void* const* regions;
  void* own_region;
  int32_t timeout_ms;
} tops_gla_p2p_args;
TOPS_API size_t tops_gla_p2p_region_size(const tops_gla_p2p_args* a);
TOPS_API int tops_gla_p2p_alloc(size_t bytes, void** region);
TOPS_API int tops_gla_p2p_free(void* region);
TOPS_API int tops_gla_ipc_handle(const void* region, void* handle);
TOPS_API int tops_gla_ipc_open(const void* handle, void** region);
TOPS_API int tops_gla_ipc_close(void* region);
TOPS_API int tops_gla_p2p_exchange(const tops_gla_p2p_args* a, void* stream);
/* The two halves of p2p_exchange apart, for a producer that pushes its own state:
 * p2p_combine is the wait + prefix / suffix kernel alone (the push must have been made by
 * one of the span_begin_p2p calls below, or by p2p_exchange's own push, for this epoch).
 * chunk_{fwd,bwd}_span_begin_p2p are tops_gla_chunk_{fwd,bwd}_span_begin with the state
 * exchange's push fused into the kernel that computes the span's own state: the rank's
 * (S | D) -- backward (L | D), D = the forward's span decay passed in -- goes straight from
 * that kernel into every rank's region, followed by the epoch flags; no local copy of S or
 * L is written.  The forward still writes `decay` (kept for the backward).  x->N, H, K, V
 * must be the problem's B, H, K, V; x's rank, world, regions and own_region are used. */
TOPS_API int tops_gla_p2p_combine(const tops_gla_p2p_args* a, void* stream);
TOPS_API int tops_gla_chunk_fwd_span_begin_p2p(const tops_gla_chunk_fwd_args* a, float* decay,
                                               const tops_gla_p2p_args* x, void* stream);
TOPS_API int tops_gla_chunk_bwd_span_begin_p2p(const tops_gla_chunk_bwd_args* a, const float* decay,
                                               const tops_gla_p2p_args* x, void* stream);

/* ---- GLA layer pieces around the chunked op ------------ */

/* Fused RMSNorm x swish output gate over rows of V: y = x * rstd * w * silu(g),
 * rstd = 1/sqrt(mean(x^2) + eps) (written to rstd[rows], fp32, for the backward).
 * x, g, w, y in `dtype` (TOPS_F32 or TOPS_BF16); w may be NULL (no affine weight).
 * Replaces FusedRMSNormGated (tops/modules/fused_norm_gate.py:28; gold
 * tests/src/modules/fused_norm_gate.py:30-44) used by tops/layers/gla.py:323-329.
 * V: a multiple of 16 bytes, at most 512 (fp32) / 1024 (bf16) elements. */
TOPS_API int tops_gla_norm_gate_fwd(int64_t rows, int32_t V, int32_t dtype, float eps, const void* x, const void* g,
                                    const void* w, void* y, float* rstd, void* stream);
/* Backward: dx, dg (dtype) and, when dw != NULL, dw[V] (dtype, deterministic sum over
 * rows through the workspace). */
TOPS_API size_t tops_gla_norm_gate_bwd_workspace_size(int64_t rows, int32_t V);
TOPS_API int tops_gla_norm_gate_bwd(int64_t rows, int32_t V, int32_t dtype, const void* dy, const void* x,
                                    const void* g, const void* w, const float* rstd, void* dx, void* dg, void* dw,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Gate activation gk = logsigmoid(x) / normalizer, max(gk, clamp_min) when has_clamp;
 * x in dtype, gk fp32 (tops/layers/gla.py:285-287).  Backward: dx = dgk * sigmoid(-x) /
 * normalizer (0 where clamped). */
TOPS_API int tops_gla_gate_logsigmoid_fwd(int64_t n, int32_t dtype, float normalizer, float clamp_min,
                                          int32_t has_clamp, const void* x, float* out, void* stream);
TOPS_API int tops_gla_gate_logsigmoid_bwd(int64_t n, int32_t dtype, float normalizer, float clamp_min,
                                          int32_t has_clamp, const void* x, const float* dy, void* dx, void* stream);

/* ---- XLA custom calls (JAX frontend) ---------------------------------------
 * Status-returning legacy custom-call signature used by jax custom_call lowering:
 * (cudaStream_t, void** buffers, const char* opaque, size_t opaque_len,
 *  XlaCustomCallStatus*).  `opaque` is a tops_gla_xla_desc; the buffer order is
 * documented at each definition (csrc/xla_custom_call.cu).  They replace the
 * reference's in-process pl.pallas_call launches (tops/ops/gla/chunk.py:1147-1164,
 * tops/ops/gla/fused_recurrent.py:343-362) for JAX callers. */
typedef struct tops_gla_xla_desc {
  int32_t B, T, H, K, V, chunk_size, dtype;
  float scale;
  int32_t has_g, has_h0, out_final, has_dht, want_dh0, reverse;
  uint64_t saved_bytes, workspace_bytes;
} tops_gla_xla_desc;

TOPS_API void tops_gla_xla_chunk_fwd(void* stream, void** buffers, const char* opaque, size_t opaque_len,
                                     void* status);
TOPS_API void tops_gla_xla_chunk_bwd(void* stream, void** buffers, const char* opaque, size_t opaque_len,
                                     void* status);
TOPS_API void tops_gla_xla_recurrent_fwd(void* stream, void** buffers, const char* opaque, size_t opaque_len,
                                         void* status);

#ifdef __cplusplus
}
#endif

#endif /* TOPS_GLA_H_ */
