/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) Gated DeltaNet hot path.
 *
 * The Gated DeltaNet (GDN) layer of Qwen3.5/3.8-27B keeps, per sequence and
 * value head, an fp32 state S of shape (Dv, Dk) = (128, 128), row-contiguous
 * over Dk, and per token applies
 *
 *     alpha = exp(-exp(A_log) * softplus(a + dt_bias)),  beta = sigmoid(b)
 *     kS    = S k                                      (per row v: sum_dk S[v,dk] k[dk])
 *     S     = alpha * (S - beta * kS k^T) + beta * v k^T
 *     o     = S q
 *
 * Every entry point takes caller-owned device pointers, plain sizes and a
 * cudaStream_t (passed as void*), allocates nothing unless stated, throws
 * nothing and returns GDN_OK or a negative GDN_ERR_* code.  Arguments are
 * validated before any CUDA call; a rejected call touches no memory.  There is
 * no CPU fallback: without a usable GPU a call returns GDN_ERR_CUDA.
 *
 * Layouts (row-major, innermost last):
 *     q, k      (B, T, Hk, Dk)       bf16 (default) or fp32 (GDN_F_QKV_F32)
 *     v         (B, T, Hv, Dv)       same dtype as q, k
 *     a, b      (B, T, Hv)           fp32 gate pre-activations (or alpha/beta)
 *     A_log, dt_bias (Hv)            fp32
 *     state     (B, Hv, Dv, Dk)      fp32
 *     o         (B, T, Hv, Dv)       fp32 (default) or bf16 (GDN_F_O_BF16)
 *     ckpt      (B, Hv, T, Dv, Dk)   fp32 state after every position
 * Key head i serves value heads i*r .. i*r+r-1 with r = Hv / Hk
 * (repeat_interleave, python/qwen35.py:592-594).  Dk = Dv = 128.
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define GDN_OK             0
#define GDN_ERR_NULL      -1   /* a required pointer is NULL                   */
#define GDN_ERR_SHAPE     -2   /* unsupported or inconsistent sizes            */
#define GDN_ERR_ALIGN     -3   /* a pointer breaks its alignment rule          */
#define GDN_ERR_FLAGS     -4   /* unknown or contradictory flag bits           */
#define GDN_ERR_ALIAS     -5   /* buffers overlap in a way the call forbids    */
#define GDN_ERR_CUDA      -6   /* a CUDA call failed; see gdn_last_error()     */
#define GDN_ERR_RANGE     -7   /* an index argument is out of range            */

/* ---- flags of gdn_recurrent_fwd ---------------------------------------- */
#define GDN_F_QKV_F32       0x1u  /* q, k, v are fp32 (default bf16)                   */
#define GDN_F_O_BF16        0x2u  /* o is written as bf16 (default fp32)              */
#define GDN_F_GATES_DIRECT  0x4u  /* a holds alpha and b holds beta; A_log, dt_bias unused */
#define GDN_F_QK_L2NORM     0x8u  /* l2-normalise q, k per head (eps 1e-6 inside the
                                     rsqrt) and scale q by Dk^-1/2 inside the kernel */
#define GDN_F_OVERLAP_PREV  0x10u /* gdn_recurrent_fwd only: launch as a programmatic
                                     dependent of the previous kernel in the stream, so
                                     the launch and the state loads overlap its tail;
                                     every other input is read after it has completed.
                                     The caller guarantees that the previous kernel does
                                     not write this call's state_in (e.g. consecutive
                                     layers of a decode step).  Kernels further back are
                                     complete before the state loads start (the kernel
                                     lets its own dependents launch only after its wait),
                                     so two layers used in turn are safe.  Pays off at
                                     small batch (launch-latency bound), neutral at large
                                     batch. */

/* ---- flags of the front-end / back-end kernels --------------------------- */
#define GDN_F_CONV_BF16_OPS 0x100u  /* conv: MLX's per-op bf16 arithmetic (each product and
                                       partial sum rounded) instead of fp32 accumulation */
#define GDN_F_CONV_NO_SILU  0x200u  /* conv: skip the SiLU after the convolution */
#define GDN_F_NORM_IN_BF16  0x400u  /* gated norm: o is bf16 (default fp32) */
#define GDN_F_NORM_OUT_F32  0x800u  /* gated norm: out is fp32 (default bf16) */

/* Human-readable text of the last error on the calling thread ("" if none). */
const char* gdn_last_error(void);

/* Library version: major * 10000 + minor * 100 + patch. */
int gdn_version(void);

/*
 * gdn_take_device_error -- synchronise `stream`, then read and clear the
 * current device's kernel error word: 0 when no kernel of this library gave
 * up on a bounded wait since the last call, nonzero otherwise.  No
 * counterpart in the reference (MLX reports errors as exceptions).
 */
int gdn_take_device_error(void* stream, int* code);

/*
 * gdn_recurrent_fwd -- decode (T = 1) and speculative verify (T = k+1) step.
 *
 * Replaces delta::run (cpp/src/delta.hpp:66-68, cpp/src/delta.cpp:137-173) and
 * gated_delta_metal (python/delta_kernel.py:126-165), with the gate
 * computation of GatedDeltaNet::operator() (cpp/src/model.cpp:608-612) moved
 * inside the kernel: the north-star signature (q,k,v,a,b,A_log,dt_bias,state
 * -> o,state').
 *
 * state_in   NULL means a zero initial state.
 * state_out  may equal state_in (in-place update) but must not otherwise
 *            overlap it; may be NULL when ckpt is given (the final state is
 *            then ckpt[:, :, T-1]).
 * ckpt       NULL, or the per-position states (DeltaCache record mode,
 *            cpp/src/delta.cpp:87-94 "collect").
 * Alignment: state_in, state_out, ckpt 16 B; q, k 8 B (bf16) or 16 B (fp32).
 * T = 0 copies state_in to state_out.  B = 0 is a no-op.
 */
int gdn_recurrent_fwd(const void* q, const void* k, const void* v,
                      const float* a, const float* b,
                      const float* A_log, const float* dt_bias,
                      const float* state_in, float* state_out,
                      void* o, float* ckpt,
                      int B, int T, int Hk, int Hv, int Dk, int Dv,
                      unsigned flags, void* stream);

/*
 * gdn_recurrent_fwd_from_ckpt -- the same step, starting each sequence from a
 * committed speculative checkpoint instead of a dense state: the rollback of
 * DeltaCache::commit (cpp/src/model.cpp:439-457) done as an index, with no
 * copy.  For sequence b with n = commit_n[b] (device int32, 0 <= n <= Tsrc):
 * n == 0 starts from state_prev[b], otherwise from ckpt_src[b, :, n-1]
 * (ckpt_src laid out (B, Hv, Tsrc, Dv, Dk)).  A sequence whose n is out of
 * range gets a zero state, its o and states are still written, and *err_flag
 * (device int32, may be NULL) is set to 1.  state_out must not overlap
 * ckpt_src or state_prev; ckpt (the new checkpoints) must not overlap either.
 */
int gdn_recurrent_fwd_from_ckpt(const void* q, const void* k, const void* v,
                                const float* a, const float* b,
                                const float* A_log, const float* dt_bias,
                                const float* state_prev, const float* ckpt_src,
                                const int32_t* commit_n, int Tsrc,
                                float* state_out, void* o, float* ckpt,
                                int32_t* err_flag,
                                int B, int T, int Hk, int Hv, int Dk, int Dv,
                                unsigned flags, void* stream);

/*
 * gdn_recurrent_fwd_pool -- the decode / verify step over a serving batch whose
 * states live in a slot pool instead of a dense (B, Hv, D, D) array: sequence
 * b reads and writes slot slots[b] (device int32) of pool (n_slots, Hv, D, D)
 * fp32, so a continuous-batching engine changes the batch by rewriting
 * `slots` (a CUDA graph of the step stays valid) and never compacts states.
 * This is the HBM layout of DeltaCache::state across a batch
 * (cpp/src/model.hpp:211-227 keeps one dense state per sequence).
 *   start     pool[slot]; with commit_n / ckpt_src (both or neither) as in
 *             gdn_recurrent_fwd_from_ckpt: n == 0 -> pool[slot], 1..Tsrc ->
 *             ckpt_src[b, :, n-1] ((B, Hv, Tsrc, D, D), the previous block's).
 *   pool_write GDN_POOL_FINAL: pool[slot] := the state after position T-1;
 *             GDN_POOL_START: pool[slot] := the start state (a committed
 *             checkpoint materialised -- DeltaCache::commit, cpp/src/model.cpp:
 *             439-457 -- before a new record-mode block; with T = 0 it is only
 *             that); GDN_POOL_KEEP: the pool is not written (record mode).
 * Slots must be distinct within a call.  A slot outside [0, n_slots) gets a
 * zero start state, its o and ckpt are written, the pool is not, and
 * *err_flag (may be NULL) is set to 1.  Other arguments as gdn_recurrent_fwd.
 */
#define GDN_POOL_KEEP  0
#define GDN_POOL_FINAL 1
#define GDN_POOL_START 2
int gdn_recurrent_fwd_pool(const void* q, const void* k, const void* v,
                           const float* a, const float* b,
                           const float* A_log, const float* dt_bias,
                           float* pool, const int32_t* slots, int n_slots,
                           const float* ckpt_src, const int32_t* commit_n, int Tsrc,
                           int pool_write, void* o, float* ckpt, int32_t* err_flag,
                           int B, int T, int Hk, int Hv, int Dk, int Dv,
                           unsigned flags, void* stream);

/*
 * gdn_delta_run -- literal swap for delta::run (cpp/src/delta.hpp:66-68):
 * fp32, head-expanded q, k (B,L,H,Dk), v (B,L,H,Dv), precomputed alpha, beta
 * (B,L,H); S NULL for zeros; states (B,H,L,Dv,Dk) or NULL (collect = false).
 * Equivalent to gdn_recurrent_fwd with Hk = Hv = H and
 * GDN_F_QKV_F32 | GDN_F_GATES_DIRECT.
 */
int gdn_delta_run(const float* q, const float* k, const float* v,
                  const float* alpha, const float* beta, const float* S,
                  float* o, float* S_out, float* states,
                  int B, int L, int H, int Dk, int Dv, void* stream);

/*
 * gdn_chunked_fwd -- prefill: the chunked (WY / UT) form of the recurrence
 * over whole sequences, on the tensor cores.  Replaces chunked_delta
 * (python/qwen35.py:365-431) together with its gate, l2norm, q-scale and
 * head-repeat prologue (python/qwen35.py:586-600): q, k are the raw conv
 * outputs, normalised inside the kernel when GDN_F_QK_L2NORM is set.
 * Matches the reference's chunk size (64) and its clip of alpha at 1e-6.
 *   q, k   bf16, element (token t, key head i, d) at q[t*q_stride + i*128 + d]
 *   v      bf16, element (t, value head h, d) at v[t*v_stride + h*128 + d]
 *          (for the conv output (T, 10240): q = y, k = y + 2048,
 *          v = y + 4096, all strides 10240)
 *   a, b   (T, Hv) fp32 gate pre-activations; A_log, dt_bias (Hv) fp32
 *   state_in, state_out (B, Hv, Dv, Dk) fp32; NULL in = zeros; may be equal
 *   o      (T, Hv, Dv) fp32 (GDN_F_O_BF16: bf16), token-major like the input
 *   cu_seqlens  NULL (B sequences of T tokens; token t of sequence b is row
 *          b*T + t) or device int32 (B+1) offsets of packed sequences.
 * Flags: GDN_F_QK_L2NORM, GDN_F_O_BF16.  Strides multiples of 8 elements;
 * q, k, v, states 16-byte aligned.  One CTA per (sequence, value head).
 */
int gdn_chunked_fwd(const void* q, const void* k, const void* v,
                    long long q_stride, long long k_stride, long long v_stride,
                    const float* a, const float* b, const float* A_log, const float* dt_bias,
                    const float* state_in, float* state_out, void* o,
                    const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv,
                    unsigned flags, void* stream);

/*
 * gdn_chunked_workspace_bytes -- device workspace with which
 * gdn_chunked_fwd_ws runs B sequences of T tokens (packed = 0), or B packed
 * sequences of T tokens in all (packed != 0, an upper bound that holds for
 * any cu_seqlens), in one pass: 89 KiB per (64-token chunk, value head).
 * 0 for bad sizes.
 */
size_t gdn_chunked_workspace_bytes(int B, int T, int Hv, int packed);

/*
 * gdn_chunked_workspace_min_bytes -- the smallest workspace gdn_chunked_fwd_ws
 * accepts for B sequences and Hv value heads: one chunk per sequence per
 * window, plus B*Hv*64 KiB for the state carried between windows when the
 * call has no state_out (has_state_out == 0).  Smaller-than-one-pass
 * workspaces run the call window by window (chunks [c0, c0 + w) of every
 * sequence per window, w as large as the workspace allows), with the same
 * results.  0 for bad sizes.
 */
size_t gdn_chunked_workspace_min_bytes(int B, int Hv, int has_state_out);

/*
 * gdn_chunked_fwd_ws -- gdn_chunked_fwd split in two launches: the
 * state-independent part of every (chunk, value head) in parallel, written
 * to `workspace`, then the state chain per (sequence, value head) reading it
 * back.  Same arguments, results and flags as gdn_chunked_fwd (the same
 * function of the inputs as chunked_delta, python/qwen35.py:365-431); the
 * split exposes (chunks x heads) of parallel work where gdn_chunked_fwd
 * has (sequences x heads).  workspace: device memory, 256-byte aligned, at
 * least gdn_chunked_workspace_min_bytes(B, Hv, state_out != NULL) bytes
 * (gdn_chunked_workspace_bytes(B, T, Hv, cu_seqlens != NULL) for one pass;
 * less runs in windows), no initial contents needed, not overlapping the
 * states or o; calls that share one workspace must be ordered on a stream.
 */
int gdn_chunked_fwd_ws(const void* q, const void* k, const void* v,
                       long long q_stride, long long k_stride, long long v_stride,
                       const float* a, const float* b, const float* A_log, const float* dt_bias,
                       const float* state_in, float* state_out, void* o,
                       const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv,
                       unsigned flags, void* workspace, size_t workspace_size, void* stream);

/*
 * gdn_chunked_norm_fwd_ws -- gdn_chunked_fwd_ws with the gated RMSNorm of
 * gdn_gated_rmsnorm_fwd fused into the scan's epilogue: writes
 *     out[t*out_stride + (out_head0 + h)*128 + d]
 *         = bf16( o[t,h,d] * rsqrt(mean_d o[t,h,:]^2 + eps) * gamma[d] * silu(z[t,h,d]) )
 * instead of o (the reference's norm(o, z), cpp/src/model.cpp:350-354 and
 * :625-627, python/qwen35.py:159-180).  z: bf16, element (t, h, d) at
 * z[t*z_stride + h*128 + d], 16-byte aligned with z_stride a multiple of 8
 * (its rows are bulk-copied); gamma (128) fp32.  out_stride / out_head0 place
 * this call's Hv heads inside a wider row (e.g. the all-heads output of a
 * head-sharded layer); out 16-byte aligned, out_stride a multiple of 8.
 * Flags: GDN_F_QK_L2NORM only.  Other arguments and the workspace as
 * gdn_chunked_fwd_ws.
 */
int gdn_chunked_norm_fwd_ws(const void* q, const void* k, const void* v,
                            long long q_stride, long long k_stride, long long v_stride,
                            const float* a, const float* b, const float* A_log, const float* dt_bias,
                            const float* state_in, float* state_out,
                            const void* z, long long z_stride, const float* gamma, float eps,
                            void* out, long long out_stride, int out_head0,
                            const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv,
                            unsigned flags, void* workspace, size_t workspace_size, void* stream);

/*
 * gdn_spec_verify -- the acceptance step of an MTP speculative-verify block
 * on the device (python/speculative.py:161-190, cpp/src/session.cpp:495-511),
 * so the rollback index feeds gdn_recurrent_fwd_from_ckpt and
 * gdn_conv_commit without a host round trip.  Per sequence b:
 *   accept_i = q_i[d_i] > 0 ? u_accept[b,i] * q_i[d_i] <= p_i[d_i] : p_i[d_i] > 0
 *   accept_len[b] = j = number of leading accepted drafts, commit_n[b] = j + 1
 *   token[b] = inverse-CDF draw with uniform u_sample[b] from p_k (j == k)
 *              or from normalize(max(p_j - q_j, 0)) (p_j when that is empty),
 *              i.e. the smallest v with u * sum(r) < sum_{x<=v} r[x]
 *   p (B, k+1, V) fp32 target distributions of the verify pass
 *   q (B, k, V) fp32 draft distributions; draft (B, k) int32 draft tokens
 *   u_accept (B, k), u_sample (B) fp32 uniforms in [0, 1)
 * 1 <= k <= 32, V <= 4,194,304.  A draft token outside [0, V) is treated as
 * rejected and sets *err_flag.
 */
int gdn_spec_verify(const float* p, const float* q, const int32_t* draft,
                    const float* u_accept, const float* u_sample, int B, int k, long long V,
                    int32_t* accept_len, int32_t* commit_n, int32_t* token, int32_t* err_flag,
                    void* stream);

/*
 * gdn_chunked_norm_gather_ws -- gdn_chunked_norm_fwd_ws of one rank of a
 * head-sharded layer whose epilogue writes the normed rows straight into the
 * all-heads output buffer of every rank over NVLink (the reference's layer
 * boundary, cpp/src/model.cpp:625-641, with the per-head outputs gathered):
 * compute and the all-gather are one kernel, no separate collective.
 *   out_ranks[r]  device pointer of rank r's output buffer (this process's
 *                 view of it, e.g. a CUDA IPC / symmetric-memory mapping),
 *                 out_elems bf16 elements each, 16-byte aligned; this rank's
 *                 heads land at head offset out_head0 of every row
 *   flag_ranks[r] rank r's array of `world` uint32 counters (same kind of
 *                 mapping); after its scan this call adds 1 to
 *                 flag_ranks[r][rank] for every r (release, system scope)
 * 1 <= world <= 8.  The host arrays are read during the call.  A consumer
 * waits with gdn_gather_wait before reading its buffer; buffers must not be
 * read by a consumer while a later call writes them (alternate two).
 */
int gdn_chunked_norm_gather_ws(const void* q, const void* k, const void* v,
                               long long q_stride, long long k_stride, long long v_stride,
                               const float* a, const float* b, const float* A_log, const float* dt_bias,
                               const float* state_in, float* state_out,
                               const void* z, long long z_stride, const float* gamma, float eps,
                               void* const* out_ranks, uint32_t* const* flag_ranks, int world, int rank,
                               long long out_elems, long long out_stride, int out_head0,
                               const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv,
                               unsigned flags, void* workspace, size_t workspace_size, void* stream);

/*
 * gdn_gather_wait -- stream-ordered wait until every rank r < world has
 * signalled at least `expected` calls in flags[r] (this rank's counter array
 * of gdn_chunked_norm_gather_ws), with acquire semantics at system scope.
 * Bounded: after about 4 s it sets *err_flag and the device error word
 * (gdn_take_device_error) and returns.
 */
int gdn_gather_wait(const uint32_t* flags, int world, unsigned expected, int32_t* err_flag, void* stream);

/*
 * gdn_gather_wait_timeout -- gdn_gather_wait with the caller's limit,
 * 1 <= limit_ms <= 60000 milliseconds of %globaltimer polling.  No
 * counterpart in the reference (it runs on one device).
 */
int gdn_gather_wait_timeout(const uint32_t* flags, int world, unsigned expected, unsigned limit_ms,
                            int32_t* err_flag, void* stream);

/*
 * gdn_ipc_export / gdn_ipc_open / gdn_ipc_close -- share a device buffer with
 * the other processes of a head-sharded layer for gdn_chunked_norm_gather_ws:
 * export writes the 64-byte CUDA IPC handle of the allocation holding `ptr`
 * and ptr's offset in it; a peer opens it with its own device current (peer
 * access from that device is enabled lazily) and gets the mapping's base
 * (for gdn_ipc_close) and the buffer's address.  Plain peer mappings.
 */
int gdn_ipc_export(const void* ptr, void* handle_out, size_t* offset_out);
int gdn_ipc_open(const void* handle, size_t offset, void** base_out, void** ptr_out);
int gdn_ipc_close(void* base);

/* Size of the fixed device scratch that gdn_chunked_fwd_static uses. */
#define GDN_CHUNKED_STATIC_SCRATCH_BYTES (64ull << 20)

/*
 * gdn_chunked_fwd_static -- gdn_chunked_fwd_ws without a caller workspace:
 * the same two launches and results, with the scratch in a fixed 64 MiB
 * device array of the library (GDN_CHUNKED_STATIC_SCRATCH_BYTES), so the call
 * allocates no memory.  No counterpart in the reference; it serves callers
 * that cannot allocate device memory at call time.
 *   Arguments, flags and results as gdn_chunked_fwd.
 *   Limit: a call whose records fit the scratch runs in one pass, a longer
 *   one in windows of chunks (bit-identical results); only a call with
 *   gdn_chunked_workspace_min_bytes(B, Hv, state_out != NULL) above
 *   GDN_CHUNKED_STATIC_SCRATCH_BYTES (one record per sequence and value head
 *   no longer fits, e.g. B x Hv above about 730 with state_out, 430 without) returns GDN_ERR_SHAPE and
 *   touches nothing.
 *   The first call on each device looks up the scratch's address
 *   (cudaGetSymbolAddress, with that device current) and sets the kernels'
 *   shared-memory attributes; make that first call before any stream capture,
 *   and before an engine hands the device's free memory to its own pools:
 *   the 64 MiB array belongs to the module that holds every chunked kernel,
 *   so every process that uses any chunked entry point pays it on each
 *   device, reserved when that module is loaded there (lazily, at its first
 *   use, under CUDA's default lazy loading).  The address is cached per
 *   device for the life of the process: do not use the library across a
 *   cudaDeviceReset.
 *   Nothing in the scratch needs to start at zero.  There is one scratch per
 *   device: calls on the same device that overlap in time (different streams
 *   or host threads without ordering between them) race on it.
 */
int gdn_chunked_fwd_static(const void* q, const void* k, const void* v,
                           long long q_stride, long long k_stride, long long v_stride,
                           const float* a, const float* b, const float* A_log, const float* dt_bias,
                           const float* state_in, float* state_out, void* o,
                           const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv,
                           unsigned flags, void* stream);

/*
 * gdn_conv1d_fwd -- causal depthwise conv1d (kernel K = 4, no bias) over the
 * concatenated q|k|v channels, then SiLU: the front end of
 * GatedDeltaNet::operator() (DepthwiseConv::operator(), cpp/src/model.cpp:
 * 385-395, and the silu at :588; python/qwen35.py:642-660, :581).
 *   x      (B, T, C) bf16, or packed (T, C) when cu_seqlens is given
 *   w      (C, K) bf16 -- the stored (C, 1, K) conv1d weight
 *   state_in  (B, K-1, C) bf16 carried window, NULL for zeros
 *   state_out (B, K-1, C) bf16 or NULL: the last K-1 rows of [state_in; x_b]
 *   y      like x, bf16: silu(conv) (GDN_F_CONV_NO_SILU: conv only)
 *   cu_seqlens  NULL (B sequences of T tokens) or device int32 (B+1) offsets
 *          of B packed sequences: cu[0] = 0, nondecreasing, cu[B] = T.
 * fp32 products and sums by default; GDN_F_CONV_BF16_OPS rounds every
 * product and partial sum to bf16 as MLX does for bf16 activations.
 * C a multiple of 8; x, w, y, states 16-byte aligned; y must not overlap x.
 */
int gdn_conv1d_fwd(const void* x, const void* w, const void* state_in, void* state_out, void* y,
                   const int32_t* cu_seqlens, int B, int T, int C, int K, unsigned flags,
                   void* stream);

/*
 * gdn_conv_commit -- conv half of DeltaCache::commit (cpp/src/model.cpp:
 * 446-447, python/qwen35.py:320-323) after a recorded block of T tokens:
 * state_out[b] = rows n .. n+K-2 of [state_prev[b]; x[b]] with n = commit_n[b]
 * (device int32, 0 <= n <= T).  Out-of-range n uses n = 0 and sets *err_flag.
 *   state_prev (B, K-1, C) bf16 or NULL (zeros); x (B, T, C) bf16.
 */
int gdn_conv_commit(const void* state_prev, const void* x, const int32_t* commit_n, void* state_out,
                    int32_t* err_flag, int B, int T, int C, int K, void* stream);

/*
 * gdn_conv1d_fwd_pool / gdn_conv_ring_append -- the conv window of a serving
 * batch as a ring per pool slot (no counterpart in the reference, whose
 * DeltaCache::conv is one dense (1, K-1, C) window per sequence rebuilt by
 * concatenation, cpp/src/model.cpp:385-395, 446-447).  ring is (n_slots, K-1,
 * C) bf16 and ring_pos (n_slots) int32 the row of each slot's oldest entry.
 * gdn_conv1d_fwd_pool is gdn_conv1d_fwd reading sequence b's carried window
 * from slot slots[b] (oldest first from ring_pos) and writing no state.
 * gdn_conv_ring_append then moves the first n_b tokens of each sequence into
 * its ring (n_b = counts[b], or the sequence's length when counts is NULL;
 * 0 <= n_b <= length): a decode step writes one row instead of shifting K-1,
 * and after a speculative block counts = commit_n is the conv half of
 * DeltaCache::commit.  Call append after every conv reading the same slots
 * (stream order).  Slots must be distinct within a call; a slot outside
 * [0, n_slots) or an n_b out of range reads a zero window / appends nothing
 * and sets *err_flag (may be NULL).  A fresh slot needs a zeroed ring and
 * ring_pos = 0.
 */
int gdn_conv1d_fwd_pool(const void* x, const void* w, const void* ring, const int32_t* ring_pos,
                        const int32_t* slots, int n_slots, void* y, const int32_t* cu_seqlens,
                        int B, int T, int C, int K, unsigned flags, int32_t* err_flag, void* stream);
int gdn_conv_ring_append(const void* x, void* ring, int32_t* ring_pos, const int32_t* slots, int n_slots,
                         const int32_t* counts, const int32_t* cu_seqlens, int B, int T, int C, int K,
                         int32_t* err_flag, void* stream);

/*
 * gdn_gated_rmsnorm_fwd -- normalise, then gate (GatedRMSNorm,
 * cpp/src/model.cpp:350-354, python/qwen35.py:159-180):
 *   out = o * rsqrt(mean(o^2) + eps) * gamma * silu(z)
 * over rows of D = 128.  o (rows, D) fp32 (GDN_F_NORM_IN_BF16: bf16), z (rows,
 * D) bf16, gamma (D) fp32 used as stored (not zero-centred), out (rows, D)
 * bf16 (GDN_F_NORM_OUT_F32: fp32).  out may equal o when both are the same
 * dtype and width.
 */
int gdn_gated_rmsnorm_fwd(const void* o, const void* z, const float* gamma, void* out, long long rows,
                          int D, float eps, unsigned flags, void* stream);

/*
 * gdn_gemm_bf16 -- C = A B^T on the tensor cores (tcgen05, fp32 accumulation,
 * bf16 rounding of C): the block's plain projections, in_proj_z / in_proj_a /
 * in_proj_b (weights cpp/src/model.cpp:174-176, applied at :608-609 and :625;
 * python/qwen35.py:561-563, 597-598, 628) and out_proj (cpp/src/model.cpp:177,
 * 641; python/qwen35.py:564, 640), which MLX runs as bf16 matmuls.  A (M, K) with row stride
 * lda, B (N, K) with row stride ldb (a Linear's weight as stored), both bf16;
 * N, K, lda, ldb multiples of 8, A and B 16-byte aligned.  C (M, ldc) bf16,
 * 16-byte aligned, ldc a multiple of 8.  With C32 non-null, columns n_f32 ..
 * N-1 (n_f32 a multiple of 8) are written to C32 as fp32 holding the
 * bf16-rounded values -- the .astype(float32) of the a / b projections
 * (cpp/src/model.cpp:608-609) -- as a stack of (M, ld32) matrices (column
 * n_f32 + j goes to matrix j / ld32, column j % ld32; ld32 = N - n_f32 gives
 * one (M, N - n_f32) matrix, ld32 = Hv gives a then b as two contiguous (M,
 * Hv) arrays), and C receives columns 0 .. n_f32-1 only.
 * Allocates nothing (the tensor maps are kernel parameters).
 */
int gdn_gemm_bf16(const void* A, const void* B, void* C, float* C32, int M, int N, int K, long long lda,
                  long long ldb, long long ldc, long long ld32, int n_f32, void* stream);

/*
 * gdn_in_proj_conv -- in_proj_qkv followed by the causal depthwise conv1d
 * (kernel 4) and SiLU in one tensor-core kernel (weights cpp/src/model.cpp:
 * 173, applied at :586-588, DepthwiseConv cpp/src/model.cpp:385-395;
 * python/qwen35.py:560, 577-578, 642-660):
 *     p = bf16(x W^T)                       (the projection's own rounding)
 *     y[t, c] = silu(sum_j w[c, j] * [window; p_seq][t + j, c]),  j = 0..3
 * with fp32 tap arithmetic exactly as gdn_conv1d_fwd's default mode, so y is
 * bit-identical to gdn_conv1d_fwd applied to gdn_gemm_bf16's output; the
 * projection never reaches HBM.  x (tokens, K) bf16 with row stride ldx,
 * packed with cu_seqlens (B+1) int32, or B sequences of T tokens when
 * cu_seqlens is NULL; W (N, K) with row stride ldw; conv_w (N, 4) bf16;
 * state_in / state_out (B, 3, N) bf16 carried windows (state_in NULL: zeros;
 * state_out NULL: not written); y (tokens, ldy) bf16.  N, ldy multiples of 8.
 */
int gdn_in_proj_conv(const void* x, const void* W, const void* conv_w, const void* state_in, void* state_out,
                     void* y, const int32_t* cu_seqlens, int B, int T, int N, int K, long long ldx,
                     long long ldw, long long ldy, void* stream);

/*
 * gdn_tc05_selftest -- diagnostic of the tensor-core path (no counterpart in
 * the reference): one CTA computes D (128 x N) = op(A) (128 x K) * B^T with
 * B (N x K), all row-major fp32, through tcgen05.mma into tensor memory.
 * mode bit 0: operands rounded to bf16 (kind::f16) instead of tf32;
 * bit 1: A negated by the instruction descriptor; bit 2: A read from tensor
 * memory (tf32 only); bit 3: A laid out MN-major in shared memory; bit 4: B
 * laid out MN-major; bit 8 (with bit 0): fp16 instead of bf16; bit 7
 * (alone): issue no MMA and wait on the barrier
 * with a poll budget of 4096, so that the bounded wait runs out (a test of
 * the timeout path: *status and the device error word are set, D is not
 * written, the kernel returns).  N, K multiples of 16 in [16, 128].
 * *status (device int32) is set to 1 if the bounded wait for the MMA timed
 * out, and so is the device error word (gdn_take_device_error).
 */
int gdn_tc05_selftest(const float* A, const float* B, float* D, int N, int K, int mode,
                      int* status, void* stream);

/*
 * gdn_tc05_pair_selftest -- diagnostic of the CTA-pair tensor-core form (no
 * counterpart in the reference): a cluster of two CTAs computes
 * A (128 x K) * B^T, B (N x K), row-major fp32 holding tf32 values, with
 * tcgen05.mma.cta_group::2 (M = 128): CTA r supplies A rows 64r..64r+63 and
 * B rows (N/2)r..(N/2)r+N/2-1.  raw (2 x 128 x N/2 floats) receives each
 * CTA's tensor memory as it lies, lane by lane, so that a test checks the
 * accumulator layout the pair scan relies on.  N a multiple of 32 in
 * [32, 256], K a multiple of 8 in [8, 128].  *status is set to 1 (and the
 * device error word) if the bounded wait for the MMA timed out.
 */
int gdn_tc05_pair_selftest(const float* A, const float* B, float* raw, int N, int K, int* status, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* GDN_B200_H */
