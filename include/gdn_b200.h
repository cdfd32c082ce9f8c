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
 * gdn_tc05_selftest -- diagnostic of the tensor-core path (no counterpart in
 * the reference): one CTA computes D (128 x N) = op(A) (128 x K) * B^T with
 * B (N x K), all row-major fp32, through tcgen05.mma into tensor memory.
 * mode bit 0: operands rounded to bf16 (kind::f16) instead of tf32;
 * bit 1: A negated by the instruction descriptor; bit 2: A read from tensor
 * memory (tf32 only).  N, K multiples of 16 in [16, 128].  *status (device
 * int32) is set to 1 if the bounded wait for the MMA timed out.
 */
int gdn_tc05_selftest(const float* A, const float* B, float* D, int N, int K, int mode,
                      int* status, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* GDN_B200_H */
