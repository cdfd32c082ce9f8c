// Chunked (WY / UT) prefill of the Gated DeltaNet recurrence on the sm_100a
// tensor cores (tcgen05 + tensor memory).
//
// Math (python/qwen35.py:365-431, chunked_delta), per sequence b, value head
// h and chunk of C = 64 tokens, with r_k, r_q the per-token l2-norm factors
// (q additionally scaled by Dk^-1/2), Gam_i = sum_{j<=i} log(clip(alpha_j,
// 1e-6, 1)), g_i = exp(Gam_i), and the state kept as R = S^T (Dv, Dk) -- the
// reference's own (Dv, Dk) layout:
//
//   G = K K^T, P = Q K^T                        (raw bf16 rows; one MMA)
//   A[i,j] = beta_i r_ki r_kj e^{Gam_i-Gam_j} G[i,j]          (j < i)
//   T^-1   = (I + A)^-1                          (blocked forward substitution)
//   U0^T   = V^T diag(beta) T^-T                 (MMA)
//   W      = T^-1 diag(beta g r_k) K             (MMA)
//   M[i,j] = r_qi r_kj e^{Gam_i-Gam_j} P[i,j]                  (j <= i)
//   ---- everything above is independent of the state ("prep") ----
//   U^T    = U0^T - R W^T                        (MMA, R from tensor memory)
//   y^T    = R (diag(g r_q) Q)^T + U^T M^T       (MMAs)      -> o
//   R     <- g_last R + U^T diag(e^{Gam_last-Gam} r_k) K       (MMA)
//
// which is the reference's y = M U0 + Qeff S, U = U0 - Kt S,
// S <- cumg_last S + k^T (ratio U) regrouped so that every product has
// M = 128 rows and the state stays on chip between chunks.  All MMAs are
// kind::tf32 with fp32 accumulation: the bf16 inputs are exact in tf32,
// derived operands are rounded to nearest tf32 once.
//
// Two schedules share the phase functions below:
//   * fused (gdn_chunked_fwd): one CTA per (sequence, value head) runs prep
//     and state update chunk after chunk; no scratch memory.
//   * split (gdn_chunked_fwd_ws): a prep kernel runs the state-independent
//     work of every (chunk, value head) in parallel and writes its operands,
//     in the shared-memory layouts the tensor cores read, to a workspace; a
//     scan kernel per (sequence, value head) bulk-copies them in and runs
//     only the state chain, so the serial work per chunk shrinks to the
//     state-dependent MMAs and their epilogues.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "gdn_conv_math.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {

#ifdef GDN_CHUNK_TIMING
// phase cycles of one CTA in the middle of the grid (a steady-state wave, warm
// instruction cache): [0,13) fused, [8,15), [16,24) and 31 prep, [24,29) scan
__device__ long long g_chunk_timing[32];
#define GDN_TICK(slot)                                                          \
  do {                                                                          \
    if (blockIdx.x == gridDim.x / 2 && blockIdx.y == 0 && threadIdx.x == 0) {   \
      const long long now_ = clock64();                                         \
      g_chunk_timing[slot] += now_ - c.tick;                                    \
      c.tick = now_;                                                            \
    }                                                                           \
  } while (0)
#else
#define GDN_TICK(slot) \
  do {                 \
  } while (0)
#endif

namespace {

constexpr int kC = 64;          // tokens per chunk (python/qwen35.py:365)
constexpr int kThreads = 256;   // 8 warps: warp w owns TMEM lane quarter w % 4, column half w / 4

// shared memory map of the fused kernel, bytes; tensor-core operands in the
// K-major no-swizzle layout (LBO 128 B), written row-wise so that a warp's
// stores hit distinct banks
constexpr uint32_t kSbo128 = (kD * 4 / 16) * 128;   // 8-row group stride of 128-wide fp32 rows
constexpr uint32_t kSbo64 = (kC * 4 / 16) * 128;    // ... of 64-wide fp32 rows
constexpr int kPad = kC + 1;                        // row stride of X (plain)
constexpr int kPadA = kC + 4;                       // row stride of A^T (plain, 16-byte rows)
constexpr uint32_t kOffKQ = 0;                      // [K; Q] rows            128 x 128 (64 KiB)
constexpr uint32_t kOffKt = kOffKQ + 128 * kD * 4;  // K^T, scaled            128 x 64  (32 KiB)
constexpr uint32_t kOffVt = kOffKt + kD * kC * 4;   // V^T diag(beta), U^T    128 x 64  (32 KiB)
constexpr uint32_t kOffTi = kOffVt + kD * kC * 4;   // T^-1                    64 x 64  (16 KiB)
constexpr uint32_t kOffM = kOffTi + kC * kC * 4;    // M (must follow T^-1)    64 x 64  (16 KiB)
constexpr uint32_t kOffW = kOffM + kC * kC * 4;     // W rows 64 x 128 (32 KiB); X during the solve
constexpr uint32_t kOffA = kOffW + kC * kD * 4;     // A^T, plain, row stride 68
constexpr uint32_t kOffY = kOffA + kC * kPadA * 4;  // solve temporaries 3 x 16 x 16
constexpr uint32_t kOffSc = kOffY + 3 * 256 * 4;    // per-token scalars, 10 x 64
constexpr uint32_t kOffBar = kOffSc + 10 * kC * 4;  // mbarrier, TMEM base
constexpr uint32_t kSmemBytes = kOffBar + 64;

// shared memory map of the prep kernel (one CTA per (chunk, value head),
// three per SM).  Rows of K, Q and V arrive by cp.async in one layout,
// element (t, d) at kmajor_offset(t, d, 2, 2048): read as an R x K operand it
// is the K-major [K; Q] of G | P = [K; Q] K^T, read as an M x K operand with
// M = d it is the MN-major K^T / V^T of W^T and U0^T, so no row is ever
// transposed.  Regions are reused as the phases go.
constexpr uint32_t kSboKQ = (kD * 2 / 16) * 128;    // 8-row group stride of 128-wide bf16 rows (2048)
constexpr uint32_t kQK = 0;                         // K rows, bf16 (16 KiB)
constexpr uint32_t kQQ = kQK + kC * kD * 2;         // Q rows (16 KiB); V rows once G | P and Q-tilde are done
constexpr uint32_t kQA = kQQ + kC * kD * 2;         // A, row-major, row stride kPadA; then the U0 operand hi | lo
constexpr uint32_t kQX = kQA + kC * kPadA * 4;      // X = T^-1, row-major, row stride kPadA; then the W operand hi | lo
constexpr uint32_t kQY = kQX + kC * kPadA * 4;      // products of the blocked solve, 1024 floats
constexpr uint32_t kQSc = kQY + 1024 * 4;           // per-token scalars, 10 x 64
constexpr uint32_t kQGa = kQSc + 10 * kC * 4;       // log-decay prefixes, then betas, of up to kPrepGroup value heads
constexpr int kPrepGroup = 3;                       // value heads per prep CTA (at most)
constexpr uint32_t kQBar = kQGa + 2 * kPrepGroup * kC * 4;   // mbarrier, TMEM base, (sequence, chunk) broadcast
constexpr uint32_t kPrepSmem = kQBar + 64;
constexpr uint32_t kSboOp = (kC * 2 / 16) * 128;    // 8-row group stride of the 64-token bf16 operands (1024)
static_assert(2 * kC * kC * 2 <= kC * kPadA * 4, "prep: an operand pair fits the A / X region it replaces");
static_assert(3 * (kPrepSmem + 1024) <= 233472, "prep: three CTAs per SM");

constexpr uint32_t kTmemCols = 512;
// fused: [0,128) R (tf32), [128,256) R (fp32 master, state-update
// accumulator), [256,320) G|P during (a); [256,384) W (lanes 0-63) during (c);
// [384,448) U^T; [448,512) y^T
constexpr uint32_t kColR = 0, kColDR = 128, kColGP = 256, kColW = 256, kColU = 384, kColY = 448;
// prep: [0,64) G|P, then W^T; [64,128) U0^T
constexpr uint32_t kPrepTmemCols = 128;
constexpr uint32_t kPColGP = 0, kPColW = 0, kPColU = 64;

// One workspace record per (chunk, value head): the prep kernel's outputs as
// tensor-core operands (K-major, no swizzle) in three groups that the scan
// kernel bulk-copies into shared memory a chunk ahead of their use.  -W and
// Qs form one 128-row B operand, M and K-hat^T one 192-row B operand, all
// fp16 for kind::f16 products (the same 10-bit mantissa as tf32, at half the
// bytes and half the MMA instructions of the state chain); U0^T stays fp32
// (it is added in the scan's epilogue).
constexpr uint32_t kSboH128 = (kD * 2 / 16) * 128;  // 8-row group stride of 128-wide 16-bit rows (2048)
constexpr uint32_t kSboH64 = (kC * 2 / 16) * 128;   // ... of 64-wide 16-bit rows (1024)
constexpr uint32_t kRecW = 0;                       // -W, 64 x 128 fp16, SBO 2048           group 1
constexpr uint32_t kRecQ = kRecW + kC * kD * 2;     // diag(g r_q) Q, 64 x 128 fp16         group 1
constexpr uint32_t kRecM = kRecQ + kC * kD * 2;     // M, 64 x 64 fp16, SBO 1024             group 2
constexpr uint32_t kRecKh = kRecM + kC * kC * 2;    // K-hat^T, 128 x 64 fp16, SBO 1024      group 2
constexpr uint32_t kRecU = kRecKh + kD * kC * 2;    // U0^T fp32 by column quads, see u0_index  group 3
constexpr uint32_t kRecSc = kRecU + kD * kC * 4;    // [0] = g_last                          group 3
constexpr uint32_t kRecBytes = kRecSc + 1024;       // multiple of 256
// fp16 pairs and quads for the record's operands (round to nearest)
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint2 pack_h4(float a, float b, float c, float d) {
  return make_uint2(pack_h2(a, b), pack_h2(c, d));
}
// address of element (r, k) of a K-major 16-bit operand with 8-row stride sbo
__device__ __forceinline__ unsigned char* at_h(unsigned char* base, int r, int k, uint32_t sbo) {
  return base + tc::kmajor_offset(r, k, 2, sbo);
}
// float4 index of U0^T[row][4 quad .. 4 quad + 3] in the record: value rows
// 0-63 and 64-127 are two contiguous blocks of 16 quads x 64 rows.
__host__ __device__ constexpr int u0_index(int quad, int row) {
  return (row >> 6) * (16 * 64) + quad * 64 + (row & 63);
}
constexpr size_t kWsHeader = 256;                   // then the chunk prefix (B+1 int32), then records

// shared memory map of the scan kernel: the record, then U^T and the barriers
// shared memory map of the scan kernel: group 1 at [0, 64K) and group 2 at
// [64K, 112K), each with its two operands in chunk-parity order (see the
// kernel); group 3 at the record's own offsets; then U^T and the barriers
constexpr uint32_t kScanG1 = 0;
constexpr uint32_t kScanG2 = kRecM;
constexpr uint32_t kScanR = kRecBytes;              // fp16(R) 128 x 128 (32 KiB), A of the first batch
constexpr uint32_t kScanU = kScanR + kD * kD * 2;   // fp16(U^T) 128 x 64 (16 KiB), A of the second batch
constexpr uint32_t kScanBar = kScanU + kD * kC * 2; // 4 mbarriers, TMEM base at +32
constexpr uint32_t kScanNorm = kScanBar + 64;       // fused norm: partial sums of squares, 4 x 64 floats
constexpr uint32_t kScanSmem = kScanNorm + 4 * kC * 4;
// fused norm: mbarriers "y of a chunk parity is in TMEM" (arrived by the MMA
// commit) and "... has been read" (one arrival per norm warp), then the
// failure flag the norm warps poll; the first 256 bytes of kScanNorm hold
// the norm warps' per-token partial sums
constexpr uint32_t kScanYBar = kScanNorm + 768;
constexpr uint32_t kScanGl1 = kScanNorm + 640;      // g_last, copied with group 1 (for the first batch's R scaling)
constexpr uint32_t kScanFail = kScanNorm + 800;
// fused norm: z rows of three chunks (chunk ch in buffer ch % 3), 64 x 128
// bf16 each; a chunk's normed output rows overwrite its z rows in place
constexpr uint32_t kScanZ = kScanSmem;
constexpr uint32_t kZBuf = kC * kD * 2;
constexpr uint32_t kScanSmemNorm = kScanZ + 3 * kZBuf;
static_assert(kScanSmemNorm <= 232448, "scan with the fused norm: shared memory per CTA");


__host__ __device__ constexpr size_t records_offset(int B) {
  return kWsHeader + (static_cast<size_t>(B + 1) * 4 + 255) / 256 * 256;
}

struct ChunkParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long long q_stride, k_stride, v_stride;   // elements between consecutive tokens
  const float* a;
  const float* b;
  const float* A_log;
  const float* dt_bias;
  const float* state_in;
  float* state_out;
  void* o;
  const int32_t* cu;
  int B, T, Hk, Hv;
  unsigned flags;
  int* err;
  // split schedule
  unsigned char* ws;              // workspace (256-byte aligned)
  int32_t* chunk_prefix;          // (B+1) first record slot of each sequence (packed batches)
  long long n_slots;              // record slots (chunks over all sequences, or an upper bound)
  int nch_uniform;                // chunks per sequence in this window when cu == null
  size_t rec_off;                 // byte offset of the records in the workspace
  int win_c0, win_len;            // window: chunks [win_c0, win_c0 + win_len) of every sequence
  int prep_group;                 // value heads per prep CTA (they share one key head)
  float* carry;                   // state between windows (state_out, a workspace region, or null)
  // gated RMSNorm fused into the scan's epilogue (o is then the bf16 output):
  // out[t * out_stride + (out_head0 + h) * 128 + d] = rms_norm(o)[d] gamma[d] silu(z[t, h, d])
  const __nv_bfloat16* z;
  long long z_stride;             // elements between consecutive tokens of z
  const float* gamma;
  float eps;
  long long out_stride;
  int out_head0;
  // fused norm output destinations: this rank's rows go to every buffer in
  // dst (the caller's own first or not; one per rank of a head-sharded
  // layer, same layout in each), out_elems elements each
  __nv_bfloat16* dst[8];
  int n_dst;
  long long out_elems;
};

__device__ __forceinline__ float softplus_f(float x) { return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x))); }

__device__ __forceinline__ float* at(unsigned char* base, int r, int c, uint32_t sbo) {
  return reinterpret_cast<float*>(base + tc::kmajor_offset(r, c, 4, sbo));
}

// 32 bf16 starting at p (16-byte aligned) -> fp32
__device__ __forceinline__ void load32(const __nv_bfloat16* p, bool valid, float (&f)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 raw = valid ? __ldg(reinterpret_cast<const uint4*>(p) + q) : make_uint4(0, 0, 0, 0);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = __bfloat1622float2(h[e]);
      f[q * 8 + 2 * e] = t.x;
      f[q * 8 + 2 * e + 1] = t.y;
    }
  }
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]) {
  float t[16];
#pragma unroll
  for (int c = 0; c < N / 16; ++c) {
    tc::tmem_ld16(taddr + c * 16, t);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[c * 16 + i] = t[i];
  }
  tc::tmem_ld_wait();
}

__device__ __forceinline__ uint64_t desc(const unsigned char* base, uint32_t byte_off, uint32_t sbo) {
  return tc::smem_desc(ptx::smem_u32(base) + byte_off, 128, sbo);
}

// Token range of sequence b.
__device__ __forceinline__ void seq_range(const ChunkParams& p, int b, long long& s0, long long& s1) {
  if (p.cu) {
    s0 = p.cu[b];
    s1 = p.cu[b + 1];
    if (s1 < s0) s1 = s0;
  } else {
    s0 = static_cast<long long>(b) * p.T;
    s1 = s0 + p.T;
  }
}

// Per-CTA state shared by the phase functions.
struct Ctx {
  unsigned char *sKQ, *sKt, *sVt, *sTi, *sM, *sW;
  float *sX, *sA, *sY;
  float *s_pre, *s_gam, *s_g, *s_ratio, *s_beta, *s_rk, *s_rq, *s_misc, *s_kw, *s_kh;
  uint64_t* bar;
  int tid, warp, lane, quarter, half, row;
  int h, kh;
  float A_h, dtb, log_clip, qscale;
  bool l2;
  uint32_t tb, my;   // TMEM base, this warp's lane quarter
  uint32_t phase;
#ifdef GDN_CHUNK_TIMING
  long long tick;
#endif
};

// Per-token scalar arrays at sc (10 x 64 floats).
__device__ __forceinline__ void ctx_scalars(Ctx& c, float* sc) {
  c.s_pre = sc;
  c.s_gam = sc + 64;
  c.s_g = sc + 128;
  c.s_ratio = sc + 192;
  c.s_beta = sc + 256;
  c.s_rk = sc + 320;
  c.s_rq = sc + 384;
  c.s_misc = sc + 448;
  c.s_kw = sc + 512;      // beta g r_k: the K columns of W's right-hand side
  c.s_kh = sc + 576;      // e^{Gam_last-Gam} r_k: the K columns of the state update
}

// Shared-memory pointers of the fused kernel's layout.
__device__ __forceinline__ void ctx_fused_layout(Ctx& c, unsigned char* sm) {
  c.sKQ = sm + kOffKQ;
  c.sKt = sm + kOffKt;
  c.sVt = sm + kOffVt;
  c.sTi = sm + kOffTi;
  c.sM = sm + kOffM;
  c.sW = sm + kOffW;
  c.sX = reinterpret_cast<float*>(sm + kOffW);
  c.sA = reinterpret_cast<float*>(sm + kOffA);
  c.sY = reinterpret_cast<float*>(sm + kOffY);
  ctx_scalars(c, reinterpret_cast<float*>(sm + kOffSc));
  c.bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
}

// Thread geometry and per-head constants (pointers are set by a layout function).
__device__ __forceinline__ void ctx_init(Ctx& c, const ChunkParams& p, int h) {
  c.tid = threadIdx.x;
  c.warp = c.tid >> 5;
  c.lane = c.tid & 31;
  c.quarter = c.warp & 3;
  c.half = c.warp >> 2;
  c.row = c.quarter * 32 + c.lane;
  c.h = h;
  c.kh = h / (p.Hv / p.Hk);
  c.l2 = (p.flags & GDN_F_QK_L2NORM) != 0;
  c.A_h = expf(__ldg(p.A_log + h));
  c.dtb = __ldg(p.dt_bias + h);
  c.log_clip = logf(1e-6f);                  // log(clip(alpha, 1e-6, 1)), python/qwen35.py:400
  c.qscale = rsqrtf(static_cast<float>(kD));
  c.phase = 0;
  c.my = static_cast<uint32_t>(c.quarter * 32) << 16;
#ifdef GDN_CHUNK_TIMING
  c.tick = clock64();
#endif
}

// Allocate ncols columns of tensor memory and initialise the CTA's mbarriers.
__device__ __forceinline__ void tmem_setup(Ctx& c, uint32_t* tslot, uint64_t* bars, int n_bars, uint32_t ncols) {
  if (c.warp == 0) {
    tc::tmem_alloc(tslot, ncols);
    tc::tmem_relinquish();
  }
  if (c.tid == 0) {
    for (int i = 0; i < n_bars; ++i) ptx::mbar_init(bars + i, 1);
    ptx::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  c.tb = *tslot;
}

// One warp polls the MMA barrier, the others wait at the CTA barrier; false if
// the bounded wait gave up or warp 0 passes ok_in = false (then every thread
// sees false).
__device__ __forceinline__ bool mma_wait(Ctx& c, bool ok_in = true) {
  bool ok = true;
  if (c.warp == 0) ok = ptx::mbar_wait(c.bar, c.phase) && ok_in;
  c.phase ^= 1u;
  const bool all_ok = !__syncthreads_or(!ok);
  tc::fence_after_sync();
  return all_ok;
}

// ---- prep phases (state-independent) -----------------------------------------

// Gates and the in-chunk decay prefix.  s_g, s_ratio, s_misc[0] are written by
// threads 0-63 without a trailing barrier (the next phase ends with one).
// The same from gate inputs already loaded: thread i < 64 holds token i's a
// and b (valid: i < nvalid).
__device__ __forceinline__ void phase_gates_from(Ctx& c, float a_in, float b_in, bool valid) {
  if (c.tid < kC) {
    float lg = 0.f, beta = 0.f;
    if (valid) {
      lg = fmaxf(-(c.A_h * softplus_f(a_in + c.dtb)), c.log_clip);
      beta = 1.f / (1.f + expf(-b_in));
    }
    float x = lg;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, off);
      if (c.lane >= off) x += y;
    }
    c.s_pre[c.tid] = x;
    c.s_beta[c.tid] = beta;
  }
  __syncthreads();
  if (c.tid < kC) c.s_gam[c.tid] = c.s_pre[c.tid] + (c.tid >= 32 ? c.s_pre[31] : 0.f);
  __syncthreads();
  if (c.tid < kC) {
    const float gl = c.s_gam[kC - 1];
    c.s_g[c.tid] = expf(c.s_gam[c.tid]);
    c.s_ratio[c.tid] = expf(gl - c.s_gam[c.tid]);
    if (c.tid == 0) c.s_misc[0] = expf(gl);
  }
}

__device__ __forceinline__ void phase_gates(const ChunkParams& p, Ctx& c, long long t0, int nvalid) {
  float a_in = 0.f, b_in = 0.f;
  const bool valid = c.tid < kC && c.tid < nvalid;
  if (valid) {
    const size_t gi = static_cast<size_t>(t0 + c.tid) * p.Hv + c.h;
    a_in = __ldg(p.a + gi);
    b_in = __ldg(p.b + gi);
  }
  phase_gates_from(c, a_in, b_in, valid);
}

// Rows of K and Q (thread -> token i, 32-dim quarter) into [K; Q], and their norms.
__device__ __forceinline__ void phase_rows(const ChunkParams& p, Ctx& c, long long t0, long long s0, int nvalid) {
  const int i = c.tid >> 2;
  const int qd = c.tid & 3;
  const bool valid = i < nvalid;
  const long long tok = valid ? t0 + i : s0;
  float f[32];
  load32(p.k + tok * p.k_stride + c.kh * kD + qd * 32, valid, f);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 32; ++e) ss += f[e] * f[e];
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
#pragma unroll
  for (int e = 0; e < 32; e += 4)
    *reinterpret_cast<float4*>(at(c.sKQ, i, qd * 32 + e, kSbo128)) = make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
  if (qd == 0) c.s_rk[i] = c.l2 ? rsqrtf(ss + 1e-6f) : 1.f;
  load32(p.q + tok * p.q_stride + c.kh * kD + qd * 32, valid, f);
  ss = 0.f;
#pragma unroll
  for (int e = 0; e < 32; ++e) ss += f[e] * f[e];
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
#pragma unroll
  for (int e = 0; e < 32; e += 4)
    *reinterpret_cast<float4*>(at(c.sKQ, kC + i, qd * 32 + e, kSbo128)) =
        make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
  if (qd == 0) c.s_rq[i] = c.l2 ? rsqrtf(ss + 1e-6f) * c.qscale : 1.f;
  ptx::fence_proxy_async_smem();
  __syncthreads();
}

// Columns of K (or V) read from global two at a time (4-byte loads), scaled
// per token by scale[], stored as rows of the transposed operand (K-major, 64
// tokens wide) at dst, and when dst2 is set scaled by scale2[] into dst2 too.
// lt in [0,128): column pair lt & 63, token half lt >> 6.  The caller selects
// K or V at run time so that all warps share one copy of this code.
__device__ __forceinline__ void columns(const ChunkParams& p, const Ctx& c, long long t0, int nvalid, int lt,
                                        bool is_k, const float* scale, unsigned char* dst,
                                        const float* scale2 = nullptr, unsigned char* dst2 = nullptr) {
  const int pr = lt & 63;
  const int th = lt >> 6;
  const int cc = 2 * pr;
  const long long stride = is_k ? p.k_stride : p.v_stride;
  const __nv_bfloat16* src = (is_k ? p.k + c.kh * kD : p.v + c.h * kD) + cc + (t0 + th * 32) * stride;
  const int nv = nvalid - th * 32;
  __nv_bfloat162 raw[32];                   // all loads in flight before any use
#pragma unroll
  for (int j = 0; j < 32; ++j)
    raw[j] = j < nv ? *reinterpret_cast<const __nv_bfloat162*>(src + j * stride) : __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    float x0[4], x1[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int jj = th * 32 + j + e;
      const float s = scale[jj];
      const float2 f = __bfloat1622float2(raw[j + e]);
      x0[e] = tc::to_tf32(f.x * s);
      x1[e] = tc::to_tf32(f.y * s);
    }
    *reinterpret_cast<float4*>(at(dst, cc, th * 32 + j, kSbo64)) = make_float4(x0[0], x0[1], x0[2], x0[3]);
    *reinterpret_cast<float4*>(at(dst, cc + 1, th * 32 + j, kSbo64)) = make_float4(x1[0], x1[1], x1[2], x1[3]);
    if (dst2) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float s = scale2[th * 32 + j + e];
        const float2 f = __bfloat1622float2(raw[j + e]);
        x0[e] = tc::to_tf32(f.x * s);
        x1[e] = tc::to_tf32(f.y * s);
      }
      *reinterpret_cast<float4*>(at(dst2, cc, th * 32 + j, kSbo64)) = make_float4(x0[0], x0[1], x0[2], x0[3]);
      *reinterpret_cast<float4*>(at(dst2, cc + 1, th * 32 + j, kSbo64)) = make_float4(x1[0], x1[1], x1[2], x1[3]);
    }
  }
}

// K^T diag(beta g r_k) (threads 0-127) and V^T diag(beta) (threads 128-255);
// with kh_dst set, K^T diag(e^{Gam_last-Gam} r_k) into kh_dst as well.
__device__ __forceinline__ void phase_cols(const ChunkParams& p, Ctx& c, long long t0, int nvalid,
                                           unsigned char* kh_dst = nullptr) {
  if (c.tid < kC) {
    c.s_kw[c.tid] = c.s_beta[c.tid] * c.s_g[c.tid] * c.s_rk[c.tid];
    c.s_kh[c.tid] = c.s_ratio[c.tid] * c.s_rk[c.tid];
  }
  __syncthreads();
  const bool is_k = c.tid < 128;
  columns(p, c, t0, nvalid, c.tid & 127, is_k, is_k ? c.s_kw : c.s_beta, is_k ? c.sKt : c.sVt, c.s_kh,
          is_k ? kh_dst : nullptr);
  ptx::fence_proxy_async_smem();
}

// (a) [K; Q] K^T -> G (lanes 0-63), P (lanes 64-127) at TMEM column col.
__device__ __forceinline__ bool phase_mma_a(Ctx& c, uint32_t col) {
  if (c.tid == 0) {
    tc::fence_after_sync();
    const uint32_t id = tc::instr_desc(tc::kTF32, 128, kC);
    for (int j = 0; j < kD / 8; ++j)
      tc::mma_ss<tc::kTF32>(c.tb + col, desc(c.sKQ, j * 256, kSbo128), desc(c.sKQ, j * 256, kSbo128), id, j > 0);
    tc::mma_commit(c.bar);
  }
  return mma_wait(c);
}

// A (strictly lower, plain) for the solve; M (lower) in the operand layout at
// m_dst; the Q rows of [K; Q] scaled by g r_q in the operand layout at q_dst
// (the fused kernel rescales them in place).  Destinations are shared memory
// or a workspace record.
__device__ __forceinline__ void phase_epi_a(Ctx& c, uint32_t col, unsigned char* m_dst, unsigned char* q_dst) {
  float gp[32];
  tmem_ld<32>(c.tb + col + c.my + c.half * 32, gp);
  if (c.quarter < 2) {
    const int i = c.row;
    const float fi = c.s_beta[i] * c.s_rk[i];
    const float gi = c.s_gam[i];
    float* Ac = c.sA + (c.half * 32) * kPadA + i;     // A^T: column i of row j at j * kPadA + i
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int j = c.half * 32 + e;
      Ac[e * kPadA] = (j < i) ? fi * c.s_rk[j] * __expf(gi - c.s_gam[j]) * gp[e] : 0.f;
    }
  } else {
    const int i = c.row - kC;
    const float fi = c.s_rq[i];
    const float gi = c.s_gam[i];
#pragma unroll
    for (int e = 0; e < 32; e += 4) {
      float m[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = c.half * 32 + e + u;
        m[u] = (j <= i) ? tc::to_tf32(fi * c.s_rk[j] * __expf(gi - c.s_gam[j]) * gp[e + u]) : 0.f;
      }
      *reinterpret_cast<float4*>(at(m_dst, i, c.half * 32 + e, kSbo64)) = make_float4(m[0], m[1], m[2], m[3]);
    }
    if (q_dst) {
      const float sq = c.s_g[i] * c.s_rq[i];
      for (int cc = c.half * 64; cc < c.half * 64 + 64; cc += 4) {
        float4 v = *reinterpret_cast<const float4*>(at(c.sKQ, kC + i, cc, kSbo128));
        v.x = tc::to_tf32(v.x * sq);
        v.y = tc::to_tf32(v.y * sq);
        v.z = tc::to_tf32(v.z * sq);
        v.w = tc::to_tf32(v.w * sq);
        *reinterpret_cast<float4*>(at(q_dst, i, cc, kSbo128)) = v;
      }
    }
  }
  __syncthreads();
}

// T^-1 = (I + A)^-1 by forward substitution on all 64 columns at once:
// warps 2s, 2s+1 hold rows 16s .. 16s+15 of the 64 columns (one column per
// thread, in registers).  Row segments are solved in order -- an in-block
// substitution, then the rows go to X -- and as soon as segment s is in X
// every later segment subtracts its contribution, so the critical path is
// four 16-step substitutions and three 16 x 16 updates.  fp32 throughout;
// X is exactly lower triangular with a unit diagonal.
__device__ __forceinline__ void phase_solve(Ctx& c) {
  const float* sA = c.sA;
  float* sX = c.sX;
  const int seg = c.warp >> 1;
  const int j = ((c.warp & 1) << 5) + c.lane;
  float b[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) b[r] = (seg * 16 + r == j) ? 1.f : 0.f;
  for (int step = 0; step < 4; ++step) {
    if (seg == step) {
      // A[16 seg + i][16 seg + r] = A^T[16 seg + r][16 seg + i], read 4 rows i at a time
      const float* At = sA + (seg * 16) * kPadA + seg * 16;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float a[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 f = *reinterpret_cast<const float4*>(At + r * kPadA + 4 * q);
          a[4 * q] = f.x; a[4 * q + 1] = f.y; a[4 * q + 2] = f.z; a[4 * q + 3] = f.w;
        }
#pragma unroll
        for (int i = r + 1; i < 16; ++i) b[i] -= a[i] * b[r];
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) sX[(seg * 16 + r) * kPad + j] = b[r];
    }
    __syncthreads();
    if (seg > step) {
      // b_r -= sum_m A[16 seg + r][16 step + m] X[16 step + m][j], A^T rows m read 4 r at a time
      const float* At = sA + (step * 16) * kPadA + seg * 16;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float x = sX[(step * 16 + m) * kPad + j];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 f = *reinterpret_cast<const float4*>(At + m * kPadA + 4 * q);
          b[4 * q] -= f.x * x;
          b[4 * q + 1] -= f.y * x;
          b[4 * q + 2] -= f.z * x;
          b[4 * q + 3] -= f.w * x;
        }
      }
    }
  }
  {
    const int i = c.tid >> 2;
    const int c0 = (c.tid & 3) * 16;
#pragma unroll
    for (int cc = c0; cc < c0 + 16; cc += 4) {
      float x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) x[u] = ((cc + u) >> 4) <= (i >> 4) ? tc::to_tf32(sX[i * kPad + cc + u]) : 0.f;
      *reinterpret_cast<float4*>(at(c.sTi, i, cc, kSbo64)) = make_float4(x[0], x[1], x[2], x[3]);
    }
  }
  ptx::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
}

// (b) U0^T = V^T diag(beta) T^-T;  (c) W = [T^-1; *] (K^T diag(beta g r_k))^T
// (M = 128: rows 64-127 of A read the next 16 KiB of shared memory and are
// discarded).
__device__ __forceinline__ bool phase_mma_bc(Ctx& c) {
  if (c.tid == 0) {
    tc::fence_after_sync();
    const uint32_t id64 = tc::instr_desc(tc::kTF32, 128, kC);
    const uint32_t id128 = tc::instr_desc(tc::kTF32, 128, kD);
    for (int j = 0; j < kC / 8; ++j)
      tc::mma_ss<tc::kTF32>(c.tb + kColU, desc(c.sVt, j * 256, kSbo64), desc(c.sTi, j * 256, kSbo64), id64, j > 0);
    for (int j = 0; j < kC / 8; ++j)
      tc::mma_ss<tc::kTF32>(c.tb + kColW, desc(c.sTi, j * 256, kSbo64), desc(c.sKt, j * 256, kSbo64), id128, j > 0);
    tc::mma_commit(c.bar);
  }
  return mma_wait(c);
}

// W rows (warps on lanes 0-63) into w_dst; K^T diag(ratio r_k) (warps on lanes
// 64-127) into kh_dst; both in the operand layouts, in shared memory or a
// workspace record.
__device__ __forceinline__ void phase_epi_c(const ChunkParams& p, Ctx& c, long long t0, int nvalid,
                                            unsigned char* w_dst, unsigned char* kh_dst) {
  if (c.quarter < 2) {
    float w[64];
    tmem_ld<64>(c.tb + kColW + c.my + c.half * 64, w);
    const int i = c.row;
#pragma unroll
    for (int e = 0; e < 64; e += 4)
      *reinterpret_cast<float4*>(at(w_dst, i, c.half * 64 + e, kSbo128)) =
          make_float4(tc::to_tf32(w[e]), tc::to_tf32(w[e + 1]), tc::to_tf32(w[e + 2]), tc::to_tf32(w[e + 3]));
  } else {
    const int lt = (c.tid & 63) + 64 * c.half;     // 0..127 over the four warps on lanes 64-127
    columns(p, c, t0, nvalid, lt, true, c.s_kh, kh_dst);
  }
  ptx::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
}

// ---- state phases --------------------------------------------------------------

// tR = tf32(R), tDR = g_last * R (the state update accumulates onto it).
__device__ __forceinline__ void phase_r_update(Ctx& c, float gl, uint32_t col_r, uint32_t col_dr) {
  for (int cc = 0; cc < 64; cc += 16) {
    float v[16], r[16];
    tc::tmem_ld16(c.tb + col_dr + c.my + c.half * 64 + cc, v);
    tc::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      r[i] = tc::to_tf32(v[i]);
      v[i] *= gl;
    }
    tc::tmem_st16(c.tb + col_r + c.my + c.half * 64 + cc, r);
    tc::tmem_st16(c.tb + col_dr + c.my + c.half * 64 + cc, v);
  }
  tc::tmem_st_wait();
}

// U^T (TMEM) -> rows of the U^T operand in shared memory.
__device__ __forceinline__ void phase_epi_d(Ctx& c, uint32_t col_u, unsigned char* ut) {
  float u[32];
  tmem_ld<32>(c.tb + col_u + c.my + c.half * 32, u);
#pragma unroll
  for (int e = 0; e < 32; e += 4)
    *reinterpret_cast<float4*>(at(ut, c.row, c.half * 32 + e, kSbo64)) =
        make_float4(tc::to_tf32(u[e]), tc::to_tf32(u[e + 1]), tc::to_tf32(u[e + 2]), tc::to_tf32(u[e + 3]));
  ptx::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
}

// y^T (TMEM) -> o rows of the chunk: thread -> (dv = row, tokens of its half).
// No barrier at the end: the caller orders it with what follows.
__device__ __forceinline__ void phase_epi_e(const ChunkParams& p, Ctx& c, uint32_t col_y, long long t0, int nvalid) {
  float y[32];
  tmem_ld<32>(c.tb + col_y + c.my + c.half * 32, y);
  const size_t orow = static_cast<size_t>(p.Hv) * kD;
  const size_t base = (static_cast<size_t>(t0 + c.half * 32) * p.Hv + c.h) * kD + c.row;
  const int nv = nvalid - c.half * 32;
  if (p.flags & GDN_F_O_BF16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.o) + base;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < nv) o[i * orow] = __float2bfloat16_rn(y[i]);
  } else {
    float* o = static_cast<float*>(p.o) + base;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < nv) o[i * orow] = y[i];
  }
}

// Initial state row dv = row, columns [col0, col0 + ncols), into the fp32 master.
__device__ __forceinline__ void state_load(const float* state, Ctx& c, int bh, uint32_t col_dr, int col0, int ncols) {
  const float* src = state ? state + (static_cast<size_t>(bh) * kD + c.row) * kD + col0 : nullptr;
  for (int cc = 0; cc < ncols; cc += 16) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 f = src ? *reinterpret_cast<const float4*>(src + cc + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
    }
    tc::tmem_st16(c.tb + col_dr + c.my + col0 + cc, v);
  }
  tc::tmem_st_wait();
}

__device__ __forceinline__ void state_store(float* state, Ctx& c, int bh, uint32_t col_dr, int col0, int ncols) {
  if (!state) return;
  float* dst = state + (static_cast<size_t>(bh) * kD + c.row) * kD + col0;
  for (int cc = 0; cc < ncols; cc += 16) {
    float v[16];
    tc::tmem_ld16(c.tb + col_dr + c.my + col0 + cc, v);
    tc::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; i += 4)
      *reinterpret_cast<float4*>(dst + cc + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  }
}

// ---- the fused schedule -----------------------------------------------------------

__global__ void __launch_bounds__(kThreads, 1) chunked_kernel(const ChunkParams p) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const int bh = blockIdx.x;
  const int b = bh / p.Hv;
  Ctx c;
  ctx_init(c, p, bh - b * p.Hv);
  ctx_fused_layout(c, sm);
  long long s0, s1;
  seq_range(p, b, s0, s1);
  const int n_chunks = static_cast<int>((s1 - s0 + kC - 1) / kC);
  tmem_setup(c, reinterpret_cast<uint32_t*>(sm + kOffBar + 8), c.bar, 1, kTmemCols);
  state_load(p.state_in, c, bh, kColDR, c.half * 64, 64);

  bool failed = false;
  for (int ch = 0; ch < n_chunks; ++ch) {
    const long long t0 = s0 + static_cast<long long>(ch) * kC;
    const int nvalid = static_cast<int>((s1 - t0) < kC ? (s1 - t0) : kC);
    phase_gates(p, c, t0, nvalid);
    GDN_TICK(0);
    phase_rows(p, c, t0, s0, nvalid);
    GDN_TICK(1);
    phase_cols(p, c, t0, nvalid);
    GDN_TICK(2);
    phase_r_update(c, c.s_misc[0], kColR, kColDR);
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(3);
    if (!phase_mma_a(c, kColGP)) { failed = true; break; }
    GDN_TICK(4);
    phase_epi_a(c, kColGP, c.sM, c.sKQ + 8 * kSbo128);
    GDN_TICK(5);
    phase_solve(c);
    GDN_TICK(6);
    if (!phase_mma_bc(c)) { failed = true; break; }
    GDN_TICK(7);
    phase_epi_c(p, c, t0, nvalid, c.sW, c.sKt);
    GDN_TICK(8);
    // (d) U^T = U0^T - R W^T
    if (c.tid == 0) {
      tc::fence_after_sync();
      const uint32_t id = tc::instr_desc(tc::kTF32, 128, kC, /*neg_a=*/true);
      for (int j = 0; j < kD / 8; ++j)
        tc::mma_ts_tf32(c.tb + kColU, c.tb + kColR + j * 8, desc(c.sW, j * 256, kSbo128), id, 1);
      tc::mma_commit(c.bar);
    }
    if (!mma_wait(c)) { failed = true; break; }
    GDN_TICK(9);
    phase_epi_d(c, kColU, c.sVt);
    GDN_TICK(10);
    // (e) y^T = R Qs^T + U^T M^T,  (f) R += U^T diag(ratio r_k) K
    if (c.tid == 0) {
      tc::fence_after_sync();
      const uint32_t id64 = tc::instr_desc(tc::kTF32, 128, kC);
      const uint32_t id128 = tc::instr_desc(tc::kTF32, 128, kD);
      for (int j = 0; j < kD / 8; ++j)
        tc::mma_ts_tf32(c.tb + kColY, c.tb + kColR + j * 8, desc(c.sKQ, 8 * kSbo128 + j * 256, kSbo128), id64, j > 0);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(c.tb + kColY, desc(c.sVt, j * 256, kSbo64), desc(c.sM, j * 256, kSbo64), id64, 1);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(c.tb + kColDR, desc(c.sVt, j * 256, kSbo64), desc(c.sKt, j * 256, kSbo64), id128, 1);
      tc::mma_commit(c.bar);
    }
    if (!mma_wait(c)) { failed = true; break; }
    GDN_TICK(11);
    phase_epi_e(p, c, kColY, t0, nvalid);
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(12);
  }
  if (failed) {
    if (c.tid == 0) atomicExch(p.err, 1);
    ptx::mbar_wait(c.bar, c.phase ^ 1u);   // the phase mma_wait gave up on: one more bounded wait
  } else {
    state_store(p.state_out, c, bh, kColDR, c.half * 64, 64);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (c.warp == 0) tc::tmem_dealloc(c.tb, kTmemCols);
}

// ---- the split schedule: prep (parallel over chunks) -------------------------------

// Record of (slot, value head) in the workspace (256-byte aligned).
__device__ __forceinline__ unsigned char* record(const ChunkParams& p, long long slot, int h) {
  return p.ws + p.rec_off + (static_cast<size_t>(slot) * p.Hv + h) * kRecBytes;
}

// Sequence and (absolute) chunk of a record slot of the current window;
// false for an unused slot.
__device__ __forceinline__ bool slot_to_chunk(const ChunkParams& p, long long slot, int& b, int& ch) {
  if (!p.cu) {
    b = static_cast<int>(slot / p.nch_uniform);
    ch = p.win_c0 + static_cast<int>(slot - static_cast<long long>(b) * p.nch_uniform);
    return b < p.B;
  }
  if (slot >= p.chunk_prefix[p.B]) return false;
  int lo = 0, hi = p.B - 1;                 // last sequence whose first slot is <= slot
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.chunk_prefix[mid] <= slot) lo = mid;
    else hi = mid - 1;
  }
  b = lo;
  ch = p.win_c0 + static_cast<int>(slot - p.chunk_prefix[lo]);
  return true;
}

// First record slot of sequence b.
__device__ __forceinline__ long long seq_first_slot(const ChunkParams& p, int b) {
  return p.cu ? static_cast<long long>(p.chunk_prefix[b]) : static_cast<long long>(b) * p.nch_uniform;
}

// prefix[b] = number of 64-token chunks of packed sequences 0 .. b-1 that fall
// in the window [c0, c0 + wlen) (one block).
__global__ void __launch_bounds__(1024) chunk_prefix_kernel(const int32_t* cu, int B, int c0, int wlen,
                                                            int32_t* prefix) {
  __shared__ int32_t carry;
  __shared__ int32_t buf[1024];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < B; base += 1024) {
    const int b = base + threadIdx.x;
    int32_t n = 0;
    if (b < B) {
      const int32_t len = cu[b + 1] - cu[b];
      n = len > 0 ? (len + kC - 1) / kC - c0 : 0;
      n = n < 0 ? 0 : (n > wlen ? wlen : n);
    }
    buf[threadIdx.x] = n;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {       // inclusive scan
      const int32_t add = threadIdx.x >= off ? buf[threadIdx.x - off] : 0;
      __syncthreads();
      buf[threadIdx.x] += add;
      __syncthreads();
    }
    if (b < B) prefix[b] = carry + buf[threadIdx.x] - n;
    __syncthreads();
    if (threadIdx.x == 1023) carry += buf[1023];
    __syncthreads();
  }
  if (threadIdx.x == 0) prefix[B] = carry;
}

// (x0, x1) as bf16 pairs hi = bf16(x), lo = bf16(x - hi): hi + lo equals x to
// about 2^-16 relative, so two kind::f16 products (hi, then lo) carry an fp32
// operand more precisely than one tf32 product.
__device__ __forceinline__ void split_bf16(float2 x, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x.x, x.y);
  const float2 hf = __bfloat1622float2(h);
  const float2 r = __ffma2_rn(hf, make_float2(-1.f, -1.f), x);   // x - hi, exact
  const __nv_bfloat162 l = __floats2bfloat162_rn(r.x, r.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// 4 x 4 transpose across the lanes u = lane % 4 of each lane quad: lane u
// holds M[u][0..3] on entry and M[0..3][u] on return.
__device__ __forceinline__ void quad_transpose(float& v0, float& v1, float& v2, float& v3, int u) {
  const bool o1 = u & 1, o2 = u & 2;
  float s0 = __shfl_xor_sync(0xffffffffu, o1 ? v0 : v1, 1);
  float s1 = __shfl_xor_sync(0xffffffffu, o1 ? v2 : v3, 1);
  if (o1) { v0 = s0; v2 = s1; } else { v1 = s0; v3 = s1; }
  s0 = __shfl_xor_sync(0xffffffffu, o2 ? v0 : v2, 2);
  s1 = __shfl_xor_sync(0xffffffffu, o2 ? v1 : v3, 2);
  if (o2) { v0 = s0; v1 = s1; } else { v2 = s0; v3 = s1; }
}

// The rest of X = (I + A)^-1 for the unit lower-triangular 64 x 64 chunk
// matrix, once its inverted 16 x 16 diagonal blocks D_b are in X: by doubling
// over the 32 x 32 halves,
//   X[2p+1][2p] = -D[2p+1] (A[2p+1][2p] D[2p])         (p = 0, 1 at once)
//   X21         = -X22 (A21 X11)                       (32 x 32 products)
// -- the same inverse as block forward substitution, in four rounds of
// products in which every thread takes part (2 outputs per thread in the
// 16 x 16 rounds, a 2 x 2 tile in the 32 x 32 ones).  Entries above the
// diagonal of X are not stored: the products mask them.  sY holds 1024
// floats.  Ends with a barrier.
__device__ __forceinline__ void solve_doubling(const float* sA, float* sX, float* sY, int tid) {
  {
    // Y_p = A[2p+1][2p] D[2p]: block p = tid / 128, row i, columns c, c + 1
    const int p = tid >> 7, i = (tid >> 3) & 15, cc = (tid & 7) * 2;
    const float* arow = sA + (32 * p + 16 + i) * kPadA + 32 * p;
    const float* dcol = sX + (32 * p) * kPadA + 32 * p + cc;
    float2 y = make_float2(0.f, 0.f);     // packed f32x2: the two columns' fused multiply-adds
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float a = arow[k];
      y = __ffma2_rn(make_float2(a, a), *reinterpret_cast<const float2*>(dcol + k * kPadA), y);
    }
    *reinterpret_cast<float2*>(sY + p * 256 + i * 16 + cc) = y;
  }
  __syncthreads();
  {
    // X[2p+1][2p] = -D[2p+1] Y_p
    const int p = tid >> 7, i = (tid >> 3) & 15, cc = (tid & 7) * 2;
    const float* drow = sX + (32 * p + 16 + i) * kPadA + 32 * p + 16;
    float2 x = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float d = drow[k];
      x = __ffma2_rn(make_float2(-d, -d), *reinterpret_cast<const float2*>(sY + p * 256 + k * 16 + cc), x);
    }
    *reinterpret_cast<float2*>(sX + (32 * p + 16 + i) * kPadA + 32 * p + cc) = x;
  }
  __syncthreads();
  const int r2 = (tid >> 4) * 2, c2 = (tid & 15) * 2;   // a 2 x 2 tile of a 32 x 32 product
  {
    // Z = A21 X11 (A21 = A[32..63][0..31]; X11[k][j] = 0 for k < j)
    // unrolled over all 32 k with the zeros selected (the unstored entries
    // may hold anything), two partial sums per output
    const float* a0 = sA + (32 + r2) * kPadA;
    const float* a1 = a0 + kPadA;
    float2 z[2][2] = {};                  // [k parity][row], the two columns packed
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float2 x = *reinterpret_cast<const float2*>(sX + k * kPadA + c2);
      const float2 xab = make_float2(k >= c2 ? x.x : 0.f, k > c2 ? x.y : 0.f);
      const float u0 = a0[k], u1 = a1[k];
      z[k & 1][0] = __ffma2_rn(make_float2(u0, u0), xab, z[k & 1][0]);
      z[k & 1][1] = __ffma2_rn(make_float2(u1, u1), xab, z[k & 1][1]);
    }
    *reinterpret_cast<float2*>(sY + r2 * 32 + c2) = __fadd2_rn(z[0][0], z[1][0]);
    *reinterpret_cast<float2*>(sY + (r2 + 1) * 32 + c2) = __fadd2_rn(z[0][1], z[1][1]);
  }
  __syncthreads();
  {
    // X21 = -X22 Z (X22 = X[32..63][32..63]; X22[i][k] = 0 for k > i)
    const float* x0 = sX + (32 + r2) * kPadA + 32;
    const float* x1 = x0 + kPadA;
    float2 v[2][2] = {};
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const float2 z = *reinterpret_cast<const float2*>(sY + k * 32 + c2);
      const float u0 = k <= r2 ? x0[k] : 0.f, u1 = k <= r2 + 1 ? x1[k] : 0.f;
      v[k & 1][0] = __ffma2_rn(make_float2(u0, u0), z, v[k & 1][0]);
      v[k & 1][1] = __ffma2_rn(make_float2(u1, u1), z, v[k & 1][1]);
    }
    const float2 s0 = __fadd2_rn(v[0][0], v[1][0]), s1 = __fadd2_rn(v[0][1], v[1][1]);
    *reinterpret_cast<float2*>(sX + (32 + r2) * kPadA + c2) = make_float2(-s0.x, -s0.y);
    *reinterpret_cast<float2*>(sX + (33 + r2) * kPadA + c2) = make_float2(-s1.x, -s1.y);
  }
  __syncthreads();
}

// Rows [nvalid, 64) of a 64 x 128 bf16 row tile in the prep layout set to
// zero (a sequence's last chunk: the tensor copy brought the next sequence's
// rows, or zeros past the tensor's end).
__device__ __forceinline__ void prep_zero_rows(unsigned char* dst, int nvalid, int tid) {
  for (int q = tid; q < (kC - nvalid) * 16; q += kThreads)
    *reinterpret_cast<uint4*>(dst + tc::kmajor_offset(nvalid + (q >> 4), (q & 15) * 8, 2, kSboKQ)) =
        make_uint4(0, 0, 0, 0);
}

// The rows of 64 tokens t0 .. t0 + 63 of one head (channel group cg0 = 16 x
// head) by eight tensor copies, one 8-row group of the prep layout each
// (thread 0 issues; completion counted on bar).
__device__ __forceinline__ void prep_rows_tma(unsigned char* dst, const CUtensorMap* tm, long long t0, int cg0,
                                              uint64_t* bar) {
#pragma unroll
  for (int g = 0; g < kC / 8; ++g)
    ptx::tma_load_3d(dst + g * kSboKQ, tm, 0, static_cast<int>(t0) + 8 * g, cg0, bar);
}

// One right-hand product of the prep into TMEM column col (thread 0 issues):
// D^T = A^T B^T with A the 64 x 128 bf16 rows at shared address a_rows read
// MN-major (LBO = one 8-token group of 128 rows, SBO 128) and B the bf16
// hi | lo operand pair at b (K-major, 64 x 64 each), one MMA per 16 tokens.
__device__ __forceinline__ void prep_rhs_mma(const Ctx& c, uint32_t a_rows, const unsigned char* b, uint32_t col) {
  const uint32_t id = tc::instr_desc(tc::kBF16, 128, kC, false, false, /*a_mn=*/true, false);
  for (int part = 0; part < 2; ++part) {
    const uint32_t boff = part * kC * kC * 2;
    for (int j = 0; j < kC / 16; ++j) {
      const uint64_t a = tc::smem_desc(a_rows + j * 2 * kSboKQ, kSboKQ, 128);
      tc::mma_ss<tc::kBF16>(c.tb + col, a, desc(b, boff + j * 256, kSboOp), id, part + j > 0);
    }
  }
}

// U0^T (lane = value row, this warp's 32 token columns in u) to the record, by
// column quads.
__device__ __forceinline__ void prep_store_u0(const Ctx& c, unsigned char* rec, const float (&u)[32]) {
  float4* ud = reinterpret_cast<float4*>(rec + kRecU);
#pragma unroll
  for (int e = 0; e < 32; e += 4)
    ud[u0_index(c.half * 8 + e / 4, c.row)] = make_float4(u[e], u[e + 1], u[e + 2], u[e + 3]);
}

// -W to the record from W^T (lane k holds W^T[k][j] for its 32 j in w): 4 x 4
// transposes across lane quads give each lane 4 consecutive k of one j, one
// 8-byte fp16 store; thread 0 adds e^{Gam_last}.
__device__ __forceinline__ void prep_store_negw(const Ctx& c, unsigned char* rec, const float (&w)[32]) {
  const int u4 = c.lane & 3;
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    float v0 = w[e], v1 = w[e + 1], v2 = w[e + 2], v3 = w[e + 3];
    quad_transpose(v0, v1, v2, v3, u4);
    *reinterpret_cast<uint2*>(at_h(rec + kRecW, c.half * 32 + e + u4, c.row - u4, kSboH128)) =
        pack_h4(-v0, -v1, -v2, -v3);
  }
  if (c.tid == 0) reinterpret_cast<float*>(rec + kRecSc)[0] = c.s_misc[0];
}

// Gates of the group's value heads h0 .. h0 + gsz - 1: thread t < 64 gsz holds
// the gate inputs of head t / 64 at token t % 64 (valid: a token of the chunk)
// and leaves the head's in-chunk log-decay prefix Gam in gam[t] and beta in
// beta[t].  Ends after the first barrier: the caller's next barrier publishes
// gam for tokens 32-63.
__device__ __forceinline__ void phase_gates_group(const Ctx& c, float* gam, float* beta_out, int gsz, float A_h,
                                                  float dtb, float a_in, float b_in, bool valid) {
  const bool mine = c.tid < kC * gsz;           // whole warps: kC is a multiple of 32
  if (mine) {
    float lg = 0.f, beta = 0.f;
    if (valid) {
      lg = fmaxf(-(A_h * softplus_f(a_in + dtb)), c.log_clip);
      beta = 1.f / (1.f + expf(-b_in));
    }
    float x = lg;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, off);
      if (c.lane >= off) x += y;
    }
    gam[c.tid] = x;
    beta_out[c.tid] = beta;
  }
  __syncthreads();
  if (mine && (c.tid & (kC - 1)) >= 32) gam[c.tid] += gam[(c.tid & ~(kC - 1)) + 31];
}

// Per-token scalars of the group's head hh that the later phases read through
// the context (threads 0-63; rk = r_k of the token): g, e^{Gam_last-Gam}, the
// K columns of W's right-hand side (beta g r_k) and of K-hat (e^{Gam_last-Gam}
// r_k), and e^{Gam_last}.
__device__ __forceinline__ void head_scalars(Ctx& c, const float* gam, const float* beta, int t, float rk) {
  const float gl = gam[kC - 1];
  const float g = expf(gam[t]);
  const float ratio = expf(gl - gam[t]);
  c.s_g[t] = g;
  c.s_ratio[t] = ratio;
  c.s_kw[t] = beta[t] * g * rk;
  c.s_kh[t] = ratio * rk;
  if (t == 0) c.s_misc[0] = expf(gl);
}

// One CTA per (chunk, group of value heads sharing a key head), group fastest
// in the grid.  Phases:
//   rows of K, Q (tensor copies) | gates of the group's heads -> norms, Q-tilde of
//   every head to its record -> G | P = [K; Q] K^T (kind::bf16, exact
//   operands; tensor-memory columns [0, 64), kept for all heads) -> per head:
//   A (shared memory) and M to the record from G | P; V rows (tensor copies) ->
//   T^-1 = (I + A)^-1 blocked: the 16 x 16 diagonal blocks by substitution
//   while the other warps write K-hat^T to the record, then the off-diagonal
//   blocks by doubling (solve_doubling) -> the U0 / W right-hand operands
//   diag(beta) T^-T and diag(beta g r_k) T^-T as bf16 hi + lo pairs (x = hi +
//   lo to 2^-16 relative) -> U0^T = V^T B_U, W^T = K^T B_W (kind::bf16, V^T
//   and K^T MN-major straight from the rows) -> the record.  The last head
//   puts W^T over G | P and runs both products at once; the others run them
//   one after the other in columns [64, 128), the next head's V rows loading
//   as soon as U0^T is done.
__global__ void __launch_bounds__(kThreads, 3)
    chunk_prep_kernel(const ChunkParams p, const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const int gsz = p.prep_group;
  const int ngroups = p.Hv / gsz;
  const long long unit = blockIdx.x;
  const long long slot = unit / ngroups;
  const int h0 = static_cast<int>(unit - slot * ngroups) * gsz;
  Ctx c;
  ctx_init(c, p, h0);   // key head and per-CTA constants in flight during the lookup
  // gate constants of this thread's head (thread t < 64 gsz: head t / 64)
  const int ghh = c.tid / kC;
  const bool gin = ghh < gsz;
  float A_h = 0.f, dtb = 0.f;
  if (gin) {
    A_h = expf(__ldg(p.A_log + h0 + ghh));
    dtb = __ldg(p.dt_bias + h0 + ghh);
  }
  // (sequence, chunk) of this slot and the sequence's token range: for a
  // packed batch thread t < B tests sequence t (one round of loads, exactly
  // one writer), thread B marks a slot past the last chunk
  int* s_bc = reinterpret_cast<int*>(sm + kQBar + 16);
  long long* s_rng = reinterpret_cast<long long*>(sm + kQBar + 32);
  if (!p.cu) {
    if (c.tid == 0) {
      int b = 0, ch = 0;
      const bool used = slot_to_chunk(p, slot, b, ch);
      s_bc[0] = used ? b : -1;
      s_bc[1] = ch;
      seq_range(p, b, s_rng[0], s_rng[1]);
    }
  } else {
    for (int t = c.tid; t <= p.B; t += kThreads) {
      const long long lo = p.chunk_prefix[t];
      if (t < p.B) {
        const long long hi = p.chunk_prefix[t + 1];
        const long long q0 = p.cu[t], q1 = p.cu[t + 1];
        if (lo <= slot && slot < hi) {
          s_bc[0] = t;
          s_bc[1] = p.win_c0 + static_cast<int>(slot - lo);
          s_rng[0] = q0;
          s_rng[1] = q1 < q0 ? q0 : q1;
        }
      } else if (slot >= lo) {
        s_bc[0] = -1;
      }
    }
  }
  __syncthreads();
  const int b = s_bc[0];
  if (b < 0) return;
  const int ch = s_bc[1];
  ctx_scalars(c, reinterpret_cast<float*>(sm + kQSc));
  c.bar = reinterpret_cast<uint64_t*>(sm + kQBar);
  float* gamA = reinterpret_cast<float*>(sm + kQGa);   // [gsz][64]
  float* betaA = gamA + kPrepGroup * kC;                // [gsz][64]
  unsigned char* sK = sm + kQK;
  unsigned char* sQ = sm + kQQ;   // then V
  float* sA = reinterpret_cast<float*>(sm + kQA);
  float* sX = reinterpret_cast<float*>(sm + kQX);
  float* sY = reinterpret_cast<float*>(sm + kQY);
  const long long s0 = s_rng[0], s1 = s_rng[1];
  const long long t0 = s0 + static_cast<long long>(ch) * kC;
  const int nvalid = static_cast<int>((s1 - t0) < kC ? (s1 - t0) : kC);
  // gate inputs first: their latency overlaps the row copies and the TMEM set-up
  float a_in = 0.f, b_in = 0.f;
  const bool gvalid = gin && (c.tid & (kC - 1)) < nvalid;
  if (gvalid) {
    const size_t gi = static_cast<size_t>(t0 + (c.tid & (kC - 1))) * p.Hv + h0 + ghh;
    a_in = __ldg(p.a + gi);
    b_in = __ldg(p.b + gi);
  }

  // K and Q rows by tensor copies on their own barrier (one arrival per
  // phase: K | Q, then each head's V rows); rows_wait is the CTA's bounded
  // wait for the current phase
  uint64_t* rbar = reinterpret_cast<uint64_t*>(sm + kQBar + 48);
  uint32_t rphase = 0;
  bool rows_pending = false;               // a phase issued and not yet waited for (same in every thread)
  auto rows_wait = [&]() -> bool {
    bool okw = true;
    if (c.warp == 0) okw = ptx::mbar_wait(rbar, rphase);
    const bool all = !__syncthreads_or(!okw);
    if (all) {                             // else the phase stays pending for the exit's last wait
      rphase ^= 1u;
      rows_pending = false;
    }
    return all;
  };
  if (c.tid == 0) {
    ptx::mbar_init(rbar, 1);
    ptx::fence_mbar_init();
    ptx::mbar_arrive_expect_tx(rbar, 2 * kC * kD * 2);
    prep_rows_tma(sK, &tmk, t0, c.kh * (kD / 8), rbar);
    prep_rows_tma(sQ, &tmq, t0, c.kh * (kD / 8), rbar);
  }
  rows_pending = true;
  tmem_setup(c, reinterpret_cast<uint32_t*>(sm + kQBar + 8), c.bar, 1, kPrepTmemCols);
  phase_gates_group(c, gamA, betaA, gsz, A_h, dtb, a_in, b_in, gvalid);
  if (!rows_wait()) {
    // the rows never arrived: record it, give the copies one more bounded wait, leave
    if (c.tid == 0) atomicExch(p.err, 1);
    if (c.warp == 0) ptx::mbar_wait(rbar, rphase);
    tc::fence_before_sync();
    __syncthreads();
    if (c.warp == 0) tc::tmem_dealloc(c.tb, kPrepTmemCols);
    return;
  }
  if (nvalid < kC) {                       // a sequence's last chunk: rows past its end are zero
    prep_zero_rows(sK, nvalid, c.tid);
    prep_zero_rows(sQ, nvalid, c.tid);
    ptx::fence_proxy_async_smem();
    __syncthreads();
  }
  GDN_TICK(16);

  // norms (thread: token i = 8 warp + lane % 8, 32-dim quarter qd = lane / 8,
  // so that the 8 lanes of each 16-byte shared-memory wavefront read 8
  // distinct rows), the first head's per-token scalars, Q-tilde of every head
  // to its record
  {
    const int i = c.warp * 8 + (c.lane & 7), qd = c.lane >> 3;
    uint4 kr[4], qr[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      kr[m] = *reinterpret_cast<const uint4*>(sK + tc::kmajor_offset(i, qd * 32 + m * 8, 2, kSboKQ));
      qr[m] = *reinterpret_cast<const uint4*>(sQ + tc::kmajor_offset(i, qd * 32 + m * 8, 2, kSboKQ));
    }
    float sk = 0.f, sq = 0.f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const __nv_bfloat162* hk = reinterpret_cast<const __nv_bfloat162*>(&kr[m]);
      const __nv_bfloat162* hq = reinterpret_cast<const __nv_bfloat162*>(&qr[m]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fk = __bfloat1622float2(hk[e]);
        const float2 fq = __bfloat1622float2(hq[e]);
        sk += fk.x * fk.x + fk.y * fk.y;
        sq += fq.x * fq.x + fq.y * fq.y;
      }
    }
    sk += __shfl_xor_sync(0xffffffffu, sk, 8);
    sk += __shfl_xor_sync(0xffffffffu, sk, 16);
    sq += __shfl_xor_sync(0xffffffffu, sq, 8);
    sq += __shfl_xor_sync(0xffffffffu, sq, 16);
    const float rk = c.l2 ? rsqrtf(sk + 1e-6f) : 1.f;
    const float rq = c.l2 ? rsqrtf(sq + 1e-6f) * c.qscale : 1.f;
    if (qd == 0) {
      c.s_rk[i] = rk;
      c.s_rq[i] = rq;
      head_scalars(c, gamA, betaA, i, rk);
    }
    for (int hh = 0; hh < gsz; ++hh) {
      unsigned char* rq_dst = record(p, slot, h0 + hh) + kRecQ;
      const float s = expf(gamA[hh * kC + i]) * rq;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const __nv_bfloat162* hq = reinterpret_cast<const __nv_bfloat162*>(&qr[m]);
        uint32_t x[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(hq[e]);
          const float2 fs = __fmul2_rn(f, make_float2(s, s));
          x[e] = pack_h2(fs.x, fs.y);
        }
        *reinterpret_cast<uint4*>(at_h(rq_dst, i, qd * 32 + m * 8, kSboH128)) = make_uint4(x[0], x[1], x[2], x[3]);
      }
    }
  }
  __syncthreads();
  GDN_TICK(17);

  // (a) G | P = [K; Q] K^T at TMEM columns [0, 64), read by every head
  if (c.tid == 0) {
    tc::fence_after_sync();
    const uint32_t id = tc::instr_desc(tc::kBF16, 128, kC);
    for (int j = 0; j < kD / 16; ++j)
      tc::mma_ss<tc::kBF16>(c.tb + kPColGP, desc(sK, j * 256, kSboKQ), desc(sK, j * 256, kSboKQ), id, j > 0);
    tc::mma_commit(c.bar);
  }
  bool ok = mma_wait(c);
  GDN_TICK(18);
  // the Q rows are no longer read: the first head's V rows into their place,
  // landing during its solve
  if (ok && c.tid == 0) {
    ptx::mbar_arrive_expect_tx(rbar, kC * kD * 2);
    prep_rows_tma(sQ, &tmv, t0, h0 * (kD / 8), rbar);
  }
  rows_pending = ok;
  GDN_TICK(8);

  for (int hh = 0; hh < gsz && ok; ++hh) {     // ok is the same in every thread
    const bool last = hh == gsz - 1;
    c.h = h0 + hh;
    c.s_gam = gamA + hh * kC;
    c.s_beta = betaA + hh * kC;
    unsigned char* rec = record(p, slot, c.h);
    {
      // A (lanes 0-63, row-major) and M (lanes 64-127, to the record)
      float gp[32];
      tmem_ld<32>(c.tb + kPColGP + c.my + c.half * 32, gp);
      GDN_TICK(9);
      if (c.quarter < 2) {
        const int i = c.row;
        const float fi = c.s_beta[i] * c.s_rk[i];
        const float gi = c.s_gam[i];
        float* arow = sA + i * kPadA + c.half * 32;
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 rk4 = *reinterpret_cast<const float4*>(c.s_rk + c.half * 32 + e);
          const float4 gm4 = *reinterpret_cast<const float4*>(c.s_gam + c.half * 32 + e);
          const float rk[4] = {rk4.x, rk4.y, rk4.z, rk4.w}, gm[4] = {gm4.x, gm4.y, gm4.z, gm4.w};
          float a[4];
#pragma unroll
          for (int u = 0; u < 4; u += 2) {     // ((fi r_k) e^{gi - gm}) g on channel pairs
            const int j = c.half * 32 + e + u;
            float2 t = __fmul2_rn(make_float2(fi, fi), make_float2(rk[u], rk[u + 1]));
            t = __fmul2_rn(t, make_float2(__expf(gi - gm[u]), __expf(gi - gm[u + 1])));
            t = __fmul2_rn(t, make_float2(gp[e + u], gp[e + u + 1]));
            a[u] = (j < i) ? t.x : 0.f;
            a[u + 1] = (j + 1 < i) ? t.y : 0.f;
          }
          *reinterpret_cast<float4*>(arow + e) = make_float4(a[0], a[1], a[2], a[3]);
        }
      } else {
        const int i = c.row - kC;
        const float fi = c.s_rq[i];
        const float gi = c.s_gam[i];
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 rk4 = *reinterpret_cast<const float4*>(c.s_rk + c.half * 32 + e);
          const float4 gm4 = *reinterpret_cast<const float4*>(c.s_gam + c.half * 32 + e);
          const float rk[4] = {rk4.x, rk4.y, rk4.z, rk4.w}, gm[4] = {gm4.x, gm4.y, gm4.z, gm4.w};
          float m[4];
#pragma unroll
          for (int u = 0; u < 4; u += 2) {
            const int j = c.half * 32 + e + u;
            float2 t = __fmul2_rn(make_float2(fi, fi), make_float2(rk[u], rk[u + 1]));
            t = __fmul2_rn(t, make_float2(__expf(gi - gm[u]), __expf(gi - gm[u + 1])));
            t = __fmul2_rn(t, make_float2(gp[e + u], gp[e + u + 1]));
            m[u] = (j <= i) ? t.x : 0.f;
            m[u + 1] = (j + 1 <= i) ? t.y : 0.f;
          }
          *reinterpret_cast<uint2*>(at_h(rec + kRecM, i, c.half * 32 + e, kSboH64)) = pack_h4(m[0], m[1], m[2], m[3]);
        }
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(19);

    // diagonal blocks D_bb = (I + A_bb)^-1 (warps 0-1: block bb, column cc) ...
    if (c.tid < 64) {
      const int bb = c.tid >> 4, cc = c.tid & 15;
      const float* ab = sA + (16 * bb) * kPadA + 16 * bb;
      float x[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) x[r] = (r == cc) ? 1.f : 0.f;
#pragma unroll
      for (int r = 0; r < 15; ++r) {
        const float xr = x[r];
#pragma unroll
        for (int i = r + 1; i < 16; ++i) x[i] -= ab[i * kPadA + r] * xr;
      }
      float* xb = sX + (16 * bb) * kPadA + 16 * bb + cc;
#pragma unroll
      for (int r = 0; r < 16; ++r) xb[r * kPadA] = x[r];
    } else {
      // ... while warps 2-7 write K-hat^T = K^T diag(e^{Gam_last-Gam} r_k) to the
      // record.  Job J: the 8 x 8 core matrices (token groups 4 (J / 16) .. +3,
      // k group J % 16) of the K rows, transposed by ldmatrix: lane L holds
      // k = 8 kg + L / 4 at tokens 2 (L % 4), +1 of each; lanes L, L ^ 1 swap
      // halves so that each holds 4 consecutive tokens of one matrix.
      const int p2 = c.lane & 3;
      const bool odd = p2 & 1;
      for (int J = c.warp - 2; J < 32; J += kThreads / 32 - 2) {
        const int kg = J & 15, tgb = (J >> 4) * 4;
        uint32_t r[4];
        ptx::ldmatrix_x4_trans(sK + (tgb + (c.lane >> 3)) * kSboKQ + kg * 128 + (c.lane & 7) * 16, r);
        const int k = kg * 8 + (c.lane >> 2);
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const uint32_t mine = odd ? r[2 * pr + 1] : r[2 * pr];
          const uint32_t got = __shfl_xor_sync(0xffffffffu, odd ? r[2 * pr] : r[2 * pr + 1], 1);
          const uint32_t lo = odd ? got : mine, hi = odd ? mine : got;   // tokens t, t+1 | t+2, t+3
          const int t = (tgb + 2 * pr + (odd ? 1 : 0)) * 8 + 2 * (p2 & 2);
          const float4 sc = *reinterpret_cast<const float4*>(c.s_kh + t);
          const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lo));
          const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hi));
          *reinterpret_cast<uint2*>(at_h(rec + kRecKh, k, t, kSboH64)) =
              [&] {
                const float2 p0 = __fmul2_rn(f0, make_float2(sc.x, sc.y));
                const float2 p1 = __fmul2_rn(f1, make_float2(sc.z, sc.w));
                return pack_h4(p0.x, p0.y, p1.x, p1.y);
              }();
        }
      }
    }
    __syncthreads();
    GDN_TICK(20);
    solve_doubling(sA, sX, sY, c.tid);
    GDN_TICK(13);

    // right-hand operands, K-major (row j, token t), bf16 hi | lo:
    // B_U[j][t] = beta_t X[j][t] over A, B_W[j][t] = beta_t g_t r_kt X[j][t] over X
    {
      uint4 uh[2], ul[2], wh[2], wl[2];
#pragma unroll
      for (int it = 0; it < 2; ++it) {
        const int item = c.tid + it * kThreads;
        const int j = (item >> 6) * 8 + (item & 7), tg = (item >> 3) & 7;
        const float4 x0 = *reinterpret_cast<const float4*>(sX + j * kPadA + tg * 8);
        const float4 x1 = *reinterpret_cast<const float4*>(sX + j * kPadA + tg * 8 + 4);
        const float4 b0 = *reinterpret_cast<const float4*>(c.s_beta + tg * 8);
        const float4 b1 = *reinterpret_cast<const float4*>(c.s_beta + tg * 8 + 4);
        const float4 w0 = *reinterpret_cast<const float4*>(c.s_kw + tg * 8);
        const float4 w1 = *reinterpret_cast<const float4*>(c.s_kw + tg * 8 + 4);
        const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        const float bs[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint32_t hu[4], lu[4], hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = tg * 8 + 2 * e;
          const float xa = t <= j ? xs[2 * e] : 0.f, xb = t + 1 <= j ? xs[2 * e + 1] : 0.f;
          const float2 x2 = make_float2(xa, xb);
          split_bf16(__fmul2_rn(x2, make_float2(bs[2 * e], bs[2 * e + 1])), hu[e], lu[e]);
          split_bf16(__fmul2_rn(x2, make_float2(ws[2 * e], ws[2 * e + 1])), hw[e], lw[e]);
        }
        uh[it] = make_uint4(hu[0], hu[1], hu[2], hu[3]);
        ul[it] = make_uint4(lu[0], lu[1], lu[2], lu[3]);
        wh[it] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        wl[it] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      GDN_TICK(14);
      __syncthreads();                  // every X value is read before the operands overwrite A and X
      GDN_TICK(21);
#pragma unroll
      for (int it = 0; it < 2; ++it) {
        const int item = c.tid + it * kThreads;
        const int j = (item >> 6) * 8 + (item & 7), tg = (item >> 3) & 7;
        const uint32_t off = tc::kmajor_offset(j, tg * 8, 2, kSboOp);
        *reinterpret_cast<uint4*>(sm + kQA + off) = uh[it];
        *reinterpret_cast<uint4*>(sm + kQA + kC * kC * 2 + off) = ul[it];
        *reinterpret_cast<uint4*>(sm + kQX + off) = wh[it];
        *reinterpret_cast<uint4*>(sm + kQX + kC * kC * 2 + off) = wl[it];
      }
    }
    ptx::fence_proxy_async_smem();      // the operands above, for the MMAs
    tc::fence_before_sync();
    ok = rows_wait();                   // this head's V rows (and the barrier for the operands)
    if (!ok) break;
    if (nvalid < kC) {
      prep_zero_rows(sQ, nvalid, c.tid);
      ptx::fence_proxy_async_smem();
      __syncthreads();
    }
    GDN_TICK(22);

    // U0^T = V^T B_U^T, W^T = K^T B_W^T; A operands MN-major (LBO = one
    // 8-token group of 128 rows, SBO 128), one MMA per 16 tokens, hi then lo
    const uint32_t a_v = ptx::smem_u32(sQ), a_k = ptx::smem_u32(sK);
    if (last) {
      if (c.tid == 0) {
        tc::fence_after_sync();
        prep_rhs_mma(c, a_v, sm + kQA, kPColU);
        prep_rhs_mma(c, a_k, sm + kQX, kPColW);   // over G | P, read for the last time above
        tc::mma_commit(c.bar);
      }
      ok = mma_wait(c);
      GDN_TICK(23);
      if (ok) {
        float u[32], w[32];
        tc::tmem_ld16(c.tb + kPColU + c.my + c.half * 32, *reinterpret_cast<float(*)[16]>(u));
        tc::tmem_ld16(c.tb + kPColU + c.my + c.half * 32 + 16, *reinterpret_cast<float(*)[16]>(u + 16));
        tc::tmem_ld16(c.tb + kPColW + c.my + c.half * 32, *reinterpret_cast<float(*)[16]>(w));
        tc::tmem_ld16(c.tb + kPColW + c.my + c.half * 32 + 16, *reinterpret_cast<float(*)[16]>(w + 16));
        tc::tmem_ld_wait();
        prep_store_u0(c, rec, u);
        prep_store_negw(c, rec, w);
      }
    } else {
      // U0^T, then W^T in the same columns: G | P stays for the next head
      if (c.tid == 0) {
        tc::fence_after_sync();
        prep_rhs_mma(c, a_v, sm + kQA, kPColU);
        tc::mma_commit(c.bar);
      }
      ok = mma_wait(c);
      if (ok) {
        // the V rows are read: the next head's into their place
        if (c.tid == 0) {
          ptx::mbar_arrive_expect_tx(rbar, kC * kD * 2);
          prep_rows_tma(sQ, &tmv, t0, (c.h + 1) * (kD / 8), rbar);
        }
        rows_pending = true;
        float u[32];
        tc::tmem_ld16(c.tb + kPColU + c.my + c.half * 32, *reinterpret_cast<float(*)[16]>(u));
        tc::tmem_ld16(c.tb + kPColU + c.my + c.half * 32 + 16, *reinterpret_cast<float(*)[16]>(u + 16));
        tc::tmem_ld_wait();
        prep_store_u0(c, rec, u);
      }
      tc::fence_before_sync();
      __syncthreads();                  // U0^T is out of its columns before W^T overwrites them
      if (ok) {
        if (c.tid == 0) {
          tc::fence_after_sync();
          prep_rhs_mma(c, a_k, sm + kQX, kPColU);
          tc::mma_commit(c.bar);
        }
        ok = mma_wait(c);
      }
      GDN_TICK(23);
      if (ok) {
        float w[32];
        tc::tmem_ld16(c.tb + kPColU + c.my + c.half * 32, *reinterpret_cast<float(*)[16]>(w));
        tc::tmem_ld16(c.tb + kPColU + c.my + c.half * 32 + 16, *reinterpret_cast<float(*)[16]>(w + 16));
        tc::tmem_ld_wait();
        prep_store_negw(c, rec, w);
        if (c.tid < kC) head_scalars(c, gamA + (hh + 1) * kC, betaA + (hh + 1) * kC, c.tid, c.s_rk[c.tid]);
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(31);
  }
  if (!ok) {
    if (c.tid == 0) atomicExch(p.err, 1);
    ptx::mbar_wait(c.bar, c.phase ^ 1u);
  }
  if (rows_pending && c.warp == 0) ptx::mbar_wait(rbar, rphase);   // no row copy outlives the CTA
  tc::fence_before_sync();
  __syncthreads();
  if (c.warp == 0) tc::tmem_dealloc(c.tb, kPrepTmemCols);
}

// ---- the split schedule: scan (serial over chunks, per sequence and head) ---------

// 17 warps: warps 0-15 are the epilogue workers -- warp w reaches TMEM lanes
// 32 (w % 4) .. +31 and owns column group w / 4 (a quarter of each
// accumulator's columns); warp 16 waits for the bulk copies and the MMAs, and
// its lane 0 issues both, so that its issue stalls never delay the workers.
constexpr int kScanWorkers = 512;
constexpr int kScanThreads = kScanWorkers + 32;
constexpr int kScanThreadsNorm = kScanThreads + 256;   // + 8 norm warps: two groups of the 4 TMEM lane quarters

template <bool NORM>
__global__ void __launch_bounds__(NORM ? kScanThreadsNorm : kScanThreads, 1) chunk_scan_kernel(const ChunkParams p) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const float4* sU0 = reinterpret_cast<const float4*>(sm + kRecU);
  unsigned char* sU = sm + kScanU;
  // [0] MMA; record groups [1] -W | Qs, [2] M | K-hat^T, [3] U0^T | g_last
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kScanBar);
  const int bh = blockIdx.x;
  const int b = bh / p.Hv;
  Ctx c;
  ctx_init(c, p, bh - b * p.Hv);
  c.bar = bars;
  const bool mw = c.warp == kScanWorkers / 32;     // the MMA / copy warp
  const bool worker = c.warp < kScanWorkers / 32;
  const bool nw = NORM && c.warp > kScanWorkers / 32;   // a norm warp
  const bool issuer = mw && c.lane == 0;
  uint64_t* ybar = reinterpret_cast<uint64_t*>(sm + kScanYBar);   // [0..1] y ready, [2..3] y read, by parity
  volatile int* s_fail = reinterpret_cast<volatile int*>(sm + kScanFail);
  // barriers of the chain (workers + copy warp); the norm warps keep their own
  auto chain_sync = [&]() { asm volatile("bar.sync 7, %0;" ::"n"(kScanThreads) : "memory"); };
  auto chain_or = [&](bool pred) -> bool {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 7, %2, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred)), "n"(kScanThreads)
        : "memory");
    return r != 0;
  };
  const int cg = (c.warp >> 2) & 3;                // column group of a worker
  long long s0, s1;
  seq_range(p, b, s0, s1);
  // this window's chunks of the sequence
  int n_chunks = static_cast<int>((s1 - s0 + kC - 1) / kC) - p.win_c0;
  n_chunks = n_chunks < 0 ? 0 : (n_chunks > p.win_len ? p.win_len : n_chunks);
  if (p.win_c0 > 0 && n_chunks == 0) return;       // finished in an earlier window: its state is in place
  const long long slot0 = seq_first_slot(p, b);
  // TMEM columns: [0,128) unused | U (even) | y (even) | R fp32 [256,384) | y (odd) | U (odd).
  // The first MMA batch writes [U | y] (even) or [y | U] (odd) in one N = 128
  // product, the second [y | R] or [R | y] in one N = 192 product; odd chunks
  // mirror the order of the stacked B operands in shared memory to match.
  // Both batches are kind::f16: fp16(R) and fp16(U^T) from shared memory.
  constexpr uint32_t cDR = 256;
  if (NORM && c.tid == 0) {
    ptx::mbar_init(ybar + 0, 1);
    ptx::mbar_init(ybar + 1, 1);
    ptx::mbar_init(ybar + 2, 8);
    ptx::mbar_init(ybar + 3, 8);
    *s_fail = 0;
  }
  tmem_setup(c, reinterpret_cast<uint32_t*>(sm + kScanBar + 32), bars, 4, kTmemCols);
  if (worker) state_load(p.win_c0 == 0 ? p.state_in : p.carry, c, bh, cDR, cg * 32, 32);
  const uint32_t lane_cols = c.tb + c.my + cg * 32;   // a worker's 32 columns of R / R fp32

  // record groups issued and waited for, counted by the copy warp only
  int issued[4] = {0, 0, 0, 0}, done[4] = {0, 0, 0, 0};
  // group g of chunk ch; groups 1, 2 put their two operands in chunk-parity order
  auto load = [&](int g, int ch) {
    if (issuer) {
      const unsigned char* rec = record(p, slot0 + ch, c.h);
      const bool odd = ch & 1;
      if (g == 1) {
        ptx::mbar_arrive_expect_tx(&bars[1], 2 * kC * kD * 2 + 16);   // one arrival: the barrier counts 1
        ptx::bulk_g2s(sm + kScanG1 + (odd ? kC * kD * 2 : 0), rec + kRecW, kC * kD * 2, &bars[1]);
        ptx::bulk_g2s(sm + kScanG1 + (odd ? 0 : kC * kD * 2), rec + kRecQ, kC * kD * 2, &bars[1]);
        ptx::bulk_g2s(sm + kScanGl1, rec + kRecSc, 16, &bars[1]);
      } else if (g == 2) {
        ptx::mbar_arrive_expect_tx(&bars[2], kC * kC * 2 + kD * kC * 2);
        ptx::bulk_g2s(sm + kScanG2 + (odd ? kD * kC * 2 : 0), rec + kRecM, kC * kC * 2, &bars[2]);
        ptx::bulk_g2s(sm + kScanG2 + (odd ? 0 : kC * kC * 2), rec + kRecKh, kD * kC * 2, &bars[2]);
      } else {
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive_expect_tx(&bars[3], kRecBytes - kRecU);
        for (uint32_t off = kRecU; off < kRecBytes; off += 16384)
          ptx::bulk_g2s(sm + off, rec + off, kRecBytes - off < 16384 ? kRecBytes - off : 16384, &bars[3]);
      }
    }
    if (mw) ++issued[g];
  };
  // the copy warp waits for group g of chunk ch (true elsewhere)
  auto wait_group = [&](int g, int ch) -> bool {
    if (!mw) return true;
    const bool ok = ptx::mbar_wait(&bars[g], ch & 1);
    done[g] += ok;
    return ok;
  };
  // MMA completion: the copy warp polls, the CTA agrees (false if it gave up)
  // (g3_ch >= 0: also group 3 of that chunk; g1_ch >= 0: also group 1)
  auto mma_done = [&](bool ok_in, int g3_ch = -1, int g1_ch = -1) -> bool {
    bool ok = ok_in;
    if (mw) ok = ok && ptx::mbar_wait(c.bar, c.phase);
    if (g3_ch >= 0) ok = wait_group(3, g3_ch) && ok;
    if (g1_ch >= 0) ok = wait_group(1, g1_ch) && ok;
    c.phase ^= 1u;
    const bool all = !chain_or(!ok);
    tc::fence_after_sync();
    return all;
  };
  // R (fp32 master, a worker's 32 columns) -> fp16(R), the next first batch's
  // A operand; then R *= gl in place for the next second batch, which adds
  // U^T K-hat^T to g_last R (one pass over R per chunk)
  auto r_pass = [&](float gl) {
    float v[16], w[16];
    tc::tmem_ld16(lane_cols + cDR, v);
    tc::tmem_ld16(lane_cols + cDR + 16, w);
    tc::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; i += 8) {          // row c.row, keys 32 cg ..
      *reinterpret_cast<uint4*>(at_h(sm + kScanR, c.row, cg * 32 + i, kSboH128)) =
          make_uint4(pack_h2(v[i], v[i + 1]), pack_h2(v[i + 2], v[i + 3]), pack_h2(v[i + 4], v[i + 5]),
                     pack_h2(v[i + 6], v[i + 7]));
      *reinterpret_cast<uint4*>(at_h(sm + kScanR, c.row, cg * 32 + 16 + i, kSboH128)) =
          make_uint4(pack_h2(w[i], w[i + 1]), pack_h2(w[i + 2], w[i + 3]), pack_h2(w[i + 4], w[i + 5]),
                     pack_h2(w[i + 6], w[i + 7]));
    }
    ptx::fence_proxy_async_smem();
#pragma unroll
    for (int i = 0; i < 16; i += 2) {          // packed f32x2
      const float2 a = __fmul2_rn(make_float2(v[i], v[i + 1]), make_float2(gl, gl));
      const float2 b = __fmul2_rn(make_float2(w[i], w[i + 1]), make_float2(gl, gl));
      v[i] = a.x;
      v[i + 1] = a.y;
      w[i] = b.x;
      w[i + 1] = b.y;
    }
    tc::tmem_st16(lane_cols + cDR, v);
    tc::tmem_st16(lane_cols + cDR + 16, w);
    tc::tmem_st_wait();
  };
  // U^T = (R (-W)^T from TMEM) + U0^T (shared memory) -> fp16 rows of the U^T operand
  auto epi_u = [&](uint32_t col_u) {
    float u[16];
    tc::tmem_ld16(c.tb + col_u + c.my + cg * 16, u);
    tc::tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 f = sU0[u0_index(cg * 4 + e / 4, c.row)];
      const float2 lo = __fadd2_rn(make_float2(u[e], u[e + 1]), make_float2(f.x, f.y));
      const float2 hi = __fadd2_rn(make_float2(u[e + 2], u[e + 3]), make_float2(f.z, f.w));
      u[e] = lo.x;
      u[e + 1] = lo.y;
      u[e + 2] = hi.x;
      u[e + 3] = hi.y;
    }
#pragma unroll
    for (int e = 0; e < 16; e += 8)
      *reinterpret_cast<uint4*>(at_h(sU, c.row, cg * 16 + e, kSboH64)) =
          make_uint4(pack_h2(u[e], u[e + 1]), pack_h2(u[e + 2], u[e + 3]), pack_h2(u[e + 4], u[e + 5]),
                     pack_h2(u[e + 6], u[e + 7]));
    ptx::fence_proxy_async_smem();
  };
  // ---- fused norm: the 8 norm warps (warp % 4 = TMEM lane quarter q, dv =
  // 32 q + lane; group g of 4 warps takes tokens 32 g .. 32 g + 31) normalise
  // chunk ch from its y in TMEM while the chain runs chunk ch + 1, and store
  // the bf16 rows to every destination.  z rows
  // (256 bytes per token) come by cp.async three chunks ahead into buffer
  // ch % 3, which the normed rows then overwrite in place to be stored as
  // 16-byte pieces.  Handshakes: ybar[ch & 1] (the MMA commit after the
  // second batch of chunk ch) says y is complete; ybar[2 + (ch & 1)] (one
  // arrival per norm warp) says it has been read, before the first batch of
  // chunk ch + 2 overwrites those columns.
  auto norm_chunks = [&]() {
    const int grp = (c.tid - kScanThreads) >> 7;     // token half of the chunk
    const int nt = (c.tid - kScanThreads) & 127;     // thread of the group
    const int bar_id = 5 + grp;
    const float gam = __ldg(p.gamma + c.row);
    float4* s_tok = reinterpret_cast<float4*>(sm + kScanNorm + grp * 256);   // [token of the round] sums by quarter
    auto nbar = [&]() { asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory"); };
    auto load_z = [&](int ch) {
      const long long t0 = s0 + static_cast<long long>(p.win_c0 + ch) * kC;
      const int nvalid = static_cast<int>((s1 - t0) < kC ? (s1 - t0) : kC);
      unsigned char* zb = sm + kScanZ + (ch % 3) * kZBuf;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int piece = nt + k * 128;
        const int tok = grp * 32 + (piece >> 4);
        const int seg = (piece & 15) * 8;
        if (tok < nvalid)
          ptx::cp_async16(zb + (tok * kD + seg) * 2, p.z + (t0 + tok) * p.z_stride + c.h * kD + seg);
      }
      ptx::cp_async_commit();
    };
    // a bounded wait that also gives up once the chain has failed
    auto wait_or_fail = [&](uint64_t* bar, uint32_t parity) -> bool {
      for (uint32_t i = 0; i < ptx::kSpinLimit; ++i) {
        if (ptx::mbar_try_wait(bar, parity)) return true;
        if (*s_fail) return false;
      }
      return false;
    };
    for (int ch = 0; ch < 3 && ch < n_chunks; ++ch) load_z(ch);
    for (int ch = 0; ch < n_chunks; ++ch) {
      // every norm thread takes the same branch: a thread that gave up makes all stop
      uint32_t any_fail;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
          "bar.red.or.pred p, %2, 128, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(any_fail)
          : "r"(static_cast<uint32_t>(!wait_or_fail(&ybar[ch & 1], (ch >> 1) & 1))), "r"(bar_id)
          : "memory");
      if (any_fail) {
        if (nt == 0) atomicExch(p.err, 1);
        break;
      }
      tc::fence_after_sync();
      const int newer = n_chunks - 1 - ch;           // z groups committed after this chunk's
      if (newer >= 2) ptx::cp_async_wait<2>();
      else if (newer == 1) ptx::cp_async_wait<1>();
      else ptx::cp_async_wait<0>();
      nbar();                                        // every norm thread's z pieces of the chunk have landed
      const uint32_t col_y = (ch & 1) ? 384 : 192;
      const long long t0 = s0 + static_cast<long long>(p.win_c0 + ch) * kC;
      const int nvalid = static_cast<int>((s1 - t0) < kC ? (s1 - t0) : kC);
      __nv_bfloat16* zt = reinterpret_cast<__nv_bfloat16*>(sm + kScanZ + (ch % 3) * kZBuf);
      // this warp's y of the chunk (both rounds) out of TMEM first, and its
      // columns released at once: the chain's first batch two chunks on
      // waits only for these loads, not for the norm arithmetic
      float ya[16], yb[16];
      tc::tmem_ld16(c.tb + col_y + c.my + grp * 32, ya);
      tc::tmem_ld16(c.tb + col_y + c.my + grp * 32 + 16, yb);
      tc::tmem_ld_wait();
      tc::fence_before_sync();
      __syncwarp();
      if (c.lane == 0) ptx::mbar_arrive(&ybar[2 + (ch & 1)]);
#pragma unroll
      for (int r = 0; r < 2; ++r) {                  // 16 tokens per round
        const int tb = grp * 32 + r * 16;            // first token of the round
        const float(&y)[16] = r ? yb : ya;
        // sums of y^2 over this warp's 32 dv for the 16 tokens: halve the
        // token set per exchange (8 + 4 + 2 + 1 shuffles), then one more; the
        // pair of lanes 2t, 2t + 1 ends with token t
        float s8[8], s4[4], s2[2], s1v;
        const bool b16 = c.lane & 16, b8 = c.lane & 8, b4 = c.lane & 4, b2 = c.lane & 2;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float lo = y[i] * y[i], hi = y[i + 8] * y[i + 8];
          s8[i] = (b16 ? hi : lo) + __shfl_xor_sync(0xffffffffu, b16 ? lo : hi, 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) s4[i] = (b8 ? s8[i + 4] : s8[i]) + __shfl_xor_sync(0xffffffffu, b8 ? s8[i] : s8[i + 4], 8);
#pragma unroll
        for (int i = 0; i < 2; ++i) s2[i] = (b4 ? s4[i + 2] : s4[i]) + __shfl_xor_sync(0xffffffffu, b4 ? s4[i] : s4[i + 2], 4);
        s1v = (b2 ? s2[1] : s2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? s2[0] : s2[1], 2);
        s1v += __shfl_xor_sync(0xffffffffu, s1v, 1);
        if ((c.lane & 1) == 0) reinterpret_cast<float*>(s_tok)[(c.lane >> 1) * 4 + c.quarter] = s1v;
        nbar();
        const float4 pp = s_tok[c.lane & 15];
        const float rr = rsqrtf((pp.x + pp.y + pp.z + pp.w) / static_cast<float>(kD) + p.eps);
#pragma unroll
        for (int i = 0; i < 16; ++i) {               // normed rows over the z they gate (same element)
          const float ri = __shfl_sync(0xffffffffu, rr, i);
          __nv_bfloat16* e = zt + (tb + i) * kD + c.row;
          const float zz = __bfloat162float(*e);
          const float sg = rcp_approx(1.f + ex2_approx(zz * -1.4426950408889634f));   // sigmoid(z), 2^(-z log2 e)
          *e = __float2bfloat16_rn((y[i] * ri * gam) * (zz * sg));
        }
        nbar();
#pragma unroll
        for (int k = 0; k < 2; ++k) {                // 16 rows x 16 pieces of 16 bytes
          const int piece = nt + k * 128;
          const int tok = tb + (piece >> 4);
          const int seg = (piece & 15) * 8;
          if (tok < nvalid) {
            const uint4 v = *reinterpret_cast<const uint4*>(zt + tok * kD + seg);
            const long long off = (t0 + tok) * p.out_stride + static_cast<long long>(p.out_head0 + c.h) * kD + seg;
            if (off + 8 <= p.out_elems) {
#pragma unroll
              for (int d = 0; d < 8; ++d)
                if (d < p.n_dst) *reinterpret_cast<uint4*>(p.dst[d] + off) = v;
            } else {
              atomicExch(p.err, 1);
            }
          }
        }
      }
      nbar();                                        // buffer ch % 3 fully stored: refill it
      if (ch + 3 < n_chunks) load_z(ch + 3);
    }
    ptx::cp_async_wait<0>();                         // no z copy may land after the CTA exits
  };
  // o rows of chunk ch from y^T (plain scan): a worker's dv = row, tokens cg*16 + part*8 .. +7
  auto epi_o = [&](int ch, int part) {
    const uint32_t col_y = (ch & 1) ? 384 : 192;
    const long long t0 = s0 + static_cast<long long>(p.win_c0 + ch) * kC;
    const int nvalid = static_cast<int>((s1 - t0) < kC ? (s1 - t0) : kC);
    const int tok = cg * 16 + part * 8;
    const int nv = nvalid - tok;
    float y[8];
    tc::tmem_ld8(c.tb + col_y + c.my + tok, y);
    tc::tmem_ld_wait();
    const size_t orow = static_cast<size_t>(p.Hv) * kD;
    const size_t base = (static_cast<size_t>(t0 + tok) * p.Hv + c.h) * kD + c.row;
    if (p.flags & GDN_F_O_BF16) {
      __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.o) + base;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < nv) o[i * orow] = __float2bfloat16_rn(y[i]);
    } else {
      float* o = static_cast<float*>(p.o) + base;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < nv) o[i * orow] = y[i];
    }
  };

  bool failed = false;
  if (nw) {
    if (n_chunks > 0) norm_chunks();
  } else {
    if (n_chunks > 0) {
      load(1, 0);
      load(2, 0);
      load(3, 0);
      const bool ok = wait_group(1, 0);      // g_last of chunk 0
      if (chain_or(!ok)) {
        failed = true;
      } else {
        tc::fence_after_sync();
        if (worker) r_pass(reinterpret_cast<const float*>(sm + kScanGl1)[0]);   // fp16(R_0), g_last R_0
      }
      tc::fence_before_sync();
      chain_sync();
    }
    for (int ch = 0; ch < n_chunks && !failed; ++ch) {
      const bool odd = ch & 1;
      const uint32_t col_b1 = odd ? 384 : 128;       // [y | U] or [U | y]
      const uint32_t col_b2 = odd ? 256 : 192;       // [R | y] or [y | R]
      const uint32_t col_u = odd ? 448 : 128;
      // -W | Qs of this chunk are in shared memory (waited for with the previous
      // second batch; U0^T is waited for under the first batch, before the
      // epilogue that adds it)
      tc::fence_after_sync();
      GDN_TICK(29);
      bool yok = true;
      if (issuer) {              // first batch: [U | y] = R [-W; Qs]^T (U0^T is added in the epilogue)
        // the norm warps have read y of chunk ch - 2, whose columns this batch overwrites
        if (NORM && ch >= 2) yok = ptx::mbar_wait(&ybar[2 + (ch & 1)], ((ch >> 1) - 1) & 1);
        if (yok) {
          tc::fence_after_sync();
          const uint32_t id = tc::instr_desc(tc::kF16, 128, 2 * kC);
          for (int j = 0; j < kD / 16; ++j)
            tc::mma_ss<tc::kF16>(c.tb + col_b1, desc(sm + kScanR, j * 256, kSboH128),
                                 desc(sm + kScanG1, j * 256, kSboH128), id, j > 0);
          tc::mma_commit(c.bar);
        }
      } else if (worker && !NORM && ch > 0) {   // under it: half of the previous o
        epi_o(ch - 1, 0);
      }
      tc::fence_before_sync();
      if (!mma_done(yok, ch)) { failed = true; break; }
      GDN_TICK(24);
      if (ch + 1 < n_chunks) load(1, ch + 1);
      if (worker) epi_u(col_u);
      bool ok = wait_group(2, ch);
      tc::fence_before_sync();
      if (chain_or(!ok)) { failed = true; break; }
      tc::fence_after_sync();
      GDN_TICK(25);
      if (issuer) {              // second batch: [y | R] += U^T [M; K-hat^T]^T
        const uint32_t id = tc::instr_desc(tc::kF16, 128, kC + kD);
        for (int j = 0; j < kC / 16; ++j)
          tc::mma_ss<tc::kF16>(c.tb + col_b2, desc(sU, j * 256, kSboH64), desc(sm + kScanG2, j * 256, kSboH64), id, 1);
        tc::mma_commit(c.bar);
        if (NORM) tc::mma_commit(&ybar[ch & 1]);   // y of chunk ch complete: the norm warps take it
      } else if (worker && !NORM && ch > 0) {
        epi_o(ch - 1, 1);        // under it: the other half of the previous o
      }
      if (ch + 1 < n_chunks) load(3, ch + 1);
      tc::fence_before_sync();
      if (!mma_done(true, -1, ch + 1 < n_chunks ? ch + 1 : -1)) { failed = true; break; }   // + group 1 of ch + 1
      GDN_TICK(26);
      if (ch + 1 < n_chunks) {
        load(2, ch + 1);
        if (worker) r_pass(reinterpret_cast<const float*>(sm + kScanGl1)[0]);   // fp16(R), g_last(ch + 1) R
      }
      tc::fence_before_sync();
      chain_sync();
      GDN_TICK(27);
    }
    if (!NORM && !failed && n_chunks > 0 && worker) {
      epi_o(n_chunks - 1, 0);
      epi_o(n_chunks - 1, 1);
    }
    if (failed) {
      // bounded waits for the MMA and the bulk copies still in flight; the norm warps stop
      if (c.tid == 0) {
        atomicExch(p.err, 1);
        if (NORM) *s_fail = 1;
      }
      if (mw) {
        ptx::mbar_wait(c.bar, c.phase ^ 1u);
        for (int g = 1; g <= 3; ++g)
          if (issued[g] > done[g]) ptx::mbar_wait(&bars[g], done[g] & 1);
      }
    } else if (worker) {
      state_store(p.carry, c, bh, cDR, cg * 32, 32);
    }
  }
  if (NORM && p.n_dst > 1) __threadfence_system();  // peer stores performed before the call's signal
  tc::fence_before_sync();
  __syncthreads();
  if (c.warp == 0) tc::tmem_dealloc(c.tb, kTmemCols);
}

// ---- host side ----------------------------------------------------------------

int set_smem_attr(const void* fn, uint32_t bytes, bool (&done)[64]) {
  static std::mutex mu;
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != GDN_OK) return rc;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev & 63]) {
    rc = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
                     "chunked kernel smem attribute");
    if (rc != GDN_OK) return rc;
    done[dev & 63] = true;
  }
  return GDN_OK;
}

// Argument checks shared by the chunked entry points; fills p without the
// workspace fields.
// Value heads per prep CTA for `r` value heads per key head: the largest
// divisor of r that is at most kPrepGroup.
int prep_group_size(int r) {
  for (int g = kPrepGroup; g > 1; --g)
    if (r % g == 0) return g;
  return 1;
}

int chunked_args(ChunkParams& p, const void* q, const void* k, const void* v, long long q_stride, long long k_stride,
                 long long v_stride, const float* a, const float* b, const float* A_log, const float* dt_bias,
                 const float* state_in, float* state_out, void* o, const int32_t* cu_seqlens, int B, int T, int Hk,
                 int Hv, int Dk, int Dv, unsigned flags) {
  if (flags & ~(GDN_F_O_BF16 | GDN_F_QK_L2NORM)) return fail(GDN_ERR_FLAGS, "unknown flag bits 0x%x", flags);
  if (B < 0 || T < 0 || Hk <= 0 || Hv <= 0) return fail(GDN_ERR_SHAPE, "bad sizes B=%d T=%d Hk=%d Hv=%d", B, T, Hk, Hv);
  if (Dk != kD || Dv != kD) return fail(GDN_ERR_SHAPE, "Dk=%d Dv=%d: only 128x128 heads are built", Dk, Dv);
  if (Hv % Hk) return fail(GDN_ERR_SHAPE, "Hv=%d is not a multiple of Hk=%d", Hv, Hk);
  if (static_cast<long long>(B) * Hv >= (1LL << 31)) return fail(GDN_ERR_SHAPE, "B*Hv too large");
  const long long total = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  if (B > 0 && total > 0 && (!q || !k || !v || !a || !b || !o))
    return fail(GDN_ERR_NULL, "q, k, v, a, b and o are required");
  if (B > 0 && (!A_log || !dt_bias)) return fail(GDN_ERR_NULL, "A_log and dt_bias are required");
  if (q_stride < static_cast<long long>(Hk) * kD || k_stride < static_cast<long long>(Hk) * kD ||
      v_stride < static_cast<long long>(Hv) * kD)
    return fail(GDN_ERR_SHAPE, "token strides too small for the heads");
  if (q_stride % 8 || k_stride % 8 || v_stride % 8)
    return fail(GDN_ERR_ALIGN, "token strides must be multiples of 8 elements (16 bytes)");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(state_in, 16) || !aligned(state_out, 16) ||
      !aligned(a, 4) || !aligned(b, 4) || !aligned(o, (flags & GDN_F_O_BF16) ? 2 : 4) || !aligned(cu_seqlens, 4))
    return fail(GDN_ERR_ALIGN, "q, k, v and states 16-byte aligned; a, b, o element-aligned");
  const size_t sbytes = static_cast<size_t>(B) * Hv * kD * kD * 4;
  const size_t obytes = static_cast<size_t>(total) * Hv * kD * ((flags & GDN_F_O_BF16) ? 2 : 4);
  if (state_in != state_out && overlap(state_in, sbytes, state_out, sbytes))
    return fail(GDN_ERR_ALIAS, "state_out partially overlaps state_in");
  if (overlap(o, obytes, state_in, sbytes) || overlap(o, obytes, state_out, sbytes))
    return fail(GDN_ERR_ALIAS, "o overlaps a state buffer");
  if (B == 0) return GDN_OK;               // nothing to launch: no CUDA call either
  int* err = nullptr;
  int rc = device_error_ptr(&err);
  if (rc != GDN_OK) return rc;
  p = ChunkParams{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                  static_cast<const __nv_bfloat16*>(v), q_stride, k_stride, v_stride, a, b, A_log, dt_bias,
                  state_in, state_out, o, cu_seqlens, B, cu_seqlens ? 0 : T, Hk, Hv, flags, err,
                  nullptr, nullptr, 0, 0, 0, 0, 0, prep_group_size(Hv / Hk), nullptr, nullptr, 0, nullptr, 0.f, 0, 0,
                  {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr}, 0, 0};
  return GDN_OK;
}

// Record slots of a window of `w` chunks per sequence: exact for uniform
// batches, an upper bound for packed ones (at most w chunks per sequence, at
// most one partial chunk per sequence overall).
long long window_slots(int B, int T, bool packed, long long w) {
  const long long nch = (static_cast<long long>(T) + kC - 1) / kC;
  const long long ww = w < nch ? w : nch;
  if (!packed) return static_cast<long long>(B) * ww;
  const long long cap = nch + B;
  return static_cast<long long>(B) * ww < cap ? static_cast<long long>(B) * ww : cap;
}

long long chunk_slots(int B, int T, bool packed) { return window_slots(B, T, packed, 1LL << 40); }

size_t records_base(int B) { return records_offset(B); }

// The whole call in one window.
size_t workspace_bytes(int B, int T, int Hv, bool packed) {
  return records_base(B) + static_cast<size_t>(chunk_slots(B, T, packed)) * Hv * kRecBytes;
}

// Smallest workspace: one chunk per sequence per window, plus the state
// carried between windows when the caller keeps no state_out.
size_t workspace_min_bytes(int B, int Hv, bool carry) {
  return records_base(B) + (carry ? static_cast<size_t>(B) * Hv * kD * kD * 4 : 0) +
         static_cast<size_t>(B) * Hv * kRecBytes;
}

struct SplitPlan {
  int win_len = 0, n_windows = 0;
  size_t carry_off = 0, rec_off = 0;
};

// Windows that fit `ws_size` bytes: one if the whole call fits, else the
// largest window of chunks per sequence that does.
bool plan_split(int B, int T, int Hv, bool packed, bool has_state_out, size_t ws_size, SplitPlan& pl) {
  const long long nch = (static_cast<long long>(T) + kC - 1) / kC;
  if (ws_size >= workspace_bytes(B, T, Hv, packed)) {
    pl.win_len = static_cast<int>(nch > 0 ? nch : 1);
    pl.n_windows = 1;
    pl.rec_off = records_base(B);
    return true;
  }
  pl.carry_off = records_base(B);
  pl.rec_off = pl.carry_off + (has_state_out ? 0 : static_cast<size_t>(B) * Hv * kD * kD * 4);
  if (ws_size < pl.rec_off) return false;
  const size_t per_chunk = static_cast<size_t>(B) * Hv * kRecBytes;
  const long long w = static_cast<long long>((ws_size - pl.rec_off) / per_chunk);
  if (w < 1) return false;
  pl.win_len = static_cast<int>(w < nch ? w : nch);
  pl.n_windows = static_cast<int>((nch + pl.win_len - 1) / pl.win_len);
  return true;
}

// Tensor maps of the prep's row copies: q, k (Hk heads) and v (Hv heads) as
// 3-D tensors (8 elements, tokens, 16-byte channel groups) so that one box of
// 8 x 8 x 16 lands as one 8-row group of the K-major no-swizzle layout (16
// core matrices of 8 rows x 16 bytes); tokens past the tensor read as zeros.
struct RowMaps {
  CUtensorMap q, k, v;
};

int make_rows_tmap(CUtensorMap* tm, const void* base, long long tokens, int heads, long long stride) {
  void* fn = nullptr;
  const int rc = tensor_map_encoder(&fn);
  if (rc != GDN_OK) return rc;
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  const cuuint64_t dims[3] = {8, static_cast<cuuint64_t>(tokens), static_cast<cuuint64_t>(heads) * (kD / 8)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride) * 2, 16};
  const cuuint32_t box[3] = {8, 8, kD / 8};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = reinterpret_cast<Encode>(fn)(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
                                                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(GDN_ERR_CUDA, "cuTensorMapEncodeTiled (prefill rows) failed (CUresult %d)", static_cast<int>(r));
  return GDN_OK;
}

// One window's launches: the chunk prefix (packed), the prep, the scan.
int launch_window(ChunkParams p, int T, int w, int win_len, const RowMaps& rm, cudaStream_t st) {
  const bool packed = p.cu != nullptr;
  const long long nch = (static_cast<long long>(T) + kC - 1) / kC;
  p.win_c0 = w * win_len;
  const long long left = nch - p.win_c0;
  p.nch_uniform = packed ? 0 : static_cast<int>(left < win_len ? left : win_len);
  p.n_slots = packed ? window_slots(p.B, T, true, win_len) : static_cast<long long>(p.B) * p.nch_uniform;
  if (p.n_slots > 0x7fffffffLL) return fail(GDN_ERR_SHAPE, "too many chunks for one launch");
  int rc;
  if (packed) {
    chunk_prefix_kernel<<<1, 1024, 0, st>>>(p.cu, p.B, p.win_c0, win_len, p.chunk_prefix);
    rc = cuda_status(cudaGetLastError(), "chunk prefix launch");
    if (rc != GDN_OK) return rc;
  }
  if (p.n_slots > 0) {
    if (p.n_slots * p.Hv > 0x7fffffffLL) return fail(GDN_ERR_SHAPE, "too many (chunk, head) pairs for one launch");
    chunk_prep_kernel<<<static_cast<unsigned>(p.n_slots * (p.Hv / p.prep_group)), kThreads, kPrepSmem, st>>>(
        p, rm.q, rm.k, rm.v);
    rc = cuda_status(cudaGetLastError(), "chunk prep launch");
    if (rc != GDN_OK) return rc;
  }
  const unsigned chains = static_cast<unsigned>(p.B * p.Hv);
  if (p.z) chunk_scan_kernel<true><<<chains, kScanThreadsNorm, kScanSmemNorm, st>>>(p);
  else chunk_scan_kernel<false><<<chains, kScanThreads, kScanSmem, st>>>(p);
  return cuda_status(cudaGetLastError(), "chunk scan launch");
}

// Launch the split schedule on a workspace of ws_size bytes (at least
// workspace_min_bytes()): one pass, or windows in order on `st`.
int run_split(ChunkParams p, int T, unsigned char* ws, size_t ws_size, cudaStream_t st) {
  const bool packed = p.cu != nullptr;
  SplitPlan pl;
  if (!plan_split(p.B, T, p.Hv, packed, p.state_out != nullptr, ws_size, pl))
    return fail(GDN_ERR_SHAPE, "workspace of %zu bytes, at least %zu needed (%zu for one window)", ws_size,
                workspace_min_bytes(p.B, p.Hv, p.state_out == nullptr), workspace_bytes(p.B, T, p.Hv, packed));
  p.ws = ws;
  static bool attr_prep[64] = {false}, attr_scan[64] = {false};
  int rc = set_smem_attr(reinterpret_cast<const void*>(chunk_prep_kernel), kPrepSmem, attr_prep);
  if (rc != GDN_OK) return rc;
  static bool attr_scan_norm[64] = {false};
  const void* scan = p.z ? reinterpret_cast<const void*>(chunk_scan_kernel<true>)
                         : reinterpret_cast<const void*>(chunk_scan_kernel<false>);
  rc = set_smem_attr(scan, p.z ? kScanSmemNorm : kScanSmem, p.z ? attr_scan_norm : attr_scan);
  if (rc != GDN_OK) return rc;
  p.chunk_prefix = reinterpret_cast<int32_t*>(ws + kWsHeader);
  p.rec_off = pl.rec_off;
  p.carry = p.state_out ? p.state_out : (pl.n_windows > 1 ? reinterpret_cast<float*>(ws + pl.carry_off) : nullptr);
  p.win_len = pl.win_len;
  RowMaps rm;
  const long long tokens = packed ? static_cast<long long>(T) : static_cast<long long>(p.B) * T;
  if (tokens > 0) {
    if (tokens > 0x7fffff00LL) return fail(GDN_ERR_SHAPE, "too many tokens for one call");
    rc = make_rows_tmap(&rm.q, p.q, tokens, p.Hk, p.q_stride);
    if (rc == GDN_OK) rc = make_rows_tmap(&rm.k, p.k, tokens, p.Hk, p.k_stride);
    if (rc == GDN_OK) rc = make_rows_tmap(&rm.v, p.v, tokens, p.Hv, p.v_stride);
    if (rc != GDN_OK) return rc;
  }
  for (int w = 0; w < pl.n_windows; ++w) {
    rc = launch_window(p, T, w, pl.win_len, rm, st);
    if (rc != GDN_OK) return rc;
  }
  return GDN_OK;
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_chunked_fwd(const void* q, const void* k, const void* v, long long q_stride, long long k_stride,
                               long long v_stride, const float* a, const float* b, const float* A_log,
                               const float* dt_bias, const float* state_in, float* state_out, void* o,
                               const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv,
                               unsigned flags, void* stream) {
  clear_error();
  ChunkParams p;
  int rc = chunked_args(p, q, k, v, q_stride, k_stride, v_stride, a, b, A_log, dt_bias, state_in, state_out, o,
                        cu_seqlens, B, T, Hk, Hv, Dk, Dv, flags);
  if (rc != GDN_OK || B == 0) return rc;
  static bool attr[64] = {false};
  rc = set_smem_attr(reinterpret_cast<const void*>(chunked_kernel), kSmemBytes, attr);
  if (rc != GDN_OK) return rc;
  chunked_kernel<<<static_cast<unsigned>(B * Hv), kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(p);
  return cuda_status(cudaGetLastError(), "chunked kernel launch");
}

extern "C" size_t gdn_chunked_workspace_bytes(int B, int T, int Hv, int packed) {
  if (B < 0 || T < 0 || Hv <= 0) return 0;
  return workspace_bytes(B, T, Hv, packed != 0);
}

extern "C" size_t gdn_chunked_workspace_min_bytes(int B, int Hv, int has_state_out) {
  if (B < 0 || Hv <= 0) return 0;
  return workspace_min_bytes(B, Hv, has_state_out == 0);
}

extern "C" int gdn_chunked_fwd_ws(const void* q, const void* k, const void* v, long long q_stride,
                                  long long k_stride, long long v_stride, const float* a, const float* b,
                                  const float* A_log, const float* dt_bias, const float* state_in,
                                  float* state_out, void* o, const int32_t* cu_seqlens, int B, int T, int Hk,
                                  int Hv, int Dk, int Dv, unsigned flags, void* workspace,
                                  size_t workspace_size, void* stream) {
  clear_error();
  ChunkParams p;
  int rc = chunked_args(p, q, k, v, q_stride, k_stride, v_stride, a, b, A_log, dt_bias, state_in, state_out, o,
                        cu_seqlens, B, T, Hk, Hv, Dk, Dv, flags);
  if (rc != GDN_OK || B == 0) return rc;
  if (!workspace) return fail(GDN_ERR_NULL, "workspace is required (%zu bytes for one window)",
                              workspace_bytes(B, T, Hv, cu_seqlens != nullptr));
  if (!aligned(workspace, 256)) return fail(GDN_ERR_ALIGN, "workspace must be 256-byte aligned");
  const size_t sbytes = static_cast<size_t>(B) * Hv * kD * kD * 4;
  const long long total = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  const size_t obytes = static_cast<size_t>(total) * Hv * kD * ((flags & GDN_F_O_BF16) ? 2 : 4);
  if (overlap(workspace, workspace_size, state_in, sbytes) || overlap(workspace, workspace_size, state_out, sbytes) ||
      overlap(workspace, workspace_size, o, obytes))
    return fail(GDN_ERR_ALIAS, "workspace overlaps a state or o");
  if (Hv > 65535) return fail(GDN_ERR_SHAPE, "too many value heads for one launch");
  return run_split(p, T, static_cast<unsigned char*>(workspace), workspace_size, static_cast<cudaStream_t>(stream));
}

namespace gdn {
namespace {

// Shared checks and launch of the fused-norm split schedule writing to n_dst
// destinations of out_elems elements each.
int run_norm(const void* q, const void* k, const void* v, long long q_stride, long long k_stride,
             long long v_stride, const float* a, const float* b, const float* A_log, const float* dt_bias,
             const float* state_in, float* state_out, const void* z, long long z_stride, const float* gamma,
             float eps, void* const* dst, int n_dst, long long out_elems, long long out_stride, int out_head0,
             const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv, unsigned flags,
             void* workspace, size_t workspace_size, cudaStream_t stream) {
  if (flags & ~GDN_F_QK_L2NORM) return fail(GDN_ERR_FLAGS, "only GDN_F_QK_L2NORM applies (out is bf16)");
  if (n_dst < 1 || n_dst > 8 || !dst) return fail(GDN_ERR_SHAPE, "1 to 8 output destinations");
  ChunkParams p;
  int rc = chunked_args(p, q, k, v, q_stride, k_stride, v_stride, a, b, A_log, dt_bias, state_in, state_out, dst[0],
                        cu_seqlens, B, T, Hk, Hv, Dk, Dv, flags | GDN_F_O_BF16);
  if (rc != GDN_OK || B == 0) return rc;
  const long long total = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  if (total > 0 && (!z || !gamma)) return fail(GDN_ERR_NULL, "z and gamma are required");
  if (out_head0 < 0 || out_stride < (static_cast<long long>(out_head0) + Hv) * kD || z_stride < static_cast<long long>(Hv) * kD)
    return fail(GDN_ERR_SHAPE, "out_stride / out_head0 / z_stride do not fit Hv heads of 128");
  const long long used = total > 0 ? (total - 1) * out_stride + (static_cast<long long>(out_head0) + Hv) * kD : 0;
  if (out_elems < used) return fail(GDN_ERR_SHAPE, "output of %lld elements, %lld needed", out_elems, used);
  if (out_stride % 8) return fail(GDN_ERR_ALIGN, "out_stride must be a multiple of 8 elements (16 bytes)");
  for (int d = 0; d < n_dst; ++d)
    if (!dst[d] || !aligned(dst[d], 16)) return fail(GDN_ERR_ALIGN, "output %d is null or not 16-byte aligned", d);
  if (!aligned(z, 16) || z_stride % 8 || !aligned(gamma, 4) || !(eps >= 0.f))
    return fail(GDN_ERR_ALIGN, "z 16-byte aligned with z_stride a multiple of 8, gamma 4-byte aligned, eps >= 0");
  if (!workspace) return fail(GDN_ERR_NULL, "workspace is required (%zu bytes for one window)",
                              workspace_bytes(B, T, Hv, cu_seqlens != nullptr));
  if (!aligned(workspace, 256)) return fail(GDN_ERR_ALIGN, "workspace must be 256-byte aligned");
  const size_t sbytes = static_cast<size_t>(B) * Hv * kD * kD * 4;
  const size_t obytes = static_cast<size_t>(used) * 2;
  if (overlap(workspace, workspace_size, state_in, sbytes) || overlap(workspace, workspace_size, state_out, sbytes) ||
      overlap(workspace, workspace_size, dst[0], obytes) || overlap(dst[0], obytes, state_in, sbytes) ||
      overlap(dst[0], obytes, state_out, sbytes))
    return fail(GDN_ERR_ALIAS, "workspace, out and the states must not overlap");
  if (Hv > 65535) return fail(GDN_ERR_SHAPE, "too many value heads for one launch");
  p.z = static_cast<const __nv_bfloat16*>(z);
  p.z_stride = z_stride;
  p.gamma = gamma;
  p.eps = eps;
  p.out_stride = out_stride;
  p.out_head0 = out_head0;
  for (int d = 0; d < n_dst; ++d) p.dst[d] = static_cast<__nv_bfloat16*>(dst[d]);
  p.n_dst = n_dst;
  p.out_elems = out_elems;
  return run_split(p, T, static_cast<unsigned char*>(workspace), workspace_size, stream);
}

struct FlagPtrs {
  uint32_t* f[8];
};

// One thread per destination rank: after the call's scan kernels (which
// fenced their peer stores at system scope), count one more finished call
// in every rank's flag word of this rank.
__global__ void gather_signal_kernel(FlagPtrs fp, int rank, int world) {
  const int r = threadIdx.x;
  if (r < world) {
    __threadfence_system();
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(fp.f[r] + rank) : "memory");
  }
}

// Wait until every rank has signalled `expected` calls (bounded: limit_ns of
// polling by %globaltimer, then *err = 1, the device error word set, return).
__global__ void gather_wait_kernel(const uint32_t* flags, int world, uint32_t expected, int32_t* err,
                                   unsigned long long limit_ns, int* dev_err) {
  const int r = threadIdx.x;
  if (r >= world) return;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
    if (static_cast<int32_t>(v - expected) >= 0) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > limit_ns) {
      atomicExch(err, 1);
      atomicExch(dev_err, 1);
      return;
    }
    __nanosleep(200);
  }
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_chunked_norm_fwd_ws(const void* q, const void* k, const void* v, long long q_stride,
                                       long long k_stride, long long v_stride, const float* a, const float* b,
                                       const float* A_log, const float* dt_bias, const float* state_in,
                                       float* state_out, const void* z, long long z_stride, const float* gamma,
                                       float eps, void* out, long long out_stride, int out_head0,
                                       const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv,
                                       unsigned flags, void* workspace, size_t workspace_size, void* stream) {
  clear_error();
  const long long total = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  const long long used = total > 0 ? (total - 1) * out_stride + (static_cast<long long>(out_head0) + Hv) * 128 : 0;
  void* dst[1] = {out};
  return run_norm(q, k, v, q_stride, k_stride, v_stride, a, b, A_log, dt_bias, state_in, state_out, z, z_stride,
                  gamma, eps, dst, 1, used, out_stride, out_head0, cu_seqlens, B, T, Hk, Hv, Dk, Dv, flags, workspace,
                  workspace_size, static_cast<cudaStream_t>(stream));
}

extern "C" int gdn_chunked_norm_gather_ws(const void* q, const void* k, const void* v, long long q_stride,
                                          long long k_stride, long long v_stride, const float* a, const float* b,
                                          const float* A_log, const float* dt_bias, const float* state_in,
                                          float* state_out, const void* z, long long z_stride, const float* gamma,
                                          float eps, void* const* out_ranks, uint32_t* const* flag_ranks, int world,
                                          int rank, long long out_elems, long long out_stride, int out_head0,
                                          const int32_t* cu_seqlens, int B, int T, int Hk, int Hv, int Dk, int Dv,
                                          unsigned flags, void* workspace, size_t workspace_size, void* stream) {
  clear_error();
  if (world < 1 || world > 8 || rank < 0 || rank >= world || !out_ranks || !flag_ranks)
    return fail(GDN_ERR_SHAPE, "world %d, rank %d: need 1 <= world <= 8, 0 <= rank < world, pointer arrays", world,
                rank);
  FlagPtrs fp{};
  for (int r = 0; r < world; ++r) {
    if (!flag_ranks[r] || !aligned(flag_ranks[r], 4)) return fail(GDN_ERR_ALIGN, "flag word array %d", r);
    fp.f[r] = flag_ranks[r];
  }
  // this rank's own buffer first, so the output checks apply to it
  void* dst[8];
  for (int r = 0; r < world; ++r) dst[r] = out_ranks[(rank + r) % world];
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = run_norm(q, k, v, q_stride, k_stride, v_stride, a, b, A_log, dt_bias, state_in, state_out, z, z_stride,
                    gamma, eps, dst, world, out_elems, out_stride, out_head0, cu_seqlens, B, T, Hk, Hv, Dk, Dv, flags,
                    workspace, workspace_size, st);
  if (rc != GDN_OK) return rc;
  gather_signal_kernel<<<1, 32, 0, st>>>(fp, rank, world);
  return cuda_status(cudaGetLastError(), "gather signal launch");
}

extern "C" int gdn_gather_wait_timeout(const uint32_t* flags, int world, unsigned expected, unsigned limit_ms,
                                       int32_t* err_flag, void* stream) {
  clear_error();
  if (world < 1 || world > 8) return fail(GDN_ERR_SHAPE, "world %d: need 1 <= world <= 8", world);
  if (limit_ms < 1 || limit_ms > 60000) return fail(GDN_ERR_RANGE, "limit_ms %u: need 1 .. 60000", limit_ms);
  if (!flags || !err_flag) return fail(GDN_ERR_NULL, "flags and err_flag are required");
  if (!aligned(flags, 4) || !aligned(err_flag, 4)) return fail(GDN_ERR_ALIGN, "flags, err_flag 4-byte aligned");
  int* dev_err = nullptr;
  int rc = device_error_ptr(&dev_err);
  if (rc != GDN_OK) return rc;
  gather_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      flags, world, expected, err_flag, static_cast<unsigned long long>(limit_ms) * 1000000ull, dev_err);
  return cuda_status(cudaGetLastError(), "gather wait launch");
}

extern "C" int gdn_gather_wait(const uint32_t* flags, int world, unsigned expected, int32_t* err_flag, void* stream) {
  return gdn_gather_wait_timeout(flags, world, expected, 4000u, err_flag, stream);
}

// Scratch of gdn_chunked_fwd_static: a fixed device array, so that the call
// allocates nothing.  Nothing in it needs to start at zero: the prefix kernel
// writes the chunk prefix and the prep kernel every record before the scan
// kernel reads them.  One per device; overlapping calls on a device race on it.
static __device__ __align__(256) unsigned char g_chunked_static_scratch[GDN_CHUNKED_STATIC_SCRATCH_BYTES];

namespace gdn {
namespace {

// Address of g_chunked_static_scratch on the current device, looked up once per
// device (cudaGetSymbolAddress with that device current) and cached for the
// life of the process: the library must not be used across a
// cudaDeviceReset (the cached address would then be stale).
int static_scratch_ptr(unsigned char** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != GDN_OK) return rc;
  if (dev < 0 || dev >= 64) return fail(GDN_ERR_CUDA, "device ordinal %d beyond the 64 the library tracks", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* a = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&a, g_chunked_static_scratch), "cudaGetSymbolAddress(static scratch)");
    if (rc != GDN_OK) return rc;
    addr[dev] = a;
  }
  *out = static_cast<unsigned char*>(addr[dev]);
  return GDN_OK;
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_chunked_fwd_static(const void* q, const void* k, const void* v, long long q_stride,
                                      long long k_stride, long long v_stride, const float* a, const float* b,
                                      const float* A_log, const float* dt_bias, const float* state_in,
                                      float* state_out, void* o, const int32_t* cu_seqlens, int B, int T, int Hk,
                                      int Hv, int Dk, int Dv, unsigned flags, void* stream) {
  clear_error();
  ChunkParams p;
  int rc = chunked_args(p, q, k, v, q_stride, k_stride, v_stride, a, b, A_log, dt_bias, state_in, state_out, o,
                        cu_seqlens, B, T, Hk, Hv, Dk, Dv, flags);
  if (rc != GDN_OK || B == 0) return rc;
  // the call runs in one pass when its records fit the scratch, else in
  // windows of chunks (bit-identical); only a call whose smallest window
  // (one chunk of every sequence, plus the carried state without state_out)
  // does not fit is refused
  const size_t need = workspace_min_bytes(B, Hv, state_out == nullptr);
  if (need > GDN_CHUNKED_STATIC_SCRATCH_BYTES)
    return fail(GDN_ERR_SHAPE,
                "gdn_chunked_fwd_static: B=%d Hv=%d needs at least %zu bytes of scratch, more than the %llu of the "
                "static scratch; split the batch or use gdn_chunked_fwd_ws",
                B, Hv, need, static_cast<unsigned long long>(GDN_CHUNKED_STATIC_SCRATCH_BYTES));
  if (Hv > 65535) return fail(GDN_ERR_SHAPE, "too many value heads for one launch");
  unsigned char* ws = nullptr;
  rc = static_scratch_ptr(&ws);
  if (rc != GDN_OK) return rc;
  return run_split(p, T, ws, GDN_CHUNKED_STATIC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream));
}

#ifdef GDN_CHUNK_TIMING
extern "C" int gdn_debug_chunk_timing(long long* out, int reset) {
  int rc = cuda_status(cudaMemcpyFromSymbol(out, gdn::g_chunk_timing, sizeof(long long) * 32), "timing read");
  if (rc == GDN_OK && reset) {
    long long z[32] = {0};
    rc = cuda_status(cudaMemcpyToSymbol(gdn::g_chunk_timing, z, sizeof(z)), "timing reset");
  }
  return rc;
}
#endif
