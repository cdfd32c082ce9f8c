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
//   W^T    = K^T diag(beta g r_k) T^-T           (MMA)
//   U^T    = U0^T - R W^T                        (MMA, R from tensor memory)
//   M[i,j] = r_qi r_kj e^{Gam_i-Gam_j} P[i,j]                  (j <= i)
//   y^T    = R (diag(g r_q) Q)^T + U^T M^T       (MMAs)      -> o
//   R     <- g_last R + U^T diag(e^{Gam_last-Gam} r_k) K       (MMA)
//
// which is the reference's y = M U0 + Qeff S, U = U0 - Kt S,
// S <- cumg_last S + k^T (ratio U) regrouped so that every product has
// M = 128 rows (Dv, Dk or the 128 rows of [K; Q]) and the state never leaves
// the chip between chunks.  One CTA (4 warps, thread t <-> TMEM lane t) owns
// one (sequence, value head); the 512 tensor-memory columns hold
//   [0,128)   R rounded to tf32 (A operand of U and y)
//   [128,256) R in full fp32, also the accumulator of the state update
//   [256,320) G (lanes 0-63) and P (lanes 64-127)
//   [320,384) W^T    [384,448) U^T    [448,512) y^T
// All MMAs are kind::tf32 with fp32 accumulation: the bf16 inputs are exact
// in tf32, derived operands are rounded to nearest tf32 once.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {

#ifdef GDN_CHUNK_TIMING
__device__ long long g_chunk_timing[16];
#define GDN_TICK(slot)                                                          \
  do {                                                                          \
    if (blockIdx.x == 0 && threadIdx.x == 0) {                                  \
      const long long now_ = clock64();                                         \
      g_chunk_timing[slot] += now_ - tick_;                                     \
      tick_ = now_;                                                             \
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

// shared memory map, bytes; tensor-core operands in the K-major no-swizzle
// layout (LBO 128 B), written row-wise so that a warp's stores hit distinct banks
constexpr uint32_t kSbo128 = (kD * 4 / 16) * 128;   // 8-row group stride of 128-wide fp32 rows
constexpr uint32_t kSbo64 = (kC * 4 / 16) * 128;    // ... of 64-wide fp32 rows
constexpr int kPad = kC + 1;                        // row stride of the plain solve arrays
constexpr uint32_t kOffKQ = 0;                      // [K; Q] rows            128 x 128 (64 KiB)
constexpr uint32_t kOffKt = kOffKQ + 128 * kD * 4;  // K^T, scaled            128 x 64  (32 KiB)
constexpr uint32_t kOffVt = kOffKt + kD * kC * 4;   // V^T diag(beta), U^T    128 x 64  (32 KiB)
constexpr uint32_t kOffTi = kOffVt + kD * kC * 4;   // T^-1                    64 x 64  (16 KiB)
constexpr uint32_t kOffM = kOffTi + kC * kC * 4;    // M (must follow T^-1)    64 x 64  (16 KiB)
constexpr uint32_t kOffW = kOffM + kC * kC * 4;     // W rows 64 x 128 (32 KiB); X during the solve
constexpr uint32_t kOffA = kOffW + kC * kD * 4;     // A, plain, row stride 65
constexpr uint32_t kOffY = kOffA + kC * kPad * 4;   // solve temporaries 3 x 16 x 16
constexpr uint32_t kOffSc = kOffY + 3 * 256 * 4;    // per-token scalars, 8 x 64
constexpr uint32_t kOffBar = kOffSc + 8 * kC * 4;   // mbarrier, TMEM base
constexpr uint32_t kSmemBytes = kOffBar + 64;

constexpr uint32_t kTmemCols = 512;
// [0,128) R (tf32), [128,256) R (fp32 master, state-update accumulator),
// [256,320) G|P during (a); [256,384) W (lanes 0-63) during (c);
// [384,448) U^T; [448,512) y^T
constexpr uint32_t kColR = 0, kColDR = 128, kColGP = 256, kColW = 256, kColU = 384, kColY = 448;

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

__global__ void __launch_bounds__(kThreads, 1) chunked_kernel(const ChunkParams p) {
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* sKQ = sm + kOffKQ;
  unsigned char* sKt = sm + kOffKt;
  unsigned char* sVt = sm + kOffVt;   // V^T diag(beta), later U^T
  unsigned char* sTi = sm + kOffTi;
  unsigned char* sM = sm + kOffM;
  unsigned char* sW = sm + kOffW;
  float* sX = reinterpret_cast<float*>(sm + kOffW);   // T^-1 in plain form while solving
  float* sA = reinterpret_cast<float*>(sm + kOffA);
  float* sY = reinterpret_cast<float*>(sm + kOffY);
  float* sc = reinterpret_cast<float*>(sm + kOffSc);
  float* s_pre = sc;            // warp-local prefix of log-decay
  float* s_gam = sc + 64;       // Gam_i
  float* s_g = sc + 128;        // exp(Gam_i)
  float* s_ratio = sc + 192;    // exp(Gam_last - Gam_i)
  float* s_beta = sc + 256;
  float* s_rk = sc + 320;
  float* s_rq = sc + 384;
  float* s_misc = sc + 448;     // [0] g_last
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kOffBar + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int quarter = warp & 3;       // TMEM lanes 32*quarter ..
  const int half = warp >> 2;         // column half of the epilogues
  const int row = quarter * 32 + lane;  // TMEM lane of this thread
  const int bh = blockIdx.x;
  const int b = bh / p.Hv;
  const int h = bh - b * p.Hv;
  const int kh = h / (p.Hv / p.Hk);
  long long s0, s1;
  if (p.cu) {
    s0 = p.cu[b];
    s1 = p.cu[b + 1];
    if (s1 < s0) s1 = s0;
  } else {
    s0 = static_cast<long long>(b) * p.T;
    s1 = s0 + p.T;
  }
  const int n_chunks = static_cast<int>((s1 - s0 + kC - 1) / kC);
  const bool l2 = (p.flags & GDN_F_QK_L2NORM) != 0;
  const float A_h = expf(__ldg(p.A_log + h));
  const float dtb = __ldg(p.dt_bias + h);
  const float log_clip = logf(1e-6f);          // log(clip(alpha, 1e-6, 1)), python/qwen35.py:400
  const float qscale = rsqrtf(static_cast<float>(kD));

  if (warp == 0) {
    tc::tmem_alloc(tslot, kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    ptx::mbar_init(bar, 1);
    ptx::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tb = *tslot;
  const uint32_t my = static_cast<uint32_t>(quarter * 32) << 16;      // this warp's lane quarter
  const uint32_t tR = tb + kColR + my, tDR = tb + kColDR + my, tGP = tb + kColGP + my;
  const uint32_t tW = tb + kColW + my, tU = tb + kColU + my, tY = tb + kColY + my;

  // initial state: row dv = row, columns [64*half, 64*half+64), into the fp32 master
  {
    const float* src = p.state_in ? p.state_in + (static_cast<size_t>(bh) * kD + row) * kD + half * 64 : nullptr;
    for (int c = 0; c < 64; c += 16) {
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 f = src ? *reinterpret_cast<const float4*>(src + c + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
      }
      tc::tmem_st16(tDR + half * 64 + c, v);
    }
    tc::tmem_st_wait();
  }

  uint32_t phase = 0;
  bool failed = false;
#ifdef GDN_CHUNK_TIMING
  long long tick_ = clock64();
#endif
  // one warp polls the MMA barrier, the others wait at the CTA barrier
  auto mma_wait = [&]() -> bool {
    bool ok = true;
    if (warp == 0) ok = ptx::mbar_wait(bar, phase);
    phase ^= 1u;
    const bool all_ok = !__syncthreads_or(!ok);
    tc::fence_after_sync();
    return all_ok;
  };
  auto desc = [](const unsigned char* base, uint32_t byte_off, uint32_t sbo) {
    return tc::smem_desc(ptx::smem_u32(base) + byte_off, 128, sbo);
  };

  for (int ch = 0; ch < n_chunks; ++ch) {
    const long long t0 = s0 + static_cast<long long>(ch) * kC;
    const int nvalid = static_cast<int>((s1 - t0) < kC ? (s1 - t0) : kC);

    // ---- per-token gates and the in-chunk decay prefix ----------------------
    if (tid < kC) {
      float lg = 0.f, beta = 0.f;
      if (tid < nvalid) {
        const size_t gi = static_cast<size_t>(t0 + tid) * p.Hv + h;
        lg = fmaxf(-(A_h * softplus_f(__ldg(p.a + gi) + dtb)), log_clip);
        beta = 1.f / (1.f + expf(-__ldg(p.b + gi)));
      }
      float x = lg;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
      }
      s_pre[tid] = x;
      s_beta[tid] = beta;
    }
    __syncthreads();
    if (tid < kC) s_gam[tid] = s_pre[tid] + (tid >= 32 ? s_pre[31] : 0.f);
    __syncthreads();
    if (tid < kC) {
      const float gl = s_gam[kC - 1];
      s_g[tid] = expf(s_gam[tid]);
      s_ratio[tid] = expf(gl - s_gam[tid]);
      if (tid == 0) s_misc[0] = expf(gl);
    }
    GDN_TICK(0);

    // ---- rows of K and Q (thread -> token i, 32-dim quarter qd) and their norms
    {
      const int i = tid >> 2;
      const int qd = tid & 3;
      const bool valid = i < nvalid;
      const long long tok = valid ? t0 + i : s0;
      float f[32];
      load32(p.k + tok * p.k_stride + kh * kD + qd * 32, valid, f);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 32; ++e) ss += f[e] * f[e];
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
#pragma unroll
      for (int e = 0; e < 32; e += 4)
        *reinterpret_cast<float4*>(at(sKQ, i, qd * 32 + e, kSbo128)) = make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
      if (qd == 0) s_rk[i] = l2 ? rsqrtf(ss + 1e-6f) : 1.f;
      load32(p.q + tok * p.q_stride + kh * kD + qd * 32, valid, f);
      ss = 0.f;
#pragma unroll
      for (int e = 0; e < 32; ++e) ss += f[e] * f[e];
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
#pragma unroll
      for (int e = 0; e < 32; e += 4)
        *reinterpret_cast<float4*>(at(sKQ, kC + i, qd * 32 + e, kSbo128)) =
            make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
      if (qd == 0) s_rq[i] = l2 ? rsqrtf(ss + 1e-6f) * qscale : 1.f;
    }
    __syncthreads();
    GDN_TICK(1);

    // ---- columns: K^T diag(beta g r_k) and V^T diag(beta), read column-wise
    //      from global two columns per 4-byte load (threads 0-63: K columns
    //      2p, 2p+1 for tokens of half th; threads 128-191 likewise for V),
    //      stored row-wise
    {
      const int pr = tid & 63;                   // column pair
      const int th = (tid >> 6) & 1;             // token half
      const bool is_k = tid < 128;
      const int c = 2 * pr;
      const long long stride = is_k ? p.k_stride : p.v_stride;
      const __nv_bfloat16* src = (is_k ? p.k + kh * kD : p.v + h * kD) + c + (t0 + th * 32) * stride;
      unsigned char* dst = is_k ? sKt : sVt;
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
          const float sc_ = is_k ? s_beta[jj] * s_g[jj] * s_rk[jj] : s_beta[jj];
          const float2 f = __bfloat1622float2(raw[j + e]);
          x0[e] = tc::to_tf32(f.x * sc_);
          x1[e] = tc::to_tf32(f.y * sc_);
        }
        *reinterpret_cast<float4*>(at(dst, c, th * 32 + j, kSbo64)) = make_float4(x0[0], x0[1], x0[2], x0[3]);
        *reinterpret_cast<float4*>(at(dst, c + 1, th * 32 + j, kSbo64)) = make_float4(x1[0], x1[1], x1[2], x1[3]);
      }
    }
    ptx::fence_proxy_async_smem();
    GDN_TICK(2);

    // ---- state operand for this chunk: tR = tf32(R), tDR = g_last * R ---------
    {
      const float gl = s_misc[0];
      for (int c = 0; c < 64; c += 16) {
        float v[16], r[16];
        tc::tmem_ld16(tDR + half * 64 + c, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          r[i] = tc::to_tf32(v[i]);
          v[i] *= gl;
        }
        tc::tmem_st16(tR + half * 64 + c, r);
        tc::tmem_st16(tDR + half * 64 + c, v);
      }
      tc::tmem_st_wait();
    }
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(3);

    // ---- (a)  [K; Q] K^T -> G (lanes 0-63), P (lanes 64-127) --------------------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t id = tc::instr_desc(tc::kTF32, 128, kC);
      for (int j = 0; j < kD / 8; ++j)
        tc::mma_ss<tc::kTF32>(tb + kColGP, desc(sKQ, j * 256, kSbo128), desc(sKQ, j * 256, kSbo128), id, j > 0);
      tc::mma_commit(bar);
    }
    if (!mma_wait()) {
      failed = true;
      break;
    }
    GDN_TICK(4);

    // ---- A (strictly lower, plain), M (lower), Q rows rescaled by g r_q --------
    {
      float gp[32];
      tmem_ld<32>(tGP + half * 32, gp);
      if (quarter < 2) {
        const int i = row;
        const float fi = s_beta[i] * s_rk[i];
        const float gi = s_gam[i];
        float* Ar = sA + i * kPad + half * 32;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = half * 32 + e;
          Ar[e] = (j < i) ? fi * s_rk[j] * expf(gi - s_gam[j]) * gp[e] : 0.f;
        }
      } else {
        const int i = row - kC;
        const float fi = s_rq[i];
        const float gi = s_gam[i];
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          float m[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = half * 32 + e + u;
            m[u] = (j <= i) ? tc::to_tf32(fi * s_rk[j] * expf(gi - s_gam[j]) * gp[e + u]) : 0.f;
          }
          *reinterpret_cast<float4*>(at(sM, i, half * 32 + e, kSbo64)) = make_float4(m[0], m[1], m[2], m[3]);
        }
        const float sq = s_g[i] * s_rq[i];
        for (int c = half * 64; c < half * 64 + 64; c += 4) {
          float4* qp = reinterpret_cast<float4*>(at(sKQ, kC + i, c, kSbo128));
          float4 v = *qp;
          v.x = tc::to_tf32(v.x * sq);
          v.y = tc::to_tf32(v.y * sq);
          v.z = tc::to_tf32(v.z * sq);
          v.w = tc::to_tf32(v.w * sq);
          *qp = v;
        }
      }
    }
    __syncthreads();
    GDN_TICK(5);

    // ---- T^-1 = (I + A)^-1: 16x16 diagonal blocks by substitution, then block
    //      diagonals X_ij = -X_ii sum_{k=j}^{i-1} A_ik X_kj; plain arrays, row stride 65
    if (tid < kC) {
      const int blk = tid >> 4, c = tid & 15;
      const float* Ab = sA + (blk * 16) * kPad + blk * 16;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) col[r] = (r == c) ? 1.f : 0.f;
#pragma unroll
      for (int r = 1; r < 16; ++r) {
        if (r > c) {
          float s = 0.f;
#pragma unroll
          for (int m = 0; m < r; ++m)
            if (m >= c) s += Ab[r * kPad + m] * col[m];
          col[r] = -s;
        }
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) sX[(blk * 16 + r) * kPad + blk * 16 + c] = col[r];
    }
    __syncthreads();
    for (int d = 1; d < 4; ++d) {
      const int nt = 4 - d;
      for (int e = tid; e < nt * 256; e += kThreads) {
        const int t = e >> 8, r = (e >> 4) & 15, c = e & 15;
        const int bj = t, bi = t + d;
        const float* Ar = sA + (bi * 16 + r) * kPad;
        float y = 0.f;
        for (int kb = bj; kb < bi; ++kb) {
#pragma unroll
          for (int m = 0; m < 16; ++m) y += Ar[kb * 16 + m] * sX[(kb * 16 + m) * kPad + bj * 16 + c];
        }
        sY[e] = y;
      }
      __syncthreads();
      for (int e = tid; e < nt * 256; e += kThreads) {
        const int t = e >> 8, r = (e >> 4) & 15, c = e & 15;
        const int bj = t, bi = t + d;
        const float* Xr = sX + (bi * 16 + r) * kPad + bi * 16;
        float x = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m) x += Xr[m] * sY[(t << 8) + (m << 4) + c];
        sX[(bi * 16 + r) * kPad + bj * 16 + c] = -x;
      }
      __syncthreads();
    }
    // T^-1 into the operand layout, rounded to tf32, zeros above the diagonal blocks
    {
      const int i = tid >> 2;
      const int c0 = (tid & 3) * 16;
#pragma unroll
      for (int c = c0; c < c0 + 16; c += 4) {
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = ((c + u) >> 4) <= (i >> 4) ? tc::to_tf32(sX[i * kPad + c + u]) : 0.f;
        *reinterpret_cast<float4*>(at(sTi, i, c, kSbo64)) = make_float4(x[0], x[1], x[2], x[3]);
      }
    }
    ptx::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(6);

    // ---- (b) U0^T = V^T diag(beta) T^-T;  (c) W = [T^-1; *] (K^T diag(beta g r_k))^T
    //      (M = 128: rows 64-127 of A read the M buffer and are discarded)
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t id64 = tc::instr_desc(tc::kTF32, 128, kC);
      const uint32_t id128 = tc::instr_desc(tc::kTF32, 128, kD);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(tb + kColU, desc(sVt, j * 256, kSbo64), desc(sTi, j * 256, kSbo64), id64, j > 0);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(tb + kColW, desc(sTi, j * 256, kSbo64), desc(sKt, j * 256, kSbo64), id128, j > 0);
      tc::mma_commit(bar);
    }
    if (!mma_wait()) {
      failed = true;
      break;
    }
    GDN_TICK(7);

    // ---- W rows into the operand buffer (warps on lanes 0-63); K^T rescaled
    //      by ratio r_k for the state update (warps on lanes 64-127)
    if (quarter < 2) {
      float w[64];
      tmem_ld<64>(tW + half * 64, w);
      const int i = row;
#pragma unroll
      for (int e = 0; e < 64; e += 4)
        *reinterpret_cast<float4*>(at(sW, i, half * 64 + e, kSbo128)) =
            make_float4(tc::to_tf32(w[e]), tc::to_tf32(w[e + 1]), tc::to_tf32(w[e + 2]), tc::to_tf32(w[e + 3]));
    } else {
      const int lt = (tid & 63) + 64 * half;     // 0..127 over the four warps on lanes 64-127
      const int pr = lt & 63;
      const int th = lt >> 6;
      const int c = 2 * pr;
      const __nv_bfloat16* src = p.k + kh * kD + c + (t0 + th * 32) * p.k_stride;
      const int nv = nvalid - th * 32;
      __nv_bfloat162 raw[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        raw[j] = j < nv ? *reinterpret_cast<const __nv_bfloat162*>(src + j * p.k_stride) : __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float x0[4], x1[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jj = th * 32 + j + e;
          const float sc_ = s_ratio[jj] * s_rk[jj];
          const float2 f = __bfloat1622float2(raw[j + e]);
          x0[e] = tc::to_tf32(f.x * sc_);
          x1[e] = tc::to_tf32(f.y * sc_);
        }
        *reinterpret_cast<float4*>(at(sKt, c, th * 32 + j, kSbo64)) = make_float4(x0[0], x0[1], x0[2], x0[3]);
        *reinterpret_cast<float4*>(at(sKt, c + 1, th * 32 + j, kSbo64)) = make_float4(x1[0], x1[1], x1[2], x1[3]);
      }
    }
    ptx::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(8);

    // ---- (d) U^T = U0^T - R W^T ----------------------------------------------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t id = tc::instr_desc(tc::kTF32, 128, kC, /*neg_a=*/true);
      for (int j = 0; j < kD / 8; ++j) tc::mma_ts_tf32(tb + kColU, tb + kColR + j * 8, desc(sW, j * 256, kSbo128), id, 1);
      tc::mma_commit(bar);
    }
    if (!mma_wait()) {
      failed = true;
      break;
    }
    GDN_TICK(9);

    // ---- U^T rows into shared memory (the V^T buffer) -------------------------
    {
      float u[32];
      tmem_ld<32>(tU + half * 32, u);
#pragma unroll
      for (int e = 0; e < 32; e += 4)
        *reinterpret_cast<float4*>(at(sVt, row, half * 32 + e, kSbo64)) =
            make_float4(tc::to_tf32(u[e]), tc::to_tf32(u[e + 1]), tc::to_tf32(u[e + 2]), tc::to_tf32(u[e + 3]));
    }
    ptx::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(10);

    // ---- (e) y^T = R Qs^T + U^T M^T,  (f) R += U^T diag(ratio r_k) K ---------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t id64 = tc::instr_desc(tc::kTF32, 128, kC);
      const uint32_t id128 = tc::instr_desc(tc::kTF32, 128, kD);
      for (int j = 0; j < kD / 8; ++j)
        tc::mma_ts_tf32(tb + kColY, tb + kColR + j * 8, desc(sKQ, 8 * kSbo128 + j * 256, kSbo128), id64, j > 0);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(tb + kColY, desc(sVt, j * 256, kSbo64), desc(sM, j * 256, kSbo64), id64, 1);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(tb + kColDR, desc(sVt, j * 256, kSbo64), desc(sKt, j * 256, kSbo64), id128, 1);
      tc::mma_commit(bar);
    }
    if (!mma_wait()) {
      failed = true;
      break;
    }
    GDN_TICK(11);

    // ---- o rows of the chunk: thread -> (dv = row, tokens of its half) --------
    {
      float y[32];
      tmem_ld<32>(tY + half * 32, y);
      const size_t orow = static_cast<size_t>(p.Hv) * kD;
      const size_t base = (static_cast<size_t>(t0 + half * 32) * p.Hv + h) * kD + row;
      const int nv = nvalid - half * 32;
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
    tc::fence_before_sync();
    __syncthreads();
    GDN_TICK(12);
  }

  if (failed) {
    if (tid == 0) atomicExch(p.err, 1);
    ptx::mbar_wait(bar, phase);      // one more bounded chance for an MMA in flight
  } else if (p.state_out) {
    float* dst = p.state_out + (static_cast<size_t>(bh) * kD + row) * kD + half * 64;
    for (int c = 0; c < 64; c += 16) {
      float v[16];
      tc::tmem_ld16(tDR + half * 64 + c, v);
      tc::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(dst + c + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tb, kTmemCols);
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
  if (flags & ~(GDN_F_O_BF16 | GDN_F_QK_L2NORM)) return fail(GDN_ERR_FLAGS, "unknown flag bits 0x%x", flags);
  if (B < 0 || T < 0 || Hk <= 0 || Hv <= 0) return fail(GDN_ERR_SHAPE, "bad sizes B=%d T=%d Hk=%d Hv=%d", B, T, Hk, Hv);
  if (Dk != kD || Dv != kD) return fail(GDN_ERR_SHAPE, "Dk=%d Dv=%d: only 128x128 heads are built", Dk, Dv);
  if (Hv % Hk) return fail(GDN_ERR_SHAPE, "Hv=%d is not a multiple of Hk=%d", Hv, Hk);
  if (static_cast<long long>(B) * Hv >= (1LL << 31)) return fail(GDN_ERR_SHAPE, "B*Hv too large");
  if (B == 0) return GDN_OK;
  const long long total = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  if (total > 0 && (!q || !k || !v || !a || !b || !o)) return fail(GDN_ERR_NULL, "q, k, v, a, b and o are required");
  if (!A_log || !dt_bias) return fail(GDN_ERR_NULL, "A_log and dt_bias are required");
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
  int* err = nullptr;
  int rc = device_error_ptr(&err);
  if (rc != GDN_OK) return rc;
  {
    static bool attr_set[64] = {false};
    static std::mutex mu;
    int dev = 0;
    rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc != GDN_OK) return rc;
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev & 63]) {
      rc = cuda_status(cudaFuncSetAttribute(chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(kSmemBytes)),
                       "chunked kernel smem attribute");
      if (rc != GDN_OK) return rc;
      attr_set[dev & 63] = true;
    }
  }
  ChunkParams p{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                static_cast<const __nv_bfloat16*>(v), q_stride, k_stride, v_stride, a, b, A_log, dt_bias,
                state_in, state_out, o, cu_seqlens, B, cu_seqlens ? 0 : T, Hk, Hv, flags, err};
  chunked_kernel<<<static_cast<unsigned>(B * Hv), kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(p);
  return cuda_status(cudaGetLastError(), "chunked kernel launch");
}

#ifdef GDN_CHUNK_TIMING
extern "C" int gdn_debug_chunk_timing(long long* out, int reset) {
  int rc = cuda_status(cudaMemcpyFromSymbol(out, gdn::g_chunk_timing, sizeof(long long) * 16), "timing read");
  if (rc == GDN_OK && reset) {
    long long z[16] = {0};
    rc = cuda_status(cudaMemcpyToSymbol(gdn::g_chunk_timing, z, sizeof(z)), "timing reset");
  }
  return rc;
}
#endif
