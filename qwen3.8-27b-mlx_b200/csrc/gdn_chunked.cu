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
namespace {

constexpr int kC = 64;          // tokens per chunk (python/qwen35.py:365)
constexpr int kThreads = 128;

// shared memory map, bytes; operands in the K-major no-swizzle layout
constexpr uint32_t kSbo128 = (kD * 4 / 16) * 128;   // 8-row group stride of 128-wide fp32 rows
constexpr uint32_t kSbo64 = (kC * 4 / 16) * 128;    // ... of 64-wide fp32 rows
constexpr uint32_t kOffKQ = 0;                      // [K; Q]   128 x 128  (64 KiB)
constexpr uint32_t kOffKt = kOffKQ + 128 * kD * 4;  // K^T      128 x 64   (32 KiB)
constexpr uint32_t kOffVt = kOffKt + kD * kC * 4;   // V^T, U^T 128 x 64   (32 KiB)
constexpr uint32_t kOffTi = kOffVt + kD * kC * 4;   // T^-1      64 x 64   (16 KiB)
constexpr uint32_t kOffM = kOffTi + kC * kC * 4;    // M         64 x 64   (16 KiB)
constexpr uint32_t kOffW = kOffM + kC * kC * 4;     // W         64 x 128  (32 KiB)
constexpr uint32_t kOffA = kOffW + kC * kD * 4;     // A, plain row-major 64 x 64 (16 KiB)
constexpr uint32_t kOffY = kOffA + kC * kC * 4;     // solve temporaries 3 x 16 x 16
constexpr uint32_t kOffSc = kOffY + 3 * 256 * 4;    // per-token scalars, 8 x 64
constexpr uint32_t kOffBar = kOffSc + 8 * kC * 4;   // mbarrier, TMEM base
constexpr uint32_t kSmemBytes = kOffBar + 64;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColR = 0, kColDR = 128, kColGP = 256, kColW = 320, kColU = 384, kColY = 448;

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

// 64 bf16 starting at p (16-byte aligned) -> fp32
__device__ __forceinline__ void load64(const __nv_bfloat16* p, bool valid, float (&f)[64]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
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

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  float t[16];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
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
  const uint32_t tR = tb + kColR, tDR = tb + kColDR, tGP = tb + kColGP;
  const uint32_t tW = tb + kColW, tU = tb + kColU, tY = tb + kColY;
  const uint32_t my = static_cast<uint32_t>(warp * 32) << 16;     // this warp's lane quarter

  // initial state row dv = tid into the fp32 master
  {
    const float* src = p.state_in ? p.state_in + (static_cast<size_t>(bh) * kD + tid) * kD : nullptr;
    for (int c = 0; c < kD; c += 16) {
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 f = src ? *reinterpret_cast<const float4*>(src + c + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
      }
      tc::tmem_st16(tDR + my + c, v);
    }
    tc::tmem_st_wait();
  }

  uint32_t phase = 0;
  bool failed = false;
  auto mma_wait = [&]() -> bool {
    const bool ok = ptx::mbar_wait(bar, phase);
    phase ^= 1u;
    tc::fence_after_sync();
    return !__syncthreads_or(!ok);
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
    __syncthreads();

    // ---- stage K, Q, V of the chunk: thread -> (token i, half hf of 64 dims) --
    {
      const int i = tid >> 1;
      const int hf = tid & 1;
      const bool valid = i < nvalid;
      const long long tok = t0 + i;
      float f[64];
      // K: raw rows of [K; Q], and K^T diag(beta g r_k)
      load64(p.k + (valid ? tok : s0) * p.k_stride + kh * kD + hf * 64, valid, f);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 64; ++e) ss += f[e] * f[e];
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float rk = l2 ? rsqrtf(ss + 1e-6f) : 1.f;
#pragma unroll
      for (int e = 0; e < 64; e += 4)
        *reinterpret_cast<float4*>(at(sKQ, i, hf * 64 + e, kSbo128)) = make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
      const float sk = s_beta[i] * s_g[i] * rk;
#pragma unroll
      for (int e = 0; e < 64; ++e) *at(sKt, hf * 64 + e, i, kSbo64) = tc::to_tf32(f[e] * sk);
      // Q: raw rows (rescaled by g r_q after the G/P product)
      load64(p.q + (valid ? tok : s0) * p.q_stride + kh * kD + hf * 64, valid, f);
      ss = 0.f;
#pragma unroll
      for (int e = 0; e < 64; ++e) ss += f[e] * f[e];
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float rq = l2 ? rsqrtf(ss + 1e-6f) * qscale : 1.f;
#pragma unroll
      for (int e = 0; e < 64; e += 4)
        *reinterpret_cast<float4*>(at(sKQ, kC + i, hf * 64 + e, kSbo128)) =
            make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
      // V^T diag(beta)
      load64(p.v + (valid ? tok : s0) * p.v_stride + h * kD + hf * 64, valid, f);
      const float bv = s_beta[i];
#pragma unroll
      for (int e = 0; e < 64; ++e) *at(sVt, hf * 64 + e, i, kSbo64) = tc::to_tf32(f[e] * bv);
      if (hf == 0) {
        s_rk[i] = rk;
        s_rq[i] = rq;
      }
    }
    ptx::fence_proxy_async_smem();

    // ---- state operand for this chunk: tR = tf32(R), tDR = g_last * R ---------
    {
      const float gl = s_misc[0];
      for (int c = 0; c < kD; c += 16) {
        float v[16], r[16];
        tc::tmem_ld16(tDR + my + c, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          r[i] = tc::to_tf32(v[i]);
          v[i] *= gl;
        }
        tc::tmem_st16(tR + my + c, r);
        tc::tmem_st16(tDR + my + c, v);
      }
      tc::tmem_st_wait();
    }
    tc::fence_before_sync();
    __syncthreads();

    // ---- (a)  [K; Q] K^T -> G, P ----------------------------------------------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t id = tc::instr_desc(tc::kTF32, 128, kC);
      for (int j = 0; j < kD / 8; ++j)
        tc::mma_ss<tc::kTF32>(tGP, desc(sKQ, j * 256, kSbo128), desc(sKQ, j * 256, kSbo128), id, j > 0);
      tc::mma_commit(bar);
    }
    if (!mma_wait()) {
      failed = true;
      break;
    }

    // ---- A (strictly lower) and M (lower), Q rows rescaled -----------------
    {
      float row[64];
      tmem_ld64(tGP + my, row);
      if (warp < 2) {
        const int i = tid;
        const float fi = s_beta[i] * s_rk[i];
        const float gi = s_gam[i];
        float* Ar = sA + i * kC;
#pragma unroll
        for (int j = 0; j < kC; ++j) Ar[j] = (j < i) ? fi * s_rk[j] * expf(gi - s_gam[j]) * row[j] : 0.f;
      } else {
        const int i = tid - kC;
        const float fi = s_rq[i];
        const float gi = s_gam[i];
#pragma unroll
        for (int j = 0; j < kC; j += 4) {
          float m[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            m[e] = (j + e <= i) ? tc::to_tf32(fi * s_rk[j + e] * expf(gi - s_gam[j + e]) * row[j + e]) : 0.f;
          *reinterpret_cast<float4*>(at(sM, i, j, kSbo64)) = make_float4(m[0], m[1], m[2], m[3]);
        }
        const float sq = s_g[i] * s_rq[i];
        for (int c = 0; c < kD; c += 4) {
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
    // zero T^-1 (its upper blocks stay zero)
    for (int e = tid; e < kC * kC; e += kThreads) *at(sTi, e >> 6, e & 63, kSbo64) = 0.f;
    __syncthreads();

    // ---- T^-1 = (I + A)^-1: 16x16 diagonal blocks, then block diagonals ------
    if (tid < kC) {
      const int blk = tid >> 4, c = tid & 15;
      const float* Ab = sA + (blk * 16) * kC + blk * 16;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) col[r] = (r == c) ? 1.f : 0.f;
#pragma unroll
      for (int r = 1; r < 16; ++r) {
        if (r > c) {
          float s = 0.f;
#pragma unroll
          for (int m = 0; m < r; ++m)
            if (m >= c) s += Ab[r * kC + m] * col[m];
          col[r] = -s;
        }
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) *at(sTi, blk * 16 + r, blk * 16 + c, kSbo64) = col[r];
    }
    __syncthreads();
    for (int d = 1; d < 4; ++d) {
      const int nt = 4 - d;
      for (int e = tid; e < nt * 256; e += kThreads) {
        const int t = e >> 8, r = (e >> 4) & 15, c = e & 15;
        const int bj = t, bi = t + d;
        float y = 0.f;
        for (int kb = bj; kb < bi; ++kb) {
#pragma unroll
          for (int m = 0; m < 16; ++m) y += sA[(bi * 16 + r) * kC + kb * 16 + m] * *at(sTi, kb * 16 + m, bj * 16 + c, kSbo64);
        }
        sY[e] = y;
      }
      __syncthreads();
      for (int e = tid; e < nt * 256; e += kThreads) {
        const int t = e >> 8, r = (e >> 4) & 15, c = e & 15;
        const int bj = t, bi = t + d;
        float x = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m) x += *at(sTi, bi * 16 + r, bi * 16 + m, kSbo64) * sY[(t << 8) + (m << 4) + c];
        *at(sTi, bi * 16 + r, bj * 16 + c, kSbo64) = -x;
      }
      __syncthreads();
    }
    for (int e = tid; e < kC * kC; e += kThreads) {
      float* x = at(sTi, e >> 6, e & 63, kSbo64);
      *x = tc::to_tf32(*x);
    }
    ptx::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();

    // ---- (b) U0^T = V^T diag(beta) T^-T,  (c) W^T = K^T diag(beta g r_k) T^-T --
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t id = tc::instr_desc(tc::kTF32, 128, kC);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(tU, desc(sVt, j * 256, kSbo64), desc(sTi, j * 256, kSbo64), id, j > 0);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(tW, desc(sKt, j * 256, kSbo64), desc(sTi, j * 256, kSbo64), id, j > 0);
      tc::mma_commit(bar);
    }
    if (!mma_wait()) {
      failed = true;
      break;
    }

    // ---- W (row-major operand), K^T rescaled for the state update -----------
    {
      float w[64];
      tmem_ld64(tW + my, w);
      const int dk = tid;
#pragma unroll
      for (int i = 0; i < kC; ++i) *at(sW, i, dk, kSbo128) = tc::to_tf32(w[i]);
#pragma unroll
      for (int j = 0; j < kC; j += 4) {
        float kk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) kk[e] = tc::to_tf32(*at(sKQ, j + e, dk, kSbo128) * s_ratio[j + e] * s_rk[j + e]);
        *reinterpret_cast<float4*>(at(sKt, dk, j, kSbo64)) = make_float4(kk[0], kk[1], kk[2], kk[3]);
      }
    }
    ptx::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();

    // ---- (d) U^T = U0^T - R W^T ----------------------------------------------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t id = tc::instr_desc(tc::kTF32, 128, kC, /*neg_a=*/true);
      for (int j = 0; j < kD / 8; ++j) tc::mma_ts_tf32(tU, tR + j * 8, desc(sW, j * 256, kSbo128), id, 1);
      tc::mma_commit(bar);
    }
    if (!mma_wait()) {
      failed = true;
      break;
    }

    // ---- U^T into shared memory (the V^T buffer) ------------------------------
    {
      float u[64];
      tmem_ld64(tU + my, u);
      const int dv = tid;
#pragma unroll
      for (int i = 0; i < kC; i += 4)
        *reinterpret_cast<float4*>(at(sVt, dv, i, kSbo64)) =
            make_float4(tc::to_tf32(u[i]), tc::to_tf32(u[i + 1]), tc::to_tf32(u[i + 2]), tc::to_tf32(u[i + 3]));
    }
    ptx::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();

    // ---- (e) y^T = R Qs^T + U^T M^T,  (f) R += U^T diag(ratio r_k) K ---------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t id64 = tc::instr_desc(tc::kTF32, 128, kC);
      const uint32_t id128 = tc::instr_desc(tc::kTF32, 128, kD);
      for (int j = 0; j < kD / 8; ++j)
        tc::mma_ts_tf32(tY, tR + j * 8, desc(sKQ, 8 * kSbo128 + j * 256, kSbo128), id64, j > 0);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(tY, desc(sVt, j * 256, kSbo64), desc(sM, j * 256, kSbo64), id64, 1);
      for (int j = 0; j < kC / 8; ++j)
        tc::mma_ss<tc::kTF32>(tDR, desc(sVt, j * 256, kSbo64), desc(sKt, j * 256, kSbo64), id128, 1);
      tc::mma_commit(bar);
    }
    if (!mma_wait()) {
      failed = true;
      break;
    }

    // ---- o rows of the chunk -------------------------------------------------
    {
      float y[64];
      tmem_ld64(tY + my, y);
      const int dv = tid;
      if (p.flags & GDN_F_O_BF16) {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.o);
#pragma unroll
        for (int i = 0; i < kC; ++i)
          if (i < nvalid) o[(static_cast<size_t>(t0 + i) * p.Hv + h) * kD + dv] = __float2bfloat16_rn(y[i]);
      } else {
        float* o = static_cast<float*>(p.o);
#pragma unroll
        for (int i = 0; i < kC; ++i)
          if (i < nvalid) o[(static_cast<size_t>(t0 + i) * p.Hv + h) * kD + dv] = y[i];
      }
    }
    tc::fence_before_sync();
    __syncthreads();
  }

  if (failed) {
    if (tid == 0) atomicExch(p.err, 1);
    ptx::mbar_wait(bar, phase);      // one more bounded chance for an MMA in flight
  } else if (p.state_out) {
    float* dst = p.state_out + (static_cast<size_t>(bh) * kD + tid) * kD;
    for (int c = 0; c < kD; c += 16) {
      float v[16];
      tc::tmem_ld16(tDR + my + c, v);
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
