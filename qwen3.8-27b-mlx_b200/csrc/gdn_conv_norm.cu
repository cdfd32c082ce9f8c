// Front end and back end of the Gated DeltaNet block, sm_100a:
//
//   * gdn_conv1d_fwd: causal depthwise conv1d (kernel 4, no bias) over the
//     concatenated q|k|v channels with its carried window, then SiLU
//     (cpp/src/model.cpp:385-395 and :588; python/qwen35.py:642-660).
//   * gdn_conv_commit: the conv half of DeltaCache::commit
//     (cpp/src/model.cpp:446-447): window = rows n .. n+K-2 of [state; x].
//   * gdn_gated_rmsnorm_fwd: normalise, then gate
//     (cpp/src/model.cpp:350-354): rms_norm(o, gamma, eps) * silu(z).
//
// All three are HBM-bound streams of bf16 activations: 16-byte vector loads
// and stores, one pass over the data, fp32 arithmetic in registers.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "gdn_conv_math.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {
namespace {

constexpr int kConvK = 4;            // linear_conv_kernel_dim (python/qwen35.py:92)
constexpr int kConvVec = 8;          // channels per thread (one 16-byte bf16 vector)
constexpr int kConvThreads = 128;
constexpr int kConvRun = 64;         // tokens per thread
constexpr int kConvBatch = 4;        // rows per cp.async group
constexpr int kConvStages = 4;       // groups per thread in the shared-memory ring (stages x batch = 16 rows, 256 bytes)
constexpr int kConvSmBlocks = 148;   // SMs of a B200, for sizing the prefill grid
constexpr int kConvShortT = 16;      // uniform batches of at most this many tokens per sequence: one thread per token

struct alignas(16) Bf16x8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const Bf16x8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ Bf16x8 pack8(const float (&f)[8]) {
  Bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

// Sequence of packed token `tok` (binary search over cu_seqlens[0..B]).
__device__ __forceinline__ int seq_of(const int32_t* cu, int B, long long tok) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= tok) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

struct ConvParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w;          // (C, K)
  const __nv_bfloat16* state_in;   // (B, K-1, C) or null
  __nv_bfloat16* state_out;        // (B, K-1, C) or null
  __nv_bfloat16* y;
  const int32_t* cu;               // (B+1) or null: uniform B x T
  long long total;                 // tokens
  int B, T, C;
  unsigned flags;
  // ring pool mode: state_in is (n_slots, K-1, C), sequence b's window is
  // slot slots[b] read oldest first from row ring_pos[slot]
  const int32_t* slots;
  const int32_t* ring_pos;
  int n_slots;
  int32_t* err;
  int run;                         // tokens per block of the prefill kernel (set by run_conv)
};

// One output vector of 8 channels: the K taps over the window rows r0 (oldest)
// .. r2 and the current row x, then the SiLU.
template <bool BF16_OPS>
__device__ __forceinline__ Bf16x8 conv_taps(const float (&r0)[kConvVec], const float (&r1)[kConvVec],
                                           const float (&r2)[kConvVec], const float (&xv)[kConvVec],
                                           const float (&w)[kConvK][kConvVec], bool silu) {
  float out[kConvVec];
  if constexpr (BF16_OPS) {   // MLX per-op bf16: each product and each partial sum rounded
#pragma unroll
    for (int e = 0; e < kConvVec; ++e) {
      float acc = bf16r(r0[e] * w[0][e]);
      acc = bf16r(acc + bf16r(r1[e] * w[1][e]));
      acc = bf16r(acc + bf16r(r2[e] * w[2][e]));
      acc = bf16r(acc + bf16r(xv[e] * w[3][e]));
      if (silu) acc = bf16r(acc * bf16r(sigmoid_f(acc)));
      out[e] = acc;
    }
  } else {
    // fp32 accumulation, two channels per packed f32x2 instruction, taps in
    // order (oldest first); the bf16 output rounding dwarfs the error of the
    // approximate exponential and reciprocal (a few ulp of fp32)
#pragma unroll
    for (int e = 0; e < kConvVec; e += 2) {
      float2 acc = conv_pair(make_float2(r0[e], r0[e + 1]), make_float2(r1[e], r1[e + 1]),
                             make_float2(r2[e], r2[e + 1]), make_float2(xv[e], xv[e + 1]),
                             make_float2(w[0][e], w[0][e + 1]), make_float2(w[1][e], w[1][e + 1]),
                             make_float2(w[2][e], w[2][e + 1]), make_float2(w[3][e], w[3][e + 1]));
      if (silu) acc = silu2(acc);
      out[e] = acc.x;
      out[e + 1] = acc.y;
    }
  }
  return pack8(out);
}

// The 8 channels x K taps of w (C, K) starting at channel c0 (32 contiguous bf16).
__device__ __forceinline__ void load_taps(const __nv_bfloat16* wt, int c0, float (&w)[kConvK][kConvVec]) {
  const Bf16x8* wp = reinterpret_cast<const Bf16x8*>(wt + static_cast<size_t>(c0) * kConvK);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float f[8];
    unpack8(wp[q], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int flat = q * 8 + e;                 // = channel_offset * K + tap
      w[flat % kConvK][flat / kConvK] = f[e];
    }
  }
}

// Row srow (0 = oldest) of sequence seq's carried window at channel c0: the
// dense (B, K-1, C) state, or its pool slot's ring; null for a zero row (no
// state, or a bad slot, which is reported).
__device__ __forceinline__ const __nv_bfloat16* window_row(const ConvParams& p, int seq, int srow, int c0) {
  if (!p.state_in) return nullptr;
  if (!p.slots) return p.state_in + (static_cast<long long>(seq) * (kConvK - 1) + srow) * p.C + c0;
  const int sl = p.slots[seq];
  if (sl < 0 || sl >= p.n_slots) {
    if (p.err) atomicExch(p.err, 1);
    return nullptr;
  }
  int hd = p.ring_pos[sl] % (kConvK - 1);
  if (hd < 0) hd += kConvK - 1;
  return p.state_in + (static_cast<long long>(sl) * (kConvK - 1) + (hd + srow) % (kConvK - 1)) * p.C + c0;
}

// Short uniform sequences (decode T = 1, verify T = k+1): one thread per
// (token, 8 channels), so a batch of single tokens spreads over the whole GPU
// instead of walking 64 sequences per thread.  The thread of a sequence's
// last token also writes the carried window (dense state_out).
template <bool BF16_OPS>
__global__ void __launch_bounds__(kConvThreads) conv1d_tok_kernel(const ConvParams p, int nvb) {
  const long long tok = blockIdx.x / nvb;
  const int c0 = ((blockIdx.x - static_cast<int>(tok) * nvb) * kConvThreads + threadIdx.x) * kConvVec;
  if (c0 >= p.C || tok >= p.total) return;
  const int seq = static_cast<int>(tok / p.T);
  const int t = static_cast<int>(tok - static_cast<long long>(seq) * p.T);
  const bool silu = !(p.flags & GDN_F_CONV_NO_SILU);
  float w[kConvK][kConvVec];
  load_taps(p.w, c0, w);
  Bf16x8 raw[kConvK - 1], xr;
  bool have[kConvK - 1];
#pragma unroll
  for (int j = 0; j < kConvK - 1; ++j) {        // window rows t-3 .. t-1 of [state; x_seq]
    const int pos = t - (kConvK - 1) + j;
    const __nv_bfloat16* src = pos >= 0 ? p.x + (tok - t + pos) * p.C + c0
                                        : window_row(p, seq, (kConvK - 1) + pos, c0);
    have[j] = src != nullptr;
    if (src) raw[j] = *reinterpret_cast<const Bf16x8*>(src);
  }
  xr = *reinterpret_cast<const Bf16x8*>(p.x + tok * p.C + c0);
  float win[kConvK - 1][kConvVec], xv[kConvVec];
#pragma unroll
  for (int j = 0; j < kConvK - 1; ++j) {
    if (have[j]) {
      unpack8(raw[j], win[j]);
    } else {
#pragma unroll
      for (int e = 0; e < kConvVec; ++e) win[j][e] = 0.f;
    }
  }
  unpack8(xr, xv);
  *reinterpret_cast<Bf16x8*>(p.y + tok * p.C + c0) = conv_taps<BF16_OPS>(win[0], win[1], win[2], xv, w, silu);
  if (p.state_out && t == p.T - 1) {
    // the carried window: rows T .. T+K-2 of [state (K-1 rows); x_seq (T rows)]
#pragma unroll
    for (int r = 0; r < kConvK - 1; ++r) {
      const int row = p.T + r;
      Bf16x8 v;
      if (row >= kConvK - 1) {
        v = *reinterpret_cast<const Bf16x8*>(p.x + (tok - t + (row - (kConvK - 1))) * p.C + c0);
      } else if (const __nv_bfloat16* sp = window_row(p, seq, row, c0)) {
        v = *reinterpret_cast<const Bf16x8*>(sp);
      } else {
        float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        v = pack8(z);
      }
      *reinterpret_cast<Bf16x8*>(p.state_out + (static_cast<long long>(seq) * (kConvK - 1) + r) * p.C + c0) = v;
    }
  }
}

// One thread: 8 channels x a run of up to p.run (<= 64) consecutive packed
// tokens, with the 3-row causal window in registers, so every x element is
// read once (plus a 3-row halo at the start of the run).  Rows stream in
// through a per-thread ring of cp.async groups in shared memory (4 groups of
// 4 rows, 32 KiB per block, six blocks per SM), so 12 rows are in flight while
// 4 are computed.  The window lives in a ring of 4 row slots: before row u of
// a 4-row batch, slots (u+1)%4, (u+2)%4, (u+3)%4 hold rows t-3, t-2, t-1 and
// row t lands in slot u, so the window moves without copies.  Batches that
// cross no sequence boundary and hold no sequence's last row (nearly all)
// take a branch-free path.
template <bool BF16_OPS>
__global__ void __launch_bounds__(kConvThreads, 6) conv1d_kernel(const ConvParams p) {
  const long long t_begin = static_cast<long long>(blockIdx.y) * p.run;
  if (t_begin >= p.total) return;
  // one binary search of cu_seqlens per block, shared through shared memory
  __shared__ int s_seq;
  if (p.cu && threadIdx.x == 0) s_seq = seq_of(p.cu, p.B, t_begin);
  __syncthreads();
  const int c0 = (blockIdx.x * kConvThreads + threadIdx.x) * kConvVec;
  if (c0 >= p.C) return;
  const long long t_end = t_begin + p.run < p.total ? t_begin + p.run : p.total;
  const bool silu = !(p.flags & GDN_F_CONV_NO_SILU);
  constexpr bool bf16_ops = BF16_OPS;

  float w[kConvK][kConvVec];
  load_taps(p.w, c0, w);

  // token range of sequence `seq`: packed offsets, or seq*T .. seq*T+T
  auto seq_begin = [&](int sq) -> long long { return p.cu ? p.cu[sq] : static_cast<long long>(sq) * p.T; };
  auto seq_end = [&](int sq) -> long long { return p.cu ? p.cu[sq + 1] : static_cast<long long>(sq + 1) * p.T; };
  int seq = p.cu ? s_seq : static_cast<int>(t_begin / p.T);
  long long s_begin = seq_begin(seq);
  long long s_end = seq_end(seq);

  float win[4][kConvVec];
  // rows t-3 .. t-1 of [state; x] for the sequence that holds t, into the
  // slots (u+1)%4 .. (u+3)%4 (u: t's place in its batch)
  auto load_window = [&](long long t, int u) {
#pragma unroll
    for (int j = 0; j < kConvK - 1; ++j) {
      float(&dst)[kConvVec] = win[(u + 1 + j) & 3];
      const long long pos = t - s_begin - (kConvK - 1) + j;     // position in the sequence
      const long long row = s_begin + pos;                       // packed row (guards a bad cu_seqlens)
      if (pos >= 0 && row >= 0 && row < p.total) {
        unpack8(*reinterpret_cast<const Bf16x8*>(p.x + row * p.C + c0), dst);
      } else if (p.state_in && pos < 0 && pos >= -(kConvK - 1)) {
        const __nv_bfloat16* sp = window_row(p, seq, static_cast<int>((kConvK - 1) + pos), c0);   // oldest first
        if (sp) {
          unpack8(*reinterpret_cast<const Bf16x8*>(sp), dst);
        } else {
#pragma unroll
          for (int e = 0; e < kConvVec; ++e) dst[e] = 0.f;
        }
      } else {
#pragma unroll
        for (int e = 0; e < kConvVec; ++e) dst[e] = 0.f;
      }
    }
  };
  load_window(t_begin, 0);

  // x rows go through a per-thread ring of kConvStages groups in shared
  // memory by cp.async: batches k + 1 .. k + kConvStages - 1 stream in while
  // batch k is computed, and the rows hold no registers while in flight.
  // Each thread reads only its own slots, so no barrier is needed.
  __shared__ Bf16x8 stage[kConvStages][kConvBatch][kConvThreads];
  auto issue = [&](long long tb, int sbuf) {
    const __nv_bfloat16* src = p.x + tb * p.C + c0;
#pragma unroll
    for (int u = 0; u < kConvBatch; ++u)
      if (tb + u < t_end) ptx::cp_async16(&stage[sbuf][u][threadIdx.x], src + static_cast<long long>(u) * p.C);
    ptx::cp_async_commit();
  };
#pragma unroll
  for (int g = 0; g < kConvStages - 1; ++g) {            // one commit group per stage, empty past the run
    if (t_begin + g * kConvBatch < t_end) issue(t_begin + g * kConvBatch, g);
    else ptx::cp_async_commit();
  }
  int sbuf = 0;
  for (long long tb = t_begin; tb < t_end; tb += kConvBatch, sbuf = (sbuf + 1) % kConvStages) {
    const long long nxt = tb + (kConvStages - 1) * kConvBatch;  // into the stage read in the previous batch
    if (nxt < t_end) issue(nxt, (sbuf + kConvStages - 1) % kConvStages);
    else ptx::cp_async_commit();
    ptx::cp_async_wait<kConvStages - 1>();                // this batch's group has landed
    __nv_bfloat16* yb = p.y + tb * p.C + c0;
    if (tb + kConvBatch <= t_end && tb + kConvBatch < s_end) {
#pragma unroll
      for (int u = 0; u < kConvBatch; ++u) {
        unpack8(stage[sbuf][u][threadIdx.x], win[u]);
        *reinterpret_cast<Bf16x8*>(yb + static_cast<long long>(u) * p.C) =
            conv_taps<bf16_ops>(win[(u + 1) & 3], win[(u + 2) & 3], win[(u + 3) & 3], win[u], w, silu);
      }
      continue;
    }
#pragma unroll
    for (int u = 0; u < kConvBatch; ++u) {
      const long long t = tb + u;
      if (t >= t_end) break;
      if (t >= s_end && seq < p.B - 1) {   // crossed into the next sequence
        ++seq;
        s_begin = seq_begin(seq);
        s_end = seq_end(seq);
        while (t >= s_end && seq < p.B - 1) {   // skip empty packed sequences
          ++seq;
          s_begin = seq_begin(seq);
          s_end = seq_end(seq);
        }
        load_window(t, u);
      }
      unpack8(stage[sbuf][u][threadIdx.x], win[u]);
      *reinterpret_cast<Bf16x8*>(yb + static_cast<long long>(u) * p.C) =
          conv_taps<bf16_ops>(win[(u + 1) & 3], win[(u + 2) & 3], win[(u + 3) & 3], win[u], w, silu);
      if (p.state_out && t == s_end - 1) {
        // the carried window: the last K-1 rows of [state; x], oldest first
#pragma unroll
        for (int j = 0; j < kConvK - 1; ++j)
          *reinterpret_cast<Bf16x8*>(p.state_out + (static_cast<long long>(seq) * (kConvK - 1) + j) * p.C + c0) =
              pack8(win[(u + 2 + j) & 3]);
      }
    }
  }
}

// Sequences of length 0 still get their window carried: state_out = state_in.
__global__ void conv_empty_kernel(const ConvParams p) {
  const int seq = blockIdx.y;
  const long long len = p.cu ? static_cast<long long>(p.cu[seq + 1] - p.cu[seq]) : p.T;
  if (len != 0) return;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * kConvVec;
  if (c0 >= p.C) return;
  for (int j = 0; j < kConvK - 1; ++j) {
    const size_t off = (static_cast<size_t>(seq) * (kConvK - 1) + j) * p.C + c0;
    Bf16x8 v;
    if (p.state_in) {
      v = *reinterpret_cast<const Bf16x8*>(p.state_in + off);
    } else {
      float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      v = pack8(z);
    }
    *reinterpret_cast<Bf16x8*>(p.state_out + off) = v;
  }
}

// commit: window of sequence b = rows n_b .. n_b+K-2 of [state_prev; x_b].
__global__ void conv_commit_kernel(const __nv_bfloat16* state_prev, const __nv_bfloat16* x, const int32_t* n,
                                   __nv_bfloat16* state_out, int T, int C, int32_t* err) {
  const int b = blockIdx.y;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * kConvVec;
  if (c0 >= C) return;
  const int nb = n[b];
  const bool ok = nb >= 0 && nb <= T;
  if (!ok && err && c0 == 0) atomicExch(err, 1);
  for (int j = 0; j < kConvK - 1; ++j) {
    const int row = (ok ? nb : 0) + j;                    // row of [state (K-1 rows); x (T rows)]
    Bf16x8 v;
    if (row < kConvK - 1) {
      if (state_prev) {
        v = *reinterpret_cast<const Bf16x8*>(state_prev + (static_cast<size_t>(b) * (kConvK - 1) + row) * C + c0);
      } else {
        float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        v = pack8(z);
      }
    } else {
      v = *reinterpret_cast<const Bf16x8*>(x + (static_cast<size_t>(b) * T + (row - (kConvK - 1))) * C + c0);
    }
    *reinterpret_cast<Bf16x8*>(state_out + (static_cast<size_t>(b) * (kConvK - 1) + j) * C + c0) = v;
  }
}

// Ring append: the first n_b tokens of sequence b (n_b = counts[b], or its
// length) enter the ring of slot slots[b]: token i goes to row
// (ring_pos + i) % (K-1), only the last K-1 of them matter, and ring_pos
// advances by n_b.  One block per sequence, so the position is read by every
// thread before thread 0 moves it.
__global__ void __launch_bounds__(256) conv_ring_append_kernel(const __nv_bfloat16* x, __nv_bfloat16* ring,
                                                              int32_t* ring_pos, const int32_t* slots, int n_slots,
                                                              const int32_t* counts, const int32_t* cu, int T, int C,
                                                              int32_t* err) {
  constexpr int W = kConvK - 1;
  const int b = blockIdx.x;
  const long long s_begin = cu ? static_cast<long long>(cu[b]) : static_cast<long long>(b) * T;
  const long long len = cu ? static_cast<long long>(cu[b + 1]) - cu[b] : T;
  const int sl = slots[b];
  const long long n = counts ? static_cast<long long>(counts[b]) : len;
  if (!(sl >= 0 && sl < n_slots && n >= 0 && n <= len)) {        // uniform over the block
    if (threadIdx.x == 0 && err) atomicExch(err, 1);
    return;
  }
  if (n == 0) return;
  int hd = ring_pos[sl] % W;
  if (hd < 0) hd += W;
  __syncthreads();
  const long long first = n > W ? n - W : 0;
  const int nv = C / kConvVec;
  const long long work = (n - first) * nv;
  for (long long idx = threadIdx.x; idx < work; idx += blockDim.x) {
    const long long i = first + idx / nv;
    const int c0 = static_cast<int>(idx % nv) * kConvVec;
    const int r = static_cast<int>((hd + i) % W);
    *reinterpret_cast<Bf16x8*>(ring + (static_cast<size_t>(sl) * W + r) * C + c0) =
        *reinterpret_cast<const Bf16x8*>(x + (s_begin + i) * C + c0);
  }
  if (threadIdx.x == 0) ring_pos[sl] = static_cast<int32_t>((hd + n) % W);
}

// Gated RMSNorm: one warp per (token, head) row of 128; lane j holds 4
// consecutive elements.  out = o * rsqrt(mean(o^2) + eps) * gamma * silu(z).
__global__ void __launch_bounds__(256) gated_rmsnorm_kernel(const void* o, const __nv_bfloat16* z, const float* gamma,
                                                           void* out, long long rows, float eps, unsigned flags) {
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const size_t base = static_cast<size_t>(row) * kD + lane * 4;
  // z and gamma do not depend on the row's norm: their loads go out with o's
  const uint2 zr = *reinterpret_cast<const uint2*>(z + base);
  const float4 g = *reinterpret_cast<const float4*>(gamma + lane * 4);
  float x[4];
  if (flags & GDN_F_NORM_IN_BF16) {
    const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(o) + base);
    const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    x[0] = lo.x; x[1] = lo.y; x[2] = hi.x; x[3] = hi.y;
  } else {
    const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(o) + base);
    x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
  }
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float r = rsqrtf(ss / static_cast<float>(kD) + eps);
  const float2 zlo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zr.x));
  const float2 zhi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zr.y));
  const float zz[4] = {zlo.x, zlo.y, zhi.x, zhi.y};
  const float gg[4] = {g.x, g.y, g.z, g.w};
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)    // sigmoid(z) = 1 / (1 + 2^(-z log2 e)), hardware exp2 and reciprocal
    y[i] = (x[i] * r * gg[i]) * (zz[i] * rcp_approx(1.f + ex2_approx(zz[i] * -1.4426950408889634f)));
  if (flags & GDN_F_NORM_OUT_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + base) = make_float4(y[0], y[1], y[2], y[3]);
  } else {
    __nv_bfloat162 a = __floats2bfloat162_rn(y[0], y[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(y[2], y[3]);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + base) = w;
  }
}

int run_conv(const ConvParams& p, void* stream);

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_conv1d_fwd(const void* x, const void* w, const void* state_in, void* state_out, void* y,
                              const int32_t* cu_seqlens, int B, int T, int C, int K, unsigned flags,
                              void* stream) {
  clear_error();
  if (flags & ~(GDN_F_CONV_BF16_OPS | GDN_F_CONV_NO_SILU))
    return fail(GDN_ERR_FLAGS, "unknown conv flag bits 0x%x", flags);
  if (K != kConvK) return fail(GDN_ERR_SHAPE, "K=%d: only the model's kernel size 4 is built", K);
  if (B < 0 || T < 0 || C <= 0 || C % kConvVec)
    return fail(GDN_ERR_SHAPE, "bad sizes B=%d T=%d C=%d (C must be a positive multiple of 8)", B, T, C);
  if (B == 0) return GDN_OK;
  const long long total = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  if (!w || (total > 0 && (!x || !y))) return fail(GDN_ERR_NULL, "w, and x and y when there are tokens, are required");
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16) || !aligned(state_in, 16) || !aligned(state_out, 16))
    return fail(GDN_ERR_ALIGN, "conv buffers must be 16-byte aligned");
  const size_t xbytes = static_cast<size_t>(total) * C * 2;
  const size_t sbytes = static_cast<size_t>(B) * (kConvK - 1) * C * 2;
  if (total > 0 && (y == x || overlap(y, xbytes, x, xbytes)))
    return fail(GDN_ERR_ALIAS, "y must not overlap x (the halo rows are re-read)");
  if (overlap(state_out, sbytes, state_in, sbytes) || overlap(state_out, sbytes, x, xbytes) ||
      overlap(state_out, sbytes, y, xbytes))
    return fail(GDN_ERR_ALIAS, "state_out overlaps an input or y");
  ConvParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
               static_cast<const __nv_bfloat16*>(state_in), static_cast<__nv_bfloat16*>(state_out),
               static_cast<__nv_bfloat16*>(y), cu_seqlens, total, B, cu_seqlens ? 0 : T, C, flags,
               nullptr, nullptr, 0, nullptr};
  return run_conv(p, stream);
}

namespace gdn {
namespace {

int run_conv(const ConvParams& p_in, void* stream) {
  ConvParams p = p_in;
  const int C = p.C, B = p.B;
  const long long total = p.total;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned gx = static_cast<unsigned>((C / kConvVec + kConvThreads - 1) / kConvThreads);
  if (total > 0 && !p.cu && p.T <= kConvShortT) {
    const int nvb = static_cast<int>((C / kConvVec + kConvThreads - 1) / kConvThreads);
    const long long blocks = total * nvb;
    if (blocks > 0x7fffffffLL) return fail(GDN_ERR_SHAPE, "too many tokens (%lld)", total);
    if (p.flags & GDN_F_CONV_BF16_OPS) conv1d_tok_kernel<true><<<static_cast<unsigned>(blocks), kConvThreads, 0, st>>>(p, nvb);
    else conv1d_tok_kernel<false><<<static_cast<unsigned>(blocks), kConvThreads, 0, st>>>(p, nvb);
    int rc = cuda_status(cudaGetLastError(), "conv1d launch");
    if (rc != GDN_OK) return rc;
  } else if (total > 0) {
    // runs of 64 tokens, or 32 / 16 when that leaves the GPU less than two
    // waves of blocks (short prefills: the 3-row halo per run costs less
    // than idle SMs)
    const long long min_blocks = 2LL * kConvSmBlocks * 6;
    p.run = kConvRun;
    while (p.run > 4 * kConvBatch && ((total + p.run - 1) / p.run) * gx < min_blocks) p.run /= 2;
    const long long gy = (total + p.run - 1) / p.run;
    if (gy > 65535) return fail(GDN_ERR_SHAPE, "at most %d tokens per call", 65535 * kConvRun);
    if (p.flags & GDN_F_CONV_BF16_OPS) conv1d_kernel<true><<<dim3(gx, static_cast<unsigned>(gy)), kConvThreads, 0, st>>>(p);
    else conv1d_kernel<false><<<dim3(gx, static_cast<unsigned>(gy)), kConvThreads, 0, st>>>(p);
    int rc = cuda_status(cudaGetLastError(), "conv1d launch");
    if (rc != GDN_OK) return rc;
  }
  if (p.state_out) {
    if (B > 65535) return fail(GDN_ERR_SHAPE, "B=%d too large", B);
    conv_empty_kernel<<<dim3(gx, static_cast<unsigned>(B)), kConvThreads, 0, st>>>(p);
    int rc = cuda_status(cudaGetLastError(), "conv1d empty-sequence launch");
    if (rc != GDN_OK) return rc;
  }
  return GDN_OK;
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_conv1d_fwd_pool(const void* x, const void* w, const void* ring, const int32_t* ring_pos,
                                   const int32_t* slots, int n_slots, void* y, const int32_t* cu_seqlens, int B,
                                   int T, int C, int K, unsigned flags, int32_t* err_flag, void* stream) {
  clear_error();
  if (flags & ~(GDN_F_CONV_BF16_OPS | GDN_F_CONV_NO_SILU))
    return fail(GDN_ERR_FLAGS, "unknown conv flag bits 0x%x", flags);
  if (K != kConvK) return fail(GDN_ERR_SHAPE, "K=%d: only the model's kernel size 4 is built", K);
  if (B < 0 || T < 0 || C <= 0 || C % kConvVec || n_slots <= 0)
    return fail(GDN_ERR_SHAPE, "bad sizes B=%d T=%d C=%d n_slots=%d", B, T, C, n_slots);
  if (B == 0) return GDN_OK;
  const long long total = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  if (!w || !ring || !ring_pos || !slots || (total > 0 && (!x || !y)))
    return fail(GDN_ERR_NULL, "w, ring, ring_pos, slots, and x and y when there are tokens, are required");
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16) || !aligned(ring, 16) || !aligned(ring_pos, 4) ||
      !aligned(slots, 4) || !aligned(err_flag, 4))
    return fail(GDN_ERR_ALIGN, "x, w, y, ring 16-byte aligned; ring_pos, slots, err_flag 4-byte");
  const size_t xbytes = static_cast<size_t>(total) * C * 2;
  const size_t rbytes = static_cast<size_t>(n_slots) * (kConvK - 1) * C * 2;
  if (total > 0 && (y == x || overlap(y, xbytes, x, xbytes)))
    return fail(GDN_ERR_ALIAS, "y must not overlap x (the halo rows are re-read)");
  if (overlap(y, xbytes, ring, rbytes)) return fail(GDN_ERR_ALIAS, "y overlaps the ring pool");
  ConvParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
               static_cast<const __nv_bfloat16*>(ring), nullptr, static_cast<__nv_bfloat16*>(y), cu_seqlens, total, B,
               cu_seqlens ? 0 : T, C, flags, slots, ring_pos, n_slots, err_flag};
  return run_conv(p, stream);
}

extern "C" int gdn_conv_ring_append(const void* x, void* ring, int32_t* ring_pos, const int32_t* slots, int n_slots,
                                    const int32_t* counts, const int32_t* cu_seqlens, int B, int T, int C, int K,
                                    int32_t* err_flag, void* stream) {
  clear_error();
  if (K != kConvK) return fail(GDN_ERR_SHAPE, "K=%d: only 4 is built", K);
  if (B < 0 || T < 0 || C <= 0 || C % kConvVec || n_slots <= 0)
    return fail(GDN_ERR_SHAPE, "bad sizes B=%d T=%d C=%d n_slots=%d", B, T, C, n_slots);
  if (B == 0) return GDN_OK;
  const long long total = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  if (!ring || !ring_pos || !slots || (total > 0 && !x))
    return fail(GDN_ERR_NULL, "ring, ring_pos, slots, and x when there are tokens, are required");
  if (!aligned(x, 16) || !aligned(ring, 16) || !aligned(ring_pos, 4) || !aligned(slots, 4) || !aligned(counts, 4) ||
      !aligned(err_flag, 4))
    return fail(GDN_ERR_ALIGN, "x, ring 16-byte aligned; ring_pos, slots, counts, err_flag 4-byte");
  const size_t xbytes = static_cast<size_t>(total) * C * 2;
  const size_t rbytes = static_cast<size_t>(n_slots) * (kConvK - 1) * C * 2;
  if (overlap(x, xbytes, ring, rbytes)) return fail(GDN_ERR_ALIAS, "x overlaps the ring pool");
  if (B > 0x7fffffff) return fail(GDN_ERR_SHAPE, "B too large");
  conv_ring_append_kernel<<<static_cast<unsigned>(B), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(ring), ring_pos, slots, n_slots, counts,
      cu_seqlens, cu_seqlens ? 0 : T, C, err_flag);
  return cuda_status(cudaGetLastError(), "conv ring append launch");
}

extern "C" int gdn_conv_commit(const void* state_prev, const void* x, const int32_t* commit_n, void* state_out,
                               int32_t* err_flag, int B, int T, int C, int K, void* stream) {
  clear_error();
  if (K != kConvK) return fail(GDN_ERR_SHAPE, "K=%d: only 4 is built", K);
  if (B < 0 || T < 0 || C <= 0 || C % kConvVec) return fail(GDN_ERR_SHAPE, "bad sizes B=%d T=%d C=%d", B, T, C);
  if (B == 0) return GDN_OK;
  if (!commit_n || !state_out || (!x && T > 0)) return fail(GDN_ERR_NULL, "commit_n, state_out and x are required");
  if (!aligned(state_prev, 16) || !aligned(x, 16) || !aligned(state_out, 16) || !aligned(commit_n, 4) ||
      !aligned(err_flag, 4))
    return fail(GDN_ERR_ALIGN, "buffers must be 16-byte aligned (commit_n, err_flag 4-byte)");
  const size_t sbytes = static_cast<size_t>(B) * (kConvK - 1) * C * 2;
  const size_t xbytes = static_cast<size_t>(B) * T * C * 2;
  if (overlap(state_out, sbytes, state_prev, sbytes) || overlap(state_out, sbytes, x, xbytes))
    return fail(GDN_ERR_ALIAS, "state_out overlaps state_prev or x");
  if (B > 65535) return fail(GDN_ERR_SHAPE, "B=%d too large", B);
  const unsigned gx = static_cast<unsigned>((C / kConvVec + kConvThreads - 1) / kConvThreads);
  conv_commit_kernel<<<dim3(gx, static_cast<unsigned>(B)), kConvThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(state_prev), static_cast<const __nv_bfloat16*>(x), commit_n,
      static_cast<__nv_bfloat16*>(state_out), T, C, err_flag);
  return cuda_status(cudaGetLastError(), "conv commit launch");
}

extern "C" int gdn_gated_rmsnorm_fwd(const void* o, const void* z, const float* gamma, void* out, long long rows,
                                     int D, float eps, unsigned flags, void* stream) {
  clear_error();
  if (flags & ~(GDN_F_NORM_IN_BF16 | GDN_F_NORM_OUT_F32)) return fail(GDN_ERR_FLAGS, "unknown norm flags 0x%x", flags);
  if (D != kD || rows < 0) return fail(GDN_ERR_SHAPE, "D=%d rows=%lld: only D = 128 is built", D, rows);
  if (rows == 0) return GDN_OK;
  if (!o || !z || !gamma || !out) return fail(GDN_ERR_NULL, "o, z, gamma and out are required");
  if (!aligned(o, 16) || !aligned(z, 8) || !aligned(gamma, 16) || !aligned(out, 16))
    return fail(GDN_ERR_ALIGN, "o, gamma, out 16-byte and z 8-byte aligned");
  const size_t ib = static_cast<size_t>(rows) * kD * ((flags & GDN_F_NORM_IN_BF16) ? 2 : 4);
  const size_t ob = static_cast<size_t>(rows) * kD * ((flags & GDN_F_NORM_OUT_F32) ? 4 : 2);
  if (out != o && overlap(out, ob, o, ib)) return fail(GDN_ERR_ALIAS, "out partially overlaps o");
  if (overlap(out, ob, z, static_cast<size_t>(rows) * kD * 2)) return fail(GDN_ERR_ALIAS, "out overlaps z");
  if ((rows + 7) / 8 > 0x7fffffffLL) return fail(GDN_ERR_SHAPE, "too many rows");
  gated_rmsnorm_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      o, static_cast<const __nv_bfloat16*>(z), gamma, out, rows, eps, flags);
  return cuda_status(cudaGetLastError(), "gated rmsnorm launch");
}
