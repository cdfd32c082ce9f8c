// Decode / speculative-verify kernel of the Gated DeltaNet recurrence, sm_100a.
//
// The step is pure state streaming: per sequence and value head the fp32
// state S (128 x 128, 64 KiB) is read once and written once per call, and
// every per-token input is a few hundred bytes.  So the kernel is built for
// HBM bandwidth, not arithmetic:
//
//   * one warp owns R consecutive state rows of one (sequence, value head);
//     lane j holds columns 4j..4j+3 of every row as a float4, so a row is one
//     fully coalesced 512-byte load (LDG.128 per lane) and one 512-byte store;
//   * the time loop (T = 1 decode, T = k+1 verify) runs with the rows in
//     registers, so S crosses HBM once per call whatever T is;
//   * both reductions (k.S[v,:] and q.S[v,:]) are warp butterflies over the
//     32 lanes; the R rows of a warp reduce together for ILP;
//   * q, k of the key head (16 heads serve 48 value heads) are read once per
//     warp per step straight from their bf16 form; the gates
//     alpha = exp(-exp(A_log) softplus(a + dt_bias)) and beta = sigmoid(b)
//     are computed in-kernel (cpp/src/model.cpp:608-612);
//   * state traffic uses streaming cache hints (ld.global.cs / st.global.cs):
//     it is touched exactly once and must not evict the small shared inputs;
//   * bytes in flight, not instructions, bound the kernel, so a warp owns up
//     to R = 8 rows (4 KiB of loads outstanding per warp);
//   * per-position checkpoints (DeltaCache record mode) are streamed out in
//     the same pass, and the rollback of DeltaCache::commit is an index into
//     them (gdn_recurrent_fwd_from_ckpt), not a copy.
//
// Arithmetic per row follows delta::run_reference (cpp/src/delta.cpp:175-204):
// kS = sum k*S, S = a*(S - (b*kS)*k) + (b*v)*k, o = sum q*S, in fp32.
#include <cuda_bf16.h>
#include <cuda_runtime.h>


#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr float kL2Eps = 1e-6f;                    // ops::l2norm eps (cpp/src/ops.hpp:19-20)

struct RecParams {
  const void* q;
  const void* k;
  const void* v;
  const float* a;
  const float* b;
  const float* A_log;
  const float* dt_bias;
  const float* state_in;    // dense (B,Hv,D,D) start state, or state_prev in ckpt mode; may be null
  const float* ckpt_src;    // (B,Hv,Tsrc,D,D) committed checkpoints (ckpt mode)
  const int32_t* commit_n;  // (B) commit index per sequence (ckpt mode)
  int32_t* err_flag;
  float* state_out;
  void* o;
  float* ckpt;
  int B, T, Hk, Hv, Tsrc;
  unsigned flags;
  // state pool mode: sequence b's state lives in slot slots[b] of a
  // (n_slots, Hv, D, D) pool (state_in == state_out == the pool); pool_write
  // says what the call leaves there (GDN_POOL_KEEP / _FINAL / _START)
  const int32_t* slots;
  int n_slots;
  int pool_write;
};

__device__ __forceinline__ float4 ld_stream4(const float* p) {
  return __ldcs(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ void st_stream4(float* p, float4 v) {
  __stcs(reinterpret_cast<float4*>(p), v);
}

template <bool BF16>
__device__ __forceinline__ float4 ld_in4(const void* base, size_t idx);

template <>
__device__ __forceinline__ float4 ld_in4<true>(const void* base, size_t idx) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(base) + idx));
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

template <>
__device__ __forceinline__ float4 ld_in4<false>(const void* base, size_t idx) {
  return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx));
}

template <bool BF16>
__device__ __forceinline__ float ld_in1(const void* base, size_t idx) {
  if constexpr (BF16) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
  } else {
    return __ldg(static_cast<const float*>(base) + idx);
  }
}

__device__ __forceinline__ float dot4(float4 x, float4 y) {
  return x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
}

// Sum each of x[0..N) over the 32 lanes of the warp; every lane gets the sums.
template <int N>
__device__ __forceinline__ void warp_sum(float (&x)[N]) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
    for (int i = 0; i < N; ++i) x[i] += __shfl_xor_sync(0xffffffffu, x[i], off);
  }
}

// softplus(x) = logaddexp(0, x) (cpp/src/ops.cpp:22-25), in its stable form.
__device__ __forceinline__ float softplus_f(float x) {
  return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)));
}

// PM: 0 dense states; 1 pool, written back after the last position when
// pool_write is GDN_POOL_FINAL; 2 pool, the start state written back
// (GDN_POOL_START).  The start-state store is its own instantiation so that
// the other modes carry no store between the state loads and the token loads.
// 8 resident 128-thread blocks per SM (64 registers, no spills at R = 8):
// the loads in flight per SM, not the instruction count, set the achieved
// bandwidth -- 6 blocks at the compiler's own 80 registers streamed ~7% less.
template <bool BF16, int R, int PM>
__global__ void __launch_bounds__(128, 8) recurrent_kernel(const RecParams p) {
  constexpr bool POOL = PM != 0;
  constexpr int kRowsPerBlock = 4 * R;
  constexpr int kBlocksPerHead = kD / kRowsPerBlock;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int bh = blockIdx.x / kBlocksPerHead;
  const int row0 = (blockIdx.x - bh * kBlocksPerHead) * kRowsPerBlock + warp * R;
  const int b = bh / p.Hv;
  const int h = bh - b * p.Hv;
  const int kh = h / (p.Hv / p.Hk);
  const int col = lane * 4;
  // Start state of this (sequence, head): the dense state, or its pool slot.
  size_t sidx = static_cast<size_t>(bh);
  bool slot_ok = true;
  if constexpr (POOL) {
    const int sl = __ldg(p.slots + b);
    slot_ok = sl >= 0 && sl < p.n_slots;
    sidx = static_cast<size_t>(slot_ok ? sl : 0) * p.Hv + h;
    if (!slot_ok && p.err_flag && threadIdx.x == 0) atomicExch(p.err_flag, 1);
  }
  const float* src = (p.state_in && slot_ok) ? p.state_in + sidx * kD * kD : nullptr;
  if (p.commit_n) {
    const int n = p.commit_n[b];
    if (n > 0 && n <= p.Tsrc) {
      src = p.ckpt_src + (static_cast<size_t>(bh) * p.Tsrc + (n - 1)) * kD * kD;
    } else if (n != 0) {
      src = nullptr;
      if (p.err_flag && threadIdx.x == 0) atomicExch(p.err_flag, 1);
    }
  }
  float4 s[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    s[r] = src ? ld_stream4(src + static_cast<size_t>(row0 + r) * kD + col)
               : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if constexpr (PM == 2) {
    // a committed checkpoint (or a zero start) materialised in the slot; a
    // start from the slot itself leaves it as it is
    float* pool_row = p.state_out + (sidx * kD + row0) * kD + col;
    if (slot_ok && src != p.state_out + sidx * kD * kD) {
#pragma unroll
      for (int r = 0; r < R; ++r) st_stream4(pool_row + static_cast<size_t>(r) * kD, s[r]);
    }
  }
  // launched with GDN_F_OVERLAP_PREV: the state rows above are in flight while
  // the previous grid finishes; the token inputs are read only after it has
  // completed (a no-op for an ordinary launch)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Only now may the next kernel in the stream begin launching.  Triggering
  // after the wait means a dependent launch N + 1 starts only once every
  // block of launch N has seen launch N - 1 complete, so dependents never
  // chain further than one kernel: a launch's early state loads can overlap
  // the previous kernel only, never one further back that might still be
  // writing those states (two layers used in turn, A B A B, stay correct).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const bool direct = (p.flags & GDN_F_GATES_DIRECT) != 0;
  const bool l2 = (p.flags & GDN_F_QK_L2NORM) != 0;
  const bool raw_gates = !direct && p.T > 0;       // A_log may be null when T == 0
  const float A = raw_gates ? expf(__ldg(p.A_log + h)) : 0.f;
  const float dtb = raw_gates ? __ldg(p.dt_bias + h) : 0.f;
  const float qscale = rsqrtf(static_cast<float>(kD));

  for (int t = 0; t < p.T; ++t) {
    const size_t tok = static_cast<size_t>(b) * p.T + t;
    const size_t qk = (tok * p.Hk + kh) * kD + col;
    float4 kk = ld_in4<BF16>(p.k, qk);
    float4 qq = ld_in4<BF16>(p.q, qk);
    if (l2) {
      float ss[2] = {dot4(kk, kk), dot4(qq, qq)};
      warp_sum<2>(ss);
      const float rk = rsqrtf(ss[0] + kL2Eps);
      const float rq = rsqrtf(ss[1] + kL2Eps);
      kk = make_float4(kk.x * rk, kk.y * rk, kk.z * rk, kk.w * rk);
      qq = make_float4(qq.x * rq * qscale, qq.y * rq * qscale, qq.z * rq * qscale, qq.w * rq * qscale);
    }
    const size_t gi = tok * p.Hv + h;
    float alpha, beta;
    if (direct) {
      alpha = __ldg(p.a + gi);
      beta = __ldg(p.b + gi);
    } else {
      alpha = expf(-(A * softplus_f(__ldg(p.a + gi) + dtb)));
      beta = 1.f / (1.f + expf(-__ldg(p.b + gi)));
    }
    float vr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) vr[r] = ld_in1<BF16>(p.v, gi * kD + row0 + r);

    float ks[R];
#pragma unroll
    for (int r = 0; r < R; ++r) ks[r] = dot4(kk, s[r]);
    warp_sum<R>(ks);

    float ov[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float bk = beta * ks[r];
      const float bv = beta * vr[r];
      s[r].x = alpha * (s[r].x - bk * kk.x) + bv * kk.x;
      s[r].y = alpha * (s[r].y - bk * kk.y) + bv * kk.y;
      s[r].z = alpha * (s[r].z - bk * kk.z) + bv * kk.z;
      s[r].w = alpha * (s[r].w - bk * kk.w) + bv * kk.w;
      ov[r] = dot4(qq, s[r]);
    }
    warp_sum<R>(ov);

    if (p.ckpt) {
      float* dst = p.ckpt + ((static_cast<size_t>(bh) * p.T + t) * kD + row0) * kD + col;
#pragma unroll
      for (int r = 0; r < R; ++r) st_stream4(dst + static_cast<size_t>(r) * kD, s[r]);
    }
    if (lane < R) {
      float val = ov[0];
#pragma unroll
      for (int r = 1; r < R; ++r) val = (lane == r) ? ov[r] : val;
      const size_t oi = gi * kD + row0 + lane;
      if (p.flags & GDN_F_O_BF16) {
        static_cast<__nv_bfloat16*>(p.o)[oi] = __float2bfloat16_rn(val);
      } else {
        static_cast<float*>(p.o)[oi] = val;
      }
    }
  }

  if (p.state_out && (PM == 0 || (PM == 1 && slot_ok && p.pool_write == GDN_POOL_FINAL))) {
    float* dst = p.state_out + (sidx * kD + row0) * kD + col;
#pragma unroll
    for (int r = 0; r < R; ++r) st_stream4(dst + static_cast<size_t>(r) * kD, s[r]);
  }
}


template <bool BF16, int R, int PM>
cudaError_t launch_one(const RecParams& p, unsigned grid, cudaStream_t st) {
  if (!(p.flags & GDN_F_OVERLAP_PREV)) {
    recurrent_kernel<BF16, R, PM><<<grid, 128, 0, st>>>(p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, recurrent_kernel<BF16, R, PM>, p);
}

template <bool BF16, int PM>
cudaError_t launch_rows(const RecParams& p, int R, cudaStream_t st) {
  const long long bh = static_cast<long long>(p.B) * p.Hv;
  R = (R == 1 || R == 2 || R == 8) ? R : 4;
  const unsigned grid = static_cast<unsigned>(bh * (kD / (4 * R)));
  switch (R) {
    case 1: return launch_one<BF16, 1, PM>(p, grid, st);
    case 2: return launch_one<BF16, 2, PM>(p, grid, st);
    case 8: return launch_one<BF16, 8, PM>(p, grid, st);
    default: return launch_one<BF16, 4, PM>(p, grid, st);
  }
}

template <int PM>
cudaError_t launch_mode(const RecParams& p, bool bf16, int R, cudaStream_t st) {
  return bf16 ? launch_rows<true, PM>(p, R, st) : launch_rows<false, PM>(p, R, st);
}

// Rows per warp.  Bytes in flight per SM set the achieved HBM bandwidth:
// with R rows a warp has R x 512 B of loads outstanding.  Measured on B200,
// one layer at B = 256 (in-place update, bf16 q/k/v/o): R = 1, 2, 4, 8 ->
// 2.5, 4.2, 5.5, 6.2 TB/s.  Small batches take fewer rows only down to about
// 2.5 blocks per SM: a 48-layer step at B = 1, 2, 3 took 150, 204, 239 us this
// way against 202, 220, 267 us when a full wave of blocks was kept.
int rows_per_warp(long long bh) {
#ifdef GDN_REC_ROWS
  (void)bh;
  return GDN_REC_ROWS;
#else
  const long long min_blocks = 148LL * 5 / 2;   // at B = 1 (48 heads): R = 4, 384 blocks
  for (int R = 8; R > 1; R >>= 1)
    if (bh * (kD / (4 * R)) >= min_blocks) return R;
  return 1;
#endif
}

// Launch the decode / verify kernel over B x Hv (sequence, value head) pairs
// with the rows per warp that rows_per_warp() picks for that count.
int run_recurrent(const RecParams& p, void* stream) {
  if (p.B == 0) return GDN_OK;
  const long long bh = static_cast<long long>(p.B) * p.Hv;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = (p.flags & GDN_F_QKV_F32) == 0;
  const int R = rows_per_warp(bh);
  const cudaError_t e = !p.slots ? launch_mode<0>(p, bf16, R, st)
                        : p.pool_write == GDN_POOL_START ? launch_mode<2>(p, bf16, R, st)
                                                         : launch_mode<1>(p, bf16, R, st);
  return cuda_status(e, "gdn recurrent kernel launch");
}

constexpr unsigned kKnownFlags = GDN_F_QKV_F32 | GDN_F_O_BF16 | GDN_F_GATES_DIRECT | GDN_F_QK_L2NORM | GDN_F_OVERLAP_PREV;

// Checks shared by both recurrent entry points.
int check_common(const void* q, const void* k, const void* v, const float* a, const float* b,
                 const float* A_log, const float* dt_bias, const void* o, int B, int T, int Hk,
                 int Hv, int Dk, int Dv, unsigned flags) {
  if (flags & ~kKnownFlags) return fail(GDN_ERR_FLAGS, "unknown flag bits 0x%x", flags & ~kKnownFlags);
  if (B < 0 || T < 0 || Hk <= 0 || Hv <= 0)
    return fail(GDN_ERR_SHAPE, "bad sizes B=%d T=%d Hk=%d Hv=%d", B, T, Hk, Hv);
  if (Dk != kD || Dv != kD) return fail(GDN_ERR_SHAPE, "Dk=%d Dv=%d: only 128x128 heads are built", Dk, Dv);
  if (Hv % Hk != 0) return fail(GDN_ERR_SHAPE, "Hv=%d is not a multiple of Hk=%d", Hv, Hk);
  if (static_cast<long long>(B) * Hv * kD >= (1LL << 31))
    return fail(GDN_ERR_SHAPE, "B*Hv=%lld too large for one launch", static_cast<long long>(B) * Hv);
  if (B == 0 || T == 0) return GDN_OK;
  if (!q || !k || !v) return fail(GDN_ERR_NULL, "q, k and v are required when T > 0");
  if (!a || !b) return fail(GDN_ERR_NULL, "a and b are required when T > 0");
  if (!(flags & GDN_F_GATES_DIRECT) && (!A_log || !dt_bias))
    return fail(GDN_ERR_NULL, "A_log and dt_bias are required unless GDN_F_GATES_DIRECT");
  if (!o) return fail(GDN_ERR_NULL, "o is required when T > 0");
  const size_t vec = (flags & GDN_F_QKV_F32) ? 16 : 8;
  if (!aligned(q, vec) || !aligned(k, vec))
    return fail(GDN_ERR_ALIGN, "q and k must be %zu-byte aligned", vec);
  const size_t el = (flags & GDN_F_QKV_F32) ? 4 : 2;
  if (!aligned(v, el) || !aligned(a, 4) || !aligned(b, 4))
    return fail(GDN_ERR_ALIGN, "v, a, b must be element-aligned");
  if (!aligned(o, (flags & GDN_F_O_BF16) ? 2 : 4)) return fail(GDN_ERR_ALIGN, "o must be element-aligned");
  return GDN_OK;
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_recurrent_fwd(const void* q, const void* k, const void* v, const float* a,
                                 const float* b, const float* A_log, const float* dt_bias,
                                 const float* state_in, float* state_out, void* o, float* ckpt,
                                 int B, int T, int Hk, int Hv, int Dk, int Dv, unsigned flags,
                                 void* stream) {
  clear_error();
  int rc = check_common(q, k, v, a, b, A_log, dt_bias, o, B, T, Hk, Hv, Dk, Dv, flags);
  if (rc != GDN_OK) return rc;
  if (B == 0) return GDN_OK;
  if (!state_out && !ckpt) return fail(GDN_ERR_NULL, "state_out and ckpt are both NULL");
  if (!aligned(state_in, 16) || !aligned(state_out, 16) || !aligned(ckpt, 16))
    return fail(GDN_ERR_ALIGN, "state_in, state_out and ckpt must be 16-byte aligned");
  const size_t sbytes = static_cast<size_t>(B) * Hv * kD * kD * sizeof(float);
  const size_t cbytes = sbytes * static_cast<size_t>(T);
  const size_t obytes = static_cast<size_t>(B) * T * Hv * kD * ((flags & GDN_F_O_BF16) ? 2 : 4);
  if (state_in != state_out && overlap(state_in, sbytes, state_out, sbytes))
    return fail(GDN_ERR_ALIAS, "state_out partially overlaps state_in");
  if (overlap(ckpt, cbytes, state_in, sbytes) || overlap(ckpt, cbytes, state_out, sbytes))
    return fail(GDN_ERR_ALIAS, "ckpt overlaps a state buffer");
  if (overlap(o, obytes, state_in, sbytes) || overlap(o, obytes, state_out, sbytes) ||
      overlap(o, obytes, ckpt, cbytes))
    return fail(GDN_ERR_ALIAS, "o overlaps a state or checkpoint buffer");
  RecParams p{q, k, v, a, b, A_log, dt_bias, state_in, nullptr, nullptr, nullptr,
              state_out, o, T > 0 ? ckpt : nullptr, B, T, Hk, Hv, 0, flags, nullptr, 0, 0};
  return run_recurrent(p, stream);
}

extern "C" int gdn_recurrent_fwd_from_ckpt(const void* q, const void* k, const void* v,
                                           const float* a, const float* b, const float* A_log,
                                           const float* dt_bias, const float* state_prev,
                                           const float* ckpt_src, const int32_t* commit_n,
                                           int Tsrc, float* state_out, void* o, float* ckpt,
                                           int32_t* err_flag, int B, int T, int Hk, int Hv,
                                           int Dk, int Dv, unsigned flags, void* stream) {
  clear_error();
  int rc = check_common(q, k, v, a, b, A_log, dt_bias, o, B, T, Hk, Hv, Dk, Dv, flags);
  if (rc != GDN_OK) return rc;
  if (B == 0) return GDN_OK;
  if (flags & GDN_F_OVERLAP_PREV)
    return fail(GDN_ERR_FLAGS, "GDN_F_OVERLAP_PREV: commit_n may come from the previous kernel");
  if (!ckpt_src || !commit_n) return fail(GDN_ERR_NULL, "ckpt_src and commit_n are required");
  if (Tsrc <= 0) return fail(GDN_ERR_SHAPE, "Tsrc=%d must be positive", Tsrc);
  if (!state_out && !ckpt) return fail(GDN_ERR_NULL, "state_out and ckpt are both NULL");
  if (!aligned(state_prev, 16) || !aligned(ckpt_src, 16) || !aligned(state_out, 16) ||
      !aligned(ckpt, 16) || !aligned(commit_n, 4) || !aligned(err_flag, 4))
    return fail(GDN_ERR_ALIGN, "state buffers must be 16-byte aligned, commit_n/err_flag 4-byte");
  const size_t sbytes = static_cast<size_t>(B) * Hv * kD * kD * sizeof(float);
  const size_t srcbytes = sbytes * static_cast<size_t>(Tsrc);
  const size_t cbytes = sbytes * static_cast<size_t>(T);
  if (overlap(state_out, sbytes, ckpt_src, srcbytes) || overlap(state_out, sbytes, state_prev, sbytes) ||
      overlap(ckpt, cbytes, ckpt_src, srcbytes) || overlap(ckpt, cbytes, state_prev, sbytes) ||
      overlap(ckpt, cbytes, state_out, sbytes))
    return fail(GDN_ERR_ALIAS, "outputs overlap the committed checkpoints or state_prev");
  RecParams p{q, k, v, a, b, A_log, dt_bias, state_prev, ckpt_src, commit_n, err_flag,
              state_out, o, T > 0 ? ckpt : nullptr, B, T, Hk, Hv, Tsrc, flags, nullptr, 0, 0};
  return run_recurrent(p, stream);
}

extern "C" int gdn_recurrent_fwd_pool(const void* q, const void* k, const void* v, const float* a,
                                      const float* b, const float* A_log, const float* dt_bias, float* pool,
                                      const int32_t* slots, int n_slots, const float* ckpt_src,
                                      const int32_t* commit_n, int Tsrc, int pool_write, void* o, float* ckpt,
                                      int32_t* err_flag, int B, int T, int Hk, int Hv, int Dk, int Dv,
                                      unsigned flags, void* stream) {
  clear_error();
  int rc = check_common(q, k, v, a, b, A_log, dt_bias, o, B, T, Hk, Hv, Dk, Dv, flags);
  if (rc != GDN_OK) return rc;
  if (B == 0) return GDN_OK;
  if (flags & GDN_F_OVERLAP_PREV)
    return fail(GDN_ERR_FLAGS, "GDN_F_OVERLAP_PREV: slots and commit_n may come from the previous kernel");
  if (!pool || !slots) return fail(GDN_ERR_NULL, "pool and slots are required");
  if (n_slots <= 0 || static_cast<long long>(n_slots) * Hv * kD >= (1LL << 31))
    return fail(GDN_ERR_SHAPE, "n_slots=%d out of range", n_slots);
  if (pool_write != GDN_POOL_KEEP && pool_write != GDN_POOL_FINAL && pool_write != GDN_POOL_START)
    return fail(GDN_ERR_FLAGS, "pool_write=%d is not GDN_POOL_KEEP, _FINAL or _START", pool_write);
  if ((ckpt_src == nullptr) != (commit_n == nullptr))
    return fail(GDN_ERR_NULL, "ckpt_src and commit_n go together");
  if (commit_n && Tsrc <= 0) return fail(GDN_ERR_SHAPE, "Tsrc=%d must be positive", Tsrc);
  if (!aligned(pool, 16) || !aligned(ckpt_src, 16) || !aligned(ckpt, 16) || !aligned(slots, 4) ||
      !aligned(commit_n, 4) || !aligned(err_flag, 4))
    return fail(GDN_ERR_ALIGN, "pool, ckpt_src, ckpt 16-byte aligned; slots, commit_n, err_flag 4-byte");
  const size_t sbytes = static_cast<size_t>(B) * Hv * kD * kD * sizeof(float);
  const size_t pbytes = static_cast<size_t>(n_slots) * Hv * kD * kD * sizeof(float);
  const size_t srcbytes = commit_n ? sbytes * static_cast<size_t>(Tsrc) : 0;
  const size_t cbytes = sbytes * static_cast<size_t>(T);
  const size_t obytes = static_cast<size_t>(B) * T * Hv * kD * ((flags & GDN_F_O_BF16) ? 2 : 4);
  if (overlap(pool, pbytes, ckpt_src, srcbytes) || overlap(pool, pbytes, ckpt, cbytes) ||
      overlap(pool, pbytes, o, obytes) || overlap(ckpt, cbytes, ckpt_src, srcbytes) || overlap(o, obytes, ckpt, cbytes))
    return fail(GDN_ERR_ALIAS, "pool, ckpt_src, ckpt and o must not overlap");
  RecParams p{q, k, v, a, b, A_log, dt_bias, pool, ckpt_src, commit_n, err_flag,
              pool, o, T > 0 ? ckpt : nullptr, B, T, Hk, Hv, commit_n ? Tsrc : 0, flags, slots, n_slots, pool_write};
  return run_recurrent(p, stream);
}

extern "C" int gdn_delta_run(const float* q, const float* k, const float* v, const float* alpha,
                             const float* beta, const float* S, float* o, float* S_out,
                             float* states, int B, int L, int H, int Dk, int Dv, void* stream) {
  return gdn_recurrent_fwd(q, k, v, alpha, beta, nullptr, nullptr, S, S_out, o, states, B, L, H, H,
                           Dk, Dv, GDN_F_QKV_F32 | GDN_F_GATES_DIRECT, stream);
}
