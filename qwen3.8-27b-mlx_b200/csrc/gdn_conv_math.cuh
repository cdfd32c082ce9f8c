// Arithmetic of the causal depthwise conv + SiLU (cpp/src/model.cpp:385-395,
// :588), shared by gdn_conv1d_fwd and the conv epilogue of gdn_in_proj_conv
// so that both give the same bits: fp32 taps on channel pairs (packed f32x2
// instructions of sm_100), oldest tap first, then the SiLU from the hardware's
// approximate 2^x and 1/x.
#pragma once

#include <cuda_runtime.h>

namespace gdn {

// The hardware's approximate 2^x and 1/x (PTX ex2.approx.ftz / rcp.approx.ftz).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// silu on two channels: a / (1 + e^-a) with e^-a = 2^(-a log2 e); a very
// negative a gives 2^+inf = inf, 1/inf = 0 and a signed zero.
__device__ __forceinline__ float2 silu2(float2 a) {
  constexpr float kLog2e = 1.4426950408889634f;
  const float2 t = __fmul2_rn(a, make_float2(-kLog2e, -kLog2e));
  const float2 den = __fadd2_rn(make_float2(1.f, 1.f), make_float2(ex2_approx(t.x), ex2_approx(t.y)));
  return __fmul2_rn(a, make_float2(rcp_approx(den.x), rcp_approx(den.y)));
}

// The 4 taps on a channel pair: r0 w0 + r1 w1 + r2 w2 + x w3, in that order
// (r0 the oldest window row, x the current row).
__device__ __forceinline__ float2 conv_pair(float2 r0, float2 r1, float2 r2, float2 x, float2 w0, float2 w1,
                                           float2 w2, float2 w3) {
  float2 acc = __fmul2_rn(r0, w0);
  acc = __ffma2_rn(r1, w1, acc);
  acc = __ffma2_rn(r2, w2, acc);
  return __ffma2_rn(x, w3, acc);
}

}  // namespace gdn
