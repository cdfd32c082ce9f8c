// Device self-test of the tcgen05 tensor-core path the chunked prefill kernel
// is built on: one CTA computes D (128 x N) = op(A) (128 x K) * B^T (B is
// N x K) through tcgen05.mma with the accumulator in tensor memory, using the
// same shared-memory layout, descriptors and TMEM load/store helpers as the
// prefill kernel.  Modes: tf32, bf16 or fp16 operands, A negated by the instruction
// descriptor, A read from tensor memory instead of shared memory, MN-major
// operands, D at a column offset of 64 and/or 128 (N up to 256).  A last mode
// issues no MMA at all and waits on the barrier with a small poll budget, so
// that the bounded wait runs out: the kernel must then report the timeout
// (status word and the library's device error word) and return cleanly.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {
namespace {

constexpr int kSelfTestCols = 512;   // TMEM columns: D from column 0, 64, 128 or 192; A in [384,512)

__global__ void __launch_bounds__(128) tc05_selftest_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                            float* __restrict__ D, int N, int K, int mode,
                                                            int* __restrict__ status, int* __restrict__ dev_err) {
  extern __shared__ __align__(128) unsigned char smem[];
  const bool bf = (mode & 1) != 0;                 // 16-bit operands: bf16, or fp16 with bit 8
  const bool h16 = (mode & 256) != 0;
  const int E = bf ? 2 : 4;
  const uint32_t kbytes = static_cast<uint32_t>(K * E);
  const uint32_t sbo = (kbytes / 16) * 128;
  unsigned char* sA = smem;
  unsigned char* sB = smem + 128 * kbytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sB + static_cast<size_t>(N) * kbytes);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;

  // K-major: sbo per 8 rows, lbo 128.  MN-major: sbo 128 per 16 bytes of
  // M/N, lbo per 8 K-rows = the whole M/N extent.
  const bool a_mn = (mode & 8) != 0, b_mn = (mode & 16) != 0;
  const uint32_t lboA_mn = static_cast<uint32_t>(128 * E / 16) * 128;
  const uint32_t lboB_mn = static_cast<uint32_t>(N * E / 16) * 128;
  for (int idx = tid; idx < 128 * K; idx += 128) {
    const int r = idx / K, k = idx - r * K;
    const uint32_t off = a_mn ? tc::mnmajor_offset(r, k, E, 128, lboA_mn) : tc::kmajor_offset(r, k, E, sbo);
    if (bf && h16) *reinterpret_cast<__half*>(sA + off) = __float2half_rn(A[idx]);
    else if (bf) *reinterpret_cast<__nv_bfloat16*>(sA + off) = __float2bfloat16_rn(A[idx]);
    else *reinterpret_cast<float*>(sA + off) = A[idx];
  }
  for (int idx = tid; idx < N * K; idx += 128) {
    const int r = idx / K, k = idx - r * K;
    const uint32_t off = b_mn ? tc::mnmajor_offset(r, k, E, 128, lboB_mn) : tc::kmajor_offset(r, k, E, sbo);
    if (bf && h16) *reinterpret_cast<__half*>(sB + off) = __float2half_rn(B[idx]);
    else if (bf) *reinterpret_cast<__nv_bfloat16*>(sB + off) = __float2bfloat16_rn(B[idx]);
    else *reinterpret_cast<float*>(sB + off) = B[idx];
  }
  ptx::fence_proxy_async_smem();
  if (warp == 0) {
    tc::tmem_alloc(slot, kSelfTestCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    ptx::mbar_init(bar, 1);
    ptx::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t base = *slot;
  const uint32_t tD = base + ((mode & 32) ? 64 : 0) + ((mode & 64) ? 128 : 0);
  const uint32_t tA = base + 384;

  if (mode & 4) {       // A into tensor memory: row r = lane r, one tf32 per column
    for (int c = 0; c < K; c += 16) {
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = A[static_cast<size_t>(tid) * K + c + i];
      tc::tmem_st16(tc::tmem_addr(tA, warp, c), v);
    }
    tc::tmem_st_wait();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }

  // timeout mode: nothing is committed to the barrier; a small poll budget
  const bool no_mma = (mode & 128) != 0;
  const uint32_t limit = no_mma ? (1u << 12) : ptx::kSpinLimit;
  if (tid == 0 && !no_mma) {
    const uint32_t idesc = tc::instr_desc(bf ? (h16 ? tc::kF16 : tc::kBF16) : tc::kTF32, 128, N, (mode & 2) != 0,
                                          false, a_mn, b_mn);
    const int steps = static_cast<int>(kbytes / 32);
    const int kgroups = bf ? 2 : 1;                 // K groups of 8 per MMA
    for (int j = 0; j < steps; ++j) {
      const uint64_t bd = b_mn ? tc::smem_desc(ptx::smem_u32(sB) + j * kgroups * lboB_mn, lboB_mn, 128)
                               : tc::smem_desc(ptx::smem_u32(sB) + j * 256, 128, sbo);
      if (mode & 4) {
        tc::mma_ts_tf32(tD, tA + j * 8, bd, idesc, j > 0);
      } else {
        const uint64_t ad = a_mn ? tc::smem_desc(ptx::smem_u32(sA) + j * kgroups * lboA_mn, lboA_mn, 128)
                                 : tc::smem_desc(ptx::smem_u32(sA) + j * 256, 128, sbo);
        if (bf) tc::mma_ss<tc::kBF16>(tD, ad, bd, idesc, j > 0);   // kind::f16: bf16 or fp16 by idesc
        else tc::mma_ss<tc::kTF32>(tD, ad, bd, idesc, j > 0);
      }
    }
    tc::mma_commit(bar);
  }
  bool ok = ptx::mbar_wait(bar, 0, limit);
  tc::fence_after_sync();
  if (__syncthreads_and(ok)) {
    for (int c = 0; c < N; c += 16) {
      float v[16];
      tc::tmem_ld16(tc::tmem_addr(tD, warp, c), v);
      tc::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) D[static_cast<size_t>(tid) * N + c + i] = v[i];
    }
  } else {
    if (tid == 0) {
      *status = 1;
      atomicExch(dev_err, 1);
    }
    ok = ptx::mbar_wait(bar, 0, limit);   // give an MMA in flight another bounded chance to land
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(base, kSelfTestCols);
}

// CTA-pair self-test: a cluster of two CTAs computes D (128 x N) = A B^T with
// tcgen05.mma.cta_group::2 (M = 128, tf32), the form the pair scan of the
// chunked prefill uses.  CTA r holds A rows 64r .. 64r+63 and B rows
// (N/2) r .. (N/2) r + N/2 - 1 in its own shared memory (K-major, same
// offsets in both CTAs); the leader issues the MMAs and commits to both
// CTAs' barriers.  Each CTA writes its tensor memory as it lies -- 128 lanes
// x N/2 columns -- to raw[r], so the host checks the accumulator layout.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128)
    tc05_pair_selftest_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ raw,
                              int N, int K, int* __restrict__ status, int* __restrict__ dev_err) {
  extern __shared__ __align__(128) unsigned char smem[];
  const uint32_t rank = ptx::cluster_ctarank();
  const uint32_t kbytes = static_cast<uint32_t>(K * 4);
  const uint32_t sbo = (kbytes / 16) * 128;
  const int nh = N / 2;
  unsigned char* sA = smem;
  unsigned char* sB = smem + 64 * kbytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sB + static_cast<size_t>(nh) * kbytes);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  for (int idx = tid; idx < 64 * K; idx += 128) {
    const int r = idx / K, k = idx - r * K;
    *reinterpret_cast<float*>(sA + tc::kmajor_offset(r, k, 4, sbo)) = A[(64 * rank + r) * K + k];
  }
  for (int idx = tid; idx < nh * K; idx += 128) {
    const int r = idx / K, k = idx - r * K;
    *reinterpret_cast<float*>(sB + tc::kmajor_offset(r, k, 4, sbo)) = B[(nh * rank + r) * K + k];
  }
  ptx::fence_proxy_async_smem();
  if (warp == 0) {
    tc::tmem_alloc_pair(slot, 128);
    tc::tmem_relinquish_pair();
  }
  if (tid == 0) {
    ptx::mbar_init(bar, 1);
    ptx::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  ptx::cluster_sync();                 // both CTAs' operands, barrier and tensor memory are ready
  tc::fence_after_sync();
  const uint32_t tD = *slot;
  if (rank == 0 && tid == 0) {
    const uint32_t idesc = tc::instr_desc(tc::kTF32, 128, N);
    for (int j = 0; j < K / 8; ++j)
      tc::mma_tf32_pair(tD, tc::smem_desc(ptx::smem_u32(sA) + j * 256, 128, sbo),
                        tc::smem_desc(ptx::smem_u32(sB) + j * 256, 128, sbo), idesc, j > 0);
    tc::mma_commit_pair(bar, 3);
  }
  const bool ok = ptx::mbar_wait_cluster(bar, 0);
  tc::fence_after_sync();
  if (__syncthreads_and(ok)) {
    for (int c = 0; c < nh; c += 16) {
      float v[16];
      tc::tmem_ld16(tc::tmem_addr(tD, warp, c), v);
      tc::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) raw[(static_cast<size_t>(rank) * 128 + tid) * nh + c + i] = v[i];
    }
  } else if (tid == 0) {
    *status = 1;
    atomicExch(dev_err, 1);
  }
  tc::fence_before_sync();
  __syncthreads();
  ptx::cluster_sync();                 // no CTA frees its tensor memory or exits while the pair is busy
  if (warp == 0) tc::tmem_dealloc_pair(tD, 128);
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_tc05_pair_selftest(const float* A, const float* B, float* raw, int N, int K, int* status,
                                      void* stream) {
  clear_error();
  if (N < 32 || N > 256 || N % 32 || K < 8 || K > 128 || K % 8)
    return fail(GDN_ERR_SHAPE, "N=%d K=%d: need N a multiple of 32 in [32, 256], K a multiple of 8 in [8, 128]", N,
                K);
  if (!A || !B || !raw || !status) return fail(GDN_ERR_NULL, "A, B, raw and status are required");
  if (!aligned(A, 4) || !aligned(B, 4) || !aligned(raw, 4) || !aligned(status, 4))
    return fail(GDN_ERR_ALIGN, "buffers must be 4-byte aligned");
  const size_t smem = static_cast<size_t>(64 + N / 2) * K * 4 + 16;
  int* dev_err = nullptr;
  int rc = device_error_ptr(&dev_err);
  if (rc != GDN_OK) return rc;
  rc = cuda_status(cudaFuncSetAttribute(tc05_pair_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)),
                   "tc05 pair self-test smem attribute");
  if (rc != GDN_OK) return rc;
  tc05_pair_selftest_kernel<<<2, 128, smem, static_cast<cudaStream_t>(stream)>>>(A, B, raw, N, K, status, dev_err);
  return cuda_status(cudaGetLastError(), "tc05 pair self-test launch");
}

extern "C" int gdn_tc05_selftest(const float* A, const float* B, float* D, int N, int K, int mode,
                                 int* status, void* stream) {
  clear_error();
  if (mode & ~511) return fail(GDN_ERR_FLAGS, "unknown mode bits 0x%x", mode & ~511);
  if ((mode & 256) && !(mode & 1)) return fail(GDN_ERR_FLAGS, "fp16 operands (bit 8) go with bit 0");
  if ((mode & 128) && (mode & 127)) return fail(GDN_ERR_FLAGS, "the timeout mode (bit 7) takes no other bit");
  if ((mode & 4) && (mode & 1)) return fail(GDN_ERR_FLAGS, "A from tensor memory is tested with tf32 only");
  if ((mode & 4) && (mode & 8)) return fail(GDN_ERR_FLAGS, "A from tensor memory has no MN-major form");
  // MN-major operands are exercised with bf16 only: on sm_100a with this
  // toolchain kind::tf32 with an MN-major operand completed with an all-zero
  // result, so no kernel of this library uses that combination.
  if ((mode & 24) && !(mode & 1)) return fail(GDN_ERR_FLAGS, "MN-major operands are tested with bf16 only");
  const int dcol = ((mode & 32) ? 64 : 0) + ((mode & 64) ? 128 : 0);
  if (N < 16 || N > 256 || N % 16 || K < 16 || K > 128 || K % 16 || dcol + N > 384)
    return fail(GDN_ERR_SHAPE, "N=%d K=%d at column %d: need multiples of 16, N <= 256, K <= 128, D below column 384",
                N, K, dcol);
  if (!A || !B || !D || !status) return fail(GDN_ERR_NULL, "A, B, D and status are required");
  if (!aligned(A, 4) || !aligned(B, 4) || !aligned(D, 4) || !aligned(status, 4))
    return fail(GDN_ERR_ALIGN, "buffers must be 4-byte aligned");
  const int E = (mode & 1) ? 2 : 4;
  const size_t smem = static_cast<size_t>(128 + N) * K * E + 16;
  int* dev_err = nullptr;
  int rc = device_error_ptr(&dev_err);
  if (rc != GDN_OK) return rc;
  rc = cuda_status(cudaFuncSetAttribute(tc05_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem)),
                       "tc05 self-test smem attribute");
  if (rc != GDN_OK) return rc;
  tc05_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(A, B, D, N, K, mode, status, dev_err);
  return cuda_status(cudaGetLastError(), "tc05 self-test launch");
}
