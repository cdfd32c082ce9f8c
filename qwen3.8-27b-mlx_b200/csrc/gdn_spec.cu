// On-device acceptance test of an MTP speculative-verify block, so that the
// rollback index reaches the next decode step without a host round trip.
//
// For each sequence b with k draft tokens d_i, draft distributions q_i and
// target distributions p_0 .. p_k (the verify pass), following the
// reference's rejection test (python/speculative.py:170-180,
// cpp/src/session.cpp:495-505) and residual (python/speculative.py:100-106):
//   accept_i = q_i[d_i] > 0 ? u_i * q_i[d_i] <= p_i[d_i] : p_i[d_i] > 0
//   j        = number of leading accepted drafts (0 .. k)
//   token    = a draw from p_k if j == k, else from max(p_j - q_j, 0) / sum
//              (p_j / sum(p_j) when that residual sums to <= 1e-12)
//   commit_n = j + 1, the DeltaCache::commit argument (cpp/src/session.cpp:507-511)
// The draw is by inverse CDF with a caller-given uniform w: the smallest v
// with w * total < sum_{x <= v} r[x] (the reference draws with MLX's
// categorical sampler; a fixed uniform makes the result reproducible).
// One CTA per sequence (a cluster of 8 for vocabularies of 64K entries and
// more); the row drawn from is read once for its block sums (coalesced) and
// once more for the 1024 entries around the draw (HBM-bound).
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kSpecThreads = 512;
constexpr int kMaxDraft = 32;
constexpr int kBlk = 1024;                  // vocabulary entries per warp block: 32 slices of 32
constexpr long long kMaxBlocks = 4096;      // block sums kept in shared memory (V <= 4M)

// Residual (or plain) probability of vocabulary entry x.
__device__ __forceinline__ float prob(const float* pj, const float* qj, long long x, bool resid) {
  return resid ? fmaxf(pj[x] - qj[x], 0.f) : pj[x];
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float warp_scan(float v, int lane) {   // inclusive
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float n = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += n;
  }
  return v;
}

// Sum of the distribution over warp block blk of 1024 entries (coalesced;
// 16-byte loads, 8 in flight per lane, when the rows allow), on every lane.
__device__ __forceinline__ float block_sum_one(const float* pj, const float* qj, long long V, bool resid, bool vec,
                                              long long blk, int lane) {
  float s = 0.f;
  if (vec && (blk + 1) * kBlk <= V) {
    const float4* p4 = reinterpret_cast<const float4*>(pj + blk * kBlk) + lane;
    const float4* q4 = reinterpret_cast<const float4*>(qj + blk * kBlk) + lane;
    float4 a[8], c[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = __ldg(p4 + i * 32);
    if (resid) {
#pragma unroll
      for (int i = 0; i < 8; ++i) c[i] = __ldg(q4 + i * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        s += fmaxf(a[i].x - c[i].x, 0.f) + fmaxf(a[i].y - c[i].y, 0.f) + fmaxf(a[i].z - c[i].z, 0.f) +
             fmaxf(a[i].w - c[i].w, 0.f);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) s += a[i].x + a[i].y + a[i].z + a[i].w;
    }
  } else {
    for (int i = 0; i < kBlk / 32; ++i) {
      const long long x = blk * kBlk + i * 32 + lane;
      s += x < V ? prob(pj, qj, x, resid) : 0.f;
    }
  }
  return warp_sum(s);
}

// Sums of the distribution over the warp blocks of 1024 entries, then their
// total, broadcast.
__device__ float block_sums(const float* pj, const float* qj, long long V, bool resid, bool vec, float* bsum,
                            float* s_tot) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long nb = (V + kBlk - 1) / kBlk;
  for (long long blk = warp; blk < nb; blk += kSpecThreads / 32) {
    const float s = block_sum_one(pj, qj, V, resid, vec, blk, lane);
    if (lane == 0) bsum[blk] = s;
  }
  __syncthreads();
  if (warp == 0) {
    float t = 0.f;
    for (long long blk = lane; blk < nb; blk += 32) t += bsum[blk];
    t = warp_sum(t);
    if (lane == 0) *s_tot = t;
  }
  __syncthreads();
  return *s_tot;
}

// Warp 0: the number of leading accepted drafts of sequence b (lanes >= k
// always accept; a draft outside [0, V) rejects and raises *err).
__device__ __forceinline__ int leading_accepted(const float* pb, const float* qb, const int32_t* draft,
                                                const float* u_accept, int b, int k, long long V, int32_t* err,
                                                int lane) {
  bool acc = true;
  if (lane < k) {
    const int d = draft[static_cast<size_t>(b) * k + lane];
    if (d < 0 || d >= V) {
      atomicExch(err, 1);
      acc = false;
    } else {
      const float pd = pb[static_cast<size_t>(lane) * V + d];
      const float qd = qb[static_cast<size_t>(lane) * V + d];
      acc = qd > 0.f ? u_accept[static_cast<size_t>(b) * k + lane] * qd <= pd : pd > 0.f;
    }
  }
  const unsigned rej = __ballot_sync(0xffffffffu, !acc);
  return rej ? __ffs(rej) - 1 : k;
}

// Warp 0: inverse CDF of the distribution with block sums bs(i).  The block
// holding the target is found by scanning the block sums 32 at a time; its
// 1024 entries are then staged in shared memory (stage, 32 x 33 floats) with
// every load in flight at once, lane l sums slice l, one scan over the 32
// slice sums picks the slice and one scan inside it picks the entry.  Where
// rounding of the differently ordered sums leaves the target past the chosen
// block's (or slice's) entries, the last entry with mass there is taken.
template <class BlockSum>
__device__ long long inverse_cdf(const float* pj, const float* qj, long long V, bool resid, float target,
                                 BlockSum bs, float* stage, int lane) {
  const long long nb = (V + kBlk - 1) / kBlk;
  float base = 0.f;
  long long blk = -1;
  for (long long c0 = 0; c0 < nb && blk < 0; c0 += 32) {
    const bool in = c0 + lane < nb;
    const float inc = warp_scan(in ? bs(c0 + lane) : 0.f, lane);
    const unsigned over = __ballot_sync(0xffffffffu, in && base + inc > target);
    if (over) {
      const int l = __ffs(over) - 1;
      const float before = __shfl_sync(0xffffffffu, inc, l > 0 ? l - 1 : 0);
      base += l > 0 ? before : 0.f;
      blk = c0 + l;
    } else {
      base += __shfl_sync(0xffffffffu, inc, 31);
    }
  }
  long long v = -1;
  if (blk >= 0) {
    float vals[kBlk / 32];
#pragma unroll
    for (int i = 0; i < kBlk / 32; ++i) {
      const long long x = blk * kBlk + i * 32 + lane;
      vals[i] = x < V ? prob(pj, qj, x, resid) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kBlk / 32; ++i) stage[i * 33 + lane] = vals[i];
    __syncwarp();
    float ssum = 0.f;                          // slice `lane`, in entry order
#pragma unroll 8
    for (int i = 0; i < 32; ++i) ssum += stage[lane * 33 + i];
    const float sinc = warp_scan(ssum, lane);
    const unsigned over = __ballot_sync(0xffffffffu, base + sinc > target);
    const int sl = over ? __ffs(over) - 1 : 31;
    base += sl > 0 ? __shfl_sync(0xffffffffu, sinc, sl > 0 ? sl - 1 : 0) : 0.f;
    const float e = stage[sl * 33 + lane];
    const long long x = blk * kBlk + sl * 32 + lane;
    const float inc = warp_scan(e, lane);
    const unsigned hit = __ballot_sync(0xffffffffu, x < V && base + inc > target);
    if (over && hit) {
      v = blk * kBlk + sl * 32 + __ffs(hit) - 1;
    } else {
      // the last entry with mass in the block
      for (int i = 31; i >= 0 && v < 0; --i) {
        const long long xi = blk * kBlk + i * 32 + lane;
        const unsigned pos = __ballot_sync(0xffffffffu, xi < V && stage[i * 33 + lane] > 0.f);
        if (pos) v = blk * kBlk + i * 32 + 31 - __clz(pos);
      }
    }
    __syncwarp();
  }
  if (v < 0) {
    // rounding left the target at or past the summed mass: the last entry with mass
    for (long long x0 = ((V - 1) / 32) * 32; x0 >= 0 && v < 0; x0 -= 32) {
      const long long x = x0 + lane;
      const unsigned pos = __ballot_sync(0xffffffffu, x < V && prob(pj, qj, x, resid) > 0.f);
      if (pos) v = x0 + 31 - __clz(pos);
    }
    if (v < 0) v = 0;
  }
  return v;
}

__global__ void __launch_bounds__(kSpecThreads) spec_verify_kernel(const float* __restrict__ p,
                                                                   const float* __restrict__ q,
                                                                   const int32_t* __restrict__ draft,
                                                                   const float* __restrict__ u_accept,
                                                                   const float* __restrict__ u_sample, int k,
                                                                   long long V, int32_t* accept_len,
                                                                   int32_t* commit_n, int32_t* token,
                                                                   int32_t* err) {
  extern __shared__ float bsum[];            // ceil(V / 1024) block sums
  __shared__ float s_stage[32 * 33];
  __shared__ float s_tot;
  __shared__ int s_j;
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const float* pb = p + static_cast<size_t>(b) * (k + 1) * V;
  const float* qb = q + static_cast<size_t>(b) * k * V;
  // 1. acceptance of the k drafts, first rejection
  if (tid < 32) {
    const int j = leading_accepted(pb, qb, draft, u_accept, b, k, V, err, tid);
    if (tid == 0) s_j = j;
  }
  __syncthreads();
  const int j = s_j;
  const float* pj = pb + static_cast<size_t>(j) * V;
  const float* qj = qb + static_cast<size_t>(j < k ? j : 0) * V;
  // 2. the distribution to draw from: residual of row j, or p_k (p_j if that residual is empty)
  bool resid = j < k;
  const bool vec = (V % 4 == 0) && (reinterpret_cast<uintptr_t>(p) % 16 == 0) && (reinterpret_cast<uintptr_t>(q) % 16 == 0);
  float total = block_sums(pj, qj, V, resid, vec, bsum, &s_tot);
  if (resid && !(total > 1e-12f)) {
    resid = false;
    total = block_sums(pj, qj, V, false, vec, bsum, &s_tot);
  }
  // 3. inverse CDF by warp 0
  if (tid < 32) {
    const long long v = inverse_cdf(pj, qj, V, resid, u_sample[b] * total, [&](long long i) { return bsum[i]; }, s_stage,
                                       tid);
    if (tid == 0) {
      token[b] = static_cast<int32_t>(v);
      accept_len[b] = j;
      commit_n[b] = j + 1;
    }
  }
}

// Large vocabularies: a cluster of kCluster CTAs per sequence shares the
// block-sum pass (CTA r sums blocks [r*per, (r+1)*per) into its own shared
// memory) and the sums are read across the cluster through distributed
// shared memory, so a batch of 32 sequences spreads over 256 SMs' worth of
// CTAs instead of 32.  Block sums and their total are formed exactly as in
// spec_verify_kernel, so the results are the same bits.
constexpr int kCluster = 8;

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kSpecThreads, 2)
    spec_verify_cluster_kernel(const float* __restrict__ p, const float* __restrict__ q,
                               const int32_t* __restrict__ draft, const float* __restrict__ u_accept,
                               const float* __restrict__ u_sample, int k, long long V, int32_t* accept_len,
                               int32_t* commit_n, int32_t* token, int32_t* err) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  extern __shared__ float bpart[];           // this CTA's share of the block sums, then all nb of them
  __shared__ float s_stage[32 * 33];
  __shared__ float s_tot;
  __shared__ int s_j;
  const unsigned rank = cl.block_rank();
  const int b = blockIdx.x / kCluster;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* pb = p + static_cast<size_t>(b) * (k + 1) * V;
  const float* qb = q + static_cast<size_t>(b) * k * V;
  if (tid < 32) {
    const int jj = leading_accepted(pb, qb, draft, u_accept, b, k, V, err, tid);
    if (tid == 0) s_j = jj;
  }
  __syncthreads();
  const int j = s_j;
  const float* pj = pb + static_cast<size_t>(j) * V;
  const float* qj = qb + static_cast<size_t>(j < k ? j : 0) * V;
  bool resid = j < k;
  const bool vec = (V % 4 == 0) && (reinterpret_cast<uintptr_t>(p) % 16 == 0) && (reinterpret_cast<uintptr_t>(q) % 16 == 0);
  const long long nb = (V + kBlk - 1) / kBlk;
  const long long per = (nb + kCluster - 1) / kCluster;
  const long long lo = static_cast<long long>(rank) * per;
  const long long hi = lo + per < nb ? lo + per : nb;
  auto partials = [&](bool rs) {
    for (long long blk = lo + warp; blk < hi; blk += kSpecThreads / 32) {
      const float sb = block_sum_one(pj, qj, V, rs, vec, blk, lane);
      if (lane == 0) bpart[blk - lo] = sb;
    }
  };
  auto bs = [&](long long i) -> float {
    return *cl.map_shared_rank(bpart + (i % per), static_cast<unsigned>(i / per));
  };
  float* ball = bpart + per;                  // a local copy of every block sum
  auto total_all = [&]() -> float {           // every CTA, the same order as block_sums
    if (tid < 32) {
      float t = 0.f;
#pragma unroll 4
      for (long long blk = lane; blk < nb; blk += 32) {
        const float sb = bs(blk);
        ball[blk] = sb;
        t += sb;
      }
      t = warp_sum(t);
      if (lane == 0) s_tot = t;
    }
    __syncthreads();
    return s_tot;
  };
  partials(resid);
  cl.sync();
  float total = total_all();
  if (resid && !(total > 1e-12f)) {           // the same decision in every CTA of the cluster
    resid = false;
    cl.sync();                                // every CTA has read the residual sums
    partials(false);
    cl.sync();
    total = total_all();
  }
  if (rank == 0 && tid < 32) {
    const long long v = inverse_cdf(pj, qj, V, resid, u_sample[b] * total, [&](long long i) { return ball[i]; },
                                    s_stage, lane);
    if (lane == 0) {
      token[b] = static_cast<int32_t>(v);
      accept_len[b] = j;
      commit_n[b] = j + 1;
    }
  }
  cl.sync();                                  // no CTA leaves while its block sums may still be read
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_spec_verify(const float* p, const float* q, const int32_t* draft, const float* u_accept,
                               const float* u_sample, int B, int k, long long V, int32_t* accept_len,
                               int32_t* commit_n, int32_t* token, int32_t* err_flag, void* stream) {
  clear_error();
  if (B < 0 || k < 1 || k > kMaxDraft || V < 1 || V > kMaxBlocks * kBlk)
    return fail(GDN_ERR_SHAPE, "B=%d k=%d V=%lld: need B >= 0, 1 <= k <= %d, 1 <= V <= %lld", B, k, V, kMaxDraft,
                kMaxBlocks * kBlk);
  if (B == 0) return GDN_OK;
  if (!p || !q || !draft || !u_accept || !u_sample || !accept_len || !commit_n || !token || !err_flag)
    return fail(GDN_ERR_NULL, "every pointer is required");
  if (!aligned(p, 4) || !aligned(q, 4) || !aligned(draft, 4) || !aligned(u_accept, 4) || !aligned(u_sample, 4) ||
      !aligned(accept_len, 4) || !aligned(commit_n, 4) || !aligned(token, 4) || !aligned(err_flag, 4))
    return fail(GDN_ERR_ALIGN, "buffers must be 4-byte aligned");
  const size_t smem = static_cast<size_t>((V + kBlk - 1) / kBlk) * sizeof(float);
  if (smem > 48 * 1024) {
    int rc = cuda_status(cudaFuncSetAttribute(spec_verify_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(smem)),
                         "spec verify smem attribute");
    if (rc != GDN_OK) return rc;
  }
  const long long nb = (V + kBlk - 1) / kBlk;
  if (nb >= 64 && static_cast<long long>(B) * kCluster <= 0x7fffffffLL) {
    const size_t psmem = static_cast<size_t>((nb + kCluster - 1) / kCluster + nb) * sizeof(float);
    spec_verify_cluster_kernel<<<static_cast<unsigned>(B) * kCluster, kSpecThreads, psmem,
                                 static_cast<cudaStream_t>(stream)>>>(p, q, draft, u_accept, u_sample, k, V,
                                                                      accept_len, commit_n, token, err_flag);
    return cuda_status(cudaGetLastError(), "spec verify (cluster) launch");
  }
  spec_verify_kernel<<<static_cast<unsigned>(B), kSpecThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      p, q, draft, u_accept, u_sample, k, V, accept_len, commit_n, token, err_flag);
  return cuda_status(cudaGetLastError(), "spec verify launch");
}
