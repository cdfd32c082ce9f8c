// The Gated DeltaNet block's projections on the sm_100a tensor cores:
//
//   * gdn_gemm_bf16:     C = A B^T  (A (M, K), B (N, K) bf16 row-major, fp32
//                        accumulation, bf16 C; optionally the last columns as
//                        fp32 to a second buffer) -- in_proj_z / in_proj_a /
//                        in_proj_b (cpp/src/model.cpp:174-176, 608-609, 625)
//                        and out_proj (cpp/src/model.cpp:177, 641);
//   * gdn_in_proj_conv:  y = silu(conv1d(x W_qkv^T, window)) -- in_proj_qkv
//                        (cpp/src/model.cpp:173, 586) with the causal depthwise
//                        conv (kernel 4) and SiLU (cpp/src/model.cpp:385-395,
//                        587-588) in the epilogue, so the projection output
//                        never goes to HBM.
//
// One persistent CTA per SM walks the output tiles (128 rows x 256 columns;
// the rows of consecutive tiles share A and sweep B, so A streams from HBM
// once and B stays in L2).  Warp roles: warp 0 issues TMA loads of A and B
// K-blocks (64 bf16 = 128 bytes wide, 128-byte swizzle) into a 4-stage ring;
// warp 1 owns the tensor memory and its lane 0 issues tcgen05.mma (kind::f16,
// M = 128, N = 256, K = 16) into one of two 256-column accumulators; warps 2-5
// drain the other accumulator (tcgen05.ld) and store it, so a tile's
// epilogue runs under the next tile's MMAs.  Every wait is bounded.
//
// The conv epilogue needs the 3 projection rows before each tile's first
// token: its tiles overlap by those rows (a tile computes rows t0-3 .. t0+124
// and writes tokens t0 .. t0+124), the 2.4% extra MMA work buying a fused
// conv with no halo exchange between CTAs.  Channel chunks of 32 go through a
// shared-memory row buffer (bf16, the projection's own rounding) from which
// each thread forms its token's 4 taps, exactly as gdn_conv1d_fwd does.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "gdn_conv_math.cuh"
#include "gdn_internal.h"
#include "gdn_ptx.cuh"

namespace gdn {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;          // accumulator rows per CTA, columns, K block
constexpr int kGemmThreads = 192;                      // producer, MMA, 4 epilogue warps
constexpr uint32_t kTileA = kBM * kBK * 2;             // 16 KiB
constexpr uint32_t kConvRow = 80;                      // 32 bf16 + 16 B pad: conflict-free 16-byte rows
constexpr int kHalo = 3;                               // conv kernel 4 -> 3 rows before each token
constexpr int kConvTileRows = kBM - kHalo;             // tokens written per CTA tile in the conv epilogue

// Shared-memory map of one CTA.  Single CTA: 4 stages of A (128 x 64) and B
// (256 x 64).  CTA pair: 6 stages of A (128 x 64) and half of B (128 x 64).
template <bool PAIR>
struct Layout {
  static constexpr int kStages = PAIR ? 6 : 4;
  static constexpr uint32_t kTileB = (PAIR ? kBN / 2 : kBN) * kBK * 2;
  static constexpr uint32_t kOffB = kStages * kTileA;
  static constexpr uint32_t kOffStage = kOffB + kStages * kTileB;   // conv row buffers (2 x 128 rows x 80 B)
  static constexpr uint32_t kOffBars = kOffStage + 2 * kBM * kConvRow;
  static constexpr uint32_t kSmem = kOffBars + 256 + 1024;          // barriers; 1 KiB to align the base
};
static_assert(Layout<false>::kSmem <= 232448 && Layout<true>::kSmem <= 232448, "gemm: shared memory per CTA");

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles;
  long long tiles;
  int group;             // row bands per raster group (tile_coords)
  // plain epilogue
  __nv_bfloat16* C;
  long long ldc;
  float* C32;            // columns >= n_f32 go here as fp32 (bf16-rounded) instead, or null
  long long ld32;
  int n_f32;
  // conv epilogue
  const __nv_bfloat16* conv_w;      // (N, 4)
  const __nv_bfloat16* state_in;    // (B, 3, N) or null (zeros)
  __nv_bfloat16* state_out;         // (B, 3, N) or null
  const int32_t* cu;                // (B + 1) or null: uniform B x T
  int B, T;
  int* err;
};

__device__ __forceinline__ int seq_of_tok(const int32_t* cu, int B, long long tok) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= tok) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Element (row, c >= n_f32) of the fp32 tail: its columns form a stack of
// (M, ld32) matrices, column j = c - n_f32 in matrix j / ld32.
__device__ __forceinline__ float* f32_at(const GemmParams& p, long long row, int c) {
  const int j = c - p.n_f32;
  const int blk = j / static_cast<int>(p.ld32);
  return p.C32 + (static_cast<long long>(blk) * p.M + row) * p.ld32 + (j - blk * static_cast<int>(p.ld32));
}

// Tile t -> (row band mt, column tile nt).  Bands go in groups of p.group:
// inside a group the column tiles are the outer index.  group = 1 is plain
// band order: the tiles in flight (one per SM) share a few A bands and sweep
// all of B, which then has to stay in L2; a larger group makes them share one
// group of A bands and a few B column slices instead, at the price of reading
// B from HBM once per group (the host picks it from the size of B).
__device__ __forceinline__ void tile_coords(const GemmParams& p, long long t, int& mt, int& nt) {
  const long long per_group = static_cast<long long>(p.group) * p.n_tiles;
  const int g = static_cast<int>(t / per_group);
  const long long j = t - g * per_group;
  const int bands = min(p.group, p.m_tiles - g * p.group);   // the last group may be short
  nt = static_cast<int>(j / bands);
  mt = g * p.group + static_cast<int>(j - static_cast<long long>(nt) * bands);
}

// CTA pairs (PAIR): a cluster of 2 CTAs computes a 256 x 256 tile with
// tcgen05 cta_group::2 -- each CTA loads its own 128 A rows and 128 of the
// 256 B rows into its shared memory (no multicast), the pair's leader issues
// the M = 256 MMAs, and each CTA's tensor memory holds its 128 accumulator
// rows.  Both CTAs' loads complete on the leader's stage barrier; the
// leader's commits arrive on both CTAs' stage-free and accumulator-ready
// barriers; both CTAs' epilogue warps report a drained accumulator to the
// leader.  Per SM this halves the B operand traffic of the single-CTA tile.
template <bool CONV, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
  using L = Layout<PAIR>;
  constexpr int kStages = L::kStages;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::kOffBars);   // [kStages] TMA -> MMA (the leader's counts both CTAs)
  uint64_t* empty = full + kStages;                                 // [kStages] MMA -> TMA
  uint64_t* tfull = empty + kStages;                                // [2] MMA -> epilogue
  uint64_t* tempty = tfull + 2;                                     // [2] epilogue -> MMA (the leader's counts both CTAs)
  volatile int* s_fail = reinterpret_cast<volatile int*>(tempty + 2);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(tempty + 3);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (p.K + kBK - 1) / kBK;
  const uint32_t rank = PAIR ? ptx::cluster_ctarank() : 0;
  const bool leader = rank == 0;
  const long long unit = PAIR ? (blockIdx.x >> 1) : blockIdx.x;       // this CTA's (pair's) first tile
  const long long units = PAIR ? (gridDim.x >> 1) : gridDim.x;
  // accumulator row 0 of this CTA: output row (plain) or token (conv, 3 halo rows first)
  auto row_base = [&](int mt) -> long long {
    if constexpr (CONV) return static_cast<long long>(mt) * (PAIR ? 2 * kConvTileRows : kConvTileRows) - kHalo +
                               static_cast<long long>(rank) * kConvTileRows;
    else return static_cast<long long>(mt) * (PAIR ? 2 * kBM : kBM) + static_cast<long long>(rank) * kBM;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(full + i, 1);
      ptx::mbar_init(empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(tfull + i, 1);
      ptx::mbar_init(tempty + i, PAIR ? 8 : 4);
    }
    *s_fail = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tc::tmem_alloc_pair(s_tmem, 512);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(s_tmem, 512);
      tc::tmem_relinquish();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if constexpr (PAIR) ptx::cluster_sync();     // both CTAs' barriers and tensor memory are ready
  tc::fence_after_sync();
  const uint32_t tbase = *s_tmem;

  // a bounded wait that also gives up once another role of this CTA has failed
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    for (uint32_t i = 0; i < ptx::kSpinLimit; ++i) {
      if (ptx::mbar_try_wait(bar, parity)) return true;
      if ((i & 1023) == 1023 && *s_fail) return false;
    }
    return false;
  };
  auto give_up = [&]() {
    *s_fail = 1;
    atomicExch(p.err, 1);
  };

  if (warp == 0) {
    // ---- TMA producer (each CTA loads its own A rows and B rows) ----
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int last[kStages];                         // parity of the last load into each stage, -1 for none
#pragma unroll
      for (int i = 0; i < kStages; ++i) last[i] = -1;
      for (long long t = unit; t < p.tiles && ok; t += units) {
        int mt, nt;
        tile_coords(p, t, mt, nt);
        const int row0 = static_cast<int>(row_base(mt));
        const int brow0 = nt * kBN + (PAIR ? static_cast<int>(rank) * (kBN / 2) : 0);
        for (int kb = 0; kb < nk; ++kb) {
          if (!wait(empty + s, ph ^ 1u)) { ok = false; break; }
          if constexpr (PAIR) {
            const uint32_t cl_full = ptx::mapa(ptx::smem_u32(full + s), 0);
            if (leader) ptx::mbar_arrive_expect_tx(full + s, 2 * (kTileA + L::kTileB));
            ptx::tma_load_2d_pair(sm + s * kTileA, &tmA, kb * kBK, row0, cl_full);
            ptx::tma_load_2d_pair(sm + L::kOffB + s * L::kTileB, &tmB, kb * kBK, brow0, cl_full);
          } else {
            ptx::mbar_arrive_expect_tx(full + s, kTileA + L::kTileB);
            ptx::tma_load_2d(sm + s * kTileA, &tmA, kb * kBK, row0, full + s);
            ptx::tma_load_2d(sm + L::kOffB + s * L::kTileB, &tmB, kb * kBK, brow0, full + s);
          }
          last[s] = static_cast<int>(ph);
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok) give_up();
      // no copy may land after the CTA has exited: the leader's stage barriers
      // count both CTAs' copies (the peer's exit waits for the leader at the
      // closing cluster barrier)
      if (leader) {
#pragma unroll
        for (int i = 0; i < kStages; ++i)
          if (last[i] >= 0) ptx::mbar_wait(full + i, static_cast<uint32_t>(last[i]));
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (the leader's lane 0) ----
    if (lane == 0 && leader) {
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      const uint32_t idesc = tc::instr_desc(tc::kBF16, PAIR ? 2 * kBM : kBM, kBN);
      const uint32_t a0 = ptx::smem_u32(sm), b0 = ptx::smem_u32(sm + L::kOffB);
      for (long long t = unit; t < p.tiles && ok; t += units, ++it) {
        const int acc = it & 1;
        if (!wait(tempty + acc, ((it >> 1) & 1) ^ 1u)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t d = tbase + acc * kBN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!wait(full + s, ph)) { ok = false; break; }
          tc::fence_after_sync();
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = tc::smem_desc_sw128(a0 + s * kTileA + k * 32);
            const uint64_t bd = tc::smem_desc_sw128(b0 + s * L::kTileB + k * 32);
            if constexpr (PAIR) tc::mma_bf16_pair(d, ad, bd, idesc, (kb | k) != 0);
            else tc::mma_ss<tc::kBF16>(d, ad, bd, idesc, (kb | k) != 0);
          }
          // the stage is free (in both CTAs) once these MMAs have read it
          if constexpr (PAIR) tc::mma_commit_pair(empty + s, 3);
          else tc::mma_commit(empty + s);
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
        if (ok) {                               // the accumulator is complete
          if constexpr (PAIR) tc::mma_commit_pair(tfull + acc, 3);
          else tc::mma_commit(tfull + acc);
        }
      }
      if (!ok) give_up();
      // drain: every MMA issued has completed before the tensor memory is released
      if (it > 0) ptx::mbar_wait(tfull + ((it - 1) & 1), ((it - 1) >> 1) & 1);
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 of this CTA ----
    const int q = warp & 3;
    const int r = q * 32 + lane;                 // accumulator row of this thread
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t cl_tempty0 = PAIR ? ptx::mapa(ptx::smem_u32(tempty), 0) : 0;
    int it = 0;
    bool ok = true;
    for (long long t = unit; t < p.tiles && ok; t += units, ++it) {
      const int acc = it & 1;
      int mt, nt;
      tile_coords(p, t, mt, nt);
      ok = wait(tfull + acc, (it >> 1) & 1);
      if (!ok) break;
      tc::fence_after_sync();
      const int col0 = nt * kBN;
      if constexpr (!CONV) {
        const long long row = row_base(mt) + r;
        const bool live = row < p.M;
#pragma unroll 1
        for (int cc = 0; cc < kBN; cc += 32) {
          float v[32];
          tc::tmem_ld16(lane_base + acc * kBN + cc, *reinterpret_cast<float(*)[16]>(v));
          tc::tmem_ld16(lane_base + acc * kBN + cc + 16, *reinterpret_cast<float(*)[16]>(v + 16));
          tc::tmem_ld_wait();
          const int c0 = col0 + cc;
          if (!live || c0 >= p.N) continue;
          if (p.C32 && c0 >= p.n_f32) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c0 + e < p.N) *f32_at(p, row, c0 + e) = __bfloat162float(__float2bfloat16_rn(v[e]));
          } else {
            __nv_bfloat16* dst = p.C + row * p.ldc + c0;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              if (c0 + g * 8 >= p.N || (p.C32 && c0 + g * 8 >= p.n_f32)) break;
              uint4 u;
              uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[g * 8 + 2 * e], v[g * 8 + 2 * e + 1]);
                w[e] = *reinterpret_cast<const uint32_t*>(&h);
              }
              *reinterpret_cast<uint4*>(dst + g * 8) = u;
            }
            if (p.C32) {                         // a chunk straddling n_f32: its fp32 tail
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (c0 + e < p.N && c0 + e >= p.n_f32) *f32_at(p, row, c0 + e) = __bfloat162float(__float2bfloat16_rn(v[e]));
            }
          }
        }
      } else {
        const long long tok = row_base(mt) + r;
        const bool out = r >= kHalo && tok < p.M;
        int seq = 0;
        long long st = 0, en = 0;
        if (out) {
          if (p.cu) {
            seq = seq_of_tok(p.cu, p.B, tok);
            st = p.cu[seq];
            en = p.cu[seq + 1];
          } else {
            seq = static_cast<int>(tok / p.T);
            st = static_cast<long long>(seq) * p.T;
            en = st + p.T;
          }
        }
#pragma unroll 1
        for (int cc = 0; cc < kBN; cc += 32) {
          unsigned char* buf = sm + L::kOffStage + ((cc >> 5) & 1) * (kBM * kConvRow);
          {
            float v[32];
            tc::tmem_ld16(lane_base + acc * kBN + cc, *reinterpret_cast<float(*)[16]>(v));
            tc::tmem_ld16(lane_base + acc * kBN + cc + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tc::tmem_ld_wait();
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 u;
              uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[g * 8 + 2 * e], v[g * 8 + 2 * e + 1]);
                w[e] = *reinterpret_cast<const uint32_t*>(&h);
              }
              *reinterpret_cast<uint4*>(buf + r * kConvRow + g * 16) = u;
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");   // the 4 epilogue warps
          const int c0 = col0 + cc;
          if (out && c0 < p.N) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const int c = c0 + g * 8;
              if (c >= p.N) break;
              // taps of channels c .. c+7: w (N, 4) -> w[tap][e]
              float w[4][8];
              {
                const uint4* wp = reinterpret_cast<const uint4*>(p.conv_w + static_cast<long long>(c) * 4);
#pragma unroll
                for (int qd = 0; qd < 4; ++qd) {
                  const uint4 raw = __ldg(wp + qd);
                  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
                  for (int e2 = 0; e2 < 4; ++e2) {
                    const float2 f = __bfloat1622float2(h[e2]);
                    const int flat = qd * 8 + 2 * e2;           // = channel offset * 4 + tap
                    w[flat % 4][flat / 4] = f.x;
                    w[(flat + 1) % 4][(flat + 1) / 4] = f.y;
                  }
                }
              }
              // window rows tok-3 .. tok-1 (sequence rows from the buffer, earlier ones from the carried window)
              float win[3][8], xv[8];
#pragma unroll
              for (int j = 0; j < 3; ++j) {
                const long long u = tok - kHalo + j;
                uint4 raw = make_uint4(0, 0, 0, 0);
                if (u >= st) raw = *reinterpret_cast<const uint4*>(buf + (r - kHalo + j) * kConvRow + g * 16);
                else if (p.state_in)
                  raw = *reinterpret_cast<const uint4*>(p.state_in + (static_cast<long long>(seq) * 3 + (u - st + 3)) * p.N + c);
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
                for (int e2 = 0; e2 < 4; ++e2) {
                  const float2 f = __bfloat1622float2(h[e2]);
                  win[j][2 * e2] = f.x;
                  win[j][2 * e2 + 1] = f.y;
                }
              }
              {
                const uint4 raw = *reinterpret_cast<const uint4*>(buf + r * kConvRow + g * 16);
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
                for (int e2 = 0; e2 < 4; ++e2) {
                  const float2 f = __bfloat1622float2(h[e2]);
                  xv[2 * e2] = f.x;
                  xv[2 * e2 + 1] = f.y;
                }
              }
              uint4 o;
              uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
              for (int e2 = 0; e2 < 4; ++e2) {
                // the arithmetic of gdn_conv1d_fwd's fp32 mode, so the results match it bit for bit
                const int e = 2 * e2;
                const float2 a = silu2(conv_pair(
                    make_float2(win[0][e], win[0][e + 1]), make_float2(win[1][e], win[1][e + 1]),
                    make_float2(win[2][e], win[2][e + 1]), make_float2(xv[e], xv[e + 1]),
                    make_float2(w[0][e], w[0][e + 1]), make_float2(w[1][e], w[1][e + 1]),
                    make_float2(w[2][e], w[2][e + 1]), make_float2(w[3][e], w[3][e + 1])));
                const __nv_bfloat162 hh = __floats2bfloat162_rn(a.x, a.y);
                ow[e2] = *reinterpret_cast<const uint32_t*>(&hh);
              }
              *reinterpret_cast<uint4*>(p.C + tok * p.ldc + c) = o;
              if (p.state_out && tok == en - 1) {
                // the carried window: the last 3 rows of [state_in; x_seq]
#pragma unroll
                for (int rr = 0; rr < 3; ++rr) {
                  const long long u = tok - 2 + rr;
                  uint4 raw = make_uint4(0, 0, 0, 0);
                  if (u >= st) raw = *reinterpret_cast<const uint4*>(buf + (r - 2 + rr) * kConvRow + g * 16);
                  else if (p.state_in)
                    raw = *reinterpret_cast<const uint4*>(p.state_in + (static_cast<long long>(seq) * 3 + (u - st + 3)) * p.N + c);
                  *reinterpret_cast<uint4*>(p.state_out + (static_cast<long long>(seq) * 3 + rr) * p.N + c) = raw;
                }
              }
            }
          }
        }
      }
      // this warp is done with the accumulator (the leader counts both CTAs' warps)
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) ptx::mbar_arrive_cluster(cl_tempty0 + acc * 8);
        else ptx::mbar_arrive(tempty + acc);
      }
    }
    if (!ok && lane == 0) give_up();
  }
  tc::fence_before_sync();
  __syncthreads();
  if constexpr (PAIR) ptx::cluster_sync();     // the leader's MMAs into this CTA's tensor memory are done
  if (warp == 1) {
    if constexpr (PAIR) tc::tmem_dealloc_pair(tbase, 512);
    else tc::tmem_dealloc(tbase, 512);
  }
}

// The carried conv window of empty packed sequences: state_in (or zeros)
// unchanged; sequences with tokens get theirs from the epilogue of their last token.
__global__ void conv_window_empty_kernel(const __nv_bfloat16* state_in, __nv_bfloat16* state_out,
                                         const int32_t* cu, int N) {
  const int seq = blockIdx.y;
  if (cu[seq + 1] > cu[seq]) return;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * N / 8; i += gridDim.x * blockDim.x) {
    const long long off = static_cast<long long>(seq) * 3 * N + static_cast<long long>(i) * 8;
    *reinterpret_cast<uint4*>(state_out + off) =
        state_in ? *reinterpret_cast<const uint4*>(state_in + off) : make_uint4(0, 0, 0, 0);
  }
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (!cached[dev & 63]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev & 63] = n > 0 ? n : 148;
  }
  return cached[dev & 63];
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so that
// the library loads (and reports GDN_ERR_CUDA) on a machine without a driver.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* out) {
  void* fn = nullptr;
  const int rc = tensor_map_encoder(&fn);
  if (rc == GDN_OK) *out = reinterpret_cast<EncodeTiledFn>(fn);
  return rc;
}

// Tensor map of a row-major (rows, K) bf16 matrix with row stride ld
// elements, read in boxes of box_rows x 64 with the 128-byte swizzle.
int make_tmap(CUtensorMap* tm, const void* base, long long rows, long long K, long long ld, int box_rows) {
  EncodeTiledFn encode = nullptr;
  int rc = encode_fn(&encode);
  if (rc != GDN_OK) return rc;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GDN_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return GDN_OK;
}

int gemm_args(const void* A, const void* B, int M, int N, int K, long long lda, long long ldb) {
  if (M < 0 || N <= 0 || K <= 0) return fail(GDN_ERR_SHAPE, "bad sizes M=%d N=%d K=%d", M, N, K);
  if (M > 0 && (!A || !B)) return fail(GDN_ERR_NULL, "A and B are required");
  if (K % 8 || lda % 8 || ldb % 8 || lda < K || ldb < K)
    return fail(GDN_ERR_SHAPE, "K and the row strides of A, B must be multiples of 8 elements, at least K");
  if (!aligned(A, 16) || !aligned(B, 16)) return fail(GDN_ERR_ALIGN, "A and B must be 16-byte aligned");
  return GDN_OK;
}

// Launch on a CTA pair per 256 x 256 tile when there are enough of them to
// fill the GPU, else on single CTAs with 128 x 256 tiles.
template <bool CONV>
int launch_gemm(const void* A, const void* B, long long lda, long long ldb, GemmParams& p, long long a_rows,
                cudaStream_t st) {
  static std::mutex mu;
  static bool attr[2][2][64] = {{{false}}};
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != GDN_OK) return rc;
  const int sms = sm_count();
  const long long rows_per_tile = CONV ? kConvTileRows : kBM;
  const long long pair_tiles = (p.M + 2 * rows_per_tile - 1) / (2 * rows_per_tile) * p.n_tiles;
  const bool pair = pair_tiles >= sms / 2;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr[CONV][pair][dev & 63]) {
      rc = pair ? cuda_status(cudaFuncSetAttribute(gemm_kernel<CONV, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(Layout<true>::kSmem)),
                              "gemm smem attribute")
                : cuda_status(cudaFuncSetAttribute(gemm_kernel<CONV, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(Layout<false>::kSmem)),
                              "gemm smem attribute");
      if (rc != GDN_OK) return rc;
      attr[CONV][pair][dev & 63] = true;
    }
  }
  rc = device_error_ptr(&p.err);
  if (rc != GDN_OK) return rc;
  p.m_tiles = static_cast<int>((p.M + (pair ? 2 : 1) * rows_per_tile - 1) / ((pair ? 2 : 1) * rows_per_tile));
  p.tiles = static_cast<long long>(p.m_tiles) * p.n_tiles;
  // B larger than ~80 MB does not stay in L2 next to the A bands in flight:
  // group about 40 MB of A tile rows and read B once per group
  const double b_bytes = static_cast<double>(p.N) * p.K * 2;
  const double band_bytes = static_cast<double>((pair ? 2 : 1) * kBM) * p.K * 2;
#ifdef GDN_GEMM_GROUP
  p.group = GDN_GEMM_GROUP;                    // tuning builds only
  (void)b_bytes;
  (void)band_bytes;
#else
  p.group = b_bytes > 80e6 ? static_cast<int>(40e6 / band_bytes + 0.5) : 1;
#endif
  if (p.group > p.m_tiles) p.group = p.m_tiles;
  if (p.group < 1) p.group = 1;
  CUtensorMap ta, tb;
  rc = make_tmap(&ta, A, a_rows, p.K, lda, kBM);
  if (rc != GDN_OK) return rc;
  rc = make_tmap(&tb, B, p.N, p.K, ldb, pair ? kBN / 2 : kBN);
  if (rc != GDN_OK) return rc;
  if (!pair) {
    const long long grid = p.tiles < sms ? p.tiles : sms;
    gemm_kernel<CONV, false><<<static_cast<unsigned>(grid), kGemmThreads, Layout<false>::kSmem, st>>>(ta, tb, p);
    return cuda_status(cudaGetLastError(), "gemm launch");
  }
  const long long pairs = p.tiles < sms / 2 ? p.tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = Layout<true>::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, gemm_kernel<CONV, true>, ta, tb, p), "gemm pair launch");
}

}  // namespace

int tensor_map_encoder(void** out) {
  static std::once_flag once;
  static void* fn = nullptr;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = p;
  });
  if (!fn) return err != cudaSuccess ? cuda_status(err, "cuTensorMapEncodeTiled lookup")
                                     : fail(GDN_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  *out = fn;
  return GDN_OK;
}

}  // namespace gdn

using namespace gdn;

extern "C" int gdn_gemm_bf16(const void* A, const void* B, void* C, float* C32, int M, int N, int K, long long lda,
                             long long ldb, long long ldc, long long ld32, int n_f32, void* stream) {
  clear_error();
  int rc = gemm_args(A, B, M, N, K, lda, ldb);
  if (rc != GDN_OK) return rc;
  if (M > 0 && !C) return fail(GDN_ERR_NULL, "C is required");
  if (N % 8) return fail(GDN_ERR_SHAPE, "N=%d must be a multiple of 8", N);
  if (ldc % 8 || ldc < (C32 ? (n_f32 < N ? n_f32 : N) : N) || !aligned(C, 16))
    return fail(GDN_ERR_SHAPE, "C: row stride a multiple of 8 elements covering its columns, 16-byte aligned");
  if (C32) {
    if (n_f32 < 0 || n_f32 > N || n_f32 % 8 || ld32 <= 0 || !aligned(C32, 4))
      return fail(GDN_ERR_SHAPE, "C32: n_f32 in [0, N] and a multiple of 8, ld32 > 0");
  }
  if (M == 0) return GDN_OK;
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.n_tiles = (N + kBN - 1) / kBN;
  p.C = static_cast<__nv_bfloat16*>(C);
  p.ldc = ldc;
  p.C32 = C32;
  p.ld32 = ld32;
  p.n_f32 = C32 ? n_f32 : N;
  return launch_gemm<false>(A, B, lda, ldb, p, M, static_cast<cudaStream_t>(stream));
}

extern "C" int gdn_in_proj_conv(const void* x, const void* W, const void* conv_w, const void* state_in,
                                void* state_out, void* y, const int32_t* cu_seqlens, int B, int T, int N, int K,
                                long long ldx, long long ldw, long long ldy, void* stream) {
  clear_error();
  const long long M = cu_seqlens ? static_cast<long long>(T) : static_cast<long long>(B) * T;
  if (B < 0 || T < 0 || M > 0x7fffffffLL) return fail(GDN_ERR_SHAPE, "bad sizes B=%d T=%d", B, T);
  int rc = gemm_args(x, W, static_cast<int>(M), N, K, ldx, ldw);
  if (rc != GDN_OK) return rc;
  if (N % 8 || ldy % 8 || ldy < N) return fail(GDN_ERR_SHAPE, "N and ldy must be multiples of 8, ldy >= N");
  if (M > 0 && (!y || !conv_w)) return fail(GDN_ERR_NULL, "y and conv_w are required");
  if (!aligned(y, 16) || !aligned(conv_w, 16) || !aligned(state_in, 16) || !aligned(state_out, 16) ||
      !aligned(cu_seqlens, 4))
    return fail(GDN_ERR_ALIGN, "y, conv_w and the windows 16-byte aligned, cu_seqlens 4-byte aligned");
  const size_t ybytes = static_cast<size_t>(M) * ldy * 2, sbytes = static_cast<size_t>(B) * 3 * N * 2;
  if (overlap(y, ybytes, x, static_cast<size_t>(M) * ldx * 2) || overlap(state_out, sbytes, state_in, sbytes) ||
      overlap(state_out, sbytes, y, ybytes))
    return fail(GDN_ERR_ALIAS, "y, x and the windows must not overlap");
  if (M == 0 || B == 0) return GDN_OK;
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = N;
  p.K = K;
  p.n_tiles = (N + kBN - 1) / kBN;
  p.C = static_cast<__nv_bfloat16*>(y);
  p.ldc = ldy;
  p.conv_w = static_cast<const __nv_bfloat16*>(conv_w);
  p.state_in = static_cast<const __nv_bfloat16*>(state_in);
  p.state_out = static_cast<__nv_bfloat16*>(state_out);
  p.cu = cu_seqlens;
  p.B = B;
  p.T = T;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cu_seqlens && state_out) {
    conv_window_empty_kernel<<<dim3((3 * N / 8 + 255) / 256, B), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(state_in), static_cast<__nv_bfloat16*>(state_out), cu_seqlens, N);
    rc = cuda_status(cudaGetLastError(), "conv window launch");
    if (rc != GDN_OK) return rc;
  }
  return launch_gemm<true>(x, W, ldx, ldw, p, M, st);
}
