// qf_w8a16.cu -- sm_100a W8A16 small-M GEMM and int8 draft LM head with fused row statistics.
//
// Replaces the Triton kernel `_w8a16_kernel` and its launcher of EurekaZang/qwen-a100-fastpath
// (plugin/qwen_fastpath/w8a16.py:15-44, :71-83) and the logits/argmax of the int8 draft head
// (plugin/qwen_fastpath/patches.py:157-185).
//
//   y[m, n] = scale[n] * sum_k x[m, k] * w[n, k]      x bf16 [M <= 16, K], w int8 [N, K] row-major
//
// The contraction streams N*K int8 weight bytes once and is bound by HBM bandwidth at these M.  Design:
//
// * Stream-K split: the iteration space (tile of 128 output channels) x (128-wide k stage) is cut into
//   G <= #SM equal contiguous ranges, one persistent CTA each, so every shape fills all SMs with no tail.
//   Tiles that straddle CTAs are reduced by the CTA that finishes last (fp32 partials in the workspace,
//   summed in CTA order, so results are deterministic), and the tile counter is reset for the next call.
//   No memset or cast launches (the reference zero-fills an fp32 buffer and casts, w8a16.py:78-79, :83).
// * One producer warp issues TMA loads (cp.async.bulk.tensor, 128-byte swizzle) of the weight box
//   [128 rows x 128 bytes] and of the two activation boxes [8*NT rows x 64 bf16] of a stage into a
//   mbarrier ring.  Weights carry an L2 evict-first hint; activations evict-last (every CTA reads them).
//   With programmatic dependent launch the weight boxes of the first stages are issued before
//   griddepcontrol.wait, i.e. while the previous kernel on the stream is still running.
// * Eight consumer warps: warp (q, h) owns rows [32q, 32q+32) of the tile and half of the 16-byte k
//   chunks of each stage.  Lane (g, t) takes chunk c = (t ^ h) | ((t & 1) << 2): with the 128B swizzle this
//   makes both the weight reads (16 B of rows g and g+8) and the activation reads conflict-free.  Weights
//   are converted int8 -> bf16 exactly in registers and fed to mma.sync m16n8k16 as the 16-row A operand
//   ("swap AB"); the M <= 16 tokens are the 8-column B operand (NT = 1 or 2 column tiles).  The k order
//   inside a chunk is permuted identically for A and B, which leaves the dot product unchanged.
// * Epilogue: fp32 accumulator * scale, one rounding to bf16 (or fp32 export), optional bias as a second
//   bf16 rounding exactly like the reference's `y + bias`.  The head epilogue also reduces the bf16 logits
//   of each tile to per-row (max, first argmax, sum exp) and the last tile to finish folds all tiles.
// * Every wait on an mbarrier is bounded (global timer); on expiry the CTA records QF_ERR_TIMEOUT in the
//   workspace, stops waiting and drains its own TMA copies before exiting.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/qf_b200.h"
#include "qf_ptx.cuh"

namespace qf {

constexpr int kBN = 128;                    // output channels per tile
constexpr int kBK = 128;                    // k per stage (int8 bytes of one swizzled weight-box row)
#ifndef QF_MT_PER_WARP
#define QF_MT_PER_WARP 1
#endif
constexpr int kMTiles = kBN / 16;                     // 16-row MMA tiles per 128-row tile
constexpr int kJ = QF_MT_PER_WARP;                    // m-tiles per consumer warp
constexpr int kConsumerWarps = 2 * kMTiles / kJ;      // each m-tile group is shared by two warps (k halves)
constexpr int kProducerWarp = kConsumerWarps;       // TMA issue (one lane)
constexpr int kConverterWarp = kConsumerWarps + 1;  // bf16 -> fp16 activations of each stage
constexpr int kThreads = (kConsumerWarps + 2) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kWStageBytes = kBN * kBK;     // 16 KiB
constexpr int kMaxGrid = 256;
constexpr int kMaxTiles = QF_MAX_N / kBN;   // tile-counter capacity
constexpr int kBarPairBase = 1;             // named barriers 1..8: warp pairs of an m-tile; 9: all consumers
constexpr int kBarConsumers = 9;
constexpr uint64_t kWaitBudgetNs = 4000000000ull;  // 4 s

// workspace layout (bytes); the prefix [0, kWsZeroBytes) must be zero before the first call
constexpr size_t kWsHeader = 256;                              // [0]: error flag, [1]: head tiles-done
constexpr size_t kWsCounters = kWsHeader;                       // int32[kMaxTiles]
constexpr size_t kWsZeroBytes = kWsCounters + sizeof(int) * kMaxTiles;
constexpr size_t kWsPartials = (kWsZeroBytes + 1023) / 1024 * 1024;
constexpr size_t kPartialSlotFloats = kBN * 16;                 // [128 rows][16 tokens]
constexpr size_t kWsStats = kWsPartials + sizeof(float) * kPartialSlotFloats * 2 * kMaxGrid;

template <int NT> struct Cfg {
  static constexpr int kStages = NT == 1 ? 5 : 4;
  static constexpr int kXBoxBytes = 8 * NT * 128;               // [8*NT rows][64 bf16]
  static constexpr int kXStageBytes = 2 * kXBoxBytes;
  static constexpr int kXPairs = kXStageBytes / 8;              // 8-byte blocks converted to fp16 per stage
  static constexpr int kOffX = kStages * kWStageBytes;
  static constexpr int kOffX16 = kOffX + kStages * kXStageBytes;
  static constexpr int kOffRed = kOffX16 + kStages * kXStageBytes;
  static constexpr int kRedBytes = (kConsumerWarps * 32 * 4 * NT * 4) > (kConsumerWarps * 16 * 16)
                                       ? kConsumerWarps * 32 * 4 * NT * 4 : kConsumerWarps * 16 * 16;
  static constexpr int kOffStat = kOffRed + kRedBytes;
  static constexpr int kStatBytes = kMTiles * 16 * 16;          // float4 per (m-tile, token)
  static constexpr int kOffBar = kOffStat + kStatBytes;         // full[S], empty[S], xready[S]
  static constexpr int kOffFlag = kOffBar + 3 * kStages * 8;    // abort, last, inexact[S]
  static constexpr int kSmemBytes = kOffFlag + 8 + 4 * kStages + 1024;  // + alignment slack
  static constexpr uint32_t kTxBytes = kWStageBytes + kXStageBytes;
};

struct Params {
  const float* scale;
  const __nv_bfloat16* bias;
  void* y;
  int64_t ldy;
  int y_f32;
  int M, N, K;
  int kiters, ntiles, T, G;
  uint8_t* ws;
  // head
  __nv_bfloat16* logits;
  int64_t ldl;
  int n_valid;
  long long vocab_offset;
  float* row_max;
  long long* row_argmax;
  float* row_lse;
  int f16_path;  // 1: convert activations to fp16 per stage (cheaper weight dequant); 0: exact bf16 path
};

struct RowStat {
  float m;  // max bf16 logit (as fp32)
  int a;    // its column (first on ties)
  float s;  // sum of exp(v - m)
};

__device__ __forceinline__ RowStat stat_combine(const RowStat& x, const RowStat& y) {
  RowStat r;
  r.m = fmaxf(x.m, y.m);
  r.a = (y.m > x.m || (y.m == x.m && y.a < x.a)) ? y.a : x.a;
  const float sx = (x.m == -INFINITY) ? 0.f : x.s * expf(x.m - r.m);
  const float sy = (y.m == -INFINITY) ? 0.f : y.s * expf(y.m - r.m);
  r.s = sx + sy;
  return r;
}

__device__ __forceinline__ RowStat stat_shfl_xor(const RowStat& v, int mask) {
  RowStat o;
  o.m = __shfl_xor_sync(0xffffffffu, v.m, mask);
  o.a = __shfl_xor_sync(0xffffffffu, v.a, mask);
  o.s = __shfl_xor_sync(0xffffffffu, v.s, mask);
  return o;
}

__device__ __forceinline__ long long split_start(int c, int T, int G) {
  return (static_cast<long long>(c) * T) / G;
}
// CTA whose range holds iteration i: largest c with split_start(c) <= i.
__device__ __forceinline__ int cta_of(int i, int T, int G) {
  return static_cast<int>(((static_cast<long long>(i) + 1) * G - 1) / T);
}

__device__ __forceinline__ void record_error(uint8_t* ws, int code) {
  atomicExch(reinterpret_cast<int*>(ws), code);
}

// Bounded mbarrier wait; gives up (returns false) after kWaitBudgetNs or once the CTA aborted.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (*abort_flag) return false;
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitBudgetNs) return false;
  }
}

// Output of one value of a finished tile (GEMM mode).
__device__ __forceinline__ void store_out(const Params& p, int n, int m, float v) {
  if (n >= p.N || m >= p.M) return;
  if (p.y_f32) {
    if (p.bias) v += __bfloat162float(p.bias[n]);
    static_cast<float*>(p.y)[static_cast<int64_t>(m) * p.ldy + n] = v;
  } else {
    __nv_bfloat16 r = __float2bfloat16_rn(v);
    if (p.bias) r = __float2bfloat16_rn(__bfloat162float(r) + __bfloat162float(p.bias[n]));
    static_cast<__nv_bfloat16*>(p.y)[static_cast<int64_t>(m) * p.ldy + n] = r;
  }
}

// One 16-k chunk (16 bytes of each of the rows g and g+8) of the lane's m-tile: four m16n8k16 MMAs per token
// tile.  xa / xb hold the 16 activations of the same k (words 0-3 and 4-7) for each token tile.
template <int NT, bool F16>
__device__ __forceinline__ void mma_chunk(float (&acc)[NT][4], const uint4& ra, const uint4& rb, const uint4 (&xa)[NT],
                                          const uint4 (&xb)[NT]) {
  const uint32_t wa[4] = {ra.x, ra.y, ra.z, ra.w};
  const uint32_t wb[4] = {rb.x, rb.y, rb.z, rb.w};
#pragma unroll
  for (int kq = 0; kq < 4; ++kq) {
    uint32_t a0, a1, a2, a3;
    if constexpr (F16) {
      dequant_i8x4_f16(wa[kq], a0, a2);
      dequant_i8x4_f16(wb[kq], a1, a3);
    } else {
      dequant_i8x4_bf16(wa[kq], a0, a2);
      dequant_i8x4_bf16(wb[kq], a1, a3);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const uint32_t b0 = kq == 0 ? xa[nt].x : kq == 1 ? xa[nt].z : kq == 2 ? xb[nt].x : xb[nt].z;
      const uint32_t b1 = kq == 0 ? xa[nt].y : kq == 1 ? xa[nt].w : kq == 2 ? xb[nt].y : xb[nt].w;
      if constexpr (F16)
        mma_f16_m16n8k16(acc[nt], a0, a1, a2, a3, b0, b1);
      else
        mma_bf16_m16n8k16(acc[nt], a0, a1, a2, a3, b0, b1);
    }
  }
}

template <int NT, bool HEAD>
__global__ void __launch_bounds__(kThreads, NT == 1 ? 2 : 1)
    w8a16_streamk_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                         const Params p) {
  using C = Cfg<NT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + C::kOffX;
  uint8_t* sX16 = smem + C::kOffX16;
  float* sRed = reinterpret_cast<float*>(smem + C::kOffRed);
  float4* sStat = reinterpret_cast<float4*>(smem + C::kOffStat);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::kOffBar);  // TMA bytes of the stage landed
  uint64_t* empty_bar = full_bar + S;                                   // all consumer warps read the stage
  uint64_t* xready_bar = empty_bar + S;                                 // fp16 activations of the stage written
  volatile int* sAbort = reinterpret_cast<volatile int*>(smem + C::kOffFlag);
  volatile int* sLast = sAbort + 1;
  volatile int* sInexact = sAbort + 2;  // [S]: an activation of the stage is outside the fp16 range

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int it_begin = static_cast<int>(split_start(cta, p.T, p.G));
  const int it_end = static_cast<int>(split_start(cta + 1, p.T, p.G));
  const int n_iter = it_end - it_begin;
  const bool use_f16 = p.f16_path != 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kConsumerWarps);  // one arrival per consumer warp
      mbar_init(&xready_bar[s], 1);              // the converter warp's lane 0
      sInexact[s] = 0;
    }
    *sAbort = 0;
    *sLast = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ producer (one lane)
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      const int npre = n_iter < S ? n_iter : S;
      for (int i = 0; i < npre; ++i) {  // weights do not depend on the previous kernel
        const int gi = it_begin + i;
        const int tile = gi / p.kiters;
        const int kk = gi - tile * p.kiters;
        mbar_arrive_expect_tx(&full_bar[i], C::kTxBytes);
        tma_load_2d(sW + i * kWStageBytes, &tmap_w, &full_bar[i], kk * kBK, tile * kBN, pol_w);
      }
      pdl_wait();
      for (int i = 0; i < npre; ++i) {
        const int gi = it_begin + i;
        const int kk = gi % p.kiters;
        uint8_t* xs = sX + i * C::kXStageBytes;
        tma_load_2d(xs, &tmap_x, &full_bar[i], kk * kBK, 0, pol_x);
        tma_load_2d(xs + C::kXBoxBytes, &tmap_x, &full_bar[i], kk * kBK + 64, 0, pol_x);
      }
      int issued = npre;
      for (int i = npre; i < n_iter; ++i) {
        const int s = i % S;
        const uint32_t u = static_cast<uint32_t>(i / S);
        if (!mbar_wait_bounded(&empty_bar[s], (u & 1u) ^ 1u, sAbort)) {
          record_error(p.ws, QF_ERR_TIMEOUT);
          *sAbort = 1;
          break;
        }
        const int gi = it_begin + i;
        const int tile = gi / p.kiters;
        const int kk = gi - tile * p.kiters;
        mbar_arrive_expect_tx(&full_bar[s], C::kTxBytes);
        tma_load_2d(sW + s * kWStageBytes, &tmap_w, &full_bar[s], kk * kBK, tile * kBN, pol_w);
        uint8_t* xs = sX + s * C::kXStageBytes;
        tma_load_2d(xs, &tmap_x, &full_bar[s], kk * kBK, 0, pol_x);
        tma_load_2d(xs + C::kXBoxBytes, &tmap_x, &full_bar[s], kk * kBK + 64, 0, pol_x);
        issued = i + 1;
      }
      // Drain: every copy this CTA issued must land before shared memory is released.
      const int first = issued > S ? issued - S : 0;
      for (int i = first; i < issued; ++i) {
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&full_bar[i % S], static_cast<uint32_t>(i / S) & 1u)) {
          if (global_timer_ns() - t0 > kWaitBudgetNs) {
            record_error(p.ws, QF_ERR_TIMEOUT);
            break;
          }
        }
      }
    }
    return;
  }

  if (warp == kConverterWarp) {
    // ------------------------------------------------------------------ activation converter (one warp)
    // bf16 -> fp16 of each landed stage, 8-byte blocks per lane, same offsets in the fp16 buffer with pairs
    // permuted to (k, k+2), (k+1, k+3); flags the stage if a value is outside the fp16 range.
    if (!use_f16) return;
    pdl_wait();
    const uint32_t sX_u32 = smem_u32(sX), sX16_u32 = smem_u32(sX16);
    for (int i = 0; i < n_iter; ++i) {
      const int st = i % S;
      if (!mbar_wait_bounded(&full_bar[st], static_cast<uint32_t>(i / S) & 1u, sAbort)) {
        if (!*sAbort) record_error(p.ws, QF_ERR_TIMEOUT);
        *sAbort = 1;
      }
      uint32_t bad = 0;
#pragma unroll
      for (int j = 0; j < C::kXPairs / 32; ++j) {
        const uint32_t off = static_cast<uint32_t>(st * C::kXStageBytes + (lane + 32 * j) * 8);
        uint32_t w0, w1, o0, o1;
        lds64(sX_u32 + off, w0, w1);
        bad |= bf16x4_to_f16_pairs(w0, w1, o0, o1);
        sts64(sX16_u32 + off, o0, o1);
      }
      const bool any_bad = __any_sync(0xffffffffu, bad != 0);
      __syncwarp();
      if (lane == 0) {
        sInexact[st] = any_bad ? 1 : 0;
        mbar_arrive(&xready_bar[st]);  // release: the warp's fp16 stores and the flag
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers (16 warps)
  pdl_wait();  // activations, outputs and workspace belong to the previous kernel until it completes
  const int q = warp >> 1;   // m-tile group: rows [16*kJ*q, 16*kJ*(q + 1)) of the 128-row tile
  const int h = warp & 1;    // which half of the 16-byte k chunks of each stage
  const int g = lane >> 2;
  const int t = lane & 3;
  const int c = (t ^ h) | ((t & 1) << 2);  // this lane's 16-k chunk of each stage
  const uint32_t sW_u32 = smem_u32(sW);
  const uint32_t sX_u32 = smem_u32(sX);
  const uint32_t sX16_u32 = smem_u32(sX16);
  const uint32_t w_off = static_cast<uint32_t>((16 * kJ * q + g) * 128 + ((c ^ g) << 4));
  const uint32_t x_off = static_cast<uint32_t>((c >> 2) * C::kXBoxBytes + g * 128);
  const uint32_t x_u0 = static_cast<uint32_t>(((2 * (c & 3)) ^ g) << 4);
  const uint32_t x_u1 = static_cast<uint32_t>(((2 * (c & 3) + 1) ^ g) << 4);

  int* counters = reinterpret_cast<int*>(p.ws + kWsCounters);
  float* partials = reinterpret_cast<float*>(p.ws + kWsPartials);
  float4* tile_stats = reinterpret_cast<float4*>(p.ws + kWsStats);
  const int first_tile = it_begin / p.kiters;
  const int ctid = threadIdx.x;  // 0..511 among consumers

  float acc[kJ][NT][4];
#pragma unroll
  for (int j = 0; j < kJ; ++j)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][nt][e] = 0.f;

  int tile = first_tile;
  int kk = it_begin - first_tile * p.kiters;
  for (int i = 0; i < n_iter; ++i) {
    const int s = i % S;
    if (!mbar_wait_bounded(use_f16 ? &xready_bar[s] : &full_bar[s], static_cast<uint32_t>(i / S) & 1u, sAbort)) {
      if (!*sAbort) record_error(p.ws, QF_ERR_TIMEOUT);
      *sAbort = 1;
    }
    const bool f16 = use_f16 && sInexact[s] == 0;
    const uint32_t xbase = (f16 ? sX16_u32 : sX_u32) + s * C::kXStageBytes + x_off;
    uint4 xa[NT], xb[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      xa[nt] = lds128(xbase + nt * 1024 + x_u0);
      xb[nt] = lds128(xbase + nt * 1024 + x_u1);
    }
    const uint32_t wbase = sW_u32 + s * kWStageBytes + w_off;
    uint4 ra[kJ], rb[kJ];
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      ra[j] = lds128(wbase + j * 2048);
      rb[j] = lds128(wbase + j * 2048 + 1024);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);  // release: this warp's reads of the slot are done
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      if (f16)
        mma_chunk<NT, true>(acc[j], ra[j], rb[j], xa, xb);
      else
        mma_chunk<NT, false>(acc[j], ra[j], rb[j], xa, xb);
    }

    // ------------------------------------------------------------ tile epilogue
    const int cur_tile = tile;
    const bool tile_end = (kk == p.kiters - 1) || (i == n_iter - 1);
    if (++kk == p.kiters) {
      kk = 0;
      ++tile;
    }
    if (!tile_end) continue;

    // fold the two k-halves held by warps (q, 0) and (q, 1): with one m-tile per warp, warp (q, 0) keeps it;
    // with two, warp (q, h) keeps m-tile h of the group
    float v[NT][4];
    const int keep = kJ == 1 ? 0 : h;      // which of this warp's m-tiles it finishes
    const bool owner = kJ == 1 ? (h == 0) : true;
    {
      float* mine = sRed + ((kJ == 1 ? q : warp) * 32 + lane) * 4 * NT;
      if (kJ == 1 ? (h == 1) : true) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) mine[nt * 4 + e] = (kJ == 1 || keep == 1) ? acc[0][nt][e] : acc[kJ - 1][nt][e];
      }
      named_bar_sync(kBarPairBase + q, 64);
      const float* other = kJ == 1 ? mine : sRed + ((warp ^ 1) * 32 + lane) * 4 * NT;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) v[nt][e] = (keep == 0 ? acc[0][nt][e] : acc[kJ - 1][nt][e]) + other[nt * 4 + e];
      named_bar_sync(kBarPairBase + q, 64);
    }
#pragma unroll
    for (int j = 0; j < kJ; ++j)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][nt][e] = 0.f;

    const int mt = kJ * q + keep;  // m-tile finished by this warp (if owner)
    const int rl0 = 16 * mt + g;   // local rows rl0 and rl0 + 8
    const int tile_it0 = cur_tile * p.kiters;
    const bool whole = (tile_it0 >= it_begin) && (tile_it0 + p.kiters <= it_end);
    bool finish = whole;
    if (!whole) {
      if (owner) {
        const int which = (cur_tile == first_tile) ? 0 : 1;
        float* slot = partials + static_cast<size_t>(2 * cta + which) * kPartialSlotFloats;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int col = 8 * nt + 2 * t;
          *reinterpret_cast<float2*>(slot + rl0 * 16 + col) = make_float2(v[nt][0], v[nt][1]);
          *reinterpret_cast<float2*>(slot + (rl0 + 8) * 16 + col) = make_float2(v[nt][2], v[nt][3]);
        }
        __threadfence();
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      if (ctid == 0) {
        const int c_first = cta_of(tile_it0, p.T, p.G);
        const int c_last = cta_of(min(tile_it0 + p.kiters, p.T) - 1, p.T, p.G);
        const int old = atomicAdd(&counters[cur_tile], 1);
        *sLast = (old == c_last - c_first) ? 1 : 0;
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      finish = *sLast != 0;
      if (finish && owner) {
        __threadfence();
        const int c_first = cta_of(tile_it0, p.T, p.G);
        const int c_last = cta_of(min(tile_it0 + p.kiters, p.T) - 1, p.T, p.G);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) v[nt][e] = 0.f;
        for (int cc = c_first; cc <= c_last; ++cc) {
          const int ft = static_cast<int>(split_start(cc, p.T, p.G) / p.kiters);
          const float* sl = partials + static_cast<size_t>(2 * cc + (cur_tile == ft ? 0 : 1)) * kPartialSlotFloats;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int col = 8 * nt + 2 * t;
            const float2 a = __ldcg(reinterpret_cast<const float2*>(sl + rl0 * 16 + col));
            const float2 b = __ldcg(reinterpret_cast<const float2*>(sl + (rl0 + 8) * 16 + col));
            v[nt][0] += a.x; v[nt][1] += a.y; v[nt][2] += b.x; v[nt][3] += b.y;
          }
        }
        if (ctid == 0) counters[cur_tile] = 0;  // ready for the next call on this workspace
      }
    }
    if (!finish) continue;

    const int n0 = cur_tile * kBN + rl0;
    const int n1 = n0 + 8;
    if constexpr (!HEAD) {
      if (owner) {
        const float s0 = n0 < p.N ? __ldg(p.scale + n0) : 0.f;
        const float s1 = n1 < p.N ? __ldg(p.scale + n1) : 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m0 = 8 * nt + 2 * t;
          store_out(p, n0, m0, v[nt][0] * s0);
          store_out(p, n0, m0 + 1, v[nt][1] * s0);
          store_out(p, n1, m0, v[nt][2] * s1);
          store_out(p, n1, m0 + 1, v[nt][3] * s1);
        }
      }
    } else {
      // bf16 logits, then per-token statistics of this tile over the same bf16 values
      if (owner) {
        const float s0 = n0 < p.N ? __ldg(p.scale + n0) : 0.f;
        const float s1 = n1 < p.N ? __ldg(p.scale + n1) : 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const int m = 8 * nt + 2 * t + b;
            const __nv_bfloat16 r0 = __float2bfloat16_rn(v[nt][b] * s0);
            const __nv_bfloat16 r1 = __float2bfloat16_rn(v[nt][2 + b] * s1);
            if (p.logits && m < p.M) {
              if (n0 < p.N) p.logits[static_cast<int64_t>(m) * p.ldl + n0] = r0;
              if (n1 < p.N) p.logits[static_cast<int64_t>(m) * p.ldl + n1] = r1;
            }
            RowStat st{-INFINITY, INT_MAX, 0.f};
            if (n0 < p.n_valid) st = RowStat{__bfloat162float(r0), n0, 1.f};
            if (n1 < p.n_valid) st = stat_combine(st, RowStat{__bfloat162float(r1), n1, 1.f});
            st = stat_combine(st, stat_shfl_xor(st, 4));
            st = stat_combine(st, stat_shfl_xor(st, 8));
            st = stat_combine(st, stat_shfl_xor(st, 16));
            if (g == 0) sStat[mt * 16 + m] = make_float4(st.m, __int_as_float(st.a), st.s, 0.f);
          }
        }
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      if (warp == 0) {
        if (lane < 8 * NT) {
          RowStat st{-INFINITY, INT_MAX, 0.f};
          for (int w = 0; w < kMTiles; ++w) {
            const float4 f = sStat[w * 16 + lane];
            st = stat_combine(st, RowStat{f.x, __float_as_int(f.y), f.z});
          }
          tile_stats[static_cast<size_t>(cur_tile) * 16 + lane] = make_float4(st.m, __int_as_float(st.a), st.s, 0.f);
          __threadfence();
        }
        __syncwarp();
        if (lane == 0) {
          const unsigned old = atomicAdd(reinterpret_cast<unsigned*>(p.ws) + 1, 1u);
          *sLast = (old == static_cast<unsigned>(p.ntiles - 1)) ? 1 : 0;
        }
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      if (*sLast) {
        // the last finished tile folds all tiles (fixed order: strided per thread, then a fixed tree)
        __threadfence();
        for (int m = 0; m < p.M; ++m) {
          RowStat st{-INFINITY, INT_MAX, 0.f};
          for (int j = ctid; j < p.ntiles; j += kConsumerThreads) {
            const float4 f = __ldcg(tile_stats + static_cast<size_t>(j) * 16 + m);
            st = stat_combine(st, RowStat{f.x, __float_as_int(f.y), f.z});
          }
#pragma unroll
          for (int off = 1; off < 32; off <<= 1) st = stat_combine(st, stat_shfl_xor(st, off));
          if (lane == 0) reinterpret_cast<float4*>(sRed)[warp * 16 + m] = make_float4(st.m, __int_as_float(st.a), st.s, 0.f);
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);
        if (warp == 0 && lane < p.M) {
          RowStat st{-INFINITY, INT_MAX, 0.f};
          for (int w = 0; w < kConsumerWarps; ++w) {
            const float4 f = reinterpret_cast<const float4*>(sRed)[w * 16 + lane];
            st = stat_combine(st, RowStat{f.x, __float_as_int(f.y), f.z});
          }
          p.row_max[lane] = st.m;
          p.row_argmax[lane] = static_cast<long long>(st.a) + p.vocab_offset;
          p.row_lse[lane] = st.m + logf(st.s);
        }
        if (ctid == 0) reinterpret_cast<unsigned*>(p.ws)[1] = 0u;
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);  // sStat / sRed / sLast reuse by the next tile
    }
  }
}

// K == 0: the sum is empty; the reference's kernel then stores 0 * scale (+ bias).
__global__ void fill_empty_k_kernel(const Params p) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(p.M) * p.N) return;
  const int m = static_cast<int>(idx / p.N);
  const int n = static_cast<int>(idx - static_cast<int64_t>(m) * p.N);
  store_out(p, n, m, 0.f);
}

// ================================================================================== host side
namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

struct DeviceInfo {
  int ok = 0;          // 1 = checked and sm_100, -1 = wrong arch
  int sm_count = 0;
  unsigned smem_set = 0;  // bit per kernel instance with the dynamic smem attribute set
};
std::mutex g_mu;
DeviceInfo g_dev[64];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int device_info(int* dev_out, DeviceInfo** info_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(QF_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.ok == 0) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    d.ok = (major == 10 && minor == 0) ? 1 : -1;
    d.sm_count = sms;
  }
  if (d.ok != 1) return fail(QF_ERR_ARCH, "libqf_b200 is built for sm_100a (B200); this device is not compute capability 10.0");
  if (!g_encode) {
    cudaDriverEntryPointQueryResult qres;
    void* fn = nullptr;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres);
    if (e != cudaSuccess || qres != cudaDriverEntryPointSuccess || !fn)
      return fail(QF_ERR_DRIVER, "cuTensorMapEncodeTiled entry point not found");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  *dev_out = dev;
  *info_out = &d;
  return QF_OK;
}

// Optional upper bound on the stream-K grid (environment QF_GRID_CAP, read once): lets tests exercise other
// split patterns, e.g. one CTA per whole problem.
int grid_cap() {
  static const int cap = [] {
    const char* v = std::getenv("QF_GRID_CAP");
    return v ? std::atoi(v) : 0;
  }();
  return cap;
}

// Activation path (environment QF_F16_PATH, read once): 1 (default) converts each stage's activations to
// fp16 for the cheaper exact weight conversion; 0 keeps every stage on the bf16 path.
int f16_path() {
  static const int v = [] {
    const char* e = std::getenv("QF_F16_PATH");
    return e ? std::atoi(e) : 1;
  }();
  return v;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t inner,
              uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QF_ERR_DRIVER, "cuTensorMapEncodeTiled rejected the tensor (error " + std::to_string(r) + ")");
  return QF_OK;
}

template <int NT, bool HEAD>
int launch_streamk(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, Params& p, DeviceInfo* dinfo,
                   unsigned flags, cudaStream_t stream) {
  using C = Cfg<NT>;
  auto kern = w8a16_streamk_kernel<NT, HEAD>;
  const unsigned bit = 1u << ((NT - 1) * 2 + (HEAD ? 1 : 0));
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!(dinfo->smem_set & bit)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
      if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      dinfo->smem_set |= bit;
    }
  }
  CUtensorMap tw, tx;
  int rc = encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.N),
                     static_cast<uint64_t>(ldw), kBK, kBN);
  if (rc) return rc;
  const uint64_t xstride = (p.M > 1) ? static_cast<uint64_t>(ldx) * 2 : (static_cast<uint64_t>(p.K) * 2 + 15) / 16 * 16;
  rc = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.M),
                 xstride, 64, 8 * NT);
  if (rc) return rc;

  p.f16_path = f16_path();
  p.kiters = (p.K + kBK - 1) / kBK;
  p.ntiles = (p.N + kBN - 1) / kBN;
  p.T = p.kiters * p.ntiles;
  int G = dinfo->sm_count;
  if (G > kMaxGrid) G = kMaxGrid;
  if (grid_cap() > 0 && G > grid_cap()) G = grid_cap();
  if (G > p.T) G = p.T;
  p.G = G;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & QF_FLAG_PDL) ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, p);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("launch: ") + cudaGetErrorString(e));
  return QF_OK;
}

int check_common(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale, int M, int N, int K,
                 void* ws, size_t ws_bytes) {
  if (M < 0 || N < 0 || K < 0) return fail(QF_ERR_SHAPE, "negative size");
  if (M > QF_MAX_M) return fail(QF_ERR_SHAPE, "M > 16: the small-M path handles at most 16 rows");
  if (N > QF_MAX_N) return fail(QF_ERR_SHAPE, "N above QF_MAX_N");
  if (M == 0 || N == 0) return QF_OK;
  if (!scale || !ws) return fail(QF_ERR_INVALID, "null scale or workspace");
  if (ws_bytes < qf_w8a16_workspace_bytes(M, N, K)) return fail(QF_ERR_WORKSPACE, "workspace too small");
  if (reinterpret_cast<uintptr_t>(ws) % 256) return fail(QF_ERR_ALIGN, "workspace must be 256-byte aligned");
  if (K == 0) return QF_OK;
  if (!x || !w) return fail(QF_ERR_INVALID, "null x or w");
  if (ldw < K) return fail(QF_ERR_STRIDE, "ldw < K");
  if (M > 1 && ldx < K) return fail(QF_ERR_STRIDE, "ldx < K");
  if (reinterpret_cast<uintptr_t>(w) % 16 || ldw % 16)
    return fail(QF_ERR_ALIGN, "w must be 16-byte aligned with ldw % 16 == 0");
  if (reinterpret_cast<uintptr_t>(x) % 16 || (M > 1 && ldx % 8))
    return fail(QF_ERR_ALIGN, "x must be 16-byte aligned with ldx % 8 == 0");
  return QF_OK;
}

}  // namespace
}  // namespace qf

using namespace qf;

extern "C" {

size_t qf_w8a16_workspace_bytes(int M, int N, int K) {
  (void)M;
  (void)K;
  const size_t ntiles = N > 0 ? (static_cast<size_t>(N) + kBN - 1) / kBN : 0;
  return kWsStats + ntiles * 16 * sizeof(float4);
}

int qf_w8a16_gemm(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale, const void* bias,
                  void* y, int64_t ldy, int y_dtype, int M, int N, int K, void* ws, size_t ws_bytes, unsigned flags,
                  void* stream) {
  int rc = check_common(x, ldx, w, ldw, scale, M, N, K, ws, ws_bytes);
  if (rc) return rc;
  if (M == 0 || N == 0) return QF_OK;
  if (y_dtype != QF_DTYPE_BF16 && y_dtype != QF_DTYPE_F32) return fail(QF_ERR_DTYPE, "y_dtype must be bf16 or fp32");
  if (!y) return fail(QF_ERR_INVALID, "null y");
  if (M > 1 && ldy < N) return fail(QF_ERR_STRIDE, "ldy < N");
  int dev;
  DeviceInfo* dinfo;
  rc = device_info(&dev, &dinfo);
  if (rc) return rc;
  Params p = {};
  p.scale = scale;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = y;
  p.ldy = ldy;
  p.y_f32 = y_dtype == QF_DTYPE_F32;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ws = static_cast<uint8_t*>(ws);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    const int64_t total = static_cast<int64_t>(M) * N;
    fill_empty_k_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, cudaGetErrorString(e));
  }
  if (M <= 8) return launch_streamk<1, false>(x, ldx, w, ldw, p, dinfo, flags, st);
  return launch_streamk<2, false>(x, ldx, w, ldw, p, dinfo, flags, st);
}

int qf_w8a16_head(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale, void* logits,
                  int64_t ldl, int M, int N, int K, int n_valid, int64_t vocab_offset, float* row_max,
                  int64_t* row_argmax, float* row_lse, void* ws, size_t ws_bytes, unsigned flags, void* stream) {
  int rc = check_common(x, ldx, w, ldw, scale, M, N, K, ws, ws_bytes);
  if (rc) return rc;
  if (M == 0) return QF_OK;
  if (N == 0 || K == 0) return fail(QF_ERR_SHAPE, "the head needs N >= 1 and K >= 1");
  if (n_valid < 1 || n_valid > N) return fail(QF_ERR_SHAPE, "n_valid must be in [1, N]");
  if (!row_max || !row_argmax || !row_lse) return fail(QF_ERR_INVALID, "null row statistics output");
  if (logits && M > 1 && ldl < N) return fail(QF_ERR_STRIDE, "ldl < N");
  int dev;
  DeviceInfo* dinfo;
  rc = device_info(&dev, &dinfo);
  if (rc) return rc;
  Params p = {};
  p.scale = scale;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ws = static_cast<uint8_t*>(ws);
  p.logits = static_cast<__nv_bfloat16*>(logits);
  p.ldl = ldl;
  p.n_valid = n_valid;
  p.vocab_offset = vocab_offset;
  p.row_max = row_max;
  p.row_argmax = reinterpret_cast<long long*>(row_argmax);
  p.row_lse = row_lse;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M <= 8) return launch_streamk<1, true>(x, ldx, w, ldw, p, dinfo, flags, st);
  return launch_streamk<2, true>(x, ldx, w, ldw, p, dinfo, flags, st);
}

int qf_workspace_status(void* ws, void* stream, int* status) {
  if (!ws || !status) return fail(QF_ERR_INVALID, "null argument");
  int v = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, ws, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && v != 0) e = cudaMemsetAsync(ws, 0, sizeof(int), st);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, cudaGetErrorString(e));
  *status = v;
  return QF_OK;
}

const char* qf_strerror(int code) {
  switch (code) {
    case QF_OK: return "ok";
    case QF_ERR_INVALID: return "invalid argument";
    case QF_ERR_SHAPE: return "unsupported shape";
    case QF_ERR_STRIDE: return "leading dimension too small";
    case QF_ERR_ALIGN: return "alignment requirement not met";
    case QF_ERR_ARCH: return "device is not sm_100 (B200)";
    case QF_ERR_WORKSPACE: return "workspace missing or too small";
    case QF_ERR_LAUNCH: return "CUDA launch error";
    case QF_ERR_DTYPE: return "unsupported dtype";
    case QF_ERR_TIMEOUT: return "device-side wait timed out";
    case QF_ERR_DRIVER: return "CUDA driver entry point error";
    default: return "unknown error";
  }
}

const char* qf_last_error_detail(void) { return g_err.c_str(); }

int qf_abi_version(void) { return QF_ABI_VERSION; }

}  // extern "C"

// ================================================================================== allocation-free entry
// qf_w8a16_gemm_noalloc: the same stream-K GEMM with its scratch (split-tile counters and fp32 partial tiles)
// in a fixed array of this library instead of a caller-provided workspace, for callers that cannot allocate
// device memory themselves (a host that embeds only this library and has no device allocator, e.g. a Go or
// Java binding over the C ABI, or a latency-critical path that must not call cudaMalloc, which can
// synchronise the device).  The array lives in every GPU that loads the library until the process exits.
namespace qf {
namespace {

constexpr int kNoAllocMaxGrid = 160;                 // CTAs: partial-tile slots are 2 per CTA
constexpr size_t kNoAllocBytes = kWsPartials + sizeof(float) * kPartialSlotFloats * 2 * kNoAllocMaxGrid;
static_assert(kNoAllocBytes == QF_NOALLOC_SCRATCH_BYTES, "header value out of date");

__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of the scratch array for the current device, looked up once per device (with that device
// current).  The host-side symbol is only a stand-in, never a device address.
int noalloc_scratch(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) return fail(QF_ERR_LAUNCH, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return QF_OK;
}

}  // namespace
}  // namespace qf

extern "C" int qf_w8a16_gemm_noalloc(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale,
                                     const void* bias, void* y, int64_t ldy, int y_dtype, int M, int N, int K,
                                     unsigned flags, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(QF_ERR_SHAPE, "negative size");
  if (M > QF_MAX_M) return fail(QF_ERR_SHAPE, "M > 16: the small-M path handles at most 16 rows");
  if (N > QF_NOALLOC_MAX_N)
    return fail(QF_ERR_SHAPE, "N above QF_NOALLOC_MAX_N (65536): the fixed scratch of the allocation-free entry "
                              "point holds tile counters for at most that many output channels");
  if (M == 0 || N == 0) return QF_OK;
  if (!scale || !y) return fail(QF_ERR_INVALID, "null scale or y");
  if (y_dtype != QF_DTYPE_BF16 && y_dtype != QF_DTYPE_F32) return fail(QF_ERR_DTYPE, "y_dtype must be bf16 or fp32");
  if (M > 1 && ldy < N) return fail(QF_ERR_STRIDE, "ldy < N");
  if (K > 0) {
    if (!x || !w) return fail(QF_ERR_INVALID, "null x or w");
    if (ldw < K) return fail(QF_ERR_STRIDE, "ldw < K");
    if (M > 1 && ldx < K) return fail(QF_ERR_STRIDE, "ldx < K");
    if (reinterpret_cast<uintptr_t>(w) % 16 || ldw % 16)
      return fail(QF_ERR_ALIGN, "w must be 16-byte aligned with ldw % 16 == 0");
    if (reinterpret_cast<uintptr_t>(x) % 16 || (M > 1 && ldx % 8))
      return fail(QF_ERR_ALIGN, "x must be 16-byte aligned with ldx % 8 == 0");
  }
  int dev;
  DeviceInfo* dinfo;
  int rc = device_info(&dev, &dinfo);
  if (rc) return rc;
  if (dinfo->sm_count > kNoAllocMaxGrid)
    return fail(QF_ERR_SHAPE, "device has more SMs than the allocation-free scratch provides partial-tile slots for");
  void* scratch = nullptr;
  rc = noalloc_scratch(dev, &scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: clear the error word and this call's tile counters.
  const size_t ntiles = (static_cast<size_t>(N) + kBN - 1) / kBN;
  cudaError_t e = cudaMemsetAsync(scratch, 0, kWsCounters + sizeof(int) * ntiles, st);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  Params p = {};
  p.scale = scale;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = y;
  p.ldy = ldy;
  p.y_f32 = y_dtype == QF_DTYPE_F32;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ws = static_cast<uint8_t*>(scratch);
  if (K == 0) {
    const int64_t total = static_cast<int64_t>(M) * N;
    fill_empty_k_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(p);
    e = cudaGetLastError();
    return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, cudaGetErrorString(e));
  }
  if (M <= 8) return launch_streamk<1, false>(x, ldx, w, ldw, p, dinfo, flags, st);
  return launch_streamk<2, false>(x, ldx, w, ldw, p, dinfo, flags, st);
}
