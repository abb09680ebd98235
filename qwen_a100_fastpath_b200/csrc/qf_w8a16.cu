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
// * Tiles of BN output channels (BN = 128, 64 or 32, picked per shape) and pipeline stages of BN x KS weight
//   bytes (the per-shape choice uses KS = 32768 / BN: 32 KiB stages of 256, 512 or 1024 contiguous bytes of each
//   weight row; 16 KiB stages exist for tuning).  One persistent CTA per SM, or, for small GEMMs whose tile
//   count lies between half and all of the SMs, one CTA per tile (pick_tiles).
// * Data-parallel + stream-K schedule: with ntiles = q*G + r, every CTA owns q whole tiles ("DP") and a share of
//   the r * kiters stages of the remaining r tiles ("SK").  Each CTA runs its SK share first: the SK tiles'
//   partial sums are handed to the epilogue warp, which reduces them (fp32 partials in the workspace, summed in
//   CTA order, so results are deterministic) while the consumer warps stream the DP tiles.  When every tile is
//   split (q == 0) each tile's reducing CTA gets a longer share, so the other shares finish first.  No memset
//   or cast launches are needed (the reference zero-fills an fp32 buffer for atomics and casts afterwards,
//   w8a16.py:78-79, :83).
// * One producer lane issues per stage B = KS/128 weight boxes [BN rows x 128 bytes] and 2B activation boxes
//   [8*NT tokens x 64 bf16] (cp.async.bulk.tensor, 128-byte swizzle, no multicast) into a ring of up to 10
//   stages guarded by mbarriers.  With programmatic dependent launch the weight boxes of the first stages are
//   issued before griddepcontrol.wait, while the previous kernel on the stream still runs.
// * Eight consumer warps.  Warp (u, h): unit u = (weight box b, group of MW = 2 or 4 m-tiles), h = half of each
//   box's 16-byte k chunks; lane (g, t) takes chunk c = (t ^ h) | ((t & 1) << 2), which keeps both the swizzled
//   weight reads and the activation reads free of bank conflicts.  Weights are converted to exact 16-bit floats in
//   registers and fed to mma.sync m16n8k16 as the 16-row A operand ("swap AB"); the M <= 16 tokens are the
//   8-column B operand (NT = 1 or 2 token tiles).  fp16 path (default): each warp converts its activation
//   fragments bf16 -> fp16 (pairs (k, k+2), (k+1, k+3)) and the weights with one lop3 per byte pair; if any
//   activation of the warp's chunk is outside the fp16 range the warp uses the bf16 path for that stage.  The
//   weight conversion is exact in both paths; the fp16 activation is exact except below fp16's normal range
//   (|x| < 2^-14), where it rounds to an fp16 subnormal (absolute error <= 2^-25 per activation, far below the
//   fp32 accumulation noise).  QF_F16_PATH=0 (under QF_TEST_OVERRIDES=1) keeps every product exact.
// * Tensor-core consumers (TC instances, opt-in: 128-row tiles of 256-byte stages, 9..16 tokens): the eight consumer
//   warps convert their rows to exact bf16 and store them into tensor memory (warp w: lanes 32 (w % 4) .., weight
//   box w / 4 of the stage), and one thread of an eleventh warp issues tcgen05.mma kind::f16 with that A operand,
//   the activation boxes as the 16-column B operand straight from shared memory and the tile's fp32 sums in tensor
//   memory (two A buffers and two accumulators, so conversion, MMA and the tile-end read-out overlap).  At a tile
//   end the consumers copy the sums into the shared-memory layout the epilogue warp reads.  Every product is exact
//   (bf16 x int8-valued bf16).  Measured on B200 it is slower than the mma.sync consumers at every shape (gate_up at
//   16 tokens 47.7 against 34.5 us): an M = 128, N = 16, K = 16 MMA costs about as long as a wide one, so the 16 MMAs
//   of a 32 KiB stage take longer than HBM needs to deliver the stage (removing the MMAs, not the tensor-memory
//   stores, brings it back to 33.8 us; two or four independent accumulators change nothing).  Kept for measurement
//   and tests (QF_TC=1); the mma.sync consumers are the default.
// * Epilogue: fp32 accumulator * scale, one rounding to bf16 (or fp32 export), optional bias as the reference's
//   second bf16 rounding (`y + bias`); a dedicated warp finishes each tile while the consumers stream the next,
//   and the consumers finish a CTA's last tile together.  The head additionally reduces each tile's bf16 logits
//   to per-row (max, first argmax, sum exp) -- and, in the drawing instance, a Gumbel-max draw -- and the last
//   CTA to finish folds all CTAs' statistics in a fixed order.
// * Every wait on an mbarrier is bounded (global timer); on expiry the CTA records QF_ERR_TIMEOUT in the
//   workspace, stops waiting, and the producer drains its own TMA copies before the CTA exits.
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
#include "qf_comm.cuh"
#include "qf_host.h"
#include "qf_ptx.cuh"

namespace qf {

constexpr int kConsumerWarps = 8;
constexpr int kProducerWarp = 8;            // TMA issue (one lane)
constexpr int kEpilogueWarp = 9;            // tile epilogues and stream-K reductions
constexpr int kThreads = 10 * 32;
constexpr int kMmaWarp = 10;                // TC instances: tcgen05.mma issue (one lane)
constexpr int kTcThreads = 11 * 32;
constexpr uint32_t kTcCols = 512;           // TC: A buffers 2 x 128 columns, accumulators 2 x 16
constexpr uint32_t kTcColD = 256;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kMaxBN = 128;
constexpr int kMaxGrid = 256;
constexpr int kMaxTiles = QF_MAX_N / kMaxBN;  // tile counters (tiles narrower than 128 rows only when N < 64*SMs)
constexpr int kMaxSplit = 8;                // stream-K: at most about this many CTAs share a split tile
constexpr int kBarConsumers = 1;            // named barriers (0 is __syncthreads)
constexpr int kBarReady = 2;                // consumers -> epilogue warp: a tile's partial sums are in sRed
constexpr int kBarFree = 3;                 // epilogue warp -> consumers: sRed has been read
constexpr int kBarEnd = 4;                  // consumers + epilogue warp at the end (head only)
constexpr int kBarCoop = 5;                 // epilogue warp -> consumers: peers' partial sums staged for the last tile
constexpr uint64_t kWaitBudgetNs = 4000000000ull;  // 4 s
constexpr uint32_t kPeerWaitNs = 100000u;          // stream-K reducer: wait for the other CTAs' partials (100 us)
constexpr int kSkSkewStages = 3;                   // default stream-K share skew (stages) when every tile is split

// workspace layout (bytes); the prefix [0, kWsZeroBytes) must be zero before the first call
constexpr size_t kWsHeader = 256;                              // [0] error flag, [2] CTAs done (head)
constexpr size_t kWsCounters = kWsHeader;                       // int32[kMaxTiles]
constexpr size_t kWsZeroBytes = kWsCounters + sizeof(int) * kMaxTiles;
constexpr size_t kWsPartials = (kWsZeroBytes + 1023) / 1024 * 1024;
constexpr size_t kSlotSsq = kMaxBN * 16;                         // fused RMSNorm: per-token sum of z^2 [16]
constexpr size_t kPartialSlotFloats = kSlotSsq + 16;             // [BN rows][8*NT tokens], then the sums
constexpr size_t kWsCtaStats = kWsPartials + sizeof(float) * kPartialSlotFloats * 2 * kMaxGrid;  // head
constexpr size_t kWsCtaDraws = kWsCtaStats + sizeof(float4) * 16 * kMaxGrid;  // float4 [16 tokens][kMaxGrid CTAs]
constexpr size_t kWsBytes = kWsCtaDraws + sizeof(float4) * 16 * kMaxGrid;     // head draws, same layout

constexpr int kNormMaxK = 8192;  // fused RMSNorm: gamma staged in shared memory, K <= this

template <int BN, int NT, int KS, bool NORM = false> struct Geo {
  static constexpr int B = KS / 128;                            // 128-byte weight boxes per stage
  static constexpr int MT = BN / 16;                            // m-tiles per tile (8, 4, 2)
  // m-tiles per consumer warp: 4 where the stage's boxes still split evenly over the four warp pairs, else 2.
  // A warp converts its activation fragments once per box and reuses them for all MW of its m-tiles.
  static constexpr int MW = (MT >= 4 && (B * (MT / 4)) % 4 == 0) ? 4 : 2;
  static constexpr int NMW = MT / MW;                           // m-tile groups (one per consumer warp pair)
  static constexpr int BPW = B * NMW / 4;                       // weight boxes per consumer warp per stage
  static constexpr int kWBoxBytes = BN * 128;
  static constexpr int kWBytes = BN * KS;                       // weight bytes per stage
  static constexpr int kXBoxBytes = 8 * NT * 128;               // [8*NT tokens][64 bf16] (rows >= M stay zero)
  static constexpr int kXBoxesBytes = 2 * B * kXBoxBytes;     // activation boxes of a stage
  static constexpr int kXStageBytes = (NORM ? 2 : 1) * kXBoxesBytes;  // + the residual's boxes (fused RMSNorm)
  // fused RMSNorm: gamma [kNormMaxK + 1024] bf16 (zero past K), then the consumer warps' per-token sums of z^2 of
  // the tile just handed off [8 warps][16 tokens]
  static constexpr int kNormBytes = NORM ? (kNormMaxK + 1024) * 2 + 8 * 16 * 4 : 0;
  static constexpr int kStageBytes = kWBytes + kXStageBytes;
  static constexpr int kRedBytes = kConsumerWarps * MW * 32 * 4 * NT * 4;  // [warp][m-tile of group][lane][4NT]
  static constexpr int kStatBytes = 8 * 16 * 16;                          // float4 [m-tile][token]
  static constexpr int kOutStride = BN + 8;                               // bf16 [16 tokens][BN + 8] (padded)
  static constexpr int kOutBytes = 16 * kOutStride * 2;
  static constexpr int kFixedBytes = kRedBytes + kStatBytes + kOutBytes + 2 * 16 * 8 + 64 + 1024 + kNormBytes;
  static constexpr int kBudget = 226 * 1024;
  static constexpr int kStagesFit = (kBudget - kFixedBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 10 ? 10 : kStagesFit;
  static constexpr int kOffX = kStages * kWBytes;
  static constexpr int kOffRed = kOffX + kStages * kXStageBytes;
  static constexpr int kOffStat = kOffRed + kRedBytes;
  static constexpr int kOffOut = kOffStat + kStatBytes;
  static constexpr int kOffBar = kOffOut + kOutBytes;         // full[S], empty[S], then 8 for the TC instances
  static constexpr int kOffFlag = kOffBar + 2 * kStages * 8 + 64;  // abort, last, coop, tensor-memory address
  static constexpr int kOffNorm = kOffFlag + 64;               // fused RMSNorm data
  static constexpr int kSmemBytes = kOffNorm + kNormBytes + 1024;  // + alignment slack
  static_assert(BPW >= 1 && B * NMW == 4 * BPW && 4 % NMW == 0, "the four warp pairs cover the stage's boxes evenly");
  static_assert(kStages >= 3, "pipeline too shallow");
  static_assert(2 * kStages * 8 + 64 <= 2 * 16 * 8, "barriers within their reservation");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

struct Params {
  const __nv_bfloat16* x;  // activations (read directly by the fused RMSNorm prologue)
  int64_t ldx;
  const float* scale;
  const __nv_bfloat16* bias;
  void* y;
  int64_t ldy;
  int y_f32;
  int M, N, K;
  int kiters, ntiles, G;
  int q;       // whole (DP) tiles per CTA: tiles r + cta + j * G, j < q
  int r;       // stream-K tiles 0 .. r-1
  int Tsk;     // r * kiters stream-K stages, split over the first Gsk CTAs
  int Gsk;
  int sk_skew; // q == 0: extra stages of each tile's reducing CTA over the other shares (0: even shares)
  uint32_t peer_wait_ns;  // how long a stream-K reducer waits for the other shares' partial sums
  uint8_t* ws;
  int f16_path;
  uint32_t x_tx;  // activation bytes per stage: 2 B boxes of M rows x 128 bytes
  int out_vec;     // bf16 output rows (y or logits) can be written with 16-byte stores
  int silu_I;      // > 0: gate_up with SiLU(gate) * up fused; the weight holds gate rows [0, I), up rows [I, 2I)
  // fused RMSNorm of the activations (NORM instances): z = x (+ residual), a = bf16(bf16(z) * gamma) feeds the MMA,
  // every token's accumulators are scaled by rsqrt(mean(z^2) + eps); bf16(z) is written to res_out
  const __nv_bfloat16* res;
  int64_t ldr;
  const __nv_bfloat16* gamma;
  __nv_bfloat16* res_out;
  int64_t ldro;
  float eps;
  // fused all-reduce of y over the tensor-parallel ranks (row-parallel layers); ar_world == 0: off
  int ar_world, ar_rank, ar_max_count;
  uint8_t* ar_bufs[QF_AR_MAX_RANKS];
  // head
  __nv_bfloat16* logits;
  int64_t ldl;
  int n_valid;
  long long vocab_offset;
  float* row_max;
  long long* row_argmax;
  float* row_lse;
  // head: the statistics are of the scaled logits s = logit * inv_temp (1 for the greedy head); the drawing head
  // instance (HEAD == 2) also makes a Gumbel-max draw from softmax(s) per row: argmax_j s_j + g(seed, offset, j, m)
  float inv_temp;
  uint32_t seed_lo, seed_hi, off_lo, off_hi;
  long long* row_sample;
  float* row_sample_score;
  float* row_sample_logit;
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

// Gumbel-max draw: the largest perturbed score z = s + g, its column (smaller column on ties) and its s.
struct SampleArg {
  float z;
  int a;
  float s;
};
__device__ __forceinline__ SampleArg sa_max(const SampleArg& x, const SampleArg& y) {
  return (y.z > x.z || (y.z == x.z && y.a < x.a)) ? y : x;
}
__device__ __forceinline__ SampleArg sa_shfl_xor(const SampleArg& v, int mask) {
  return SampleArg{__shfl_xor_sync(0xffffffffu, v.z, mask), __shfl_xor_sync(0xffffffffu, v.a, mask),
                   __shfl_xor_sync(0xffffffffu, v.s, mask)};
}

// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011): ten rounds of two 32x32 -> 64-bit products, with a Weyl key schedule between rounds.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// Random words of (global column j, tokens 4q .. 4q + 3) for this draw: Philox4x32-10 of the counter
// (j, q, offset lo, offset hi) under the key (seed lo, seed hi); word e belongs to token 4q + e.
__device__ __forceinline__ uint4 draw_words(const Params& p, long long j, int q) {
  return philox4x32_10(make_uint4(static_cast<uint32_t>(j), static_cast<uint32_t>(q), p.off_lo, p.off_hi), p.seed_lo,
                       p.seed_hi);
}

// Standard Gumbel noise from a random word: u = (w >> 9 + 1/2) * 2^-23, exact in fp32, in (0, 1); g = -log(E),
// E = -log(u) ~ Exp(1).  The inner logarithm needs full precision (for u near 1, -log u is tiny and an absolute
// error would dominate it); the outer one takes the fast approximation (E >= 6e-8: its absolute error in g is
// below 1e-5, far under the spacing of competing perturbed scores that matters for the draw).
__device__ __forceinline__ float gumbel_of(uint32_t w) {
  const float u = (static_cast<float>(w >> 9) + 0.5f) * 1.1920928955078125e-07f;
  return -__logf(-logf(u));
}

__device__ __forceinline__ RowStat stat_shfl_xor(const RowStat& v, int mask) {
  RowStat o;
  o.m = __shfl_xor_sync(0xffffffffu, v.m, mask);
  o.a = __shfl_xor_sync(0xffffffffu, v.a, mask);
  o.s = __shfl_xor_sync(0xffffffffu, v.s, mask);
  return o;
}

// Start of CTA c's stream-K range.  Even shares of the Tsk stages over Gsk CTAs, or, when every tile is split
// (q == 0, sk_skew = d > 0), uneven shares: each tile's first stage falls in a "long" range of L = S + d stages
// and the other CTAs get "short" ranges of S stages inside one tile.  A short CTA finishes about d stages before
// the long ones, so its partial sums are in place when the tile's reducer (the long CTA, whose part of the tile
// comes last in its range) reaches its end.  With T tiles of K stages over G CTAs: CTA c is long iff
// c = floor(t G / T) for a tile t, nL = ceil(c T / G) long CTAs precede it, S = T (K - d) / G, and
// G * start(c) = nL (T K + (G - T) d) + (c - nL) T (K - d), rounded to the nearest stage (the host enables the
// skew only where G * T * K fits in 31 bits).
__device__ __forceinline__ int split_start(int c, const Params& p) {
  if (p.sk_skew == 0) return static_cast<int>((static_cast<long long>(c) * p.Tsk) / p.Gsk);
  const int T = p.r, K = p.kiters, G = p.Gsk, d = p.sk_skew;
  const int nl = (c * T + G - 1) / G;
  const int pos = nl * (T * K + (G - T) * d) + (c - nl) * T * (K - d);
  return (pos + G / 2) / G;
}
// First and last CTA whose stream-K ranges hold stages of split tile `tile`.
__device__ __forceinline__ void tile_ctas(int tile, const Params& p, int& c_first, int& c_last) {
  const long long i0 = static_cast<long long>(tile) * p.kiters;
  const long long i1 = min(i0 + p.kiters, static_cast<long long>(p.Tsk)) - 1;
  if (p.sk_skew == 0) {  // the largest c with c * Tsk / Gsk <= i
    c_first = static_cast<int>(((i0 + 1) * p.Gsk - 1) / p.Tsk);
    c_last = static_cast<int>(((i1 + 1) * p.Gsk - 1) / p.Tsk);
    return;
  }
  // uneven shares: the tile starts in long CTA floor(tile G / T); its last stages belong to the next tile's long
  // CTA if that range starts inside this tile, else to the short CTA before it
  c_first = (tile * p.Gsk) / p.r;
  const int nxt = ((tile + 1) * p.Gsk) / p.r;
  c_last = (tile + 1 < p.r && split_start(nxt, p) <= i1) ? nxt : nxt - 1;
}

__device__ __forceinline__ int ctid_early() { return static_cast<int>(threadIdx.x); }  // consumer thread 0..255

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

// Weight row (output channel) behind row r of tile `tile`.  With the fused SiLU gate (silu_I > 0) a tile holds BN/2
// gate rows in its first half and the matching up rows in its second half.  Returns -1 for rows past the end.
template <int BN, bool SILU>
__device__ __forceinline__ int weight_row(const Params& p, int tile, int r) {
  if constexpr (!SILU) {
    const int n = tile * BN + r;
    return n < p.N ? n : -1;
  }
  constexpr int H = BN / 2;
  const int j = tile * H + (r < H ? r : r - H);
  if (j >= p.silu_I) return -1;
  return r < H ? j : p.silu_I + j;
}

// Fused gate_up activation for a finished tile staged in sOut ([M][BN + 8] bf16: gate in columns [0, BN/2), up in
// [BN/2, BN)): y[m, j] = bf16( bf16(silu(g)) * u ), silu(g) = g / (1 + exp(-g)) in fp32 -- the two roundings of
// vLLM's SiluAndMul on bf16 tensors (F.silu(x[..., :I]) * x[..., I:]).  16-byte stores of 8 outputs.
template <int BN>
__device__ __forceinline__ void silu_mul_store(const Params& p, int tile, int lane, const __nv_bfloat16* sOut) {
  constexpr int OS = BN + 8;
  constexpr int H = BN / 2;
  constexpr int HC = H / 8;
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
  for (int idx = lane; idx < p.M * HC; idx += 32) {
    const int m = idx / HC;
    const int c = (idx - m * HC) * 8;
    const int j = tile * H + c;
    const __nv_bfloat16* gp = sOut + m * OS + c;
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float gv = __bfloat162float(gp[e]);
      const __nv_bfloat16 act = __float2bfloat16_rn(gv / (1.0f + expf(-gv)));
      o[e] = __float2bfloat16_rn(__bfloat162float(act) * __bfloat162float(gp[H + e]));
    }
    __nv_bfloat16* out = y + static_cast<int64_t>(m) * p.ldy + j;
    if (p.out_vec && j + 8 <= p.silu_I) {
      *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(o);
    } else {
      for (int e = 0; e < 8; ++e)
        if (j + e < p.silu_I) out[e] = o[e];
    }
  }
}

// Walks a CTA's stages in order: its stream-K share of tiles 0..r-1, then its whole tiles.
struct StageIter {
  int tile, kk, i;
  bool sk;
  int n_sk, n_iter, sk_begin, sk_end;
  __device__ __forceinline__ void init(const Params& p, int cta) {
    if (cta < p.Gsk) {
      sk_begin = split_start(cta, p);
      sk_end = split_start(cta + 1, p);
    } else {
      sk_begin = sk_end = 0;
    }
    n_sk = sk_end - sk_begin;
    n_iter = n_sk + p.q * p.kiters;
    i = 0;
    sk = n_sk > 0;
    if (sk) {
      tile = sk_begin / p.kiters;
      kk = sk_begin - tile * p.kiters;
    } else {
      tile = p.r + cta;
      kk = 0;
    }
  }
  __device__ __forceinline__ void next(const Params& p) {
    ++i;
    if (++kk == p.kiters) {
      kk = 0;
      tile += sk ? 1 : p.G;
    }
    if (sk && i == n_sk) {
      sk = false;
      tile = p.r + static_cast<int>(blockIdx.x);
      kk = 0;
    }
  }
};

// One 16-k chunk (16 bytes of each of the rows g and g+8 of an m-tile): four m16n8k16 MMAs per token tile.
// xa / xb hold the 16 activations of the same k (words 0-3 and 4-7) for each token tile.
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

// Fused RMSNorm, per 8 bf16 columns: a = bf16(bf16(x + r) * g) (z rounded to bf16 as the residual the norm reads,
// then times gamma, one more rounding); the token's rsqrt(mean z^2 + eps) is applied to its accumulators later.
// ss accumulates z^2 (z in fp32, before rounding); zw receives bf16(z) (the new residual).
__device__ __forceinline__ uint32_t norm_pair(uint32_t x, uint32_t r, uint32_t g, float& ss, uint32_t& zw) {
  const float z0 = __uint_as_float(x << 16) + __uint_as_float(r << 16);
  const float z1 = __uint_as_float(x & 0xFFFF0000u) + __uint_as_float(r & 0xFFFF0000u);
  ss = fmaf(z0, z0, ss);
  ss = fmaf(z1, z1, ss);
  const __nv_bfloat162 z = __floats2bfloat162_rn(z0, z1);
  zw = *reinterpret_cast<const uint32_t*>(&z);
  const __nv_bfloat162 a = __floats2bfloat162_rn(__uint_as_float(zw << 16) * __uint_as_float(g << 16),
                                                 __uint_as_float(zw & 0xFFFF0000u) * __uint_as_float(g & 0xFFFF0000u));
  return *reinterpret_cast<const uint32_t*>(&a);
}
__device__ __forceinline__ uint4 norm_words(const uint4& x, const uint4& r, const uint4& g, float& ss, uint4& z) {
  return make_uint4(norm_pair(x.x, r.x, g.x, ss, z.x), norm_pair(x.y, r.y, g.y, ss, z.y),
                    norm_pair(x.z, r.z, g.z, ss, z.z), norm_pair(x.w, r.w, g.w, ss, z.w));
}
// rsqrt(mean z^2 + eps) from a token's sum of squares over the K columns.
__device__ __forceinline__ float norm_factor(const Params& p, float ss) {
  return rsqrtf(ss / static_cast<float>(p.K) + p.eps);
}

// (max, first argmax) of bf16 logits: larger value wins, equal values keep the smaller column.
struct MaxArg {
  float m;
  int a;
};
__device__ __forceinline__ MaxArg ma_max(const MaxArg& x, const MaxArg& y) {
  return (y.m > x.m || (y.m == x.m && y.a < x.a)) ? y : x;
}
__device__ __forceinline__ MaxArg ma_shfl_xor(const MaxArg& v, int mask) {
  return MaxArg{__shfl_xor_sync(0xffffffffu, v.m, mask), __shfl_xor_sync(0xffffffffu, v.a, mask)};
}

// Fused all-reduce of one finished output tile (bf16 rows staged in sOut, [M][BN + 8]) by the epilogue warp: write
// the tile as self-validating lines (qf_comm.cuh) into slot [rank] of every other rank's symmetric buffer (peer
// stores over NVLink; the tile occupies elements [tile*BN*M, (tile+1)*BN*M) of a slot, token-major), then for every
// group of 4 outputs wait (bounded) for the other ranks' lines in this rank's buffer, sum all ranks' values in rank
// order in fp32 (this rank's from sOut), round once to bf16 and store y.  Every rank computes the same bits.
template <int BN>
__device__ __forceinline__ void ar_publish_reduce(const Params& p, int tile, int lane, const __nv_bfloat16* sOut,
                                                  uint32_t epoch, uint64_t bound_ns) {
  constexpr int OS = BN + 8;
  constexpr int LPR = BN / 4;  // lines per token row of the tile
  const int par = static_cast<int>(epoch & 1u);
  const int nl = p.M * LPR;
  const int l0 = tile * BN * p.M / 4;
  for (int idx = lane; idx < nl; idx += 32) {
    const int m = idx / LPR;
    const uint2 v = *reinterpret_cast<const uint2*>(sOut + m * OS + (idx - m * LPR) * 4);
    const uint4 line = make_uint4(v.x, epoch, v.y, epoch);
    for (int r = 0; r < p.ar_world; ++r)
      if (r != p.ar_rank) st_volatile_v4(ar_line(p.ar_bufs[r], par, p.ar_rank, p.ar_max_count, l0 + idx), line);
  }
  uint8_t* own = p.ar_bufs[p.ar_rank];
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
  uint64_t deadline = 0;
  int timed_out = 0;
  for (int idx = lane; idx < nl; idx += 32) {
    const int m = idx / LPR;
    const int col = (idx - m * LPR) * 4;
    const int n = tile * BN + col;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int r = 0; r < p.ar_world; ++r) {
      const uint2 v = (r == p.ar_rank)
                          ? *reinterpret_cast<const uint2*>(sOut + m * OS + col)
                          : ar_wait_line(ar_line(own, par, r, p.ar_max_count, l0 + idx), epoch, bound_ns, &deadline,
                                         &timed_out);
      bf16x2_acc(a0, a1, v.x);
      bf16x2_acc(a2, a3, v.y);
    }
    __nv_bfloat16* out = y + static_cast<int64_t>(m) * p.ldy + n;
    if (p.out_vec && n + 4 <= p.N) {
      const __nv_bfloat162 b01 = __floats2bfloat162_rn(a0, a1);
      const __nv_bfloat162 b23 = __floats2bfloat162_rn(a2, a3);
      *reinterpret_cast<uint2*>(out) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&b01), *reinterpret_cast<const uint32_t*>(&b23));
    } else {
      const float av[4] = {a0, a1, a2, a3};
      for (int k = 0; k < 4; ++k)
        if (n + k < p.N) out[k] = __float2bfloat16_rn(av[k]);
    }
  }
  if (__any_sync(0xffffffffu, timed_out) && lane == 0)
    atomicExch(reinterpret_cast<uint32_t*>(own), static_cast<uint32_t>(QF_ERR_TIMEOUT));
}

// Reduction of a stream-K tile from every contributor's slot (CTAs c_first .. c_last, in that order), by the
// contributor that arrived last when the tile's designated reducer did not wait for the others: finishes the tile
// (scale + store, or logits + tile statistics for the head) and re-arms the tile's counter.
template <int BN, int NT, int HEAD, bool AR, bool SILU, bool NORM>
__device__ __forceinline__ void split_reduce_all(const Params& p, int tile, int lane, int c_first, int c_last,
                                                 int* counters, const float* partials, float4* sTile,
                                                 __nv_bfloat16* sOut, uint32_t ar_epoch, uint64_t ar_bound) {
  // fused RMSNorm: token `lane` (< 16) sums the contributors' sums of squares (CTA order) into its factor
  float rfac = 1.f;
  if constexpr (NORM) {
    float ss = 0.f;
    if (lane < 16) {
      for (int cc = c_first; cc <= c_last; ++cc) {
        const int ft = split_start(cc, p) / p.kiters;
        ss += __ldcg(partials + static_cast<size_t>(2 * cc + (tile == ft ? 0 : 1)) * kPartialSlotFloats + kSlotSsq + lane);
      }
      rfac = norm_factor(p, ss);
    }
  }
  // Slot = [BN rows][8*NT tokens] fp32, read as float4: lane takes float4 f = lane + 32 j (row f / (2 NT),
  // tokens 4 (lane % (2 NT)) + 0..3).  All of a contributor's loads (and those of U contributors) are issued
  // before they are added, in ascending CTA order.
  constexpr int F4 = BN * 2 * NT;
  constexpr int PER = F4 / 32;
  constexpr int PC = PER > 8 ? 8 : PER;   // float4 per lane per pass (bounded registers)
  constexpr int U = PC >= 8 ? 1 : 8 / PC;  // contributors whose loads are in flight together
  const int m_base = 4 * (lane % (2 * NT));
  RowStat st[4];
  SampleArg sz[4];  // head with sampling: Gumbel-max draw per token m_base + e
#pragma unroll
  for (int pass = 0; pass < PER / PC; ++pass) {
    float4 v[PC];
#pragma unroll
    for (int j = 0; j < PC; ++j) v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int cc = c_first; cc <= c_last; cc += U) {
      float4 a[U][PC];
#pragma unroll
      for (int uu = 0; uu < U; ++uu) {
        if (cc + uu <= c_last) {
          const int ft = split_start(cc + uu, p) / p.kiters;
          const float4* sl = reinterpret_cast<const float4*>(
              partials + static_cast<size_t>(2 * (cc + uu) + (tile == ft ? 0 : 1)) * kPartialSlotFloats);
#pragma unroll
          for (int j = 0; j < PC; ++j) a[uu][j] = __ldcg(sl + lane + 32 * (pass * PC + j));
        }
      }
#pragma unroll
      for (int uu = 0; uu < U; ++uu) {
        if (cc + uu <= c_last) {
#pragma unroll
          for (int j = 0; j < PC; ++j) {
            v[j].x += a[uu][j].x;
            v[j].y += a[uu][j].y;
            v[j].z += a[uu][j].z;
            v[j].w += a[uu][j].w;
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < PC; ++j) {
      const int row = (lane + 32 * (pass * PC + j)) / (2 * NT);
      const int wr = weight_row<BN, SILU>(p, tile, row);
      const int n = wr < 0 ? p.N : wr;  // past the end: masked below
      const float sc = wr >= 0 ? __ldg(p.scale + wr) : 0.f;
      float vv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      if constexpr (NORM) {
#pragma unroll
        for (int e = 0; e < 4; ++e) vv[e] *= __shfl_sync(0xffffffffu, rfac, m_base + e);
      }
      uint4 wd = make_uint4(0u, 0u, 0u, 0u);  // head with sampling: noise words of (row, tokens m_base ..)
      if (HEAD == 2 && n < p.n_valid) wd = draw_words(p, n + p.vocab_offset, m_base / 4);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = m_base + e;
        if constexpr (!HEAD) {
          if constexpr (AR || SILU)  // staged like finish_tile, published / activated below
            sOut[m * (BN + 8) + row] = __float2bfloat16_rn(vv[e] * sc);
          else
            store_out(p, n, m, vv[e] * sc);
        } else {
          const __nv_bfloat16 rv = __float2bfloat16_rn(vv[e] * sc);
          if (p.logits && m < p.M && n < p.N) p.logits[static_cast<int64_t>(m) * p.ldl + n] = rv;
          const float sv = HEAD == 2 ? __bfloat162float(rv) * p.inv_temp : __bfloat162float(rv);
          const RowStat one = n < p.n_valid ? RowStat{sv, n, 1.f} : RowStat{-INFINITY, INT_MAX, 0.f};
          st[e] = (pass == 0 && j == 0) ? one : stat_combine(st[e], one);
          if constexpr (HEAD == 2) {
            const uint32_t u = e == 0 ? wd.x : e == 1 ? wd.y : e == 2 ? wd.z : wd.w;
            const SampleArg z1 = n < p.n_valid ? SampleArg{sv + gumbel_of(u), n, sv} : SampleArg{-INFINITY, INT_MAX, 0.f};
            sz[e] = (pass == 0 && j == 0) ? z1 : sa_max(sz[e], z1);
          }
        }
      }
    }
  }
  if constexpr (HEAD) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      RowStat sr = st[e];
#pragma unroll
      for (int off = 2 * NT; off < 32; off <<= 1) sr = stat_combine(sr, stat_shfl_xor(sr, off));
      if (lane < 2 * NT)
        sTile[m_base + e] = make_float4(sr.m, __int_as_float(sr.a), sr.s, 0.f);
      if constexpr (HEAD == 2) {
        SampleArg zr = sz[e];
#pragma unroll
        for (int off = 2 * NT; off < 32; off <<= 1) zr = sa_max(zr, sa_shfl_xor(zr, off));
        if (lane < 2 * NT) sTile[16 + m_base + e] = make_float4(zr.z, __int_as_float(zr.a), zr.s, 0.f);
      }
    }
  }
  if constexpr (AR) {
    __syncwarp();
    ar_publish_reduce<BN>(p, tile, lane, sOut, ar_epoch, ar_bound);
  } else if constexpr (SILU) {
    __syncwarp();
    silu_mul_store<BN>(p, tile, lane, sOut);
    __syncwarp();
  }
  if (lane == 0) counters[tile] = 0;  // ready for the next call on this workspace
}

// Finishes a whole tile from the epilogue warp's fragment sums (lane (g, t): rows 16 mt + g and 16 mt + g + 8,
// tokens 8 nt + 2 t and 8 nt + 2 t + 1): scale, bf16 rounding (+ the bias as a second rounding), rows staged in
// shared memory and written with 16-byte stores (GEMM output or head logits), and for the head the tile's per-token
// (max, first argmax, sum exp) of its bf16 logits.
template <int BN, int NT, int HEAD, bool AR, bool SILU>
__device__ __forceinline__ void finish_tile(const Params& p, int tile, int lane, const float (&v)[BN / 16][NT][4],
                                            const float (&sc)[BN / 16][2], __nv_bfloat16* sOut, float4* sTile,
                                            uint32_t ar_epoch, uint64_t ar_bound) {
  constexpr int MT = BN / 16;
  constexpr int OS = BN + 8;
  const int g = lane >> 2;
  const int t = lane & 3;
  if constexpr (!HEAD) {
    if (p.y_f32) {  // fp32 export: plain stores
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int n0 = tile * BN + 16 * mt + g;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int m0 = 8 * nt + 2 * t;
          store_out(p, n0, m0, v[mt][nt][0] * sc[mt][0]);
          store_out(p, n0, m0 + 1, v[mt][nt][1] * sc[mt][0]);
          store_out(p, n0 + 8, m0, v[mt][nt][2] * sc[mt][1]);
          store_out(p, n0 + 8, m0 + 1, v[mt][nt][3] * sc[mt][1]);
        }
      }
      return;
    }
  }
  MaxArg mx[NT][2];  // head: per token 8 nt + 2 t + bq over this lane's rows
  const float inv_t = HEAD == 2 ? p.inv_temp : 1.0f;  // the greedy head's statistics are of the logits themselves
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int bq = 0; bq < 2; ++bq) mx[nt][bq] = MaxArg{-INFINITY, INT_MAX};
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int n0 = tile * BN + 16 * mt + g;
    const int n1 = n0 + 8;
    float b0 = 0.f, b1 = 0.f;
    if constexpr (!HEAD) {
      if (p.bias) {
        if (n0 < p.N) b0 = __bfloat162float(p.bias[n0]);
        if (n1 < p.N) b1 = __bfloat162float(p.bias[n1]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int bq = 0; bq < 2; ++bq) {
        const int m = 8 * nt + 2 * t + bq;
        __nv_bfloat16 r0 = __float2bfloat16_rn(v[mt][nt][bq] * sc[mt][0]);
        __nv_bfloat16 r1 = __float2bfloat16_rn(v[mt][nt][2 + bq] * sc[mt][1]);
        if constexpr (!HEAD) {
          if (p.bias) {
            r0 = __float2bfloat16_rn(__bfloat162float(r0) + b0);
            r1 = __float2bfloat16_rn(__bfloat162float(r1) + b1);
          }
        } else {
          if (n0 < p.n_valid) mx[nt][bq] = ma_max(mx[nt][bq], MaxArg{__bfloat162float(r0) * inv_t, n0});
          if (n1 < p.n_valid) mx[nt][bq] = ma_max(mx[nt][bq], MaxArg{__bfloat162float(r1) * inv_t, n1});
        }
        sOut[m * OS + 16 * mt + g] = r0;
        sOut[m * OS + 16 * mt + g + 8] = r1;
      }
  }
  __syncwarp();
  __nv_bfloat16* dst = HEAD ? p.logits : static_cast<__nv_bfloat16*>(p.y);
  const int64_t ld = HEAD ? p.ldl : p.ldy;
  if constexpr (AR) {
    ar_publish_reduce<BN>(p, tile, lane, sOut, ar_epoch, ar_bound);
  } else if constexpr (SILU) {
    silu_mul_store<BN>(p, tile, lane, sOut);
  } else if (dst) {
    constexpr int CH = BN / 8;
    for (int idx = lane; idx < p.M * CH; idx += 32) {
      const int m = idx / CH;
      const int ch = idx - m * CH;
      const int n = tile * BN + ch * 8;
      const __nv_bfloat16* src = sOut + m * OS + ch * 8;
      __nv_bfloat16* out = dst + static_cast<int64_t>(m) * ld + n;
      if (p.out_vec && n + 8 <= p.N) {
        *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(src);
      } else {
        for (int e = 0; e < 8; ++e)
          if (n + e < p.N) out[e] = src[e];
      }
    }
  }
  __syncwarp();  // staging tile free for the next tile
  if constexpr (HEAD) {
    // pass 1: the tile's max / first argmax per token over the 8 lanes g; pass 2: sum of exp(v - max) (one
    // exponential per logit), added over g in a fixed order
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int bq = 0; bq < 2; ++bq) {
        mx[nt][bq] = ma_max(mx[nt][bq], ma_shfl_xor(mx[nt][bq], 4));
        mx[nt][bq] = ma_max(mx[nt][bq], ma_shfl_xor(mx[nt][bq], 8));
        mx[nt][bq] = ma_max(mx[nt][bq], ma_shfl_xor(mx[nt][bq], 16));
      }
    float se[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int bq = 0; bq < 2; ++bq) se[nt][bq] = 0.f;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int n0 = tile * BN + 16 * mt + g;
      const int n1 = n0 + 8;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int bq = 0; bq < 2; ++bq) {
          const float mref = mx[nt][bq].m;
          if (mref != -INFINITY) {
            const float r0 = __bfloat162float(__float2bfloat16_rn(v[mt][nt][bq] * sc[mt][0])) * inv_t;
            const float r1 = __bfloat162float(__float2bfloat16_rn(v[mt][nt][2 + bq] * sc[mt][1])) * inv_t;
            if (n0 < p.n_valid) se[nt][bq] += expf(r0 - mref);
            if (n1 < p.n_valid) se[nt][bq] += expf(r1 - mref);
          }
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int bq = 0; bq < 2; ++bq) {
        float sum = se[nt][bq];
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        sum += __shfl_xor_sync(0xffffffffu, sum, 8);
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        if (g == 0)
          sTile[8 * nt + 2 * t + bq] = make_float4(mx[nt][bq].m, __int_as_float(mx[nt][bq].a), sum, 0.f);
      }
    if constexpr (HEAD == 2) {
      // Gumbel-max draw over the tile's logits as staged in sOut: lane l takes rows l, l + 32, ...; one Philox call
      // per (row, token quad) gives the noise of four tokens; z = s + g, then the best z per token over the warp.
      // The noise lies in [-2.81, 16.64] (u in [2^-24, 1 - 2^-24]), so a logit more than 19.45 below the tile's
      // largest s can never beat that element's z: its noise is not drawn (an exact pruning; kDrawPrune = 20.5
      // leaves room for rounding).
      constexpr float kDrawPrune = 20.5f;
      int* sList = reinterpret_cast<int*>(sTile + 32);  // candidate rows of the tile (BN ints, after the statistics)
      __syncwarp();  // the tile maxima of s (sTile[m].x) written above
      for (int q = 0; 4 * q < p.M; ++q) {
        float thr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)  // padded token rows draw nothing
          thr[e] = 4 * q + e < p.M ? sTile[4 * q + e].x - kDrawPrune : INFINITY;
        // candidates: rows holding a logit within kDrawPrune of its token's tile maximum, compacted so that the
        // Philox calls and logarithms run on full warps
        int cnt = 0;
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) {
          const int r = lane + 32 * i;
          bool need = false;
#pragma unroll
          for (int e = 0; e < 4; ++e)
            need |= __bfloat162float(sOut[(4 * q + e) * OS + r]) * p.inv_temp >= thr[e];
          need = need && tile * BN + r < p.n_valid;
          const uint32_t mask = __ballot_sync(0xffffffffu, need);
          if (need) sList[cnt + __popc(mask & ((1u << lane) - 1u))] = r;
          cnt += __popc(mask);
        }
        __syncwarp();
        SampleArg best[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) best[e] = SampleArg{-INFINITY, INT_MAX, 0.f};
        for (int c = lane; c < cnt; c += 32) {
          const int r = sList[c];
          const int n = tile * BN + r;
          const uint4 w = draw_words(p, n + p.vocab_offset, q);
          const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float sv = __bfloat162float(sOut[(4 * q + e) * OS + r]) * p.inv_temp;
            if (sv >= thr[e]) best[e] = sa_max(best[e], SampleArg{sv + gumbel_of(wv[e]), n, sv});
          }
        }
        const int ne = p.M - 4 * q < 4 ? p.M - 4 * q : 4;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (e < ne) {
            SampleArg b = best[e];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) b = sa_max(b, sa_shfl_xor(b, off));
            if (lane == 0) sTile[16 + 4 * q + e] = make_float4(b.z, __int_as_float(b.a), b.s, 0.f);
          }
        }
        __syncwarp();  // sList is rewritten for the next quad
      }
    }
  }
}

// Scale and bias of the rows 16 w + g and 16 w + g + 8 of `tile` for consumer lane (w, g): what coop_finish_tile
// needs, loaded when the consumers start so that their memory latency stays off the launch's critical path.
struct RowScale {
  float s0, s1, b0, b1;
};
template <int BN>
__device__ __forceinline__ RowScale load_row_scale(const Params& p, int tile, int warp, int g) {
  RowScale r{0.f, 0.f, 0.f, 0.f};
  if (tile < 0 || 16 * warp >= BN) return r;
  const int n0 = tile * BN + 16 * warp + g;
  const int n1 = n0 + 8;
  if (n0 < p.N) r.s0 = __ldg(p.scale + n0);
  if (n1 < p.N) r.s1 = __ldg(p.scale + n1);
  if (p.bias) {
    if (n0 < p.N) r.b0 = __bfloat162float(p.bias[n0]);
    if (n1 < p.N) r.b1 = __bfloat162float(p.bias[n1]);
  }
  return r;
}

// The CTA's last tile, finished by the eight consumer warps together instead of the epilogue warp alone (nothing is
// left to overlap with it, so it sits on the launch's critical path): warp w sums m-tile w from the warps' partial
// sums in sRed -- starting from the stream-K peers' sums in sPeer when `peers` -- in the epilogue warp's order, so the
// bits are the same as finish_tile's, then all consumers store the staged rows.  `rs` holds the m-tile's scales and
// bias (load_row_scale).  Plain GEMM instances with bf16 output only.
template <int BN, int NT, int MW, int NMW, bool NORM>
__device__ __forceinline__ void coop_finish_tile(const Params& p, int tile, int warp, const float* sRed,
                                                 const float* sPeer, bool peers, __nv_bfloat16* sOut,
                                                 const RowScale& rs, const float* sSsq) {
  constexpr int MT = BN / 16;
  constexpr int OS = BN + 8;
  static_assert(MT <= kConsumerWarps, "one m-tile per consumer warp");
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  // fused RMSNorm: this lane's tokens 8 nt + 2 t + bq, from the consumer warps' sums of squares (and the stream-K
  // peers', staged after their partial sums)
  float rtk[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int bq = 0; bq < 2; ++bq) {
      rtk[nt][bq] = 1.f;
      if constexpr (NORM) {
        const int m = 8 * nt + 2 * t + bq;
        float ss = peers ? sPeer[MT * 32 * 4 * NT + m] : 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) ss += sSsq[w * 16 + m];
        rtk[nt][bq] = norm_factor(p, ss);
      }
    }
  if (warp < MT) {
    const int mt = warp;
    float v[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) v[nt][e] = peers ? sPeer[(mt * 32 + lane) * 4 * NT + nt * 4 + e] : 0.f;
#pragma unroll
    for (int bb = 0; bb < 4 / NMW; ++bb)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int src = 2 * (bb * NMW + mt / MW) + hh;
        const float* o = sRed + ((src * MW + mt % MW) * 32 + lane) * 4 * NT;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) v[nt][e] += o[nt * 4 + e];
      }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int bq = 0; bq < 2; ++bq) {
        const int m = 8 * nt + 2 * t + bq;
        __nv_bfloat16 r0 = __float2bfloat16_rn(v[nt][bq] * rtk[nt][bq] * rs.s0);
        __nv_bfloat16 r1 = __float2bfloat16_rn(v[nt][2 + bq] * rtk[nt][bq] * rs.s1);
        if (p.bias) {
          r0 = __float2bfloat16_rn(__bfloat162float(r0) + rs.b0);
          r1 = __float2bfloat16_rn(__bfloat162float(r1) + rs.b1);
        }
        sOut[m * OS + 16 * mt + g] = r0;
        sOut[m * OS + 16 * mt + g + 8] = r1;
      }
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  constexpr int CH = BN / 8;
  __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.y);
  for (int idx = threadIdx.x; idx < p.M * CH; idx += kConsumerThreads) {
    const int m = idx / CH;
    const int ch = idx - m * CH;
    const int n = tile * BN + ch * 8;
    const __nv_bfloat16* src = sOut + m * OS + ch * 8;
    __nv_bfloat16* out = dst + static_cast<int64_t>(m) * p.ldy + n;
    if (p.out_vec && n + 8 <= p.N) {
      *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(src);
    } else {
      for (int e = 0; e < 8; ++e)
        if (n + e < p.N) out[e] = src[e];
    }
  }
}

// Head: folds a finished tile's per-token statistics (sTile[m], written by the epilogue warp) into lane m's running
// statistics of this CTA, in the order the CTA finishes its tiles.
template <int HEAD>
__device__ __forceinline__ void fold_tile(const Params& p, int lane, float4* sTile, RowStat& run, SampleArg& run_z) {
  __syncwarp();
  if (lane < p.M) {
    const float4 f = sTile[lane];
    run = stat_combine(run, RowStat{f.x, __float_as_int(f.y), f.z});
    if constexpr (HEAD == 2) {
      const float4 z = sTile[16 + lane];
      run_z = sa_max(run_z, SampleArg{z.x, __float_as_int(z.y), z.z});
    }
  }
  __syncwarp();
}

template <int BN, int NT, int KS, int HEAD, bool AR, bool SILU, bool NORM, bool TC>
__global__ void __launch_bounds__(TC ? kTcThreads : kThreads, 1)
    w8a16_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 const __grid_constant__ CUtensorMap tmap_r, const Params p) {
  static_assert(!TC || (BN == 128 && KS == 256 && NT == 2 && !NORM),
                "tensor-core consumers: 128-row tiles, 256-byte stages, two token tiles, no fused RMSNorm");
  static_assert(!(HEAD && AR), "the head is vocab-parallel: no all-reduce");
  static_assert(!(SILU && (HEAD || AR)), "the fused gate is for the column-parallel gate_up only");
  static_assert(!(NORM && (HEAD || AR)), "the fused RMSNorm is for the column-parallel qkv and gate_up");
  using C = Geo<BN, NT, KS, NORM>;
  constexpr int S = C::kStages;
  constexpr int B = C::B;
  constexpr int MT = C::MT;
  constexpr int MW = C::MW;
  constexpr int NMW = C::NMW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + C::kOffX;
  float* sRed = reinterpret_cast<float*>(smem + C::kOffRed);
  float4* sStat = reinterpret_cast<float4*>(smem + C::kOffStat);
  __nv_bfloat16* sOut = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffOut);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::kOffBar);  // TMA bytes of the stage landed
  uint64_t* empty_bar = full_bar + S;                                   // all consumer warps read the stage
  volatile int* sAbort = reinterpret_cast<volatile int*>(smem + C::kOffFlag);
  volatile int* sLast = sAbort + 1;
  volatile int* sCoop = sAbort + 2;  // last tile: 0 epilogue warp finishes it, 1 consumers, 2 consumers + peers' sums
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(smem + C::kOffFlag + 12);  // TC: tensor-memory base address
  // TC: a_full[2] (consumers -> MMA: A buffer stored), a_free[2] (MMA commit: A buffer read), d_full[2] (MMA commit:
  // the tile's sums are complete), d_free[2] (consumers -> MMA: sums read out)
  uint64_t* a_full = full_bar + 2 * S;
  uint64_t* a_free = a_full + 2;
  uint64_t* d_full = a_full + 4;
  uint64_t* d_free = a_full + 6;
  // fused RMSNorm: the consumer warps' per-token sums of z^2 of the tile being handed off, [8 warps][16 tokens]
  float* sSsq = reinterpret_cast<float*>(smem + C::kOffNorm + (kNormMaxK + 1024) * 2);
  // the CTA's last tile is finished by the consumer warps (plain GEMM instances with bf16 output)
  constexpr bool kCoopLast = !HEAD && !AR && !SILU;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmap_w);
    prefetch_tensormap(&tmap_x);
    if (NORM && p.res) prefetch_tensormap(&tmap_r);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], TC ? 1 : kConsumerWarps);  // one arrival per consumer warp (TC: the MMA commit)
    }
    if constexpr (TC) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&a_full[b], kConsumerWarps);
        mbar_init(&a_free[b], 1);
        mbar_init(&d_full[b], 1);
        mbar_init(&d_free[b], kConsumerWarps);
      }
    }
    *sAbort = 0;
    *sLast = 0;
    *sCoop = 0;
    fence_mbar_init();
  }
  if (TC && warp == kMmaWarp) tmem_alloc(sTmem, kTcCols);
  if constexpr (TC) tc_fence_before();
  __syncthreads();
  if constexpr (TC) tc_fence_after();
  pdl_launch_dependents();

  StageIter it;
  it.init(p, cta);
  const int n_iter = it.n_iter;
  // first and last tile of this CTA's stream-K range (partial unless the range covers them whole)
  const int sk_t0 = it.n_sk > 0 ? it.sk_begin / p.kiters : -1;
  const int sk_t1 = it.n_sk > 0 ? (it.sk_end - 1) / p.kiters : -1;

  if constexpr (TC) {
    if (warp == kMmaWarp) {
      // ---------------------------------------------------------------- MMA issue (one lane), TC instances
      // Per stage: wait for the consumers' bf16 rows of both weight boxes (A buffer i % 2), then 16 MMAs of K = 16:
      // D [128 rows x 16 tokens] (+)= A [128 x 16] x X^T, X the stage's activation boxes read in place (K-major,
      // 128-byte swizzle, 8-token groups 1 KiB apart; k step j at +32 bytes in box j / 4).  Commits release the A
      // buffer, the stage's shared memory (weights converted, activations read) and, at a tile end, the sums.
      const uint32_t tmem = *sTmem;
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_bf16(128, 16, false, false);
        StageIter mi = it;
        bool tile_start = true;
        int tcn = 0;  // tiles started before the current one
        for (int i = 0; i < n_iter; ++i) {
          const int s = i % S;
          const int buf = i & 1;
          const bool tile_end = (mi.kk == p.kiters - 1) || (mi.sk && i == mi.n_sk - 1);
          mi.next(p);
          const int d = tcn & 1;
          bool ok = true;
          if (tile_start && tcn >= 2) ok = mbar_wait_bounded(&d_free[d], ((tcn >> 1) - 1) & 1, sAbort);
          ok = ok && mbar_wait_bounded(&a_full[buf], (i >> 1) & 1, sAbort);
          if (!ok && !*sAbort) {
            record_error(p.ws, QF_ERR_TIMEOUT);
            *sAbort = 1;
          }
          tc_fence_after();
          if (!*sAbort) {
            const uint32_t xs = smem_u32(sX + s * C::kXStageBytes);
#pragma unroll
            for (int j = 0; j < KS / 16; ++j)
              mma_bf16_ts(tmem + kTcColD + 16 * d, tmem + 128 * buf + 8 * j,
                          smem_desc_k128_sw128(xs + (j >> 2) * C::kXBoxBytes + (j & 3) * 32), idesc,
                          (tile_start && j == 0) ? 0u : 1u);
          }
          // commits arrive even after an abort (nothing pending), so every role passes its waits
          mma_commit(&a_free[buf]);
          mma_commit(&empty_bar[s]);
          if (tile_end) {
            mma_commit(&d_full[d]);
            ++tcn;
          }
          tile_start = tile_end;
        }
        // the consumers' read-out of the last tile precedes the release of tensor memory (bounded, abort or not)
        if (tcn > 0) {
          const uint32_t par = static_cast<uint32_t>(((tcn - 1) >> 1) & 1);
          const uint64_t t0 = global_timer_ns();
          while (!mbar_try_wait(&d_free[(tcn - 1) & 1], par) && global_timer_ns() - t0 < kWaitBudgetNs) {
          }
        }
      }
      __syncwarp();
      tc_fence_after();
      tmem_dealloc(tmem, kTcCols);
      return;
    }
  }

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ producer (one lane)
    if (lane == 0) {
      const int npre = n_iter < S ? n_iter : S;
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      StageIter pi = it;
      for (int i = 0; i < npre; ++i) {  // weights do not depend on the previous kernel
        mbar_arrive_expect_tx(&full_bar[i], C::kWBytes + p.x_tx);
#pragma unroll
        for (int b = 0; b < B; ++b) {
          uint8_t* dst = sW + i * C::kWBytes + b * C::kWBoxBytes;
          if constexpr (!SILU) {
            tma_load_2d(dst, &tmap_w, &full_bar[i], pi.kk * KS + b * 128, pi.tile * BN, pol_w);
          } else {  // half-height boxes: gate rows, then the matching up rows
            tma_load_2d(dst, &tmap_w, &full_bar[i], pi.kk * KS + b * 128, pi.tile * (BN / 2), pol_w);
            tma_load_2d(dst + (BN / 2) * 128, &tmap_w, &full_bar[i], pi.kk * KS + b * 128,
                        p.silu_I + pi.tile * (BN / 2), pol_w);
          }
        }
        pi.next(p);
      }
      pdl_wait();
      StageIter xi = it;
      for (int i = 0; i < npre; ++i) {
        uint8_t* xs = sX + i * C::kXStageBytes;
#pragma unroll
        for (int b = 0; b < 2 * B; ++b)
          tma_load_2d(xs + b * C::kXBoxBytes, &tmap_x, &full_bar[i], xi.kk * KS + b * 64, 0, pol_x);
        if (NORM && p.res) {
#pragma unroll
          for (int b = 0; b < 2 * B; ++b)
            tma_load_2d(xs + C::kXBoxesBytes + b * C::kXBoxBytes, &tmap_r, &full_bar[i], xi.kk * KS + b * 64, 0, pol_x);
        }
        xi.next(p);
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
        mbar_arrive_expect_tx(&full_bar[s], C::kWBytes + p.x_tx);
#pragma unroll
        for (int b = 0; b < B; ++b) {
          uint8_t* dst = sW + s * C::kWBytes + b * C::kWBoxBytes;
          if constexpr (!SILU) {
            tma_load_2d(dst, &tmap_w, &full_bar[s], pi.kk * KS + b * 128, pi.tile * BN, pol_w);
          } else {  // half-height boxes: gate rows, then the matching up rows
            tma_load_2d(dst, &tmap_w, &full_bar[s], pi.kk * KS + b * 128, pi.tile * (BN / 2), pol_w);
            tma_load_2d(dst + (BN / 2) * 128, &tmap_w, &full_bar[s], pi.kk * KS + b * 128,
                        p.silu_I + pi.tile * (BN / 2), pol_w);
          }
        }
        uint8_t* xs = sX + s * C::kXStageBytes;
#pragma unroll
        for (int b = 0; b < 2 * B; ++b)
          tma_load_2d(xs + b * C::kXBoxBytes, &tmap_x, &full_bar[s], pi.kk * KS + b * 64, 0, pol_x);
        if (NORM && p.res) {
#pragma unroll
          for (int b = 0; b < 2 * B; ++b)
            tma_load_2d(xs + C::kXBoxesBytes + b * C::kXBoxBytes, &tmap_r, &full_bar[s], pi.kk * KS + b * 64, 0, pol_x);
        }
        pi.next(p);
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

  int* counters = reinterpret_cast<int*>(p.ws + kWsCounters);
  float* partials = reinterpret_cast<float*>(p.ws + kWsPartials);
  float4* cta_stats = reinterpret_cast<float4*>(p.ws + kWsCtaStats);
  float4* cta_draws = reinterpret_cast<float4*>(p.ws + kWsCtaDraws);
  // tile ends of this CTA: every tile its stream-K range touches, then its q whole tiles
  const int n_ends = (it.n_sk > 0 ? sk_t1 - sk_t0 + 1 : 0) + p.q;

  if (warp == kEpilogueWarp) {
    // ------------------------------------------------------------------ epilogue warp
    // Walks the consumers' stage sequence; at each tile end it takes the eight consumer warps' partial sums from
    // shared memory, adds them in a fixed order and finishes the tile while the consumers stream the next one.
    // Stream-K tiles: a CTA that holds a later part of a tile (its first tile) stores its partial sums and counts
    // itself in; the CTA holding the tile's first k-stages (its last stream-K tile, always the last to finish
    // it) is the tile's reducer: it waits for the others' count, prefetches their sums while its own stages still
    // stream, and finishes the tile.  If that wait exceeds p.peer_wait_ns (CTAs not co-resident), the reducer hands
    // off like the others and the last one to count itself in reduces every slot.
    pdl_wait();
    const int g = lane >> 2;
    const int t = lane & 3;
    int tc = -1, tr = -1;  // this CTA's contributor tile and reducer tile
    if (it.n_sk > 0) {
#pragma unroll
      for (int side = 0; side < 2; ++side) {
        const int tt = side == 0 ? sk_t0 : sk_t1;
        if (side == 1 && tt == sk_t0) break;
        const bool whole_tt = tt * p.kiters >= it.sk_begin && (tt + 1) * p.kiters <= it.sk_end;
        if (whole_tt) continue;
        if (tt * p.kiters >= it.sk_begin) tr = tt;
        else tc = tt;
      }
    }
    // CTAs sharing the contributor tile and the reducer tile, kept in shared memory for the tile ends
    __shared__ int s_tile_ctas[2][2];
    if (lane == 0) {
      if (tc >= 0) tile_ctas(tc, p, s_tile_ctas[0][0], s_tile_ctas[0][1]);
      if (tr >= 0) tile_ctas(tr, p, s_tile_ctas[1][0], s_tile_ctas[1][1]);
    }
    __syncwarp();
    uint32_t ar_epoch = 0;  // fused all-reduce: this call's epoch (previous calls on these buffers + 1)
    uint64_t ar_bound = 0;  // and the bound of its waits on the other ranks
    if constexpr (AR) {
      uint32_t e = 0;
      if (lane == 0) e = *reinterpret_cast<volatile uint32_t*>(p.ar_bufs[p.ar_rank] + 4) + 1u;
      ar_epoch = __shfl_sync(0xffffffffu, e, 0);
      ar_bound = ar_wait_bound_ns(p.ar_bufs[p.ar_rank]);
    }
    StageIter et = it;
    int tcount = 0;
    RowStat run{-INFINITY, INT_MAX, 0.f};  // head: lane m folds token m's statistics over this CTA's tiles
    SampleArg run_z{-INFINITY, INT_MAX, 0.f};  // head with sampling: lane m's draw over this CTA's tiles
    for (int i = 0; i < n_iter; ++i) {
      const int tile = et.tile;
      const bool sk = et.sk;
      const bool tile_end = (et.kk == p.kiters - 1) || (sk && i == et.n_sk - 1);
      et.next(p);
      if (!tile_end) continue;
      const bool is_red = sk && tile == tr;
      const bool is_con = sk && tile == tc;
      float sc[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int w0 = weight_row<BN, SILU>(p, tile, 16 * mt + g);
        const int w1 = weight_row<BN, SILU>(p, tile, 16 * mt + g + 8);
        sc[mt][0] = w0 >= 0 ? __ldg(p.scale + w0) : 0.f;
        sc[mt][1] = w1 >= 0 ? __ldg(p.scale + w1) : 0.f;
      }
      int c_first = 0, c_last = 0;
      if (is_red || is_con) {
        c_first = s_tile_ctas[is_red ? 1 : 0][0];
        c_last = s_tile_ctas[is_red ? 1 : 0][1];
      }
      // the tile's sums: the reducer starts from the later CTAs' partials (in CTA order), then adds its own
      float v[MT][NT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) v[mt][nt][e] = 0.f;
      bool red_ok = false;
      float peer_ss = 0.f;  // fused RMSNorm: the later CTAs' sums of squares of token `lane` (< 16)
      if (is_red) {
        int ok = 0;
        if (lane == 0 && p.peer_wait_ns > 0) {  // 0: hand off at once
          const int want = c_last - c_first;
          const uint64_t t0 = global_timer_ns();
          while (true) {
            if (ld_acquire_gpu(counters + tile) == want) {
              ok = 1;
              break;
            }
            if (global_timer_ns() - t0 > p.peer_wait_ns) break;
            sleep_ns(128);
          }
        }
        red_ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
        __syncwarp();  // lane 0's acquire orders the other lanes' loads of the peers' slots
        if (red_ok) {
#pragma unroll 2
          for (int cc = c_first + 1; cc <= c_last; ++cc) {  // the tile is each later CTA's first: slot 0
            const float* sl = partials + static_cast<size_t>(2 * cc) * kPartialSlotFloats;
            if (NORM && lane < 16) peer_ss += __ldcg(sl + kSlotSsq + lane);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                const int row = 16 * mt + g;
                const int col = 8 * nt + 2 * t;
                const float2 a = __ldcg(reinterpret_cast<const float2*>(sl + row * 8 * NT + col));
                const float2 b = __ldcg(reinterpret_cast<const float2*>(sl + (row + 8) * 8 * NT + col));
                v[mt][nt][0] += a.x;
                v[mt][nt][1] += a.y;
                v[mt][nt][2] += b.x;
                v[mt][nt][3] += b.y;
              }
          }
        }
      }
      const bool coop_tile = kCoopLast && !p.y_f32 && tcount == n_ends - 1;
      const bool coop = coop_tile && !is_con && (!is_red || red_ok);
      if (coop_tile) {
        if (lane == 0) *sCoop = coop ? (is_red ? 2 : 1) : 0;
        __syncwarp();
      }
      named_bar_sync(kBarReady, kConsumerThreads + 32);
      if (coop) {
        // the consumers finish the tile; the weight ring is idle now (every stage consumed): stage the peers' sums
        // there in the consumers' accumulator layout
        if (is_red) {
          float* sPeer = reinterpret_cast<float*>(sW);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) sPeer[(mt * 32 + lane) * 4 * NT + nt * 4 + e] = v[mt][nt][e];
          if (NORM && lane < 16) sPeer[MT * 32 * 4 * NT + lane] = peer_ss;
          named_bar_arrive(kBarCoop, kConsumerThreads + 32);
          if (lane == 0) counters[tile] = 0;  // every other contributor has counted itself in: re-arm
        }
        ++tcount;
        continue;
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int bb = 0; bb < 4 / NMW; ++bb)  // warps (u = bb * NMW + mt / MW, h) hold m-tile mt
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int src = 2 * (bb * NMW + mt / MW) + hh;
            const float* o = sRed + ((src * MW + mt % MW) * 32 + lane) * 4 * NT;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) v[mt][nt][e] += o[nt * 4 + e];
          }
      }
      float own_ss = 0.f;  // fused RMSNorm: this CTA's sum of squares of token `lane` (< 16) for the tile
      if constexpr (NORM) {
        if (lane < 16) {
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) own_ss += sSsq[w * 16 + lane];
        }
      }
      if (tcount + 1 < n_ends) named_bar_arrive(kBarFree, kConsumerThreads + 32);
      ++tcount;

      if (is_red && red_ok) {
        if (lane == 0) counters[tile] = 0;  // every other contributor has counted itself in: re-arm
      } else if (is_red || is_con) {
        const int which = (tile == sk_t0) ? 0 : 1;
        float* slot = partials + static_cast<size_t>(2 * cta + which) * kPartialSlotFloats;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {  // [BN rows][8*NT tokens]
            const int row = 16 * mt + g;
            const int col = 8 * nt + 2 * t;
            __stcg(reinterpret_cast<float2*>(slot + row * 8 * NT + col), make_float2(v[mt][nt][0], v[mt][nt][1]));
            __stcg(reinterpret_cast<float2*>(slot + (row + 8) * 8 * NT + col),
                   make_float2(v[mt][nt][2], v[mt][nt][3]));
          }
        if (NORM && lane < 16) __stcg(slot + kSlotSsq + lane, own_ss);
        __syncwarp();  // the slot stores of all lanes precede lane 0's release
        int last = 0;
        if (lane == 0)  // last only after a reducer gave up waiting
          last = atom_add_acq_rel_gpu(reinterpret_cast<uint32_t*>(counters + tile), 1u) ==
                 static_cast<uint32_t>(c_last - c_first);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          split_reduce_all<BN, NT, HEAD, AR, SILU, NORM>(p, tile, lane, c_first, c_last, counters, partials, sStat, sOut,
                                                         ar_epoch, ar_bound);
          if constexpr (HEAD) fold_tile<HEAD>(p, lane, sStat, run, run_z);
        }
        continue;
      }
      if constexpr (NORM) {  // the whole tile's sums (this CTA's, plus the later CTAs' for a reduced split tile)
        const float rfac = norm_factor(p, own_ss + peer_ss);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int bq = 0; bq < 2; ++bq) {
            const float r = __shfl_sync(0xffffffffu, rfac, 8 * nt + 2 * t + bq);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              v[mt][nt][bq] *= r;
              v[mt][nt][2 + bq] *= r;
            }
          }
      }
      finish_tile<BN, NT, HEAD, AR, SILU>(p, tile, lane, v, sc, sOut, sStat, ar_epoch, ar_bound);
      if constexpr (HEAD) fold_tile<HEAD>(p, lane, sStat, run, run_z);
    }
    if (AR && lane == 0) {  // the last CTA to finish advances the buffers' epoch for the next call
      uint32_t* hdr = reinterpret_cast<uint32_t*>(p.ar_bufs[p.ar_rank]);
      if (atomicAdd(hdr + 2, 1u) == static_cast<uint32_t>(p.G - 1)) {
        hdr[2] = 0u;
        hdr[1] = ar_epoch;
      }
    }
    if constexpr (HEAD) {
      if (lane < p.M) {
        cta_stats[lane * kMaxGrid + cta] = make_float4(run.m, __int_as_float(run.a), run.s, 0.f);
        if constexpr (HEAD == 2) cta_draws[lane * kMaxGrid + cta] = make_float4(run_z.z, __int_as_float(run_z.a), run_z.s, 0.f);
      }
      named_bar_sync(kBarEnd, kConsumerThreads + 32);
    }
    return;
  }

  // -------------------------------------------------------------------- consumers (8 warps)
  {
    // Token rows M .. 8*NT-1 of every activation box are never written by the copies (the boxes are M rows high):
    // zero them once so that those MMA columns compute zeros.  The copies write only rows < M of the same boxes.
    const int zrows = 8 * NT - p.M;
    const int per_box = zrows * 8;  // 16-byte units
    for (int idx = threadIdx.x; idx < S * (NORM ? 4 : 2) * B * per_box; idx += kConsumerThreads) {
      const int box = idx / per_box;
      const int rem = idx - box * per_box;
      *reinterpret_cast<uint4*>(sX + box * C::kXBoxBytes + (p.M + rem / 8) * 128 + (rem % 8) * 16) =
          make_uint4(0u, 0u, 0u, 0u);
    }
    if constexpr (TC) {
      // the tile sums go to one holder slot per m-tile; the other slots the epilogue adds stay zero
      for (int idx = threadIdx.x; idx < C::kRedBytes / 16; idx += kConsumerThreads)
        reinterpret_cast<uint4*>(sRed)[idx] = make_uint4(0u, 0u, 0u, 0u);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // zeroed token rows feed the tensor cores
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
  }
  pdl_wait();  // activations, outputs and workspace belong to the previous kernel until it completes
  if constexpr (NORM) {
    // gamma into shared memory, zero past K (the stages' k range reaches past K where the copies zero-fill)
    uint4* sGam = reinterpret_cast<uint4*>(smem + C::kOffNorm);
    const int kch = p.K / 8;  // K % 8 == 0 (host check)
    for (int i = ctid_early(); i < (kNormMaxK + 1024) / 8; i += kConsumerThreads)
      sGam[i] = i < kch ? __ldg(reinterpret_cast<const uint4*>(p.gamma) + i) : make_uint4(0u, 0u, 0u, 0u);
    named_bar_sync(kBarConsumers, kConsumerThreads);
  }
  // Warp (u, h), u = warp / 2: m-tile group mg = u % NMW (m-tiles MW * mg ..), weight boxes
  // b = u / NMW + j * (4 / NMW), j < BPW.
  const int h = warp & 1;           // which half of each box's 16-byte k chunks
  const int u = warp >> 1;
  const int mg = u % NMW;
  const int b0 = u / NMW;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int c = (t ^ h) | ((t & 1) << 2);  // this lane's 16-k chunk of the box
  const uint32_t sW_u32 = smem_u32(sW);
  const uint32_t sX_u32 = smem_u32(sX);
  const uint32_t w_off = static_cast<uint32_t>(b0 * C::kWBoxBytes + (16 * MW * mg + g) * 128 + ((c ^ g) << 4));
  const uint32_t x_off = static_cast<uint32_t>((2 * b0 + (c >> 2)) * C::kXBoxBytes + g * 128);
  const uint32_t x_u0 = static_cast<uint32_t>(((2 * (c & 3)) ^ g) << 4);
  const uint32_t x_u1 = static_cast<uint32_t>(((2 * (c & 3) + 1) ^ g) << 4);
  const int ctid = threadIdx.x;  // 0..255 among consumers
  const bool use_f16 = p.f16_path != 0;
  const uint32_t tmem = TC ? *sTmem : 0u;
  const uint32_t tc_lanes = static_cast<uint32_t>(32 * (warp & 3)) << 16;  // TC: this warp's tensor-memory lanes
  int tcount = 0;
  // scales and bias of the CTA's last tile (its last whole tile, else the last tile of its stream-K share), which the
  // consumers may finish themselves
  RowScale last_rs{0.f, 0.f, 0.f, 0.f};
  if constexpr (kCoopLast) {
    if (!p.y_f32 && n_iter > 0)
      last_rs = load_row_scale<BN>(p, p.q > 0 ? p.r + cta + (p.q - 1) * p.G : (it.sk_end - 1) / p.kiters, warp, g);
  }

  // fused RMSNorm: this lane's sum of z^2 over the current tile's stages, for tokens g + 8 nt; counted by the warps
  // of m-tile group 0 only, which between them read every activation of a stage once
  float ssq[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) ssq[nt] = 0.f;

  float acc[MW][NT][4];
#pragma unroll
  for (int j = 0; j < MW; ++j)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][nt][e] = 0.f;

  for (int i = 0; i < n_iter; ++i) {
    const int s = i % S;
    if (!mbar_wait_bounded(&full_bar[s], static_cast<uint32_t>(i / S) & 1u, sAbort)) {
      if (!*sAbort) record_error(p.ws, QF_ERR_TIMEOUT);
      *sAbort = 1;
    }
    if constexpr (TC) {
      // row 32 (warp % 4) + lane of weight box warp / 4 as exact bf16 into A buffer i % 2 (columns 64 (warp / 4) ..,
      // k pairs per column), once the MMAs of stage i - 2 have read that buffer
      const int buf = i & 1;
      if (i >= 2 && !mbar_wait_bounded(&a_free[buf], ((i >> 1) - 1) & 1, sAbort)) {
        if (!*sAbort) record_error(p.ws, QF_ERR_TIMEOUT);
        *sAbort = 1;
      }
      tc_fence_after();
      const int row = 32 * (warp & 3) + lane;
      const uint32_t wrow = sW_u32 + s * C::kWBytes + (warp >> 2) * C::kWBoxBytes + row * 128;
      uint32_t a0[32], a1[32];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const uint4 v = lds128(wrow + ((cc ^ (row & 7)) << 4));
        uint32_t* dst = cc < 4 ? a0 + 8 * cc : a1 + 8 * (cc - 4);
        dequant_i8x4_bf16(v.x, dst[0], dst[1]);
        dequant_i8x4_bf16(v.y, dst[2], dst[3]);
        dequant_i8x4_bf16(v.z, dst[4], dst[5]);
        dequant_i8x4_bf16(v.w, dst[6], dst[7]);
      }
      const uint32_t ta = tmem + tc_lanes + 128 * buf + 64 * (warp >> 2);
      tmem_st_32x32b_x32(ta, a0);
      tmem_st_32x32b_x32(ta + 32, a1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[buf]);
    } else {
#pragma unroll
    for (int jb = 0; jb < C::BPW; ++jb) {
      const int db = jb * (4 / NMW);  // box offset from b0
      const uint32_t xbase = sX_u32 + s * C::kXStageBytes + x_off + 2 * db * C::kXBoxBytes;
      uint4 xa[NT], xb[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        xa[nt] = lds128(xbase + nt * 1024 + x_u0);
        xb[nt] = lds128(xbase + nt * 1024 + x_u1);
      }
      if constexpr (NORM) {
        // a = bf16(bf16(x + residual) * gamma) for this lane's 16 k columns of each token row
        const int k0 = it.kk * KS + 64 * (2 * (b0 + db) + (c >> 2)) + 16 * (c & 3);
        const uint32_t gbase = smem_u32(smem + C::kOffNorm) + static_cast<uint32_t>(k0 * 2);
        const uint4 ga = lds128(gbase), gb = lds128(gbase + 16);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          uint4 ra = make_uint4(0u, 0u, 0u, 0u), rb = ra;
          if (p.res) {
            ra = lds128(xbase + C::kXBoxesBytes + nt * 1024 + x_u0);
            rb = lds128(xbase + C::kXBoxesBytes + nt * 1024 + x_u1);
          }
          float ss = 0.f;
          uint4 za, zb;
          xa[nt] = norm_words(xa[nt], ra, ga, ss, za);
          xb[nt] = norm_words(xb[nt], rb, gb, ss, zb);
          if (mg == 0) {
            ssq[nt] += ss;
            // the new residual bf16(z): written by whichever CTAs stream tile 0 (its stages cover every k once)
            const int m = g + 8 * nt;
            if (it.tile == 0 && p.res_out && m < p.M && k0 < p.K) {
              uint4* dst = reinterpret_cast<uint4*>(p.res_out + static_cast<int64_t>(m) * p.ldro + k0);
              dst[0] = za;
              if (k0 + 8 < p.K) dst[1] = zb;
            }
          }
        }
      }
      const uint32_t wbase = sW_u32 + s * C::kWBytes + w_off + db * C::kWBoxBytes;
      uint4 ra[MW], rb[MW];  // m-tile j: rows g and g + 8 of the tile's 16
#pragma unroll
      for (int j = 0; j < MW; ++j) {
        ra[j] = lds128(wbase + j * 2048);
        rb[j] = lds128(wbase + j * 2048 + 1024);
      }
      if (jb == C::BPW - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);  // release: this warp's reads of the slot are done
      }

      bool f16 = false;
      uint4 xa16[NT], xb16[NT];
      if (use_f16) {
        uint32_t bad = 0;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          bad |= bf16x4_to_f16_pairs(xa[nt].x, xa[nt].y, xa16[nt].x, xa16[nt].y);
          bad |= bf16x4_to_f16_pairs(xa[nt].z, xa[nt].w, xa16[nt].z, xa16[nt].w);
          bad |= bf16x4_to_f16_pairs(xb[nt].x, xb[nt].y, xb16[nt].x, xb16[nt].y);
          bad |= bf16x4_to_f16_pairs(xb[nt].z, xb[nt].w, xb16[nt].z, xb16[nt].w);
        }
        f16 = !__any_sync(0xffffffffu, bad != 0);
      }
      if (f16) {
#pragma unroll
        for (int j = 0; j < MW; ++j) mma_chunk<NT, true>(acc[j], ra[j], rb[j], xa16, xb16);
      } else {
#pragma unroll
        for (int j = 0; j < MW; ++j) mma_chunk<NT, false>(acc[j], ra[j], rb[j], xa, xb);
      }
    }
    }

    // ------------------------------------------------------------ tile end: hand the sums to the epilogue warp
    const bool tile_end = (it.kk == p.kiters - 1) || (it.sk && i == it.n_sk - 1);
    const int cur_tile = it.tile;
    it.next(p);
    if (!tile_end) continue;
    if constexpr (TC) {
      // the tile's sums: tokens 8 (warp / 4) .. + 7 of row 32 (warp % 4) + lane, from accumulator tcount % 2
      const int d = tcount & 1;
      if (!mbar_wait_bounded(&d_full[d], (tcount >> 1) & 1, sAbort)) {
        if (!*sAbort) record_error(p.ws, QF_ERR_TIMEOUT);
        *sAbort = 1;
      }
      tc_fence_after();
      uint32_t r8[8];
      tmem_ld_32x32b_x8(tmem + tc_lanes + kTcColD + 16 * d + 8 * (warp >> 2), r8);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_free[d]);
      if (tcount > 0) named_bar_sync(kBarFree, kConsumerThreads + 32);  // the previous tile's sums have been read
      // into the slot of the first warp holding the m-tile in the mma.sync layout: lane (g, t) holds rows g, g + 8 and
      // tokens 8 nt + 2 t, + 1 as acc[nt][0..3]
      const int row = 32 * (warp & 3) + lane;
      const int mt = row >> 4;
      float* slot = sRed + ((2 * (mt / MW) * MW + mt % MW) * 32 + 4 * (row & 7)) * 4 * NT + 4 * (warp >> 2) +
                    2 * ((row >> 3) & 1);
#pragma unroll
      for (int tt = 0; tt < 4; ++tt)
        *reinterpret_cast<float2*>(slot + tt * 4 * NT) =
            make_float2(__uint_as_float(r8[2 * tt]), __uint_as_float(r8[2 * tt + 1]));
    } else {
    if (tcount > 0) named_bar_sync(kBarFree, kConsumerThreads + 32);  // the previous tile's sums have been read
    {
      float* mine = sRed + (warp * MW * 32 + lane) * 4 * NT;
#pragma unroll
      for (int j = 0; j < MW; ++j)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            mine[j * 32 * 4 * NT + nt * 4 + e] = acc[j][nt][e];
            acc[j][nt][e] = 0.f;
          }
      if constexpr (NORM) {  // the tile's sums of squares per token (lanes 4 g .. 4 g + 3 hold token g's parts)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float v = ssq[nt];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          if (t == 0) sSsq[warp * 16 + 8 * nt + g] = v;
          ssq[nt] = 0.f;
        }
        if (NT == 1 && lane < 8) sSsq[warp * 16 + 8 + lane] = 0.f;
      }
    }
    }
    if (kCoopLast && !p.y_f32 && i == n_iter - 1) {  // the CTA's last tile: finished here unless the epilogue
      named_bar_sync(kBarReady, kConsumerThreads + 32);  // warp keeps it (stream-K contribution)
      const int mode = *sCoop;
      if (mode == 2) named_bar_sync(kBarCoop, kConsumerThreads + 32);
      if (mode != 0)
        coop_finish_tile<BN, NT, MW, NMW, NORM>(p, cur_tile, warp, sRed, reinterpret_cast<const float*>(sW), mode == 2,
                                                sOut, last_rs, sSsq);
    } else {
      named_bar_arrive(kBarReady, kConsumerThreads + 32);
    }
    ++tcount;
  }

  if constexpr (HEAD) {
    // the CTA that finishes last folds the per-tile statistics of all tiles (fixed order)
    // kBarEnd orders every tile-statistics store of this CTA before thread 0's release; the last CTA's acquire
    // (and the barrier after it) orders its reads after all CTAs' stores.
    named_bar_sync(kBarEnd, kConsumerThreads + 32);
    if (ctid == 0) {
      const uint32_t old = atom_add_acq_rel_gpu(reinterpret_cast<uint32_t*>(p.ws) + 2, 1u);
      *sLast = (old == static_cast<uint32_t>(p.G - 1)) ? 1 : 0;
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (*sLast) {
      // Warp w folds tokens w and w + 8: lane l combines CTAs l, l + 32, ... in order, then a butterfly over the
      // lanes.  The combine is symmetric, so every lane ends with the same bits, and the order is fixed.
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int m = warp + kConsumerWarps * k;
        if (m < p.M) {
          RowStat st{-INFINITY, INT_MAX, 0.f};
          for (int c = lane; c < p.G; c += 32) {
            const float4 f = __ldcg(cta_stats + m * kMaxGrid + c);
            st = stat_combine(st, RowStat{f.x, __float_as_int(f.y), f.z});
          }
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) st = stat_combine(st, stat_shfl_xor(st, off));
          if (lane == 0) {
            p.row_max[m] = st.m;
            p.row_argmax[m] = static_cast<long long>(st.a) + p.vocab_offset;
            p.row_lse[m] = st.m + logf(st.s);
          }
          if constexpr (HEAD == 2) {
            SampleArg sz{-INFINITY, INT_MAX, 0.f};
            for (int c = lane; c < p.G; c += 32) {
              const float4 f = __ldcg(cta_draws + m * kMaxGrid + c);
              sz = sa_max(sz, SampleArg{f.x, __float_as_int(f.y), f.z});
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) sz = sa_max(sz, sa_shfl_xor(sz, off));
            if (lane == 0) {
              p.row_sample[m] = static_cast<long long>(sz.a) + p.vocab_offset;
              p.row_sample_score[m] = sz.z;
              p.row_sample_logit[m] = sz.s;
            }
          }
        }
      }
      if (ctid == 0) reinterpret_cast<unsigned*>(p.ws)[2] = 0u;
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
thread_local std::string g_err;

// Records the message behind a failing entry point (qf_last_error_detail) and returns its code.
int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

namespace {

struct DeviceInfo {
  int ok = 0;             // 1 = checked and sm_100, -1 = wrong arch
  int sm_count = 0;
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
  if (d.ok != 1)
    return fail(QF_ERR_ARCH, "libqf_b200 is built for sm_100a (B200); this device is not compute capability 10.0");
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

// Test and tuning knobs (QF_GRID_CAP, QF_TILES, QF_SK_SKEW, QF_PEER_WAIT_NS, QF_F16_PATH) are read only when the
// environment also sets QF_TEST_OVERRIDES=1, so that a stray variable in a deployment cannot change the schedule or
// the arithmetic path.  Each is read once per process.
const char* test_env(const char* name) {
  static const bool on = [] {
    const char* v = std::getenv("QF_TEST_OVERRIDES");
    return v != nullptr && std::strcmp(v, "1") == 0;
  }();
  return on ? std::getenv(name) : nullptr;
}

// Optional upper bound on the grid (QF_GRID_CAP): lets tests exercise other schedules.
int grid_cap() {
  static const int cap = [] {
    const char* v = test_env("QF_GRID_CAP");
    return v ? std::atoi(v) : 0;
  }();
  return cap;
}

// Stream-K reducer wait in ns (QF_PEER_WAIT_NS; default kPeerWaitNs).  0 means no wait at
// all: the tests set it so that every reducer hands off and the last-arriving share reduces the tile
// (split_reduce_all), the path that otherwise runs only when the CTAs of a launch are not all resident.
uint32_t peer_wait_ns() {
  static const uint32_t v = [] {
    const char* e = test_env("QF_PEER_WAIT_NS");
    return e ? static_cast<uint32_t>(std::strtoul(e, nullptr, 10)) : kPeerWaitNs;
  }();
  return v;
}

// Stream-K share skew in stages (QF_SK_SKEW; default kSkSkewStages): how many stages
// longer the reducing CTA's share of a split tile is than the other shares, when every tile is split.
int sk_skew_stages() {
  static const int v = [] {
    const char* e = test_env("QF_SK_SKEW");
    return e ? std::atoi(e) : kSkSkewStages;
  }();
  return v;
}

// Activation path (QF_F16_PATH): 1 (default) converts activations to fp16 for the cheaper
// exact weight conversion (warps fall back to bf16 where activations leave the fp16 range); 0 keeps bf16.
int f16_path() {
  static const int v = [] {
    const char* e = test_env("QF_F16_PATH");
    return e ? std::atoi(e) : 1;
  }();
  return v;
}

// Tensor-core consumers for the 128 x 256 tiles at 9..16 tokens (QF_TC=1 under QF_TEST_OVERRIDES=1); off by default,
// the measured choice (the mma.sync consumers are faster at every shape).
int tc_mode() {
  static const int v = [] {
    const char* e = test_env("QF_TC");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(QF_ERR_DRIVER, "cuTensorMapEncodeTiled rejected the tensor (error " + std::to_string(r) + ")");
  return QF_OK;
}

// Tile shape (BN rows x KS k-bytes per stage) and, for small GEMMs, a data-parallel grid.  Longer contiguous runs
// per weight row stream faster from HBM3e (512-byte runs reach the plain read rate, 128-byte runs about 80 % of
// it), narrow tiles cost activation copies (2M/BN of the weight bytes) and per-tile epilogues, and too few tiles
// move work into stream-K splits, whose cross-CTA reduction (2-4 us of partial-sum stores, counters and reloads)
// dominates a GEMM of a few MB.  The rule below is the measured best (or within 3 %) on B200 over the Qwen decoder
// shapes and their 2/4/8-way shards at M = 1, 5 and 16:
//   a tile height BN in {128, 64, 32} (largest first) giving T = N/BN tiles with SMs/2 <= T <= SMs and at most
//   160 KiB of weights per tile (320 KiB when T >= 0.9 SMs)   -> BN x (32768/BN), T CTAs of one whole tile each
//   N >= ~1.8 x 128 x SMs  (gate_up, vocab head)            -> 128 x 256, stream-K
//   N >= ~0.9 x 64 x SMs   (qkv, gate_up shards)            -> 64 x 512, stream-K
//   smaller N with N*K >= 5120*6144 (o_proj, down)           -> 64 x 512, stream-K
//   otherwise (narrow shards)                                -> 32 x 1024, stream-K
// *dp_grid is the data-parallel grid (0: stream-K over all SMs).
void pick_tiles(int N, int K, int sms, int* bn, int* ks, int* dp_grid) {
  *dp_grid = 0;
  for (int h = 128; h >= 32; h >>= 1) {
    const long long t = (N + h - 1) / h;
    const long long bytes = static_cast<long long>(h) * K;
    const bool fits = bytes <= 160 * 1024 || (10 * t >= 9LL * sms && bytes <= 320 * 1024);
    if (2 * t >= sms && t <= sms && fits) {
      *bn = h;
      *ks = 32768 / h;
      *dp_grid = static_cast<int>(t);
      return;
    }
  }
  const long long t128 = (N + 127) / 128, t64 = (N + 63) / 64;
  if (10 * t128 >= 18LL * sms) {
    *bn = 128;
    *ks = 256;
  } else if (10 * t64 >= 9LL * sms || static_cast<long long>(N) * K >= 5120LL * 6144) {
    *bn = 64;
    *ks = 512;
  } else {
    *bn = 32;
    *ks = 1024;
  }
}

template <int BN, int NT, int KS, int HEAD, bool AR, bool SILU, bool NORM, bool TC = false>
int launch(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, Params& p, DeviceInfo* dinfo, int dev,
           unsigned flags, cudaStream_t stream) {
  using C = Geo<BN, NT, KS, NORM>;
  auto kern = w8a16_kernel<BN, NT, KS, HEAD, AR, SILU, NORM, TC>;
  static bool smem_attr_set[64] = {};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!smem_attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
      if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      smem_attr_set[dev] = true;
    }
  }
  CUtensorMap tw, tx;
  int rc = encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.N),
                     static_cast<uint64_t>(ldw), 128, p.silu_I ? BN / 2 : BN);
  if (rc) return rc;
  // activation boxes are M rows high: only the real tokens are copied
  const uint64_t xstride = (p.M > 1) ? static_cast<uint64_t>(ldx) * 2 : (static_cast<uint64_t>(p.K) * 2 + 15) / 16 * 16;
  rc = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.M),
                 xstride, 64, static_cast<uint32_t>(p.M));
  if (rc) return rc;
  CUtensorMap tr = tx;  // fused RMSNorm: the residual, same shape as x
  if (NORM && p.res) {
    const uint64_t rstride = (p.M > 1) ? static_cast<uint64_t>(p.ldr) * 2 : xstride;
    rc = encode_2d(&tr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.res, static_cast<uint64_t>(p.K),
                   static_cast<uint64_t>(p.M), rstride, 64, static_cast<uint32_t>(p.M));
    if (rc) return rc;
  }

  p.f16_path = f16_path();
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = p.M > 1 ? ldx : p.K;
  p.x_tx = static_cast<uint32_t>((NORM && p.res ? 2 : 1) * 2 * C::B * p.M * 128);
  p.kiters = (p.K + KS - 1) / KS;
  p.ntiles = p.silu_I ? (p.silu_I + BN / 2 - 1) / (BN / 2) : (p.N + BN - 1) / BN;
  if (p.ntiles > kMaxTiles) return fail(QF_ERR_SHAPE, "too many tiles for this tile height");
  if (p.ar_world && (p.ntiles > QF_AR_MAX_CHUNKS || static_cast<long long>(p.ntiles) * BN * p.M > p.ar_max_count))
    return fail(QF_ERR_SHAPE, "output too large for the all-reduce buffers (max_count) or more than "
                              "QF_AR_MAX_CHUNKS tiles");
  const long long total = static_cast<long long>(p.kiters) * p.ntiles;
  int G = dinfo->sm_count;
  if (G > kMaxGrid) G = kMaxGrid;
  if (p.G > 0 && G > p.G) G = p.G;  // data-parallel grid chosen with the tile shape
  if (grid_cap() > 0 && G > grid_cap()) G = grid_cap();
  if (G > total) G = static_cast<int>(total);
  p.G = G;
  p.q = p.ntiles / G;
  p.r = p.ntiles - p.q * G;
  p.Tsk = p.r * p.kiters;
  // At most about kMaxSplit CTAs share a stream-K tile: fewer, longer shares keep the fixup short (it reads every
  // contributor's partial) at a small cost in balance.
  long long gsk = p.Tsk < G ? p.Tsk : G;
  if (gsk > static_cast<long long>(kMaxSplit) * p.r) gsk = static_cast<long long>(kMaxSplit) * p.r;
  p.Gsk = static_cast<int>(gsk);
  if (p.q == 0) p.G = p.Gsk;  // all work is stream-K: CTAs without a share are not launched
  p.peer_wait_ns = peer_wait_ns();
  p.sk_skew = 0;
  if (p.q == 0 && p.Gsk > p.r && static_cast<long long>(p.Gsk) * p.Tsk < (1LL << 31)) {
    // every tile split: uneven shares, the short ones keeping at least two stages
    const int dmax = p.kiters - (2 * p.Gsk + p.r - 1) / p.r;
    p.sk_skew = sk_skew_stages() < dmax ? sk_skew_stages() : dmax;
    if (p.sk_skew < 0) p.sk_skew = 0;
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.G);
  cfg.blockDim = dim3(TC ? kTcThreads : kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & QF_FLAG_PDL) ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, tr, p);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("launch: ") + cudaGetErrorString(e));
  return QF_OK;
}

template <int BN, int KS, int HEAD, bool AR, bool SILU, bool NORM>
int launch_nt(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, Params& p, DeviceInfo* dinfo, int dev,
              unsigned flags, cudaStream_t st) {
  if (p.M <= 8) return launch<BN, 1, KS, HEAD, AR, SILU, NORM>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  // the fused RMSNorm also stages the residual: with two token tiles the 512- and 1024-byte stages would leave fewer
  // than three ring stages, so those tile heights run with half the k bytes per stage
  constexpr int KS2 = (NORM && KS >= 512 && BN * KS >= 32768) ? KS / 2 : KS;
  if constexpr (BN == 128 && KS2 == 256 && !NORM) {
    if (tc_mode() == 1) return launch<BN, 2, KS2, HEAD, AR, SILU, NORM, true>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  }
  return launch<BN, 2, KS2, HEAD, AR, SILU, NORM>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
}

// Optional fixed tile shape (QF_TILES="BN:KS"; 0 = the per-shape choice): used by the
// tests to run every kernel instance, and for tuning.
struct TileShape {
  int bn = 0, ks = 0;
};
const TileShape& tile_override() {
  static const TileShape v = [] {
    TileShape t;
    if (const char* e = test_env("QF_TILES")) {
      if (std::sscanf(e, "%d:%d", &t.bn, &t.ks) != 2) t = TileShape{};
    }
    return t;
  }();
  return v;
}

template <int HEAD, bool AR = false, bool SILU = false, bool NORM = false>
int launch_any(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, Params& p, DeviceInfo* dinfo, int dev,
               unsigned flags, cudaStream_t st) {
  int bn = tile_override().bn, ks = tile_override().ks, dp_grid = 0;
  if (bn == 0) pick_tiles(p.N, p.K, dinfo->sm_count, &bn, &ks, &dp_grid);
  p.G = dp_grid;  // launch() takes it as an upper bound of the grid
  if (bn == 128 && ks == 128) return launch_nt<128, 128, HEAD, AR, SILU, NORM>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  if (bn == 128 && ks == 256) return launch_nt<128, 256, HEAD, AR, SILU, NORM>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  if (bn == 64 && ks == 256) return launch_nt<64, 256, HEAD, AR, SILU, NORM>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  if (bn == 64 && ks == 512) return launch_nt<64, 512, HEAD, AR, SILU, NORM>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  if (bn == 32 && ks == 512) return launch_nt<32, 512, HEAD, AR, SILU, NORM>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  if (bn == 32 && ks == 1024) return launch_nt<32, 1024, HEAD, AR, SILU, NORM>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  return fail(QF_ERR_SHAPE, "no kernel instance for the chosen tile shape");
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
  (void)N;
  return kWsBytes;
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
  p.out_vec = reinterpret_cast<uintptr_t>(y) % 16 == 0 && (M == 1 || ldy % 8 == 0);
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
  return launch_any<0>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
}

int qf_w8a16_gemm_silu_mul(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale, void* y,
                           int64_t ldy, int M, int N, int K, void* ws, size_t ws_bytes, unsigned flags, void* stream) {
  int rc = check_common(x, ldx, w, ldw, scale, M, N, K, ws, ws_bytes);
  if (rc) return rc;
  if (N % 2) return fail(QF_ERR_SHAPE, "N must be even (gate rows [0, N/2), up rows [N/2, N))");
  if (M == 0 || N == 0) return QF_OK;
  if (K == 0) return fail(QF_ERR_SHAPE, "the fused gate needs K >= 1");
  if (!y) return fail(QF_ERR_INVALID, "null y");
  if (M > 1 && ldy < N / 2) return fail(QF_ERR_STRIDE, "ldy < N / 2");
  int dev;
  DeviceInfo* dinfo;
  rc = device_info(&dev, &dinfo);
  if (rc) return rc;
  Params p = {};
  p.scale = scale;
  p.y = y;
  p.ldy = ldy;
  p.out_vec = reinterpret_cast<uintptr_t>(y) % 16 == 0 && (M == 1 || ldy % 8 == 0);
  p.M = M;
  p.N = N;
  p.K = K;
  p.ws = static_cast<uint8_t*>(ws);
  p.silu_I = N / 2;
  return launch_any<0, false, true>(x, ldx, w, ldw, p, dinfo, dev, flags, static_cast<cudaStream_t>(stream));
}

int qf_w8a16_gemm_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, const void* gamma, float eps,
                          void* residual_out, int64_t ldro, const int8_t* w, int64_t ldw, const float* scale, void* y,
                          int64_t ldy, int M, int N, int K, int silu_mul, void* ws, size_t ws_bytes, unsigned flags,
                          void* stream) {
  int rc = check_common(x, ldx, w, ldw, scale, M, N, K, ws, ws_bytes);
  if (rc) return rc;
  if (M == 0 || N == 0) return QF_OK;
  if (K < 8 || K % 8 || K > kNormMaxK) return fail(QF_ERR_SHAPE, "the fused RMSNorm needs K % 8 == 0 and 8 <= K <= 8192");
  if (silu_mul && N % 2) return fail(QF_ERR_SHAPE, "N must be even with the fused SiLU gate");
  if (!y || !gamma) return fail(QF_ERR_INVALID, "null y or gamma");
  if (!(eps >= 0.f) || !std::isfinite(eps)) return fail(QF_ERR_INVALID, "eps must be finite and >= 0");
  if (M > 1 && ldy < (silu_mul ? N / 2 : N)) return fail(QF_ERR_STRIDE, "ldy too small");
  if (reinterpret_cast<uintptr_t>(gamma) % 16) return fail(QF_ERR_ALIGN, "gamma must be 16-byte aligned");
  if (residual) {
    if (M > 1 && ldr < K) return fail(QF_ERR_STRIDE, "ldr < K");
    if (reinterpret_cast<uintptr_t>(residual) % 16 || (M > 1 && ldr % 8))
      return fail(QF_ERR_ALIGN, "residual must be 16-byte aligned with ldr % 8 == 0");
  }
  if (residual_out) {
    if (M > 1 && ldro < K) return fail(QF_ERR_STRIDE, "ldro < K");
    if (reinterpret_cast<uintptr_t>(residual_out) % 16 || (M > 1 && ldro % 8))
      return fail(QF_ERR_ALIGN, "residual_out must be 16-byte aligned with ldro % 8 == 0");
    // every CTA reads the whole of x and residual: residual_out must not overlap them
    const uintptr_t o0 = reinterpret_cast<uintptr_t>(residual_out);
    const uintptr_t o1 = o0 + 2 * (static_cast<uint64_t>(M - 1) * (M > 1 ? ldro : K) + K);
    const void* ins[2] = {x, residual};
    const int64_t lds[2] = {ldx, ldr};
    for (int j = 0; j < 2; ++j) {
      if (!ins[j]) continue;
      const uintptr_t i0 = reinterpret_cast<uintptr_t>(ins[j]);
      const uintptr_t i1 = i0 + 2 * (static_cast<uint64_t>(M - 1) * (M > 1 ? lds[j] : K) + K);
      if (o0 < i1 && i0 < o1) return fail(QF_ERR_INVALID, "residual_out overlaps x or residual");
    }
  }
  int dev;
  DeviceInfo* dinfo;
  rc = device_info(&dev, &dinfo);
  if (rc) return rc;
  Params p = {};
  p.scale = scale;
  p.y = y;
  p.ldy = ldy;
  p.out_vec = reinterpret_cast<uintptr_t>(y) % 16 == 0 && (M == 1 || ldy % 8 == 0);
  p.M = M;
  p.N = N;
  p.K = K;
  p.ws = static_cast<uint8_t*>(ws);
  p.res = static_cast<const __nv_bfloat16*>(residual);
  p.ldr = M > 1 ? ldr : K;
  p.gamma = static_cast<const __nv_bfloat16*>(gamma);
  p.res_out = static_cast<__nv_bfloat16*>(residual_out);
  p.ldro = M > 1 ? ldro : K;
  p.eps = eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (silu_mul) {
    p.silu_I = N / 2;
    return launch_any<0, false, true, true>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
  }
  return launch_any<0, false, false, true>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
}

int qf_w8a16_gemm_allreduce(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale, void* y,
                            int64_t ldy, int M, int N, int K, void* ws, size_t ws_bytes, int rank, int world,
                            void* const* bufs, int max_count, unsigned flags, void* stream) {
  int rc = check_common(x, ldx, w, ldw, scale, M, N, K, ws, ws_bytes);
  if (rc) return rc;
  if (world < 1 || world > QF_AR_MAX_RANKS) return fail(QF_ERR_INVALID, "world size must be 1..8");
  if (rank < 0 || rank >= world) return fail(QF_ERR_INVALID, "rank out of range");
  if (max_count <= 0 || max_count % 8) return fail(QF_ERR_SHAPE, "max_count must be a positive multiple of 8");
  if (M == 0 || N == 0) return QF_OK;
  if (K == 0) return fail(QF_ERR_SHAPE, "the fused all-reduce needs K >= 1");
  if (!y || !bufs) return fail(QF_ERR_INVALID, "null y or buffer list");
  if (M > 1 && ldy < N) return fail(QF_ERR_STRIDE, "ldy < N");
  for (int r = 0; r < world; ++r)
    if (!bufs[r] || reinterpret_cast<uintptr_t>(bufs[r]) % 256)
      return fail(QF_ERR_ALIGN, "buffers must be non-null and 256-byte aligned");
  int dev;
  DeviceInfo* dinfo;
  rc = device_info(&dev, &dinfo);
  if (rc) return rc;
  Params p = {};
  p.scale = scale;
  p.y = y;
  p.ldy = ldy;
  p.out_vec = reinterpret_cast<uintptr_t>(y) % 16 == 0 && (M == 1 || ldy % 8 == 0);
  p.M = M;
  p.N = N;
  p.K = K;
  p.ws = static_cast<uint8_t*>(ws);
  p.ar_world = world;
  p.ar_rank = rank;
  p.ar_max_count = max_count;
  for (int r = 0; r < world; ++r) p.ar_bufs[r] = static_cast<uint8_t*>(bufs[r]);
  return launch_any<0, true>(x, ldx, w, ldw, p, dinfo, dev, flags, static_cast<cudaStream_t>(stream));
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
  p.out_vec = reinterpret_cast<uintptr_t>(logits) % 16 == 0 && (M == 1 || ldl % 8 == 0);
  p.n_valid = n_valid;
  p.vocab_offset = vocab_offset;
  p.row_max = row_max;
  p.row_argmax = reinterpret_cast<long long*>(row_argmax);
  p.row_lse = row_lse;
  p.inv_temp = 1.0f;
  return launch_any<1>(x, ldx, w, ldw, p, dinfo, dev, flags, static_cast<cudaStream_t>(stream));
}

int qf_w8a16_head_sample(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale,
                         void* logits, int64_t ldl, int M, int N, int K, int n_valid, int64_t vocab_offset,
                         float inv_temperature, uint64_t seed, uint64_t offset, float* row_max,
                         int64_t* row_argmax, float* row_lse, int64_t* row_sample, float* row_sample_score,
                         float* row_sample_logit, void* ws, size_t ws_bytes, unsigned flags, void* stream) {
  int rc = check_common(x, ldx, w, ldw, scale, M, N, K, ws, ws_bytes);
  if (rc) return rc;
  if (M == 0) return QF_OK;
  if (N == 0 || K == 0) return fail(QF_ERR_SHAPE, "the head needs N >= 1 and K >= 1");
  if (n_valid < 1 || n_valid > N) return fail(QF_ERR_SHAPE, "n_valid must be in [1, N]");
  if (!row_max || !row_argmax || !row_lse || !row_sample || !row_sample_score || !row_sample_logit)
    return fail(QF_ERR_INVALID, "null row statistics output");
  if (!(inv_temperature > 0.f) || !std::isfinite(inv_temperature))
    return fail(QF_ERR_INVALID, "inv_temperature must be finite and > 0");
  if (vocab_offset < 0 || vocab_offset + N > (1LL << 32)) return fail(QF_ERR_SHAPE, "vocabulary beyond 2^32 columns");
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
  p.out_vec = reinterpret_cast<uintptr_t>(logits) % 16 == 0 && (M == 1 || ldl % 8 == 0);
  p.n_valid = n_valid;
  p.vocab_offset = vocab_offset;
  p.row_max = row_max;
  p.row_argmax = reinterpret_cast<long long*>(row_argmax);
  p.row_lse = row_lse;
  p.inv_temp = inv_temperature;
  p.seed_lo = static_cast<uint32_t>(seed);
  p.seed_hi = static_cast<uint32_t>(seed >> 32);
  p.off_lo = static_cast<uint32_t>(offset);
  p.off_hi = static_cast<uint32_t>(offset >> 32);
  p.row_sample = reinterpret_cast<long long*>(row_sample);
  p.row_sample_score = row_sample_score;
  p.row_sample_logit = row_sample_logit;
  return launch_any<2>(x, ldx, w, ldw, p, dinfo, dev, flags, static_cast<cudaStream_t>(stream));
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
// qf_w8a16_gemm_noalloc: the same GEMM with its scratch (split-tile counters and fp32 partial tiles) in a fixed
// array of this library instead of a caller-provided workspace, for callers that cannot allocate device memory
// themselves (a host that embeds only this library and has no device allocator, e.g. a Go or Java binding over
// the C ABI, or a latency-critical path that must not call cudaMalloc, which can synchronise the device).  The
// array lives in every GPU that loads the library until the process exits.
namespace qf {
namespace {

constexpr int kNoAllocMaxGrid = 160;                 // CTAs: partial-tile slots are 2 per CTA
constexpr size_t kNoAllocBytes = kWsPartials + sizeof(float) * kPartialSlotFloats * 2 * kNoAllocMaxGrid;
static_assert(kNoAllocBytes == QF_NOALLOC_SCRATCH_BYTES, "header value out of date");
// Tiles are at least 32 output channels high and the array holds kMaxTiles tile counters.
static_assert(static_cast<long long>(QF_NOALLOC_MAX_N) <= 32LL * kMaxTiles, "tile counters of the fixed scratch");

__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of the scratch array for the current device, looked up once per device (with that device
// current).  The host-side symbol is only a stand-in, never a device address.  The first lookup also zeroes the
// error word and the tile counters, enqueued on `stream` ahead of the first kernel; from then on every kernel
// leaves its counters at zero again, as on a caller's workspace.
int noalloc_scratch(int dev, cudaStream_t stream, void** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(QF_ERR_LAUNCH, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    e = cudaMemsetAsync(ptr, 0, kWsZeroBytes, stream);
    if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
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
    return fail(QF_ERR_SHAPE, "N above QF_NOALLOC_MAX_N (262144): the fixed scratch of the allocation-free entry "
                              "point holds 8192 tile counters, and tiles are at least 32 output channels high");
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
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  rc = noalloc_scratch(dev, st, &scratch);
  if (rc) return rc;
  // The array keeps the previous call's contents.  What must start at zero -- the tile counters -- was zeroed when
  // the array was first used on this device, and every call leaves it at zero again; the error word stays set
  // until qf_w8a16_noalloc_status reads it.
  Params p = {};
  p.scale = scale;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = y;
  p.ldy = ldy;
  p.y_f32 = y_dtype == QF_DTYPE_F32;
  p.out_vec = reinterpret_cast<uintptr_t>(y) % 16 == 0 && (M == 1 || ldy % 8 == 0);
  p.M = M;
  p.N = N;
  p.K = K;
  p.ws = static_cast<uint8_t*>(scratch);
  if (K == 0) {
    const int64_t total = static_cast<int64_t>(M) * N;
    fill_empty_k_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, cudaGetErrorString(e));
  }
  return launch_any<0>(x, ldx, w, ldw, p, dinfo, dev, flags, st);
}

extern "C" int qf_w8a16_noalloc_status(void* stream, int* status) {
  if (!status) return fail(QF_ERR_INVALID, "null status");
  int dev;
  DeviceInfo* dinfo;
  int rc = device_info(&dev, &dinfo);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  rc = noalloc_scratch(dev, st, &scratch);
  if (rc) return rc;
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, scratch, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  // A call that gave up waiting may have left tile counters set: start the next call from a clean array.
  if (e == cudaSuccess && v != 0) e = cudaMemsetAsync(scratch, 0, kWsZeroBytes, st);
  if (e == cudaSuccess && v != 0) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, cudaGetErrorString(e));
  *status = v;
  return QF_OK;
}
