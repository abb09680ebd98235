// qf_spec_attn.cu -- sm_100a split-KV, GQA-packed attention for uniform speculative-verification batches.
//
// Replaces gqa_packed_spec_attention of EurekaZang/qwen-a100-fastpath (plugin/qwen_fastpath/spec_attn.py:139-173,
// Triton kernels :17-136), to which the plugin routes uniform speculative-decode batches (patches.py:10-69).
// Semantics (spec_attn.py:141-146): num_reqs requests x Q query tokens each (token b*Q + qi); query qi of request b
// attends the cached keys [0, seq_lens[b] - Q + qi] of a paged cache (page block_table[b][pos / page], slot
// pos % page), softmax scale `scale`, G = H / HKV query heads per KV head; a row with no key gives zeros (:129-130).
//
// Design (B200):
// * The R = Q*G query rows that share a KV head are packed into one tile (16-row m-tiles), so a request's KV head is
//   read once for all of them, as in the reference.  The keys [0, seq_len) -- the cached prefix and the Q in-flight
//   tokens alike, the causal limit applied as a per-row mask -- are split into n_split chunks of >= 128 tokens
//   (multiples of 32): chunk = ceil(seq_len / S) rounded up, S = SMs / (num_reqs * HKV) splits per (request,
//   KV head), so one launch of S x (num_reqs * HKV) CTAs fills the SMs once.
// * The chunk's K and V are streamed with TMA -- one 4-D tensor map per cache (head dim, slot, KV head, page; or
//   slot and KV head swapped, whichever has the smaller stride first), 64-column x 16-token boxes with the 128-byte
//   swizzle, the page looked up in the block table for every 16 tokens (page sizes are multiples of 16) -- into a
//   ring of 32-token stages: an mbarrier per stage counts the bytes in, and the last warp to finish with a stage
//   (a shared-memory acq_rel counter) refills it.  There is no producer warp, so the CTA is 8 warps and every warp
//   may hold 255 registers (the D = 256 output tile alone is 128 per thread).  Warp (m-tile mt, slice ts) takes
//   every W-th 16-token slice: S = Q K^T with mma.sync m16n8k16 (Q and K fragments by ldmatrix from the swizzled
//   tiles), online softmax in base 2 with fp32 statistics, P rounded to bf16 in registers as the A operand of
//   O += P V (V fragments by ldmatrix.trans).  The W warps of an m-tile merge their (max, sum, O) in shared memory.
// * A request with one split writes its output directly.  Otherwise each CTA writes its normalized partial output
//   and base-2 log-sum-exp, and a second kernel (one CTA per output row, programmatic dependent launch) merges the
//   splits by the log-sum-exp rule, recomputing the split arithmetic from seq_lens: nothing depends on a host-side
//   value, so both launches are CUDA-graph safe.
// * A 16-token box may bring in slots past the chunk's end (same page, possibly never written): they are masked in
//   S, and their V rows are zeroed in shared memory before P V, so stale values (NaN included) never reach the
//   output.
// * Arithmetic intensity: 2 * 2 * R_pad * D flop per 4 * D bytes of K and V, i.e. R_pad flop per byte (R_pad = 16 x
//   m-tiles, 32 for Q*G <= 32): at the measured HBM bandwidth that is about 0.2 PFLOP/s, a third of what the
//   mma.sync pipe sustains, so the kernel is HBM-bound; tcgen05 tiles (M >= 64 rows) would leave most rows empty.
// * Every mbarrier wait is bounded (4 s): on expiry the CTA records QF_ERR_TIMEOUT in the workspace header, the
//   warps stop, and one thread waits (bounded) for the copies still in flight before the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/qf_b200.h"
#include "qf_host.h"
#include "qf_ptx.cuh"

namespace qf {
namespace {

constexpr int kSaSlice = 16;        // tokens per consumer slice (one k-step of P V)
constexpr int kSaStageTok = 32;     // tokens per ring stage (two slices)
constexpr int kSaMinChunk = 128;    // smallest split, tokens
constexpr int kSaMaxSplits = 160;
constexpr int kSaBtCache = 512;     // block-table entries of a chunk kept in shared memory
constexpr size_t kSaHeader = 256;   // workspace: [0] error word
constexpr uint64_t kSaWaitNs = 4000000000ull;

template <int D, int MT> struct SaGeo {
  static constexpr int W = MT == 1 ? 8 : MT == 2 ? 4 : 2;  // slices in flight (warps per m-tile)
  static constexpr int CW = MT * W;                         // warps
  static constexpr int kThreads = CW * 32;
  static constexpr int kBoxes = D / 64;                     // 64-column boxes per token row
  static constexpr int kBoxBytes = kSaSlice * 128;          // [16 tokens][64 bf16], 128-byte swizzle
  static constexpr int kSliceBytes = kBoxes * kBoxBytes;    // one slice of K or of V
  static constexpr int kStageBytes = 4 * kSliceBytes;       // K slice 0, K slice 1, V slice 0, V slice 1
  static constexpr int kQBoxBytes = 16 * MT * 128;          // [16 MT rows][64 bf16] per box
  // the deepest ring that fits beside the Q tile, the block-table cache and the barriers (227 KiB per CTA)
  static constexpr int kStagesFit = (227 * 1024 - kBoxes * kQBoxBytes - 4 * kSaBtCache - 2048) / kStageBytes;
  static constexpr int kStages = kStagesFit > 12 ? 12 : kStagesFit;
  static constexpr int kOffQ = kStages * kStageBytes;
  static constexpr int kOffBt = kOffQ + kBoxes * kQBoxBytes;  // int [kSaBtCache]: the chunk's pages
  static constexpr int kOffBar = kOffBt + 4 * kSaBtCache;
  static constexpr int kOffCnt = kOffBar + kStages * 8;     // per stage: warps done with it
  static constexpr int kOffMisc = kOffCnt + kStages * 4;     // abort flag, stages issued
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;   // + slack for the 1024-byte alignment
  // merge scratch in the ring once every stage is consumed: per warp O [16][D + 8] fp32 (padded rows), then
  // the row maxima [16] and sums [16]
  static constexpr int kMergeO = 16 * (D + 8);
  static constexpr int kMergeWarp = kMergeO + 32;
  static_assert(kStages >= 3, "ring too shallow");
  static_assert(CW * kMergeWarp * 4 <= kStages * kStageBytes, "merge scratch exceeds the ring");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
  static_assert(D % 64 == 0 && (D / 8) % W == 0, "columns per merging warp");
};

struct SaParams {
  const __nv_bfloat16* q;  // [num_reqs * Q tokens][H][D]
  int64_t sq_t, sq_h;
  const int* block_table;  // [num_reqs][*]
  int64_t s_bt;
  const int* seq_lens;     // [num_reqs]
  __nv_bfloat16* out;      // [num_reqs * Q tokens][H][D]
  int64_t so_t, so_h;
  float* o_part;           // [num_reqs][HKV][max_splits][R][D], normalized partial outputs
  float* lse_part;         // [num_reqs][HKV][max_splits][R], base-2 log-sum-exp of the scaled scores
  int* err;
  int Q, G, R, HKV, page, max_splits;
  int head_inner;          // tensor-map coordinate order: 0 = (d, slot, head, page), 1 = (d, head, slot, page)
  float qk_scale;          // scale * log2(e)
};

// Split arithmetic shared by both kernels: chunk length (tokens, a multiple of 32) and number of active splits.
__device__ __forceinline__ void sa_split(int seq_len, int max_splits, int& chunk, int& n_split) {
  const int L = seq_len > 0 ? seq_len : 0;
  int c = (L + max_splits - 1) / max_splits;
  c = c < kSaMinChunk ? kSaMinChunk : c;
  chunk = (c + kSaStageTok - 1) / kSaStageTok * kSaStageTok;
  n_split = L > 0 ? (L + chunk - 1) / chunk : 1;
}

// Byte offset of 16-byte chunk c (0 .. D/8 - 1) of row r in a tile stored as 64-column boxes of 128-byte rows with the
// 128-byte swizzle (chunk index XOR row % 8; box bases 1024-byte aligned), box_bytes apart.
__device__ __forceinline__ uint32_t sw_off(int r, int c, int box_bytes) {
  return static_cast<uint32_t>((c >> 3) * box_bytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ bool sa_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (*abort_flag) return false;
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kSaWaitNs) return false;
  }
}

__device__ __forceinline__ void sa_abort(const SaParams& p, volatile int* abort_flag) {
  if (!*abort_flag) atomicExch(p.err, QF_ERR_TIMEOUT);
  *abort_flag = 1;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Shared-memory add with acquire + release semantics at CTA scope: the caller's earlier accesses of the stage are
// complete for whoever sees the new count, and the last warp to count itself sees everyone else's.
__device__ __forceinline__ uint32_t atom_add_acq_rel_cta_shared(uint32_t* ptr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(smem_u32(ptr)), "r"(v) : "memory");
  return old;
}

// Issues the TMA copies of stage st (its one or two 16-token slices below `end`) into its ring slot.
template <int D, int MT>
__device__ __forceinline__ void sa_issue(const CUtensorMap* tk, const CUtensorMap* tv, const SaParams& p, uint8_t* smem,
                                         uint64_t* full, const int* bt, const int* sBt, int pg0, int hkv, int start,
                                         int end, int st, uint64_t pol) {
  using C = SaGeo<D, MT>;
  const int slot = st % C::kStages;
  const int p0 = start + st * kSaStageTok;
  const int nsl = end - p0 > kSaSlice ? 2 : 1;  // slices holding a token < end
  mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nsl * 2 * C::kSliceBytes));
  uint8_t* dst = smem + slot * C::kStageBytes;
  for (int sl = 0; sl < nsl; ++sl) {
    const int pos = p0 + sl * kSaSlice;
    const int pg = pos / p.page;
    const int blk = pg - pg0 < kSaBtCache ? sBt[pg - pg0] : __ldg(bt + pg);
    const int off = pos - pg * p.page;
    const int c1 = p.head_inner ? hkv : off;
    const int c2 = p.head_inner ? off : hkv;
#pragma unroll
    for (int i = 0; i < C::kBoxes; ++i) {
      tma_load_4d(dst + sl * C::kSliceBytes + i * C::kBoxBytes, tk, &full[slot], 64 * i, c1, c2, blk, pol);
      tma_load_4d(dst + (2 + sl) * C::kSliceBytes + i * C::kBoxBytes, tv, &full[slot], 64 * i, c1, c2, blk, pol);
    }
  }
}

template <int D, int MT>
__global__ void __launch_bounds__(SaGeo<D, MT>::kThreads, 1)
    spec_attn_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                     const SaParams p) {
  using C = SaGeo<D, MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint32_t* done = reinterpret_cast<uint32_t*>(smem + C::kOffCnt);
  volatile int* sAbort = reinterpret_cast<volatile int*>(smem + C::kOffMisc);
  int* sIssued = reinterpret_cast<int*>(smem + C::kOffMisc + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int b = blockIdx.y / p.HKV;
  const int hkv = blockIdx.y - b * p.HKV;

  pdl_launch_dependents();  // the merge kernel may be scheduled now; it waits for this grid before reading
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      done[i] = 0;
    }
    *sAbort = 0;
    *sIssued = 0;
    fence_mbar_init();
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
  }
  __syncthreads();
  pdl_wait();  // queries, cache, block table and lengths are written by earlier kernels
  const int seq_len = __ldg(p.seq_lens + b);
  int chunk, n_split;
  sa_split(seq_len, p.max_splits, chunk, n_split);
  if (split >= n_split) return;
  const int start = split * chunk;
  const int end = min(start + chunk, max(seq_len, 0));
  const int n_stages = end > start ? (end - start + kSaStageTok - 1) / kSaStageTok : 0;
  const int* bt = p.block_table + static_cast<int64_t>(b) * p.s_bt;
  const uint64_t pol = policy_evict_first();  // the cache is read once
  // the chunk's pages into shared memory in one round trip (the copies of every stage need one)
  int* sBt = reinterpret_cast<int*>(smem + C::kOffBt);
  const int pg0 = start / p.page;
  if (n_stages > 0) {
    const int npg = (end - 1) / p.page - pg0 + 1;
    for (int i = threadIdx.x; i < npg && i < kSaBtCache; i += C::kThreads) sBt[i] = __ldg(bt + pg0 + i);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // the first ring's worth of stages
    const int n0 = n_stages < C::kStages ? n_stages : C::kStages;
    for (int st = 0; st < n0; ++st) sa_issue<D, MT>(&tk, &tv, p, smem, full, bt, sBt, pg0, hkv, start, end, st, pol);
    *sIssued = n0;
  }

  // ------------------------------------------------------------------------------------------------ consumers
  const int mt = warp % MT;
  const int ts = warp / MT;
  const int g = lane >> 2;
  const int t = lane & 3;
  uint8_t* sQ = smem + C::kOffQ;
  const int hq0 = hkv * p.G;
  // the packed query rows r = qi * G + gg (token b * Q + qi, head hq0 + gg) into the swizzled Q tile; rows >= R zero
  for (int idx = threadIdx.x; idx < 16 * MT * (D / 8); idx += C::CW * 32) {
    const int r = idx / (D / 8);
    const int c = idx - r * (D / 8);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < p.R) {
      const int qi = r / p.G;
      const int gg = r - qi * p.G;
      v = *reinterpret_cast<const uint4*>(p.q + static_cast<int64_t>(b * p.Q + qi) * p.sq_t +
                                          static_cast<int64_t>(hq0 + gg) * p.sq_h + c * 8);
    }
    *reinterpret_cast<uint4*>(sQ + sw_off(r, c, C::kQBoxBytes)) = v;
  }
  __syncthreads();

  const uint32_t ring_u = smem_u32(smem);
  const uint32_t q_u = smem_u32(sQ);
  const int a_row = 16 * mt + (lane & 15);                      // Q fragment rows / chunks (ldmatrix lanes)
  const int a_ch = lane >> 4;
  const int k_tok = (lane & 7) + ((lane >> 4) << 3);            // K: matrices (tok 0-7 | 8-15) x (k 0-7 | 8-15)
  const int k_ch = (lane >> 3) & 1;
  const int v_tok = (lane & 7) + (((lane >> 3) & 1) << 3);      // V (transposed): (tok 0-7, 8-15) x (d 0-7 | 8-15)
  const int v_ch = lane >> 4;
  const int lim0 = seq_len - p.Q;                               // row r sees slots <= lim0 + r / G
  const int lim_a = lim0 + (16 * mt + g) / p.G;
  const int lim_b = lim0 + (16 * mt + g + 8) / p.G;

  float m_run[2] = {-INFINITY, -INFINITY};  // rows g, g + 8 (base-2, scaled)
  float l_run[2] = {0.f, 0.f};              // this lane's part of the row sums
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;

  for (int st = 0; st < n_stages; ++st) {
    const int j0 = 2 * st;
    const int my = (j0 % C::W) == ts ? 0 : ((j0 + 1) % C::W) == ts ? 1 : -1;
    if (my < 0) continue;
    const int slot = st % C::kStages;
    int got = 1;
    if (lane == 0) {
      got = sa_wait(&full[slot], (st / C::kStages) & 1, sAbort) ? 1 : 0;
      if (!got) sa_abort(p, sAbort);
    }
    got = __shfl_sync(0xffffffffu, got, 0);
    if (!got) break;
    const int pos0 = start + st * kSaStageTok + my * kSaSlice;
    if (pos0 < end) {
      const uint32_t kb = ring_u + slot * C::kStageBytes + my * C::kSliceBytes;
      const uint32_t vb = kb + 2 * C::kSliceBytes;
      if (pos0 + kSaSlice > end) {  // slots past the chunk's end: V rows to zero before P V
        uint8_t* vg = smem + slot * C::kStageBytes + (2 + my) * C::kSliceBytes;
        const int valid = end - pos0;
        for (int idx = lane; idx < (kSaSlice - valid) * (D / 8); idx += 32) {
          const int tk = valid + idx / (D / 8);
          const int c = idx - (tk - valid) * (D / 8);
          *reinterpret_cast<uint4*>(vg + sw_off(tk, c, C::kBoxBytes)) = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }
      // S = Q K^T for 16 rows x 16 slots, two accumulator sets (even / odd k-steps) for independent MMA chains; the
      // fragments of k-step kk + 1 are loaded before the MMAs of kk is issued
      float sa[2][4], sb[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sa[nt][e] = sb[nt][e] = 0.f;
      uint32_t fa[2][4], fb[2][4];
      ldsm_x4(q_u + sw_off(a_row, a_ch, C::kQBoxBytes), fa[0][0], fa[0][1], fa[0][2], fa[0][3]);
      ldsm_x4(kb + sw_off(k_tok, k_ch, C::kBoxBytes), fb[0][0], fb[0][1], fb[0][2], fb[0][3]);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int c = kk & 1;
        if (kk + 1 < D / 16) {
          ldsm_x4(q_u + sw_off(a_row, 2 * (kk + 1) + a_ch, C::kQBoxBytes), fa[c ^ 1][0], fa[c ^ 1][1], fa[c ^ 1][2],
                  fa[c ^ 1][3]);
          ldsm_x4(kb + sw_off(k_tok, 2 * (kk + 1) + k_ch, C::kBoxBytes), fb[c ^ 1][0], fb[c ^ 1][1], fb[c ^ 1][2],
                  fb[c ^ 1][3]);
        }
        float (&s0)[4] = c ? sb[0] : sa[0];
        float (&s1)[4] = c ? sb[1] : sa[1];
        mma_bf16_m16n8k16(s0, fa[c][0], fa[c][1], fa[c][2], fa[c][3], fb[c][0], fb[c][1]);
        mma_bf16_m16n8k16(s1, fa[c][0], fa[c][1], fa[c][2], fa[c][3], fb[c][2], fb[c][3]);
      }
      // the first V fragments do not depend on P: load them before the softmax
      uint32_t fv[2][4];
      ldsm_x4_trans(vb + sw_off(v_tok, v_ch, C::kBoxBytes), fv[0][0], fv[0][1], fv[0][2], fv[0][3]);
      // scaled scores (base 2), masked past the chunk's end and past each row's causal limit
      const bool unmasked = pos0 + kSaSlice <= end && pos0 + kSaSlice - 1 <= lim0;
      float x[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = (sa[nt][e] + sb[nt][e]) * p.qk_scale;
          if (!unmasked) {
            const int pos = pos0 + 8 * nt + 2 * t + (e & 1);
            if (pos >= end || pos > (e < 2 ? lim_a : lim_b)) v = -INFINITY;
          }
          x[nt][e] = v;
        }
      // online softmax: row maxima over the four lanes of a row, rescale of the running sums and outputs
      float mx0 = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
      float mx1 = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m_run[0], mx0);
      const float mn1 = fmaxf(m_run[1], mx1);
      const float mu0 = mn0 == -INFINITY ? 0.f : mn0;  // no key yet: any finite reference keeps 2^(-inf) = 0
      const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = ex2_approx(m_run[0] - mu0);
      const float al1 = ex2_approx(m_run[1] - mu1);
      m_run[0] = mn0;
      m_run[1] = mn1;
      float pr[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) pr[nt][e] = ex2_approx(x[nt][e] - (e < 2 ? mu0 : mu1));
      l_run[0] = l_run[0] * al0 + ((pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]));
      l_run[1] = l_run[1] * al1 + ((pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]));
      if (!__all_sync(0xffffffffu, al0 == 1.f && al1 == 1.f)) {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[n][0] *= al0;
          o[n][1] *= al0;
          o[n][2] *= al1;
          o[n][3] *= al1;
        }
      }
      // O += P V: P (bf16) as the A operand straight from the score registers
      const uint32_t pa0 = pack_bf16x2(pr[0][0], pr[0][1]);
      const uint32_t pa1 = pack_bf16x2(pr[0][2], pr[0][3]);
      const uint32_t pa2 = pack_bf16x2(pr[1][0], pr[1][1]);
      const uint32_t pa3 = pack_bf16x2(pr[1][2], pr[1][3]);
#pragma unroll
      for (int j = 0; j < D / 16; ++j) {
        const int c = j & 1;
        if (j + 1 < D / 16)
          ldsm_x4_trans(vb + sw_off(v_tok, 2 * (j + 1) + v_ch, C::kBoxBytes), fv[c ^ 1][0], fv[c ^ 1][1], fv[c ^ 1][2],
                        fv[c ^ 1][3]);
        mma_bf16_m16n8k16(o[2 * j], pa0, pa1, pa2, pa3, fv[c][0], fv[c][1]);
        mma_bf16_m16n8k16(o[2 * j + 1], pa0, pa1, pa2, pa3, fv[c][2], fv[c][3]);
      }
    }
    __syncwarp();
    if (lane == 0 && atom_add_acq_rel_cta_shared(&done[slot], 1u) == 2 * MT - 1) {
      // the last of the stage's 2 MT warps: the slot is free; refill it with stage st + kStages
      done[slot] = 0;
      if (st + C::kStages < n_stages) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // our generic accesses before the copies
        sa_issue<D, MT>(&tk, &tv, p, smem, full, bt, sBt, pg0, hkv, start, end, st + C::kStages, pol);
        atomicMax(sIssued, st + C::kStages + 1);
      }
    }
  }

  // ---------------------------------------------------------------------- merge of the W warps of each m-tile
  __syncthreads();  // every stage consumed: the ring becomes merge scratch
  if (*sAbort) {
    // a wait expired: copies of the last issued stages may still be in flight; let them land (bounded) and stop
    if (threadIdx.x == 0) {
      const int issued = *sIssued;
      for (int s2 = issued > C::kStages ? issued - C::kStages : 0; s2 < issued; ++s2) {
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&full[s2 % C::kStages], (s2 / C::kStages) & 1) && global_timer_ns() - t0 < kSaWaitNs) {
        }
      }
    }
    return;
  }
  float* scr = reinterpret_cast<float*>(smem);
  float* mine = scr + warp * C::kMergeWarp;
  l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], 1);
  l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], 2);
  l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], 1);
  l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], 2);
  if (t == 0) {
    mine[C::kMergeO + g] = m_run[0];
    mine[C::kMergeO + 8 + g] = m_run[1];
    mine[C::kMergeO + 16 + g] = l_run[0];
    mine[C::kMergeO + 24 + g] = l_run[1];
  }
  __syncthreads();
  float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
  for (int w2 = 0; w2 < C::W; ++w2) {
    const float* o2 = scr + (mt + MT * w2) * C::kMergeWarp + C::kMergeO;
    M0 = fmaxf(M0, o2[g]);
    M1 = fmaxf(M1, o2[8 + g]);
  }
  const float Mu0 = M0 == -INFINITY ? 0.f : M0;
  const float Mu1 = M1 == -INFINITY ? 0.f : M1;
  float L0 = 0.f, L1 = 0.f;
#pragma unroll
  for (int w2 = 0; w2 < C::W; ++w2) {
    const float* o2 = scr + (mt + MT * w2) * C::kMergeWarp + C::kMergeO;
    L0 += o2[16 + g] * ex2_approx(o2[g] - Mu0);
    L1 += o2[24 + g] * ex2_approx(o2[8 + g] - Mu1);
  }
  const float f0 = L0 > 0.f ? ex2_approx(m_run[0] - Mu0) / L0 : 0.f;  // this warp's share, normalized
  const float f1 = L1 > 0.f ? ex2_approx(m_run[1] - Mu1) / L1 : 0.f;
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    *reinterpret_cast<float2*>(mine + g * (D + 8) + 8 * n + 2 * t) = make_float2(o[n][0] * f0, o[n][1] * f0);
    *reinterpret_cast<float2*>(mine + (g + 8) * (D + 8) + 8 * n + 2 * t) = make_float2(o[n][2] * f1, o[n][3] * f1);
  }
  __syncthreads();
  // warp (mt, ts) sums columns [ts * D / W, (ts + 1) * D / W) of the m-tile's rows over the W warps and stores them
  constexpr int kCols = D / C::W;
  constexpr int kQuads = kCols / 4;
  const bool single = n_split == 1;
  const int64_t part_row0 = (static_cast<int64_t>(b * p.HKV + hkv) * p.max_splits + split) * p.R;
  for (int idx = lane; idx < 16 * kQuads; idx += 32) {
    const int row = idx / kQuads;
    const int col = ts * kCols + 4 * (idx - row * kQuads);
    const int r = 16 * mt + row;
    if (r >= p.R) continue;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w2 = 0; w2 < C::W; ++w2) {
      const float4 v = *reinterpret_cast<const float4*>(scr + (mt + MT * w2) * C::kMergeWarp + row * (D + 8) + col);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    if (single) {
      const int qi = r / p.G;
      __nv_bfloat16* dst = p.out + static_cast<int64_t>(b * p.Q + qi) * p.so_t +
                           static_cast<int64_t>(hq0 + r - qi * p.G) * p.so_h + col;
      uint2 w;
      w.x = pack_bf16x2(acc.x, acc.y);
      w.y = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(dst) = w;
    } else {
      *reinterpret_cast<float4*>(p.o_part + (part_row0 + r) * D + col) = acc;
    }
  }
  if (!single && ts == 0 && t == 0) {
    const int ra = 16 * mt + g;
    if (ra < p.R) p.lse_part[part_row0 + ra] = L0 > 0.f ? M0 + log2f(L0) : -INFINITY;
    if (ra + 8 < p.R) p.lse_part[part_row0 + ra + 8] = L1 > 0.f ? M1 + log2f(L1) : -INFINITY;
  }
}

// Loads issued in program order (volatile asm: the compiler neither sinks them below a branch nor drops them), plain
// weak global loads like the compiler's own.
__device__ __forceinline__ int ld_issue_s32(const int* ptr) {
  int v;
  asm volatile("ld.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr));
  return v;
}
__device__ __forceinline__ float ld_issue_f32(const float* ptr) {
  float v;
  asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(ptr));
  return v;
}
__device__ __forceinline__ float4 ld_issue_f32x4(const float4* ptr) {
  float4 v;
  asm volatile("ld.global.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(ptr));
  return v;
}

// Merge of the splits: one CTA of 256 threads per output row (request, KV head, packed row r); thread (group sg,
// column quad c) sums the splits s = sg, sg + NG, ... of its four columns.  The request's length, every split's
// log-sum-exp and the first kMergeSpec splits of each thread are loaded at once, before the split count is known (the
// slots of every possible split lie in the workspace; those at or past the count are never used), so the merge costs
// one memory round trip after the dependency wait instead of three.  out = sum_s 2^(lse_s - m) o_s /
// sum_s 2^(lse_s - m), m = max_s lse_s (zeros when every split is empty).  Rows of requests with a single split were
// written by the attention kernel.
constexpr int kMergeSpec = 12;
template <int D>
__global__ void __launch_bounds__(256) spec_attn_merge_kernel(const SaParams p) {
  constexpr int NQ = D / 4;    // float4 columns per row
  constexpr int NG = 256 / NQ; // split groups
  static_assert(kSaMaxSplits <= 256, "one log-sum-exp per thread");
  __shared__ float sW[kSaMaxSplits];
  __shared__ float sRed[8];
  __shared__ float4 sAcc[NG][NQ];
  pdl_launch_dependents();  // the next kernel's prologue may overlap this one; it reads nothing written here before
                            // its own griddepcontrol.wait
  pdl_wait();  // the partial outputs of the attention kernel
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int r = row % p.R;
  const int bh = row / p.R;
  const int b = bh / p.HKV;
  const int hkv = bh - b * p.HKV;
  const int sg = tid / NQ;
  const int c = tid - sg * NQ;
  const int64_t row0 = static_cast<int64_t>(bh) * p.max_splits * p.R + r;  // split s at row0 + s * R
  const float4* src = reinterpret_cast<const float4*>(p.o_part + row0 * D) + c;
  const int seq_len = ld_issue_s32(p.seq_lens + b);
  const float l_any = tid < p.max_splits ? ld_issue_f32(p.lse_part + row0 + static_cast<int64_t>(tid) * p.R) : 0.f;
  float4 v[kMergeSpec];
#pragma unroll
  for (int k = 0; k < kMergeSpec; ++k) {
    const int s = sg + k * NG;
    v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s < p.max_splits) v[k] = ld_issue_f32x4(src + static_cast<int64_t>(s) * p.R * NQ);
  }
  int chunk, n_split;
  sa_split(seq_len, p.max_splits, chunk, n_split);
  if (n_split == 1) return;
  const float l = tid < n_split ? l_any : -INFINITY;
  float m = l;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((tid & 31) == 0) sRed[tid >> 5] = m;
  __syncthreads();
  m = sRed[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, sRed[w]);
  const float mu = m == -INFINITY ? 0.f : m;
  const float w = tid < n_split ? ex2_approx(l - mu) : 0.f;
  if (tid < n_split) sW[tid] = w;
  float den = w;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
  __syncthreads();  // every thread has read sRed's maxima
  if ((tid & 31) == 0) sRed[tid >> 5] = den;
  __syncthreads();
  den = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) den += sRed[i];
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int k = 0; k < kMergeSpec; ++k) {
    const int s = sg + k * NG;
    if (s < n_split) {  // slots past the count may hold anything, NaN included: never touched
      const float ws = sW[s];
      acc.x = fmaf(ws, v[k].x, acc.x);
      acc.y = fmaf(ws, v[k].y, acc.y);
      acc.z = fmaf(ws, v[k].z, acc.z);
      acc.w = fmaf(ws, v[k].w, acc.w);
    }
  }
#pragma unroll 4
  for (int s = sg + kMergeSpec * NG; s < n_split; s += NG) {
    const float ws = sW[s];
    const float4 u = src[static_cast<int64_t>(s) * p.R * NQ];
    acc.x = fmaf(ws, u.x, acc.x);
    acc.y = fmaf(ws, u.y, acc.y);
    acc.z = fmaf(ws, u.z, acc.z);
    acc.w = fmaf(ws, u.w, acc.w);
  }
  sAcc[sg][c] = acc;
  __syncthreads();
  if (tid < NQ) {
    float4 t = sAcc[0][tid];
#pragma unroll
    for (int g2 = 1; g2 < NG; ++g2) {
      const float4 u = sAcc[g2][tid];
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    const int qi = r / p.G;
    __nv_bfloat16* dst = p.out + static_cast<int64_t>(b * p.Q + qi) * p.so_t +
                         static_cast<int64_t>(hkv * p.G + r - qi * p.G) * p.so_h + 4 * tid;
    uint2 o;
    o.x = pack_bf16x2(t.x * inv, t.y * inv);
    o.y = pack_bf16x2(t.z * inv, t.w * inv);
    *reinterpret_cast<uint2*>(dst) = o;
  }
}

// =============================================================================================== tcgen05 path
// Head sizes 128 and 256: the score and value products run on the 5th-generation tensor cores, one 64-token tile of
// the chunk at a time, accumulators in tensor memory.
//   S [64 rows x 64 tokens] = Q [rows x D] . K^T      (M = 64: the R = Q * G packed rows, zero-padded; N = 64 tokens;
//                                                       K-major A from the query tile, K-major B from the K tile)
//   O [64 rows x D] += P [rows x 64 tokens] . V        (M = 64, N = D; P^T-free: P is the K-major A operand, V is
//                                                       read in place as an MN-major B operand)
// An M = 64 accumulator puts row r in tensor-memory lane r % 16 + 32 (r / 16): lanes 0-15 of each of the four softmax
// warps own a row each, so a row's maximum, exponentials and sum are thread-local (no shuffles, no exchange between
// warps).  The padding rows cost tensor-core time only, which the kernel has to spare (the MMAs are a few percent of
// it).  Roles (7 warps): warp 0 streams K and V with TMA into a ring of 8 KiB pieces (K: one 64-column block of the
// tile's 64 tokens; V: 16 (D = 256) or 32 (D = 128) tokens of every column) -- lane q arms piece q of the tile, then
// every lane issues one 16-token box, since one issuing thread caps the copy rate well below HBM bandwidth; it starts
// as soon as the barriers exist, while warps 1-6 load the query tile; warp 1 allocates tensor memory and its lane 0
// issues the score MMAs, warp 6 lane 0 the value MMAs (two S buffers: the scores of tile i + 1 run while the softmax
// of tile i does), each releasing pieces with tcgen05.commit; warps 2-5 are the softmax: base-2 scores of the
// thread's row from tcgen05.ld, a reference maximum raised only when the row's maximum grows by more than 2^8 (then
// the row's O and sum are rescaled in place), P rounded to bf16 and stored as the row of the A operand, and at the end
// O / l written as outputs or split partials like the mma.sync kernel.
template <int D, int RP> struct SaTcGeo {
  static constexpr int kThreads = 224;
  static constexpr int kTile = 64;                   // tokens per tile
  static constexpr int kRows = 64;                   // M of both products
  // Only RP (32 or 64) rows of the query tile and of P are stored: with RP = 32 the M = 64 operands read their rows
  // 32-63 from the memory that follows (the next 64-column block, the other P buffer, or the pad below), which only
  // feeds accumulator rows that are never output.
  static constexpr int kPiece = 8192;
  static constexpr int kKPieces = D / 64;            // K: [64 tokens][64 columns] per piece
  static constexpr int kVTok = kPiece / (2 * D);     // V: tokens per piece, all D columns
  static constexpr int kVPieces = kTile / kVTok;
  static constexpr int kPiecesPerTile = kKPieces + kVPieces;
  static constexpr int kVLbo = kVTok * 128;          // V piece: 64-column blocks of kVTok 128-byte rows
  static constexpr int kQBytes = (D / 64) * RP * 128;
  static constexpr int kPBytes = RP * 128;           // P: [RP rows][64 tokens x 2 B]
  static constexpr int kPad = (kRows - RP) * 128;    // readable bytes after the last operand block
  static constexpr int kMiscBytes = 4 * kSaBtCache + 1024;
  static constexpr int kRingFit = (227 * 1024 - kQBytes - 2 * kPBytes - kPad - kMiscBytes - 1024) / kPiece;
  static constexpr int kRing = kRingFit > 32 ? 32 : kRingFit;
  static constexpr int kOffQ = kRing * kPiece;
  static constexpr int kOffP = kOffQ + kQBytes;
  static constexpr int kOffBt = kOffP + 2 * kPBytes + kPad;
  static constexpr int kOffBar = kOffBt + 4 * kSaBtCache;
  // barriers: full[kRing], empty[kRing], s_full[2], s_free[2], p_full[2], pv_done[2], drain, q_ready
  static constexpr int kNumBars = 2 * kRing + 10;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;             // tensor-memory address, abort flag
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;
  static constexpr uint32_t kColS = 0;                               // S buffers b at b * 64
  static constexpr uint32_t kColO = 2 * kTile;                       // O: D columns
  static constexpr uint32_t kTmemCols = 2 * kTile + D <= 256 ? 256 : 512;
  static_assert(kRing >= 2 * kPiecesPerTile, "ring shallower than two tiles");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
  static_assert(D == 128 || D == 256, "tcgen05 path head sizes");
  static_assert(RP == 32 || RP == 64, "stored rows");
};

template <int D, int RP>
__global__ void __launch_bounds__(224, 1)
    spec_attn_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                        const SaParams p) {
  using C = SaTcGeo<D, RP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kRing;
  uint64_t* s_full = bars + 2 * C::kRing;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_full + 4;
  uint64_t* pv_done = s_full + 6;
  uint64_t* drain = s_full + 8;
  uint64_t* q_ready = s_full + 9;  // the query tile is in shared memory (one arrival per loading warp)
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);
  int* sBt = reinterpret_cast<int*>(smem + C::kOffBt);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int b = blockIdx.y / p.HKV;
  const int hkv = blockIdx.y - b * p.HKV;

  pdl_launch_dependents();  // the merge kernel may be scheduled now; it waits for this grid before reading
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kRing; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 2);  // one commit from each MMA lane
    mbar_init(q_ready, C::kThreads / 32 - 1);
    *sAbort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
  }
  if (warp == 1) tmem_alloc(sTmem, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // queries, cache, block table and lengths are written by earlier kernels
  const int seq_len = __ldg(p.seq_lens + b);
  int chunk, n_split;
  sa_split(seq_len, p.max_splits, chunk, n_split);
  const uint32_t tmem = *sTmem;
  if (split < n_split) {
    const int start = split * chunk;
    const int end = min(start + chunk, max(seq_len, 0));
    const int n_tiles = end > start ? (end - start + C::kTile - 1) / C::kTile : 0;
    const int* bt = p.block_table + static_cast<int64_t>(b) * p.s_bt;
    const int pg0 = start / p.page;
    uint8_t* sQ = smem + C::kOffQ;
    const int hq0 = hkv * p.G;
    if (warp == 0) {
      // the chunk's pages for the producer only (no CTA barrier: the copies start while the others load the queries)
      if (n_tiles > 0) {
        const int npg = (end - 1) / p.page - pg0 + 1;
        for (int i = lane; i < npg && i < kSaBtCache; i += 32) sBt[i] = __ldg(bt + pg0 + i);
      }
      __syncwarp();
    } else {
      // the packed query rows (r = qi * G + gg) as the K-major A operand: per 64-column block, RP rows x 128 B
      // swizzled; the score lanes wait for q_ready
      for (int idx = threadIdx.x - 32; idx < RP * (D / 8); idx += C::kThreads - 32) {
        const int r = idx / (D / 8);
        const int c = idx - r * (D / 8);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < p.R) {
          const int qi = r / p.G;
          v = *reinterpret_cast<const uint4*>(p.q + static_cast<int64_t>(b * p.Q + qi) * p.sq_t +
                                              static_cast<int64_t>(hq0 + r - qi * p.G) * p.sq_h + c * 8);
        }
        *reinterpret_cast<uint4*>(sQ + sw_off(r, c, RP * 128)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the query tile is read by the tensor cores
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }

    if (warp == 0) {
      // ---------------------------------------------------------------------------------------- TMA producer
      constexpr int kKBoxes = C::kKPieces * (C::kTile / 16);             // K: 16-token boxes per 64-column block
      constexpr int kVBoxes = C::kVPieces * (C::kVTok / 16) * (D / 64);  // V: per 16-token box, every column block
      static_assert(kKBoxes + kVBoxes <= 32, "one box per lane");
      const uint64_t pol = policy_evict_first();
      bool ok = true;
      int issued = 0;  // tiles whose copies are all issued
      for (int i = 0; i < n_tiles && ok; ++i) {
        const int base = start + C::kTile * i;
        const int pc0 = i * C::kPiecesPerTile;
        if (lane < C::kPiecesPerTile) {  // lane q2 arms piece q2 of the tile: its slot, then its byte count
          const int q2 = lane;
          const int pc = pc0 + q2;
          const int slot = pc % C::kRing;
          if (pc >= C::kRing && !sa_wait(&empty[slot], ((pc / C::kRing) - 1) & 1, sAbort)) {
            sa_abort(p, sAbort);
            ok = false;
          } else {
            int nb;  // bytes of the piece below `end`
            if (q2 < C::kKPieces) {
              nb = min(C::kTile / 16, (end - base + 15) / 16) * 2048;
            } else {
              const int t0 = base + (q2 - C::kKPieces) * C::kVTok;
              nb = (t0 < end ? min(C::kVTok / 16, (end - t0 + 15) / 16) : 0) * (D / 64) * 2048;
            }
            mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nb));
          }
        }
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        if (lane < kKBoxes + kVBoxes) {  // lane l issues one box of the tile
          int q2, pos, col, off_b;
          if (lane < kKBoxes) {  // K: piece = column block, box = 16 tokens of the tile
            q2 = lane / (C::kTile / 16);
            const int g = lane - q2 * (C::kTile / 16);
            pos = base + 16 * g;
            col = 64 * q2;
            off_b = g * 2048;
          } else {               // V: piece = kVTok tokens, box = (16 tokens, column block)
            const int l2 = lane - kKBoxes;
            const int per = (C::kVTok / 16) * (D / 64);
            const int v = l2 / per;
            const int g = (l2 - v * per) / (D / 64);
            const int j = l2 - v * per - g * (D / 64);
            q2 = C::kKPieces + v;
            pos = base + v * C::kVTok + 16 * g;
            col = 64 * j;
            off_b = j * C::kVLbo + g * 2048;
          }
          if (pos < end) {
            const int slot = (pc0 + q2) % C::kRing;
            const int pg = pos / p.page;
            const int blk = pg - pg0 < kSaBtCache ? sBt[pg - pg0] : __ldg(bt + pg);
            const int off = pos - pg * p.page;
            tma_load_4d(smem + slot * C::kPiece + off_b, lane < kKBoxes ? &tk : &tv, &full[slot], col,
                        p.head_inner ? hkv : off, p.head_inner ? off : hkv, blk, pol);
          }
        }
        issued = i + 1;
      }
      if (*sAbort && lane == 0) {  // let the issued copies of the last pieces land (one bounded wait in all)
        const int pcn = issued * C::kPiecesPerTile;
        const uint64_t t0 = global_timer_ns();
        for (int q2 = pcn > C::kRing ? pcn - C::kRing : 0; q2 < pcn; ++q2) {
          while (!mbar_try_wait(&full[q2 % C::kRing], (q2 / C::kRing) & 1) && global_timer_ns() - t0 < kSaWaitNs) {
          }
        }
      }
    } else if (warp == 1 || warp == 6) {
      // ---------------------------------------------------------------------------------------- MMA issuers
      // warp 1 lane 0 issues the score products, warp 6 lane 0 the value products: neither waits for the other's
      // inputs (scores need K pieces and a free S buffer, values need P and V pieces)
      if (lane == 0) {
        constexpr uint32_t idesc_s = idesc_bf16(C::kRows, C::kTile, false, false);
        constexpr uint32_t idesc_o = idesc_bf16(C::kRows, D, false, true);
        const uint32_t sm_base = smem_u32(smem);
        const uint32_t q_base = smem_u32(sQ);
        const uint32_t p_base = smem_u32(smem + C::kOffP);
        bool ok = true;
        // pieces are numbered in the producer's order (tile i: its K pieces, then its V pieces); the scores of tile
        // i + 1 consume K pieces before the V pieces of tile i
        auto wait_piece = [&](int pc, int& slot) -> bool {
          slot = pc % C::kRing;
          if (!sa_wait(&full[slot], (pc / C::kRing) & 1, sAbort)) {
            sa_abort(p, sAbort);
            return false;
          }
          tc_fence_after();
          return true;
        };
        if (warp == 1 && !sa_wait(q_ready, 0, sAbort)) {
          sa_abort(p, sAbort);
          ok = false;
        }
        auto issue_s = [&](int i) -> bool {
          const int sb = i & 1;
          if (i >= 2 && !sa_wait(&s_free[sb], ((i >> 1) - 1) & 1, sAbort)) {
            sa_abort(p, sAbort);
            return false;
          }
          tc_fence_after();
          for (int j = 0; j < C::kKPieces; ++j) {
            int slot;
            if (!wait_piece(i * C::kPiecesPerTile + j, slot)) return false;
            const uint32_t a0 = q_base + j * RP * 128;
            const uint32_t b0 = sm_base + slot * C::kPiece;
#pragma unroll
            for (int s2 = 0; s2 < 4; ++s2)
              mma_bf16_ss(tmem + C::kColS + sb * C::kTile, smem_desc_k128_sw128(a0 + 32 * s2),
                          smem_desc_k128_sw128(b0 + 32 * s2), idesc_s, (j | s2) != 0);
            mma_commit(&empty[slot]);
          }
          mma_commit(&s_full[sb]);
          return true;
        };
        auto issue_pv = [&](int i) -> bool {
          const int sb = i & 1;
          if (!sa_wait(&p_full[sb], (i >> 1) & 1, sAbort)) {
            sa_abort(p, sAbort);
            return false;
          }
          tc_fence_after();
          const int base = start + C::kTile * i;
          for (int v = 0; v < C::kVPieces; ++v) {
            int slot;
            if (!wait_piece(i * C::kPiecesPerTile + C::kKPieces + v, slot)) return false;
            const uint32_t b0 = sm_base + slot * C::kPiece;
#pragma unroll
            for (int s2 = 0; s2 < C::kVTok / 16; ++s2) {
              const int tk0 = v * C::kVTok + 16 * s2;  // token of the k-step within the tile
              if (base + tk0 >= end) continue;       // past the chunk: no keys, no copies
              mma_bf16_ss(tmem + C::kColO, smem_desc_k128_sw128(p_base + sb * C::kPBytes + (tk0 >> 4) * 32),
                          smem_desc_mn_sw128(b0 + s2 * 2048, C::kVLbo, 1024), idesc_o, (i | tk0) != 0);
            }
            mma_commit(&empty[slot]);
          }
          mma_commit(&pv_done[sb]);
          return true;
        };
        if (warp == 1) {
          for (int i = 0; i < n_tiles && ok; ++i) ok = issue_s(i);
        } else {
          for (int i = 0; i < n_tiles && ok; ++i) ok = issue_pv(i);
        }
        // every issued MMA of both lanes has completed before the roles finish (and tensor memory is freed)
        mma_commit(drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(drain, 0) && global_timer_ns() - t0 < kSaWaitNs) {
        }
      }
    } else {
      // ---------------------------------------------------------------------------------------- softmax warps
      // lanes 0-15 of warp w own packed row r = 16 (w % 4) + lane (tensor-memory lane 32 (w % 4) + lane)
      const int q4 = warp & 3;
      const bool row_lane = lane < 16;
      const int r = 16 * q4 + (lane & 15);
      const uint32_t lane_off = static_cast<uint32_t>(32 * q4) << 16;
      uint8_t* prow = smem + C::kOffP + r * 128;  // this row of P (slot 0)
      const bool live = row_lane && r < p.R;
      const int lim = seq_len - p.Q + (live ? r / p.G : 0);  // the row sees keys <= lim
      float m_run = -INFINITY;  // reference maximum (base 2)
      float l_run = 0.f;        // sum of 2^(s - m_run)
      bool ok = true;
      // every wait's outcome is made warp-uniform: tcgen05.ld / st are warp-collective
      auto wait_or_abort = [&](uint64_t* bar, uint32_t parity) -> bool {
        bool got = sa_wait(bar, parity, sAbort);
        if (!got) sa_abort(p, sAbort);
        return __all_sync(0xffffffffu, got);
      };
      for (int i = 0; i < n_tiles && ok; ++i) {
        const int sb = i & 1;
        const int base = start + C::kTile * i;
        if (!(ok = wait_or_abort(&s_full[sb], (i >> 1) & 1))) break;
        tc_fence_after();
        float x[C::kTile];
#pragma unroll
        for (int g2 = 0; g2 < C::kTile / 32; ++g2) {
          uint32_t r32[32];
          tmem_ld_32x32b_x32(tmem + lane_off + C::kColS + sb * C::kTile + 32 * g2, r32);
#pragma unroll
          for (int j = 0; j < 32; ++j) x[32 * g2 + j] = __uint_as_float(r32[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        // base-2 scaled scores; keys past the chunk's end or the row's causal limit are -inf
        const int kmax = min(end, lim + 1) - base;  // tokens [0, kmax) of the tile are keys of this row
#pragma unroll
        for (int t = 0; t < C::kTile; ++t) x[t] = (live && t < kmax) ? x[t] * p.qk_scale : -INFINITY;
        float mx[16];  // the row maximum as a tree (independent chains)
#pragma unroll
        for (int j = 0; j < 16; ++j) mx[j] = fmaxf(fmaxf(x[j], x[j + 16]), fmaxf(x[j + 32], x[j + 48]));
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
          for (int j = 0; j < w; ++j) mx[j] = fmaxf(mx[j], mx[j + w]);
        const float tmax = mx[0];
        // raise the reference only when the row's maximum grows by more than 2^8 (or first appears): P stays below 2^8
        const bool want = tmax > m_run + 8.f || (m_run == -INFINITY && tmax > -INFINITY);
        float al = 1.f;
        if (want) {
          const float mn = fmaxf(m_run, tmax);
          al = m_run == -INFINITY ? 0.f : ex2_approx(m_run - mn);
          l_run *= al;
          m_run = mn;
        }
        if (i > 0 && __any_sync(0xffffffffu, want)) {
          // O holds P V of the earlier tiles: scale the raised rows (factor 1 for the others) once the last P V landed
          if (!(ok = wait_or_abort(&pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1))) break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r32[32];
            const uint32_t ta = tmem + lane_off + C::kColO + 32 * c;
            tmem_ld_32x32b_x32(ta, r32);
#pragma unroll
            for (int j = 0; j < 32; ++j) r32[j] = __float_as_uint(__uint_as_float(r32[j]) * al);
            tmem_st_32x32b_x32(ta, r32);
          }
          tc_fence_before();
        }
        // P = 2^(x - m) in bf16 as this row of the A operand in slot sb (free once P V of tile i - 2 has completed)
        if (i >= 2 && !(ok = wait_or_abort(&pv_done[sb], ((i >> 1) - 1) & 1))) break;
        const float mu = m_run == -INFINITY ? 0.f : m_run;
        float ls[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) ls[j] = 0.f;
        uint32_t pk[C::kTile / 2];
#pragma unroll
        for (int t = 0; t < C::kTile; t += 2) {
          const float p0 = ex2_approx(x[t] - mu);
          const float p1 = ex2_approx(x[t + 1] - mu);
          ls[(t >> 1) & 7] += p0 + p1;
          pk[t / 2] = pack_bf16x2(p0, p1);
        }
        l_run += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
        if (row_lane && r < RP) {
          uint8_t* dst = prow + sb * C::kPBytes;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(dst + ((c ^ (r & 7)) << 4)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
        // slots past the chunk's end inside a 16-token step that still has keys were copied from their page (maybe
        // never written): zero their V rows so that P = 0 cannot meet a NaN
        const int kend = end - base;  // tokens [kend, 16 * ceil(kend / 16)) of the tile
        if (kend < C::kTile && (kend & 15)) {
          const int st0 = kend & ~15;
          const int vv = st0 / C::kVTok;
          const int pcv = i * C::kPiecesPerTile + C::kKPieces + vv;
          if (!(ok = wait_or_abort(&full[pcv % C::kRing], (pcv / C::kRing) & 1))) break;
          const int nz = (16 - (kend & 15)) * (D / 64) * 8;  // 16-byte words to clear
          for (int idx = 32 * (warp - 2) + lane; idx < nz; idx += 128) {
            const int w16 = idx & 7;
            const int rest = idx >> 3;
            const int j = rest % (D / 64);
            const int t = kend + rest / (D / 64);
            *reinterpret_cast<uint4*>(smem + (pcv % C::kRing) * C::kPiece + j * C::kVLbo + (t - vv * C::kVTok) * 128 +
                                      16 * w16) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P (and zeroed V) for the tensor cores
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
      }
      if (ok && n_tiles > 0 && wait_or_abort(&pv_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1)) {
        // O / l for this row (D columns of its tensor-memory lane)
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        const bool single = n_split == 1;
        const int64_t part_row0 = (static_cast<int64_t>(b * p.HKV + hkv) * p.max_splits + split) * p.R;
        const int qi = live ? r / p.G : 0;
        __nv_bfloat16* orow =
            p.out + static_cast<int64_t>(b * p.Q + qi) * p.so_t + static_cast<int64_t>(hq0 + r - qi * p.G) * p.so_h;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r32[32];
          tmem_ld_32x32b_x32(tmem + lane_off + C::kColO + 32 * c, r32);
          if (live) {
            if (single) {
#pragma unroll
              for (int j = 0; j < 32; j += 8)
                *reinterpret_cast<uint4*>(orow + 32 * c + j) =
                    make_uint4(pack_bf16x2(__uint_as_float(r32[j]) * inv, __uint_as_float(r32[j + 1]) * inv),
                               pack_bf16x2(__uint_as_float(r32[j + 2]) * inv, __uint_as_float(r32[j + 3]) * inv),
                               pack_bf16x2(__uint_as_float(r32[j + 4]) * inv, __uint_as_float(r32[j + 5]) * inv),
                               pack_bf16x2(__uint_as_float(r32[j + 6]) * inv, __uint_as_float(r32[j + 7]) * inv));
            } else {
              float* prt = p.o_part + (part_row0 + r) * D + 32 * c;
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(prt + j) =
                    make_float4(__uint_as_float(r32[j]) * inv, __uint_as_float(r32[j + 1]) * inv,
                                __uint_as_float(r32[j + 2]) * inv, __uint_as_float(r32[j + 3]) * inv);
            }
          }
        }
        if (live && !single) p.lse_part[part_row0 + r] = l_run > 0.f ? m_run + log2f(l_run) : -INFINITY;
      } else if (ok && n_tiles == 0 && n_split == 1 && live) {
        // no key at all (seq_len <= 0): zeros
        const int qi = r / p.G;
        __nv_bfloat16* orow =
            p.out + static_cast<int64_t>(b * p.Q + qi) * p.so_t + static_cast<int64_t>(hq0 + r - qi * p.G) * p.so_h;
        for (int d = 0; d < D; d += 8) *reinterpret_cast<uint4*>(orow + d) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// ----------------------------------------------------------------------------------------------- host side
std::mutex g_sa_mu;
int g_sa_sms[64] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_sa_encode = nullptr;

int sa_device(int* dev, int* sms) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (*dev < 0 || *dev >= 64) return fail(QF_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(g_sa_mu);
  if (g_sa_sms[*dev] == 0) {
    int major = 0, minor = 0, n = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, *dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, *dev);
    g_sa_sms[*dev] = (major == 10 && minor == 0) ? n : -1;
  }
  if (g_sa_sms[*dev] < 0)
    return fail(QF_ERR_ARCH, "libqf_b200 is built for sm_100a (B200); this device is not compute capability 10.0");
  if (!g_sa_encode) {
    cudaDriverEntryPointQueryResult qres;
    void* fn = nullptr;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres);
    if (e != cudaSuccess || qres != cudaDriverEntryPointSuccess || !fn)
      return fail(QF_ERR_DRIVER, "cuTensorMapEncodeTiled entry point not found");
    g_sa_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  *sms = g_sa_sms[*dev];
  return QF_OK;
}

int sa_max_splits(int sms, int num_reqs, int hkv) {
  const long long units = static_cast<long long>(num_reqs) * hkv;
  long long s = units > 0 ? sms / units : 1;
  if (s < 1) s = 1;
  if (s > kSaMaxSplits) s = kSaMaxSplits;
  return static_cast<int>(s);
}

size_t sa_ws_bytes(int num_reqs, int hkv, int R, int D, int splits) {
  const size_t rows = static_cast<size_t>(num_reqs) * hkv * splits * R;
  return kSaHeader + (rows * D * 4 + 255) / 256 * 256 + rows * 4;
}

// Cache [page][slot][head][d] with element strides (s_b, s_t, s_h, 1) as a 4-D tensor map with 64 x 16-slot boxes;
// the slot and head dimensions are ordered by stride (smaller first).
int sa_encode(CUtensorMap* map, const void* base, int D, int page, int hkv, int num_blocks, int64_t s_b, int64_t s_t,
              int64_t s_h) {
  const bool head_inner = s_h < s_t;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(head_inner ? hkv : page),
                        static_cast<cuuint64_t>(head_inner ? page : hkv), static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>((head_inner ? s_h : s_t) * 2),
                           static_cast<cuuint64_t>((head_inner ? s_t : s_h) * 2), static_cast<cuuint64_t>(s_b * 2)};
  cuuint32_t box[4] = {64, head_inner ? 1u : static_cast<cuuint32_t>(kSaSlice),
                       head_inner ? static_cast<cuuint32_t>(kSaSlice) : 1u, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = g_sa_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(QF_ERR_DRIVER, "cuTensorMapEncodeTiled rejected the KV cache view (error " + std::to_string(r) + ")");
  return QF_OK;
}

// The merge launch shared by both attention kernels (skipped when every request has one split).
template <int D>
int sa_launch_merge(const SaParams& p, int num_reqs, cudaStream_t st) {
  if (p.max_splits == 1) return QF_OK;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t mc = {};
  mc.gridDim = dim3(static_cast<unsigned>(num_reqs * p.HKV * p.R));
  mc.blockDim = dim3(256);
  mc.stream = st;
  mc.attrs = attr;
  mc.numAttrs = 1;  // scheduled behind the attention grid; reads its outputs after griddepcontrol.wait
  const cudaError_t e = cudaLaunchKernelEx(&mc, spec_attn_merge_kernel<D>, p);
  return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, std::string("merge launch: ") + cudaGetErrorString(e));
}

template <int D, int MT>
int sa_launch(const CUtensorMap& tk, const CUtensorMap& tv, const SaParams& p, int num_reqs, int dev, unsigned flags,
              cudaStream_t st) {
  using C = SaGeo<D, MT>;
  static bool attr_set[64] = {};
  {
    std::lock_guard<std::mutex> lk(g_sa_mu);
    if (!attr_set[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(spec_attn_kernel<D, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 C::kSmemBytes);
      if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      attr_set[dev] = true;
    }
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.max_splits), static_cast<unsigned>(num_reqs * p.HKV));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & QF_FLAG_PDL) ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, spec_attn_kernel<D, MT>, tk, tv, p);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("attention launch: ") + cudaGetErrorString(e));
  return sa_launch_merge<D>(p, num_reqs, st);
}

template <int D, int RP>
int sa_launch_tc(const CUtensorMap& tk, const CUtensorMap& tv, const SaParams& p, int num_reqs, int dev,
                 unsigned flags, cudaStream_t st) {
  using C = SaTcGeo<D, RP>;
  static bool attr_set[64] = {};
  {
    std::lock_guard<std::mutex> lk(g_sa_mu);
    if (!attr_set[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(spec_attn_tc_kernel<D, RP>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
      if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      attr_set[dev] = true;
    }
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.max_splits), static_cast<unsigned>(num_reqs * p.HKV));
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & QF_FLAG_PDL) ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, spec_attn_tc_kernel<D, RP>, tk, tv, p);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("attention launch: ") + cudaGetErrorString(e));
  return sa_launch_merge<D>(p, num_reqs, st);
}

// QF_ATTN_MMA_SYNC=1 (read only with QF_TEST_OVERRIDES=1) keeps head sizes 128 / 256 on the mma.sync kernel, so
// that tests can run both kernels on the same shapes.
bool force_mma_sync() {
  static const bool on = [] {
    const char* t = std::getenv("QF_TEST_OVERRIDES");
    const char* v = std::getenv("QF_ATTN_MMA_SYNC");
    return t && std::strcmp(t, "1") == 0 && v && std::strcmp(v, "1") == 0;
  }();
  return on;
}

template <int D>
int sa_dispatch_mt(int MT, const CUtensorMap& tk, const CUtensorMap& tv, const SaParams& p, int num_reqs, int dev,
                   unsigned flags, cudaStream_t st) {
  switch (MT) {
    case 1: return sa_launch<D, 1>(tk, tv, p, num_reqs, dev, flags, st);
    case 2: return sa_launch<D, 2>(tk, tv, p, num_reqs, dev, flags, st);
    case 3: return sa_launch<D, 3>(tk, tv, p, num_reqs, dev, flags, st);
    default: return sa_launch<D, 4>(tk, tv, p, num_reqs, dev, flags, st);
  }
}

bool aligned16(const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; }

}  // namespace
}  // namespace qf

using namespace qf;

extern "C" {

size_t qf_spec_attn_workspace_bytes(int num_reqs, int q_len, int num_heads, int num_kv_heads, int head_size) {
  if (num_reqs <= 0 || q_len <= 0 || num_kv_heads <= 0 || num_heads <= 0 || head_size <= 0) return kSaHeader;
  int dev = 0, sms = 0;
  if (sa_device(&dev, &sms) != QF_OK) sms = kSaMaxSplits;  // no usable device: the largest split count
  const int R = q_len * (num_heads / num_kv_heads);
  return sa_ws_bytes(num_reqs, num_kv_heads, R, head_size, sa_max_splits(sms, num_reqs, num_kv_heads));
}

int qf_spec_attn(const void* q, int64_t sq_t, int64_t sq_h, const void* k_cache, int64_t sk_b, int64_t sk_t,
                 int64_t sk_h, const void* v_cache, int64_t sv_b, int64_t sv_t, int64_t sv_h, int num_blocks,
                 int page_size, const int32_t* block_table, int64_t s_bt, const int32_t* seq_lens, void* out,
                 int64_t so_t, int64_t so_h, int num_reqs, int q_len, int num_heads, int num_kv_heads, int head_size,
                 float scale, void* ws, size_t ws_bytes, unsigned flags, void* stream) {
  if (num_reqs < 0 || q_len < 1 || num_heads < 1 || num_kv_heads < 1 || num_blocks < 1)
    return fail(QF_ERR_SHAPE, "num_reqs >= 0, q_len, num_heads, num_kv_heads and num_blocks >= 1 required");
  if (num_reqs == 0) return QF_OK;
  if (num_heads % num_kv_heads) return fail(QF_ERR_SHAPE, "num_heads must be a multiple of num_kv_heads");
  if (head_size != 64 && head_size != 128 && head_size != 256)
    return fail(QF_ERR_SHAPE, "head_size must be 64, 128 or 256");
  const int G = num_heads / num_kv_heads;
  const long long R = static_cast<long long>(q_len) * G;
  if (R > 64) return fail(QF_ERR_SHAPE, "q_len * num_heads / num_kv_heads must be <= 64");
  if (page_size < 16 || page_size % 16) return fail(QF_ERR_SHAPE, "page_size must be a positive multiple of 16");
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(QF_ERR_INVALID, "scale must be finite and > 0");
  if (!q || !k_cache || !v_cache || !block_table || !seq_lens || !out || !ws) return fail(QF_ERR_INVALID, "null pointer");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return fail(QF_ERR_ALIGN, "q, k_cache, v_cache and out must be 16-byte aligned");
  const int64_t st8[10] = {sq_t, sq_h, sk_b, sk_t, sk_h, sv_b, sv_t, sv_h, so_t, so_h};
  for (int i = 0; i < 10; ++i)
    if (st8[i] <= 0 || st8[i] % 8) return fail(QF_ERR_STRIDE, "strides must be positive multiples of 8 elements");
  if ((sk_h < sk_t) != (sv_h < sv_t)) return fail(QF_ERR_STRIDE, "k_cache and v_cache must share one slot/head order");
  if (s_bt < 1) return fail(QF_ERR_STRIDE, "block_table row stride must be >= 1");
  if (reinterpret_cast<uintptr_t>(ws) % 256) return fail(QF_ERR_ALIGN, "workspace must be 256-byte aligned");
  int dev = 0, sms = 0;
  int rc = sa_device(&dev, &sms);
  if (rc) return rc;
  const int splits = sa_max_splits(sms, num_reqs, num_kv_heads);
  if (ws_bytes < sa_ws_bytes(num_reqs, num_kv_heads, static_cast<int>(R), head_size, splits))
    return fail(QF_ERR_WORKSPACE, "workspace too small (qf_spec_attn_workspace_bytes)");
  if (static_cast<long long>(num_reqs) * num_kv_heads > 65535) return fail(QF_ERR_SHAPE, "num_reqs * num_kv_heads > 65535");
  CUtensorMap tk, tv;
  rc = sa_encode(&tk, k_cache, head_size, page_size, num_kv_heads, num_blocks, sk_b, sk_t, sk_h);
  if (rc) return rc;
  rc = sa_encode(&tv, v_cache, head_size, page_size, num_kv_heads, num_blocks, sv_b, sv_t, sv_h);
  if (rc) return rc;
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  const size_t rows = static_cast<size_t>(num_reqs) * num_kv_heads * splits * R;
  SaParams p = {};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.sq_t = sq_t;
  p.sq_h = sq_h;
  p.block_table = block_table;
  p.s_bt = s_bt;
  p.seq_lens = seq_lens;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.so_t = so_t;
  p.so_h = so_h;
  p.o_part = reinterpret_cast<float*>(wsb + kSaHeader);
  p.lse_part = reinterpret_cast<float*>(wsb + kSaHeader + (rows * head_size * 4 + 255) / 256 * 256);
  p.err = reinterpret_cast<int*>(wsb);
  p.Q = q_len;
  p.G = G;
  p.R = static_cast<int>(R);
  p.HKV = num_kv_heads;
  p.page = page_size;
  p.max_splits = splits;
  p.head_inner = sk_h < sk_t ? 1 : 0;
  p.qk_scale = scale * 1.4426950408889634f;
  const int MT = static_cast<int>((R + 15) / 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_size >= 128 && !force_mma_sync()) {  // tensor-core (tcgen05) kernel
    if (head_size == 256)
      return R <= 32 ? sa_launch_tc<256, 32>(tk, tv, p, num_reqs, dev, flags, st)
                     : sa_launch_tc<256, 64>(tk, tv, p, num_reqs, dev, flags, st);
    return R <= 32 ? sa_launch_tc<128, 32>(tk, tv, p, num_reqs, dev, flags, st)
                   : sa_launch_tc<128, 64>(tk, tv, p, num_reqs, dev, flags, st);
  }
  if (head_size == 256) return sa_dispatch_mt<256>(MT, tk, tv, p, num_reqs, dev, flags, st);
  if (head_size == 128) return sa_dispatch_mt<128>(MT, tk, tv, p, num_reqs, dev, flags, st);
  return sa_dispatch_mt<64>(MT, tk, tv, p, num_reqs, dev, flags, st);
}

}  // extern "C"
