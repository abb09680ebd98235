// qf_w8a8.cu -- sm_100a int8 x int8 GEMM for the rows the small-M path does not take (prefill, M > 16).
//
// Replaces the W8A8 fallback of EurekaZang/qwen-a100-fastpath's qf_int8_linear (plugin/qwen_fastpath/patches.py:99-100):
//   x_q, x_s = ops.scaled_int8_quant(x, symmetric=True)          (dynamic per-token int8 activations)
//   y = ops.cutlass_scaled_mm(x_q, w_q, scale_a=x_s, scale_b=w_s, out_dtype=bf16, bias=bias)
// Both live in vLLM's compiled extension (pinned vllm==0.31.0 by the reference's requirements.lock; not part of the
// reference source).  Their published arithmetic, restated here:
//   quantization, per token row m:  a = max_k |x[m,k]|;  s_x[m] = a / 127;  q[m,k] = rni_sat_s8(x[m,k] * (127 / a))
//     (fp32, round half to even, saturated to [-128, 127]; a zero row gives q = 0, s_x = 0);
//   GEMM epilogue (CUTLASS "scaled" epilogue):  y[m,n] = bf16( s_x[m] * (s_w[n] * float(acc[m,n])) [+ bias[n]] ),
//     acc = exact int32 sum_k q[m,k] * w[n,k]; with a bias the last step is one fused multiply-add.
//
// Design (B200):
// * qf_quantize_tokens_kernel: one CTA per token row, 16-byte loads, the row's absmax by warp shuffles, int8 rows
//   written to the caller's workspace with the row stride padded to 16 bytes (TMA rule).
// * w8a8_kernel<BN>: persistent, one CTA per SM over 128 x BN output tiles (token rows x channels).  Warp 0 (one
//   lane) streams the tiles' k-slices with TMA (128-byte rows, 128-byte swizzle, no multicast) into a ring of
//   stages guarded by mbarriers; warp 1 allocates 2 x BN tensor-memory columns (two accumulators) and one of its
//   lanes issues tcgen05.mma kind::i8 (M = 128, N = BN, K = 32 per instruction, four per 128-byte stage), releasing
//   each stage with tcgen05.commit; warps 2-5 read a finished accumulator with tcgen05.ld (warp w reads lanes
//   32 (w % 4) .. +31, i.e. token rows), apply the scales (and bias), round to bf16 and store, while the MMAs of the
//   next tile fill the other accumulator.  Tiles are taken channel-block-major so consecutive CTAs share a weight
//   block through L2.
// * Every mbarrier wait is bounded (4 s): on expiry the CTA records QF_ERR_TIMEOUT in the workspace header, the
//   roles stop, the MMA lane waits (bounded) for its issued MMAs, the producer drains its copies, and the tensor
//   memory is freed before the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <string>

#include "../../include/qf_b200.h"
#include "qf_host.h"
#include "qf_ptx.cuh"

namespace qf {
namespace {

constexpr int kPfThreads = 192;          // warp 0 TMA, warp 1 MMA + tensor memory, warps 2-5 epilogue
constexpr int kPfBM = 128;               // token rows per tile (tcgen05 M)
constexpr int kPfBK = 128;               // k bytes per stage: one 128-byte swizzle row
constexpr int kPfMaxGrid = 256;
constexpr uint64_t kPfWaitNs = 4000000000ull;
constexpr size_t kPfHeader = 256;        // workspace: [0] error word

template <int BN> struct PfGeo {
  static constexpr int kABytes = kPfBM * kPfBK;
  static constexpr int kBBytes = BN * kPfBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagesFit = (200 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kOffBar = kStages * kStageBytes;
  // full[S], empty[S], acc_full[2], acc_empty[2], mma_done
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;   // tmem address, abort flag
  static constexpr int kOffScale = kOffMisc + 16;           // float s_w[BN], float bias[BN] of the current tile
  static constexpr int kSmemBytes = kOffScale + 2 * BN * 4 + 1024;
  static_assert(kStages >= 3, "ring too shallow");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
  static_assert(kTmemCols <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "tensor memory columns");
};

struct PfParams {
  const float* sx;        // per-token scales [M]
  const float* sw;        // per-channel scales [N]
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;
  int64_t ldy;
  int M, N, K;
  int mtiles, ntiles, kiters;
  int* err;
};

__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (*abort_flag) return false;
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kPfWaitNs) return false;
  }
}

__device__ __forceinline__ void pf_abort(const PfParams& p, volatile int* abort_flag) {
  if (!*abort_flag) atomicExch(p.err, QF_ERR_TIMEOUT);
  *abort_flag = 1;
}

// Per-token symmetric int8 quantization: q[m, k] = rni_sat_s8(x[m, k] * (127 / a)), s_x[m] = a / 127, a = max|x[m, :]|.
// Columns [K, ldq) of q are zeroed.  One CTA of 256 threads per row.
__global__ void __launch_bounds__(256) quantize_tokens_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                              int K, int8_t* __restrict__ q, int64_t ldq,
                                                              float* __restrict__ sx, int vec) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const __nv_bfloat16* row = x + static_cast<int64_t>(m) * ldx;
  int8_t* qrow = q + static_cast<int64_t>(m) * ldq;
  float a = 0.f;
  const int nvec = vec ? K / 8 : 0;
  for (int c = threadIdx.x; c < nvec; c += 256) {
    const uint4 u = reinterpret_cast<const uint4*>(row)[c];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a = fmaxf(a, fabsf(__uint_as_float(w[j] << 16)));
      a = fmaxf(a, fabsf(__uint_as_float(w[j] & 0xFFFF0000u)));
    }
  }
  for (int k = nvec * 8 + threadIdx.x; k < K; k += 256) a = fmaxf(a, fabsf(__bfloat162float(row[k])));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
  __shared__ float s_red[8];
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = a;
  __syncthreads();
  a = s_red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) a = fmaxf(a, s_red[i]);
  const float inv = __fdiv_rn(127.0f, a);  // +inf for a zero row: 0 * inf = NaN converts to 0
  if (threadIdx.x == 0) sx[m] = __fdiv_rn(a, 127.0f);
  for (int c = threadIdx.x; c < nvec; c += 256) {
    const uint4 u = reinterpret_cast<const uint4*>(row)[c];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int b0 = f32_to_s8_rni_sat(__fmul_rn(__uint_as_float(w[2 * j] << 16), inv));
      const int b1 = f32_to_s8_rni_sat(__fmul_rn(__uint_as_float(w[2 * j] & 0xFFFF0000u), inv));
      const int b2 = f32_to_s8_rni_sat(__fmul_rn(__uint_as_float(w[2 * j + 1] << 16), inv));
      const int b3 = f32_to_s8_rni_sat(__fmul_rn(__uint_as_float(w[2 * j + 1] & 0xFFFF0000u), inv));
      o[j] = (static_cast<uint32_t>(b0) & 0xFF) | ((static_cast<uint32_t>(b1) & 0xFF) << 8) |
             ((static_cast<uint32_t>(b2) & 0xFF) << 16) | ((static_cast<uint32_t>(b3) & 0xFF) << 24);
    }
    reinterpret_cast<uint2*>(qrow)[c] = make_uint2(o[0], o[1]);
  }
  for (int k = nvec * 8 + threadIdx.x; k < K; k += 256)
    qrow[k] = static_cast<int8_t>(f32_to_s8_rni_sat(__fmul_rn(__bfloat162float(row[k]), inv)));
  for (int k = K + threadIdx.x; k < ldq; k += 256) qrow[k] = 0;
}

template <int BN>
__global__ void __launch_bounds__(kPfThreads, 1)
    w8a8_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                const PfParams p) {
  using C = PfGeo<BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);
  float* s_sw = reinterpret_cast<float*>(smem + C::kOffScale);
  float* s_bias = s_sw + BN;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntotal = p.mtiles * p.ntiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_normal();
      const uint64_t pol_x = policy_evict_last();
      bool waited = false;  // activations come from the quantization kernel before this one
      int it = 0;
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntotal && ok; t += gridDim.x) {
        const int n0 = (t / p.mtiles) * BN;
        const int m0 = (t % p.mtiles) * kPfBM;
        for (int kb = 0; kb < p.kiters; ++kb, ++it) {
          const int s = it % S;
          if (!pf_wait(&empty[s], ((it / S) & 1) ^ 1, s_abort)) {
            pf_abort(p, s_abort);
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + s * C::kStageBytes;
          uint8_t* b_dst = a_dst + C::kABytes;
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          tma_load_2d(b_dst, &tmap_w, &full[s], kb * kPfBK, n0, pol_w);
          if (!waited) {
            pdl_wait();
            waited = true;
          }
          tma_load_2d(a_dst, &tmap_x, &full[s], kb * kPfBK, m0, pol_x);
          issued = it + 1;
        }
      }
      if (!waited) pdl_wait();
      // every copy issued must land before the shared memory is released
      const int first = issued > S ? issued - S : 0;
      for (int i = first; i < issued; ++i) {
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&full[i % S], static_cast<uint32_t>(i / S) & 1u)) {
          if (global_timer_ns() - t0 > kPfWaitNs) {
            pf_abort(p, s_abort);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(kPfBM, BN);
      const uint32_t smem_base = smem_u32(smem);
      int it = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntotal && ok; t += gridDim.x, ++local) {
        const int b = local & 1;
        if (!pf_wait(&acc_empty[b], ((local >> 1) & 1) ^ 1, s_abort)) {
          pf_abort(p, s_abort);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * BN);
        for (int kb = 0; kb < p.kiters; ++kb, ++it) {
          const int s = it % S;
          if (!pf_wait(&full[s], (it / S) & 1, s_abort)) {
            pf_abort(p, s_abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_base + s * C::kStageBytes;
          const uint64_t a_desc = smem_desc_k128_sw128(a_addr);
          const uint64_t b_desc = smem_desc_k128_sw128(a_addr + C::kABytes);
#pragma unroll
          for (int k = 0; k < kPfBK / 32; ++k)  // K = 32 bytes per instruction: +2 in the 16-byte address field
            mma_i8(d, a_desc + 2 * k, b_desc + 2 * k, idesc, (kb | k) != 0);
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
      // all issued MMAs complete before the tensor memory can be freed
      mma_commit(mma_done);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(mma_done, 0)) {
        if (global_timer_ns() - t0 > kPfWaitNs) {
          pf_abort(p, s_abort);
          break;
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5, token rows)
    const int q = warp & 3;         // tensor-memory lane quarter this warp may read
    const int et = threadIdx.x - 64;  // 0..127 among the epilogue threads
    pdl_wait();                       // scales of the tokens come from the quantization kernel
    int local = 0;
    for (int t = blockIdx.x; t < ntotal; t += gridDim.x, ++local) {
      const int n0 = (t / p.mtiles) * BN;
      const int m0 = (t % p.mtiles) * kPfBM;
      const int b = local & 1;
      // this tile's channel scales and bias, staged once for the four warps
      named_bar_sync(1, 128);  // the previous tile's readers are done
      for (int j = et; j < BN; j += 128) {
        const int n = n0 + j;
        s_sw[j] = n < p.N ? __ldg(p.sw + n) : 0.f;
        s_bias[j] = (p.bias && n < p.N) ? __bfloat162float(p.bias[n]) : 0.f;
      }
      named_bar_sync(1, 128);
      const int m = m0 + 32 * q + lane;
      const float sxm = m < p.M ? __ldg(p.sx + m) : 0.f;
      // lane 0 waits and the warp follows its answer (tcgen05.ld needs the whole warp); after an abort the loop
      // keeps its shape (the named barriers above) and only skips the work
      int have = 0;
      if (lane == 0) {
        have = pf_wait(&acc_full[b], (local >> 1) & 1, s_abort) ? 1 : 0;
        if (!have) pf_abort(p, s_abort);
      }
      have = __shfl_sync(0xffffffffu, have, 0);
      tc_fence_after();
      __nv_bfloat16* yrow = p.y + static_cast<int64_t>(m) * p.ldy;
      const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.y) | static_cast<uintptr_t>(p.ldy * 2)) & 15) == 0;
#pragma unroll 1
      for (int c = 0; have && c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(b * BN + 32 * c), r);
        if (m < p.M) {
          __align__(16) __nv_bfloat16 o[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float tv = __fmul_rn(static_cast<float>(static_cast<int>(r[j])), s_sw[32 * c + j]);
            const float v = p.bias ? __fmaf_rn(sxm, tv, s_bias[32 * c + j]) : __fmul_rn(sxm, tv);
            o[j] = __float2bfloat16_rn(v);
          }
          const int nb = n0 + 32 * c;
          if (vec_ok && nb + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(yrow + nb)[j] = reinterpret_cast<const uint4*>(o)[j];
          } else {
            for (int j = 0; j < 32; ++j)
              if (nb + j < p.N) yrow[nb + j] = o[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// ----------------------------------------------------------------------------------------------- host side
std::mutex g_pf_mu;
int g_pf_sms[64] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_pf_encode = nullptr;

int pf_device(int* dev, int* sms) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (*dev < 0 || *dev >= 64) return fail(QF_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lk(g_pf_mu);
  if (g_pf_sms[*dev] == 0) {
    int major = 0, minor = 0, n = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, *dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, *dev);
    g_pf_sms[*dev] = (major == 10 && minor == 0) ? n : -1;
  }
  if (g_pf_sms[*dev] < 0)
    return fail(QF_ERR_ARCH, "libqf_b200 is built for sm_100a (B200); this device is not compute capability 10.0");
  if (!g_pf_encode) {
    cudaDriverEntryPointQueryResult qres;
    void* fn = nullptr;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres);
    if (e != cudaSuccess || qres != cudaDriverEntryPointSuccess || !fn)
      return fail(QF_ERR_DRIVER, "cuTensorMapEncodeTiled entry point not found");
    g_pf_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  *sms = g_pf_sms[*dev];
  return QF_OK;
}

int pf_encode(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kPfBK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_pf_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(QF_ERR_DRIVER, "cuTensorMapEncodeTiled rejected the tensor (error " + std::to_string(r) + ")");
  return QF_OK;
}

size_t pf_ldq(int K) { return (static_cast<size_t>(K) + 15) / 16 * 16; }
size_t pf_q_bytes(int M, int K) { return (static_cast<size_t>(M) * pf_ldq(K) + 255) / 256 * 256; }

template <int BN>
int pf_launch(const CUtensorMap& tx, const CUtensorMap& tw, PfParams& p, int dev, int sms, unsigned flags,
              cudaStream_t st) {
  using C = PfGeo<BN>;
  static bool attr_set[64] = {};
  {
    std::lock_guard<std::mutex> lk(g_pf_mu);
    if (!attr_set[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(w8a8_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 C::kSmemBytes);
      if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      attr_set[dev] = true;
    }
  }
  p.ntiles = (p.N + BN - 1) / BN;
  const int total = p.mtiles * p.ntiles;
  int G = sms < kPfMaxGrid ? sms : kPfMaxGrid;
  if (G > total) G = total;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // the weight stream of the first stages overlaps the quantization kernel
  (void)flags;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w8a8_kernel<BN>, tx, tw, p);
  return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, std::string("launch: ") + cudaGetErrorString(e));
}

}  // namespace
}  // namespace qf

using namespace qf;

extern "C" {

size_t qf_w8a8_workspace_bytes(int M, int K) {
  if (M <= 0 || K <= 0) return kPfHeader;
  return kPfHeader + pf_q_bytes(M, K) + sizeof(float) * static_cast<size_t>(M);
}

int qf_w8a8_gemm(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* w_scale, const void* bias,
                 void* y, int64_t ldy, int M, int N, int K, void* ws, size_t ws_bytes, unsigned flags, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(QF_ERR_SHAPE, "negative size");
  if (M == 0 || N == 0) return QF_OK;
  if (K == 0) return fail(QF_ERR_SHAPE, "K must be >= 1");
  if (N > (1 << 30) || M > (1 << 30)) return fail(QF_ERR_SHAPE, "M or N too large");
  if (!x || !w || !w_scale || !y || !ws) return fail(QF_ERR_INVALID, "null pointer");
  if (ldw < K || (M > 1 && ldx < K) || (M > 1 && ldy < N)) return fail(QF_ERR_STRIDE, "leading dimension too small");
  if (reinterpret_cast<uintptr_t>(w) % 16 || ldw % 16)
    return fail(QF_ERR_ALIGN, "w must be 16-byte aligned with ldw % 16 == 0");
  if (reinterpret_cast<uintptr_t>(x) % 2) return fail(QF_ERR_ALIGN, "x must be 2-byte aligned");
  if (reinterpret_cast<uintptr_t>(ws) % 256) return fail(QF_ERR_ALIGN, "workspace must be 256-byte aligned");
  if (ws_bytes < qf_w8a8_workspace_bytes(M, K)) return fail(QF_ERR_WORKSPACE, "workspace too small");
  int dev = 0, sms = 0;
  int rc = pf_device(&dev, &sms);
  if (rc) return rc;
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  int8_t* xq = reinterpret_cast<int8_t*>(wsb + kPfHeader);
  float* sx = reinterpret_cast<float*>(wsb + kPfHeader + pf_q_bytes(M, K));
  const size_t ldq = pf_ldq(K);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // 1. per-token quantization (PDL: it may start while the previous kernel on the stream finishes)
  const int vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0 && (M == 1 || ldx % 8 == 0)) ? 1 : 0;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(M));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (flags & QF_FLAG_PDL) ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, quantize_tokens_kernel, static_cast<const __nv_bfloat16*>(x),
                                             ldx, K, xq, static_cast<int64_t>(ldq), sx, vec);
    if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("quantize launch: ") + cudaGetErrorString(e));
  }
  // 2. the GEMM
  PfParams p = {};
  p.sx = sx;
  p.sw = w_scale;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = M > 1 ? ldy : N;
  p.M = M;
  p.N = N;
  p.K = K;
  p.mtiles = (M + kPfBM - 1) / kPfBM;
  p.kiters = (K + kPfBK - 1) / kPfBK;
  p.err = reinterpret_cast<int*>(wsb);
  CUtensorMap tx, tw;
  rc = pf_encode(&tx, xq, ldq, static_cast<uint64_t>(M), ldq, kPfBM);
  if (rc) return rc;
  // channel-block height: the widest tile that still gives every SM a tile
  const long long mt = p.mtiles;
  int bn = 256;
  if (mt * ((N + 255) / 256) < sms) bn = (mt * ((N + 127) / 128) < sms) ? 64 : 128;
  rc = pf_encode(&tw, w, static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint64_t>(ldw),
                 static_cast<uint32_t>(bn));
  if (rc) return rc;
  if (bn == 256) return pf_launch<256>(tx, tw, p, dev, sms, flags, st);
  if (bn == 128) return pf_launch<128>(tx, tw, p, dev, sms, flags, st);
  return pf_launch<64>(tx, tw, p, dev, sms, flags, st);
}

}  // extern "C"
