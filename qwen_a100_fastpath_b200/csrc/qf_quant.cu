// qf_quant.cu -- load-time int8 quantizer of the draft LM head on the device.
//
// Replaces the per-row symmetric quantizer the reference runs in torch when the draft model loads
// (plugin/qwen_fastpath/patches.py:143-147): for every row of the bf16 lm_head weight [V, H],
//   s = max(max_k |w[k]|, 1e-8) / 127        (fp32, IEEE division)
//   q[k] = clamp(round_half_even(w[k] / s), -127, 127)
// One CTA per row: the row is read once into registers, reduced to its absolute maximum, then divided and rounded
// with the same fp32 operations as the reference, so the result is bit-identical.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/qf_b200.h"
#include "qf_host.h"

namespace qf {
namespace {

constexpr int kQThreads = 256;
constexpr int kQPerThread = 32;  // elements per thread held in registers: rows up to 8192 wide

__global__ void __launch_bounds__(kQThreads) quantize_rows_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw,
                                                                  int H, int8_t* __restrict__ q, int64_t ldq,
                                                                  float* __restrict__ scale) {
  const int row = blockIdx.x;
  const __nv_bfloat16* wr = w + static_cast<int64_t>(row) * ldw;
  float v[kQPerThread];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kQPerThread; ++j) {
    const int k = threadIdx.x + j * kQThreads;
    v[j] = k < H ? __bfloat162float(wr[k]) : 0.f;
    amax = fmaxf(amax, fabsf(v[j]));
  }
  __shared__ float s_red[kQThreads / 32];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = s_red[0];
#pragma unroll
  for (int i = 1; i < kQThreads / 32; ++i) m = fmaxf(m, s_red[i]);
  const float s = fmaxf(m, 1e-8f) / 127.0f;
  if (threadIdx.x == 0) scale[row] = s;
  int8_t* qr = q + static_cast<int64_t>(row) * ldq;
#pragma unroll
  for (int j = 0; j < kQPerThread; ++j) {
    const int k = threadIdx.x + j * kQThreads;
    if (k < H) qr[k] = static_cast<int8_t>(fminf(fmaxf(rintf(v[j] / s), -127.f), 127.f));
  }
}

}  // namespace
}  // namespace qf

using namespace qf;

extern "C" int qf_quantize_rows_int8(const void* w, int64_t ldw, int V, int H, int8_t* q, int64_t ldq, float* scale,
                                     void* stream) {
  if (V < 0 || H < 0) return fail(QF_ERR_SHAPE, "negative size");
  if (H > kQThreads * kQPerThread) return fail(QF_ERR_SHAPE, "rows wider than 8192 elements");
  if (V == 0 || H == 0) return QF_OK;
  if (!w || !q || !scale) return fail(QF_ERR_INVALID, "null pointer");
  if (ldw < H || ldq < H) return fail(QF_ERR_STRIDE, "row stride smaller than the row");
  quantize_rows_kernel<<<static_cast<unsigned>(V), kQThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(w), ldw, H, q, ldq, scale);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, std::string("launch: ") + cudaGetErrorString(e));
}
