// qf_allreduce.cu -- one-shot all-reduce of bf16 vectors between the tensor-parallel ranks of one node, over
// NVLink peer memory.
//
// Under tensor parallelism the row-parallel layers of the decode path (o_proj, down) end with a sum of every
// rank's bf16 partial output [M, 5120]; vLLM issues an NCCL all-reduce for it after RowParallelLinear (the
// reference plugin leaves that call to vLLM).  At decode sizes (M <= 16: at most 160 KB per rank) the all-reduce
// is pure latency, so this kernel does it in one pass:
//
//   * every rank owns one symmetric buffer (cudaMalloc'd, shared with the other ranks through CUDA IPC);
//   * CTA c of every rank takes elements [c*1024, (c+1)*1024): it stores its input chunk into slot [rank] of every
//     rank's buffer (peer stores over NVLink), then sets flag [rank][c] in every rank's buffer to the call's
//     epoch (st.release.sys);
//   * it waits (bounded) until all ranks' flags [*][c] in its own buffer carry the epoch, then sums the W slots in
//     rank order in fp32 and rounds once to bf16: every rank computes the same bits, deterministic.
//
// Epochs live in device memory (the buffer header), so the call is CUDA-graph capturable: each launch reads
// epoch = header.epoch + 1 and the last CTA to finish stores it back.  Slots and flags are double-buffered by
// epoch parity: a rank can only reach epoch e + 2 after every rank has pushed epoch e + 1, i.e. finished reading
// epoch e, so a slot is never overwritten while a peer still reads it.  A flag wait that exceeds kArWaitNs
// records QF_ERR_TIMEOUT in the header (read by qf_allreduce_status) and the CTA continues.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>

#include "../../include/qf_b200.h"
#include "qf_comm.cuh"
#include "qf_host.h"
#include "qf_ptx.cuh"

namespace qf {
namespace {

constexpr int kArThreads = 128;
constexpr int kArChunk = 1024;                  // bf16 elements per CTA

struct ArParams {
  const __nv_bfloat16* in;
  __nv_bfloat16* out;
  int count;      // elements, multiple of 8
  int max_count;  // slot capacity (elements) of every buffer
  int rank;
  int world;
  uint8_t* bufs[QF_AR_MAX_RANKS];  // every rank's buffer, this rank's at [rank]
};


__global__ void __launch_bounds__(kArThreads) allreduce_kernel(const ArParams p) {
  // The next kernel may be scheduled now (its weight prefetch overlaps this kernel; it reads this kernel's
  // output only after its own griddepcontrol.wait).  The input is the previous kernel's output.
  pdl_launch_dependents();
  pdl_wait();
  uint8_t* own = p.bufs[p.rank];
  uint32_t* hdr = reinterpret_cast<uint32_t*>(own);
  __shared__ uint32_t s_epoch;
  __shared__ int s_timeout;
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(hdr + 1) + 1u;
    s_timeout = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int par = static_cast<int>(epoch & 1u);
  const int c = blockIdx.x;
  const int e0 = c * kArChunk;
  const int nv = min(kArChunk, p.count - e0) / 8;  // 16-byte vectors in this chunk

  // 1. push this rank's chunk into slot [rank] of every rank's buffer
  const uint4* src = reinterpret_cast<const uint4*>(p.in + e0);
  for (int i = threadIdx.x; i < nv; i += kArThreads) {
    const uint4 v = src[i];
    for (int r = 0; r < p.world; ++r) ar_slot(p.bufs[r], par, p.rank, p.max_count, e0)[i] = v;
  }
  __syncthreads();
  // 2. publish: after the CTA barrier, thread r raises flag [rank][c] on rank r with a system-scope release,
  //    which orders the whole CTA's stores above before the flag
  if (threadIdx.x < p.world) st_release_sys(ar_flag(p.bufs[threadIdx.x], par, p.rank, c), epoch);
  // 3. wait for every rank's chunk c (flags only grow: a stale value is epoch - 2)
  if (threadIdx.x < p.world) {
    const uint32_t* f = ar_flag(own, par, threadIdx.x, c);
    if (ld_acquire_sys(f) != epoch) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_sys(f) != epoch) {
        if (global_timer_ns() - t0 > kArWaitNs) {
          s_timeout = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (s_timeout && threadIdx.x == 0) atomicExch(hdr, static_cast<uint32_t>(QF_ERR_TIMEOUT));
  // 4. sum the ranks' slots in rank order (fp32), one rounding to bf16
  for (int i = threadIdx.x; i < nv; i += kArThreads) {
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    for (int r = 0; r < p.world; ++r) {
      const uint4 v = __ldcg(ar_slot(own, par, r, p.max_count, e0) + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[2 * k] += __uint_as_float(w[k] << 16);
        acc[2 * k + 1] += __uint_as_float(w[k] & 0xFFFF0000u);
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
      ow[k] = *reinterpret_cast<const uint32_t*>(&b);
    }
    reinterpret_cast<uint4*>(p.out + e0)[i] = o;
  }
  // 5. the last CTA to finish advances the epoch for the next launch on this rank
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t done = atomicAdd(hdr + 2, 1u);
    if (done == gridDim.x - 1) {
      hdr[2] = 0u;
      hdr[1] = epoch;
    }
  }
}

}  // namespace
}  // namespace qf

using namespace qf;

extern "C" {

size_t qf_allreduce_buffer_bytes(int max_count) {
  if (max_count <= 0) return 0;
  return kArData + sizeof(uint16_t) * 2 * QF_AR_MAX_RANKS * static_cast<size_t>(max_count);
}

int qf_symm_alloc(size_t bytes, void** dev_ptr) {
  if (!dev_ptr || bytes == 0) return fail(QF_ERR_INVALID, "null output pointer or zero size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return fail(QF_ERR_LAUNCH, std::string("symmetric buffer allocation: ") + cudaGetErrorString(e));
  }
  *dev_ptr = p;
  return QF_OK;
}

int qf_symm_free(void* dev_ptr) {
  if (!dev_ptr) return QF_OK;
  const cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, std::string("cudaFree: ") + cudaGetErrorString(e));
}

int qf_ipc_handle(void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return fail(QF_ERR_INVALID, "null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == QF_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, dev_ptr);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  std::memcpy(handle_out, &h, sizeof(h));
  return QF_OK;
}

int qf_ipc_open(const void* handle, void** peer_ptr) {
  if (!handle || !peer_ptr) return fail(QF_ERR_INVALID, "null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  *peer_ptr = p;
  return QF_OK;
}

int qf_ipc_close(void* peer_ptr) {
  if (!peer_ptr) return QF_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
}

int qf_allreduce_bf16(const void* in, void* out, int count, int max_count, int rank, int world,
                      void* const* bufs, unsigned flags, void* stream) {
  if (world < 1 || world > QF_AR_MAX_RANKS) return fail(QF_ERR_INVALID, "world size must be 1..8");
  if (rank < 0 || rank >= world) return fail(QF_ERR_INVALID, "rank out of range");
  if (count < 0 || count > max_count) return fail(QF_ERR_SHAPE, "count must be in [0, max_count]");
  if (max_count > QF_AR_MAX_CHUNKS * 1024) return fail(QF_ERR_SHAPE, "max_count above QF_AR_MAX_CHUNKS * 1024");
  if (count % 8 || max_count % 8) return fail(QF_ERR_SHAPE, "count and max_count must be multiples of 8");
  if (count == 0) return QF_OK;
  if (!in || !out || !bufs) return fail(QF_ERR_INVALID, "null pointer");
  if (reinterpret_cast<uintptr_t>(in) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(QF_ERR_ALIGN, "in and out must be 16-byte aligned");
  ArParams p = {};
  p.in = static_cast<const __nv_bfloat16*>(in);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.count = count;
  p.max_count = max_count;
  p.rank = rank;
  p.world = world;
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || reinterpret_cast<uintptr_t>(bufs[r]) % 256) return fail(QF_ERR_ALIGN, "buffers must be 256-byte aligned");
    p.bufs[r] = static_cast<uint8_t*>(bufs[r]);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((count + 1023) / 1024));
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & QF_FLAG_PDL) ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, allreduce_kernel, p);
  return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, std::string("launch: ") + cudaGetErrorString(e));
}

int qf_allreduce_status(void* own_buf, void* stream, int* status) {
  if (!own_buf || !status) return fail(QF_ERR_INVALID, "null argument");
  int v = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, own_buf, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && v != 0) e = cudaMemsetAsync(own_buf, 0, sizeof(int), st);
  if (e != cudaSuccess) return fail(QF_ERR_LAUNCH, cudaGetErrorString(e));
  *status = v;
  return QF_OK;
}

}  // extern "C"
