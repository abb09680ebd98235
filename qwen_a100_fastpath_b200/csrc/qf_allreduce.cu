// qf_allreduce.cu -- one-shot all-reduce of bf16 vectors between the tensor-parallel ranks of one node, over
// NVLink peer memory.
//
// Under tensor parallelism the row-parallel layers of the decode path (o_proj, down) end with a sum of every
// rank's bf16 partial output [M, 5120]; vLLM issues an NCCL all-reduce for it after RowParallelLinear (the
// reference plugin leaves that call to vLLM).  At decode sizes (M <= 16: at most 160 KB per rank) the all-reduce
// is pure latency, so this kernel does it in one pass with self-validating lines (qf_comm.cuh):
//
//   * every rank owns one symmetric buffer (cudaMalloc'd, shared with the other ranks through CUDA IPC);
//   * CTA c of every rank takes elements [c*1024, (c+1)*1024): it writes its input chunk as lines
//     {v0v1, epoch, v2v3, epoch} into slot [rank] of every other rank's buffer (peer stores over NVLink);
//   * it then reads, for every element group, the other ranks' lines from its own buffer (spinning, bounded, until
//     both halves carry the call's epoch) and sums all ranks' values in rank order in fp32, its own taken from its
//     input, with one rounding to bf16: every rank computes the same bits, deterministic.
//
// No fence or flag round trip is needed: a line is valid exactly when both of its 8-byte halves carry the epoch.
// Epochs live in device memory (the buffer header), so the call is CUDA-graph capturable: each launch reads
// epoch = header.epoch + 1 and the last CTA to finish stores it back.  Lines are double-buffered by epoch parity: a
// rank reaches epoch e + 2 only after every rank has written its lines of epoch e + 1, i.e. finished reading epoch
// e, so a line is never overwritten while a peer still reads it.  A wait that exceeds its bound (2 s, or what
// qf_allreduce_set_wait stored in the header) records QF_ERR_TIMEOUT in the header (read by qf_allreduce_status) and
// the CTA continues.
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
  __shared__ uint64_t s_bound;
  __shared__ int s_timeout;
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(hdr + 1) + 1u;
    s_bound = ar_wait_bound_ns(own);
    s_timeout = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const uint64_t bound = s_bound;
  const int par = static_cast<int>(epoch & 1u);
  const int e0 = blockIdx.x * kArChunk;
  const int nl = min(kArChunk, p.count - e0) / 4;  // lines (4 elements each) in this chunk
  const uint2* src = reinterpret_cast<const uint2*>(p.in + e0);

  // 1. write this rank's chunk as lines into slot [rank] of every other rank's buffer
  for (int i = threadIdx.x; i < nl; i += kArThreads) {
    const uint2 v = src[i];
    const uint4 line = make_uint4(v.x, epoch, v.y, epoch);
    for (int r = 0; r < p.world; ++r)
      if (r != p.rank) st_volatile_v4(ar_line(p.bufs[r], par, p.rank, p.max_count, e0 / 4 + i), line);
  }
  // 2. sum every rank's values in rank order (this rank's from its input), fp32, one rounding
  uint64_t deadline = 0;
  int timed_out = 0;
  for (int i = threadIdx.x; i < nl; i += kArThreads) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int r = 0; r < p.world; ++r) {
      const uint2 v = (r == p.rank) ? src[i]
                                    : ar_wait_line(ar_line(own, par, r, p.max_count, e0 / 4 + i), epoch, bound,
                                                   &deadline, &timed_out);
      bf16x2_acc(a0, a1, v.x);
      bf16x2_acc(a2, a3, v.y);
    }
    const __nv_bfloat162 b01 = __floats2bfloat162_rn(a0, a1);
    const __nv_bfloat162 b23 = __floats2bfloat162_rn(a2, a3);
    reinterpret_cast<uint2*>(p.out + e0)[i] =
        make_uint2(*reinterpret_cast<const uint32_t*>(&b01), *reinterpret_cast<const uint32_t*>(&b23));
  }
  if (timed_out) s_timeout = 1;
  // 3. the last CTA to finish advances the epoch for the next launch on this rank
  __syncthreads();
  if (threadIdx.x == 0) {
    if (s_timeout) atomicExch(hdr, static_cast<uint32_t>(QF_ERR_TIMEOUT));
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
  return kArData + 4 * 2 * QF_AR_MAX_RANKS * static_cast<size_t>(max_count);  // 16-byte line per 4 elements
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

int qf_allreduce_set_wait(void* own_buf, unsigned wait_us, void* stream) {
  if (!own_buf) return fail(QF_ERR_INVALID, "null buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint32_t v = wait_us;
  cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(own_buf) + 12, &v, sizeof(v), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return e == cudaSuccess ? QF_OK : fail(QF_ERR_LAUNCH, cudaGetErrorString(e));
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
