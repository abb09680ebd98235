// qf_comm.cuh -- layout of the symmetric (CUDA IPC) buffers shared by the tensor-parallel ranks of one node, used
// by the one-shot all-reduce kernel and by the GEMM's fused all-reduce epilogue.
//
// Each rank's buffer:
//   [0, 256)              header, u32: [0] sticky error word, [1] epoch (calls completed), [2] CTAs done
//   [256, kArData)        u32 flags[2 parity][QF_AR_MAX_RANKS source rank][QF_AR_MAX_CHUNKS chunk or tile]
//   [kArData, ...)        bf16 data[2 parity][QF_AR_MAX_RANKS source rank][max_count]
// A call with epoch e (= header[1] + 1) uses parity e & 1; a flag holding e marks its chunk ready.
#pragma once
#include <cstddef>
#include <cstdint>

#include "../../include/qf_b200.h"

namespace qf {

constexpr size_t kArHeader = 256;
constexpr size_t kArFlags = kArHeader;
constexpr size_t kArData = kArFlags + sizeof(uint32_t) * 2 * QF_AR_MAX_RANKS * QF_AR_MAX_CHUNKS;
static_assert(kArData % 256 == 0, "data alignment");
constexpr uint64_t kArWaitNs = 2000000000ull;  // bound of every cross-GPU wait (2 s)

__device__ __forceinline__ uint4* ar_slot(uint8_t* buf, int par, int src, int max_count, int e0) {
  return reinterpret_cast<uint4*>(buf + kArData +
                                  (static_cast<size_t>(par * QF_AR_MAX_RANKS + src) * max_count + e0) * 2);
}
__device__ __forceinline__ uint32_t* ar_flag(uint8_t* buf, int par, int src, int chunk) {
  return reinterpret_cast<uint32_t*>(buf + kArFlags) + (par * QF_AR_MAX_RANKS + src) * QF_AR_MAX_CHUNKS + chunk;
}

}  // namespace qf
