// qf_comm.cuh -- layout of the symmetric (CUDA IPC) buffers shared by the tensor-parallel ranks of one node, used
// by the one-shot all-reduce kernel and by the GEMM's fused all-reduce epilogue.
//
// Each rank's buffer:
//   [0, 256)      header, u32: [0] sticky error word, [1] epoch (calls completed), [2] CTAs done,
//                 [3] bound of every wait on the other ranks in microseconds (0: kArWaitNs)
//   [256, ...)    16-byte lines [2 parity][QF_AR_MAX_RANKS source rank][max_count / 4]
// A line carries 4 bf16 values with the call's epoch stored twice, {v0v1, epoch, v2v3, epoch}: each 8-byte half is
// written and read as one access, so a reader that sees the epoch in both halves has both payload words of this
// call, without a fence or a separate flag (peers write the lines over NVLink; the owner polls them in its own
// memory).  A call with epoch e (= header[1] + 1) uses parity e & 1; lines left from call e - 2 carry e - 2.
#pragma once
#include <cstddef>
#include <cstdint>

#include "../../include/qf_b200.h"
#include "qf_ptx.cuh"

namespace qf {

constexpr size_t kArHeader = 256;
constexpr size_t kArData = kArHeader;
constexpr uint64_t kArWaitNs = 2000000000ull;  // default bound of every cross-GPU wait (2 s)

// Bound (ns) of the waits of a call on this rank's buffer: header word 3 in microseconds, or kArWaitNs if it is 0.
__device__ __forceinline__ uint64_t ar_wait_bound_ns(const uint8_t* own) {
  const uint32_t us = *reinterpret_cast<const volatile uint32_t*>(own + 12);
  return us ? static_cast<uint64_t>(us) * 1000ull : kArWaitNs;
}

// Line `line` (= element / 4) of slot [par][src].
__device__ __forceinline__ uint4* ar_line(uint8_t* buf, int par, int src, int max_count, int line) {
  return reinterpret_cast<uint4*>(buf + kArData) +
         (static_cast<size_t>(par * QF_AR_MAX_RANKS + src) * (max_count / 4) + line);
}

__device__ __forceinline__ void st_volatile_v4(uint4* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_volatile_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Waits (bounded: *deadline_ns is set to now + bound_ns on first use) until both halves of the line carry `epoch`;
// returns the payload {v0v1, v2v3}.  Sets *timed_out and returns whatever the line holds if the bound expires.
__device__ __forceinline__ uint2 ar_wait_line(const uint4* p, uint32_t epoch, uint64_t bound_ns, uint64_t* deadline_ns,
                                              int* timed_out) {
  uint4 v = ld_volatile_v4(p);
  int spins = 0;
  while ((v.y != epoch || v.w != epoch) && !*timed_out) {
    if (++spins == 64) {
      spins = 0;
      const uint64_t now = global_timer_ns();
      if (*deadline_ns == 0) *deadline_ns = now + bound_ns;
      else if (now > *deadline_ns) *timed_out = 1;
    }
    v = ld_volatile_v4(p);
  }
  return make_uint2(v.x, v.z);
}

__device__ __forceinline__ void bf16x2_acc(float& a, float& b, uint32_t w) {
  a += __uint_as_float(w << 16);
  b += __uint_as_float(w & 0xFFFF0000u);
}

}  // namespace qf
