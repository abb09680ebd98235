// qf_ptx.cuh -- thin inline-PTX wrappers used by the sm_100a kernels of libqf_b200.
//
// Only documented PTX ISA forms are used: mbarrier (arrive / expect_tx / try_wait.parity), the tiled TMA
// loads cp.async.bulk.tensor.2d / .4d (no multicast), createpolicy for L2 eviction hints, griddepcontrol for
// programmatic dependent launch, bar.sync on named barriers, ldmatrix (.trans), ex2.approx, mma.sync m16n8k16
// bf16 / f16, and the tcgen05 forms listed further down.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace qf {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier --------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy and to the other threads of the CTA.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- TMA (tiled, 2-D, no multicast) -----------------------------------------------------------
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Coordinates: c0 = innermost (element index along the contiguous dimension), c1 = row.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Four-dimensional tiled load (same form, coordinates c0 innermost .. c3 outermost).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Brings a kernel-parameter tensor map into the TMA unit's descriptor cache before its first copy.
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- programmatic dependent launch -------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- cross-CTA flags -----------------------------------------------------------------------------
__device__ __forceinline__ int ld_acquire_gpu(const int* ptr) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ void sleep_ns(uint32_t ns) { asm volatile("nanosleep.u32 %0;" ::"r"(ns)); }
// Atomic add with acquire + release semantics at GPU scope: the caller's earlier writes (and those ordered before
// it by a CTA or warp barrier) are visible to whoever observes the new value, and writes released by earlier
// adders are visible to the caller afterwards.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* ptr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(ptr), "r"(v) : "memory");
  return old;
}

// ---- named barriers (id 0 is __syncthreads) -----------------------------------------------------
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Signal barrier `id` without waiting (the waiting side uses named_bar_sync with the same count).
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- shared / global loads ---------------------------------------------------------------------
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// ---- tensor-core MMA (legacy warp-level path, still issued on sm_100) ---------------------------
// D[16x8] += A[16x16] (row) * B[16x8] (col), bf16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_bf16_m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                  uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16_m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                 uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four 8x8 b16 matrices from shared memory; lane l supplies the address of row (l % 8) of matrix (l / 8), and
// register j receives matrix j in the mma fragment layout (thread (g, t) holds row g, columns 2t, 2t + 1; with .trans
// the matrix is transposed on the way).
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// 2^x by the special-function unit (PTX ex2.approx.ftz.f32: relative error about 2^-22; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void lds64(uint32_t addr, uint32_t& a, uint32_t& b) {
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
}
__device__ __forceinline__ void sts64(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}

// ---- exact int8 -> fp16 ----------------------------------------------------------------------------
// Four signed bytes (k, k+1, k+2, k+3) -> a02 = f16x2{k, k+2}, a13 = f16x2{k+1, k+3}.
// One lop3 builds, for bytes 0 and 2, the fp16 bit patterns 0x64uu with uu = byte ^ 0x80 (= byte + 128):
// out = mask ? (w ^ C) : C with mask 0x00FF00FF and C = 0x64806480 (lut 0x6A), i.e. the fp16 values
// 1024 + byte + 128; the same on w >> 8 gives bytes 1 and 3.  Subtracting 1152 leaves the byte exactly
// (fp16 holds every integer up to 2048).  The pairing (k, k+2) / (k+1, k+3) is matched by the activation
// layout the kernel builds.
__device__ __forceinline__ void dequant_i8x4_f16(uint32_t w, uint32_t& a02, uint32_t& a13) {
  uint32_t lo, hi;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(lo) : "r"(w), "r"(0x00FF00FFu), "r"(0x64806480u));
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(hi) : "r"(w >> 8), "r"(0x00FF00FFu), "r"(0x64806480u));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(a02) : "r"(lo), "r"(0x64806480u));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(a13) : "r"(hi), "r"(0x64806480u));
}

// Two bf16x2 words (x0, x1), (x2, x3) -> f16x2 (x0, x2), (x1, x3), the activation pairing of
// dequant_i8x4_f16.  Returns non-zero if any value is outside the fp16 range (|x| >= 65536, Inf, NaN):
// the magnitude bits plus 0x3880 reach bit 15 exactly when they are >= 0x4780 (bf16 65536).  Values below
// fp16's normal range (|x| < 2^-14) become fp16 subnormals, which keep 2^-24 absolute resolution: not exact
// there, but within 2^-25 of the bf16 value.
__device__ __forceinline__ uint32_t bf16x4_to_f16_pairs(uint32_t w0, uint32_t w1, uint32_t& o0, uint32_t& o1) {
  const float x0 = __uint_as_float(w0 << 16), x1 = __uint_as_float(w0 & 0xFFFF0000u);
  const float x2 = __uint_as_float(w1 << 16), x3 = __uint_as_float(w1 & 0xFFFF0000u);
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(o0) : "f"(x2), "f"(x0));
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(o1) : "f"(x3), "f"(x1));
  const uint32_t t0 = (w0 & 0x7FFF7FFFu) + 0x38803880u;
  const uint32_t t1 = (w1 & 0x7FFF7FFFu) + 0x38803880u;
  return (t0 | t1) & 0x80008000u;
}

// ---- exact int8 -> bf16 ---------------------------------------------------------------------------
// Four signed bytes (k, k+1, k+2, k+3) -> lo = bf16x2{k, k+1}, hi = bf16x2{k+2, k+3}.
// Each byte b is biased to u = b + 128 (xor 0x80), placed in the low mantissa byte of the fp32 2^23
// (bit pattern 0x4B0000uu = 8388608 + u), and 8388608 + 128 is subtracted: an exact fp32 integer in
// [-128, 127].  Such integers have at most 8 significant bits, so their upper 16 bits are the exact bf16.
__device__ __forceinline__ void dequant_i8x4_bf16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f;
  const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f;
  const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f;
  const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f;
  lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
  hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632);
}

}  // namespace qf

// ---- tcgen05 (5th-generation tensor cores, accumulators in tensor memory) ----------------------------------------
namespace qf {

__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Allocates `ncols` (power of two, 32..512) tensor-memory columns for this CTA; the address lands in *smem_dst.
// Executed by one whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] x B[smem desc]^T, signed int8 operands, int32 accumulators (one thread issues).
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on the mbarrier when every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive 32-bit columns of the warp's 32 tensor-memory lanes: thread t gets lane (lane base + t).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored as 128-byte rows with the 128-byte swizzle (what
// a TMA box of 128 bytes x rows with CU_TENSOR_MAP_SWIZZLE_128B writes; tile base 1024-byte aligned): start address,
// leading-dimension offset 16 B (unused for this layout), stride between 8-row groups 1024 B, descriptor version 1,
// layout type 2 (128-byte swizzle).  A k offset of j*32 bytes inside the 128-byte row is start address + j*32.
__device__ __forceinline__ uint64_t smem_desc_k128_sw128(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::i8: int32 accumulator, signed int8 A and B, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// D[tmem] (+)= A[smem desc] x B[smem desc]^T, bf16 operands, fp32 accumulators (kind::f16; one thread issues).
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem desc]^T, bf16 operands, fp32 accumulators (kind::f16; one thread issues).  A sits in
// tensor memory K-major: row m on lane m, k along the columns, two 16-bit elements per 32-bit column (the lower k in
// the low half), so a K = 16 step spans 8 columns.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 8 consecutive 32-bit columns of the warp's 32 tensor-memory lanes: thread t gets lane (lane base + t).
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Instruction descriptor of tcgen05.mma kind::f16 with bf16 A and B and an fp32 accumulator, M x N; a_mn / b_mn
// select the MN-major (transposed) operand layout instead of K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn ? (1u << 15) : 0u) | (b_mn ? (1u << 16) : 0u) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Shared-memory descriptor of an MN-major operand stored as 128-byte swizzle atoms (64 consecutive 16-bit elements
// along M or N per 128-byte row, 8 rows along K per 1024-byte atom, which is what a 64-column TMA box with the
// 128-byte swizzle writes): atoms `lbo` bytes apart along M/N, 8-row groups `sbo` bytes apart along K.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16) |
         (static_cast<uint64_t>(sbo >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Stores 32 consecutive 32-bit columns of the warp's 32 tensor-memory lanes (thread t writes lane base + t), then
// waits for this thread's stores to complete unless `wait` is false.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32], bool wait = true) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  if (wait) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// fp32 -> int8 with round-to-nearest-even and saturation to [-128, 127]; NaN -> 0.
__device__ __forceinline__ int f32_to_s8_rni_sat(float v) {
  int r;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(v));
  return static_cast<int>(static_cast<int8_t>(r & 0xFF));
}

}  // namespace qf
