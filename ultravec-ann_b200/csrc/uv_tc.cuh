// uv_tc.cuh -- sm_100a tensor-core plumbing used by the scan's prefilter:
// tcgen05 (TMEM allocation, MMA issue/commit, TMEM loads, ordering fences),
// mbarriers with bounded waits, and the shared-memory matrix descriptors.
//
// Operand layout: K-major with the 128-byte swizzle.  A tile of R rows x 64
// fp16 (one "atom column") is R x 128 bytes, rows 128 B apart, 8-row groups
// 1024 B apart; the 16-byte chunk c of row r sits at chunk position c ^ (r & 7).
// Wider K is a sequence of such atom columns, each R * 128 bytes.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace uvb {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- mbarriers ----
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
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
// Wait for the phase with the given parity to complete, giving up after
// `limit` polls (each try_wait itself blocks for a hardware-defined slice).
// Returns false on timeout; the caller records the error and winds down.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; i++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// After an abort: wait (bounded) until the last load armed on each of the
// `stages` barriers has landed, so that no bulk copy is still writing into
// shared memory when the CTA exits.  `issued` = stage uses armed so far.
__device__ __forceinline__ void drain_stages(uint64_t *full, int stages, int64_t issued,
                                             uint32_t limit) {
  for (int s = 0; s < stages; s++) {
    if (issued <= s) continue;
    const int64_t last = issued - 1 - ((issued - 1 - s) % stages);  // last use of stage s
    for (uint32_t i = 0; i < limit; i++)
      if (mbar_try_wait(&full[s], (uint32_t)((last / stages) & 1))) break;
  }
}

// Arrive and add `bytes` to the transaction count the phase waits for.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// ---- TMA: one 2-D tile of a tensor map into this CTA's shared memory, its
// bytes counted on `bar`.  c0 is the inner (contiguous) coordinate.  No
// cluster multicast: the tile lands in the issuing CTA only.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int c0, int c1,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      :
      : "r"(smem_u32(dst)), "l"((uint64_t)tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Generic-proxy shared-memory writes made visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 ordering ----
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- TMEM allocation (one full warp) ----
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// ---- descriptors ----
// Shared-memory matrix descriptor: start >> 4 in [0,14), leading byte offset
// >> 4 in [16,30) (unused by swizzled K-major layouts, set to 16 B), stride
// byte offset >> 4 in [32,46) (1024 B between 8-row groups), version 1 in
// [46,48), base offset 0, layout type 2 (128-byte swizzle) in [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// The same for a K-major tile with the 32-byte swizzle (rows of 16 fp16,
// 8-row groups 256 B apart, layout type 6): one K step per atom.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(256u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)6 << 61;
  return d;
}
// Byte offset of the 16-byte chunk c (0 or 1) of row r in a K-major
// 32-byte-swizzled tile: chunk position c ^ ((r >> 2) & 1).
__host__ __device__ __forceinline__ uint32_t sw32_chunk_offset(int r, int c) {
  return (uint32_t)(r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
}

// Instruction descriptor of kind::f16: f32 accumulator (bits 4-5 = 1), A and
// B fp16 (format 0), both K-major, N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- MMA (issued by one thread) ----
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :
      : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every previously issued MMA of this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// ---- TMEM -> registers: 32 lanes x 32 columns, one column per register ----
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// TMEM -> registers: 32 lanes x 16 columns (thread = lane, r[j] = column j)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Byte offset of the 16-byte chunk holding elements [8c, 8c+8) of row r in a
// K-major 128-byte-swizzled tile of `rows` rows (c counts along all of K).
__host__ __device__ __forceinline__ uint32_t sw128_chunk_offset(int r, int c, int rows) {
  const int atom = c >> 3;   // 64 fp16 per 128-byte row of an atom column
  const int cc = c & 7;
  return (uint32_t)(atom * rows * 128 + r * 128 + ((cc ^ (r & 7)) << 4));
}

}  // namespace tc
}  // namespace uvb
