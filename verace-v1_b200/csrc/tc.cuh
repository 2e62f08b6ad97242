// Blackwell (sm_100a) tensor-core primitives written as inline PTX: tcgen05 MMA with
// shared-memory operand descriptors, tensor-memory (TMEM) allocation and loads,
// mbarrier completion tracking with bounded waits, and bf16 hi/lo operand splitting.
//
// Operand layouts used by the kernels (no swizzle, the canonical "interleaved" form):
// a core matrix is 8 rows x 16 bytes (8 bf16) stored contiguously (128 bytes).  A
// descriptor gives two strides: SBO between core matrices adjacent along M (or N) and
// LBO between core matrices adjacent along K.
//  * K-major tile of R rows x K columns (k contiguous inside a core row): element
//    (r, k) at byte ((k/8)*R + r)*16 + (k%8)*2.   SBO = 128, LBO = R*16;
//    advancing K by 16 moves the start address by 2*R*16 bytes.
//  * The same bytes read as an MN-major operand whose M index is k and whose K index
//    is r (m contiguous inside a core row): SBO = R*16, LBO = 128; advancing K by 16
//    moves the start address by 256 bytes.  So one staged tile of k/v vectors serves
//    as the K-major A of W^T H and as the MN-major A of W Cm.
//  * MN-major tile built directly (n contiguous inside a core row): element (k, n) at
//    byte ((k/8)*NG + n/8)*128 + (k%8)*16 + (n%8)*2 with NG = N/8.  SBO = 128,
//    LBO = NG*128; advancing K by 16 moves the start address by 2*NG*128 bytes.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace verace {
namespace tc {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory matrix descriptor (sm_100 format: version 1, no swizzle).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// Shared-memory matrix descriptor for the 128-byte-swizzled canonical layouts (atoms of
// 8 rows x 128 bytes, 1024-byte aligned; the hardware XORs address bits [4,7) with
// bits [7,10)).  K-major: rows of 64 bf16 k-elements, SBO = 1024 between 8-row groups,
// LBO unused (16); a K step of 16 inside an atom adds 32 bytes to the start address.
// MN-major: 64 contiguous m-elements per 128-byte row, rows are k; SBO = 1024 between
// 8-k-row groups, LBO = byte distance between 64-element m blocks.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return sdesc(saddr, lbo, sbo) | ((uint64_t)2u << 61);
}

// Instruction descriptor for kind::f16 with bf16 A/B and an fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major,
                                                  bool negate_a = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((negate_a ? 1u : 0u) << 13) |
         ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A * B, issued by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrive on `mbar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(mbar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(mbar)), "r"(count) : "memory");
}

// Invalidate an mbarrier with no pending operations, so that it can be initialised again.
__device__ __forceinline__ void mbar_inval(uint64_t* mbar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_addr(mbar)) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Wait for the phase with parity `parity` of `mbar` to complete; gives up after
// `max_polls` polls and returns false (the caller records a timeout status).
// Wait strategy: 2 (default) = try_wait with a 20 ns suspend-time hint (measured 3-6 %
// faster than 0 = plain try_wait and 1 = a test_wait spin on the tcgen05 kernels).
#ifndef VERACE_MBAR_WAIT
#define VERACE_MBAR_WAIT 2
#endif
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, uint32_t max_polls) {
  const uint32_t a = smem_addr(mbar);
  for (uint32_t it = 0; it < max_polls; ++it) {
    uint32_t done;
#if VERACE_MBAR_WAIT == 1
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
#elif VERACE_MBAR_WAIT == 2
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(20u)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
#endif
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async proxy
// (the tensor core reads operands through it).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMEM allocation: executed by one whole warp; the base address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Load 16 consecutive fp32 columns of this thread's TMEM lane.  A warp may only touch
// lanes [32*(warp%4), 32*(warp%4)+32); `taddr` must carry that lane base in bits 16+.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive fp32 columns of this thread's TMEM lane (same lane rule as
// tmem_ld16), then wait until the stores are done.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16-byte asynchronous global -> shared copy (zero-filled when !valid; `gmem` must still
// be a valid address).  Completion: cp_async_commit(), then cp_async_wait_all().
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// mbarrier arrive (count 1) and arrive-with-expected-transaction-bytes.
__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(mbar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(mbar)), "r"(bytes)
               : "memory");
}
// TMA tiled loads into this CTA's own shared memory: box at coordinates (x innermost),
// completion counted in bytes on `mbar`.
__device__ __forceinline__ void tma_load_2d(void* smem, const void* tmap, int x, int y, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(smem)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(mbar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem, const void* tmap, int x, int y, int z, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_addr(smem)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_addr(mbar))
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* smem, const void* tmap, int x, int y, int z, int w, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          smem_addr(smem)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(mbar))
      : "memory");
}
// L2 eviction-priority policies (for the cache-hinted copies below): evict_last for data
// that is read again soon (a scan's resident state), evict_first for data streamed once.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_load_2d_hint(void* smem, const void* tmap, int x, int y, uint64_t* mbar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(smem)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(mbar)), "l"(policy)
      : "memory");
}
// Prefetch a box of a tensor into L2 (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(tmap), "r"(x), "r"(y) : "memory");
}
// TMA tiled store shared -> global (bulk-group completion), and its group controls.
__device__ __forceinline__ void tma_store_2d(const void* tmap, int x, int y, const void* smem) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(tmap), "r"(x),
               "r"(y), "r"(smem_addr(smem))
               : "memory");
}
// TMA tiled reduce shared -> global: global += smem element-wise (fp32 add for an fp32 map).
__device__ __forceinline__ void tma_reduce_add_2d(const void* tmap, int x, int y, const void* smem) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(tmap),
               "r"(x), "r"(y), "r"(smem_addr(smem))
               : "memory");
}
__device__ __forceinline__ void tma_store_2d_hint(const void* tmap, int x, int y, const void* smem, uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;" ::"l"(
                   tmap), "r"(x), "r"(y), "r"(smem_addr(smem)), "l"(policy)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d_hint(const void* tmap, int x, int y, const void* smem,
                                                       uint64_t policy) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;" ::"l"(
          tmap), "r"(x), "r"(y), "r"(smem_addr(smem)), "l"(policy)
      : "memory");
}
// 16-byte global store with an L2 eviction-priority policy.
__device__ __forceinline__ void st_global_hint(void* gmem, uint4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(gmem), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w), "l"(policy)
               : "memory");
}
// Order this thread's completed bulk (async-proxy) global writes before later async-proxy reads.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N committed bulk groups still read their shared-memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until at most N committed bulk groups are still in flight (writes performed)
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Plain bulk copy global -> shared (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem, const void* gmem, uint32_t bytes, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem)),
      "l"(gmem), "r"(bytes), "r"(smem_addr(mbar))
      : "memory");
}
__device__ __forceinline__ void bulk_load_hint(void* smem, const void* gmem, uint32_t bytes, uint64_t* mbar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(smem)),
      "l"(gmem), "r"(bytes), "r"(smem_addr(mbar)), "l"(policy)
      : "memory");
}
// Named barrier over `count` threads (id 1..15; id 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// fp32 -> (hi, lo) bf16 pair with x ~= hi + lo (16 significant bits).
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

// Pack 8 floats into 16 bytes of bf16 hi and 16 bytes of bf16 lo.
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
  __nv_bfloat16 h[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) split_bf16(x[i], h[i], l[i]);
  hi = *reinterpret_cast<const uint4*>(h);
  lo = *reinterpret_cast<const uint4*>(l);
}

}  // namespace tc
}  // namespace verace
