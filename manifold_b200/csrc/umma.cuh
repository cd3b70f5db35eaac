// Blackwell (sm_100a) tensor-core primitives, written as inline PTX:
// tiled TMA loads (cp.async.bulk.tensor, no multicast), tcgen05 tensor-memory
// allocation, tcgen05.mma (kind::f16, one CTA), tcgen05.commit onto an
// mbarrier and tcgen05.ld of the fp32 accumulator.
//
// Shared-memory operand tiles are K-major with the 128-byte swizzle that the
// TMA engine writes (CU_TENSOR_MAP_SWIZZLE_128B): row r of a tile starts at
// r * 128 bytes and its 16-byte units are XOR-permuted by (r & 7).  The UMMA
// matrix descriptor for that layout: start address >> 4, stride byte offset
// 1024 (one 8-row atom), descriptor version 1, layout type 2 (SWIZZLE_128B).
// Each tile base is 1024-byte aligned, so the K offset inside the 128-byte
// row is added to the start address directly.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace gfn {
namespace umma {

// ------------------------------------------------------------------ TMA
GFN_DEV void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

GFN_DEV void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

GFN_DEV void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

GFN_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Spin on an mbarrier phase without sleeping (the pipeline's producer and
// MMA threads sit on the critical path).  Bounded in wall-clock time: after
// `limit_ns` (default one second) it records GFN_DEVERR_MBAR_TIMEOUT and
// returns false; the caller then leaves its loop, so a broken pipeline ends
// the launch within about a second instead of hanging the GPU.
GFN_DEV bool mbar_wait_spin(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 1000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) break;
  }
  gfn_flag_error(kDevErrMbarTimeout);
  return false;
}

// The same with a short sleep between polls, for threads off the critical
// path (the epilogue warps waiting for an accumulator).
GFN_DEV bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 1000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
      __nanosleep(20);
    }
    if (global_ns() - t0 > limit_ns) break;
  }
  gfn_flag_error(kDevErrMbarTimeout);
  return false;
}

// Plain (count-1) arrive on an mbarrier of this CTA.
GFN_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ------------------------------------------------------------------ TMEM
// Allocates `ncols` (power of two >= 32) tensor-memory columns; the base
// address lands in *slot (shared memory).  Whole warp.
GFN_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

GFN_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

GFN_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// Programmatic dependent launch: launch_dependents lets the next kernel of the
// stream start its prologue on SMs this grid frees; wait blocks until the
// previous kernel of the stream has completed and its writes are visible.
// Both are no-ops for a kernel launched without the attribute.
GFN_DEV void gdc_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
GFN_DEV void gdc_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

GFN_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ------------------------------------------------------------------ MMA
// K-major, 128-byte-swizzled operand tile at shared address `saddr`.
GFN_DEV uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);        // start address
  d |= (uint64_t)1 << 16;                         // leading byte offset (unused for K-major SW128)
  d |= (uint64_t)(1024u >> 4) << 32;              // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                         // SWIZZLE_128B
  return d;
}

// K-major tile with a `swz`-byte swizzle (64 or 128): rows of `swz` bytes,
// 8-row atoms of 8 * swz bytes.
template <int SWZ>
GFN_DEV uint64_t desc_kmajor(uint32_t saddr) {
  static_assert(SWZ == 64 || SWZ == 128, "swizzle");
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)((8u * SWZ) >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(SWZ == 128 ? 2 : 4) << 61;
  return d;
}

// Instruction descriptor of kind::f16 with fp16 A and B (both K-major), fp32
// accumulator, shape M x N.
constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4)                          // D format: f32
         | (0u << 7) | (0u << 10)           // A, B format: f16
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// D[tmem] (+)= A[smem] . B[smem]^T, issued by one thread.
GFN_DEV void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma this thread issued so far has
// completed (and its shared-memory operands may be overwritten).
GFN_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 accumulator columns of this warp's 32 lanes (lane i of
// the warp reads TMEM lane (taddr >> 16) + i).  The load and its wait sit in
// one asm statement, so no use of the registers can be scheduled between them.
GFN_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive fp32 accumulator columns (see tmem_ld32).
GFN_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 8 consecutive fp32 accumulator columns (see tmem_ld32).
GFN_DEV void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

template <int N>
GFN_DEV void tmem_ld(uint32_t taddr, float (&v)[N]) {
  if constexpr (N == 8) tmem_ld8(taddr, v);
  else if constexpr (N == 16) tmem_ld16(taddr, v);
  else tmem_ld32(taddr, v);
}

GFN_DEV uint32_t elect_one_lane() { return (threadIdx.x & 31) == 0; }

}  // namespace umma
}  // namespace gfn
