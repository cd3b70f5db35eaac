// Device helpers shared by the gfn_b200 kernels (sm_100a).
//
// Inline PTX for the Blackwell data-movement primitives the recurrence uses:
// mbarrier transaction barriers, 1-D bulk async copies (the untiled TMA
// engine, cp.async.bulk) global -> shared, thread-block-cluster barriers and
// distributed-shared-memory (DSMEM) stores into a peer CTA's shared memory.
// No multicast variant is used anywhere in this library.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#define GFN_DEV __device__ __forceinline__

// Device-side error word.  Kernels OR bits into it instead of trapping; the
// host reads it back with gfn_get_device_error().
__device__ int gfn_device_err;

// Bits: 1 = an mbarrier wait gave up (bulk copy never landed),
//       2 = a token id outside [0, vocab).
constexpr int kDevErrMbarTimeout = 1;
constexpr int kDevErrBadToken = 2;
constexpr int kDevErrF16Range = 4;

GFN_DEV void gfn_flag_error(int bits) { atomicOr(&gfn_device_err, bits); }

// Each translation unit of the library has its own copy of gfn_device_err
// (no relocatable device code); this reads (and optionally clears) the copy
// of the unit it is compiled into.
static inline cudaError_t gfn_unit_error_word(int* v, int reset, cudaStream_t s) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(v, gfn_device_err, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && reset && *v) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(gfn_device_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  return e;
}

GFN_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
GFN_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

GFN_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

GFN_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

GFN_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Bounded wait: gives up after ~2^22 polls (well over a second with the
// backoff), records GFN_DEVERR_MBAR_TIMEOUT and returns false.  The caller
// keeps executing the same barrier sequence so that no peer CTA is left
// waiting on it; the results of such a launch are garbage and the host
// reports the error.
GFN_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t sleep_ns = 32) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    // Back off at once: a warp spinning on a barrier must not take issue
    // slots from the compute warps sharing its scheduler.
    __nanosleep(sleep_ns);
  }
  gfn_flag_error(kDevErrMbarTimeout);
  return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned, bytes a multiple of 16.
GFN_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- cluster
GFN_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Full cluster barrier (all threads of all CTAs), release/acquire at
// cluster scope so DSMEM stores before it are visible after it.
GFN_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
GFN_DEV uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
  return out;
}

GFN_DEV void dsmem_st(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

GFN_DEV void dsmem_st2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}

// ---------------------------------------------------------------- math
// The reference's elementwise formulas, written in the same operation order
// as its PyTorch expressions so float32 rounding matches.
GFN_DEV float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }
GFN_DEV float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }
GFN_DEV float soft_clamp20(float g) { return 20.f * tanhf(g / 20.f); }
GFN_DEV float saturate100(float v) { return 100.f * tanhf(v / 100.f); }

GFN_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
