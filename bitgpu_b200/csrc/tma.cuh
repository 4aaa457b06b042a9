// TMA (cp.async.bulk.tensor) + mbarrier helpers for sm_100a, with bounded waits.
//
// Every mbarrier wait in this library spins at most kSpinLimit polls; on expiry the kernel
// records BG_ETIMEOUT in a device flag (read by bg_device_status) and returns instead of
// hanging the GPU.  No multicast form of any bulk copy is used anywhere.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace bg {

constexpr uint32_t kSpinLimit = 1u << 20;  // far above any legitimate wait; a fault fails fast

// Per-translation-unit timeout flag (no relocatable device code): each .cu that includes this
// header exposes a host poll function that reads and clears its copy; bg_device_status polls all.
static __device__ int g_device_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity; false (and the device error flag set) after
// `limit` polls.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t *bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(&g_device_error, BG_ETIMEOUT);
  return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  return mbar_wait_limit(bar, parity, kSpinLimit);
}

// Whole-warp form: every lane polls, then the warp reconverges (__all_sync) before the
// .sync.aligned instructions that follow (ldmatrix, mma.sync, movmatrix, tcgen05.ld/st), and the
// timeout decision is the same on every lane.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity) {
  const bool ok = mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Host: encode a rank-4 tiled tensor map (driver entry point fetched through the runtime, so the
// library does not link libcuda).  dims/strides in elements/bytes as cuTensorMapEncodeTiled.
int make_tmap_4d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, const uint64_t dims[4],
                 const uint64_t strides_bytes[3], const uint32_t box[4], CUtensorMapSwizzle swz);

}  // namespace bg
