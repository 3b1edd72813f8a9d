// common.cuh -- sm_100a helpers shared by the GDN kernels: mbarriers, 1-D bulk
// (TMA) copies, bounded waits and the device status word.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "gdn_b200.h"

namespace gdn {

// Device status bits (gdn_b200_device_status reads them back).
constexpr uint32_t kStatusWaitTimeout = GDN_STATUS_WAIT_TIMEOUT;
constexpr uint32_t kStatusBadSlot = GDN_STATUS_BAD_SLOT;

// Address of the library's device status word on the current device.
// Resolved once per device with cudaGetSymbolAddress (runtime/status.cu).
uint32_t* device_status_ptr();

// Bounded waits give up after this long (ns of %globaltimer).
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

#ifdef __CUDACC__
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Makes initialised mbarriers visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the hardware may suspend the thread for up to
// `suspend_ns` while the phase is incomplete (it resumes when the phase
// completes), so a waiting thread issues few instructions.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete; false after
// `timeout_ns` without completion (the caller reports and leaves).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t timeout_ns = kWaitTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_suspend(bar, parity, 100000u)) return true;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  }
}

// CTA-wide bounded wait: thread 0 waits, the others are parked at the
// barrier (no instruction issue).  Uniform result; must be reached by every
// thread of the CTA.
__device__ __forceinline__ bool mbar_wait_cta(uint64_t* bar, uint32_t parity, uint64_t timeout_ns = kWaitTimeoutNs) {
  bool ok = true;
  if (threadIdx.x == 0) ok = mbar_wait_bounded(bar, parity, timeout_ns);
  return !__syncthreads_or(!ok);
}

// 1-D bulk copy global -> shared, completing `bytes` on the mbarrier.
// dst, src 16-byte aligned, bytes a multiple of 16; into this CTA only.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
#endif  // __CUDACC__

// Host-side helpers -------------------------------------------------------
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

// SM count of the current device (cached per device).
int sm_count();

// Byte strides between consecutive (slot, head) tiles of a state pool's
// codes, scales and global scales (128 x 128 tiles).  tile_stride 0: three
// dense arrays (8192, 1024 and 4 bytes per tile).  Otherwise the record
// layout, every array advancing by tile_stride: a multiple of 16 of at least
// 9220 bytes, with the three pointers 16-, 16- and 4-byte aligned.  False
// when the stride or the alignment is not usable.
inline bool pool_strides(int64_t tile_stride, const void* codes, const void* scales, const void* gscale,
                         int64_t* code_stride, int64_t* scale_stride, int64_t* gs_stride) {
  if (tile_stride == 0) {
    *code_stride = 8192;
    *scale_stride = 1024;
    *gs_stride = 4;
  } else {
    if (tile_stride < 9220 || tile_stride % 16) return false;
    *code_stride = *scale_stride = *gs_stride = tile_stride;
  }
  return aligned16(codes) && aligned16(scales) && (reinterpret_cast<uintptr_t>(gscale) & 3u) == 0;
}

// Raises `func`'s dynamic shared-memory limit to `bytes` on the current
// device, once per (kernel, device); safe to call from any host thread.
// Returns GDN_OK or GDN_ERR_CUDA.
int allow_dynamic_smem(const void* func, int bytes);

}  // namespace gdn
