// peer_allreduce.cu -- the sum all-reduce that ends a tensor-parallel layer's
// out-projection, over NVLink peer memory, one process per GPU.
//
// The reference's layer ends in the out-projection (src/ops/qwen35_gdn_patch.py:
// 118-121); under tensor parallelism each rank holds a partial [B, hidden]
// product and the layer output is their sum.  At decode sizes (a few MiB) a
// library all-reduce is latency-bound; this one is a single kernel with two
// cross-GPU hand-offs.
//
// Each rank owns one peer buffer (cudaMalloc, exported with cudaIpcGetMemHandle
// and mapped by every other rank with cudaIpcOpenMemHandle):
//   [0, cap)         in   : this rank's summand (copied in by the kernel)
//   [cap, 2 cap)     red  : the reduced vector, written by the rank owning each slice
//   [2 cap, ...)     flags: uint32 [2 hand-offs][kMaxBlocks][kMaxRanks] arrival epochs,
//                           then uint32 [kMaxBlocks] this rank's per-CTA call counters
// A call with n ranks and `count` bf16 elements (count % (8 n) == 0) splits the
// vector into n slices; rank s reduces slice s (two-shot).  CTA b of every rank
// handles the same chunks (512 16-byte vectors each) of every slice, chunk c with
// c = b (mod grid), so CTA b only ever waits for CTA b of the other ranks:
//   1. copy this rank's summand into `in`; hand-off 0 to every rank;
//   2. once every rank's hand-off 0 has arrived: sum the n ranks' `in` over this
//      rank's slice in fp32 (rank order 0..n-1), round to bf16 once and store the
//      sum into every rank's `red`; hand-off 1 to every rank;
//   3. once every rank's hand-off 1 has arrived: copy `red` to the output.
// Each hand-off is a st.release.sys of the call's epoch into the receiver's flag
// after a CTA barrier; the receiver's ld.acquire.sys of it orders its later loads.
// The epoch is the CTA's call counter + 1, kept in device memory and advanced by
// the kernel, so the replays of a captured CUDA graph stay in step.  No rank
// writes `in` or `red` of a call before every rank has finished reading them
// in the previous call (each CTA's step 1 follows its own step 3, which waited
// for every rank's step 2).  Every wait gives up after timeout_ns, sets
// GDN_STATUS_WAIT_TIMEOUT and the CTA returns.
#include <cstdint>
#include <cstring>

#include <cuda_bf16.h>

#include "../common.cuh"

namespace gdn {
int sm_count();

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 160;
constexpr int kThreads = 512;          // one 16-byte vector per thread per chunk
constexpr int64_t kChunkVecs = kThreads;
constexpr int64_t kFlagBytes = (2 * kMaxBlocks * kMaxRanks + kMaxBlocks) * 4;
constexpr int64_t kFlagArea = 16384;
static_assert(kFlagBytes <= kFlagArea, "flag area");

struct ArArgs {
  uint8_t* base[kMaxRanks];  // every rank's peer buffer as mapped in this process
  int32_t rank, nranks;
  int64_t cap;               // bytes of `in` (and of `red`)
  const uint4* src;
  uint4* dst;
  int64_t slice_vecs;        // 16-byte vectors per slice
  uint64_t timeout_ns;
  uint32_t* status;
};

__device__ __forceinline__ uint32_t* flag_at(uint8_t* base, int64_t cap, int hand, int blk, int from) {
  return reinterpret_cast<uint32_t*>(base + 2 * cap) + (hand * kMaxBlocks + blk) * kMaxRanks + from;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Hand-off `hand` of epoch e from this CTA to CTA b of every rank, then wait
// (bounded) until CTA b of every rank has handed off to this one.  Uniform
// result over the CTA.
__device__ bool hand_off(const ArArgs& a, int hand, uint32_t e) {
  const int b = blockIdx.x, t = threadIdx.x;
  __syncthreads();  // every thread's stores of this step precede the releases below
  bool ok = true;
  if (t < a.nranks) {
    st_release_sys(flag_at(a.base[t], a.cap, hand, b, a.rank), e);
    const uint32_t* f = flag_at(a.base[a.rank], a.cap, hand, b, t);
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if (globaltimer_ns() - t0 > a.timeout_ns) {
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

__global__ void __launch_bounds__(kThreads) peer_allreduce_kernel(ArArgs a) {
  const int b = blockIdx.x, t = threadIdx.x;
  const int n = a.nranks;
  uint32_t* const counter = reinterpret_cast<uint32_t*>(a.base[a.rank] + 2 * a.cap) + 2 * kMaxBlocks * kMaxRanks + b;
  const uint32_t e = *counter + 1u;
  const int64_t chunks = (a.slice_vecs + kChunkVecs - 1) / kChunkVecs;
  uint4* const in_own = reinterpret_cast<uint4*>(a.base[a.rank]);
  const uint4* const red_own = reinterpret_cast<const uint4*>(a.base[a.rank] + a.cap);

  // 1. this rank's summand into its `in` (chunks of every slice)
  for (int s = 0; s < n; ++s)
    for (int64_t c = b; c < chunks; c += gridDim.x) {
      const int64_t v = c * kChunkVecs + t;
      if (v < a.slice_vecs) in_own[s * a.slice_vecs + v] = a.src[s * a.slice_vecs + v];  // src may be dst: no read-only path
    }
  if (!hand_off(a, 0, e)) {
    if (t == 0) atomicOr(a.status, kStatusWaitTimeout);
    return;
  }

  // 2. this rank's slice: sum of every rank's `in`, stored into every rank's `red`
  const int64_t off = (int64_t)a.rank * a.slice_vecs;
  for (int64_t c = b; c < chunks; c += gridDim.x) {
    const int64_t v = c * kChunkVecs + t;
    if (v >= a.slice_vecs) continue;
    uint4 x[kMaxRanks];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
      if (p < n) x[p] = __ldcg(reinterpret_cast<const uint4*>(a.base[p]) + off + v);
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) {
      if (p < n) {
        const uint32_t w[4] = {x[p].x, x[p].y, x[p].z, x[p].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[q]));
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
    }
    uint32_t packed[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      packed[q] = *reinterpret_cast<const uint32_t*>(&h);
    }
    const uint4 r = make_uint4(packed[0], packed[1], packed[2], packed[3]);
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
      if (p < n) reinterpret_cast<uint4*>(a.base[p] + a.cap)[off + v] = r;
  }
  if (!hand_off(a, 1, e)) {
    if (t == 0) atomicOr(a.status, kStatusWaitTimeout);
    return;
  }

  // 3. the reduced vector out (chunks of every slice)
  for (int s = 0; s < n; ++s)
    for (int64_t c = b; c < chunks; c += gridDim.x) {
      const int64_t v = c * kChunkVecs + t;
      if (v < a.slice_vecs) a.dst[s * a.slice_vecs + v] = __ldcg(red_own + s * a.slice_vecs + v);
    }
  if (t == 0) *counter = e;
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_peer_buffer_bytes(int64_t capacity_bytes, int64_t* total_bytes) {
  if (!total_bytes || capacity_bytes <= 0 || capacity_bytes % 16) return GDN_ERR_ARGS;
  *total_bytes = 2 * capacity_bytes + kFlagArea;
  return GDN_OK;
}

extern "C" int gdn_peer_buffer_create(int64_t capacity_bytes, void** base, void* ipc_handle) {
  int64_t total = 0;
  if (!base || !ipc_handle || gdn_peer_buffer_bytes(capacity_bytes, &total) != GDN_OK) return GDN_ERR_ARGS;
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)total) != cudaSuccess) return GDN_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, (size_t)total) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return GDN_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *base = p;
  return GDN_OK;
}

extern "C" int gdn_peer_buffer_open(const void* ipc_handle, void** base) {
  if (!ipc_handle || !base) return GDN_ERR_ARGS;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return GDN_ERR_CUDA;
  *base = p;
  return GDN_OK;
}

extern "C" int gdn_peer_buffer_close(void* base) {
  if (!base) return GDN_ERR_ARGS;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

extern "C" int gdn_peer_buffer_destroy(void* base) {
  if (!base) return GDN_ERR_ARGS;
  return cudaFree(base) == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

extern "C" int gdn_peer_allreduce_bf16(const gdn_peer_allreduce_params* p, cudaStream_t stream) {
  if (!p || !p->src || !p->dst || p->nranks < 1 || p->nranks > kMaxRanks || p->rank < 0 ||
      p->rank >= p->nranks || p->count <= 0 || p->capacity_bytes <= 0 || p->capacity_bytes % 16)
    return GDN_ERR_ARGS;
  if (p->count % (8 * (int64_t)p->nranks) || p->count * 2 > p->capacity_bytes) return GDN_ERR_ARGS;
  if ((reinterpret_cast<uintptr_t>(p->src) | reinterpret_cast<uintptr_t>(p->dst)) & 15) return GDN_ERR_ALIGN;
  ArArgs a{};
  for (int r = 0; r < p->nranks; ++r) {
    if (!p->bases[r] || (reinterpret_cast<uintptr_t>(p->bases[r]) & 15)) return GDN_ERR_ARGS;
    a.base[r] = static_cast<uint8_t*>(p->bases[r]);
  }
  a.rank = p->rank;
  a.nranks = p->nranks;
  a.cap = p->capacity_bytes;
  a.src = reinterpret_cast<const uint4*>(p->src);
  a.dst = reinterpret_cast<uint4*>(p->dst);
  a.slice_vecs = p->count / 8 / p->nranks;
  a.timeout_ns = p->timeout_ns ? p->timeout_ns : kWaitTimeoutNs;
  a.status = device_status_ptr();
  if (!a.status) return GDN_ERR_CUDA;
  const int64_t chunks = (a.slice_vecs + kChunkVecs - 1) / kChunkVecs;
  int grid = sm_count();
  if (grid > kMaxBlocks) grid = kMaxBlocks;
  if (grid > chunks) grid = (int)chunks;
  peer_allreduce_kernel<<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
