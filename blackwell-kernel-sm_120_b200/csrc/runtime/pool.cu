// pool.cu -- slot gather / scatter for the NVFP4 state pool.
//
// The reference keeps one state per (layer, batch index) in a Python dict
// (src/ops/qwen35_gdn_patch.py:30-57, GDNStateCache).  Here a layer's states
// live in one pool of `num_slots` slots, each slot holding HV value-head tiles
// of D x D NVFP4 state plus one fp32 global scale per tile:
//   codes  [num_slots, HV, D, D/2]  u8
//   scales [num_slots, HV, D, D/16] u8
//   gscale [num_slots, HV]          f32
// Sequences address their slot through an int32 slot index; a negative index
// is padding (vLLM's PAD_SLOT_ID = -1).  The decode and prefill kernels fuse
// the slot lookup into their loads; these two kernels move whole slots between
// the pool and a dense [n, HV, ...] staging area (snapshots, prefix copies,
// continuous-batching compaction).  HBM-bound copies with 16-byte accesses.
#include <cstdint>

#include "../common.cuh"

namespace gdn {
namespace {

constexpr int kThreads = 256;

// Copies n slot records.  One CTA per (record i, 16 KiB chunk); kGather picks
// the direction.  Record = HV*D*D/2 code bytes, HV*D*D/16 scale bytes, HV gs.
template <bool kGather>
__global__ void __launch_bounds__(kThreads) pool_copy_kernel(const uint8_t* __restrict__ src_codes,
                                                             const uint8_t* __restrict__ src_scales,
                                                             const float* __restrict__ src_gs,
                                                             uint8_t* __restrict__ dst_codes,
                                                             uint8_t* __restrict__ dst_scales,
                                                             float* __restrict__ dst_gs,
                                                             const int32_t* __restrict__ slot_idx,
                                                             int64_t num_slots, int32_t HV, int64_t code_rec,
                                                             int64_t scale_rec, int32_t n, uint32_t* status) {
  const int i = blockIdx.y;
  if (i >= n) return;
  const int32_t slot = __ldg(slot_idx + i);
  const bool valid = slot >= 0 && slot < num_slots;
  // a slot past the pool is treated as padding and reported
  if (slot >= num_slots && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(status, kStatusBadSlot);
  if (!valid && !kGather) return;  // scatter: padding rows are skipped
  // Gather reads pool[slot] into dense[i]; scatter reads dense[i] into pool[slot].
  const int64_t src_rec = kGather ? (int64_t)slot : (int64_t)i;
  const int64_t dst_rec = kGather ? (int64_t)i : (int64_t)slot;
  const int64_t code_vecs = code_rec / 16, scale_vecs = scale_rec / 16;
  const int64_t total = code_vecs + scale_vecs;
  for (int64_t e = blockIdx.x * (int64_t)kThreads + threadIdx.x; e < total; e += (int64_t)gridDim.x * kThreads) {
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (e < code_vecs) {
      if (valid) val = __ldg(reinterpret_cast<const uint4*>(src_codes + src_rec * code_rec) + e);
      reinterpret_cast<uint4*>(dst_codes + dst_rec * code_rec)[e] = val;
    } else {
      const int64_t f = e - code_vecs;
      if (valid) val = __ldg(reinterpret_cast<const uint4*>(src_scales + src_rec * scale_rec) + f);
      reinterpret_cast<uint4*>(dst_scales + dst_rec * scale_rec)[f] = val;
    }
  }
  if (blockIdx.x == 0) {
    for (int h = threadIdx.x; h < HV; h += kThreads)
      dst_gs[dst_rec * HV + h] = valid ? src_gs[src_rec * HV + h] : 0.0f;
  }
}

int pool_copy(bool gather, const uint8_t* sc, const uint8_t* ss, const float* sg, uint8_t* dc, uint8_t* ds,
              float* dg, int64_t num_slots, int32_t HV, int32_t D, const int32_t* slot_idx, int32_t n,
              cudaStream_t stream) {
  if (!sc || !ss || !sg || !dc || !ds || !dg || !slot_idx || HV <= 0 || D <= 0 || n < 0 || num_slots < 0)
    return GDN_ERR_ARGS;
  if (D % 16) return GDN_ERR_UNSUPPORTED;
  if (!aligned16(sc) || !aligned16(ss) || !aligned16(dc) || !aligned16(ds)) return GDN_ERR_ALIGN;
  if (n == 0) return GDN_OK;
  uint32_t* status = device_status_ptr();
  if (!status) return GDN_ERR_CUDA;
  const int64_t code_rec = (int64_t)HV * D * D / 2;
  const int64_t scale_rec = (int64_t)HV * D * D / 16;
  const int64_t vecs = (code_rec + scale_rec) / 16;
  int64_t gx = (vecs + kThreads - 1) / kThreads;
  if (gx > 64) gx = 64;
  dim3 grid((unsigned)gx, (unsigned)n);
  if (gather)
    pool_copy_kernel<true><<<grid, kThreads, 0, stream>>>(sc, ss, sg, dc, ds, dg, slot_idx, num_slots, HV, code_rec,
                                                          scale_rec, n, status);
  else
    pool_copy_kernel<false><<<grid, kThreads, 0, stream>>>(sc, ss, sg, dc, ds, dg, slot_idx, num_slots, HV,
                                                           code_rec, scale_rec, n, status);
  return launch_status();
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_pool_gather(const uint8_t* pool_codes, const uint8_t* pool_scales, const float* pool_gscale,
                               int64_t num_slots, int32_t num_v_heads, int32_t head_dim, const int32_t* slot_idx,
                               int32_t n, uint8_t* dense_codes, uint8_t* dense_scales, float* dense_gscale,
                               cudaStream_t stream) {
  return gdn::pool_copy(true, pool_codes, pool_scales, pool_gscale, dense_codes, dense_scales, dense_gscale,
                        num_slots, num_v_heads, head_dim, slot_idx, n, stream);
}

extern "C" int gdn_pool_scatter(const uint8_t* dense_codes, const uint8_t* dense_scales, const float* dense_gscale,
                                int64_t num_slots, int32_t num_v_heads, int32_t head_dim, const int32_t* slot_idx,
                                int32_t n, uint8_t* pool_codes, uint8_t* pool_scales, float* pool_gscale,
                                cudaStream_t stream) {
  return gdn::pool_copy(false, dense_codes, dense_scales, dense_gscale, pool_codes, pool_scales, pool_gscale,
                        num_slots, num_v_heads, head_dim, slot_idx, n, stream);
}
