// gdn_decode.cu -- fused recurrent NVFP4 Gated DeltaNet decode step (sm_100a).
//
// One CTA owns one (sequence, value head) state tile at a time: a 128 x 128
// NVFP4 tile (8192 B codes + 1024 B scales + 4 B global scale) in the slot of
// the state pool named by slot_idx.  Per tile:
//   alpha = exp(g), S_a = alpha * S, u = S_a^T k, w = beta (v - u),
//   S' = S_a + k w^T, o = q_scale * S'^T q = q_scale (S_a^T q + (k.q) w),
// then S' is requantised in place with a fresh global scale
// gs' = amax(S') / gden and the reference block quantiser
// (src/kernel/gdn_state_update_ref.cu:93-141) applied to y = S' * (1/gs').
// There is no counterpart of this step in the reference (its only update is
// S' = alpha S + beta k v^T, gdn_state_update_ref.cu:51-67); the recurrence is
// the gated delta rule (Yang, Kautz & Hatamizadeh, ICLR 2025).
//
// Structure (HBM-bound: 18,432 B of state read+written per tile):
//   * persistent grid of 2 CTAs per SM; each CTA walks tiles blockIdx.x,
//     blockIdx.x + gridDim.x, ...
//   * a 4-stage ring of 1-D bulk (TMA) copies keeps the next tiles' codes,
//     scales, q, k, v in flight into shared memory while the current tile is
//     computed; one mbarrier per stage, bounded waits;
//   * 256 threads; thread (warp w, lane l) owns the 16-column scale block
//     cb = l & 7 of rows 4w + (l >> 3) + 32m, m = 0..3 (64 elements in
//     registers), so block amax and requantisation stay inside the thread and
//     every code row is read and written as whole 8-byte pieces;
//   * u and S_a^T q are reduced with two warp-shuffle steps and one pass
//     through shared memory.  The shuffles carry no selects: lanes of the
//     upper half-warp accumulate the two products in swapped registers, and
//     lanes with (l >> 3) odd hold their two code words in swapped order;
//   * decode uses cvt.rn.f16x2.e2m1x2, encode cvt.rn.satfinite.e2m1x2.f32
//     (see intrinsics/nvfp4_codec.cuh for the exactness argument);
//   * new codes and scales are stored straight from registers (8-byte stores,
//     256 contiguous bytes per warp instruction).
#include <cstdint>
#include <cuda_bf16.h>

#include "../common.cuh"
#include "../intrinsics/nvfp4_codec.cuh"

namespace gdn {
namespace {

constexpr int kD = 128;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 4;
constexpr uint32_t kCodeBytes = kD * kD / 2;    // 8192
constexpr uint32_t kScaleBytes = kD * kD / 16;  // 1024
constexpr uint32_t kVecBytes = kD * 2;          // 256
constexpr uint32_t kStageTx = kCodeBytes + kScaleBytes + 3 * kVecBytes;

struct __align__(128) Stage {
  uint8_t codes[kCodeBytes];
  uint8_t scales[kScaleBytes];
  __nv_bfloat16 q[kD];
  __nv_bfloat16 k[kD];
  __nv_bfloat16 v[kD];
};

struct __align__(128) DecodeSmem {
  Stage st[kStages];
  float red[kWarps][2 * kD];  // per-warp partial u (0..127) and S_a^T q (128..255)
  float w[kD];
  float amax[kWarps];
  float dec_tab[256];
  uint64_t full[kStages];
};

struct DecodeArgs {
  int32_t B, HK, HV, group;
  int64_t num_slots, ntiles;
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_stride, k_stride, v_stride;
  const float* g;
  const float* beta;
  const int32_t* slot_idx;
  uint8_t* pool_codes;
  uint8_t* pool_scales;
  float* pool_gs;
  __nv_bfloat16* out;
  float q_scale, gden;
  float* debug_y;
  uint32_t* status;
};

// Thread 0: queue tile `tile` into stage `s`.
__device__ __forceinline__ void issue_tile(const DecodeArgs& a, DecodeSmem& sm, int s, int64_t tile) {
  const int b = (int)(tile / a.HV), h = (int)(tile % a.HV);
  const int32_t slot = __ldg(a.slot_idx + b);
  uint64_t* bar = &sm.full[s];
  if (slot < 0 || slot >= a.num_slots) {
    mbar_arrive(bar);  // nothing to load: complete the phase
    return;
  }
  const int hk = h / a.group;
  const int64_t pt = (int64_t)slot * a.HV + h;
  Stage& st = sm.st[s];
  mbar_arrive_expect_tx(bar, kStageTx);
  bulk_g2s(st.codes, a.pool_codes + pt * kCodeBytes, kCodeBytes, bar);
  bulk_g2s(st.scales, a.pool_scales + pt * kScaleBytes, kScaleBytes, bar);
  bulk_g2s(st.q, a.q + b * a.q_stride + (int64_t)hk * kD, kVecBytes, bar);
  bulk_g2s(st.k, a.k + b * a.k_stride + (int64_t)hk * kD, kVecBytes, bar);
  bulk_g2s(st.v, a.v + b * a.v_stride + (int64_t)h * kD, kVecBytes, bar);
}

__device__ __forceinline__ uint16_t f2bf_bits(float f) {
  const __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<const uint16_t*>(&b);
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 2) gdn_decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cb = lane & 7;     // column block: columns 16cb .. 16cb+15
  const int rq = lane >> 3;    // row within the warp's quad
  const int sh = rq & 1;       // this lane holds its two code words swapped
  const int skq = rq >> 1;     // this lane accumulates (q, k) instead of (k, q)

  sm.dec_tab[tid] = scale_decode((uint32_t)tid, kMode);
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const int64_t G = gridDim.x;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      const int64_t t = blockIdx.x + s * G;
      if (t < a.ntiles) issue_tile(a, sm, s, t);
    }
  }

  bool timed_out = false;
  int64_t n = 0;
  for (;; ++n) {
    const int64_t tile = blockIdx.x + n * G;
    if (tile >= a.ntiles) break;
    const int s = (int)(n % kStages);
    const uint32_t par = (uint32_t)((n / kStages) & 1);
    const bool ok = mbar_wait_bounded(&sm.full[s], par);
    if (__syncthreads_or(!ok)) { timed_out = true; break; }

    const int b = (int)(tile / a.HV), h = (int)(tile % a.HV);
    const int32_t slot = __ldg(a.slot_idx + b);
    __nv_bfloat16* ob = a.out + ((int64_t)b * a.HV + h) * kD;
    if (slot < 0 || slot >= a.num_slots) {
      if (tid < kD / 2) reinterpret_cast<uint32_t*>(ob)[tid] = 0u;
      if (tid == 0) {
        if (slot >= a.num_slots) atomicOr(a.status, kStatusBadSlot);
        const int64_t nt = blockIdx.x + (n + kStages) * G;
        if (nt < a.ntiles) issue_tile(a, sm, s, nt);
      }
      continue;
    }
    const int64_t pt = (int64_t)slot * a.HV + h;
    const Stage& st = sm.st[s];
    const float gs_old = __ldg(a.pool_gs + pt);
    const float alpha = expf(__ldg(a.g + (int64_t)b * a.HV + h));
    const float bt = __ldg(a.beta + (int64_t)b * a.HV + h);
    const float c = alpha * gs_old;  // S_a = e2m1 * scale * c

    // ---- decode + partial products over this thread's 4 rows ----
    float x[4][16];
    float kr[4];
    float A[16], Bq[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) { A[i] = 0.0f; Bq[i] = 0.0f; }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int r = 4 * warp + rq + 32 * m;
      const uint8_t* crow = st.codes + r * 64 + 8 * cb;
      const uint32_t w0 = *reinterpret_cast<const uint32_t*>(crow + 4 * sh);
      const uint32_t w1 = *reinterpret_cast<const uint32_t*>(crow + 4 * (sh ^ 1));
      const float sig = sm.dec_tab[st.scales[r * 8 + cb]] * c;
      uint32_t hh[4];
      cvt_e2m1x8_to_f16x2(w0, hh);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = f16x2_to_f32x2(hh[j]);
        x[m][2 * j] = f.x * sig;
        x[m][2 * j + 1] = f.y * sig;
      }
      cvt_e2m1x8_to_f16x2(w1, hh);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = f16x2_to_f32x2(hh[j]);
        x[m][8 + 2 * j] = f.x * sig;
        x[m][8 + 2 * j + 1] = f.y * sig;
      }
      kr[m] = bf2f(st.k[r]);
      const float qr = bf2f(st.q[r]);
      const float ka = skq ? qr : kr[m];
      const float kb = skq ? kr[m] : qr;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        A[i] = fmaf(x[m][i], ka, A[i]);
        Bq[i] = fmaf(x[m][i], kb, Bq[i]);
      }
    }
    // Step 1 (lanes l, l^16): keep A, add the partner's B.  Lanes with skq = 0
    // end with u partials, skq = 1 with S_a^T q partials.
#pragma unroll
    for (int i = 0; i < 16; ++i) A[i] += __shfl_xor_sync(0xffffffffu, Bq[i], 16);
    // Step 2 (lanes l, l^8): registers 0..7 hold this lane's own half of the
    // block's columns (swapped lanes hold columns 8..15 there).
#pragma unroll
    for (int i = 0; i < 8; ++i) A[i] += __shfl_xor_sync(0xffffffffu, A[i + 8], 8);
    {
      float4* dst = reinterpret_cast<float4*>(&sm.red[warp][skq * kD + 16 * cb + 8 * sh]);
      dst[0] = make_float4(A[0], A[1], A[2], A[3]);
      dst[1] = make_float4(A[4], A[5], A[6], A[7]);
    }
    // k.q for the readout (warps 0..3 need it), and v_t for column t.
    float kq = 0.0f, vt = 0.0f;
    if (warp < 4) {
#pragma unroll
      for (int i = 0; i < 4; ++i) kq = fmaf(bf2f(st.k[4 * lane + i]), bf2f(st.q[4 * lane + i]), kq);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);
      vt = bf2f(st.v[tid]);
    }
    __syncthreads();  // S1: stage s fully read, partials published
    if (tid == 0) {
      const int64_t nt = blockIdx.x + (n + kStages) * G;
      if (nt < a.ntiles) issue_tile(a, sm, s, nt);
    }
    if (tid < kD) {
      float u = 0.0f, p = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) { u += sm.red[w][tid]; p += sm.red[w][kD + tid]; }
      const float wj = bt * (vt - u);
      sm.w[tid] = wj;
      const float o0 = a.q_scale * fmaf(kq, wj, p);
      const float o1 = __shfl_down_sync(0xffffffffu, o0, 1);
      if ((tid & 1) == 0)
        reinterpret_cast<uint32_t*>(ob)[tid >> 1] = (uint32_t)f2bf_bits(o0) | ((uint32_t)f2bf_bits(o1) << 16);
    }
    __syncthreads();  // S2: w published

    // ---- rank-1 update, block and tile amax ----
    float wr[16];
    {
      const float4* w4a = reinterpret_cast<const float4*>(&sm.w[16 * cb + 8 * sh]);
      const float4* w4b = reinterpret_cast<const float4*>(&sm.w[16 * cb + 8 * (sh ^ 1)]);
      float4 t0 = w4a[0], t1 = w4a[1], t2 = w4b[0], t3 = w4b[1];
      wr[0] = t0.x; wr[1] = t0.y; wr[2] = t0.z; wr[3] = t0.w;
      wr[4] = t1.x; wr[5] = t1.y; wr[6] = t1.z; wr[7] = t1.w;
      wr[8] = t2.x; wr[9] = t2.y; wr[10] = t2.z; wr[11] = t2.w;
      wr[12] = t3.x; wr[13] = t3.y; wr[14] = t3.z; wr[15] = t3.w;
    }
    float am[4];
    float tmax = 0.0f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
#pragma unroll
      for (int i = 0; i < 16; ++i) x[m][i] = fmaf(kr[m], wr[i], x[m][i]);
      float mx = x[m][0];
#pragma unroll
      for (int i = 1; i < 16; ++i) mx = absmax_nan(mx, x[m][i]);
      am[m] = fabsf(mx);
      float ok_max = am[m];
      if (isnan(ok_max)) {  // rare: the reference's amax ignores NaN
        ok_max = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) ok_max = fmaxf(ok_max, fabsf(x[m][i]));
      }
      tmax = fmaxf(tmax, ok_max);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    if (lane == 0) sm.amax[warp] = tmax;
    __syncthreads();  // S3: tile amax
    float amax = sm.amax[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) amax = fmaxf(amax, sm.amax[w]);
    const float gs_new = (amax > 0.0f) ? __fdiv_rn(amax, a.gden) : 1.0f;
    const float inv_gs = __frcp_rn(gs_new);

    // ---- requantise and store ----
    uint8_t* pcodes = a.pool_codes + pt * kCodeBytes;
    uint8_t* pscales = a.pool_scales + pt * kScaleBytes;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int r = 4 * warp + rq + 32 * m;
      float y[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) y[i] = __fmul_rn(x[m][i], inv_gs);
      uint32_t w0, w1;
      const uint32_t sc = quantize16<false>(y, __fmul_rn(am[m], inv_gs), kMode, w0, w1);
      *reinterpret_cast<uint2*>(pcodes + r * 64 + 8 * cb) = sh ? make_uint2(w1, w0) : make_uint2(w0, w1);
      pscales[r * 8 + cb] = (uint8_t)sc;
      if (a.debug_y) {
        float* dy = a.debug_y + (((int64_t)b * a.HV + h) * kD + r) * kD + 16 * cb;
        float4* da = reinterpret_cast<float4*>(dy + 8 * sh);
        float4* db = reinterpret_cast<float4*>(dy + 8 * (sh ^ 1));
        da[0] = make_float4(y[0], y[1], y[2], y[3]);
        da[1] = make_float4(y[4], y[5], y[6], y[7]);
        db[0] = make_float4(y[8], y[9], y[10], y[11]);
        db[1] = make_float4(y[12], y[13], y[14], y[15]);
      }
    }
    if (tid == 0) a.pool_gs[pt] = gs_new;
  }

  if (timed_out) {
    // Report, then give the copies this CTA queued a bounded chance to land
    // before its shared memory is released.
    if (tid == 0) {
      atomicOr(a.status, kStatusWaitTimeout);
      for (int64_t m = n; m < n + kStages; ++m) {
        const int64_t t = blockIdx.x + m * G;
        if (t >= a.ntiles) break;
        mbar_wait_bounded(&sm.full[m % kStages], (uint32_t)((m / kStages) & 1), kWaitTimeoutNs / 4);
      }
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_decode(const gdn_decode_params* p, cudaStream_t stream) {
  if (!p) return GDN_ERR_ARGS;
  if (!p->q || !p->k || !p->v || !p->g || !p->beta || !p->slot_idx || !p->pool_codes || !p->pool_scales ||
      !p->pool_gscale || !p->out)
    return GDN_ERR_ARGS;
  if (p->batch < 0 || p->num_k_heads <= 0 || p->num_v_heads <= 0 || p->num_slots < 0) return GDN_ERR_ARGS;
  if (p->num_v_heads % p->num_k_heads) return GDN_ERR_ARGS;
  if (p->head_dim != kD) return GDN_ERR_UNSUPPORTED;
  if (p->scale_mode != kScaleRef240 && p->scale_mode != kScaleFn448) return GDN_ERR_UNSUPPORTED;
  if (p->batch == 0) return GDN_OK;
  DecodeArgs a;
  a.B = p->batch;
  a.HK = p->num_k_heads;
  a.HV = p->num_v_heads;
  a.group = p->num_v_heads / p->num_k_heads;
  a.num_slots = p->num_slots;
  a.ntiles = (int64_t)p->batch * p->num_v_heads;
  a.q = p->q;
  a.k = p->k;
  a.v = p->v;
  a.q_stride = p->q_stride ? p->q_stride : (int64_t)p->num_k_heads * kD;
  a.k_stride = p->k_stride ? p->k_stride : (int64_t)p->num_k_heads * kD;
  a.v_stride = p->v_stride ? p->v_stride : (int64_t)p->num_v_heads * kD;
  // Bulk copies need 16-byte aligned sources: bases aligned, strides multiples of 8 elements.
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(p->pool_codes) ||
      !aligned16(p->pool_scales) || !aligned16(p->out) || (a.q_stride | a.k_stride | a.v_stride) % 8 ||
      (p->debug_y && !aligned16(p->debug_y)))
    return GDN_ERR_ALIGN;
  a.g = p->g;
  a.beta = p->beta;
  a.slot_idx = p->slot_idx;
  a.pool_codes = p->pool_codes;
  a.pool_scales = p->pool_scales;
  a.pool_gs = p->pool_gscale;
  a.out = p->out;
  a.q_scale = p->q_scale > 0.0f ? p->q_scale : 0.08838834764831845f;  // 1/sqrt(128)
  a.gden = p->gscale_den > 0.0f ? p->gscale_den : default_gden(p->scale_mode);
  // The fast quantiser path skips its range test; that is exact while gden <= 1e6.
  if (!(a.gden >= 6.0f && a.gden <= 1.0e6f)) return GDN_ERR_ARGS;
  a.debug_y = p->debug_y;
  a.status = device_status_ptr();
  if (!a.status) return GDN_ERR_CUDA;

  const int smem = (int)sizeof(DecodeSmem);
  const int64_t max_ctas = (int64_t)sm_count() * 2;
  const int grid = (int)(a.ntiles < max_ctas ? a.ntiles : max_ctas);
  // Opt in to > 48 KB of dynamic shared memory once per device and kernel.
  static bool attr_set[2][64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GDN_ERR_CUDA;
  const int mi = p->scale_mode == kScaleRef240 ? 0 : 1;
  if (!attr_set[mi][dev]) {
    const cudaError_t e = mi == 0 ? cudaFuncSetAttribute(gdn_decode_kernel<kScaleRef240>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem)
                                  : cudaFuncSetAttribute(gdn_decode_kernel<kScaleFn448>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return GDN_ERR_CUDA;
    attr_set[mi][dev] = true;
  }
  if (mi == 0)
    gdn_decode_kernel<kScaleRef240><<<grid, kThreads, smem, stream>>>(a);
  else
    gdn_decode_kernel<kScaleFn448><<<grid, kThreads, smem, stream>>>(a);
  return launch_status();
}
