// gdn_decode.cu -- fused recurrent NVFP4 Gated DeltaNet decode step (sm_100a).
//
// Per (sequence, value head) tile -- a 128 x 128 NVFP4 state S[i][j] (i over
// d_k, j over d_v; 8192 B codes + 1024 B scales + one fp32 global scale gs)
// in the pool slot named by slot_idx:
//   alpha = exp(g), S_a = alpha S, u = S_a^T k, w = beta (v - u),
//   S' = S_a + k w^T, o = q_scale S'^T q = q_scale (S_a^T q + (k.q) w),
// then S' is requantised in place with a fresh global scale
// gs' = amax(S') / gden and the reference block quantiser
// (src/kernel/gdn_state_update_ref.cu:93-141) applied to y = S' / gs'.
// The reference has no counterpart of this step (its only update is
// S' = alpha S + beta k v^T, gdn_state_update_ref.cu:51-67); the recurrence is
// the gated delta rule (Yang, Kautz & Hatamizadeh, ICLR 2025).
//
// The decode and the rank-1 update run on the tensor cores.  With
// c = alpha gs and S_dq = e2m1 * block scale (so S = gs S_dq):
//   MMA1'   D1' = I * S_dq^T          block-scaled E2M1 MMA against an identity
//                                     (lane = column j; double-buffered)
//   SIMT    [u p] / c = D1' [k q]     each w thread reduces its own row of D1'
//   MMA1    D1  = S_dq * I            the tile again, lane = row i
//   MMA_r1  D1 += k (w / c)^T         tf32 rank-1 update, w / c split hi + lo
// so S' = c D1 and the requantiser reads y = D1 * (c / gs') straight from TMEM.
// The codes arrive by one 2-D TMA copy with 64-byte swizzle that both decode
// MMAs read in place.
//
// Warp roles (one CTA per SM, 14 warps):
//   warp 13     producer: walks the CTA's tiles, loads the per-tile scalars,
//               queues the TMA copies into a 6-stage ring, zeroes the outputs
//               of padding tiles;
//   warp 12     MMA: scale-factor permutation, the [k q] operand, every MMA
//               and commit; it issues tile n+1's MMA1' before waiting for
//               tile n's w;
//   warps 8-11  w: u, p -> w, o (stored) and the rank-1 operand;
//   warps 0-7   requantise D1 and store the tile.
// Every wait is bounded; a timeout in any role stops all of them.
#include <cstdint>
#include <mutex>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include "../common.cuh"
#include "../intrinsics/nvfp4_codec.cuh"
#include "../tcgen05.cuh"
#include "tile_requant.cuh"

namespace gdn {
namespace {

constexpr int kD = 128;
constexpr int kQWarps = 8;
constexpr int kWWarp0 = 8;
constexpr int kMmaWarp = 12;
constexpr int kProdWarp = 13;
constexpr int kThreads = 14 * 32;
constexpr int kStages = 6;
constexpr uint32_t kCodeBytes = kD * kD / 2;    // 8192
constexpr uint32_t kScaleBytes = kD * kD / 16;  // 1024
constexpr uint32_t kVecBytes = kD * 2;          // 256
constexpr uint32_t kStageTx = kCodeBytes + kScaleBytes + 3 * kVecBytes;
constexpr float kDropBelow = 1e-30f;            // alpha * gs below this: the decayed state is zero

// TMEM columns (512 allocated)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColD1 = 0;     // 128: D1 (lane i)
constexpr uint32_t kColD1t = 128;  // 2 x 128: D1' (lane j), double-buffered
constexpr uint32_t kColSF = 384;   // 3 x 8: the tile's scale factors (tile n uses n % 3: the
                                   // slot is rewritten only after tile n - 3's MMA1 is known complete)
constexpr uint32_t kColOne = 408;  // 8: unit scale factors of the identity

struct TileMeta {
  int64_t pt;       // slot * HV + h
  int32_t b, h;
  float c;          // alpha * gs (1 when the decayed state is dropped)
  float inv_c;
  float beta;
  int32_t drop;     // alpha * gs < kDropBelow: S_a = 0
  int32_t end;      // no more tiles
};

struct __align__(1024) Stage {
  uint8_t codes[kCodeBytes];  // 64-byte swizzled rows (TMA), read in place by MMA1' and MMA1
  uint8_t scales[kScaleBytes];
  __nv_bfloat16 q[kD];
  __nv_bfloat16 k[kD];
  __nv_bfloat16 v[kD];
  TileMeta meta;
};

struct InfoW {
  TileMeta m;
  float kq;
  int32_t stage;
};

struct __align__(1024) DecodeSmem {
  Stage st[kStages];
  uint8_t ident[kCodeBytes];  // identity, no-swizzle K-major: byte b of row r at (b % 16) + 16 r + 2048 (b / 16)
  uint8_t sf_one[kScaleBytes];
  uint8_t sfb[2][kScaleBytes];  // tcgen05.cp 32x128b layout, 2 K-steps
  float4 kq4[2][kD / 2];        // (k_i, k_i+1, q_i, q_i+1), even i
  uint8_t ak[2][kD * 8 * 4];    // [128][8] fp32 K-major: columns 0, 1 = k
  uint8_t bw[2][kD * 8 * 4];    // [128][8] fp32 K-major: columns 0, 1 = hi, lo of w / c
  InfoW iw[2];
  TileMeta iq;
  float amax[2][kQWarps];
  float inv_tab[256];
  uint64_t full[kStages], empty[kStages], bar_t[2], bar_w, bar_d, bar_q, bar_fin;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ int canon(int row, int byte) { return (byte & 15) + 16 * row + 2048 * (byte >> 4); }
// [rows][K] fp32 K-major, 16-byte K chunks 128 bytes apart, 8-row groups sbo apart.
__device__ __forceinline__ uint32_t kf32(int row, int k, uint32_t sbo) {
  return (row & 7) * 16 + (k & 3) * 4 + (row >> 3) * sbo + (k >> 2) * 128;
}
__device__ __forceinline__ uint64_t desc_codes(const uint8_t* codes, int kstep) {
  // K-major, 64-byte swizzle: 8-row groups 512 bytes apart, K step = 32 bytes (64 E2M1 values)
  return tc::smem_desc(codes + 32 * kstep, 16, 512) | (4ull << 61);
}

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

// Bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_suspend(bar, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ uint16_t f2bf_bits(float f) {
  const __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<const uint16_t*>(&b);
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_decode_kernel(const DecodeArgs a, const __grid_constant__ CUtensorMap tm_codes) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  volatile int* abort_flag = &sm.abort_flag;
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // the swizzled stages need 1024-byte alignment
    if (tid == 0) atomicOr(a.status, kStatusWaitTimeout);
    return;
  }

  // ---- once per CTA: tables, constant operands, barriers, TMEM ----
  if (tid < 256) sm.inv_tab[tid] = scale_inverse(scale_decode((uint32_t)tid, kMode));
  for (int e = tid; e < (int)kCodeBytes; e += kThreads) {
    const int r = e >> 6, byte = e & 63;
    uint8_t val = 0;
    if (2 * byte == r) val = 0x02;      // E2M1 1.0 in the low nibble (k = 2 byte)
    if (2 * byte + 1 == r) val = 0x20;  // ... or the high nibble (k = 2 byte + 1)
    sm.ident[canon(r, byte)] = val;
  }
  if (tid < 256) reinterpret_cast<uint32_t*>(sm.sf_one)[tid] = 0x38383838u;  // UE4M3 1.0
  for (int e = tid; e < 2 * kD * 8; e += kThreads) {
    reinterpret_cast<float*>(sm.ak)[e] = 0.0f;
    reinterpret_cast<float*>(sm.bw)[e] = 0.0f;
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) mbar_init(&sm.bar_t[b], 2);
    mbar_init(&sm.bar_w, 4);
    mbar_init(&sm.bar_d, 2);
    mbar_init(&sm.bar_q, kQWarps);
    mbar_init(&sm.bar_fin, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&sm.tmem_base, kTmemCols);
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t T = sm.tmem_base;

  if (warp == kProdWarp) {
    // =================================== producer ===================================
    if (lane == 0) {
      int64_t t = blockIdx.x;
      int32_t tb = (int32_t)(blockIdx.x / (uint32_t)a.HV), th = (int32_t)(blockIdx.x % (uint32_t)a.HV);
      const int32_t step_b = (int32_t)(gridDim.x / (uint32_t)a.HV), step_h = (int32_t)(gridDim.x % (uint32_t)a.HV);
      for (int n = 0;; ++n) {
        const int s = n % kStages;
        if (n >= kStages && !wait_bar(&sm.empty[s], (uint32_t)(((n / kStages) - 1) & 1), abort_flag)) break;
        Stage& st = sm.st[s];
        // next valid tile (padding tiles: zero output, flag out-of-range slots)
        int32_t slot = -1;
        int b = 0, h = 0;
        while (t < a.ntiles) {
          b = tb;
          h = th;
          slot = __ldg(a.slot_idx + b);
          t += gridDim.x;
          th += step_h;
          tb += step_b;
          if (th >= a.HV) { th -= a.HV; ++tb; }
          if (slot >= 0 && slot < a.num_slots) break;
          uint4* ob = reinterpret_cast<uint4*>(a.out + ((int64_t)b * a.HV + h) * kD);
#pragma unroll
          for (int e = 0; e < 16; ++e) ob[e] = make_uint4(0u, 0u, 0u, 0u);
          if (slot >= a.num_slots) atomicOr(a.status, kStatusBadSlot);
          slot = -1;
        }
        TileMeta& m = st.meta;
        if (slot < 0) {  // walk over: an end marker in this stage
          m.end = 1;
          mbar_arrive(&sm.full[s]);
          break;
        }
        const int64_t pt = (int64_t)slot * a.HV + h;
        const int hk = h / a.group;
        const float c = expf(__ldg(a.g + (int64_t)b * a.HV + h)) * __ldg(a.pool_gs + pt);
        m.pt = pt;
        m.b = b;
        m.h = h;
        m.drop = (c >= 0.0f && c < kDropBelow) ? 1 : 0;
        m.c = m.drop ? 1.0f : c;
        m.inv_c = 1.0f / m.c;
        m.beta = __ldg(a.beta + (int64_t)b * a.HV + h);
        m.end = 0;
        uint64_t* bar = &sm.full[s];
        mbar_arrive_expect_tx(bar, kStageTx);  // also publishes the metadata
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
            "[%4];" ::"r"(smem_u32(st.codes)),
            "l"(&tm_codes), "r"(0), "r"((int32_t)(pt * kD)), "r"(smem_u32(bar))
            : "memory");
        bulk_g2s(st.scales, a.pool_scales + pt * kScaleBytes, kScaleBytes, bar);
        bulk_g2s(st.q, a.q + b * a.q_stride + (int64_t)hk * kD, kVecBytes, bar);
        bulk_g2s(st.k, a.k + b * a.k_stride + (int64_t)hk * kD, kVecBytes, bar);
        bulk_g2s(st.v, a.v + b * a.v_stride + (int64_t)h * kD, kVecBytes, bar);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ===================================== MMA =====================================
    const uint32_t id_mx = tc::idesc_mxf4nvf4(128, 128);
    const uint32_t id_r1 = tc::idesc_tf32(128, 128);
    if (lane == 0)
      for (int kt = 0; kt < 2; ++kt) tc::cp_32x128b_warpx4(T + kColOne + 4 * kt, tc::smem_desc(sm.sf_one + 512 * kt, 0, 128));
    bool ok = true;
    // Tile n's operands (after its stage landed): scale factors, k/q for the w
    // warps, then MMA1' into D1'[n & 1].  Returns false at the end marker.
    auto front = [&](int n, bool& more) -> bool {
      const int s = n % kStages;
      if (!wait_bar(&sm.full[s], (uint32_t)((n / kStages) & 1), abort_flag)) return false;
      Stage& st = sm.st[s];
      more = !st.meta.end;
      if (!more) return true;
      uint32_t* sfw = reinterpret_cast<uint32_t*>(sm.sfb[n & 1]);
      const uint32_t* scw = reinterpret_cast<const uint32_t*>(st.scales);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int qd = lane + 32 * r;
        const int t = qd >> 7, m0 = (qd & 127) >> 2, m1 = qd & 3;
        sfw[t * 128 + m0 * 4 + m1] = scw[(32 * m1 + m0) * 2 + t];
      }
      float kq = 0.0f;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int i2 = lane + 32 * r;  // pair (2 i2, 2 i2 + 1)
        const __nv_bfloat162 k2 = reinterpret_cast<const __nv_bfloat162*>(st.k)[i2];
        const __nv_bfloat162 q2 = reinterpret_cast<const __nv_bfloat162*>(st.q)[i2];
        const float4 f = make_float4(__low2float(k2), __high2float(k2), __low2float(q2), __high2float(q2));
        sm.kq4[n & 1][i2] = f;
        kq = fmaf(f.x, f.z, fmaf(f.y, f.w, kq));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);
      // D1'[n & 1] was last read by the w warps for tile n - 2 (bar_w waited since)
      tc::fence_smem_to_async();
      __syncwarp();
      if (lane == 0) {
        InfoW& iw = sm.iw[n & 1];
        iw.m = st.meta;
        iw.kq = kq;
        iw.stage = s;
        const uint32_t sf = T + kColSF + 8 * (n % 3);
        for (int kt = 0; kt < 2; ++kt) tc::cp_32x128b_warpx4(sf + 4 * kt, tc::smem_desc(sm.sfb[n & 1] + 512 * kt, 0, 128));
        for (int kt = 0; kt < 2; ++kt)
          tc::mma_mxf4nvf4(T + kColD1t + 128 * (n & 1), tc::smem_desc(sm.ident + 4096 * kt, 2048, 128),
                           desc_codes(st.codes, kt), id_mx, T + kColOne + 4 * kt, sf + 4 * kt, kt > 0);
        mbar_arrive(&sm.bar_t[n & 1]);  // publishes iw, kq4
        tc::commit(&sm.bar_t[n & 1]);
      }
      __syncwarp();
      return true;
    };
    bool more = true;
    ok = front(0, more);
    int n = 0;
    for (; ok && more; ++n) {
      const int s = n % kStages;
      Stage& st = sm.st[s];
      // tile n + 1's decode goes ahead of tile n's update (D1'[(n + 1) & 1] is
      // free: the w warps finished tile n - 1, waited for in the last iteration)
      bool more_next = false;
      if (!front(n + 1, more_next)) { ok = false; break; }
      // MMA1(n) + MMA_r1(n) into D1 once w(n) is ready and the requantisers read D1 (tile n - 1)
      if (!wait_bar(&sm.bar_w, (uint32_t)(n & 1), abort_flag)) { ok = false; break; }
      if (n >= 1 && !wait_bar(&sm.bar_q, (uint32_t)((n - 1) & 1), abort_flag)) { ok = false; break; }
      tc::fence_after_sync();
      uint8_t* ak = sm.ak[n & 1];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = lane + 32 * r;
        const float kv = bf2f(st.k[i]);
        *reinterpret_cast<float*>(ak + kf32(i, 0, 256)) = kv;
        *reinterpret_cast<float*>(ak + kf32(i, 1, 256)) = kv;
      }
      tc::fence_smem_to_async();
      __syncwarp();
      if (lane == 0) {
        sm.iq = st.meta;
        const uint32_t sf = T + kColSF + 8 * (n % 3);
        if (!st.meta.drop)
          for (int kt = 0; kt < 2; ++kt)
            tc::mma_mxf4nvf4(T + kColD1, desc_codes(st.codes, kt), tc::smem_desc(sm.ident + 4096 * kt, 2048, 128),
                             id_mx, sf + 4 * kt, T + kColOne + 4 * kt, kt > 0);
        tc::mma_tf32_ss(T + kColD1, tc::smem_desc(ak, 128, 256), tc::smem_desc(sm.bw[n & 1], 128, 256), id_r1,
                        st.meta.drop ? 0u : 1u);
        mbar_arrive(&sm.bar_d);  // publishes iq
        tc::commit(&sm.bar_d);
        tc::commit(&sm.empty[s]);
      }
      __syncwarp();
      more = more_next;
    }
    // end: tell the w and requantiser warps (n = number of tiles)
    if (ok) {
      const int N = n;
      // w warps: an end marker in iw[N & 1] (they finished tile N - 2: bar_w(N - 1) seen)
      if (lane == 0) {
        sm.iw[N & 1].m.end = 1;
        mbar_arrive(&sm.bar_t[N & 1]);
        mbar_arrive(&sm.bar_t[N & 1]);
      }
      if (N >= 1) ok = wait_bar(&sm.bar_q, (uint32_t)((N - 1) & 1), abort_flag);
      if (ok && lane == 0) {
        sm.iq.end = 1;
        mbar_arrive(&sm.bar_d);
        mbar_arrive(&sm.bar_d);
      }
    }
    if (!ok) *abort_flag = 1;
    // every tcgen05 operation this warp issued has completed before TMEM is freed
    if (lane == 0) {
      tc::commit(&sm.bar_fin);
      mbar_wait_bounded(&sm.bar_fin, 0, kWaitTimeoutNs / 4);
    }
    __syncwarp();
  } else if (warp >= kWWarp0) {
    // ================================ w and outputs ================================
    const int j = 32 * (warp & 3) + lane;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    for (int n = 0;; ++n) {
      if (!wait_bar(&sm.bar_t[n & 1], (uint32_t)((n >> 1) & 1), abort_flag)) break;
      const InfoW iw = sm.iw[n & 1];
      if (iw.m.end) break;
      tc::fence_after_sync();
      // u / c, p / c = row j of D1' against k, q
      float2 su = make_float2(0.0f, 0.0f), sp = make_float2(0.0f, 0.0f);
      const float4* kq4 = sm.kq4[n & 1];
#pragma unroll
      for (int c32 = 0; c32 < 4; ++c32) {
        float2 x[16];
        tc::ld_32x32b_x32(T + lane_base + kColD1t + 128 * (n & 1) + 32 * c32, reinterpret_cast<float*>(x));
        tc::ld_wait();
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const float4 kq = kq4[16 * c32 + p];
          su = __ffma2_rn(x[p], make_float2(kq.x, kq.y), su);
          sp = __ffma2_rn(x[p], make_float2(kq.z, kq.w), sp);
        }
      }
      tc::fence_before_sync();
      const TileMeta& m = iw.m;
      const float c = m.drop ? 0.0f : m.c;
      const float u = su.x + su.y, p = sp.x + sp.y;
      const float vj = bf2f(sm.st[iw.stage].v[j]);
      const float wj = m.beta * (vj - c * u);
      const float o = a.q_scale * fmaf(iw.kq, wj, c * p);
      const float o1 = __shfl_down_sync(0xffffffffu, o, 1);
      if ((j & 1) == 0)
        reinterpret_cast<uint32_t*>(a.out + ((int64_t)m.b * a.HV + m.h) * kD)[j >> 1] =
            (uint32_t)f2bf_bits(o) | ((uint32_t)f2bf_bits(o1) << 16);
      const float wc = wj * m.inv_c;
      const float hi = __uint_as_float(__float_as_uint(wc) & 0xFFFFE000u);
      uint8_t* bw = sm.bw[n & 1];
      *reinterpret_cast<float*>(bw + kf32(j, 0, 256)) = hi;
      *reinterpret_cast<float*>(bw + kf32(j, 1, 256)) = wc - hi;
      tc::fence_smem_to_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.bar_w);
    }
  } else {
    // ================================ requantisation ================================
    const int quad = warp & 3, half = warp >> 2;
    const int row = 32 * quad + lane;  // TMEM lane = state row i
    const uint32_t lane_base = (uint32_t)(32 * quad) << 16;
    for (int n = 0;; ++n) {
      if (!wait_bar(&sm.bar_d, (uint32_t)(n & 1), abort_flag)) break;
      const TileMeta m = sm.iq;
      if (m.end) break;
      tc::fence_after_sync();
      float2 x[32];
      {
        const uint32_t ta = T + lane_base + kColD1 + 64 * half;
        tc::ld_32x32b_x32(ta, reinterpret_cast<float*>(x));
        tc::ld_32x32b_x32(ta + 32, reinterpret_cast<float*>(x) + 32);
        tc::ld_wait();
      }
      // D1 and iq are read: release them to the MMA warp
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.bar_q);
      // block abs-max: three-input max, NaN-propagating (a NaN block takes the exact path)
      float am[4];
      float tmax = 0.0f;
#pragma unroll
      for (int blk = 0; blk < 4; ++blk) {
        const float2* xb = x + 8 * blk;
        float m0, m1;
        asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(xb[0].x), "f"(xb[0].y), "f"(xb[1].x));
        asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(xb[1].y), "f"(xb[2].x), "f"(xb[2].y));
        asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[3].x), "f"(xb[3].y));
        asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(m1), "f"(xb[4].x), "f"(xb[4].y));
        asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[5].x), "f"(xb[5].y));
        asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(m1), "f"(xb[6].x), "f"(xb[6].y));
        asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[7].x), "f"(xb[7].y));
        float mb;
        asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(mb) : "f"(m0), "f"(m1), "f"(0.0f));
        am[blk] = mb;
        float ok_max = mb;
        if (isnan(mb)) {  // rare: the reference's amax ignores NaN
          ok_max = 0.0f;
#pragma unroll
          for (int p = 0; p < 8; ++p) ok_max = fmaxf(ok_max, fmaxf(fabsf(xb[p].x), fabsf(xb[p].y)));
        }
        tmax = fmaxf(tmax, ok_max);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      if (lane == 0) sm.amax[n & 1][warp] = tmax;
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight requantiser warps
      float amax = sm.amax[n & 1][0];
#pragma unroll
      for (int w = 1; w < kQWarps; ++w) amax = fmaxf(amax, sm.amax[n & 1][w]);
      // S' = c D1: gs' = amax(S') / gden; y = D1 (c / gs')
      const float amax_s = m.c * amax;
      const float gs_new = (amax_s > 0.0f) ? __fdiv_rn(amax_s, a.gden) : 1.0f;
      const float mult = __fmul_rn(m.c, __frcp_rn(gs_new));
      uint32_t words[8], scw;
      requant_half_row<kMode>(
          x, am, mult, sm.inv_tab, words, scw,
          a.debug_y ? a.debug_y + (((int64_t)m.b * a.HV + m.h) * kD + row) * kD + 64 * half : nullptr);
      uint4* dst = reinterpret_cast<uint4*>(a.pool_codes + m.pt * kCodeBytes + row * 64 + 32 * half);
      dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
      dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
      *reinterpret_cast<uint32_t*>(a.pool_scales + m.pt * kScaleBytes + row * 8 + 4 * half) = scw;
      if (tid == 0) a.pool_gs[m.pt] = gs_new;
    }
  }

  if (*abort_flag && tid == 0) atomicOr(a.status, kStatusWaitTimeout);
  // Every tcgen05 operation has completed (or was abandoned after a timeout);
  // release the tensor memory.
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(T, kTmemCols);
}

}  // namespace
}  // namespace gdn

using namespace gdn;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

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
  // The codes are addressed as rows of a 2-D tensor map (int32 row coordinate).
  if (a.ntiles > INT32_MAX || p->num_slots * (int64_t)p->num_v_heads * kD > INT32_MAX) return GDN_ERR_UNSUPPORTED;
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

  CUtensorMap tm;
  {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return GDN_ERR_CUDA;
    const int64_t rows = p->num_slots > 0 ? p->num_slots * (int64_t)p->num_v_heads * kD : kD;
    const cuuint64_t dims[2] = {64, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {64};
    const cuuint32_t box[2] = {64, kD};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p->pool_codes, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GDN_ERR_CUDA;
  }

  const int smem = (int)sizeof(DecodeSmem);
  const int64_t max_ctas = sm_count();
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
    gdn_decode_kernel<kScaleRef240><<<grid, kThreads, smem, stream>>>(a, tm);
  else
    gdn_decode_kernel<kScaleFn448><<<grid, kThreads, smem, stream>>>(a, tm);
  return launch_status();
}
