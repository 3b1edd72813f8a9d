// gdn_decode.cu -- fused recurrent NVFP4 Gated DeltaNet decode step (sm_100a).
//
// Per (sequence, value head) tile -- a 128 x 128 NVFP4 state S[i][j] (i over
// d_k, j over d_v; 8192 B codes + 1024 B scales + one fp32 global scale gs)
// in the pool slot named by slot_idx:
//   alpha = exp(g), S_a = alpha S, u = S_a^T k, w = beta (v - u),
//   S' = S_a + k w^T, o = q_scale S'^T q = q_scale (S_a^T q + (k.q) w),
// then S' is requantised in place with a fresh power-of-two-adjusted global
// scale and the reference block quantiser (src/kernel/gdn_state_update_ref.cu:93-141)
// applied to y = S' / gs'.
// The reference has no counterpart of this step (its only update is
// S' = alpha S + beta k v^T, gdn_state_update_ref.cu:51-67); the recurrence is
// the gated delta rule (Yang, Kautz & Hatamizadeh, ICLR 2025).
//
// The decode and the rank-1 update run on the tensor cores.  With
// S_dq = e2m1 * block scale (so S = gs S_dq), an identity of E2M1 0.5 at
// scale 2^-6 (so that the decoded tile is 2^-7 S_dq) and c = 2^7 alpha gs:
//   MMA1'   D1' = I * S_dq^T          block-scaled E2M1 MMA against the identity
//                                     (lane = column j)
//   SIMT    [u p] / c = D1' [k q]     each w thread reduces half a row of D1'
//   MMA1    D1  = S_dq * I            the tile again, lane = row i (double-buffered)
//   MMA_r1  D1 += k (w / c)^T         tf32 rank-1 update, w / c split hi + lo
// so S' = c D1.  The new global scale is gs' = c 2^-k with k >= 0 the
// largest integer for which max |D1| 2^k <= gden, and the quantiser input is
// y = D1 2^k.  Scaling by 2^k is exact, so each block's E2M1 codes follow from
// D1 and the block's own maximum alone (tile_requant.cuh); the identity's
// 2^-7 keeps max |D1| below gden, and so k >= 0, unless the rank-1 term is
// more than ~127x the decayed state (then an exact path runs).  The
// requantiser reads D1 straight from TMEM in two passes (block maxima, then
// codes) so that a thread never holds more than 32 values.  The codes arrive
// by one 2-D TMA copy with 64-byte swizzle that both decode MMAs read in
// place.
//
// Warp roles (one CTA per SM, 28 warps):
//   warp 25     producer: walks the CTA's tiles, loads the per-tile scalars
//               into a metadata ring, queues the TMA copies into an 8-stage
//               ring, zeroes the outputs of padding tiles;
//   warp 26     staging: once a stage lands, permutes its scale factors into
//               the tcgen05.cp layout and writes the fp32 k / q operands;
//   warp 24     MMA front: tile n's scale-factor copies and MMA1';
//   warp 27     MMA back: tile n's MMA1 and rank-1 update (the two issue in
//               parallel: a tcgen05 operation takes ~65-140 cycles to issue);
//   warps 0-23  three worker groups of 8 warps; group g takes the tiles
//               n = g (mod 3) and owns one 128-column TMEM buffer X_g, which
//               holds first D1'(n) (phase A: u, p -> w, o and the rank-1
//               operand) and then D1(n) (phase B: the requantiser).  Three
//               tiles are in flight, and no tile waits for another tile's
//               buffer to be read.
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
constexpr int kGroups = 3;        // worker groups of 8 warps: warps 0-23
constexpr int kMmaWarp = 24;      // issues the scale-factor copies and MMA1'
constexpr int kProdWarp = 25;
constexpr int kStageWarp = 26;
constexpr int kMmaBackWarp = 27;  // issues MMA1 and the rank-1 update
constexpr int kThreads = 28 * 32;
constexpr int kStages = 8;
constexpr int kRing = 16;  // metadata ring entries
constexpr uint32_t kCodeBytes = kD * kD / 2;    // 8192
constexpr uint32_t kScaleBytes = kD * kD / 16;  // 1024
constexpr uint32_t kVecBytes = kD * 2;          // 256
constexpr uint32_t kStageTx = kCodeBytes + kScaleBytes + 3 * kVecBytes;
constexpr float kDropBelow = 1e-30f;            // alpha * gs below this: the decayed state is zero
constexpr float kIdentInv = 128.0f;             // 1 / (the identity's value 0.5 x its scale 2^-6)
constexpr int kMaxShift = 100;                  // the fast requantiser path takes 0 <= k <= kMaxShift

// Named hardware barriers (0 is __syncthreads): group g uses kBarG0 + g
constexpr int kBarG0 = 1;

// TMEM columns (512 allocated)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColX = 0;      // 3 x 128: X_g, D1'(n) (lane j) then D1(n) (lane i) of group g's tile
constexpr uint32_t kColSF = 384;   // 4 x 8: the tile's scale factors (tile n uses n % 4: the
                                   // slot is rewritten only after tile n - 4's MMA1 is known complete)
constexpr uint32_t kColOne = 416;  // 8: the identity's scale factors (UE4M3 2^-6)
constexpr int kSfSlots = 4;

struct TileMeta {
  int64_t pt;       // slot * HV + h
  int32_t b, h;
  float c;          // 2^7 alpha gs, S' = c D1 (1 when the decayed state is dropped)
  float inv_c;
  float beta;
  float kq;         // k . q
  int32_t drop;     // alpha * gs < kDropBelow: S_a = 0
  int32_t end;      // no more tiles
};

struct __align__(1024) Stage {
  uint8_t codes[kCodeBytes];  // 64-byte swizzled rows (TMA), read in place by MMA1' and MMA1
  uint8_t scales[kScaleBytes];
  __nv_bfloat16 q[kD];
  __nv_bfloat16 k[kD];
  __nv_bfloat16 v[kD];
  uint8_t sfp[kScaleBytes];   // scale factors in the tcgen05.cp 32x128b layout, 2 K-steps
  float4 kq4[kD / 2];         // (k_i, k_i+1, q_i, q_i+1), even i
  uint8_t ak[kD * 8 * 4];     // [128][8] fp32 K-major: columns 0, 1 = k, the rest 0
  __nv_bfloat16 z[kD];        // the output gate (fused gated RMS norm only)
};

struct __align__(1024) DecodeSmem {
  Stage st[kStages];
  uint8_t ident[kCodeBytes];  // identity (E2M1 0.5), no-swizzle K-major: byte b of row r at (b % 16) + 16 r + 2048 (b / 16)
  uint8_t sf_one[kScaleBytes];  // the identity's scale factors, UE4M3 2^-6
  uint8_t bw[kGroups][kD * 8 * 4];  // per group, [128][8] fp32 K-major: columns 0, 1 = hi, lo of w / c
  float2 red[kGroups][kD];          // per group, partial [u p] / c of the second half of each row of D1'
  TileMeta ring[kRing];             // metadata of valid tile n at n % kRing
  uint32_t amax_bits[kGroups][2];   // per group, per tile parity: tile max |D1| as float bits
  float nrm[kGroups][4];            // fused norm: per group, per output warp, sum of x^2
  float inv_tab[256];
  uint32_t rtab[8];                 // scale_inv_w's reciprocal significands
  uint64_t full[kStages], ready[kStages], empty[kStages];
  // per group: bar_t D1' in X_g (MMA1' committed), bar_r D1' read, bar_w w formed, bar_d D1
  // in X_g (MMA1 and the rank-1 update committed), bar_x X_g free (D1 read)
  uint64_t bar_t[kGroups], bar_r[kGroups], bar_w[kGroups], bar_d[kGroups], bar_x[kGroups], bar_fin[2];
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
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier that also ORs `flag` over the participating threads: every
// thread gets the same answer, so a group leaves its loop together.
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, int flag) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.s32 q, %1, 0; bar.red.or.pred p, %2, %3, q; selp.u32 %0, 1, 0, p; }"
      : "=r"(r)
      : "r"(flag), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
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
  int64_t code_stride, scale_stride, gs_stride;  // bytes between consecutive (slot, head) tiles
  __nv_bfloat16* out;
  float q_scale, gden;
  float* debug_y;
  uint32_t* status;
  // fused prologue (A_log == nullptr: g and beta are read)
  const float* A_log;
  const float* dt_bias;
  const __nv_bfloat16* gate_a;
  const __nv_bfloat16* gate_b;
  int64_t gate_stride;
  int32_t qk_l2norm;
  // fused gated RMS norm of the output (norm_weight == nullptr: plain output)
  const float* norm_weight;
  const __nv_bfloat16* gate_z;
  int64_t z_stride;
  float norm_eps;
  int32_t norm_act;
};

// The global scale of pool tile pt (slot * HV + head).
__device__ __forceinline__ float* gs_at(const DecodeArgs& a, int64_t pt) {
  return reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.pool_gs) + pt * a.gs_stride);
}

// softplus(x) = log(1 + exp(x)), the identity above 20 (torch.nn.functional.softplus, beta 1).
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

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

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

static_assert(sizeof(Stage) == 16384, "a stage is 16 KB");

template <int kMode, bool kDebug, bool kNorm>
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
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (tid == i) sm.rtab[i] = scale_inv_w_entry(i);
  for (int e = tid; e < (int)kCodeBytes; e += kThreads) {
    const int r = e >> 6, byte = e & 63;
    uint8_t val = 0;
    if (2 * byte == r) val = 0x01;      // E2M1 0.5 in the low nibble (k = 2 byte)
    if (2 * byte + 1 == r) val = 0x10;  // ... or the high nibble (k = 2 byte + 1)
    sm.ident[canon(r, byte)] = val;
  }
  if (tid < 256) reinterpret_cast<uint32_t*>(sm.sf_one)[tid] = 0x08080808u;  // UE4M3 2^-6
  for (int e = tid; e < kGroups * kD * 8; e += kThreads) reinterpret_cast<float*>(sm.bw)[e] = 0.0f;
  for (int e = tid; e < kStages * kD * 8; e += kThreads)
    reinterpret_cast<float*>(sm.st[e / (kD * 8)].ak)[e % (kD * 8)] = 0.0f;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.ready[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int g = 0; g < kGroups; ++g) {
      mbar_init(&sm.bar_t[g], 2);   // the front warp's arrival + its commit
      mbar_init(&sm.bar_w[g], 4);   // the group's four output warps
      mbar_init(&sm.bar_d[g], 2);   // the back warp's arrival + its commit
      mbar_init(&sm.bar_x[g], 8);   // the group's eight warps
      mbar_init(&sm.bar_r[g], 8);   // likewise
      sm.amax_bits[g][0] = sm.amax_bits[g][1] = 0u;
    }
    mbar_init(&sm.bar_fin[0], 1);
    mbar_init(&sm.bar_fin[1], 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&sm.tmem_base, kTmemCols);
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t T = sm.tmem_base;
  // Launched as a programmatic dependent: the set-up above (shared and tensor
  // memory only) overlaps the previous kernel's tail; nothing in global memory
  // is read or written before every grid this one depends on has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The next launch in the stream may start its set-up as SMs free up.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == kProdWarp) {
    // =================================== producer ===================================
    // Lane l loads the scalars of tile t0 + l * gridDim.x for a batch of 32
    // tiles at a time; lane 0 queues the copies in tile order.  The next
    // batch's independent loads (slot, g and beta or the gate inputs) are in
    // flight while this batch is queued, and its dependent global-scale load
    // follows the queueing, so the first copy waits for one batch only.
    struct Scal {
      int64_t pt;
      int32_t b, h, slot;
      float c, beta;
      int32_t live;  // tile index < ntiles
    };
    struct Raw {
      int32_t b, h, slot, live;
      float x0, x1, x2, x3;  // g, beta; or gate a, gate b, A_log, dt_bias
    };
    auto issue_batch = [&](int64_t tb) -> Raw {
      Raw r{0, 0, -1, 0, 0.0f, 0.0f, 0.0f, 0.0f};
      const int64_t t = tb + (int64_t)lane * gridDim.x;
      if (t < a.ntiles) {
        r.live = 1;
        r.b = (int32_t)(t / a.HV);
        r.h = (int32_t)(t - (int64_t)r.b * a.HV);
        r.slot = __ldg(a.slot_idx + r.b);
        if (a.A_log) {
          const int64_t ai = (int64_t)r.b * a.gate_stride + r.h;
          r.x0 = __bfloat162float(a.gate_a[ai]);
          r.x1 = __bfloat162float(a.gate_b[ai]);
          r.x2 = __ldg(a.A_log + r.h);
          r.x3 = __ldg(a.dt_bias + r.h);
        } else {
          const int64_t gi = (int64_t)r.b * a.HV + r.h;
          r.x0 = __ldg(a.g + gi);
          r.x1 = __ldg(a.beta + gi);
        }
      }
      return r;
    };
    auto finish_batch = [&](const Raw& r) -> Scal {
      Scal q{0, r.b, r.h, r.slot, 0.0f, 0.0f, r.live};
      if (r.live && r.slot >= 0 && r.slot < a.num_slots) {
        q.pt = (int64_t)r.slot * a.HV + r.h;
        float gv, bv;
        if (a.A_log) {  // fused gating: g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
          gv = -expf(r.x2) * softplus_f(r.x0 + r.x3);
          bv = 1.0f / (1.0f + expf(-r.x1));
        } else {
          gv = r.x0;
          bv = r.x1;
        }
        q.c = expf(gv) * __ldg(gs_at(a, q.pt));
        q.beta = bv;
      }
      return q;
    };
    int64_t tb0 = blockIdx.x;
    const int64_t batch_step = 32ll * gridDim.x;
    Scal cur = finish_batch(issue_batch(tb0));
    int n = 0;
    bool done = false, ok = true;
    while (!done && ok) {
      const Raw nxt = issue_batch(tb0 + batch_step);
      for (int l = 0; l < 32; ++l) {
        const int live = __shfl_sync(0xffffffffu, cur.live, l);
        if (!live) { done = true; break; }
        const int32_t slot = __shfl_sync(0xffffffffu, cur.slot, l);
        const int32_t b = __shfl_sync(0xffffffffu, cur.b, l);
        const int32_t h = __shfl_sync(0xffffffffu, cur.h, l);
        if (slot < 0 || slot >= a.num_slots) {  // padding: zero output, flag out-of-range slots
          reinterpret_cast<uint2*>(a.out + ((int64_t)b * a.HV + h) * kD)[lane] = make_uint2(0u, 0u);
          if (lane == 0 && slot >= a.num_slots) atomicOr(a.status, kStatusBadSlot);
          continue;
        }
        const int64_t pt = __shfl_sync(0xffffffffu, cur.pt, l);
        const float c = __shfl_sync(0xffffffffu, cur.c, l);
        const float beta = __shfl_sync(0xffffffffu, cur.beta, l);
        const int s = n % kStages;
        if (lane == 0) {
          if (n >= kStages && !wait_bar(&sm.empty[s], (uint32_t)(((n / kStages) - 1) & 1), abort_flag)) ok = false;
          if (ok) {
            Stage& st = sm.st[s];
            TileMeta& m = sm.ring[n % kRing];
            m.pt = pt;
            m.b = b;
            m.h = h;
            m.drop = (c >= 0.0f && c < kDropBelow) ? 1 : 0;
            m.c = m.drop ? 1.0f : c * kIdentInv;
            m.inv_c = 1.0f / m.c;
            m.beta = beta;
            m.end = 0;
            const int hk = h / a.group;
            uint64_t* bar = &sm.full[s];
            mbar_arrive_expect_tx(bar, kStageTx + (kNorm && a.gate_z ? kVecBytes : 0u));  // also publishes the metadata
            asm volatile(
                "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
                "%3, %4}], [%5];" ::"r"(smem_u32(st.codes)),
                "l"(&tm_codes), "r"(0), "r"(0), "r"((int32_t)pt), "r"(smem_u32(bar))
                : "memory");
            bulk_g2s(st.scales, a.pool_scales + pt * a.scale_stride, kScaleBytes, bar);
            bulk_g2s(st.q, a.q + b * a.q_stride + (int64_t)hk * kD, kVecBytes, bar);
            bulk_g2s(st.k, a.k + b * a.k_stride + (int64_t)hk * kD, kVecBytes, bar);
            bulk_g2s(st.v, a.v + b * a.v_stride + (int64_t)h * kD, kVecBytes, bar);
            if (kNorm && a.gate_z) bulk_g2s(st.z, a.gate_z + b * a.z_stride + (int64_t)h * kD, kVecBytes, bar);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        ++n;
      }
      cur = finish_batch(nxt);
      tb0 += batch_step;
    }
    // walk over: an end marker in the ring
    if (ok && lane == 0) {
      const int s = n % kStages;
      if (n < kStages || wait_bar(&sm.empty[s], (uint32_t)(((n / kStages) - 1) & 1), abort_flag)) {
        sm.ring[n % kRing].end = 1;
        mbar_arrive(&sm.full[s]);
      }
    }
    __syncwarp();
  } else if (warp == kStageWarp) {
    // =================================== staging ===================================
    for (int n = 0;; ++n) {
      const int s = n % kStages;
      if (!wait_bar(&sm.full[s], (uint32_t)((n / kStages) & 1), abort_flag)) break;
      TileMeta& m = sm.ring[n % kRing];
      Stage& st = sm.st[s];
      if (!m.end) {
        uint32_t* sfw = reinterpret_cast<uint32_t*>(st.sfp);
        const uint32_t* scw = reinterpret_cast<const uint32_t*>(st.scales);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int qd = lane + 32 * r;
          const int t = qd >> 7, m0 = (qd & 127) >> 2, m1 = qd & 3;
          sfw[t * 128 + m0 * 4 + m1] = scw[(32 * m1 + m0) * 2 + t];
        }
        float kq = 0.0f;
        // optional unit-L2 scaling of k and q (fp32), x / sqrt(sum x^2 + 1e-6)
        float sk = 1.0f, sq = 1.0f;
        if (a.qk_l2norm) {
          float nk = 0.0f, nq = 0.0f;
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int i2 = lane + 32 * r;
            const float2 k2 = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(st.k)[i2]);
            const float2 q2 = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(st.q)[i2]);
            nk = fmaf(k2.x, k2.x, fmaf(k2.y, k2.y, nk));
            nq = fmaf(q2.x, q2.x, fmaf(q2.y, q2.y, nq));
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            nk += __shfl_xor_sync(0xffffffffu, nk, o);
            nq += __shfl_xor_sync(0xffffffffu, nq, o);
          }
          sk = 1.0f / sqrtf(nk + 1e-6f);
          sq = 1.0f / sqrtf(nq + 1e-6f);
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int i2 = lane + 32 * r;  // pair (2 i2, 2 i2 + 1)
          const __nv_bfloat162 k2 = reinterpret_cast<const __nv_bfloat162*>(st.k)[i2];
          const __nv_bfloat162 q2 = reinterpret_cast<const __nv_bfloat162*>(st.q)[i2];
          const float4 f = make_float4(__low2float(k2) * sk, __high2float(k2) * sk, __low2float(q2) * sq,
                                       __high2float(q2) * sq);
          st.kq4[i2] = f;
          kq = fmaf(f.x, f.z, fmaf(f.y, f.w, kq));
          *reinterpret_cast<float2*>(st.ak + kf32(2 * i2, 0, 256)) = make_float2(f.x, f.x);
          *reinterpret_cast<float2*>(st.ak + kf32(2 * i2 + 1, 0, 256)) = make_float2(f.y, f.y);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);
        if (lane == 0) m.kq = kq;
        tc::fence_smem_to_async();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.ready[s]);  // publishes sfp, kq4, ak and m.kq
      if (m.end) break;
    }
  } else if (warp == kMmaWarp || warp == kMmaBackWarp) {
    // ===================================== MMA =====================================
    // Two issuing warps, since one tcgen05 operation takes ~65-150 cycles to
    // issue: the front warp copies tile n's scale factors to TMEM and decodes
    // D1' = I S_dq^T into the buffer X_g of tile n's group g = n % 3; the back
    // warp decodes D1 = S_dq I into the same buffer and adds the rank-1 update
    // once the group has formed w.  Operations of different threads are not
    // ordered with each other, so each side waits for what the other issued
    // through barriers it already shares with the other roles:
    //   * the back warp's MMA1(n) reads scale-factor slot n % 4 and overwrites
    //     D1'(n) after the group arrived on bar_w(n), which it does after
    //     bar_t(n), the commit of the front warp's copies and MMA1'(n), and
    //     after every warp of the group loaded D1'(n);
    //   * the front warp rewrites slot n % 4 for tile n + 4 after empty(n),
    //     the back warp's commit of tile n's last MMA (a stage's empty barrier
    //     completes once per use, so its phase cannot run ahead), and writes
    //     D1'(n) into X_g after bar_x(n - 3), the group's last load of
    //     D1(n - 3).
    // Every shared-memory descriptor, TMEM address and mbarrier address is
    // formed once here: a stage's descriptors are the first stage's plus the
    // stage offset (the start-address field holds address >> 4).
    const bool front_warp = warp == kMmaWarp;
    const uint32_t id_mx = tc::idesc_mxf4nvf4(128, 128);
    const uint32_t id_r1 = tc::idesc_tf32(128, 128);
    constexpr uint32_t kStageDesc = sizeof(Stage) >> 4;
    constexpr uint32_t kBwDesc = sizeof(sm.bw[0]) >> 4;
    const uint64_t d_ident0 = tc::smem_desc(sm.ident, 2048, 128);
    const uint64_t d_ident1 = tc::smem_desc(sm.ident + 4096, 2048, 128);
    const uint64_t d_codes = desc_codes(sm.st[0].codes, 0);  // + 2: the second K step (32 bytes)
    const uint64_t d_sfp = tc::smem_desc(sm.st[0].sfp, 0, 128);  // + 32: the second K step (512 bytes)
    const uint64_t d_ak = tc::smem_desc(sm.st[0].ak, 128, 256);
    const uint64_t d_bw = tc::smem_desc(sm.bw[0], 128, 256);  // + g kBwDesc: group g's
    const uint32_t t_one = T + kColOne;
    const uint32_t b_t0 = smem_u32(&sm.bar_t[0]), b_d0 = smem_u32(&sm.bar_d[0]), b_empty0 = smem_u32(&sm.empty[0]);
    if (front_warp && lane == 0)
      for (int kt = 0; kt < 2; ++kt) tc::cp_32x128b_warpx4(t_one + 4 * kt, tc::smem_desc(sm.sf_one + 512 * kt, 0, 128));
    bool ok = true;
    int n = 0;
    if (front_warp) {
      // Tile t's scale factors are copied as soon as its stage is staged and
      // slot t % 4 is free, ahead of MMA1'(t), which may wait for its buffer.
      auto copy_sf = [&](int t) -> int {  // 1: copied, 0: t is the end marker, -1: gave up
        const uint32_t st_i = (uint32_t)t & (kStages - 1);
        if (!wait_bar(&sm.ready[st_i], (uint32_t)((t / kStages) & 1), abort_flag)) return -1;
        if (sm.ring[t & (kRing - 1)].end) return 0;
        // slot t % 4 was last read by tile t - 4's MMA1
        if (t >= kSfSlots && !wait_bar(&sm.empty[(t - kSfSlots) & (kStages - 1)],
                                       (uint32_t)(((t - kSfSlots) / kStages) & 1), abort_flag))
          return -1;
        tc::fence_after_sync();
        if (lane == 0) {
          const uint64_t so = st_i * kStageDesc;
          const uint32_t sf = T + kColSF + 8 * (uint32_t)(t & (kSfSlots - 1));
          tc::cp_32x128b_warpx4(sf, d_sfp + so);
          tc::cp_32x128b_warpx4(sf + 4, d_sfp + so + 32);
        }
        __syncwarp();
        return 1;
      };
      int r = copy_sf(0);
      for (; r == 1; ++n) {
        const int g = n % kGroups;
        // X_g is free once the group has loaded tile n - 3's D1
        if (n >= kGroups && !wait_bar(&sm.bar_x[g], (uint32_t)(((n - kGroups) / kGroups) & 1), abort_flag)) {
          r = -1;
          break;
        }
        tc::fence_after_sync();
        if (lane == 0) {
          const uint64_t so = ((uint32_t)n & (kStages - 1)) * kStageDesc;
          const uint32_t sf = T + kColSF + 8 * (uint32_t)(n & (kSfSlots - 1));
          const uint32_t x = T + kColX + 128 * (uint32_t)g;
          tc::mma_mxf4nvf4_c<false>(x, d_ident0, d_codes + so, id_mx, t_one, sf);
          tc::mma_mxf4nvf4_c<true>(x, d_ident1, d_codes + so + 2, id_mx, t_one + 4, sf + 4);
          mbar_arrive(&sm.bar_t[g]);  // publishes the ring entry to the group
          tc::commit_at(b_t0 + 8 * g);
        }
        __syncwarp();
        r = copy_sf(n + 1);  // on 0 the loop's increment leaves n at the end marker
      }
      if (r < 0) {
        ok = false;
      } else if (r == 0) {
        // Release every group into an end marker (tiles n, n + 1, n + 2; the
        // producer wrote ring[n]).  The two arrivals for tile e may complete
        // bar_t's next phase only after the group has waited on the phase of
        // its previous tile e - 3 (else both phases would be complete when it
        // looks, and its parity wait would miss them): wait until the group has
        // finished tile e - 3 (bar_x).  Ring entries n + 1 and n + 2 held tiles
        // n - 15 and n - 14, which every role has finished with.
        for (int e = n; ok && e < n + kGroups; ++e) {
          const int g = e % kGroups;
          if (e >= kGroups && !wait_bar(&sm.bar_x[g], (uint32_t)(((e - kGroups) / kGroups) & 1), abort_flag)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            if (e > n) sm.ring[e & (kRing - 1)].end = 1;
            mbar_arrive(&sm.bar_t[g]);
            mbar_arrive(&sm.bar_t[g]);
          }
          __syncwarp();
        }
      }
    } else {
      for (;; ++n) {
        const uint32_t s = (uint32_t)n & (kStages - 1);
        const int g = n % kGroups;
        if (!wait_bar(&sm.ready[s], (uint32_t)((n / kStages) & 1), abort_flag)) { ok = false; break; }
        if (sm.ring[n & (kRing - 1)].end) break;
        const uint64_t so = s * kStageDesc;
        const int drop = sm.ring[n & (kRing - 1)].drop;
        const uint32_t sf = T + kColSF + 8 * (uint32_t)(n & (kSfSlots - 1));
        const uint32_t d = T + kColX + 128 * (uint32_t)g;
        // MMA1(n) into X_g once every warp of the group has read D1'(n), which
        // is early in its phase A: the decode overlaps the dot products
        if (!wait_bar(&sm.bar_r[g], (uint32_t)((n / kGroups) & 1), abort_flag)) { ok = false; break; }
        tc::fence_after_sync();
        if (lane == 0 && !drop) {
          tc::mma_mxf4nvf4_c<false>(d, d_codes + so, d_ident0, id_mx, sf, t_one);
          tc::mma_mxf4nvf4_c<true>(d, d_codes + so + 2, d_ident1, id_mx, sf + 4, t_one + 4);
        }
        __syncwarp();
        // MMA_r1(n) once the group has formed w(n)
        if (!wait_bar(&sm.bar_w[g], (uint32_t)((n / kGroups) & 1), abort_flag)) { ok = false; break; }
        tc::fence_after_sync();
        if (lane == 0) {
          tc::mma_tf32_ss(d, d_ak + so, d_bw + (uint64_t)g * kBwDesc, id_r1, drop ? 0u : 1u);
          mbar_arrive(&sm.bar_d[g]);  // publishes the ring entry to the group's requantiser phase
          tc::commit_at(b_d0 + 8 * g);
          tc::commit_at(b_empty0 + 8 * s);
        }
        __syncwarp();
      }
    }
    if (!ok) *abort_flag = 1;
    // every tcgen05 operation this warp issued has completed before TMEM is freed
    if (lane == 0) {
      uint64_t* fin = &sm.bar_fin[front_warp ? 0 : 1];
      tc::commit(fin);
      mbar_wait_bounded(fin, 0, kWaitTimeoutNs / 4);
    }
    __syncwarp();
  } else {
    // ================================ worker groups ================================
    // Group g = warp / 8 takes the tiles n = g (mod 3).  Its warp w (0-7) reads
    // lane quadrant w % 4 and column half w / 4 of X_g, so `row` is j (over
    // d_v) in phase A, where X_g holds D1', and i (over d_k) in phase B, where
    // it holds D1.
    const int grp = warp >> 3;
    const int quad = warp & 3, half = (warp >> 2) & 1;
    const int row = 32 * quad + lane;
    const uint32_t lane_base = (uint32_t)(32 * quad) << 16;
    const uint32_t ta = T + lane_base + kColX + 128 * grp + 64 * half;
    const int bar_id = kBarG0 + grp;
    const int lead = 256 * grp;                   // the group's first thread
    const uint32_t gden_bits = __float_as_uint(a.gden);
    constexpr uint32_t kSat = kMode ? 0x7Eu : 0x77u;
    const float norm_wj = kNorm ? __ldg(a.norm_weight + row) : 0.0f;
    uint8_t* const bw = sm.bw[grp];
    for (int l = 0;; ++l) {
      const int n = kGroups * l + grp;
      // ------------- phase A: [u p] / c = D1' [k q], then w, o and the rank-1 operand -------------
      // one thread waits; the others sleep on the group's hardware barrier
      if (tid == lead) wait_bar(&sm.bar_t[grp], (uint32_t)(l & 1), abort_flag);
      if (named_bar_or(bar_id, 256, *abort_flag)) break;
      const TileMeta m = sm.ring[n % kRing];
      if (m.end) break;
      // fused norm: this thread's bf16 output and gate, normed after phase B's
      // first barrier (where every output warp's sum of x^2 is visible)
      float pend_x = 0.0f, pend_z = 0.0f;
      {
        const Stage& st = sm.st[n % kStages];
        tc::fence_after_sync();
        // this warp's half (64 columns i) of row j of D1', 32 at a time
        float2 su0 = make_float2(0.0f, 0.0f), sp0 = su0, su1 = su0, sp1 = su0;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          float2 x[16];
          tc::ld_32x32b_x32(ta + 32 * h2, reinterpret_cast<float*>(x));
          tc::ld_wait();
          if (h2 == 1) {
            // D1' is read: the back warp may decode D1 into X_g
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.bar_r[grp]);
          }
          const float4* kq4 = st.kq4 + 32 * half + 16 * h2;
#pragma unroll
          for (int p = 0; p < 16; p += 2) {
            const float4 ka = kq4[p], kb = kq4[p + 1];
            su0 = __ffma2_rn(x[p], make_float2(ka.x, ka.y), su0);
            sp0 = __ffma2_rn(x[p], make_float2(ka.z, ka.w), sp0);
            su1 = __ffma2_rn(x[p + 1], make_float2(kb.x, kb.y), su1);
            sp1 = __ffma2_rn(x[p + 1], make_float2(kb.z, kb.w), sp1);
          }
        }
        const float2 su = __fadd2_rn(su0, su1), sp = __fadd2_rn(sp0, sp1);
        if (half) sm.red[grp][row] = make_float2(su.x + su.y, sp.x + sp.y);
        named_bar(bar_id, 256);
        // bw[grp] is free: its last reader, tile n - 3's rank-1 MMA, completed
        // before the group's bar_d wait of that tile
        if (!half) {
          const int j = row;
          const float2 r = sm.red[grp][j];
          const float c = m.drop ? 0.0f : m.c;
          const float u = su.x + su.y + r.x, p = sp.x + sp.y + r.y;
          const float vj = bf2f(st.v[j]);
          const float wj = m.beta * (vj - c * u);
          // the stage may be refilled once w is published: the output gate is read first
          if (kNorm) pend_z = a.gate_z ? bf2f(st.z[j]) : 0.0f;
          // the rank-1 operand first (the back warp's MMA waits for it), the output after
          const float wc = wj * m.inv_c;
          const float hi = __uint_as_float(__float_as_uint(wc) & 0xFFFFE000u);
          *reinterpret_cast<float*>(bw + kf32(j, 0, 256)) = hi;
          *reinterpret_cast<float*>(bw + kf32(j, 1, 256)) = wc - hi;
          tc::fence_smem_to_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.bar_w[grp]);
          const float o = a.q_scale * fmaf(m.kq, wj, c * p);
          if (kNorm) {
            // gated RMS norm over the head: x = the bf16 output; this warp's sum of x^2 now
            pend_x = __bfloat162float(__float2bfloat16_rn(o));
            float sq = pend_x * pend_x;
#pragma unroll
            for (int s5 = 16; s5 > 0; s5 >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, s5);
            if (lane == 0) sm.nrm[grp][quad] = sq;
          } else {
            const float o1 = __shfl_down_sync(0xffffffffu, o, 1);
            if ((j & 1) == 0)
              reinterpret_cast<uint32_t*>(a.out + ((int64_t)m.b * a.HV + m.h) * kD)[j >> 1] =
                  pack_bf16x2(o, o1);  // one paired conversion (faster than two single ones)
          }
        }
      }
      // ---------------------------- phase B: requantise D1 ----------------------------
      if (tid == lead) wait_bar(&sm.bar_d[grp], (uint32_t)(l & 1), abort_flag);
      if (named_bar_or(bar_id, 256, *abort_flag)) break;
      if (kNorm && !half) {
        // x * rsqrt(mean(x^2) + eps) * weight * act(z), vLLM's RMSNormGated (norm before gate)
        const float* nr = sm.nrm[grp];
        const float rs = rsqrtf(((nr[0] + nr[1]) + (nr[2] + nr[3])) * (1.0f / kD) + a.norm_eps);
        float y = (pend_x * rs) * norm_wj;
        if (a.gate_z) {
          const float sg = 1.0f / (1.0f + expf(-pend_z));
          y = y * (a.norm_act ? sg : pend_z * sg);
        }
        const float y1 = __shfl_down_sync(0xffffffffu, y, 1);
        if ((row & 1) == 0)
          reinterpret_cast<uint32_t*>(a.out + ((int64_t)m.b * a.HV + m.h) * kD)[row >> 1] = pack_bf16x2(y, y1);
      }
      tc::fence_after_sync();
      // pass 1: block maxima of this thread's 64 values, columns 32-63 first (columns
      // 0-31 stay in registers for pass 2), and each block's provisional scale
      float am[4];
      uint32_t ws[4];
      float2 x0[16];
      {
        float2 x[16];
        tc::ld_32x32b_x32(ta + 32, reinterpret_cast<float*>(x));
        tc::ld_wait();
        float a2[2];
        block_amax3_raw<2>(x, a2);
        am[2] = a2[0];
        am[3] = a2[1];
      }
      {
        tc::ld_32x32b_x32(ta, reinterpret_cast<float*>(x0));
        tc::ld_wait();
        float a2[2];
        block_amax3_raw<2>(x0, a2);
        am[0] = a2[0];
        am[1] = a2[1];
      }
      // this thread's max |D1|: NaN if a block holds one; then (rarely) the
      // NaN-ignoring maximum, which the reference's tile amax takes.  The
      // reload is warp-wide (tcgen05.ld is .sync.aligned); lanes without a NaN
      // get their own maximum again.
      float tmax = max3_nan(am[0], am[1], max3_nan(am[2], am[3], 0.0f));
      if (__any_sync(0xffffffffu, isnan(tmax))) {
        tmax = amax_ignore_nan(x0);
#pragma unroll
        for (int q = 0; q < 2; ++q) {  // columns 32-63, 16 at a time (x0 stays live)
          float y[16];
          tc::ld_32x32b_x16(ta + 32 + 16 * q, y);
          tc::ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) tmax = fmaxf(tmax, fabsf(y[e]));
        }
      }
      // the warp's maximum in one reduction (non-negative floats order as their bits)
      const uint32_t wmax = __reduce_max_sync(0xffffffffu, __float_as_uint(tmax));
      if (lane == 0) atomicMax(&sm.amax_bits[grp][l & 1], wmax);
#pragma unroll
      for (int b = 0; b < 4; ++b) ws[b] = scale_w(am[b]);
      named_bar(bar_id, 256);
      // A = max |D1| over the tile (NaN ignored); gs' = c 2^-k, y = D1 2^k
      const uint32_t ab = sm.amax_bits[grp][l & 1];
      if (tid == lead) sm.amax_bits[grp][(l + 1) & 1] = 0u;  // the next tile's slot: every thread of the
                                                             // group read it (tile l - 1) before the barrier above
      int k = pow2_headroom(ab, gden_bits);
      const bool fast = ab >= 0x00800000u && ab < 0x7F800000u && k >= 0 && k <= kMaxShift;
      float mult, gs_new;
      if (ab != 0u && ab < 0x7F800000u) {  // finite A > 0
        k = k < -126 ? -126 : (k > 126 ? 126 : k);
        mult = exp2i(k);
        gs_new = m.c * exp2i(-k);
      } else if (ab == 0u) {  // an all-zero tile: gs' = 1, y = S'
        mult = m.c;
        gs_new = 1.0f;
      } else {  // an infinite value: gs' = inf, y = D1 * 0
        mult = 0.0f;
        gs_new = __uint_as_float(0x7F800000u);
      }
      // pass 2: codes, one pair of 16-value blocks per TMEM load and per 16-byte store
      uint8_t* codes = a.pool_codes + m.pt * a.code_stride + row * 64 + 32 * half;
      float* dbg = kDebug ? a.debug_y + (((int64_t)m.b * a.HV + m.h) * kD + row) * kD + 64 * half : nullptr;
      uint32_t scw = 0;
#pragma unroll
      for (int bp = 0; bp < 2; ++bp) {
        float2 x[16];
        if (bp == 0) {
#pragma unroll
          for (int e = 0; e < 16; ++e) x[e] = x0[e];
        } else {
          tc::ld_32x32b_x32(ta + 32, reinterpret_cast<float*>(x));
          tc::ld_wait();
          // D1 is read: X_g is free for the group's next tile
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.bar_x[grp]);
        }
        uint32_t words[4];
        if (fast) {
          // both blocks as normal, unclamped scale bytes: RN(y inv) = RN(D1 scale_inv_w)
          uint32_t fix = 0;
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const int bi = 2 * bp + b;
            const uint32_t fin = ws[bi] + 8u * (uint32_t)k - 960u;
            fix |= (fin - 8u > kSat - 8u) ? (1u << b) : 0u;
            const float inv0 = scale_inv_w(ws[bi], sm.rtab);
            const float2 inv2 = make_float2(inv0, inv0);
            words[2 * b] = e2m1_encode8(x + 8 * b, inv2);
            words[2 * b + 1] = e2m1_encode8(x + 8 * b + 4, inv2);
            scw |= (fin & 0xFFu) << (8 * bi);
          }
          // rare: a zero, subnormal-scale, saturated or NaN block takes the exact
          // path on y = D1 2^k (one warp-uniform test per pair of blocks)
          if (__any_sync(0xffffffffu, fix != 0)) {
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              if (fix & (1u << b)) {
                const int bi = 2 * bp + b;
                const float a1[1] = {am[bi]};
                uint32_t w2[2], sc;
                requant_blocks<kMode, 1>(*reinterpret_cast<const float2(*)[8]>(x + 8 * b), a1, mult, sm.inv_tab, w2,
                                         sc, nullptr);
                words[2 * b] = w2[0];
                words[2 * b + 1] = w2[1];
                scw = (scw & ~(0xFFu << (8 * bi))) | (sc << (8 * bi));
              }
            }
          }
        } else {
          const float a2[2] = {am[2 * bp], am[2 * bp + 1]};
          uint32_t sc2;
          requant_blocks<kMode, 2>(x, a2, mult, sm.inv_tab, words, sc2, nullptr);
          scw |= sc2 << (16 * bp);
        }
        *reinterpret_cast<uint4*>(codes + 16 * bp) = make_uint4(words[0], words[1], words[2], words[3]);
        if (kDebug) {
          float4* dy = reinterpret_cast<float4*>(dbg + 32 * bp);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            dy[e] = make_float4(__fmul_rn(x[2 * e].x, mult), __fmul_rn(x[2 * e].y, mult),
                                __fmul_rn(x[2 * e + 1].x, mult), __fmul_rn(x[2 * e + 1].y, mult));
        }
      }
      *reinterpret_cast<uint32_t*>(a.pool_scales + m.pt * a.scale_stride + row * 8 + 4 * half) = scw;
      if (tid == lead) *gs_at(a, m.pt) = gs_new;
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
  if (!p->q || !p->k || !p->v || (!p->A_log && (!p->g || !p->beta)) || !p->slot_idx || !p->pool_codes ||
      !p->pool_scales || !p->pool_gscale || !p->out)
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
  // A sequence's q/k/v rows must not overlap the next sequence's.
  if (a.q_stride < (int64_t)p->num_k_heads * kD || a.k_stride < (int64_t)p->num_k_heads * kD ||
      a.v_stride < (int64_t)p->num_v_heads * kD)
    return GDN_ERR_ARGS;
  // The codes are addressed as tiles of a 3-D tensor map (int32 tile coordinate).
  if (a.ntiles > INT32_MAX || p->num_slots * (int64_t)p->num_v_heads > INT32_MAX) return GDN_ERR_UNSUPPORTED;
  if (!pool_strides(p->pool_tile_stride, p->pool_codes, p->pool_scales, p->pool_gscale, &a.code_stride,
                    &a.scale_stride, &a.gs_stride))
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
  a.A_log = p->A_log;
  a.dt_bias = p->dt_bias;
  a.gate_a = p->gate_a;
  a.gate_b = p->gate_b;
  a.gate_stride = p->gate_stride ? p->gate_stride : p->num_v_heads;
  a.qk_l2norm = p->qk_l2norm;
  if (a.A_log && (!a.dt_bias || !a.gate_a || !a.gate_b || a.gate_stride < p->num_v_heads)) return GDN_ERR_ARGS;
  a.norm_weight = p->norm_weight;
  a.gate_z = p->norm_weight ? p->gate_z : nullptr;
  a.z_stride = p->z_stride ? p->z_stride : (int64_t)p->num_v_heads * kD;
  a.norm_eps = p->norm_eps;
  a.norm_act = p->norm_act;
  if (a.norm_weight) {
    if (!(a.norm_eps > 0.0f && a.norm_eps < 1.0f) || (a.norm_act != 0 && a.norm_act != 1)) return GDN_ERR_ARGS;
    if (p->debug_y) return GDN_ERR_UNSUPPORTED;  // the fused norm has no debug variant
    if (a.gate_z && (!aligned16(a.gate_z) || a.z_stride % 8 || a.z_stride < (int64_t)p->num_v_heads * kD))
      return GDN_ERR_ALIGN;
  }

  CUtensorMap tm;
  {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return GDN_ERR_CUDA;
    // [tiles][128 rows][64 bytes]: one box is one tile's codes, whatever the tile stride
    const int64_t tiles = p->num_slots > 0 ? p->num_slots * (int64_t)p->num_v_heads : 1;
    const cuuint64_t dims[3] = {64, (cuuint64_t)kD, (cuuint64_t)tiles};
    const cuuint64_t strides[2] = {64, (cuuint64_t)a.code_stride};
    const cuuint32_t box[3] = {64, kD, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, p->pool_codes, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GDN_ERR_CUDA;
  }

  const int smem = (int)sizeof(DecodeSmem);
  const int64_t max_ctas = sm_count();
  const int grid = (int)(a.ntiles < max_ctas ? a.ntiles : max_ctas);
  const int mi = (p->scale_mode == kScaleRef240 ? 0 : 1) + (p->debug_y ? 2 : 0) + (a.norm_weight ? 4 : 0);
  void (*kern)(const DecodeArgs, const CUtensorMap) =
      mi == 0 ? gdn_decode_kernel<kScaleRef240, false, false>
      : mi == 1 ? gdn_decode_kernel<kScaleFn448, false, false>
      : mi == 2 ? gdn_decode_kernel<kScaleRef240, true, false>
      : mi == 3 ? gdn_decode_kernel<kScaleFn448, true, false>
      : mi == 4 ? gdn_decode_kernel<kScaleRef240, false, true>
                : gdn_decode_kernel<kScaleFn448, false, true>;
  // > 48 KB of dynamic shared memory: opted in once per (kernel, device), under a lock.
  if (allow_dynamic_smem(reinterpret_cast<const void*>(kern), smem) != GDN_OK) return GDN_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a, tm) != cudaSuccess) {
    (void)cudaGetLastError();
    return GDN_ERR_LAUNCH;
  }
  return launch_status();
}
