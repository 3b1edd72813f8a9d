// gdn_decode.cu -- fused recurrent NVFP4 Gated DeltaNet decode step (sm_100a).
//
// One CTA owns one (sequence, value head) state tile at a time: a 128 x 128
// NVFP4 tile S[i][j] (i over d_k, j over d_v; 8192 B codes + 1024 B scales +
// one fp32 global scale) in the pool slot named by slot_idx.  Per tile:
//   alpha = exp(g), S_a = alpha S, u = S_a^T k, w = beta (v - u),
//   S' = S_a + k w^T, o = q_scale S'^T q = q_scale (S_a^T q + (k.q) w),
// then S' is requantised in place with a fresh global scale
// gs' = amax(S') / gden and the reference block quantiser
// (src/kernel/gdn_state_update_ref.cu:93-141) applied to y = S' (1/gs').
// The reference has no counterpart of this step (its only update is
// S' = alpha S + beta k v^T, gdn_state_update_ref.cu:51-67); the recurrence is
// the gated delta rule (Yang, Kautz & Hatamizadeh, ICLR 2025).
//
// The tensor cores decode the tile twice, both times exactly, with one
// block-scaled E2M1 MMA (kind::mxf4nvf4) against a constant identity operand:
//   MMA1' D = I * S^T with the tile's E4M3 scales as B scale factors
//         -> e2m1 * scale with TMEM lane = j, column = i.  Each thread then
//         holds one column j over 64 rows i and forms its partial sums of
//         u = S_a^T k and S_a^T q with packed f32x2 FMAs (no reduction across
//         lanes; the two row halves meet in shared memory);
//   MMA1  D = S * I with the scales as A scale factors -> lane = i, column = j,
//         the layout the requantiser wants: each thread holds one row i and
//         64 columns j, i.e. four whole 16-element scale blocks.
// The identity operand and its unit scale factors are built once per CTA.
// MMA1 runs while the threads compute the partial sums; the next tile's
// operands are staged and its MMA1' issued before the current tile is
// updated and requantised, so the tensor-core round trips overlap SIMT work.
// Requantisation uses cvt.rn.satfinite.e2m1x2.f32 with the tie correction of
// intrinsics/nvfp4_codec.cuh; all element arithmetic is packed f32x2.
//
// Pipeline: persistent grid of 2 CTAs per SM (256 TMEM columns each); a
// 4-stage ring of 1-D bulk copies prefetches the next tiles' codes, scales,
// q, k, v; per-tile scalars are loaded one tile ahead; every wait is bounded.
//
// Scale bytes are read by the tensor cores as UE4M3: identical to the
// reference decode for every byte the quantiser writes (0x00..0x77 in the
// reference mode, 0x00..0x7E in the E4M3FN mode).
#include <cstdint>
#include <cuda_bf16.h>

#include "../common.cuh"
#include "../intrinsics/nvfp4_codec.cuh"
#include "../tcgen05.cuh"
#include "tile_requant.cuh"

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
constexpr uint32_t kTmemCols = 256;
// TMEM columns
constexpr uint32_t kColD = 0;      // 128: dequantised tile (transposed, then not)
constexpr uint32_t kColSF = 128;   // 8: the tile's scale factors (2 K-steps x 4 columns)
constexpr uint32_t kColOne = 136;  // 8: unit scale factors of the identity

struct __align__(128) Stage {
  uint8_t codes[kCodeBytes];  // row-major, 64 B per row
  uint8_t scales[kScaleBytes];
  __nv_bfloat16 q[kD];
  __nv_bfloat16 k[kD];
  __nv_bfloat16 v[kD];
};

struct __align__(1024) DecodeSmem {
  Stage st[kStages];
  // MMA operands, no-swizzle K-major layout: byte b of row r at
  // (b % 16) + 16 r + 2048 (b / 16).
  uint8_t codes[kCodeBytes];
  uint8_t ident[kCodeBytes];
  uint8_t sf[kScaleBytes];  // scale factors, tcgen05.cp 32x128b layout, 2 K-steps
  uint8_t sf_one[kScaleBytes];
  float4 kq4[kD / 2];       // (k_i, k_i+1, q_i, q_i+1) for even i: the matvec operands
  float red[2][2][kD];      // [row half][u or S^T q][column]
  float w[kD];
  float amax[kWarps];
  float inv_tab[256];
  uint64_t full[kStages];
  uint64_t bar_dt, bar_d;
  uint32_t tmem_base;
};

__device__ __forceinline__ int canon(int row, int byte) { return (byte & 15) + 16 * row + 2048 * (byte >> 4); }

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
  // Tile t = b * HV + h.  A CTA visits t = blockIdx.x + n * gridDim.x; the
  // (b, h) step between visits is precomputed on the host so the kernel never
  // divides.
  int32_t step_b, step_h;
};

// (sequence, value head) of a tile, advanced without division.
struct TileIdx {
  int32_t b, h;
  __device__ __forceinline__ void advance(int32_t db, int32_t dh, int32_t HV) {
    h += dh;
    b += db;
    if (h >= HV) { h -= HV; ++b; }
  }
};

// Thread 0: queue the tile (t.b, t.h) into stage `s`.
__device__ __forceinline__ void issue_tile(const DecodeArgs& a, DecodeSmem& sm, int s, TileIdx t) {
  const int b = t.b, h = t.h;
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

struct Scalars {
  int32_t slot;
  float gs, g, beta;
};

__device__ __forceinline__ Scalars load_scalars(const DecodeArgs& a, TileIdx t) {
  Scalars sc{-1, 0.0f, 0.0f, 0.0f};
  if (t.b < a.B) {
    const int b = t.b, h = t.h;
    sc.slot = __ldg(a.slot_idx + b);
    sc.g = __ldg(a.g + (int64_t)b * a.HV + h);
    sc.beta = __ldg(a.beta + (int64_t)b * a.HV + h);
    if (sc.slot >= 0 && sc.slot < a.num_slots) sc.gs = __ldg(a.pool_gs + (int64_t)sc.slot * a.HV + h);
  }
  return sc;
}

// Everything a tile carries from its staging to its store.
struct TileCtx {
  TileIdx idx;
  int64_t pt;    // pool tile index slot * HV + h
  float c;       // alpha * old global scale
  float beta;
  float kq;      // k . q (threads of warps 0..3)
  float vj;      // v_j (threads of warps 0..3)
  float k_row;   // k_i of this thread's row
};

template <int kMode>
__global__ void __launch_bounds__(kThreads, 2) gdn_decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3;         // TMEM lane subpartition of this warp
  const int half = warp >> 2;        // which 64 TMEM columns this warp reads
  const int row = 32 * quad + lane;  // TMEM lane: column j after MMA1', row i after MMA1

  // ---- once per CTA: tables, identity operand, unit scale factors, barriers, TMEM ----
  sm.inv_tab[tid] = scale_inverse(scale_decode((uint32_t)tid, kMode));
  for (int e = tid; e < (int)kCodeBytes; e += kThreads) {
    const int r = e >> 6, byte = e & 63;
    uint8_t val = 0;
    if (2 * byte == r) val = 0x02;      // E2M1 1.0 in the low nibble (k = 2 byte)
    if (2 * byte + 1 == r) val = 0x20;  // ... or the high nibble (k = 2 byte + 1)
    sm.ident[canon(r, byte)] = val;
  }
  reinterpret_cast<uint32_t*>(sm.sf_one)[tid] = 0x38383838u;  // UE4M3 1.0
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
    mbar_init(&sm.bar_dt, 1);
    mbar_init(&sm.bar_d, 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&sm.tmem_base, kTmemCols);
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t T = sm.tmem_base;
  const uint32_t id_mx = tc::idesc_mxf4nvf4(128, 128);
  const TileIdx first{(int32_t)(blockIdx.x / (uint32_t)a.HV), (int32_t)(blockIdx.x % (uint32_t)a.HV)};
  TileIdx ahead = first;  // thread 0: the tile whose copies are queued next
  if (tid == 0) {
    for (int t = 0; t < 2; ++t) tc::cp_32x128b_warpx4(T + kColOne + 4 * t, tc::smem_desc(sm.sf_one + 512 * t, 0, 128));
    for (int s = 0; s < kStages; ++s) {
      if (ahead.b < a.B) issue_tile(a, sm, s, ahead);
      ahead.advance(a.step_b, a.step_h, a.HV);
    }
  }

  bool failed = false;
  uint32_t par = 0;  // phase of bar_dt / bar_d (one completion per valid tile each)
  int64_t n = 0;     // local index of the next tile to stage
  TileIdx sidx = first;             // the next tile to stage
  TileIdx pidx = first;             // the tile whose scalars are prefetched next
  Scalars scal = load_scalars(a, pidx);
  pidx.advance(a.step_b, a.step_h, a.HV);

  // Waits for local tile n, writes zeros for padding tiles, and for the next
  // valid tile stages its MMA operands, fills `ctx` and issues its MMA1'.
  // Returns false when this CTA has no tile left (or a wait timed out).
  auto stage_next = [&](TileCtx& ctx) -> bool {
    for (;; ++n, sidx.advance(a.step_b, a.step_h, a.HV)) {
      if (sidx.b >= a.B) return false;
      const Scalars cur = scal;
      scal = load_scalars(a, pidx);
      pidx.advance(a.step_b, a.step_h, a.HV);
      const int s = (int)(n % kStages);
      if (!mbar_wait_cta(&sm.full[s], (uint32_t)((n / kStages) & 1))) { failed = true; return false; }
      const int b = sidx.b, h = sidx.h;
      if (cur.slot < 0 || cur.slot >= a.num_slots) {
        __nv_bfloat16* ob = a.out + ((int64_t)b * a.HV + h) * kD;
        if (tid < kD / 2) reinterpret_cast<uint32_t*>(ob)[tid] = 0u;
        if (tid == 0) {
          if (cur.slot >= a.num_slots) atomicOr(a.status, kStatusBadSlot);
          if (ahead.b < a.B) issue_tile(a, sm, s, ahead);
          ahead.advance(a.step_b, a.step_h, a.HV);
        }
        continue;
      }
      Stage& st = sm.st[s];
      ctx.idx = sidx;
      ctx.pt = (int64_t)cur.slot * a.HV + h;
      ctx.c = expf(cur.g) * cur.gs;
      ctx.beta = cur.beta;
      {
        // codes -> no-swizzle K-major: thread moves 32 bytes (two 16-byte chunks) of row tid/2
        const int r = tid >> 1, c0 = 2 * (tid & 1);
        const uint4* src = reinterpret_cast<const uint4*>(st.codes + r * 64 + 16 * c0);
        const uint4 x0 = src[0], x1 = src[1];
        *reinterpret_cast<uint4*>(sm.codes + 2048 * c0 + 16 * r) = x0;
        *reinterpret_cast<uint4*>(sm.codes + 2048 * (c0 + 1) + 16 * r) = x1;
        // scale factors: word (t*128 + m0*4 + m1) <- scales of row 32 m1 + m0, blocks 4t..4t+3
        const int t = tid >> 7, m0 = (tid & 127) >> 2, m1 = tid & 3;
        reinterpret_cast<uint32_t*>(sm.sf)[t * 128 + m0 * 4 + m1] =
            reinterpret_cast<const uint32_t*>(st.scales)[(32 * m1 + m0) * 2 + t];
      }
      if (tid < kD / 2) {
        const __nv_bfloat162 k2 = reinterpret_cast<const __nv_bfloat162*>(st.k)[tid];
        const __nv_bfloat162 q2 = reinterpret_cast<const __nv_bfloat162*>(st.q)[tid];
        sm.kq4[tid] = make_float4(__low2float(k2), __high2float(k2), __low2float(q2), __high2float(q2));
      }
      ctx.k_row = bf2f(st.k[row]);
      ctx.kq = 0.0f;
      ctx.vj = 0.0f;
      if (warp < 4) {
        float kq = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) kq = fmaf(bf2f(st.k[4 * lane + i]), bf2f(st.q[4 * lane + i]), kq);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);
        ctx.kq = kq;
        ctx.vj = bf2f(st.v[tid]);
      }
      tc::fence_smem_to_async();
      tc::fence_before_sync();
      __syncthreads();  // operands staged, stage s consumed
      tc::fence_after_sync();
      if (tid == 0) {
        if (ahead.b < a.B) issue_tile(a, sm, s, ahead);
        ahead.advance(a.step_b, a.step_h, a.HV);
        // MMA1': D = I * S^T (lane j, column i)
        for (int t = 0; t < 2; ++t) tc::cp_32x128b_warpx4(T + kColSF + 4 * t, tc::smem_desc(sm.sf + 512 * t, 0, 128));
        for (int t = 0; t < 2; ++t)
          tc::mma_mxf4nvf4(T + kColD, tc::smem_desc(sm.ident + 4096 * t, 2048, 128),
                           tc::smem_desc(sm.codes + 4096 * t, 2048, 128), id_mx, T + kColOne + 4 * t,
                           T + kColSF + 4 * t, t > 0);
        tc::commit(&sm.bar_dt);
      }
      ++n;
      sidx.advance(a.step_b, a.step_h, a.HV);
      return true;
    }
  };

  TileCtx cur, nxt;
  bool have = stage_next(cur);
  while (have) {
    const int b = cur.idx.b, h = cur.idx.h;
    __nv_bfloat16* ob = a.out + ((int64_t)b * a.HV + h) * kD;

    // ---- 1: the transposed tile -> partial S^T k, S^T q over this thread's 64 rows ----
    if (!mbar_wait_cta(&sm.bar_dt, par)) { failed = true; break; }
    tc::fence_after_sync();
    float2 x[32];
    {
      const uint32_t ta = T + ((uint32_t)(32 * quad) << 16) + kColD + 64 * half;
      tc::ld_32x32b_x32(ta, reinterpret_cast<float*>(x));
      tc::ld_32x32b_x32(ta + 32, reinterpret_cast<float*>(x) + 32);
      tc::ld_wait();
    }
    tc::fence_before_sync();
    __syncthreads();  // D read by every thread: MMA1 may overwrite it
    tc::fence_after_sync();
    if (tid == 0) {
      // MMA1: D = S * I (lane i, column j)
      for (int t = 0; t < 2; ++t)
        tc::mma_mxf4nvf4(T + kColD, tc::smem_desc(sm.codes + 4096 * t, 2048, 128),
                         tc::smem_desc(sm.ident + 4096 * t, 2048, 128), id_mx, T + kColSF + 4 * t,
                         T + kColOne + 4 * t, t > 0);
      tc::commit(&sm.bar_d);
    }
    {
      // x[p] = (S[64 half + 2p][j], S[64 half + 2p + 1][j]) * scale (unscaled by c)
      float2 su = make_float2(0.0f, 0.0f), sp = make_float2(0.0f, 0.0f);
      const float4* kq4 = sm.kq4 + 32 * half;
#pragma unroll
      for (int p = 0; p < 32; ++p) {
        const float4 kq = kq4[p];
        su = __ffma2_rn(x[p], make_float2(kq.x, kq.y), su);
        sp = __ffma2_rn(x[p], make_float2(kq.z, kq.w), sp);
      }
      sm.red[half][0][row] = su.x + su.y;
      sm.red[half][1][row] = sp.x + sp.y;
    }
    __syncthreads();  // partial sums of both row halves published
    if (warp < 4) {
      const int j = tid;
      const float u = cur.c * (sm.red[0][0][j] + sm.red[1][0][j]);
      const float pq = cur.c * (sm.red[0][1][j] + sm.red[1][1][j]);
      const float wj = cur.beta * (cur.vj - u);
      sm.w[j] = wj;
      const float o0 = a.q_scale * fmaf(cur.kq, wj, pq);
      const float o1 = __shfl_down_sync(0xffffffffu, o0, 1);
      if ((j & 1) == 0)
        reinterpret_cast<uint32_t*>(ob)[j >> 1] = (uint32_t)f2bf_bits(o0) | ((uint32_t)f2bf_bits(o1) << 16);
    }

    // ---- 2: the tile (lane i) -> registers ----
    const bool ok_d = mbar_wait_cta(&sm.bar_d, par);  // also publishes w
    par ^= 1;
    if (!ok_d) { failed = true; break; }
    tc::fence_after_sync();
    {
      const uint32_t ta = T + ((uint32_t)(32 * quad) << 16) + kColD + 64 * half;
      tc::ld_32x32b_x32(ta, reinterpret_cast<float*>(x));
      tc::ld_32x32b_x32(ta + 32, reinterpret_cast<float*>(x) + 32);
      tc::ld_wait();
    }
    tc::fence_before_sync();

    // ---- 3: stage the next tile and start its MMA1' (overlaps 4-5) ----
    have = stage_next(nxt);

    // ---- 4: rank-1 update of this thread's row, block and tile amax ----
    const float2 c2 = make_float2(cur.c, cur.c), k2 = make_float2(cur.k_row, cur.k_row);
    const float4* w4 = reinterpret_cast<const float4*>(sm.w + 64 * half);  // w of this thread's columns
    float am[4];
    float tmax = 0.0f;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
      float mx = 0.0f;
#pragma unroll
      for (int p = 0; p < 8; p += 2) {
        const float4 wv = w4[4 * blk + p / 2];
        float2& v0 = x[8 * blk + p];
        float2& v1 = x[8 * blk + p + 1];
        v0 = __ffma2_rn(k2, make_float2(wv.x, wv.y), __fmul2_rn(v0, c2));
        v1 = __ffma2_rn(k2, make_float2(wv.z, wv.w), __fmul2_rn(v1, c2));
        mx = (p == 0) ? absmax_nan(v0.x, v0.y) : absmax_nan(absmax_nan(mx, v0.x), v0.y);
        mx = absmax_nan(absmax_nan(mx, v1.x), v1.y);
      }
      am[blk] = fabsf(mx);
      float ok_max = am[blk];
      if (isnan(ok_max)) {  // rare: the reference's amax ignores NaN
        ok_max = 0.0f;
#pragma unroll
        for (int p = 0; p < 8; ++p) ok_max = fmaxf(ok_max, fmaxf(fabsf(x[8 * blk + p].x), fabsf(x[8 * blk + p].y)));
      }
      tmax = fmaxf(tmax, ok_max);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    if (lane == 0) sm.amax[warp] = tmax;
    __syncthreads();  // tile amax
    float amax = sm.amax[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) amax = fmaxf(amax, sm.amax[w]);
    const float gs_new = (amax > 0.0f) ? __fdiv_rn(amax, a.gden) : 1.0f;
    const float inv_gs = __frcp_rn(gs_new);

    // ---- 5: requantise this thread's four blocks, store ----
    uint32_t words[8];
    uint32_t scw;
    requant_half_row<kMode>(x, am, inv_gs, sm.inv_tab, words, scw,
                            a.debug_y ? a.debug_y + (((int64_t)b * a.HV + h) * kD + row) * kD + 64 * half : nullptr);
    uint4* dst = reinterpret_cast<uint4*>(a.pool_codes + cur.pt * kCodeBytes + row * 64 + 32 * half);
    dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
    dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
    *reinterpret_cast<uint32_t*>(a.pool_scales + cur.pt * kScaleBytes + row * 8 + 4 * half) = scw;
    if (tid == 0) a.pool_gs[cur.pt] = gs_new;
    cur = nxt;
  }

  if (failed && tid == 0) {
    // Report, then give the copies this CTA queued a bounded chance to land
    // before its shared memory is released.
    atomicOr(a.status, kStatusWaitTimeout);
    // local tiles n .. n + kStages - 1 may have copies queued
    TileIdx t = sidx;
    for (int64_t m = n; m < n + kStages; ++m, t.advance(a.step_b, a.step_h, a.HV)) {
      if (t.b >= a.B) break;
      mbar_wait_bounded(&sm.full[m % kStages], (uint32_t)((m / kStages) & 1), kWaitTimeoutNs / 4);
    }
  }
  // Every tcgen05 operation of this CTA has been waited on (or abandoned after
  // a timeout); release the tensor memory.
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(T, kTmemCols);
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
  if (a.ntiles > INT32_MAX) return GDN_ERR_UNSUPPORTED;
  a.step_b = grid / a.HV;
  a.step_h = grid % a.HV;
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
