// gdn_prefill.cu -- chunked NVFP4 Gated DeltaNet prefill (sm_100a).
//
// The gated delta rule of gdn_decode.cu applied to every token of packed
// variable-length sequences, in chunks of C = 64 tokens (WY/UT form; Yang,
// Kautz & Hatamizadeh, "Gated Delta Networks", ICLR 2025).  For one
// (sequence, value head) and a chunk with initial state S (d_k x d_v), local
// tokens r, s in [0, C), cumulative log decay G_r = g_0 + .. + g_r and
// gamma_r = exp(G_r):
//   A[r][s]  = beta_r (k_r . k_s) exp(G_r - G_s)            s < r   (else 0)
//   T        = (I + A)^-1                                     (unit lower triangular)
//   U        = T diag(beta) V,   W = T diag(beta gamma) K
//   V_new    = U - W S                                        (the delta-rule w of every token)
//   O        = q_scale (diag(gamma) Q S + P V_new),  P[r][s] = (q_r . k_s) exp(G_r - G_s), s <= r
//   S_next   = gamma_{C-1} S + sum_s exp(G_{C-1} - G_s) k_s V_new_s^T
// which equals the token-by-token recurrence exactly (in exact arithmetic).
// The reference has no prefill (its serving loop calls the d x d update once
// per token and sequence, src/ops/qwen35_gdn_patch.py:98-116).
//
// One CTA owns one (sequence, value head) at a time and walks its chunks in
// order.  The state stays in tensor memory for the whole sequence, transposed
// (TMEM lane = j over d_v, column = i over d_k), so that it is directly the A
// operand of the two tf32 products that read it.  Per chunk:
//   P1 (bf16)  [K; Q] K^T             -> K K^T and Q K^T in one M = 128 MMA
//   SIMT       A, P, the blocked 16 x 16 triangular inverse T
//   P2 (bf16)  U^T = V^T (T diag beta)^T
//   P3 (bf16)  W^T = K^T (T diag(beta gamma))^T
//   P4 (tf32)  U^T - S^T W^T          (accumulates onto U^T: V_new^T)
//   P6a (tf32) S^T (q_scale diag(gamma) Q)^T
//   P6b (tf32) + V_new^T P^T          -> O^T
//   P7 (bf16)  S^T <- gamma S^T + V_new'^T K  (V_new' = V_new scaled by exp(G_{C-1} - G_s))
// q, k, v rows arrive by 1-D bulk copies (one per 256-byte row) into a padded
// staging buffer; the next chunk's copies are issued as soon as the current
// chunk's operands are built, so they overlap the rest of the chunk.  At the
// end of a sequence the state is requantised into its pool slot with the
// reference block quantiser (tile_requant.cuh).  Every wait is bounded.
//
// All MMA operands use the no-swizzle K-major layout: 8-row x 16-byte core
// matrices, 16-byte K chunks 128 bytes apart (LBO), 8-row groups SBO apart.
#include <cstdint>
#include <cuda_bf16.h>

#include "../common.cuh"
#include "../intrinsics/nvfp4_codec.cuh"
#include "../tcgen05.cuh"
#include "tile_requant.cuh"

namespace gdn {
namespace {

constexpr int kD = 128;
constexpr int kC = 64;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kCodeBytes = kD * kD / 2;
constexpr uint32_t kScaleBytes = kD * kD / 16;
constexpr uint32_t kRowBytes = kD * 2;  // one bf16 q/k/v row
constexpr uint32_t kStgRow = 272;       // staged row pitch (16 bytes of padding against bank conflicts)
constexpr uint32_t kStgBytes = kC * kStgRow;

// Shared-memory map (bytes).  Regions are reused by phase; see each use.
constexpr uint32_t kOffStgK = 0;
constexpr uint32_t kOffStgQ = kStgBytes;
constexpr uint32_t kOffStgV = 2 * kStgBytes;
constexpr uint32_t kOffR1 = 3 * kStgBytes;      // [K;Q] bf16 -> solve scratch -> -W fp32
constexpr uint32_t kSizeR1 = 39936;
constexpr uint32_t kOffKt = kOffR1 + kSizeR1;   // K^T bf16 [d_k][C]
constexpr uint32_t kOffR2 = kOffKt + 16384;     // V^T bf16, T', T'' -> V_new^T fp32 (or initial-state operands)
constexpr uint32_t kOffR3 = kOffR2 + 32768;     // Q' fp32 -> V_new'^T bf16
constexpr uint32_t kOffPm = kOffR3 + 32768;     // P fp32 [C][C]
constexpr uint32_t kOffMisc = kOffPm + 16384;
constexpr int kLd = 68;                         // solve scratch row pitch (floats)
constexpr uint32_t kFPitch = 132;               // final-state transpose row pitch (floats)
constexpr uint32_t kWnSbo = 4608;               // -W: 32 K chunks of 144 bytes per 8-row group
constexpr uint32_t kWnLbo = 144;

static_assert(kOffR1 % 128 == 0 && kOffR2 % 128 == 0 && kOffR3 % 128 == 0 && kOffPm % 128 == 0, "alignment");
static_assert(2 * 64 * kLd * 4 + 16 * kLd * 4 <= kSizeR1, "solve scratch fits R1");
static_assert(8 * kWnSbo <= kSizeR1, "-W fits R1");
static_assert(kOffR1 + 128 * kFPitch * 4 <= kOffR3, "final-state transpose fits R1..R2");

// TMEM columns (512 allocated: one CTA per SM)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;     // 128: state S^T (lane j, column i)
constexpr uint32_t kColKQ = 128;  // 64: [K K^T; Q K^T]
constexpr uint32_t kColU = 192;   // 64: U^T, then V_new^T
constexpr uint32_t kColW = 256;   // 64: W^T (lane i, column r)
constexpr uint32_t kColO = 320;   // 64: O^T
constexpr uint32_t kColSF = 384;  // 8: initial-state scale factors
constexpr uint32_t kColOne = 392; // 8: unit scale factors

struct Misc {
  float gw[kC];    // warp-inclusive scans of g
  float G[kC];     // cumulative log decay
  float bet[kC];   // beta
  float bg[kC];    // beta * gamma
  float de[kC];    // exp(G_last - G)
  float inv_tab[256];
  float amax[kWarps];
  uint64_t bar_stg, bar_mma;
  uint32_t tmem_base;
};
constexpr uint32_t kSmemBytes = kOffMisc + sizeof(Misc);
static_assert(kSmemBytes <= 232448, "shared memory");

struct PrefillArgs {
  int32_t N, HK, HV, group, nitems;
  int64_t T, num_slots;
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_stride, k_stride, v_stride;
  const float* g;
  const float* beta;
  const int32_t* cu;
  const int32_t* slot_idx;
  const uint8_t* has_init;
  uint8_t* pool_codes;
  uint8_t* pool_scales;
  float* pool_gs;
  __nv_bfloat16* out;
  float q_scale, gden;
  float* debug_y;
  uint32_t* status;
};

// Byte offsets in the K-major no-swizzle layouts.
__device__ __forceinline__ uint32_t kbf16(int row, int k, uint32_t sbo) {
  return (row & 7) * 16 + (k & 7) * 2 + (row >> 3) * sbo + (k >> 3) * 128;
}
__device__ __forceinline__ uint32_t kf32(int row, int k, uint32_t sbo) {
  return (row & 7) * 16 + (k & 3) * 4 + (row >> 3) * sbo + (k >> 2) * 128;
}
__device__ __forceinline__ uint32_t kwn(int r, int i) {
  return (r & 7) * 16 + (i & 3) * 4 + (r >> 3) * kWnSbo + (i >> 2) * kWnLbo;
}
__device__ __forceinline__ int canon(int row, int byte) { return (byte & 15) + 16 * row + 2048 * (byte >> 4); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// Position in the CTA's work list: item = n * HV + h, chunk of that sequence.
struct Cursor {
  int32_t item, n, h;
  int64_t bos, len;
  int64_t chunk;
};

// Moves c to the first item >= c.item (stride gridDim.x) with at least one token.
__device__ __forceinline__ void cursor_seek(const PrefillArgs& a, Cursor& c, bool report) {
  for (; c.item < a.nitems; c.item += gridDim.x) {
    c.n = c.item / a.HV;
    c.h = c.item - c.n * a.HV;
    const int32_t b0 = __ldg(a.cu + c.n), b1 = __ldg(a.cu + c.n + 1);
    if (b0 < 0 || b1 < b0 || (int64_t)b1 > a.T) {
      if (report) atomicOr(a.status, GDN_STATUS_BAD_SEQLENS);
      continue;
    }
    if (b1 == b0) continue;
    c.bos = b0;
    c.len = b1 - b0;
    c.chunk = 0;
    return;
  }
}

__device__ __forceinline__ void cursor_next(const PrefillArgs& a, Cursor& c, bool report) {
  if ((c.chunk + 1) * kC < c.len) {
    ++c.chunk;
    return;
  }
  c.item += gridDim.x;
  cursor_seek(a, c, report);
}

__device__ __forceinline__ int chunk_len(const Cursor& c) {
  const int64_t rest = c.len - c.chunk * kC;
  return rest < kC ? (int)rest : kC;
}

// Warp 0: queue the q, k, v rows of chunk c into the staging buffer.
__device__ __forceinline__ void issue_chunk(const PrefillArgs& a, uint8_t* smem, uint64_t* bar, const Cursor& c,
                                            int lane) {
  const int64_t t0 = c.bos + c.chunk * kC;
  const int len = chunk_len(c);
  const int64_t hk = c.h / a.group;
  if (lane == 0) mbar_arrive_expect_tx(bar, 3u * kRowBytes * (uint32_t)len);
  __syncwarp();
  for (int r = lane; r < len; r += 32) {
    const int64_t t = t0 + r;
    bulk_g2s(smem + kOffStgK + r * kStgRow, a.k + t * a.k_stride + hk * kD, kRowBytes, bar);
    bulk_g2s(smem + kOffStgQ + r * kStgRow, a.q + t * a.q_stride + hk * kD, kRowBytes, bar);
    bulk_g2s(smem + kOffStgV + r * kStgRow, a.v + t * a.v_stride + (int64_t)c.h * kD, kRowBytes, bar);
  }
}

// Threads 0..63: g and beta of token `r` of chunk c (0 past the chunk end).
__device__ __forceinline__ void load_gb(const PrefillArgs& a, const Cursor& c, int r, float& gv, float& bv) {
  gv = 0.0f;
  bv = 0.0f;
  if (r < chunk_len(c)) {
    const int64_t idx = (c.bos + c.chunk * kC + r) * a.HV + c.h;
    gv = __ldg(a.g + idx);
    bv = __ldg(a.beta + idx);
  }
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1) gdn_prefill_kernel(const PrefillArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  Misc& ms = *reinterpret_cast<Misc*>(smem + kOffMisc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int lrow = 32 * quad + lane;  // this thread's TMEM lane
  const uint32_t lane_base = (uint32_t)(32 * quad) << 16;

  uint8_t* const stg_k = smem + kOffStgK;
  uint8_t* const stg_q = smem + kOffStgQ;
  uint8_t* const stg_v = smem + kOffStgV;
  uint8_t* const a1 = smem + kOffR1;
  float* const Am = reinterpret_cast<float*>(smem + kOffR1);
  float* const Tm = Am + 64 * kLd;
  float* const Xm = Tm + 64 * kLd;
  uint8_t* const wn = smem + kOffR1;
  uint8_t* const kt = smem + kOffKt;
  uint8_t* const vt = smem + kOffR2;
  uint8_t* const tp = smem + kOffR2 + 16384;   // T diag(beta gamma)
  uint8_t* const tpp = smem + kOffR2 + 24576;  // T diag(beta)
  uint8_t* const vn = smem + kOffR2;           // V_new^T fp32
  uint8_t* const qp = smem + kOffR3;
  uint8_t* const vnp = smem + kOffR3;          // V_new'^T bf16
  uint8_t* const pm = smem + kOffPm;

  ms.inv_tab[tid] = scale_inverse(scale_decode((uint32_t)tid, kMode));
  if (tid == 0) {
    mbar_init(&ms.bar_stg, 1);
    mbar_init(&ms.bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&ms.tmem_base, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t T = ms.tmem_base;
  const uint32_t id_bf16_64 = tc::idesc_bf16(128, 64);
  const uint32_t id_bf16_128 = tc::idesc_bf16(128, 128);
  const uint32_t id_tf32_64 = tc::idesc_tf32(128, 64);
  const uint32_t id_mx = tc::idesc_mxf4nvf4(128, 128);

  Cursor cur{(int32_t)blockIdx.x, 0, 0, 0, 0, 0};
  cursor_seek(a, cur, tid == 0);
  Cursor ahead = cur;
  float g_pre = 0.0f, b_pre = 0.0f;
  bool stg_pending = false, mma_pending = false, failed = false;
  uint32_t stg_par = 0, mma_par = 0;
  if (cur.item < a.nitems) {
    if (warp == 0) issue_chunk(a, smem, &ms.bar_stg, ahead, lane);
    if (tid < kC) load_gb(a, ahead, tid, g_pre, b_pre);
    stg_pending = true;
    cursor_next(a, ahead, false);
  }

  // Issues the queued MMAs' commit (thread 0) and waits for them (all).
  auto mma_wait = [&]() -> bool {
    mma_pending = true;
    if (!mbar_wait_cta(&ms.bar_mma, mma_par)) return false;
    mma_par ^= 1;
    mma_pending = false;
    tc::fence_after_sync();
    return true;
  };
  auto sync_for_mma = [&]() {
    tc::fence_smem_to_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  };

  int32_t slot = -1;
  bool s_zero = true;  // the state in TMEM is not valid yet (zero initial state)
  while (cur.item < a.nitems) {
    const int h = cur.h;
    const int64_t t0 = cur.bos + cur.chunk * kC;
    const int len = chunk_len(cur);
    const bool last = (cur.chunk + 1) * kC >= cur.len;

    // ---- sequence start: slot and initial state ----
    if (cur.chunk == 0) {
      slot = a.slot_idx ? __ldg(a.slot_idx + cur.n) : -1;
      if (slot >= a.num_slots) {
        if (tid == 0) atomicOr(a.status, GDN_STATUS_BAD_SLOT);
        slot = -1;
      }
      if (slot < 0) slot = -1;
      const bool has = slot >= 0 && a.has_init && __ldg(a.has_init + cur.n) != 0;
      s_zero = !has;
      if (has) {
        // Decode the NVFP4 tile straight into TMEM with one block-scaled MMA
        // against the identity: D = I * S^T (lane j, column i).
        const int64_t pt = (int64_t)slot * a.HV + h;
        uint8_t* const codes = smem + kOffR2;
        uint8_t* const ident = codes + kCodeBytes;
        uint8_t* const sf = ident + kCodeBytes;
        uint8_t* const sf_one = sf + kScaleBytes;
        {
          const int r = tid >> 1, c0 = 2 * (tid & 1);
          const uint4* src = reinterpret_cast<const uint4*>(a.pool_codes + pt * kCodeBytes + r * 64 + 16 * c0);
          const uint4 x0 = __ldg(src), x1 = __ldg(src + 1);
          *reinterpret_cast<uint4*>(codes + 2048 * c0 + 16 * r) = x0;
          *reinterpret_cast<uint4*>(codes + 2048 * (c0 + 1) + 16 * r) = x1;
          const int t = tid >> 7, m0 = (tid & 127) >> 2, m1 = tid & 3;
          reinterpret_cast<uint32_t*>(sf)[t * 128 + m0 * 4 + m1] =
              __ldg(reinterpret_cast<const uint32_t*>(a.pool_scales + pt * kScaleBytes) + (32 * m1 + m0) * 2 + t);
          reinterpret_cast<uint32_t*>(sf_one)[tid] = 0x38383838u;  // UE4M3 1.0
          for (int e = tid; e < (int)kCodeBytes; e += kThreads) {
            const int rr = e >> 6, byte = e & 63;
            uint8_t val = 0;
            if (2 * byte == rr) val = 0x02;      // E2M1 1.0, low nibble
            if (2 * byte + 1 == rr) val = 0x20;  // high nibble
            ident[canon(rr, byte)] = val;
          }
        }
        const float gs = __ldg(a.pool_gs + pt);
        sync_for_mma();
        if (tid == 0) {
          for (int t = 0; t < 2; ++t) {
            tc::cp_32x128b_warpx4(T + kColSF + 4 * t, tc::smem_desc(sf + 512 * t, 0, 128));
            tc::cp_32x128b_warpx4(T + kColOne + 4 * t, tc::smem_desc(sf_one + 512 * t, 0, 128));
          }
          for (int t = 0; t < 2; ++t)
            tc::mma_mxf4nvf4(T + kColS, tc::smem_desc(ident + 4096 * t, 2048, 128),
                             tc::smem_desc(codes + 4096 * t, 2048, 128), id_mx, T + kColOne + 4 * t,
                             T + kColSF + 4 * t, t > 0);
          tc::commit(&ms.bar_mma);
        }
        if (!mma_wait()) { failed = true; break; }
        float sv[32];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const uint32_t ta = T + lane_base + kColS + 64 * half + 32 * p;
          tc::ld_32x32b_x32(ta, sv);
          tc::ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) sv[c] *= gs;
          tc::st_32x32b_x32(ta, sv);
        }
        tc::st_wait();
        tc::fence_before_sync();
      }
    }

    // ---- 0: staged rows -> MMA operands; g, beta -> cumulative decay ----
    if (!mbar_wait_cta(&ms.bar_stg, stg_par)) { failed = true; break; }
    stg_par ^= 1;
    stg_pending = false;
    const float gv = g_pre, bv = b_pre;
    if (tid < kC) {
      float s = gv;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      ms.gw[tid] = s;
      ms.bet[tid] = bv;
    }
    // [K; Q] rows (bf16, 128 x 128): thread moves 16-byte chunks; rows past the chunk end are zero.
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int e = tid + kThreads * it;
      const int row_lo = e & 7, c = (e >> 3) & 15, row_hi = e >> 7;
      const int row = row_lo + 8 * row_hi;
      const int r = row & 63;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (r < len) val = *reinterpret_cast<const uint4*>((row < 64 ? stg_k : stg_q) + r * kStgRow + 16 * c);
      *reinterpret_cast<uint4*>(a1 + row_lo * 16 + row_hi * 2048 + c * 128) = val;
    }
    tc::fence_smem_to_async();
    __syncthreads();
    if (tid == 0) {
      // P1: [K K^T; Q K^T] = [K; Q] K^T  (M = 128, N = 64, K = 128)
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t d = tc::smem_desc(a1 + 256 * ks, 128, 2048);
        tc::mma_bf16_ss(T + kColKQ, d, d, id_bf16_64, ks > 0);
      }
      tc::commit(&ms.bar_mma);
    }
    if (tid < kC) {
      const float G = ms.gw[tid] + (tid >= 32 ? ms.gw[31] : 0.0f);
      const float Glast = ms.gw[63] + ms.gw[31];
      const float gm = __expf(G);
      ms.G[tid] = G;
      ms.bg[tid] = bv * gm;
      ms.de[tid] = __expf(Glast - G);
    }
    // K^T, V^T (bf16 [d][C]): thread gathers 8 tokens of one column.
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int e = tid + kThreads * it;
      const int i = e & 127, s8 = e >> 7;
      uint32_t wk[4], wv[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int s = 8 * s8 + 2 * t;
        uint32_t k0 = 0, k1 = 0, v0 = 0, v1 = 0;
        if (s < len) {
          k0 = reinterpret_cast<const uint16_t*>(stg_k + s * kStgRow)[i];
          v0 = reinterpret_cast<const uint16_t*>(stg_v + s * kStgRow)[i];
        }
        if (s + 1 < len) {
          k1 = reinterpret_cast<const uint16_t*>(stg_k + (s + 1) * kStgRow)[i];
          v1 = reinterpret_cast<const uint16_t*>(stg_v + (s + 1) * kStgRow)[i];
        }
        wk[t] = k0 | (k1 << 16);
        wv[t] = v0 | (v1 << 16);
      }
      const uint32_t off = (i & 7) * 16 + (i >> 3) * 1024 + s8 * 128;
      *reinterpret_cast<uint4*>(kt + off) = make_uint4(wk[0], wk[1], wk[2], wk[3]);
      *reinterpret_cast<uint4*>(vt + off) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    __syncthreads();  // G, bg, de published
    const float Glast = ms.G[kC - 1];
    // Q' = q_scale gamma_r q_r (fp32 [C][d_k])
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int e = tid + kThreads * it;
      const int r_lo = e & 7, i4 = (e >> 3) & 31, r_hi = e >> 8;
      const int r = r_lo + 8 * r_hi;
      float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (r < len) {
        const float sc = a.q_scale * __expf(ms.G[r]);
        const uint2 raw = *reinterpret_cast<const uint2*>(stg_q + r * kStgRow + 8 * i4);
        const __nv_bfloat162 q01 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
        const __nv_bfloat162 q23 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
        o = make_float4(sc * __low2float(q01), sc * __high2float(q01), sc * __low2float(q23), sc * __high2float(q23));
      }
      *reinterpret_cast<float4*>(qp + r_lo * 16 + r_hi * 4096 + i4 * 128) = o;
    }
    tc::fence_smem_to_async();
    __syncthreads();  // staging consumed: queue the next chunk
    if (ahead.item < a.nitems) {
      if (warp == 0) issue_chunk(a, smem, &ms.bar_stg, ahead, lane);
      if (tid < kC) load_gb(a, ahead, tid, g_pre, b_pre);
      stg_pending = true;
      cursor_next(a, ahead, false);
    }

    // ---- 1: A (strictly lower, for the solve) and P (lower incl. diagonal) ----
    if (!mma_wait()) { failed = true; break; }
    {
      float vals[32];
      tc::ld_32x32b_x32(T + lane_base + kColKQ + 32 * half, vals);
      tc::ld_wait();
      const int sb = 32 * half;
      if (quad < 2) {
        const int r = lrow;
        const float Gr = ms.G[r], br = ms.bet[r];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          float o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int s = sb + 4 * c4 + e;
            o[e] = (s < r) ? br * vals[4 * c4 + e] * __expf(Gr - ms.G[s]) : 0.0f;
          }
          *reinterpret_cast<float4*>(Am + r * kLd + sb + 4 * c4) = make_float4(o[0], o[1], o[2], o[3]);
        }
      } else {
        const int r = lrow - 64;
        const float Gr = ms.G[r];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          float o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int s = sb + 4 * c4 + e;
            o[e] = (s <= r) ? a.q_scale * vals[4 * c4 + e] * __expf(Gr - ms.G[s]) : 0.0f;
          }
          *reinterpret_cast<float4*>(pm + kf32(r, sb + 4 * c4, 2048)) = make_float4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    tc::fence_before_sync();
    __syncthreads();

    // ---- 2: T = (I + A)^-1 in 16 x 16 blocks ----
    if (tid < 64) {
      // diagonal blocks by forward substitution, one column per thread
      const int b = tid >> 4, c = tid & 15;
      float x[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const float* arow = Am + (16 * b + r) * kLd + 16 * b;
        float acc = 0.0f;
#pragma unroll
        for (int s = 0; s < r; ++s) acc = fmaf(arow[s], x[s], acc);
        x[r] = (r < c) ? 0.0f : (r == c ? 1.0f : -acc);
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) Tm[(16 * b + r) * kLd + 16 * b + c] = x[r];
    } else {
      // zero the blocks above the diagonal
      for (int e = tid - 64; e < 6 * 256; e += kThreads - 64) {
        const int blk = e >> 8, idx = e & 255;
        const int bi = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
        const int bj = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
        Tm[(16 * bi + (idx >> 4)) * kLd + 16 * bj + (idx & 15)] = 0.0f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int ib = 1; ib < 4; ++ib) {
      const int r = tid & 15, jj = tid >> 4;
      // X = A[block row ib][0 : 16 ib] T[0 : 16 ib][0 : 16 ib]
#pragma unroll
      for (int m = 0; m < ib; ++m) {
        const int j = jj + 16 * m;
        const float* arow = Am + (16 * ib + r) * kLd;
        float acc = 0.0f;
#pragma unroll
        for (int kk = 16 * m; kk < 16 * ib; ++kk) acc = fmaf(arow[kk], Tm[kk * kLd + j], acc);
        Xm[r * kLd + j] = acc;
      }
      __syncthreads();
      // T[block row ib][0 : 16 ib] = -D_ib X
#pragma unroll
      for (int m = 0; m < ib; ++m) {
        const int j = jj + 16 * m;
        const float* drow = Tm + (16 * ib + r) * kLd + 16 * ib;
        float acc = 0.0f;
#pragma unroll
        for (int t = 0; t < 16; ++t) acc = fmaf(drow[t], Xm[t * kLd + j], acc);
        Tm[(16 * ib + r) * kLd + j] = -acc;
      }
      __syncthreads();
    }
    // T' = T diag(beta gamma), T'' = T diag(beta) as bf16 B operands ([r][s], K = s)
#pragma unroll
    for (int sp = 0; sp < 2; ++sp) {
      const int r = tid & 63, s8 = 2 * (tid >> 6) + sp;
      const float4 t0v = *reinterpret_cast<const float4*>(Tm + r * kLd + 8 * s8);
      const float4 t1v = *reinterpret_cast<const float4*>(Tm + r * kLd + 8 * s8 + 4);
      const float tv[8] = {t0v.x, t0v.y, t0v.z, t0v.w, t1v.x, t1v.y, t1v.z, t1v.w};
      uint32_t pa[4], pb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int s = 8 * s8 + 2 * e;
        pa[e] = pack_bf16(tv[2 * e] * ms.bg[s], tv[2 * e + 1] * ms.bg[s + 1]);
        pb[e] = pack_bf16(tv[2 * e] * ms.bet[s], tv[2 * e + 1] * ms.bet[s + 1]);
      }
      const uint32_t off = kbf16(r, 8 * s8, 1024);
      *reinterpret_cast<uint4*>(tp + off) = make_uint4(pa[0], pa[1], pa[2], pa[3]);
      *reinterpret_cast<uint4*>(tpp + off) = make_uint4(pb[0], pb[1], pb[2], pb[3]);
    }
    sync_for_mma();
    const bool s0 = s_zero;
    if (tid == 0) {
      // P2: U^T = V^T T''^T  (M = d_v, N = C, K = C)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16_ss(T + kColU, tc::smem_desc(vt + 256 * ks, 128, 1024), tc::smem_desc(tpp + 256 * ks, 128, 1024),
                        id_bf16_64, ks > 0);
      if (!s0) {
        // P3: W^T = K^T T'^T  (M = d_k)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ss(T + kColW, tc::smem_desc(kt + 256 * ks, 128, 1024),
                          tc::smem_desc(tp + 256 * ks, 128, 1024), id_bf16_64, ks > 0);
      }
      tc::commit(&ms.bar_mma);
    }
    if (!mma_wait()) { failed = true; break; }

    // ---- 3: V_new^T = U^T - S^T W^T and O^T = S^T Q'^T (skipped while S = 0) ----
    if (!s0) {
      float vals[32];
      tc::ld_32x32b_x32(T + lane_base + kColW + 32 * half, vals);
      tc::ld_wait();
      const int i = lrow;
#pragma unroll
      for (int c = 0; c < 32; ++c) *reinterpret_cast<float*>(wn + kwn(32 * half + c, i)) = -vals[c];
      sync_for_mma();
      if (tid == 0) {
#pragma unroll
        for (int ks = 0; ks < 16; ++ks)
          tc::mma_tf32_ts(T + kColU, T + kColS + 8 * ks, tc::smem_desc(wn + 2 * kWnLbo * ks, kWnLbo, kWnSbo),
                          id_tf32_64, 1);
#pragma unroll
        for (int ks = 0; ks < 16; ++ks)
          tc::mma_tf32_ts(T + kColO, T + kColS + 8 * ks, tc::smem_desc(qp + 256 * ks, 128, 4096), id_tf32_64,
                          ks > 0);
        tc::commit(&ms.bar_mma);
      }
      if (!mma_wait()) { failed = true; break; }
    }

    // ---- 4: V_new^T -> operands; decay the state ----
    {
      float vals[32];
      tc::ld_32x32b_x32(T + lane_base + kColU + 32 * half, vals);
      tc::ld_wait();
      const int j = lrow, sb = 32 * half;
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4)
        *reinterpret_cast<float4*>(vn + kf32(j, sb + 4 * c4, 2048)) =
            make_float4(vals[4 * c4], vals[4 * c4 + 1], vals[4 * c4 + 2], vals[4 * c4 + 3]);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 8 * c8 + 2 * e;
          w[e] = pack_bf16(vals[c] * ms.de[sb + c], vals[c + 1] * ms.de[sb + c + 1]);
        }
        *reinterpret_cast<uint4*>(vnp + kbf16(j, sb + 8 * c8, 1024)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      if (!s0) {
        const float gC = __expf(Glast);
        float sv[32];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const uint32_t ta = T + lane_base + kColS + 64 * half + 32 * p;
          tc::ld_32x32b_x32(ta, sv);
          tc::ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) sv[c] *= gC;
          tc::st_32x32b_x32(ta, sv);
        }
        tc::st_wait();
      }
    }
    sync_for_mma();
    if (tid == 0) {
      // P6b: O^T += V_new^T P^T  (M = d_v, N = C, K = C)
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        tc::mma_tf32_ss(T + kColO, tc::smem_desc(vn + 256 * ks, 128, 2048), tc::smem_desc(pm + 256 * ks, 128, 2048),
                        id_tf32_64, !s0 || ks > 0);
      // P7: S^T += V_new'^T K  (M = d_v, N = d_k, K = C)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16_ss(T + kColS, tc::smem_desc(vnp + 256 * ks, 128, 1024), tc::smem_desc(kt + 256 * ks, 128, 1024),
                        id_bf16_128, !s0 || ks > 0);
      tc::commit(&ms.bar_mma);
    }
    if (!mma_wait()) { failed = true; break; }
    s_zero = false;

    // ---- 5: O^T -> out (bf16 [T, HV, d_v]) ----
    {
      float vals[32];
      tc::ld_32x32b_x32(T + lane_base + kColO + 32 * half, vals);
      tc::ld_wait();
      const int64_t row_stride = (int64_t)a.HV * kD;
      __nv_bfloat16* ob = a.out + (t0 + 32 * half) * row_stride + (int64_t)h * kD + lrow;
#pragma unroll
      for (int c = 0; c < 32; ++c)
        if (32 * half + c < len) ob[c * row_stride] = __float2bfloat16_rn(vals[c]);
    }
    tc::fence_before_sync();

    // ---- sequence end: requantise the state into its slot ----
    if (last) {
      float* F = reinterpret_cast<float*>(smem + kOffR1);
      float sv[32];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        tc::ld_32x32b_x32(T + lane_base + kColS + 64 * half + 32 * p, sv);
        tc::ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) F[(64 * half + 32 * p + c) * kFPitch + lrow] = sv[c];
      }
      tc::fence_before_sync();
      __syncthreads();
      if (slot >= 0) {
        const int i = tid & 127, hh = tid >> 7;
        float2 x[32];
        const float4* src = reinterpret_cast<const float4*>(F + i * kFPitch + 64 * hh);
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const float4 f = src[p];
          x[2 * p] = make_float2(f.x, f.y);
          x[2 * p + 1] = make_float2(f.z, f.w);
        }
        float am[4];
        float tmax = block_amax4(x, am);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        if (lane == 0) ms.amax[warp] = tmax;
        __syncthreads();
        float amax = ms.amax[0];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) amax = fmaxf(amax, ms.amax[w]);
        const float gs_new = (amax > 0.0f) ? __fdiv_rn(amax, a.gden) : 1.0f;
        const int64_t pt = (int64_t)slot * a.HV + h;
        uint32_t words[8], scw;
        requant_half_row<kMode>(
            x, am, __frcp_rn(gs_new), ms.inv_tab, words, scw,
            a.debug_y ? a.debug_y + (((int64_t)cur.n * a.HV + h) * kD + i) * kD + 64 * hh : nullptr);
        uint4* dst = reinterpret_cast<uint4*>(a.pool_codes + pt * kCodeBytes + i * 64 + 32 * hh);
        dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
        dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
        *reinterpret_cast<uint32_t*>(a.pool_scales + pt * kScaleBytes + i * 8 + 4 * hh) = scw;
        if (tid == 0) a.pool_gs[pt] = gs_new;
      }
      __syncthreads();  // the transpose buffer is free again
    }
    cursor_next(a, cur, tid == 0);
  }

  if (failed && tid == 0) {
    // Report, then give the copies and MMAs still queued a bounded chance to
    // finish before the shared and tensor memory are released.
    atomicOr(a.status, kStatusWaitTimeout);
    if (stg_pending) mbar_wait_bounded(&ms.bar_stg, stg_par, kWaitTimeoutNs / 4);
    if (mma_pending) mbar_wait_bounded(&ms.bar_mma, mma_par, kWaitTimeoutNs / 4);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(T, kTmemCols);
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_prefill(const gdn_prefill_params* p, cudaStream_t stream) {
  if (!p) return GDN_ERR_ARGS;
  if (p->num_seqs < 0 || p->num_k_heads <= 0 || p->num_v_heads <= 0 || p->total_tokens < 0 || p->num_slots < 0)
    return GDN_ERR_ARGS;
  if (p->num_v_heads % p->num_k_heads) return GDN_ERR_ARGS;
  if (p->head_dim != kD) return GDN_ERR_UNSUPPORTED;
  if (p->scale_mode != kScaleRef240 && p->scale_mode != kScaleFn448) return GDN_ERR_UNSUPPORTED;
  if (p->num_seqs == 0 || p->total_tokens == 0) return GDN_OK;
  if (!p->q || !p->k || !p->v || !p->g || !p->beta || !p->cu_seqlens || !p->out) return GDN_ERR_ARGS;
  if (p->slot_idx && (!p->pool_codes || !p->pool_scales || !p->pool_gscale)) return GDN_ERR_ARGS;
  if (p->total_tokens > INT32_MAX) return GDN_ERR_UNSUPPORTED;  // cu_seqlens are int32
  const int64_t nitems = (int64_t)p->num_seqs * p->num_v_heads;
  if (nitems > INT32_MAX / 2) return GDN_ERR_UNSUPPORTED;
  PrefillArgs a;
  a.N = p->num_seqs;
  a.HK = p->num_k_heads;
  a.HV = p->num_v_heads;
  a.group = p->num_v_heads / p->num_k_heads;
  a.nitems = (int32_t)nitems;
  a.T = p->total_tokens;
  a.num_slots = p->num_slots;
  a.q = p->q;
  a.k = p->k;
  a.v = p->v;
  a.q_stride = p->q_stride ? p->q_stride : (int64_t)p->num_k_heads * kD;
  a.k_stride = p->k_stride ? p->k_stride : (int64_t)p->num_k_heads * kD;
  a.v_stride = p->v_stride ? p->v_stride : (int64_t)p->num_v_heads * kD;
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(p->out) ||
      (a.q_stride | a.k_stride | a.v_stride) % 8 || (p->debug_y && !aligned16(p->debug_y)) ||
      (p->slot_idx && (!aligned16(p->pool_codes) || !aligned16(p->pool_scales))))
    return GDN_ERR_ALIGN;
  a.g = p->g;
  a.beta = p->beta;
  a.cu = p->cu_seqlens;
  a.slot_idx = p->slot_idx;
  a.has_init = p->has_initial_state;
  a.pool_codes = p->pool_codes;
  a.pool_scales = p->pool_scales;
  a.pool_gs = p->pool_gscale;
  a.out = p->out;
  a.q_scale = p->q_scale > 0.0f ? p->q_scale : 0.08838834764831845f;  // 1/sqrt(128)
  a.gden = p->gscale_den > 0.0f ? p->gscale_den : default_gden(p->scale_mode);
  if (!(a.gden >= 6.0f && a.gden <= 1.0e6f)) return GDN_ERR_ARGS;
  a.debug_y = p->debug_y;
  a.status = device_status_ptr();
  if (!a.status) return GDN_ERR_CUDA;

  const int smem = (int)kSmemBytes;
  const int64_t max_ctas = sm_count();
  const int grid = (int)(nitems < max_ctas ? nitems : max_ctas);
  static bool attr_set[2][64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GDN_ERR_CUDA;
  const int mi = p->scale_mode == kScaleRef240 ? 0 : 1;
  if (!attr_set[mi][dev]) {
    const cudaError_t e = mi == 0 ? cudaFuncSetAttribute(gdn_prefill_kernel<kScaleRef240>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem)
                                  : cudaFuncSetAttribute(gdn_prefill_kernel<kScaleFn448>,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return GDN_ERR_CUDA;
    attr_set[mi][dev] = true;
  }
  if (mi == 0)
    gdn_prefill_kernel<kScaleRef240><<<grid, kThreads, smem, stream>>>(a);
  else
    gdn_prefill_kernel<kScaleFn448><<<grid, kThreads, smem, stream>>>(a);
  return launch_status();
}
