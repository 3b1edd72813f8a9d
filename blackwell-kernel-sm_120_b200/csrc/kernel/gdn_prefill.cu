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
//   V_new    = U - W S = U - (T diag(beta gamma)) (K S)       (the delta-rule w of every token)
//   O        = q_scale diag(gamma) Q S + P V_new,  P[r][s] = q_scale (q_r . k_s) exp(G_r - G_s), s <= r
//   S_next   = gamma_{C-1} S + sum_s exp(G_{C-1} - G_s) k_s V_new_s^T
// which equals the token-by-token recurrence exactly (in exact arithmetic).
// The reference has no prefill (its serving loop calls the d x d update once
// per token and sequence, src/ops/qwen35_gdn_patch.py:98-116).
//
// One CTA owns one (sequence, value head) at a time and walks its chunks in
// order, in two warp groups that overlap consecutive chunks:
//   prep  (warps 0-7)   the state-independent half of chunk c + 1: P1 = [K; Q] K^T
//                       on the tensor cores, the gates, A and P, the triangular
//                       solve T = (I + A)^-1 (SIMT), T diag(beta) and
//                       -T diag(beta gamma), and P2: U^T = V^T (T diag beta)^T;
//   chain (warps 8-15)  the state chain of chunk c: Y | O1 = S^T [K; Q]^T,
//                       P4: V_new^T = U^T + Y (-T diag(beta gamma))^T (tf32, Y
//                       read from TMEM), V_new^T packed to bf16 in TMEM, the
//                       state decay, P6: O2 = V_new^T P^T and P7: S^T +=
//                       V_new'^T K (both with A in TMEM), the outputs and the
//                       bf16 copy of S for the next chunk.
// The fp32 state stays in tensor memory for the whole sequence, transposed
// (TMEM lane = j over d_v, column = i over d_k).  k and q arrive by TMA
// tensor copies (128-byte swizzle) into a two-stage ring, v into its own
// buffer; the MMAs read them in place.  The groups hand over through
// double-buffered shared memory and TMEM, ordered by mbarriers.  At the end
// of a sequence the state is requantised into its pool slot with the
// reference block quantiser (tile_requant.cuh).  Every wait is bounded.
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
constexpr int kC = 64;
constexpr int kThreads = 512;       // prep warps 0-7, chain warps 8-15
constexpr int kGroup = 256;         // threads per group
constexpr int kBarPrep = 1, kBarChain = 2;  // named hardware barriers of the groups
constexpr int kPrepIssuer = 224;  // prep's MMA / copy issuer: warp 7, which the gate scan does not use
constexpr uint32_t kCodeBytes = kD * kD / 2;
constexpr uint32_t kScaleBytes = kD * kD / 16;

// 64-row x 128-byte TMA boxes, 128-byte swizzled.
constexpr uint32_t kBox = 8192;
constexpr uint32_t kStK0 = 0, kStQ0 = kBox, kStK1 = 2 * kBox, kStQ1 = 3 * kBox;  // one k/q stage
constexpr uint32_t kStageKQ = 4 * kBox;
constexpr uint32_t kV0 = 0, kV1 = kBox;  // the v buffer

// Shared-memory map (bytes).
constexpr uint32_t kOffKQ = 0;                       // 2 k/q stages
constexpr uint32_t kOffV = 2 * kStageKQ;             // v of the chunk the prep group works on
constexpr uint32_t kOffSB = kOffV + 2 * kBox;        // chain: bf16 state copy S^T [j][i]
constexpr uint32_t kOffScr = kOffSB + 32768;         // prep: solve scratch, T diag(beta)
constexpr int kLd = 68;                              // solve scratch row pitch (floats)
constexpr int kXLd = 16;                             // X^T scratch: 64 x 16 floats (6 tiles of 8 x 20 in the solve)
constexpr int kDLd = 20;                             // diagonal-block inverse row pitch (floats)
constexpr uint32_t kSizeScr = 2 * 64 * kLd * 4 + 64 * kXLd * 4 + 64 * kDLd * 4;
constexpr uint32_t kOffHand = kOffScr + kSizeScr;    // prep -> chain, double-buffered
constexpr uint32_t kFPitch = 132;                    // final-state transpose row pitch (floats)

// One prep -> chain hand-over.
struct Hand {
  uint8_t ntp[64 * 64 * 4];  // -T diag(beta gamma), fp32 K-major [r][s]: B of P4
  uint8_t pm[64 * 64 * 2];   // P, bf16 K-major [r][s]: B of P6
  float de[kC];              // exp(G_last - G_s)
  float qg[kC];              // q_scale * gamma_r
  float gC;                  // gamma_{C-1}: the state's decay over the chunk
  float pad[63];
};
constexpr uint32_t kOffMisc = kOffHand + 2 * sizeof(Hand);

struct Misc {
  float gw[kC];    // warp-inclusive scans of g
  float G[kC];     // cumulative log decay
  float bet[kC];   // beta
  float bg[kC];    // beta * gamma
  float al[kC];    // exp(g): one token's decay
  float inv_tab[256];
  float amax[8];
  float nrm[4][kC];  // q/k L2 norm: sums of squares of each token's k (0, 1) and q (2, 3) halves
  float dk[kC];      // 1 / |k_s| (with the norm in the kernel)
  float dq[kC];      // 1 / |q_r|
  uint64_t bar_kq[2];     // k/q stage loaded
  uint64_t bar_v;         // v loaded
  uint64_t bar_p1;        // prep: P1 done
  uint64_t bar_p2[2];     // prep: hand-over written (arrive) and P2 done (commit)
  uint64_t bar_hfree[2];  // chain: hand-over and U[b] read (P4, P6, P7 done)
  uint64_t bar_cm;        // chain: its MMAs done
  uint64_t bar_seq;       // chain: a sequence's final state written, the prep scratch is free
  uint32_t tmem_base;
};
constexpr uint32_t kSmemBytes = kOffMisc + sizeof(Misc);
static_assert(kOffKQ % 1024 == 0 && kOffV % 1024 == 0 && kStageKQ % 1024 == 0, "swizzled boxes: 1024-byte aligned");
static_assert(sizeof(Hand) % 16 == 0 && kOffHand % 16 == 0, "hand-over alignment");
static_assert(kSmemBytes <= 232448, "shared memory");
static_assert(128 * kFPitch * 4 <= 32768 + kSizeScr, "final-state transpose fits SB + scratch");
static_assert(2 * kCodeBytes + 2 * kScaleBytes <= 32768, "initial-state operands fit SB");
static_assert(64 * 64 * 2 <= 64 * kLd * 4, "T diag(beta) fits the A scratch");

// TMEM columns (512 allocated: one CTA per SM)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;     // 128: state S^T (lane j, column i), fp32
constexpr uint32_t kColY = 128;   // 64: Y = S^T K^T   } one N = 128 product
constexpr uint32_t kColO1 = 192;  // 64: S^T Q^T       } S^T [K; Q]^T
constexpr uint32_t kColO2 = 256;  // 64: V_new^T P^T
constexpr uint32_t kColSF = 256;  // 8: initial-state scale factors (sequence start only, over O2)
constexpr uint32_t kColOne = 264; // 8: unit scale factors (likewise)
constexpr uint32_t kColKQ = 320;  // 64: [K K^T; Q K^T] (prep)
constexpr uint32_t kColU = 384;   // 2 x 64: U^T -> V_new^T (fp32) -> [V_new^T | V_new'^T] (bf16 pairs)

struct PrefillArgs {
  int32_t N, HK, HV, group, nitems;
  int64_t T, num_slots;
  const float* g;
  const float* beta;
  const int32_t* cu;
  const int32_t* slot_idx;
  const uint8_t* has_init;
  uint8_t* pool_codes;
  uint8_t* pool_scales;
  float* pool_gs;
  int64_t code_stride, scale_stride, gs_stride;  // bytes between consecutive (slot, head) tiles
  __nv_bfloat16* out;
  float q_scale, gden;
  float* debug_y;
  uint32_t* status;
  int32_t qk_l2norm;  // q and k scaled to unit L2 norm per token and head in the kernel
  // fused gating (A_log == nullptr: g and beta are read)
  const float* A_log;
  const float* dt_bias;
  const __nv_bfloat16* gate_a;
  const __nv_bfloat16* gate_b;
  int64_t gate_stride;
};

// The global scale of pool tile pt (slot * HV + head).
__device__ __forceinline__ float* gs_at(const PrefillArgs& a, int64_t pt) {
  return reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.pool_gs) + pt * a.gs_stride);
}

// Byte offsets in the no-swizzle K-major layouts (16-byte K chunks 128 bytes
// apart, 8-row groups sbo apart).
__device__ __forceinline__ uint32_t kbf16(int row, int k, uint32_t sbo) {
  return (row & 7) * 16 + (k & 7) * 2 + (row >> 3) * sbo + (k >> 3) * 128;
}
__device__ __forceinline__ uint32_t kf32(int row, int k, uint32_t sbo) {
  return (row & 7) * 16 + (k & 3) * 4 + (row >> 3) * sbo + (k >> 2) * 128;
}
__device__ __forceinline__ int canon(int row, int byte) { return (byte & 15) + 16 * row + 2048 * (byte >> 4); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// Named barrier over one warp group.
__device__ __forceinline__ void group_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "n"(kGroup) : "memory");
}
// Named barrier over one warp group that also ORs a predicate across it.
__device__ __forceinline__ bool group_or(int id, bool p) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred pi, po; setp.ne.u32 pi, %1, 0; bar.red.or.pred po, %2, %3, pi; selp.u32 %0, 1, 0, po; }"
      : "=r"(r)
      : "r"((uint32_t)p), "r"(id), "n"(kGroup)
      : "memory");
  return r != 0;
}
// The group's leader waits (bounded); every thread of the group learns the outcome.
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, bool leader, int id) {
  bool ok = true;
  if (leader) ok = mbar_wait_bounded(bar, parity);
  return !group_or(id, !ok);
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

// Queue one of chunk c's four k and q boxes into a stage (part 0 also sets
// the stage's byte count; the four parts are issued by four threads, since
// one copy takes ~100 cycles to issue).  Rows past the end of the tensors
// arrive as zeros; rows past the end of the sequence are masked by the
// consumers (beta = 0, rows not stored).
__device__ __forceinline__ void issue_kq_part(const PrefillArgs& a, uint8_t* stage, uint64_t* bar, const Cursor& c,
                                              const CUtensorMap* tq, const CUtensorMap* tk, int part) {
  const int t0 = (int)(c.bos + c.chunk * kC);
  const int hk = c.h / a.group;
  if (part == 0) mbar_arrive_expect_tx(bar, kStageKQ);
  const uint32_t off = part == 0 ? kStK0 : part == 1 ? kStK1 : part == 2 ? kStQ0 : kStQ1;
  tc::tma_load_3d(stage + off, part < 2 ? tk : tq, 64 * (part & 1), hk, t0, bar);
}

__device__ __forceinline__ void issue_v_part(const PrefillArgs& a, uint8_t* vbuf, uint64_t* bar, const Cursor& c,
                                             const CUtensorMap* tv, int part) {
  const int t0 = (int)(c.bos + c.chunk * kC);
  if (part == 0) mbar_arrive_expect_tx(bar, 2 * kBox);
  tc::tma_load_3d(vbuf + (part ? kV1 : kV0), tv, 64 * part, c.h, t0, bar);
}

// Threads 0..63: g and beta of token `r` of chunk c (0 past the chunk end).
__device__ __forceinline__ void load_gb(const PrefillArgs& a, const Cursor& c, int r, float& gv, float& bv) {
  gv = 0.0f;
  bv = 0.0f;
  if (c.item < a.nitems && r < chunk_len(c)) {
    const int64_t idx = (c.bos + c.chunk * kC + r) * a.HV + c.h;
    if (a.A_log) {  // g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) (vLLM's gating)
      const int64_t gi = (c.bos + c.chunk * kC + r) * a.gate_stride + c.h;
      const float xa = __bfloat162float(a.gate_a[gi]) + __ldg(a.dt_bias + c.h);
      const float sp = xa > 20.0f ? xa : log1pf(expf(xa));  // torch.nn.functional.softplus, threshold 20
      gv = -expf(__ldg(a.A_log + c.h)) * sp;
      bv = 1.0f / (1.0f + expf(-__bfloat162float(a.gate_b[gi])));
    } else {
      gv = __ldg(a.g + idx);
      bv = __ldg(a.beta + idx);
    }
  }
}

// K-major descriptor of rows [0, 64 or 128) of a stage's K or [K; Q], K step ks (16 elements).
__device__ __forceinline__ uint64_t stage_kmajor(const uint8_t* stage, uint32_t box0, int ks) {
  return tc::smem_desc_sw128(stage + box0 + (ks < 4 ? 0u : 2u * kBox) + 32u * (ks & 3), 16, 1024);
}

// The slot of a sequence (-1: none or out of range) and whether it starts from the pool state.
__device__ __forceinline__ int32_t seq_slot(const PrefillArgs& a, int n, bool report, bool& has) {
  int32_t slot = a.slot_idx ? __ldg(a.slot_idx + n) : -1;
  if (slot >= a.num_slots) {
    if (report) atomicOr(a.status, GDN_STATUS_BAD_SLOT);
    slot = -1;
  }
  if (slot < 0) slot = -1;
  has = slot >= 0 && a.has_init && __ldg(a.has_init + n) != 0;
  return slot;
}


__device__ __forceinline__ void mma_16x8x8_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// d (16 x 8) += a (16 x 8) b (8 x 8) on the tensor cores with fp32 operands
// read as tf32 (the MMA uses the top 19 bits of each, i.e. truncates the
// significand to 10 bits; fp32 accumulate).  Warp-level fragments (PTX mma.m16n8k8
// .tf32): lane l, group g = l / 4, t = l % 4, holds a at rows g, g + 8 and
// columns t, t + 4 (a0 = [g][t], a1 = [g + 8][t], a2 = [g][t + 4],
// a3 = [g + 8][t + 4]), b at rows t, t + 4 of column g, and d at rows g,
// g + 8, columns 2t, 2t + 1.
__device__ __forceinline__ void mma_16x8x8_f(float (&d)[4], float a0, float a1, float a2, float a3, float b0,
                                             float b1) {
  mma_16x8x8_tf32(d, __float_as_uint(a0), __float_as_uint(a1), __float_as_uint(a2), __float_as_uint(a3),
                  __float_as_uint(b0), __float_as_uint(b1));
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_prefill_kernel(const PrefillArgs a, const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ __align__(1024) uint8_t smem[];
  Misc& ms = *reinterpret_cast<Misc*>(smem + kOffMisc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = (warp >> 2) & 1;
  const int lrow = 32 * quad + lane;  // this thread's TMEM lane
  const uint32_t lane_base = (uint32_t)(32 * quad) << 16;

  // The swizzled boxes need a 1024-byte aligned window.
  if ((smem_u32(smem) & 1023u) != 0) {
    if (tid == 0) atomicOr(a.status, kStatusWaitTimeout);
    return;
  }
  Hand* const hand = reinterpret_cast<Hand*>(smem + kOffHand);
  uint8_t* const vbuf = smem + kOffV;
  uint8_t* const sb = smem + kOffSB;

  if (tid < 256) ms.inv_tab[tid] = scale_inverse(scale_decode((uint32_t)tid, kMode));
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ms.bar_kq[b], 1);
      mbar_init(&ms.bar_p2[b], 2);
      mbar_init(&ms.bar_hfree[b], 1);
    }
    mbar_init(&ms.bar_v, 1);
    mbar_init(&ms.bar_p1, 1);
    mbar_init(&ms.bar_cm, 1);
    mbar_init(&ms.bar_seq, 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&ms.tmem_base, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t T = ms.tmem_base;
  bool failed = false;

  if (warp < 8) {
    // ================================== prep ==================================
    float* const Am = reinterpret_cast<float*>(smem + kOffScr);
    float* const Tt = Am + 64 * kLd;   // T^T: Tt[j * kLd + r] = T[r][j]
    float* const Xt = Tt + 64 * kLd;   // per-warp X^T tiles of the block-row solve (8 x 20 floats each)
    float* const Dm = Xt + 64 * kXLd;  // the diagonal blocks of T, row-major: Dm[(16 b + r) * kDLd + c]
    uint8_t* const tpp = smem + kOffScr;  // T diag(beta), bf16 K-major [r][s], over A once A is consumed
    const uint32_t id_kq = tc::idesc_bf16(128, 64);
    const uint32_t id_u = tc::idesc_bf16(128, 64, true, false);
    Cursor cur{(int32_t)blockIdx.x, 0, 0, 0, 0, 0};
    cursor_seek(a, cur, false);
    float g_pre = 0.0f, b_pre = 0.0f;
    if (tid < kC) load_gb(a, cur, tid, g_pre, b_pre);
    uint32_t g = 0, nseq = 0;
    while (cur.item < a.nitems) {
      const int b = g & 1;
      uint8_t* const stage = smem + kOffKQ + b * kStageKQ;
      Hand& hd = hand[b];
      const bool last = (cur.chunk + 1) * kC >= cur.len;

      // ---- P1 = [K; Q] K^T as soon as the stage has landed (the issuer, while warps 0-1 scan the gates) ----
      bool kq_ok = true;
      if (tid == kPrepIssuer) {
        kq_ok = mbar_wait_bounded(&ms.bar_kq[b], (g >> 1) & 1);
        if (kq_ok) {
          tc::fence_after_sync();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t dk = stage_kmajor(stage, kStK0, ks);
            tc::mma_bf16_ss(T + kColKQ, dk, dk, id_kq, ks > 0);  // rows 64..127 of A are Q's box
          }
          tc::commit(&ms.bar_p1);
        }
      }
      // ---- gates ----
      const float gv = g_pre, bv = b_pre;
      if (tid < kC) {
        float s = gv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, s, o);
          if (lane >= o) s += y;
        }
        ms.gw[tid] = s;
        Cursor nx = cur;  // prefetch g, beta of the next chunk
        cursor_next(a, nx, false);
        load_gb(a, nx, tid, g_pre, b_pre);
      }
      group_sync(kBarPrep);
      if (a.qk_l2norm) {
        // Sum of squares of one token's half-row of k or q (the issuer saw the
        // stage land before the barrier above).  The 128-byte swizzle only
        // permutes the 16-byte chunks of a row, so a row's sum reads it as stored.
        const int box = tid >> 6, r = tid & 63;
        const uint32_t off = box == 0 ? kStK0 : box == 1 ? kStK1 : box == 2 ? kStQ0 : kStQ1;
        const uint4* row = reinterpret_cast<const uint4*>(stage + off + 128 * r);
        float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 w = row[c];
          const uint32_t ws4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws4[e]));
            acc = __ffma2_rn(f, f, acc);
          }
        }
        ms.nrm[box][r] = acc.x + acc.y;
      }
      float h_de = 0.0f, h_qg = 0.0f, h_gC = 0.0f;
      if (tid < kC) {
        const float G = ms.gw[tid] + (tid >= 32 ? ms.gw[31] : 0.0f);
        const float Glast = ms.gw[63] + ms.gw[31];
        const float gm = __expf(G);
        ms.G[tid] = G;
        ms.bet[tid] = bv;
        ms.bg[tid] = bv * gm;
        ms.al[tid] = __expf(gv);
        h_de = __expf(Glast - G);
        h_qg = a.q_scale * gm;
        h_gC = __expf(Glast);
      }
      // ---- P1 done (and with it the previous chunk's P2: the v buffer and T diag(beta) are free), and
      //      the hand-over buffer free (the chain has finished chunk g - 2): one wait for the group ----
      {
        bool ok = kq_ok;
        if (tid == kPrepIssuer) {
          if (ok && g >= 2) ok = mbar_wait_bounded(&ms.bar_hfree[b], ((g - 2) >> 1) & 1);
          if (ok) ok = mbar_wait_bounded(&ms.bar_p1, g & 1);
        }
        if (group_or(kBarPrep, !ok)) { failed = true; break; }
      }
      tc::fence_after_sync();
      if (tid < kC) {
        if (a.qk_l2norm) {
          // x / sqrt(sum x^2 + 1e-6) of k_s and q_r folded into every product
          // that reads k or q: A, P (below), -T diag(beta gamma) (through bg),
          // the state update (through de) and the output (through qg)
          const float dk = 1.0f / sqrtf((ms.nrm[0][tid] + ms.nrm[1][tid]) + 1e-6f);
          const float dq = 1.0f / sqrtf((ms.nrm[2][tid] + ms.nrm[3][tid]) + 1e-6f);
          ms.dk[tid] = dk;
          ms.dq[tid] = dq;
          ms.bg[tid] *= dk;
          h_de *= dk;
          h_qg *= dq;
        }
        hd.de[tid] = h_de;
        hd.qg[tid] = h_qg;
        if (tid == 0) hd.gC = h_gC;
      }
      if (a.qk_l2norm) group_sync(kBarPrep);
      if (tid == kPrepIssuer || tid == kPrepIssuer - 32)
        issue_v_part(a, vbuf, &ms.bar_v, cur, &tm_v, tid == kPrepIssuer ? 0 : 1);

      // ---- A (strictly lower, for the solve) and P (lower incl. diagonal) ----
      // The decay exp(G_r - G_s) of this thread's columns s in [sb0, sb0 + 32)
      // comes from one exp at the last column s_hi <= r and a running product of
      // per-token decays towards smaller s (exp(G_r - G_{s-1}) = exp(G_r - G_s)
      // exp(g_s)): one exp per thread instead of one per element.
      {
        float vals[32];
        tc::ld_32x32b_x32(T + lane_base + kColKQ + 32 * half, vals);
        tc::ld_wait();
        const int sb0 = 32 * half;
        const bool arow = quad < 2;                  // rows 0-63: K K^T -> A; rows 64-127: Q K^T -> P
        const int r = arow ? lrow : lrow - 64;
        const int s_hi = arow ? r - 1 : r;           // last column kept
        const float Gr = ms.G[r];
        float scale = arow ? ms.bet[r] : a.q_scale;
        if (a.qk_l2norm) scale *= arow ? ms.dk[r] : ms.dq[r];
        const int s_top = s_hi < sb0 + 31 ? s_hi : sb0 + 31;
        float f = (s_top >= sb0) ? __expf(Gr - ms.G[s_top]) : 0.0f;
        float alv[33];  // exp(g) of tokens sb0 .. sb0 + 32, in registers before the chain
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 t = *reinterpret_cast<const float4*>(ms.al + sb0 + 4 * c4);
          alv[4 * c4] = t.x;
          alv[4 * c4 + 1] = t.y;
          alv[4 * c4 + 2] = t.z;
          alv[4 * c4 + 3] = t.w;
        }
        alv[32] = half ? 1.0f : ms.al[32];  // token 64 does not exist (never used: s < s_top <= 63)
#pragma unroll
        for (int e = 31; e >= 0; --e) {
          const int s = sb0 + e;
          if (s < s_top) f *= alv[e + 1];
          vals[e] = (s <= s_top) ? scale * vals[e] * f : 0.0f;
        }
        if (a.qk_l2norm) {  // column s: 1 / |k_s|
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            const float4 d4 = *reinterpret_cast<const float4*>(ms.dk + sb0 + 4 * c4);
            vals[4 * c4] *= d4.x;
            vals[4 * c4 + 1] *= d4.y;
            vals[4 * c4 + 2] *= d4.z;
            vals[4 * c4 + 3] *= d4.w;
          }
        }
        if (arow) {
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4)
            *reinterpret_cast<float4*>(Am + r * kLd + sb0 + 4 * c4) =
                make_float4(vals[4 * c4], vals[4 * c4 + 1], vals[4 * c4 + 2], vals[4 * c4 + 3]);
        } else {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8)
            *reinterpret_cast<uint4*>(hd.pm + kbf16(r, sb0 + 8 * c8, 1024)) =
                make_uint4(pack_bf16(vals[8 * c8], vals[8 * c8 + 1]), pack_bf16(vals[8 * c8 + 2], vals[8 * c8 + 3]),
                           pack_bf16(vals[8 * c8 + 4], vals[8 * c8 + 5]), pack_bf16(vals[8 * c8 + 6], vals[8 * c8 + 7]));
        }
      }
      tc::fence_before_sync();  // KQ is read before the next P1 overwrites it
      group_sync(kBarPrep);
      // ---- 2: T = (I + A)^-1 in 16 x 16 blocks ----
      // T is kept transposed (a column of T is a contiguous row of Tt) so that
      // the block products read both operands with 16-byte loads.
      if (tid < 64) {
        // diagonal blocks by forward substitution, one column per thread
        const int b = tid >> 4, c = tid & 15;
        float x[16];
  #pragma unroll
        for (int r = 0; r < 16; ++r) {
          const float4* arow = reinterpret_cast<const float4*>(Am + (16 * b + r) * kLd + 16 * b);
          float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  #pragma unroll
          for (int s4 = 0; s4 < (r + 3) / 4; ++s4) {
            const float4 av = arow[s4];
            const float aa[4] = {av.x, av.y, av.z, av.w};
  #pragma unroll
            for (int e = 0; e < 4; ++e)
              if (4 * s4 + e < r) acc[e] = fmaf(aa[e], x[4 * s4 + e], acc[e]);
          }
          const float sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
          x[r] = (r < c) ? 0.0f : (r == c ? 1.0f : -sum);
        }
        float4* tcol = reinterpret_cast<float4*>(Tt + (16 * b + c) * kLd + 16 * b);
  #pragma unroll
        for (int r4 = 0; r4 < 4; ++r4) tcol[r4] = make_float4(x[4 * r4], x[4 * r4 + 1], x[4 * r4 + 2], x[4 * r4 + 3]);
  #pragma unroll
        for (int r = 0; r < 16; ++r) Dm[(16 * b + r) * kDLd + c] = x[r];
      } else {
        // zero the blocks above the diagonal: T[i][j] = Tt[j][i] with block(i) < block(j)
        for (int e = tid - 64; e < 6 * 256; e += kGroup - 64) {
          const int blk = e >> 8, idx = e & 255;
          const int bi = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
          const int bj = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
          Tt[(16 * bj + (idx >> 4)) * kLd + 16 * bi + (idx & 15)] = 0.0f;
        }
      }
      group_sync(kBarPrep);
      // Block rows 1-3 on warp-level tensor-core MMAs (m16n8k8, tf32 operands):
      // warp w < 2 ib owns the 8 columns n0 = 8 w of block row ib and needs no
      // other warp until the row is done.
      // X = A[block row ib][.] T[.][n0 : n0 + 8] over the K steps where that
      // column strip of T is nonzero, then T[block row ib][n0 : n0 + 8] =
      // -D_ib X through an 8 x 16 scratch tile of its own (pitch 20:
      // conflict-free fragment stores and loads).  The m16n8k8 shape fits these
      // 16-row products; tcgen05 MMAs start at 64 rows.
      const int fg = lane >> 2, ft = lane & 3;  // fragment group and thread-in-group
  #pragma unroll
      for (int ib = 1; ib < 4; ++ib) {
        if (warp < 2 * ib) {
          const int n0 = 8 * warp;
          float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int k = 16 * (n0 >> 4); k < 16 * ib; k += 8) {
            const float* ar = Am + (16 * ib + fg) * kLd + k + ft;
            const float* tr = Tt + (n0 + fg) * kLd + k + ft;
            mma_16x8x8_f(acc, ar[0], ar[8 * kLd], ar[4], ar[8 * kLd + 4], tr[0], tr[4]);
          }
          float* const xw = Xt + 160 * warp;  // X^T tile: xw[n * 20 + k] = X[k][n0 + n]
          xw[(2 * ft) * 20 + fg] = acc[0];
          xw[(2 * ft + 1) * 20 + fg] = acc[1];
          xw[(2 * ft) * 20 + fg + 8] = acc[2];
          xw[(2 * ft + 1) * 20 + fg + 8] = acc[3];
          __syncwarp();
          float acc2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  #pragma unroll
          for (int k2 = 0; k2 < 16; k2 += 8) {
            const float* dr = Dm + (16 * ib + fg) * kDLd + k2 + ft;
            const float* xr = xw + fg * 20 + k2 + ft;
            mma_16x8x8_f(acc2, dr[0], dr[8 * kDLd], dr[4], dr[8 * kDLd + 4], xr[0], xr[4]);
          }
          Tt[(n0 + 2 * ft) * kLd + 16 * ib + fg] = -acc2[0];
          Tt[(n0 + 2 * ft + 1) * kLd + 16 * ib + fg] = -acc2[1];
          Tt[(n0 + 2 * ft) * kLd + 16 * ib + fg + 8] = -acc2[2];
          Tt[(n0 + 2 * ft + 1) * kLd + 16 * ib + fg + 8] = -acc2[3];
          __syncwarp();  // the scratch tile is read before the next block row rewrites it
        }
        group_sync(kBarPrep);
      }
      // ---- T diag(beta) as bf16 (over A, consumed by the solve), -T diag(beta gamma) as fp32 ----
#pragma unroll
      for (int sp = 0; sp < 2; ++sp) {
        const int r = tid & 63, s8 = 2 * (tid >> 6) + sp;
        float tv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) tv[e] = Tt[(8 * s8 + e) * kLd + r];
        uint32_t pb[4];
        float nt[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) nt[e] = -tv[e] * ms.bg[8 * s8 + e];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          pb[e] = pack_bf16(tv[2 * e] * ms.bet[8 * s8 + 2 * e], tv[2 * e + 1] * ms.bet[8 * s8 + 2 * e + 1]);
        *reinterpret_cast<uint4*>(tpp + kbf16(r, 8 * s8, 1024)) = make_uint4(pb[0], pb[1], pb[2], pb[3]);
        *reinterpret_cast<float4*>(hd.ntp + kf32(r, 8 * s8, 2048)) = make_float4(nt[0], nt[1], nt[2], nt[3]);
        *reinterpret_cast<float4*>(hd.ntp + kf32(r, 8 * s8 + 4, 2048)) = make_float4(nt[4], nt[5], nt[6], nt[7]);
      }
      tc::fence_smem_to_async();
      // ---- v landed: P2 into U[b] (free since bar_hfree above); hand over to the chain ----
      if (!group_wait(&ms.bar_v, g & 1, tid == kPrepIssuer, kBarPrep)) { failed = true; break; }
      if (tid == kPrepIssuer) {
        tc::fence_after_sync();
        // P2: U^T = V^T T''^T  (A = V as MN-major, M = d_v, N = C, K = C)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ss(T + kColU + 64 * b, tc::smem_desc_sw128(vbuf + kV0 + 2048 * ks, kBox, 1024),
                          tc::smem_desc(tpp + 256 * ks, 128, 1024), id_u, ks > 0);
        mbar_arrive(&ms.bar_p2[b]);  // the hand-over (written before the barrier above) is published
        tc::commit(&ms.bar_p2[b]);
      }
      if (last) {
        // the chain transposes the final state through this group's scratch: wait for it
        if (!group_wait(&ms.bar_seq, nseq & 1, tid == kPrepIssuer, kBarPrep)) { failed = true; break; }
        ++nseq;
      }
      ++g;
      cursor_next(a, cur, false);
    }
  } else {
    // ================================== chain ==================================
    const int ctid = tid - kGroup;  // 0..255
    const uint32_t id_yo = tc::idesc_bf16(128, 128);
    const uint32_t id_o2 = tc::idesc_bf16(128, 64);
    const uint32_t id_s = tc::idesc_bf16(128, 128, false, true);
    const uint32_t id_tf = tc::idesc_tf32(128, 64);
    const uint32_t id_mx = tc::idesc_mxf4nvf4(128, 128);
    const int64_t row_stride = (int64_t)a.HV * kD;
    Cursor cur{(int32_t)blockIdx.x, 0, 0, 0, 0, 0};
    cursor_seek(a, cur, ctid == 0);
    Cursor ahead = cur;  // next chunk whose k/q to load
    for (int b = 0; b < 2; ++b) {
      if (ahead.item < a.nitems) {
        if (lane == 0 && warp < 12) issue_kq_part(a, smem + kOffKQ + b * kStageKQ, &ms.bar_kq[b], ahead, &tm_q, &tm_k, warp - 8);
        cursor_next(a, ahead, false);
      }
    }
    uint32_t g = 0, cm_par = 0;
    int32_t slot = -1;
    bool s_zero = true;  // the state is zero (not yet in TMEM / the bf16 copy)
    auto cm_wait = [&]() -> bool {
      const bool ok = group_wait(&ms.bar_cm, cm_par, ctid == 0, kBarChain);
      cm_par ^= 1u;
      tc::fence_after_sync();
      return ok;
    };
    while (cur.item < a.nitems) {
      const int b = g & 1;
      uint8_t* const stage = smem + kOffKQ + b * kStageKQ;
      Hand& hd = hand[b];
      const int h = cur.h;
      const int64_t t0 = cur.bos + cur.chunk * kC;
      const int len = chunk_len(cur);
      const bool last = (cur.chunk + 1) * kC >= cur.len;
      const uint32_t ub = T + kColU + 64 * b;

      // ---- sequence start: slot and initial state ----
      if (cur.chunk == 0) {
        bool has = false;
        slot = seq_slot(a, cur.n, ctid == 0, has);
        s_zero = !has;
        if (has) {
          // Decode the NVFP4 tile straight into TMEM with one block-scaled MMA
          // against the identity: D = I * S^T (lane j, column i).
          const int64_t pt = (int64_t)slot * a.HV + h;
          uint8_t* const codes = sb;
          uint8_t* const ident = codes + kCodeBytes;
          uint8_t* const sf = ident + kCodeBytes;
          uint8_t* const sf_one = sf + kScaleBytes;
          {
            const int r = ctid >> 1, c0 = 2 * (ctid & 1);
            const uint4* src = reinterpret_cast<const uint4*>(a.pool_codes + pt * a.code_stride + r * 64 + 16 * c0);
            const uint4 x0 = __ldg(src), x1 = __ldg(src + 1);
            *reinterpret_cast<uint4*>(codes + 2048 * c0 + 16 * r) = x0;
            *reinterpret_cast<uint4*>(codes + 2048 * (c0 + 1) + 16 * r) = x1;
            const int t = ctid >> 7, m0 = (ctid & 127) >> 2, m1 = ctid & 3;
            reinterpret_cast<uint32_t*>(sf)[t * 128 + m0 * 4 + m1] =
                __ldg(reinterpret_cast<const uint32_t*>(a.pool_scales + pt * a.scale_stride) + (32 * m1 + m0) * 2 + t);
            reinterpret_cast<uint32_t*>(sf_one)[ctid] = 0x38383838u;  // UE4M3 1.0
            for (int e = ctid; e < (int)kCodeBytes; e += kGroup) {
              const int rr = e >> 6, byte = e & 63;
              uint8_t val = 0;
              if (2 * byte == rr) val = 0x02;      // E2M1 1.0, low nibble
              if (2 * byte + 1 == rr) val = 0x20;  // high nibble
              ident[canon(rr, byte)] = val;
            }
          }
          const float gs = __ldg(gs_at(a, pt));
          tc::fence_smem_to_async();
          tc::fence_before_sync();
          group_sync(kBarChain);
          if (ctid == 0) {
            tc::fence_after_sync();
            for (int t = 0; t < 2; ++t) {
              tc::cp_32x128b_warpx4(T + kColSF + 4 * t, tc::smem_desc(sf + 512 * t, 0, 128));
              tc::cp_32x128b_warpx4(T + kColOne + 4 * t, tc::smem_desc(sf_one + 512 * t, 0, 128));
            }
            for (int t = 0; t < 2; ++t)
              tc::mma_mxf4nvf4(T + kColS, tc::smem_desc(ident + 4096 * t, 2048, 128),
                               tc::smem_desc(codes + 4096 * t, 2048, 128), id_mx, T + kColOne + 4 * t,
                               T + kColSF + 4 * t, t > 0);
            tc::commit(&ms.bar_cm);
          }
          if (!cm_wait()) { failed = true; break; }
          // S *= gs in TMEM; the bf16 copy for the state products (over the decode operands)
          float sv[32];
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            const uint32_t ta = T + lane_base + kColS + 64 * half + 32 * p;
            tc::ld_32x32b_x32(ta, sv);
            tc::ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) sv[c] *= gs;
            tc::st_32x32b_x32(ta, sv);
            group_sync(kBarChain);  // every thread's reads of the decode operands precede the overwrite
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
              const int i = 64 * half + 32 * p + 8 * c8;
              *reinterpret_cast<uint4*>(sb + kbf16(lrow, i, 2048)) =
                  make_uint4(pack_bf16(sv[8 * c8], sv[8 * c8 + 1]), pack_bf16(sv[8 * c8 + 2], sv[8 * c8 + 3]),
                             pack_bf16(sv[8 * c8 + 4], sv[8 * c8 + 5]), pack_bf16(sv[8 * c8 + 6], sv[8 * c8 + 7]));
            }
          }
          tc::st_wait();
          tc::fence_smem_to_async();
          tc::fence_before_sync();
          group_sync(kBarChain);
        }
      }
      const bool s0 = s_zero;

      // ---- Y | O1 = S^T [K; Q]^T once the stage has landed ----
      if (!group_wait(&ms.bar_kq[b], (g >> 1) & 1, ctid == 0, kBarChain)) { failed = true; break; }
      if (ctid == 0 && !s0) {
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16_ss(T + kColY, tc::smem_desc(sb + 256 * ks, 128, 2048), stage_kmajor(stage, kStK0, ks), id_yo,
                          ks > 0);
      }
      // ---- the prep group's hand-over: P4, V_new^T = U^T + Y (-T')^T ----
      if (!group_wait(&ms.bar_p2[b], (g >> 1) & 1, ctid == 0, kBarChain)) { failed = true; break; }
      if (ctid == 0) {
        tc::fence_after_sync();
        if (!s0) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            tc::mma_tf32_ts(ub, T + kColY + 8 * ks, tc::smem_desc(hd.ntp + 256 * ks, 128, 2048), id_tf, 1);
        }
        tc::commit(&ms.bar_cm);
      }
      if (!cm_wait()) { failed = true; break; }

      // ---- V_new^T -> bf16 [V_new^T | V_new^T diag(exp(G_last - G))] in U[b]; decay the state ----
      {
        float vals[32];
        tc::ld_32x32b_x32(ub + lane_base + 32 * half, vals);
        tc::ld_wait();
        uint32_t wn[16], wd[16];
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const int s = 32 * half + 2 * p;
          wn[p] = pack_bf16(vals[2 * p], vals[2 * p + 1]);
          wd[p] = pack_bf16(vals[2 * p] * hd.de[s], vals[2 * p + 1] * hd.de[s + 1]);
        }
        tc::fence_before_sync();
        group_sync(kBarChain);  // every lane's V_new^T is read before U[b] is overwritten
        tc::fence_after_sync();
        tc::st_32x32b_x16(ub + lane_base + 16 * half, wn);
        tc::st_32x32b_x16(ub + lane_base + 32 + 16 * half, wd);
        if (!s0) {
          const float gC = hd.gC;
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
        }
        tc::st_wait();
      }
      tc::fence_before_sync();
      group_sync(kBarChain);
      if (ctid == 0) {
        tc::fence_after_sync();
        // P6: O2 = V_new^T P^T  (A = V_new^T bf16 in TMEM, M = d_v, N = C, K = C)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ts(T + kColO2, ub + 8 * ks, tc::smem_desc(hd.pm + 256 * ks, 128, 1024), id_o2, ks > 0);
        // P7: S^T += V_new'^T K  (A in TMEM, B = K as MN-major, N = d_k)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ts(T + kColS, ub + 32 + 8 * ks, tc::smem_desc_sw128(stage + kStK0 + 2048 * ks, 2 * kBox, 1024),
                          id_s, !s0 || ks > 0);
        tc::commit(&ms.bar_cm);
        tc::commit(&ms.bar_hfree[b]);  // the hand-over and U[b] are free once these complete
      }
      if (!cm_wait()) { failed = true; break; }
      s_zero = false;
      // The stage is free: queue the chunk after next into it.
      if (ahead.item < a.nitems) {
        if (lane == 0 && warp >= 12) issue_kq_part(a, stage, &ms.bar_kq[b], ahead, &tm_q, &tm_k, warp - 12);
        cursor_next(a, ahead, false);
      }

      // ---- bf16 copy of the updated state for the next chunk's state products ----
      if (!last) {
        float sv[32];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          tc::ld_32x32b_x32(T + lane_base + kColS + 64 * half + 32 * p, sv);
          tc::ld_wait();
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const int i = 64 * half + 32 * p + 8 * c8;
            *reinterpret_cast<uint4*>(sb + kbf16(lrow, i, 2048)) =
                make_uint4(pack_bf16(sv[8 * c8], sv[8 * c8 + 1]), pack_bf16(sv[8 * c8 + 2], sv[8 * c8 + 3]),
                           pack_bf16(sv[8 * c8 + 4], sv[8 * c8 + 5]), pack_bf16(sv[8 * c8 + 6], sv[8 * c8 + 7]));
          }
        }
        tc::fence_smem_to_async();
      }
      // ---- outputs O = diag(q_scale gamma) O1 + O2 -> bf16, straight to global (lanes j: 64-byte rows) ----
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {
        float v2[16], v1[16];
        const uint32_t col = 32 * half + 16 * hc;
        tc::ld_32x32b_x16(T + lane_base + kColO2 + col, v2);
        if (!s0) tc::ld_32x32b_x16(T + lane_base + kColO1 + col, v1);
        tc::ld_wait();
        // Rows r, r + 1 per step: an even lane j stores (j, j + 1) of row r, an odd lane (j - 1, j) of
        // row r + 1, after one shuffle with its neighbour: 4-byte stores, one paired conversion.
        const bool odd = lane & 1;
        uint32_t* orow = reinterpret_cast<uint32_t*>(a.out + (t0 + col + (odd ? 1 : 0)) * row_stride +
                                                     (int64_t)h * kD + (lrow & ~1));
#pragma unroll
        for (int c = 0; c < 16; c += 2) {
          const int r = col + c;
          const float o0 = s0 ? v2[c] : fmaf(hd.qg[r], v1[c], v2[c]);
          const float o1 = s0 ? v2[c + 1] : fmaf(hd.qg[r + 1], v1[c + 1], v2[c + 1]);
          const float x = __shfl_xor_sync(0xffffffffu, odd ? o0 : o1, 1);
          const uint32_t pk = odd ? pack_bf16(x, o1) : pack_bf16(o0, x);
          if (r + (odd ? 1 : 0) < len) *orow = pk;
          orow += row_stride;  // two rows of row_stride / 2 words
        }
      }
      tc::fence_before_sync();
      group_sync(kBarChain);  // the bf16 state copy is complete and O1, O2 are read

      // ---- sequence end: requantise the state into its slot (through the prep scratch, which is idle) ----
      if (last) {
        float* F = reinterpret_cast<float*>(smem + kOffSB);
        float sv[32];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          tc::ld_32x32b_x32(T + lane_base + kColS + 64 * half + 32 * p, sv);
          tc::ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) F[(64 * half + 32 * p + c) * kFPitch + lrow] = sv[c];
        }
        tc::fence_before_sync();
        group_sync(kBarChain);
        if (slot >= 0) {
          const int i = ctid & 127, hh = ctid >> 7;
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
          if (lane == 0) ms.amax[warp - 8] = tmax;
          group_sync(kBarChain);
          float amax = ms.amax[0];
#pragma unroll
          for (int w = 1; w < 8; ++w) amax = fmaxf(amax, ms.amax[w]);
          const float gs_new = (amax > 0.0f) ? __fdiv_rn(amax, a.gden) : 1.0f;
          const int64_t pt = (int64_t)slot * a.HV + h;
          uint32_t words[8], scw;
          requant_half_row<kMode>(
              x, am, __frcp_rn(gs_new), ms.inv_tab, words, scw,
              a.debug_y ? a.debug_y + (((int64_t)cur.n * a.HV + h) * kD + i) * kD + 64 * hh : nullptr);
          uint4* dst = reinterpret_cast<uint4*>(a.pool_codes + pt * a.code_stride + i * 64 + 32 * hh);
          dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
          dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
          *reinterpret_cast<uint32_t*>(a.pool_scales + pt * a.scale_stride + i * 8 + 4 * hh) = scw;
          if (ctid == 0) *gs_at(a, pt) = gs_new;
        }
        group_sync(kBarChain);  // the transpose buffer is read
        if (ctid == 0) mbar_arrive(&ms.bar_seq);  // the prep group's scratch is free again
      }
      ++g;
      cursor_next(a, cur, ctid == 0);
    }
  }

  if (failed && (tid == 0 || tid == kGroup)) {
    // Report, then give the copies and MMAs still queued a bounded time to
    // finish before the shared and tensor memory are released.
    atomicOr(a.status, kStatusWaitTimeout);
    const uint64_t t_end = globaltimer_ns() + 200000ull;
    while (globaltimer_ns() < t_end) {
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(T, kTmemCols);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
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

// Tensor map over rows [T][heads][128] bf16 (token stride in elements): boxes of
// 64 tokens x 64 features of one head, 128-byte swizzled, zero fill past T.
bool make_row_map(CUtensorMap* m, const void* base, int64_t heads, int64_t T, int64_t token_stride) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)heads, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)token_stride * 2};
  const cuuint32_t box[3] = {64, 1, 64};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
  if (!p->q || !p->k || !p->v || (!p->A_log && (!p->g || !p->beta)) || !p->cu_seqlens || !p->out)
    return GDN_ERR_ARGS;
  const int64_t gate_stride = p->gate_stride ? p->gate_stride : p->num_v_heads;
  if (p->A_log && (!p->dt_bias || !p->gate_a || !p->gate_b || gate_stride < p->num_v_heads)) return GDN_ERR_ARGS;
  if (p->slot_idx && (!p->pool_codes || !p->pool_scales || !p->pool_gscale)) return GDN_ERR_ARGS;
  int64_t code_stride = 0, scale_stride = 0, gs_stride = 0;
  if (p->slot_idx && !pool_strides(p->pool_tile_stride, p->pool_codes, p->pool_scales, p->pool_gscale,
                                   &code_stride, &scale_stride, &gs_stride))
    return GDN_ERR_ALIGN;
  if (p->total_tokens > INT32_MAX) return GDN_ERR_UNSUPPORTED;  // cu_seqlens are int32
  const int64_t nitems = (int64_t)p->num_seqs * p->num_v_heads;
  if (nitems > INT32_MAX / 2) return GDN_ERR_UNSUPPORTED;
  const int64_t q_stride = p->q_stride ? p->q_stride : (int64_t)p->num_k_heads * kD;
  const int64_t k_stride = p->k_stride ? p->k_stride : (int64_t)p->num_k_heads * kD;
  const int64_t v_stride = p->v_stride ? p->v_stride : (int64_t)p->num_v_heads * kD;
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->out) ||
      (q_stride | k_stride | v_stride) % 8 || (p->debug_y && !aligned16(p->debug_y)) ||
      (p->slot_idx && (!aligned16(p->pool_codes) || !aligned16(p->pool_scales))))
    return GDN_ERR_ALIGN;
  if (q_stride < (int64_t)p->num_k_heads * kD || k_stride < (int64_t)p->num_k_heads * kD ||
      v_stride < (int64_t)p->num_v_heads * kD)
    return GDN_ERR_ARGS;
  PrefillArgs a;
  a.N = p->num_seqs;
  a.HK = p->num_k_heads;
  a.HV = p->num_v_heads;
  a.group = p->num_v_heads / p->num_k_heads;
  a.nitems = (int32_t)nitems;
  a.T = p->total_tokens;
  a.num_slots = p->num_slots;
  a.g = p->g;
  a.beta = p->beta;
  a.cu = p->cu_seqlens;
  a.slot_idx = p->slot_idx;
  a.has_init = p->has_initial_state;
  a.pool_codes = p->pool_codes;
  a.pool_scales = p->pool_scales;
  a.pool_gs = p->pool_gscale;
  a.code_stride = code_stride;
  a.scale_stride = scale_stride;
  a.gs_stride = gs_stride;
  a.out = p->out;
  a.q_scale = p->q_scale > 0.0f ? p->q_scale : 0.08838834764831845f;  // 1/sqrt(128)
  a.gden = p->gscale_den > 0.0f ? p->gscale_den : default_gden(p->scale_mode);
  if (!(a.gden >= 6.0f && a.gden <= 1.0e6f)) return GDN_ERR_ARGS;
  a.debug_y = p->debug_y;
  a.status = device_status_ptr();
  if (!a.status) return GDN_ERR_CUDA;
  a.qk_l2norm = p->qk_l2norm;
  a.A_log = p->A_log;
  a.dt_bias = p->dt_bias;
  a.gate_a = p->gate_a;
  a.gate_b = p->gate_b;
  a.gate_stride = gate_stride;
  CUtensorMap tq, tk, tv;
  if (!make_row_map(&tq, p->q, p->num_k_heads, p->total_tokens, q_stride) ||
      !make_row_map(&tk, p->k, p->num_k_heads, p->total_tokens, k_stride) ||
      !make_row_map(&tv, p->v, p->num_v_heads, p->total_tokens, v_stride))
    return GDN_ERR_CUDA;

  const int smem = (int)kSmemBytes;
  const int64_t max_ctas = sm_count();
  const int grid = (int)(nitems < max_ctas ? nitems : max_ctas);
  const int mi = p->scale_mode == kScaleRef240 ? 0 : 1;
  const void* kern = mi == 0 ? reinterpret_cast<const void*>(gdn_prefill_kernel<kScaleRef240>)
                             : reinterpret_cast<const void*>(gdn_prefill_kernel<kScaleFn448>);
  if (allow_dynamic_smem(kern, smem) != GDN_OK) return GDN_ERR_CUDA;
  if (mi == 0)
    gdn_prefill_kernel<kScaleRef240><<<grid, kThreads, smem, stream>>>(a, tq, tk, tv);
  else
    gdn_prefill_kernel<kScaleFn448><<<grid, kThreads, smem, stream>>>(a, tq, tk, tv);
  return launch_status();
}
