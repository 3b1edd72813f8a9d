/*
 * gdn_oracle.c -- CPU oracle for the NVFP4 Gated DeltaNet state-update path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: it is loaded by the
 * tests, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg, and by
 * nothing else.  The product (the CUDA kernels behind include/gdn_b200.h) never
 * links, loads or calls it, and has no CPU fallback.
 *
 * What it restates (citations are paths inside the reference project
 * bojak83318/blackwell-kernel-sm_120):
 *   - E2M1 nibble decode          src/intrinsics/gdn_fp4_intrinsics.cuh:27-45
 *                                  (duplicate: src/kernel/gdn_state_update_ref.cu:20-34)
 *   - UE4M3 scale decode          src/intrinsics/gdn_fp4_intrinsics.cuh:48-68
 *   - UE4M3 scale encode          src/intrinsics/gdn_fp4_intrinsics.cuh:71-123
 *   - NVFP4 dequantise (host)     src/kernel/gdn_state_update_ref.cu:75-89
 *   - NVFP4 quantise (host)       src/kernel/gdn_state_update_ref.cu:93-141
 *   - legacy update S'=aS+b k v^T src/kernel/gdn_state_update_ref.cu:51-67
 *   - legacy op path              src/kernel/gdn_state_update_ref.cu:202-262
 * Parts with no counterpart in the reference (built from the published
 * mathematics: Yang, Kautz & Hatamizadeh, "Gated Delta Networks", ICLR 2025;
 * Yang et al., "Parallelizing Linear Transformers with the Delta Rule over
 * Sequence Length", NeurIPS 2024):
 *   - per-head fp32 global scale on top of the reference block quantiser
 *   - the gated delta-rule decode step with GQA and readout o = S^T q
 *   - the recurrent and chunked (WY/UT, chunk 64) forms of a prefill
 *
 * Scale modes.  Mode 0 ("ref240") is the reference codec unchanged: scales
 * saturate at 240 (0x77) and codes 0x78..0xFF decode to inf/NaN/negative as the
 * reference does.  Mode 1 ("fn448") keeps every rounding rule of the reference
 * encoder but extends the range to the E4M3FN format (saturation 448 = 0x7E;
 * exponent field 15 is a normal binade, 0x7F/0xFF are NaN).  The two modes give
 * identical bytes for every block whose local scale is below 240.
 *
 * Build: gcc -O2 -fPIC -shared -ffp-contract=off (see oracle/Makefile).  FMA
 * contraction is off so that every float expression below rounds exactly as
 * written; the legacy update exposes its contraction explicitly via fmaf().
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

static inline float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_from_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf16_to_f32(uint16_t b) { return f32_from_bits((uint32_t)b << 16); }

/* ---- codec ---------------------------------------------------------------- */

/* E2M1 nibble [s e1 e0 m] -> float.  gdn_fp4_intrinsics.cuh:27-45: exponent 0 is
 * subnormal (m * 0.5), otherwise (1 + m/2) * 2^(e-1); sign bit negates. */
ORC_API float orc_e2m1_decode(uint32_t nib) {
  nib &= 0xFu;
  uint32_t s = (nib >> 3) & 1u, e = (nib >> 1) & 3u, m = nib & 1u;
  float mag = (e == 0) ? (m ? 0.5f : 0.0f) : ldexpf(1.0f + 0.5f * (float)m, (int)e - 1);
  return s ? -mag : mag;
}

/* Scale byte -> float.  gdn_fp4_intrinsics.cuh:48-68 for mode 0 (bias 7,
 * exponent 0 subnormal m*2^-9, exponent 15 -> inf (m==0) / NaN, sign honoured).
 * Mode 1 reads exponent 15 as a normal binade except mantissa 7 (NaN). */
ORC_API float orc_scale_decode(uint32_t b, int mode) {
  b &= 0xFFu;
  uint32_t s = b >> 7, e = (b >> 3) & 0xFu, m = b & 7u;
  float mag;
  if (e == 0) {
    mag = m ? ldexpf((float)m / 8.0f, -6) : 0.0f;
  } else if (e == 15 && mode == 0) {
    mag = m ? NAN : INFINITY;
  } else if (e == 15 && m == 7) {
    mag = NAN;
  } else {
    mag = ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);
  }
  return s ? -mag : mag;
}

/* float -> scale byte, following gdn_fp4_intrinsics.cuh:71-123 step by step:
 *   non-finite or <= 0            -> 0
 *   >= saturation                 -> 0x77 (mode 0) / 0x7E (mode 1)
 *   < 2^-6 (subnormal)            -> int(x / 2^-9 + 0.5f) clamped to [0, 7]
 *   otherwise e = ilogb(x), n = x * 2^-e; n >= 1.875 -> (n/2, e+1);
 *   mantissa = int((n - 1) * 8 + 0.5f), carry into the exponent if it reaches 8. */
ORC_API uint32_t orc_scale_encode(float x, int mode) {
  const int max_field = mode ? 15 : 14;
  const float sat = mode ? 448.0f : 240.0f;
  const uint32_t sat_code = mode ? 0x7Eu : 0x77u;
  if (!isfinite(x) || x <= 0.0f) return 0;
  if (x >= sat) return sat_code;
  if (x < ldexpf(1.0f, -6)) {
    const float unit = ldexpf(1.0f, -9);
    int m = (int)(x / unit + 0.5f);
    if (m <= 0) return 0;
    if (m > 7) m = 7;
    return (uint32_t)m;
  }
  int e = ilogbf(x);
  float n = ldexpf(x, -e);
  if (n >= 1.875f) { n *= 0.5f; ++e; }
  int field = e + 7;
  if (field > max_field) { field = max_field; n = mode ? 1.75f : 1.875f; }
  if (field <= 0) return 0;
  int m = (int)((n - 1.0f) * 8.0f + 0.5f);
  if (m > 7) { m = 0; ++field; if (field > max_field) { field = max_field; m = mode ? 6 : 7; } }
  uint32_t code = ((uint32_t)field << 3) | (uint32_t)m;
  return code > sat_code ? sat_code : code;
}

/* Nearest E2M1 magnitude with a strict '<' scan, so an exact tie keeps the
 * smaller magnitude; the sign is (x < 0), so -0.0 encodes as 0x0
 * (gdn_state_update_ref.cu:117-135). */
static inline uint32_t e2m1_encode_ref(float x) {
  static const float mags[8] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  float ax = fabsf(x);
  uint32_t best = 0;
  float best_err = fabsf(ax - mags[0]);
  for (uint32_t k = 1; k < 8; ++k) {
    float err = fabsf(ax - mags[k]);
    if (err < best_err) { best_err = err; best = k; }
  }
  return best | ((x < 0.0f) ? 8u : 0u);
}

ORC_API uint32_t orc_e2m1_encode(float x) { return e2m1_encode_ref(x); }

/* Reference block quantiser, gdn_state_update_ref.cu:93-141: 16-element
 * blocks; amax via fmaxf(|x|); local scale amax/6 (1.0 for an all-zero block);
 * inverse of the DECODED scale (0 if it is not > 0); nibble pairs packed with
 * the even element in the low nibble. */
ORC_API void orc_quantise(const float* in, uint8_t* codes, uint8_t* scales, int64_t n, int mode) {
  for (int64_t b = 0; b < n / 16; ++b) {
    const float* blk = in + b * 16;
    float amax = 0.0f;
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(blk[i]));
    float local = (amax > 0.0f) ? (amax / 6.0f) : 1.0f;
    uint32_t enc = orc_scale_encode(local, mode);
    scales[b] = (uint8_t)enc;
    float dec = orc_scale_decode(enc, mode);
    float inv = (dec > 0.0f) ? (1.0f / dec) : 0.0f;
    for (int i = 0; i < 16; i += 2) {
      uint32_t n0 = e2m1_encode_ref(blk[i] * inv);
      uint32_t n1 = e2m1_encode_ref(blk[i + 1] * inv);
      codes[(b * 16 + i) / 2] = (uint8_t)(n0 | (n1 << 4));
    }
  }
}

/* gdn_state_update_ref.cu:75-89: out[i] = e2m1(nibble i) * scale(i / 16). */
ORC_API void orc_dequantise(const uint8_t* codes, const uint8_t* scales, float* out, int64_t n, int mode) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t byte = codes[i / 2];
    uint32_t nib = (i % 2 == 0) ? (byte & 0xFu) : (byte >> 4);
    out[i] = orc_e2m1_decode(nib) * orc_scale_decode(scales[i / 16], mode);
  }
}

/* ---- per-tile global scale (new; no reference counterpart) -----------------
 * gs = amax / gden (1.0 for an all-zero tile); the reference quantiser runs on
 * y = x * (1.0f / gs); dequantisation is (e2m1 * scale) * gs. */
ORC_API float orc_global_scale(const float* x, int64_t n, float gden) {
  float amax = 0.0f;
  for (int64_t i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(x[i]));
  return (amax > 0.0f) ? (amax / gden) : 1.0f;
}

ORC_API void orc_quantise_tile_gs(const float* x, int64_t n, uint8_t* codes, uint8_t* scales,
                                  float* gs_out, float* y_out, int mode, float gden) {
  float gs = orc_global_scale(x, n, gden);
  float inv = 1.0f / gs;
  float* y = y_out ? y_out : (float*)malloc((size_t)n * sizeof(float));
  for (int64_t i = 0; i < n; ++i) y[i] = x[i] * inv;
  orc_quantise(y, codes, scales, n, mode);
  *gs_out = gs;
  if (!y_out) free(y);
}

ORC_API void orc_dequantise_tile_gs(const uint8_t* codes, const uint8_t* scales, float gs,
                                    float* out, int64_t n, int mode) {
  orc_dequantise(codes, scales, out, n, mode);
  for (int64_t i = 0; i < n; ++i) out[i] = out[i] * gs;
}

/* ---- legacy op (gdn_state_update_ref.cu:51-67 and :202-262) ----------------
 * S'[r*d+c] = alpha*S[r*d+c] + beta*k[r]*v[c] (row = k index, col = v index).
 * The reference kernel's source expression is (alpha*s) + ((beta*k)*v); the
 * CUDA compiler may contract it, so the three roundings are selectable:
 *   variant 0: fmaf(alpha, s, (beta*k)*v)
 *   variant 1: fmaf(beta*k, v, alpha*s)
 *   variant 2: no contraction. */
static inline float legacy_elem(float s, float kr, float vc, float alpha, float beta, int variant) {
  float bk = beta * kr;
  if (variant == 0) return fmaf(alpha, s, bk * vc);
  if (variant == 1) return fmaf(bk, vc, alpha * s);
  float a = alpha * s, b = bk * vc;
  return a + b;
}

ORC_API void orc_legacy_update_f32(const float* S, const uint16_t* k, const uint16_t* v, float* out,
                                   float alpha, float beta, int d, int variant) {
  for (int r = 0; r < d; ++r) {
    float kr = bf16_to_f32(k[r]);
    for (int c = 0; c < d; ++c)
      out[(int64_t)r * d + c] = legacy_elem(S[(int64_t)r * d + c], kr, bf16_to_f32(v[c]), alpha, beta, variant);
  }
}

/* The whole reference op path: dequantise -> update -> quantise (mode 0). */
ORC_API void orc_legacy_op(const uint8_t* S_data, const uint8_t* S_scales, const uint16_t* k,
                           const uint16_t* v, uint8_t* out_data, uint8_t* out_scales,
                           float alpha, float beta, int d, int variant) {
  int64_t n = (int64_t)d * d;
  float* S = (float*)malloc((size_t)n * sizeof(float));
  float* T = (float*)malloc((size_t)n * sizeof(float));
  orc_dequantise(S_data, S_scales, S, n, 0);
  orc_legacy_update_f32(S, k, v, T, alpha, beta, d, variant);
  orc_quantise(T, out_data, out_scales, n, 0);
  free(S);
  free(T);
}

/* ---- gated delta rule, one decode step over a slot-indexed NVFP4 pool ------
 * For sequence b and value head h (key head hk = h / (HV/HK)):
 *   alpha = exp(g);  S_a = alpha * S;  u = S_a^T k;  w = beta * (v - u)
 *   S' = S_a + k w^T;  o = q_scale * S'^T q
 * S is [dk][dv] (dv contiguous), the NVFP4 tile layout of the pool.  Sums run
 * in double; the new state is rounded to fp32, given a fresh global scale and
 * quantised by the reference quantiser.  A negative slot marks padding: the
 * pool is not touched and o is zero.  Optional y_out receives the fp32
 * quantiser inputs per tile ([B][HV][D*D]). */
/* ---- decode-step requantisation (new; the decode kernel's rule) -------------
 * S' = c * D with c = 2^7 * RN(expf(g) * gs) (c = 1 when RN(expf(g) * gs) is
 * below 1e-30, where the decode kernel drops the decayed state) and
 * D = RN(S' / c).  With A = max |D| (NaN ignored):
 *   A finite > 0: k = the largest integer with A * 2^k <= gden, clamped to
 *                 [-126, 126]; gs' = c * 2^-k and y = D * 2^k;
 *   A = 0:        gs' = 1 and y = D * c;
 *   A = inf:      gs' = inf and y = D * 0;
 * then the reference quantiser on y. */
static void requant_pow2(const float* Sn, int64_t n, float c, uint8_t* codes, uint8_t* scales, float* gs_out,
                         float* y_out, int mode, float gden) {
  float* y = y_out ? y_out : (float*)malloc((size_t)n * sizeof(float));
  float A = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    y[i] = (float)((double)Sn[i] / (double)c);
    A = fmaxf(A, fabsf(y[i]));
  }
  float mult, gs;
  if (A > 0.0f && isfinite(A)) {
    int k = 0;
    while (ldexpf(A, k + 1) <= gden && k < 126) ++k;
    while (ldexpf(A, k) > gden && k > -126) --k;
    mult = ldexpf(1.0f, k);
    gs = c * ldexpf(1.0f, -k);
  } else if (A == 0.0f) {
    mult = c;
    gs = 1.0f;
  } else {
    mult = 0.0f;
    gs = INFINITY;
  }
  for (int64_t i = 0; i < n; ++i) y[i] = y[i] * mult;
  orc_quantise(y, codes, scales, n, mode);
  *gs_out = gs;
  if (!y_out) free(y);
}

ORC_API void orc_gdn_decode(int B, int HK, int HV, int D,
                            const uint16_t* q, const uint16_t* k, const uint16_t* v,
                            const float* g, const float* beta, const int32_t* slot,
                            uint8_t* pool_codes, uint8_t* pool_scales, float* pool_gs,
                            uint16_t* o_bf16, float* o_f32, float q_scale, int mode, float gden,
                            float* y_out) {
  const int64_t DD = (int64_t)D * D;
  const int group = HV / HK;
  float* S = (float*)malloc((size_t)DD * sizeof(float));
  float* Sn = (float*)malloc((size_t)DD * sizeof(float));
  double* u = (double*)malloc((size_t)D * sizeof(double));
  double* w = (double*)malloc((size_t)D * sizeof(double));
  double* oo = (double*)malloc((size_t)D * sizeof(double));
  for (int b = 0; b < B; ++b) {
    for (int h = 0; h < HV; ++h) {
      const int hk = h / group;
      const uint16_t* qb = q + ((int64_t)b * HK + hk) * D;
      const uint16_t* kb = k + ((int64_t)b * HK + hk) * D;
      const uint16_t* vb = v + ((int64_t)b * HV + h) * D;
      const int64_t ob = ((int64_t)b * HV + h) * D;
      const int32_t s = slot[b];
      if (s < 0) {
        for (int j = 0; j < D; ++j) {
          if (o_bf16) o_bf16[ob + j] = 0;
          if (o_f32) o_f32[ob + j] = 0.0f;
        }
        continue;
      }
      const int64_t t = (int64_t)s * HV + h;
      uint8_t* pc = pool_codes + t * (DD / 2);
      uint8_t* ps = pool_scales + t * (DD / 16);
      const float pool_gs_in = pool_gs[t];
      orc_dequantise_tile_gs(pc, ps, pool_gs_in, S, DD, mode);
      /* the decode kernel drops the decayed state when alpha * gs < 1e-30 in fp32 */
      const float cg = expf(g[(int64_t)b * HV + h]) * pool_gs_in;
      const int drop = cg >= 0.0f && cg < 1e-30f;
      const double alpha = drop ? 0.0 : exp((double)g[(int64_t)b * HV + h]);
      const double bt = beta[(int64_t)b * HV + h];
      for (int j = 0; j < D; ++j) u[j] = 0.0;
      for (int i = 0; i < D; ++i) {
        const double ki = bf16_to_f32(kb[i]);
        for (int j = 0; j < D; ++j) u[j] += alpha * (double)S[(int64_t)i * D + j] * ki;
      }
      for (int j = 0; j < D; ++j) { w[j] = bt * ((double)bf16_to_f32(vb[j]) - u[j]); oo[j] = 0.0; }
      for (int i = 0; i < D; ++i) {
        const double ki = bf16_to_f32(kb[i]), qi = bf16_to_f32(qb[i]);
        for (int j = 0; j < D; ++j) {
          const double sn = alpha * (double)S[(int64_t)i * D + j] + ki * w[j];
          Sn[(int64_t)i * D + j] = (float)sn;
          oo[j] += sn * qi;
        }
      }
      for (int j = 0; j < D; ++j) {
        const float of = (float)(oo[j] * (double)q_scale);
        if (o_f32) o_f32[ob + j] = of;
        if (o_bf16) {
          /* round-to-nearest-even fp32 -> bf16 */
          uint32_t ub = bits_from_f32(of);
          uint32_t r = ub + 0x7FFFu + ((ub >> 16) & 1u);
          o_bf16[ob + j] = (uint16_t)(isnan(of) ? 0x7FC0u : (r >> 16));
        }
      }
      const float c = drop ? 1.0f : cg * 128.0f;
      requant_pow2(Sn, DD, c, pc, ps, &pool_gs[t], y_out ? y_out + ((int64_t)b * HV + h) * DD : NULL, mode, gden);
    }
  }
  free(S); free(Sn); free(u); free(w); free(oo);
}

/* ---- unquantised recurrence for one (sequence, head) ------------------------
 * S (double, [D][D], in/out) runs T tokens; q/k rows are D apart (caller
 * passes pointers already offset to this head with the given token stride);
 * o receives T rows of D outputs (q_scale applied).  Used as the fp32/f64
 * reference for SQNR and for prefill parity. */
ORC_API void orc_gdn_recurrent_f64(int T, int D, double* S,
                                   const float* q, const float* k, const float* v,
                                   int64_t qk_stride, int64_t v_stride,
                                   const float* g, const float* beta, int64_t gb_stride,
                                   double* o, int64_t o_stride, double q_scale) {
  double* u = (double*)malloc((size_t)D * sizeof(double));
  for (int t = 0; t < T; ++t) {
    const float* qt = q + t * qk_stride;
    const float* kt = k + t * qk_stride;
    const float* vt = v + t * v_stride;
    const double a = exp((double)g[t * gb_stride]);
    const double bt = beta[t * gb_stride];
    for (int j = 0; j < D; ++j) u[j] = 0.0;
    for (int i = 0; i < D; ++i) {
      for (int j = 0; j < D; ++j) {
        S[i * D + j] *= a;
        u[j] += S[i * D + j] * kt[i];
      }
    }
    for (int j = 0; j < D; ++j) u[j] = bt * (vt[j] - u[j]);
    double* ot = o + t * o_stride;
    for (int j = 0; j < D; ++j) ot[j] = 0.0;
    for (int i = 0; i < D; ++i) {
      for (int j = 0; j < D; ++j) {
        S[i * D + j] += kt[i] * u[j];
        ot[j] += S[i * D + j] * qt[i];
      }
    }
    for (int j = 0; j < D; ++j) ot[j] *= q_scale;
  }
  free(u);
}

/* ---- chunked (WY / UT) form of the same recurrence ---------------------------
 * Per chunk of C tokens with cumulative log decay gam_t (within the chunk):
 *   L[t][s]  = exp(gam_t - gam_s) * (k_t . k_s)      for s < t
 *   Tm       = (I + diag(beta) L)^-1                  (unit lower triangular)
 *   Ut       = Tm diag(beta) V,   W = Tm diag(beta * exp(gam)) K
 *   U        = Ut - W S0
 *   O        = diag(exp(gam)) Q S0 + ((Q K^T) o M) U,  M[t][s] = exp(gam_t - gam_s), s <= t
 *   S_end    = exp(gam_C) S0 + (K o exp(gam_C - gam))^T U
 * Same arguments as orc_gdn_recurrent_f64 plus the chunk length C. */
ORC_API void orc_gdn_chunked_f64(int T, int D, int C, double* S,
                                 const float* q, const float* k, const float* v,
                                 int64_t qk_stride, int64_t v_stride,
                                 const float* g, const float* beta, int64_t gb_stride,
                                 double* o, int64_t o_stride, double q_scale) {
  double* gam = (double*)malloc((size_t)C * sizeof(double));
  double* L = (double*)malloc((size_t)C * C * sizeof(double));
  double* Tm = (double*)malloc((size_t)C * C * sizeof(double));
  double* U = (double*)malloc((size_t)C * D * sizeof(double));
  double* W = (double*)malloc((size_t)C * D * sizeof(double));
  double* A = (double*)malloc((size_t)C * C * sizeof(double));
  double* Sn = (double*)malloc((size_t)D * D * sizeof(double));
  for (int c0 = 0; c0 < T; c0 += C) {
    const int n = (T - c0 < C) ? (T - c0) : C;
    double acc = 0.0;
    for (int t = 0; t < n; ++t) { acc += g[(int64_t)(c0 + t) * gb_stride]; gam[t] = acc; }
#define KK(t, i) ((double)k[(int64_t)(c0 + (t)) * qk_stride + (i)])
#define QQ(t, i) ((double)q[(int64_t)(c0 + (t)) * qk_stride + (i)])
#define VV(t, j) ((double)v[(int64_t)(c0 + (t)) * v_stride + (j)])
#define BB(t) ((double)beta[(int64_t)(c0 + (t)) * gb_stride])
    for (int t = 0; t < n; ++t)
      for (int s = 0; s < n; ++s) {
        double dk = 0.0, dq = 0.0;
        for (int i = 0; i < D; ++i) { dk += KK(t, i) * KK(s, i); dq += QQ(t, i) * KK(s, i); }
        L[t * C + s] = (s < t) ? exp(gam[t] - gam[s]) * dk : 0.0;
        A[t * C + s] = (s <= t) ? exp(gam[t] - gam[s]) * dq : 0.0;
      }
    /* forward substitution: Tm (I + diag(beta) L) = I, row by row */
    for (int t = 0; t < n; ++t) {
      for (int s = 0; s < n; ++s) Tm[t * C + s] = (s == t) ? 1.0 : 0.0;
      for (int s = 0; s < t; ++s) {
        const double f = BB(t) * L[t * C + s];
        for (int r = 0; r <= s; ++r) Tm[t * C + r] -= f * Tm[s * C + r];
      }
    }
    for (int t = 0; t < n; ++t) {
      for (int j = 0; j < D; ++j) {
        double su = 0.0, sw = 0.0;
        for (int s = 0; s <= t; ++s) {
          su += Tm[t * C + s] * BB(s) * VV(s, j);
          sw += Tm[t * C + s] * BB(s) * exp(gam[s]) * KK(s, j);
        }
        U[t * D + j] = su;
        W[t * D + j] = sw;
      }
    }
    for (int t = 0; t < n; ++t)
      for (int j = 0; j < D; ++j) {
        double ws = 0.0;
        for (int i = 0; i < D; ++i) ws += W[t * D + i] * S[i * D + j];
        U[t * D + j] -= ws;
      }
    for (int t = 0; t < n; ++t) {
      double* ot = o + (int64_t)(c0 + t) * o_stride;
      const double et = exp(gam[t]);
      for (int j = 0; j < D; ++j) {
        double acc2 = 0.0;
        for (int i = 0; i < D; ++i) acc2 += QQ(t, i) * S[i * D + j];
        acc2 *= et;
        for (int s = 0; s <= t; ++s) acc2 += A[t * C + s] * U[s * D + j];
        ot[j] = acc2 * q_scale;
      }
    }
    const double eC = exp(gam[n - 1]);
    for (int i = 0; i < D; ++i)
      for (int j = 0; j < D; ++j) {
        double acc3 = eC * S[i * D + j];
        for (int s = 0; s < n; ++s) acc3 += exp(gam[n - 1] - gam[s]) * KK(s, i) * U[s * D + j];
        Sn[i * D + j] = acc3;
      }
    memcpy(S, Sn, (size_t)D * D * sizeof(double));
#undef KK
#undef QQ
#undef VV
#undef BB
  }
  free(gam); free(L); free(Tm); free(U); free(W); free(A); free(Sn);
}

/* SQNR in dB of `test` against `ref`: 10 log10(sum ref^2 / sum (ref-test)^2). */
ORC_API double orc_sqnr_db(const double* ref, const double* test, int64_t n) {
  double num = 0.0, den = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    num += ref[i] * ref[i];
    const double e = ref[i] - test[i];
    den += e * e;
  }
  if (den == 0.0) return INFINITY;
  return 10.0 * log10(num / den);
}

/* ---- sweeps and fixtures ------------------------------------------------------ */

/* Encodes every float whose bit pattern is lo + i*stride (i < count). */
ORC_API void orc_scale_encode_sweep(uint32_t lo, uint32_t stride, uint64_t count, int mode, uint8_t* out) {
  for (uint64_t i = 0; i < count; ++i) {
    uint32_t u = lo + (uint32_t)(i * stride);
    out[i] = (uint8_t)orc_scale_encode(f32_from_bits(u), mode);
  }
}

/* Block scale byte for every block max |y| with bit pattern lo + i: the
 * reference quantiser's local scale amax/6 (1.0 for amax 0) through the scale
 * encoder (gdn_state_update_ref.cu:105-108). */
ORC_API void orc_block_scale_sweep(uint32_t lo, uint64_t count, int mode, uint8_t* out) {
  for (uint64_t i = 0; i < count; ++i) {
    const float amax = f32_from_bits(lo + (uint32_t)i);
    const float local = (amax > 0.0f) ? (amax / 6.0f) : 1.0f;
    out[i] = (uint8_t)orc_scale_encode(local, mode);
  }
}

/* E2M1 nibble (the reference scan) of every value with bit pattern lo + i. */
ORC_API void orc_e2m1_sweep(uint32_t lo, uint64_t count, uint8_t* out) {
  for (uint64_t i = 0; i < count; ++i) out[i] = (uint8_t)e2m1_encode_ref(f32_from_bits(lo + (uint32_t)i));
}

/* The reference's M3 gate draws its inputs from the C library's rand() after
 * srand(42) (tests/test_gdn_correctness.cu:50-54, :101-104, :200):
 *   x = lo + (hi - lo) * ((float)rand() / (float)RAND_MAX)   in float. */
ORC_API void orc_libc_srand(unsigned seed) { srand(seed); }

ORC_API void orc_libc_fill_uniform(float* x, int64_t n, float lo, float hi) {
  for (int64_t i = 0; i < n; ++i) {
    float r = (float)rand() / (float)RAND_MAX;
    x[i] = lo + (hi - lo) * r;
  }
}
