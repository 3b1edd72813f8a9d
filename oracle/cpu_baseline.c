/*
 * cpu_baseline.c -- the CPU path of one NVFP4 Gated DeltaNet decode step,
 * timed beside the GPU kernel by bench.py (its cpu_baseline leg and
 * `--impl reference`).  TEST/BENCH INFRASTRUCTURE ONLY; never on the product
 * path.
 *
 * Per (sequence, value head) tile, exactly the steps of the reference's op
 * path (src/kernel/gdn_state_update_ref.cu:202-262) widened to the gated delta
 * rule:
 *   1. dequantise the NVFP4 tile on the host
 *      (nvfp4_dequantise_host, gdn_state_update_ref.cu:75-89), times the
 *      tile's global scale;
 *   2. the fp32 state update: alpha = exp(g), S_a = alpha S, u = S_a^T k,
 *      w = beta (v - u), S' = S_a + k w^T, o = q_scale S'^T q;
 *   3. requantise on the host (nvfp4_quantise_host, gdn_state_update_ref.cu:93-141)
 *      after the global scale gs' = amax / gden.
 * Built twice by oracle/Makefile: against the reference's own host codec
 * (GDN_CPU_USE_REF, oracle/_ref/libgdn_cpu_ref.so) and against the oracle's
 * restatement (oracle/_build/libgdn_cpu_port.so).  Tiles run in parallel with
 * OpenMP over (sequence, head).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#define API __attribute__((visibility("default")))

#ifdef GDN_CPU_USE_REF
void ref_nvfp4_quantise(const float* in, uint8_t* codes, uint8_t* scales, int n);
void ref_nvfp4_dequantise(const uint8_t* codes, const uint8_t* scales, float* out, int n);
#define DEQUANT(c, s, o, n, mode) ref_nvfp4_dequantise((c), (s), (o), (int)(n))
#define QUANT(i, c, s, n, mode) ref_nvfp4_quantise((i), (c), (s), (int)(n))
API int cpu_baseline_uses_reference(void) { return 1; }
#else
void orc_quantise(const float* in, uint8_t* codes, uint8_t* scales, int64_t n, int mode);
void orc_dequantise(const uint8_t* codes, const uint8_t* scales, float* out, int64_t n, int mode);
#define DEQUANT(c, s, o, n, mode) orc_dequantise((c), (s), (o), (n), (mode))
#define QUANT(i, c, s, n, mode) orc_quantise((i), (c), (s), (n), (mode))
API int cpu_baseline_uses_reference(void) { return 0; }
#endif

static inline float bf(uint16_t b) { uint32_t u = (uint32_t)b << 16; float f; memcpy(&f, &u, 4); return f; }
static inline uint16_t to_bf(float f) {
  uint32_t u; memcpy(&u, &f, 4);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

/* One decode step over tiles [t_begin, t_end) of the B*HV tile grid.  Returns
 * the number of tiles processed.  nthreads <= 0 uses all OpenMP threads. */
API int64_t cpu_gdn_decode(int B, int HK, int HV, int D,
                           const uint16_t* q, const uint16_t* k, const uint16_t* v,
                           const float* g, const float* beta, const int32_t* slot,
                           uint8_t* pool_codes, uint8_t* pool_scales, float* pool_gs,
                           uint16_t* o, float q_scale, int mode, float gden,
                           int64_t t_begin, int64_t t_end, int nthreads) {
  const int64_t DD = (int64_t)D * D;
  const int group = HV / HK;
  if (t_end > (int64_t)B * HV) t_end = (int64_t)B * HV;
  if (nthreads > 0) omp_set_num_threads(nthreads);
  int64_t done = 0;
#pragma omp parallel reduction(+ : done)
  {
    float* S = (float*)malloc((size_t)DD * sizeof(float));
    float* u = (float*)malloc((size_t)D * sizeof(float));
    float* oo = (float*)malloc((size_t)D * sizeof(float));
#pragma omp for schedule(static)
    for (int64_t t = t_begin; t < t_end; ++t) {
      const int b = (int)(t / HV), h = (int)(t % HV), hk = h / group;
      const int32_t s = slot[b];
      uint16_t* ob = o + t * D;
      if (s < 0) { memset(ob, 0, (size_t)D * 2); continue; }
      const int64_t pt = (int64_t)s * HV + h;
      uint8_t* pc = pool_codes + pt * (DD / 2);
      uint8_t* ps = pool_scales + pt * (DD / 16);
      const uint16_t* qb = q + ((int64_t)b * HK + hk) * D;
      const uint16_t* kb = k + ((int64_t)b * HK + hk) * D;
      const uint16_t* vb = v + t * D;
      DEQUANT(pc, ps, S, DD, mode);
      const float alpha = expf(g[t]) * pool_gs[pt];
      const float bt = beta[t];
      for (int j = 0; j < D; ++j) u[j] = 0.0f;
      for (int i = 0; i < D; ++i) {
        const float ki = bf(kb[i]);
        float* Si = S + (int64_t)i * D;
        for (int j = 0; j < D; ++j) { Si[j] *= alpha; u[j] += Si[j] * ki; }
      }
      for (int j = 0; j < D; ++j) { u[j] = bt * (bf(vb[j]) - u[j]); oo[j] = 0.0f; }
      float amax = 0.0f;
      for (int i = 0; i < D; ++i) {
        const float ki = bf(kb[i]), qi = bf(qb[i]);
        float* Si = S + (int64_t)i * D;
        for (int j = 0; j < D; ++j) {
          Si[j] += ki * u[j];
          oo[j] += Si[j] * qi;
          amax = fmaxf(amax, fabsf(Si[j]));
        }
      }
      for (int j = 0; j < D; ++j) ob[j] = to_bf(oo[j] * q_scale);
      const float gs = (amax > 0.0f) ? amax / gden : 1.0f;
      const float inv = 1.0f / gs;
      for (int64_t e = 0; e < DD; ++e) S[e] *= inv;
      QUANT(S, pc, ps, DD, mode);
      pool_gs[pt] = gs;
      ++done;
    }
    free(S); free(u); free(oo);
  }
  return done;
}

API int cpu_max_threads(void) { return omp_get_max_threads(); }
