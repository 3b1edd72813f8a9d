/*
 * gdn_b200.h -- C ABI of libgdn_b200.so, the B200 (sm_100a) NVFP4 Gated
 * DeltaNet state-update library.
 *
 * Conventions
 *   - Plain C types only: device pointers, sizes, a cudaStream_t.  Every call
 *     is stream-ordered and non-blocking: no allocation, no host
 *     synchronisation, no host round trip (gdn_b200_device_status and the
 *     set-up calls of the peer all-reduce are the exceptions and say so).
 *     The caller owns every buffer.
 *   - Calls are stateless and safe from any host thread; ordering is per
 *     stream.  The library's only host state is set up once per device under
 *     a lock (the device status word's address, the SM count, the kernels'
 *     shared-memory opt-in).  Errors are integer status codes (GDN_OK == 0).
 *   - bf16 arrays are IEEE bfloat16 (__nv_bfloat16 in C++, uint16_t bit
 *     patterns in C).
 *   - Device pointers handed to the bulk-copy (TMA) kernels must be 16-byte
 *     aligned and rows of bf16 vectors must start on 16-byte boundaries
 *     (strides that are multiples of 8 elements).
 *
 * NVFP4 state format (the reference's, src/kernel/gdn_state_update_ref.cu:16-18,
 * plus a per-tile global scale): E2M1 codes two per byte, the even element in
 * the low nibble; one E4M3-style scale byte per 16 contiguous elements; for the
 * pooled GDN state one fp32 global scale per (slot, value head) tile.  A state
 * tile is S[k][v] (d_k rows, d_v contiguous), so scale blocks run along d_v.
 *
 * Reference interfaces (paths in bojak83318/blackwell-kernel-sm_120):
 *   launch_gdn_state_update   src/kernel/gdn_state_update_ref.cu:202-262,
 *                             declared by src/ops/gdn_op.cu:32-40 and
 *                             tests/test_gdn_correctness.cu:32-36
 *   launch_gdn_ref            src/kernel/gdn_state_update_ref.cu:147-176
 *   nvfp4 (de)quantise        src/kernel/gdn_state_update_ref.cu:75-141 (host)
 *                             and :178-197 (device dequantise)
 *   decode / prefill / pool   no counterpart in the reference (its only batched
 *                             kernel, src/kernel/gdn_state_update.cu:112-182,
 *                             is unreachable); the parameter blocks follow the
 *                             batched layout of gdn_state_update.cu:65-75
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stdint.h>
#include <cuda_runtime_api.h>

/* Symbols of this header are the library's only exports. */
#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

#ifdef __cplusplus
#include <cuda_bf16.h>
typedef __nv_bfloat16 gdn_bf16_t;
extern "C" {
#else
typedef uint16_t gdn_bf16_t;
#endif

/* ---- status codes --------------------------------------------------------
 * 0 and 1 keep the reference's meaning (gdn_state_update_ref.cu:214-217);
 * 3 keeps "kernel launch failed" (:232-236).  The reference's 2/4/5/6
 * (cudaMalloc, stream sync, D2H, H2D failures) cannot occur: nothing here
 * allocates, synchronises or copies through the host. */
#define GDN_OK 0
#define GDN_ERR_ARGS 1        /* null pointer, non-positive or inconsistent size */
#define GDN_ERR_LAUNCH 3      /* kernel launch failed (cudaGetLastError) */
#define GDN_ERR_UNSUPPORTED 7 /* shape or mode outside what this build implements */
#define GDN_ERR_ALIGN 8       /* pointer or stride not 16-byte aligned */
#define GDN_ERR_CUDA 9        /* a CUDA runtime query failed */

/* Device status bits, set by kernels and read by gdn_b200_device_status. */
#define GDN_STATUS_WAIT_TIMEOUT 0x1u /* a bounded wait gave up; the kernel left early */
#define GDN_STATUS_BAD_SLOT 0x2u     /* a slot index >= num_slots was skipped */
#define GDN_STATUS_BAD_SEQLENS 0x4u  /* a sequence with invalid cu_seqlens bounds was skipped */

/* Scale modes. */
#define GDN_SCALE_REF240 0 /* the reference codec: scales saturate at 240 (0x77) */
#define GDN_SCALE_FN448 1  /* reference rounding, E4M3FN range: saturate at 448 (0x7E) */

/* ---- legacy op (kept byte-compatible) -------------------------------------- */

/* One d x d state update S' = alpha*S + beta * k v^T, NVFP4 in and out, no
 * global scale, reference quantiser (mode GDN_SCALE_REF240).  Same prototype
 * and return codes as the reference (gdn_state_update_ref.cu:202-262); unlike
 * it, this one runs entirely on the GPU, stream-ordered, with no cudaMalloc and
 * no host synchronisation.  S_data [d*d/2], S_scales [d*d/16], k, v [d];
 * requires d*d % 16 == 0.  In-place (out == in) is allowed. */
GDN_API int launch_gdn_state_update(const uint8_t* S_data, const uint8_t* S_scales, const gdn_bf16_t* k,
                            const gdn_bf16_t* v, uint8_t* S_out_data, uint8_t* S_out_scales,
                            float alpha, float beta, int d, cudaStream_t stream);

/* fp32 reference update (gdn_state_update_ref.cu:147-176): dequantise the
 * NVFP4 state and write S_out = alpha*S + beta*k v^T in fp32 [d*d].  Same
 * prototype (void); errors surface through cudaGetLastError as in the
 * reference.  Fused into one kernel: no temporary buffer. */
GDN_API void launch_gdn_ref(const uint8_t* S_data, const uint8_t* S_scales, const gdn_bf16_t* k,
                    const gdn_bf16_t* v, float* S_out, float alpha, float beta, int d,
                    cudaStream_t stream);

/* The legacy update with an explicit rounding of alpha*s + (beta*k)*v, chosen
 * per call (no counterpart in the reference, whose compiler picks one):
 * rounding 0 = fmaf(alpha, s, (beta*k)*v), 1 = fmaf(beta*k, v, alpha*s),
 * 2 = no FMA.  launch_gdn_state_update and launch_gdn_ref always use 1, the
 * rounding of the reference kernel as compiled for sm_100a.  With S_out_f32
 * set it writes the fp32 update as launch_gdn_ref does (S_out_data and
 * S_out_scales unused); otherwise the NVFP4 result as launch_gdn_state_update
 * does.  Returns GDN_ERR_ARGS for a rounding outside 0..2. */
GDN_API int gdn_legacy_update_rounding(const uint8_t* S_data, const uint8_t* S_scales, const gdn_bf16_t* k,
                                       const gdn_bf16_t* v, uint8_t* S_out_data, uint8_t* S_out_scales,
                                       float* S_out_f32, float alpha, float beta, int d, int rounding,
                                       cudaStream_t stream);

/* ---- NVFP4 codec ----------------------------------------------------------- */

/* Device twin of nvfp4_quantise_host (gdn_state_update_ref.cu:93-141): n % 16 == 0,
 * codes [n/2], scales [n/16].  Bit-exact with the reference for every fp32
 * input in mode GDN_SCALE_REF240. */
GDN_API int gdn_nvfp4_quantize(const float* x, uint8_t* codes, uint8_t* scales, int64_t n,
                       int32_t scale_mode, cudaStream_t stream);

/* Device twin of nvfp4_dequantise_host (gdn_state_update_ref.cu:75-89; device
 * form :178-197). */
GDN_API int gdn_nvfp4_dequantize(const uint8_t* codes, const uint8_t* scales, float* out, int64_t n,
                         int32_t scale_mode, cudaStream_t stream);

/* Per-tile global scale (new): for each of num_tiles tiles of tile_elems
 * (a multiple of 16) elements, gs = amax/gscale_den (1.0 for an all-zero tile),
 * then the reference quantiser on y = x * (1/gs).  gscale_den <= 0 selects
 * 6*240 (mode 0) or 6*448 (mode 1).  gscale [num_tiles]. */
GDN_API int gdn_nvfp4_quantize_tiles(const float* x, int64_t num_tiles, int64_t tile_elems, uint8_t* codes,
                             uint8_t* scales, float* gscale, int32_t scale_mode, float gscale_den,
                             cudaStream_t stream);

/* Inverse: out = (e2m1 * scale) * gs. */
GDN_API int gdn_nvfp4_dequantize_tiles(const uint8_t* codes, const uint8_t* scales, const float* gscale,
                               int64_t num_tiles, int64_t tile_elems, float* out,
                               int32_t scale_mode, cudaStream_t stream);

/* ---- fused recurrent decode (one token per sequence) ------------------------
 * For each sequence b and value head h (key head h / (HV/HK)):
 *   alpha = exp(g);  S_a = alpha*S;  u = S_a^T k;  w = beta*(v - u)
 *   S' = S_a + k w^T;  out = q_scale * S'^T q
 * S is the NVFP4 tile at pool slot slot_idx[b]; S' is written back in place
 * with a fresh global scale gs' in [A/gscale_den, 2A/gscale_den), A = max |S'|:
 * a power-of-two multiple of alpha*gs, so that the E2M1 codes of every block
 * follow from S'/(alpha*gs) alone; codes and scales are those of the reference
 * quantiser applied to S'/gs'.  A negative slot marks padding (out = 0, pool
 * untouched); a slot >= num_slots is skipped the same way and flagged in the
 * device status.  Non-negative slots must be distinct.  head_dim must be 128. */
typedef struct gdn_decode_params {
  int32_t batch;          /* B */
  int32_t num_k_heads;    /* HK */
  int32_t num_v_heads;    /* HV, a multiple of HK */
  int32_t head_dim;       /* d_k = d_v */
  int64_t num_slots;      /* pool slots */
  const gdn_bf16_t* q;    /* [B, HK, D], sequence stride q_stride */
  const gdn_bf16_t* k;    /* [B, HK, D], sequence stride k_stride */
  const gdn_bf16_t* v;    /* [B, HV, D], sequence stride v_stride */
  int64_t q_stride;       /* elements between sequences; 0 = HK*D */
  int64_t k_stride;       /* 0 = HK*D */
  int64_t v_stride;       /* 0 = HV*D */
  const float* g;         /* [B, HV] log decay */
  const float* beta;      /* [B, HV] */
  const int32_t* slot_idx; /* [B] */
  uint8_t* pool_codes;    /* [num_slots, HV, D, D/2] */
  uint8_t* pool_scales;   /* [num_slots, HV, D, D/16] */
  float* pool_gscale;     /* [num_slots, HV] */
  gdn_bf16_t* out;        /* [B, HV, D] */
  float q_scale;          /* <= 0 selects 1/sqrt(D) */
  int32_t scale_mode;     /* GDN_SCALE_* */
  float gscale_den;       /* <= 0 selects 6*saturation */
  float* debug_y;         /* optional [B, HV, D, D]: the fp32 quantiser inputs */
  /* Optional fused prologue (the gating and q/k normalisation vLLM runs before
   * the recurrence; all NULL / 0 to skip).  With A_log set, g and beta are
   * computed in the kernel from the gate projections and the g / beta fields
   * are not read:
   *   g = -exp(A_log[h]) * softplus(gate_a[b, h] + dt_bias[h]),  beta = sigmoid(gate_b[b, h])
   * (softplus with threshold 20, as torch.nn.functional.softplus). */
  const float* A_log;       /* [HV] */
  const float* dt_bias;     /* [HV] */
  const gdn_bf16_t* gate_a; /* [B, HV], sequence stride gate_stride */
  const gdn_bf16_t* gate_b; /* [B, HV], sequence stride gate_stride */
  int64_t gate_stride;      /* elements between sequences; 0 = HV */
  int32_t qk_l2norm;        /* != 0: q and k scaled to unit L2 norm per head, x / sqrt(sum x^2 + 1e-6), in fp32 */
  /* Optional fused epilogue: the gated RMS norm vLLM's GDN layer applies to
   * the attention output before its out-projection (RMSNormGated with
   * norm_before_gate, one group per head).  With norm_weight set, out holds
   *   x * rsqrt(mean_d(x^2) + norm_eps) * norm_weight[d] * act(z[b, h, d])
   * where x is the bf16 attention output and act is SiLU (norm_act 0) or the
   * sigmoid (1); with gate_z NULL there is no gate.  fp32 arithmetic, bf16
   * result.  The state update is unchanged. */
  const float* norm_weight; /* [D] or NULL */
  const gdn_bf16_t* gate_z; /* [B, HV, D], sequence stride z_stride, or NULL */
  int64_t z_stride;         /* elements between sequences (a multiple of 8); 0 = HV * D */
  float norm_eps;           /* > 0 */
  int32_t norm_act;         /* 0: SiLU, 1: sigmoid */
  /* Pool layout.  0: the three dense arrays above.  Otherwise the record
   * layout, in which every (slot, head) tile is one record of this many bytes
   * (a multiple of 16, at least 9220) holding its codes at byte 0, its scales
   * at byte 8192 and its global scale at byte 9216: pool_codes, pool_scales
   * and pool_gscale then point at bytes 0, 8192 and 9216 of the first record,
   * and all three advance by the record size.  A serving engine that
   * allocates one byte array per layer for its recurrent state (vLLM's
   * mamba state cache) holds the pool in it this way. */
  int64_t pool_tile_stride;
} gdn_decode_params;

GDN_API int gdn_decode(const gdn_decode_params* params, cudaStream_t stream);

/* ---- chunked prefill (many tokens per sequence) -----------------------------
 * The same recurrence as gdn_decode applied to every token of variable-length
 * sequences, computed in chunks of 64 tokens in the WY/UT form.  Sequence n
 * owns tokens [cu_seqlens[n], cu_seqlens[n+1]) of the packed q/k/v/g/beta/out
 * rows.  Its initial state is the pool tile at slot_idx[n] when
 * has_initial_state[n] != 0 (zero otherwise); its final state is quantised
 * into that slot with a fresh global scale.  slot_idx == NULL (or a negative
 * slot) runs the sequence from a zero state and keeps no final state.
 * The reference has no prefill; its per-token Python loop
 * (src/ops/qwen35_gdn_patch.py:98-116) is what this replaces. */
typedef struct gdn_prefill_params {
  int32_t num_seqs;       /* N */
  int32_t num_k_heads;    /* HK */
  int32_t num_v_heads;    /* HV, a multiple of HK */
  int32_t head_dim;       /* d_k = d_v = 128 */
  int64_t total_tokens;   /* rows of q, k, v, g, beta, out */
  int64_t num_slots;      /* pool slots */
  const gdn_bf16_t* q;    /* [T, HK, D], token stride q_stride */
  const gdn_bf16_t* k;    /* [T, HK, D] */
  const gdn_bf16_t* v;    /* [T, HV, D] */
  int64_t q_stride;       /* elements between tokens; 0 = HK*D */
  int64_t k_stride;       /* 0 = HK*D */
  int64_t v_stride;       /* 0 = HV*D */
  const float* g;         /* [T, HV] log decay */
  const float* beta;      /* [T, HV] */
  const int32_t* cu_seqlens;         /* [N + 1], non-decreasing, within [0, T] */
  const int32_t* slot_idx;           /* [N] or NULL */
  const uint8_t* has_initial_state;  /* [N] (bool) or NULL = all zero */
  uint8_t* pool_codes;    /* [num_slots, HV, D, D/2] */
  uint8_t* pool_scales;   /* [num_slots, HV, D, D/16] */
  float* pool_gscale;     /* [num_slots, HV] */
  gdn_bf16_t* out;        /* [T, HV, D] */
  float q_scale;          /* <= 0 selects 1/sqrt(D) */
  int32_t scale_mode;     /* GDN_SCALE_* */
  float gscale_den;       /* <= 0 selects 6*saturation */
  float* debug_y;         /* optional [N, HV, D, D]: fp32 quantiser inputs of the final states */
  int64_t pool_tile_stride; /* pool layout, as in gdn_decode_params (0: dense arrays) */
  int32_t qk_l2norm;      /* != 0: q and k scaled to unit L2 norm per token and head, x / sqrt(sum x^2 + 1e-6),
                             in fp32 inside the kernel (vLLM's use_qk_l2norm_in_kernel) */
  /* Optional fused gating, as in gdn_decode_params: with A_log set, g and beta
   * are computed in the kernel for every token t and value head h from the
   * gate projections, and the g / beta fields are not read:
   *   g = -exp(A_log[h]) * softplus(gate_a[t, h] + dt_bias[h]),  beta = sigmoid(gate_b[t, h])
   * (softplus with threshold 20, as torch.nn.functional.softplus). */
  const float* A_log;       /* [HV] */
  const float* dt_bias;     /* [HV] */
  const gdn_bf16_t* gate_a; /* [T, HV], token stride gate_stride */
  const gdn_bf16_t* gate_b; /* [T, HV], token stride gate_stride */
  int64_t gate_stride;      /* elements between tokens; 0 = HV */
} gdn_prefill_params;

GDN_API int gdn_prefill(const gdn_prefill_params* params, cudaStream_t stream);

/* ---- state pool ------------------------------------------------------------ */

/* Copies tiles pool[slot_idx[i]] -> dense[i] for i < n (negative slot: the
 * dense tile is zeroed).  Tile = HV heads of D x D states.  A slot >=
 * num_slots is treated as padding and sets GDN_STATUS_BAD_SLOT. */
GDN_API int gdn_pool_gather(const uint8_t* pool_codes, const uint8_t* pool_scales, const float* pool_gscale,
                    int64_t num_slots, int32_t num_v_heads, int32_t head_dim,
                    const int32_t* slot_idx, int32_t n, uint8_t* dense_codes,
                    uint8_t* dense_scales, float* dense_gscale, cudaStream_t stream);

/* Copies dense[i] -> pool[slot_idx[i]] (negative slot: skipped; a slot >=
 * num_slots is skipped and sets GDN_STATUS_BAD_SLOT). */
GDN_API int gdn_pool_scatter(const uint8_t* dense_codes, const uint8_t* dense_scales,
                     const float* dense_gscale, int64_t num_slots, int32_t num_v_heads,
                     int32_t head_dim, const int32_t* slot_idx, int32_t n, uint8_t* pool_codes,
                     uint8_t* pool_scales, float* pool_gscale, cudaStream_t stream);

/* ---- the out-projection's all-reduce over peer memory ------------------------ */
/* No counterpart in the reference, whose layer ends in a single-GPU out-projection
 * (src/ops/qwen35_gdn_patch.py:118-121).  Under tensor parallelism every rank holds
 * a partial [B, hidden] bf16 product and the layer output is their sum: one
 * process per GPU, every rank's peer buffer mapped into every other rank. */

/* Bytes of one rank's peer buffer for summands of up to capacity_bytes
 * (a multiple of 16): 2 * capacity_bytes plus 16 KiB of flags. */
GDN_API int gdn_peer_buffer_bytes(int64_t capacity_bytes, int64_t* total_bytes);

/* Set-up, once per rank (allocates with cudaMalloc, zeroes and synchronises
 * the current device): this rank's peer buffer and its CUDA IPC handle
 * (64 bytes, cudaIpcMemHandle_t) to send to the other ranks. */
GDN_API int gdn_peer_buffer_create(int64_t capacity_bytes, void** base, void* ipc_handle);
/* Set-up: maps another rank's peer buffer from its IPC handle. */
GDN_API int gdn_peer_buffer_open(const void* ipc_handle, void** base);
/* Tear-down: unmaps another rank's buffer / frees this rank's.  Call them only
 * when no rank has an all-reduce in flight. */
GDN_API int gdn_peer_buffer_close(void* base);
GDN_API int gdn_peer_buffer_destroy(void* base);

typedef struct gdn_peer_allreduce_params {
  void* bases[8];          /* every rank's peer buffer as mapped in this process (bases[rank]: its own) */
  int32_t rank, nranks;    /* 1 <= nranks <= 8 */
  int64_t capacity_bytes;  /* as passed to gdn_peer_buffer_create, the same on every rank */
  const gdn_bf16_t* src;   /* this rank's summand [count], 16-byte aligned */
  gdn_bf16_t* dst;         /* the sum [count] (may equal src), 16-byte aligned */
  int64_t count;           /* multiple of 8 * nranks, 2 * count <= capacity_bytes */
  uint64_t timeout_ns;     /* bound on each wait for the other ranks (0: 2 s) */
} gdn_peer_allreduce_params;

/* dst = the sum over the ranks of their src (fp32 sum in rank order, one
 * rounding to bf16; every rank gets the same bytes).  Every rank must make the
 * same sequence of calls with the same count; the kernel of one call waits for
 * the other ranks' kernels of that call (bounded: a wait that runs out sets
 * GDN_STATUS_WAIT_TIMEOUT and the kernel ends early, after which the buffers
 * must be re-created).  Calls of one rank must not overlap on the GPU.  The
 * kernel keeps its own call count in the buffer, so a call captured in a CUDA
 * graph may be replayed.  Stream-ordered. */
GDN_API int gdn_peer_allreduce_bf16(const gdn_peer_allreduce_params* params, cudaStream_t stream);

/* ---- library ----------------------------------------------------------------- */

/* Reads (and with clear != 0 resets) the device status word of the current
 * device after synchronising `stream`.  This call blocks the host. */
GDN_API int gdn_b200_device_status(uint32_t* status_out, int clear, cudaStream_t stream);

/* Self-test of the bounded wait behind GDN_STATUS_WAIT_TIMEOUT (no counterpart
 * in the reference, whose waits are host-side).  One thread on the device waits
 * on an mbarrier phase that completes, then on one that nothing completes;
 * the second wait must give up after timeout_us (1 .. 2,000,000) and set
 * GDN_STATUS_WAIT_TIMEOUT.  result: device int32[3] = {first wait succeeded,
 * second wait succeeded, microseconds the second waited}.  Stream-ordered. */
GDN_API int gdn_b200_selftest_wait(uint32_t timeout_us, int32_t* result, cudaStream_t stream);

/* Self-test of the device codec (no counterpart in the reference): runs a
 * production encoder over the fp32 values whose bit patterns are lo_bits,
 * lo_bits + 1, ..., lo_bits + count - 1 (lo_bits + count <= 2^32) and writes
 * one byte per value to the device array out [count]:
 *   which 0: the block scale byte the requantisers write for a block whose
 *            max |y| is that value (finite, >= 0), in scale_mode;
 *   which 1: the E2M1 nibble of that value at inverse scale 1.
 * The tests compare every finite input against the reference's encoders.
 * Stream-ordered. */
GDN_API int gdn_b200_selftest_codec(int32_t which, uint32_t lo_bits, int64_t count, int32_t scale_mode,
                                    uint8_t* out, cudaStream_t stream);

GDN_API const char* gdn_b200_error_string(int code);
GDN_API const char* gdn_b200_version(void);

#ifdef __cplusplus
}
#endif
#endif /* GDN_B200_H_ */
