// ref_shim.cu -- C entry points onto the reference's own NVFP4 host code.
//
// TEST INFRASTRUCTURE ONLY (the oracle's reference leg).  Compiled by
// oracle/Makefile together with the reference source file
// src/kernel/gdn_state_update_ref.cu (and its header
// src/intrinsics/gdn_fp4_intrinsics.cuh, found through -I) into
// oracle/_ref/libgdn_ref.so.  Nothing here restates reference code: each
// function forwards to the reference's implementation so that the tests can
// call it through ctypes.
#include <cstdint>
#include "gdn_fp4_intrinsics.cuh"

// Declared (not defined) here; the definitions are the reference's,
// src/kernel/gdn_state_update_ref.cu:75-89 and :93-141.
void nvfp4_dequantise_host(const uint8_t* data_packed, const uint8_t* scales, float* out_fp32,
                           int num_elements);
void nvfp4_quantise_host(const float* in_fp32, uint8_t* data_packed, uint8_t* scales,
                         int num_elements);

extern "C" {
void ref_nvfp4_quantise(const float* in, uint8_t* codes, uint8_t* scales, int n) {
  nvfp4_quantise_host(in, codes, scales, n);
}
void ref_nvfp4_dequantise(const uint8_t* codes, const uint8_t* scales, float* out, int n) {
  nvfp4_dequantise_host(codes, scales, out, n);
}
float ref_decode_e2m1(uint32_t nib) { return sm120::intrinsics::decode_e2m1_to_f32((uint8_t)nib); }
float ref_decode_ue4m3(uint32_t b) { return sm120::intrinsics::decode_ue4m3_to_f32((uint8_t)b); }
uint32_t ref_encode_ue4m3(float x) { return sm120::intrinsics::encode_f32_to_ue4m3(x); }
// Batch form for exhaustive sweeps: encodes every float whose bit pattern is
// lo + i*stride for i < count, writing one byte each.
void ref_encode_ue4m3_sweep(uint32_t lo, uint32_t stride, uint64_t count, uint8_t* out) {
  for (uint64_t i = 0; i < count; ++i) {
    uint32_t u = lo + (uint32_t)(i * stride);
    float f;
    __builtin_memcpy(&f, &u, 4);
    out[i] = sm120::intrinsics::encode_f32_to_ue4m3(f);
  }
}
// The reference's block scale byte for every block max |y| with bit pattern
// lo + i: its two lines local_scale = amax > 0 ? amax / 6 : 1 and the encoder
// call (gdn_state_update_ref.cu:105-108), the encoder being the reference's own.
void ref_block_scale_sweep(uint32_t lo, uint64_t count, uint8_t* out) {
  for (uint64_t i = 0; i < count; ++i) {
    const uint32_t u = lo + (uint32_t)i;
    float amax;
    __builtin_memcpy(&amax, &u, 4);
    const float local = (amax > 0.0f) ? (amax / 6.0f) : 1.0f;
    out[i] = sm120::intrinsics::encode_f32_to_ue4m3(local);
  }
}
// The reference's E2M1 nibble of every value v with bit pattern lo + i and
// |v| <= 6, through its own nvfp4_quantise_host: each call quantises the block
// {6, v_0, ..., v_14}, whose max is 6, so its scale decodes to exactly 1.0 and
// element j + 1's nibble is the reference's nearest-E2M1 of v_j.
void ref_e2m1_sweep(uint32_t lo, uint64_t count, uint8_t* out) {
  float blk[16];
  uint8_t codes[8], scale;
  for (uint64_t i0 = 0; i0 < count; i0 += 15) {
    const int n = (count - i0) < 15 ? (int)(count - i0) : 15;
    blk[0] = 6.0f;
    for (int j = 0; j < 15; ++j) {
      const uint32_t u = lo + (uint32_t)(i0 + (j < n ? j : 0));
      __builtin_memcpy(&blk[j + 1], &u, 4);
    }
    nvfp4_quantise_host(blk, codes, &scale, 16);
    for (int j = 0; j < n; ++j) {
      const int e = j + 1;
      out[i0 + j] = (uint8_t)((codes[e / 2] >> (4 * (e & 1))) & 0xFu);
    }
  }
}
}
