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
}
