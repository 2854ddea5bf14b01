// Device helpers shared by the quantizer and GEMV kernels (sm_100a).
//
// Format facts (KURN split layout; ggml block formats):
//   q4_0  32 values per block: 16 quant bytes in WQ, byte i holds value i (low nibble) and value i+16 (high nibble),
//         value = d * (nibble - 8), d = f16 in WS.                       (patches/0001-language-extra-kurn.patch:16-17)
//   tq2_0 256 values per block: 64 quant bytes, value v in byte (v/128)*32 + v%32 at bits 2*((v%128)/32),
//         value = d * (crumb - 1).                                         (patch:18-19, 58-63)
//   q8_0  32 int8 per block + f32 copy of the f16-rounded scale.           (patch:20-21, 104-114)
//   q8_K  256 int8 per block + f32 scale.                                  (patch:117-131)
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2q {

// ---------------------------------------------------------------------------------------------------------------
// Integer dot products
// ---------------------------------------------------------------------------------------------------------------

// c + sum of the four signed-byte products of a and b (PTX dp4a.s32.s32), the reference's ktl.dp4a (patch:73-81).
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }

// c + sum of (unsigned byte of a) * (signed byte of b) (PTX dp4a.u32.s32). Used on masked weight words whose bytes
// can reach 0xF0 / 0xC0: the product is then 2^k times the field value, removed exactly by an arithmetic shift.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ---------------------------------------------------------------------------------------------------------------
// Memory
// ---------------------------------------------------------------------------------------------------------------

// 16-byte streaming load of read-only weight data: no L1 allocation (each byte is used once per launch).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ld_stream_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// f16 bit pattern -> f32 (exact), the reference's ktl.f16_bits_to_f32 (patch:33-36).
__device__ __forceinline__ float f16_bits_to_f32(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }

// ---------------------------------------------------------------------------------------------------------------
// Activation quantizers. Only correctly rounded float operations: IEEE division, single multiplies (never fused),
// roundf (half away from zero), round half to even (rintf, or an exact add of 1.5 * 2^23: q8_K_bits), f16
// conversion with round-to-nearest-even.
// ---------------------------------------------------------------------------------------------------------------

// q8_0 for one 32-value block held by 8 consecutive lanes (4 values each, lanes aligned to a multiple of 8).
// Returns the 4 quants packed little-endian in one word, and d (unrounded f32) in *d_out.
// Follows ggml quantize_row_q8_0_ref as restated in ktl.q8_0_quantize (patch:104-114).
__device__ __forceinline__ uint32_t q8_0_quant4(float4 v, float* d_out) {
  float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
  const int q0 = (int)roundf(__fmul_rn(v.x, id));
  const int q1 = (int)roundf(__fmul_rn(v.y, id));
  const int q2 = (int)roundf(__fmul_rn(v.z, id));
  const int q3 = (int)roundf(__fmul_rn(v.w, id));
  *d_out = d;
  return (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
         ((uint32_t)(q3 & 0xff) << 24);
}

// f32(f16_rne(d)): the scale stored for a q8_0 block (the f16 ggml keeps, widened back to f32).
__device__ __forceinline__ float q8_0_stored_scale(float d) { return __half2float(__float2half_rn(d)); }

// q = min(127, rint(p)) of a q8_K product p = fl(iscale * x), |p| <= 127 + ulp, without the conversion unit:
// fl(min(p, 127) + 1.5 * 2^23) is exactly 1.5 * 2^23 + rint(min(p, 127)) (round to nearest even at unit spacing),
// whose bits are 0x4B400000 + q, so their low byte is q's byte. min before rounding equals min after it because 127
// is an integer; a NaN product gives 127 either way (fminf).
__device__ __forceinline__ uint32_t q8_K_bits(float p) {
  return __float_as_uint(__fadd_rn(fminf(p, 127.0f), 12582912.0f));
}

// The low bytes of four words, packed little-endian (a -> byte 0).
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// q8_K for one 256-value block held by a full warp (8 consecutive values per lane: lane l holds values 8l..8l+7).
// Writes the 8 quants packed into q_lo/q_hi (little-endian) and returns d (0 for an all-zero block).
// Follows ggml quantize_row_q8_K_ref as restated in ktl.q8_K_quantize (patch:117-131): the signed value with the
// largest magnitude, lowest index on ties; iscale = -127/max; q = min(127, nearest-even(iscale*x)); d = 1/iscale.
__device__ __forceinline__ float q8_K_quant8(const float (&v)[8], int lane, uint32_t* q_lo, uint32_t* q_hi) {
  float lmax = 0.0f;
  int lidx = 8;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = fabsf(v[i]);
    if (a > lmax) {  // strict: keeps the first index among equal magnitudes
      lmax = a;
      lidx = i;
    }
  }
  float amax = lmax;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // lowest index whose |x| equals amax; lanes without a match propose 256
  int first = (lmax == amax && lidx < 8) ? lane * 8 + lidx : 256;
  if (amax == 0.0f) first = 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
  float mine = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) mine = ((first & 7) == i) ? v[i] : mine;
  const float mx = __shfl_sync(0xffffffffu, mine, first >> 3);
  const bool nz = amax != 0.0f;
  const float iscale = __fdiv_rn(-127.0f, nz ? mx : 1.0f);
  uint32_t b8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) b8[i] = q8_K_bits(__fmul_rn(iscale, v[i]));
  *q_lo = nz ? pack_low_bytes(b8[0], b8[1], b8[2], b8[3]) : 0u;
  *q_hi = nz ? pack_low_bytes(b8[4], b8[5], b8[6], b8[7]) : 0u;
  return nz ? __fdiv_rn(1.0f, iscale) : 0.0f;
}

// Sum of the four signed bytes of a word.
__device__ __forceinline__ int bytesum(uint32_t w) { return __dp4a((int)w, 0x01010101, 0); }

// Programmatic dependent launch: wait until the preceding grid on the stream has completed and its writes are
// visible, then let the next grid launch (its CTAs start prefetching their own weights while this grid finishes).
// Only immutable inputs (weights) may be read before this point; activations, outputs and flags only after it.
// Without a programmatic dependency both instructions are no-ops.
__device__ __forceinline__ void pdl_wait_then_trigger() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace b2q
