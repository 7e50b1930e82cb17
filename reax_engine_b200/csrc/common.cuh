// common.cuh -- shared device helpers of the NVFP4 MoE library (sm_100a).
//
// NVFP4 numerics follow the reference's quantiser (engine/fp4.py:27-52, engine/fp4_triton.py:16-27):
//   s  = e4m3_rn(min(bamax / (6 g), 448)),  sf = max(float(s) * g, 1e-30),  q = x / sf  (IEEE division),
//   code = index of q on the e2m1 grid, ties to the even index, sign bit = (q < 0).
// All float operations that the oracle reproduces use explicit _rn intrinsics so that nvcc cannot contract
// them into FMAs.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/reaxmoe.h"

namespace reaxmoe {

constexpr int kMaxExperts = 256;
constexpr int kMaxTopk = 16;
constexpr int kMaxRanks = 64;     // expert-parallel ranks
constexpr int kPermUnits = 3;     // 32-element units per lane and token in the permute kernels: hidden <= 3072
constexpr int kSegTokens = 128;   // tokens per routing segment (count / permute CTA)

__host__ __device__ inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Scale-atom row blocks needed for S routed slots over E experts: sum_e ceil(count_e / 128) <= S/128 + E.
__host__ __device__ inline int64_t sf_row_blocks(int64_t slots, int experts) { return slots / 128 + experts + 1; }

// Byte offset of scale (row, 16-element block kb) in the 128x4 atom layout of a matrix with K/64 atom columns
// (engine/fp4.py:16-24; engine/fp4_triton.py:38-39).
__host__ __device__ inline int64_t sf_offset(int64_t row, int kb, int k64) {
  return ((row >> 7) * k64 + (kb >> 2)) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + (kb & 3);
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// e4m3 (fn) round-to-nearest-even of a value in [0, 448] (torch .to(float8_e4m3fn) at engine/fp4.py:47).
__device__ __forceinline__ uint32_t e4m3_rn(float x) {
  return (uint32_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// e2m1 code of q (already divided by the block scale): thresholds at the grid midpoints, ties to the even
// index (engine/fp4.py:27-36; the same comparisons as engine/fp4_triton.py:24-26).
__device__ __forceinline__ uint32_t e2m1_code(float q) {
  const float a = fabsf(q);
  uint32_t idx = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.0f);
  return idx | ((q < 0.0f) ? 8u : 0u);
}

// Division-free e2m1 decision thresholds for one block with scale sf. The reference rounds q = fl(x / sf) to fp32
// and then compares q with the grid midpoints m (q > m for the midpoints that tie down, q >= m for those that tie
// up). Because every midpoint has an even fp32 significand, fl(x / sf) > m  <=>  x / sf > m + ulp(m)/2 and
// fl(x / sf) >= m  <=>  x / sf >= m - ulp-(m)/2 exactly. Each shifted midpoint c has at most 25 significant bits,
// so c * sf (<= 49 bits) is exact in fp64. T[i] is then the float threshold such that, for any float a = |x|,
// (a > T[i]) is exactly the i-th comparison: T = RD(c * sf) for the strict ones, the largest float below c * sf
// for the non-strict ones.
__device__ __forceinline__ void e2m1_thresholds(float sf, float (&T)[7]) {
  const double c[7] = {0.25 + 0x1p-26, 0.75 - 0x1p-25, 1.25 + 0x1p-24, 1.75 - 0x1p-24,
                       2.5 + 0x1p-23,  3.5 - 0x1p-23,  5.0 + 0x1p-22};
  const double s = (double)sf;
#pragma unroll
  for (int i = 0; i < 7; ++i) {
    const double P = c[i] * s;
    float f = __double2float_rd(P);
    if ((i & 1) && (double)f == P) f = __int_as_float(__float_as_int(f) - 1);  // P > 0 always
    T[i] = f;
  }
}

// The sign of fl(x / sf) is set iff x < 0 and the quotient does not underflow to -0, i.e. |x| > sf * 2^-150 (a
// quotient of exactly 2^-150 rounds to 0, ties to even). With z = RD(sf * 2^-150) (exact in fp64, then rounded down
// to float), |x| > sf * 2^-150  <=>  |x| > z for any float |x|.
__device__ __forceinline__ float zero_threshold(float sf) { return __double2float_rd((double)sf * 0x1p-150); }

// e2m1 code of x / sf, identical to e2m1_code(__fdiv_rn(x, sf)) for the thresholds T and zero threshold z of sf.
__device__ __forceinline__ uint32_t e2m1_code_t(float x, const float (&T)[7], float z) {
  const float a = fabsf(x);
  const uint32_t idx = (a > T[0]) + (a > T[1]) + (a > T[2]) + (a > T[3]) + (a > T[4]) + (a > T[5]) + (a > T[6]);
  return idx | ((x < 0.0f && a > z) ? 8u : 0u);
}

// Quantise one 16-element block with dequant-side global scale g. Returns the e4m3 scale byte; writes the
// 8 packed bytes (element 2i in the low nibble of byte i) into lo/hi words. Numerics of engine/fp4.py:45-51.
__device__ __forceinline__ uint32_t quant_block16(const float (&v)[16], float g, uint32_t& lo, uint32_t& hi) {
  float bamax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bamax = fmaxf(bamax, fabsf(v[i]));
  const float s = fminf(__fdiv_rn(bamax, __fmul_rn(6.0f, g)), 448.0f);
  const uint32_t s8 = e4m3_rn(s);
  const float sf = fmaxf(__fmul_rn(e4m3_to_f32(s8), g), 1e-30f);
  float T[7];
  e2m1_thresholds(sf, T);
  const float z = zero_threshold(sf);
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i >> 3] |= e2m1_code_t(v[i], T, z) << ((i & 7) * 4);
  lo = w[0];
  hi = w[1];
  return s8;
}

// The same quantisation for 16 values that are exactly bf16 (packed pairs, element 2i in the low half of xw[i]),
// two elements per instruction. For a bf16 value a and a float threshold T >= 0, a > T  <=>  a > Tb with Tb = T
// truncated to bf16 (T's upper 16 bits): Tb <= T < the next bf16 above Tb. So the decisions run as bf16x2
// comparisons against truncated thresholds, as a 3-level binary search over the 7 (non-decreasing) thresholds:
// bit 2 = a > T3; bit 1 = a > (bit2 ? T5 : T1); bit 0 = a > T[4*bit2 + 2*bit1]. The sign bit is x < 0 and
// |x| > z (zero_threshold, truncated to bf16 the same way), as in the fp32 path: -0, NaN and quotients that underflow
// to -0 get no sign.
__device__ __forceinline__ uint32_t bf2_gt(uint32_t a, uint32_t b) {
  return __hgt2_mask(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
}
__device__ __forceinline__ uint32_t quant_block16_bf16(const uint32_t (&xw)[8], float g, uint32_t& lo, uint32_t& hi) {
  uint32_t ab[8];
  __nv_bfloat162 m2;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ab[i] = xw[i] & 0x7FFF7FFFu;
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&ab[i]);
    m2 = i == 0 ? v : __hmax2(m2, v);
  }
  const float bamax = fmaxf(__low2float(m2), __high2float(m2));
  const float s = fminf(__fdiv_rn(bamax, __fmul_rn(6.0f, g)), 448.0f);
  const uint32_t s8 = e4m3_rn(s);
  const float sf = fmaxf(__fmul_rn(e4m3_to_f32(s8), g), 1e-30f);
  float T[7];
  e2m1_thresholds(sf, T);
  uint32_t tb[7];
#pragma unroll
  for (int i = 0; i < 7; ++i) tb[i] = (__float_as_uint(T[i]) >> 16) * 0x00010001u;
  const uint32_t zb = (__float_as_uint(zero_threshold(sf)) >> 16) * 0x00010001u;
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t a = ab[i];
    const uint32_t m2b = bf2_gt(a, tb[3]);
    const uint32_t t1 = (m2b & tb[5]) | (~m2b & tb[1]);
    const uint32_t m1b = bf2_gt(a, t1);
    const uint32_t ta = (m1b & tb[6]) | (~m1b & tb[4]);
    const uint32_t tc = (m1b & tb[2]) | (~m1b & tb[0]);
    const uint32_t t0 = (m2b & ta) | (~m2b & tc);
    const uint32_t m0b = bf2_gt(a, t0);
    const uint32_t neg = __hlt2_mask(*reinterpret_cast<const __nv_bfloat162*>(&xw[i]), __float2bfloat162_rn(0.0f)) &
                         bf2_gt(a, zb);
    const uint32_t idx = (m2b & 0x00040004u) | (m1b & 0x00020002u) | (m0b & 0x00010001u) | (neg & 0x00080008u);
    const uint32_t byte = (idx & 0xFu) | ((idx >> 12) & 0xF0u);
    w[i >> 2] |= byte << (8 * (i & 3));
  }
  lo = w[0];
  hi = w[1];
  return s8;
}

// Unpack 8 bf16 (one uint4) to floats.
__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return l | (h << 16);
}

// 256-bit global store of 8 words (one full 32-byte sector per lane; sm_100 vector width).
__device__ __forceinline__ void st_global_v8(void* ptr, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(ptr), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// Device status word: first error wins.
__device__ __forceinline__ void set_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

}  // namespace reaxmoe
