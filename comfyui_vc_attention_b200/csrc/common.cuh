// Shared device helpers for the VC-Attention sm_100a kernels.
//
// Every floating-point step that the parity tests compare bit for bit is
// written with explicit round-to-nearest intrinsics (__fadd_rn, __fmul_rn,
// __fdiv_rn, __fmaf_rn) so that nvcc cannot contract or reorder it.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/vcattn.h"

namespace vcattn {

constexpr float kE4M3Max = 448.0f;
constexpr float kTiny = 1e-30f;               // clamp(min=1e-30) of quant.py
constexpr float kLog2e = 1.4426950408889634f;  // expcast.py:47

// Device-side status word: kernels that give up on a bounded wait, or find an
// argument they cannot honour, record a code here instead of trapping.
struct DeviceStatus {
  int code;
  int where;
};

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

// float -> bf16 (round to nearest even), returned as a float holding the value.
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Input element loaders: the reference accepts bf16 / fp16 / fp32 tensors.
template <int DT> struct Elem;
template <> struct Elem<VCATTN_DTYPE_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float load(const T* p) { return __bfloat162float(*p); }
};
template <> struct Elem<VCATTN_DTYPE_F16> {
  using T = __half;
  static __device__ __forceinline__ float load(const T* p) { return __half2float(*p); }
};
template <> struct Elem<VCATTN_DTYPE_F32> {
  using T = float;
  static __device__ __forceinline__ float load(const T* p) { return *p; }
};

// Four consecutive input elements -> float4 (pointer aligned to 4 elements).
template <int DT>
__device__ __forceinline__ float4 load4(const void* base, int64_t elem_off) {
  if constexpr (DT == VCATTN_DTYPE_BF16) {
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(base) + elem_off);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
  } else if constexpr (DT == VCATTN_DTYPE_F16) {
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __half*>(base) + elem_off);
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&u.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
  } else {
    return *reinterpret_cast<const float4*>(static_cast<const float*>(base) + elem_off);
  }
}

// RNE + saturate-to-finite E4M3 encode of two floats (cvt.rn.satfinite).
// +-0 inputs give code 0x00, as quant.py:56-84 does (its sign bit is x < 0).
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  lo = __fadd_rn(lo, 0.0f);   // -0 -> +0
  hi = __fadd_rn(hi, 0.0f);
  const __nv_fp8x2_storage_t s = __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint16_t>(s);
}

__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  return static_cast<uint32_t>(e4m3x2(a, b)) | (static_cast<uint32_t>(e4m3x2(c, d)) << 16);
}

// Four E4M3 codes of a word (byte i = element i) -> their exact values.
__device__ __forceinline__ float4 e4m3x4_to_float4(uint32_t w) {
  const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w & 0xffffu), __NV_E4M3);
  const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w >> 16), __NV_E4M3);
  return make_float4(__half2float(__half(__half_raw{lo.x})), __half2float(__half(__half_raw{lo.y})),
                     __half2float(__half(__half_raw{hi.x})), __half2float(__half(__half_raw{hi.y})));
}

// E4M3 byte -> float (exact).
__device__ __forceinline__ float e4m3_to_float(uint32_t code) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(code & 0xff), __NV_E4M3);
  return __half2float(__half(h));
}

// E2M1 encode of two floats (RNE, satfinite) -> one byte, low nibble = first.
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  lo = __fadd_rn(lo, 0.0f);
  hi = __fadd_rn(hi, 0.0f);
  uint32_t out;
  asm volatile(
      "{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\t"
      "cvt.u32.u8 %0, t;\n\t}\n"
      : "=r"(out) : "f"(lo), "f"(hi));
  return out;
}

// Three-input max / min (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Per-row E4M3 scale of quant.py:107-126: max(amax, 1e-30) / 448 (IEEE).
__device__ __forceinline__ float e4m3_row_scale(float amax) {
  return __fdiv_rn(fmaxf(amax, kTiny), kE4M3Max);
}

// x / s for many x and one s, from y = RN(1 / s) (an IEEE division): Markstein's correction
// (P. Markstein, IBM J. Res. Dev. 34(1), 1990): q0 = RN(x y), r = x - q0 s
// exactly (fma), q = RN(q0 + r y).  It is the correctly rounded quotient
// whenever x / s and the residual stay in the normal range.  The E4M3 codes
// only use quotients up to 448, and any quotient below 2^-10 becomes code 0
// whatever its last bit, so the codes equal those of an IEEE division.
struct DivBy {
  float s, y;
  __device__ __forceinline__ explicit DivBy(float s_) : s(s_), y(0.f) {
#ifdef __CUDA_ARCH__
    y = __fdiv_rn(1.0f, s_);
#endif
  }
  __device__ __forceinline__ float operator()(float x) const {
    const float q0 = __fmul_rn(x, y);
    const float r = __fmaf_rn(-q0, s, x);
    return __fmaf_rn(r, y, q0);
  }
};

// In-register Walsh-Hadamard transform of a 128-wide row spread over a warp
// (lane l holds elements 4l..4l+3), followed by the IEEE division by
// fp32(sqrt(128)).  Same butterfly pairing and the same a+b / a-b as the fp32
// reference transform (hadamard.py:37-65), so the result is bit-identical.
__device__ __forceinline__ void fwht128_warp(float v[4], int lane) {
  // h = 1 and h = 2 live inside the lane.
  float a0 = __fadd_rn(v[0], v[1]), a1 = __fsub_rn(v[0], v[1]);
  float a2 = __fadd_rn(v[2], v[3]), a3 = __fsub_rn(v[2], v[3]);
  v[0] = __fadd_rn(a0, a2); v[2] = __fsub_rn(a0, a2);
  v[1] = __fadd_rn(a1, a3); v[3] = __fsub_rn(a1, a3);
  // h = 4 .. 64: partner lane = lane ^ (h / 4).
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    // lower lane: v + p, upper lane: p - v, both as one fma with a +-1
    // multiplier (rounded once, identical to the add / subtract)
    const float sg = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float p = __shfl_xor_sync(0xffffffffu, v[t], m);
      v[t] = __fmaf_rn(sg, v[t], p);
    }
  }
  // IEEE division by r = fp32(sqrt(128)) = 0x1.6a09e6p+3.  Markstein's
  // correction from y = RN(1/r) = 0x1.6a09e6p-4 equals __fdiv_rn(x, r) for
  // every fp32 x with 2^-100 <= |x| <= 2^100: an exhaustive run over all 2^32
  // inputs on B200 found 1 595 509 differences, all with |x| <= 2.2e-32 (the
  // residual leaves the normal range) or x = -0 (sign of zero).  A row holding
  // any value outside that range takes the division itself.
  const float r = 11.313708498984761f;
  const float y = 0.0883883461356163f;
  bool slow = false;
#pragma unroll
  for (int t = 0; t < 4; ++t) slow |= !(fabsf(v[t]) >= 0x1p-100f && fabsf(v[t]) <= 0x1p+100f);
  if (__any_sync(0xffffffffu, slow)) {
#pragma unroll
    for (int t = 0; t < 4; ++t) v[t] = __fdiv_rn(v[t], r);
  } else {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float q0 = __fmul_rn(v[t], y);
      v[t] = __fmaf_rn(__fmaf_rn(-q0, r, v[t]), y, q0);
    }
  }
}

// 64-wide variant: lanes 0..15 hold a row (4 elements each), lanes 16..31 a
// second row.  Partner masks stay below 16 so the halves never mix.
__device__ __forceinline__ void fwht64_halfwarp(float v[4], int lane) {
  float a0 = __fadd_rn(v[0], v[1]), a1 = __fsub_rn(v[0], v[1]);
  float a2 = __fadd_rn(v[2], v[3]), a3 = __fsub_rn(v[2], v[3]);
  v[0] = __fadd_rn(a0, a2); v[2] = __fsub_rn(a0, a2);
  v[1] = __fadd_rn(a1, a3); v[3] = __fsub_rn(a1, a3);
#pragma unroll
  for (int m = 1; m < 16; m <<= 1) {
    const float sg = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float p = __shfl_xor_sync(0xffffffffu, v[t], m);
      v[t] = __fmaf_rn(sg, v[t], p);
    }
  }
  // division by fp32(sqrt(64)) = 8: the scaling by 2^-3 is the same rounding
#pragma unroll
  for (int t = 0; t < 4; ++t) v[t] = __fmul_rn(v[t], 0.125f);
}

}  // namespace vcattn
