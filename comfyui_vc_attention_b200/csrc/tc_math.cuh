// Shared arithmetic of the tcgen05 attention kernels: packed fp32 helpers,
// the one-FMA ExpCast byte packer, the output staging store and per-warp
// mbarrier arrivals.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace vcattn {
namespace tc {

// One arrival per warp: the lanes' earlier shared-memory and tensor-memory
// work is ordered before lane 0's (release) arrive by __syncwarp.
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// ---- packed fp32 helpers ---------------------------------------------------
__device__ __forceinline__ void mul2(float& a, float& b, float x, float y) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "mul.rn.f32x2 rc, ra, rb;\n\tmov.b64 {%0, %1}, rc;\n\t}\n"
      : "+f"(a), "+f"(b)
      : "f"(x), "f"(y));
}
// (a, b) = (x0, x1) * (y0, y1) + (a, b)
__device__ __forceinline__ void fma2(float& a, float& b, float x0, float x1, float y0, float y1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%0, %1};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\tmov.b64 {%0, %1}, rc;\n\t}\n"
      : "+f"(a), "+f"(b)
      : "f"(x0), "f"(x1), "f"(y0), "f"(y1));
}
__device__ __forceinline__ void add2(float& a, float& b, float x, float y) {
  asm("{\n\t.reg .b64 ra, rb;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "add.rn.f32x2 ra, ra, rb;\n\tmov.b64 {%0, %1}, ra;\n\t}\n"
      : "+f"(a), "+f"(b)
      : "f"(x), "f"(y));
}
__device__ __forceinline__ float fma_sat(float a, float b, float c) {
  float d;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Four ExpCast codes (fma.sat to [0,1] in units of 128 codes, then + 98304
// rounds to an integer in the low byte) packed into one word.  The word of
// c = 98304 + code / 128 is 0x47c00000 + code, so a + (b << 8) holds
// code_a | code_b << 8 in its low half (no carry out of the low byte); one
// byte permute joins the halves.
__device__ __forceinline__ uint32_t expcast4(float x0, float x1, float x2, float x3, float As, float Bs) {
  float c0 = fma_sat(x0, As, Bs), c1 = fma_sat(x1, As, Bs);
  float c2 = fma_sat(x2, As, Bs), c3 = fma_sat(x3, As, Bs);
  add2(c0, c1, 98304.0f, 98304.0f);
  add2(c2, c3, 98304.0f, 98304.0f);
  const uint32_t lo = __float_as_uint(c0) + (__float_as_uint(c1) << 8);
  const uint32_t hi = __float_as_uint(c2) + (__float_as_uint(c3) << 8);
  return __byte_perm(lo, hi, 0x5410);
}
// Four E4M3(exp2(x * Ae + Be)) bytes packed into one word.
__device__ __forceinline__ uint32_t exp4(float x0, float x1, float x2, float x3, float Ae, float Be) {
  float t0 = Be, t1 = Be, t2 = Be, t3 = Be;
  fma2(t0, t1, x0, x1, Ae, Ae);
  fma2(t2, t3, x2, x3, Ae, Ae);
  return e4m3x4(exp2f(t0), exp2f(t1), exp2f(t2), exp2f(t3));
}

// Two adjacent output values of one row, converted and written to the
// staging tile.
template <int ODT>
__device__ __forceinline__ void stage2(uint8_t* base, float v0, float v1) {
  if constexpr (ODT == VCATTN_DTYPE_BF16) {
    *reinterpret_cast<__nv_bfloat162*>(base) = __floats2bfloat162_rn(v0, v1);
  } else if constexpr (ODT == VCATTN_DTYPE_F16) {
    *reinterpret_cast<__half2*>(base) = __floats2half2_rn(v0, v1);
  } else {
    *reinterpret_cast<float2*>(base) = make_float2(v0, v1);
  }
}

}  // namespace tc
}  // namespace vcattn
