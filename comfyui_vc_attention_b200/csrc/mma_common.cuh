// Helpers shared by the register-MMA (mma.sync m16n8k32 E4M3) attention
// kernels: dense (attn_mma.cu) and block-sparse (attn_sparse.cu).
#pragma once

#include "kernels.cuh"

namespace vcattn {
namespace mmak {

constexpr int kWarps = 4;
constexpr int kRowsPerCta = 16 * kWarps;

__device__ __forceinline__ void mma_e4m3(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ExpCast byte, in the operation order of expcast.py:67-69.
__device__ __forceinline__ float expcast_code(float s, float m, float c0) {
  const float u = __fadd_rn(__fmul_rn(__fsub_rn(s, m), kLog2e), 8.0f);
  float c = rintf(__fmaf_rn(u, 8.0f, c0));    // u * 8 is exact, so the FMA is the add
  return fminf(fmaxf(c, 0.0f), 120.0f);
}

template <int ODT>
__device__ __forceinline__ void store_out2(void* out, int64_t off, float a, float b) {
  if constexpr (ODT == VCATTN_DTYPE_BF16) {
    *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(out) + off) = __floats2bfloat162_rn(a, b);
  } else if constexpr (ODT == VCATTN_DTYPE_F16) {
    *reinterpret_cast<__half2*>(static_cast<__half*>(out) + off) = __floats2half2_rn(a, b);
  } else {
    *reinterpret_cast<float2*>(static_cast<float*>(out) + off) = make_float2(a, b);
  }
}

template <int BR, int D>
struct TileSmem {
  static constexpr int kKStride = D + 16;     // bytes; conflict-free B loads
  static constexpr int kVStride = BR + 16;    // bytes
  static constexpr int kKBytes = BR * kKStride;
  static constexpr int kVBytes = D * kVStride;
  static constexpr int kStage = kKBytes + kVBytes + BR * 4 + 2 * D * 4 + 2 * D * 4;
  // per stage: K | Vt | ks[BR] | vs[D] | mu[D] | cvec[D] | mvec[D]
};

template <int BR, int D>
__device__ __forceinline__ void load_tile(uint8_t* st, const AttnParams& p, int g, int j, int tid) {
  using S = TileSmem<BR, D>;
  const int nb = p.n_pad / BR;
  const uint8_t* kg = p.k8 + (static_cast<int64_t>(g) * p.n_pad + static_cast<int64_t>(j) * BR) * D;
  for (int c = tid; c < BR * D / 16; c += kWarps * 32) {
    const int row = c / (D / 16), col = c % (D / 16);
    cp_async16(st + row * S::kKStride + col * 16, kg + row * D + col * 16);
  }
  const uint8_t* vg = p.v8t + (static_cast<int64_t>(g) * nb + j) * D * BR;
  uint8_t* vs = st + S::kKBytes;
  for (int c = tid; c < D * BR / 16; c += kWarps * 32) {
    const int row = c / (BR / 16), col = c % (BR / 16);
    cp_async16(vs + row * S::kVStride + col * 16, vg + row * BR + col * 16);
  }
  float* ks = reinterpret_cast<float*>(st + S::kKBytes + S::kVBytes);
  const float* ksg = p.k_scale + static_cast<int64_t>(g) * p.n_pad + static_cast<int64_t>(j) * BR;
  for (int c = tid; c < BR / 4; c += kWarps * 32) cp_async16(ks + c * 4, ksg + c * 4);
  float* vsc = ks + BR;
  float* mu = vsc + D;
  const float* vsg = p.v_scale + (static_cast<int64_t>(g) * nb + j) * D;
  const float* mug = p.mu + (static_cast<int64_t>(g) * nb + j) * D;
  for (int c = tid; c < D / 4; c += kWarps * 32) {
    cp_async16(vsc + c * 4, vsg + c * 4);
    cp_async16(mu + c * 4, mug + c * 4);
  }
}



// One exact KV tile (triton_attn.py:254-318, the body :324-382 shares):
// S = Q K^T on E4M3, scale by qs * ks * sm_scale, mask padding keys, online
// softmax with P as E4M3 (exp2 * 448 cast or the ExpCast byte in the
// reference's operation order), r = rowsum(P) / 448, then
// o = alpha * o + (P V8) * vs / 448 + r * mu * vs.  `st` is a staged tile
// (TileSmem layout); every thread of the CTA calls this together.
template <int BR, int D, bool EXPCAST>
__device__ __forceinline__ void exact_tile(uint8_t* st, const uint32_t (&qa)[D / 32][4], float qs0, float qs1,
                                           int kv0, int N, float sm_scale, float c0, int tid, int gid, int tig,
                                           float (&o)[D / 8][4], float (&m_i)[2], float (&l_i)[2]) {
  using S = TileSmem<BR, D>;
  const uint8_t* ks8 = st;
  const uint8_t* vt8 = st + S::kKBytes;
  const float* ksc = reinterpret_cast<const float*>(st + S::kKBytes + S::kVBytes);
  const float* vsc = ksc + BR;
  const float* mu = vsc + D;
  float* cvec = const_cast<float*>(mu + D);
  float* mvec = cvec + D;
  for (int d = tid; d < D; d += kWarps * 32) {
    cvec[d] = __fdiv_rn(vsc[d], 448.0f);           // vs / P_SCALE
    mvec[d] = __fmul_rn(mu[d], vsc[d]);            // mu * vs
  }
  __syncthreads();

  // ---- S = Q K^T -------------------------------------------------------
  float s[BR / 8][4];
#pragma unroll
  for (int n = 0; n < BR / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < D / 32; ++kk) {
#pragma unroll
    for (int n = 0; n < BR / 8; ++n) {
      const uint8_t* kr = ks8 + (n * 8 + gid) * S::kKStride + kk * 32 + tig * 4;
      mma_e4m3(s[n], qa[kk], *reinterpret_cast<const uint32_t*>(kr),
               *reinterpret_cast<const uint32_t*>(kr + 16));
    }
  }
  // ---- scale, mask, row max -------------------------------------------
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int n = 0; n < BR / 8; ++n) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = n * 8 + tig * 2 + e;
      const float kscv = ksc[col];
      const bool valid = kv0 + col < N;
      float v0 = __fmul_rn(__fmul_rn(s[n][e], __fmul_rn(qs0, kscv)), sm_scale);
      float v1 = __fmul_rn(__fmul_rn(s[n][2 + e], __fmul_rn(qs1, kscv)), sm_scale);
      v0 = valid ? v0 : -1.0e30f;
      v1 = valid ? v1 : -1.0e30f;
      s[n][e] = v0;
      s[n][2 + e] = v1;
      mx0 = fmaxf(mx0, v0);
      mx1 = fmaxf(mx1, v1);
    }
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  float mn[2] = {fmaxf(m_i[0], mx0), fmaxf(m_i[1], mx1)};
  float alpha[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (mn[r] == -INFINITY) mn[r] = 0.f;
    alpha[r] = (m_i[r] == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m_i[r], mn[r]), kLog2e));
  }
  // ---- P bytes (A operand of PV), row sums ------------------------------
  uint32_t pa[BR / 32][4];
  float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
  for (int n = 0; n < BR / 8; ++n) {
    uint32_t b01, b23;   // bytes for (row gid: e=0,1) and (row gid+8: e=0,1)
    if constexpr (EXPCAST) {
      const float e0 = expcast_code(s[n][0], mn[0], c0), e1 = expcast_code(s[n][1], mn[0], c0);
      const float e2 = expcast_code(s[n][2], mn[1], c0), e3 = expcast_code(s[n][3], mn[1], c0);
      b01 = static_cast<uint32_t>(e0) | (static_cast<uint32_t>(e1) << 8);
      b23 = static_cast<uint32_t>(e2) | (static_cast<uint32_t>(e3) << 8);
    } else {
      const float e0 = __fmul_rn(exp2f(__fmul_rn(__fsub_rn(s[n][0], mn[0]), kLog2e)), 448.0f);
      const float e1 = __fmul_rn(exp2f(__fmul_rn(__fsub_rn(s[n][1], mn[0]), kLog2e)), 448.0f);
      const float e2 = __fmul_rn(exp2f(__fmul_rn(__fsub_rn(s[n][2], mn[1]), kLog2e)), 448.0f);
      const float e3 = __fmul_rn(exp2f(__fmul_rn(__fsub_rn(s[n][3], mn[1]), kLog2e)), 448.0f);
      b01 = e4m3x2(e0, e1);
      b23 = e4m3x2(e2, e3);
    }
    rs0 += e4m3_to_float(b01 & 0xff) + e4m3_to_float(b01 >> 8);
    rs1 += e4m3_to_float(b23 & 0xff) + e4m3_to_float(b23 >> 8);
    const int ks = n >> 2, q = n & 3;    // 32-key step, n8 block within it
    const int reg_r0 = (q < 2) ? 0 : 2;  // a0/a2 hold row gid, a1/a3 row gid+8
    const int shift = (q & 1) * 16;
    if (q == 0 || q == 2) {
      pa[ks][reg_r0] = b01;
      pa[ks][reg_r0 + 1] = b23;
    } else {
      pa[ks][reg_r0] |= b01 << shift;
      pa[ks][reg_r0 + 1] |= b23 << shift;
    }
  }
  rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
  rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
  rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
  rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
  const float r0 = __fdiv_rn(rs0, 448.0f), r1 = __fdiv_rn(rs1, 448.0f);
  // ---- PV, per-tile scale, mean restoration -----------------------------
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) {
    float t[4] = {0.f, 0.f, 0.f, 0.f};
    const uint8_t* vr = vt8 + (nd * 8 + gid) * S::kVStride + tig * 2;
#pragma unroll
    for (int ks = 0; ks < BR / 32; ++ks) {
      const uint8_t* v = vr + ks * 32;
      const uint32_t b0 = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(v)) |
                          (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(v + 8)) << 16);
      const uint32_t b1 = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(v + 16)) |
                          (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(v + 24)) << 16);
      mma_e4m3(t, pa[ks], b0, b1);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = nd * 8 + tig * 2 + e;
      const float cv = cvec[col], mv = mvec[col];
      float a0 = __fmul_rn(o[nd][e], alpha[0]);
      a0 = __fadd_rn(a0, __fmul_rn(t[e], cv));
      o[nd][e] = __fadd_rn(a0, __fmul_rn(r0, mv));
      float a1 = __fmul_rn(o[nd][2 + e], alpha[1]);
      a1 = __fadd_rn(a1, __fmul_rn(t[2 + e], cv));
      o[nd][2 + e] = __fadd_rn(a1, __fmul_rn(r1, mv));
    }
  }
  l_i[0] = __fadd_rn(__fmul_rn(l_i[0], alpha[0]), r0);
  l_i[1] = __fadd_rn(__fmul_rn(l_i[1], alpha[1]), r1);
  m_i[0] = mn[0];
  m_i[1] = mn[1];
}

}  // namespace mmak
}  // namespace vcattn
