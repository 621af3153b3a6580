// Fused dense FP8 VC-Attention on the 5th-generation tensor cores (tcgen05).
//
// Same semantics as triton_attn.py:203-322: for every KV tile j (one value
// block of BR keys)
//   s   = (q8 . k8) * qs * ks * sm_scale
//   P   = ExpCast byte of s against the running row max (one FMA form), or
//         E4M3(exp2((s - m) * log2e) * 448)
//   acc = alpha * acc + (P @ V8) * (vs / 448) + (rowsum(P) / 448) * (mu * vs)
//   l   = alpha * l + rowsum(P) / 448 ;  O = acc / l
//
// One CTA = 128 query rows of one (batch, head); 12 warps (register-limited
// blocks are sized in whole warpgroups, so the 168-register budget needs 384
// threads, of which warps 2-3 are idle):
//   warp 0      TMA producer (Q once; K, V codes + ks, vs, mu per tile, 3 stages)
//   warp 1      MMA issuer and TMEM owner
//   warps 4-7   softmax: thread = query row = TMEM lane; P row -> shared memory
//   warps 8-11  correction: thread = row; O row in registers
// A warp reads TMEM lanes 32 * (warp % 4) .. +31, so each group of four
// consecutive warps covers the 128 rows once.
// TMEM columns: S double buffer [0,128) [128,256), PV tile T [256,384),
// row sum R [384,400) (from an N=16 MMA of P against a ones block).
// Operands in shared memory use the 128-byte swizzle: Q, K and P K-major, V
// MN-major (straight from the prepare layout).  Every wait is bounded.
#include <cuda.h>
#include <cstdio>
#include <mutex>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace vcattn {

__device__ tc::DevStatus g_attn_tc_status;

namespace {

using namespace tc;
char g_tc_diag[256];

constexpr int kBM = 128;
constexpr int kD = 128;
constexpr int kStages = 3;
constexpr int kThreads = 384;   // 12 warps (3 warpgroups) at <= 168 registers each
constexpr uint32_t kColS = 0, kColT = 256, kColR = 384;

template <int BR>
struct TcSmem {
  alignas(1024) uint8_t q[kBM * 128];
  alignas(1024) uint8_t k[kStages][BR * 128];
  alignas(1024) uint8_t v[kStages][BR * 128];
  alignas(1024) uint8_t p[2][kBM * 128];
  alignas(1024) uint8_t ones[16 * 128];
  alignas(16) float ks[kStages][BR];
  alignas(16) float vs[kStages][kD];
  alignas(16) float mu[kStages][kD];
  alignas(16) float cm[4][2][kD];    // per tile: vs / 448 and mu * vs (softmax -> correction)
  alignas(16) float alpha[4][kBM];
  alignas(8) uint64_t q_full;
  alignas(8) uint64_t kv_full[kStages];
  alignas(8) uint64_t kv_empty[kStages];
  alignas(8) uint64_t s_full[2];
  alignas(8) uint64_t s_free[2];
  alignas(8) uint64_t p_full[2];
  alignas(8) uint64_t p_free[2];
  alignas(8) uint64_t t_full;
  alignas(8) uint64_t t_free;
  alignas(8) uint64_t a_full[4];   // alpha of tile j ready (ring of 4, softmax -> correction)
  alignas(8) uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct TcArgs {
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  const float* mu;
  int H, N, n_pad, nb;
  float sm_scale;
  float c120;   // 64 + 56 + beta (ExpCast)
  void* out;
  int64_t osb, osh, osn;
};

// ---- packed fp32 helpers ---------------------------------------------------
__device__ __forceinline__ void mul2(float& a, float& b, float x, float y) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "mul.rn.f32x2 rc, ra, rb;\n\tmov.b64 {%0, %1}, rc;\n\t}\n"
      : "+f"(a), "+f"(b)
      : "f"(x), "f"(y));
}
// (a, b) = (a, b) * (s, s) + (x, y) * (c0, c1) style helpers
__device__ __forceinline__ void fma2(float& a, float& b, float x0, float x1, float y0, float y1) {
  // (a, b) = (x0, x1) * (y0, y1) + (a, b)
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
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fma_sat(float a, float b, float c) {
  float d;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
template <int ODT>
__device__ __forceinline__ void store_row(void* out, int64_t off, const float (&o)[kD], float l) {
  if constexpr (ODT == VCATTN_DTYPE_BF16) {
    __nv_bfloat16* p = static_cast<__nv_bfloat16*>(out) + off;
#pragma unroll
    for (int c = 0; c < kD; c += 8) {
      uint4 w;
      __nv_bfloat162 t0 = __floats2bfloat162_rn(__fdiv_rn(o[c], l), __fdiv_rn(o[c + 1], l));
      __nv_bfloat162 t1 = __floats2bfloat162_rn(__fdiv_rn(o[c + 2], l), __fdiv_rn(o[c + 3], l));
      __nv_bfloat162 t2 = __floats2bfloat162_rn(__fdiv_rn(o[c + 4], l), __fdiv_rn(o[c + 5], l));
      __nv_bfloat162 t3 = __floats2bfloat162_rn(__fdiv_rn(o[c + 6], l), __fdiv_rn(o[c + 7], l));
      w.x = *reinterpret_cast<uint32_t*>(&t0); w.y = *reinterpret_cast<uint32_t*>(&t1);
      w.z = *reinterpret_cast<uint32_t*>(&t2); w.w = *reinterpret_cast<uint32_t*>(&t3);
      *reinterpret_cast<uint4*>(p + c) = w;
    }
  } else if constexpr (ODT == VCATTN_DTYPE_F16) {
    __half* p = static_cast<__half*>(out) + off;
#pragma unroll
    for (int c = 0; c < kD; c += 8) {
      uint4 w;
      __half2 t0 = __floats2half2_rn(__fdiv_rn(o[c], l), __fdiv_rn(o[c + 1], l));
      __half2 t1 = __floats2half2_rn(__fdiv_rn(o[c + 2], l), __fdiv_rn(o[c + 3], l));
      __half2 t2 = __floats2half2_rn(__fdiv_rn(o[c + 4], l), __fdiv_rn(o[c + 5], l));
      __half2 t3 = __floats2half2_rn(__fdiv_rn(o[c + 6], l), __fdiv_rn(o[c + 7], l));
      w.x = *reinterpret_cast<uint32_t*>(&t0); w.y = *reinterpret_cast<uint32_t*>(&t1);
      w.z = *reinterpret_cast<uint32_t*>(&t2); w.w = *reinterpret_cast<uint32_t*>(&t3);
      *reinterpret_cast<uint4*>(p + c) = w;
    }
  } else {
    float* p = static_cast<float*>(out) + off;
#pragma unroll
    for (int c = 0; c < kD; c += 4) {
      *reinterpret_cast<float4*>(p + c) =
          make_float4(__fdiv_rn(o[c], l), __fdiv_rn(o[c + 1], l), __fdiv_rn(o[c + 2], l), __fdiv_rn(o[c + 3], l));
    }
  }
}

template <int BR, bool EXPCAST, int ODT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  TcSmem<BR>& sm = *reinterpret_cast<TcSmem<BR>*>(smem_raw + pad);
  DevStatus* status = &g_attn_tc_status;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.y;
  const int row0 = blockIdx.x * kBM;
  const int nb = a.nb;

  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1 + kBM);   // PV commit + the 128 softmax threads
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.s_free[b], kBM);
      mbar_init(&sm.p_full[b], kBM);
      mbar_init(&sm.p_free[b], 1);
    }
    mbar_init(&sm.t_full, 1);
    mbar_init(&sm.t_free, kBM);
    for (int r = 0; r < 4; ++r) mbar_init(&sm.a_full[r], kBM);
    mbar_init(&sm.drain, 1);
    fence_mbar_init();
  }
  // Constant ones block (B operand of the row-sum MMA): row 0 = E4M3 1.0.
  for (int i = tid; i < 16 * 128; i += kThreads) sm.ones[i] = (i < 128) ? 0x38 : 0x00;
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp < 4) {
  // Register budget per warpgroup (launched at 168 x 384 = 64512):
  // 128 x 56 (producer, MMA, 2 idle) + 128 x 200 (softmax) + 128 x 232 (correction) = 62464.
  asm volatile("setmaxnreg.dec.sync.aligned.u32 56;\n" ::: "memory");
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int issued = 0;
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_expect_tx(&sm.q_full, kBM * 128);
      tma_load_2d(sm.q, &tm_q, 0, g * a.n_pad + row0, &sm.q_full);
      const uint32_t tile_bytes = 2u * BR * 128u + BR * 4u + 2u * kD * 4u;
      for (int j = 0; j < nb; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&sm.kv_empty[s], ((j / kStages) + 1) & 1, abort, status, 1)) break;
        mbar_expect_tx(&sm.kv_full[s], tile_bytes);
        const int krow = g * a.n_pad + j * BR;
        tma_load_2d(sm.k[s], &tm_k, 0, krow, &sm.kv_full[s]);
        tma_load_2d(sm.v[s], &tm_v, 0, krow, &sm.kv_full[s]);
        bulk_load(sm.ks[s], a.k_scale + static_cast<int64_t>(krow), BR * 4, &sm.kv_full[s]);
        const int64_t vo = (static_cast<int64_t>(g) * nb + j) * kD;
        bulk_load(sm.vs[s], a.v_scale + vo, kD * 4, &sm.kv_full[s]);
        bulk_load(sm.mu[s], a.mu + vo, kD * 4, &sm.kv_full[s]);
        issued = j + 1;
      }
      // Drain: on an abandoned run, let the copies already issued land.
      if (*abort) {
        for (int j = max(0, issued - kStages); j < issued; ++j) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&sm.kv_full[j % kStages], (j / kStages) & 1) && clock64() - t0 < kWaitCycles / 4) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_qk = idesc_e4m3(kBM, BR, false);
      const uint32_t id_pv = idesc_e4m3(kBM, kD, true);
      const uint32_t id_r = idesc_e4m3(kBM, 16, false);
      const uint32_t q_addr = smem_u32(sm.q);
      const uint32_t ones_addr = smem_u32(sm.ones);
      bool ok = mbar_wait(&sm.q_full, 0, abort, status, 2);
      for (int j = 0; ok && j <= nb; ++j) {
        if (j < nb) {
          const int s = j % kStages, b = j & 1;
          ok = mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 3);
          if (ok && j >= 2) ok = mbar_wait(&sm.s_free[b], ((j >> 1) + 1) & 1, abort, status, 4);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm.k[s]);
#pragma unroll
          for (int kk = 0; kk < kD / 32; ++kk)
            mma_f8(tbase + kColS + b * 128, desc_kmajor(q_addr + kk * 32), desc_kmajor(k_addr + kk * 32), id_qk,
                   kk > 0);
          tc_commit(&sm.s_full[b]);
        }
        if (j >= 1) {
          const int i = j - 1, bi = i & 1, si = i % kStages;
          ok = mbar_wait(&sm.p_full[bi], (i >> 1) & 1, abort, status, 5);
          if (ok && i >= 1) ok = mbar_wait(&sm.t_free, (i - 1) & 1, abort, status, 6);
          if (!ok) break;
          tc_fence_after();
          const uint32_t p_addr = smem_u32(sm.p[bi]);
          const uint32_t v_addr = smem_u32(sm.v[si]);
#pragma unroll
          for (int kk = 0; kk < BR / 32; ++kk)
            mma_f8(tbase + kColT, desc_kmajor(p_addr + kk * 32), desc_mnmajor(v_addr + kk * 32 * 128), id_pv,
                   kk > 0);
#pragma unroll
          for (int kk = 0; kk < BR / 32; ++kk)
            mma_f8(tbase + kColR, desc_kmajor(p_addr + kk * 32), desc_kmajor(ones_addr + kk * 32), id_r, kk > 0);
          tc_commit(&sm.t_full);
          tc_commit(&sm.kv_empty[si]);
          tc_commit(&sm.p_free[bi]);
        }
      }
      // Every MMA issued must finish before TMEM is released.
      tc_commit(&sm.drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(&sm.drain, 0) && clock64() - t0 < kWaitCycles) {
      }
    }
    __syncwarp();
  }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 200;\n" ::: "memory");
    // ------------------------------------------------------------ softmax
    const int t = (warp & 3) * 32 + lane;          // query row within the tile = TMEM lane
    const uint32_t lane_base = tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int row = row0 + t;
    const float qs = (row < a.n_pad) ? a.q_scale[static_cast<int64_t>(g) * a.n_pad + row] : 0.f;
    const float qsm = __fmul_rn(qs, a.sm_scale);
    // ExpCast: c = A * (x - m) + c120 with A = 8 log2e qs sm; evaluated as
    // fma.sat(x, A/128, B/128) so the clamp at 0 is free and the /128 scale
    // makes a + 98304 round the code to an integer in the low bits.
    const float A = __fmul_rn(8.0f * kLog2e, qsm);
    const float As = A * (1.0f / 128.0f);
    const float Ae = __fmul_rn(qsm, kLog2e);       // exp path: p = exp2(Ae (x - m)) * 448
    float m = -INFINITY;
    for (int j = 0; j < nb; ++j) {
      const int b = j & 1, s = j % kStages;
      if (!mbar_wait(&sm.s_full[b], (j >> 1) & 1, abort, status, 7)) break;
      if (!mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 8)) break;
      tc_fence_after();
      float x[BR];
#pragma unroll
      for (int c = 0; c < BR; c += 32) tmem_ld32(lane_base + kColS + b * 128 + c, *reinterpret_cast<float(*)[32]>(&x[c]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&sm.s_free[b]);
      const float* ks = sm.ks[s];
#pragma unroll
      for (int c = 0; c < BR; c += 4) {
        const float4 kv = *reinterpret_cast<const float4*>(ks + c);
        mul2(x[c], x[c + 1], kv.x, kv.y);
        mul2(x[c + 2], x[c + 3], kv.z, kv.w);
      }
      const int valid = a.N - j * BR;                 // columns >= valid are padding keys
      if (valid < BR) {
#pragma unroll
        for (int c = 0; c < BR; ++c)
          if (c >= valid) x[c] = -1.0e30f;
      }
      float m0 = m, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < BR; c += 8) {
        m0 = fmax3(m0, x[c], x[c + 1]);
        m1 = fmax3(m1, x[c + 2], x[c + 3]);
        m2 = fmax3(m2, x[c + 4], x[c + 5]);
        m3 = fmax3(m3, x[c + 6], x[c + 7]);
      }
      const float m_new = fmax3(m0, m1, fmaxf(m2, m3));
      const float alpha = (m == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m, m_new), Ae));
      uint32_t packed[BR / 4];
      if constexpr (EXPCAST) {
        const float Bs = __fmaf_rn(-As, m_new, a.c120 * (1.0f / 128.0f));
#pragma unroll
        for (int c = 0; c < BR; c += 4) {
          float c0 = fma_sat(x[c], As, Bs), c1 = fma_sat(x[c + 1], As, Bs);
          float c2 = fma_sat(x[c + 2], As, Bs), c3 = fma_sat(x[c + 3], As, Bs);
          add2(c0, c1, 98304.0f, 98304.0f);
          add2(c2, c3, 98304.0f, 98304.0f);
          const uint32_t lo = __byte_perm(__float_as_uint(c0), __float_as_uint(c1), 0x0040);
          const uint32_t hi = __byte_perm(__float_as_uint(c2), __float_as_uint(c3), 0x0040);
          packed[c / 4] = __byte_perm(lo, hi, 0x5410);
        }
      } else {
        const float Be = __fmaf_rn(-Ae, m_new, 8.807354922057604f);   // log2(448)
#pragma unroll
        for (int c = 0; c < BR; c += 4) {
          float e0 = x[c], e1 = x[c + 1], e2 = x[c + 2], e3 = x[c + 3];
          float t0 = Be, t1 = Be, t2 = Be, t3 = Be;
          fma2(t0, t1, e0, e1, Ae, Ae);
          fma2(t2, t3, e2, e3, Ae, Ae);
          packed[c / 4] = e4m3x4(exp2f(t0), exp2f(t1), exp2f(t2), exp2f(t3));
        }
      }
      if (j >= 2 && !mbar_wait(&sm.p_free[b], ((j >> 1) + 1) & 1, abort, status, 9)) break;
      uint8_t* prow = sm.p[b] + t * 128;
#pragma unroll
      for (int c = 0; c < BR / 16; ++c) {
        *reinterpret_cast<uint4*>(prow + ((c ^ (t & 7)) << 4)) =
            make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&sm.p_full[b]);
      // Per-tile column factors for the correction warps (thread t = channel t).
      const float vsc = sm.vs[s][t];
      sm.cm[j & 3][0][t] = __fdiv_rn(vsc, 448.0f);
      sm.cm[j & 3][1][t] = __fmul_rn(sm.mu[s][t], vsc);
      sm.alpha[j & 3][t] = alpha;
      mbar_arrive(&sm.kv_empty[s]);
      mbar_arrive(&sm.a_full[j & 3]);
      m = m_new;
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 232;\n" ::: "memory");
    // ------------------------------------------------------------ correction
    const int t = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    float o[kD];
#pragma unroll
    for (int c = 0; c < kD; ++c) o[c] = 0.f;
    float l = 0.f;
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
      const int ri = i & 3;
      ok = mbar_wait(&sm.t_full, i & 1, abort, status, 10) &&
           mbar_wait(&sm.a_full[ri], (i >> 2) & 1, abort, status, 12);
      if (!ok) break;
      tc_fence_after();
      const float alpha = sm.alpha[ri][t];
      const float* cv = sm.cm[ri][0];
      const float* mv = sm.cm[ri][1];
      const bool rescale = !__all_sync(0xffffffffu, alpha == 1.0f);
      float tv[64];
      const float rsum = tmem_ld1(lane_base + kColR);
      tmem_ld32(lane_base + kColT, *reinterpret_cast<float(*)[32]>(&tv[0]));
      tmem_ld32(lane_base + kColT + 32, *reinterpret_cast<float(*)[32]>(&tv[32]));
      tmem_ld_wait();
      const float r = __fdiv_rn(rsum, 448.0f);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h == 1) {
          tmem_ld32(lane_base + kColT + 64, *reinterpret_cast<float(*)[32]>(&tv[0]));
          tmem_ld32(lane_base + kColT + 96, *reinterpret_cast<float(*)[32]>(&tv[32]));
          tmem_ld_wait();
          tc_fence_before();
          mbar_arrive(&sm.t_free);          // T fully read: the next PV may start
        }
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const int col = h * 64 + c;
          if (rescale) mul2(o[col], o[col + 1], alpha, alpha);
          const float2 cc = *reinterpret_cast<const float2*>(cv + col);
          const float2 mm = *reinterpret_cast<const float2*>(mv + col);
          fma2(o[col], o[col + 1], tv[c], tv[c + 1], cc.x, cc.y);
          fma2(o[col], o[col + 1], r, r, mm.x, mm.y);
        }
      }
      l = __fadd_rn(__fmul_rn(l, alpha), r);
    }
    const int row = row0 + t;
    if (ok && !*abort && row < a.N) {
      const int b = g / a.H, h = g % a.H;
      store_row<ODT>(a.out, b * a.osb + h * a.osh + static_cast<int64_t>(row) * a.osn, o, l);
    }
  }
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ---- host side ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D map over (rows, 128 bytes) with a (box_rows x 128) box and 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {128, rows};
  cuuint64_t strides[1] = {128};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BR, bool EC, int ODT>
cudaError_t launch_tc(const AttnParams& p, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  const uint64_t rows = static_cast<uint64_t>(p.B) * p.H * p.n_pad;
  if (!make_map(&mq, p.q8, rows, kBM) || !make_map(&mk, p.k8, rows, BR) || !make_map(&mv, p.v8, rows, BR))
    return cudaErrorInvalidValue;
  TcArgs a{};
  a.q_scale = p.q_scale; a.k_scale = p.k_scale; a.v_scale = p.v_scale; a.mu = p.mu;
  a.H = p.H; a.N = p.N; a.n_pad = p.n_pad; a.nb = p.n_pad / BR;
  a.sm_scale = p.sm_scale;
  a.c120 = static_cast<float>(64.0 + 56.0 + p.beta);
  a.out = p.out; a.osb = p.osb; a.osh = p.osh; a.osn = p.osn;
  const size_t smem = sizeof(TcSmem<BR>) + 1024;
  auto k = attn_tc_kernel<BR, EC, ODT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid((p.n_pad + kBM - 1) / kBM, p.B * p.H);
  k<<<grid, kThreads, smem, st>>>(mq, mk, mv, a);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, k);
    snprintf(g_tc_diag, sizeof(g_tc_diag),
             "regs=%d maxThreadsPerBlock=%d staticSmem=%zu dynSmem=%zu maxDynSmem=%d local=%zu threads=%d",
             fa.numRegs, fa.maxThreadsPerBlock, fa.sharedSizeBytes, smem, fa.maxDynamicSharedSizeBytes,
             fa.localSizeBytes, kThreads);
  }
  return e;
}

template <int BR>
cudaError_t dispatch_tc(const AttnParams& p, cudaStream_t st) {
  const bool ec = (p.flags & VCATTN_EXPCAST) != 0;
  switch (p.out_dtype) {
    case VCATTN_DTYPE_BF16:
      return ec ? launch_tc<BR, true, VCATTN_DTYPE_BF16>(p, st) : launch_tc<BR, false, VCATTN_DTYPE_BF16>(p, st);
    case VCATTN_DTYPE_F16:
      return ec ? launch_tc<BR, true, VCATTN_DTYPE_F16>(p, st) : launch_tc<BR, false, VCATTN_DTYPE_F16>(p, st);
    default:
      return ec ? launch_tc<BR, true, VCATTN_DTYPE_F32>(p, st) : launch_tc<BR, false, VCATTN_DTYPE_F32>(p, st);
  }
}

}  // namespace

cudaError_t launch_attn_tc(const AttnParams& p, cudaStream_t st) {
  if (p.D != 128) return cudaErrorNotSupported;
  return p.block_rows == 128 ? dispatch_tc<128>(p, st) : dispatch_tc<64>(p, st);
}

const char* attn_tc_diag() { return g_tc_diag; }

cudaError_t attn_tc_status(int* code, int* where, int* block, bool reset) {
  tc::DevStatus s{};
  cudaError_t e = cudaMemcpyFromSymbol(&s, g_attn_tc_status, sizeof(s));
  if (e != cudaSuccess) return e;
  *code = s.code;
  *where = s.where;
  *block = s.block;
  if (reset) {
    tc::DevStatus z{};
    e = cudaMemcpyToSymbol(g_attn_tc_status, &z, sizeof(z));
  }
  return e;
}

}  // namespace vcattn
