// Fused dense VC-Attention with NVFP4 QK^T on the 5th-generation tensor cores.
//
// The NVFP4 branch of triton_attn.py:227-239, 263-271 with the tensor-scaled
// NVFP4 of quant.py:172-204: Q and K are E2M1 codes with an E4M3 micro scale
// per 16 elements and one fp32 tensor scale g per (b, h), so
//   s   = dot_blockscaled(q4, k4) * (g_q * g_k * sm_scale)
// (no per-token scale); P, V, ExpCast and the V-Smooth accumulation are those
// of the FP8 kernel:
//   acc = alpha * acc + (P @ V8) * (vs / 448) + (rowsum(P) / 448) * (mu * vs)
//   l   = alpha * l + rowsum(P) / 448 ;  O = acc / l
//
// One CTA = 128 query rows of one (batch, head); 16 warps in 4 warpgroups:
//   warp 0       TMA producer (Q codes + scale atoms once; per tile the K
//                codes and scale atoms, the V codes, vs and mu)
//   warp 1       MMA issuer and TMEM owner: tcgen05.cp of the scale atoms,
//                QK^T with tcgen05.mma.kind::mxf4nvf4.block_scale (K = 64 per
//                instruction), PV and the row-sum MMA in E4M3
//   warps 2-3    per-tile factors vs / 448 and mu * vs
//   warps 4-7    softmax: thread = query row = TMEM lane; row max over S, then
//                P bytes written back to TMEM
//   warps 8-15   correction, two warpgroups of 64 channels each
// TMEM columns: S double buffer [0,128) [128,256) (P over its first 32
// columns), PV tile T [256,384), row sum R [384,400), Q scale factors
// [400,408), K scale factors double buffer [408,416) [416,424).
// Q / K codes use the 64-byte swizzle (rows of 64 bytes), V the 128-byte
// swizzle MN-major in token order.  Every wait is bounded.
#include <cuda.h>
#include <cstdio>
#include <mutex>

#include "kernels.cuh"
#include "tc_common.cuh"
#include "tc_math.cuh"

namespace vcattn {

__device__ tc::DevStatus g_attn_fp4_status;

namespace {

using namespace tc;
char g_fp4_diag[256];

constexpr int kBM = 128;
constexpr int kD = 128;
constexpr int kStages = 4;
constexpr int kRing = 4;        // alpha / column-factor hand-off depth
constexpr int kThreads = 512;   // 16 warps = 4 warpgroups
constexpr uint32_t kColS = 0, kColT = 256, kColR = 384, kColSFA = 400, kColSFB = 408;

template <int BR>
struct TcSmem {
  // q, k and v are contiguous: after the last tile they stage the output.
  alignas(1024) uint8_t q[kBM * 64];
  alignas(1024) uint8_t k[kStages][BR * 64];
  alignas(1024) uint8_t v[kStages][BR * 128];
  alignas(1024) uint8_t ones[16 * 128];
  alignas(128) uint8_t sfa[2 * 512];
  alignas(128) uint8_t sfb[kStages][2 * 512];
  alignas(16) float vs[kStages][kD];
  alignas(16) float mu[kStages][kD];
  alignas(16) float cm[kRing][2][kD];   // vs / 448 and mu * vs per channel
  alignas(16) float alpha[kRing][kBM];  // per query row
  alignas(8) uint64_t q_full;
  alignas(8) uint64_t kv_full[kStages];
  alignas(8) uint64_t kv_empty[kStages];
  alignas(8) uint64_t s_full[2];
  alignas(8) uint64_t p_full[2];
  alignas(8) uint64_t t_full;
  alignas(8) uint64_t t_free;
  alignas(8) uint64_t a_full[kRing];
  alignas(8) uint64_t a_free[kRing];
  alignas(8) uint64_t cm_full[kRing];
  alignas(8) uint64_t cm_free[kRing];
  alignas(8) uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct TcArgs {
  const uint8_t* q_sf;   // (G, NP/128, 2, 512) scale-factor atoms
  const uint8_t* k_sf;
  const float* q_g;      // (G) tensor scales
  const float* k_g;
  const float* v_scale;
  const float* mu;
  int H, N, n_pad, nb;
  float sm_scale;
  float c120;   // 64 + 56 + beta (ExpCast)
  void* out;
  int64_t osb, osh, osn;
};

template <int BR, bool EXPCAST, int ODT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  constexpr int NCH = BR / 32;   // 32-column chunks of S
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  TcSmem<BR>& sm = *reinterpret_cast<TcSmem<BR>*>(smem_raw + pad);
  DevStatus* status = &g_attn_fp4_status;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.y;
  const int row0 = blockIdx.x * kBM;
  const int nb = a.nb;

  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1 + 2);   // PV commit + column-factor warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.p_full[b], 4);
    }
    mbar_init(&sm.t_full, 1);
    mbar_init(&sm.t_free, 8);
    for (int r = 0; r < kRing; ++r) {
      mbar_init(&sm.a_full[r], 4);
      mbar_init(&sm.a_free[r], 8);
      mbar_init(&sm.cm_full[r], 2);
      mbar_init(&sm.cm_free[r], 8);
    }
    mbar_init(&sm.drain, 1);
    fence_mbar_init();
  }
  // All-ones block (B operand of the row-sum MMA): every R column = rowsum(P).
  for (int i = tid; i < 16 * 128; i += kThreads) sm.ones[i] = 0x38;
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
  // Register budget per warpgroup (launched at 128 x 512 = 65536):
  // 128 x (48 producer/MMA/factors + 112 softmax + 2 x 168 correction) = 63488.
  asm volatile("setmaxnreg.dec.sync.aligned.u32 48;\n" ::: "memory");
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int issued = 0;
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      const int tiles = a.n_pad / 128;
      mbar_expect_tx(&sm.q_full, kBM * 64 + 1024);
      tma_load_2d(sm.q, &tm_q, 0, g * a.n_pad + row0, &sm.q_full);
      bulk_load(sm.sfa, a.q_sf + (static_cast<int64_t>(g) * tiles + blockIdx.x) * 1024, 1024, &sm.q_full);
      const uint32_t tile_bytes = BR * 64u + BR * 128u + 1024u + 2u * kD * 4u;
      for (int j = 0; j < nb; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&sm.kv_empty[s], ((j / kStages) + 1) & 1, abort, status, 1)) break;
        mbar_expect_tx(&sm.kv_full[s], tile_bytes);
        const int krow = g * a.n_pad + j * BR;
        tma_load_2d(sm.k[s], &tm_k, 0, krow, &sm.kv_full[s]);
        tma_load_2d(sm.v[s], &tm_v, 0, krow, &sm.kv_full[s]);
        bulk_load(sm.sfb[s], a.k_sf + (static_cast<int64_t>(g) * tiles + j) * 1024, 1024, &sm.kv_full[s]);
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
    // The whole warp runs the loop; the elected lane issues.
    {
      const uint32_t leader = elect_one();
      const uint32_t id_qk = idesc_nvfp4(kBM, BR);
      const uint32_t id_pv = idesc_e4m3(kBM, kD, true);
      const uint32_t id_r = idesc_e4m3(kBM, 16, false);
      const uint32_t q_addr = smem_u32(sm.q);
      const uint32_t ones_addr = smem_u32(sm.ones);
      bool ok = mbar_wait(&sm.q_full, 0, abort, status, 2);
      if (ok) {
        tc_fence_after();
        for (int at = 0; at < 2; ++at)
          tmem_cp_sf_if(tbase + kColSFA + 4 * at, desc_sf(smem_u32(sm.sfa + 512 * at)), leader);
      }
      for (int j = 0; ok && j <= nb; ++j) {
        if (j < nb) {
          // S_b was last read as P by PV_{j-2}, issued earlier by this thread:
          // tcgen05.mma from one thread run in order, so no extra wait.
          const int s = j % kStages, b = j & 1;
          ok = mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 3);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm.k[s]);
          // K scale atoms of tile j into SFB_b; SFB_b was last read by QK_{j-2},
          // complete before PV_{j-2} was issued (p_full(j-2) follows s_full(j-2)).
          const uint32_t sfb = tbase + kColSFB + 8 * b;
          for (int at = 0; at < 2; ++at) tmem_cp_sf_if(sfb + 4 * at, desc_sf(smem_u32(sm.sfb[s] + 512 * at)), leader);
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
            mma_nvfp4_if(tbase + kColS + b * 128, desc_kmajor64(q_addr + kk * 32), desc_kmajor64(k_addr + kk * 32),
                         id_qk, tbase + kColSFA + 4 * kk, sfb + 4 * kk, kk > 0, leader);
          tc_commit_if(&sm.s_full[b], leader);
        }
        if (j >= 1) {
          const int i = j - 1, bi = i & 1, si = i % kStages;
          ok = i >= 1 ? mbar_wait2(&sm.p_full[bi], (i >> 1) & 1, &sm.t_free, (i - 1) & 1, abort, status, 5)
                      : mbar_wait(&sm.p_full[bi], (i >> 1) & 1, abort, status, 5);
          if (!ok) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sm.v[si]);
          const uint32_t p_t = tbase + kColS + bi * 128;   // keys [32kk, 32kk+32) at columns 8kk..8kk+7
#pragma unroll
          for (int kk = 0; kk < BR / 32; ++kk)
            mma_f8_ts_if(tbase + kColT, p_t + 8 * kk, desc_mnmajor(v_addr + kk * 32 * 128), id_pv, kk > 0, leader);
#pragma unroll
          for (int kk = 0; kk < BR / 32; ++kk)
            mma_f8_ts_if(tbase + kColR, p_t + 8 * kk, desc_kmajor(ones_addr + kk * 32), id_r, kk > 0, leader);
          tc_commit_if(&sm.t_full, leader);
          tc_commit_if(&sm.kv_empty[si], leader);
        }
      }
      // Every MMA issued must finish before TMEM is released.
      tc_commit_if(&sm.drain, leader);
      const long long t0 = clock64();
      while (!mbar_try_wait(&sm.drain, 0) && clock64() - t0 < kWaitCycles) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ column factors
    const int c2 = tid - 64;   // 0..63
    for (int j = 0; j < nb; ++j) {
      const int s = j % kStages, ring = j % kRing;
      if (!mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 13)) break;
      if (j >= kRing && !mbar_wait(&sm.cm_free[ring], ((j / kRing) + 1) & 1, abort, status, 14)) break;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = c2 + 64 * h;
        const float vsc = sm.vs[s][c];
        sm.cm[ring][0][c] = __fdiv_rn(vsc, 448.0f);
        sm.cm[ring][1][c] = __fmul_rn(sm.mu[s][c], vsc);
      }
      warp_arrive(&sm.cm_full[ring], lane);
      warp_arrive(&sm.kv_empty[s], lane);
    }
  }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 112;\n" ::: "memory");
    // ------------------------------------------------------------ softmax
    const int t = (warp & 3) * 32 + lane;          // query row within the tile = TMEM lane
    const uint32_t lane_base = tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int row = row0 + t;
    const int aidx = (warp & 3) * 32 + lane;
    (void)row;
    // one score scale for the whole head: g_q * g_k * sm_scale
    const float qsm = __fmul_rn(__fmul_rn(a.q_g[g], a.k_g[g]), a.sm_scale);
    // ExpCast: c = A * (x - m) + c120 with A = 8 log2e qs sm; evaluated as
    // fma.sat(x, A/128, B/128) so the clamp at 0 is free and the /128 scale
    // makes a + 98304 round the code to an integer in the low bits.
    const float A = __fmul_rn(8.0f * kLog2e, qsm);
    const float As = A * (1.0f / 128.0f);
    const float Ae = __fmul_rn(qsm, kLog2e);       // exp path: p = exp2(Ae (x - m)) * 448
    float m = -INFINITY;
    for (int j = 0; j < nb; ++j) {
      const int b = j & 1, ring = j % kRing;
      if (!mbar_wait(&sm.s_full[b], (j >> 1) & 1, abort, status, 7)) break;
      tc_fence_after();
      const uint32_t sb = lane_base + kColS + b * 128;
      const int valid = a.N - j * BR;                 // key columns >= valid are padding
      // pass 1: row max of S (already in score units up to the head scale)
      float xa[32], xb[32];
      float m0 = m, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
      tmem_ld32(sb, xa);
      tmem_ld_wait_regs(xa);
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        float (&cur)[32] = (ch & 1) ? xb : xa;
        float (&nxt)[32] = (ch & 1) ? xa : xb;
        if (ch + 1 < NCH) tmem_ld32(sb + 32 * (ch + 1), nxt);
        if (valid < 32 * (ch + 1)) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (32 * ch + c >= valid) cur[c] = -1.0e30f;
        }
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          m0 = fmax3(m0, cur[c], cur[c + 1]);
          m1 = fmax3(m1, cur[c + 2], cur[c + 3]);
          m2 = fmax3(m2, cur[c + 4], cur[c + 5]);
          m3 = fmax3(m3, cur[c + 6], cur[c + 7]);
        }
        if (ch + 1 < NCH) tmem_ld_wait_regs(nxt);
      }
      const float m_new = fmax3(m0, m1, fmaxf(m2, m3));
      // pass 2: P bytes; chunk ch lands in columns [8ch, 8ch+8), which pass 2
      // has already read (chunk 0's scores)
      tmem_ld32(sb, xa);
      tmem_ld_wait_regs(xa);
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        float (&cur)[32] = (ch & 1) ? xb : xa;
        float (&nxt)[32] = (ch & 1) ? xa : xb;
        if (ch + 1 < NCH) tmem_ld32(sb + 32 * (ch + 1), nxt);
        if (valid < 32 * (ch + 1)) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (32 * ch + c >= valid) cur[c] = -1.0e30f;
        }
        uint32_t packed[8];
        if constexpr (EXPCAST) {
          const float Bs = __fmaf_rn(-As, m_new, a.c120 * (1.0f / 128.0f));
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            float c0 = fma_sat(cur[c], As, Bs), c1 = fma_sat(cur[c + 1], As, Bs);
            float c2 = fma_sat(cur[c + 2], As, Bs), c3 = fma_sat(cur[c + 3], As, Bs);
            add2(c0, c1, 98304.0f, 98304.0f);
            add2(c2, c3, 98304.0f, 98304.0f);
            const uint32_t lo = __byte_perm(__float_as_uint(c0), __float_as_uint(c1), 0x0040);
            const uint32_t hi = __byte_perm(__float_as_uint(c2), __float_as_uint(c3), 0x0040);
            packed[c / 4] = __byte_perm(lo, hi, 0x5410);
          }
        } else {
          const float Be = __fmaf_rn(-Ae, m_new, 8.807354922057604f);   // log2(448)
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            float t0 = Be, t1 = Be, t2 = Be, t3 = Be;
            fma2(t0, t1, cur[c], cur[c + 1], Ae, Ae);
            fma2(t2, t3, cur[c + 2], cur[c + 3], Ae, Ae);
            packed[c / 4] = e4m3x4(exp2f(t0), exp2f(t1), exp2f(t2), exp2f(t3));
          }
        }
        tmem_st8(sb + 8 * ch, packed);
        if (ch + 1 < NCH) tmem_ld_wait_regs(nxt);
      }
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(&sm.p_full[b], lane);
      const float alpha = (m == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m, m_new), Ae));
      if (j >= kRing && !mbar_wait(&sm.a_free[ring], ((j / kRing) + 1) & 1, abort, status, 10)) break;
      sm.alpha[ring][aidx] = alpha;
      warp_arrive(&sm.a_full[ring], lane);
      m = m_new;
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 168;\n" ::: "memory");
    // ------------------------------------------------------------ correction
    // Warpgroup cg owns channels [64 cg, 64 cg + 64); thread = query row
    // r = 32 (w%4) + lane (TMEM lane r), T read with the 32x32b shape.
    const int cg = (warp >> 2) - 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lb = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    float o[64];   // channels 64 cg + c
#pragma unroll
    for (int c = 0; c < 64; ++c) o[c] = 0.f;
    float l = 0.f;
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
      const int ring = i % kRing;
      ok = mbar_wait(&sm.t_full, i & 1, abort, status, 11) &&
           mbar_wait(&sm.a_full[ring], (i / kRing) & 1, abort, status, 12) &&
           mbar_wait(&sm.cm_full[ring], (i / kRing) & 1, abort, status, 15);
      if (!ok) break;
      tc_fence_after();
      float ta[32], tb[32];
      float rs = tmem_ld1(lb + kColR);
      tmem_ld32(lb + kColT + 64 * cg, ta);
      tmem_ld32(lb + kColT + 64 * cg + 32, tb);
      const float al = sm.alpha[ring][r];
      tmem_ld_wait();
      asm volatile("" : "+f"(rs));
      reg_fence(ta);
      reg_fence(tb);
      tc_fence_before();
      warp_arrive(&sm.t_free, lane);     // T and R read: the next PV may start
      warp_arrive(&sm.a_free[ring], lane);
      const bool rescale = !__all_sync(0xffffffffu, al == 1.0f);
      const float rr = rs * (1.0f / 448.0f);
      const float4* f4 = reinterpret_cast<const float4*>(sm.cm[ring][0] + 64 * cg);
      const float4* g4 = reinterpret_cast<const float4*>(sm.cm[ring][1] + 64 * cg);
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const float* src = (q < 8) ? ta + 4 * q : tb + 4 * (q - 8);
        const float4 fv = f4[q];
        const float4 gv = g4[q];
        float* oc = o + 4 * q;
        if (rescale) {
          mul2(oc[0], oc[1], al, al);
          mul2(oc[2], oc[3], al, al);
        }
        fma2(oc[0], oc[1], src[0], src[1], fv.x, fv.y);
        fma2(oc[2], oc[3], src[2], src[3], fv.z, fv.w);
        fma2(oc[0], oc[1], rr, rr, gv.x, gv.y);
        fma2(oc[2], oc[3], rr, rr, gv.z, gv.w);
      }
      warp_arrive(&sm.cm_free[ring], lane);
      l = __fadd_rn(__fmul_rn(l, al), rr);
    }
    if (ok && !*abort) {
      // Stage this warp's 32 rows x 64 channels (padded stride), then write
      // them out as whole 16-byte row chunks.
      constexpr int ES = (ODT == VCATTN_DTYPE_F32) ? 4 : 2;
      constexpr int RS = 64 * ES + 16;
      static_assert(8 * 32 * RS <= static_cast<int>(sizeof(TcSmem<BR>::q) + sizeof(TcSmem<BR>::k) +
                                                    sizeof(TcSmem<BR>::v)),
                    "output staging must fit in the operand buffers");
      uint8_t* stage = sm.q + (cg * 4 + wq) * 32 * RS;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 16 / ES) {
        uint4 w;
#pragma unroll
        for (int e = 0; e < 16 / ES; e += 2)
          stage2<ODT>(reinterpret_cast<uint8_t*>(&w) + e * ES, __fdiv_rn(o[c0 + e], l), __fdiv_rn(o[c0 + e + 1], l));
        *reinterpret_cast<uint4*>(stage + lane * RS + c0 * ES) = w;
      }
      __syncwarp();
      constexpr int CPR = 64 * ES / 16;   // 16-byte chunks per staged row
      const int bq = g / a.H, hq = g % a.H;
      uint8_t* out = static_cast<uint8_t*>(a.out) + (bq * a.osb + hq * a.osh + 64 * cg) * ES;
      for (int idx = lane; idx < 32 * CPR; idx += 32) {
        const int rloc = idx / CPR, ch = idx % CPR;
        const int orow = row0 + wq * 32 + rloc;
        if (orow < a.N)
          *reinterpret_cast<uint4*>(out + static_cast<int64_t>(orow) * a.osn * ES + ch * 16) =
              *reinterpret_cast<const uint4*>(stage + rloc * RS + ch * 16);
      }
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

// 2-D map over (rows, 64 bytes) with a (box_rows x 64) box and 64-byte swizzle.
bool make_map64(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {64, rows};
  cuuint64_t strides[1] = {64};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BR, bool EC, int ODT>
cudaError_t launch_tc(const AttnParams& p, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  const uint64_t rows = static_cast<uint64_t>(p.B) * p.H * p.n_pad;
  if (!make_map64(&mq, p.q4, rows, kBM) || !make_map64(&mk, p.k4, rows, BR) || !make_map(&mv, p.v8, rows, BR))
    return cudaErrorInvalidValue;
  TcArgs a{};
  a.q_sf = p.q4_sf; a.k_sf = p.k4_sf; a.q_g = p.q4_g; a.k_g = p.k4_g; a.v_scale = p.v_scale; a.mu = p.mu;
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
    snprintf(g_fp4_diag, sizeof(g_fp4_diag),
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

cudaError_t launch_attn_nvfp4(const AttnParams& p, cudaStream_t st) {
  if (p.D != 128 || p.block_rows != 128 || p.n_pad % 128 != 0) return cudaErrorNotSupported;
  return dispatch_tc<128>(p, st);
}

const char* attn_nvfp4_diag() { return g_fp4_diag; }

cudaError_t attn_nvfp4_status(int* code, int* where, int* block, bool reset) {
  tc::DevStatus s{};
  cudaError_t e = cudaMemcpyFromSymbol(&s, g_attn_fp4_status, sizeof(s));
  if (e != cudaSuccess) return e;
  *code = s.code;
  *where = s.where;
  *block = s.block;
  if (reset) {
    tc::DevStatus z{};
    e = cudaMemcpyToSymbol(g_attn_fp4_status, &z, sizeof(z));
  }
  return e;
}

}  // namespace vcattn
