// Fused dense FP8 VC-Attention, two 128-row query tiles per CTA, with the
// output accumulated by the tensor cores in tensor memory.
//
// Semantics of triton_attn.py:203-322 (the value block BR = 128 is the KV
// tile), arithmetic of attn_tc.cu, except where O lives.  attn_tc.cu keeps O
// in registers because each KV tile's P.V result carries its own
// per-(block, channel) scale vs_j.  Here the P.V MMA adds into O itself, so O
// is held in units of the current block's scale u_j = max(vs_j, floor_j):
// before PV_j the correction warps rescale O by alpha_j * u_{j-1} / u_j per
// (row, channel) and add block j-1's mean term R_{j-1} * mu_{j-1} (in units
// of u_{j-1}); the epilogue multiplies by u_last / 448 and divides by l.
// floor_j = 2^-80 * max over blocks i <= j of |mu_i vs_i| + 448 vs_i keeps O
// finite when a block's scale sits at the amax clamp (a constant channel):
// O is a convex combination of V rows, so |O_hat| < l * 448 * 2^80.
// oracle.attention_codes_units(running_floor=True, floor_exp=-80) restates
// this order of operations.
//
// With O out of the registers, one CTA runs two query tiles A (rows
// row0..row0+127) and B (the next 128): while one tile's softmax and
// correction run, the tensor cores work on the other's QK^T and P.V.
//
// 16 warps in 4 warpgroups (launched at 128 registers; setmaxnreg 40 / 176 /
// 176 / 120):
//   warp 0       TMA producer (Q_A, Q_B once; K, V codes + ks, vs, mu per tile)
//   warp 1       MMA issuer and TMEM owner
//   warps 2-3    per-tile factors u_{j-1}/u_j and the mean in units of u
//   warps 4-7    softmax of tile A: thread = query row = TMEM lane; also
//                the row sum R_j (read after P.V) and l
//   warps 8-11   softmax of tile B
//   warps 12-15  correction (O rescale in TMEM) of A and B, then the epilogue
// TMEM columns: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512).
// P_X (E4M3 bytes, keys 4c..4c+3 in column c) goes over the first 32 columns
// of S_X; R_X (an N=16 MMA of P_X against an all-ones block) over columns
// 32..47 of S_X, read by the softmax warps before QK_X(j+1) overwrites S_X.
// MMA issue order per KV tile j: PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1).
// Every wait is bounded.
#include <cuda.h>
#include <cstdio>

#include "kernels.cuh"
#include "tc_common.cuh"
#include "tc_math.cuh"

namespace vcattn {

__device__ tc::DevStatus g_attn_tc2_status;

namespace {

using namespace tc;
char g_tc2_diag[256];

constexpr int kBR = 128;         // KV tile = value block
constexpr int kBM = 128;         // rows per query tile
constexpr int kD = 128;
constexpr int kStages = 3;
constexpr int kRing = 4;
constexpr int kThreads = 512;
constexpr uint32_t kColO = 256;
constexpr float kFloorScale = 8.2718061255302767e-25f;   // 2^-80

struct Tc2Smem {
  alignas(1024) uint8_t q[2][kBM * 128];
  alignas(1024) uint8_t k[kStages][kBR * 128];
  alignas(1024) uint8_t v[kStages][kBR * 128];
  alignas(1024) uint8_t ones[16 * 128];
  alignas(16) float ks[kStages][kBR];
  alignas(16) float vs[kStages][kD];
  alignas(16) float mu[kStages][kD];
  alignas(16) float fac[kRing][2][kD];     // u_{j-1}/u_j and mu_{j-1} in units of u_{j-1}
  alignas(16) float fin[2][kD];            // u_last / 448 and mu_last in units of u_last
  alignas(16) float alpha[2][kRing][kBM];  // per query tile and row
  alignas(16) float rprev[2][kRing][kBM];  // R_{j-1} per row
  alignas(16) float lfin[2][kBM];          // l and R_last per row at the end
  alignas(16) float rfin[2][kBM];
  alignas(8) uint64_t q_full;
  alignas(8) uint64_t kv_full[kStages];
  alignas(8) uint64_t kv_empty[kStages];
  alignas(8) uint64_t s_full[2];
  alignas(8) uint64_t p_full[2];
  alignas(8) uint64_t pv_done[2];
  alignas(8) uint64_t r_read[2];
  alignas(8) uint64_t o_ready[2];
  alignas(8) uint64_t a_full[2][kRing];
  alignas(8) uint64_t a_free[2][kRing];
  alignas(8) uint64_t f_full[kRing];
  alignas(8) uint64_t f_free[kRing];
  alignas(8) uint64_t fin_f;
  alignas(8) uint64_t fin_s[2];
  alignas(8) uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct Tc2Args {
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

// ECM: 0 = E4M3 of exp2, 1 = one-FMA ExpCast, 2 = ExpCast in the reference's
// operation order on s = (S * (qs * ks)) * sm_scale.
template <int ECM, int ODT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Tc2Args a) {
  constexpr int NCH = kBR / 32;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Tc2Smem& sm = *reinterpret_cast<Tc2Smem*>(smem_raw + pad);
  DevStatus* status = &g_attn_tc2_status;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.y;
  const int row0 = blockIdx.x * (2 * kBM);
  const int nb = a.nb;

  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1 + 2);   // MMA commit after PV_B + factor warps
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&sm.s_full[x], 1);
      mbar_init(&sm.p_full[x], 4);
      mbar_init(&sm.pv_done[x], 1);
      mbar_init(&sm.r_read[x], 4);
      mbar_init(&sm.o_ready[x], 4);
      mbar_init(&sm.fin_s[x], 4);
      for (int r = 0; r < kRing; ++r) {
        mbar_init(&sm.a_full[x][r], 4);
        mbar_init(&sm.a_free[x][r], 4);
      }
    }
    for (int r = 0; r < kRing; ++r) {
      mbar_init(&sm.f_full[r], 2);
      mbar_init(&sm.f_free[r], 4);
    }
    mbar_init(&sm.fin_f, 2);
    mbar_init(&sm.drain, 1);
    fence_mbar_init();
  }
  for (int i = tid; i < 16 * 128; i += kThreads) sm.ones[i] = 0x38;   // E4M3 1.0
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
    // Register budget (launched at 128 x 512 = 65536):
    // 128 x (40 producer/MMA/factors + 176 + 176 softmax + 120 correction) = 65536.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 40;\n" ::: "memory");
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      int issued = 0;
      if (lane == 0) {
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        mbar_expect_tx(&sm.q_full, 2 * kBM * 128);
        tma_load_2d(sm.q[0], &tm_q, 0, g * a.n_pad + row0, &sm.q_full);
        tma_load_2d(sm.q[1], &tm_q, 0, g * a.n_pad + row0 + kBM, &sm.q_full);
        const uint32_t tile_bytes = 2u * kBR * 128u + kBR * 4u + 2u * kD * 4u;
        for (int j = 0; j < nb; ++j) {
          const int s = j % kStages;
          if (j >= kStages && !mbar_wait(&sm.kv_empty[s], ((j / kStages) + 1) & 1, abort, status, 1)) break;
          mbar_expect_tx(&sm.kv_full[s], tile_bytes);
          const int krow = g * a.n_pad + j * kBR;
          tma_load_2d(sm.k[s], &tm_k, 0, krow, &sm.kv_full[s]);
          tma_load_2d(sm.v[s], &tm_v, 0, krow, &sm.kv_full[s]);
          bulk_load(sm.ks[s], a.k_scale + static_cast<int64_t>(krow), kBR * 4, &sm.kv_full[s]);
          const int64_t vo = (static_cast<int64_t>(g) * nb + j) * kD;
          bulk_load(sm.vs[s], a.v_scale + vo, kD * 4, &sm.kv_full[s]);
          bulk_load(sm.mu[s], a.mu + vo, kD * 4, &sm.kv_full[s]);
          issued = j + 1;
        }
        if (*abort) {   // let the copies already issued land before the CTA exits
          for (int j = max(0, issued - kStages); j < issued; ++j) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&sm.kv_full[j % kStages], (j / kStages) & 1) && clock64() - t0 < kWaitCycles / 4) {
            }
          }
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      // ---------------------------------------------------------- MMA issuer
      const uint32_t leader = elect_one();
      const uint32_t id_qk = idesc_e4m3(kBM, kBR, false);
      const uint32_t id_pv = idesc_e4m3(kBM, kD, true);
      const uint32_t id_r = idesc_e4m3(kBM, 16, false);
      const uint32_t ones_addr = smem_u32(sm.ones);
      auto issue_qk = [&](int x, int j) {
        const uint32_t q_addr = smem_u32(sm.q[x]);
        const uint32_t k_addr = smem_u32(sm.k[j % kStages]);
#pragma unroll
        for (int kk = 0; kk < kD / 32; ++kk)
          mma_f8_if(tbase + x * 128, desc_kmajor(q_addr + kk * 32), desc_kmajor(k_addr + kk * 32), id_qk, kk > 0,
                    leader);
        tc_commit_if(&sm.s_full[x], leader);
      };
      auto issue_pv = [&](int x, int j) {
        const uint32_t v_addr = smem_u32(sm.v[j % kStages]);
        const uint32_t p_t = tbase + x * 128;   // P positions [32kk, 32kk+32) at columns 8kk..8kk+7
#pragma unroll
        for (int kk = 0; kk < kBR / 32; ++kk)
          mma_f8_ts_if(tbase + kColO + x * 128, p_t + 8 * kk, desc_mnmajor(v_addr + kk * 32 * 128), id_pv,
                       (j > 0 || kk > 0) ? 1u : 0u, leader);
#pragma unroll
        for (int kk = 0; kk < kBR / 32; ++kk)
          mma_f8_ts_if(tbase + x * 128 + 32, p_t + 8 * kk, desc_kmajor(ones_addr + kk * 32), id_r, kk > 0, leader);
        tc_commit_if(&sm.pv_done[x], leader);
      };
      bool ok = mbar_wait(&sm.q_full, 0, abort, status, 2) && mbar_wait(&sm.kv_full[0], 0, abort, status, 3);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        issue_qk(1, 0);
      }
      for (int j = 0; ok && j < nb; ++j) {
        const int sn = (j + 1) % kStages;
        for (int x = 0; x < 2 && ok; ++x) {
          // PV_X(j): P_X(j) stored, O_X rescaled for block j (from j = 1)
          ok = j >= 1 ? mbar_wait2(&sm.p_full[x], j & 1, &sm.o_ready[x], (j - 1) & 1, abort, status, 4 + x)
                      : mbar_wait(&sm.p_full[x], 0, abort, status, 4 + x);
          if (!ok) break;
          tc_fence_after();
          issue_pv(x, j);
          if (x == 1) tc_commit_if(&sm.kv_empty[j % kStages], leader);
          // QK_X(j+1): K_{j+1} landed, R_X(j) read out of S_X
          if (j + 1 < nb) {
            ok = mbar_wait2(&sm.kv_full[sn], ((j + 1) / kStages) & 1, &sm.r_read[x], j & 1, abort, status, 6 + x);
            if (!ok) break;
            tc_fence_after();
            issue_qk(x, j + 1);
          }
        }
      }
      tc_commit_if(&sm.drain, leader);   // every MMA issued completes before TMEM is released
      const long long t0 = clock64();
      while (!mbar_try_wait(&sm.drain, 0) && clock64() - t0 < kWaitCycles) {
      }
      __syncwarp();
    } else {
      // ---------------------------------------------------------- factors
      // Per channel c: u_j = max(vs_j, 2^-80 * running max of |mu vs| + 448 vs);
      // slot (j-1) % kRing holds u_{j-1} / u_j and mu_{j-1} in units of u_{j-1}.
      const int c2 = tid - 64;   // channels c2 and c2 + 64
      float mrun[2] = {0.f, 0.f}, uprev[2] = {0.f, 0.f}, muprev[2] = {0.f, 0.f};
      bool ok = true;
      for (int j = 0; j < nb; ++j) {
        const int s = j % kStages;
        ok = mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 13);
        if (!ok) break;
        const int slot = (j - 1) % kRing;
        if (j >= 1 + kRing && !(ok = mbar_wait(&sm.f_free[slot], (((j - 1) / kRing) + 1) & 1, abort, status, 14)))
          break;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = c2 + 64 * h;
          const float vsc = sm.vs[s][c], muc = sm.mu[s][c];
          const float bound = __fadd_rn(fabsf(__fmul_rn(muc, vsc)), __fmul_rn(448.0f, vsc));
          mrun[h] = fmaxf(mrun[h], bound);
          const float u = fmaxf(vsc, __fmul_rn(mrun[h], kFloorScale));
          if (j >= 1) {
            sm.fac[slot][0][c] = __fdiv_rn(uprev[h], u);
            sm.fac[slot][1][c] = muprev[h];
          }
          uprev[h] = u;
          muprev[h] = __fmul_rn(muc, __fdiv_rn(vsc, u));
        }
        if (j >= 1) warp_arrive(&sm.f_full[slot], lane);
        warp_arrive(&sm.kv_empty[s], lane);
      }
      if (ok) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          sm.fin[0][c2 + 64 * h] = __fdiv_rn(uprev[h], 448.0f);
          sm.fin[1][c2 + 64 * h] = muprev[h];
        }
        warp_arrive(&sm.fin_f, lane);
      }
    }
  } else if (warp < 12) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 176;\n" ::: "memory");
    // ------------------------------------------------------------ softmax
    const int x = (warp - 4) >> 2;                 // query tile
    const int t = (warp & 3) * 32 + lane;          // row = TMEM lane
    const uint32_t lane_base = tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t sb = lane_base + x * 128;
    const int qrow = row0 + x * kBM + t;
    const float qs = (qrow < a.n_pad) ? a.q_scale[static_cast<int64_t>(g) * a.n_pad + qrow] : 0.f;
    const float qsm = __fmul_rn(qs, a.sm_scale);
    const float As = __fmul_rn(8.0f * kLog2e, qsm) * (1.0f / 128.0f);
    const float Ae = (ECM == 2) ? kLog2e : __fmul_rn(qsm, kLog2e);
    float m = -INFINITY, l = 0.f, rprev = 0.f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      const int s = j % kStages;
      ok = mbar_wait2(&sm.s_full[x], j & 1, &sm.kv_full[s], (j / kStages) & 1, abort, status, 7 + 2 * x);
      if (!ok) break;
      tc_fence_after();
      float xs[kBR];
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) tmem_ld32(sb + 32 * ch, *reinterpret_cast<float(*)[32]>(xs + 32 * ch));
      tmem_ld_wait();
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) reg_fence(*reinterpret_cast<float(*)[32]>(xs + 32 * ch));
      const float4* k4 = reinterpret_cast<const float4*>(sm.ks[s]);
      if constexpr (ECM == 2) {
#pragma unroll
        for (int q = 0; q < kBR / 4; ++q) {
          const float4 kv = k4[q];
          xs[4 * q] = __fmul_rn(__fmul_rn(xs[4 * q], __fmul_rn(qs, kv.x)), a.sm_scale);
          xs[4 * q + 1] = __fmul_rn(__fmul_rn(xs[4 * q + 1], __fmul_rn(qs, kv.y)), a.sm_scale);
          xs[4 * q + 2] = __fmul_rn(__fmul_rn(xs[4 * q + 2], __fmul_rn(qs, kv.z)), a.sm_scale);
          xs[4 * q + 3] = __fmul_rn(__fmul_rn(xs[4 * q + 3], __fmul_rn(qs, kv.w)), a.sm_scale);
        }
      } else {
#pragma unroll
        for (int q = 0; q < kBR / 4; ++q) {
          const float4 kv = k4[q];
          mul2(xs[4 * q], xs[4 * q + 1], kv.x, kv.y);
          mul2(xs[4 * q + 2], xs[4 * q + 3], kv.z, kv.w);
        }
      }
      const int valid = a.N - j * kBR;   // keys >= valid are padding
      if (valid < kBR) {
#pragma unroll
        for (int c = 0; c < kBR; ++c)
          if (c >= valid) xs[c] = -1.0e30f;
      }
      float m0 = m, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBR; c += 8) {
        m0 = fmax3(m0, xs[c], xs[c + 1]);
        m1 = fmax3(m1, xs[c + 2], xs[c + 3]);
        m2 = fmax3(m2, xs[c + 4], xs[c + 5]);
        m3 = fmax3(m3, xs[c + 6], xs[c + 7]);
      }
      const float mn = fmax3(m0, m1, fmaxf(m2, m3));
      const float al = (m == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m, mn), Ae));
      if (j >= 1) {
        // alpha_j and R_{j-1} for the correction of O_X before PV_X(j)
        const int slot = (j - 1) % kRing;
        if (j >= 1 + kRing &&
            !(ok = mbar_wait(&sm.a_free[x][slot], (((j - 1) / kRing) + 1) & 1, abort, status, 11 + 20 * x)))
          break;
        sm.alpha[x][slot][t] = al;
        sm.rprev[x][slot][t] = rprev;
        warp_arrive(&sm.a_full[x][slot], lane);
      }
      if constexpr (ECM == 2) {
        const float c0 = a.c120 - 64.0f;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          uint32_t packed[8];
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            const float* xc = xs + 32 * ch + 4 * w;
            uint32_t word = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float u = __fadd_rn(__fmul_rn(__fsub_rn(xc[e], mn), kLog2e), 8.0f);
              const float c = fminf(fmaxf(rintf(__fmaf_rn(u, 8.0f, c0)), 0.0f), 120.0f);
              word |= static_cast<uint32_t>(c) << (8 * e);
            }
            packed[w] = word;
          }
          tmem_st8(sb + 8 * ch, packed);
        }
      } else if constexpr (ECM == 1) {
        const float Bs = __fmaf_rn(-As, mn, a.c120 * (1.0f / 128.0f));
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          uint32_t packed[8];
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            const float* xc = xs + 32 * ch + 4 * w;
            packed[w] = expcast4(xc[0], xc[1], xc[2], xc[3], As, Bs);
          }
          tmem_st8(sb + 8 * ch, packed);
        }
      } else {
        const float Be = __fmaf_rn(-Ae, mn, 8.807354922057604f);   // log2(448)
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          uint32_t packed[8];
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            const float* xc = xs + 32 * ch + 4 * w;
            packed[w] = exp4(xc[0], xc[1], xc[2], xc[3], Ae, Be);
          }
          tmem_st8(sb + 8 * ch, packed);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(&sm.p_full[x], lane);
      // R_j (row sum of the P bytes, from the N=16 MMA after P.V) out of S_X
      // before QK_X(j+1) overwrites it
      ok = mbar_wait(&sm.pv_done[x], j & 1, abort, status, 12 + 20 * x);
      if (!ok) break;
      tc_fence_after();
      float r = tmem_ld1(sb + 32);
      tmem_ld_wait();
      asm volatile("" : "+f"(r));
      tc_fence_before();
      warp_arrive(&sm.r_read[x], lane);
      l = __fadd_rn(__fmul_rn(l, al), r * (1.0f / 448.0f));
      rprev = r;
      m = mn;
    }
    if (ok) {
      sm.lfin[x][t] = l;
      sm.rfin[x][t] = rprev;
      warp_arrive(&sm.fin_s[x], lane);
    }
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 120;\n" ::: "memory");
    // ------------------------------------------------------------ correction
    // O_X <- (O_X + R_{j-1} mu_{j-1}) * alpha_j * u_{j-1} / u_j, per row
    // (TMEM lane r) and channel, in place in tensor memory.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lb = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    bool ok = true;
    for (int j = 1; j < nb && ok; ++j) {
      const int slot = (j - 1) % kRing;
      ok = mbar_wait(&sm.f_full[slot], ((j - 1) / kRing) & 1, abort, status, 15);
      if (!ok) break;
      const float4* f4 = reinterpret_cast<const float4*>(sm.fac[slot][0]);
      const float4* h4 = reinterpret_cast<const float4*>(sm.fac[slot][1]);
      for (int x = 0; x < 2; ++x) {
        ok = mbar_wait2(&sm.a_full[x][slot], ((j - 1) / kRing) & 1, &sm.pv_done[x], (j - 1) & 1, abort, status,
                        16 + x);
        if (!ok) break;
        tc_fence_after();
        const float al = sm.alpha[x][slot][r];
        const float rp = sm.rprev[x][slot][r];
        warp_arrive(&sm.a_free[x][slot], lane);
        const bool rescale = !__all_sync(0xffffffffu, al == 1.0f);
        const uint32_t oc = lb + kColO + x * 128;
#pragma unroll
        for (int ch = 0; ch < kD / 32; ++ch) {
          float o[32];
          tmem_ld32(oc + 32 * ch, o);
          tmem_ld_wait();
          reg_fence(o);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 fv = f4[8 * ch + q];
            const float4 hv = h4[8 * ch + q];
            float* op = o + 4 * q;
            fma2(op[0], op[1], rp, rp, hv.x, hv.y);
            fma2(op[2], op[3], rp, rp, hv.z, hv.w);
            float f0 = fv.x, f1 = fv.y, f2 = fv.z, f3 = fv.w;
            if (rescale) {
              mul2(f0, f1, al, al);
              mul2(f2, f3, al, al);
            }
            mul2(op[0], op[1], f0, f1);
            mul2(op[2], op[3], f2, f3);
          }
          tmem_st32(oc + 32 * ch, o);
        }
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(&sm.o_ready[x], lane);
      }
      if (ok) warp_arrive(&sm.f_free[slot], lane);
    }
    // ------------------------------------------------------------ epilogue
    // out = (O_hat + R_last mu_last) * u_last / 448 / l
    if (ok) ok = mbar_wait(&sm.fin_f, 0, abort, status, 18);
    constexpr int ES = (ODT == VCATTN_DTYPE_F32) ? 4 : 2;
    const int bq = g / a.H, hq = g % a.H;
    uint8_t* obase = static_cast<uint8_t*>(a.out) + (bq * a.osb + hq * a.osh) * ES;
    for (int x = 0; x < 2 && ok; ++x) {
      ok = mbar_wait2(&sm.pv_done[x], (nb - 1) & 1, &sm.fin_s[x], 0, abort, status, 19 + x);
      if (!ok) break;
      tc_fence_after();
      const float l = sm.lfin[x][r];
      const float rl = sm.rfin[x][r];
      const int orow = row0 + x * kBM + r;
      uint8_t* orow_p = obase + static_cast<int64_t>(orow) * a.osn * ES;
      const float4* s4 = reinterpret_cast<const float4*>(sm.fin[0]);
      const float4* m4 = reinterpret_cast<const float4*>(sm.fin[1]);
#pragma unroll
      for (int ch = 0; ch < kD / 32; ++ch) {
        float o[32];
        tmem_ld32(lb + kColO + x * 128 + 32 * ch, o);
        tmem_ld_wait();
        reg_fence(o);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 sv = s4[8 * ch + q];
          const float4 mv = m4[8 * ch + q];
          float* op = o + 4 * q;
          fma2(op[0], op[1], rl, rl, mv.x, mv.y);
          fma2(op[2], op[3], rl, rl, mv.z, mv.w);
          mul2(op[0], op[1], sv.x, sv.y);
          mul2(op[2], op[3], sv.z, sv.w);
#pragma unroll
          for (int e = 0; e < 4; ++e) op[e] = __fdiv_rn(op[e], l);
        }
        if (orow < a.N) {
#pragma unroll
          for (int c0 = 0; c0 < 32; c0 += 16 / ES) {
            uint4 w;
#pragma unroll
            for (int e = 0; e < 16 / ES; e += 2)
              stage2<ODT>(reinterpret_cast<uint8_t*>(&w) + e * ES, o[c0 + e], o[c0 + e + 1]);
            *reinterpret_cast<uint4*>(orow_p + (32 * ch + c0) * ES) = w;
          }
        }
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

EncodeTiledFn encode_fn2() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D map over (rows, 128 bytes) with a (box_rows x 128) box and 128-byte swizzle.
bool make_map2(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn2();
  if (!fn) return false;
  cuuint64_t dims[2] = {128, rows};
  cuuint64_t strides[1] = {128};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EC, int ODT>
cudaError_t launch_tc2(const AttnParams& p, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  const uint64_t rows = static_cast<uint64_t>(p.B) * p.H * p.n_pad;
  if (!make_map2(&mq, p.q8, rows, kBM) || !make_map2(&mk, p.k8, rows, kBR) || !make_map2(&mv, p.v8, rows, kBR))
    return cudaErrorInvalidValue;
  Tc2Args a{};
  a.q_scale = p.q_scale; a.k_scale = p.k_scale; a.v_scale = p.v_scale; a.mu = p.mu;
  a.H = p.H; a.N = p.N; a.n_pad = p.n_pad; a.nb = p.n_pad / kBR;
  a.sm_scale = p.sm_scale;
  a.c120 = static_cast<float>(64.0 + 56.0 + p.beta);
  a.out = p.out; a.osb = p.osb; a.osh = p.osh; a.osn = p.osn;
  const size_t smem = sizeof(Tc2Smem) + 1024;
  auto k = attn_tc2_kernel<EC, ODT>;
  // The setmaxnreg split above hands out exactly 128 x 512 registers: a build
  // that launched with fewer would leave the softmax warps' increase waiting.
  static int regs = -1;
  if (regs < 0) {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) return cudaErrorInvalidDeviceFunction;
    regs = fa.numRegs;
  }
  if (regs != 128) {
    snprintf(g_tc2_diag, sizeof(g_tc2_diag), "attn_tc2_kernel built with %d registers per thread, needs 128", regs);
    return cudaErrorInvalidConfiguration;
  }
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid((p.n_pad + 2 * kBM - 1) / (2 * kBM), p.B * p.H);
  k<<<grid, kThreads, smem, st>>>(mq, mk, mv, a);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, k);
    snprintf(g_tc2_diag, sizeof(g_tc2_diag),
             "regs=%d maxThreadsPerBlock=%d staticSmem=%zu dynSmem=%zu maxDynSmem=%d local=%zu threads=%d",
             fa.numRegs, fa.maxThreadsPerBlock, fa.sharedSizeBytes, smem, fa.maxDynamicSharedSizeBytes,
             fa.localSizeBytes, kThreads);
  }
  return e;
}

}  // namespace

bool attn_tc2_supported(const AttnParams& p) { return p.D == 128 && p.block_rows == 128; }

cudaError_t launch_attn_tc2(const AttnParams& p, cudaStream_t st) {
  if (!attn_tc2_supported(p)) return cudaErrorNotSupported;
  const int ec = (p.flags & VCATTN_EXPCAST) ? ((p.flags & VCATTN_EXPCAST_EXACT) ? 2 : 1) : 0;
  switch (p.out_dtype) {
    case VCATTN_DTYPE_BF16:
      return ec == 1 ? launch_tc2<1, VCATTN_DTYPE_BF16>(p, st)
                     : ec == 2 ? launch_tc2<2, VCATTN_DTYPE_BF16>(p, st) : launch_tc2<0, VCATTN_DTYPE_BF16>(p, st);
    case VCATTN_DTYPE_F16:
      return ec == 1 ? launch_tc2<1, VCATTN_DTYPE_F16>(p, st)
                     : ec == 2 ? launch_tc2<2, VCATTN_DTYPE_F16>(p, st) : launch_tc2<0, VCATTN_DTYPE_F16>(p, st);
    default:
      return ec == 1 ? launch_tc2<1, VCATTN_DTYPE_F32>(p, st)
                     : ec == 2 ? launch_tc2<2, VCATTN_DTYPE_F32>(p, st) : launch_tc2<0, VCATTN_DTYPE_F32>(p, st);
  }
}

const char* attn_tc2_diag() { return g_tc2_diag; }

cudaError_t attn_tc2_status(int* code, int* where, int* block, bool reset) {
  tc::DevStatus s{};
  cudaError_t e = cudaMemcpyFromSymbol(&s, g_attn_tc2_status, sizeof(s));
  if (e != cudaSuccess) return e;
  *code = s.code;
  *where = s.where;
  *block = s.block;
  if (reset) {
    tc::DevStatus z{};
    e = cudaMemcpyToSymbol(g_attn_tc2_status, &z, sizeof(z));
  }
  return e;
}

}  // namespace vcattn
