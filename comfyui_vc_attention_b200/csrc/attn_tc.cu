// Fused dense FP8 VC-Attention on the 5th-generation tensor cores (tcgen05).
//
// Same semantics as triton_attn.py:203-322: for every KV tile j (one value
// block of BR keys)
//   s   = (q8 . k8) * qs * ks * sm_scale
//   P   = ExpCast byte of s against the running row max (one FMA form, or
//         with VCATTN_EXPCAST_EXACT the operation order of expcast.py:67-69),
//         or E4M3(exp2((s - m) * log2e) * 448)
//   acc = alpha * acc + (P @ V8) * (vs / 448) + (rowsum(P) / 448) * (mu * vs)
//   l   = alpha * l + rowsum(P) / 448 ;  O = acc / l
//
// One CTA = 128 query rows of one (batch, head); 12 warps in 3 warpgroups:
//   warp 0       TMA producer (Q once; K, V codes + ks, vs, mu per tile)
//   warp 1       MMA issuer and TMEM owner
//   warps 2-3    per-tile factors vs / 448 and mu * vs
//   warps 4-7    softmax: thread = query row = TMEM lane; the row's scores
//                come in with four 32x32b loads behind one wait, the row max
//                needs no shuffles, and the P bytes go back in key order
//   warps 8-11   correction: O in registers, one query row (TMEM lane) per
//                thread, T read with the 32x32b shape
// (The 16x256b shape, which splits a row over four threads, sustains about a
// quarter of the 32x32b tensor-memory bandwidth.)  ks and the per-channel
// factors are read as shared-memory broadcasts.
// TMEM columns: S double buffer [0,128) [128,256); the P bytes (E4M3, keys
// 4c..4c+3 in column c) go over the first BR/4 columns of their S buffer and
// feed the PV MMA from tensor memory; PV tile T_j double buffer [256,384)
// [384,512); the row sum R_j (an N=16 MMA of P_j against an all-ones block)
// goes to the first 16 columns of the other T buffer, whose first quarter
// (T_{j-1}) the correction warps have already read.  Every MMA gate points at
// least one MMA back, so the in-order tensor pipe never drains while a
// handshake completes.
// P is in key order, so V rows are read in token order (prepared without
// VCATTN_V_MMA_ORDER).  Q, K K-major, V MN-major, in the 128-byte swizzle for
// head dim 128 and the 64-byte swizzle for head dim 64.
// Every wait is bounded.
#include <cuda.h>
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "kernels.cuh"
#include "tc_common.cuh"
#include "tc_math.cuh"

namespace vcattn {

__device__ tc::DevStatus g_attn_tc_status;

namespace {

using namespace tc;
char g_tc_diag[256];
// Bounded-wait test hook (vcattn_inject_stall): the producer stops before
// this KV tile in the launches that follow (-1: never).
int g_stall_tile = -1;

constexpr int kBM = 128;
constexpr int kStages = 4;
constexpr int kRing = 4;        // per-tile factor / alpha hand-off depth
constexpr int kThreads = 384;   // 12 warps = 3 warpgroups
constexpr uint32_t kColS = 0, kColT = 256;
// Factor tables in fragment order: the 32 entries lane group q (= lane % 4)
// reads are contiguous, groups 36 floats apart so their float4 reads fall
// in different banks.

// D = 128: Q, K, V rows of 128 bytes in the 128-byte swizzle; D = 64: rows
// of 64 bytes in the 64-byte swizzle (8-row atoms of 512 bytes).
template <int BR, int D>
struct TcSmem {
  // q, k and v are contiguous: after the last tile they stage the output.
  alignas(1024) uint8_t q[kBM * D];
  alignas(1024) uint8_t k[kStages][BR * D];
  alignas(1024) uint8_t v[kStages][BR * D];
  alignas(1024) uint8_t ones[16 * 128];
  alignas(16) float ks[kStages][BR];
  alignas(16) float vs[kStages][D];
  alignas(16) float mu[kStages][D];
  alignas(16) float cm[kRing][2][D];             // vs / 448 and mu * vs per channel
  alignas(16) float alpha[kRing][kBM];            // per query row
  alignas(8) uint64_t q_full;
  alignas(8) uint64_t kv_full[kStages];
  alignas(8) uint64_t kv_empty[kStages];
  alignas(8) uint64_t s_full[2];
  alignas(8) uint64_t p_full[2];
  alignas(8) uint64_t t_full[2];
  // Correction of tile i has read R_i and the first quarter of T_i (and all
  // of T_{i-1}): PV_{i+1} / R_{i+1} may write T_{(i+1)&1} and T_i[0,16).
  alignas(8) uint64_t t_rel;
  alignas(8) uint64_t a_full[kRing];
  alignas(8) uint64_t a_free[kRing];
  alignas(8) uint64_t f_full[kRing];
  alignas(8) uint64_t f_free[kRing];
  alignas(8) uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int kvn;     // keys taking part in this CTA's head
  int g;       // head (b * H + h)
  int row0;    // first query row
  int slot;    // KV piece of a split query tile (partial output slot), or -1
  int j0;      // first KV tile of this CTA (0 unless it runs one piece of a split query tile)
  int ntl;     // KV tiles this CTA visits
  int kv0;     // kvn - j0 * BR: keys of this CTA's tile range from its first tile on
  int nload;   // KV tiles the producer loads (fewer only under vcattn_inject_stall)
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
  const int32_t* kv_len;   // (B,) keys taking part per batch entry, or null (all N)
  int stall_tile;          // tests: the producer stops before this KV tile (-1: never)
  // Grid: CTA t < n_main runs query tile t of the flattened (head, query
  // tile) order whole; CTA n_main + u runs KV piece u % pieces of query tile
  // n_main + u / pieces and writes its unnormalised partial to part_o
  // ([u][D][128]), part_l and part_m ([u][128]: row sum and log2-domain max).
  int qt;                  // query tiles per head
  int n_main;
  int pieces;              // >= 1
  int tp;                  // KV tiles per piece
  float* part_o;
  float* part_l;
  float* part_m;
};

// ECM: 0 = E4M3 of exp2, 1 = one-FMA ExpCast, 2 = ExpCast in the reference's
// operation order on s = (S * (qs * ks)) * sm_scale (parity runs).
template <int D>
__device__ __forceinline__ uint64_t operand_desc(uint32_t saddr) {
  // the same descriptor serves K-major Q/K and MN-major V (the instruction
  // descriptor carries the major-ness): one swizzle atom across the row
  if constexpr (D == 128) return desc_kmajor(saddr);
  else return desc_kmajor64(saddr);
}

template <int BR, int D, int ECM, int ODT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  constexpr int NCH = BR / 32;   // 32-key chunks per tile
  constexpr int kD = D;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  TcSmem<BR, D>& sm = *reinterpret_cast<TcSmem<BR, D>*>(smem_raw + pad);
  DevStatus* status = &g_attn_tc_status;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = a.nb;

  if (tid == 0) {
    // (head, query tile) of this CTA, kept in shared memory (read where used,
    // so that no role holds them in registers through its loop)
    const int cta = static_cast<int>(blockIdx.x);
    const int slot = cta < a.n_main ? -1 : cta - a.n_main;
    const int tq = slot < 0 ? cta : a.n_main + slot / a.pieces;
    const int g = tq / a.qt;
    sm.g = g;
    sm.row0 = (tq - g * a.qt) * kBM;
    sm.slot = slot;
    // Keys at (permuted) positions >= kvn take no part (reference.py
    // valid_len, padding sorted to the tail by grouping.py:181-183); only the
    // tiles holding keys below kvn are visited.
    sm.kvn = a.kv_len ? min(a.N, max(1, a.kv_len[g / a.H])) : a.N;
    const int tiles = (sm.kvn + BR - 1) / BR;
    int j0 = 0, nt = tiles;
    if (slot >= 0) {
      j0 = (slot % a.pieces) * a.tp;
      nt = max(0, min(a.tp, tiles - j0));
    }
    sm.j0 = j0;
    sm.kv0 = sm.kvn - j0 * BR;
    sm.ntl = nt;
    sm.nload = a.stall_tile >= 0 ? min(nt, a.stall_tile) : nt;

    sm.abort = 0;
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1 + 2);   // PV commit + factor warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.p_full[b], 4);
      mbar_init(&sm.t_full[b], 1);
    }
    mbar_init(&sm.t_rel, 4);
    for (int r = 0; r < kRing; ++r) {
      mbar_init(&sm.a_full[r], 4);
      mbar_init(&sm.a_free[r], 4);
      mbar_init(&sm.f_full[r], 2);
      mbar_init(&sm.f_free[r], 4);
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
#define VC_TILES_VISITED (sm.ntl)

  if (warp < 4) {
  // Register budget per warpgroup (launched at 168 x 384 = 64512):
  // 128 x (40 producer/MMA/factors + 200 softmax + 248 correction) = 62464.
  asm volatile("setmaxnreg.dec.sync.aligned.u32 40;\n" ::: "memory");
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int issued = 0;
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_expect_tx(&sm.q_full, kBM * kD);
      const int g = sm.g, j0 = sm.j0;
      tma_load_2d(sm.q, &tm_q, 0, g * a.n_pad + sm.row0, &sm.q_full);
      const uint32_t tile_bytes = 2u * BR * kD + BR * 4u + 2u * kD * 4u;
      // (under vcattn_inject_stall the copies of tile nload on never come,
      // and the waits on them time out)
      for (int j = 0; j < sm.nload; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&sm.kv_empty[s], ((j / kStages) + 1) & 1, abort, status, 1)) break;
        mbar_expect_tx(&sm.kv_full[s], tile_bytes);
        const int krow = g * a.n_pad + (j0 + j) * BR;
        tma_load_2d(sm.k[s], &tm_k, 0, krow, &sm.kv_full[s]);
        tma_load_2d(sm.v[s], &tm_v, 0, krow, &sm.kv_full[s]);
        bulk_load(sm.ks[s], a.k_scale + static_cast<int64_t>(krow), BR * 4, &sm.kv_full[s]);
        const int64_t vo = (static_cast<int64_t>(g) * nb + j0 + j) * kD;
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
    {
      const uint32_t leader = elect_one();
      const uint32_t id_qk = idesc_e4m3(kBM, BR, false);
      const uint32_t id_pv = idesc_e4m3(kBM, kD, true);
      const uint32_t id_r = idesc_e4m3(kBM, 16, false);
      const uint32_t q_addr = smem_u32(sm.q);
      const uint32_t ones_addr = smem_u32(sm.ones);
      bool ok = mbar_wait(&sm.q_full, 0, abort, status, 2);
      for (int j = 0; ok && j <= VC_TILES_VISITED; ++j) {
        if (j < VC_TILES_VISITED) {
          // S_b was last read as P by PV_{j-2}, issued earlier by this thread
          // (tcgen05.mma from one thread run in order), after p_full(j-2).
          const int s = j % kStages, b = j & 1;
          ok = mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 3);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm.k[s]);
#pragma unroll
          for (int kk = 0; kk < kD / 32; ++kk)
            mma_f8_if(tbase + kColS + b * 128, operand_desc<D>(q_addr + kk * 32), operand_desc<D>(k_addr + kk * 32),
                      id_qk, kk > 0, leader);
          tc_commit_if(&sm.s_full[b], leader);
        }
        if (j >= 1) {
          const int i = j - 1, bi = i & 1, si = i % kStages;
          // T_bi last held T_{i-2} and R_{i-1}; R_i goes over the first
          // quarter of T_{i-1}: all three read once tile i-1 is released.
          ok = i >= 1 ? mbar_wait2(&sm.p_full[bi], (i >> 1) & 1, &sm.t_rel, (i - 1) & 1, abort, status, 5)
                      : mbar_wait(&sm.p_full[bi], (i >> 1) & 1, abort, status, 5);
          if (!ok) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sm.v[si]);
          const uint32_t p_t = tbase + kColS + bi * 128;   // A positions [32kk, 32kk+32) at columns 8kk..8kk+7
#pragma unroll
          for (int kk = 0; kk < BR / 32; ++kk)
            mma_f8_ts_if(tbase + kColT + bi * 128, p_t + 8 * kk, operand_desc<D>(v_addr + kk * 32 * kD), id_pv,
                         kk > 0, leader);
#pragma unroll
          for (int kk = 0; kk < BR / 32; ++kk)
            mma_f8_ts_if(tbase + kColT + (bi ^ 1) * 128, p_t + 8 * kk, desc_kmajor(ones_addr + kk * 32), id_r, kk > 0, leader);
          tc_commit_if(&sm.t_full[bi], leader);
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
    // ------------------------------------------------------------ per-tile factors
    const int c2 = tid - 64;   // 0..63
    for (int j = 0; j < VC_TILES_VISITED; ++j) {
      const int s = j % kStages, ring = j % kRing;
      if (!mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 13)) break;
      if (j >= kRing && !mbar_wait(&sm.f_free[ring], ((j / kRing) + 1) & 1, abort, status, 14)) break;
#pragma unroll
      for (int h = 0; h < kD / 64; ++h) {
        const int c = c2 + 64 * h;
        const float vsc = sm.vs[s][c];
        sm.cm[ring][0][c] = __fdiv_rn(vsc, 448.0f);
        sm.cm[ring][1][c] = __fmul_rn(sm.mu[s][c], vsc);
      }
      warp_arrive(&sm.f_full[ring], lane);
      warp_arrive(&sm.kv_empty[s], lane);
    }
  }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 200;\n" ::: "memory");
    // ------------------------------------------------------------ softmax
    // Thread = query row t = 32 (w%4) + lane = TMEM lane t: the whole row of S
    // in registers (32x32b loads, one wait), the row max without shuffles,
    // P for keys 4c..4c+3 in column c (key order: V is read in token order).
    const int t = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int row0 = sm.row0;
    const int64_t qrow = static_cast<int64_t>(sm.g) * a.n_pad + row0 + t;
    const float qs = (row0 + t < a.n_pad) ? a.q_scale[qrow] : 0.f;
    const float qsm = __fmul_rn(qs, a.sm_scale);
    // ExpCast: c = A * (x - m) + c120 with A = 8 log2e qs sm; evaluated as
    // fma.sat(x, A/128, B/128) so the clamp at 0 is free and the /128 scale
    // makes a + 98304 round the code to an integer in the low bits.
    const float As = __fmul_rn(8.0f * kLog2e, qsm) * (1.0f / 128.0f);
    // The row max is kept in x units (x = S * ks), or in score units s for ECM 2.
    const float Ae = (ECM == 2) ? kLog2e : __fmul_rn(qsm, kLog2e);
    float m = -INFINITY;
    for (int j = 0; j < VC_TILES_VISITED; ++j) {
      const int b = j & 1, ring = j % kRing, s = j % kStages;
      // ks of tile j came with its K/V stage (bulk copy completed on kv_full)
      if (!mbar_wait2(&sm.s_full[b], (j >> 1) & 1, &sm.kv_full[s], (j / kStages) & 1, abort, status, 7)) break;
      tc_fence_after();
      const uint32_t sb = lane_base + kColS + b * 128;
      float x[BR];
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
        tmem_ld32(sb + 32 * ch, *reinterpret_cast<float(*)[32]>(x + 32 * ch));
      tmem_ld_wait();
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) reg_fence(*reinterpret_cast<float(*)[32]>(x + 32 * ch));
      const float4* k4 = reinterpret_cast<const float4*>(sm.ks[s]);
      if constexpr (ECM == 2) {
        // s = (S * (qs * ks)) * sm_scale, rounded at each step
#pragma unroll
        for (int q = 0; q < BR / 4; ++q) {
          const float4 kv = k4[q];
          x[4 * q] = __fmul_rn(__fmul_rn(x[4 * q], __fmul_rn(qs, kv.x)), a.sm_scale);
          x[4 * q + 1] = __fmul_rn(__fmul_rn(x[4 * q + 1], __fmul_rn(qs, kv.y)), a.sm_scale);
          x[4 * q + 2] = __fmul_rn(__fmul_rn(x[4 * q + 2], __fmul_rn(qs, kv.z)), a.sm_scale);
          x[4 * q + 3] = __fmul_rn(__fmul_rn(x[4 * q + 3], __fmul_rn(qs, kv.w)), a.sm_scale);
        }
      } else {
#pragma unroll
        for (int q = 0; q < BR / 4; ++q) {
          const float4 kv = k4[q];
          mul2(x[4 * q], x[4 * q + 1], kv.x, kv.y);
          mul2(x[4 * q + 2], x[4 * q + 3], kv.z, kv.w);
        }
      }
      const int valid = sm.kv0 - j * BR;                 // keys >= valid are padding or masked
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
      const float mn = fmax3(m0, m1, fmaxf(m2, m3));
      const float al = (m == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m, mn), Ae));
      // P words: chunk ch (keys 32 ch .. 32 ch + 31) to columns 8 ch .. 8 ch + 7
      if constexpr (ECM == 2) {
        // expcast.py:67-69: u = (s - m) * log2e + 8 ; c = u * 8 + (56 + beta)
        // (u * 8 is exact, so one FMA rounds the sum once, as torch does)
        const float c0 = a.c120 - 64.0f;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          uint32_t packed[8];
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            const float* xc = x + 32 * ch + 4 * w;
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
            const float* xc = x + 32 * ch + 4 * w;
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
            const float* xc = x + 32 * ch + 4 * w;
            packed[w] = exp4(xc[0], xc[1], xc[2], xc[3], Ae, Be);
          }
          tmem_st8(sb + 8 * ch, packed);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(&sm.p_full[b], lane);
      if (j >= kRing && !mbar_wait(&sm.a_free[ring], ((j / kRing) + 1) & 1, abort, status, 10)) break;
      sm.alpha[ring][t] = al;
      warp_arrive(&sm.a_full[ring], lane);
      m = mn;
    }
    // split piece: its row max in the log2 domain, for the combine
    if (sm.slot >= 0) a.part_m[sm.slot * kBM + t] = __fmul_rn(m, Ae);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 248;\n" ::: "memory");
    // ------------------------------------------------------------ correction
    // Thread = query row r = 32 (w%4) + lane (TMEM lane r), O[D] in
    // registers; T read with the 32x32b shape, 64 columns per load batch.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lb = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    float o[kD];
#pragma unroll
    for (int c = 0; c < kD; ++c) o[c] = 0.f;
    float l = 0.f;
    bool ok = true;
    for (int i = 0; i < VC_TILES_VISITED; ++i) {
      const int ring = i % kRing, tb = i & 1;
      ok = mbar_wait(&sm.t_full[tb], (i >> 1) & 1, abort, status, 11);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tcol = kColT + tb * 128;
      float xa[32], xb[32];
      float rs = tmem_ld1(lb + kColT + (tb ^ 1) * 128);   // R_i sits in T_{(i+1)&1}
      tmem_ld32(lb + tcol, xa);
      tmem_ld32(lb + tcol + 32, xb);
      tmem_ld_wait();
      asm volatile("" : "+f"(rs));
      reg_fence(xa);
      reg_fence(xb);
      tc_fence_before();
      warp_arrive(&sm.t_rel, lane);   // PV_{i+1} may write T_{(i+1)&1}, R_{i+1} the first quarter of T_i
      ok = mbar_wait2(&sm.a_full[ring], (i / kRing) & 1, &sm.f_full[ring], (i / kRing) & 1, abort, status, 12);
      if (!ok) break;
      const float al = sm.alpha[ring][r];
      warp_arrive(&sm.a_free[ring], lane);
      const bool rescale = !__all_sync(0xffffffffu, al == 1.0f);
      const float rr = rs * (1.0f / 448.0f);
      const float4* f4 = reinterpret_cast<const float4*>(sm.cm[ring][0]);
      const float4* g4 = reinterpret_cast<const float4*>(sm.cm[ring][1]);
#pragma unroll
      for (int half = 0; half < kD / 64; ++half) {
        if (half == 1) {
          tmem_ld32(lb + tcol + 64, xa);
          tmem_ld32(lb + tcol + 96, xb);
          tmem_ld_wait();
          reg_fence(xa);
          reg_fence(xb);
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float* src = (q < 8) ? xa + 4 * q : xb + 4 * (q - 8);
          const float4 fv = f4[16 * half + q];
          const float4 gv = g4[16 * half + q];
          float* oc = o + 64 * half + 4 * q;
          if (rescale) {
            mul2(oc[0], oc[1], al, al);
            mul2(oc[2], oc[3], al, al);
          }
          fma2(oc[0], oc[1], src[0], src[1], fv.x, fv.y);
          fma2(oc[2], oc[3], src[2], src[3], fv.z, fv.w);
          fma2(oc[0], oc[1], rr, rr, gv.x, gv.y);
          fma2(oc[2], oc[3], rr, rr, gv.z, gv.w);
        }
      }
      warp_arrive(&sm.f_free[ring], lane);
      l = __fadd_rn(__fmul_rn(l, al), rr);
    }
    const int slot = sm.slot;
    if (ok && !*abort && slot >= 0) {
      // split piece: unnormalised O (channel-major, coalesced over rows) and l
      float* po = a.part_o + static_cast<int64_t>(slot) * kD * kBM + r;
#pragma unroll
      for (int c = 0; c < kD; ++c) po[c * kBM] = o[c];
      a.part_l[slot * kBM + r] = l;
    } else if (ok && !*abort) {
      // Stage this warp's 32 rows (padded stride), then write them out as
      // whole 16-byte row chunks.
      constexpr int ES = (ODT == VCATTN_DTYPE_F32) ? 4 : 2;
      constexpr int RS = kD * ES + 16;
      static_assert(kBM * RS <= static_cast<int>(sizeof(TcSmem<BR, D>::q) + sizeof(TcSmem<BR, D>::k) +
                                                 sizeof(TcSmem<BR, D>::v)),
                    "output staging must fit in the operand buffers");
      uint8_t* stage = sm.q + wq * 32 * RS;
#pragma unroll
      for (int c0 = 0; c0 < kD; c0 += 16 / ES) {
        uint4 w;
#pragma unroll
        for (int e = 0; e < 16 / ES; e += 2)
          stage2<ODT>(reinterpret_cast<uint8_t*>(&w) + e * ES, __fdiv_rn(o[c0 + e], l), __fdiv_rn(o[c0 + e + 1], l));
        *reinterpret_cast<uint4*>(stage + lane * RS + c0 * ES) = w;
      }
      __syncwarp();
      constexpr int CPR = kD * ES / 16;   // 16-byte chunks per row
      const int g = sm.g, row0 = sm.row0;
      const int bq = g / a.H, hq = g % a.H;
      uint8_t* out = static_cast<uint8_t*>(a.out) + (bq * a.osb + hq * a.osh) * ES;
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
#undef VC_TILES_VISITED

constexpr int kMaxPieces = 32;

// The split query tiles: out = sum_p w_p O_p / sum_p w_p l_p with
// w_p = exp2(m_p - max_p m_p) (m_p in the log2 domain), one thread per row.
template <int D, int ODT>
__global__ void __launch_bounds__(kBM) attn_tc_combine_kernel(const TcArgs a) {
  const int e = blockIdx.x, r = threadIdx.x;
  const int tq = a.n_main + e;
  const int g = tq / a.qt;
  const int row = (tq - g * a.qt) * kBM + r;
  if (row >= a.N) return;
  const int u0 = e * a.pieces;
  float mx = -INFINITY;
  for (int q = 0; q < a.pieces; ++q) mx = fmaxf(mx, a.part_m[(u0 + q) * kBM + r]);
  float w[kMaxPieces];
  float den = 0.f;
#pragma unroll
  for (int q = 0; q < kMaxPieces; ++q) {
    w[q] = q < a.pieces ? exp2f(__fsub_rn(a.part_m[(u0 + q) * kBM + r], mx)) : 0.f;
    if (q < a.pieces) den = __fmaf_rn(w[q], a.part_l[(u0 + q) * kBM + r], den);
  }
  constexpr int ES = (ODT == VCATTN_DTYPE_F32) ? 4 : 2;
  const int bq = g / a.H, hq = g % a.H;
  uint8_t* out = static_cast<uint8_t*>(a.out) + ((bq * a.osb + hq * a.osh) + static_cast<int64_t>(row) * a.osn) * ES;
  const float* po = a.part_o + static_cast<int64_t>(u0) * D * kBM + r;
  for (int c = 0; c < D; c += 2) {
    float n0 = 0.f, n1 = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxPieces; ++q) {
      if (q < a.pieces) {
        n0 = __fmaf_rn(w[q], po[(static_cast<int64_t>(q) * D + c) * kBM], n0);
        n1 = __fmaf_rn(w[q], po[(static_cast<int64_t>(q) * D + c + 1) * kBM], n1);
      }
    }
    stage2<ODT>(out + c * ES, __fdiv_rn(n0, den), __fdiv_rn(n1, den));
  }
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

// 2-D map over (rows, D bytes) with a (box_rows x D) box: the 128-byte
// swizzle for D = 128, the 64-byte swizzle for D = 64.
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows, int D) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), rows};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(D)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(D), box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return n > 0 ? n : 148;
}

// Which query tiles run split over their KV tiles (see TcArgs).  Auto: when
// the CTAs end in a partial wave holding at most half of the SMs, its query
// tiles run in about SMs / (tiles in that wave) pieces each, so the last wave
// takes a fraction of a CTA's time instead of a whole one.
struct SplitPlan {
  int qt, n_main, pieces, tp, nsplit;
};

SplitPlan plan_split(const AttnParams& p) {
  SplitPlan s{};
  s.qt = (p.n_pad + kBM - 1) / kBM;
  const int ctas = p.B * p.H * s.qt;
  const int tiles = (p.N + p.block_rows - 1) / p.block_rows;
  s.n_main = ctas;
  s.pieces = 1;
  s.tp = tiles;
  s.nsplit = 0;
  if (p.kv_len != nullptr || g_stall_tile >= 0 || p.kv_split == 1 || p.part == nullptr || tiles < 2) return s;
  int r = ctas, want = p.kv_split;
  if (p.kv_split <= 0) {
    const int nsm = sm_count();
    r = ctas % nsm;
    if (ctas <= nsm || r == 0 || r > nsm / 2) return s;
    want = nsm / r;
  }
  want = std::min(want, std::min(tiles, kMaxPieces));
  if (want < 2) return s;
  const int tp = (tiles + want - 1) / want;
  const int pieces = (tiles + tp - 1) / tp;
  if (pieces < 2) return s;
  s.n_main = ctas - r;
  s.pieces = pieces;
  s.tp = tp;
  s.nsplit = r * pieces;
  return s;
}

template <int BR, int D, int EC, int ODT>
cudaError_t launch_tc(const AttnParams& p, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  const uint64_t rows = static_cast<uint64_t>(p.B) * p.H * p.n_pad;
  if (!make_map(&mq, p.q8, rows, kBM, D) || !make_map(&mk, p.k8, rows, BR, D) ||
      !make_map(&mv, p.v8, rows, BR, D))
    return cudaErrorInvalidValue;
  TcArgs a{};
  a.q_scale = p.q_scale; a.k_scale = p.k_scale; a.v_scale = p.v_scale; a.mu = p.mu;
  a.H = p.H; a.N = p.N; a.n_pad = p.n_pad; a.nb = p.n_pad / BR;
  a.sm_scale = p.sm_scale;
  a.c120 = static_cast<float>(64.0 + 56.0 + p.beta);
  a.out = p.out; a.osb = p.osb; a.osh = p.osh; a.osn = p.osn;
  a.kv_len = p.kv_len;
  a.stall_tile = g_stall_tile;
  const SplitPlan sp = plan_split(p);
  a.qt = sp.qt;
  a.n_main = sp.n_main;
  a.pieces = sp.pieces;
  a.tp = sp.tp;
  if (sp.nsplit > 0) {
    float* part = static_cast<float*>(p.part);
    a.part_o = part;
    a.part_l = part + static_cast<size_t>(sp.nsplit) * D * kBM;
    a.part_m = a.part_l + static_cast<size_t>(sp.nsplit) * kBM;
  }
  const size_t smem = sizeof(TcSmem<BR, D>) + 1024;
  auto k = attn_tc_kernel<BR, D, EC, ODT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned ctas = static_cast<unsigned>(sp.n_main + sp.nsplit);
  k<<<ctas, kThreads, smem, st>>>(mq, mk, mv, a);
  e = cudaGetLastError();
  if (e == cudaSuccess && sp.nsplit > 0) {
    attn_tc_combine_kernel<D, ODT><<<sp.nsplit / sp.pieces, kBM, 0, st>>>(a);
    e = cudaGetLastError();
  }
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

template <int BR, int D>
cudaError_t dispatch_tc(const AttnParams& p, cudaStream_t st) {
  const int ec = (p.flags & VCATTN_EXPCAST) ? ((p.flags & VCATTN_EXPCAST_EXACT) ? 2 : 1) : 0;
  switch (p.out_dtype) {
    case VCATTN_DTYPE_BF16:
      return ec == 1 ? launch_tc<BR, D, 1, VCATTN_DTYPE_BF16>(p, st)
                     : ec == 2 ? launch_tc<BR, D, 2, VCATTN_DTYPE_BF16>(p, st)
                               : launch_tc<BR, D, 0, VCATTN_DTYPE_BF16>(p, st);
    case VCATTN_DTYPE_F16:
      return ec == 1 ? launch_tc<BR, D, 1, VCATTN_DTYPE_F16>(p, st)
                     : ec == 2 ? launch_tc<BR, D, 2, VCATTN_DTYPE_F16>(p, st)
                               : launch_tc<BR, D, 0, VCATTN_DTYPE_F16>(p, st);
    default:
      return ec == 1 ? launch_tc<BR, D, 1, VCATTN_DTYPE_F32>(p, st)
                     : ec == 2 ? launch_tc<BR, D, 2, VCATTN_DTYPE_F32>(p, st)
                               : launch_tc<BR, D, 0, VCATTN_DTYPE_F32>(p, st);
  }
}

}  // namespace

cudaError_t launch_attn_tc(const AttnParams& p, cudaStream_t st) {
  if (p.D == 128) return p.block_rows == 128 ? dispatch_tc<128, 128>(p, st) : dispatch_tc<64, 128>(p, st);
  if (p.D == 64) return p.block_rows == 128 ? dispatch_tc<128, 64>(p, st) : dispatch_tc<64, 64>(p, st);
  return cudaErrorNotSupported;
}

const char* attn_tc_diag() { return g_tc_diag; }

void set_attn_tc_stall(int tile) { g_stall_tile = tile; }

size_t attn_tc_split_bytes(const AttnParams& p) {
  AttnParams q = p;
  q.part = reinterpret_cast<void*>(16);   // plan as if a workspace were given
  const SplitPlan sp = plan_split(q);
  return static_cast<size_t>(sp.nsplit) * kBM * (p.D + 2) * sizeof(float);
}

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
