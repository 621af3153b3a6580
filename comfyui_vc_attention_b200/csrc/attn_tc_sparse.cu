// Fused block-sparse FP8 VC-Attention on the tcgen05 tensor cores.
//
// Semantics of triton_attn.py:384-501 (the Sol-Attn routed kernel): for each
// query block (64 rows) the KV blocks are walked in groups of 16.  A group's
// approximated blocks (keep = 0) are folded first with a per-row proxy,
//   x_ap = q8 . bf16(k_mean_j)              (scores s = x * qs * sm_scale)
//   m'   = max(m, max_j x_ap) ; alpha = exp2((m - m') qs sm log2e)
//   p_ap = exp2((x_ap - m') qs sm log2e) * len_j
//   acc  = alpha acc + bf16(p_ap) @ bf16(v_mean) ; l = alpha l + sum p_ap
// and its kept blocks then run the exact tile of the dense kernel in
// ascending order.  Skipped blocks are never loaded.
//
// One CTA = 128 query rows = two routing query blocks (A: rows 0-63, B: rows
// 64-127).  KV tiles are value blocks of BR = 128 or 64 keys; head dims 128
// (128-byte swizzled operand rows) and 64 (64-byte swizzle) are built.  The CTA walks one step list: per group an approximation step if
// either query block approximates a block of it, then the union of both
// blocks' kept tiles.  A warp's rows lie in one query block (TMEM quadrants
// 0-1 are block A, 2-3 block B), so a step that does not concern a warp's
// block is a uniform no-op for it: P = 0 and alpha = 1 leave its rows'
// running max, sum and accumulator exactly unchanged.
//
// Pipeline (roles, TMEM and barriers) is that of attn_tc.cu; approximation
// steps use the same slots:
//   QK slot:  S_b[0,16)  = Q(bf16) . K_mean(bf16)^T      tcgen05.mma kind::f16
//   softmax:  P_ap (bf16) into S_b[0,8), alpha, sum p_ap into shared memory
//   PV slot:  T_b = P_ap @ V_mean(bf16)                   tcgen05.mma kind::f16,
//             A from tensor memory, two N = 64 halves
//   correction: acc = alpha acc + T_b ; l = alpha l + sum p_ap
// The group's bf16 k_mean / v_mean operand tiles come prepared (route tiles
// of prepare.cu, already in the swizzled layout) and are bulk-copied into the
// step's K / V stage; the softmax warps convert Q to bf16 once per CTA when
// the CTA has a proxy step.  Every wait is bounded.
#include <cuda.h>
#include <cuda_fp8.h>
#include <cstdio>
#include <mutex>

#include "kernels.cuh"
#include "tc_common.cuh"
#include "tc_math.cuh"

namespace vcattn {

__device__ tc::DevStatus g_attn_sparse_tc_status;

namespace {

using namespace tc;
char g_sp_diag[256];

constexpr int kBM = 128;
constexpr int kGroup = 16;
constexpr int kQBlock = 64;
constexpr int kStages = 4;
constexpr int kRing = 4;
constexpr int kThreads = 512;
constexpr int kMaxSteps = 1024 + 64;    // nb + groups: N up to 128K tokens (BR = 128), 64K (BR = 64)
constexpr uint32_t kColS = 0, kColT = 256;
constexpr int kFStride = 36;
__host__ __device__ constexpr int ks_index(int k) {
  return ((k >> 1) & 3) * kFStride + (k >> 5) * 8 + ((k >> 3) & 3) * 2 + (k & 1);
}
// Byte offset of (row r, byte c) in a 128-byte-swizzled tile with 128-byte rows.
__host__ __device__ constexpr int sw128(int r, int c) { return r * 128 + ((((c >> 4) ^ (r & 7)) & 7) << 4) + (c & 15); }
// Q, K and V operand descriptors: one swizzle atom across the row (the
// instruction descriptor carries the major-ness).
template <int D>
__device__ __forceinline__ uint64_t operand_desc(uint32_t saddr) {
  if constexpr (D == 128) return desc_kmajor(saddr);
  else return desc_kmajor64(saddr);
}

// Step list entry: info = index (block or group) | kind << 31 (1 = approximation);
// mask = kept bits (bit 0 block A, bit 1 block B) of an exact step, or the
// approximated-block bits of an approximation step (A: 0-15, B: 16-31).
struct Step {
  uint32_t info, mask;
};
__device__ __forceinline__ bool step_is_ap(const Step& s) { return (s.info >> 31) != 0; }
__device__ __forceinline__ int step_index(const Step& s) { return static_cast<int>(s.info & 0xffffu); }

template <int BR, int D>
struct SpSmem {
  alignas(1024) uint8_t q[kBM * D];
  alignas(1024) uint8_t k[kStages][BR * D];   // exact: K codes; proxy: bf16 k_mean tile (D * 32 bytes)
  alignas(1024) uint8_t v[kStages][BR * D];   // exact: V codes; proxy: bf16 v_mean tile (D * 32 bytes)
  alignas(1024) uint8_t qb[D / 64][kBM * 128];   // Q as bf16, 64-element K atoms
  alignas(1024) uint8_t ones[16 * 128];
  alignas(16) float ks[kStages][BR];
  alignas(16) float vs[kStages][D];
  alignas(16) float mu[kStages][D];
  alignas(16) float cm[kRing][2][4 * kFStride];
  alignas(16) float ksf[kRing][4 * kFStride];
  alignas(16) float alpha[kRing][kBM];   // per query row
  alignas(16) float lsum[kRing][kBM];    // approximation steps: sum p_ap, per query row
  Step steps[kMaxSteps];
  int nsteps;
  int has_ap;
  alignas(8) uint64_t q_full;
  alignas(8) uint64_t qb_full;
  alignas(8) uint64_t kv_full[kStages];
  alignas(8) uint64_t kv_empty[kStages];
  alignas(8) uint64_t s_full[2];
  alignas(8) uint64_t p_full[2];
  alignas(8) uint64_t t_full[2];
  alignas(8) uint64_t t_rel;
  alignas(8) uint64_t a_full[kRing];
  alignas(8) uint64_t a_free[kRing];
  alignas(8) uint64_t f_full[kRing];
  alignas(8) uint64_t f_free[kRing];
  alignas(8) uint64_t drain;
  uint32_t tmem_base;
  int abort;
};


struct SpArgs {
  const uint8_t* q8;   // (G, NP, D) codes, read directly only by the D = 64 proxy conversion
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  const float* mu;
  const uint8_t* ap_tiles;
  const uint8_t* keep;
  int H, N, n_pad, nb, nqb, ngroups;
  float sm_scale;
  float c120;
  void* out;
  int64_t osb, osh, osn;
};

// Instruction descriptor of kind::f16 with bf16 A and B and f32 accumulate.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(b_mn_major) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}
__device__ __forceinline__ void mma_bf16_if(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate, uint32_t leader) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.ne.b32 e, %5, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(leader)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_ts_if(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate, uint32_t leader) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.ne.b32 e, %5, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(leader)
      : "memory");
}
__device__ __forceinline__ uint16_t bf16_bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return static_cast<uint32_t>(bf16_bits(lo)) | (static_cast<uint32_t>(bf16_bits(hi)) << 16);
}
__device__ __forceinline__ void tmem_st_16x256b_x1(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void tmem_ld_16x256b_x2(uint32_t taddr, float (&v)[8]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

// P codes of one tile (NCH chunks of 32 keys, 8 columns each) into TMEM.
template <int NCH>
__device__ __forceinline__ void store_p(uint32_t taddr, const uint32_t (&r)[4 * NCH]) {
  if constexpr (NCH == 4) tmem_st_16x256b_x4(taddr, r);
  else tmem_st_16x256b_x2(taddr, r);
}

template <int BR, int D, bool EXPCAST, int ODT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_sparse_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const SpArgs a) {
  constexpr int NCH = BR / 32;   // 32-key chunks per tile
  static_assert(sizeof(SpSmem<BR, D>) + 1024 <= 232448, "shared memory of the sparse kernel exceeds 227 KB");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  SpSmem<BR, D>& sm = *reinterpret_cast<SpSmem<BR, D>*>(smem_raw + pad);
  DevStatus* status = &g_attn_sparse_tc_status;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.y;
  const int row0 = blockIdx.x * kBM;
  const int nb = a.nb;

  if (tid == 0) {
    sm.abort = 0;
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.qb_full, 8);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1 + 2);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.p_full[b], 8);
      mbar_init(&sm.t_full[b], 1);
    }
    mbar_init(&sm.t_rel, 4);
    for (int r = 0; r < kRing; ++r) {
      mbar_init(&sm.a_full[r], 8);
      mbar_init(&sm.a_free[r], 4);
      mbar_init(&sm.f_full[r], 2);
      mbar_init(&sm.f_free[r], 8 + 4);
    }
    mbar_init(&sm.drain, 1);
    fence_mbar_init();
  }
  for (int i = tid; i < 16 * 128; i += kThreads) sm.ones[i] = 0x38;
  // Step list (warp 0): lane l handles group gbase + l; its 16 keep bytes of
  // each query block are independent loads, and a warp scan of the steps per
  // group gives every lane its slot in the list.
  if (warp == 0) {
    const int qa = 2 * blockIdx.x, qbk = 2 * blockIdx.x + 1;
    const uint8_t* keep_a = a.keep + (static_cast<int64_t>(g) * a.nqb + qa) * nb;
    const uint8_t* keep_b = a.keep + (static_cast<int64_t>(g) * a.nqb + qbk) * nb;
    const bool has_b = qbk < a.nqb;
    const int ngr = (nb + kGroup - 1) / kGroup;
    int n_base = 0, any_ap = 0;
    for (int gbase = 0; gbase < ngr; gbase += 32) {
      const int gi = gbase + lane;
      uint32_t km_a = 0, km_b = 0, vm = 0;
      if (gi < ngr) {
        const int b0 = gi * kGroup;
#pragma unroll
        for (int i = 0; i < kGroup; ++i) {
          if (b0 + i < nb) {
            vm |= 1u << i;
            km_a |= static_cast<uint32_t>(keep_a[b0 + i] != 0) << i;
            if (has_b) km_b |= static_cast<uint32_t>(keep_b[b0 + i] != 0) << i;
          }
        }
      }
      const uint32_t am = (vm & ~km_a) | (has_b ? (vm & ~km_b) << 16 : 0u);   // approximated: A 0-15, B 16-31
      const uint32_t ku = km_a | km_b;                                        // union of kept blocks
      const int has_ap = am != 0;
      const int cnt = has_ap + __popc(ku);
      int s_incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int ts = __shfl_up_sync(0xffffffffu, s_incl, o);
        if (lane >= o) s_incl += ts;
      }
      int n = n_base + s_incl - cnt;
      if (gi < ngr) {
        if (has_ap) {
          if (n < kMaxSteps) {
            sm.steps[n].info = static_cast<uint32_t>(gi) | (1u << 31);
            sm.steps[n].mask = am;
          }
          ++n;
        }
        for (uint32_t rest = ku; rest != 0; rest &= rest - 1) {
          const int bj = __ffs(rest) - 1;
          if (n < kMaxSteps) {
            sm.steps[n].info = static_cast<uint32_t>(gi * kGroup + bj);
            sm.steps[n].mask = ((km_a >> bj) & 1u) | (((km_b >> bj) & 1u) << 1);
          }
          ++n;
        }
      }
      n_base += __shfl_sync(0xffffffffu, s_incl, 31);
      any_ap |= __any_sync(0xffffffffu, has_ap != 0);
    }
    if (lane == 0) {
      sm.nsteps = n_base;
      sm.has_ap = any_ap != 0;
    }
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;
  const int nst = sm.nsteps;
  if (nst > kMaxSteps) {   // host checks nb; this only guards the shared list
    if (tid == 0 && atomicCAS(&status->code, 0, 3) == 0) {
      status->where = 99;
      status->block = blockIdx.x + gridDim.x * blockIdx.y;
    }
    __syncthreads();
    if (warp == 1) tmem_dealloc(tbase, 512);
    return;
  }

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 40;\n" ::: "memory");
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int issued = 0;
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_expect_tx(&sm.q_full, kBM * D);
      tma_load_2d(sm.q, &tm_q, 0, g * a.n_pad + row0, &sm.q_full);
      const uint32_t tile_bytes = 2u * BR * D + BR * 4u + 2u * D * 4u;
      for (int j = 0; j < nst; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&sm.kv_empty[s], ((j / kStages) + 1) & 1, abort, status, 1)) break;
        const Step st = sm.steps[j];
        if (step_is_ap(st)) {
          // the first D / 64 atoms of the tile's k_mean and v_mean halves
          const uint8_t* tile = a.ap_tiles + (static_cast<int64_t>(g) * a.ngroups + step_index(st)) * 8192;
          mbar_expect_tx(&sm.kv_full[s], 64u * D);
          bulk_load(sm.k[s], tile, 32 * D, &sm.kv_full[s]);
          bulk_load(sm.v[s], tile + 4096, 32 * D, &sm.kv_full[s]);
        } else {
          const int blk = step_index(st);
          mbar_expect_tx(&sm.kv_full[s], tile_bytes);
          const int krow = g * a.n_pad + blk * BR;
          tma_load_2d(sm.k[s], &tm_k, 0, krow, &sm.kv_full[s]);
          tma_load_2d(sm.v[s], &tm_v, 0, krow, &sm.kv_full[s]);
          bulk_load(sm.ks[s], a.k_scale + static_cast<int64_t>(krow), BR * 4, &sm.kv_full[s]);
          const int64_t vo = (static_cast<int64_t>(g) * nb + blk) * D;
          bulk_load(sm.vs[s], a.v_scale + vo, D * 4, &sm.kv_full[s]);
          bulk_load(sm.mu[s], a.mu + vo, D * 4, &sm.kv_full[s]);
        }
        issued = j + 1;
      }
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
      const uint32_t id_pv = idesc_e4m3(kBM, D, true);
      const uint32_t id_r = idesc_e4m3(kBM, 16, false);
      const uint32_t id_qka = idesc_bf16(kBM, kGroup, false);
      const uint32_t id_pva = idesc_bf16(kBM, 64, true);
      const uint32_t q_addr = smem_u32(sm.q);
      const uint32_t qb_addr = smem_u32(sm.qb[0]);
      const uint32_t ones_addr = smem_u32(sm.ones);
      bool ok = mbar_wait(&sm.q_full, 0, abort, status, 2);
      bool qb_ready = false;
      for (int j = 0; ok && j <= nst; ++j) {
        if (j < nst) {
          const int s = j % kStages, b = j & 1;
          const Step st = sm.steps[j];
          ok = mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 3);
          if (!ok) break;
          if (step_is_ap(st)) {
            // bf16 k_mean tile in stage s; Q in bf16 once per CTA.
            if (!qb_ready) ok = qb_ready = mbar_wait(&sm.qb_full, 0, abort, status, 18);
            if (!ok) break;
            tc_fence_after();
            const uint32_t kmb_addr = smem_u32(sm.k[s]);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              mma_bf16_if(tbase + kColS + b * 128, desc_kmajor(qb_addr + (kk >> 2) * (kBM * 128) + (kk & 3) * 32),
                          desc_kmajor(kmb_addr + (kk >> 2) * (kGroup * 128) + (kk & 3) * 32), id_qka, kk > 0,
                          leader);
          } else {
            tc_fence_after();
            const uint32_t k_addr = smem_u32(sm.k[s]);
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk)
              mma_f8_if(tbase + kColS + b * 128, operand_desc<D>(q_addr + kk * 32), operand_desc<D>(k_addr + kk * 32),
                        id_qk, kk > 0, leader);
          }
          tc_commit_if(&sm.s_full[b], leader);
        }
        if (j >= 1) {
          const int i = j - 1, bi = i & 1, si = i % kStages;
          const Step st = sm.steps[i];
          ok = i >= 1 ? mbar_wait2(&sm.p_full[bi], (i >> 1) & 1, &sm.t_rel, (i - 1) & 1, abort, status, 5)
                      : mbar_wait(&sm.p_full[bi], (i >> 1) & 1, abort, status, 5);
          if (!ok) break;
          tc_fence_after();
          const uint32_t p_t = tbase + kColS + bi * 128;
          if (step_is_ap(st)) {
            const uint32_t vmb_addr = smem_u32(sm.v[si]);
#pragma unroll
            for (int h = 0; h < D / 64; ++h)
              mma_bf16_ts_if(tbase + kColT + bi * 128 + 64 * h, p_t, desc_mnmajor(vmb_addr + 2048 * h), id_pva, 0,
                             leader);
          } else {
            const uint32_t v_addr = smem_u32(sm.v[si]);
#pragma unroll
            for (int kk = 0; kk < NCH; ++kk)
              mma_f8_ts_if(tbase + kColT + bi * 128, p_t + 8 * kk, operand_desc<D>(v_addr + kk * 32 * D), id_pv, kk > 0,
                           leader);
#pragma unroll
            for (int kk = 0; kk < NCH; ++kk)
              mma_f8_ts_if(tbase + kColT + (bi ^ 1) * 128, p_t + 8 * kk, desc_kmajor(ones_addr + kk * 32), id_r,
                           kk > 0, leader);
          }
          tc_commit_if(&sm.t_full[bi], leader);
          tc_commit_if(&sm.kv_empty[si], leader);
        }
      }
      tc_commit_if(&sm.drain, leader);
      const long long t0 = clock64();
      while (!mbar_try_wait(&sm.drain, 0) && clock64() - t0 < kWaitCycles) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ per-tile factors
    const int c2 = tid - 64;   // 0..63
    for (int j = 0; j < nst; ++j) {
      const int s = j % kStages, ring = j % kRing;
      if (!mbar_wait(&sm.kv_full[s], (j / kStages) & 1, abort, status, 13)) break;
      if (j >= kRing && !mbar_wait(&sm.f_free[ring], ((j / kRing) + 1) & 1, abort, status, 14)) break;
      const Step st = sm.steps[j];
      if (!step_is_ap(st)) {
#pragma unroll
        for (int h = 0; h < D / 64; ++h) {
          const int c = c2 + 64 * h;
          const float vsc = sm.vs[s][c];
          sm.cm[ring][0][c] = __fdiv_rn(vsc, 448.0f);
          sm.cm[ring][1][c] = __fmul_rn(sm.mu[s][c], vsc);
        }
#pragma unroll
        for (int kc = c2; kc < BR; kc += 64) sm.ksf[ring][ks_index(kc)] = sm.ks[s][kc];
      }
      warp_arrive(&sm.f_full[ring], lane);
      warp_arrive(&sm.kv_empty[s], lane);
    }
  }
  } else if (warp < 12) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 112;\n" ::: "memory");
    // ------------------------------------------------------------ softmax
    const int sg = (warp >> 2) - 1;
    const int wq = warp & 3, q = lane & 3, rl = lane >> 2;
    const int qsel = wq >> 1;   // query block of this warp's rows (0 = A, 1 = B)
    const int ra = wq * 32 + 16 * sg + rl;
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(wq * 32 + 16 * sg) << 16);
    const int64_t qrow = static_cast<int64_t>(g) * a.n_pad + row0;
    const float qs_a = (row0 + ra < a.n_pad) ? a.q_scale[qrow + ra] : 0.f;
    const float qs_b = (row0 + ra + 8 < a.n_pad) ? a.q_scale[qrow + ra + 8] : 0.f;
    const float qsm_a = __fmul_rn(qs_a, a.sm_scale), qsm_b = __fmul_rn(qs_b, a.sm_scale);
    const float As_a = __fmul_rn(8.0f * kLog2e, qsm_a) * (1.0f / 128.0f);
    const float As_b = __fmul_rn(8.0f * kLog2e, qsm_b) * (1.0f / 128.0f);
    const float Ae_a = __fmul_rn(qsm_a, kLog2e), Ae_b = __fmul_rn(qsm_b, kLog2e);
    bool run = true;
    if (sm.has_ap) {
      // Q codes -> bf16 operand of the proxy MMA (K-major, 128-byte swizzle,
      // D / 64 atoms of 64 elements): each thread converts D / 32 16-byte
      // chunks.  D = 128 reads the TMA-loaded tile; D = 64 reads the codes
      // from global memory (L2), rows past the head's padded end as zeros.
      constexpr int CPR = D / 16;   // 16-byte code chunks per row
      run = mbar_wait(&sm.q_full, 0, abort, status, 19);
      const int t = run ? tid - 128 : kBM * CPR;
      for (int ci = t; ci < kBM * CPR; ci += 256) {
        const int r = ci / CPR, c = ci % CPR;
        uint4 raw = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (D == 128) {
          raw = *reinterpret_cast<const uint4*>(sm.q + sw128(r, 16 * c));
        } else if (row0 + r < a.n_pad) {
          raw = *reinterpret_cast<const uint4*>(a.q8 + (static_cast<int64_t>(g) * a.n_pad + row0 + r) * D + 16 * c);
        }
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t two = (w[i >> 1] >> (16 * (i & 1))) & 0xffffu;
          const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
          o[i] = pack_bf16x2(f.x, f.y);
        }
        uint8_t* dst = sm.qb[c >> 2];
        const int cb = (c & 3) * 32;
        *reinterpret_cast<uint4*>(dst + sw128(r, cb)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(dst + sw128(r, cb + 16)) = make_uint4(o[4], o[5], o[6], o[7]);
      }
      fence_proxy_async_smem();
      if (run) warp_arrive(&sm.qb_full, lane);
    }
    float m_a = -INFINITY, m_b = -INFINITY;
    for (int j = 0; run && j < nst; ++j) {
      const int b = j & 1, ring = j % kRing;
      if (!mbar_wait(&sm.s_full[b], (j >> 1) & 1, abort, status, 7)) break;
      if (!mbar_wait(&sm.f_full[ring], (j / kRing) & 1, abort, status, 8)) break;
      tc_fence_after();
      const Step st = sm.steps[j];
      const uint32_t sb = lane_base + kColS + b * 128;
      float al_a = 1.0f, al_b = 1.0f, ls_a = 0.f, ls_b = 0.f;
      if (step_is_ap(st)) {
        const uint32_t am = (st.mask >> (16 * qsel)) & 0xffffu;
        uint32_t pk[4] = {0u, 0u, 0u, 0u};
        if (am != 0) {
          // Proxies of blocks 2q, 2q+1 (v[0..3]) and 8+2q, 9+2q (v[4..7]).
          float v[8];
          tmem_ld_16x256b_x2(sb, v);
          tmem_ld_wait();
          asm volatile("" : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]),
                       "+f"(v[7]));
          const int blk0 = step_index(st) * kGroup;
          const int bl[4] = {2 * q, 2 * q + 1, 8 + 2 * q, 9 + 2 * q};
          float xa[4], xb[4];
          float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const bool ap = (am >> bl[i]) & 1u;
            const int rr = (i >> 1) * 4 + (i & 1);   // register of row a for block i
            xa[i] = ap ? v[rr] : -INFINITY;
            xb[i] = ap ? v[rr + 2] : -INFINITY;
            mx_a = fmaxf(mx_a, xa[i]);
            mx_b = fmaxf(mx_b, xb[i]);
          }
          mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
          mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
          mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
          mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
          const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
          al_a = (m_a == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m_a, mn_a), Ae_a));
          al_b = (m_b == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m_b, mn_b), Ae_b));
          float pa[4], pb[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const bool ap = (am >> bl[i]) & 1u;
            const float len = ap ? static_cast<float>(min(BR, a.N - (blk0 + bl[i]) * BR)) : 0.f;
            pa[i] = ap ? __fmul_rn(exp2f(__fmul_rn(__fsub_rn(xa[i], mn_a), Ae_a)), len) : 0.f;
            pb[i] = ap ? __fmul_rn(exp2f(__fmul_rn(__fsub_rn(xb[i], mn_b), Ae_b)), len) : 0.f;
            ls_a += pa[i];
            ls_b += pb[i];
          }
          ls_a += __shfl_xor_sync(0xffffffffu, ls_a, 1);
          ls_b += __shfl_xor_sync(0xffffffffu, ls_b, 1);
          ls_a += __shfl_xor_sync(0xffffffffu, ls_a, 2);
          ls_b += __shfl_xor_sync(0xffffffffu, ls_b, 2);
          // A positions 4q..4q+3 = blocks bl[0..3]; column 2q holds 4q, 4q+1.
          pk[0] = pack_bf16x2(pa[0], pa[1]);
          pk[1] = pack_bf16x2(pa[2], pa[3]);
          pk[2] = pack_bf16x2(pb[0], pb[1]);
          pk[3] = pack_bf16x2(pb[2], pb[3]);
          m_a = mn_a;
          m_b = mn_b;
        }
        // 16x256b.x1 register order: (row a, col 2q), (row a, col 2q+1),
        // (row b, col 2q), (row b, col 2q+1).
        const uint32_t st4[4] = {pk[0], pk[1], pk[2], pk[3]};
        tmem_st_16x256b_x1(sb, st4);
        warp_arrive(&sm.f_free[ring], lane);
      } else if (((st.mask >> qsel) & 1u) == 0) {
        // Tile kept only by the other query block: P = 0, alpha = 1.
        uint32_t zero[4 * NCH];
#pragma unroll
        for (int i = 0; i < 4 * NCH; ++i) zero[i] = 0u;
        store_p<NCH>(sb, zero);
        warp_arrive(&sm.f_free[ring], lane);
      } else {
        float x[NCH][16];
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) tmem_ld_16x256b_x4(sb + 32 * ch, x[ch]);
        tmem_ld_wait();
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) reg_fence16(x[ch]);
        const float* kf = sm.ksf[ring] + q * kFStride;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          const float4 k0 = *reinterpret_cast<const float4*>(kf + 8 * ch);
          const float4 k1 = *reinterpret_cast<const float4*>(kf + 8 * ch + 4);
          const float kr[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            mul2(x[ch][4 * r], x[ch][4 * r + 1], kr[2 * r], kr[2 * r + 1]);
            mul2(x[ch][4 * r + 2], x[ch][4 * r + 3], kr[2 * r], kr[2 * r + 1]);
          }
        }
        warp_arrive(&sm.f_free[ring], lane);
        const int valid = a.N - step_index(st) * BR;
        if (valid < BR) {
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
              for (int e = 0; e < 2; ++e)
                if (32 * ch + 8 * r + 2 * q + e >= valid) x[ch][4 * r + e] = x[ch][4 * r + 2 + e] = -1.0e30f;
        }
        float ma0 = m_a, ma1 = -INFINITY, mb0 = m_b, mb1 = -INFINITY;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          ma0 = fmax3(ma0, x[ch][0], x[ch][1]);
          mb0 = fmax3(mb0, x[ch][2], x[ch][3]);
          ma1 = fmax3(ma1, x[ch][4], x[ch][5]);
          mb1 = fmax3(mb1, x[ch][6], x[ch][7]);
          ma0 = fmax3(ma0, x[ch][8], x[ch][9]);
          mb0 = fmax3(mb0, x[ch][10], x[ch][11]);
          ma1 = fmax3(ma1, x[ch][12], x[ch][13]);
          mb1 = fmax3(mb1, x[ch][14], x[ch][15]);
        }
        float mn_a = fmaxf(ma0, ma1), mn_b = fmaxf(mb0, mb1);
        mn_a = fmaxf(mn_a, __shfl_xor_sync(0xffffffffu, mn_a, 1));
        mn_b = fmaxf(mn_b, __shfl_xor_sync(0xffffffffu, mn_b, 1));
        mn_a = fmaxf(mn_a, __shfl_xor_sync(0xffffffffu, mn_a, 2));
        mn_b = fmaxf(mn_b, __shfl_xor_sync(0xffffffffu, mn_b, 2));
        al_a = (m_a == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m_a, mn_a), Ae_a));
        al_b = (m_b == -INFINITY) ? 0.f : exp2f(__fmul_rn(__fsub_rn(m_b, mn_b), Ae_b));
        uint32_t packed[4 * NCH];
        if constexpr (EXPCAST) {
          const float Bs_a = __fmaf_rn(-As_a, mn_a, a.c120 * (1.0f / 128.0f));
          const float Bs_b = __fmaf_rn(-As_b, mn_b, a.c120 * (1.0f / 128.0f));
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
            packed[4 * ch + 0] = expcast4(x[ch][0], x[ch][1], x[ch][4], x[ch][5], As_a, Bs_a);
            packed[4 * ch + 1] = expcast4(x[ch][8], x[ch][9], x[ch][12], x[ch][13], As_a, Bs_a);
            packed[4 * ch + 2] = expcast4(x[ch][2], x[ch][3], x[ch][6], x[ch][7], As_b, Bs_b);
            packed[4 * ch + 3] = expcast4(x[ch][10], x[ch][11], x[ch][14], x[ch][15], As_b, Bs_b);
          }
        } else {
          const float Be_a = __fmaf_rn(-Ae_a, mn_a, 8.807354922057604f);   // log2(448)
          const float Be_b = __fmaf_rn(-Ae_b, mn_b, 8.807354922057604f);
#pragma unroll
          for (int ch = 0; ch < NCH; ++ch) {
            packed[4 * ch + 0] = exp4(x[ch][0], x[ch][1], x[ch][4], x[ch][5], Ae_a, Be_a);
            packed[4 * ch + 1] = exp4(x[ch][8], x[ch][9], x[ch][12], x[ch][13], Ae_a, Be_a);
            packed[4 * ch + 2] = exp4(x[ch][2], x[ch][3], x[ch][6], x[ch][7], Ae_b, Be_b);
            packed[4 * ch + 3] = exp4(x[ch][10], x[ch][11], x[ch][14], x[ch][15], Ae_b, Be_b);
          }
        }
        store_p<NCH>(sb, packed);
        m_a = mn_a;
        m_b = mn_b;
      }
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(&sm.p_full[b], lane);
      if (j >= kRing && !mbar_wait(&sm.a_free[ring], ((j / kRing) + 1) & 1, abort, status, 10)) break;
      if (q < 2) {
        const int slot = ra + 8 * q;
        sm.alpha[ring][slot] = q ? al_b : al_a;
        sm.lsum[ring][slot] = q ? ls_b : ls_a;
      }
      warp_arrive(&sm.a_full[ring], lane);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 248;\n" ::: "memory");
    // ------------------------------------------------------------ correction
    // Thread = query row r = 32 (w%4) + lane (TMEM lane r), O[D] in
    // registers; T read with the 32x32b shape, 64 columns per load batch.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lb = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    float o[D];
#pragma unroll
    for (int c = 0; c < D; ++c) o[c] = 0.f;
    float l = 0.f;
    bool ok = true;
    for (int i = 0; i < nst; ++i) {
      const int ring = i % kRing, tb = i & 1;
      ok = mbar_wait(&sm.t_full[tb], (i >> 1) & 1, abort, status, 11);
      if (!ok) break;
      tc_fence_after();
      const bool ap = step_is_ap(sm.steps[i]);
      const uint32_t tcol = kColT + tb * 128;
      float xa[32], xb[32];
      float rs = 0.f;
      if (!ap) rs = tmem_ld1(lb + kColT + (tb ^ 1) * 128);   // R_i sits in T_{(i+1)&1}
      tmem_ld32(lb + tcol, xa);
      tmem_ld32(lb + tcol + 32, xb);
      tmem_ld_wait();
      asm volatile("" : "+f"(rs));
      reg_fence(xa);
      reg_fence(xb);
      tc_fence_before();
      warp_arrive(&sm.t_rel, lane);
      ok = mbar_wait2(&sm.a_full[ring], (i / kRing) & 1, &sm.f_full[ring], (i / kRing) & 1, abort, status, 12);
      if (!ok) break;
      const float al = sm.alpha[ring][r];
      const float rr = ap ? sm.lsum[ring][r] : rs * (1.0f / 448.0f);
      warp_arrive(&sm.a_free[ring], lane);
      const bool rescale = !__all_sync(0xffffffffu, al == 1.0f);
      const float4* f4 = reinterpret_cast<const float4*>(sm.cm[ring][0]);
      const float4* g4 = reinterpret_cast<const float4*>(sm.cm[ring][1]);
#pragma unroll
      for (int half = 0; half < D / 64; ++half) {
        if (half == 1) {
          tmem_ld32(lb + tcol + 64, xa);
          tmem_ld32(lb + tcol + 96, xb);
          tmem_ld_wait();
          reg_fence(xa);
          reg_fence(xb);
        }
        if (ap) {
          // acc = alpha acc + T (values already in output units)
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float* src = (q < 8) ? xa + 4 * q : xb + 4 * (q - 8);
            float* oc = o + 64 * half + 4 * q;
            if (rescale) {
              mul2(oc[0], oc[1], al, al);
              mul2(oc[2], oc[3], al, al);
            }
            add2(oc[0], oc[1], src[0], src[1]);
            add2(oc[2], oc[3], src[2], src[3]);
          }
        } else {
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
      }
      warp_arrive(&sm.f_free[ring], lane);
      l = __fadd_rn(__fmul_rn(l, al), rr);
    }
    if (ok && !*abort) {
      constexpr int ES = (ODT == VCATTN_DTYPE_F32) ? 4 : 2;
      constexpr int RS = D * ES + 16;
      using SM = SpSmem<BR, D>;
      static_assert(kBM * RS <= static_cast<int>(sizeof(SM::q) + sizeof(SM::k) + sizeof(SM::v)),
                    "output staging must fit in the operand buffers");
      uint8_t* stage = sm.q + wq * 32 * RS;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 16 / ES) {
        uint4 w;
#pragma unroll
        for (int e = 0; e < 16 / ES; e += 2)
          stage2<ODT>(reinterpret_cast<uint8_t*>(&w) + e * ES, __fdiv_rn(o[c0 + e], l), __fdiv_rn(o[c0 + e + 1], l));
        *reinterpret_cast<uint4*>(stage + lane * RS + c0 * ES) = w;
      }
      __syncwarp();
      constexpr int CPR = D * ES / 16;
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

// (rows, D) E4M3 codes; D = 128: 128-byte swizzle, D = 64: 64-byte swizzle.
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

template <int BR, int D, bool EC, int ODT>
cudaError_t launch_sp(const AttnParams& p, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  const uint64_t rows = static_cast<uint64_t>(p.B) * p.H * p.n_pad;
  if (!make_map(&mq, p.q8, rows, kBM, D) || !make_map(&mk, p.k8, rows, BR, D) || !make_map(&mv, p.v8, rows, BR, D))
    return cudaErrorInvalidValue;
  SpArgs a{};
  a.q8 = p.q8;
  a.q_scale = p.q_scale; a.k_scale = p.k_scale; a.v_scale = p.v_scale; a.mu = p.mu;
  a.ap_tiles = p.ap_tiles; a.keep = p.keep;
  a.H = p.H; a.N = p.N; a.n_pad = p.n_pad; a.nb = p.n_pad / BR; a.nqb = p.n_pad / kQBlock;
  a.ngroups = (a.nb + kGroup - 1) / kGroup;
  a.sm_scale = p.sm_scale;
  a.c120 = static_cast<float>(64.0 + 56.0 + p.beta);
  a.out = p.out; a.osb = p.osb; a.osh = p.osh; a.osn = p.osn;
  const size_t smem = sizeof(SpSmem<BR, D>) + 1024;
  auto k = attn_tc_sparse_kernel<BR, D, EC, ODT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid((p.n_pad + kBM - 1) / kBM, p.B * p.H);
  k<<<grid, kThreads, smem, st>>>(mq, mk, mv, a);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, k);
    snprintf(g_sp_diag, sizeof(g_sp_diag), "regs=%d dynSmem=%zu maxDynSmem=%d local=%zu", fa.numRegs, smem,
             fa.maxDynamicSharedSizeBytes, fa.localSizeBytes);
  }
  return e;
}

template <int BR, int D>
cudaError_t launch_sp_shape(const AttnParams& p, cudaStream_t st) {
  const bool ec = (p.flags & VCATTN_EXPCAST) != 0;
  switch (p.out_dtype) {
    case VCATTN_DTYPE_BF16:
      return ec ? launch_sp<BR, D, true, VCATTN_DTYPE_BF16>(p, st) : launch_sp<BR, D, false, VCATTN_DTYPE_BF16>(p, st);
    case VCATTN_DTYPE_F16:
      return ec ? launch_sp<BR, D, true, VCATTN_DTYPE_F16>(p, st) : launch_sp<BR, D, false, VCATTN_DTYPE_F16>(p, st);
    default:
      return ec ? launch_sp<BR, D, true, VCATTN_DTYPE_F32>(p, st) : launch_sp<BR, D, false, VCATTN_DTYPE_F32>(p, st);
  }
}

}  // namespace

bool attn_sparse_tc_supported(const AttnParams& p) {
  const bool br_ok = p.block_rows == 128 || p.block_rows == 64;
  return (p.D == 128 || p.D == 64) && br_ok && p.q_block == kQBlock && p.group == kGroup &&
         p.n_pad % p.block_rows == 0 &&
         p.n_pad / p.block_rows + (p.n_pad / p.block_rows + kGroup - 1) / kGroup <= kMaxSteps;
}

cudaError_t launch_attn_sparse_tc(const AttnParams& p, cudaStream_t st) {
  if (!attn_sparse_tc_supported(p)) return cudaErrorNotSupported;
  if (p.block_rows == 128) return p.D == 128 ? launch_sp_shape<128, 128>(p, st) : launch_sp_shape<128, 64>(p, st);
  return p.D == 128 ? launch_sp_shape<64, 128>(p, st) : launch_sp_shape<64, 64>(p, st);
}

const char* attn_sparse_tc_diag() { return g_sp_diag; }

cudaError_t attn_sparse_tc_status(int* code, int* where, int* block, bool reset) {
  tc::DevStatus s{};
  cudaError_t e = cudaMemcpyFromSymbol(&s, g_attn_sparse_tc_status, sizeof(s));
  if (e != cudaSuccess) return e;
  *code = s.code;
  *where = s.where;
  *block = s.block;
  if (reset) {
    tc::DevStatus z{};
    e = cudaMemcpyToSymbol(g_attn_sparse_tc_status, &z, sizeof(z));
  }
  return e;
}

}  // namespace vcattn
