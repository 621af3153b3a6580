// Nearest-centroid assignment of the V-Smooth k-means (grouping.py:86-100)
// on the 5th-generation tensor cores, with labels identical to the
// sequential-FMA definition of the CUDA-core assign_kernel.
//
// Definition (fixed by the restatement the labels are checked against):
//   acc_c = fp32 FMA chain over channels 0..D-1 of v . c   (bf16 products exact)
//   sim_c = fp32(bf16(acc_c) * 2 - |c|^2)                  (|c|^2 sequential fp32)
//   label = first argmax_c sim_c
//
// The tensor cores give every dot product a_c in another summation order.
// Both orders approximate the real dot d_c to within gamma * sum_j |v_j c_j|
// <= 2^-13 |v| |c| (128 fp32 additions, Cauchy-Schwarz); E = 2^-12 |v| cmax
// bounds |a_c - acc_c| with a factor 2 to spare for the tensor core's internal
// adder.  With s_c = fp32(2 a_c - |c|^2),
//   |s_c - sim_c| <= 2E + ulp_bf16(|acc_c|) + 2 ulp_fp32(|s_c|) =: Delta,
// so every index whose exact sim can reach the maximum has s_c >= M - 2 Delta
// (M = max_c s_c).  Those candidates are resolved exactly: when a_c is more
// than E away from both bf16 rounding boundaries around it, bf16(acc_c) =
// bf16(a_c) and sim_c follows without recomputation; otherwise the token's
// dot with that centroid is recomputed as the sequential FMA chain from the
// bf16 rows staged in shared memory.  The recomputations are queued per
// token (a bit per column of the 32-column block) and run one per lane per
// round, so a warp pays one sequential chain per round rather than one per
// column any of its tokens flagged.  The best is the highest sim, ties going
// to the lower index (numpy's / torch's first-argmax rule), which does not
// depend on the order candidates are visited in.
//
// One CTA = 128 tokens (MMA M) of one (batch, head); warps 0-15 are the
// epilogue (thread = token = TMEM lane, four warps per row splitting the
// columns), warp 16 loads (TMA, 128-byte swizzle)
// and issues tcgen05.mma kind::f16 (bf16 x bf16 -> f32) over centroid chunks
// of up to 256 (MMA N), 512 centroids per TMEM pass.  Every wait is bounded.
#include <cuda.h>
#include <cstdlib>
#include <mutex>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace vcattn {

__device__ tc::DevStatus g_kmeans_tc_status;

namespace {

using namespace tc;

constexpr int kTok = 128;       // tokens per CTA
constexpr int kChunkC = 256;    // centroids per MMA
constexpr int kGroupC = 512;    // centroids per TMEM pass
constexpr int kMaxParts = 4;    // column parts per row (epilogue warps = 4 x parts)
constexpr int kHalfA = kTok * 128;       // bytes of one 64-channel half of the token tile
constexpr int kHalfB = kChunkC * 128;    // bytes of one 64-channel half of a centroid chunk

struct alignas(16) AsCtl {   // 16-byte size: the -|c|^2 table after it is read as float4
  alignas(8) uint64_t a_full;
  alignas(8) uint64_t b_full[2];
  alignas(8) uint64_t acc_full[2];
  alignas(8) uint64_t grp_done;
  alignas(8) uint64_t drain;
  alignas(8) uint64_t xa, xb;   // epilogue exchanges: row maxima, best candidates
  uint32_t tmem_base;
  int abort;
  int c2max_bits;
  int pad_;
  float mx[kMaxParts][kTok];   // per column part: row maximum of the scores
  float bs[kMaxParts][kTok];   // per column part: best exact sim and its index
  int bi[kMaxParts][kTok];
};

struct AssignArgs {
  const float* c2;          // (G, k) |c|^2, sequential fp32
  int H, N, k, kbox;        // kbox: centroid rows per TMA box (min(256, k rounded up to 16))
  int32_t* labels;
  const int32_t* key_offset;
  int nkeys, nchunks;
  int32_t* counts;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mma_bf16_ss_if(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate, uint32_t leader) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.ne.b32 e, %5, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(leader)
      : "memory");
}
__host__ __device__ constexpr uint32_t idesc_bf16_kk(int M, int N) {
  // f32 accumulate, A = B = bf16, both K-major
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// Channels 8c .. 8c+7 (c = 0..15) of row r of a 128-byte-swizzled K-major
// tile whose two 64-channel halves are `half_bytes` apart: the 16-byte chunk
// c % 8 of the row sits at chunk position (c % 8) ^ (r % 8).
__device__ __forceinline__ uint4 swz_chunk(const uint8_t* tile, int half_bytes, int r, int c) {
  const int pos = (c & 7) ^ (r & 7);
  return *reinterpret_cast<const uint4*>(tile + (c >> 3) * half_bytes + r * 128 + (pos << 4));
}

// acc + a * b for the low (or high) bf16 halves of two words: the mixed
// precision FMA rounds the exact a * b + acc once to fp32, the same result as
// the fp32 FMA of the widened operands (bf16 values are exact in fp32).
__device__ __forceinline__ float fma_lo(uint32_t a, uint32_t b, float acc) {
  float d;
  asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\tmov.b32 {a0, a1}, %1;\n\tmov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.bf16 %0, a0, b0, %3;\n\t}\n" : "=f"(d) : "r"(a), "r"(b), "f"(acc));
  return d;
}
__device__ __forceinline__ float fma_hi(uint32_t a, uint32_t b, float acc) {
  float d;
  asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\tmov.b32 {a0, a1}, %1;\n\tmov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.bf16 %0, a1, b1, %3;\n\t}\n" : "=f"(d) : "r"(a), "r"(b), "f"(acc));
  return d;
}

// Sequential fp32 FMA chain of a token row and a centroid row (both bf16 in
// swizzled shared memory), channels in increasing order.
__device__ __noinline__ float exact_dot(const uint8_t* ta, int r, const uint8_t* tb, int cr) {
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const uint4 a = swz_chunk(ta, kHalfA, r, c);
    const uint4 b = swz_chunk(tb, kHalfB, cr, c);
    acc = fma_lo(a.x, b.x, acc);
    acc = fma_hi(a.x, b.x, acc);
    acc = fma_lo(a.y, b.y, acc);
    acc = fma_hi(a.y, b.y, acc);
    acc = fma_lo(a.z, b.z, acc);
    acc = fma_hi(a.z, b.z, acc);
    acc = fma_lo(a.w, b.w, acc);
    acc = fma_hi(a.w, b.w, acc);
  }
  return acc;
}

// bf16(acc) of a candidate from its tensor-core dot `a`: equal to bf16(a)
// when a lies more than E inside the rounding interval of bf16(a) (returns
// true and sets *bf); otherwise the dot must be recomputed in the defining
// order.
__device__ __forceinline__ bool cand_certified(float a, float E, float* bf) {
  *bf = bf16_round(a);
  const uint32_t ab = __float_as_uint(fabsf(*bf));
  if (ab >= (8u << 23) && ab < 0x7f800000u) {
    const float ulp = __uint_as_float((ab & 0x7f800000u) - (7u << 23));   // bf16 spacing above |bf|
    const float dn = (ab & 0x007f0000u) ? ulp : 0.5f * ulp;              // spacing below |bf|
    const float d = fabsf(a) - fabsf(*bf);                               // exact: same binade or adjacent
    return (d + E < 0.5f * ulp) && (E - d < 0.5f * dn);
  }
  return false;
}

// First-argmax update: a higher sim wins, an equal sim wins only with a
// lower index, so candidates may be visited in any order.
__device__ __forceinline__ void take_best(float sim, int idx, float& bsim, int& bidx) {
  if (sim > bsim || (sim == bsim && idx < bidx)) {
    bsim = sim;
    bidx = idx;
  }
}

template <int NCH, int EW>
__global__ void __launch_bounds__(32 * (EW + 1), 1)
    assign_tc_kernel(const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_c,
                     const AssignArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* sa = smem_raw + pad;                     // token tile: 2 halves x 16 KB
  uint8_t* sb = sa + 2 * kHalfA;                    // centroid chunks: NCH x 2 halves x 32 KB
  AsCtl& ctl = *reinterpret_cast<AsCtl*>(sb + NCH * 2 * kHalfB);
  float* nc2 = reinterpret_cast<float*>(&ctl + 1);  // -|c|^2 of the head's k centroids
  DevStatus* status = &g_kmeans_tc_status;
  constexpr int kEpiWarps = EW;             // 4 row quadrants x P column parts
  constexpr int P = EW / 4;
  constexpr int kThreadsA = 32 * (EW + 1);   // + 1 load / MMA warp
  static_assert(P >= 1 && P <= kMaxParts && (NCH * 8) % P == 0, "parts must split the blocks");

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.y;
  const int row0 = blockIdx.x * kTok;
  const int k = a.k;
  const int ngroups = (k + kGroupC - 1) / kGroupC;

  if (tid == 0) {
    ctl.abort = 0;
    ctl.c2max_bits = 0;
    mbar_init(&ctl.a_full, 1);
    for (int c = 0; c < 2; ++c) {
      mbar_init(&ctl.b_full[c], 1);
      mbar_init(&ctl.acc_full[c], 1);
    }
    mbar_init(&ctl.grp_done, kEpiWarps);
    mbar_init(&ctl.xa, kEpiWarps);
    mbar_init(&ctl.xb, kEpiWarps);
    mbar_init(&ctl.drain, 1);
    fence_mbar_init();
  }
  if (warp == kEpiWarps) {
    tmem_alloc(&ctl.tmem_base, 256 * NCH);
    tmem_relinquish();
  }
  __syncthreads();
  float m2 = 0.f;
  for (int i = tid; i < k; i += kThreadsA) {
    const float c2 = a.c2[static_cast<int64_t>(g) * k + i];
    nc2[i] = -c2;
    m2 = fmaxf(m2, c2);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
  if (lane == 0) atomicMax(&ctl.c2max_bits, __float_as_int(m2));   // non-negative floats order as ints
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ctl.tmem_base;
  volatile int* abort = &ctl.abort;

  if (warp == kEpiWarps) {
    // ------------------------------------------------------------ loads + MMA
    const uint32_t leader = elect_one();
    const int b_ = g / a.H, h_ = g % a.H;
    if (leader) {
      prefetch_tmap(&tm_v);
      prefetch_tmap(&tm_c);
      mbar_expect_tx(&ctl.a_full, 2 * kHalfA);
      tma_load_4d(sa, &tm_v, 0, row0, h_, b_, &ctl.a_full);
      tma_load_4d(sa + kHalfA, &tm_v, 64, row0, h_, b_, &ctl.a_full);
    }
    const uint32_t a_addr = smem_u32(sa), b_addr = smem_u32(sb);
    bool ok = true;
    for (int gi = 0; gi < ngroups && ok; ++gi) {
      // The previous pass's epilogue has read TMEM and the centroid rows.
      if (gi > 0 && !(ok = mbar_wait(&ctl.grp_done, (gi - 1) & 1, abort, status, 1))) break;
      const int ncg = min(kGroupC, k - gi * kGroupC);
      const int nchk = (ncg + kChunkC - 1) / kChunkC;
      if (leader) {
        for (int c = 0; c < nchk; ++c) {
          mbar_expect_tx(&ctl.b_full[c], 2u * a.kbox * 128u);
          const int y = gi * kGroupC + c * kChunkC;
          tma_load_3d(sb + c * 2 * kHalfB, &tm_c, 0, y, g, &ctl.b_full[c]);
          tma_load_3d(sb + c * 2 * kHalfB + kHalfB, &tm_c, 64, y, g, &ctl.b_full[c]);
        }
      }
      __syncwarp();
      if (!(ok = mbar_wait(&ctl.a_full, 0, abort, status, 2))) break;
      for (int c = 0; c < nchk; ++c) {
        if (!(ok = mbar_wait(&ctl.b_full[c], gi & 1, abort, status, 3))) break;
        tc_fence_after();
        const int n = min(kChunkC, ((ncg - c * kChunkC) + 15) & ~15);
        const uint32_t idesc = idesc_bf16_kk(kTok, n);
        const uint32_t bc = b_addr + c * 2 * kHalfB;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ss_if(tbase + c * kChunkC, desc_kmajor(a_addr + h * kHalfA + kk * 32),
                           desc_kmajor(bc + h * kHalfB + kk * 32), idesc, (h | kk) != 0, leader);
        tc_commit_if(&ctl.acc_full[c], leader);
      }
    }
    // Every MMA issued must finish before TMEM is released.
    tc_commit_if(&ctl.drain, leader);
    const long long t0 = clock64();
    while (!mbar_try_wait(&ctl.drain, 0) && clock64() - t0 < kWaitCycles) {
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w reads TMEM lane quadrant qd = w % 4 (rows 32 qd .. +31) and
    // column part pt = w / 4 of each pass (BPP blocks of 32 columns, all in
    // chunk cpt).  With several parts, their row maxima and best candidates
    // are exchanged through shared memory and merged in column order.
    constexpr int BPP = NCH * 8 / P;
    const int qd = warp & 3, pt = warp >> 2;
    const int cpt = (pt * BPP) >> 3;
    const int r = qd * 32 + lane;
    const int t = row0 + r;
    const bool live = t < a.N;
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(qd * 32) << 16);
    const float c2max = __int_as_float(ctl.c2max_bits);
    bool ok = mbar_wait(&ctl.a_full, 0, abort, status, 4);
    float vv = 0.f, vw = 0.f;
    if (ok) {
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 a4 = swz_chunk(sa, kHalfA, r, c);
        vv = fma_lo(a4.x, a4.x, vv);
        vw = fma_hi(a4.x, a4.x, vw);
        vv = fma_lo(a4.y, a4.y, vv);
        vw = fma_hi(a4.y, a4.y, vw);
        vv = fma_lo(a4.z, a4.z, vv);
        vw = fma_hi(a4.z, a4.z, vw);
        vv = fma_lo(a4.w, a4.w, vv);
        vw = fma_hi(a4.w, a4.w, vw);
      }
      vv += vw;
    }
    // Upper bounds (fp32 rounding of the norms covered by the 1 + 2^-10 factors).
    const float S = sqrtf(vv) * sqrtf(c2max) * (1.0f + 0x1p-10f);
    const float E = S * 0x1p-12f;
    const float Delta = (S * (0x1p-11f + 0x1p-7f + 0x1p-19f) + c2max * 0x1p-22f) * 1.0625f;
    float best_sim = -INFINITY;   // running result, kept by the part-0 warps
    int best = 0;
    for (int gi = 0; ok && gi < ngroups; ++gi) {
      const int ncg = min(kGroupC, k - gi * kGroupC);
      const int ncc = cpt * kChunkC < ncg ? min(kChunkC, ncg - cpt * kChunkC) : 0;
      if (ncc > 0) {
        if (!(ok = mbar_wait(&ctl.acc_full[cpt], gi & 1, abort, status, 5))) break;
        tc_fence_after();
      }
      float gm[BPP];
      float Mp = -INFINITY;
#pragma unroll
      for (int j = 0; j < BPP; ++j) {
        const int blk = (pt * BPP + j) & 7;
        gm[j] = -INFINITY;
        if (32 * blk < ncc) {
          float x[32];
          tmem_ld32(lane_base + cpt * kChunkC + 32 * blk, x);
          tmem_ld_wait_regs(x);
          const int col0 = gi * kGroupC + cpt * kChunkC + 32 * blk;
          const int nv = min(32, k - col0);
          float m0 = -INFINITY, m1 = -INFINITY;
          if (nv == 32) {
            const float4* nc4 = reinterpret_cast<const float4*>(nc2 + col0);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 n4 = nc4[q];
              const float s0 = __fmaf_rn(x[4 * q], 2.0f, n4.x), s1 = __fmaf_rn(x[4 * q + 1], 2.0f, n4.y);
              const float s2 = __fmaf_rn(x[4 * q + 2], 2.0f, n4.z), s3 = __fmaf_rn(x[4 * q + 3], 2.0f, n4.w);
              m0 = fmaxf(m0, fmaxf(s0, s1));
              m1 = fmaxf(m1, fmaxf(s2, s3));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nv) m0 = fmaxf(m0, __fmaf_rn(x[i], 2.0f, nc2[col0 + i]));
          }
          gm[j] = fmaxf(m0, m1);
          Mp = fmaxf(Mp, gm[j]);
        }
      }
      float M = Mp;
      if constexpr (P > 1) {
        ctl.mx[pt][r] = Mp;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl.xa);
        if (!(ok = mbar_wait(&ctl.xa, gi & 1, abort, status, 6))) break;
#pragma unroll
        for (int q = 0; q < P; ++q) M = fmaxf(M, ctl.mx[q][r]);
      }
      const float T = M - 2.0f * Delta;
      // Candidates: every index whose score is within 2 Delta of the maximum.
      // The warp reloads each 32-column block any of its lanes flagged.
      uint32_t flags = 0;
#pragma unroll
      for (int j = 0; j < BPP; ++j) flags |= (gm[j] >= T ? 1u : 0u) << j;
      uint32_t wflags = __reduce_or_sync(0xffffffffu, flags);
      float bsim = -INFINITY;
      int bidx = 0;
#pragma unroll 1
      while (wflags != 0u) {
        const int j = __ffs(wflags) - 1;
        wflags &= wflags - 1u;
        const int blk = (pt * BPP + j) & 7;
        float x[32];
        tmem_ld32(lane_base + cpt * kChunkC + 32 * blk, x);
        tmem_ld_wait_regs(x);
        const int col0 = gi * kGroupC + cpt * kChunkC + 32 * blk;
        const int nv = min(32, k - col0);
        const uint8_t* tb = sb + cpt * 2 * kHalfB;
        // This token's candidates of the block as a bitmask (no branches),
        // then the columns some lane flagged: certified candidates are taken
        // now, the others queue in `pend`.
        uint32_t cm = 0;
        if ((flags >> j) & 1u) {
          if (nv == 32) {
            const float4* nc4 = reinterpret_cast<const float4*>(nc2 + col0);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 n4 = nc4[q];
              cm |= (__fmaf_rn(x[4 * q], 2.0f, n4.x) >= T ? 1u : 0u) << (4 * q);
              cm |= (__fmaf_rn(x[4 * q + 1], 2.0f, n4.y) >= T ? 1u : 0u) << (4 * q + 1);
              cm |= (__fmaf_rn(x[4 * q + 2], 2.0f, n4.z) >= T ? 1u : 0u) << (4 * q + 2);
              cm |= (__fmaf_rn(x[4 * q + 3], 2.0f, n4.w) >= T ? 1u : 0u) << (4 * q + 3);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nv && __fmaf_rn(x[i], 2.0f, nc2[col0 + i]) >= T) cm |= 1u << i;
          }
        }
        const uint32_t wcm = __reduce_or_sync(0xffffffffu, cm);
        uint32_t pend = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if ((wcm >> i) & 1u) {                 // warp-uniform
            if ((cm >> i) & 1u) {
              float bf;
              if (cand_certified(x[i], E, &bf))
                take_best(__fadd_rn(__fmul_rn(bf, 2.0f), nc2[col0 + i]), col0 + i, bsim, bidx);
              else
                pend |= 1u << i;
            }
          }
        }
        // Queued candidates: each lane recomputes its next one as the
        // sequential FMA chain, all lanes in parallel, one chain per round.
        while (__any_sync(0xffffffffu, pend != 0u)) {
          if (pend != 0u) {
            const int i = __ffs(pend) - 1;
            pend &= pend - 1u;
            const float acc = exact_dot(sa, r, tb, 32 * blk + i);
            take_best(__fadd_rn(__fmul_rn(bf16_round(acc), 2.0f), nc2[col0 + i]), col0 + i, bsim, bidx);
          }
        }
      }
      if constexpr (P > 1) {
        ctl.bs[pt][r] = bsim;
        ctl.bi[pt][r] = bidx;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (P > 1) mbar_arrive(&ctl.xb);
        if (gi + 1 < ngroups) mbar_arrive(&ctl.grp_done);   // TMEM and the centroid rows are free
      }
      if constexpr (P > 1) {
        if (!(ok = mbar_wait(&ctl.xb, gi & 1, abort, status, 7))) break;
        if (pt == 0) {
          // parts in increasing column order; a later part wins only when strictly greater
#pragma unroll
          for (int q = 0; q < P; ++q) {
            if (ctl.bs[q][r] > best_sim) {
              best_sim = ctl.bs[q][r];
              best = ctl.bi[q][r];
            }
          }
        }
      } else if (bsim > best_sim) {
        best_sim = bsim;
        best = bidx;
      }
    }
    // Label and the counting-sort histogram of the stable sort (one 32-token
    // chunk per warp), as in assign_kernel.
    if (pt == 0) {
      const unsigned live_mask = __ballot_sync(0xffffffffu, live);
      if (ok && !*abort && live) {
        a.labels[static_cast<int64_t>(g) * a.N + t] = best;
        const int key = best + (a.key_offset ? a.key_offset[t] : 0);
        const unsigned same = __match_any_sync(live_mask, key);
        if ((same & ((1u << lane) - 1u)) == 0u && key >= 0 && key < a.nkeys)
          a.counts[(static_cast<int64_t>(g) * a.nkeys + key) * a.nchunks + t / 32] = __popc(same);
      }
    }
  }
  __syncthreads();
  if (warp == kEpiWarps) tmem_dealloc(tbase, 256 * NCH);
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

template <int NCH>
size_t assign_smem_bytes(int k) {   // same for every epilogue width
  return 1024 + 2 * kHalfA + static_cast<size_t>(NCH) * 2 * kHalfB + sizeof(AsCtl) + ((static_cast<size_t>(k) * 4 + 15) & ~static_cast<size_t>(15));
}

template <int NCH, int EW>
cudaError_t run_assign(const CUtensorMap& mv, const CUtensorMap& mc, const AssignArgs& a, int G, cudaStream_t st) {
  const size_t smem = assign_smem_bytes<NCH>(a.k);
  auto kern = assign_tc_kernel<NCH, EW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid((a.N + kTok - 1) / kTok, G);
  kern<<<grid, 32 * (EW + 1), smem, st>>>(mv, mc, a);
  return cudaGetLastError();
}

}  // namespace

bool assign_tc_supported(const KMeansParams& p) {
  if (p.D != 128 || p.dtype != VCATTN_DTYPE_BF16 || p.k < 1 || p.k > 4096) return false;
  const char* env = std::getenv("VCATTN_KMEANS_SIMT");   // force the CUDA-core assign (parity tests)
  if (env && env[0] == '1') return false;
  return encode_fn() != nullptr;
}

bool assign_tc_maps(const KMeansParams& p, const uint16_t* cb16, void* maps) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  CUtensorMap* mv = static_cast<CUtensorMap*>(maps);
  CUtensorMap* mc = mv + 1;
  const vcattn_bhnd& v = *p.v;
  cuuint64_t vdims[4] = {128, static_cast<cuuint64_t>(p.N), static_cast<cuuint64_t>(p.H),
                         static_cast<cuuint64_t>(p.B)};
  cuuint64_t vstr[3] = {static_cast<cuuint64_t>(v.sn) * 2, static_cast<cuuint64_t>(v.sh) * 2,
                        static_cast<cuuint64_t>(v.sb) * 2};
  cuuint32_t vbox[4] = {64, kTok, 1, 1};
  cuuint32_t es4[4] = {1, 1, 1, 1};
  if (fn(mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(v.data), vdims, vstr, vbox, es4,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  const int G = p.B * p.H;
  const cuuint32_t kbox = static_cast<cuuint32_t>(p.k >= kChunkC ? kChunkC : ((p.k + 15) & ~15));
  cuuint64_t cdims[3] = {128, static_cast<cuuint64_t>(p.k), static_cast<cuuint64_t>(G)};
  cuuint64_t cstr[2] = {256, static_cast<cuuint64_t>(p.k) * 256};
  cuuint32_t cbox[3] = {64, kbox, 1};
  cuuint32_t es3[3] = {1, 1, 1};
  return fn(mc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(cb16), cdims, cstr, cbox, es3,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_assign_tc(const KMeansParams& p, const void* maps, const float* c2, int32_t* labels,
                             const int32_t* key_offset, int nkeys, int nchunks, int32_t* counts, cudaStream_t st) {
  const CUtensorMap* mv = static_cast<const CUtensorMap*>(maps);
  AssignArgs a{};
  a.c2 = c2;
  a.H = p.H;
  a.N = p.N;
  a.k = p.k;
  a.kbox = p.k >= kChunkC ? kChunkC : ((p.k + 15) & ~15);
  a.labels = labels;
  a.key_offset = key_offset;
  a.nkeys = nkeys;
  a.nchunks = nchunks;
  a.counts = counts;
  const int G = p.B * p.H;
  // Epilogue width by k: 16 warps for two chunks per pass (one CTA per SM),
  // 8 or 4 for one chunk (two CTAs per SM overlap their loads and epilogues).
  if (p.k > kChunkC) return run_assign<2, 16>(mv[0], mv[1], a, G, st);
  if (p.k > 128) return run_assign<1, 8>(mv[0], mv[1], a, G, st);
  return run_assign<1, 4>(mv[0], mv[1], a, G, st);
}

cudaError_t kmeans_tc_status(int* code, int* where, int* block, bool reset) {
  tc::DevStatus s{};
  cudaError_t e = cudaMemcpyFromSymbol(&s, g_kmeans_tc_status, sizeof(s));
  if (e != cudaSuccess) return e;
  *code = s.code;
  *where = s.where;
  *block = s.block;
  if (reset) {
    tc::DevStatus z{};
    e = cudaMemcpyToSymbol(g_kmeans_tc_status, &z, sizeof(z));
  }
  return e;
}

}  // namespace vcattn
