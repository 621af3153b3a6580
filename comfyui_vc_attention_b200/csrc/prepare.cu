// Prepare kernels: permute, Hadamard-rotate, smooth and quantise Q/K/V into
// the Prepared layout of triton_attn.py:504-579, plus the routing statistics
// of triton_attn.py:716-735.
//
// All kernels are HBM-bound.  One warp owns one token row (D = 128: four
// elements per lane; D = 64: sixteen lanes per row), so every load and store
// of a row is a single coalesced transaction and the Hadamard butterfly runs
// in registers with warp shuffles.  Means are accumulated in float64 and
// rounded once, which makes them independent of the reduction order.
#include "kernels.cuh"

namespace vcattn {

// ---------------------------------------------------------------------------
// Row access helpers.  A warp handles one row; lane l owns 4 consecutive
// elements (D = 128) or, for D = 64, lanes 0..15 own row r and lanes 16..31
// row r+1 of a row pair.
// ---------------------------------------------------------------------------
template <int D> struct RowMap;
template <> struct RowMap<128> {
  static constexpr int kRowsPerWarp = 1;
  static __device__ __forceinline__ int sub(int lane) { return 0; }
  static __device__ __forceinline__ int col(int lane) { return lane * 4; }
  static __device__ __forceinline__ float amax(float v) { return warp_max(v); }
  static __device__ __forceinline__ void fwht(float v[4], int lane) { fwht128_warp(v, lane); }
};
template <> struct RowMap<64> {
  static constexpr int kRowsPerWarp = 2;
  static __device__ __forceinline__ int sub(int lane) { return lane >> 4; }
  static __device__ __forceinline__ int col(int lane) { return (lane & 15) * 4; }
  static __device__ __forceinline__ float amax(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
  }
  static __device__ __forceinline__ void fwht(float v[4], int lane) { fwht64_halfwarp(v, lane); }
};

__device__ __forceinline__ int source_row(const int32_t* perm, int perm_rows, int g, int n, int t) {
  if (perm == nullptr) return t;
  const int pr = (perm_rows == 1) ? 0 : g;
  return perm[static_cast<int64_t>(pr) * n + t];
}

// ---------------------------------------------------------------------------
// K token mean (smooth_k, triton_attn.py:545-546): partial float64 sums of the
// rotated K per (head, chunk of kChunkRows tokens).  The mean is permutation
// invariant, so it is taken over the unpermuted rows.
// ---------------------------------------------------------------------------
constexpr int kChunkRows = 256;

// Fixed-order reduction of per-lane float64 accumulators: lane l of warp w
// holds channels col(l)..col(l)+3; thread d < D sums warps 0..7 and, for
// D = 64, both half-warps, always in the same order.
template <int D>
__device__ __forceinline__ double reduce_lanes(double (*red)[32][4], int nwarps, int d) {
  const int l = d / 4, i = d % 4;
  double tot = 0.0;
  for (int w = 0; w < nwarps; ++w) {
    tot += red[w][l][i];
    if (D == 64) tot += red[w][l + 16][i];
  }
  return tot;
}

template <int DT, int D>
__global__ void __launch_bounds__(256, 3) kmean_partial_kernel(
    vcattn_bhnd k, int H, int N, int flags, double* __restrict__ partial) {
  using RM = RowMap<D>;
  __shared__ double red[8][32][4];
  const int g = blockIdx.y, chunk = blockIdx.x;
  const int b = g / H, h = g % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  const int t0 = chunk * kChunkRows;
  const int t1 = min(N, t0 + kChunkRows);
  // Rows advance in warp-uniform steps so every lane reaches the shuffles;
  // kBatch rows are loaded before any is used (memory-level parallelism).
  constexpr int kBatch = 8;
  constexpr int kStep = 8 * RM::kRowsPerWarp;
  for (int base = t0 + warp * RM::kRowsPerWarp; base < t1; base += kBatch * kStep) {
    float v[kBatch][4];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int t = base + u * kStep + RM::sub(lane);
      v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0.f;
      if (t < t1) {
        const int64_t off = b * k.sb + h * k.sh + static_cast<int64_t>(t) * k.sn + RM::col(lane);
        const float4 x = load4<DT>(k.data, off);
        v[u][0] = x.x; v[u][1] = x.y; v[u][2] = x.z; v[u][3] = x.w;
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (flags & VCATTN_HADAMARD) RM::fwht(v[u], lane);
      if (base + u * kStep + RM::sub(lane) < t1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] += static_cast<double>(v[u][i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) red[warp][lane][i] = acc[i];
  __syncthreads();
  if (threadIdx.x < D)
    partial[(static_cast<int64_t>(g) * gridDim.x + chunk) * D + threadIdx.x] =
        reduce_lanes<D>(red, 8, threadIdx.x);
}

template <int D>
__global__ void kmean_final_kernel(const double* __restrict__ partial, int nchunks, int N,
                                   float* __restrict__ kmean) {
  const int g = blockIdx.x, d = threadIdx.x;
  if (d >= D) return;
  // chunks in order, eight loads in flight at a time
  const double* pp = partial + static_cast<int64_t>(g) * nchunks * D + d;
  double tot = 0.0;
  int c = 0;
  for (; c + 8 <= nchunks; c += 8) {
    double x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] = pp[static_cast<int64_t>(c + u) * D];
#pragma unroll
    for (int u = 0; u < 8; ++u) tot += x[u];
  }
  for (; c < nchunks; ++c) tot += pp[static_cast<int64_t>(c) * D];
  kmean[g * D + d] = __fdiv_rn(__double2float_rn(tot), static_cast<float>(N));
}

// ---------------------------------------------------------------------------
// Q / K rows: rotate, (K) subtract the token mean, per-row E4M3.
// One CTA covers `rows` consecutive output rows (a routing block when
// statistics are requested) so that block sums reduce in a fixed order.
// ---------------------------------------------------------------------------
struct QKArgs {
  vcattn_bhnd x;
  int H, N, n_pad, flags;
  const int32_t* perm;   // K only
  int perm_rows;
  const float* kmean;    // (G, D) or nullptr
  uint8_t* codes;        // (G, NP, D)
  float* scale;          // (G, NP)
  int rows;              // rows per CTA
  float* blk_mean;       // (G, NP/rows, D) mean of the rotated rows, or nullptr
  float* blk_qbar;       // (G, NP/rows, D) sum of fp32(q8 * fp32(qs*sm)), or nullptr
  float sm_scale;
};

// STATS: the routing block statistics are requested (blk_mean / blk_qbar),
// kept as float64 accumulators.  Both variants run four CTAs per SM (64
// registers): the kernel is latency-bound, and the statistics variant is
// faster at four CTAs with a few bytes of spills than at three without.
template <int DT, int D, bool STATS>
__global__ void __launch_bounds__(256, 4) quant_rows_kernel(QKArgs a) {
  using RM = RowMap<D>;
  const int g = blockIdx.y;
  const int b = g / a.H, h = g % a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * a.rows;
  const bool want_mean = STATS && a.blk_mean != nullptr;
  const bool want_qbar = STATS && a.blk_qbar != nullptr;
  double msum[4] = {0.0, 0.0, 0.0, 0.0};
  double qsum[4] = {0.0, 0.0, 0.0, 0.0};
  float km[4] = {0.f, 0.f, 0.f, 0.f};
  if (a.kmean != nullptr) {
    const float4 t = *reinterpret_cast<const float4*>(a.kmean + g * D + RM::col(lane));
    km[0] = t.x; km[1] = t.y; km[2] = t.z; km[3] = t.w;
  }
  const int nwarps = blockDim.x >> 5;
  // kBatch rows per warp are loaded before any is used (memory-level
  // parallelism); rows = 64 or 128 gives 8 or 16 rows per warp.
  constexpr int kBatch = 4;
  const int step = nwarps * RM::kRowsPerWarp;
  for (int base0 = warp * RM::kRowsPerWarp; base0 < a.rows; base0 += kBatch * step) {
  float vb[kBatch][4];
#pragma unroll
  for (int u = 0; u < kBatch; ++u) {
    const int t = r0 + base0 + u * step + RM::sub(lane);
    vb[u][0] = vb[u][1] = vb[u][2] = vb[u][3] = 0.f;
    if (base0 + u * step < a.rows && t < a.N) {
      const int src = source_row(a.perm, a.perm_rows, g, a.N, t);
      const int64_t off = b * a.x.sb + h * a.x.sh + static_cast<int64_t>(src) * a.x.sn + RM::col(lane);
      const float4 x = load4<DT>(a.x.data, off);
      vb[u][0] = x.x; vb[u][1] = x.y; vb[u][2] = x.z; vb[u][3] = x.w;
    }
  }
#pragma unroll
  for (int u = 0; u < kBatch; ++u) {
    if (base0 + u * step >= a.rows) break;
    const int t = r0 + base0 + u * step + RM::sub(lane);
    float* v = vb[u];
    const bool real = t < a.N;
    if (a.flags & VCATTN_HADAMARD) RM::fwht(v, lane);
    if (real && a.kmean != nullptr) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __fsub_rn(v[i], km[i]);
    }
    if (!real) { v[0] = v[1] = v[2] = v[3] = 0.f; }
    float am = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    am = RM::amax(am);
    uint32_t packed = 0;
    float sc = 0.f;
    if (real) {
      sc = e4m3_row_scale(am);
      const DivBy div(sc);
      packed = e4m3x4(div(v[0]), div(v[1]), div(v[2]), div(v[3]));
    }
    if (t < a.n_pad) {
      *reinterpret_cast<uint32_t*>(a.codes + (static_cast<int64_t>(g) * a.n_pad + t) * D + RM::col(lane)) = packed;
      if ((lane & (32 / RM::kRowsPerWarp - 1)) == 0) a.scale[static_cast<int64_t>(g) * a.n_pad + t] = sc;
      if (want_mean) {
#pragma unroll
        for (int i = 0; i < 4; ++i) msum[i] += static_cast<double>(v[i]);
      }
      if (want_qbar && real) {
        const float w = __fmul_rn(sc, a.sm_scale);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float q8 = e4m3_to_float((packed >> (8 * i)) & 0xff);
          qsum[i] += static_cast<double>(__fmul_rn(q8, w));
        }
      }
    }
  }
  }
  if constexpr (!STATS) return;
  if (!want_mean && !want_qbar) return;
  __shared__ double red_m[8][32][4];
  __shared__ double red_q[8][32][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    red_m[warp][lane][i] = msum[i];
    red_q[warp][lane][i] = qsum[i];
  }
  __syncthreads();
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
    const int64_t o = (static_cast<int64_t>(g) * gridDim.x + blockIdx.x) * D + d;
    if (want_mean)
      a.blk_mean[o] = __fdiv_rn(__double2float_rn(reduce_lanes<D>(red_m, nwarps, d)),
                                static_cast<float>(a.rows));
    if (want_qbar) a.blk_qbar[o] = __double2float_rn(reduce_lanes<D>(red_q, nwarps, d));
  }
}

// ---------------------------------------------------------------------------
// Head dim 128 with four lanes per row.  Lane 4 s + c of a warp owns channels
// 32 c .. 32 c + 31 of the warp's row s (eight rows per warp at a time), so
// the butterfly strides 1 .. 16 run inside the lane and only strides 32 and
// 64 cross lanes (partners lane ^ 1 and lane ^ 2): 8 warp shuffles per row
// instead of 25, the row maximum reduces over four lanes, and the E4M3 row
// scale and its reciprocal are divided out by four lanes instead of 32.  The
// butterfly pairs, their order and every rounding are those of fwht128_warp
// (hadamard.py:37-65), so the bytes are identical.
// ---------------------------------------------------------------------------

// 32 consecutive input elements (16-byte aligned) -> float.
template <int DT>
__device__ __forceinline__ void load32(const void* base, int64_t off, float v[32]) {
  if constexpr (DT == VCATTN_DTYPE_F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
    float4 x[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) x[q] = p[q];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v[4 * q] = x[q].x; v[4 * q + 1] = x[q].y; v[4 * q + 2] = x[q].z; v[4 * q + 3] = x[q].w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + off);
    uint4 x[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) x[q] = p[q];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t w[4] = {x[q].x, x[q].y, x[q].z, x[q].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if constexpr (DT == VCATTN_DTYPE_BF16) {
          v[8 * q + 2 * e] = __uint_as_float(w[e] << 16);
          v[8 * q + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          v[8 * q + 2 * e] = f.x;
          v[8 * q + 2 * e + 1] = f.y;
        }
      }
    }
  }
}

// Walsh-Hadamard transform of a 128-wide row over the four lanes that hold
// it (32 consecutive elements each), then the IEEE division by
// fp32(sqrt(128)) (Markstein's correction on the values where it equals the
// division, as in fwht128_warp; the choice of path is per lane, which gives
// the same quotients).
__device__ __forceinline__ void fwht128_quad(float v[32], int lane) {
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if ((i & h) == 0) {
        const float x = v[i], y = v[i + h];
        v[i] = __fadd_rn(x, y);
        v[i + h] = __fsub_rn(x, y);
      }
    }
  }
#pragma unroll
  for (int m = 1; m <= 2; m <<= 1) {
    // lower lane: v + p, upper lane: p - v, as one fma with a +-1 multiplier
    const float sg = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float p = __shfl_xor_sync(0xffffffffu, v[i], m);
      v[i] = __fmaf_rn(sg, v[i], p);
    }
  }
  const float r = 11.313708498984761f;
  const float y = 0.0883883461356163f;
  float lo = fabsf(v[0]), hi = fabsf(v[0]);
#pragma unroll
  for (int i = 1; i < 31; i += 2) {
    lo = fmin3(lo, fabsf(v[i]), fabsf(v[i + 1]));
    hi = fmax3(hi, fabsf(v[i]), fabsf(v[i + 1]));
  }
  lo = fminf(lo, fabsf(v[31]));
  hi = fmaxf(hi, fabsf(v[31]));
  if (!(lo >= 0x1p-100f && hi <= 0x1p+100f)) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __fdiv_rn(v[i], r);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float q0 = __fmul_rn(v[i], y);
      v[i] = __fmaf_rn(__fmaf_rn(-q0, r, v[i]), y, q0);
    }
  }
}

// Q / K rows (D = 128): the work of quant_rows_kernel in the four-lane
// layout.  A CTA still covers `rows` consecutive output rows; it takes them
// 64 at a time (eight warps x eight rows).  With STATS the rotated rows (and
// for Q the dequantised fp32(q8 * fp32(qs * sm))) of each 64-row pass go
// through shared memory, where one thread per channel adds them in float64.
template <int DT, bool STATS>
__global__ void __launch_bounds__(256, 3) quant_rows4_kernel(QKArgs a) {
  constexpr int D = 128;
  constexpr int kPad = D + 4;
  const int g = blockIdx.y;
  const int b = g / a.H, h = g % a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = lane >> 2, c = lane & 3;
  const int r0 = blockIdx.x * a.rows;
  const bool want_mean = STATS && a.blk_mean != nullptr;
  const bool want_qbar = STATS && a.blk_qbar != nullptr;
  extern __shared__ float stat_sm[];   // STATS: [64][kPad] rows, then [64][kPad] q-bar terms
  __shared__ float km_sm[D];
  __shared__ double half_sm[2][D];
  double msum = 0.0, qsum = 0.0;       // thread d < 128: channel d of the CTA's block
  if (a.kmean != nullptr && threadIdx.x < D) km_sm[threadIdx.x] = a.kmean[g * D + threadIdx.x];
  __syncthreads();
  for (int p0 = 0; p0 < a.rows; p0 += 64) {
    const int rl = p0 + warp * 8 + slot;
    const int t = r0 + rl;
    const bool mine = rl < a.rows && t < a.n_pad;
    const bool real = mine && t < a.N;
    float v[32];
    if (real) {
      const int src = source_row(a.perm, a.perm_rows, g, a.N, t);
      load32<DT>(a.x.data, b * a.x.sb + h * a.x.sh + static_cast<int64_t>(src) * a.x.sn + 32 * c, v);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.f;
    }
    if (a.flags & VCATTN_HADAMARD) fwht128_quad(v, lane);
    if (real && a.kmean != nullptr) {
      const float4* km = reinterpret_cast<const float4*>(km_sm + 32 * c);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 m = km[q];
        v[4 * q] = __fsub_rn(v[4 * q], m.x);
        v[4 * q + 1] = __fsub_rn(v[4 * q + 1], m.y);
        v[4 * q + 2] = __fsub_rn(v[4 * q + 2], m.z);
        v[4 * q + 3] = __fsub_rn(v[4 * q + 3], m.w);
      }
    }
    if (!real) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.f;
    }
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i += 2) am = fmax3(am, fabsf(v[i]), fabsf(v[i + 1]));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    uint32_t pk[8];
    float sc = 0.f;
    if (real) {
      sc = e4m3_row_scale(am);
      const DivBy div(sc);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        pk[q] = e4m3x4(div(v[4 * q]), div(v[4 * q + 1]), div(v[4 * q + 2]), div(v[4 * q + 3]));
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) pk[q] = 0u;
    }
    if (mine) {
      uint4* dst = reinterpret_cast<uint4*>(a.codes + (static_cast<int64_t>(g) * a.n_pad + t) * D + 32 * c);
      dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      if (c == 0) a.scale[static_cast<int64_t>(g) * a.n_pad + t] = sc;
    }
    if constexpr (STATS) {
      if (want_mean || want_qbar) {
        float* row_m = stat_sm + (warp * 8 + slot) * kPad + 32 * c;
        float* row_q = row_m + 64 * kPad;
        if (want_mean) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(row_m + 4 * q) =
                mine ? make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (want_qbar) {
          const float w = __fmul_rn(sc, a.sm_scale);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
            if (real) {
              const float4 q8 = e4m3x4_to_float4(pk[q]);
              f = make_float4(__fmul_rn(q8.x, w), __fmul_rn(q8.y, w), __fmul_rn(q8.z, w), __fmul_rn(q8.w, w));
            }
            *reinterpret_cast<float4*>(row_q + 4 * q) = f;
          }
        }
        __syncthreads();
        // all 256 threads: channel d = tid % 128, rows 32 (tid / 128) .. + 31
        // with four accumulators, then the two halves
        const int d = threadIdx.x & (D - 1), hr = (threadIdx.x >> 7) * 32;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          if (which == 0 ? !want_mean : !want_qbar) continue;
          const float* col = stat_sm + (which * 64 + hr) * kPad + d;
          double s4[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
          for (int r = 0; r < 32; r += 4) {
#pragma unroll
            for (int u = 0; u < 4; ++u) s4[u] += static_cast<double>(col[(r + u) * kPad]);
          }
          half_sm[threadIdx.x >> 7][d] = (s4[0] + s4[1]) + (s4[2] + s4[3]);
          __syncthreads();
          if (threadIdx.x < D) {
            const double part = half_sm[0][d] + half_sm[1][d];
            if (which == 0) msum += part; else qsum += part;
          }
          __syncthreads();
        }
      }
    }
  }
  if constexpr (STATS) {
    if (threadIdx.x < D && (want_mean || want_qbar)) {
      const int64_t o = (static_cast<int64_t>(g) * gridDim.x + blockIdx.x) * D + threadIdx.x;
      if (want_mean) a.blk_mean[o] = __fdiv_rn(__double2float_rn(msum), static_cast<float>(a.rows));
      if (want_qbar) a.blk_qbar[o] = __double2float_rn(qsum);
    }
  }
}
constexpr size_t kStatSmem4 = 2 * 64 * (128 + 4) * sizeof(float);

// K token mean (D = 128) in the four-lane layout: 256 rows per CTA in four
// passes of 64.  Each pass's rotated rows go through shared memory, where all
// 256 threads add them in float64: thread i takes channel i % 128 of rows
// 32 (i / 128) .. + 31 with four accumulators, kept across the passes; the
// two halves are added at the end.
template <int DT>
__global__ void __launch_bounds__(256, 3) kmean_partial4_kernel(vcattn_bhnd k, int H, int N, int flags,
                                                                 double* __restrict__ partial) {
  constexpr int D = 128;
  constexpr int kPad = D + 4;
  __shared__ float rows_sm[64 * kPad];
  __shared__ double half_sm[2][D];
  const int g = blockIdx.y, chunk = blockIdx.x;
  const int b = g / H, h = g % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = lane >> 2, c = lane & 3;
  const int d = threadIdx.x & (D - 1), hr = (threadIdx.x >> 7) * 32;
  const int t0 = chunk * kChunkRows;
  double s4[4] = {0.0, 0.0, 0.0, 0.0};
  for (int p0 = 0; p0 < kChunkRows; p0 += 64) {
    const int t = t0 + p0 + warp * 8 + slot;
    float v[32];
    if (t < N) {
      load32<DT>(k.data, b * k.sb + h * k.sh + static_cast<int64_t>(t) * k.sn + 32 * c, v);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.f;
    }
    if (flags & VCATTN_HADAMARD) fwht128_quad(v, lane);
    float* row = rows_sm + (warp * 8 + slot) * kPad + 32 * c;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4*>(row + 4 * q) =
          t < N ? make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    const float* col = rows_sm + hr * kPad + d;
#pragma unroll
    for (int r = 0; r < 32; r += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u) s4[u] += static_cast<double>(col[(r + u) * kPad]);
    }
    __syncthreads();
  }
  half_sm[threadIdx.x >> 7][d] = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  __syncthreads();
  if (threadIdx.x < D)
    partial[(static_cast<int64_t>(g) * gridDim.x + chunk) * D + d] = half_sm[0][d] + half_sm[1][d];
}

// ---------------------------------------------------------------------------
// V: gather by perm, zero-pad, block demean, per-(block x channel) E4M3,
// mu / scale (triton_attn.py:555-567, quant.py:219-237).  One CTA per
// (head, value block); the block is staged in shared memory as fp32.
// ---------------------------------------------------------------------------
struct VArgs {
  vcattn_bhnd x;
  int H, N, n_pad, br;
  const int32_t* perm;
  int perm_rows;
  uint8_t* codes;    // (G, NP, D) or nullptr
  uint8_t* codes_t;  // (G, NB, D, br) or nullptr
  float* scale;      // (G, NB, D)
  float* mu;         // (G, NB, D) block mean / scale
  float* mean;       // (G, NB, D) block mean, or nullptr
  bool mma_order;    // codes rows in the tcgen05 kernel's key order
};

// Slot of value-block row r when VCATTN_V_MMA_ORDER is set: a 4 x 4
// transpose of (row / 8 % 4, row / 2 % 4) inside each 32-row chunk.
__host__ __device__ __forceinline__ int mma_key_slot(int r) {
  return (r & ~31) | (((r >> 1) & 3) << 3) | (((r >> 3) & 3) << 1) | (r & 1);
}

// Each warp keeps the rows it owns in registers through the three passes
// (block mean, residual max, codes); lanes own four channels as in the row
// kernels, so every load and row-major store is a whole coalesced row.  The
// transposed codes go through a shared byte tile whose 4-byte words are
// XOR-swizzled by row / 4, which keeps both its row-major writes and its
// column reads free of bank conflicts.
template <int DT, int D, int BR>
__global__ void __launch_bounds__(512, 2) quant_v_kernel(VArgs a) {
  using RM = RowMap<D>;
  constexpr int kWarps = 16;   // 16 warps, two CTAs per SM: 32 row-holding warps
  constexpr int kSteps = BR / (kWarps * RM::kRowsPerWarp);   // rows per lane
  constexpr int kWords = D / 4;                              // 4-byte code words per row
  __shared__ double red[kWarps][32][4];
  __shared__ float mu_s[D], sc_s[D];
  __shared__ uint32_t ct[BR * kWords];
  const int g = blockIdx.y, j = blockIdx.x;
  const int b = g / a.H, h = g % a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = a.n_pad / BR;
  const int col = RM::col(lane);
  // pass 1: load (zero past N), float64 channel sums
  float x[kSteps][4];
#pragma unroll
  for (int k = 0; k < kSteps; ++k) {
    const int r = (k * kWarps + warp) * RM::kRowsPerWarp + RM::sub(lane);
    const int t = j * BR + r;
    x[k][0] = x[k][1] = x[k][2] = x[k][3] = 0.f;
    if (t < a.N) {
      const int src = source_row(a.perm, a.perm_rows, g, a.N, t);
      const float4 v = load4<DT>(a.x.data, b * a.x.sb + h * a.x.sh + static_cast<int64_t>(src) * a.x.sn + col);
      x[k][0] = v.x; x[k][1] = v.y; x[k][2] = v.z; x[k][3] = v.w;
    }
  }
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
  for (int k = 0; k < kSteps; ++k)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += static_cast<double>(x[k][i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) red[warp][lane][i] = acc[i];
  __syncthreads();
  if (threadIdx.x < D)
    mu_s[threadIdx.x] = __fdiv_rn(__double2float_rn(reduce_lanes<D>(red, kWarps, threadIdx.x)), static_cast<float>(BR));
  __syncthreads();
  // pass 2: residual max per channel
  float mu[4], am[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 4; ++i) mu[i] = mu_s[col + i];
#pragma unroll
  for (int k = 0; k < kSteps; ++k)
#pragma unroll
    for (int i = 0; i < 4; ++i) am[i] = fmaxf(am[i], fabsf(__fsub_rn(x[k][i], mu[i])));
#pragma unroll
  for (int i = 0; i < 4; ++i) red[warp][lane][i] = am[i];
  __syncthreads();
  if (threadIdx.x < D) {
    const int d = threadIdx.x, l = d / 4, i = d % 4;
    float m = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      m = fmaxf(m, static_cast<float>(red[w][l][i]));
      if (D == 64) m = fmaxf(m, static_cast<float>(red[w][l + 16][i]));
    }
    const float sc = e4m3_row_scale(m);
    sc_s[d] = sc;
    const int64_t so = (static_cast<int64_t>(g) * nb + j) * D + d;
    a.scale[so] = sc;
    a.mu[so] = __fdiv_rn(mu_s[d], sc);
    if (a.mean) a.mean[so] = mu_s[d];
  }
  __syncthreads();
  // pass 3: codes
  const DivBy dv[4] = {DivBy(sc_s[col]), DivBy(sc_s[col + 1]), DivBy(sc_s[col + 2]), DivBy(sc_s[col + 3])};
#pragma unroll
  for (int k = 0; k < kSteps; ++k) {
    const int r = (k * kWarps + warp) * RM::kRowsPerWarp + RM::sub(lane);
    const uint32_t w = e4m3x4(dv[0](__fsub_rn(x[k][0], mu[0])), dv[1](__fsub_rn(x[k][1], mu[1])),
                              dv[2](__fsub_rn(x[k][2], mu[2])), dv[3](__fsub_rn(x[k][3], mu[3])));
    if (a.codes) {
      const int slot = a.mma_order ? mma_key_slot(r) : r;
      *reinterpret_cast<uint32_t*>(a.codes + (static_cast<int64_t>(g) * a.n_pad + j * BR + slot) * D + col) = w;
    }
    if (a.codes_t) ct[r * kWords + ((col >> 2) ^ ((r >> 2) & (kWords - 1)))] = w;
  }
  if (a.codes_t) {
    __syncthreads();
    // thread -> (channel d, rows 4rq..4rq+3): one packed word of the
    // transposed block; a warp writes 128 consecutive bytes of one channel
    uint8_t* dst = a.codes_t + (static_cast<int64_t>(g) * nb + j) * D * BR;
    for (int item = threadIdx.x; item < D * (BR / 4); item += blockDim.x) {
      const int d = item / (BR / 4), rq = item % (BR / 4);
      const int wd = d >> 2, bs = 8 * (d & 3);
      uint32_t packed = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = 4 * rq + i;
        const uint32_t word = ct[r * kWords + (wd ^ ((r >> 2) & (kWords - 1)))];
        packed |= ((word >> bs) & 0xffu) << (8 * i);
      }
      *reinterpret_cast<uint32_t*>(dst + static_cast<int64_t>(d) * BR + 4 * rq) = packed;
    }
  }
}

// ---------------------------------------------------------------------------
// Routing threshold + keep mask (triton_attn.py:449-459 and :716-735).
// One CTA per (head, kRouteQB routing query blocks).  Thread t takes KV
// blocks t, t + 256, ...: it reads its k_mean row once (16-byte loads, the
// row's lines stay in L1 across the four-channel steps) and forms the float64
// dots of that row with all kRouteQB query blocks (q vectors as shared-memory
// broadcasts): the threshold proxy fp32(q_cent . k_mean_j) * scale and the
// routing score fp32(q_bar . bf16(k_mean_j)) / q_block.  Each dot is summed
// in float64 and rounded once, so its fp32 value does not depend on the order
// of the partial sums.  Warp w then reduces the threshold of query block w.
// ---------------------------------------------------------------------------
constexpr int kRouteQB = 8;

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int D>
__global__ void __launch_bounds__(256) route_mask_kernel(const float* __restrict__ k_mean,
                                                         const float* __restrict__ q_cent,
                                                         const float* __restrict__ q_bar, int nqb, int nb, int q_block,
                                                         int br, float tau, int local_blocks, int sink_blocks,
                                                         float sm_scale, uint8_t* __restrict__ keep,
                                                         float* __restrict__ thresh_out) {
  extern __shared__ float rsm[];                 // proxy, score [kRouteQB][nb]
  // the eight query vectors as doubles: each is converted once, not once per
  // k_mean row (the float -> double conversions bounded this kernel)
  __shared__ __align__(16) double qcs[kRouteQB][D];
  __shared__ __align__(16) double qbs[kRouteQB][D];
  float* proxy = rsm;
  float* score = rsm + kRouteQB * nb;
  const int g = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < kRouteQB * D; e += blockDim.x) {
    const int w = e / D, d = e % D, i = blockIdx.x * kRouteQB + w;
    const bool ok = i < nqb;
    qcs[w][d] = ok ? static_cast<double>(q_cent[(static_cast<int64_t>(g) * nqb + i) * D + d]) : 0.0;
    qbs[w][d] = ok ? static_cast<double>(q_bar[(static_cast<int64_t>(g) * nqb + i) * D + d]) : 0.0;
  }
  __syncthreads();
  const float inv_q = static_cast<float>(q_block);
  for (int j = tid; j < nb; j += blockDim.x) {
    const float* km = k_mean + (static_cast<int64_t>(g) * nb + j) * D;
    double d1[kRouteQB], d2[kRouteQB];
#pragma unroll
    for (int w = 0; w < kRouteQB; ++w) d1[w] = d2[w] = 0.0;
#pragma unroll 2
    for (int d = 0; d < D; d += 4) {
      const float4 kv = *reinterpret_cast<const float4*>(km + d);
      const double kf[4] = {static_cast<double>(kv.x), static_cast<double>(kv.y), static_cast<double>(kv.z),
                            static_cast<double>(kv.w)};
      const double kb[4] = {static_cast<double>(bf16_round(kv.x)), static_cast<double>(bf16_round(kv.y)),
                            static_cast<double>(bf16_round(kv.z)), static_cast<double>(bf16_round(kv.w))};
#pragma unroll
      for (int w = 0; w < kRouteQB; ++w) {
        const double2 c01 = *reinterpret_cast<const double2*>(&qcs[w][d]);
        const double2 c23 = *reinterpret_cast<const double2*>(&qcs[w][d + 2]);
        const double2 b01 = *reinterpret_cast<const double2*>(&qbs[w][d]);
        const double2 b23 = *reinterpret_cast<const double2*>(&qbs[w][d + 2]);
        const double cv[4] = {c01.x, c01.y, c23.x, c23.y}, bv[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          d1[w] = fma(cv[e], kf[e], d1[w]);
          d2[w] = fma(bv[e], kb[e], d2[w]);
        }
      }
    }
#pragma unroll
    for (int w = 0; w < kRouteQB; ++w) {
      proxy[w * nb + j] = __fmul_rn(__double2float_rn(d1[w]), sm_scale);
      score[w * nb + j] = __fdiv_rn(__double2float_rn(d2[w]), inv_q);
    }
  }
  __syncthreads();
  const int qi = blockIdx.x * kRouteQB + warp;   // this warp's routing query block
  if (qi >= nqb) return;
  // threshold of the query block: mean + tau * std of its proxies
  const float* pr = proxy + warp * nb;
  const float* sc = score + warp * nb;
  double part = 0.0;
  for (int j = lane; j < nb; j += 32) part += static_cast<double>(pr[j]);
  const float mean = __fdiv_rn(__double2float_rn(warp_sum_f64(part)), static_cast<float>(nb));
  part = 0.0;
  for (int j = lane; j < nb; j += 32) {
    const float dv = __fsub_rn(pr[j], mean);
    part += static_cast<double>(__fmul_rn(dv, dv));
  }
  const float var = __fdiv_rn(__double2float_rn(warp_sum_f64(part)), static_cast<float>(nb));
  const float thr = __fadd_rn(mean, __fmul_rn(tau, __fsqrt_rn(var)));
  if (lane == 0 && thresh_out) thresh_out[static_cast<int64_t>(g) * nqb + qi] = thr;
  const int qb_kv = (qi * q_block) / br;
  uint8_t* krow = keep + (static_cast<int64_t>(g) * nqb + qi) * nb;
  for (int j = lane; j < nb; j += 32) {
    const bool k = (sc[j] > thr) || (abs(qb_kv - j) <= local_blocks) || (j < sink_blocks);
    krow[j] = k ? 1 : 0;
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// NVFP4 Q / K (quant.py:172-204 applied to each (b, h) slab of the rotated,
// smoothed rows): one fp32 tensor scale g per head, an E4M3 micro scale per
// 16 consecutive elements along D and E2M1 codes packed two per byte (low
// nibble = even element).  Pass A takes the head's |x| max (integer atomicMax
// on the float bits of non-negative values); pass B quantises.  Lanes own
// four consecutive elements, so a 16-element block spans four lanes.
// ---------------------------------------------------------------------------
struct NvArgs {
  vcattn_bhnd x;
  int H, N, n_pad, flags;
  const int32_t* perm;   // K only
  int perm_rows;
  const float* kmean;    // (G, D) or nullptr
  unsigned* amax;        // (G) float bits
  uint8_t* codes;        // (G, NP, D/2)
  uint8_t* micro;        // (G, NP, D/16)
  uint8_t* micro_mma;    // (G, ceil(NP/128), D/64, 512) scale-factor atoms of the block-scaled MMA, or nullptr
  float* gout;           // (G)
  int rows;              // rows per CTA
};

template <int DT, int D, bool QUANT>
__global__ void __launch_bounds__(256, 4) nvfp4_rows_kernel(NvArgs a) {
  using RM = RowMap<D>;
  const int g = blockIdx.y;
  const int b = g / a.H, h = g % a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * a.rows;
  float km[4] = {0.f, 0.f, 0.f, 0.f};
  if (a.kmean != nullptr) {
    const float4 t = *reinterpret_cast<const float4*>(a.kmean + g * D + RM::col(lane));
    km[0] = t.x; km[1] = t.y; km[2] = t.z; km[3] = t.w;
  }
  float gs = 0.f;
  if constexpr (QUANT) {
    gs = fmaxf(__fdiv_rn(fmaxf(__uint_as_float(a.amax[g]), kTiny), 6.0f * kE4M3Max), kTiny);
    if (blockIdx.x == 0 && threadIdx.x == 0) a.gout[g] = gs;
  }
  float mx = 0.f;
  const int nwarps = blockDim.x >> 5;
  constexpr int kBatch = 4;
  const int step = nwarps * RM::kRowsPerWarp;
  for (int base0 = warp * RM::kRowsPerWarp; base0 < a.rows; base0 += kBatch * step) {
    float vb[kBatch][4];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int t = r0 + base0 + u * step + RM::sub(lane);
      vb[u][0] = vb[u][1] = vb[u][2] = vb[u][3] = 0.f;
      if (base0 + u * step < a.rows && t < a.N) {
        const int src = source_row(a.perm, a.perm_rows, g, a.N, t);
        const float4 x = load4<DT>(a.x.data, b * a.x.sb + h * a.x.sh + static_cast<int64_t>(src) * a.x.sn + RM::col(lane));
        vb[u][0] = x.x; vb[u][1] = x.y; vb[u][2] = x.z; vb[u][3] = x.w;
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (base0 + u * step >= a.rows) break;
      const int t = r0 + base0 + u * step + RM::sub(lane);
      float* v = vb[u];
      const bool real = t < a.N;
      if (a.flags & VCATTN_HADAMARD) RM::fwht(v, lane);
      if (!real) { v[0] = v[1] = v[2] = v[3] = 0.f; }
      else if (a.kmean != nullptr) {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fsub_rn(v[i], km[i]);
      }
      float bm = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
      if constexpr (!QUANT) {
        mx = fmaxf(mx, bm);
      } else {
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
        bm = fmaxf(bm, kTiny);
        const float micro = __fdiv_rn(__fdiv_rn(bm, 6.0f), gs);
        const uint32_t mcode = e4m3x2(fminf(micro, kE4M3Max), 0.f) & 0xffu;
        const float denom = fmaxf(__fmul_rn(gs, e4m3_to_float(mcode)), kTiny);
        if (t < a.n_pad) {
          const int64_t row = static_cast<int64_t>(g) * a.n_pad + t;
          const uint32_t lo = e2m1x2(__fdiv_rn(v[0], denom), __fdiv_rn(v[1], denom));
          const uint32_t hi = e2m1x2(__fdiv_rn(v[2], denom), __fdiv_rn(v[3], denom));
          *reinterpret_cast<uint16_t*>(a.codes + row * (D / 2) + RM::col(lane) / 2) =
              static_cast<uint16_t>(lo | (hi << 8));
          if ((lane & 3) == 0) {
            const int kb = RM::col(lane) / 16;
            a.micro[row * (D / 16) + kb] = static_cast<uint8_t>(mcode);
            if (a.micro_mma != nullptr) {
              // 128-row tile, 512-byte atom per 4 scales: byte 16 (m%32) + 4 (m/32) + kb%4
              const int m = t & 127;
              const int64_t tiles = (a.n_pad + 127) / 128;
              const int64_t atom = ((static_cast<int64_t>(g) * tiles + (t >> 7)) * (D / 64) + (kb >> 2)) * 512;
              a.micro_mma[atom + (m & 31) * 16 + (m >> 5) * 4 + (kb & 3)] = static_cast<uint8_t>(mcode);
            }
          }
        }
      }
    }
  }
  if constexpr (!QUANT) {
    mx = warp_max(mx);
    if (lane == 0) atomicMax(a.amax + g, __float_as_uint(mx));
  }
}

template <int DT, int D>
static cudaError_t prepare_nvfp4_impl(const NvfpParams& p, cudaStream_t st) {
  const int G = p.B * p.H;
  float* kmean = nullptr;
  const int nchunks = (p.N + kChunkRows - 1) / kChunkRows;
  double* partial = reinterpret_cast<double*>(p.workspace);
  unsigned* amax = reinterpret_cast<unsigned*>(reinterpret_cast<float*>(partial + static_cast<size_t>(G) * nchunks * D) +
                                               static_cast<size_t>(G) * D);
  if (p.flags & VCATTN_SMOOTH_K) {
    kmean = reinterpret_cast<float*>(partial + static_cast<size_t>(G) * nchunks * D);
    kmean_partial_kernel<DT, D><<<dim3(nchunks, G), 256, 0, st>>>(*p.k, p.H, p.N, p.flags, partial);
    kmean_final_kernel<D><<<G, D, 0, st>>>(partial, nchunks, p.N, kmean);
  }
  cudaMemsetAsync(amax, 0, 2 * static_cast<size_t>(G) * sizeof(unsigned), st);
  const int rows = 128;
  const dim3 grid((p.n_pad + rows - 1) / rows, G);
  NvArgs aq{};
  aq.x = *p.q; aq.H = p.H; aq.N = p.N; aq.n_pad = p.n_pad; aq.flags = p.flags;
  aq.amax = amax; aq.codes = p.q4; aq.micro = p.q4_scale; aq.micro_mma = p.q4_sf_mma; aq.gout = p.q4_g; aq.rows = rows;
  NvArgs ak = aq;
  ak.x = *p.k; ak.perm = p.perm; ak.perm_rows = p.perm_rows; ak.kmean = kmean;
  ak.amax = amax + G; ak.codes = p.k4; ak.micro = p.k4_scale; ak.micro_mma = p.k4_sf_mma; ak.gout = p.k4_g;
  nvfp4_rows_kernel<DT, D, false><<<grid, 256, 0, st>>>(aq);
  nvfp4_rows_kernel<DT, D, false><<<grid, 256, 0, st>>>(ak);
  nvfp4_rows_kernel<DT, D, true><<<grid, 256, 0, st>>>(aq);
  nvfp4_rows_kernel<DT, D, true><<<grid, 256, 0, st>>>(ak);
  return cudaGetLastError();
}

cudaError_t launch_prepare_nvfp4(const NvfpParams& p, cudaStream_t st) {
  if (p.D == 128) {
    switch (p.dtype) {
      case VCATTN_DTYPE_BF16: return prepare_nvfp4_impl<VCATTN_DTYPE_BF16, 128>(p, st);
      case VCATTN_DTYPE_F16: return prepare_nvfp4_impl<VCATTN_DTYPE_F16, 128>(p, st);
      default: return prepare_nvfp4_impl<VCATTN_DTYPE_F32, 128>(p, st);
    }
  }
  switch (p.dtype) {
    case VCATTN_DTYPE_BF16: return prepare_nvfp4_impl<VCATTN_DTYPE_BF16, 64>(p, st);
    case VCATTN_DTYPE_F16: return prepare_nvfp4_impl<VCATTN_DTYPE_F16, 64>(p, st);
    default: return prepare_nvfp4_impl<VCATTN_DTYPE_F32, 64>(p, st);
  }
}

size_t prepare_workspace_bytes(int G, int N, int D) {
  const size_t nchunks = (N + kChunkRows - 1) / kChunkRows;
  return static_cast<size_t>(G) * nchunks * D * sizeof(double) + static_cast<size_t>(G) * D * sizeof(float) +
         2 * static_cast<size_t>(G) * sizeof(unsigned) + 256;
}

// The Q / K row pass: the four-lane kernel for D = 128, the warp-per-row
// kernel for D = 64.
template <int DT, int D>
static void launch_rows(const QKArgs& a, dim3 grid, bool stats, cudaStream_t st) {
  if constexpr (D == 128) {
    if (stats) {
      cudaFuncSetAttribute(quant_rows4_kernel<DT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kStatSmem4));
      quant_rows4_kernel<DT, true><<<grid, 256, kStatSmem4, st>>>(a);
    } else {
      quant_rows4_kernel<DT, false><<<grid, 256, 0, st>>>(a);
    }
  } else {
    if (stats) quant_rows_kernel<DT, D, true><<<grid, 256, 0, st>>>(a);
    else quant_rows_kernel<DT, D, false><<<grid, 256, 0, st>>>(a);
  }
}

template <int DT, int D>
static cudaError_t prepare_impl(const PrepareParams& p, cudaStream_t st) {
  const int G = p.B * p.H;
  const int nb = p.n_pad / p.block_rows;
  float* kmean = nullptr;
  if ((p.flags & VCATTN_SMOOTH_K) && p.k8 != nullptr) {
    const int nchunks = (p.N + kChunkRows - 1) / kChunkRows;
    double* partial = reinterpret_cast<double*>(p.workspace);
    kmean = reinterpret_cast<float*>(partial + static_cast<size_t>(G) * nchunks * D);
    if constexpr (D == 128) kmean_partial4_kernel<DT><<<dim3(nchunks, G), 256, 0, st>>>(*p.k, p.H, p.N, p.flags, partial);
    else kmean_partial_kernel<DT, D><<<dim3(nchunks, G), 256, 0, st>>>(*p.k, p.H, p.N, p.flags, partial);
    kmean_final_kernel<D><<<G, D, 0, st>>>(partial, nchunks, p.N, kmean);
  }
  const bool route = p.route != nullptr;
  // Q rows
  if (p.q8 != nullptr) {
    QKArgs a{};
    a.x = *p.q; a.H = p.H; a.N = p.N; a.n_pad = p.n_pad; a.flags = p.flags;
    a.perm = nullptr; a.perm_rows = 0; a.kmean = nullptr;
    a.codes = p.q8; a.scale = p.q_scale;
    a.rows = route ? p.route->q_block : 64;
    a.blk_mean = route ? p.route->q_cent : nullptr;
    a.blk_qbar = route ? p.route->q_bar : nullptr;
    a.sm_scale = route ? p.route->sm_scale : 0.f;
    const int grid_x = (p.n_pad + a.rows - 1) / a.rows;
    launch_rows<DT, D>(a, dim3(grid_x, G), route, st);
  }
  // K rows (gathered by perm)
  if (p.k8 != nullptr) {
    QKArgs a{};
    a.x = *p.k; a.H = p.H; a.N = p.N; a.n_pad = p.n_pad; a.flags = p.flags;
    a.perm = p.perm; a.perm_rows = p.perm_rows; a.kmean = kmean;
    a.codes = p.k8; a.scale = p.k_scale;
    a.rows = p.block_rows;
    a.blk_mean = route ? p.route->k_mean : nullptr;
    a.blk_qbar = nullptr;
    launch_rows<DT, D>(a, dim3(nb, G), route, st);
  }
  // V blocks
  {
    VArgs a{};
    a.x = *p.v; a.H = p.H; a.N = p.N; a.n_pad = p.n_pad; a.br = p.block_rows;
    a.perm = p.perm; a.perm_rows = p.perm_rows;
    a.codes = p.v8; a.codes_t = p.v8t; a.scale = p.v_scale; a.mu = p.mu; a.mean = p.v_mean;
    a.mma_order = (p.flags & VCATTN_V_MMA_ORDER) != 0;
    if (p.block_rows == 128) quant_v_kernel<DT, D, 128><<<dim3(nb, G), 512, 0, st>>>(a);
    else quant_v_kernel<DT, D, 64><<<dim3(nb, G), 512, 0, st>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_prepare(const PrepareParams& p, cudaStream_t st) {
  if (p.D == 128) {
    switch (p.dtype) {
      case VCATTN_DTYPE_BF16: return prepare_impl<VCATTN_DTYPE_BF16, 128>(p, st);
      case VCATTN_DTYPE_F16: return prepare_impl<VCATTN_DTYPE_F16, 128>(p, st);
      default: return prepare_impl<VCATTN_DTYPE_F32, 128>(p, st);
    }
  }
  switch (p.dtype) {
    case VCATTN_DTYPE_BF16: return prepare_impl<VCATTN_DTYPE_BF16, 64>(p, st);
    case VCATTN_DTYPE_F16: return prepare_impl<VCATTN_DTYPE_F16, 64>(p, st);
    default: return prepare_impl<VCATTN_DTYPE_F32, 64>(p, st);
  }
}

// ---------------------------------------------------------------------------
// bf16 operand tiles of the proxy fold of the tcgen05 sparse kernel, one
// 8 KB tile per (head, group of 16 KV blocks), laid out so that a linear
// copy into 1024-byte aligned shared memory gives the 128-byte swizzle:
//   [0, 4096)    bf16(k_mean) K-major: atom a (channels 64a..64a+63) at 2048 a,
//                row n = block g0+n, byte c at sw128(n, c)
//   [4096, 8192) bf16(v_mean) MN-major: half h (channels 64h..) at 4096 + 2048 h,
//                row k = block g0 + route_tile_block(k), byte c at sw128(k, c)
// Blocks past the last one are zero.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int route_tile_block(int k) {
  return ((k & 3) < 2) ? 2 * (k >> 2) + (k & 3) : 8 + 2 * (k >> 2) + (k & 3) - 2;
}
__host__ __device__ constexpr int tile_sw128(int r, int c) {
  return r * 128 + ((((c >> 4) ^ (r & 7)) & 7) << 4) + (c & 15);
}

__global__ void __launch_bounds__(256) route_tiles_kernel(const float* __restrict__ k_mean,
                                                          const float* __restrict__ v_mean, int nb, int ngroups,
                                                          int D, uint8_t* __restrict__ tiles) {
  const int grp = blockIdx.x, g = blockIdx.y;
  const int g0 = grp * 16;
  uint8_t* t = tiles + (static_cast<int64_t>(g) * ngroups + grp) * 8192;
  // 16 rows x 64 channel pairs for each of k_mean and v_mean
  for (int e = threadIdx.x; e < 2 * 16 * 64; e += blockDim.x) {
    const int which = e >> 10, r = (e >> 6) & 15, pair = e & 63;
    const int ch = 2 * pair;                       // channel of the low half
    const int blk = g0 + (which == 0 ? r : route_tile_block(r));
    float v0 = 0.f, v1 = 0.f;
    if (blk < nb && ch < D) {   // head dim 64: channels 64-127 of the tile stay zero
      const float* src = (which == 0 ? k_mean : v_mean) + (static_cast<int64_t>(g) * nb + blk) * D + ch;
      v0 = src[0];
      v1 = src[1];
    }
    const uint32_t word = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v0))) |
                          (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v1))) << 16);
    const int half = ch >> 6, c = (ch & 63) * 2;
    *reinterpret_cast<uint32_t*>(t + which * 4096 + half * 2048 + tile_sw128(r, c)) = word;
  }
}

cudaError_t launch_route_tiles(const float* k_mean, const float* v_mean, int G, int nb, int D, uint8_t* tiles,
                               cudaStream_t st) {
  const int ngroups = (nb + 15) / 16;
  if (G <= 0 || ngroups <= 0) return cudaSuccess;
  route_tiles_kernel<<<dim3(ngroups, G), 256, 0, st>>>(k_mean, v_mean, nb, ngroups, D, tiles);
  return cudaGetLastError();
}

cudaError_t launch_route_mask(const RouteParams& p, cudaStream_t st) {
  const int nqb = p.n_pad / p.q_block;
  const int nb = p.n_pad / p.block_rows;
  const dim3 grid((nqb + kRouteQB - 1) / kRouteQB, p.G);
  const size_t smem = 2 * static_cast<size_t>(kRouteQB) * nb * sizeof(float);
  // above 48 KB of dynamic shared memory from 768 KV blocks on
  cudaError_t e = cudaFuncSetAttribute(route_mask_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(route_mask_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  if (p.D == 128) {
    route_mask_kernel<128><<<grid, 256, smem, st>>>(
        p.k_mean, p.q_cent, p.q_bar, nqb, nb, p.q_block, p.block_rows, p.tau, p.local_blocks,
        p.sink_blocks, p.sm_scale, p.keep, p.thresh);
  } else {
    route_mask_kernel<64><<<grid, 256, smem, st>>>(
        p.k_mean, p.q_cent, p.q_bar, nqb, nb, p.q_block, p.block_rows, p.tau, p.local_blocks,
        p.sink_blocks, p.sm_scale, p.keep, p.thresh);
  }
  return cudaGetLastError();
}

}  // namespace vcattn
