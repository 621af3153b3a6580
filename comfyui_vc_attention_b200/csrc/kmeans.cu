// V-Smooth k-means grouping and the stable label sort that yields the
// permutation (grouping.py:71-186).
//
// Arithmetic is fixed so that labels, centroids and the permutation are bit
// exact against the CPU restatement:
//   * assignment: the bf16 GEMM of grouping.py:98 is a per-(token, centroid)
//     fp32 FMA chain over channels in increasing order (bf16 products are
//     exact, so this equals a sequential fp32 sum), rounded to bf16, times 2,
//     minus |c|^2 (sequential fp32), first argmax;
//   * update: fp32 sums in token order, which is what index_add_ does
//     (grouping.py:277-278), then / count and bf16 rounding;
//   * sort: a stable counting sort over (key, 32-token chunk) pairs.
#include "kernels.cuh"

namespace vcattn {

namespace {

constexpr int kChunk = 32;        // tokens per counting-sort chunk (one warp)
constexpr int kAssignThreads = 128;
constexpr int kCentTile = 64;     // centroids staged in shared memory per pass

struct KmWs {
  int32_t* labels;
  int32_t* counts;
  int32_t* offsets;
  float* cent;
  float* seeds;
  uint16_t* cb16;   // (G, k, D) bf16 centroids: B operand of the tensor-core assign
  float* c2;        // (G, k) |c|^2, sequential fp32 over channels
  int32_t* tsum;    // (G, scan tiles) tile sums of the counting-sort scan
};

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

KmWs carve(void* base, int G, int N, int D, int k, int nkeys) {
  const size_t nchunks = (N + kChunk - 1) / kChunk;
  const size_t nk = static_cast<size_t>(nkeys > k ? nkeys : k);
  char* p = static_cast<char*>(base);
  KmWs w;
  w.labels = reinterpret_cast<int32_t*>(p); p += align256(sizeof(int32_t) * G * static_cast<size_t>(N));
  w.counts = reinterpret_cast<int32_t*>(p); p += align256(sizeof(int32_t) * G * nk * nchunks);
  w.offsets = reinterpret_cast<int32_t*>(p); p += align256(sizeof(int32_t) * G * nk * nchunks);
  w.cent = reinterpret_cast<float*>(p); p += align256(sizeof(float) * G * static_cast<size_t>(k) * D);
  w.seeds = reinterpret_cast<float*>(p); p += align256(sizeof(float) * G * static_cast<size_t>(k) * D);
  w.cb16 = reinterpret_cast<uint16_t*>(p); p += align256(sizeof(uint16_t) * G * static_cast<size_t>(k) * D);
  w.c2 = reinterpret_cast<float*>(p); p += align256(sizeof(float) * G * static_cast<size_t>(k));
  w.tsum = reinterpret_cast<int32_t*>(p);
  return w;
}

template <int DT>
__device__ __forceinline__ float load_bf16_value(const vcattn_bhnd& v, int b, int h, int t, int d) {
  const int64_t off = b * v.sb + h * v.sh + static_cast<int64_t>(t) * v.sn + d;
  if constexpr (DT == VCATTN_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(v.data)[off]);
  else if constexpr (DT == VCATTN_DTYPE_F16) return bf16_round(__half2float(static_cast<const __half*>(v.data)[off]));
  else return bf16_round(static_cast<const float*>(v.data)[off]);
}

// The bf16 copy of centroid (g, c) and its |c|^2 as a sequential fp32 FMA
// chain over channels (what the assignment subtracts).  One CTA of D threads,
// thread d holding channel d.
__device__ __forceinline__ void centroid_side(float val, int D, int64_t row, uint16_t* cb16, float* c2) {
  __shared__ float sq[128];
  const int d = threadIdx.x;
  cb16[row * D + d] = static_cast<uint16_t>(__float_as_uint(val) >> 16);   // val holds a bf16 value
  sq[d] = val;
  __syncthreads();
  if (d == 0) {
    float acc = 0.f;
    for (int j = 0; j < D; ++j) acc = __fmaf_rn(sq[j], sq[j], acc);
    c2[row] = acc;
  }
}

// grouping.py:71-83: centroid c = bf16(mean of the samples at
// round(linspace(0, N-1, m))[c*m_per : (c+1)*m_per]).  Launched with D threads.
template <int DT>
__global__ void seed_kernel(vcattn_bhnd v, int H, int N, int D, int k, int m, int m_per,
                            float* seeds, float* cent, const uint16_t* warm, uint16_t* cb16, float* c2) {
  const int g = blockIdx.y, c = blockIdx.x, d = threadIdx.x;
  const int b = g / H, h = g % H;
  float step = 0.f;
  if (m > 1) step = __fdiv_rn(static_cast<float>(N - 1), static_cast<float>(m - 1));
  double s = 0.0;
  for (int i = 0; i < m_per; ++i) {
    const int pos = c * m_per + i;
    int idx = 0;
    if (m > 1) {
      const float f = (pos < m / 2) ? __fmaf_rn(step, static_cast<float>(pos), 0.0f)
                                    : __fmaf_rn(-step, static_cast<float>(m - 1 - pos), static_cast<float>(N - 1));
      idx = static_cast<int>(rintf(f));
    }
    s += static_cast<double>(load_bf16_value<DT>(v, b, h, idx, d));
  }
  const float mean = bf16_round(__fdiv_rn(__double2float_rn(s), static_cast<float>(m_per)));
  const int64_t o = (static_cast<int64_t>(g) * k + c) * D + d;
  seeds[o] = mean;
  const float cv = warm ? bf16_bits_to_float(warm[o]) : mean;
  cent[o] = cv;
  centroid_side(cv, D, static_cast<int64_t>(g) * k + c, cb16, c2);
}

// Row of D bf16 values packed two per register.
template <int DT, int D>
__device__ __forceinline__ void load_row_bf16x2(const vcattn_bhnd& v, int b, int h, int t, uint32_t (&r)[D / 2]) {
  const int64_t off = b * v.sb + h * v.sh + static_cast<int64_t>(t) * v.sn;
  if constexpr (DT == VCATTN_DTYPE_BF16) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(v.data) + off);
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const uint4 x = p[i];
      r[4 * i + 0] = x.x; r[4 * i + 1] = x.y; r[4 * i + 2] = x.z; r[4 * i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < D / 2; ++i) {
      float lo, hi;
      if constexpr (DT == VCATTN_DTYPE_F16) {
        const __half* p = static_cast<const __half*>(v.data) + off;
        lo = __half2float(p[2 * i]); hi = __half2float(p[2 * i + 1]);
      } else {
        const float* p = static_cast<const float*>(v.data) + off;
        lo = p[2 * i]; hi = p[2 * i + 1];
      }
      const uint32_t bl = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
      const uint32_t bh = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
      r[i] = bl | (bh << 16);
    }
  }
}

// grouping.py:86-100: nearest centroid per token (one thread per token), then
// per-warp counts of the sort key for the stable counting sort.
template <int DT, int D>
__global__ void __launch_bounds__(kAssignThreads) assign_kernel(
    vcattn_bhnd v, int H, int N, int k, const float* __restrict__ cent,
    int32_t* __restrict__ labels, const int32_t* __restrict__ key_offset, int nkeys, int nchunks,
    int32_t* __restrict__ counts) {
  __shared__ __align__(16) float cT[D][kCentTile];   // channel-major centroid tile
  __shared__ float c2[kCentTile];
  const int g = blockIdx.y;
  const int b = g / H, h = g % H;
  const int t = blockIdx.x * kAssignThreads + threadIdx.x;
  const bool live = t < N;
  uint32_t row[D / 2];
  if (live) load_row_bf16x2<DT, D>(v, b, h, t, row);
  else {
#pragma unroll
    for (int i = 0; i < D / 2; ++i) row[i] = 0u;
  }
  float best = -INFINITY;
  int label = 0;
  for (int c0 = 0; c0 < k; c0 += kCentTile) {
    const int nc = min(kCentTile, k - c0);
    __syncthreads();
    for (int i = threadIdx.x; i < kCentTile * D; i += kAssignThreads) {
      const int c = i / D, d = i % D;
      cT[d][c] = (c < nc) ? cent[(static_cast<int64_t>(g) * k + c0 + c) * D + d] : 0.f;
    }
    __syncthreads();
    if (threadIdx.x < kCentTile) {
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = __fmaf_rn(cT[d][threadIdx.x], cT[d][threadIdx.x], acc);
      c2[threadIdx.x] = acc;
    }
    __syncthreads();
    for (int cc = 0; cc < nc; cc += 8) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int i = 0; i < D / 2; ++i) {
        const float v0 = __uint_as_float(row[i] << 16);
        const float v1 = __uint_as_float(row[i] & 0xffff0000u);
        const float4 a0 = *reinterpret_cast<const float4*>(&cT[2 * i][cc]);
        const float4 a1 = *reinterpret_cast<const float4*>(&cT[2 * i][cc + 4]);
        const float4 b0 = *reinterpret_cast<const float4*>(&cT[2 * i + 1][cc]);
        const float4 b1 = *reinterpret_cast<const float4*>(&cT[2 * i + 1][cc + 4]);
        acc[0] = __fmaf_rn(v0, a0.x, acc[0]); acc[1] = __fmaf_rn(v0, a0.y, acc[1]);
        acc[2] = __fmaf_rn(v0, a0.z, acc[2]); acc[3] = __fmaf_rn(v0, a0.w, acc[3]);
        acc[4] = __fmaf_rn(v0, a1.x, acc[4]); acc[5] = __fmaf_rn(v0, a1.y, acc[5]);
        acc[6] = __fmaf_rn(v0, a1.z, acc[6]); acc[7] = __fmaf_rn(v0, a1.w, acc[7]);
        acc[0] = __fmaf_rn(v1, b0.x, acc[0]); acc[1] = __fmaf_rn(v1, b0.y, acc[1]);
        acc[2] = __fmaf_rn(v1, b0.z, acc[2]); acc[3] = __fmaf_rn(v1, b0.w, acc[3]);
        acc[4] = __fmaf_rn(v1, b1.x, acc[4]); acc[5] = __fmaf_rn(v1, b1.y, acc[5]);
        acc[6] = __fmaf_rn(v1, b1.z, acc[6]); acc[7] = __fmaf_rn(v1, b1.w, acc[7]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (cc + j < nc) {
          const float sim = __fsub_rn(__fmul_rn(bf16_round(acc[j]), 2.0f), c2[cc + j]);
          if (sim > best) { best = sim; label = c0 + cc + j; }
        }
      }
    }
  }
  // Counting-sort histogram: one chunk per warp.
  const unsigned live_mask = __ballot_sync(0xffffffffu, live);
  if (live) {
    labels[static_cast<int64_t>(g) * N + t] = label;
    const int key = label + (key_offset ? key_offset[t] : 0);
    const unsigned same = __match_any_sync(live_mask, key);
    const int lane = threadIdx.x & 31;
    // Keys outside [0, nkeys) (a malformed key_offset) are dropped, never written.
    if ((same & ((1u << lane) - 1u)) == 0u && key >= 0 && key < nkeys) {
      const int chunk = t / kChunk;
      counts[(static_cast<int64_t>(g) * nkeys + key) * nchunks + chunk] = __popc(same);
    }
  }
}

// Exclusive scan of counts[g] in (key, chunk) order, per head, in three
// data-parallel steps over tiles of kScanTile entries: tile sums, a scan of
// the tile sums per head, then each tile's scan plus its offset.
constexpr int kScanThreads = 256;
constexpr int kScanPer = 16;                            // entries per thread
constexpr int kScanTile = kScanThreads * kScanPer;      // 4096

__device__ __forceinline__ int32_t block_sum256(int32_t x) {
  __shared__ int32_t ws[kScanThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = x;
  __syncthreads();
  int32_t t = 0;
#pragma unroll
  for (int w = 0; w < kScanThreads / 32; ++w) t += ws[w];
  return t;
}

__global__ void __launch_bounds__(kScanThreads) scan_tile_sum_kernel(const int32_t* __restrict__ counts,
                                                                     int64_t len, int ntiles,
                                                                     int32_t* __restrict__ tsum) {
  const int g = blockIdx.y, tile = blockIdx.x;
  const int32_t* c = counts + static_cast<int64_t>(g) * len;
  const int64_t base = static_cast<int64_t>(tile) * kScanTile;
  int32_t x = 0;
#pragma unroll
  for (int j = 0; j < kScanPer; ++j) {
    const int64_t i = base + j * kScanThreads + threadIdx.x;   // coalesced
    if (i < len) x += c[i];
  }
  x = block_sum256(x);
  if (threadIdx.x == 0) tsum[static_cast<int64_t>(g) * ntiles + tile] = x;
}

// Exclusive scan of the ntiles tile sums of one head, in place (one CTA per head).
__global__ void __launch_bounds__(1024) scan_tiles_kernel(int32_t* __restrict__ tsum, int ntiles) {
  __shared__ int32_t part[1024];
  int32_t* ts = tsum + static_cast<int64_t>(blockIdx.x) * ntiles;
  int32_t carry = 0;
  for (int b = 0; b < ntiles; b += 1024) {
    const int i = b + threadIdx.x;
    const int32_t v = i < ntiles ? ts[i] : 0;
    part[threadIdx.x] = v;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
      const int32_t x = (threadIdx.x >= off) ? part[threadIdx.x - off] : 0;
      __syncthreads();
      part[threadIdx.x] += x;
      __syncthreads();
    }
    if (i < ntiles) ts[i] = carry + part[threadIdx.x] - v;
    const int32_t total = part[1023];
    __syncthreads();
    carry += total;
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const int32_t* __restrict__ counts,
                                                                  int64_t len, int ntiles,
                                                                  const int32_t* __restrict__ tsum,
                                                                  int32_t* __restrict__ offsets) {
  __shared__ int32_t wsum[kScanThreads / 32];
  const int g = blockIdx.y, tile = blockIdx.x;
  const int32_t* c = counts + static_cast<int64_t>(g) * len;
  int32_t* o = offsets + static_cast<int64_t>(g) * len;
  const int64_t base = static_cast<int64_t>(tile) * kScanTile + static_cast<int64_t>(threadIdx.x) * kScanPer;
  int32_t v[kScanPer];
  int32_t run = 0;
#pragma unroll
  for (int j = 0; j < kScanPer; ++j) {
    v[j] = (base + j < len) ? c[base + j] : 0;
    run += v[j];
  }
  // exclusive scan of the thread totals: warp shuffles, then warp totals
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t inc = run;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += y;
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  int32_t wpre = 0;
#pragma unroll
  for (int w = 0; w < kScanThreads / 32; ++w) wpre += (w < warp) ? wsum[w] : 0;
  int32_t acc = tsum[static_cast<int64_t>(g) * ntiles + tile] + wpre + inc - run;
#pragma unroll
  for (int j = 0; j < kScanPer; ++j) {
    if (base + j < len) o[base + j] = acc;
    acc += v[j];
  }
}

// Stable scatter: position = offset(key, chunk) + rank among equal keys in the warp.
__global__ void __launch_bounds__(kAssignThreads) scatter_kernel(
    const int32_t* __restrict__ labels, const int32_t* __restrict__ key_offset, int N, int nkeys,
    int nchunks, const int32_t* __restrict__ offsets, int32_t* __restrict__ sorted) {
  const int g = blockIdx.y;
  const int t = blockIdx.x * kAssignThreads + threadIdx.x;
  const bool live = t < N;
  const unsigned live_mask = __ballot_sync(0xffffffffu, live);
  if (!live) return;
  const int key = labels[static_cast<int64_t>(g) * N + t] + (key_offset ? key_offset[t] : 0);
  const unsigned same = __match_any_sync(live_mask, key);
  const int lane = threadIdx.x & 31;
  const int rank = __popc(same & ((1u << lane) - 1u));
  if (key < 0 || key >= nkeys) return;
  const int pos = offsets[(static_cast<int64_t>(g) * nkeys + key) * nchunks + t / kChunk] + rank;
  if (pos >= 0 && pos < N) sorted[static_cast<int64_t>(g) * N + pos] = t;
}

// Clusters above kBigCluster members with bf16 rows at 16-byte aligned
// strides are summed by the BIG launch, which stages member rows in shared
// memory; the other launch leaves them out.
constexpr int kBigCluster = 512;
constexpr int kStageM = 64;   // member rows per staged batch (64 x 256 B)

__device__ __forceinline__ bool staged_rows_ok(const vcattn_bhnd& v, int D) {
  const uint64_t bits = reinterpret_cast<uint64_t>(v.data) | static_cast<uint64_t>(v.sb * 2) |
                        static_cast<uint64_t>(v.sh * 2) | static_cast<uint64_t>(v.sn * 2);
  return D == 128 && (bits & 15u) == 0 && v.sb >= 0 && v.sh >= 0 && v.sn >= 0;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// grouping.py:103-124: fp32 sums in token order, / max(count, 1), re-seed
// clusters with count <= 1, bf16.  One CTA per (cluster, head), D threads,
// thread = channel.
template <int DT, bool BIG>
__global__ void update_kernel(vcattn_bhnd v, int H, int N, int D, int k, int nchunks,
                              const int32_t* __restrict__ offsets, const int32_t* __restrict__ sorted,
                              const float* __restrict__ seeds, float* __restrict__ cent,
                              uint16_t* __restrict__ cent_out, uint16_t* __restrict__ cb16, float* __restrict__ c2) {
  const int g = blockIdx.y, c = blockIdx.x, d = threadIdx.x;
  const int b = g / H, h = g % H;
  const int64_t base = static_cast<int64_t>(g) * k * nchunks;
  const int start = offsets[base + static_cast<int64_t>(c) * nchunks];
  const int end = (c + 1 < k) ? offsets[base + static_cast<int64_t>(c + 1) * nchunks] : N;
  const int32_t* mem = sorted + static_cast<int64_t>(g) * N;
  const bool big = DT == VCATTN_DTYPE_BF16 && end - start > kBigCluster && staged_rows_ok(v, D);
  if (big != BIG) return;   // uniform per CTA: the other launch owns this cluster
  float acc = 0.f;
  if constexpr (BIG && DT == VCATTN_DTYPE_BF16) {
    // Member rows in batches of kStageM, gathered into shared memory with
    // cp.async (16 bytes per copy) while the previous batch is summed; each
    // thread adds its channel of the staged rows in member order, so the sum
    // is the same sequence of fp32 adds as the direct loop below.
    __shared__ __align__(16) uint16_t rows[2][kStageM][128];
    __shared__ int sidx[2][kStageM];
    const __nv_bfloat16* vb = static_cast<const __nv_bfloat16*>(v.data) + b * v.sb + h * v.sh;
    const int cnt = end - start;
    const int nbatch = (cnt + kStageM - 1) / kStageM;
    auto member = [&](int bt) -> int {
      const int m = start + bt * kStageM + d;
      return (d < kStageM && bt < nbatch && m < end) ? mem[m] : 0;
    };
    auto issue = [&](int bt, int buf) {
      const int nm = min(kStageM, cnt - bt * kStageM);
      for (int q = d; q < nm * 16; q += 128) {
        const int u = q >> 4, ch = q & 15;
        cp_async16(&rows[buf][u][ch * 8], vb + static_cast<int64_t>(sidx[buf][u]) * v.sn + ch * 8);
      }
      cp_async_commit();
    };
    if (d < kStageM) sidx[0][d] = member(0);
    __syncthreads();
    issue(0, 0);
    int pend = member(1);
    for (int bt = 0; bt < nbatch; ++bt) {
      const int cur = bt & 1;
      if (bt + 1 < nbatch) {
        if (d < kStageM) sidx[cur ^ 1][d] = pend;
        __syncthreads();
        issue(bt + 1, cur ^ 1);
        pend = member(bt + 2);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const int nm = min(kStageM, cnt - bt * kStageM);
      for (int u = 0; u < nm; ++u) acc = __fadd_rn(acc, __uint_as_float(static_cast<uint32_t>(rows[cur][u][d]) << 16));
      __syncthreads();   // rows[cur] is refilled by the next iteration's copies
    }
  } else {
  // The sum runs in member order (one fp32 add after another); only the
  // loads run ahead: kB member values are in flight per batch, and the next
  // batch's member indices are fetched while the current values arrive, so a
  // large cluster costs about one memory round trip per kB members.
  constexpr int kB = 8;
  int nid[kB];
#pragma unroll
  for (int u = 0; u < kB; ++u) nid[u] = (start + u < end) ? mem[start + u] : 0;
  for (int i = start; i < end; i += kB) {
    float x[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) x[u] = (i + u < end) ? load_bf16_value<DT>(v, b, h, nid[u], d) : 0.f;
    const int in = i + kB;
#pragma unroll
    for (int u = 0; u < kB; ++u) nid[u] = (in + u < end) ? mem[in + u] : 0;
#pragma unroll
    for (int u = 0; u < kB; ++u)
      if (i + u < end) acc = __fadd_rn(acc, x[u]);
  }
  }
  const int cnt = end - start;
  const int64_t o = (static_cast<int64_t>(g) * k + c) * D + d;
  const float cntc = static_cast<float>(cnt > 1 ? cnt : 1);
  const float nv = (cnt <= 1) ? seeds[o] : bf16_round(__fdiv_rn(acc, cntc));
  cent[o] = nv;
  if (cent_out) cent_out[o] = __bfloat16_as_ushort(__float2bfloat16_rn(nv));
  centroid_side(nv, D, static_cast<int64_t>(g) * k + c, cb16, c2);
}

__global__ void copy_centroids_kernel(const float* __restrict__ cent, uint16_t* __restrict__ out, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(cent[i]));
}

template <int DT, int D>
cudaError_t kmeans_impl(const KMeansParams& p, cudaStream_t st) {
  const int G = p.B * p.H;
  const int k = p.k;
  const int nkeys = p.key_offset ? p.nkeys : k;
  const int nchunks = (p.N + kChunk - 1) / kChunk;
  KmWs w = carve(p.workspace, G, p.N, D, k, nkeys);
  int32_t* labels = p.labels_out ? p.labels_out : w.labels;
  const int m = (p.N < 4 * k) ? p.N : 4 * k;          // init_samples_per_centroid = 4
  const int m_per = (m / k) > 1 ? (m / k) : 1;
  seed_kernel<DT><<<dim3(k, G), D, 0, st>>>(*p.v, p.H, p.N, D, k, m, m_per, w.seeds, w.cent, p.warm, w.cb16,
                                            w.c2);
  const dim3 agrid((p.N + kAssignThreads - 1) / kAssignThreads, G, 1);
  // Tensor-core assignment when the token rows can be tiled by TMA (bf16,
  // D = 128); the CUDA-core kernel otherwise.  Both give the same labels.
  alignas(64) unsigned char maps[256];
  const bool tc = assign_tc_supported(p) && assign_tc_maps(p, w.cb16, maps);
  cudaError_t err = cudaSuccess;
  auto sort_pass = [&](const int32_t* koff, int nkey, int32_t* out_sorted) {
    const size_t cnt_bytes = sizeof(int32_t) * static_cast<size_t>(G) * nkey * nchunks;
    cudaMemsetAsync(w.counts, 0, cnt_bytes, st);
    if (tc) {
      const cudaError_t e = launch_assign_tc(p, maps, w.c2, labels, koff, nkey, nchunks, w.counts, st);
      if (e != cudaSuccess && err == cudaSuccess) err = e;
    } else {
      assign_kernel<DT, D><<<agrid, kAssignThreads, 0, st>>>(
          *p.v, p.H, p.N, k, w.cent, labels, koff, nkey, nchunks, w.counts);
    }
    const int64_t len = static_cast<int64_t>(nkey) * nchunks;
    const int ntiles = static_cast<int>((len + kScanTile - 1) / kScanTile);
    scan_tile_sum_kernel<<<dim3(ntiles, G), kScanThreads, 0, st>>>(w.counts, len, ntiles, w.tsum);
    scan_tiles_kernel<<<G, 1024, 0, st>>>(w.tsum, ntiles);
    scan_apply_kernel<<<dim3(ntiles, G), kScanThreads, 0, st>>>(w.counts, len, ntiles, w.tsum, w.offsets);
    scatter_kernel<<<dim3(agrid.x, G), kAssignThreads, 0, st>>>(labels, koff, p.N, nkey, nchunks,
                                                              w.offsets, out_sorted);
  };
  const int iters = p.iters;
  for (int it = 0; it < iters; ++it) {
    sort_pass(nullptr, k, p.perm_out);
    update_kernel<DT, false><<<dim3(k, G), D, 0, st>>>(*p.v, p.H, p.N, D, k, nchunks, w.offsets, p.perm_out,
                                                      w.seeds, w.cent, nullptr, w.cb16, w.c2);
    if constexpr (DT == VCATTN_DTYPE_BF16)
      update_kernel<DT, true><<<dim3(k, G), D, 0, st>>>(*p.v, p.H, p.N, D, k, nchunks, w.offsets, p.perm_out,
                                                       w.seeds, w.cent, nullptr, w.cb16, w.c2);
  }
  copy_centroids_kernel<<<static_cast<unsigned>((static_cast<int64_t>(G) * k * D + 255) / 256), 256, 0, st>>>(
      w.cent, p.centroids_out, static_cast<int64_t>(G) * k * D);
  sort_pass(p.key_offset, nkeys, p.perm_out);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace

size_t kmeans_workspace_bytes(int G, int N, int D, int k, int nkeys) {
  const size_t nchunks = (N + kChunk - 1) / kChunk;
  const size_t nk = static_cast<size_t>(nkeys > k ? nkeys : k);
  return align256(sizeof(int32_t) * G * static_cast<size_t>(N)) +
         2 * align256(sizeof(int32_t) * G * nk * nchunks) +
         2 * align256(sizeof(float) * G * static_cast<size_t>(k) * D) +
         align256(sizeof(uint16_t) * G * static_cast<size_t>(k) * D) + align256(sizeof(float) * G * static_cast<size_t>(k)) +
         align256(sizeof(int32_t) * G * ((nk * nchunks + 4095) / 4096)) + 256;
}

cudaError_t launch_kmeans(const KMeansParams& p, cudaStream_t st) {
  if (p.D == 128) {
    switch (p.dtype) {
      case VCATTN_DTYPE_BF16: return kmeans_impl<VCATTN_DTYPE_BF16, 128>(p, st);
      case VCATTN_DTYPE_F16: return kmeans_impl<VCATTN_DTYPE_F16, 128>(p, st);
      default: return kmeans_impl<VCATTN_DTYPE_F32, 128>(p, st);
    }
  }
  switch (p.dtype) {
    case VCATTN_DTYPE_BF16: return kmeans_impl<VCATTN_DTYPE_BF16, 64>(p, st);
    case VCATTN_DTYPE_F16: return kmeans_impl<VCATTN_DTYPE_F16, 64>(p, st);
    default: return kmeans_impl<VCATTN_DTYPE_F32, 64>(p, st);
  }
}

}  // namespace vcattn
