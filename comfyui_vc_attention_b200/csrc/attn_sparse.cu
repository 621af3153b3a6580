// Fused block-sparse FP8 VC-Attention (triton_attn.py:384-501), register MMA.
//
// One CTA = 64 query rows = one routing query block, so the keep mask
// (vcattn_route_mask) is uniform across the CTA.  KV blocks are walked in
// groups of 16, in the reference's order:
//   1. the group's approximated blocks are folded at once: per-row proxy
//      s_ap = (q8 . bf16(k_mean_j)) * (qs * sm_scale) from a bf16 MMA, the
//      running max and alpha updated over them, p_ap = exp2((s_ap - m) log2e)
//      weighted by the block's real length, o = alpha o + bf16(p_ap) @
//      bf16(v_mean), l = alpha l + rowsum(p_ap);
//   2. the group's kept blocks run the exact tile, in increasing order.
// Kept tiles stream through the same double-buffered cp.async stages as the
// dense kernel; skipped blocks are never loaded.
#include "mma_common.cuh"

namespace vcattn {
namespace {

using namespace mmak;

constexpr int kGroup = 16;
constexpr int kKmStride = 8;   // bf16 padding per k_mean row (bank spread)

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two E4M3 bytes (low byte first) -> bf16x2, exact (E4M3 values are bf16 values).
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint32_t two) {
  const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two & 0xffff), __NV_E4M3);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
  const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<const uint32_t*>(&b);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}

template <int D>
struct SparseSmem {
  // bf16 k_mean rows of the group [kGroup][D + pad] and v_mean transposed [D][kGroup]
  static constexpr int kKmBytes = kGroup * (D + kKmStride) * 2;
  static constexpr int kVmBytes = D * kGroup * 2;
};

// Fold the approximated blocks of group `gi` (triton_attn.py:449-486).
template <int BR, int D>
__device__ __forceinline__ void approx_group(const AttnParams& p, int g, int gi, int nb, const uint8_t* keep_row,
                                             uint16_t* kmb, uint16_t* vmbT, const uint32_t (&qa)[D / 32][4],
                                             float qsm0, float qsm1, int tid, int gid, int tig,
                                             float (&o)[D / 8][4], float (&m_i)[2], float (&l_i)[2]) {
  const int b0 = gi * kGroup;
  // Is any block of the group approximated?  (uniform across the CTA)
  bool any = false;
  for (int j = 0; j < kGroup; ++j) {
    const int blk = b0 + j;
    if (blk < nb && keep_row[blk] == 0) any = true;
  }
  if (!any) return;
  __syncthreads();   // previous users of the k_mean / v_mean tiles are done
  const float* km = p.k_mean + (static_cast<int64_t>(g) * nb + b0) * D;
  const float* vm = p.v_mean + (static_cast<int64_t>(g) * nb + b0) * D;
  for (int i = tid; i < kGroup * D; i += kWarps * 32) {
    const int j = i / D, d = i % D;
    const bool ok = b0 + j < nb;
    const float kv = ok ? km[static_cast<int64_t>(j) * D + d] : 0.f;
    const float vv = ok ? vm[static_cast<int64_t>(j) * D + d] : 0.f;
    kmb[j * (D + kKmStride) + d] = __bfloat16_as_ushort(__float2bfloat16_rn(kv));
    vmbT[d * kGroup + j] = __bfloat16_as_ushort(__float2bfloat16_rn(vv));
  }
  __syncthreads();
  // ---- per-row proxy: (16 rows x 16 blocks) per warp, bf16 MMA over D ----
  float pc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
  for (int kk = 0; kk < D / 32; ++kk) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      // E4M3 bytes d = 32kk + 16 half + 4 tig + {0..3} of rows gid / gid+8
      const uint32_t r0 = qa[kk][half * 2], r1 = qa[kk][half * 2 + 1];
      const uint32_t a0 = e4m3x2_to_bf16x2(r0), a2 = e4m3x2_to_bf16x2(r0 >> 16);
      const uint32_t a1 = e4m3x2_to_bf16x2(r1), a3 = e4m3x2_to_bf16x2(r1 >> 16);
      const int dbase = 32 * kk + 16 * half + 4 * tig;
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const uint16_t* kr = kmb + (n * 8 + gid) * (D + kKmStride) + dbase;
        const uint32_t bb0 = *reinterpret_cast<const uint32_t*>(kr);
        const uint32_t bb1 = *reinterpret_cast<const uint32_t*>(kr + 2);
        mma_bf16(pc[n], a0, a1, a2, a3, bb0, bb1);
      }
    }
  }
  // ---- scores of the approximated blocks, max, alpha --------------------
  float sap[2][4];
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int blk = b0 + n * 8 + tig * 2 + e;
      const bool ap = blk < nb && keep_row[blk] == 0;
      sap[n][e] = ap ? __fmul_rn(pc[n][e], qsm0) : -INFINITY;
      sap[n][2 + e] = ap ? __fmul_rn(pc[n][2 + e], qsm1) : -INFINITY;
      mx0 = fmaxf(mx0, sap[n][e]);
      mx1 = fmaxf(mx1, sap[n][2 + e]);
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
  // ---- p_ap = exp2(s_ap - m) * block length -----------------------------
  float pap[2][4];
  float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int blk = b0 + n * 8 + tig * 2 + e;
      const bool ap = blk < nb && keep_row[blk] == 0;
      const float len = ap ? static_cast<float>(min(BR, p.N - blk * BR)) : 0.f;
      const float p0 = ap ? exp2f(__fmul_rn(__fsub_rn(sap[n][e], mn[0]), kLog2e)) : 0.f;
      const float p1 = ap ? exp2f(__fmul_rn(__fsub_rn(sap[n][2 + e], mn[1]), kLog2e)) : 0.f;
      pap[n][e] = __fmul_rn(p0, len);
      pap[n][2 + e] = __fmul_rn(p1, len);
      ls0 += pap[n][e];
      ls1 += pap[n][2 + e];
    }
  }
  ls0 += __shfl_xor_sync(0xffffffffu, ls0, 1);
  ls0 += __shfl_xor_sync(0xffffffffu, ls0, 2);
  ls1 += __shfl_xor_sync(0xffffffffu, ls1, 1);
  ls1 += __shfl_xor_sync(0xffffffffu, ls1, 2);
  // ---- o = alpha o + bf16(p_ap) @ bf16(v_mean) ---------------------------
  const uint32_t a0 = pack_bf16x2(pap[0][0], pap[0][1]), a1 = pack_bf16x2(pap[0][2], pap[0][3]);
  const uint32_t a2 = pack_bf16x2(pap[1][0], pap[1][1]), a3 = pack_bf16x2(pap[1][2], pap[1][3]);
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) {
    float t[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t* vr = vmbT + (nd * 8 + gid) * kGroup + tig * 2;
    mma_bf16(t, a0, a1, a2, a3, *reinterpret_cast<const uint32_t*>(vr), *reinterpret_cast<const uint32_t*>(vr + 8));
    o[nd][0] = __fadd_rn(__fmul_rn(o[nd][0], alpha[0]), t[0]);
    o[nd][1] = __fadd_rn(__fmul_rn(o[nd][1], alpha[0]), t[1]);
    o[nd][2] = __fadd_rn(__fmul_rn(o[nd][2], alpha[1]), t[2]);
    o[nd][3] = __fadd_rn(__fmul_rn(o[nd][3], alpha[1]), t[3]);
  }
  l_i[0] = __fadd_rn(__fmul_rn(l_i[0], alpha[0]), ls0);
  l_i[1] = __fadd_rn(__fmul_rn(l_i[1], alpha[1]), ls1);
  m_i[0] = mn[0];
  m_i[1] = mn[1];
}

template <int BR, int D, bool EXPCAST, int ODT>
__global__ void __launch_bounds__(kWarps * 32) attn_sparse_kernel(AttnParams p) {
  using S = TileSmem<BR, D>;
  using SS = SparseSmem<D>;
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* kmb = reinterpret_cast<uint16_t*>(smem + 2 * S::kStage);
  uint16_t* vmbT = reinterpret_cast<uint16_t*>(smem + 2 * S::kStage + SS::kKmBytes);
  int* kept = reinterpret_cast<int*>(smem + 2 * S::kStage + SS::kKmBytes + SS::kVmBytes);
  __shared__ int nkept_s;

  const int g = blockIdx.y, qi = blockIdx.x;
  const int b = g / p.H, h = g % p.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int row0 = qi * kRowsPerCta + warp * 16;
  const int nb = p.n_pad / BR;
  const int nqb = p.n_pad / p.q_block;
  const uint8_t* keep_row = p.keep + (static_cast<int64_t>(g) * nqb + qi) * nb;

  // Ordered list of the kept blocks (warp 0, ballot compaction).
  if (warp == 0) {
    int cnt = 0;
    for (int base = 0; base < nb; base += 32) {
      const int blk = base + lane;
      const bool k = blk < nb && keep_row[blk] != 0;
      const unsigned m = __ballot_sync(0xffffffffu, k);
      if (k) kept[cnt + __popc(m & ((1u << lane) - 1u))] = blk;
      cnt += __popc(m);
    }
    if (lane == 0) nkept_s = cnt;
  }

  uint32_t qa[D / 32][4];
  {
    const uint8_t* q0 = p.q8 + (static_cast<int64_t>(g) * p.n_pad + row0 + gid) * D;
    const uint8_t* q1 = q0 + 8 * D;
#pragma unroll
    for (int kk = 0; kk < D / 32; ++kk) {
      qa[kk][0] = *reinterpret_cast<const uint32_t*>(q0 + kk * 32 + tig * 4);
      qa[kk][1] = *reinterpret_cast<const uint32_t*>(q1 + kk * 32 + tig * 4);
      qa[kk][2] = *reinterpret_cast<const uint32_t*>(q0 + kk * 32 + 16 + tig * 4);
      qa[kk][3] = *reinterpret_cast<const uint32_t*>(q1 + kk * 32 + 16 + tig * 4);
    }
  }
  const float qs0 = p.q_scale[static_cast<int64_t>(g) * p.n_pad + row0 + gid];
  const float qs1 = p.q_scale[static_cast<int64_t>(g) * p.n_pad + row0 + gid + 8];
  const float qsm0 = __fmul_rn(qs0, p.sm_scale), qsm1 = __fmul_rn(qs1, p.sm_scale);
  const float c0 = static_cast<float>(56.0 + p.beta);

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_i[2] = {-INFINITY, -INFINITY};
  float l_i[2] = {0.f, 0.f};

  __syncthreads();
  const int nkept = nkept_s;
  const int ngroups = (nb + kGroup - 1) / kGroup;
  if (nkept > 0) load_tile<BR, D>(smem, p, g, kept[0], tid);
  cp_async_commit();
  int next_group = 0;
  for (int ki = 0; ki < nkept; ++ki) {
    const int blk = kept[ki];
    const int grp = blk / kGroup;
    while (next_group <= grp) {
      approx_group<BR, D>(p, g, next_group, nb, keep_row, kmb, vmbT, qa, qsm0, qsm1, tid, gid, tig, o, m_i, l_i);
      ++next_group;
    }
    uint8_t* st = smem + (ki & 1) * S::kStage;
    if (ki + 1 < nkept) load_tile<BR, D>(smem + ((ki + 1) & 1) * S::kStage, p, g, kept[ki + 1], tid);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    exact_tile<BR, D, EXPCAST>(st, qa, qs0, qs1, blk * BR, p.N, p.sm_scale, c0, tid, gid, tig, o, m_i, l_i);
    __syncthreads();
  }
  while (next_group < ngroups) {
    approx_group<BR, D>(p, g, next_group, nb, keep_row, kmb, vmbT, qa, qsm0, qsm1, tid, gid, tig, o, m_i, l_i);
    ++next_group;
  }
  cp_async_wait<0>();
  // ---- epilogue ----------------------------------------------------------
  const int ra = row0 + gid, rb = row0 + gid + 8;
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) {
    const int col = nd * 8 + tig * 2;
    if (ra < p.N)
      store_out2<ODT>(p.out, b * p.osb + h * p.osh + static_cast<int64_t>(ra) * p.osn + col,
                      __fdiv_rn(o[nd][0], l_i[0]), __fdiv_rn(o[nd][1], l_i[0]));
    if (rb < p.N)
      store_out2<ODT>(p.out, b * p.osb + h * p.osh + static_cast<int64_t>(rb) * p.osn + col,
                      __fdiv_rn(o[nd][2], l_i[1]), __fdiv_rn(o[nd][3], l_i[1]));
  }
}

template <int BR, int D, bool EXPCAST, int ODT>
cudaError_t launch_one(const AttnParams& p, cudaStream_t st) {
  using S = TileSmem<BR, D>;
  using SS = SparseSmem<D>;
  const int nb = p.n_pad / BR;
  const size_t smem = 2 * S::kStage + SS::kKmBytes + SS::kVmBytes + static_cast<size_t>(nb) * sizeof(int);
  auto k = attn_sparse_kernel<BR, D, EXPCAST, ODT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid(p.n_pad / kRowsPerCta, p.B * p.H);
  k<<<grid, kWarps * 32, smem, st>>>(p);
  return cudaGetLastError();
}

template <int BR, int D>
cudaError_t dispatch(const AttnParams& p, cudaStream_t st) {
  const bool ec = (p.flags & VCATTN_EXPCAST) != 0;
  switch (p.out_dtype) {
    case VCATTN_DTYPE_BF16:
      return ec ? launch_one<BR, D, true, VCATTN_DTYPE_BF16>(p, st) : launch_one<BR, D, false, VCATTN_DTYPE_BF16>(p, st);
    case VCATTN_DTYPE_F16:
      return ec ? launch_one<BR, D, true, VCATTN_DTYPE_F16>(p, st) : launch_one<BR, D, false, VCATTN_DTYPE_F16>(p, st);
    default:
      return ec ? launch_one<BR, D, true, VCATTN_DTYPE_F32>(p, st) : launch_one<BR, D, false, VCATTN_DTYPE_F32>(p, st);
  }
}

}  // namespace

cudaError_t launch_attn_sparse_mma(const AttnParams& p, cudaStream_t st) {
  if (p.q_block != kRowsPerCta || p.group != kGroup) return cudaErrorInvalidValue;
  if (p.D == 128) return p.block_rows == 128 ? dispatch<128, 128>(p, st) : dispatch<64, 128>(p, st);
  return p.block_rows == 128 ? dispatch<128, 64>(p, st) : dispatch<64, 64>(p, st);
}

}  // namespace vcattn
