// Fused dense FP8 VC-Attention, register-MMA form (mma.sync m16n8k32 E4M3).
//
// Semantics of triton_attn.py:203-322 (one KV tile == one value block):
//   s    = dot(q8, k8) * (qs * ks) * sm_scale        (invalid keys -> -1e30)
//   m'   = max(m, rowmax(s)); alpha = exp2((m - m') * log2e)
//   P    = E4M3(exp2((s - m') * log2e) * 448)   or the ExpCast byte
//   r    = rowsum(P) / 448
//   acc  = alpha * acc + (P @ V8) * (vs / 448) + r * (mu * vs)
//   l    = alpha * l + r ;  O = acc / l
//
// CTA = 4 warps x 16 query rows.  K and the block-transposed V codes of each
// KV tile are staged in shared memory by cp.async (double buffered).  The
// S accumulator layout of m16n8k32 is reused directly as the A operand of the
// PV product by visiting keys in the order (32s + 2t + {0,1}, 32s + 8 + 2t +
// {0,1}) within each 32-key step; the V operand is read in the same order.
#include "mma_common.cuh"

namespace vcattn {
namespace {

using namespace mmak;

template <int BR, int D, bool EXPCAST, int ODT>
__global__ void __launch_bounds__(kWarps * 32) attn_mma_kernel(AttnParams p) {
  using S = TileSmem<BR, D>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int g = blockIdx.y;
  const int b = g / p.H, h = g % p.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int row0 = blockIdx.x * kRowsPerCta + warp * 16;
  const int nb = p.n_pad / BR;

  // Q fragments for the warp's 16 rows (rows >= n_pad never occur: n_pad is a
  // multiple of 64 and the grid covers n_pad).
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
  const float c0 = static_cast<float>(56.0 + p.beta);

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_i[2] = {-INFINITY, -INFINITY};
  float l_i[2] = {0.f, 0.f};

  load_tile<BR, D>(smem, p, g, 0, tid);
  cp_async_commit();
  for (int j = 0; j < nb; ++j) {
    uint8_t* st = smem + (j & 1) * S::kStage;
    if (j + 1 < nb) load_tile<BR, D>(smem + ((j + 1) & 1) * S::kStage, p, g, j + 1, tid);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    exact_tile<BR, D, EXPCAST>(st, qa, qs0, qs1, j * BR, p.N, p.sm_scale, c0, tid, gid, tig, o, m_i, l_i);
    __syncthreads();   // the stage is refilled next iteration
  }
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
  const size_t smem = 2 * S::kStage;
  auto k = attn_mma_kernel<BR, D, EXPCAST, ODT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid(p.n_pad / kRowsPerCta, p.B * p.H);
  k<<<grid, kWarps * 32, smem, st>>>(p);
  return cudaGetLastError();
}

template <int BR, int D>
cudaError_t dispatch_flags(const AttnParams& p, cudaStream_t st) {
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

cudaError_t launch_attn_mma(const AttnParams& p, cudaStream_t st) {
  if (p.D == 128) return p.block_rows == 128 ? dispatch_flags<128, 128>(p, st) : dispatch_flags<64, 128>(p, st);
  return p.block_rows == 128 ? dispatch_flags<128, 64>(p, st) : dispatch_flags<64, 64>(p, st);
}

}  // namespace vcattn
