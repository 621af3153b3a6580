// Internal launcher interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include "common.cuh"

namespace vcattn {

struct PrepareParams {
  const vcattn_bhnd *q, *k, *v;
  int dtype, B, H, N, D, n_pad, block_rows, flags;
  const int32_t* perm;
  int perm_rows;
  uint8_t *q8, *k8, *v8, *v8t;
  float *q_scale, *k_scale, *v_scale, *mu, *v_mean;
  const vcattn_route_stats* route;
  void* workspace;
};

// NVFP4 Q / K (no V): the kernels reuse the prepare workspace (K mean,
// per-head maxima).
struct NvfpParams {
  const vcattn_bhnd *q, *k;
  int dtype, B, H, N, D, n_pad, block_rows, flags;
  const int32_t* perm;
  int perm_rows;
  uint8_t *q4, *q4_scale, *k4, *k4_scale;
  uint8_t *q4_sf_mma, *k4_sf_mma;   // scale-factor atoms of the block-scaled MMA, or nullptr
  float *q4_g, *k4_g;
  void* workspace;
};

struct RouteParams {
  const float *k_mean, *q_cent, *q_bar;
  int G, N, n_pad, D, block_rows, q_block;
  float tau, sm_scale;
  int local_blocks, sink_blocks;
  uint8_t* keep;
  float* thresh;
};

struct KMeansParams {
  const vcattn_bhnd* v;
  int dtype, B, H, N, D, k, iters;
  const uint16_t* warm;
  const int32_t* key_offset;
  int nkeys;
  uint16_t* centroids_out;
  int32_t* perm_out;
  int32_t* labels_out;
  void* workspace;
};

struct AttnParams {
  const uint8_t *q8, *k8, *v8, *v8t;
  const float *q_scale, *k_scale, *v_scale, *mu;
  // block-sparse extras (nullptr for the dense kernel)
  const float *k_mean, *v_mean;
  const uint8_t* keep;
  const uint8_t* ap_tiles;   // bf16 proxy tiles (vcattn_route_tiles) of the tcgen05 sparse kernel
  int q_block, group;
  // NVFP4 QK^T (nullptr for the FP8 kernels)
  const uint8_t *q4, *k4, *q4_sf, *k4_sf;
  const float *q4_g, *k4_g;
  int B, H, N, n_pad, D, block_rows;
  float sm_scale;
  double beta;
  int flags;
  void* out;
  int out_dtype;
  int64_t osb, osh, osn;
  const int32_t* kv_len;   // (B,) keys taking part per batch entry (dense tcgen05 kernel), or nullptr
  // dense tcgen05 kernel, KV split of query tiles: 0 = the last partial wave
  // of CTAs (auto), 1 = none, k >= 2 = every query tile in k pieces; the
  // partials go to `part` (attn_tc_split_bytes bytes)
  int kv_split;
  void* part;
};

size_t prepare_workspace_bytes(int G, int N, int D);
size_t kmeans_workspace_bytes(int G, int N, int D, int k, int nkeys);

cudaError_t launch_prepare(const PrepareParams& p, cudaStream_t st);
cudaError_t launch_prepare_nvfp4(const NvfpParams& p, cudaStream_t st);
cudaError_t launch_route_mask(const RouteParams& p, cudaStream_t st);
cudaError_t launch_route_tiles(const float* k_mean, const float* v_mean, int G, int nb, int D, uint8_t* tiles,
                               cudaStream_t st);
cudaError_t launch_kmeans(const KMeansParams& p, cudaStream_t st);
// Tensor-core nearest-centroid assignment (kmeans_tc.cu): labels identical to
// the CUDA-core assign.  `maps` holds two CUtensorMap (256 bytes, 64-aligned):
// the token rows of p.v and the bf16 centroid table cb16 (G, k, 128).
bool assign_tc_supported(const KMeansParams& p);
bool assign_tc_maps(const KMeansParams& p, const uint16_t* cb16, void* maps);
cudaError_t launch_assign_tc(const KMeansParams& p, const void* maps, const float* c2, int32_t* labels,
                             const int32_t* key_offset, int nkeys, int nchunks, int32_t* counts, cudaStream_t st);
cudaError_t kmeans_tc_status(int* code, int* where, int* block, bool reset);
cudaError_t launch_attn_mma(const AttnParams& p, cudaStream_t st);
cudaError_t launch_attn_tc(const AttnParams& p, cudaStream_t st);
cudaError_t launch_attn_nvfp4(const AttnParams& p, cudaStream_t st);
cudaError_t attn_nvfp4_status(int* code, int* where, int* block, bool reset);
const char* attn_nvfp4_diag();
cudaError_t attn_tc_status(int* code, int* where, int* block, bool reset);
const char* attn_tc_diag();
// Bounded-wait test hook of the dense tcgen05 kernel (vcattn_inject_stall).
void set_attn_tc_stall(int tile);
size_t attn_tc_split_bytes(const AttnParams& p);
cudaError_t launch_attn_sparse_mma(const AttnParams& p, cudaStream_t st);
bool attn_sparse_tc_supported(const AttnParams& p);
cudaError_t launch_attn_sparse_tc(const AttnParams& p, cudaStream_t st);
cudaError_t attn_sparse_tc_status(int* code, int* where, int* block, bool reset);
const char* attn_sparse_tc_diag();
cudaError_t launch_codecs_e4m3(const float* x, int64_t n, uint8_t* out, cudaStream_t st);
cudaError_t launch_codecs_fp4(const float* x, int64_t n, uint8_t* out, cudaStream_t st);
cudaError_t launch_expcast(const float* s, const float* m, int rows, int cols, double beta, int mode,
                           uint8_t* out, cudaStream_t st);

}  // namespace vcattn
