// extern "C" entry points of libvcattn.so (declared in include/vcattn.h).
//
// Each entry point validates its arguments on the host, honours host-side
// fault injection, enqueues kernels on the caller's stream and returns a
// status code.  No entry point allocates device memory.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "kernels.cuh"
#include "tc_math.cuh"

namespace vcattn {

// ---------------------------------------------------------------------------
// Standalone codec kernels (bit-exact tests of the in-kernel encoders).
// ---------------------------------------------------------------------------
__global__ void e4m3_encode_kernel(const float* __restrict__ x, int64_t n, uint8_t* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = static_cast<uint8_t>(e4m3x2(x[i], 0.f) & 0xff);
}

__global__ void fp4_encode_kernel(const float* __restrict__ x, int64_t n, uint8_t* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = static_cast<uint8_t>(e2m1x2(x[i], 0.f) & 0xf);
}

// mode 1: the operation sequence of expcast.py:67-69 (what the attention
// kernel evaluates under VCATTN_EXPCAST_EXACT).
__global__ void expcast_exact_kernel(const float* __restrict__ s, const float* __restrict__ m, int rows, int cols,
                                     float c0, uint8_t* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(rows) * cols) return;
  const int r = static_cast<int>(i / cols);
  const float u = __fadd_rn(__fmul_rn(__fsub_rn(s[i], m[r]), kLog2e), 8.0f);
  const float c = fminf(fmaxf(rintf(__fmaf_rn(u, 8.0f, c0)), 0.0f), 120.0f);
  out[i] = static_cast<uint8_t>(c);
}

// mode 0: the attention kernels' own one-FMA form, through the same device
// function (tc::expcast4) and the same folding of the per-row constants: with
// the score s = x * qsm (here qsm = 1, x = s), As = 8 log2e qsm / 128 and
// Bs = fma(-As, m, (64 + 56 + beta) / 128); the code is fma.sat(x, As, Bs)
// rounded by the 98304 magic add.  Four consecutive columns per thread.
__global__ void expcast_fast_kernel(const float* __restrict__ s, const float* __restrict__ m, int rows, int cols,
                                    float c120, uint8_t* __restrict__ out) {
  const int quads = (cols + 3) / 4;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(rows) * quads) return;
  const int r = static_cast<int>(i / quads);
  const int c = static_cast<int>(i % quads) * 4;
  const float qsm = 1.0f;
  const float As = __fmul_rn(8.0f * kLog2e, qsm) * (1.0f / 128.0f);
  const float Bs = __fmaf_rn(-As, m[r], c120 * (1.0f / 128.0f));
  const float* row = s + static_cast<int64_t>(r) * cols;
  float x[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) x[e] = (c + e < cols) ? row[c + e] : -INFINITY;
  const uint32_t word = tc::expcast4(x[0], x[1], x[2], x[3], As, Bs);
  uint8_t* o = out + static_cast<int64_t>(r) * cols + c;
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (c + e < cols) o[e] = static_cast<uint8_t>(word >> (8 * e));
}

cudaError_t launch_codecs_e4m3(const float* x, int64_t n, uint8_t* out, cudaStream_t st) {
  if (n > 0) e4m3_encode_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(x, n, out);
  return cudaGetLastError();
}
cudaError_t launch_codecs_fp4(const float* x, int64_t n, uint8_t* out, cudaStream_t st) {
  if (n > 0) fp4_encode_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(x, n, out);
  return cudaGetLastError();
}
cudaError_t launch_expcast(const float* s, const float* m, int rows, int cols, double beta, int mode,
                           uint8_t* out, cudaStream_t st) {
  const float c0 = static_cast<float>(56.0 + beta);
  const float c120 = static_cast<float>(64.0 + 56.0 + beta);
  if (mode == 1) {
    const int64_t n = static_cast<int64_t>(rows) * cols;
    if (n > 0) expcast_exact_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(s, m, rows, cols, c0, out);
  } else {
    const int64_t n = static_cast<int64_t>(rows) * ((cols + 3) / 4);
    if (n > 0) expcast_fast_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(s, m, rows, cols, c120, out);
  }
  return cudaGetLastError();
}

}  // namespace vcattn

using namespace vcattn;

namespace {

thread_local std::string g_last_error;
std::mutex g_inject_mu;
std::string g_inject;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return VCATTN_OK;
  return fail(VCATTN_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

bool injected(const char* name) {
  std::lock_guard<std::mutex> lk(g_inject_mu);
  return !g_inject.empty() && g_inject == name;
}

int elem_size(int dtype) { return dtype == VCATTN_DTYPE_F32 ? 4 : 2; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Views are read with 16-byte (kmeans rows) or 8/16-byte (prepare) vector
// loads: base 16-byte aligned and every stride a multiple of 16 bytes.
bool view_ok(const vcattn_bhnd* v, int dtype) {
  if (v == nullptr || v->data == nullptr || !aligned16(v->data)) return false;
  const int64_t q = 16 / elem_size(dtype);
  return (v->sb % q) == 0 && (v->sh % q) == 0 && (v->sn % q) == 0;
}

bool dtype_ok(int dtype) {
  return dtype == VCATTN_DTYPE_BF16 || dtype == VCATTN_DTYPE_F16 || dtype == VCATTN_DTYPE_F32;
}

#define VC_CHECK(cond, msg) \
  do {                      \
    if (!(cond)) return fail(VCATTN_ERR_ARG, msg); \
  } while (0)

}  // namespace

namespace vcattn {
// Lets entry points defined in other translation units report through
// vcattn_last_error().
int record_error(int code, const char* msg) { return fail(code, msg); }
void clear_error() { g_last_error.clear(); }
bool fault_injected(const char* entry_point) { return injected(entry_point); }

// Argument checks of vcattn_prepare_fp8, shared with vcattn_prepare_fp8_noalloc
// (everything but the workspace).  Messages start with `name`.
int prepare_fp8_checks(const char* name, const vcattn_bhnd* q, const vcattn_bhnd* k, const vcattn_bhnd* v,
                       int dtype, int B, int H, int N, int D, const int32_t* perm, int perm_rows, int block_rows,
                       const uint8_t* q8, const float* q_scale, const uint8_t* k8, const float* k_scale,
                       const uint8_t* v8, const float* v_scale, const float* mu, const uint8_t* v8t,
                       const vcattn_route_stats* route) {
  const std::string n(name);
  VC_CHECK(dtype_ok(dtype), n + ": unsupported dtype");
  VC_CHECK(D == 64 || D == 128, n + ": D must be 64 or 128");
  VC_CHECK(B > 0 && H > 0 && N > 0, n + ": empty shape");
  VC_CHECK(block_rows == 64 || block_rows == 128, n + ": block_rows must be 64 or 128");
  VC_CHECK(view_ok(q, dtype) && view_ok(k, dtype) && view_ok(v, dtype),
           n + ": q/k/v must be 16-byte aligned with 16-byte multiple strides");
  VC_CHECK(perm == nullptr || perm_rows == 1 || perm_rows == B * H, n + ": perm_rows must be 1 or G");
  // Q (or K) codes are skipped when both their code and scale buffers are
  // null (the NVFP4 path only needs V here); routing needs both.
  VC_CHECK((q8 == nullptr) == (q_scale == nullptr) && (k8 == nullptr) == (k_scale == nullptr),
           n + ": q8/q_scale and k8/k_scale must be given (or left out) together");
  VC_CHECK(v_scale && mu && (v8 || v8t), n + ": null output");
  VC_CHECK(route == nullptr || (q8 && k8), n + ": routing statistics need the Q and K codes");
  VC_CHECK((q8 == nullptr || aligned16(q8)) && (k8 == nullptr || aligned16(k8)) && (v8 == nullptr || aligned16(v8)) &&
               (v8t == nullptr || aligned16(v8t)),
           n + ": code buffers must be 16-byte aligned");
  const int n_pad = (N + block_rows - 1) / block_rows * block_rows;
  if (route) {
    VC_CHECK(route->q_block == 64 || route->q_block == 128, n + ": route q_block must be 64 or 128");
    VC_CHECK(n_pad % route->q_block == 0, n + ": n_pad must be a multiple of q_block");
  }
  return VCATTN_OK;
}
}  // namespace vcattn

extern "C" {

int vcattn_abi_version(void) { return 1; }

const char* vcattn_last_error(void) { return g_last_error.c_str(); }

void vcattn_inject_fault(const char* entry_point) {
  std::lock_guard<std::mutex> lk(g_inject_mu);
  g_inject = entry_point ? entry_point : "";
}

void vcattn_inject_stall(int tile) {
  std::lock_guard<std::mutex> lk(g_inject_mu);
  set_attn_tc_stall(tile);
}

size_t vcattn_kmeans_workspace_bytes(int G, int N, int D, int k, int nkeys) {
  if (G <= 0 || N <= 0 || D <= 0 || k <= 0) return 0;
  return kmeans_workspace_bytes(G, N, D, k, nkeys);
}

int vcattn_kmeans(const vcattn_bhnd* v, int dtype, int B, int H, int N, int D, int k, int iters,
                  const uint16_t* warm_centroids, const int32_t* key_offset, int nkeys,
                  uint16_t* centroids_out, int32_t* perm_out, int32_t* labels_out, void* workspace,
                  size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_kmeans")) return fail(VCATTN_ERR_INJECTED, "vcattn_kmeans: injected fault");
  VC_CHECK(dtype_ok(dtype), "vcattn_kmeans: unsupported dtype");
  VC_CHECK(D == 64 || D == 128, "vcattn_kmeans: D must be 64 or 128");
  VC_CHECK(B > 0 && H > 0 && N > 0, "vcattn_kmeans: empty shape");
  VC_CHECK(k >= 1 && k <= N && k <= 4096, "vcattn_kmeans: need 1 <= k <= min(N, 4096)");
  VC_CHECK(iters >= 0 && iters <= 1000, "vcattn_kmeans: iters out of range");
  VC_CHECK(view_ok(v, dtype), "vcattn_kmeans: v must be 16-byte aligned with 16-byte multiple strides");
  VC_CHECK(centroids_out && perm_out, "vcattn_kmeans: null output");
  VC_CHECK(key_offset == nullptr || nkeys >= k, "vcattn_kmeans: nkeys must be >= k");
  const int G = B * H;
  const size_t need = kmeans_workspace_bytes(G, N, D, k, key_offset ? nkeys : k);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(VCATTN_ERR_WORKSPACE, "vcattn_kmeans: workspace too small (need " + std::to_string(need) + " bytes)");
  VC_CHECK(aligned16(workspace), "vcattn_kmeans: workspace must be 16-byte aligned");
  KMeansParams p{};
  p.v = v; p.dtype = dtype; p.B = B; p.H = H; p.N = N; p.D = D; p.k = k; p.iters = iters;
  p.warm = warm_centroids; p.key_offset = key_offset; p.nkeys = key_offset ? nkeys : k;
  p.centroids_out = centroids_out; p.perm_out = perm_out; p.labels_out = labels_out;
  p.workspace = workspace;
  return cuda_status(launch_kmeans(p, static_cast<cudaStream_t>(stream)), "vcattn_kmeans");
}

size_t vcattn_prepare_workspace_bytes(int G, int N, int D) {
  if (G <= 0 || N <= 0 || D <= 0) return 0;
  return prepare_workspace_bytes(G, N, D);
}

int vcattn_prepare_fp8(const vcattn_bhnd* q, const vcattn_bhnd* k, const vcattn_bhnd* v, int dtype, int B,
                       int H, int N, int D, const int32_t* perm, int perm_rows, int block_rows, int flags,
                       uint8_t* q8, float* q_scale, uint8_t* k8, float* k_scale, uint8_t* v8,
                       float* v_scale, float* mu, uint8_t* v8t, const vcattn_route_stats* route,
                       void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_prepare_fp8")) return fail(VCATTN_ERR_INJECTED, "vcattn_prepare_fp8: injected fault");
  const int rc = prepare_fp8_checks("vcattn_prepare_fp8", q, k, v, dtype, B, H, N, D, perm, perm_rows, block_rows,
                                    q8, q_scale, k8, k_scale, v8, v_scale, mu, v8t, route);
  if (rc != VCATTN_OK) return rc;
  const int G = B * H;
  const int n_pad = (N + block_rows - 1) / block_rows * block_rows;
  const size_t need = prepare_workspace_bytes(G, N, D);
  if ((flags & VCATTN_SMOOTH_K) && k8 != nullptr && (workspace == nullptr || workspace_bytes < need))
    return fail(VCATTN_ERR_WORKSPACE, "vcattn_prepare_fp8: workspace too small (need " + std::to_string(need) + " bytes)");
  PrepareParams p{};
  p.q = q; p.k = k; p.v = v; p.dtype = dtype; p.B = B; p.H = H; p.N = N; p.D = D; p.n_pad = n_pad;
  p.block_rows = block_rows; p.flags = flags; p.perm = perm; p.perm_rows = perm ? perm_rows : 0;
  p.q8 = q8; p.k8 = k8; p.v8 = v8; p.v8t = v8t;
  p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.mu = mu;
  p.v_mean = route ? route->v_mean : nullptr;
  p.route = route; p.workspace = workspace;
  return cuda_status(launch_prepare(p, static_cast<cudaStream_t>(stream)), "vcattn_prepare_fp8");
}

int vcattn_prepare_nvfp4(const vcattn_bhnd* q, const vcattn_bhnd* k, int dtype, int B, int H, int N, int D,
                         const int32_t* perm, int perm_rows, int block_rows, int flags, uint8_t* q4,
                         uint8_t* q4_scale, float* q4_g, uint8_t* k4, uint8_t* k4_scale, float* k4_g,
                         uint8_t* q4_sf_mma, uint8_t* k4_sf_mma, void* workspace, size_t workspace_bytes,
                         void* stream) {
  g_last_error.clear();
  if (injected("vcattn_prepare_nvfp4")) return fail(VCATTN_ERR_INJECTED, "vcattn_prepare_nvfp4: injected fault");
  VC_CHECK(dtype_ok(dtype), "vcattn_prepare_nvfp4: unsupported dtype");
  VC_CHECK(D == 64 || D == 128, "vcattn_prepare_nvfp4: D must be 64 or 128");
  VC_CHECK(B > 0 && H > 0 && N > 0, "vcattn_prepare_nvfp4: empty shape");
  VC_CHECK(block_rows == 64 || block_rows == 128, "vcattn_prepare_nvfp4: block_rows must be 64 or 128");
  VC_CHECK(view_ok(q, dtype) && view_ok(k, dtype),
           "vcattn_prepare_nvfp4: q/k must be 16-byte aligned with 16-byte multiple strides");
  VC_CHECK(perm == nullptr || perm_rows == 1 || perm_rows == B * H, "vcattn_prepare_nvfp4: perm_rows must be 1 or G");
  VC_CHECK(q4 && q4_scale && q4_g && k4 && k4_scale && k4_g, "vcattn_prepare_nvfp4: null output");
  const int G = B * H;
  const size_t need = prepare_workspace_bytes(G, N, D);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(VCATTN_ERR_WORKSPACE, "vcattn_prepare_nvfp4: workspace too small (need " + std::to_string(need) + " bytes)");
  NvfpParams p{};
  p.q = q; p.k = k; p.dtype = dtype; p.B = B; p.H = H; p.N = N; p.D = D;
  p.n_pad = (N + block_rows - 1) / block_rows * block_rows;
  p.block_rows = block_rows; p.flags = flags; p.perm = perm; p.perm_rows = perm ? perm_rows : 0;
  p.q4 = q4; p.q4_scale = q4_scale; p.q4_g = q4_g; p.k4 = k4; p.k4_scale = k4_scale; p.k4_g = k4_g;
  p.q4_sf_mma = q4_sf_mma; p.k4_sf_mma = k4_sf_mma;
  p.workspace = workspace;
  return cuda_status(launch_prepare_nvfp4(p, static_cast<cudaStream_t>(stream)), "vcattn_prepare_nvfp4");
}

int vcattn_route_mask(const vcattn_route_stats* route, int G, int N, int n_pad, int D, int block_rows, float tau,
                      int local_blocks, int sink_blocks, float sm_scale, uint8_t* keep, float* thresh,
                      void* stream) {
  g_last_error.clear();
  if (injected("vcattn_route_mask")) return fail(VCATTN_ERR_INJECTED, "vcattn_route_mask: injected fault");
  VC_CHECK(route && route->k_mean && route->q_cent && route->q_bar, "vcattn_route_mask: missing statistics");
  VC_CHECK(D == 64 || D == 128, "vcattn_route_mask: D must be 64 or 128");
  VC_CHECK(block_rows == 64 || block_rows == 128, "vcattn_route_mask: block_rows must be 64 or 128");
  VC_CHECK(n_pad / block_rows <= 2048, "vcattn_route_mask: at most 2048 KV blocks per head");
  VC_CHECK(route->q_block > 0 && n_pad % route->q_block == 0 && n_pad % block_rows == 0,
           "vcattn_route_mask: inconsistent padding");
  VC_CHECK(keep != nullptr, "vcattn_route_mask: null keep");
  RouteParams p{};
  p.k_mean = route->k_mean; p.q_cent = route->q_cent; p.q_bar = route->q_bar;
  p.G = G; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows; p.q_block = route->q_block;
  p.tau = tau; p.sm_scale = sm_scale; p.local_blocks = local_blocks; p.sink_blocks = sink_blocks;
  p.keep = keep; p.thresh = thresh;
  return cuda_status(launch_route_mask(p, static_cast<cudaStream_t>(stream)), "vcattn_route_mask");
}

int vcattn_route_tiles(const float* k_mean, const float* v_mean, int G, int n_pad, int D, int block_rows,
                       uint8_t* tiles, void* stream) {
  g_last_error.clear();
  VC_CHECK(k_mean && v_mean && tiles, "vcattn_route_tiles: null pointer");
  VC_CHECK((D == 128 || D == 64) && (block_rows == 128 || block_rows == 64),
           "vcattn_route_tiles: needs D and block_rows in {64, 128}");
  VC_CHECK(G > 0 && n_pad > 0 && n_pad % block_rows == 0, "vcattn_route_tiles: bad shape");
  VC_CHECK(aligned16(tiles), "vcattn_route_tiles: tiles must be 16-byte aligned");
  return cuda_status(launch_route_tiles(k_mean, v_mean, G, n_pad / block_rows, D, tiles,
                                        static_cast<cudaStream_t>(stream)),
                     "vcattn_route_tiles");
}

static int attn_common_checks(const char* name, const uint8_t* q8, const float* q_scale, const uint8_t* k8,
                              const float* k_scale, const uint8_t* v8t, const float* v_scale, const float* mu,
                              int B, int H, int N, int n_pad, int D, int block_rows, void* out, int out_dtype) {
  const std::string n(name);
  VC_CHECK(q8 && q_scale && k8 && k_scale && v8t && v_scale && mu && out, n + ": null pointer");
  VC_CHECK(D == 64 || D == 128, n + ": D must be 64 or 128");
  VC_CHECK(block_rows == 64 || block_rows == 128, n + ": block_rows must be 64 or 128");
  VC_CHECK(B > 0 && H > 0 && N > 0, n + ": empty shape");
  VC_CHECK(n_pad >= N && n_pad % block_rows == 0 && n_pad - N < block_rows, n + ": n_pad inconsistent with N");
  VC_CHECK(dtype_ok(out_dtype), n + ": unsupported output dtype");
  VC_CHECK(aligned16(q8) && aligned16(k8) && aligned16(v8t) && aligned16(k_scale) && aligned16(v_scale) &&
               aligned16(mu),
           n + ": operand buffers must be 16-byte aligned");
  return VCATTN_OK;
}

int vcattn_attn_fp8(const uint8_t* q8, const float* q_scale, const uint8_t* k8, const float* k_scale,
                    const uint8_t* v8, const float* v_scale, const float* mu, int B, int H, int N, int n_pad,
                    int D, int block_rows, float sm_scale, int flags, double expcast_beta, void* out,
                    int out_dtype, int64_t out_sb, int64_t out_sh, int64_t out_sn, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_attn_fp8")) return fail(VCATTN_ERR_INJECTED, "vcattn_attn_fp8: injected fault");
  const int rc = attn_common_checks("vcattn_attn_fp8", q8, q_scale, k8, k_scale, v8, v_scale, mu, B, H, N, n_pad,
                                    D, block_rows, out, out_dtype);
  if (rc != VCATTN_OK) return rc;
  VC_CHECK(aligned16(out) && (out_sn % 8) == 0 && (out_sh % 8) == 0 && (out_sb % 8) == 0,
           "vcattn_attn_fp8: out must be 16-byte aligned with 8-element multiple strides");
  AttnParams p{};
  p.q8 = q8; p.k8 = k8; p.v8 = v8; p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.mu = mu;
  p.B = B; p.H = H; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows;
  p.sm_scale = sm_scale; p.beta = expcast_beta; p.flags = flags;
  p.out = out; p.out_dtype = out_dtype; p.osb = out_sb; p.osh = out_sh; p.osn = out_sn;
  const cudaError_t e = launch_attn_tc(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(VCATTN_ERR_CUDA, std::string("vcattn_attn_fp8: ") + cudaGetErrorString(e) + " [" + attn_tc_diag() + "]");
  return VCATTN_OK;
}

size_t vcattn_attn_split_workspace_bytes(int B, int H, int N, int n_pad, int D, int block_rows, int kv_split) {
  if (B <= 0 || H <= 0 || N <= 0 || n_pad < N || (D != 64 && D != 128) || (block_rows != 64 && block_rows != 128))
    return 0;
  AttnParams p{};
  p.B = B; p.H = H; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows; p.kv_split = kv_split;
  return attn_tc_split_bytes(p);
}

int vcattn_attn_fp8_split(const uint8_t* q8, const float* q_scale, const uint8_t* k8, const float* k_scale,
                          const uint8_t* v8, const float* v_scale, const float* mu, int B, int H, int N, int n_pad,
                          int D, int block_rows, float sm_scale, int flags, double expcast_beta, void* out,
                          int out_dtype, int64_t out_sb, int64_t out_sh, int64_t out_sn, int kv_split,
                          void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_attn_fp8_split")) return fail(VCATTN_ERR_INJECTED, "vcattn_attn_fp8_split: injected fault");
  const int rc = attn_common_checks("vcattn_attn_fp8_split", q8, q_scale, k8, k_scale, v8, v_scale, mu, B, H, N,
                                    n_pad, D, block_rows, out, out_dtype);
  if (rc != VCATTN_OK) return rc;
  VC_CHECK(aligned16(out) && (out_sn % 8) == 0 && (out_sh % 8) == 0 && (out_sb % 8) == 0,
           "vcattn_attn_fp8_split: out must be 16-byte aligned with 8-element multiple strides");
  VC_CHECK(kv_split >= 0, "vcattn_attn_fp8_split: kv_split must be >= 0");
  AttnParams p{};
  p.q8 = q8; p.k8 = k8; p.v8 = v8; p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.mu = mu;
  p.B = B; p.H = H; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows;
  p.sm_scale = sm_scale; p.beta = expcast_beta; p.flags = flags;
  p.out = out; p.out_dtype = out_dtype; p.osb = out_sb; p.osh = out_sh; p.osn = out_sn;
  p.kv_split = kv_split;
  const size_t need = attn_tc_split_bytes(p);
  if (need > 0) {
    VC_CHECK(workspace != nullptr && workspace_bytes >= need && aligned16(workspace),
             "vcattn_attn_fp8_split: workspace missing, unaligned or smaller than "
             "vcattn_attn_split_workspace_bytes()");
    p.part = workspace;
  }
  const cudaError_t e = launch_attn_tc(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(VCATTN_ERR_CUDA,
                std::string("vcattn_attn_fp8_split: ") + cudaGetErrorString(e) + " [" + attn_tc_diag() + "]");
  return VCATTN_OK;
}

int vcattn_attn_fp8_masked(const uint8_t* q8, const float* q_scale, const uint8_t* k8, const float* k_scale,
                           const uint8_t* v8, const float* v_scale, const float* mu, const int32_t* kv_len, int B,
                           int H, int N, int n_pad, int D, int block_rows, float sm_scale, int flags,
                           double expcast_beta, void* out, int out_dtype, int64_t out_sb, int64_t out_sh,
                           int64_t out_sn, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_attn_fp8_masked")) return fail(VCATTN_ERR_INJECTED, "vcattn_attn_fp8_masked: injected fault");
  const int rc = attn_common_checks("vcattn_attn_fp8_masked", q8, q_scale, k8, k_scale, v8, v_scale, mu, B, H, N,
                                    n_pad, D, block_rows, out, out_dtype);
  if (rc != VCATTN_OK) return rc;
  VC_CHECK(kv_len != nullptr, "vcattn_attn_fp8_masked: null kv_len");
  VC_CHECK(aligned16(out) && (out_sn % 8) == 0 && (out_sh % 8) == 0 && (out_sb % 8) == 0,
           "vcattn_attn_fp8_masked: out must be 16-byte aligned with 8-element multiple strides");
  AttnParams p{};
  p.q8 = q8; p.k8 = k8; p.v8 = v8; p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.mu = mu;
  p.B = B; p.H = H; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows;
  p.sm_scale = sm_scale; p.beta = expcast_beta; p.flags = flags;
  p.out = out; p.out_dtype = out_dtype; p.osb = out_sb; p.osh = out_sh; p.osn = out_sn;
  p.kv_len = kv_len;
  const cudaError_t e = launch_attn_tc(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(VCATTN_ERR_CUDA,
                std::string("vcattn_attn_fp8_masked: ") + cudaGetErrorString(e) + " [" + attn_tc_diag() + "]");
  return VCATTN_OK;
}

int vcattn_attn_fp8_mma(const uint8_t* q8, const float* q_scale, const uint8_t* k8, const float* k_scale,
                        const uint8_t* v8t, const float* v_scale, const float* mu, int B, int H, int N, int n_pad,
                        int D, int block_rows, float sm_scale, int flags, double expcast_beta, void* out,
                        int out_dtype, int64_t out_sb, int64_t out_sh, int64_t out_sn, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_attn_fp8_mma")) return fail(VCATTN_ERR_INJECTED, "vcattn_attn_fp8_mma: injected fault");
  const int rc = attn_common_checks("vcattn_attn_fp8_mma", q8, q_scale, k8, k_scale, v8t, v_scale, mu, B, H, N,
                                    n_pad, D, block_rows, out, out_dtype);
  if (rc != VCATTN_OK) return rc;
  AttnParams p{};
  p.q8 = q8; p.k8 = k8; p.v8t = v8t; p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.mu = mu;
  p.B = B; p.H = H; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows;
  p.sm_scale = sm_scale; p.beta = expcast_beta; p.flags = flags;
  p.out = out; p.out_dtype = out_dtype; p.osb = out_sb; p.osh = out_sh; p.osn = out_sn;
  return cuda_status(launch_attn_mma(p, static_cast<cudaStream_t>(stream)), "vcattn_attn_fp8_mma");
}

int vcattn_attn_status(int* code, int* where, int* block, int reset) {
  g_last_error.clear();
  VC_CHECK(code && where && block, "vcattn_attn_status: null output");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "vcattn_attn_status");
  int c2 = 0, w2 = 0, b2 = 0;
  e = attn_tc_status(code, where, block, reset != 0);
  if (e == cudaSuccess) e = attn_nvfp4_status(&c2, &w2, &b2, reset != 0);
  if (e == cudaSuccess && *code == 0 && c2 != 0) {
    *code = c2;
    *where = 100 + w2;   // waits of the NVFP4 kernel are reported as 100 + site
    *block = b2;
  }
  int c3 = 0, w3 = 0, b3 = 0;
  if (e == cudaSuccess) e = attn_sparse_tc_status(&c3, &w3, &b3, reset != 0);
  if (e == cudaSuccess && *code == 0 && c3 != 0) {
    *code = c3;
    *where = 200 + w3;   // and those of the tcgen05 sparse kernel as 200 + site
    *block = b3;
  }
  int c4 = 0, w4 = 0, b4 = 0;
  if (e == cudaSuccess) e = kmeans_tc_status(&c4, &w4, &b4, reset != 0);
  if (e == cudaSuccess && *code == 0 && c4 != 0) {
    *code = c4;
    *where = 300 + w4;   // and those of the tensor-core k-means assignment as 300 + site
    *block = b4;
  }
  return cuda_status(e, "vcattn_attn_status");
}

int vcattn_attn_nvfp4(const uint8_t* q4, const uint8_t* q4_sf_mma, const float* q4_g, const uint8_t* k4,
                      const uint8_t* k4_sf_mma, const float* k4_g, const uint8_t* v8, const float* v_scale,
                      const float* mu, int B, int H, int N, int n_pad, int D, int block_rows, float sm_scale,
                      int flags, double expcast_beta, void* out, int out_dtype, int64_t out_sb, int64_t out_sh,
                      int64_t out_sn, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_attn_nvfp4")) return fail(VCATTN_ERR_INJECTED, "vcattn_attn_nvfp4: injected fault");
  VC_CHECK(q4 && q4_sf_mma && q4_g && k4 && k4_sf_mma && k4_g && v8 && v_scale && mu && out,
           "vcattn_attn_nvfp4: null pointer");
  VC_CHECK(D == 128 && block_rows == 128, "vcattn_attn_nvfp4: needs D = 128 and block_rows = 128");
  VC_CHECK(B > 0 && H > 0 && N > 0, "vcattn_attn_nvfp4: empty shape");
  VC_CHECK(n_pad >= N && n_pad % 128 == 0 && n_pad - N < 128, "vcattn_attn_nvfp4: n_pad inconsistent with N");
  VC_CHECK(dtype_ok(out_dtype), "vcattn_attn_nvfp4: unsupported output dtype");
  VC_CHECK(aligned16(q4) && aligned16(k4) && aligned16(v8) && aligned16(q4_sf_mma) && aligned16(k4_sf_mma) &&
               aligned16(v_scale) && aligned16(mu),
           "vcattn_attn_nvfp4: operand buffers must be 16-byte aligned");
  VC_CHECK(aligned16(out) && (out_sn % 8) == 0 && (out_sh % 8) == 0 && (out_sb % 8) == 0,
           "vcattn_attn_nvfp4: out must be 16-byte aligned with 8-element multiple strides");
  AttnParams p{};
  p.q4 = q4; p.k4 = k4; p.q4_sf = q4_sf_mma; p.k4_sf = k4_sf_mma; p.q4_g = q4_g; p.k4_g = k4_g;
  p.v8 = v8; p.v_scale = v_scale; p.mu = mu;
  p.B = B; p.H = H; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows;
  p.sm_scale = sm_scale; p.beta = expcast_beta; p.flags = flags;
  p.out = out; p.out_dtype = out_dtype; p.osb = out_sb; p.osh = out_sh; p.osn = out_sn;
  const cudaError_t e = launch_attn_nvfp4(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(VCATTN_ERR_CUDA, std::string("vcattn_attn_nvfp4: ") + cudaGetErrorString(e) + " [" + attn_nvfp4_diag() + "]");
  return VCATTN_OK;
}

int vcattn_attn_fp8_sparse(const uint8_t* q8, const float* q_scale, const uint8_t* k8, const float* k_scale,
                           const uint8_t* v8t, const float* v_scale, const float* mu, const float* k_mean,
                           const float* v_mean, const uint8_t* keep, int q_block, int group, int B, int H,
                           int N, int n_pad, int D, int block_rows, float sm_scale, int flags,
                           double expcast_beta, void* out, int out_dtype, int64_t out_sb, int64_t out_sh,
                           int64_t out_sn, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_attn_fp8_sparse")) return fail(VCATTN_ERR_INJECTED, "vcattn_attn_fp8_sparse: injected fault");
  const int rc = attn_common_checks("vcattn_attn_fp8_sparse", q8, q_scale, k8, k_scale, v8t, v_scale, mu, B, H, N,
                                    n_pad, D, block_rows, out, out_dtype);
  if (rc != VCATTN_OK) return rc;
  VC_CHECK(k_mean && v_mean && keep, "vcattn_attn_fp8_sparse: missing routing inputs");
  VC_CHECK(q_block == 64 && n_pad % q_block == 0, "vcattn_attn_fp8_sparse: q_block must be 64");
  VC_CHECK(group == 16, "vcattn_attn_fp8_sparse: group must be 16 (TritonConfig.group default)");
  AttnParams p{};
  p.q8 = q8; p.k8 = k8; p.v8t = v8t; p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.mu = mu;
  p.k_mean = k_mean; p.v_mean = v_mean; p.keep = keep; p.q_block = q_block; p.group = group;
  p.B = B; p.H = H; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows;
  p.sm_scale = sm_scale; p.beta = expcast_beta; p.flags = flags;
  p.out = out; p.out_dtype = out_dtype; p.osb = out_sb; p.osh = out_sh; p.osn = out_sn;
  return cuda_status(launch_attn_sparse_mma(p, static_cast<cudaStream_t>(stream)), "vcattn_attn_fp8_sparse");
}

int vcattn_attn_fp8_sparse_tc(const uint8_t* q8, const float* q_scale, const uint8_t* k8, const float* k_scale,
                              const uint8_t* v8, const float* v_scale, const float* mu, const uint8_t* ap_tiles,
                              const uint8_t* keep, int q_block, int group, int B, int H,
                              int N, int n_pad, int D, int block_rows, float sm_scale, int flags,
                              double expcast_beta, void* out, int out_dtype, int64_t out_sb, int64_t out_sh,
                              int64_t out_sn, void* stream) {
  g_last_error.clear();
  if (injected("vcattn_attn_fp8_sparse_tc"))
    return fail(VCATTN_ERR_INJECTED, "vcattn_attn_fp8_sparse_tc: injected fault");
  const int rc = attn_common_checks("vcattn_attn_fp8_sparse_tc", q8, q_scale, k8, k_scale, v8, v_scale, mu, B, H, N,
                                    n_pad, D, block_rows, out, out_dtype);
  if (rc != VCATTN_OK) return rc;
  VC_CHECK(ap_tiles && keep, "vcattn_attn_fp8_sparse_tc: missing routing inputs");
  VC_CHECK(aligned16(ap_tiles), "vcattn_attn_fp8_sparse_tc: ap_tiles must be 16-byte aligned");
  VC_CHECK(aligned16(out) && (out_sn % 8) == 0 && (out_sh % 8) == 0 && (out_sb % 8) == 0,
           "vcattn_attn_fp8_sparse_tc: out must be 16-byte aligned with 8-element multiple strides");
  AttnParams p{};
  p.q8 = q8; p.k8 = k8; p.v8 = v8; p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.mu = mu;
  p.ap_tiles = ap_tiles; p.keep = keep; p.q_block = q_block; p.group = group;
  p.B = B; p.H = H; p.N = N; p.n_pad = n_pad; p.D = D; p.block_rows = block_rows;
  p.sm_scale = sm_scale; p.beta = expcast_beta; p.flags = flags;
  p.out = out; p.out_dtype = out_dtype; p.osb = out_sb; p.osh = out_sh; p.osn = out_sn;
  VC_CHECK(attn_sparse_tc_supported(p),
           "vcattn_attn_fp8_sparse_tc: needs D and block_rows in {64, 128}, q_block = 64, group = 16 and at most "
           "1024 KV blocks (N <= 131072 at block_rows 128, 65536 at 64)");
  const cudaError_t e = launch_attn_sparse_tc(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(VCATTN_ERR_CUDA,
                std::string("vcattn_attn_fp8_sparse_tc: ") + cudaGetErrorString(e) + " [" + attn_sparse_tc_diag() + "]");
  return VCATTN_OK;
}

int vcattn_e4m3_encode(const float* x, int64_t n, uint8_t* out, void* stream) {
  g_last_error.clear();
  VC_CHECK(n >= 0 && (n == 0 || (x && out)), "vcattn_e4m3_encode: bad arguments");
  return cuda_status(launch_codecs_e4m3(x, n, out, static_cast<cudaStream_t>(stream)), "vcattn_e4m3_encode");
}

int vcattn_fp4_encode(const float* x, int64_t n, uint8_t* out, void* stream) {
  g_last_error.clear();
  VC_CHECK(n >= 0 && (n == 0 || (x && out)), "vcattn_fp4_encode: bad arguments");
  return cuda_status(launch_codecs_fp4(x, n, out, static_cast<cudaStream_t>(stream)), "vcattn_fp4_encode");
}

int vcattn_expcast_codes(const float* s, const float* m, int rows, int cols, double beta, int mode, uint8_t* out,
                         void* stream) {
  g_last_error.clear();
  VC_CHECK(rows >= 0 && cols >= 0 && (rows * static_cast<int64_t>(cols) == 0 || (s && m && out)),
           "vcattn_expcast_codes: bad arguments");
  VC_CHECK(mode == 0 || mode == 1, "vcattn_expcast_codes: mode must be 0 or 1");
  return cuda_status(launch_expcast(s, m, rows, cols, beta, mode, out, static_cast<cudaStream_t>(stream)),
                     "vcattn_expcast_codes");
}

}  // extern "C"
