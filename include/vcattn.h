/*
 * vcattn.h -- C ABI of the B200 (sm_100a) VC-Attention hot path.
 *
 * One shared library, libvcattn.so, built from comfyui_vc_attention_b200/csrc.
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as void*, enqueues its kernels on that stream and returns a status
 * code (0 = VCATTN_OK).  Nothing here aborts, traps or synchronises the device
 * unless the entry point says so.  Device buffers are borrowed and no entry
 * point allocates device memory.  Scratch memory is a caller-provided
 * workspace whose size the matching *_workspace_bytes() function reports,
 * except for vcattn_prepare_fp8_noalloc, whose scratch is a fixed 16 MiB
 * array held inside the library on every GPU that loads it.
 *
 * The reference (bingling360/comfyui_vc_attention) is Python + Triton, so its
 * "FFI" for this path is the Python call boundary; each function below names
 * the reference interface (file:line inside that project) whose work it
 * performs.  The Python host layer (comfyui_vc_attention_b200.vc_attention)
 * binds these with ctypes under the reference's own function names.
 *
 * Layout conventions
 *   B, H, N, D   batch, heads, tokens, head dim (D in {64, 128}); G = B*H.
 *   NP           N rounded up to a multiple of block_rows; NB = NP/block_rows.
 *   "(G, NP, D)" means a dense row-major array, head-major.
 *   Codes are E4M3 bytes (float8_e4m3fn bit patterns), scales are fp32.
 */
#ifndef VCATTN_H_
#define VCATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VCATTN_API __attribute__((visibility("default")))
#else
#define VCATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define VCATTN_OK 0
#define VCATTN_ERR_ARG 1        /* unsupported shape / option / alignment     */
#define VCATTN_ERR_CUDA 2       /* a CUDA call failed; see vcattn_last_error() */
#define VCATTN_ERR_WORKSPACE 3  /* workspace smaller than *_workspace_bytes()  */
#define VCATTN_ERR_DEVICE 4     /* a kernel reported failure in its status word */
#define VCATTN_ERR_INJECTED 5   /* host-side fault injection (tests)           */

/* ---- element types ----------------------------------------------------- */
#define VCATTN_DTYPE_BF16 0
#define VCATTN_DTYPE_F16 1
#define VCATTN_DTYPE_F32 2

/* ---- prepare flags (triton_attn.py:504-512 hadamard / smooth_k) --------- */
#define VCATTN_HADAMARD 1
#define VCATTN_SMOOTH_K 2
/* V codes (v8) in the tcgen05 sparse kernel's key order: inside every 32-row
 * chunk of a value block, row 8a + 2b + e is stored at slot 8b + 2a + e (a, b
 * in 0..3, e in 0..1).  The order is its own inverse.
 * vcattn_attn_fp8_sparse_tc requires it; vcattn_attn_fp8 and
 * vcattn_attn_nvfp4 read token order (without the flag); the other outputs are
 * unaffected.  No counterpart in the reference. */
#define VCATTN_V_MMA_ORDER 4

/* ---- attention flags (TritonConfig, triton_attn.py:93-129) ------------- */
#define VCATTN_EXPCAST 1        /* write P bytes with ExpCast (expcast.py:52-70) */
/* With VCATTN_EXPCAST: evaluate ExpCast in the reference's operation order
 * (expcast.py:67-69) on s = (S * (qs * ks)) * sm_scale instead of the one-FMA
 * form.  Slower; for parity runs.  vcattn_attn_fp8 only. */
#define VCATTN_EXPCAST_EXACT 2

/* A strided (B, H, N, D) view: element (b,h,n,d) sits at
 * data + b*sb + h*sh + n*sn + d (strides in elements, d contiguous).  This is
 * what lets the 3-D (B, N, H*D) ComfyUI layout (patch.py:331-337) be read
 * without a transpose copy. */
typedef struct vcattn_bhnd {
  const void* data;
  int64_t sb, sh, sn;
} vcattn_bhnd;

/* Optional routing statistics produced by vcattn_prepare_fp8 for the
 * block-sparse kernel (triton_attn.py:716-735).  Any pointer may be NULL. */
typedef struct vcattn_route_stats {
  int q_block;     /* rows per routing query block (TritonConfig.block_m)     */
  float* k_mean;   /* (G, NB, D)  block mean of the rotated, smoothed, permuted K */
  float* q_cent;   /* (G, NP/q_block, D) query-block mean of the rotated Q      */
  float* q_bar;    /* (G, NP/q_block, D) sum over the block of q8 * (qs * sm_scale) */
  float* v_mean;   /* (G, NB, D)  value block mean (the skipped-block value)      */
  float sm_scale;  /* softmax scale folded into q_bar                           */
} vcattn_route_stats;

/* ---- library ------------------------------------------------------------ */
VCATTN_API int vcattn_abi_version(void);
/* Text of the last error on the calling thread ("" if none). */
VCATTN_API const char* vcattn_last_error(void);
/* Host-side fault injection for the router's fallback tests: while set, the
 * named entry point (e.g. "vcattn_attn_fp8") returns VCATTN_ERR_INJECTED
 * without launching anything.  NULL or "" clears it. */
VCATTN_API void vcattn_inject_fault(const char* entry_point);
/* Bounded-wait test hook (no counterpart in the reference).  While set
 * (tile >= 0), the dense tcgen05 kernel of vcattn_attn_fp8 and
 * vcattn_attn_fp8_masked issues no copies from KV tile `tile` on, so the
 * waits on that tile find nothing to wait for: each gives up after its limit
 * (about 2 s of SM clocks), the CTA drains its copies and MMAs, frees its
 * tensor memory and returns, and vcattn_attn_status() reports code 1 and the
 * wait that gave up.  No fault, trap or unbounded wait is involved.
 * tile = -1 restores normal launches. */
VCATTN_API void vcattn_inject_stall(int tile);

/* ---- V-Smooth grouping: grouping.py:127-147 (kmeans) + :150-186
 *      (build_permutation) ------------------------------------------------
 * v: (B,H,N,D) view, any of the three dtypes (rounded to bf16 first, as
 *    grouping.py:299 does).  k clusters; iters Lloyd iterations (warm_iters
 *    when warm_centroids != NULL).  key_offset (N,) int32 or NULL is added to
 *    the cluster label before the stable sort (modality / padding keys,
 *    grouping.py:176-183); nkeys bounds the keys (k when key_offset is NULL).
 * Outputs: centroids_out (G,k,D) bf16 bits, perm_out (G,N) int32, and
 *    labels_out (G,N) int32 (may be NULL).
 * bf16 input with D = 128 is assigned on the tensor cores (tcgen05, labels
 * certified equal to the sequential-FMA definition; bounded waits report
 * through vcattn_attn_status as 300 + site); other inputs on the CUDA cores.
 * Environment VCATTN_KMEANS_SIMT=1 forces the CUDA-core assignment. */
VCATTN_API size_t vcattn_kmeans_workspace_bytes(int G, int N, int D, int k, int nkeys);
VCATTN_API int vcattn_kmeans(const vcattn_bhnd* v, int dtype, int B, int H, int N, int D,
                  int k, int iters, const uint16_t* warm_centroids,
                  const int32_t* key_offset, int nkeys,
                  uint16_t* centroids_out, int32_t* perm_out, int32_t* labels_out,
                  void* workspace, size_t workspace_bytes, void* stream);

/* ---- prepare: triton_attn.py:504-579 (the portable Prepared producer) ----
 * perm: (perm_rows, N) int32 gather index applied to K and V; perm_rows is 0
 *    (no permutation), 1 (shared by every head) or G.
 * Outputs (all dense, zero-padded to NP rows):
 *    q8, k8, v8 (G,NP,D) E4M3 codes; q_scale, k_scale (G,NP); v_scale,
 *    mu (G,NB,D) with mu = block mean / v_scale.
 *    v8t: NULL, or the same V codes stored block-transposed (G,NB,D,block_rows)
 *    (the operand layout of the register-MMA attention kernels); v8 may be
 *    NULL when only v8t is wanted.
 *    q8 + q_scale (or k8 + k_scale) may both be NULL: those rows are then not
 *    quantised (the NVFP4 QK path takes its Q / K from vcattn_prepare_nvfp4).
 * route: NULL, or routing statistics to fill (block-sparse path; needs the
 *    Q and K codes). */
VCATTN_API size_t vcattn_prepare_workspace_bytes(int G, int N, int D);
VCATTN_API int vcattn_prepare_fp8(const vcattn_bhnd* q, const vcattn_bhnd* k, const vcattn_bhnd* v,
                       int dtype, int B, int H, int N, int D,
                       const int32_t* perm, int perm_rows, int block_rows, int flags,
                       uint8_t* q8, float* q_scale, uint8_t* k8, float* k_scale,
                       uint8_t* v8, float* v_scale, float* mu, uint8_t* v8t,
                       const vcattn_route_stats* route,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ---- NVFP4 Q / K: quant.py:172-204 per (b, h) slab; replaces the NVFP4 half
 * of triton_attn.py:693-702 (nvfp4_pack, whose Triton path has no tensor
 * scale) with the tensor-scaled form of configs[3].
 * Quantises the same rotated (VCATTN_HADAMARD) and, for K, smoothed
 * (VCATTN_SMOOTH_K, over the N real rows) and perm-gathered rows as
 * vcattn_prepare_fp8, zero-padded to NP = ceil(N / block_rows) * block_rows:
 *    q4, k4 (G,NP,D/2): E2M1 codes, two per byte, low nibble = even element
 *       (token-major for both; the reference stores K transposed);
 *    q4_scale, k4_scale (G,NP,D/16): E4M3 micro scale per 16 elements;
 *    q4_g, k4_g (G): fp32 tensor scale g = max(amax, 1e-30) / 2688 per head.
 * x = fp4(x / max(g * micro, 1e-30)) * micro * g.
 * q4_sf_mma, k4_sf_mma: NULL, or the same micro scales again in the layout
 *    the block-scaled tcgen05 MMA reads (G, ceil(NP/128), D/64, 512): per
 *    128-row tile and 4 scales one 512-byte atom, row m / scale kb at byte
 *    16 (m % 32) + 4 (m / 32) + kb % 4.
 * The workspace is the one of vcattn_prepare_workspace_bytes (always needed
 * here). */
VCATTN_API int vcattn_prepare_nvfp4(const vcattn_bhnd* q, const vcattn_bhnd* k, int dtype, int B, int H, int N,
                                    int D, const int32_t* perm, int perm_rows, int block_rows, int flags,
                                    uint8_t* q4, uint8_t* q4_scale, float* q4_g, uint8_t* k4, uint8_t* k4_scale,
                                    float* k4_g, uint8_t* q4_sf_mma, uint8_t* k4_sf_mma, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* ---- prepare without a workspace (no counterpart in the reference) ------
 * Same inputs, outputs and results as vcattn_prepare_fp8, for callers that
 * cannot allocate device memory: a host that owns every device byte through
 * its own pool and forbids plugins to allocate, or a plain FFI binding with no
 * device allocator.  Its scratch is a 16 MiB array inside the library, which
 * every GPU that loads the library holds until the process exits.  Shapes
 * whose scratch exceeds it (G * ceil(N/256) * D * 8 + G * D * 4 + G * 8 + 256
 * bytes when VCATTN_SMOOTH_K is set and k8 is given) are rejected with VCATTN_ERR_ARG before any launch.
 * The first call on a device looks the array's address up (with that device
 * current) and should come before any stream capture; the address is cached
 * per device together with the id of its CUDA context, and looked up again
 * once that context has changed (after a cudaDeviceReset()).  All calls share
 * the array: calls that overlap on the GPU race and must be serialised.
 * Argument checks, host fault injection and error codes are those of
 * vcattn_prepare_fp8 (Q or K codes may be left out in pairs); shapes that
 * need no K mean (no VCATTN_SMOOTH_K, or k8 NULL) use no scratch at all. */
VCATTN_API int vcattn_prepare_fp8_noalloc(const vcattn_bhnd* q, const vcattn_bhnd* k, const vcattn_bhnd* v,
                                          int dtype, int B, int H, int N, int D,
                                          const int32_t* perm, int perm_rows, int block_rows, int flags,
                                          uint8_t* q8, float* q_scale, uint8_t* k8, float* k_scale,
                                          uint8_t* v8, float* v_scale, float* mu, uint8_t* v8t,
                                          const vcattn_route_stats* route, void* stream);

/* ---- routing mask: triton_attn.py:449-459 with the threshold of :716-735 -
 * keep (G, NP/q_block, NB) uint8: 1 = exact tile, 0 = block-mean approximation.
 * thresh (G, NP/q_block) fp32 output (may be NULL). */
VCATTN_API int vcattn_route_mask(const vcattn_route_stats* route, int G, int N, int n_pad, int D,
                      int block_rows, float tau, int local_blocks, int sink_blocks,
                      float sm_scale, uint8_t* keep, float* thresh, void* stream);

/* ---- fused attention with NVFP4 QK^T: the QK_FP4 branch of
 * triton_attn.py:227-239, 263-271 (+ launch :831-844), tensor-scaled NVFP4.
 * q4, k4 (G,NP,D/2), the scale-factor atoms q4_sf_mma, k4_sf_mma and the
 * tensor scales q4_g, k4_g from vcattn_prepare_nvfp4; v8, v_scale, mu from
 * vcattn_prepare_fp8 WITHOUT VCATTN_V_MMA_ORDER (token-order V rows).
 * s = dot_blockscaled(q4, k4) * g_q * g_k * sm_scale; P, V as in
 * vcattn_attn_fp8.  D = 128, block_rows = 128.  Bounded waits report through
 * vcattn_attn_status() (site numbers offset by 100). */
VCATTN_API int vcattn_attn_nvfp4(const uint8_t* q4, const uint8_t* q4_sf_mma, const float* q4_g,
                                 const uint8_t* k4, const uint8_t* k4_sf_mma, const float* k4_g,
                                 const uint8_t* v8, const float* v_scale, const float* mu, int B, int H, int N,
                                 int n_pad, int D, int block_rows, float sm_scale, int flags,
                                 double expcast_beta, void* out, int out_dtype, int64_t out_sb,
                                 int64_t out_sh, int64_t out_sn, void* stream);

/* ---- fused dense FP8 attention: triton_attn.py:203-322 (+ launch :831-844)
 * The tcgen05 kernel (D = 64 or 128, block_rows 64 or 128).  Consumes the prepare
 * outputs in the Prepared layout (v8 row-major (G,NP,D) in token order, i.e.
 * prepared without VCATTN_V_MMA_ORDER); writes O (B,H,N,D)
 * through the out view (out_dtype one of the three dtypes; strides in
 * elements).  Its bounded waits report through vcattn_attn_status(). */
VCATTN_API int vcattn_attn_fp8(const uint8_t* q8, const float* q_scale, const uint8_t* k8,
                    const float* k_scale, const uint8_t* v8, const float* v_scale,
                    const float* mu, int B, int H, int N, int n_pad, int D,
                    int block_rows, float sm_scale, int flags, double expcast_beta,
                    void* out, int out_dtype, int64_t out_sb, int64_t out_sh, int64_t out_sn,
                    void* stream);

/* ---- the same with query tiles split over their KV tiles (no counterpart in
 * the reference).  A split query tile runs as several CTAs, each over a
 * contiguous range of its KV tiles with its own running max, and a second
 * kernel combines the partials (O = sum w_p O_p / sum w_p l_p, w_p =
 * exp2(m_p - max m)).  kv_split 0 (auto): only when the CTAs would end in a
 * partial wave holding at most half of the SMs are that wave's query tiles
 * split, so the last wave takes a fraction of a CTA's time; 1: no split
 * (identical to vcattn_attn_fp8); k >= 2: every query tile in k pieces (at
 * most 32).  Split tiles round their P bytes relative to each piece's own
 * maximum, so their output differs from the unsplit kernel's at the level of
 * the FP8 rounding; unsplit tiles are bit-identical to vcattn_attn_fp8.
 * workspace: at least vcattn_attn_split_workspace_bytes() bytes, 16-byte
 * aligned (may be null when that is 0); the plan depends on the current
 * device's SM count. */
VCATTN_API size_t vcattn_attn_split_workspace_bytes(int B, int H, int N, int n_pad, int D,
                                                    int block_rows, int kv_split);
VCATTN_API int vcattn_attn_fp8_split(const uint8_t* q8, const float* q_scale, const uint8_t* k8,
                          const float* k_scale, const uint8_t* v8, const float* v_scale,
                          const float* mu, int B, int H, int N, int n_pad, int D,
                          int block_rows, float sm_scale, int flags, double expcast_beta,
                          void* out, int out_dtype, int64_t out_sb, int64_t out_sh, int64_t out_sn,
                          int kv_split, void* workspace, size_t workspace_bytes, void* stream);

/* ---- masked (key-padding) dense FP8 attention: reference.py:162-294 with
 * valid_len (keys at positions >= valid_len masked out), per batch entry.
 * The reference applies valid_len to the permuted key order, after
 * build_permutation(valid_len=...) has sorted the padding keys to the tail
 * (grouping.py:176-183); its Triton path does not run masked attention
 * (README.md:514-515).  Same operands as vcattn_attn_fp8; kv_len is a device
 * array (B,) int32: in batch entry b only keys 0 .. kv_len[b]-1 of the
 * (permuted) order take part (values below 1 count as 1, above N as N), and
 * KV tiles past the last such key are not visited.  D = 64 or 128. */
VCATTN_API int vcattn_attn_fp8_masked(const uint8_t* q8, const float* q_scale, const uint8_t* k8,
                    const float* k_scale, const uint8_t* v8, const float* v_scale,
                    const float* mu, const int32_t* kv_len, int B, int H, int N, int n_pad, int D,
                    int block_rows, float sm_scale, int flags, double expcast_beta,
                    void* out, int out_dtype, int64_t out_sb, int64_t out_sh, int64_t out_sn,
                    void* stream);

/* Same computation on the register-MMA (mma.sync m16n8k32) kernel, for head
 * dims 64 and 128; V as the block-transposed v8t (G,NB,D,block_rows).  P bytes
 * follow the reference's ExpCast operation order exactly.  Not on the
 * product path (the router and vc_attention_cuda use the tcgen05 kernels);
 * kept as a second, independently written implementation for the tests. */
VCATTN_API int vcattn_attn_fp8_mma(const uint8_t* q8, const float* q_scale, const uint8_t* k8,
                    const float* k_scale, const uint8_t* v8t, const float* v_scale,
                    const float* mu, int B, int H, int N, int n_pad, int D,
                    int block_rows, float sm_scale, int flags, double expcast_beta,
                    void* out, int out_dtype, int64_t out_sb, int64_t out_sh, int64_t out_sn,
                    void* stream);

/* Device status word of the tcgen05 kernels: code 0 = ok, 1 = a bounded wait
 * expired (the kernel gave up and returned); where = which wait (NVFP4
 * attention 100 + site, sparse attention 200 + site, the tensor-core k-means
 * assignment of vcattn_kmeans 300 + site); block = the first failing CTA.
 * Synchronises the current device.  reset != 0 clears it. */
VCATTN_API int vcattn_attn_status(int* code, int* where, int* block, int reset);

/* ---- fused block-sparse FP8 attention: triton_attn.py:384-501 ----------
 * keep from vcattn_route_mask; k_mean/v_mean (G,NB,D) fp32; q_block rows per
 * routing query block; group KV blocks routed together. */
VCATTN_API int vcattn_attn_fp8_sparse(const uint8_t* q8, const float* q_scale, const uint8_t* k8,
                           const float* k_scale, const uint8_t* v8t, const float* v_scale,
                           const float* mu, const float* k_mean, const float* v_mean,
                           const uint8_t* keep, int q_block, int group,
                           int B, int H, int N, int n_pad, int D, int block_rows,
                           float sm_scale, int flags, double expcast_beta,
                           void* out, int out_dtype, int64_t out_sb, int64_t out_sh,
                           int64_t out_sn, void* stream);

/* ---- bf16 proxy tiles of the tcgen05 sparse kernel (triton_attn.py:460-486
 * operands): per (head, group of 16 KV blocks) one 8192-byte tile holding
 * bf16(k_mean) and bf16(v_mean) of the group in the kernel's 128-byte
 * swizzled shared-memory layout.  tiles: G * ceil(NB/16) * 8192 bytes.
 * D and block_rows in {64, 128}; with D = 64 channels 64-127 of each half are
 * zero. */
VCATTN_API int vcattn_route_tiles(const float* k_mean, const float* v_mean, int G, int n_pad, int D,
                       int block_rows, uint8_t* tiles, void* stream);

/* ---- fused block-sparse FP8 attention on tcgen05: triton_attn.py:384-501 ---
 * Same routing semantics as vcattn_attn_fp8_sparse, with the V codes v8
 * (G,NP,D) in the tcgen05 key order (prepare flag VCATTN_V_MMA_ORDER)
 * instead of the block-transposed v8t, and the proxy operands as the tiles
 * of vcattn_route_tiles instead of fp32 k_mean / v_mean.  One CTA runs two
 * routing query blocks: needs D and block_rows in {64, 128}, q_block = 64,
 * group = 16 and at most 1024 KV blocks (n_pad / block_rows).  Bounded waits
 * report through vcattn_attn_status as 200 + site. */
VCATTN_API int vcattn_attn_fp8_sparse_tc(const uint8_t* q8, const float* q_scale, const uint8_t* k8,
                              const float* k_scale, const uint8_t* v8, const float* v_scale,
                              const float* mu, const uint8_t* ap_tiles,
                              const uint8_t* keep, int q_block, int group,
                              int B, int H, int N, int n_pad, int D, int block_rows,
                              float sm_scale, int flags, double expcast_beta,
                              void* out, int out_dtype, int64_t out_sb, int64_t out_sh,
                              int64_t out_sn, void* stream);

/* ---- element codecs, exposed for bit-exact tests ------------------------
 * vcattn_e4m3_encode: quant.py:56-84.  vcattn_fp4_encode: quant.py:144-161
 * (one code per byte).  vcattn_expcast_codes: expcast.py:52-70 on a (rows,
 * cols) score tile and its (rows,) running maxima; mode 0 runs the attention
 * kernels' own one-FMA device routine (same folding of the per-row constants,
 * unit score scale), mode 1 the reference's operation sequence. */
VCATTN_API int vcattn_e4m3_encode(const float* x, int64_t n, uint8_t* out, void* stream);
VCATTN_API int vcattn_fp4_encode(const float* x, int64_t n, uint8_t* out, void* stream);
VCATTN_API int vcattn_expcast_codes(const float* s, const float* m, int rows, int cols, double beta,
                         int mode, uint8_t* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VCATTN_H_ */
