// vcattn_prepare_fp8_noalloc: the prepare entry point for callers that cannot
// allocate device memory.
//
// vcattn_prepare_fp8 needs a caller-provided scratch workspace (the float64
// partial sums of the K token mean).  Some callers have no way to provide one:
// a plugin host that owns every device byte through its own pool and forbids
// its plugins from allocating, or a plain FFI binding (ctypes, cgo, JNI) that
// has no device allocator at hand.  This variant takes the same inputs and
// outputs and uses a fixed scratch array that lives in the library itself.
//
// The scratch is a file-scope __device__ array of kScratchBytes (16 MiB).
// Every GPU that loads the library holds it until the process exits.  Host
// code cannot pass the array's name to a kernel (on the host the name is only
// a stand-in, not a device address), so the first call on each device looks
// the address up with cudaGetSymbolAddress while that device is current and
// caches it; that first call should come before any stream capture.
//
// All calls share the array and it keeps the last call's contents.  Nothing
// in it needs to start at zero: every partial sum is written before it is
// read.  Calls that overlap on the GPU (on different streams, or from
// different threads) race on the array and must be serialised by the caller.
#include <mutex>
#include <string>

#include "kernels.cuh"

namespace vcattn {
int record_error(int code, const char* msg);
void clear_error();
}  // namespace vcattn

namespace {

constexpr size_t kScratchBytes = static_cast<size_t>(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_prepare_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_prepare_scratch on the current device (set up once).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_prepare_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool view_ok(const vcattn_bhnd* v, int dtype) {
  if (v == nullptr || v->data == nullptr || !aligned16(v->data)) return false;
  const int64_t q = 16 / (dtype == VCATTN_DTYPE_F32 ? 4 : 2);
  return (v->sb % q) == 0 && (v->sh % q) == 0 && (v->sn % q) == 0;
}

int arg_error(const std::string& msg) { return vcattn::record_error(VCATTN_ERR_ARG, msg.c_str()); }

}  // namespace

extern "C" VCATTN_API int vcattn_prepare_fp8_noalloc(
    const vcattn_bhnd* q, const vcattn_bhnd* k, const vcattn_bhnd* v, int dtype, int B, int H, int N, int D,
    const int32_t* perm, int perm_rows, int block_rows, int flags, uint8_t* q8, float* q_scale, uint8_t* k8,
    float* k_scale, uint8_t* v8, float* v_scale, float* mu, uint8_t* v8t, const vcattn_route_stats* route,
    void* stream) {
  const char* fn = "vcattn_prepare_fp8_noalloc";
  vcattn::clear_error();
  if (!(dtype == VCATTN_DTYPE_BF16 || dtype == VCATTN_DTYPE_F16 || dtype == VCATTN_DTYPE_F32))
    return arg_error(std::string(fn) + ": unsupported dtype");
  if (!(D == 64 || D == 128)) return arg_error(std::string(fn) + ": D must be 64 or 128");
  if (B <= 0 || H <= 0 || N <= 0) return arg_error(std::string(fn) + ": empty shape");
  if (!(block_rows == 64 || block_rows == 128))
    return arg_error(std::string(fn) + ": block_rows must be 64 or 128");
  const int G = B * H;
  // The size limit is checked before anything else touches the buffers.
  const size_t need = (flags & VCATTN_SMOOTH_K) ? vcattn::prepare_workspace_bytes(G, N, D) : 0;
  if (need > kScratchBytes)
    return arg_error(std::string(fn) + ": shape needs " + std::to_string(need) +
                     " bytes of scratch, above this entry point's fixed " + std::to_string(kScratchBytes) +
                     "-byte limit; use vcattn_prepare_fp8 with a workspace");
  if (!(view_ok(q, dtype) && view_ok(k, dtype) && view_ok(v, dtype)))
    return arg_error(std::string(fn) + ": q/k/v must be 16-byte aligned with 16-byte multiple strides");
  if (!(perm == nullptr || perm_rows == 1 || perm_rows == G))
    return arg_error(std::string(fn) + ": perm_rows must be 1 or G");
  if (!(q8 && q_scale && k8 && k_scale && v_scale && mu && (v8 || v8t)))
    return arg_error(std::string(fn) + ": null output");
  if (!(aligned16(q8) && aligned16(k8) && (v8 == nullptr || aligned16(v8)) && (v8t == nullptr || aligned16(v8t))))
    return arg_error(std::string(fn) + ": code buffers must be 16-byte aligned");
  const int n_pad = (N + block_rows - 1) / block_rows * block_rows;
  if (route) {
    if (!(route->q_block == 64 || route->q_block == 128) || n_pad % route->q_block != 0)
      return arg_error(std::string(fn) + ": route q_block must be 64 or 128 and divide n_pad");
  }
  void* scratch = nullptr;
  cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess)
    return vcattn::record_error(VCATTN_ERR_CUDA, (std::string(fn) + ": cudaGetSymbolAddress: " +
                                                  cudaGetErrorString(e)).c_str());
  vcattn::PrepareParams p{};
  p.q = q; p.k = k; p.v = v; p.dtype = dtype; p.B = B; p.H = H; p.N = N; p.D = D; p.n_pad = n_pad;
  p.block_rows = block_rows; p.flags = flags; p.perm = perm; p.perm_rows = perm ? perm_rows : 0;
  p.q8 = q8; p.k8 = k8; p.v8 = v8; p.v8t = v8t;
  p.q_scale = q_scale; p.k_scale = k_scale; p.v_scale = v_scale; p.mu = mu;
  p.v_mean = route ? route->v_mean : nullptr;
  p.route = route; p.workspace = scratch;
  e = vcattn::launch_prepare(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return vcattn::record_error(VCATTN_ERR_CUDA, (std::string(fn) + ": " + cudaGetErrorString(e)).c_str());
  return VCATTN_OK;
}
