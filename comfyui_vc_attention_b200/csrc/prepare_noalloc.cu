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
// caches it; that first call should come before any stream capture.  The cache
// remembers which CUDA context the address belongs to: after a
// cudaDeviceReset() the device gets a new primary context (and a new copy of
// the array), and the next call looks the address up again.
//
// All calls share the array and it keeps the last call's contents.  Nothing
// in it needs to start at zero: every partial sum is written before it is
// read.  Calls that overlap on the GPU (on different streams, or from
// different threads) race on the array and must be serialised by the caller.
#include <cuda.h>

#include <mutex>
#include <string>

#include "kernels.cuh"

namespace vcattn {
int record_error(int code, const char* msg);
void clear_error();
bool fault_injected(const char* entry_point);
int prepare_fp8_checks(const char* name, const vcattn_bhnd* q, const vcattn_bhnd* k, const vcattn_bhnd* v,
                       int dtype, int B, int H, int N, int D, const int32_t* perm, int perm_rows, int block_rows,
                       const uint8_t* q8, const float* q_scale, const uint8_t* k8, const float* k_scale,
                       const uint8_t* v8, const float* v_scale, const float* mu, const uint8_t* v8t,
                       const vcattn_route_stats* route);
}  // namespace vcattn

namespace {

constexpr size_t kScratchBytes = static_cast<size_t>(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_prepare_scratch[kScratchBytes];

struct ScratchSlot {
  void* ptr = nullptr;
  unsigned long long ctx_id = 0;
};

std::mutex g_mu;
ScratchSlot g_slot[kMaxDevices];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id (for the life of the process) of the calling thread's current
// context, or 0 when it cannot be read.
unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_prepare_scratch on the current device (looked up once
// per device and context).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  ScratchSlot& slot = g_slot[dev];
  if (slot.ptr != nullptr) {
    const unsigned long long id = current_ctx_id();
    if (id != 0 && id == slot.ctx_id) {
      *out = slot.ptr;
      return cudaSuccess;
    }
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_prepare_scratch);   // also makes the primary context current
  if (e != cudaSuccess) return e;
  slot.ptr = p;
  slot.ctx_id = current_ctx_id();
  *out = p;
  return cudaSuccess;
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
  if (vcattn::fault_injected(fn))
    return vcattn::record_error(VCATTN_ERR_INJECTED, "vcattn_prepare_fp8_noalloc: injected fault");
  if (!(D == 64 || D == 128)) return arg_error(std::string(fn) + ": D must be 64 or 128");
  if (B <= 0 || H <= 0 || N <= 0) return arg_error(std::string(fn) + ": empty shape");
  // The size limit is checked before anything else touches the buffers.  The
  // scratch holds the K token mean, needed when K is smoothed and quantised.
  const int G = B * H;
  const size_t need = ((flags & VCATTN_SMOOTH_K) && k8 != nullptr) ? vcattn::prepare_workspace_bytes(G, N, D) : 0;
  if (need > kScratchBytes)
    return arg_error(std::string(fn) + ": shape needs " + std::to_string(need) +
                     " bytes of scratch, above this entry point's fixed " + std::to_string(kScratchBytes) +
                     "-byte limit; use vcattn_prepare_fp8 with a workspace");
  const int rc = vcattn::prepare_fp8_checks(fn, q, k, v, dtype, B, H, N, D, perm, perm_rows, block_rows, q8, q_scale,
                                            k8, k_scale, v8, v_scale, mu, v8t, route);
  if (rc != VCATTN_OK) return rc;
  const int n_pad = (N + block_rows - 1) / block_rows * block_rows;
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
