// moe_forward_static_scratch: the MoE forward for callers that cannot allocate
// device memory.
//
// moe_forward needs a caller-provided workspace (moe_workspace_bytes(T) bytes of
// device memory for the normalised activations, the routing tables, the
// dispatched rows and the expert outputs).  Some callers have no way to provide
// one: a host reached through a thin FFI (a Go, Java or C program that only owns
// the activation buffers it passes in), a process whose memory pool has already
// claimed the GPU so that one more cudaMalloc fails, or a serving loop that must
// not call cudaMalloc because it synchronises the device.  For them this file
// keeps one fixed scratch area in the library itself and runs exactly the
// kernels moe_forward runs, with that area as the workspace.
//
// The scratch is a file-scope __device__ array of MOE_STATIC_SCRATCH_BYTES
// (32 MiB).  Every GPU on which the library's module is loaded holds those
// 32 MiB until the process exits.  The name `g_static_scratch` is only a
// host-side handle in host code; the device address is obtained once per device
// with cudaGetSymbolAddress (below) and passed to the kernels.
#include <mutex>
#include <string>

#include "common.cuh"
#include "moe_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = MOE_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) char g_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on `device`, looked up the first time a
// device is used (with that device current) and cached afterwards.
cudaError_t scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[device] == nullptr) {
    void* ptr = nullptr;
    cudaError_t st = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (st != cudaSuccess) return st;
    g_scratch_addr[device] = ptr;
  }
  *out = g_scratch_addr[device];
  return cudaSuccess;
}

int fail(int code, const std::string& msg) {
  moe::set_error(msg);
  return code;
}

int cuda_fail(cudaError_t st, const char* what) {
  return fail(MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(st));
}

}  // namespace

#define MOE_NA_CUDA(call)                                  \
  do {                                                     \
    cudaError_t st_ = (call);                              \
    if (st_ != cudaSuccess) return cuda_fail(st_, #call);  \
  } while (0)

// Makes `device` current for the lifetime of the object and puts the caller's
// current device back afterwards, so that a host thread driving several GPUs
// keeps the device it had selected.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    st_ = cudaGetDevice(&prev_);
    if (st_ == cudaSuccess && prev_ != device) {
      st_ = cudaSetDevice(device);
      switched_ = st_ == cudaSuccess;
    }
  }
  ~DeviceGuard() {
    if (switched_) cudaSetDevice(prev_);
  }
  cudaError_t status() const { return st_; }

 private:
  int prev_ = 0;
  bool switched_ = false;
  cudaError_t st_ = cudaSuccess;
};

extern "C" int moe_forward_static_scratch(MoePlan* plan, const float* x_dev, float* out_dev,
                                          int32_t T, void* stream) {
  using namespace moe;
  if (!plan) return fail(MOE_ERR_INVALID, "null plan");
  Plan& p = plan->p;
  if (!p.bound) return fail(MOE_ERR_NOT_BOUND, "moe_bind_layer has not been called");
  if (p.n_local != p.E)
    return fail(MOE_ERR_UNSUPPORTED,
                "this plan holds a share of the experts: use the moe_ep_* entry points");
  if (T < 0 || T > p.cfg.max_tokens) return fail(MOE_ERR_INVALID, "T outside [0, max_tokens]");
  if (T == 0) return MOE_OK;
  if (!x_dev || !out_dev) return fail(MOE_ERR_INVALID, "null x / out");
  if (moe::misaligned16(x_dev) || moe::misaligned16(out_dev))
    return fail(MOE_ERR_INVALID, "x and out must be 16-byte aligned");
  if (x_dev == out_dev) return fail(MOE_ERR_INVALID, "x and out may not alias");
  if (p.device < 0 || p.device >= kMaxDevices)
    return fail(MOE_ERR_UNSUPPORTED, "device ordinal beyond the static scratch table");
  const WsLayout L = ws_layout(p, T);
  if (L.total > kStaticScratchBytes)
    return fail(MOE_ERR_WORKSPACE,
                "this layer needs " + std::to_string(L.total) + " bytes of scratch for T=" +
                    std::to_string(T) + ", more than the " + std::to_string(kStaticScratchBytes) +
                    "-byte static scratch; use moe_forward with a workspace or a smaller T");
  // The symbol lookup below needs the plan's device current; the guard puts the
  // caller's device back on every return path.
  DeviceGuard guard(p.device);
  MOE_NA_CUDA(guard.status());
  void* scratch = nullptr;
  MOE_NA_CUDA(scratch_address(p.device, &scratch));

  // Same kernel sequence as moe_forward.  The router's split counters must
  // start at zero: launch_route clears them with a stream memset at the start of
  // every call, and the tile-list builders zero the split-K arrival counters.
  // Every other scratch byte a kernel reads is written earlier in the same call,
  // so nothing else has to be cleared between calls.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(scratch);
  if (p.E == 0) {  // dense MLP plan: normalised rows and the shared-expert tile map
    MOE_NA_CUDA(launch_row_prep(p, L, ws, x_dev, T, s));
    MOE_NA_CUDA(launch_shared_tiles(p, L, ws, T, s));
  } else {
    MOE_NA_CUDA(launch_route(p, L, ws, x_dev, T, true, s));
  }
  MOE_NA_CUDA(launch_gemm(p, L, ws, false, T, s));
  MOE_NA_CUDA(launch_gemm(p, L, ws, true,
                       GemmIO{T * p.K, T, reinterpret_cast<__half*>(ws + L.y), nullptr, p.n_local}, s));
  MOE_NA_CUDA(launch_combine_half(p, x_dev, reinterpret_cast<const __half*>(ws + L.y),
                             reinterpret_cast<float*>(ws + L.y_s),
                             reinterpret_cast<int32_t*>(ws + L.slot_row),
                             reinterpret_cast<float*>(ws + L.wts),
                             reinterpret_cast<float*>(ws + L.sgate), out_dev, T, s));
  return MOE_OK;
}
