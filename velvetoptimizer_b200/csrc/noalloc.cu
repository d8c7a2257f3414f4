// vmoe_forward_no_alloc: the MoE forward with its scratch in a static device array.
//
// Who needs this: callers that cannot call cudaMalloc (or any allocator) at the moment
// they run the layer -- an inference server's request thread working under a fixed
// memory budget that forbids growing device allocations, a real-time loop where an
// allocation could stall or fail mid-request, or a host runtime (e.g. a Rust or C engine
// without a caching allocator) that has no way to hand out a workspace.  They still own
// and pass x, out and the optional outputs; only the intermediate scratch (routing tables,
// the permuted activations, the gate/up and down results) comes from here.
//
// The scratch is one file-scope __device__ array of kNoAllocWorkspaceBytes (64 MiB).
// Every GPU that loads this library reserves it until the process exits, whether or not
// this entry point is used.  Host code cannot use the array's name as a device address
// (in host code it names a host-side stand-in), so the device address is looked up once
// per device with cudaGetSymbolAddress, with that device current, and cached together
// with the unique id of the CUDA context it belongs to.  That lookup happens inside the
// FIRST call on each device; make that first call before any CUDA stream capture begins.
// If the device's context is later destroyed and recreated (cudaDeviceReset), the next
// call sees a new context id and looks the address up again -- but a reset also frees
// every handle's weights, so handles must be recreated after one anyway.
//
// All calls share the one array: two calls whose GPU work overlaps (different streams,
// different handles on the same device, or another thread) race on it and corrupt each
// other's results.  Serialise them (one stream, or events).  The array keeps whatever the
// previous call left; nothing in the forward reads scratch it has not first written in the
// same call (routing tables, slots, offsets and all rows that reach the output are rewritten
// every time), so no clearing is needed between calls.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>

#include "../../include/vesper_moe.h"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocWorkspaceBytes = static_cast<size_t>(VMOE_NO_ALLOC_WORKSPACE_BYTES);
static_assert(kNoAllocWorkspaceBytes % 256 == 0, "workspace size must keep 256-byte alignment");

__device__ __align__(256) unsigned char g_no_alloc_workspace[kNoAllocWorkspaceBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct CachedAddress {
  unsigned long long ctx_id = 0;  // unique id of the context the address belongs to
  void* ptr = nullptr;
};
CachedAddress g_workspace_on_device[kMaxDevices];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context (0 when it cannot be read).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    looked_up = true;
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx &&
      get_id(ctx, &id) == CUDA_SUCCESS)
    return id;
  return 0;
}

// Device address of the static workspace on `device`: looked up with that device current
// on the first call (and again if the device's context was recreated), then cached.
cudaError_t workspace_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  cudaError_t e = cudaSuccess;
  if (prev != device) e = cudaSetDevice(device);
  if (e == cudaSuccess) {
    CachedAddress& c = g_workspace_on_device[device];
    const unsigned long long id = current_context_id();
    if (!c.ptr || id != c.ctx_id) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_no_alloc_workspace);
      if (e == cudaSuccess) {
        c.ptr = p;
        c.ctx_id = id;
      }
    }
    if (e == cudaSuccess) *out = c.ptr;
  }
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return e;
}

}  // namespace

extern "C" int vmoe_forward_no_alloc(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                                     float* router_logits, int32_t* topk_idx, float* topk_w,
                                     int32_t* expert_counts, float* aux_loss, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  if (tokens < 0) {
    char msg[128];
    snprintf(msg, sizeof(msg), "vmoe_forward_no_alloc: tokens must be >= 0 (got %lld)",
             static_cast<long long>(tokens));
    return vmoe::set_handle_error(h, VMOE_ERR_INVALID_ARG, msg);
  }
  size_t need = 0;
  int rc = vmoe_workspace_size(h, tokens, &need);
  if (rc != VMOE_OK) return vmoe::set_handle_error(h, rc, "vmoe_forward_no_alloc: workspace size");
  if (need > kNoAllocWorkspaceBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "vmoe_forward_no_alloc: %lld tokens need %zu bytes of scratch but the static "
             "workspace holds %zu bytes (%zu MiB); use vmoe_forward with a caller workspace",
             static_cast<long long>(tokens), need, kNoAllocWorkspaceBytes,
             kNoAllocWorkspaceBytes >> 20);
    return vmoe::set_handle_error(h, VMOE_ERR_WORKSPACE, msg);
  }
  const int device = vmoe::handle_device(h);
  if (device < 0 || device >= kMaxDevices)
    return vmoe::set_handle_error(h, VMOE_ERR_INVALID_ARG, "device index out of range");
  void* ws = nullptr;
  const cudaError_t e = workspace_address(device, &ws);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "cudaGetSymbolAddress of the static workspace failed: %s",
             cudaGetErrorString(e));
    return vmoe::set_handle_error(h, VMOE_ERR_CUDA, msg);
  }
  return vmoe_forward(h, x, tokens, out, router_logits, topk_idx, topk_w, expert_counts,
                      aux_loss, ws, kNoAllocWorkspaceBytes, stream);
}
