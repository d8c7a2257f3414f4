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
// per device with cudaGetSymbolAddress, with that device current, and cached.  That
// lookup happens inside the FIRST call on each device; make that first call before any
// CUDA stream capture begins.
//
// All calls share the one array: two calls whose GPU work overlaps (different streams,
// different handles on the same device, or another thread) race on it and corrupt each
// other's results.  Serialise them (one stream, or events).  The array keeps whatever the
// previous call left; nothing in the forward reads scratch it has not first written in the
// same call (routing tables, slots, offsets and all rows that reach the output are rewritten
// every time), so no clearing is needed between calls.
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
void* g_workspace_on_device[kMaxDevices] = {};

// Device address of the static workspace on `device` (looked up once, then cached).
cudaError_t workspace_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_workspace_on_device[device]) {
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaError_t e = cudaSuccess;
    if (prev != device) e = cudaSetDevice(device);
    void* p = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_no_alloc_workspace);
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return e;
    g_workspace_on_device[device] = p;
  }
  *out = g_workspace_on_device[device];
  return cudaSuccess;
}

}  // namespace

extern "C" int vmoe_forward_no_alloc(vmoe_handle* h, const void* x, int64_t tokens, void* out,
                                     float* router_logits, int32_t* topk_idx, float* topk_w,
                                     int32_t* expert_counts, float* aux_loss, void* stream) {
  if (!h) return VMOE_ERR_INVALID_ARG;
  size_t need = 0;
  int rc = vmoe_workspace_size(h, tokens, &need);
  if (rc != VMOE_OK) return rc;
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
