// coalibi_bwd_noalloc: the backward with its scratch taken from a fixed,
// library-owned device array instead of a caller-provided workspace.
//
// Who needs it: callers that cannot hand us a workspace because they cannot
// allocate device memory at the point of the call -- a plugin host or C/FFI
// caller that owns only the tensors it passes and has no device allocator to
// share, or code that must not call cudaMalloc there because cudaMalloc can
// synchronise the whole device and, inside a process whose memory is managed by
// a caching allocator, competes with it for the same pool.
//
// The backward's scratch (the per-row delta and the per-32-key carries -- z
// suffix and dA prefix -- that pass A hands to pass B) lives in
// kNoallocScratchBytes of file-scope __device__ memory.  Every GPU that loads this library holds that much memory until the
// process exits.  Problems whose scratch would exceed it are rejected with
// COALIBI_ERR_WORKSPACE before anything is launched.
//
// All calls on a device share the one array and it keeps whatever the last call
// wrote; nothing in it has to start at zero, because every word the kernels
// read is written earlier in the same call.  Two calls whose kernels overlap on
// the GPU (different streams, or different host threads) race on the array and
// corrupt each other's results: serialise them.
//
// The device address of the array is looked up with cudaGetSymbolAddress once
// per device, with that device current, by the first call made on that device
// (a failed lookup is not remembered: the next call tries again).  Make that
// first call before any stream capture begins.  The address is not looked up
// again afterwards, so it is stale after cudaDeviceReset on that device.
//
// Like every entry point of the library, the call leaves the calling thread's
// current CUDA context as it found it.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "coalibi.h"
#include "ctx_guard.h"

namespace coalibi {
void set_last_error_detail(const char* msg);
int check_common(int B, int Hq, int Hkv, int Sq, int Skv, int D, int dtype, int slopes_dtype);
}

namespace {

constexpr size_t kNoallocScratchBytes = COALIBI_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// Host code must not use &g_noalloc_scratch as a device address: on the host
// this name denotes a shadow object.  The device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

struct NoallocDevice {
  std::mutex mu;
  void* ptr = nullptr;  // set once, by the first successful lookup on the device
};
NoallocDevice g_noalloc[kMaxDevices];

}  // namespace

extern "C" int coalibi_bwd_noalloc(const CoalibiBwdArgs* args, void* stream) {
  if (args == nullptr || args->q == nullptr) return COALIBI_ERR_NULL_POINTER;
  // Shape and size checks first: pure arithmetic, nothing touches the device.
  if (int rc = coalibi::check_common(args->B, args->Hq, args->Hkv, args->Sq, args->Skv, args->D, args->dtype,
                                     args->slopes_dtype))
    return rc;
  // the smallest scratch any path of the backward can run in (the path that fits
  // the array is chosen inside coalibi_bwd)
  const size_t need = coalibi_bwd_workspace_min_bytes(args->B, args->Hq, args->Hkv, args->Sq, args->Skv, args->D);
  if (need == 0) return COALIBI_ERR_SHAPE;
  if (need > kNoallocScratchBytes) {
    char msg[200];
    snprintf(msg, sizeof(msg),
             "coalibi_bwd_noalloc: this problem needs %zu bytes of backward scratch, more than the %zu-byte "
             "static scratch; use coalibi_bwd with a caller workspace",
             need, kNoallocScratchBytes);
    coalibi::set_last_error_detail(msg);
    return COALIBI_ERR_WORKSPACE;
  }
  // Per-device state is touched with the device that owns q current; the guard
  // puts the caller's context back on return.
  coalibi::CtxGuard guard;
  if (int rc = coalibi::enter_device(args->q, stream)) return rc;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return COALIBI_ERR_DEVICE;
  }
  NoallocDevice& st = g_noalloc[dev];
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(st.mu);
    if (st.ptr == nullptr) {
      void* p = nullptr;
      const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (err != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        char msg[160];
        snprintf(msg, sizeof(msg), "coalibi_bwd_noalloc: cudaGetSymbolAddress failed: %s",
                 cudaGetErrorString(err));
        coalibi::set_last_error_detail(msg);
        return COALIBI_ERR_LAUNCH;
      }
      st.ptr = p;
    }
    scratch = st.ptr;
  }
  CoalibiBwdArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kNoallocScratchBytes;
  return coalibi_bwd(&a, stream);
}
