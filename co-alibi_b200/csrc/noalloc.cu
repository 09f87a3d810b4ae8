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
// The backward's scratch (the per-row delta and the per-64-key carries pass A
// hands to pass B) lives in kNoallocScratchBytes of file-scope __device__
// memory.  Every GPU that loads this library holds that much memory until the
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
// per device, with that device current, by the first call made on that device.
// Make that first call before any stream capture begins.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "coalibi.h"

namespace coalibi {
void set_last_error_detail(const char* msg);
}

namespace {

constexpr size_t kNoallocScratchBytes = COALIBI_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// Host code must not use &g_noalloc_scratch as a device address: on the host
// this name denotes a shadow object.  The device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

struct NoallocDevice {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};
NoallocDevice g_noalloc[kMaxDevices];

}  // namespace

extern "C" int coalibi_bwd_noalloc(const CoalibiBwdArgs* args, void* stream) {
  if (args == nullptr || args->q == nullptr) return COALIBI_ERR_NULL_POINTER;
  // Size check first: pure arithmetic, nothing touches the device.
  const size_t need = coalibi_bwd_workspace_bytes(args->B, args->Hq, args->Hkv, args->Sq, args->Skv, args->D);
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
  // Make the device that owns q current before touching per-device state.
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, args->q) != cudaSuccess || attr.device < 0 || attr.device >= kMaxDevices) {
    cudaGetLastError();
    return COALIBI_ERR_DEVICE;
  }
  if (cudaSetDevice(attr.device) != cudaSuccess) {
    cudaGetLastError();
    return COALIBI_ERR_DEVICE;
  }
  NoallocDevice& st = g_noalloc[attr.device];
  std::call_once(st.once, [&st] {
    void* p = nullptr;
    st.err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    st.ptr = (st.err == cudaSuccess) ? p : nullptr;
  });
  if (st.err != cudaSuccess || st.ptr == nullptr) {
    char msg[160];
    snprintf(msg, sizeof(msg), "coalibi_bwd_noalloc: cudaGetSymbolAddress failed: %s",
             cudaGetErrorString(st.err));
    coalibi::set_last_error_detail(msg);
    return COALIBI_ERR_LAUNCH;
  }
  CoalibiBwdArgs a = *args;
  a.workspace = st.ptr;
  a.workspace_bytes = kNoallocScratchBytes;
  return coalibi_bwd(&a, stream);
}
