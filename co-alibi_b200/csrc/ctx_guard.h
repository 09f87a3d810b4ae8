// Scoped save / restore of the calling thread's current CUDA context.
//
// The C-ABI entry points switch to the device that owns their tensors (the
// tensor-map encoder and the launches need that device's context current).  A
// CtxGuard constructed first in an entry point records the context that was
// current on the calling thread -- possibly none -- and makes it current again
// when the entry point returns, so a caller's device selection is the same after
// the call as before it.
#pragma once

#include <cuda.h>

namespace coalibi {

class CtxGuard {
 public:
  CtxGuard();
  ~CtxGuard();
  CtxGuard(const CtxGuard&) = delete;
  CtxGuard& operator=(const CtxGuard&) = delete;

 private:
  CUcontext saved_ = nullptr;
  bool saved_ok_ = false;
};

// Make the device that owns `ptr` current on this thread, run the once-per-device
// set-up, and check that `stream` (NULL: the legacy default stream) belongs to
// that device.  Returns COALIBI_OK or an error code (detail in coalibi_last_error).
int enter_device(const void* ptr, void* stream);

}  // namespace coalibi
