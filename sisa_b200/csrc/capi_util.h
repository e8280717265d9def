// capi_util.h - argument checks and device binding shared by the C-ABI entry points (defined in capi.cu).
#pragma once
#include <cstdint>

#include "sisa_b200.h"

namespace sisa {

// Records `msg` for sisa_last_error() and returns `code`.
int capi_fail(int code, const char* msg);
// B, H, L >= 1 and within the grid limits of the kernels.
int capi_check_dims(int64_t B, int64_t H, int64_t L);
// Non-null, 16-byte aligned view with positive row stride and 16-byte multiples as strides.
int capi_check_view(const sisa_view4* v, int elem_bytes, const char* name);
int capi_check_dtype(int dtype);

// Makes the device that owns an entry point's data current on the calling thread for the length of
// the call. The destructor gives the thread back the context it had before bind() (or none), so an
// entry point never changes its caller's current device. Tensor-map encoding needs a current context,
// which a thread that has not touched CUDA yet (an autograd worker, a foreign host thread) lacks.
class DeviceScope {
 public:
  DeviceScope() = default;
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
  ~DeviceScope();
  // Binds the device of `ptr` (device or managed memory). Returns SISA_OK or an error code.
  int bind(const void* ptr);
  int device() const { return device_; }

 private:
  void* prev_ = nullptr;   // the CUcontext that was current before bind()
  bool bound_ = false;
  int device_ = -1;
};

}  // namespace sisa
