// Host-side helpers shared by the C ABI translation units.
#pragma once
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>
#include <cuda.h>
#include <cuda_runtime.h>
#include "../../include/fxb200.h"

namespace fxb {

// Records the message for fxb_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

// Wraps a CUDA runtime status; FXB_OK when success.
int check_cuda(cudaError_t e, const char* what);

// Counts kernel launches made by this library (fxb_launch_count).
void count_launch();

// Launch-time check: picks up configuration errors of the launch just made
// and counts the launch.
inline int check_launch(const char* what) {
  count_launch();
  return check_cuda(cudaGetLastError(), what);
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch is on unless FXB_PDL=0 in the environment.
bool pdl_enabled();

// Launches kernel `k` with programmatic dependent launch allowed: its CTAs may
// be scheduled (and run their prologue: barrier init, tensor-memory
// allocation, descriptor prefetch) while the previous kernel on the stream is
// draining. Every kernel of this library calls pdl_wait() (griddepcontrol.wait:
// the previous kernel has completed and its writes are visible) before its
// first global-memory access, so stream order is preserved.
// A launch error is left for the check_launch() that follows every launch.
template <typename... KArgs, typename... Args>
void pdl_launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  (void)cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int32_t dt) {
  switch (dt) {
    case FXB_DTYPE_F32: return 4;
    case FXB_DTYPE_F16: return 2;
    case FXB_DTYPE_BF16: return 2;
    default: return 0;
  }
}

// Device address of the error word of the current device (kernels OR bits
// into it when a bounded wait expires); nullptr + error set on failure.
int* dev_error_ptr();

// Identity of the calling thread's current CUDA context (0 if none). Caches
// of device addresses are keyed on it as well as on the device ordinal: a
// cudaDeviceReset() ends the primary context, the next call creates a new one
// and addresses looked up in the old one are stale.
uintptr_t context_token();

// Cached SM count of the current device.
int num_sms();

// cuTensorMapEncodeTiled obtained through the runtime's driver entry point
// (the library does not link libcuda directly).
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

}  // namespace fxb
