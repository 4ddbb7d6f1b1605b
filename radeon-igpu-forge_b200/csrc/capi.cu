// Library-wide C ABI: version, error reporting, device error word, SM count,
// and the tensor-map encoder used by the TMA-fed kernels.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include "common.cuh"
#include "internal.h"

// Error word set by kernels whose bounded waits expire (one per device).
__device__ int g_fxb_dev_error = 0;

namespace fxb {

static thread_local std::string t_last_error;
static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("FXB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FXB_OK;
  return set_error(FXB_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

uintptr_t context_token() {
  typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return 0;
  return reinterpret_cast<uintptr_t>(c);
}

int* dev_error_ptr() {
  static std::mutex mu;
  static int* cached[64] = {nullptr};
  static uintptr_t cached_ctx[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error(FXB_ECUDA, "dev_error_ptr: no current device");
    return nullptr;
  }
  // cudaGetDevice does not create the context; the symbol lookup below does
  // (first call on the device), so the token is read after it on a miss
  std::lock_guard<std::mutex> lock(mu);
  const uintptr_t ctx = context_token();
  if (!cached[dev] || ctx == 0 || cached_ctx[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fxb_dev_error) != cudaSuccess) {
      set_error(FXB_ECUDA, "dev_error_ptr: cudaGetSymbolAddress failed");
      return nullptr;
    }
    cached[dev] = static_cast<int*>(p);
    cached_ctx[dev] = context_token();
  }
  return cached[dev];
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn(int* err) {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  static int status = FXB_OK;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      status = FXB_ECUDA;
      return;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  *err = status;
  return fn;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  int st = FXB_OK;
  EncodeTiledFn fn = get_encode_fn(&st);
  if (!fn) return set_error(FXB_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes),
                  reinterpret_cast<const cuuint32_t*>(box), estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FXB_EINVAL, "cuTensorMapEncodeTiled failed (CUresult %d, rank %u)", (int)r,
                     rank);
  return FXB_OK;
}

}  // namespace fxb

extern "C" {

int fxb_version(void) { return 200; }  // 0.2.0: fxb_gemm_args.workspace

const char* fxb_last_error(void) { return fxb::t_last_error.c_str(); }

int fxb_device_error(int32_t* code, int32_t clear) {
  if (!code) return fxb::set_error(FXB_EINVAL, "fxb_device_error: code is NULL");
  int r = fxb::check_cuda(cudaDeviceSynchronize(), "fxb_device_error sync");
  if (r) return r;
  int v = 0;
  r = fxb::check_cuda(cudaMemcpyFromSymbol(&v, g_fxb_dev_error, sizeof(int)),
                      "fxb_device_error read");
  if (r) return r;
  *code = v;
  if (clear) {
    int z = 0;
    r = fxb::check_cuda(cudaMemcpyToSymbol(g_fxb_dev_error, &z, sizeof(int)),
                        "fxb_device_error clear");
  }
  return r;
}

uint64_t fxb_launch_count(void) { return fxb::g_launches.load(std::memory_order_relaxed); }

size_t fxb_abi_struct_size(int32_t which) {
  if (which == 0) return sizeof(fxb_gemm_args);
  if (which == 1) return sizeof(fxb_attn_args);
  return 0;
}

int fxb_num_sms(int32_t* out) {
  if (!out) return fxb::set_error(FXB_EINVAL, "fxb_num_sms: out is NULL");
  *out = fxb::num_sms();
  return FXB_OK;
}

}  // extern "C"
