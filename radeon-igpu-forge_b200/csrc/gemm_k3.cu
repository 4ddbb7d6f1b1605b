// tcgen05 GEMM kernels of one epilogue kind: fp32 C (store / residual / bias / accumulate).
#include "common.cuh"
#include "internal.h"
#include "gemm_kernel.cuh"

namespace fxb {
namespace gk {
template int gemm_dispatch<EK_F32>(bool, int, int, bool, bool, const Maps&, const GemmParams&,
                                  int, cudaStream_t);
}  // namespace gk
}  // namespace fxb
