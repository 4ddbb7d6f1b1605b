// tcgen05 GEMM kernels of one epilogue kind: GELU / bias+GELU / bias+SiLU, 16-bit C.
#include "common.cuh"
#include "internal.h"
#include "gemm_kernel.cuh"

namespace fxb {
namespace gk {
template int gemm_dispatch<EK_ACT16>(bool, int, int, bool, bool, const Maps&, const GemmParams&,
                                  int, cudaStream_t);
}  // namespace gk
}  // namespace fxb
