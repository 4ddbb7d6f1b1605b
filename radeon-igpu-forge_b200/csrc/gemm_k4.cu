// tcgen05 GEMM kernels of one epilogue kind: per-row softmax statistics of the
// logits tiles (loss-only linear cross entropy; no C written).
#include "common.cuh"
#include "internal.h"
#include "gemm_kernel.cuh"

namespace fxb {
namespace gk {
template int gemm_dispatch<EK_CESTAT>(bool, int, int, bool, bool, const Maps&, const GemmParams&,
                                      int, cudaStream_t);
}  // namespace gk
}  // namespace fxb
