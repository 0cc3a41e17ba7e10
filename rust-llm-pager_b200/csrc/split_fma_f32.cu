// CUDA-core (fp32 FMA) split kernels for float KV, every supported head_dim.
#include "split_inst.cuh"

namespace pager {
bool lookup_split_fma_f32(int head_dim, int mode, SplitKernelInfo* out) {
  switch (head_dim) {
    PAGER_MODE_CASES(float, 8, BACKEND_FMA)
    PAGER_MODE_CASES(float, 16, BACKEND_FMA)
    PAGER_MODE_CASES(float, 32, BACKEND_FMA)
    PAGER_MODE_CASES(float, 64, BACKEND_FMA)
    PAGER_MODE_CASES(float, 128, BACKEND_FMA)
    PAGER_MODE_CASES(float, 256, BACKEND_FMA)
    default: return false;
  }
}
}  // namespace pager
