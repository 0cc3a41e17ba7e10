// CUDA-core (fp32 FMA) split kernels for __half KV, every supported head_dim.
#include "split_inst.cuh"

namespace pager {
bool lookup_split_fma_f16(int head_dim, int mode, SplitKernelInfo* out) {
  switch (head_dim) {
    PAGER_FMA16_MODE_CASES(__half, 8)
    PAGER_FMA16_MODE_CASES(__half, 16)
    PAGER_FMA16_MODE_CASES(__half, 32)
    PAGER_FMA16_MODE_CASES(__half, 64)
    PAGER_FMA16_MODE_CASES(__half, 128)
    PAGER_FMA16_MODE_CASES(__half, 256)
    default: return false;
  }
}
}  // namespace pager
