// CUDA-core (fp32 FMA) split kernels for __nv_bfloat16 KV, every supported head_dim.
#include "split_inst.cuh"

namespace pager {
bool lookup_split_fma_bf16(int head_dim, int mode, SplitKernelInfo* out) {
  switch (head_dim) {
    PAGER_FMA16_MODE_CASES(__nv_bfloat16, 8)
    PAGER_FMA16_MODE_CASES(__nv_bfloat16, 16)
    PAGER_FMA16_MODE_CASES(__nv_bfloat16, 32)
    PAGER_FMA16_MODE_CASES(__nv_bfloat16, 64)
    PAGER_FMA16_MODE_CASES(__nv_bfloat16, 128)
    PAGER_FMA16_MODE_CASES(__nv_bfloat16, 256)
    default: return false;
  }
}
}  // namespace pager
