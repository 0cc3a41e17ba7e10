// Tensor-core (mma.sync m16n8k16, fp32 accumulate) split kernels: fp16 / bf16 KV, head_dim 64 / 128 / 256.
#include "split_inst.cuh"

namespace pager {
bool lookup_split_mma(int kv_dtype, int head_dim, int mode, SplitKernelInfo* out) {
  if (kv_dtype == 1) {
    switch (head_dim) {
      PAGER_MODE_CASES(__half, 64, BACKEND_MMA)
      PAGER_MODE_CASES(__half, 128, BACKEND_MMA)
      PAGER_MODE_CASES(__half, 256, BACKEND_MMA)
      default: return false;
    }
  }
  if (kv_dtype == 2) {
    switch (head_dim) {
      PAGER_MODE_CASES(__nv_bfloat16, 64, BACKEND_MMA)
      PAGER_MODE_CASES(__nv_bfloat16, 128, BACKEND_MMA)
      PAGER_MODE_CASES(__nv_bfloat16, 256, BACKEND_MMA)
      default: return false;
    }
  }
  return false;
}
}  // namespace pager
