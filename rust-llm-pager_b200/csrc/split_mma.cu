// Tensor-core (mma.sync m16n8k16, fp32 accumulate) split kernels: fp16 / bf16 KV, head_dim 64 / 128 / 256,
// every mode including the SCORES / VALUES passes of reference-exact rounding.
#include "split_inst.cuh"

namespace pager {
bool lookup_split_mma(int kv_dtype, int head_dim, int mode, SplitKernelInfo* out) {
  if (kv_dtype == 1) {
    switch (head_dim) {
      PAGER_EXACT_MODE_CASES(__half, 64)
      PAGER_EXACT_MODE_CASES(__half, 128)
      PAGER_EXACT_MODE_CASES(__half, 256)
      default: return false;
    }
  }
  if (kv_dtype == 2) {
    switch (head_dim) {
      PAGER_EXACT_MODE_CASES(__nv_bfloat16, 64)
      PAGER_EXACT_MODE_CASES(__nv_bfloat16, 128)
      PAGER_EXACT_MODE_CASES(__nv_bfloat16, 256)
      default: return false;
    }
  }
  return false;
}
}  // namespace pager
