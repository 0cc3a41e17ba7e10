// Copying one layer of host-pool blocks into the device staging buffer.
//
// The host tier can be read two ways: zero-copy by the decode kernel (mapped
// pinned memory, every byte crossing the link on SM loads) or staged by the
// copy engines: before a layer's kernel runs, each host block's chunk of that
// layer ([2, kv_heads, tokens_per_block, head_dim], contiguous inside the
// slot) is copied into a device staging buffer with cudaMemcpy2DAsync, and
// the kernel reads it from there with TMA.  Consecutive host slots that land
// in consecutive staging slots form one strided 2D copy (source pitch = the
// host slot size, destination pitch = the chunk size), so one call moves a
// whole run of blocks.  The caller issues the next layer's copies on a copy
// stream while the current layer computes.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "pager_b200.h"

namespace pager {
void set_last_error(const char* msg);
}

extern "C" int pager_stage_host_blocks(void* stage, const void* host_pool, int64_t slot_bytes,
                                       int64_t layer_offset_bytes, int64_t chunk_bytes, const int32_t* run_src,
                                       const int32_t* run_dst, const int32_t* run_len, int nruns, void* stream) {
  char buf[256];
  if (nruns < 0 || (nruns > 0 && (!stage || !host_pool || !run_src || !run_dst || !run_len))) {
    pager::set_last_error("pager_stage_host_blocks: null pointer or negative run count");
    return PAGER_ERR_INVALID;
  }
  if (nruns == 0) return PAGER_OK;
  if (chunk_bytes <= 0 || slot_bytes < chunk_bytes || layer_offset_bytes < 0 ||
      layer_offset_bytes + chunk_bytes > slot_bytes) {
    pager::set_last_error("pager_stage_host_blocks: chunk must lie inside a slot");
    return PAGER_ERR_INVALID;
  }
  const char* src = static_cast<const char*>(host_pool);
  char* dst = static_cast<char*>(stage);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int r = 0; r < nruns; ++r) {
    if (run_src[r] < 0 || run_dst[r] < 0 || run_len[r] <= 0) {
      snprintf(buf, sizeof(buf), "pager_stage_host_blocks: bad run %d (src %d, dst %d, len %d)", r, run_src[r],
               run_dst[r], run_len[r]);
      pager::set_last_error(buf);
      return PAGER_ERR_INVALID;
    }
    const cudaError_t e = cudaMemcpy2DAsync(dst + (int64_t)run_dst[r] * chunk_bytes, (size_t)chunk_bytes,
                                            src + (int64_t)run_src[r] * slot_bytes + layer_offset_bytes,
                                            (size_t)slot_bytes, (size_t)chunk_bytes, (size_t)run_len[r],
                                            cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
      snprintf(buf, sizeof(buf), "pager_stage_host_blocks: cudaMemcpy2DAsync failed: %s", cudaGetErrorString(e));
      pager::set_last_error(buf);
      return PAGER_ERR_CUDA;
    }
  }
  return PAGER_OK;
}
