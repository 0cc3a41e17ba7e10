// A variant of the fused paged decode-attention entry point that allocates
// nothing: its scratch lives in a fixed array of device memory inside this
// library instead of a buffer the caller provides.
//
// It exists for callers that cannot allocate device memory: clients that bind
// the C ABI from a host language with no CUDA allocator of its own, and serving
// loops that forbid device allocation after start-up so that their memory use
// stays fixed.  They still pass every input and output buffer; only the
// scratch moves into the library.
//
// Limits and sharing:
//   * the array holds PAGER_NOALLOC_SCRATCH_BYTES (32 MiB) and is reserved on
//     every GPU that loads the library, for as long as the process runs;
//   * a call whose scratch requirement for the backend it passes (the size
//     pager_paged_decode_scratch_bytes gives covers every backend) is larger is
//     rejected with PAGER_ERR_SCRATCH;
//   * every call on a device uses the same array and leaves its contents
//     behind; nothing in it needs to start at zero (every value the kernels
//     read was written earlier in the same call), but calls that overlap on the
//     GPU -- on different streams, or from different threads -- race on it;
//   * the first call on a device looks up the array's device address (with
//     that device current) and caches it; make that first call before any
//     stream capture.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "pager_b200.h"

namespace pager {
void set_last_error(const char* msg);  // pager_abi.cu: the message pager_last_error() returns
size_t paged_scratch_bytes_for_backend(int batch, int num_q_heads, int num_kv_heads, int head_dim, int kv_dtype,
                                       int tokens_per_block, int max_row_tokens, int backend);  // pager_abi.cu
}

namespace {

constexpr size_t kNoallocBytes = PAGER_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

std::mutex g_mu;
void* g_ptr[128];  // per device: device address of g_noalloc_scratch (host code cannot use the symbol itself)

int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 128) {
    pager::set_last_error((std::string("pager_paged_decode_attention_noalloc: cudaGetDevice failed: ") +
                           cudaGetErrorString(e)).c_str());
    return PAGER_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      pager::set_last_error((std::string("pager_paged_decode_attention_noalloc: cudaGetSymbolAddress failed: ") +
                             cudaGetErrorString(e)).c_str());
      return PAGER_ERR_CUDA;
    }
    g_ptr[dev] = p;
  }
  *out = g_ptr[dev];
  return PAGER_OK;
}

}  // namespace

extern "C" {

int pager_paged_decode_attention_noalloc(const void* q, int q_dtype, const void* dev_pool, int dev_slots,
                                         const void* host_pool, int host_slots, int kv_dtype, int num_layers,
                                         int layer, int num_kv_heads, int tokens_per_block, int head_dim,
                                         const int32_t* block_table, int max_blocks, const int32_t* num_blocks,
                                         const void* tail_k, const void* tail_v, const int32_t* tail_len,
                                         int tail_cap, const int32_t* valid_lo, const int32_t* valid_hi,
                                         const int32_t* active, int batch, int num_q_heads, float scale,
                                         float softcap, int max_row_tokens, void* out, int out_dtype,
                                         float* block_mass, float* mass_accum, int mass_mode, int backend,
                                         void* stream) {
  // sized for the backend this call asks for (the regular entry checks the same plan); a call whose
  // arguments are rejected sizes to 0 here and gets the regular entry's own error below
  const size_t need = pager::paged_scratch_bytes_for_backend(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype,
                                                             tokens_per_block, max_row_tokens, backend);
  if (need > kNoallocBytes) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "pager_paged_decode_attention_noalloc: this call needs %zu bytes of scratch, the built-in array holds "
             "%zu; use pager_paged_decode_attention with a caller-provided buffer",
             need, kNoallocBytes);
    pager::set_last_error(buf);
    return PAGER_ERR_SCRATCH;
  }
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  return pager_paged_decode_attention(q, q_dtype, dev_pool, dev_slots, host_pool, host_slots, kv_dtype, num_layers,
                                      layer, num_kv_heads, tokens_per_block, head_dim, block_table, max_blocks,
                                      num_blocks, tail_k, tail_v, tail_len, tail_cap, valid_lo, valid_hi, active,
                                      batch, num_q_heads, scale, softcap, max_row_tokens, out, out_dtype, block_mass,
                                      mass_accum, mass_mode, backend, scratch, kNoallocBytes, stream);
}

}  // extern "C"
