// Appending one decode step's new K/V into pool slots.
//
// A decode session keeps its tail (the tokens after its last full block) in a
// slot of the device pool, in the same [layers, 2, kv_heads, tokens_per_block,
// head_dim] layout as a full block, and the decode op reads it through the
// block table with valid_hi marking how many of its tokens are real.  Each
// step's new token goes straight into that slot at its position: the
// equivalent of the reference's tail concatenation
// (pager_hf/batched_decode.py:170-171, paged_model.py's DynamicCache.update)
// without rebuilding the tail, and when the tail fills up it already is a full
// block in the pool (no copy to form it, kv_utils.py:37-53).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "pager_b200.h"

namespace pager {
void set_last_error(const char* msg);
int current_status_word(int** out);
}  // namespace pager

namespace {

constexpr int kBadSlot = 6;  // same code the decode kernel uses for an out-of-range slot

struct AppendParams {
  char* pool;
  const char* k_new;  // [batch, kv_heads, head_dim]
  const char* v_new;
  const int32_t* slots;      // [batch], < 0 = skip the row
  const int32_t* positions;  // [batch], token index inside the slot
  long long pool_slots;
  int layers, layer, kv_heads, tpb, row_bytes;
  int* status;
};

template <int UNIT>
__global__ void __launch_bounds__(128) append_tokens_kernel(const AppendParams p) {
  using V = typename std::conditional<UNIT == 16, uint4, typename std::conditional<UNIT == 4, uint32_t, uint16_t>::type>::type;
  const int b = blockIdx.x;
  const int slot = p.slots[b];
  if (slot < 0) return;
  const int pos = p.positions[b];
  if (slot >= p.pool_slots || pos < 0 || pos >= p.tpb) {
    if (threadIdx.x == 0) atomicExch(p.status, kBadSlot);
    return;
  }
  const int per_row = p.row_bytes / UNIT;
  const int total = 2 * p.kv_heads * per_row;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int c = i % per_row;
    const int kvh = i / per_row;
    const int h = kvh % p.kv_heads;
    const int kv = kvh / p.kv_heads;
    const V* src = reinterpret_cast<const V*>((kv ? p.v_new : p.k_new) + ((long long)b * p.kv_heads + h) * p.row_bytes) + c;
    const long long row = ((((long long)slot * p.layers + p.layer) * 2 + kv) * p.kv_heads + h) * p.tpb + pos;
    V* dst = reinterpret_cast<V*>(p.pool + row * p.row_bytes) + c;
    *dst = *src;
  }
}

int fail(int code, const char* msg) {
  pager::set_last_error(msg);
  return code;
}

}  // namespace

namespace pager {
// The append kernels (by copy unit: 16, 4, 2 bytes), for the library's load of every kernel at its
// first call on a device.
const void* append_kernel_fn(int i) {
  return i == 0 ? reinterpret_cast<const void*>(&append_tokens_kernel<16>)
                : (i == 1 ? reinterpret_cast<const void*>(&append_tokens_kernel<4>)
                          : reinterpret_cast<const void*>(&append_tokens_kernel<2>));
}
}  // namespace pager

extern "C" int pager_append_tokens(void* pool, int dtype, int pool_slots, int num_layers, int layer,
                                   int num_kv_heads, int tokens_per_block, int head_dim, const int32_t* slots,
                                   const int32_t* positions, const void* k_new, const void* v_new, int batch,
                                   void* stream) {
  if (batch < 0 || pool_slots < 0 || num_layers <= 0 || num_kv_heads <= 0 || tokens_per_block <= 0 || head_dim <= 0)
    return fail(PAGER_ERR_INVALID, "pager_append_tokens: bad geometry");
  if (layer < 0 || layer >= num_layers) return fail(PAGER_ERR_INVALID, "pager_append_tokens: layer out of range");
  if (dtype != PAGER_DTYPE_F32 && dtype != PAGER_DTYPE_F16 && dtype != PAGER_DTYPE_BF16)
    return fail(PAGER_ERR_INVALID, "pager_append_tokens: unknown dtype code");
  if (batch == 0) return PAGER_OK;
  if (!pool || !slots || !positions || !k_new || !v_new)
    return fail(PAGER_ERR_INVALID, "pager_append_tokens: null pointer");
  const int elt = dtype == PAGER_DTYPE_F32 ? 4 : 2;
  AppendParams p;
  p.pool = static_cast<char*>(pool);
  p.k_new = static_cast<const char*>(k_new);
  p.v_new = static_cast<const char*>(v_new);
  p.slots = slots;
  p.positions = positions;
  p.pool_slots = pool_slots;
  p.layers = num_layers;
  p.layer = layer;
  p.kv_heads = num_kv_heads;
  p.tpb = tokens_per_block;
  p.row_bytes = head_dim * elt;
  const int rc = pager::current_status_word(&p.status);
  if (rc) return rc;
  const auto aligned = [](const void* x, int a) { return (reinterpret_cast<uintptr_t>(x) % a) == 0; };
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p.row_bytes % 16 == 0 && aligned(pool, 16) && aligned(k_new, 16) && aligned(v_new, 16))
    append_tokens_kernel<16><<<batch, 128, 0, st>>>(p);
  else if (elt == 4 && aligned(pool, 4) && aligned(k_new, 4) && aligned(v_new, 4))
    append_tokens_kernel<4><<<batch, 128, 0, st>>>(p);
  else if (aligned(pool, 2) && aligned(k_new, 2) && aligned(v_new, 2))
    append_tokens_kernel<2><<<batch, 128, 0, st>>>(p);
  else
    return fail(PAGER_ERR_INVALID, "pager_append_tokens: misaligned tensors");
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "pager_append_tokens launch: %s", cudaGetErrorString(e));
    return fail(PAGER_ERR_CUDA, buf);
  }
  return PAGER_OK;
}
