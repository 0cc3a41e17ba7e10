// C ABI of libpager_b200.so: argument checking, split planning, tensor-map
// encoding, the combine / mass / finalize kernels, the pinned host pool and
// the host-link probes.  Declarations and layouts: include/pager_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "pager_b200.h"
#include "pager_split.cuh"

namespace pager {

__device__ int g_status;
const void* append_kernel_fn(int i);  // pager_append.cu

bool lookup_split_mma(int kv_dtype, int head_dim, int mode, SplitKernelInfo* out);
bool lookup_split_fma_f32(int head_dim, int mode, SplitKernelInfo* out);
bool lookup_split_fma_f16(int head_dim, int mode, SplitKernelInfo* out);
bool lookup_split_fma_bf16(int head_dim, int mode, SplitKernelInfo* out);

bool lookup_split_kernel(int kv_dtype, int head_dim, int mode, int backend, SplitKernelInfo* out) {
  if (backend == BACKEND_MMA) return lookup_split_mma(kv_dtype, head_dim, mode, out);
  if (kv_dtype == 0) return lookup_split_fma_f32(head_dim, mode, out);
  if (kv_dtype == 1) return lookup_split_fma_f16(head_dim, mode, out);
  if (kv_dtype == 2) return lookup_split_fma_bf16(head_dim, mode, out);
  return false;
}

namespace {

thread_local std::string t_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PAGER_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define PAGER_CUDA(call, what)                  \
  do {                                          \
    cudaError_t e_ = (call);                    \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

constexpr unsigned long long kWaitLimitNs = 4000000000ull;  // 4 s per bounded device wait
constexpr int kMaxSplits = 1024;

void preload_kernels();  // below: loads every kernel of the library on the current device

struct DevInfo {
  bool init = false;
  int sms = 0;
  int* status = nullptr;
};
std::mutex g_mu;
DevInfo g_dev[128];
std::unordered_map<const void*, int> g_occupancy;  // per kernel (one smem config each)

int device_info(DevInfo** out) {
  int dev = 0;
  PAGER_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 128) return fail(PAGER_ERR_CUDA, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DevInfo& d = g_dev[dev];
  if (!d.init) {
    PAGER_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev), "sm count");
    void* p = nullptr;
    PAGER_CUDA(cudaGetSymbolAddress(&p, g_status), "status symbol");
    d.status = static_cast<int*>(p);
    preload_kernels();
    d.init = true;
  }
  *out = &d;
  return PAGER_OK;
}

// Resident CTAs per SM for a split kernel (sets its dynamic smem limit once per device).
int ctas_per_sm(const SplitKernelInfo& k, int* out) {
  int dev = 0;
  PAGER_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  const void* key = reinterpret_cast<const char*>(k.fn) + dev;  // per (kernel, device)
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end()) {
      *out = it->second;
      return PAGER_OK;
    }
  }
  PAGER_CUDA(cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem_bytes),
             "cudaFuncSetAttribute(max dynamic smem)");
  int n = 0;
  PAGER_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k.fn, k.threads, k.smem_bytes), "occupancy");
  if (n < 1) n = 1;
  std::lock_guard<std::mutex> lk(g_mu);
  g_occupancy[key] = n;
  *out = n;
  return PAGER_OK;
}

struct Plan {
  int tiles_per_split;
  int max_splits;
};

// Split each (row, kv head) unit's tiles into CTAs: the fewest waves of resident CTAs, then as
// many splits as that wave holds, but no split shorter than kMinSplitTiles tiles (a CTA's fixed
// cost -- prologue, pipeline fill, merge -- is worth several microseconds, and every extra wave
// adds one ramp and one drain).  Measured on B200 (paged op, HBM-resident KV, bf16 D=128 unless
// noted, split + combine/mass µs per launch at 1, 4, 9, 37 splits):
//   8 rows x 8 kv heads, 32k: 561 / 178 / 179 / 223 (this rule: 4 -> 256 CTAs, one wave)
//   1 row x 8 kv heads, 32k: 556 / 151 / 77 / 39 (37 -> 296 CTAs)
//   32 rows x 8 kv heads, 8k: 183 / 212 / 224 / 385 (1)
//   1 row x 2 kv heads, fp16 D=64, 8k: 75 / 27 / 18 / 16; 18 splits 15.8, 148 splits 29 (16)
// The block-table cache bounds the tiles per split from above.
constexpr int kMinSplitTiles = 8;

Plan plan_splits(long long units, int tiles_per_unit, int sms, int per_sm, int max_tps) {
  Plan best{1, 1};
  if (tiles_per_unit <= 0 || units <= 0) return best;
  const long long capacity = (long long)sms * per_sm;
  long long ns = capacity / units;  // most splits that keep every unit's CTAs in one wave
  if (ns < 1) ns = 1;
  const int by_length = tiles_per_unit / kMinSplitTiles;
  if (ns > by_length) ns = by_length > 1 ? by_length : 1;
  const long long by_table = (tiles_per_unit + (long long)max_tps - 1) / max_tps;  // table-cache bound
  if (ns < by_table) ns = by_table;
  if (ns > tiles_per_unit) ns = tiles_per_unit;
  if (ns > kMaxSplits) ns = kMaxSplits;  // the merge holds at most kMaxSplits partials per row
  best.tiles_per_split = (int)((tiles_per_unit + ns - 1) / ns);
  best.max_splits = (tiles_per_unit + best.tiles_per_split - 1) / best.tiles_per_split;
  return best;
}

int dtype_size(int dt) { return dt == PAGER_DTYPE_F32 ? 4 : 2; }
bool dtype_ok(int dt) { return dt == PAGER_DTYPE_F32 || dt == PAGER_DTYPE_F16 || dt == PAGER_DTYPE_BF16; }
bool head_dim_ok(int d) { return d == 8 || d == 16 || d == 32 || d == 64 || d == 128 || d == 256; }
int ilog2(int x) {
  int r = 0;
  while ((1 << r) < x) ++r;
  return r;
}
bool is_pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encoder(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) return fail(PAGER_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable (%s)", cudaGetErrorString(err));
  *out = fn;
  return PAGER_OK;
}

// 3D view [d2][d1][d0] of 16-bit / 32-bit rows, box = one panel x `box_rows` rows x 1.
int encode_3d(CUtensorMap* map, int kv_dtype, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
              uint32_t box0, uint32_t box_rows, int panel_bytes) {
  EncodeTiledFn enc;
  int rc = get_encoder(&enc);
  if (rc) return rc;
  const uint64_t row_bytes = d0 * dtype_size(kv_dtype);
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {row_bytes, row_bytes * d1};
  cuuint32_t box[3] = {box0, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMapDataType dt = kv_dtype == PAGER_DTYPE_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : kv_dtype == PAGER_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMapSwizzle sw = panel_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : panel_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : panel_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PAGER_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for dims %llu x %llu x %llu", (int)r,
                (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2);
  return PAGER_OK;
}

// ------------------------------------------------------------------ small kernels
struct CombineParams {
  int num_q_heads, head_dim;
  int tile_shift, tiles_per_split, max_splits;
  GeomArgs geom;
  const int* active;
  const float* part_m;
  const float* part_l;
  const float* part_acc;
  int op;  // 0 merge into (m,l,acc); 1 merge into (m,l); 2 acc += sum; 3 paged final -> out
  float* m;
  float* l;
  float* acc;
  void* out;
  int out_dtype;
};

enum { OP_STEP = 0, OP_STATS = 1, OP_FIXED = 2, OP_PAGED = 3 };

// Weight of a split whose running max is ms once the row's final max is M (the reference's
// guard, streaming_attention.py:171-172: a split that saw nothing valid contributes nothing).
__device__ __forceinline__ float split_weight(float ms, float M) {
  return ms == neg_inf() ? 0.f : (ms == M ? 1.f : exp2f((ms - M) * kLog2e));
}

// Final softmax statistics of one query row from its splits' partial (m, l), in split order:
// M = max(m_floor, max_s m_s), L = sum_s l_s * 2^((m_s - M) log2 e), each step rounded on its own
// (explicit fma), so the combine and the mass pass, which both need them, get identical values.
template <typename Ptr>
__device__ __forceinline__ void row_final_stats(Ptr ms, Ptr ls, int nsplit, float m_floor, float& M, float& L) {
  float mx = m_floor;
#pragma unroll 8
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, ms[s]);
  float acc = 0.f;
#pragma unroll 8
  for (int s = 0; s < nsplit; ++s) acc = __fmaf_rn(split_weight(ms[s], mx), ls[s], acc);
  M = mx;
  L = acc;
}

// One query row: merge the splits' (m, l, acc), into the incoming state (drop-in ops) or from
// scratch into the output (paged op).
__device__ __forceinline__ void combine_row(const CombineParams& c, int row) {
  __shared__ float w_s[kMaxSplits];
  __shared__ float l_s[kMaxSplits];
  __shared__ float sh_L;
  __shared__ float sh_M;
  __shared__ float sh_win;
  const int b = row / c.num_q_heads;
  if (c.active && c.active[b] == 0) return;
  int t_begin, t_end, nsplit;
  geom_tiles(row_geom(c.geom, b), c.tile_shift, c.tiles_per_split, t_begin, t_end, nsplit);
  const int D = c.head_dim;
  const long long pbase = (long long)row * c.max_splits;
  if (c.op == OP_FIXED) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float a = c.acc[(long long)row * D + d];
#pragma unroll 8
      for (int s = 0; s < nsplit; ++s) a += c.part_acc[(pbase + s) * D + d];
      c.acc[(long long)row * D + d] = a;
    }
    return;
  }
  // the splits' statistics are loaded by all threads at once, then reduced by one in split order
  for (int s = threadIdx.x; s < nsplit; s += blockDim.x) {
    w_s[s] = c.part_m[pbase + s];
    l_s[s] = c.part_l[pbase + s];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const float m_in = c.op == OP_PAGED ? neg_inf() : c.m[row];
    float Mt, L;
    row_final_stats(static_cast<const float*>(w_s), static_cast<const float*>(l_s), nsplit, m_in, Mt, L);
    for (int s = 0; s < nsplit; ++s) w_s[s] = split_weight(w_s[s], Mt);
    // reference guard (streaming_attention.py:171-172): nothing valid yet -> alpha = 0
    float w_in = 0.f;
    if (c.op != OP_PAGED && Mt != neg_inf()) w_in = (m_in == Mt) ? 1.f : exp2f((m_in - Mt) * kLog2e);
    if (c.op != OP_PAGED) L = __fmaf_rn(c.l[row], w_in, L);
    sh_L = L;
    sh_M = Mt;
    sh_win = w_in;
  }
  __syncthreads();
  const float L = sh_L;
  if (c.op == OP_STEP || c.op == OP_PAGED) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float a = c.op == OP_PAGED ? 0.f : c.acc[(long long)row * D + d] * sh_win;
#pragma unroll 8
      for (int s = 0; s < nsplit; ++s) a += w_s[s] * c.part_acc[(pbase + s) * D + d];
      if (c.op == OP_STEP)
        c.acc[(long long)row * D + d] = a;
      else
        store_any(c.out, (long long)row * D + d, c.out_dtype, a / L);
    }
  }
  if (threadIdx.x == 0 && c.op != OP_PAGED) {
    c.m[row] = sh_M;
    c.l[row] = L;
  }
}

__global__ void __launch_bounds__(128) combine_kernel(const CombineParams c) { combine_row(c, blockIdx.x); }

// accumulate_step: block_mass[b, h, off + j] = sum_{groups of local block j} p / l.
__global__ void chunk_mass_kernel(const float2* mass_part, int gstride, int group_tokens, int tpb, int tokens,
                                  const float* l, const int* active, int num_q_heads, float* block_mass,
                                  int max_blocks, int block_id_offset) {
  const int row = blockIdx.y;
  const int b = row / num_q_heads;
  if (active && active[b] == 0) return;
  const int nloc = (tokens + tpb - 1) / tpb;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= nloc) return;
  const int gpb = tpb / group_tokens;
  const int g0 = j * gpb;
  const int g1 = min(g0 + gpb, gstride);
  float s = 0.f;
  for (int gi = g0; gi < g1; ++gi) s += mass_part[(long long)row * gstride + gi].x;
  const int col = block_id_offset + j;
  if (col < max_blocks) block_mass[(long long)row * max_blocks + col] = s / l[row];
}

struct PagedMassParams {
  const float2* mass_part;
  int gstride, group_shift, tile_shift, tpb, tiles_per_split;
  GeomArgs geom;
  const int* active;
  const float* part_m;  // the splits' partial statistics, [rows, max_splits]
  const float* part_l;
  int max_splits;
  int batch, num_q_heads, max_blocks;
  float* block_mass;  // [B, Hq, max_blocks] or null
  float* mass_accum;
  int mass_mode;
};

// The combine/mass kernel of the paged op runs 256-thread CTAs: the first `rows` CTAs merge one
// query row each, the rest compute the per-block mass of 32 blocks of one row (all rows in
// batch-mean mode).  Both halves derive each head's final (M, L) from the splits' statistics the
// same way -- lanes walk the splits with an online (max, sum), shuffles merge the lanes -- so
// neither waits for the other and they agree on M and L bit for bit.
constexpr int kFinishThreads = 256;
constexpr int kFinishWarps = kFinishThreads / 32;
constexpr int kHeadsPerWarp = 4;  // heads a warp handles at once: their loads are issued together
constexpr int kMassHeadChunk = kFinishWarps * kHeadsPerWarp;
constexpr int kPreload = 8;  // partial accumulators a combine thread loads before the statistics are known

// Final (M, L) of one query row from its splits' (m, l), for every lane of the calling warp.
__device__ __forceinline__ void warp_row_stats(const float* pm, const float* pl, int nsplit, float& M, float& L) {
  const int lane = threadIdx.x & 31;
  float mx = neg_inf(), sm = 0.f;
  for (int s = lane; s < nsplit; s += 32) {
    const float mv = pm[s], lv = pl[s];
    const float nm = fmaxf(mx, mv);
    sm = sm * split_weight(mx, nm) + lv * split_weight(mv, nm);
    mx = nm;
  }
  M = warp_max(mx);
  L = warp_sum(sm * split_weight(mx, M));
}

// One query row of the paged op: out = sum_s w_s acc_s / L.  Warp 0 reduces the statistics while the
// other threads already load their columns' partial accumulators; one CTA barrier hands the split
// weights over.
__device__ __forceinline__ void paged_combine_row(const CombineParams& c, int row) {
  __shared__ float w_s[kMaxSplits];
  __shared__ float sh_L;
  const int b = row / c.num_q_heads;
  if (c.active && c.active[b] == 0) return;
  int t_begin, t_end, nsplit;
  geom_tiles(row_geom(c.geom, b), c.tile_shift, c.tiles_per_split, t_begin, t_end, nsplit);
  const int D = c.head_dim;
  const int tid = threadIdx.x;
  const long long pbase = (long long)row * c.max_splits;
  const int d = tid;  // this thread's column (head_dim <= kFinishThreads)
  float pre[kPreload];
  if (tid >= 32 && d < D) {
#pragma unroll
    for (int s = 0; s < kPreload; ++s) pre[s] = s < nsplit ? c.part_acc[(pbase + s) * D + d] : 0.f;
  }
  if (tid < 32) {
    float M, L;
    warp_row_stats(c.part_m + pbase, c.part_l + pbase, nsplit, M, L);
    for (int s = tid; s < nsplit; s += 32) w_s[s] = split_weight(c.part_m[pbase + s], M);
    if (tid == 0) sh_L = L;
  }
  __syncthreads();
  if (d >= D) return;
  if (tid < 32) {
#pragma unroll
    for (int s = 0; s < kPreload; ++s) pre[s] = s < nsplit ? c.part_acc[(pbase + s) * D + d] : 0.f;
  }
  float a = 0.f;
#pragma unroll
  for (int s = 0; s < kPreload; ++s)
    if (s < nsplit) a += w_s[s] * pre[s];
  for (int s = kPreload; s < nsplit; ++s) a += w_s[s] * c.part_acc[(pbase + s) * D + d];
  store_any(c.out, (long long)row * D + d, c.out_dtype, a / sh_L);
}

// Per-block mass of 32 blocks (lane <-> block j) of one batch row, or of every row in batch-mean
// mode.  Each warp owns kHeadsPerWarp heads of a chunk for both phases -- their final (M, L), then
// their mass: sum over the block's groups of sum(p) * 2^((m_group - M) log2 e) / L (zero for a row
// with nothing valid, streaming_attention.py:317 defaults l_final to 1 there) -- so no CTA barrier
// separates the phases; one barrier at the end sums the warps' heads.
__device__ __forceinline__ void paged_mass_cta(const PagedMassParams& p, int bx, int by) {
  __shared__ float red[kFinishWarps][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int j = bx * 32 + lane;
  const bool batch_mean = p.mass_mode == PAGER_MASS_BATCH_MEAN;
  const int b_first = batch_mean ? 0 : by;
  const int b_last = batch_mean ? p.batch : by + 1;
  const int gpb = p.tpb >> p.group_shift;
  float tot = 0.f;
  for (int b = b_first; b < b_last; ++b) {
    if (p.active && p.active[b] == 0) continue;
    const RowGeom g = row_geom(p.geom, b);
    int tb, te, ns;
    geom_tiles(g, p.tile_shift, p.tiles_per_split, tb, te, ns);
    const long long row0 = (long long)b * p.num_q_heads;
    for (int r0 = 0; r0 < p.num_q_heads; r0 += kMassHeadChunk) {
      float M[kHeadsPerWarp], L[kHeadsPerWarp];
      bool live[kHeadsPerWarp];
      {
        float mx[kHeadsPerWarp], sm[kHeadsPerWarp];
#pragma unroll
        for (int k = 0; k < kHeadsPerWarp; ++k) {
          mx[k] = neg_inf();
          sm[k] = 0.f;
          live[k] = r0 + warp + k * kFinishWarps < p.num_q_heads;
        }
        for (int s0 = 0; s0 < ns; s0 += 32) {
          const int s = s0 + lane;
          float mv[kHeadsPerWarp], lv[kHeadsPerWarp];
#pragma unroll
          for (int k = 0; k < kHeadsPerWarp; ++k) {
            const bool ok = live[k] && s < ns;
            const long long pi = (row0 + r0 + warp + k * kFinishWarps) * p.max_splits + s;
            mv[k] = ok ? p.part_m[pi] : neg_inf();
            lv[k] = ok ? p.part_l[pi] : 0.f;
          }
#pragma unroll
          for (int k = 0; k < kHeadsPerWarp; ++k) {
            const float nm = fmaxf(mx[k], mv[k]);
            sm[k] = sm[k] * split_weight(mx[k], nm) + lv[k] * split_weight(mv[k], nm);
            mx[k] = nm;
          }
        }
#pragma unroll
        for (int k = 0; k < kHeadsPerWarp; ++k) {
          M[k] = warp_max(mx[k]);
          L[k] = warp_sum(sm[k] * split_weight(mx[k], M[k]));
        }
      }
      if (j < g.nb && j < p.max_blocks) {
        float acc[kHeadsPerWarp];
#pragma unroll
        for (int k = 0; k < kHeadsPerWarp; ++k) acc[k] = 0.f;
#pragma unroll 2
        for (int gi = j * gpb; gi < (j + 1) * gpb; ++gi) {
          const int tile = (gi << p.group_shift) >> p.tile_shift;
          if (tile < tb || tile >= te) continue;  // never loaded: outside the attended range
          float2 v[kHeadsPerWarp];
#pragma unroll
          for (int k = 0; k < kHeadsPerWarp; ++k)
            v[k] = live[k] ? p.mass_part[(row0 + r0 + warp + k * kFinishWarps) * p.gstride + gi] : make_float2(0.f, 0.f);
#pragma unroll
          for (int k = 0; k < kHeadsPerWarp; ++k)
            if (v[k].x != 0.f) acc[k] += v[k].x * exp2f((v[k].y - M[k]) * kLog2e);
        }
#pragma unroll
        for (int k = 0; k < kHeadsPerWarp; ++k) {
          if (!live[k]) continue;
          const float v = L[k] > 0.f ? acc[k] / L[k] : 0.f;
          if (p.block_mass) p.block_mass[(row0 + r0 + warp + k * kFinishWarps) * p.max_blocks + j] = v;
          tot += v;
        }
      }
    }
  }
  red[warp][lane] = tot;
  __syncthreads();
  if (warp != 0 || j >= p.max_blocks || p.mass_mode == PAGER_MASS_NONE) return;
  float sum = 0.f;
#pragma unroll
  for (int w = 0; w < kFinishWarps; ++w) sum += red[w][lane];
  if (batch_mean) {
    p.mass_accum[j] += sum / (float)(p.batch * p.num_q_heads);
  } else {
    const int b = by;
    if (p.active && p.active[b] == 0) return;
    if (j >= row_geom(p.geom, b).nb) return;
    p.mass_accum[(long long)b * p.max_blocks + j] += sum / (float)p.num_q_heads;
  }
}

// Paged op, after the split kernel: CTAs [0, rows) merge, the next mass_x * mass_y compute mass.
// Launched programmatically serialized behind the split kernel, it waits for the split grid before
// reading its partials and lets the next layer's split kernel be scheduled behind it.
__global__ void __launch_bounds__(kFinishThreads) paged_finish_kernel(const CombineParams c, const PagedMassParams mp,
                                                                     int rows, int mass_x) {
  pdl_wait();
  pdl_launch_dependents();
  const int cta = blockIdx.x;
  if (cta < rows) {
    paged_combine_row(c, cta);
  } else {
    const int m = cta - rows;
    paged_mass_cta(mp, m % mass_x, m / mass_x);
  }
}

__global__ void finalize_kernel(const float* acc, const float* l, void* out, int out_dtype, long long n, int head_dim) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  store_any(out, i, out_dtype, acc[i] / l[i / head_dim]);
}

__global__ void state_init_kernel(float* m, float* l, float* acc, long long rows, int head_dim) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) {
    m[i] = neg_inf();
    l[i] = 0.f;
  }
  if (i < rows * head_dim) acc[i] = 0.f;
}

// Self-test of the bounded waits every kernel uses: one thread waits on an mbarrier that nothing
// ever arrives on; the wait gives up after limit_ns and the device status word reports a timeout.
__device__ unsigned long long g_selftest_waited_ns;

__global__ void bounded_wait_selftest_kernel(unsigned long long limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  mbar_fence_init();
  const unsigned long long t0 = global_timer_ns();
  const bool arrived = mbar_wait_bounded(&bar, 0, limit_ns);
  g_selftest_waited_ns = global_timer_ns() - t0;
  if (!arrived) atomicExch(status, kStatusTimeout);
}

__global__ void zero_copy_probe_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, long long n16) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = ld_global_16(src + i);
    const uint4 b2 = ld_global_16(src + i + stride);
    const uint4 c = ld_global_16(src + i + 2 * stride);
    const uint4 d = ld_global_16(src + i + 3 * stride);
    dst[i] = a;
    dst[i + stride] = b2;
    dst[i + 2 * stride] = c;
    dst[i + 3 * stride] = d;
  }
  for (; i < n16; i += stride) dst[i] = ld_global_16(src + i);
}

// ------------------------------------------------------------------ launches
// Launch with programmatic stream serialization: the kernel may be scheduled while the previous
// kernel in the stream drains (hiding launch latency between the paged op's kernels and across
// layers); every kernel launched this way calls pdl_wait() before it touches global memory.
cudaError_t launch_serialized(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  memset(attr, 0, sizeof(attr));
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

// ------------------------------------------------------------------ scratch layout
struct Scratch {
  float* part_m;
  float* part_l;
  float* part_acc;
  float2* mass_part;
  size_t bytes;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

Scratch layout_scratch(char* base, long long rows, int max_splits, int head_dim, long long mass_groups) {
  Scratch s;
  size_t off = 0;
  auto take = [&](size_t n) {
    char* p = base ? base + off : nullptr;
    off += align256(n);
    return p;
  };
  s.part_m = reinterpret_cast<float*>(take(sizeof(float) * rows * max_splits));
  s.part_l = reinterpret_cast<float*>(take(sizeof(float) * rows * max_splits));
  s.part_acc = reinterpret_cast<float*>(take(sizeof(float) * rows * max_splits * head_dim));
  s.mass_part = reinterpret_cast<float2*>(take(sizeof(float2) * rows * (mass_groups > 0 ? mass_groups : 0)));
  s.bytes = off;
  return s;
}

int backend_for(int requested, int kv_dtype, int head_dim) {
  if (requested == PAGER_BACKEND_MMA || requested == PAGER_BACKEND_FMA) return requested;
  if (kv_dtype != PAGER_DTYPE_F32 && (head_dim == 64 || head_dim == 128 || head_dim == 256)) return PAGER_BACKEND_MMA;
  return PAGER_BACKEND_FMA;
}

// The values pass of reference-exact rounding for a geometry: on the tensor-core kernels with at
// most 4 query heads per KV head (Llama, Mistral), the variant whose 4-row score ring leaves room for
// a sixth stage of V tiles in the same shared memory; with at most 8 (TinyLlama), the 8-row one;
// both with the swapped-operand consumers.  Otherwise the general one.
int values_mode(int n_rep, int be) {
  if (be != BACKEND_MMA) return MODE_VALUES;
  return n_rep <= 4 ? MODE_VALUES_R4 : (n_rep <= 8 ? MODE_VALUES_R8 : MODE_VALUES);
}

int check_geometry(int batch, int hq, int hkv, int head_dim, int kv_dtype, int q_dtype) {
  if (batch < 0 || hq <= 0 || hkv <= 0) return fail(PAGER_ERR_INVALID, "bad shape: batch=%d heads=%d kv_heads=%d", batch, hq, hkv);
  if (hq % hkv) return fail(PAGER_ERR_INVALID, "num_query_heads (%d) is not a multiple of num_kv_heads (%d)", hq, hkv);
  const int n_rep = hq / hkv;
  if (n_rep > kMaxRep)
    return fail(PAGER_ERR_UNSUPPORTED,
                "streaming attention's GQA query-head packing supports n_rep up to %d, got %d. This architecture's "
                "query/KV head ratio is wider than any currently supported model.",
                kMaxRep, n_rep);
  if (!head_dim_ok(head_dim)) return fail(PAGER_ERR_UNSUPPORTED, "head_dim %d not supported (8..256, power of two)", head_dim);
  if (!dtype_ok(kv_dtype) || !dtype_ok(q_dtype)) return fail(PAGER_ERR_INVALID, "unknown dtype code");
  return PAGER_OK;
}

struct ChunkArgs {
  int op;  // 0 step, 1 stats, 2 accumulate, 3 fold_fixed
  const void* q;
  int q_dtype;
  const void* k;
  const void* v;
  int kv_dtype;
  const int32_t* valid;
  const int32_t* active;
  float* m;
  float* l;
  float* acc;
  float* block_mass;
  int max_blocks, block_id_offset, tokens_per_block;
  int batch, hq, hkv, tokens, head_dim;
  float scale, softcap;
  int backend;
  void* scratch;
  size_t scratch_bytes;
  cudaStream_t stream;
};

// streaming_attention_step on fp16/bf16 KV with the tensor-core kernels rounds p exactly as the
// reference's one-pass kernel does (scores pass, scan seeded with the incoming m, values pass);
// defined below, beside the scan kernel.
bool chunk_exact(const ChunkArgs& a);
int run_chunk_exact(const ChunkArgs& a);
size_t chunk_exact_scratch(const ChunkArgs& a);

int chunk_plan(const ChunkArgs& a, SplitKernelInfo* k, Plan* plan, long long* mass_groups, int* group_tokens) {
  const int mode = a.op == 0 ? MODE_ONLINE : (a.op == 1 ? MODE_STATS : MODE_FIXED);
  const int be = backend_for(a.backend, a.kv_dtype, a.head_dim);
  if (!lookup_split_kernel(a.kv_dtype, a.head_dim, mode, be, k))
    return fail(PAGER_ERR_UNSUPPORTED, "no split kernel for dtype %d head_dim %d backend %d", a.kv_dtype, a.head_dim, be);
  DevInfo* di;
  int rc = device_info(&di);
  if (rc) return rc;
  int per_sm = 1;
  rc = ctas_per_sm(*k, &per_sm);
  if (rc) return rc;
  const int tiles = (a.tokens + k->tile - 1) / k->tile;
  *plan = plan_splits((long long)a.batch * a.hkv, tiles, di->sms, per_sm, 1 << 30);
  *group_tokens = 0;
  *mass_groups = 0;
  if (a.op == 2) {
    *group_tokens = a.tokens_per_block < k->tile ? a.tokens_per_block : k->tile;
    *mass_groups = (long long)tiles * k->tile / *group_tokens;
  }
  return PAGER_OK;
}

int run_chunk(const ChunkArgs& a) {
  int rc = check_geometry(a.batch, a.hq, a.hkv, a.head_dim, a.kv_dtype, a.q_dtype);
  if (rc) return rc;
  if (a.tokens < 0) return fail(PAGER_ERR_INVALID, "negative token count");
  if (a.batch == 0 || a.tokens == 0) return PAGER_OK;  // nothing to fold (the reference loop runs zero times)
  if (!a.q || !a.k || (a.op != 1 && !a.v) || !a.m || !a.l || (a.op != 1 && !a.acc))
    return fail(PAGER_ERR_INVALID, "null tensor pointer");
  if (!aligned16(a.k) || (a.op != 1 && !aligned16(a.v)))
    return fail(PAGER_ERR_INVALID, "k/v must be 16-byte aligned");
  if (a.op == 2) {
    if (!a.block_mass) return fail(PAGER_ERR_INVALID, "block_mass is null");
    if (!is_pow2(a.tokens_per_block) || a.tokens_per_block < 8)
      return fail(PAGER_ERR_UNSUPPORTED, "tokens_per_block must be a power of two >= 8, got %d", a.tokens_per_block);
    const int nloc = (a.tokens + a.tokens_per_block - 1) / a.tokens_per_block;
    if (a.block_id_offset < 0 || a.block_id_offset + nloc > a.max_blocks)
      return fail(PAGER_ERR_INVALID, "block_mass has %d blocks; offset %d + %d local blocks overflows it", a.max_blocks,
                  a.block_id_offset, nloc);
  }
  if (chunk_exact(a)) return run_chunk_exact(a);
  SplitKernelInfo k;
  Plan plan;
  long long mass_groups;
  int G;
  rc = chunk_plan(a, &k, &plan, &mass_groups, &G);
  if (rc) return rc;
  const long long rows = (long long)a.batch * a.hq;
  Scratch sc = layout_scratch(static_cast<char*>(a.scratch), rows, plan.max_splits, a.head_dim, mass_groups);
  if (!a.scratch || a.scratch_bytes < sc.bytes)
    return fail(PAGER_ERR_SCRATCH, "scratch too small: need %zu bytes, got %zu", sc.bytes, a.scratch_bytes);
  DevInfo* di;
  rc = device_info(&di);
  if (rc) return rc;

  CUtensorMap mk, mv;
  memset(&mk, 0, sizeof(mk));
  memset(&mv, 0, sizeof(mv));
  const uint64_t z = (uint64_t)a.batch * a.hkv;
  rc = encode_3d(&mk, a.kv_dtype, a.k, a.head_dim, a.tokens, z, k.panel_elts, k.tile, k.panel_bytes);
  if (rc) return rc;
  if (a.op != 1) {
    rc = encode_3d(&mv, a.kv_dtype, a.v, a.head_dim, a.tokens, z, k.panel_elts, k.tile, k.panel_bytes);
    if (rc) return rc;
  }
  SplitParams p;
  memset(&p, 0, sizeof(p));
  p.q = a.q;
  p.q_dtype = a.q_dtype;
  p.batch = a.batch;
  p.num_q_heads = a.hq;
  p.num_kv_heads = a.hkv;
  p.n_rep = a.hq / a.hkv;
  p.scale = a.scale;
  p.softcap = a.softcap > 0.f ? a.softcap : 0.f;
  p.source = SRC_CONTIG;
  p.geom.source = SRC_CONTIG;
  p.geom.tokens = a.tokens;
  p.geom.max_tokens = a.tokens;
  p.valid = a.valid;
  p.valid_stride = a.tokens;
  p.active = (a.op == 3) ? nullptr : a.active;
  p.m_fixed = a.m;
  p.l_fixed = a.l;
  p.tiles_per_split = plan.tiles_per_split;
  p.max_splits = plan.max_splits;
  p.part_m = sc.part_m;
  p.part_l = sc.part_l;
  p.part_acc = sc.part_acc;
  p.mass_part = sc.mass_part;
  p.mass_gstride = (int)mass_groups;
  p.group_tokens = G;
  p.log2_group = G ? ilog2(G) : 0;
  p.wait_limit_ns = kWaitLimitNs;
  p.status = di->status;

  dim3 grid(plan.max_splits, a.hkv, a.batch);
  CUtensorMap unused;
  memset(&unused, 0, sizeof(unused));
  void* args[] = {&p, &mk, &mv, &unused, &unused};
  PAGER_CUDA(cudaLaunchKernel(k.fn, grid, dim3(k.threads), args, k.smem_bytes, a.stream), "split kernel launch");

  CombineParams c;
  memset(&c, 0, sizeof(c));
  c.num_q_heads = a.hq;
  c.head_dim = a.head_dim;
  c.tile_shift = ilog2(k.tile);
  c.tiles_per_split = plan.tiles_per_split;
  c.max_splits = plan.max_splits;
  c.geom = p.geom;
  c.active = p.active;
  c.part_m = sc.part_m;
  c.part_l = sc.part_l;
  c.part_acc = sc.part_acc;
  c.op = a.op == 0 ? OP_STEP : (a.op == 1 ? OP_STATS : OP_FIXED);
  c.m = a.m;
  c.l = a.l;
  c.acc = a.acc;
  combine_kernel<<<(unsigned)rows, 128, 0, a.stream>>>(c);
  PAGER_CUDA(cudaGetLastError(), "combine launch");
  if (a.op == 2) {
    const int nloc = (a.tokens + a.tokens_per_block - 1) / a.tokens_per_block;
    dim3 g2((nloc + 127) / 128, (unsigned)rows);
    chunk_mass_kernel<<<g2, 128, 0, a.stream>>>(sc.mass_part, (int)mass_groups, G, a.tokens_per_block, a.tokens, a.l,
                                                 a.active, a.hq, a.block_mass, a.max_blocks, a.block_id_offset);
    PAGER_CUDA(cudaGetLastError(), "mass launch");
  }
  return PAGER_OK;
}

size_t chunk_scratch(const ChunkArgs& a) {
  if (check_geometry(a.batch, a.hq, a.hkv, a.head_dim, a.kv_dtype, a.q_dtype)) return 0;
  if (a.batch <= 0 || a.tokens <= 0) return 0;
  if (chunk_exact(a)) return chunk_exact_scratch(a);
  SplitKernelInfo k;
  Plan plan;
  long long mass_groups;
  int G;
  if (chunk_plan(a, &k, &plan, &mass_groups, &G)) return 0;
  return layout_scratch(nullptr, (long long)a.batch * a.hq, plan.max_splits, a.head_dim, mass_groups).bytes;
}

struct PagedPlan {
  SplitKernelInfo k;
  Plan plan;
  int G;
  long long gstride;
};

int paged_plan(int batch, int hq, int hkv, int head_dim, int kv_dtype, int tpb, int max_row_tokens, int backend,
               PagedPlan* out, int mode = MODE_ONLINE) {
  const int be = backend_for(backend, kv_dtype, head_dim);
  if (mode == MODE_VALUES) mode = values_mode(hq / hkv, be);
  if (!lookup_split_kernel(kv_dtype, head_dim, mode, be, &out->k))
    return fail(PAGER_ERR_UNSUPPORTED, "no split kernel for dtype %d head_dim %d backend %d", kv_dtype, head_dim, be);
  DevInfo* di;
  int rc = device_info(&di);
  if (rc) return rc;
  int per_sm = 1;
  rc = ctas_per_sm(out->k, &per_sm);
  if (rc) return rc;
  const int tiles = (max_row_tokens + out->k.tile - 1) / out->k.tile;
  const int max_tps = (int)((long long)(kTableCache - 2) * tpb / out->k.tile);
  out->plan = plan_splits((long long)batch * hkv, tiles, di->sms, per_sm, max_tps > 0 ? max_tps : 1);
  out->G = tpb < out->k.tile ? tpb : out->k.tile;
  out->gstride = (long long)tiles * out->k.tile / out->G;
  return PAGER_OK;
}

}  // namespace

void set_last_error(const char* msg) { t_err = msg; }

// Scratch bytes the paged op needs with the compute backend a call passes (0 when the
// arguments are rejected); pager_paged_decode_scratch_bytes sizes for the larger of two plans.
size_t paged_scratch_bytes_for_backend(int batch, int num_q_heads, int num_kv_heads, int head_dim, int kv_dtype,
                                       int tokens_per_block, int max_row_tokens, int backend) {
  if (check_geometry(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype, kv_dtype)) return 0;
  if (batch <= 0 || max_row_tokens <= 0 || !is_pow2(tokens_per_block) || tokens_per_block < 8) return 0;
  PagedPlan pp;
  if (paged_plan(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype, tokens_per_block, max_row_tokens, backend, &pp))
    return 0;
  return layout_scratch(nullptr, (long long)batch * num_q_heads, pp.plan.max_splits, head_dim, pp.gstride).bytes;
}

// Device status word of the current device, for kernels compiled in other files.
int current_status_word(int** out) {
  DevInfo* d = nullptr;
  const int rc = device_info(&d);
  if (rc) return rc;
  *out = d->status;
  return PAGER_OK;
}

}  // namespace pager

using namespace pager;

extern "C" {

const char* pager_last_error(void) { return t_err.c_str(); }

int pager_version(void) { return 1; }

int pager_device_status(int device, int* status_out) {
  if (!status_out) return fail(PAGER_ERR_INVALID, "status_out is null");
  int prev = 0;
  PAGER_CUDA(cudaGetDevice(&prev), "cudaGetDevice");
  PAGER_CUDA(cudaSetDevice(device), "cudaSetDevice");
  int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  *status_out = v;
  return PAGER_OK;
}

int pager_status_snapshot_async(int32_t* host_dst, void* stream) {
  if (!host_dst) return fail(PAGER_ERR_INVALID, "host_dst is null");
  DevInfo* di;
  const int rc = device_info(&di);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  PAGER_CUDA(cudaMemcpyAsync(host_dst, di->status, sizeof(int), cudaMemcpyDeviceToHost, st), "status snapshot");
  PAGER_CUDA(cudaMemsetAsync(di->status, 0, sizeof(int), st), "status reset");
  return PAGER_OK;
}

int pager_attn_state_init(float* m, float* l, float* acc, int64_t rows, int head_dim, void* stream) {
  if (rows < 0 || head_dim <= 0) return fail(PAGER_ERR_INVALID, "bad shape");
  if (rows == 0) return PAGER_OK;
  const long long n = rows * head_dim;
  state_init_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(m, l, acc, rows, head_dim);
  PAGER_CUDA(cudaGetLastError(), "state_init launch");
  return PAGER_OK;
}

int pager_attn_finalize(const float* acc, const float* l, void* out, int out_dtype, int64_t rows, int head_dim,
                        void* stream) {
  if (rows < 0 || head_dim <= 0 || !dtype_ok(out_dtype)) return fail(PAGER_ERR_INVALID, "bad finalize arguments");
  if (rows == 0) return PAGER_OK;
  const long long n = rows * head_dim;
  finalize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(acc, l, out, out_dtype, n, head_dim);
  PAGER_CUDA(cudaGetLastError(), "finalize launch");
  return PAGER_OK;
}

size_t pager_attn_chunk_scratch_bytes(int op, int batch, int num_q_heads, int num_kv_heads, int tokens, int head_dim,
                                      int kv_dtype, int tokens_per_block) {
  ChunkArgs a;
  memset(&a, 0, sizeof(a));
  a.op = op;
  a.q_dtype = kv_dtype;
  a.kv_dtype = kv_dtype;
  a.batch = batch;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.tokens = tokens;
  a.head_dim = head_dim;
  a.tokens_per_block = tokens_per_block > 0 ? tokens_per_block : 16;
  a.backend = PAGER_BACKEND_AUTO;
  return chunk_scratch(a);
}

#define CHUNK_COMMON                                                                                     \
  a.q = q;                                                                                               \
  a.q_dtype = q_dtype;                                                                                   \
  a.kv_dtype = kv_dtype;                                                                                 \
  a.batch = batch;                                                                                       \
  a.hq = num_q_heads;                                                                                    \
  a.hkv = num_kv_heads;                                                                                  \
  a.tokens = tokens;                                                                                     \
  a.head_dim = head_dim;                                                                                 \
  a.scale = scale;                                                                                       \
  a.softcap = softcap;                                                                                   \
  a.backend = backend;                                                                                   \
  a.scratch = scratch;                                                                                   \
  a.scratch_bytes = scratch_bytes;                                                                       \
  a.stream = (cudaStream_t)stream;

int pager_attn_step(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype, const int32_t* valid,
                    const int32_t* active, float* m, float* l, float* acc, int batch, int num_q_heads,
                    int num_kv_heads, int tokens, int head_dim, float scale, float softcap, int backend,
                    void* scratch, size_t scratch_bytes, void* stream) {
  ChunkArgs a;
  memset(&a, 0, sizeof(a));
  CHUNK_COMMON
  a.op = 0;
  a.k = k;
  a.v = v;
  a.valid = valid;
  a.active = active;
  a.m = m;
  a.l = l;
  a.acc = acc;
  return run_chunk(a);
}

int pager_attn_stats_step(const void* q, int q_dtype, const void* k, int kv_dtype, const int32_t* valid,
                          const int32_t* active, float* m, float* l, int batch, int num_q_heads, int num_kv_heads,
                          int tokens, int head_dim, float scale, float softcap, int backend, void* scratch,
                          size_t scratch_bytes, void* stream) {
  ChunkArgs a;
  memset(&a, 0, sizeof(a));
  CHUNK_COMMON
  a.op = 1;
  a.k = k;
  a.valid = valid;
  a.active = active;
  a.m = m;
  a.l = l;
  return run_chunk(a);
}

int pager_attn_accumulate_step(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype,
                               const int32_t* valid, const int32_t* active, const float* m, const float* l,
                               float* acc, float* block_mass, int max_blocks, int block_id_offset,
                               int tokens_per_block, int batch, int num_q_heads, int num_kv_heads, int tokens,
                               int head_dim, float scale, float softcap, int backend, void* scratch,
                               size_t scratch_bytes, void* stream) {
  ChunkArgs a;
  memset(&a, 0, sizeof(a));
  CHUNK_COMMON
  a.op = 2;
  a.k = k;
  a.v = v;
  a.valid = valid;
  a.active = active;
  a.m = const_cast<float*>(m);
  a.l = const_cast<float*>(l);
  a.acc = acc;
  a.block_mass = block_mass;
  a.max_blocks = max_blocks;
  a.block_id_offset = block_id_offset;
  a.tokens_per_block = tokens_per_block;
  return run_chunk(a);
}

int pager_attn_fold_fixed_step(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype,
                               const int32_t* valid, const float* m, const float* l, float* acc, int batch,
                               int num_q_heads, int num_kv_heads, int tokens, int head_dim, float scale,
                               float softcap, int backend, void* scratch, size_t scratch_bytes, void* stream) {
  ChunkArgs a;
  memset(&a, 0, sizeof(a));
  CHUNK_COMMON
  a.op = 3;
  a.k = k;
  a.v = v;
  a.valid = valid;
  a.m = const_cast<float*>(m);
  a.l = const_cast<float*>(l);
  a.acc = acc;
  return run_chunk(a);
}

size_t pager_paged_decode_scratch_bytes(int batch, int num_q_heads, int num_kv_heads, int head_dim, int kv_dtype,
                                        int tokens_per_block, int max_blocks, int max_row_tokens) {
  (void)max_blocks;
  if (check_geometry(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype, kv_dtype)) return 0;
  if (batch <= 0 || max_row_tokens <= 0 || !is_pow2(tokens_per_block) || tokens_per_block < 8) return 0;
  PagedPlan pp;
  if (paged_plan(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype, tokens_per_block, max_row_tokens,
                 PAGER_BACKEND_AUTO, &pp))
    return 0;
  PagedPlan pf;  // the FMA backend may plan differently; size for the larger of the two
  size_t extra = 0;
  if (!paged_plan(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype, tokens_per_block, max_row_tokens,
                  PAGER_BACKEND_FMA, &pf))
    extra = layout_scratch(nullptr, (long long)batch * num_q_heads, pf.plan.max_splits, head_dim, pf.gstride).bytes;
  const size_t base =
      layout_scratch(nullptr, (long long)batch * num_q_heads, pp.plan.max_splits, head_dim, pp.gstride).bytes;
  return base > extra ? base : extra;
}

int pager_paged_decode_attention(const void* q, int q_dtype, const void* dev_pool, int dev_slots,
                                 const void* host_pool, int host_slots, int kv_dtype, int num_layers, int layer,
                                 int num_kv_heads, int tokens_per_block, int head_dim, const int32_t* block_table,
                                 int max_blocks, const int32_t* num_blocks, const void* tail_k, const void* tail_v,
                                 const int32_t* tail_len, int tail_cap, const int32_t* valid_lo,
                                 const int32_t* valid_hi, const int32_t* active, int batch, int num_q_heads,
                                 float scale, float softcap, int max_row_tokens, void* out, int out_dtype,
                                 float* block_mass, float* mass_accum, int mass_mode, int backend, void* scratch,
                                 size_t scratch_bytes, void* stream) {
  return pager_paged_decode_attention_staged(q, q_dtype, dev_pool, dev_slots, host_pool, host_slots, nullptr, 0,
                                             kv_dtype, num_layers, layer, num_kv_heads, tokens_per_block, head_dim,
                                             block_table, max_blocks, num_blocks, tail_k, tail_v, tail_len, tail_cap,
                                             valid_lo, valid_hi, active, batch, num_q_heads, scale, softcap,
                                             max_row_tokens, out, out_dtype, block_mass, mass_accum, mass_mode,
                                             backend, scratch, scratch_bytes, stream);
}

}  // extern "C"

namespace pager {
namespace {

// Every argument of the paged entry points (see include/pager_b200.h).
struct PagedArgs {
  const void* q;
  int q_dtype;
  const void* dev_pool;
  int dev_slots;
  const void* host_pool;
  int host_slots;
  const void* stage_pool;
  int stage_slots;
  int kv_dtype, num_layers, layer, num_kv_heads, tokens_per_block, head_dim;
  const int32_t* block_table;
  int max_blocks;
  const int32_t* num_blocks;
  const void* tail_k;
  const void* tail_v;
  const int32_t* tail_len;
  int tail_cap;
  const int32_t* valid_lo;
  const int32_t* valid_hi;
  const int32_t* active;
  int batch, num_q_heads;
  float scale, softcap;
  int max_row_tokens;
  void* out;
  int out_dtype;
  float* block_mass;
  float* mass_accum;
  int mass_mode, backend;
  int rounding, ref_group_tokens;
  const int32_t* ref_shift;
  const int32_t* ref_tail_start;
  void* scratch;
  size_t scratch_bytes;
  void* stream;
};

// The reference's tile of row-local token j: its one-pass kernel walks each chunk it is given in
// 64-token tiles from the chunk's start (streaming_attention.py:143), the chunks being groups of
// `gs_tok` tokens of the combined block numbering (paged_model.py:993-1072; in batched_decode.py
// :238-285 a row's blocks sit `shift` tokens into that numbering) and then the tail from
// `tail_start`.  Keys are unique per tile and increase along the row.
__device__ __forceinline__ int ref_tile_key(int j, int shift, int tail_start, int gs_tok) {
  if (j >= tail_start) return 0x40000000 + ((j - tail_start) >> 6);
  const int c = shift + j;
  if (gs_tok <= 0) return c >> 6;
  const int grp = c / gs_tok;
  return grp * ((gs_tok + 63) >> 6) + ((c - grp * gs_tok) >> 6);
}

struct RefMaxParams {
  GeomArgs geom;
  const int* active;
  const float* m_in;  // incoming running max per query row (drop-in step), or null: -inf
  int rows, num_q_heads, tile_shift, tiles_per_split, group_shift, gstride, mstride, tpb;
  int rule;  // PAGER_ROUND_RUNNING or PAGER_ROUND_FINAL
  int ref_group_tokens;
  const int* ref_shift;
  const int* ref_tail_start;
  float* gmax;  // in: the SCORES pass's group maxima; out: their inclusive prefix max
  float* mref;  // out: [rows, mstride], kRefSlots entries per tile
};

constexpr int kRefMaxThreads = 256;
constexpr int kRefMaxPer = 4;  // consecutive groups per thread in each chunk of the prefix scan

// Between the SCORES and VALUES passes: per query row (one CTA), the max each group's p is formed
// against -- the reference's running max once its tile is folded in (the inclusive prefix max of
// the group maxima up to the tile's last group), or the row's final max.  The prefix max runs as a
// block-wide scan over chunks of kRefMaxThreads * kRefMaxPer groups, written back over the group
// maxima; each group then reads the prefix at its reference tile's last group.
__global__ void __launch_bounds__(kRefMaxThreads) ref_max_kernel(const RefMaxParams p) {
  __shared__ float warp_tot[kRefMaxThreads / 32];
  __shared__ float chunk_tot;
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int b = row / p.num_q_heads;
  if (p.active && p.active[b] == 0) return;  // uniform across the CTA
  const RowGeom g = row_geom(p.geom, b);
  int tb, te, ns;
  geom_tiles(g, p.tile_shift, p.tiles_per_split, tb, te, ns);
  if (ns == 0) return;
  const int g0 = (tb << p.tile_shift) >> p.group_shift;
  const int g1 = (te << p.tile_shift) >> p.group_shift;
  float* gm = p.gmax + (long long)row * p.gstride;
  float* mr = p.mref + (long long)row * p.mstride;
  float carry = p.m_in ? p.m_in[row] : neg_inf();
  for (int c0 = g0; c0 < g1; c0 += kRefMaxThreads * kRefMaxPer) {
    float v[kRefMaxPer];
    float run = neg_inf();
#pragma unroll
    for (int i = 0; i < kRefMaxPer; ++i) {
      const int gi = c0 + tid * kRefMaxPer + i;
      v[i] = gi < g1 ? gm[gi] : neg_inf();
      run = fmaxf(run, v[i]);
      v[i] = run;  // inclusive prefix within this thread's groups
    }
    float incl = run;  // inclusive scan of the threads' maxima across the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl = fmaxf(incl, t);
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    float before = carry;  // everything before this thread's groups
    for (int w = 0; w < warp; ++w) before = fmaxf(before, warp_tot[w]);
    const float excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane > 0) before = fmaxf(before, excl);
#pragma unroll
    for (int i = 0; i < kRefMaxPer; ++i) {
      const int gi = c0 + tid * kRefMaxPer + i;
      if (gi < g1) gm[gi] = fmaxf(before, v[i]);
    }
    if (tid == kRefMaxThreads - 1) chunk_tot = fmaxf(before, run);
    __syncthreads();
    carry = chunk_tot;
    __syncthreads();
  }
  // carry: the row's final max; the prefix values written above are visible to the whole CTA
  const int shift = p.ref_shift ? p.ref_shift[b] : 0;
  const int tail_start = p.ref_tail_start ? p.ref_tail_start[b] : g.nb * p.tpb;
  const int G = 1 << p.group_shift;
  const int per_tile = 1 << (p.tile_shift - p.group_shift);
  for (int gi = g0 + tid; gi < g1; gi += kRefMaxThreads) {
    float M = carry;
    if (p.rule == PAGER_ROUND_RUNNING) {
      const int key = ref_tile_key(gi * G, shift, tail_start, p.ref_group_tokens);
      int e = gi;  // the last group of the same reference tile (a tile spans at most 64 / G groups)
      while (e + 1 < g1 && ref_tile_key((e + 1) * G, shift, tail_start, p.ref_group_tokens) == key) ++e;
      M = gm[e];
    }
    const int tile = gi / per_tile;
    mr[(long long)tile * kRefSlots + (gi - tile * per_tile)] = M;
  }
}

// Loads every kernel of the library on the current device, at the library's first call there.
// With lazy module loading (the CUDA 12 default) a kernel is otherwise loaded at its first launch;
// a load while another thread captures a CUDA graph on the device fails and invalidates that
// capture, which a serving process with one scheduler thread per session can run into.
void preload_kernels() {
  cudaFuncAttributes fa;
  const int dims[] = {8, 16, 32, 64, 128, 256};
  for (int dt = 0; dt < 3; ++dt)
    for (int d : dims)
      for (int mode = 0; mode <= MODE_VALUES_R8; ++mode)
        for (int be : {BACKEND_MMA, BACKEND_FMA}) {
          SplitKernelInfo k;
          if (lookup_split_kernel(dt, d, mode, be, &k)) cudaFuncGetAttributes(&fa, k.fn);
        }
  const void* fns[] = {reinterpret_cast<const void*>(&combine_kernel), reinterpret_cast<const void*>(&chunk_mass_kernel),
                       reinterpret_cast<const void*>(&paged_finish_kernel), reinterpret_cast<const void*>(&finalize_kernel),
                       reinterpret_cast<const void*>(&state_init_kernel), reinterpret_cast<const void*>(&ref_max_kernel),
                       reinterpret_cast<const void*>(&zero_copy_probe_kernel),
                       reinterpret_cast<const void*>(&bounded_wait_selftest_kernel), append_kernel_fn(0),
                       append_kernel_fn(1), append_kernel_fn(2)};
  for (const void* f : fns) cudaFuncGetAttributes(&fa, f);
  (void)cudaGetLastError();  // a kernel this build lacks is reported at its launch, not here
}

// 2D fp32 view [d1][d0], box b0 x b1, no swizzle (score and reference-max tiles).
int encode_2d_f32(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint32_t b0, uint32_t b1) {
  EncodeTiledFn enc;
  int rc = get_encoder(&enc);
  if (rc) return rc;
  cuuint64_t dims[2] = {d0, d1};
  cuuint64_t strides[1] = {d0 * 4};
  cuuint32_t box[2] = {b0, b1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PAGER_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for a %llu x %llu fp32 view", (int)r,
                (unsigned long long)d0, (unsigned long long)d1);
  return PAGER_OK;
}

// ---- the drop-in streaming_attention_step with the reference's rounding
// The reference's one-pass kernel folds a chunk in 64-token tiles from the chunk's start, its
// running max starting at the incoming m (streaming_attention.py:143-181).  Here the scores pass
// writes each tile's scores and max (one group per tile: tiles are at most 64 tokens and aligned
// to the reference's), the scan turns them into the reference's running max seeded with m, and
// the values pass folds V; the splits then merge into the incoming (m, l, acc) as before.
struct ChunkExactLayout {
  SplitKernelInfo ks, kv;
  Plan ps, pv;
  long long tiles;
  Scratch sc;
  float* scores;
  float* gmax;
  float* mref;
  size_t bytes;
};

bool chunk_exact(const ChunkArgs& a) { return a.op == 0 && a.kv_dtype != PAGER_DTYPE_F32; }

int chunk_exact_layout(const ChunkArgs& a, char* base, ChunkExactLayout* L) {
  const int be = backend_for(a.backend, a.kv_dtype, a.head_dim);
  if (!lookup_split_kernel(a.kv_dtype, a.head_dim, MODE_SCORES, be, &L->ks) ||
      !lookup_split_kernel(a.kv_dtype, a.head_dim, values_mode(a.hq / a.hkv, be), be, &L->kv))
    return fail(PAGER_ERR_UNSUPPORTED, "no exact-rounding kernels for dtype %d head_dim %d", a.kv_dtype, a.head_dim);
  if (L->ks.tile != L->kv.tile) return fail(PAGER_ERR_CUDA, "scores and values passes disagree on the tile");
  DevInfo* di;
  int rc = device_info(&di);
  if (rc) return rc;
  int per_s = 1, per_v = 1;
  rc = ctas_per_sm(L->ks, &per_s);
  if (rc) return rc;
  rc = ctas_per_sm(L->kv, &per_v);
  if (rc) return rc;
  L->tiles = (a.tokens + L->kv.tile - 1) / L->kv.tile;
  L->ps = plan_splits((long long)a.batch * a.hkv, (int)L->tiles, di->sms, per_s, 1 << 30);
  L->pv = plan_splits((long long)a.batch * a.hkv, (int)L->tiles, di->sms, per_v, 1 << 30);
  const long long rows = (long long)a.batch * a.hq;
  L->sc = layout_scratch(base, rows, L->pv.max_splits, a.head_dim, L->tiles);
  size_t off = L->sc.bytes;
  auto take = [&](size_t n) {
    char* p = base ? base + off : nullptr;
    off += align256(n);
    return reinterpret_cast<float*>(p);
  };
  L->scores = take(sizeof(float) * rows * L->tiles * L->kv.tile);
  L->gmax = take(sizeof(float) * rows * L->tiles);
  L->mref = take(sizeof(float) * rows * L->tiles * kRefSlots);
  L->bytes = off;
  return PAGER_OK;
}

size_t chunk_exact_scratch(const ChunkArgs& a) {
  ChunkExactLayout L;
  return chunk_exact_layout(a, nullptr, &L) ? 0 : L.bytes;
}

int run_chunk_exact(const ChunkArgs& a) {
  ChunkExactLayout lay;
  int rc = chunk_exact_layout(a, static_cast<char*>(a.scratch), &lay);
  if (rc) return rc;
  if (!a.scratch || a.scratch_bytes < lay.bytes)
    return fail(PAGER_ERR_SCRATCH, "scratch too small: need %zu bytes, got %zu", lay.bytes, a.scratch_bytes);
  DevInfo* di;
  rc = device_info(&di);
  if (rc) return rc;
  const long long rows = (long long)a.batch * a.hq;
  const int n_rep = a.hq / a.hkv;
  const int tile = lay.kv.tile;
  CUtensorMap mk, mv, mS, mM;
  const uint64_t z = (uint64_t)a.batch * a.hkv;
  rc = encode_3d(&mk, a.kv_dtype, a.k, a.head_dim, a.tokens, z, lay.ks.panel_elts, tile, lay.ks.panel_bytes);
  if (rc) return rc;
  rc = encode_3d(&mv, a.kv_dtype, a.v, a.head_dim, a.tokens, z, lay.kv.panel_elts, tile, lay.kv.panel_bytes);
  if (rc) return rc;
  rc = encode_2d_f32(&mS, lay.scores, (uint64_t)(lay.tiles * tile), (uint64_t)rows, (uint32_t)tile, (uint32_t)n_rep);
  if (rc) return rc;
  rc = encode_2d_f32(&mM, lay.mref, (uint64_t)(lay.tiles * kRefSlots), (uint64_t)rows, (uint32_t)kRefSlots,
                     (uint32_t)n_rep);
  if (rc) return rc;
  SplitParams p;
  memset(&p, 0, sizeof(p));
  p.q = a.q;
  p.q_dtype = a.q_dtype;
  p.batch = a.batch;
  p.num_q_heads = a.hq;
  p.num_kv_heads = a.hkv;
  p.n_rep = n_rep;
  p.scale = a.scale;
  p.softcap = a.softcap > 0.f ? a.softcap : 0.f;
  p.source = SRC_CONTIG;
  p.geom.source = SRC_CONTIG;
  p.geom.tokens = a.tokens;
  p.geom.max_tokens = a.tokens;
  p.valid = a.valid;
  p.valid_stride = a.tokens;
  p.active = a.active;
  p.part_m = lay.sc.part_m;
  p.part_l = lay.sc.part_l;
  p.part_acc = lay.sc.part_acc;
  p.mass_part = lay.sc.mass_part;
  p.mass_gstride = (int)lay.tiles;
  p.group_tokens = tile;
  p.log2_group = ilog2(tile);
  p.scores = lay.scores;
  p.s_stride = lay.tiles * tile;
  p.gmax = lay.gmax;
  p.wait_limit_ns = kWaitLimitNs;
  p.status = di->status;
  SplitParams ps = p;
  ps.tiles_per_split = lay.ps.tiles_per_split;
  ps.max_splits = lay.ps.max_splits;
  void* sargs[] = {&ps, &mk, &mv, &mS, &mM};
  PAGER_CUDA(cudaLaunchKernel(lay.ks.fn, dim3(lay.ps.max_splits, a.hkv, a.batch), dim3(lay.ks.threads), sargs,
                              lay.ks.smem_bytes, a.stream),
             "scores kernel launch");
  RefMaxParams rp;
  memset(&rp, 0, sizeof(rp));
  rp.geom = p.geom;
  rp.active = a.active;
  rp.m_in = a.m;
  rp.rows = (int)rows;
  rp.num_q_heads = a.hq;
  rp.tile_shift = ilog2(tile);
  rp.tiles_per_split = lay.pv.tiles_per_split;
  rp.group_shift = ilog2(tile);
  rp.gstride = (int)lay.tiles;
  rp.mstride = (int)(lay.tiles * kRefSlots);
  rp.tpb = tile;
  rp.rule = PAGER_ROUND_RUNNING;
  rp.ref_tail_start = nullptr;  // a chunk has no blocks: 64-token tiles from its first token
  rp.gmax = lay.gmax;
  rp.mref = lay.mref;
  ref_max_kernel<<<(unsigned)rows, kRefMaxThreads, 0, a.stream>>>(rp);
  PAGER_CUDA(cudaGetLastError(), "reference-max launch");
  p.tiles_per_split = lay.pv.tiles_per_split;
  p.max_splits = lay.pv.max_splits;
  void* vargs[] = {&p, &mk, &mv, &mS, &mM};
  PAGER_CUDA(cudaLaunchKernel(lay.kv.fn, dim3(lay.pv.max_splits, a.hkv, a.batch), dim3(lay.kv.threads), vargs,
                              lay.kv.smem_bytes, a.stream),
             "values kernel launch");
  CombineParams c;
  memset(&c, 0, sizeof(c));
  c.num_q_heads = a.hq;
  c.head_dim = a.head_dim;
  c.tile_shift = ilog2(tile);
  c.tiles_per_split = lay.pv.tiles_per_split;
  c.max_splits = lay.pv.max_splits;
  c.geom = p.geom;
  c.active = a.active;
  c.part_m = lay.sc.part_m;
  c.part_l = lay.sc.part_l;
  c.part_acc = lay.sc.part_acc;
  c.op = OP_STEP;
  c.m = a.m;
  c.l = a.l;
  c.acc = a.acc;
  combine_kernel<<<(unsigned)rows, 128, 0, a.stream>>>(c);
  PAGER_CUDA(cudaGetLastError(), "combine launch");
  return PAGER_OK;
}

// Whether a call runs the two reference-rounding passes: fp32 KV rounds p to fp32, which changes
// nothing, so the one pass already is the reference's arithmetic there.
bool exact_rounding(int rounding, int kv_dtype) { return rounding != PAGER_ROUND_ONE_PASS && kv_dtype != PAGER_DTYPE_F32; }

struct PagedLayout {
  PagedPlan pv;  // the pass that folds V (ONLINE, or VALUES with exact rounding)
  PagedPlan ps;  // SCORES (exact rounding only)
  long long s_stride, mstride;
  Scratch sc;
  float* scores;
  float* gmax;
  float* mref;
  size_t bytes;
};

int paged_layout(int batch, int hq, int hkv, int head_dim, int kv_dtype, int tpb, int max_row_tokens, int backend,
                 int rounding, char* base, PagedLayout* L) {
  const bool exact = exact_rounding(rounding, kv_dtype);
  int rc = paged_plan(batch, hq, hkv, head_dim, kv_dtype, tpb, max_row_tokens, backend, &L->pv,
                      exact ? MODE_VALUES : MODE_ONLINE);
  if (rc) return rc;
  const long long rows = (long long)batch * hq;
  L->sc = layout_scratch(base, rows, L->pv.plan.max_splits, head_dim, L->pv.gstride);
  size_t off = L->sc.bytes;
  L->scores = L->gmax = L->mref = nullptr;
  L->s_stride = L->mstride = 0;
  if (exact) {
    rc = paged_plan(batch, hq, hkv, head_dim, kv_dtype, tpb, max_row_tokens, backend, &L->ps, MODE_SCORES);
    if (rc) return rc;
    if (L->ps.k.tile != L->pv.k.tile) return fail(PAGER_ERR_CUDA, "scores and values passes disagree on the tile");
    const long long tiles = L->pv.gstride * L->pv.G / L->pv.k.tile;
    L->s_stride = tiles * L->pv.k.tile;
    L->mstride = tiles * kRefSlots;
    auto take = [&](size_t n) {
      char* p = base ? base + off : nullptr;
      off += align256(n);
      return reinterpret_cast<float*>(p);
    };
    L->scores = take(sizeof(float) * rows * L->s_stride);
    L->gmax = take(sizeof(float) * rows * L->pv.gstride);
    L->mref = take(sizeof(float) * rows * L->mstride);
  }
  L->bytes = off;
  return PAGER_OK;
}

int run_paged(const PagedArgs& a) {
  int rc = check_geometry(a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim, a.kv_dtype, a.q_dtype);
  if (rc) return rc;
  if (a.batch == 0) return PAGER_OK;
  if (!dtype_ok(a.out_dtype)) return fail(PAGER_ERR_INVALID, "bad out dtype");
  if (!is_pow2(a.tokens_per_block) || a.tokens_per_block < 8)
    return fail(PAGER_ERR_UNSUPPORTED, "tokens_per_block must be a power of two >= 8, got %d", a.tokens_per_block);
  if (a.num_layers <= 0 || a.layer < 0 || a.layer >= a.num_layers)
    return fail(PAGER_ERR_INVALID, "layer %d out of range for %d layers", a.layer, a.num_layers);
  if (!a.q || !a.out || !a.num_blocks || a.max_blocks < 0 || (a.max_blocks > 0 && !a.block_table))
    return fail(PAGER_ERR_INVALID, "null tensor pointer");
  if (a.max_row_tokens <= 0) return fail(PAGER_ERR_INVALID, "max_row_tokens must be positive");
  if (a.tail_len && (!a.tail_k || !a.tail_v || a.tail_cap <= 0)) return fail(PAGER_ERR_INVALID, "tail tensors missing");
  if ((a.dev_pool && !aligned16(a.dev_pool)) || (a.host_pool && !aligned16(a.host_pool)) ||
      (a.tail_k && !aligned16(a.tail_k)) || (a.tail_v && !aligned16(a.tail_v)))
    return fail(PAGER_ERR_INVALID, "pools and tail tensors must be 16-byte aligned");
  if (a.dev_slots < 0 || a.host_slots < 0 || a.stage_slots < 0) return fail(PAGER_ERR_INVALID, "negative pool capacity");
  if (a.dev_slots >= (1 << 29) || a.host_slots >= (1 << 29) || a.stage_slots >= (1 << 29))
    return fail(PAGER_ERR_INVALID, "pool capacity must stay below 2^29 slots (block-table tag bits)");
  if ((long long)a.dev_slots * a.num_layers * 2 * a.num_kv_heads >= (1LL << 31) ||
      (long long)a.host_slots * a.num_layers * 2 * a.num_kv_heads >= (1LL << 31) ||
      (long long)a.stage_slots * 2 * a.num_kv_heads >= (1LL << 31))
    return fail(PAGER_ERR_INVALID, "pool too large: slots * layers * 2 * kv_heads must stay below 2^31");
  if (a.stage_pool && !aligned16(a.stage_pool)) return fail(PAGER_ERR_INVALID, "staging buffer must be 16-byte aligned");
  if (a.mass_mode != PAGER_MASS_NONE && a.mass_mode != PAGER_MASS_ROW_MEAN && a.mass_mode != PAGER_MASS_BATCH_MEAN)
    return fail(PAGER_ERR_INVALID, "unknown mass mode %d", a.mass_mode);
  if (a.mass_mode != PAGER_MASS_NONE && !a.mass_accum) return fail(PAGER_ERR_INVALID, "mass_accum is null");
  if (a.rounding != PAGER_ROUND_ONE_PASS && a.rounding != PAGER_ROUND_RUNNING && a.rounding != PAGER_ROUND_FINAL)
    return fail(PAGER_ERR_INVALID, "unknown rounding mode %d", a.rounding);
  const bool exact = exact_rounding(a.rounding, a.kv_dtype);
  if (exact) {
    if (a.rounding == PAGER_ROUND_RUNNING && a.tokens_per_block < 16 &&
        backend_for(a.backend, a.kv_dtype, a.head_dim) == PAGER_BACKEND_MMA)
      return fail(PAGER_ERR_UNSUPPORTED, "running-max reference rounding needs tokens_per_block >= 16, got %d",
                  a.tokens_per_block);
  }

  PagedLayout lay;
  rc = paged_layout(a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim, a.kv_dtype, a.tokens_per_block,
                    a.max_row_tokens, a.backend, a.rounding, static_cast<char*>(a.scratch), &lay);
  if (rc) return rc;
  if (!a.scratch || a.scratch_bytes < lay.bytes)
    return fail(PAGER_ERR_SCRATCH, "scratch too small: need %zu bytes, got %zu", lay.bytes, a.scratch_bytes);
  const PagedPlan& pp = lay.pv;
  const Scratch& sc = lay.sc;
  const long long rows = (long long)a.batch * a.num_q_heads;
  DevInfo* di;
  rc = device_info(&di);
  if (rc) return rc;

  const long long row_bytes = (long long)a.head_dim * dtype_size(a.kv_dtype);
  const long long layer_stride = 2LL * a.num_kv_heads * a.tokens_per_block * row_bytes;
  const int br = a.tokens_per_block < pp.k.tile ? a.tokens_per_block : pp.k.tile;
  CUtensorMap mk;
  memset(&mk, 0, sizeof(mk));
  if (a.dev_pool && a.dev_slots > 0) {
    const uint64_t z = (uint64_t)a.dev_slots * a.num_layers * 2 * a.num_kv_heads;
    rc = encode_3d(&mk, a.kv_dtype, a.dev_pool, a.head_dim, a.tokens_per_block, z, pp.k.panel_elts, br,
                   pp.k.panel_bytes);
    if (rc) return rc;
  }
  CUtensorMap ms;  // staging buffer [stage_slots, 2, Hkv, tpb, D]: one layer of copied host blocks
  memset(&ms, 0, sizeof(ms));
  const bool staged = a.stage_pool && a.stage_slots > 0;
  if (staged) {
    const uint64_t z = (uint64_t)a.stage_slots * 2 * a.num_kv_heads;
    rc = encode_3d(&ms, a.kv_dtype, a.stage_pool, a.head_dim, a.tokens_per_block, z, pp.k.panel_elts, br,
                   pp.k.panel_bytes);
    if (rc) return rc;
  }
  CUtensorMap mS, mM;  // exact rounding: score tiles [n_rep][TILE] and reference maxima [n_rep][kRefSlots]
  memset(&mS, 0, sizeof(mS));
  memset(&mM, 0, sizeof(mM));
  const int n_rep = a.num_q_heads / a.num_kv_heads;
  if (exact) {
    rc = encode_2d_f32(&mS, lay.scores, (uint64_t)lay.s_stride, (uint64_t)rows, (uint32_t)pp.k.tile, (uint32_t)n_rep);
    if (rc) return rc;
    rc = encode_2d_f32(&mM, lay.mref, (uint64_t)lay.mstride, (uint64_t)rows, (uint32_t)kRefSlots, (uint32_t)n_rep);
    if (rc) return rc;
  }
  SplitParams p;
  memset(&p, 0, sizeof(p));
  p.q = a.q;
  p.q_dtype = a.q_dtype;
  p.batch = a.batch;
  p.num_q_heads = a.num_q_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.n_rep = n_rep;
  p.scale = a.scale;
  p.softcap = a.softcap > 0.f ? a.softcap : 0.f;
  p.source = SRC_PAGED;
  p.dev_pool = (a.dev_pool && a.dev_slots > 0) ? static_cast<const char*>(a.dev_pool) : nullptr;
  p.host_pool = (a.host_pool && a.host_slots > 0) ? static_cast<const char*>(a.host_pool) : nullptr;
  p.stage_pool = staged ? static_cast<const char*>(a.stage_pool) : nullptr;
  p.stage_slots = staged ? a.stage_slots : 0;
  p.slot_stride_bytes = layer_stride * a.num_layers;
  p.layer_stride_bytes = layer_stride;
  p.num_layers = a.num_layers;
  p.layer = a.layer;
  p.tpb = a.tokens_per_block;
  p.log2_tpb = ilog2(a.tokens_per_block);
  p.dev_slots = a.dev_slots;
  p.host_slots = a.host_slots;
  p.block_table = a.block_table;
  p.max_blocks = a.max_blocks;
  p.tail_k = static_cast<const char*>(a.tail_k);
  p.tail_v = static_cast<const char*>(a.tail_v);
  p.tail_cap = a.tail_cap;
  p.geom.source = SRC_PAGED;
  p.geom.tpb = a.tokens_per_block;
  p.geom.num_blocks = a.num_blocks;
  p.geom.max_blocks = a.max_blocks;
  p.geom.tail_len = a.tail_len;
  p.geom.tail_cap = a.tail_len ? a.tail_cap : 0;
  p.geom.max_tokens = a.max_row_tokens;
  p.geom.valid_lo = a.valid_lo;
  p.geom.valid_hi = a.valid_hi;
  p.active = a.active;
  p.part_m = sc.part_m;
  p.part_l = sc.part_l;
  p.part_acc = sc.part_acc;
  p.mass_part = sc.mass_part;
  p.mass_gstride = (int)pp.gstride;
  p.group_tokens = pp.G;
  p.log2_group = ilog2(pp.G);
  p.scores = lay.scores;
  p.s_stride = lay.s_stride;
  p.gmax = lay.gmax;
  p.wait_limit_ns = kWaitLimitNs;
  p.status = di->status;

  cudaStream_t st = (cudaStream_t)a.stream;
  CUtensorMap* map2 = staged ? &ms : &mk;
  if (exact) {
    SplitParams ps = p;  // SCORES: its own split plan over the same tiles
    ps.tiles_per_split = lay.ps.plan.tiles_per_split;
    ps.max_splits = lay.ps.plan.max_splits;
    dim3 grid_s(lay.ps.plan.max_splits, a.num_kv_heads, a.batch);
    void* sargs[] = {&ps, &mk, map2, &mS, &mM};
    PAGER_CUDA(launch_serialized(lay.ps.k.fn, grid_s, dim3(lay.ps.k.threads), lay.ps.k.smem_bytes, st, sargs),
               "scores kernel launch");
    RefMaxParams rp;
    memset(&rp, 0, sizeof(rp));
    rp.geom = p.geom;
    rp.active = a.active;
    rp.rows = (int)rows;
    rp.num_q_heads = a.num_q_heads;
    rp.tile_shift = ilog2(pp.k.tile);
    rp.tiles_per_split = pp.plan.tiles_per_split;
    rp.group_shift = ilog2(pp.G);
    rp.gstride = (int)pp.gstride;
    rp.mstride = (int)lay.mstride;
    rp.tpb = a.tokens_per_block;
    rp.rule = a.rounding;
    rp.ref_group_tokens = a.ref_group_tokens;
    rp.ref_shift = a.ref_shift;
    rp.ref_tail_start = a.ref_tail_start;
    rp.gmax = lay.gmax;
    rp.mref = lay.mref;
    void* rargs[] = {&rp};
    PAGER_CUDA(launch_serialized(reinterpret_cast<const void*>(&ref_max_kernel), dim3((unsigned)rows),
                                 dim3(kRefMaxThreads), 0, st, rargs),
               "reference-max launch");
  }
  p.tiles_per_split = pp.plan.tiles_per_split;
  p.max_splits = pp.plan.max_splits;
  dim3 grid(pp.plan.max_splits, a.num_kv_heads, a.batch);
  void* args[] = {&p, &mk, map2, &mS, &mM};
  PAGER_CUDA(launch_serialized(pp.k.fn, grid, dim3(pp.k.threads), pp.k.smem_bytes, st, args), "split kernel launch");

  CombineParams c;
  memset(&c, 0, sizeof(c));
  c.num_q_heads = a.num_q_heads;
  c.head_dim = a.head_dim;
  c.tile_shift = ilog2(pp.k.tile);
  c.tiles_per_split = pp.plan.tiles_per_split;
  c.max_splits = pp.plan.max_splits;
  c.geom = p.geom;
  c.active = a.active;
  c.part_m = sc.part_m;
  c.part_l = sc.part_l;
  c.part_acc = sc.part_acc;
  c.op = OP_PAGED;
  c.out = a.out;
  c.out_dtype = a.out_dtype;
  PagedMassParams mp;
  memset(&mp, 0, sizeof(mp));
  int mass_x = 1, mass_y = 0;
  if ((a.block_mass || a.mass_mode != PAGER_MASS_NONE) && a.max_blocks > 0) {
    mp.mass_part = sc.mass_part;
    mp.gstride = (int)pp.gstride;
    mp.group_shift = ilog2(pp.G);
    mp.tile_shift = ilog2(pp.k.tile);
    mp.tpb = a.tokens_per_block;
    mp.tiles_per_split = pp.plan.tiles_per_split;
    mp.geom = p.geom;
    mp.active = a.active;
    mp.part_m = sc.part_m;
    mp.part_l = sc.part_l;
    mp.max_splits = pp.plan.max_splits;
    mp.batch = a.batch;
    mp.num_q_heads = a.num_q_heads;
    mp.max_blocks = a.max_blocks;
    mp.block_mass = a.block_mass;
    mp.mass_accum = a.mass_accum;
    mp.mass_mode = a.mass_mode;
    mass_x = (a.max_blocks + 31) / 32;
    mass_y = a.mass_mode == PAGER_MASS_BATCH_MEAN ? 1 : a.batch;
  }
  int rows_i = (int)rows;
  const long long ctas = rows + (long long)mass_x * mass_y;
  if (ctas >= (1LL << 31)) return fail(PAGER_ERR_INVALID, "too many rows and blocks for one launch");
  void* fargs[] = {&c, &mp, &rows_i, &mass_x};
  PAGER_CUDA(launch_serialized(reinterpret_cast<const void*>(&paged_finish_kernel), dim3((unsigned)ctas),
                               dim3(kFinishThreads), 0, st, fargs),
             "combine/mass launch");
  return PAGER_OK;
}

}  // namespace
}  // namespace pager

extern "C" {

int pager_paged_decode_attention_staged(const void* q, int q_dtype, const void* dev_pool, int dev_slots,
                                        const void* host_pool, int host_slots, const void* stage_pool,
                                        int stage_slots, int kv_dtype, int num_layers, int layer, int num_kv_heads,
                                        int tokens_per_block, int head_dim, const int32_t* block_table,
                                        int max_blocks, const int32_t* num_blocks, const void* tail_k,
                                        const void* tail_v, const int32_t* tail_len, int tail_cap,
                                        const int32_t* valid_lo, const int32_t* valid_hi, const int32_t* active,
                                        int batch, int num_q_heads, float scale, float softcap, int max_row_tokens,
                                        void* out, int out_dtype, float* block_mass, float* mass_accum,
                                        int mass_mode, int backend, void* scratch, size_t scratch_bytes,
                                        void* stream) {
  return pager_paged_decode_attention_rounded(
      q, q_dtype, dev_pool, dev_slots, host_pool, host_slots, stage_pool, stage_slots, kv_dtype, num_layers, layer,
      num_kv_heads, tokens_per_block, head_dim, block_table, max_blocks, num_blocks, tail_k, tail_v, tail_len,
      tail_cap, valid_lo, valid_hi, active, batch, num_q_heads, scale, softcap, max_row_tokens, out, out_dtype,
      block_mass, mass_accum, mass_mode, backend, PAGER_ROUND_ONE_PASS, 0, nullptr, nullptr, scratch, scratch_bytes,
      stream);
}

size_t pager_paged_decode_scratch_bytes_rounded(int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                                int kv_dtype, int tokens_per_block, int max_row_tokens,
                                                int rounding) {
  if (!exact_rounding(rounding, kv_dtype))
    return pager_paged_decode_scratch_bytes(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype, tokens_per_block,
                                            0, max_row_tokens);
  if (check_geometry(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype, kv_dtype)) return 0;
  if (batch <= 0 || max_row_tokens <= 0 || !is_pow2(tokens_per_block) || tokens_per_block < 8) return 0;
  size_t need = 0;  // the larger of the automatic backend's plan and the CUDA-core one's
  for (int be : {PAGER_BACKEND_AUTO, PAGER_BACKEND_FMA}) {
    PagedLayout lay;
    if (!paged_layout(batch, num_q_heads, num_kv_heads, head_dim, kv_dtype, tokens_per_block, max_row_tokens, be,
                      rounding, nullptr, &lay))
      need = lay.bytes > need ? lay.bytes : need;
  }
  return need;
}

int pager_paged_decode_attention_rounded(const void* q, int q_dtype, const void* dev_pool, int dev_slots,
                                         const void* host_pool, int host_slots, const void* stage_pool,
                                         int stage_slots, int kv_dtype, int num_layers, int layer, int num_kv_heads,
                                         int tokens_per_block, int head_dim, const int32_t* block_table,
                                         int max_blocks, const int32_t* num_blocks, const void* tail_k,
                                         const void* tail_v, const int32_t* tail_len, int tail_cap,
                                         const int32_t* valid_lo, const int32_t* valid_hi, const int32_t* active,
                                         int batch, int num_q_heads, float scale, float softcap, int max_row_tokens,
                                         void* out, int out_dtype, float* block_mass, float* mass_accum,
                                         int mass_mode, int backend, int rounding, int ref_group_tokens,
                                         const int32_t* ref_shift, const int32_t* ref_tail_start, void* scratch,
                                         size_t scratch_bytes, void* stream) {
  PagedArgs a;
  a.q = q;
  a.q_dtype = q_dtype;
  a.dev_pool = dev_pool;
  a.dev_slots = dev_slots;
  a.host_pool = host_pool;
  a.host_slots = host_slots;
  a.stage_pool = stage_pool;
  a.stage_slots = stage_slots;
  a.kv_dtype = kv_dtype;
  a.num_layers = num_layers;
  a.layer = layer;
  a.num_kv_heads = num_kv_heads;
  a.tokens_per_block = tokens_per_block;
  a.head_dim = head_dim;
  a.block_table = block_table;
  a.max_blocks = max_blocks;
  a.num_blocks = num_blocks;
  a.tail_k = tail_k;
  a.tail_v = tail_v;
  a.tail_len = tail_len;
  a.tail_cap = tail_cap;
  a.valid_lo = valid_lo;
  a.valid_hi = valid_hi;
  a.active = active;
  a.batch = batch;
  a.num_q_heads = num_q_heads;
  a.scale = scale;
  a.softcap = softcap;
  a.max_row_tokens = max_row_tokens;
  a.out = out;
  a.out_dtype = out_dtype;
  a.block_mass = block_mass;
  a.mass_accum = mass_accum;
  a.mass_mode = mass_mode;
  a.backend = backend;
  a.rounding = rounding;
  a.ref_group_tokens = ref_group_tokens;
  a.ref_shift = ref_shift;
  a.ref_tail_start = ref_tail_start;
  a.scratch = scratch;
  a.scratch_bytes = scratch_bytes;
  a.stream = stream;
  return run_paged(a);
}

int pager_selftest_bounded_wait(unsigned long long limit_ns, unsigned long long* waited_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 100000000ull)
    return fail(PAGER_ERR_INVALID, "limit_ns must be in (0, 100 ms], got %llu", limit_ns);
  DevInfo* di;
  const int rc = device_info(&di);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  bounded_wait_selftest_kernel<<<1, 32, 0, st>>>(limit_ns, di->status);
  PAGER_CUDA(cudaGetLastError(), "self-test launch");
  unsigned long long w = 0;
  PAGER_CUDA(cudaMemcpyFromSymbolAsync(&w, g_selftest_waited_ns, sizeof(w), 0, cudaMemcpyDeviceToHost, st),
             "self-test readback");
  PAGER_CUDA(cudaStreamSynchronize(st), "self-test sync");
  if (waited_ns) *waited_ns = w;
  return PAGER_OK;
}

int pager_host_pool_alloc(size_t bytes, void** host_ptr) {
  if (!host_ptr) return fail(PAGER_ERR_INVALID, "host_ptr is null");
  *host_ptr = nullptr;
  if (bytes == 0) return PAGER_OK;
  PAGER_CUDA(cudaHostAlloc(host_ptr, bytes, cudaHostAllocPortable | cudaHostAllocMapped), "cudaHostAlloc");
  return PAGER_OK;
}

int pager_host_pool_free(void* host_ptr) {
  if (!host_ptr) return PAGER_OK;
  PAGER_CUDA(cudaFreeHost(host_ptr), "cudaFreeHost");
  return PAGER_OK;
}

int pager_probe_h2d_copy_gbs(const void* host_src, void* dev_dst, size_t bytes, int iters, void* stream,
                             double* gbs_out) {
  if (!host_src || !dev_dst || !gbs_out || bytes == 0 || iters <= 0) return fail(PAGER_ERR_INVALID, "bad probe args");
  cudaStream_t s = (cudaStream_t)stream;
  cudaEvent_t e0, e1;
  PAGER_CUDA(cudaEventCreate(&e0), "event");
  PAGER_CUDA(cudaEventCreate(&e1), "event");
  float best = 1e30f;
  for (int i = 0; i <= iters; ++i) {
    cudaEventRecord(e0, s);
    cudaMemcpyAsync(dev_dst, host_src, bytes, cudaMemcpyHostToDevice, s);
    cudaEventRecord(e1, s);
    cudaError_t e = cudaEventSynchronize(e1);
    if (e != cudaSuccess) {
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      return cuda_fail(e, "h2d probe");
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    if (i > 0 && ms < best) best = ms;  // first copy is a warm-up
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *gbs_out = (double)bytes / (best * 1e6);
  return PAGER_OK;
}

int pager_probe_zero_copy_gbs(const void* host_src, void* dev_dst, size_t bytes, int iters, void* stream,
                              double* gbs_out) {
  if (!host_src || !dev_dst || !gbs_out || bytes < 16 || iters <= 0 || !aligned16(host_src) || !aligned16(dev_dst))
    return fail(PAGER_ERR_INVALID, "bad probe args");
  DevInfo* di;
  int rc = device_info(&di);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  cudaEvent_t e0, e1;
  PAGER_CUDA(cudaEventCreate(&e0), "event");
  PAGER_CUDA(cudaEventCreate(&e1), "event");
  const long long n16 = (long long)(bytes / 16);
  float best = 1e30f;
  for (int i = 0; i <= iters; ++i) {
    cudaEventRecord(e0, s);
    zero_copy_probe_kernel<<<di->sms * 4, 256, 0, s>>>(static_cast<const uint4*>(host_src), static_cast<uint4*>(dev_dst), n16);
    cudaEventRecord(e1, s);
    cudaError_t e = cudaEventSynchronize(e1);
    if (e != cudaSuccess) {
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      return cuda_fail(e, "zero-copy probe");
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    if (i > 0 && ms < best) best = ms;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *gbs_out = (double)(n16 * 16) / (best * 1e6);
  return PAGER_OK;
}

}  // extern "C"
