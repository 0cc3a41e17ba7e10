// Split-KV decode-attention kernel for sm_100a.
//
// One CTA = one work unit (batch row b, KV head h, split s): a contiguous run
// of TILE-token tiles of row b.  Warps 0 .. NCW-1 are consumers, the warps after
// them producers (TileCfg: NCW 3 or 4 and one producer on the tensor-core path, 6
// and 2 on the CUDA-core path).  A producer streams K/V tiles into a ring of
// shared-memory stages -- TMA tensor loads (128B-swizzled) for HBM-resident
// data, 16-byte zero-copy loads for blocks in the pinned host pool and for the
// tail -- signalling per-stage mbarriers.  Tile i goes to consumer warp
// i % NCW, which folds it into its own online softmax state (m, l, acc) for the
// n_rep query heads sharing KV head h.  At the end the warp states are merged
// and the split's partial state is written to scratch; a combine kernel merges
// splits.
//
// Modes (the reference's four kernels, pager_hf/streaming_attention.py):
//   ONLINE  one-pass (m, l, acc) fold            (_decode_attention_step_kernel :77-185)
//   STATS   (m, l) only, K only                  (_decode_attention_stats_kernel :188-261)
//   FIXED   acc += exp(s - m_final) . V          (_decode_attention_accumulate_kernel :264-352,
//                                                 _decode_attention_fold_fixed_kernel :355-430)
// In ONLINE and FIXED modes the kernel also emits per-group attention-mass
// partials (sum of p over `group_tokens` tokens, with the running max it is
// relative to), from which the per-block mass is assembled without a second
// pass over KV.
//
// Reference-exact rounding of P (the reference rounds p = exp(s - m) to the
// value dtype before P.V, with m its running max at each 64-token tile in
// sequence order, or the final max in its two-pass path; a split-KV pass
// cannot know either, so its roundings differ in about half of the bf16
// outputs).  Two more modes do the same arithmetic in two passes without
// reading K twice:
//   SCORES  K only: writes the masked fp32 scores of every attended tile and
//           the max of every `group_tokens` group; a small scan kernel turns
//           the group maxima into the reference's max for each group.
//   VALUES  V only: the producer brings each tile's scores and reference
//           maxima in by TMA next to the V tile; p is formed against the
//           reference max of its group, rounded, and folded like ONLINE.
#pragma once

#include <type_traits>

#include "pager_device.cuh"

namespace pager {

// MODE_VALUES_R4 / MODE_VALUES_R8: MODE_VALUES for at most 4 / 8 query heads per KV head, with a
// score ring of that many rows (R4: room for one more stage of V in the same shared memory) and the
// swapped-operand consumers.
enum Mode {
  MODE_ONLINE = 0, MODE_STATS = 1, MODE_FIXED = 2, MODE_SCORES = 3, MODE_VALUES = 4, MODE_VALUES_R4 = 5,
  MODE_VALUES_R8 = 6
};
enum Source { SRC_CONTIG = 0, SRC_PAGED = 1 };
enum Backend { BACKEND_MMA = 1, BACKEND_FMA = 2 };

// 6 consumer warps + 2 producer warps: 8 warps, 2 per scheduler, up to 255 registers each.
// The consumer count must be even and at most the stage count (see consumer_wait).
constexpr int kMaxRep = 16;
constexpr int kHostSlotBit = 0x40000000;   // block-table entry: slot of the pinned host pool
constexpr int kStageSlotBit = 0x20000000;  // block-table entry: slot of the device staging buffer
constexpr int kStatusTimeout = 5;
constexpr int kStatusBadBlock = 6;

struct RowGeom {
  int nb, ntok, lo, hi;
};

// Everything that defines a row's token range; shared by the split, combine
// and mass kernels so that all three agree on the tiles of every row.
struct GeomArgs {
  int source;
  int tokens;  // SRC_CONTIG: tokens per row
  int tpb;
  const int* num_blocks;
  int max_blocks;
  const int* tail_len;
  int tail_cap;
  int max_tokens;  // host-known bound; longer rows are clamped (and flagged)
  const int* valid_lo;
  const int* valid_hi;
};

// Clamps every per-row input to the buffers it indexes, so a bad row length
// can never send a load or a scratch write out of bounds.
__device__ __forceinline__ RowGeom row_geom(const GeomArgs& a, int b, bool* clamped = nullptr) {
  RowGeom g;
  bool c = false;
  if (a.source == SRC_CONTIG) {
    g.nb = 0;
    g.ntok = a.tokens;
  } else {
    int nb = a.num_blocks[b];
    if (nb < 0 || nb > a.max_blocks) {
      c = true;
      nb = nb < 0 ? 0 : a.max_blocks;
    }
    int tl = a.tail_len ? a.tail_len[b] : 0;
    if (tl < 0 || tl > a.tail_cap) {
      c = true;
      tl = tl < 0 ? 0 : a.tail_cap;
    }
    g.nb = nb;
    g.ntok = nb * a.tpb + tl;
    if (g.ntok > a.max_tokens) {
      c = true;
      g.ntok = a.max_tokens;
    }
  }
  g.lo = a.valid_lo ? max(0, a.valid_lo[b]) : 0;
  g.hi = a.valid_hi ? min(g.ntok, a.valid_hi[b]) : g.ntok;
  if (clamped) *clamped = c;
  return g;
}

__device__ __forceinline__ void geom_tiles(const RowGeom& g, int tile_shift, int tps, int& t_begin, int& t_end,
                                           int& nsplit) {
  if (g.hi <= g.lo) {
    t_begin = t_end = nsplit = 0;
    return;
  }
  t_begin = g.lo >> tile_shift;
  t_end = (g.hi + (1 << tile_shift) - 1) >> tile_shift;
  nsplit = (t_end - t_begin + tps - 1) / tps;
}

struct SplitParams {
  // queries
  const void* q;
  int q_dtype;
  int batch, num_q_heads, num_kv_heads, n_rep;
  float scale, softcap;  // softcap <= 0: off
  // source of K/V and row geometry
  GeomArgs geom;
  int source;
  const char* dev_pool;
  const char* host_pool;
  const char* stage_pool;        // one layer's host blocks copied to the device: [slots, 2, Hkv, tpb, D]
  long long slot_stride_bytes;   // SRC_PAGED: bytes per pool slot (all layers)
  long long layer_stride_bytes;  // bytes per (slot, layer) = 2 * Hkv * tpb * row bytes
  int num_layers, layer, tpb, log2_tpb;
  int dev_slots, host_slots, stage_slots;  // capacities (block-table entries are checked against them)
  const int* block_table;
  int max_blocks;
  const char* tail_k;
  const char* tail_v;
  int tail_cap;
  // validity
  const int* valid;
  long long valid_stride;
  const int* active;
  // MODE_FIXED: final statistics
  const float* m_fixed;
  const float* l_fixed;
  // decomposition
  int tiles_per_split, max_splits;
  // outputs
  float* part_m;    // [B, Hq, max_splits]
  float* part_l;    // [B, Hq, max_splits]
  float* part_acc;  // [B, Hq, max_splits, D]
  float2* mass_part;  // [B, Hq, mass_gstride]: (sum p, reference max)
  int mass_gstride;
  int group_tokens;  // 0: no mass partials
  int log2_group;
  // MODE_SCORES outputs (MODE_VALUES reads them back through its tensor maps)
  float* scores;       // [B*Hq, s_stride]: masked scores of every attended tile
  long long s_stride;  // tokens per score row (the plan's tiles * TILE)
  float* gmax;         // [B*Hq, mass_gstride]: max score of every group_tokens group
  unsigned long long wait_limit_ns;
  int* status;
};

constexpr int kRefSlots = 8;  // reference-max entries per tile in the VALUES pass (groups per tile <= 8)

constexpr int kTableCache = 1024;  // block-table entries cached in shared memory per CTA

template <typename T, int D, int MODE, int BACKEND>
struct TileCfg {
  static constexpr int ELT = sizeof(T);
  static constexpr int ROW_BYTES = D * ELT;
  // 16 KiB of KV per stage: a K and a V tile, or one tile twice as long in the passes that read
  // one of them (per-tile costs -- waits, table lookups, the online update -- then spread over as
  // many bytes as in the one-pass kernel)
  static constexpr bool SINGLE =
      MODE == MODE_STATS || MODE == MODE_SCORES || MODE == MODE_VALUES || MODE == MODE_VALUES_R4 || MODE == MODE_VALUES_R8;
  static constexpr int TILE_RAW = 16384 / ((SINGLE ? 1 : 2) * ROW_BYTES);
  static constexpr int TILE = TILE_RAW > 64 ? 64 : (TILE_RAW < 16 ? 16 : TILE_RAW);
  static constexpr int LOG2_TILE = TILE == 64 ? 6 : (TILE == 32 ? 5 : 4);
  static constexpr int PANEL_BYTES = ROW_BYTES < 128 ? ROW_BYTES : 128;
  static constexpr int NPANEL = ROW_BYTES / PANEL_BYTES;
  static constexpr int PANEL_ELTS = PANEL_BYTES / ELT;
  static constexpr int CPP = PANEL_BYTES / 16;  // 16-byte chunks per panel row
  static constexpr int CPR = ROW_BYTES / 16;    // 16-byte chunks per row
  static constexpr int SWZ_MASK = CPP - 1;
  static constexpr int PANEL_TILE_BYTES = TILE * PANEL_BYTES;
  static constexpr int TENSOR_BYTES = TILE * ROW_BYTES;
  static constexpr bool KONLY = MODE == MODE_STATS || MODE == MODE_SCORES;  // K tiles only
  static constexpr bool VONLY = MODE == MODE_VALUES || MODE == MODE_VALUES_R4 || MODE == MODE_VALUES_R8;  // V only
  static constexpr bool SWAPPED = MODE == MODE_VALUES_R4 || MODE == MODE_VALUES_R8;  // swapped-operand consumers
  static constexpr int AUX_REP = MODE == MODE_VALUES_R4 ? 4 : (MODE == MODE_VALUES_R8 ? 8 : kMaxRep);  // score rows
  static constexpr int STAGE_BYTES = (KONLY || VONLY ? 1 : 2) * TENSOR_BYTES;
  // VALUES: a second ring beside the tensor ring holds each stage's score tile [n_rep][TILE] and
  // reference maxima [n_rep][kRefSlots] (fp32, no swizzle), filled by the same full barrier.
  static constexpr int AUX_S_BYTES = VONLY ? AUX_REP * TILE * 4 : 0;
  static constexpr int AUX_BYTES = VONLY ? (AUX_S_BYTES + AUX_REP * kRefSlots * 4 + 127) / 128 * 128 : 0;
  // Shared memory outside the stage ring: Q (bf16/fp16 for mma, fp32 for fma), the fma
  // path's P buffer, the block-table cache, barriers.
  // CTA shape.  Tensor-core configs: 3 consumer warps (4 for MODE_VALUES_R4/R8) + 1 producer warp, two CTAs
  // per SM (half the shared memory each), so that one CTA's prologue, pipeline fill and merge
  // overlap the other's streaming and the grid has twice the slots to balance splits over.
  // CUDA-core configs (compute-bound): 6 consumer + 2 producer warps, one CTA per SM.
  // consumer warps: the swapped-operand values pass (at most 184 registers a thread) fits a fourth warp at
  // two CTAs per SM, which hides more of its per-tile latency (measured: 206.0 -> 199.4 us per
  // hbm-32k layer; a fourth scores warp, or a fifth values warp, measured slower)
  static constexpr int NCW = BACKEND == BACKEND_MMA ? (SWAPPED ? 4 : 3) : 6;
  static constexpr int NPW = BACKEND == BACKEND_MMA ? 1 : 2;  // producer warps (one thread each)
  static constexpr int THREADS = (NCW + NPW) * 32;
  static constexpr int MIN_BLOCKS = BACKEND == BACKEND_MMA ? 2 : 1;
  static constexpr int SMEM_BUDGET = BACKEND == BACKEND_MMA ? 110 * 1024 : 225 * 1024;
  static constexpr int Q_BYTES = VONLY ? 0 : (BACKEND == BACKEND_FMA ? kMaxRep * D * 4 : kMaxRep * D * ELT);
  static constexpr int P_BYTES = BACKEND == BACKEND_FMA ? NCW * TILE * kMaxRep * 4 : 0;
  static constexpr int EXTRA = Q_BYTES + P_BYTES + kTableCache * 4 + 1536;
  // A deep ring: each consumer warp holds a stage while it computes, the rest stay in flight.
  // With two producer warps the count is even, so that each stage is always filled by the same one.
  static constexpr int STAGES_FIT = (SMEM_BUDGET - EXTRA) / (STAGE_BYTES + AUX_BYTES);
  static constexpr int STAGES_RAW = NPW == 2 ? (STAGES_FIT & ~1) : STAGES_FIT;
  static constexpr int STAGES = STAGES_RAW > 16 ? 16 : STAGES_RAW;
  static_assert(STAGES >= NCW && (NPW == 1 || STAGES % 2 == 0), "stage ring too shallow for the consumer warps");
  static constexpr int STAGE_AREA = STAGES * STAGE_BYTES;
  static constexpr int MERGE_BYTES = NCW * kMaxRep * (2 + (KONLY ? 0 : D)) * 4;
  static_assert(MERGE_BYTES <= STAGE_AREA, "merge region must fit in the stage ring");
  static_assert((TILE & (TILE - 1)) == 0 && TILE >= 16 && TILE <= 64, "tile");
};

// Physical byte offset of logical offset `off` inside a panel written by TMA
// with the swizzle mode matching the panel width (128B / 64B / 32B / none).
template <class Cfg>
__device__ __forceinline__ uint32_t swz(uint32_t off) {
  return off ^ (((off >> 7) & Cfg::SWZ_MASK) << 4);
}

template <class Cfg>
__device__ __forceinline__ uint32_t chunk_addr(uint32_t tile_base, int row, int chunk) {
  const int panel = chunk / Cfg::CPP;
  const int cp = chunk % Cfg::CPP;
  return tile_base + panel * Cfg::PANEL_TILE_BYTES + swz<Cfg>(row * Cfg::PANEL_BYTES + cp * 16);
}

// This CTA's block-table entries, copied to shared memory in the prologue so
// that neither the producer nor the consumers wait on global loads per tile.
struct TableCache {
  const int* sm;
  int blk0, n;
};

__device__ __forceinline__ bool bit_of(uint32_t lo_bits, uint32_t hi_bits, int t) {
  return ((t < 32 ? (lo_bits >> t) : (hi_bits >> (t - 32))) & 1u) != 0;
}

// Hot fields of SplitParams copied into registers once per warp.  The kernel
// parameter block lives in parameter space and is reached through a reference;
// after every volatile shared-memory store (tickets, abort flag) the compiler
// may not assume it unchanged and re-loads each field, which put several
// hundred nanoseconds into every tile of the producer's loop.
struct Hot {
  const int* block_table;
  const char* dev_pool;
  const char* host_pool;
  const char* tail_k;
  const char* tail_v;
  const int* valid;
  int* status;
  long long valid_stride, slot_stride, layer_stride;
  unsigned long long wait_limit;
  int source, tpb, log2_tpb, max_blocks, num_layers, layer, hkv, dev_slots, host_slots, stage_slots, tail_cap;
};

__device__ __forceinline__ Hot load_hot(const SplitParams& p) {
  Hot h;
  h.block_table = p.block_table;
  h.dev_pool = p.dev_pool;
  h.host_pool = p.host_pool;
  h.tail_k = p.tail_k;
  h.tail_v = p.tail_v;
  h.valid = p.valid;
  h.status = p.status;
  h.valid_stride = p.valid_stride;
  h.slot_stride = p.slot_stride_bytes;
  h.layer_stride = p.layer_stride_bytes;
  h.wait_limit = p.wait_limit_ns;
  h.source = p.source;
  h.tpb = p.tpb;
  h.log2_tpb = p.log2_tpb;
  h.max_blocks = p.max_blocks;
  h.num_layers = p.num_layers;
  h.layer = p.layer;
  h.hkv = p.num_kv_heads;
  h.dev_slots = p.dev_slots;
  h.host_slots = p.host_slots;
  h.stage_slots = p.stage_pool != nullptr ? p.stage_slots : 0;
  h.tail_cap = p.tail_cap;
  return h;
}

// A block-table entry names a slot that exists in a pool that was passed in:
// slot (device pool), slot | kHostSlotBit (host pool, read zero-copy) or
// slot | kStageSlotBit (this layer's copy of a host block in the staging buffer).
__device__ __forceinline__ bool entry_ok(const Hot& k, int e) {
  if (e < 0) return false;
  if (e & kHostSlotBit)
    return !(e & kStageSlotBit) && k.host_pool != nullptr && (e & (kStageSlotBit - 1)) < k.host_slots;
  if (e & kStageSlotBit) return (e & (kStageSlotBit - 1)) < k.stage_slots;
  return k.dev_pool != nullptr && e < k.dev_slots;
}

__device__ __forceinline__ int entry_at(const Hot& k, const TableCache& tc, int b, int blk) {
  const int i = blk - tc.blk0;
  if (i >= 0 && i < tc.n) return tc.sm[i];
  return k.block_table[(long long)b * k.max_blocks + blk];
}

// ------------------------------------------------------------------ producer helpers

// Warp-cooperative copy of `nrows` rows (row-contiguous source, any global or
// mapped-host address) into rows [row0, row0+nrows) of a swizzled tile.
template <class Cfg>
__device__ __forceinline__ void sw_copy_rows(uint32_t tile_base, int row0, const char* src, int nrows) {
  const int lane = threadIdx.x & 31;
  const int total = nrows * Cfg::CPR;
  constexpr int U = 4;  // 4 x 16 B in flight per lane: ample for the host link, few registers
  for (int c0 = 0; c0 < total; c0 += 32 * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < total) v[u] = ld_global_16(src + (size_t)c * 16);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < total) {
        const int r = c / Cfg::CPR;
        const int cw = c % Cfg::CPR;
        st_shared_16(chunk_addr<Cfg>(tile_base, row0 + r, cw), v[u]);
      }
    }
  }
}

// Rows that TMA cannot fetch -- blocks in the pinned host pool (read zero-copy
// over the host link) and tail rows -- are copied into the stage by the
// consumer warp that owns the tile, with 16-byte loads.  `mask` has one bit per
// segment of min(TILE, tokens_per_block) rows.
template <class Cfg, bool kNeedK, bool kNeedV>
__device__ __forceinline__ void copy_sw_segments(const SplitParams& p, const TableCache& tc, const RowGeom& g, int b,
                                                 int h, int t0, uint32_t mask, uint8_t* kbuf, uint8_t* vbuf) {
  // Slow path (host-pool blocks, tail rows): fields are read from the parameter block here
  // rather than kept live across the tile loop.
  const int tpb = p.tpb;
  const int br = min(Cfg::TILE, tpb);
  const int block_tokens = g.nb * tpb;
  const long long head_bytes = (long long)tpb * Cfg::ROW_BYTES;
  const uint32_t kaddr = smem_u32(kbuf), vaddr = smem_u32(vbuf);
  for (int sg = 0; mask; ++sg, mask >>= 1) {
    if (!(mask & 1u)) continue;
    const int tok = t0 + sg * br;
    const char* ksrc;
    long long vdelta;
    int n;
    if (tok < block_tokens) {
      const int blk = tok >> p.log2_tpb;
      const int i = blk - tc.blk0;
      const int e = (i >= 0 && i < tc.n) ? tc.sm[i] : p.block_table[(long long)b * p.max_blocks + blk];
      const long long slot = e & (kHostSlotBit - 1);
      ksrc = p.host_pool + slot * p.slot_stride_bytes + (long long)p.layer * p.layer_stride_bytes +
             (long long)h * head_bytes + (long long)(tok & (tpb - 1)) * Cfg::ROW_BYTES;
      vdelta = (long long)p.num_kv_heads * head_bytes;
      n = br;
    } else {
      const long long off =
          (((long long)b * p.num_kv_heads + h) * p.tail_cap + (tok - block_tokens)) * Cfg::ROW_BYTES;
      ksrc = p.tail_k + off;
      vdelta = p.tail_v - p.tail_k;
      n = min(br, g.ntok - tok);
    }
    if (kNeedK) sw_copy_rows<Cfg>(kaddr, sg * br, ksrc, n);
    if (kNeedV) sw_copy_rows<Cfg>(vaddr, sg * br, ksrc + vdelta, n);
  }
  __syncwarp();
}

// The producers are one thread each of two warps, taking alternate tiles (the
// stage ring has an even length, so a stage is always filled by the same
// producer).  Per tile: wait for the stage to be free, issue the TMA boxes of
// every device-resident segment, record the stage's segment masks in shared
// memory (bits 0-7: segments the consumer copies itself, bits 8-15: segments
// holding data) and arrive on the stage's full barrier (release).
template <class Cfg, int MODE>
__device__ void run_producer(const SplitParams& p, const TableCache& tc, const CUtensorMap* mapk,
                             const CUtensorMap* mapv, const CUtensorMap* maps, const CUtensorMap* mapm,
                             uint8_t* stages, uint8_t* aux, uint64_t* full, uint64_t* empty, volatile int* infos,
                             int b, int h, int tile0, int ntiles, const RowGeom& g, volatile int* abort_flag,
                             int producer) {
  if ((threadIdx.x & 31) != 0) return;
  constexpr bool kNeedK = !Cfg::VONLY;
  constexpr bool kNeedV = !Cfg::KONLY;
  const Hot k = load_hot(p);
  // VALUES: the tile's scores [n_rep][TILE] and reference maxima [n_rep][kRefSlots] (rows of the query
  // heads of KV head h), fetched with the V tile under the same full barrier
  const int aux_row0 = b * p.num_q_heads + h * p.n_rep;
  const uint32_t aux_tx = Cfg::VONLY ? (uint32_t)p.n_rep * (Cfg::TILE + kRefSlots) * 4u : 0u;
  const int zc = b * k.hkv + h;  // contiguous source: (row, kv head) plane
  const int br = min(Cfg::TILE, k.tpb);
  const int nseg = Cfg::TILE / br;
  const int block_tokens = g.nb * k.tpb;
  const uint32_t seg_bytes = (uint32_t)br * Cfg::ROW_BYTES * ((kNeedK ? 1u : 0u) + (kNeedV ? 1u : 0u));
  const uint64_t once = l2_policy_evict_first();  // every tile is read once per layer
  int last = -1;
  for (int i = producer; i < ntiles; i += Cfg::NPW) {
    const int s = i % Cfg::STAGES;
    const int use = i / Cfg::STAGES;
    if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1, k.wait_limit)) {
      atomicExch(k.status, kStatusTimeout);
      *abort_flag = 1;
      break;
    }
    uint8_t* kbuf = stages + s * Cfg::STAGE_BYTES;
    uint8_t* vbuf = Cfg::VONLY ? kbuf : kbuf + Cfg::TENSOR_BYTES;
    const int t0 = (tile0 + i) * Cfg::TILE;
    uint32_t sw_mask = 0;
    uint32_t present = 0;  // segments whose rows hold data (device, host or tail)
    if (Cfg::VONLY) {
      uint8_t* a = aux + s * Cfg::AUX_BYTES;
      mbar_expect_tx(&full[s], aux_tx);
      tma_load_2d_hint(a, maps, t0, aux_row0, &full[s], once);
      tma_load_2d_hint(a + Cfg::AUX_S_BYTES, mapm, (tile0 + i) * kRefSlots, aux_row0, &full[s], once);
    }
    if (k.source == SRC_CONTIG) {
      present = 1u;  // one segment: the whole tile
      mbar_expect_tx(&full[s], (uint32_t)Cfg::STAGE_BYTES);
#pragma unroll
      for (int pn = 0; pn < Cfg::NPANEL; ++pn) {
        if (kNeedK)
          tma_load_3d_hint(kbuf + pn * Cfg::PANEL_TILE_BYTES, mapk, pn * Cfg::PANEL_ELTS, t0, zc, &full[s], once);
        if (kNeedV)
          tma_load_3d_hint(vbuf + pn * Cfg::PANEL_TILE_BYTES, mapv, pn * Cfg::PANEL_ELTS, t0, zc, &full[s], once);
      }
    } else {
      for (int sg = 0; sg < nseg; ++sg) {
        const int tok = t0 + sg * br;
        if (tok >= g.hi || tok + br <= g.lo) continue;
        if (tok >= block_tokens) {
          sw_mask |= 1u << sg;  // tail rows
          present |= 1u << sg;
          continue;
        }
        const int e = entry_at(k, tc, b, tok >> k.log2_tpb);
        if (!entry_ok(k, e)) {
          if (e >= 0) atomicExch(k.status, kStatusBadBlock);
          continue;
        }
        present |= 1u << sg;
        if (e & kHostSlotBit) {
          sw_mask |= 1u << sg;
          continue;
        }
        mbar_expect_tx(&full[s], seg_bytes);
        // device pool: plane ((slot * L + layer) * 2 + kv) * Hkv + h; staging buffer (one layer,
        // described by the second tensor map): plane (slot * 2 + kv) * Hkv + h
        const bool staged = (e & kStageSlotBit) != 0;
        const int zk = staged ? ((e & (kStageSlotBit - 1)) * 2) * k.hkv + h : ((e * k.num_layers + k.layer) * 2) * k.hkv + h;
        const CUtensorMap* map = staged ? mapv : mapk;
        const int y = tok & (k.tpb - 1);
#pragma unroll
        for (int pn = 0; pn < Cfg::NPANEL; ++pn) {
          const int off = pn * Cfg::PANEL_TILE_BYTES + sg * br * Cfg::PANEL_BYTES;
          if (kNeedK) tma_load_3d_hint(kbuf + off, map, pn * Cfg::PANEL_ELTS, y, zk, &full[s], once);
          if (kNeedV) tma_load_3d_hint(vbuf + off, map, pn * Cfg::PANEL_ELTS, y, zk + k.hkv, &full[s], once);
        }
      }
    }
    infos[s] = (int)((present << 8) | sw_mask);
    mbar_arrive(&full[s]);  // release: the consumer that acquires the phase sees infos[s]
    last = i;
  }
  // Drain: never leave the CTA with bulk copies still landing in its shared memory.
  for (int i = last; i >= 0 && i > last - Cfg::STAGES; i -= Cfg::NPW) {
    if (!mbar_wait_bounded(&full[i % Cfg::STAGES], (i / Cfg::STAGES) & 1, k.wait_limit)) {
      atomicExch(k.status, kStatusTimeout);
      *abort_flag = 1;
      break;
    }
  }
}

// Consumer-side wait for tile i on stage s = i % STAGES (use n = i / STAGES).
// Tiles of one stage go to different warps, so a warp can reach use n of a
// stage while use n-1 is still loading or being consumed; a parity wait posed
// about a phase that is not yet the current one would alias the phase two back
// and succeed early.  The warp therefore first waits for use n-1 to be
// released (empty barrier, phase n-1) and then for use n to land (full
// barrier, phase n).  The empty wait itself cannot alias: this warp's previous
// tile, i - NCW, was issued, and with STAGES >= NCW tile i - STAGES was issued
// before it by the same producer (with one producer warp trivially; with two,
// because both counts are even, so tiles i - STAGES and i - NCW have the same
// producer, which issues in order) -- after use n-2 of the stage had been
// released.  Both waits suspend in hardware (mbarrier.try_wait) and
// are bounded; lane 0 waits, then every lane observes the completed full phase
// so the TMA writes are visible to it.  *info = the stage's segment masks.
__device__ __forceinline__ bool consumer_wait(uint64_t wait_limit, int* status, uint64_t* full_bar,
                                              uint64_t* empty_bar, volatile int* info, int use,
                                              volatile int* abort_flag, uint32_t* mask) {
  const int lane = threadIdx.x & 31;
  const uint32_t parity = use & 1;
  int ok = 1;
  uint32_t m = 0;
  if (lane == 0) {
    if (use > 0) ok = mbar_wait_bounded(empty_bar, (use - 1) & 1, wait_limit) ? 1 : 0;
    if (ok) ok = mbar_wait_bounded(full_bar, parity, wait_limit) ? 1 : 0;
    if (ok) m = (uint32_t)*info;
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  *mask = __shfl_sync(0xffffffffu, m, 0);
  if (!ok) {
    if (lane == 0) {
      atomicExch(status, kStatusTimeout);
      *abort_flag = 1;
    }
    return false;
  }
  while (!mbar_try_wait(full_bar, parity)) {
  }
  return true;
}

// Valid-token bits of a tile from its token range, the segments the producer
// found present, and (chunk ops only) the caller's per-token 0/1 mask.
template <int TILE>
__device__ __forceinline__ void tile_bits_fast(const int* valid, long long valid_stride, int b, int t0,
                                               const RowGeom& g, uint32_t present, int seg_rows, uint32_t& lo_bits,
                                               uint32_t& hi_bits) {
  const int lower = max(g.lo - t0, 0);
  const int upper = min(g.hi - t0, TILE);
  uint64_t m = 0;
  if (upper > lower) {
    const uint64_t hi_part = upper >= 64 ? ~0ull : ((1ull << upper) - 1ull);
    m = hi_part & ~((1ull << lower) - 1ull);
  }
  if (present != 1u || seg_rows < TILE) {
    uint64_t pm = 0;
    const uint64_t seg = seg_rows >= 64 ? ~0ull : ((1ull << seg_rows) - 1ull);
    for (int sg = 0; sg * seg_rows < TILE; ++sg)
      if ((present >> sg) & 1u) pm |= seg << (sg * seg_rows);
    m &= pm;
  }
  if (valid) {
    const int lane = threadIdx.x & 31;
    const bool v0 = lane < TILE && ((m >> lane) & 1ull) && valid[(long long)b * valid_stride + t0 + lane] != 0;
    const bool v1 = TILE > 32 && ((m >> (32 + lane)) & 1ull) &&
                    valid[(long long)b * valid_stride + t0 + 32 + lane] != 0;
    lo_bits = __ballot_sync(0xffffffffu, v0);
    hi_bits = __ballot_sync(0xffffffffu, v1);
    return;
  }
  lo_bits = (uint32_t)m;
  hi_bits = (uint32_t)(m >> 32);
}

// Zero the V rows of masked tokens so that 0 * (stale or non-finite) never
// reaches the P.V product (the reference loads masked rows as 0).
template <class Cfg>
__device__ __forceinline__ bool zero_masked_rows(uint8_t* vbuf, uint32_t lo_bits, uint32_t hi_bits) {
  const uint32_t need_lo = Cfg::TILE >= 32 ? 0xffffffffu : ((1u << Cfg::TILE) - 1u);
  const uint32_t need_hi = Cfg::TILE == 64 ? 0xffffffffu : 0u;
  if (lo_bits == need_lo && hi_bits == need_hi) return false;
  const int lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(vbuf);
  const int total = Cfg::TILE * Cfg::CPR;
  for (int c = lane; c < total; c += 32) {
    const int r = c / Cfg::CPR;
    if (!bit_of(lo_bits, hi_bits, r)) st_shared_16(chunk_addr<Cfg>(base, r, c % Cfg::CPR), make_uint4(0, 0, 0, 0));
  }
  __syncwarp();
  return true;
}

__device__ __forceinline__ void release_stage(uint64_t* bar, bool wrote) {
  if (wrote) fence_proxy_async_smem();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ float apply_score(float raw, float scale, float softcap) {
  float x = raw * scale;
  if (softcap > 0.f) x = softcap * tanhf(x / softcap);
  return x;
}

// Merge the four consumer warps' states (held in the stage area) and write
// this split's partial state.  `mw`: m_w[4][16], l_w[4][16], acc_w[4][16][D].
template <int D, int MODE, int NCW>
__device__ void merge_and_store(const SplitParams& p, float* mw, int b, int h, int split) {
  const int tid = threadIdx.x;
  const float* m_w = mw;
  const float* l_w = mw + NCW * kMaxRep;
  const float* acc_w = mw + 2 * NCW * kMaxRep;
  const int n_rep = p.n_rep;
  const int qh0 = h * n_rep;
  if (MODE != MODE_FIXED) {
    for (int r = tid; r < n_rep; r += NCW * 32) {
      float M = neg_inf();
#pragma unroll
      for (int w = 0; w < NCW; ++w) M = fmaxf(M, m_w[w * kMaxRep + r]);
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < NCW; ++w) {
        const float mwr = m_w[w * kMaxRep + r];
        const float wt = mwr == neg_inf() ? 0.f : fast_exp2((mwr - M) * kLog2e);
        L += wt * l_w[w * kMaxRep + r];
      }
      const long long o = ((long long)b * p.num_q_heads + qh0 + r) * p.max_splits + split;
      p.part_m[o] = M;
      p.part_l[o] = L;
    }
  }
  if constexpr (MODE != MODE_STATS) {
    for (int idx = tid; idx < n_rep * D; idx += NCW * 32) {
      const int r = idx / D;
      const int d = idx % D;
      float A = 0.f;
      if (MODE == MODE_FIXED) {
#pragma unroll
        for (int w = 0; w < NCW; ++w) A += acc_w[(w * kMaxRep + r) * D + d];
      } else {
        float M = neg_inf();
#pragma unroll
        for (int w = 0; w < NCW; ++w) M = fmaxf(M, m_w[w * kMaxRep + r]);
#pragma unroll
        for (int w = 0; w < NCW; ++w) {
          const float mwr = m_w[w * kMaxRep + r];
          const float wt = mwr == neg_inf() ? 0.f : fast_exp2((mwr - M) * kLog2e);
          A += wt * acc_w[(w * kMaxRep + r) * D + d];
        }
      }
      const long long o = ((long long)b * p.num_q_heads + qh0 + r) * p.max_splits + split;
      p.part_acc[o * D + d] = A;
    }
  }
}

// ------------------------------------------------------------------ tensor-core consumer
// One warp folds one tile: S = Q K^T and O += P V with mma.sync m16n8k16
// (fp32 accumulate), the n_rep query heads in the 16-row M dimension.
// Per-lane shared-memory addresses are precomputed once: with 128-byte
// swizzled panels the XOR term only depends on the lane.
template <typename T, int D, int MODE>
__device__ void run_consumer_mma(const SplitParams& p, const TableCache& tc, uint8_t* stages, uint64_t* full,
                                 uint64_t* empty, volatile int* infos, int b, int h, int tile0, int ntiles,
                                 const RowGeom& g, volatile int* abort_flag, int split, const T* q_smem) {
  using Cfg = TileCfg<T, D, MODE, BACKEND_MMA>;
  using Op = MmaOp<T>;
  static_assert(Cfg::PANEL_BYTES == 128, "mma path expects 128-byte panels");
  constexpr int KSTEPS = D / 16;
  constexpr int NT_O = D / 8;
  constexpr int NT_S = Cfg::TILE / 8;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int gr = lane >> 2;  // fragment row (query head within the group)
  const int tq = lane & 3;
  const int n_rep = p.n_rep;
  const int qh0 = h * n_rep;
  const int l7 = lane & 7;
  const int seg_rows = p.source == SRC_CONTIG ? Cfg::TILE : min(Cfg::TILE, p.tpb);
  const int* const valid = p.valid;
  const long long valid_stride = p.valid_stride;
  const uint64_t wait_limit = p.wait_limit_ns;
  int* const status = p.status;
  const float scale = p.scale;
  const float softcap = p.softcap;
  float2* const mass_part = p.mass_part;
  const int num_q_heads = p.num_q_heads;
  const int mass_gstride = p.mass_gstride;
  const int log2_group = p.log2_group;

  // Q is kept in shared memory in the tiles' 128-byte swizzled layout (16 rows) and its
  // fragments are re-read per tile: holding them in registers across the loop spilled.
  const uint32_t qaddr = smem_u32(q_smem);
  const int qrow = l7 + ((lane >> 3) & 1) * 8;
  float mfix_l2[2] = {0.f, 0.f};
  if (MODE == MODE_FIXED) {
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int row = gr + 8 * rr;
      const float mf = row < n_rep ? p.m_fixed[(long long)b * p.num_q_heads + qh0 + row] : 0.f;
      mfix_l2[rr] = mf * kLog2e;
    }
  }

  float o[NT_O][4];
#pragma unroll
  for (int n = 0; n < NT_O; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_r[2] = {neg_inf(), neg_inf()};
  float l_r[2] = {0.f, 0.f};
  const int G = p.group_tokens;
  const bool softcap_on = softcap > 0.f;
  const uint64_t full_mask = Cfg::TILE == 64 ? ~0ull : ((1ull << Cfg::TILE) - 1ull);

  for (int i = warp; i < ntiles; i += Cfg::NCW) {
    const int s = i % Cfg::STAGES;
    if (*abort_flag) break;
    uint32_t swm;
    if (!consumer_wait(wait_limit, status, &full[s], &empty[s], &infos[s], i / Cfg::STAGES, abort_flag, &swm)) break;
    const int t0 = (tile0 + i) * Cfg::TILE;
    uint8_t* kbuf = stages + s * Cfg::STAGE_BYTES;
    uint8_t* vbuf = kbuf + Cfg::TENSOR_BYTES;
    if (swm & 0xffu) copy_sw_segments<Cfg, true, !Cfg::KONLY>(p, tc, g, b, h, t0, swm & 0xffu, kbuf, vbuf);
    uint32_t vlo, vhi;
    tile_bits_fast<Cfg::TILE>(valid, valid_stride, b, t0, g, swm >> 8, seg_rows, vlo, vhi);
    const uint64_t vmask = ((uint64_t)vhi << 32) | vlo;
    const bool all_valid = vmask == full_mask;
    const uint32_t kaddr = smem_u32(kbuf);

    float sc[NT_S][4];
#pragma unroll
    for (int j = 0; j < NT_S; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kp = 0; kp < KSTEPS / 2; ++kp) {
      uint32_t qa0[4], qa1[4];
      {
        const int c0 = 4 * kp + (lane >> 4);  // A fragment chunk of k-step 2kp; +2 for 2kp+1
        const int c1 = c0 + 2;
        ldmatrix_x4(qaddr + (c0 >> 3) * 2048 + qrow * 128 + (((c0 & 7) ^ l7) << 4), qa0[0], qa0[1], qa0[2], qa0[3]);
        ldmatrix_x4(qaddr + (c1 >> 3) * 2048 + qrow * 128 + (((c1 & 7) ^ l7) << 4), qa1[0], qa1[1], qa1[2], qa1[3]);
      }
      const int c = 4 * kp + (lane >> 3);
      const uint32_t koff = (c >> 3) * Cfg::PANEL_TILE_BYTES + l7 * 128 + (((c & 7) ^ l7) << 4);
#pragma unroll
      for (int j = 0; j < NT_S; ++j) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kaddr + koff + j * 8 * 128, b0, b1, b2, b3);
        Op::run(sc[j], qa0, b0, b1);
        Op::run(sc[j], qa1, b2, b3);
      }
    }
    // scale, softcap, token mask (streaming_attention.py:158-161)
    const uint64_t tmask = vmask >> (2 * tq);
#pragma unroll
    for (int j = 0; j < NT_S; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = sc[j][e] * scale;
        if (softcap_on) x = softcap * tanhf(x / softcap);
        if (!all_valid && !((tmask >> (8 * j + (e & 1))) & 1ull)) x = neg_inf();
        sc[j][e] = x;
      }
    }
    if constexpr (MODE == MODE_SCORES) {
      // the masked scores of the tile, and the max of each group_tokens group, per query head
      float* const srow = p.scores + (long long)(b * num_q_heads + qh0) * p.s_stride + t0 + 2 * tq;
      const uint64_t keep = l2_policy_evict_last();  // read back by the values pass of this layer
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int row = gr + 8 * rr;
        if (row < n_rep) {
#pragma unroll
          for (int j = 0; j < NT_S; ++j)
            st_global_f2_hint(srow + (long long)row * p.s_stride + 8 * j, sc[j][2 * rr], sc[j][2 * rr + 1], keep);
        }
      }
      const int ntg = G >> 3;  // S n-tiles per group
      for (int gi = 0; gi < Cfg::TILE / G; ++gi) {
        float gm[2] = {neg_inf(), neg_inf()};
#pragma unroll
        for (int j = 0; j < NT_S; ++j) {
          if (j / ntg == gi) {
            gm[0] = fmaxf(gm[0], fmaxf(sc[j][0], sc[j][1]));
            gm[1] = fmaxf(gm[1], fmaxf(sc[j][2], sc[j][3]));
          }
        }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          gm[rr] = fmaxf(gm[rr], __shfl_xor_sync(0xffffffffu, gm[rr], 1));
          gm[rr] = fmaxf(gm[rr], __shfl_xor_sync(0xffffffffu, gm[rr], 2));
        }
        if (tq == 0) {
          const long long gidx = (t0 >> log2_group) + gi;
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int row = gr + 8 * rr;
            if (row < n_rep) p.gmax[((long long)b * num_q_heads + qh0 + row) * mass_gstride + gidx] = gm[rr];
          }
        }
      }
      release_stage(&empty[s], (swm & 0xffu) != 0);
      continue;
    }
    float mref[2];
    if (MODE != MODE_FIXED) {
      float mx[2] = {neg_inf(), neg_inf()};
#pragma unroll
      for (int j = 0; j < NT_S; ++j) {
        mx[0] = fmaxf(mx[0], fmaxf(sc[j][0], sc[j][1]));
        mx[1] = fmaxf(mx[1], fmaxf(sc[j][2], sc[j][3]));
      }
      bool changed = false;
      float alpha[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
        const float m_new = fmaxf(m_r[rr], mx[rr]);
        const bool empty_row = m_new == neg_inf();  // streaming_attention.py:171-177
        alpha[rr] = empty_row ? 0.f : (m_new == m_r[rr] ? 1.f : fast_exp2((m_r[rr] - m_new) * kLog2e));
        changed |= alpha[rr] != 1.f;
        m_r[rr] = m_new;
        mref[rr] = empty_row ? 0.f : m_new * kLog2e;
      }
      if (__any_sync(0xffffffffu, changed)) {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          l_r[rr] *= alpha[rr];
          if (MODE == MODE_ONLINE) {
#pragma unroll
            for (int n = 0; n < NT_O; ++n) {
              o[n][2 * rr] *= alpha[rr];
              o[n][2 * rr + 1] *= alpha[rr];
            }
          }
        }
      }
    } else {
      mref[0] = mfix_l2[0];
      mref[1] = mfix_l2[1];
    }
    // p = exp(s - m)
#pragma unroll
    for (int j = 0; j < NT_S; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[j][e] = fast_exp2(fmaf(sc[j][e], kLog2e, -mref[e >> 1]));
    }
    if (MODE != MODE_FIXED) {
#pragma unroll
      for (int j = 0; j < NT_S; ++j) {
        l_r[0] += sc[j][0] + sc[j][1];
        l_r[1] += sc[j][2] + sc[j][3];
      }
    }
    if (MODE != MODE_STATS && G > 0) {
      const int ntg = G >> 3;  // S n-tiles per mass group
      for (int gi = 0; gi < Cfg::TILE / G; ++gi) {
        float gs[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < NT_S; ++j) {
          if (j / ntg == gi) {
            gs[0] += sc[j][0] + sc[j][1];
            gs[1] += sc[j][2] + sc[j][3];
          }
        }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          gs[rr] += __shfl_xor_sync(0xffffffffu, gs[rr], 1);
          gs[rr] += __shfl_xor_sync(0xffffffffu, gs[rr], 2);
        }
        if (tq == 0) {
          const long long gidx = (t0 >> log2_group) + gi;
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int row = gr + 8 * rr;
            if (row < n_rep)
              mass_part[((long long)b * num_q_heads + qh0 + row) * mass_gstride + gidx] =
                  make_float2(gs[rr], MODE == MODE_ONLINE ? m_r[rr] : 0.f);
          }
        }
      }
    }
    bool wrote = (swm & 0xffu) != 0;
    if (MODE != MODE_STATS) {
      if (!all_valid) wrote |= zero_masked_rows<Cfg>(vbuf, vlo, vhi);
      const uint32_t vaddr = smem_u32(vbuf);
#pragma unroll
      for (int kt = 0; kt < Cfg::TILE / 16; ++kt) {
        uint32_t pa[4];
        pa[0] = Op::pack(sc[2 * kt][0], sc[2 * kt][1]);
        pa[1] = Op::pack(sc[2 * kt][2], sc[2 * kt][3]);
        pa[2] = Op::pack(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
        pa[3] = Op::pack(sc[2 * kt + 1][2], sc[2 * kt + 1][3]);
#pragma unroll
        for (int np = 0; np < NT_O / 2; ++np) {
          uint32_t b0, b1, b2, b3;
          const int c = 2 * np + (lane >> 4);
          const uint32_t voff =
              (c >> 3) * Cfg::PANEL_TILE_BYTES + (((lane >> 3) & 1) * 8 + l7) * 128 + (((c & 7) ^ l7) << 4);
          ldmatrix_x4_trans(vaddr + voff + kt * 16 * 128, b0, b1, b2, b3);
          Op::run(o[2 * np], pa, b0, b1);
          Op::run(o[2 * np + 1], pa, b2, b3);
        }
      }
    }
    release_stage(&empty[s], wrote);
  }
  if constexpr (MODE == MODE_SCORES) return;  // no partial state: the VALUES pass folds the tiles

  // per-row l from the quad's partial sums
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
  }
  named_bar_sync(1, Cfg::NCW * 32);
  float* mw = reinterpret_cast<float*>(stages);
  float* m_w = mw;
  float* l_w = mw + Cfg::NCW * kMaxRep;
  float* acc_w = mw + 2 * Cfg::NCW * kMaxRep;
  if (tq == 0) {
    m_w[warp * kMaxRep + gr] = m_r[0];
    m_w[warp * kMaxRep + gr + 8] = m_r[1];
    l_w[warp * kMaxRep + gr] = l_r[0];
    l_w[warp * kMaxRep + gr + 8] = l_r[1];
  }
  if (MODE != MODE_STATS) {
#pragma unroll
    for (int n = 0; n < NT_O; ++n) {
      const int col = 8 * n + 2 * tq;
      acc_w[(warp * kMaxRep + gr) * D + col] = o[n][0];
      acc_w[(warp * kMaxRep + gr) * D + col + 1] = o[n][1];
      acc_w[(warp * kMaxRep + gr + 8) * D + col] = o[n][2];
      acc_w[(warp * kMaxRep + gr + 8) * D + col + 1] = o[n][3];
    }
  }
  named_bar_sync(1, Cfg::NCW * 32);
  merge_and_store<D, MODE, Cfg::NCW>(p, mw, b, h, split);
}


// ------------------------------------------------------------------ tensor-core consumer, VALUES pass
// The tile's scores and each group's reference max (the reference's running max at that group's
// 64-token tile, or its final max) arrive by TMA in the auxiliary ring.  p = exp(s - M) against the
// group's M, rounded to the KV dtype before O += P V (streaming_attention.py:177-178, :346-347),
// l and the mass partials from the unrounded p.  M never decreases along a row and a warp visits
// its tiles in order, so the warp keeps O and l relative to the latest M and rescales them when M
// grows (at most once per group; G >= 16 puts every 16-token k-step in one group, and under the
// final-max rule all groups share M).  The split's (m, l, acc) then merge like ONLINE partials.
template <typename T, int D, int MODE>
__device__ void run_consumer_mma_values(const SplitParams& p, const TableCache& tc, uint8_t* stages, uint8_t* aux,
                                        uint64_t* full, uint64_t* empty, volatile int* infos, int b, int h,
                                        int tile0, int ntiles, const RowGeom& g, volatile int* abort_flag,
                                        int split) {
  using Cfg = TileCfg<T, D, MODE, BACKEND_MMA>;
  using Op = MmaOp<T>;
  static_assert(Cfg::PANEL_BYTES == 128, "mma path expects 128-byte panels");
  constexpr int NT_O = D / 8;
  constexpr int NT_S = Cfg::TILE / 8;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int gr = lane >> 2;
  const int tq = lane & 3;
  const int n_rep = p.n_rep;
  const int qh0 = h * n_rep;
  const int l7 = lane & 7;
  const int seg_rows = p.source == SRC_CONTIG ? Cfg::TILE : min(Cfg::TILE, p.tpb);
  const int* const valid = p.valid;
  const long long valid_stride = p.valid_stride;
  const uint64_t wait_limit = p.wait_limit_ns;
  int* const status = p.status;
  float2* const mass_part = p.mass_part;
  const int num_q_heads = p.num_q_heads;
  const int mass_gstride = p.mass_gstride;
  const int log2_group = p.log2_group;
  const int G = p.group_tokens;
  const uint64_t full_mask = Cfg::TILE == 64 ? ~0ull : ((1ull << Cfg::TILE) - 1ull);

  float o[NT_O][4];
#pragma unroll
  for (int n = 0; n < NT_O; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_r[2] = {neg_inf(), neg_inf()};
  float l_r[2] = {0.f, 0.f};

  for (int i = warp; i < ntiles; i += Cfg::NCW) {
    const int s = i % Cfg::STAGES;
    if (*abort_flag) break;
    uint32_t swm;
    if (!consumer_wait(wait_limit, status, &full[s], &empty[s], &infos[s], i / Cfg::STAGES, abort_flag, &swm)) break;
    const int t0 = (tile0 + i) * Cfg::TILE;
    uint8_t* vbuf = stages + s * Cfg::STAGE_BYTES;
    const float* s_sm = reinterpret_cast<const float*>(aux + s * Cfg::AUX_BYTES);  // [n_rep][TILE]
    const float* m_sm = s_sm + Cfg::AUX_S_BYTES / 4;                               // [n_rep][kRefSlots]
    if (swm & 0xffu) copy_sw_segments<Cfg, false, true>(p, tc, g, b, h, t0, swm & 0xffu, vbuf, vbuf);
    uint32_t vlo, vhi;
    tile_bits_fast<Cfg::TILE>(valid, valid_stride, b, t0, g, swm >> 8, seg_rows, vlo, vhi);
    bool wrote = (swm & 0xffu) != 0;
    if ((((uint64_t)vhi << 32) | vlo) != full_mask) wrote |= zero_masked_rows<Cfg>(vbuf, vlo, vhi);

    // scores of rows gr and gr + 8 (masked tokens hold -inf), columns 8j + 2tq + {0, 1}
    float sc[NT_S][4];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int row = gr + 8 * rr;
#pragma unroll
      for (int j = 0; j < NT_S; ++j) {
        float2 v = make_float2(neg_inf(), neg_inf());
        if (row < n_rep) v = *reinterpret_cast<const float2*>(s_sm + row * Cfg::TILE + 8 * j + 2 * tq);
        sc[j][2 * rr] = v.x;
        sc[j][2 * rr + 1] = v.y;
      }
    }
    float gsum[2] = {0.f, 0.f};  // this lane's sum of p over the current mass group
    const uint32_t vaddr = smem_u32(vbuf);
#pragma unroll
    for (int kt = 0; kt < Cfg::TILE / 16; ++kt) {
      const int gi = (16 * kt) / G;  // the k-step's group within the tile
      // the reference max changes only where a group starts: once a tile when groups are tiles
      if (kt == 0 || G < Cfg::TILE) {
        float alpha[2];
        bool changed = false;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int row = gr + 8 * rr;
          const float mn = row < n_rep ? m_sm[row * kRefSlots + gi] : neg_inf();
          alpha[rr] = 1.f;
          if (mn > m_r[rr]) {
            alpha[rr] = m_r[rr] == neg_inf() ? 0.f : fast_exp2((m_r[rr] - mn) * kLog2e);
            m_r[rr] = mn;
            changed = true;
          }
        }
        if (__any_sync(0xffffffffu, changed)) {
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            l_r[rr] *= alpha[rr];
#pragma unroll
            for (int n = 0; n < NT_O; ++n) {
              o[n][2 * rr] *= alpha[rr];
              o[n][2 * rr + 1] *= alpha[rr];
            }
          }
        }
      }
      float mref[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) mref[rr] = m_r[rr] == neg_inf() ? 0.f : m_r[rr] * kLog2e;
#pragma unroll
      for (int jj = 2 * kt; jj < 2 * kt + 2; ++jj) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[jj][e] = fast_exp2(fmaf(sc[jj][e], kLog2e, -mref[e >> 1]));
        l_r[0] += sc[jj][0] + sc[jj][1];
        l_r[1] += sc[jj][2] + sc[jj][3];
        gsum[0] += sc[jj][0] + sc[jj][1];
        gsum[1] += sc[jj][2] + sc[jj][3];
      }
      uint32_t pa[4];
      pa[0] = Op::pack(sc[2 * kt][0], sc[2 * kt][1]);
      pa[1] = Op::pack(sc[2 * kt][2], sc[2 * kt][3]);
      pa[2] = Op::pack(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
      pa[3] = Op::pack(sc[2 * kt + 1][2], sc[2 * kt + 1][3]);
#pragma unroll
      for (int np = 0; np < NT_O / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        const int c = 2 * np + (lane >> 4);
        const uint32_t voff =
            (c >> 3) * Cfg::PANEL_TILE_BYTES + (((lane >> 3) & 1) * 8 + l7) * 128 + (((c & 7) ^ l7) << 4);
        ldmatrix_x4_trans(vaddr + voff + kt * 16 * 128, b0, b1, b2, b3);
        Op::run(o[2 * np], pa, b0, b1);
        Op::run(o[2 * np + 1], pa, b2, b3);
      }
      // a mass group ends after this k-step: (sum p, the group's reference max)
      if (G > 0 && ((16 * (kt + 1)) % G == 0 || G < 16)) {
        // G == 8 (final-max rule only): this k-step holds two groups; split the sum by n-tile
        const int ngs = G < 16 ? 2 : 1;
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          if (q2 >= ngs) break;
          float gs[2];
          if (ngs == 2) {
            const int jj = 2 * kt + q2;
            gs[0] = sc[jj][0] + sc[jj][1];
            gs[1] = sc[jj][2] + sc[jj][3];
          } else {
            gs[0] = gsum[0];
            gs[1] = gsum[1];
          }
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            gs[rr] += __shfl_xor_sync(0xffffffffu, gs[rr], 1);
            gs[rr] += __shfl_xor_sync(0xffffffffu, gs[rr], 2);
          }
          const int gl = ngs == 2 ? 2 * kt + q2 : gi;  // group index within the tile
          if (tq == 0) {
            const long long gidx = (t0 >> log2_group) + gl;
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const int row = gr + 8 * rr;
              if (row < n_rep)
                mass_part[((long long)b * num_q_heads + qh0 + row) * mass_gstride + gidx] =
                    make_float2(gs[rr], m_sm[row * kRefSlots + gl]);
            }
          }
        }
        gsum[0] = gsum[1] = 0.f;
      }
    }
    release_stage(&empty[s], wrote);
  }

#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
  }
  named_bar_sync(1, Cfg::NCW * 32);
  float* mw = reinterpret_cast<float*>(stages);
  float* m_w = mw;
  float* l_w = mw + Cfg::NCW * kMaxRep;
  float* acc_w = mw + 2 * Cfg::NCW * kMaxRep;
  if (tq == 0) {
    m_w[warp * kMaxRep + gr] = m_r[0];
    m_w[warp * kMaxRep + gr + 8] = m_r[1];
    l_w[warp * kMaxRep + gr] = l_r[0];
    l_w[warp * kMaxRep + gr + 8] = l_r[1];
  }
#pragma unroll
  for (int n = 0; n < NT_O; ++n) {
    const int col = 8 * n + 2 * tq;
    acc_w[(warp * kMaxRep + gr) * D + col] = o[n][0];
    acc_w[(warp * kMaxRep + gr) * D + col + 1] = o[n][1];
    acc_w[(warp * kMaxRep + gr + 8) * D + col] = o[n][2];
    acc_w[(warp * kMaxRep + gr + 8) * D + col + 1] = o[n][3];
  }
  named_bar_sync(1, Cfg::NCW * 32);
  merge_and_store<D, MODE_ONLINE, Cfg::NCW>(p, mw, b, h, split);
}

// The values pass with the mma operands' roles swapped, for at most 8 query heads per KV head:
// O^T[d][h] += V^T[d][t] . P^T[t][h].  V is the m16 operand (ldmatrix.trans of the token-major
// tile) and the heads fill the n8 side, so a k-step of 16 tokens takes D/16 mma instead of D/8, each
// lane forms p for one head (row gr) instead of two, and the accumulator is D/4 floats per lane.
// The arithmetic is that of run_consumer_mma_values: p against its group's reference max, rounded
// to the KV dtype, O and l rescaled when the reference max grows.  A lane keeps two views of the
// running max: m_p for head gr (its p and l) and m_c for heads 2tq, 2tq+1 (its accumulator
// columns); both follow the same reference maxima, so they agree head by head.
template <typename T, int D, int MODE>
__device__ void run_consumer_mma_values_t(const SplitParams& p, const TableCache& tc, uint8_t* stages, uint8_t* aux,
                                          uint64_t* full, uint64_t* empty, volatile int* infos, int b, int h,
                                          int tile0, int ntiles, const RowGeom& g, volatile int* abort_flag,
                                          int split) {
  using Cfg = TileCfg<T, D, MODE, BACKEND_MMA>;
  using Op = MmaOp<T>;
  static_assert(Cfg::PANEL_BYTES == 128, "mma path expects 128-byte panels");
  static_assert(Cfg::AUX_REP <= 8, "one n8 tile holds the heads");
  constexpr int MT = D / 16;  // m16 tiles over head_dim
  constexpr int NT_S = Cfg::TILE / 8;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int gr = lane >> 2;
  const int tq = lane & 3;
  const int n_rep = p.n_rep;
  const int qh0 = h * n_rep;
  const int l7 = lane & 7;
  const int db = (lane >> 3) & 1;  // ldmatrix: which 8 head_dim columns this lane's row address covers
  const int tb = (lane >> 4) & 1;  // ... and which 8 tokens
  const bool row_ok = gr < n_rep;  // head gr exists
  const int seg_rows = p.source == SRC_CONTIG ? Cfg::TILE : min(Cfg::TILE, p.tpb);
  const int* const valid = p.valid;
  const long long valid_stride = p.valid_stride;
  const uint64_t wait_limit = p.wait_limit_ns;
  int* const status = p.status;
  float2* const mass_part = p.mass_part;
  const int num_q_heads = p.num_q_heads;
  const int mass_gstride = p.mass_gstride;
  const int log2_group = p.log2_group;
  const int G = p.group_tokens;
  const uint64_t full_mask = Cfg::TILE == 64 ? ~0ull : ((1ull << Cfg::TILE) - 1ull);

  float o[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.f;
  float m_p = neg_inf(), l_p = 0.f;
  float m_c[2] = {neg_inf(), neg_inf()};

  for (int i = warp; i < ntiles; i += Cfg::NCW) {
    const int s = i % Cfg::STAGES;
    if (*abort_flag) break;
    uint32_t swm;
    if (!consumer_wait(wait_limit, status, &full[s], &empty[s], &infos[s], i / Cfg::STAGES, abort_flag, &swm)) break;
    const int t0 = (tile0 + i) * Cfg::TILE;
    uint8_t* vbuf = stages + s * Cfg::STAGE_BYTES;
    const float* s_sm = reinterpret_cast<const float*>(aux + s * Cfg::AUX_BYTES);  // [n_rep][TILE]
    const float* m_sm = s_sm + Cfg::AUX_S_BYTES / 4;                               // [n_rep][kRefSlots]
    if (swm & 0xffu) copy_sw_segments<Cfg, false, true>(p, tc, g, b, h, t0, swm & 0xffu, vbuf, vbuf);
    uint32_t vlo, vhi;
    tile_bits_fast<Cfg::TILE>(valid, valid_stride, b, t0, g, swm >> 8, seg_rows, vlo, vhi);
    bool wrote = (swm & 0xffu) != 0;
    if ((((uint64_t)vhi << 32) | vlo) != full_mask) wrote |= zero_masked_rows<Cfg>(vbuf, vlo, vhi);

    // scores of head gr (masked tokens hold -inf), tokens 8j + 2tq + {0, 1}
    float sc[NT_S][2];
#pragma unroll
    for (int j = 0; j < NT_S; ++j) {
      float2 v = make_float2(neg_inf(), neg_inf());
      if (row_ok) v = *reinterpret_cast<const float2*>(s_sm + gr * Cfg::TILE + 8 * j + 2 * tq);
      sc[j][0] = v.x;
      sc[j][1] = v.y;
    }
    float gsum = 0.f;  // this lane's sum of p over the current mass group
    const uint32_t vaddr = smem_u32(vbuf);
#pragma unroll
    for (int kt = 0; kt < Cfg::TILE / 16; ++kt) {
      const int gi = (16 * kt) / G;  // the k-step's group within the tile
      // the reference max changes only where a group starts: once a tile when groups are tiles
      // (blocks of at least 64 tokens), so the check runs at the first k-step only
      if (kt == 0 || G < Cfg::TILE) {
        const float mn = row_ok ? m_sm[gr * kRefSlots + gi] : neg_inf();
        if (mn > m_p) {
          l_p *= m_p == neg_inf() ? 0.f : fast_exp2((m_p - mn) * kLog2e);
          m_p = mn;
        }
        float alpha[2];
        bool changed = false;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int head = 2 * tq + c;
          const float mc = head < n_rep ? m_sm[head * kRefSlots + gi] : neg_inf();
          alpha[c] = 1.f;
          if (mc > m_c[c]) {
            alpha[c] = m_c[c] == neg_inf() ? 0.f : fast_exp2((m_c[c] - mc) * kLog2e);
            m_c[c] = mc;
            changed = true;
          }
        }
        if (__any_sync(0xffffffffu, changed)) {
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            o[m][0] *= alpha[0];
            o[m][1] *= alpha[1];
            o[m][2] *= alpha[0];
            o[m][3] *= alpha[1];
          }
        }
      }
      const float mref = m_p == neg_inf() ? 0.f : m_p * kLog2e;
#pragma unroll
      for (int jj = 2 * kt; jj < 2 * kt + 2; ++jj) {
        sc[jj][0] = fast_exp2(fmaf(sc[jj][0], kLog2e, -mref));
        sc[jj][1] = fast_exp2(fmaf(sc[jj][1], kLog2e, -mref));
        l_p += sc[jj][0] + sc[jj][1];
        gsum += sc[jj][0] + sc[jj][1];
      }
      // P^T as the col-major B operand: tokens 2tq + {0, 1} and 2tq + 8 + {0, 1} of head gr
      const uint32_t b0 = Op::pack(sc[2 * kt][0], sc[2 * kt][1]);
      const uint32_t b1 = Op::pack(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        uint32_t a[4];
        const int c = 2 * m + db;  // 16-byte chunk of the token row: head_dim 8c .. 8c + 7
        const uint32_t voff = (c >> 3) * Cfg::PANEL_TILE_BYTES + (tb * 8 + l7) * 128 + (((c & 7) ^ l7) << 4);
        ldmatrix_x4_trans(vaddr + voff + kt * 16 * 128, a[0], a[1], a[2], a[3]);
        Op::run(o[m], a, b0, b1);
      }
      // a mass group ends after this k-step: (sum p, the group's reference max)
      if (G > 0 && ((16 * (kt + 1)) % G == 0 || G < 16)) {
        // G == 8 (final-max rule only): this k-step holds two groups; split the sum by token half
        const int ngs = G < 16 ? 2 : 1;
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          if (q2 >= ngs) break;
          float gs = ngs == 2 ? sc[2 * kt + q2][0] + sc[2 * kt + q2][1] : gsum;
          gs += __shfl_xor_sync(0xffffffffu, gs, 1);
          gs += __shfl_xor_sync(0xffffffffu, gs, 2);
          const int gl = ngs == 2 ? 2 * kt + q2 : gi;  // group index within the tile
          if (tq == 0 && row_ok)
            mass_part[((long long)b * num_q_heads + qh0 + gr) * mass_gstride + (t0 >> log2_group) + gl] =
                make_float2(gs, m_sm[gr * kRefSlots + gl]);
        }
        gsum = 0.f;
      }
    }
    release_stage(&empty[s], wrote);
  }

  l_p += __shfl_xor_sync(0xffffffffu, l_p, 1);
  l_p += __shfl_xor_sync(0xffffffffu, l_p, 2);
  named_bar_sync(1, Cfg::NCW * 32);
  float* mw = reinterpret_cast<float*>(stages);
  float* m_w = mw;
  float* l_w = mw + Cfg::NCW * kMaxRep;
  float* acc_w = mw + 2 * Cfg::NCW * kMaxRep;
  if (tq == 0) {
    m_w[warp * kMaxRep + gr] = m_p;
    l_w[warp * kMaxRep + gr] = l_p;
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const int d = 16 * m + gr;
    acc_w[(warp * kMaxRep + 2 * tq) * D + d] = o[m][0];
    acc_w[(warp * kMaxRep + 2 * tq + 1) * D + d] = o[m][1];
    acc_w[(warp * kMaxRep + 2 * tq) * D + d + 8] = o[m][2];
    acc_w[(warp * kMaxRep + 2 * tq + 1) * D + d + 8] = o[m][3];
  }
  named_bar_sync(1, Cfg::NCW * 32);
  merge_and_store<D, MODE_ONLINE, Cfg::NCW>(p, mw, b, h, split);
}

// ------------------------------------------------------------------ CUDA-core consumer
// Lane <-> token for Q.K (q broadcast from shared memory), lane <-> head_dim
// column for P.V (p broadcast from shared memory); fp32 throughout.
template <typename T, int D, int MODE>
__device__ void run_consumer_fma(const SplitParams& p, const TableCache& tc, uint8_t* stages, uint64_t* full,
                                 uint64_t* empty, volatile int* infos, int b, int h, int tile0, int ntiles,
                                 const RowGeom& g, volatile int* abort_flag, int split, const float* q_sm,
                                 float* p_sm_all) {
  using Cfg = TileCfg<T, D, MODE, BACKEND_FMA>;
  constexpr int TILE = Cfg::TILE;
  constexpr int TPL = TILE > 32 ? TILE / 32 : 1;   // tokens per lane in Q.K
  constexpr int EPC = 16 / sizeof(T);              // elements per 16-byte chunk
  constexpr int DPL = D >= 32 ? D / 32 : 1;        // head_dim columns per lane in P.V
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int n_rep = p.n_rep;
  const int qh0 = h * n_rep;
  float* p_sm = p_sm_all + warp * TILE * kMaxRep;
  const int seg_rows = p.source == SRC_CONTIG ? Cfg::TILE : min(Cfg::TILE, p.tpb);
  const int* const valid = p.valid;
  const long long valid_stride = p.valid_stride;
  const uint64_t wait_limit = p.wait_limit_ns;
  int* const status = p.status;
  const float scale = p.scale;
  const float softcap = p.softcap;
  float2* const mass_part = p.mass_part;
  const int num_q_heads = p.num_q_heads;
  const int mass_gstride = p.mass_gstride;
  const int log2_group = p.log2_group;

  float mfix[kMaxRep];
  if (MODE == MODE_FIXED) {
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r)
      mfix[r] = r < n_rep ? p.m_fixed[(long long)b * p.num_q_heads + qh0 + r] * kLog2e : 0.f;
  }
  float acc[kMaxRep][DPL];
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r)
#pragma unroll
    for (int k = 0; k < DPL; ++k) acc[r][k] = 0.f;
  float m_r[kMaxRep], l_r[kMaxRep];  // l_r: this lane's partial sum
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r) {
    m_r[r] = neg_inf();
    l_r[r] = 0.f;
  }
  const int G = p.group_tokens;

  for (int i = warp; i < ntiles; i += Cfg::NCW) {
    const int s = i % Cfg::STAGES;
    if (*abort_flag) break;
    uint32_t swm;
    if (!consumer_wait(wait_limit, status, &full[s], &empty[s], &infos[s], i / Cfg::STAGES, abort_flag, &swm)) break;
    const int t0 = (tile0 + i) * TILE;
    uint8_t* kbuf = stages + s * Cfg::STAGE_BYTES;
    uint8_t* vbuf = kbuf + Cfg::TENSOR_BYTES;
    if (swm & 0xffu) copy_sw_segments<Cfg, true, !Cfg::KONLY>(p, tc, g, b, h, t0, swm & 0xffu, kbuf, vbuf);
    uint32_t vlo, vhi;
    tile_bits_fast<TILE>(valid, valid_stride, b, t0, g, swm >> 8, seg_rows, vlo, vhi);
    const uint32_t kaddr = smem_u32(kbuf);

    float sc[TPL][kMaxRep];
#pragma unroll
    for (int u = 0; u < TPL; ++u) {
      const int t = lane + 32 * u;
#pragma unroll
      for (int r = 0; r < kMaxRep; ++r) sc[u][r] = 0.f;
      if (t < TILE) {
#pragma unroll 2
        for (int c = 0; c < Cfg::CPR; ++c) {
          float kf[EPC];
          unpack16(ld_shared_16(chunk_addr<Cfg>(kaddr, t, c)), kf, T());
#pragma unroll
          for (int r = 0; r < kMaxRep; ++r) {
            if (r < n_rep) {
              const float* qr = q_sm + r * D + c * EPC;
#pragma unroll
              for (int e = 0; e < EPC; ++e) sc[u][r] = fmaf(qr[e], kf[e], sc[u][r]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kMaxRep; ++r) {
        const float x = apply_score(sc[u][r], scale, softcap);
        sc[u][r] = (t < TILE && bit_of(vlo, vhi, t)) ? x : neg_inf();
      }
    }
    if constexpr (MODE == MODE_SCORES) {
      // the masked scores of the tile (lane <-> token), and the max of each group_tokens group
      float* const srow = p.scores + (long long)(b * num_q_heads + qh0) * p.s_stride + t0;
      const uint64_t keep = l2_policy_evict_last();  // read back by the values pass of this layer
#pragma unroll
      for (int u = 0; u < TPL; ++u) {
        const int t = lane + 32 * u;
        if (t < TILE) {
#pragma unroll
          for (int r = 0; r < kMaxRep; ++r)
            if (r < n_rep) st_global_f1_hint(srow + (long long)r * p.s_stride + t, sc[u][r], keep);
        }
      }
      for (int gi = 0; gi < TILE / G; ++gi) {
        for (int r = 0; r < n_rep; ++r) {
          float v = neg_inf();
#pragma unroll
          for (int u = 0; u < TPL; ++u) {
            const int t = lane + 32 * u;
            if (t < TILE && t / G == gi) v = fmaxf(v, sc[u][r]);
          }
          v = warp_max(v);
          if (lane == 0) p.gmax[((long long)b * num_q_heads + qh0 + r) * mass_gstride + (t0 >> log2_group) + gi] = v;
        }
      }
      release_stage(&empty[s], (swm & 0xffu) != 0);
      continue;
    }
    float mref[kMaxRep];
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) {
      if (MODE != MODE_FIXED) {
        float mx = sc[0][r];
#pragma unroll
        for (int u = 1; u < TPL; ++u) mx = fmaxf(mx, sc[u][r]);
        mx = warp_max(mx);
        const float m_new = fmaxf(m_r[r], mx);
        const bool empty_row = m_new == neg_inf();
        const float alpha = empty_row ? 0.f : fast_exp2((m_r[r] - m_new) * kLog2e);
        l_r[r] *= alpha;
        if (MODE == MODE_ONLINE) {
#pragma unroll
          for (int k = 0; k < DPL; ++k) acc[r][k] *= alpha;
        }
        m_r[r] = m_new;
        mref[r] = empty_row ? 0.f : m_new * kLog2e;
      } else {
        mref[r] = mfix[r];
      }
    }
#pragma unroll
    for (int u = 0; u < TPL; ++u) {
#pragma unroll
      for (int r = 0; r < kMaxRep; ++r) {
        sc[u][r] = fast_exp2(fmaf(sc[u][r], kLog2e, -mref[r]));
        if (MODE != MODE_FIXED) l_r[r] += sc[u][r];
      }
    }
    if (MODE != MODE_STATS && G > 0) {
      // mass partials per group of G tokens (G >= 16, power of two)
      const int ngroups = TILE / G;
      for (int gi = 0; gi < ngroups; ++gi) {
#pragma unroll
        for (int r = 0; r < kMaxRep; ++r) {
          if (r >= n_rep) continue;
          float v = 0.f;
#pragma unroll
          for (int u = 0; u < TPL; ++u) {
            const int t = lane + 32 * u;
            if (t < TILE && t / G == gi) v += sc[u][r];
          }
          v = warp_sum(v);
          if (lane == 0) {
            const long long gidx = (t0 >> log2_group) + gi;
            mass_part[((long long)b * num_q_heads + qh0 + r) * mass_gstride + gidx] =
                make_float2(v, MODE == MODE_ONLINE ? m_r[r] : 0.f);
          }
        }
      }
    }
    bool wrote = (swm & 0xffu) != 0;
    if (MODE != MODE_STATS) {
#pragma unroll
      for (int u = 0; u < TPL; ++u) {
        const int t = lane + 32 * u;
        if (t < TILE) {
#pragma unroll
          for (int r = 0; r < kMaxRep; ++r) {
            // against the fixed (final) max, p enters P.V rounded to the KV dtype, as the
            // reference's accumulate and fold kernels round it (streaming_attention.py:346-347,
            // :427-428); l and the mass partials above took the unrounded p
            p_sm[t * kMaxRep + r] = MODE == MODE_FIXED ? to_f32(T(sc[u][r])) : sc[u][r];
          }
        }
      }
      wrote |= zero_masked_rows<Cfg>(vbuf, vlo, vhi);
      __syncwarp();
      const uint32_t vaddr = smem_u32(vbuf);
      for (int t = 0; t < TILE; ++t) {
        if (!bit_of(vlo, vhi, t)) continue;
        float pr[kMaxRep];
#pragma unroll
        for (int r4 = 0; r4 < kMaxRep; r4 += 4) {
          const float4 v4 = *reinterpret_cast<const float4*>(p_sm + t * kMaxRep + r4);
          pr[r4] = v4.x;
          pr[r4 + 1] = v4.y;
          pr[r4 + 2] = v4.z;
          pr[r4 + 3] = v4.w;
        }
#pragma unroll
        for (int k = 0; k < DPL; ++k) {
          const int d = lane + 32 * k;
          if (d < D) {
            const int byte = d * (int)sizeof(T);
            const uint32_t a = chunk_addr<Cfg>(vaddr, t, byte >> 4) + (byte & 15);
            float vv;
            if (sizeof(T) == 4) {
              asm volatile("ld.shared.f32 %0, [%1];" : "=f"(vv) : "r"(a));
            } else {
              unsigned short raw;
              asm volatile("ld.shared.u16 %0, [%1];" : "=h"(raw) : "r"(a));
              if (sizeof(T) == 2 && std::is_same<T, __half>::value)
                vv = __half2float(__ushort_as_half(raw));
              else
                vv = __uint_as_float(((uint32_t)raw) << 16);
            }
#pragma unroll
            for (int r = 0; r < kMaxRep; ++r) acc[r][k] = fmaf(pr[r], vv, acc[r][k]);
          }
        }
      }
    }
    release_stage(&empty[s], wrote);
  }
  if constexpr (MODE == MODE_SCORES) return;

#pragma unroll
  for (int r = 0; r < kMaxRep; ++r) l_r[r] = warp_sum(l_r[r]);
  named_bar_sync(1, Cfg::NCW * 32);
  float* mw = reinterpret_cast<float*>(stages);
  float* m_w = mw;
  float* l_w = mw + Cfg::NCW * kMaxRep;
  float* acc_w = mw + 2 * Cfg::NCW * kMaxRep;
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) {
      m_w[warp * kMaxRep + r] = m_r[r];
      l_w[warp * kMaxRep + r] = l_r[r];
    }
  }
  if (MODE != MODE_STATS) {
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r)
#pragma unroll
      for (int k = 0; k < DPL; ++k) {
        const int d = lane + 32 * k;
        if (d < D) acc_w[(warp * kMaxRep + r) * D + d] = acc[r][k];
      }
  }
  named_bar_sync(1, Cfg::NCW * 32);
  merge_and_store<D, MODE, Cfg::NCW>(p, mw, b, h, split);
}


// ------------------------------------------------------------------ CUDA-core consumer, VALUES pass
// As the tensor-core VALUES pass, lane <-> token: p = exp(s - M) against its group's reference max,
// rounded to the KV dtype; the warp keeps O and l relative to the tile's last (largest) M, so a
// token of an earlier group of the tile enters P.V as its rounded p times exp(M_group - M), the
// scale applied after the rounding as the reference's later rescale of its accumulator is.
template <typename T, int D, int MODE>
__device__ void run_consumer_fma_values(const SplitParams& p, const TableCache& tc, uint8_t* stages, uint8_t* aux,
                                        uint64_t* full, uint64_t* empty, volatile int* infos, int b, int h,
                                        int tile0, int ntiles, const RowGeom& g, volatile int* abort_flag,
                                        int split, float* p_sm_all) {
  using Cfg = TileCfg<T, D, MODE, BACKEND_FMA>;
  constexpr int TILE = Cfg::TILE;
  constexpr int TPL = TILE > 32 ? TILE / 32 : 1;
  constexpr int DPL = D >= 32 ? D / 32 : 1;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int n_rep = p.n_rep;
  const int qh0 = h * n_rep;
  float* p_sm = p_sm_all + warp * TILE * kMaxRep;
  const int seg_rows = p.source == SRC_CONTIG ? TILE : min(TILE, p.tpb);
  const uint64_t wait_limit = p.wait_limit_ns;
  int* const status = p.status;
  float2* const mass_part = p.mass_part;
  const int num_q_heads = p.num_q_heads;
  const int mass_gstride = p.mass_gstride;
  const int log2_group = p.log2_group;
  const int G = p.group_tokens;
  const int ngroups = TILE / G;

  float acc[kMaxRep][DPL];
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r)
#pragma unroll
    for (int k = 0; k < DPL; ++k) acc[r][k] = 0.f;
  float m_r[kMaxRep], l_r[kMaxRep];
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r) {
    m_r[r] = neg_inf();
    l_r[r] = 0.f;
  }

  for (int i = warp; i < ntiles; i += Cfg::NCW) {
    const int s = i % Cfg::STAGES;
    if (*abort_flag) break;
    uint32_t swm;
    if (!consumer_wait(wait_limit, status, &full[s], &empty[s], &infos[s], i / Cfg::STAGES, abort_flag, &swm)) break;
    const int t0 = (tile0 + i) * TILE;
    uint8_t* vbuf = stages + s * Cfg::STAGE_BYTES;
    const float* s_sm = reinterpret_cast<const float*>(aux + s * Cfg::AUX_BYTES);  // [n_rep][TILE]
    const float* m_sm = s_sm + Cfg::AUX_S_BYTES / 4;                               // [n_rep][kRefSlots]
    if (swm & 0xffu) copy_sw_segments<Cfg, false, true>(p, tc, g, b, h, t0, swm & 0xffu, vbuf, vbuf);
    uint32_t vlo, vhi;
    tile_bits_fast<TILE>(p.valid, p.valid_stride, b, t0, g, swm >> 8, seg_rows, vlo, vhi);
    bool wrote = (swm & 0xffu) != 0;
    wrote |= zero_masked_rows<Cfg>(vbuf, vlo, vhi);
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) {
      if (r >= n_rep) continue;
      const float mt = m_sm[r * kRefSlots + ngroups - 1];
      if (mt > m_r[r]) {
        const float alpha = m_r[r] == neg_inf() ? 0.f : fast_exp2((m_r[r] - mt) * kLog2e);
        l_r[r] *= alpha;
#pragma unroll
        for (int k = 0; k < DPL; ++k) acc[r][k] *= alpha;
        m_r[r] = mt;
      }
    }
    float pe[TPL][kMaxRep];  // unrounded p against the token's group max
#pragma unroll
    for (int u = 0; u < TPL; ++u) {
      const int t = lane + 32 * u;
#pragma unroll
      for (int r = 0; r < kMaxRep; ++r) {
        float e = 0.f, pr = 0.f;
        if (t < TILE && r < n_rep) {
          const float mg = m_sm[r * kRefSlots + t / G];
          if (mg != neg_inf()) {
            e = fast_exp2(fmaf(s_sm[r * TILE + t], kLog2e, -mg * kLog2e));
            const float w = fast_exp2((mg - m_r[r]) * kLog2e);
            pr = to_f32(T(e)) * w;
            l_r[r] += e * w;
          }
        }
        pe[u][r] = e;
        if (t < TILE) p_sm[t * kMaxRep + r] = pr;
      }
    }
    for (int gi = 0; gi < ngroups; ++gi) {
      for (int r = 0; r < n_rep; ++r) {
        float v = 0.f;
#pragma unroll
        for (int u = 0; u < TPL; ++u) {
          const int t = lane + 32 * u;
          if (t < TILE && t / G == gi) v += pe[u][r];
        }
        v = warp_sum(v);
        if (lane == 0)
          mass_part[((long long)b * num_q_heads + qh0 + r) * mass_gstride + (t0 >> log2_group) + gi] =
              make_float2(v, m_sm[r * kRefSlots + gi]);
      }
    }
    __syncwarp();
    const uint32_t vaddr = smem_u32(vbuf);
    for (int t = 0; t < TILE; ++t) {
      if (!bit_of(vlo, vhi, t)) continue;
      float prr[kMaxRep];
#pragma unroll
      for (int r4 = 0; r4 < kMaxRep; r4 += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(p_sm + t * kMaxRep + r4);
        prr[r4] = v4.x;
        prr[r4 + 1] = v4.y;
        prr[r4 + 2] = v4.z;
        prr[r4 + 3] = v4.w;
      }
#pragma unroll
      for (int k = 0; k < DPL; ++k) {
        const int d = lane + 32 * k;
        if (d < D) {
          const int byte = d * (int)sizeof(T);
          const uint32_t a = chunk_addr<Cfg>(vaddr, t, byte >> 4) + (byte & 15);
          unsigned short raw;
          asm volatile("ld.shared.u16 %0, [%1];" : "=h"(raw) : "r"(a));
          const float vv = std::is_same<T, __half>::value ? __half2float(__ushort_as_half(raw))
                                                          : __uint_as_float(((uint32_t)raw) << 16);
#pragma unroll
          for (int r = 0; r < kMaxRep; ++r) acc[r][k] = fmaf(prr[r], vv, acc[r][k]);
        }
      }
    }
    __syncwarp();  // p_sm is rewritten by this warp's next tile
    release_stage(&empty[s], wrote);
  }

#pragma unroll
  for (int r = 0; r < kMaxRep; ++r) l_r[r] = warp_sum(l_r[r]);
  named_bar_sync(1, Cfg::NCW * 32);
  float* mw = reinterpret_cast<float*>(stages);
  float* m_w = mw;
  float* l_w = mw + Cfg::NCW * kMaxRep;
  float* acc_w = mw + 2 * Cfg::NCW * kMaxRep;
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) {
      m_w[warp * kMaxRep + r] = m_r[r];
      l_w[warp * kMaxRep + r] = l_r[r];
    }
  }
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r)
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      const int d = lane + 32 * k;
      if (d < D) acc_w[(warp * kMaxRep + r) * D + d] = acc[r][k];
    }
  named_bar_sync(1, Cfg::NCW * 32);
  merge_and_store<D, MODE_ONLINE, Cfg::NCW>(p, mw, b, h, split);
}

// ------------------------------------------------------------------ kernel
template <typename T, int D, int MODE, int BACKEND>
struct SplitSmem {
  using Cfg = TileCfg<T, D, MODE, BACKEND>;
  static constexpr int AUX_OFF = Cfg::STAGE_AREA;  // VALUES: score / reference-max ring (128-byte stages)
  static constexpr int BAR_OFF = AUX_OFF + Cfg::STAGES * Cfg::AUX_BYTES;
  static constexpr int FLAG_OFF = BAR_OFF + 2 * Cfg::STAGES * 8;
  static constexpr int INFO_OFF = FLAG_OFF + 16;
  static constexpr int TBL_OFF = (INFO_OFF + 4 * Cfg::STAGES + 15) / 16 * 16;
  static constexpr int Q_OFF = TBL_OFF + kTableCache * 4;
  static constexpr int P_OFF = Q_OFF + Cfg::Q_BYTES;
  static constexpr int TOTAL = P_OFF + Cfg::P_BYTES + 1024;  // + slack for 1024-byte alignment
  static_assert(TOTAL <= 227 * 1024, "shared memory budget");
};

template <typename T, int D, int MODE, int BACKEND>
__global__ void __launch_bounds__(TileCfg<T, D, MODE, BACKEND>::THREADS, TileCfg<T, D, MODE, BACKEND>::MIN_BLOCKS)
    split_kernel(const __grid_constant__ SplitParams p, const __grid_constant__ CUtensorMap mapk,
                 const __grid_constant__ CUtensorMap mapv, const __grid_constant__ CUtensorMap maps,
                 const __grid_constant__ CUtensorMap mapm) {
  using Cfg = TileCfg<T, D, MODE, BACKEND>;
  using L = SplitSmem<T, D, MODE, BACKEND>;
  const int split = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  // Launched programmatically serialized (paged op): the previous kernel in the stream may still
  // be reading the partials this grid overwrites, or writing q / the pools; wait for it first,
  // then let the combine/mass kernel that follows be scheduled behind this grid.
  pdl_wait();
  pdl_launch_dependents();
  if (p.active && p.active[b] == 0) return;
  if (Cfg::VONLY && p.n_rep > Cfg::AUX_REP) {  // the host picks the variant; never overrun its score ring
    if (blockIdx.x == 0 && h == 0 && threadIdx.x == 0) atomicExch(p.status, kStatusBadBlock);
    return;
  }
  bool clamped = false;
  const RowGeom g = row_geom(p.geom, b, &clamped);
  if (clamped && split == 0 && h == 0 && threadIdx.x == 0) atomicExch(p.status, kStatusBadBlock);
  int t_begin, t_end, nsplit;
  geom_tiles(g, Cfg::LOG2_TILE, p.tiles_per_split, t_begin, t_end, nsplit);
  if (split >= nsplit) return;
  const int tile0 = t_begin + split * p.tiles_per_split;
  const int ntiles = min(p.tiles_per_split, t_end - tile0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* aux = smem + L::AUX_OFF;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + Cfg::STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::FLAG_OFF);
  volatile int* infos = reinterpret_cast<volatile int*>(smem + L::INFO_OFF);
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      infos[s] = 0;
    }
    *abort_flag = 0;
    mbar_fence_init();
    if ((p.source == SRC_CONTIG && !Cfg::VONLY) || (p.source == SRC_PAGED && p.dev_pool != nullptr))
      tma_prefetch_desc(&mapk);
    if ((p.source == SRC_CONTIG && !Cfg::KONLY) || (p.source == SRC_PAGED && p.stage_pool != nullptr))
      tma_prefetch_desc(&mapv);
    if (Cfg::VONLY) {
      tma_prefetch_desc(&maps);
      tma_prefetch_desc(&mapm);
    }
  }
  float* q_sm = reinterpret_cast<float*>(smem + L::Q_OFF);
  T* q_smem_t = reinterpret_cast<T*>(smem + L::Q_OFF);
  float* p_sm = reinterpret_cast<float*>(smem + L::P_OFF);
  int* tbl = reinterpret_cast<int*>(smem + L::TBL_OFF);
  TableCache tc{tbl, 0, 0};
  if (p.source == SRC_PAGED) {
    const int blk0 = (tile0 * Cfg::TILE) >> p.log2_tpb;
    int blk1 = ((tile0 + ntiles) * Cfg::TILE + p.tpb - 1) >> p.log2_tpb;
    blk1 = min(blk1, g.nb);
    tc.blk0 = blk0;
    tc.n = max(0, min(blk1 - blk0, kTableCache));
    for (int i = threadIdx.x; i < tc.n; i += Cfg::THREADS) tbl[i] = p.block_table[(long long)b * p.max_blocks + blk0 + i];
  }
  if (warp < Cfg::NCW && !Cfg::VONLY) {
    const long long qbase = ((long long)b * p.num_q_heads + (long long)h * p.n_rep) * D;
    for (int idx = threadIdx.x; idx < kMaxRep * D; idx += Cfg::NCW * 32) {
      const int r = idx / D;
      const float v = r < p.n_rep ? load_any(p.q, qbase + idx, p.q_dtype) : 0.f;
      if constexpr (BACKEND == BACKEND_FMA) {
        q_sm[idx] = v;
      } else {
        // 128-byte swizzled, 16 rows per 128-byte panel (the consumers' ldmatrix layout)
        const int col = idx % D;
        const int byte = col * (int)sizeof(T);
        const int chunk = byte >> 4;
        const int off = (chunk >> 3) * 2048 + r * 128 + ((((chunk & 7) ^ (r & 7)) << 4) | (byte & 15));
        *reinterpret_cast<T*>(reinterpret_cast<uint8_t*>(q_smem_t) + off) = T(v);
      }
    }
  }
  __syncthreads();

  if (warp >= Cfg::NCW) {
    run_producer<Cfg, MODE>(p, tc, &mapk, &mapv, &maps, &mapm, stages, aux, full, empty, infos, b, h, tile0, ntiles,
                            g, abort_flag, warp - Cfg::NCW);
  } else {
    if constexpr (BACKEND == BACKEND_MMA && Cfg::SWAPPED) {
      run_consumer_mma_values_t<T, D, MODE>(p, tc, stages, aux, full, empty, infos, b, h, tile0, ntiles, g, abort_flag,
                                            split);
    } else if constexpr (BACKEND == BACKEND_MMA && Cfg::VONLY) {
      run_consumer_mma_values<T, D, MODE>(p, tc, stages, aux, full, empty, infos, b, h, tile0, ntiles, g, abort_flag,
                                    split);
    } else if constexpr (BACKEND == BACKEND_MMA) {
      run_consumer_mma<T, D, MODE>(p, tc, stages, full, empty, infos, b, h, tile0, ntiles, g, abort_flag, split,
                                   q_smem_t);
    } else if constexpr (Cfg::VONLY) {
      run_consumer_fma_values<T, D, MODE>(p, tc, stages, aux, full, empty, infos, b, h, tile0, ntiles, g, abort_flag, split,
                                    p_sm);
    } else {
      run_consumer_fma<T, D, MODE>(p, tc, stages, full, empty, infos, b, h, tile0, ntiles, g, abort_flag, split,
                                   q_sm, p_sm);
    }
  }
}

// Host-side description of one instantiation.
struct SplitKernelInfo {
  const void* fn;
  int threads;
  int tile;
  int smem_bytes;
  int stages;
  int panel_elts;
  int panel_bytes;
};

template <typename T, int D, int MODE, int BACKEND>
SplitKernelInfo split_kernel_info() {
  using Cfg = TileCfg<T, D, MODE, BACKEND>;
  using L = SplitSmem<T, D, MODE, BACKEND>;
  SplitKernelInfo k;
  k.fn = reinterpret_cast<const void*>(&split_kernel<T, D, MODE, BACKEND>);
  k.threads = Cfg::THREADS;
  k.tile = Cfg::TILE;
  k.smem_bytes = L::TOTAL;
  k.stages = Cfg::STAGES;
  k.panel_elts = Cfg::PANEL_ELTS;
  k.panel_bytes = Cfg::PANEL_BYTES;
  return k;
}

// Lookup: returns false when the (dtype, D, mode, backend) combination is not built.
bool lookup_split_kernel(int kv_dtype, int head_dim, int mode, int backend, SplitKernelInfo* out);

}  // namespace pager
