/*
 * pager_b200.h -- C ABI of the B200 decode-attention library (libpager_b200.so).
 *
 * Drop-in boundary for rust-llm-pager's streaming decode-attention hot path.
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), returns an int status (PAGER_OK == 0) and never throws.
 * The message of the last failing call on the calling thread is available
 * from pager_last_error().  No torch types cross this boundary: callers own
 * all tensors; the library owns only what the pool functions hand out.
 *
 * Layouts (all row-major, contiguous):
 *   q          [batch, num_q_heads, head_dim]              q_dtype
 *   k, v       [batch, num_kv_heads, tokens, head_dim]      kv_dtype (chunk ops)
 *   m, l       [batch, num_q_heads]                         fp32, in/out
 *   acc        [batch, num_q_heads, head_dim]               fp32, in/out
 *   valid      [batch, tokens] int32 0/1 (NULL = all valid)
 *   active     [batch] int32 0/1 (NULL = all active)
 *   block_mass [batch, num_q_heads, max_blocks]             fp32
 *   KV pool    [slots, num_layers, 2 (K,V), num_kv_heads, tokens_per_block, head_dim]
 *   block table[batch, max_blocks] int32: slot index (device pool), or
 *              slot | PAGER_HOST_SLOT_BIT (pinned host pool), or -1 (absent)
 *
 * Query head h uses KV head h / n_rep with n_rep = num_q_heads / num_kv_heads
 * (GQA heads sharing a KV head are contiguous), n_rep <= 16.
 * head_dim must be one of 8, 16, 32, 64, 128, 256.
 */
#ifndef PAGER_B200_H
#define PAGER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { PAGER_DTYPE_F32 = 0, PAGER_DTYPE_F16 = 1, PAGER_DTYPE_BF16 = 2 };

enum {
  PAGER_OK = 0,
  PAGER_ERR_INVALID = 1,     /* bad shape, pointer, alignment or argument: ValueError   */
  PAGER_ERR_UNSUPPORTED = 2, /* n_rep > 16, head_dim outside the supported set          */
  PAGER_ERR_CUDA = 3,        /* CUDA runtime / launch failure                           */
  PAGER_ERR_SCRATCH = 4,     /* scratch buffer smaller than *_scratch_bytes() says      */
  PAGER_ERR_TIMEOUT = 5      /* a bounded device-side wait ran out (pager_device_status) */
};

/* Block-table tier bit: entry = host slot | PAGER_HOST_SLOT_BIT. */
#define PAGER_HOST_SLOT_BIT 0x40000000

/* Compute backends for the split kernel (PAGER_BACKEND_AUTO picks tensor-core
 * mma for fp16/bf16 at head_dim 64/128/256 and CUDA-core FMA otherwise). */
enum { PAGER_BACKEND_AUTO = 0, PAGER_BACKEND_MMA = 1, PAGER_BACKEND_FMA = 2 };

/* Mass accumulation modes of pager_paged_decode_attention. */
enum {
  PAGER_MASS_NONE = 0,
  PAGER_MASS_ROW_MEAN = 1,   /* mass_accum[b, j]  += mean over query heads            */
  PAGER_MASS_BATCH_MEAN = 2  /* mass_accum[j]     += mean over batch rows and heads   */
};

const char* pager_last_error(void);
int pager_version(void);
/* Reads (and clears) the device-side status word written by bounded waits. */
int pager_device_status(int device, int* status_out);

/* Stream-ordered form of pager_device_status for decode loops (the reference surfaces a failed
 * step per request, pager_hf/serving/scheduler.py:520-524): enqueues on `stream` a copy of the
 * current device's status word into *host_dst (page-locked host memory, so the copy is
 * asynchronous and can be captured in a CUDA graph), then a reset of the word to 0.  *host_dst is
 * valid once the stream has reached that point (e.g. after the step's synchronisation):
 * 0 = no fault, PAGER_ERR_TIMEOUT (5) = a bounded wait ran out, 6 = a block-table entry or a
 * tail write named a slot outside its pool and was skipped.  The word is per device: a kernel on
 * another stream may set it between the copy and the reset. */
int pager_status_snapshot_async(int32_t* host_dst, void* stream);

/* ---- streaming_attention_state_init (pager_hf/streaming_attention.py:444-449) */
int pager_attn_state_init(float* m, float* l, float* acc, int64_t rows, int head_dim, void* stream);

/* ---- streaming_attention_finalize (pager_hf/streaming_attention.py:668-670):
 *      out = (acc / l).to(out_dtype) */
int pager_attn_finalize(const float* acc, const float* l, void* out, int out_dtype, int64_t rows, int head_dim,
                        void* stream);

/* Scratch (device bytes) a chunk op needs; op: 0 step, 1 stats, 2 accumulate, 3 fold_fixed. */
size_t pager_attn_chunk_scratch_bytes(int op, int batch, int num_q_heads, int num_kv_heads, int tokens,
                                      int head_dim, int kv_dtype, int tokens_per_block);

/* ---- streaming_attention_step (pager_hf/streaming_attention.py:452-513):
 *      fold a chunk into (m, l, acc), in place.  With fp16/bf16 KV, p is rounded exactly as the
 *      reference's one-pass kernel rounds it (64-token tiles from the chunk's start, its running max
 *      starting at the incoming m, :143-181): a K pass to scores, a scan seeded with m, a V pass;
 *      pager_attn_chunk_scratch_bytes covers their scratch. */
int pager_attn_step(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype, const int32_t* valid,
                    const int32_t* active, float* m, float* l, float* acc, int batch, int num_q_heads,
                    int num_kv_heads, int tokens, int head_dim, float scale, float softcap, int backend,
                    void* scratch, size_t scratch_bytes, void* stream);

/* ---- streaming_attention_stats_step (pager_hf/streaming_attention.py:516-560):
 *      fold a chunk's K into (m, l) only. */
int pager_attn_stats_step(const void* q, int q_dtype, const void* k, int kv_dtype, const int32_t* valid,
                          const int32_t* active, float* m, float* l, int batch, int num_q_heads, int num_kv_heads,
                          int tokens, int head_dim, float scale, float softcap, int backend, void* scratch,
                          size_t scratch_bytes, void* stream);

/* ---- streaming_attention_accumulate_step (pager_hf/streaming_attention.py:563-621):
 *      acc += exp(s - m) . V with final (m, l); block_mass[b, h, block_id_offset + j] =
 *      sum over tokens of local block j of exp(s - m) / l.  Rows with active = 0 are untouched. */
int pager_attn_accumulate_step(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype,
                               const int32_t* valid, const int32_t* active, const float* m, const float* l,
                               float* acc, float* block_mass, int max_blocks, int block_id_offset,
                               int tokens_per_block, int batch, int num_q_heads, int num_kv_heads, int tokens,
                               int head_dim, float scale, float softcap, int backend, void* scratch,
                               size_t scratch_bytes, void* stream);

/* ---- streaming_attention_fold_fixed_step (pager_hf/streaming_attention.py:624-665):
 *      acc += exp(s - m) . V with final (m, l); no mass, no active switch. */
int pager_attn_fold_fixed_step(const void* q, int q_dtype, const void* k, const void* v, int kv_dtype,
                               const int32_t* valid, const float* m, const float* l, float* acc, int batch,
                               int num_q_heads, int num_kv_heads, int tokens, int head_dim, float scale,
                               float softcap, int backend, void* scratch, size_t scratch_bytes, void* stream);

/* ---- Fused paged decode attention: replaces the per-layer group loop of
 *      PagedModel._build_streaming_layer_forward (pager_hf/paged_model.py:993-1072) and
 *      batched_decode_step's layer forward (pager_hf/batched_decode.py:238-287), including
 *      the per-block gather of PagedModel._gather_layer_kv_group (paged_model.py:878-924).
 *      One split-KV pass over the block table (device pool blocks and pinned host pool
 *      blocks, read zero-copy) plus the tail, a combine that writes the finalized output,
 *      and the per-block attention mass (the two-pass reference's block_mass) from the
 *      same pass.
 *
 *   row b's tokens: blocks 0..num_blocks[b]-1 (tokens_per_block each), then tail_len[b]
 *   tail tokens from tail_k/tail_v [batch, num_kv_heads, tail_cap, head_dim].
 *   dev_slots/host_slots are the pools' capacities: a table entry naming a slot outside
 *   its pool (or a pool passed as NULL) is treated as absent and flagged in the device
 *   status word (pager_device_status), never dereferenced.
 *   valid_lo/valid_hi [batch] (NULL = whole row) bound the attended token range
 *   (left padding and sliding window); max_row_tokens is a host-known upper bound of
 *   num_blocks[b]*tokens_per_block + tail_len[b] over rows (sizes the split grid).
 */
size_t pager_paged_decode_scratch_bytes(int batch, int num_q_heads, int num_kv_heads, int head_dim, int kv_dtype,
                                        int tokens_per_block, int max_blocks, int max_row_tokens);

int pager_paged_decode_attention(const void* q, int q_dtype, const void* dev_pool, int dev_slots,
                                 const void* host_pool, int host_slots, int kv_dtype, int num_layers, int layer,
                                 int num_kv_heads, int tokens_per_block,
                                 int head_dim, const int32_t* block_table, int max_blocks,
                                 const int32_t* num_blocks, const void* tail_k, const void* tail_v,
                                 const int32_t* tail_len, int tail_cap, const int32_t* valid_lo,
                                 const int32_t* valid_hi, const int32_t* active, int batch, int num_q_heads,
                                 float scale, float softcap, int max_row_tokens, void* out, int out_dtype,
                                 float* block_mass, float* mass_accum, int mass_mode, int backend, void* scratch,
                                 size_t scratch_bytes, void* stream);

/* ---- The same fused paged decode attention for callers that cannot allocate device
 *      memory (a client binding this C ABI from a host language without a CUDA allocator,
 *      or a serving loop that forbids device allocation after start-up).  No counterpart in
 *      the reference: it takes every argument of pager_paged_decode_attention except the
 *      scratch buffer, and uses instead a fixed array of PAGER_NOALLOC_SCRATCH_BYTES of device
 *      memory built into the library -- reserved on every GPU that loads the library until
 *      the process exits.  Calls needing more scratch than that
 *      (pager_paged_decode_scratch_bytes) fail with PAGER_ERR_SCRATCH.  All calls on a device
 *      share the array and leave their contents in it (nothing needs to start at zero); calls
 *      that overlap on the GPU race on it.  The first call on a device looks up the array's
 *      address with that device current; make it before any stream capture.  Calls no
 *      cudaMalloc / cudaFree. */
#define PAGER_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
int pager_paged_decode_attention_noalloc(const void* q, int q_dtype, const void* dev_pool, int dev_slots,
                                         const void* host_pool, int host_slots, int kv_dtype, int num_layers,
                                         int layer, int num_kv_heads, int tokens_per_block, int head_dim,
                                         const int32_t* block_table, int max_blocks, const int32_t* num_blocks,
                                         const void* tail_k, const void* tail_v, const int32_t* tail_len,
                                         int tail_cap, const int32_t* valid_lo, const int32_t* valid_hi,
                                         const int32_t* active, int batch, int num_q_heads, float scale,
                                         float softcap, int max_row_tokens, void* out, int out_dtype,
                                         float* block_mass, float* mass_accum, int mass_mode, int backend,
                                         void* stream);

/* ---- Staged host tier.
 *      Block-table entries may also be `slot | PAGER_STAGE_SLOT_BIT`: slot of a device staging
 *      buffer [stage_slots, 2, kv_heads, tokens_per_block, head_dim] holding THIS layer's copy of
 *      a host block (filled by pager_stage_host_blocks on a copy stream).  The kernel reads staged
 *      blocks with TMA like device-pool blocks; host entries (PAGER_HOST_SLOT_BIT) are still read
 *      zero-copy.  Same arguments as pager_paged_decode_attention plus the staging buffer; every
 *      pool holds fewer than 2^29 slots.  The reference reads host blocks with synchronous
 *      pageable copies per layer and group (pager_hf/paged_model.py:878-924). */
#define PAGER_STAGE_SLOT_BIT 0x20000000
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
                                        void* stream);

/* ---- Reference-exact rounding of P.
 *      The reference rounds p = exp(s - m) to the KV dtype before its P.V product
 *      (pager_hf/streaming_attention.py:177-178; :346-347 and :427-428 in its two-pass path),
 *      with m its running max after each 64-token tile of the chunks it is handed
 *      (PagedModel._build_streaming_layer_forward, paged_model.py:1055-1072, for recent_only /
 *      sinks_recent) or the row's final max (the two-pass path of the heavy-hitter policies,
 *      paged_model.py:993-1039).  A one-pass split-KV kernel rounds against maxima the reference
 *      never uses, which moves about half of the bf16/fp16 outputs by an ulp.  These modes run two
 *      passes instead -- K to fp32 scores and group maxima, a scan to the reference's maxima, then
 *      V -- reading every K and V byte once (plus 2 * n_rep * 4 bytes of scores per token and KV
 *      head), and round p exactly as the reference does:
 *        PAGER_ROUND_ONE_PASS  the one-pass kernel (pager_paged_decode_attention_staged)
 *        PAGER_ROUND_RUNNING   the reference's one-pass path: m = running max after the reference
 *                              tile holding the token; tiles are 64 tokens from the start of each
 *                              chunk: chunks of ref_group_tokens tokens (<= 0: one chunk) of a
 *                              numbering in which row b's token j sits at ref_shift[b] + j (NULL:
 *                              j), then the tail chunk from row-local token ref_tail_start[b]
 *                              (NULL: num_blocks[b] * tokens_per_block).
 *        PAGER_ROUND_FINAL     the reference's two-pass path: m = the row's final max.
 *      fp16/bf16 KV, every head_dim (the tensor-core kernels need tokens_per_block >= 16 for
 *      PAGER_ROUND_RUNNING); fp32 KV rounds p to fp32, a no-op, so every mode runs the one pass
 *      there.  Other arguments as
 *      pager_paged_decode_attention_staged; scratch per pager_paged_decode_scratch_bytes_rounded. */
enum { PAGER_ROUND_ONE_PASS = 0, PAGER_ROUND_RUNNING = 1, PAGER_ROUND_FINAL = 2 };
size_t pager_paged_decode_scratch_bytes_rounded(int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                                int kv_dtype, int tokens_per_block, int max_row_tokens,
                                                int rounding);
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
                                         size_t scratch_bytes, void* stream);

/* Copy one layer of host-pool blocks into a staging buffer, one cudaMemcpy2DAsync per run:
 * run r copies run_len[r] consecutive host slots starting at run_src[r] into consecutive staging
 * slots starting at run_dst[r]; from each host slot it takes chunk_bytes at layer_offset_bytes
 * (slot_bytes apart).  run_* are HOST arrays.  Stream-ordered on `stream`. */
int pager_stage_host_blocks(void* stage, const void* host_pool, int64_t slot_bytes, int64_t layer_offset_bytes,
                            int64_t chunk_bytes, const int32_t* run_src, const int32_t* run_dst,
                            const int32_t* run_len, int nruns, void* stream);

/* ---- Writing one decode step's new token into pool slots.
 *      Replaces the tail concatenation of a decode step (pager_hf/batched_decode.py:170-171,
 *      the DynamicCache update of paged_model.py's patched forward): row b's new K and V
 *      (k_new / v_new [batch, kv_heads, head_dim], the pool's dtype) are written at token
 *      positions[b] of pool slot slots[b], layer `layer`.  A row with slots[b] < 0 is
 *      skipped; a slot outside [0, pool_slots) or a position outside [0, tokens_per_block)
 *      is not written and sets the device status word to 6. */
int pager_append_tokens(void* pool, int dtype, int pool_slots, int num_layers, int layer, int num_kv_heads,
                        int tokens_per_block, int head_dim, const int32_t* slots, const int32_t* positions,
                        const void* k_new, const void* v_new, int batch, void* stream);

/* ---- Self-test of the kernels' bounded waits (no counterpart in the reference).
 *      Every wait in the decode kernels (on a TMA stage, on a producer) gives up after a time
 *      limit, sets the device status word to PAGER_ERR_TIMEOUT and lets the kernel finish, so a
 *      stuck copy never hangs the GPU.  This launches one thread that waits on an mbarrier nothing
 *      arrives on, with a limit of limit_ns (at most 100 ms); afterwards pager_device_status
 *      reports 5 and *waited_ns holds the time the wait took.  Synchronises `stream`. */
int pager_selftest_bounded_wait(unsigned long long limit_ns, unsigned long long* waited_ns, void* stream);

/* ---- Pinned host pool (the host tier of KVBlockStore, pager_hf/kv_block_store.py:45-46).
 *      cudaHostAlloc(Portable | Mapped): the returned pointer is readable by kernels
 *      on every device (zero-copy) and is the host address as well. */
int pager_host_pool_alloc(size_t bytes, void** host_ptr);
int pager_host_pool_free(void* host_ptr);

/* ---- Link probes used to choose zero-copy vs copy-engine reads of host blocks.
 *      Both time `bytes` from pinned host memory into device memory on `stream`. */
int pager_probe_h2d_copy_gbs(const void* host_src, void* dev_dst, size_t bytes, int iters, void* stream,
                             double* gbs_out);
int pager_probe_zero_copy_gbs(const void* host_src, void* dev_dst, size_t bytes, int iters, void* stream,
                              double* gbs_out);

#ifdef __cplusplus
}
#endif

#endif /* PAGER_B200_H */
