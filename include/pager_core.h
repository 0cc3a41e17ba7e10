/* pager_core.h -- C ABI of the block-placement pager (host code, no GPU).
 *
 * The reference's pager is a Rust crate bound to Python with pyo3
 * (pager/src/lib.rs:9-74 -> module `pager`, class `PyPager`, class `Metrics`);
 * its placement logic is pager/src/core.rs:56-555.  This library restates that
 * logic in C++ and exports one C entry point per pyo3 method, so any host
 * language can bind it; the Python module `pager` (rust-llm-pager_b200/pager)
 * is the ctypes binding with the pyo3 class surface.
 *
 * Blocks are numbered 0, 1, 2, ... in the order they appear (one per
 * `tokens_per_block` tokens of a sequence); every block counts as 16 MiB
 * (core.rs:6) when the VRAM / RAM budgets are divided into block counts.
 * Tier codes: 0 = VRAM (device pool), 1 = RAM (pinned host pool), 2 = SSD
 * (evicted; core.rs:111-119).
 *
 * Status codes: 0 OK, 1 invalid argument (message from pager_core_last_error).
 * Not thread-safe per object: one caller at a time per pager (the reference's
 * PyPager holds the GIL for every method).
 */
#ifndef PAGER_CORE_H
#define PAGER_CORE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PAGER_CORE_API __attribute__((visibility("default")))
#else
#define PAGER_CORE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PAGER_CORE_BLOCK_BYTES ((size_t)16 * 1024 * 1024) /* core.rs:6 BLOCK_SIZE_BYTES */
#define PAGER_CORE_SINK_BLOCKS 4                          /* core.rs:7 SINK_BLOCKS */

#define PAGER_CORE_OK 0
#define PAGER_CORE_ERR_INVALID 1

/* Policy codes (core.rs:16-33).  Unknown names map to heavy_hitter. */
#define PAGER_POLICY_RECENT_ONLY 0
#define PAGER_POLICY_SINKS_RECENT 1
#define PAGER_POLICY_HEAVY_HITTER 2
#define PAGER_POLICY_SINKS_HEAVY_HITTER 3

typedef struct pager_core pager_core;

/* metrics.rs:4-27 Metrics */
typedef struct pager_core_metrics {
  uint64_t tokens;
  uint64_t vram_peak;
  uint64_t ram_peak;
  uint64_t swap_vram_ram;
  uint64_t swap_ram_ssd;
  double attention_mass_total;
  double attention_mass_vram;
} pager_core_metrics;

PAGER_CORE_API const char* pager_core_last_error(void);

/* Policy::from_name (core.rs:24-33). */
PAGER_CORE_API int pager_core_policy_code(const char* name);

/* PyPager::new (lib.rs:16-46): budgets in bytes, recent window in blocks. */
PAGER_CORE_API pager_core* pager_core_new(uint64_t vram, uint64_t ram, uint64_t recent, uint64_t rebalance_interval,
                           float promote_margin, float ram_promote_margin, const char* policy);
PAGER_CORE_API void pager_core_free(pager_core* p);

/* PyPager::on_step (lib.rs:48-50, core.rs:86-98): one decoded token's
 * per-block attention mass (n values).  Rebalances on the first token and every
 * `rebalance_interval` tokens.  Fails (status 1, nothing changed but the token
 * count and scores) when a rebalance falls due with rebalance_interval == 0,
 * where the reference panics on the modulo. */
PAGER_CORE_API int pager_core_on_step(pager_core* p, uint64_t token_idx, uint32_t layer, const float* attention, size_t n);

/* PyPager::force_rebalance (lib.rs:52-54, core.rs:100-107): grows the block
 * list to token_idx + 1 blocks, re-pins and re-places them. */
PAGER_CORE_API int pager_core_force_rebalance(pager_core* p, uint64_t token_idx);

/* PyPager::metrics (lib.rs:56-58). */
PAGER_CORE_API int pager_core_metrics_get(const pager_core* p, pager_core_metrics* out);

/* Number of blocks known to the pager. */
PAGER_CORE_API size_t pager_core_num_blocks(const pager_core* p);

/* PyPager::tiers (lib.rs:60-62): writes min(cap, num_blocks) tier codes,
 * returns num_blocks. */
PAGER_CORE_API size_t pager_core_tiers(const pager_core* p, uint8_t* out, size_t cap);

/* PyPager::vram_block_ids (lib.rs:64-66): writes min(cap, count) ids in
 * ascending order, returns count. */
PAGER_CORE_API size_t pager_core_vram_block_ids(const pager_core* p, uint64_t* out, size_t cap);

/* Per-block smoothed scores (the EMA of core.rs:144-148), for inspection:
 * writes min(cap, num_blocks) values, returns num_blocks. */
PAGER_CORE_API size_t pager_core_scores(const pager_core* p, float* out, size_t cap);

#ifdef __cplusplus
}
#endif

#endif /* PAGER_CORE_H */
