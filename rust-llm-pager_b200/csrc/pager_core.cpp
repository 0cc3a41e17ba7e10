// Block-placement pager: which KV blocks live in VRAM, pinned RAM, or are
// evicted, decided from a smoothed per-block attention score.
//
// Restates the reference's Rust pager (pager/src/core.rs:56-555, metrics in
// pager/src/metrics.rs) so that identical call sequences give identical
// placements, metrics and scores.  The points where that needs care:
//   * scores are f32 and updated as s*0.9f + a*0.1f with two roundings and no
//     fused multiply-add (core.rs:144-148; Rust never contracts; this file is
//     built with -ffp-contract=off);
//   * score comparisons treat unordered pairs (NaN) as equal (core.rs:555-557);
//   * every sort is stable (Rust's sort_by), every "worst" pick returns the
//     first of equal minima and every "best" pick the last of equal maxima
//     (Iterator::min_by / max_by);
//   * attention mass totals are f64 sums in block order (core.rs:150-164).
// One deliberate difference: the hysteresis swap loops stop after n*n swaps.
// With a non-negative margin and finite scores each swap raises the VRAM
// (or RAM) score sum by more than the margin, so they end long before that;
// a negative margin or NaN scores can make the reference loop forever.
#include "pager_core.h"

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

int fail(const std::string& msg) {
  g_err = msg;
  return PAGER_CORE_ERR_INVALID;
}

enum Tier : uint8_t { kVram = 0, kRam = 1, kSsd = 2 };

// -1 / 0 / +1 like Rust's partial_cmp(..).unwrap_or(Equal)
inline int cmp_scores(float a, float b) {
  if (a < b) return -1;
  if (a > b) return 1;
  return 0;
}

struct Block {
  uint64_t id;
  float score;
  uint8_t tier;
  bool pinned;
};

}  // namespace

struct pager_core {
  uint64_t vram_bytes, ram_bytes, recent_window, interval;
  float vram_margin, ram_margin;
  int policy;
  pager_core_metrics m;
  std::vector<Block> blocks;

  size_t count_tier(uint8_t t) const {
    size_t n = 0;
    for (const Block& b : blocks) n += b.tier == t;
    return n;
  }

  void grow_to(size_t n) {
    while (blocks.size() < n) blocks.push_back(Block{blocks.size(), 0.0f, kRam, false});
  }

  void smooth_scores(const float* a, size_t n) {
    const size_t k = std::min(n, blocks.size());
    for (size_t i = 0; i < k; ++i) {
      const float kept = blocks[i].score * 0.90f;
      const float added = a[i] * 0.10f;
      blocks[i].score = kept + added;
    }
  }

  void record_mass(const float* a, size_t n) {
    double total = 0.0, in_vram = 0.0;
    const size_t k = std::min(n, blocks.size());
    for (size_t i = 0; i < k; ++i) {
      const double s = static_cast<double>(a[i]);
      total += s;
      if (blocks[i].tier == kVram) in_vram += s;
    }
    m.attention_mass_total += total;
    m.attention_mass_vram += in_vram;
  }

  void pin(uint64_t token_idx) {
    const uint64_t recent_start = token_idx > recent_window ? token_idx - recent_window : 0;
    for (Block& b : blocks) {
      const bool recent = b.id >= recent_start;
      const bool sink = b.id < static_cast<uint64_t>(PAGER_CORE_SINK_BLOCKS);
      b.pinned = policy == PAGER_POLICY_RECENT_ONLY ? recent : (recent || sink);
    }
  }

  // indices ordered pinned-first, then by `then` (stable)
  template <class Then>
  void sort_pinned_first(std::vector<size_t>& idx, Then then) const {
    std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
      if (blocks[a].pinned != blocks[b].pinned) return blocks[a].pinned;
      return then(a, b);
    });
  }

  std::vector<size_t> all_indices() const {
    std::vector<size_t> idx(blocks.size());
    for (size_t i = 0; i < idx.size(); ++i) idx[i] = i;
    return idx;
  }

  void assign_ranked(const std::vector<size_t>& order, size_t max_vram, size_t max_ram) {
    for (size_t r = 0; r < order.size(); ++r)
      blocks[order[r]].tier = r < max_vram ? kVram : (r < max_vram + max_ram ? kRam : kSsd);
  }

  void set_all(uint8_t t) {
    for (Block& b : blocks) b.tier = t;
  }

  // first index with the smallest score among blocks passing `keep`, or -1
  template <class Keep>
  long long pick_worst(Keep keep) const {
    long long best = -1;
    for (size_t i = 0; i < blocks.size(); ++i) {
      if (!keep(blocks[i])) continue;
      if (best < 0 || cmp_scores(blocks[best].score, blocks[i].score) > 0) best = static_cast<long long>(i);
    }
    return best;
  }

  // last index with the largest score among blocks passing `keep`, or -1
  template <class Keep>
  long long pick_best(Keep keep) const {
    long long best = -1;
    for (size_t i = 0; i < blocks.size(); ++i) {
      if (!keep(blocks[i])) continue;
      if (best < 0 || cmp_scores(blocks[best].score, blocks[i].score) <= 0) best = static_cast<long long>(i);
    }
    return best;
  }

  void place_by_rank(size_t max_vram, size_t max_ram) {  // recent_only, sinks_recent (core.rs:197-216)
    std::vector<size_t> order = all_indices();
    sort_pinned_first(order, [&](size_t a, size_t b) { return blocks[a].id < blocks[b].id; });
    set_all(kSsd);
    assign_ranked(order, max_vram, max_ram);
  }

  void keep_best_in_vram(size_t max_vram) {  // core.rs:330-354
    std::vector<size_t> in_vram;
    for (size_t i = 0; i < blocks.size(); ++i)
      if (blocks[i].tier == kVram) in_vram.push_back(i);
    if (in_vram.size() <= max_vram) return;
    sort_pinned_first(in_vram, [&](size_t a, size_t b) { return cmp_scores(blocks[b].score, blocks[a].score) < 0; });
    for (size_t r = max_vram; r < in_vram.size(); ++r) blocks[in_vram[r]].tier = kRam;
  }

  void promote_into_vram(size_t max_vram) {  // core.rs:356-387
    const size_t cap = blocks.size() * blocks.size() + blocks.size() + 1;
    for (size_t it = 0; it < cap; ++it) {
      const long long best = pick_best([](const Block& b) { return b.tier != kVram; });
      if (count_tier(kVram) < max_vram) {
        if (best < 0) return;
        blocks[best].tier = kVram;
        continue;
      }
      const long long worst = pick_worst([](const Block& b) { return b.tier == kVram && !b.pinned; });
      if (worst < 0 || best < 0) return;
      const float gain = blocks[best].score - blocks[worst].score;
      if (gain <= vram_margin) return;
      const uint8_t from = blocks[best].tier;
      blocks[best].tier = kVram;
      blocks[worst].tier = from;
    }
  }

  void shrink_ram(size_t max_ram) {  // core.rs:429-448
    std::vector<size_t> in_ram;
    for (size_t i = 0; i < blocks.size(); ++i)
      if (blocks[i].tier == kRam) in_ram.push_back(i);
    if (in_ram.size() <= max_ram) return;
    std::stable_sort(in_ram.begin(), in_ram.end(),
                     [&](size_t a, size_t b) { return cmp_scores(blocks[a].score, blocks[b].score) < 0; });
    const size_t drop = in_ram.size() - max_ram;
    for (size_t r = 0; r < drop; ++r) blocks[in_ram[r]].tier = kSsd;
  }

  void fill_ram(size_t max_ram) {  // core.rs:403-427
    const size_t have = count_tier(kRam);
    if (have >= max_ram) {
      shrink_ram(max_ram);
      return;
    }
    std::vector<size_t> evicted;
    for (size_t i = 0; i < blocks.size(); ++i)
      if (blocks[i].tier == kSsd) evicted.push_back(i);
    std::stable_sort(evicted.begin(), evicted.end(),
                     [&](size_t a, size_t b) { return cmp_scores(blocks[b].score, blocks[a].score) < 0; });
    const size_t take = std::min(evicted.size(), max_ram - have);
    for (size_t r = 0; r < take; ++r) blocks[evicted[r]].tier = kRam;
  }

  void promote_into_ram(size_t max_ram) {  // core.rs:450-477
    const size_t cap = blocks.size() * blocks.size() + 1;
    for (size_t it = 0; it < cap; ++it) {
      if (count_tier(kRam) < max_ram) return;
      const long long worst = pick_worst([](const Block& b) { return b.tier == kRam; });
      const long long best = pick_best([](const Block& b) { return b.tier == kSsd; });
      if (worst < 0 || best < 0) return;
      const float gain = blocks[best].score - blocks[worst].score;
      if (gain <= ram_margin) return;
      blocks[best].tier = kRam;
      blocks[worst].tier = kSsd;
    }
  }

  void place_heavy_hitter(size_t max_vram, size_t max_ram) {  // core.rs:218-250
    if (count_tier(kVram) == 0) {
      std::vector<size_t> order = all_indices();
      sort_pinned_first(order, [&](size_t a, size_t b) { return cmp_scores(blocks[b].score, blocks[a].score) < 0; });
      assign_ranked(order, max_vram, max_ram);
      return;
    }
    for (Block& b : blocks)
      if (b.pinned) b.tier = kVram;
    keep_best_in_vram(max_vram);
    promote_into_vram(max_vram);
    fill_ram(max_ram);
    promote_into_ram(max_ram);
  }

  void place_sinks_heavy_hitter(size_t max_vram, size_t max_ram) {  // core.rs:252-313
    set_all(kSsd);
    if (max_vram == 0) return;
    std::vector<char> chosen(blocks.size(), 0);
    size_t n_chosen = 0;
    auto choose = [&](size_t i) {
      if (!chosen[i]) {
        chosen[i] = 1;
        ++n_chosen;
      }
    };
    for (size_t i = 0; i < blocks.size() && i < static_cast<size_t>(PAGER_CORE_SINK_BLOCKS); ++i) {
      if (n_chosen >= max_vram) break;
      choose(i);
    }
    const size_t left = max_vram > n_chosen ? max_vram - n_chosen : 0;
    const uint64_t half = std::max<uint64_t>(max_vram / 2, 1);
    const size_t recent_budget = static_cast<size_t>(std::min<uint64_t>(std::min<uint64_t>(recent_window, half), left));
    const size_t first_recent = blocks.size() > recent_budget ? blocks.size() - recent_budget : 0;
    for (size_t i = first_recent; i < blocks.size(); ++i) {
      if (n_chosen >= max_vram) break;
      choose(i);
    }
    std::vector<size_t> rest;
    for (size_t i = 0; i < blocks.size(); ++i)
      if (!chosen[i]) rest.push_back(i);
    std::stable_sort(rest.begin(), rest.end(),
                     [&](size_t a, size_t b) { return cmp_scores(blocks[b].score, blocks[a].score) < 0; });
    for (size_t i : rest) {
      if (n_chosen >= max_vram) break;
      choose(i);
    }
    for (size_t i = 0; i < blocks.size(); ++i)
      if (chosen[i]) blocks[i].tier = kVram;
    fill_ram(max_ram);
  }

  void count_moves(const std::vector<uint8_t>& before) {  // core.rs:511-529
    const uint64_t sz = PAGER_CORE_BLOCK_BYTES;
    for (size_t i = 0; i < before.size() && i < blocks.size(); ++i) {
      const uint8_t a = before[i], b = blocks[i].tier;
      if (a == b) continue;
      const bool crosses_vram_ram = a == kVram || b == kVram;  // VRAM<->RAM or VRAM<->SSD
      const bool crosses_ram_ssd = a == kSsd || b == kSsd;     // RAM<->SSD or VRAM<->SSD
      if (crosses_vram_ram) m.swap_vram_ram += sz;
      if (crosses_ram_ssd) m.swap_ram_ssd += sz;
    }
  }

  void place() {  // core.rs:179-195
    std::vector<uint8_t> before(blocks.size());
    for (size_t i = 0; i < blocks.size(); ++i) before[i] = blocks[i].tier;
    const size_t max_vram = static_cast<size_t>(vram_bytes / PAGER_CORE_BLOCK_BYTES);
    const size_t max_ram = static_cast<size_t>(ram_bytes / PAGER_CORE_BLOCK_BYTES);
    switch (policy) {
      case PAGER_POLICY_RECENT_ONLY:
      case PAGER_POLICY_SINKS_RECENT:
        place_by_rank(max_vram, max_ram);
        break;
      case PAGER_POLICY_SINKS_HEAVY_HITTER:
        place_sinks_heavy_hitter(max_vram, max_ram);
        break;
      default:
        place_heavy_hitter(max_vram, max_ram);
        break;
    }
    count_moves(before);
  }

  void track_peaks() {  // core.rs:531-552
    const uint64_t sz = PAGER_CORE_BLOCK_BYTES;
    m.vram_peak = std::max<uint64_t>(m.vram_peak, count_tier(kVram) * sz);
    m.ram_peak = std::max<uint64_t>(m.ram_peak, count_tier(kRam) * sz);
  }

  int rebalance(uint64_t token_idx) {  // core.rs:100-107
    if (token_idx >= static_cast<uint64_t>(SIZE_MAX / 2)) return fail("force_rebalance: token_idx too large");
    grow_to(static_cast<size_t>(token_idx) + 1);
    pin(token_idx);
    place();
    track_peaks();
    return PAGER_CORE_OK;
  }
};

extern "C" {

const char* pager_core_last_error(void) { return g_err.c_str(); }

int pager_core_policy_code(const char* name) {
  if (name) {
    if (!std::strcmp(name, "recent_only")) return PAGER_POLICY_RECENT_ONLY;
    if (!std::strcmp(name, "sinks_recent")) return PAGER_POLICY_SINKS_RECENT;
    if (!std::strcmp(name, "sinks_heavy_hitter")) return PAGER_POLICY_SINKS_HEAVY_HITTER;
  }
  return PAGER_POLICY_HEAVY_HITTER;
}

pager_core* pager_core_new(uint64_t vram, uint64_t ram, uint64_t recent, uint64_t rebalance_interval,
                           float promote_margin, float ram_promote_margin, const char* policy) {
  pager_core* p = new pager_core();
  p->vram_bytes = vram;
  p->ram_bytes = ram;
  p->recent_window = recent;
  p->interval = rebalance_interval;
  p->vram_margin = promote_margin;
  p->ram_margin = ram_promote_margin;
  p->policy = pager_core_policy_code(policy);
  std::memset(&p->m, 0, sizeof(p->m));
  return p;
}

void pager_core_free(pager_core* p) { delete p; }

int pager_core_on_step(pager_core* p, uint64_t token_idx, uint32_t /*layer*/, const float* attention, size_t n) {
  if (!p) return fail("on_step: null pager");
  if (n && !attention) return fail("on_step: null attention with n > 0");
  p->m.tokens += 1;
  p->grow_to(n);
  p->smooth_scores(attention, n);
  p->record_mass(attention, n);
  p->pin(token_idx);
  if (p->m.tokens == 1) return p->rebalance(token_idx);
  if (p->interval == 0) return fail("on_step: rebalance_interval is 0 (the reference panics on the modulo)");
  if (p->m.tokens % p->interval == 0) return p->rebalance(token_idx);
  return PAGER_CORE_OK;
}

int pager_core_force_rebalance(pager_core* p, uint64_t token_idx) {
  if (!p) return fail("force_rebalance: null pager");
  return p->rebalance(token_idx);
}

int pager_core_metrics_get(const pager_core* p, pager_core_metrics* out) {
  if (!p || !out) return fail("metrics: null argument");
  *out = p->m;
  return PAGER_CORE_OK;
}

size_t pager_core_num_blocks(const pager_core* p) { return p ? p->blocks.size() : 0; }

size_t pager_core_tiers(const pager_core* p, uint8_t* out, size_t cap) {
  if (!p) return 0;
  for (size_t i = 0; i < p->blocks.size() && i < cap; ++i) out[i] = p->blocks[i].tier;
  return p->blocks.size();
}

size_t pager_core_vram_block_ids(const pager_core* p, uint64_t* out, size_t cap) {
  if (!p) return 0;
  size_t n = 0;
  for (const Block& b : p->blocks) {
    if (b.tier != kVram) continue;
    if (n < cap) out[n] = b.id;
    ++n;
  }
  return n;
}

size_t pager_core_scores(const pager_core* p, float* out, size_t cap) {
  if (!p) return 0;
  for (size_t i = 0; i < p->blocks.size() && i < cap; ++i) out[i] = p->blocks[i].score;
  return p->blocks.size();
}

}  // extern "C"
