// Instantiation helpers: each split_*.cu file instantiates one family of
// split kernels and exposes a lookup by (head_dim, mode).
#pragma once
#include "pager_split.cuh"

#define PAGER_MODE_CASES(T, D, BE)                                                   \
  case D:                                                                            \
    switch (mode) {                                                                  \
      case pager::MODE_ONLINE: *out = pager::split_kernel_info<T, D, pager::MODE_ONLINE, BE>(); return true; \
      case pager::MODE_STATS: *out = pager::split_kernel_info<T, D, pager::MODE_STATS, BE>(); return true;   \
      case pager::MODE_FIXED: *out = pager::split_kernel_info<T, D, pager::MODE_FIXED, BE>(); return true;   \
      default: return false;                                                         \
    }
