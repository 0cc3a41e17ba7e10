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

// The two passes of reference-exact rounding (tensor-core kernels only).
#define PAGER_EXACT_MODE_CASES(T, D)                                                 \
  case D:                                                                            \
    switch (mode) {                                                                  \
      case pager::MODE_ONLINE: *out = pager::split_kernel_info<T, D, pager::MODE_ONLINE, pager::BACKEND_MMA>(); return true; \
      case pager::MODE_STATS: *out = pager::split_kernel_info<T, D, pager::MODE_STATS, pager::BACKEND_MMA>(); return true;   \
      case pager::MODE_FIXED: *out = pager::split_kernel_info<T, D, pager::MODE_FIXED, pager::BACKEND_MMA>(); return true;   \
      case pager::MODE_SCORES: *out = pager::split_kernel_info<T, D, pager::MODE_SCORES, pager::BACKEND_MMA>(); return true; \
      case pager::MODE_VALUES: *out = pager::split_kernel_info<T, D, pager::MODE_VALUES, pager::BACKEND_MMA>(); return true; \
      case pager::MODE_VALUES_R4: *out = pager::split_kernel_info<T, D, pager::MODE_VALUES_R4, pager::BACKEND_MMA>(); return true; \
      case pager::MODE_VALUES_R8: *out = pager::split_kernel_info<T, D, pager::MODE_VALUES_R8, pager::BACKEND_MMA>(); return true; \
      default: return false;                                                         \
    }

// Every mode of the CUDA-core kernels for 16-bit KV (fp32 KV rounds p to fp32, a no-op, so its
// one-pass kernel already is the reference's arithmetic and it has no exact-rounding passes).
#define PAGER_FMA16_MODE_CASES(T, D)                                                 \
  case D:                                                                            \
    switch (mode) {                                                                  \
      case pager::MODE_ONLINE: *out = pager::split_kernel_info<T, D, pager::MODE_ONLINE, pager::BACKEND_FMA>(); return true; \
      case pager::MODE_STATS: *out = pager::split_kernel_info<T, D, pager::MODE_STATS, pager::BACKEND_FMA>(); return true;   \
      case pager::MODE_FIXED: *out = pager::split_kernel_info<T, D, pager::MODE_FIXED, pager::BACKEND_FMA>(); return true;   \
      case pager::MODE_SCORES: *out = pager::split_kernel_info<T, D, pager::MODE_SCORES, pager::BACKEND_FMA>(); return true; \
      case pager::MODE_VALUES: *out = pager::split_kernel_info<T, D, pager::MODE_VALUES, pager::BACKEND_FMA>(); return true; \
      default: return false;                                                         \
    }
