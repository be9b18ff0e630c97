// dtype dispatch helpers for the host launchers
#pragma once

#include "nib_common.cuh"

namespace nib {
template <int code> struct DType;
template <> struct DType<NIB_F32> { using type = float; };
template <> struct DType<NIB_F16> { using type = __half; };
template <> struct DType<NIB_BF16> { using type = __nv_bfloat16; };
}  // namespace nib

#define NIB_CASE_T(code, T_, ...)            \
  case code: {                               \
    using T_ = ::nib::DType<code>::type;     \
    __VA_ARGS__;                             \
    break;                                   \
  }

// Expands the body with T_ bound to the C++ type of `dtype`; unknown codes
// return NIB_ERR_UNSUPPORTED from the enclosing function.
#define NIB_DISPATCH(dtype, T_, ...)                                  \
  switch (dtype) {                                                    \
    NIB_CASE_T(NIB_F32, T_, __VA_ARGS__)                              \
    NIB_CASE_T(NIB_F16, T_, __VA_ARGS__)                              \
    NIB_CASE_T(NIB_BF16, T_, __VA_ARGS__)                             \
    default:                                                          \
      ::nib::set_error("unsupported dtype code %d", (int)(dtype));    \
      return NIB_ERR_UNSUPPORTED;                                     \
  }
