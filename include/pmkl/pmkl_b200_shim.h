// pmkl_b200_shim.h -- shared pieces of the header-only C++ shim that keeps
// the reference's C++ entry points (pmkl::nlp::causal_attention_forward,
// pmkl::norm::warp_softmax_forward) and forwards them to the C ABI of
// libpmkl_b200 (pmkl_b200.h).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <stdexcept>
#include <string>

#include "pmkl_b200.h"

namespace pmkl {

// Thrown where the reference's CHECK_FAIL throws pmkl::utils::Error
// (pmkl/core/utils/exception.h:121-129).
class Error : public std::runtime_error {
   public:
    Error(const std::string &what, int status) : std::runtime_error(what), status_(status) {}
    int status() const { return status_; }

   private:
    int status_;
};

namespace detail {

template <typename T>
struct DtypeOf;
template <>
struct DtypeOf<float> {
    static constexpr int value = PMKL_DTYPE_F32;
};
template <>
struct DtypeOf<__half> {
    static constexpr int value = PMKL_DTYPE_F16;
};
template <>
struct DtypeOf<__nv_bfloat16> {
    static constexpr int value = PMKL_DTYPE_BF16;
};

inline void check(int status, const char *what) {
    if (status != PMKL_OK) throw Error(std::string(what) + ": " + pmkl_status_string(status), status);
}

}  // namespace detail
}  // namespace pmkl
