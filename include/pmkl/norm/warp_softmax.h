// pmkl/norm/warp_softmax.h -- B200 drop-in for the reference header of the
// same path (pmkl/norm/warp_softmax.h:159-201).
//
// Same template signature and argument meaning: `batch_count` rows of
// `softmax_elements` values, consecutive rows `softmax_elements_stride`
// elements apart, 0 <= softmax_elements <= 1024.  acc_t must be float
// (the B200 kernels accumulate in fp32).  Synchronises like the reference
// launcher unless `synchronize` is false.  Errors throw pmkl::Error.
#pragma once

#include <type_traits>

#include "../pmkl_b200_shim.h"

namespace pmkl {
namespace norm {

template <typename output_t, typename input_t, typename acc_t, bool is_log_softmax>
void warp_softmax_forward(output_t *dst, const input_t *src, int softmax_elements, int softmax_elements_stride,
                          int batch_count, void *stream = nullptr, bool synchronize = true) {
    static_assert(std::is_same<acc_t, float>::value, "pmkl_b200 accumulates softmax in float");
    detail::check(pmkl_warp_softmax_fwd(dst, src, softmax_elements, softmax_elements_stride, batch_count,
                                        detail::DtypeOf<input_t>::value, detail::DtypeOf<output_t>::value,
                                        is_log_softmax ? 1 : 0, stream),
                  "warp_softmax_forward");
    if (synchronize) detail::check(pmkl_stream_synchronize(stream), "warp_softmax_forward");
}

}  // namespace norm
}  // namespace pmkl
