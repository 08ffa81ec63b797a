// pmkl/nlp/causal_attention.h -- B200 drop-in for the reference header of the
// same path (pmkl/nlp/causal_attention.h:258-288).
//
// Same template signature and argument meaning: out/q/k/v are device pointers
// to [batch, heads, seq, HIDDEN_SIZE] tensors, out_m/out_l to [batch, heads,
// seq]; causal mask; scale 1/sqrt(HIDDEN_SIZE).  BLOCK_M is accepted for
// source compatibility and ignored (the B200 kernels pick their own tiles),
// and seq needs no longer be a multiple of 32.
//
// The reference launcher synchronises after every launch by default
// (pmkl/core/launcher/cuda_launcher.h:334); so does this function unless
// `synchronize` is false.  Work goes to `stream` (default: legacy default
// stream).  Errors throw pmkl::Error.
#pragma once

#include "../pmkl_b200_shim.h"

namespace pmkl {
namespace nlp {

template <typename scalar_t, int BLOCK_M = 32, int HIDDEN_SIZE = 64>
void causal_attention_forward(scalar_t *out, const scalar_t *q, const scalar_t *k, const scalar_t *v,
                              const int batch_size, const int num_heads, const int seq_length, scalar_t *out_m,
                              scalar_t *out_l, void *stream = nullptr, bool synchronize = true) {
    constexpr int dt = detail::DtypeOf<scalar_t>::value;
    detail::check(pmkl_causal_attention_fwd(q, k, v, out, out_m, out_l, batch_size, num_heads, seq_length,
                                            HIDDEN_SIZE, dt, dt, /*is_causal=*/1, /*scale=*/0.f, stream),
                  "causal_attention_forward");
    if (synchronize) detail::check(pmkl_stream_synchronize(stream), "causal_attention_forward");
}

}  // namespace nlp
}  // namespace pmkl
