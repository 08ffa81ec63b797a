// Inert stand-in for pmkl/norm/warp_softmax.h (a CUDA-only device header),
// used only when oracle/build_ref.py compiles the reference's
// test/test_softmax.cpp for its host softmax.  Never called.
#pragma once
namespace pmkl {
namespace norm {
template <typename output_t, typename input_t, typename acc_t, bool is_log_softmax>
void warp_softmax_forward(output_t *, const input_t *, int, int, int) {}
}  // namespace norm
}  // namespace pmkl
