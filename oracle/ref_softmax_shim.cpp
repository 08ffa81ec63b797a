// Compiles the reference's own host softmax (test/test_softmax.cpp:10-28)
// unmodified into a CPU library with a C entry point, for pinning the oracle
// and timing the reference's CPU softmax.  Built by oracle/build_ref.py with
// -I oracle/ref_stubs (inert launcher stand-ins) and -Dmain=... so the test's
// GPU driver main() is compiled but never run.  Test infrastructure only.
#include "test_softmax.cpp"

extern "C" void pmkl_ref_host_softmax_forward_f32(float *dst, const float *src, int elements,
                                                  int stride, int rows) {
    host_softmax_forward<float, float, float>(dst, src, elements, stride, rows);
}
