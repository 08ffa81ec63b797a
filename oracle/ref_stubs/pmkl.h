// Inert stand-in for the reference's umbrella header, used only when
// oracle/build_ref.py compiles the reference's test/test_softmax.cpp as a
// CPU library.  That file's host_softmax_forward (test_softmax.cpp:10-28) is
// the reference CPU softmax; its main() drives the GPU launcher, which is not
// wanted here.  main() is renamed at compile time and never called, so these
// declarations only have to let it compile: none of them does any work.
#pragma once
#include <cmath>
#include <cstddef>
#include <iostream>

namespace pmkl {
struct GpuLauncher {
    enum class Direction { H2D, D2H };
    static GpuLauncher *GetInstance() { return nullptr; }
    template <typename T> T *malloc(size_t) { return nullptr; }
    void memcpy(void *, void *, size_t, Direction) {}
    void stream_begin() {}
    void stream_end() {}
    void set_profiling_mode(bool) {}
};
namespace utils {
namespace host {
template <typename T> void fill_rand(T *, unsigned int, const T, const T) {}
}  // namespace host
template <typename T> bool all_close(T *, T *, unsigned int) { return false; }
}  // namespace utils
}  // namespace pmkl
