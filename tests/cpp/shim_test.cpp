// C++ drop-in test: calls the reference's C++ entry points through the B200
// shim headers, in the manner of the reference's own GPU tests
// (test/test_causal_attention.cpp:143-207, test/test_softmax.cpp:30-58), and
// checks the results against the CPU oracle with the reference's all_close
// rule (atol = rtol = 1e-5, pmkl/core/utils/measure.h:10-29).  Prints "ok"
// and exits 0 on success.  Built and run by tests/test_shim_gpu.py.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <vector>

#include "pmkl/nlp/causal_attention.h"
#include "pmkl/norm/warp_softmax.h"

extern "C" {
int pmkl_oracle_attention_fwd_f32(const float *, const float *, const float *, float *, float *, float *, int64_t,
                                  int, int, int, float);
void pmkl_oracle_softmax_fwd_f32(float *, const float *, int, int, int);
}

static uint64_t g_state = 0x9E3779B97F4A7C15ull;
static float uniform(float lo, float hi) {  // seeded, reproducible (the reference uses time(0))
    g_state = g_state * 6364136223846793005ull + 1442695040888963407ull;
    return lo + (hi - lo) * static_cast<float>((g_state >> 40) & 0xFFFFFF) / 16777216.0f;
}

static bool all_close(const std::vector<float> &a, const std::vector<float> &b, const char *what) {
    size_t bad = 0;
    for (size_t i = 0; i < a.size(); ++i)
        if (std::isnan(a[i]) || std::fabs(a[i] - b[i]) > 1e-5 + 1e-5 * std::fabs(b[i])) {
            if (bad < 5) std::printf("%s mismatch at %zu: %g vs %g\n", what, i, a[i], b[i]);
            ++bad;
        }
    return bad == 0;
}

template <typename T>
static T *to_device(const std::vector<T> &h) {
    T *d = nullptr;
    cudaMalloc(&d, h.size() * sizeof(T));
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}

template <typename T>
static std::vector<T> to_host(const T *d, size_t n) {
    std::vector<T> h(n);
    cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
    return h;
}

int main() {
    // causal attention, fp32, the reference test's shape reduced to B1 H4
    const int B = 1, H = 4, S = 256, D = 64;
    const size_t n = static_cast<size_t>(B) * H * S * D, ns = static_cast<size_t>(B) * H * S;
    std::vector<float> q(n), k(n), v(n);
    for (size_t i = 0; i < n; ++i) q[i] = uniform(-1.05f, 1.05f);
    for (size_t i = 0; i < n; ++i) k[i] = uniform(-1.05f, 1.05f);
    for (size_t i = 0; i < n; ++i) v[i] = uniform(-1.05f, 1.05f);
    float *dq = to_device(q), *dk = to_device(k), *dv = to_device(v);
    float *dout = nullptr, *dm = nullptr, *dl = nullptr;
    cudaMalloc(&dout, n * 4);
    cudaMalloc(&dm, ns * 4);
    cudaMalloc(&dl, ns * 4);
    pmkl::nlp::causal_attention_forward<float, 32, 64>(dout, dq, dk, dv, B, H, S, dm, dl);
    std::vector<float> o_ref(n), m_ref(ns), l_ref(ns);
    pmkl_oracle_attention_fwd_f32(q.data(), k.data(), v.data(), o_ref.data(), m_ref.data(), l_ref.data(), B * H, S,
                                  D, 1, 1.0f / std::sqrt(static_cast<float>(D)));
    if (!all_close(to_host(dm, ns), m_ref, "m") || !all_close(to_host(dl, ns), l_ref, "l") ||
        !all_close(to_host(dout, n), o_ref, "out"))
        return 1;

    // a bad size must throw pmkl::Error, as CHECK_FAIL throws in the reference
    bool threw = false;
    try {
        pmkl::norm::warp_softmax_forward<float, float, float, false>(dout, dq, 1025, 1025, 1);
    } catch (const pmkl::Error &) {
        threw = true;
    }
    if (!threw) return 2;

    // warp softmax, fp32, the reference test's shape (12 x 1024) in U(-10, 10)
    const int rows = 12, el = 1024;
    std::vector<float> x(static_cast<size_t>(rows) * el), y_ref(x.size());
    for (auto &e : x) e = uniform(-10.f, 10.f);
    float *dx = to_device(x), *dy = nullptr;
    cudaMalloc(&dy, x.size() * 4);
    for (int it = 0; it < 10; ++it) pmkl::norm::warp_softmax_forward<float, float, float, false>(dy, dx, el, el, rows);
    pmkl_oracle_softmax_fwd_f32(y_ref.data(), x.data(), el, el, rows);
    if (!all_close(to_host(dy, x.size()), y_ref, "softmax")) return 3;
    std::printf("ok\n");
    return 0;
}
