// pmkl_pytorch_ext -- torch binding of the B200 attention kernels.
//
// Keeps the reference extension's module name, function names, argument
// lists, return tuple and error behaviour
// (pmkl_pytorch_ext/fused_self_attention.cpp:139-220), but the compute goes
// through the C ABI of libpmkl_b200 (include/pmkl_b200.h) on the current
// CUDA stream instead of the reference's single-threaded host loops.  There is
// no CPU path: CPU tensors are rejected.
#include <array>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include "pmkl_b200.h"

namespace {

int pmkl_dtype_of(at::ScalarType t) {
    switch (t) {
        case at::ScalarType::Float:
            return PMKL_DTYPE_F32;
        case at::ScalarType::Half:
            return PMKL_DTYPE_F16;
        case at::ScalarType::BFloat16:
            return PMKL_DTYPE_BF16;
        default:
            return -1;
    }
}

void check_inputs(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v, bool allow_kv_heads = false) {
    // fused_self_attention.cpp:140-141
    TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "Input tensor shapes must match");
    if (allow_kv_heads) {
        // Grouped-query form (no reference counterpart): k and v may have fewer heads.
        TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == q.size(0) && k.size(2) == q.size(2) &&
                        k.size(3) == q.size(3) && k.size(1) > 0 && q.size(1) % k.size(1) == 0,
                    "Input tensor shapes must match (k and v may have heads dividing q's heads)");
    } else {
        TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes(), "Input tensor shapes must match");
    }
    TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(),
                "pmkl_pytorch_ext (B200 build) runs on CUDA tensors only; got a CPU tensor");
    TORCH_CHECK(q.device() == k.device() && q.device() == v.device(), "q, k and v must be on the same device");
    TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(),
                "q, k and v must have the same dtype");
    TORCH_CHECK(pmkl_dtype_of(v.scalar_type()) >= 0, "fused_self_attention: unsupported dtype ", v.scalar_type(),
                " (float32, float16 and bfloat16 are supported)");
    TORCH_CHECK(q.size(0) <= INT32_MAX && q.size(1) <= INT32_MAX && q.size(2) <= INT32_MAX && q.size(3) <= INT32_MAX,
                "fused_self_attention: sizes must fit in 32-bit integers");
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> forward_impl(const at::Tensor &q, const at::Tensor &k,
                                                            const at::Tensor &v, bool is_causal, bool out_fp32,
                                                            int64_t kernel, double scale, bool allow_kv_heads) {
    check_inputs(q, k, v, allow_kv_heads);
    const c10::cuda::CUDAGuard guard(q.device());
    const int B = static_cast<int>(q.size(0)), H = static_cast<int>(q.size(1));
    const int S = static_cast<int>(q.size(2)), D = static_cast<int>(q.size(3));
    const int Hkv = static_cast<int>(k.size(1));
    // The reference makes the inputs contiguous (fused_self_attention.cpp:160-162);
    // here they are read in place through their strides, and copied only when
    // the hidden dimension itself is strided.
    const auto rows_ok = [](const at::Tensor &t) { return t.size(3) <= 1 || t.stride(3) == 1; };
    const at::Tensor qc = rows_ok(q) ? q : q.contiguous();
    const at::Tensor kc = rows_ok(k) ? k : k.contiguous();
    const at::Tensor vc = rows_ok(v) ? v : v.contiguous();
    const int64_t qs[3] = {qc.stride(0), qc.stride(1), qc.stride(2)};
    const int64_t ks[3] = {kc.stride(0), kc.stride(1), kc.stride(2)};
    const int64_t vs[3] = {vc.stride(0), vc.stride(1), vc.stride(2)};
    // Outputs in v's dtype (fused_self_attention.cpp:148-150), contiguous.
    const auto opts = out_fp32 ? v.options().dtype(at::kFloat) : v.options();
    at::Tensor out = at::empty(q.sizes(), opts);
    at::Tensor out_m = at::empty({q.size(0), q.size(1), q.size(2)}, opts);
    at::Tensor out_l = at::empty({q.size(0), q.size(1), q.size(2)}, opts);
    const int dt = pmkl_dtype_of(v.scalar_type());
    const int odt = out_fp32 ? PMKL_DTYPE_F32 : dt;
    cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
    const int rc = pmkl_causal_attention_fwd_strided(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                                                     out_m.data_ptr(), out_l.data_ptr(), B, H, Hkv, S, D, qs, ks, vs,
                                                     nullptr, dt, odt, is_causal ? 1 : 0, static_cast<float>(scale),
                                                     static_cast<int>(kernel), stream);
    TORCH_CHECK(rc == PMKL_OK, "pmkl_causal_attention_fwd failed: ", pmkl_status_string(rc));
    return std::make_tuple(out, out_m, out_l);
}

}  // namespace

// fused_self_attention.cpp:139 -- same name, arguments and return tuple.
std::tuple<at::Tensor, at::Tensor, at::Tensor> fused_self_attention_fw(const at::Tensor &q, const at::Tensor &k,
                                                                       const at::Tensor &v, bool is_causal) {
    return forward_impl(q, k, v, is_causal, false, PMKL_ATTN_AUTO, 0.0, false);
}

// Extra entry (no reference counterpart): fp32 outputs, explicit kernel
// choice and score scale, and k, v with fewer heads than q (grouped-query:
// query head h reads K/V head h / (H / H_kv)).
std::tuple<at::Tensor, at::Tensor, at::Tensor> fused_self_attention_fw_ex(const at::Tensor &q, const at::Tensor &k,
                                                                          const at::Tensor &v, bool is_causal,
                                                                          bool out_fp32, int64_t kernel,
                                                                          double scale) {
    return forward_impl(q, k, v, is_causal, out_fp32, kernel, scale, true);
}

namespace {

std::tuple<at::Tensor, at::Tensor, at::Tensor> backward_impl(const at::Tensor &dout, const at::Tensor &q,
                                                             const at::Tensor &k, const at::Tensor &v,
                                                             const at::Tensor &out_m, const at::Tensor &out_l,
                                                             bool is_causal, int64_t kernel, double scale,
                                                             bool allow_kv_heads) {
    // fused_self_attention.cpp:178-180
    check_inputs(q, k, v, allow_kv_heads);
    TORCH_CHECK(dout.sizes() == q.sizes(), "fused_self_attention_bw: grad_output must have q's shape");
    const std::vector<int64_t> stat_shape = {q.size(0), q.size(1), q.size(2)};
    TORCH_CHECK(out_m.sizes() == stat_shape && out_l.sizes() == stat_shape,
                "fused_self_attention_bw: out_m and out_l must be [batch, heads, seq]");
    for (const at::Tensor *t : {&dout, &out_m, &out_l}) {
        TORCH_CHECK(t->device() == q.device(), "fused_self_attention_bw: all tensors must be on q's device");
        // The reference reads them as v's scalar type (fused_self_attention.cpp:205-209).
        TORCH_CHECK(t->scalar_type() == v.scalar_type(), "fused_self_attention_bw: grad_output, out_m and out_l "
                    "must have v's dtype");
    }
    const c10::cuda::CUDAGuard guard(q.device());
    const int B = static_cast<int>(q.size(0)), H = static_cast<int>(q.size(1));
    const int S = static_cast<int>(q.size(2)), D = static_cast<int>(q.size(3));
    const int Hkv = static_cast<int>(k.size(1));
    // The reference makes its inputs contiguous (fused_self_attention.cpp:179);
    // here views are read in place through their strides and copied only when
    // the hidden dimension itself is strided.
    const auto rows_ok = [](const at::Tensor &t) { return t.size(3) <= 1 || t.stride(3) == 1; };
    const at::Tensor dc = rows_ok(dout) ? dout : dout.contiguous();
    const at::Tensor qc = rows_ok(q) ? q : q.contiguous();
    const at::Tensor kc = rows_ok(k) ? k : k.contiguous();
    const at::Tensor vc = rows_ok(v) ? v : v.contiguous();
    const at::Tensor mc = out_m.contiguous(), lc = out_l.contiguous();
    // Every element is written, so empty (not zeros, :186-188) gives the same
    // result.  The gradients take their inputs' layout (dense views keep their
    // strides) and are written in place through them.
    at::Tensor dq = at::empty_like(qc), dk = at::empty_like(kc), dv = at::empty_like(vc);
    const int dt = pmkl_dtype_of(v.scalar_type());
    const size_t ws_bytes = pmkl_causal_attention_bwd_workspace_size_ex(B, H, S, D, dt, static_cast<int>(kernel));
    at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 1)}, q.options().dtype(at::kByte));
    const auto st = [](const at::Tensor &t) { return std::array<int64_t, 3>{t.stride(0), t.stride(1), t.stride(2)}; };
    const auto sdo = st(dc), sq = st(qc), sk = st(kc), sv = st(vc), sdq = st(dq), sdk = st(dk), sdv = st(dv);
    cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
    const int rc = pmkl_causal_attention_bwd_strided(
        dc.data_ptr(), qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), mc.data_ptr(), lc.data_ptr(), dq.data_ptr(),
        dk.data_ptr(), dv.data_ptr(), B, H, Hkv, S, D, sdo.data(), sq.data(), sk.data(), sv.data(), sdq.data(),
        sdk.data(), sdv.data(), dt, is_causal ? 1 : 0, static_cast<float>(scale), ws.data_ptr(), ws_bytes,
        static_cast<int>(kernel), stream);
    TORCH_CHECK(rc == PMKL_OK, "pmkl_causal_attention_bwd failed: ", pmkl_status_string(rc));
    return std::make_tuple(dq, dk, dv);
}

}  // namespace

// fused_self_attention.cpp:175 -- same name, arguments and return tuple.
std::tuple<at::Tensor, at::Tensor, at::Tensor> fused_self_attention_bw(const at::Tensor &dout, const at::Tensor &q,
                                                                       const at::Tensor &k, const at::Tensor &v,
                                                                       const at::Tensor &out_m,
                                                                       const at::Tensor &out_l, bool is_causal) {
    return backward_impl(dout, q, k, v, out_m, out_l, is_causal, PMKL_ATTN_AUTO, 0.0, false);
}

// Extra entry (no reference counterpart): explicit kernel choice and scale,
// and k, v with fewer heads than q (grouped-query: dk, dv are the sums over
// the query heads that read each K/V head) -- the backward of
// fused_self_attention_fw_ex.
std::tuple<at::Tensor, at::Tensor, at::Tensor> fused_self_attention_bw_ex(
    const at::Tensor &dout, const at::Tensor &q, const at::Tensor &k, const at::Tensor &v, const at::Tensor &out_m,
    const at::Tensor &out_l, bool is_causal, int64_t kernel, double scale) {
    return backward_impl(dout, q, k, v, out_m, out_l, is_causal, kernel, scale, true);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("fused_self_attention_fw", &fused_self_attention_fw, "fused_self_attention_fw");
    m.def("fused_self_attention_bw", &fused_self_attention_bw, "fused_self_attention_bw");
    m.def("fused_self_attention_bw_ex", &fused_self_attention_bw_ex, "fused_self_attention_bw_ex",
          pybind11::arg("dout"), pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("out_m"),
          pybind11::arg("out_l"), pybind11::arg("is_causal"), pybind11::arg("kernel") = 0,
          pybind11::arg("scale") = 0.0);
    m.def("fused_self_attention_fw_ex", &fused_self_attention_fw_ex, "fused_self_attention_fw_ex",
          pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("is_causal"),
          pybind11::arg("out_fp32") = false, pybind11::arg("kernel") = 0, pybind11::arg("scale") = 0.0);
    m.attr("KERNEL_AUTO") = static_cast<int>(PMKL_ATTN_AUTO);
    m.attr("KERNEL_SIMT") = static_cast<int>(PMKL_ATTN_SIMT);
    m.attr("KERNEL_TCGEN05") = static_cast<int>(PMKL_ATTN_TCGEN05);
}
