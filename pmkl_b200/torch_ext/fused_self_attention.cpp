// pmkl_pytorch_ext -- torch binding of the B200 attention kernels.
//
// Keeps the reference extension's module name, function names, argument
// lists, return tuple and error behaviour
// (pmkl_pytorch_ext/fused_self_attention.cpp:139-220), but the compute goes
// through the C ABI of libpmkl_b200 (include/pmkl_b200.h) on the current
// CUDA stream instead of the reference's single-threaded host loops.  There is
// no CPU path: CPU tensors are rejected.
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

void check_inputs(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v) {
    // fused_self_attention.cpp:140-141
    TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "Input tensor shapes must match");
    TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes(), "Input tensor shapes must match");
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
                                                            int64_t kernel, double scale) {
    check_inputs(q, k, v);
    const c10::cuda::CUDAGuard guard(q.device());
    const int B = static_cast<int>(q.size(0)), H = static_cast<int>(q.size(1));
    const int S = static_cast<int>(q.size(2)), D = static_cast<int>(q.size(3));
    // fused_self_attention.cpp:160-162 makes the inputs contiguous.
    const at::Tensor qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
    // Outputs in v's dtype (fused_self_attention.cpp:148-150), contiguous.
    const auto opts = out_fp32 ? v.options().dtype(at::kFloat) : v.options();
    at::Tensor out = at::empty(v.sizes(), opts);
    at::Tensor out_m = at::empty({q.size(0), q.size(1), q.size(2)}, opts);
    at::Tensor out_l = at::empty({q.size(0), q.size(1), q.size(2)}, opts);
    const int dt = pmkl_dtype_of(v.scalar_type());
    const int odt = out_fp32 ? PMKL_DTYPE_F32 : dt;
    cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
    const int rc = pmkl_causal_attention_fwd_ex(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                                                out_m.data_ptr(), out_l.data_ptr(), B, H, S, D, dt, odt,
                                                is_causal ? 1 : 0, static_cast<float>(scale),
                                                static_cast<int>(kernel), stream);
    TORCH_CHECK(rc == PMKL_OK, "pmkl_causal_attention_fwd failed: ", pmkl_status_string(rc));
    return std::make_tuple(out, out_m, out_l);
}

}  // namespace

// fused_self_attention.cpp:139 -- same name, arguments and return tuple.
std::tuple<at::Tensor, at::Tensor, at::Tensor> fused_self_attention_fw(const at::Tensor &q, const at::Tensor &k,
                                                                       const at::Tensor &v, bool is_causal) {
    return forward_impl(q, k, v, is_causal, false, PMKL_ATTN_AUTO, 0.0);
}

// Extra entry (no reference counterpart): fp32 outputs, explicit kernel
// choice and score scale, for parity tests and benchmarks.
std::tuple<at::Tensor, at::Tensor, at::Tensor> fused_self_attention_fw_ex(const at::Tensor &q, const at::Tensor &k,
                                                                          const at::Tensor &v, bool is_causal,
                                                                          bool out_fp32, int64_t kernel,
                                                                          double scale) {
    return forward_impl(q, k, v, is_causal, out_fp32, kernel, scale);
}

// fused_self_attention.cpp:175 -- same name and arguments.  The B200 build
// has no backward kernel yet.
std::tuple<at::Tensor, at::Tensor, at::Tensor> fused_self_attention_bw(const at::Tensor &dout, const at::Tensor &q,
                                                                       const at::Tensor &k, const at::Tensor &v,
                                                                       const at::Tensor &out_m,
                                                                       const at::Tensor &out_l, bool is_causal) {
    TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "Input tensor shapes must match");
    TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes(), "Input tensor shapes must match");
    TORCH_CHECK_NOT_IMPLEMENTED(false, "fused_self_attention_bw: the B200 build has no backward kernel yet");
    return std::make_tuple(at::Tensor(), at::Tensor(), at::Tensor());
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("fused_self_attention_fw", &fused_self_attention_fw, "fused_self_attention_fw");
    m.def("fused_self_attention_bw", &fused_self_attention_bw, "fused_self_attention_bw");
    m.def("fused_self_attention_fw_ex", &fused_self_attention_fw_ex, "fused_self_attention_fw_ex",
          pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("is_causal"),
          pybind11::arg("out_fp32") = false, pybind11::arg("kernel") = 0, pybind11::arg("scale") = 0.0);
    m.attr("KERNEL_AUTO") = static_cast<int>(PMKL_ATTN_AUTO);
    m.attr("KERNEL_SIMT") = static_cast<int>(PMKL_ATTN_SIMT);
    m.attr("KERNEL_TCGEN05") = static_cast<int>(PMKL_ATTN_TCGEN05);
}
