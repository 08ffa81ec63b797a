// pmkl_b200.cu -- C ABI of libpmkl_b200 (declared in include/pmkl_b200.h):
// argument checks, kernel selection, TMA descriptor set-up and launches.
//
// Host-side behaviour follows the reference's entry points:
//   pmkl::nlp::causal_attention_forward   pmkl/nlp/causal_attention.h:258-288
//   fused_self_attention_fw               pmkl_pytorch_ext/fused_self_attention.cpp:139-173
//   pmkl::norm::warp_softmax_forward      pmkl/norm/warp_softmax.h:159-201
// but never synchronises (the reference launcher syncs after every launch,
// pmkl/core/launcher/cuda_launcher.h:334) and never resets the device (the
// reference's launcher does at start-up, cuda_launcher.h:149,273).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <atomic>
#include <mutex>

#include "attention_bwd.cuh"
#include "attention_bwd_simt.cuh"
#include "attention_simt.cuh"
#include "attention_pp.cuh"
#include "attention_tc.cuh"
#include "common.cuh"
#include "pmkl_b200.h"
#include "softmax.cuh"
#include "wait_selftest.cuh"

// K+V bytes per scheduling group of the persistent attention kernel (tuned on
// B200 at config 3: 24 MiB beat 48/96 MiB and no grouping).
#ifndef PMKL_PP_GROUP_BYTES
#define PMKL_PP_GROUP_BYTES (24LL << 20)
#endif

namespace pmkl_b200 {
namespace {

constexpr int kMaxDevices = 64;

// ------------------------------------------------------------------ device checks
struct DeviceState {
    std::once_flag once;
    bool ok = false;
};
DeviceState g_dev[kMaxDevices];

int current_device_ok() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return PMKL_ERR_NO_DEVICE;
    }
    if (dev < 0 || dev >= kMaxDevices) return PMKL_ERR_NO_DEVICE;
    DeviceState &st = g_dev[dev];
    std::call_once(st.once, [&]() {
        int major = 0, minor = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) == cudaSuccess) {
            st.ok = (major == 10 && minor == 0);  // code is built for sm_100a only
        } else {
            cudaGetLastError();
        }
    });
    return st.ok ? PMKL_OK : PMKL_ERR_NO_DEVICE;
}

// Sets a kernel's dynamic shared-memory limit once per device.
template <typename K>
bool ensure_smem(K kernel, int bytes, std::once_flag (&flags)[kMaxDevices]) {
    int dev = 0;
    cudaGetDevice(&dev);
    bool ok = true;
    std::call_once(flags[dev], [&]() {
        ok = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
    });
    return ok;
}

int launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? PMKL_OK : PMKL_ERR_LAUNCH;
}

// ------------------------------------------------------------------ TMA descriptors
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = []() -> EncodeTiledFn {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// [planes, rows, cols] 16-bit tensor, 128-row x 64-column boxes, 128-byte swizzle.
bool make_tile_map(CUtensorMap *map, const void *base, int dtype, int cols, int rows, long long planes) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const CUtensorMapDataType dt =
        dtype == PMKL_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(planes)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 2,
                                   static_cast<cuuint64_t>(cols) * 2 * static_cast<cuuint64_t>(rows)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(tc::kBoxCols), 128u, 1u};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return enc(map, dt, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [batch][heads][rows][cols] 16-bit tensor with element strides st = (batch,
// head, row) and contiguous columns, viewed as 4-D {cols, rows, heads, batch}
// for 128-row x 64-column boxes with the 128-byte swizzle.  A dimension of
// extent 1 is never stepped, so its stride is replaced by a valid one.
bool make_tile_map_4d(CUtensorMap *map, const void *base, int dtype, int cols, int rows, int heads, int batch,
                      const long long (&st)[3]) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const CUtensorMapDataType dt =
        dtype == PMKL_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint64_t row_b = static_cast<cuuint64_t>(st[2]) * 2;
    const cuuint64_t head_b = heads > 1 ? static_cast<cuuint64_t>(st[1]) * 2 : row_b * static_cast<cuuint64_t>(rows);
    const cuuint64_t batch_b =
        batch > 1 ? static_cast<cuuint64_t>(st[0]) * 2 : head_b * static_cast<cuuint64_t>(heads);
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[3] = {row_b, head_b, batch_b};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(tc::kBoxCols), 128u, 1u, 1u};
    const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
    return enc(map, dt, 4, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

AttnLayout contiguous_layout(int H, int S, int D) {
    AttnLayout L;
    L.H = H;
    L.kv_group = 1;
    const long long s3[3] = {static_cast<long long>(H) * S * D, static_cast<long long>(S) * D, D};
    for (int i = 0; i < 3; ++i) L.q[i] = L.k[i] = L.v[i] = L.o[i] = s3[i];
    return L;
}

bool layout_contiguous(const AttnLayout &L, int S, int D) {
    const AttnLayout c = contiguous_layout(L.H, S, D);
    for (int i = 0; i < 3; ++i)
        if (L.q[i] != c.q[i] || L.k[i] != c.k[i] || L.v[i] != c.v[i] || L.o[i] != c.o[i]) return false;
    return L.kv_group == 1;
}

// ------------------------------------------------------------------ attention launchers
template <int D, bool BF16>
int launch_tc(const void *q, const void *k, const void *v, void *o, void *m, void *l, int S, int BH, int causal,
              float scale, int dtype, int out_dtype, cudaStream_t stream) {
    using C = tc::Cfg<D>;
    static std::once_flag smem_once[kMaxDevices];
    auto kernel = tc::attn_fwd_tc_kernel<D, BF16>;
    if (!ensure_smem(kernel, C::kSmemBytes, smem_once)) return PMKL_ERR_LAUNCH;
    CUtensorMap tq, tk, tv, to;
    const bool o16 = out_dtype != PMKL_DTYPE_F32;
    if (!make_tile_map(&tq, q, dtype, D, S, BH) || !make_tile_map(&tk, k, dtype, D, S, BH) ||
        !make_tile_map(&tv, v, dtype, D, S, BH) || !make_tile_map(&to, o16 ? o : q, dtype, D, S, BH))
        return PMKL_ERR_LAUNCH;
    tc::Params p;
    p.S = S;
    p.BH = BH;
    p.n_qt = (S + tc::kBM - 1) / tc::kBM;
    p.causal = causal;
    p.out_dtype = out_dtype;
    p.scale = scale;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.o_f32 = o;
    p.m_out = m;
    p.l_out = l;
    const long long blocks = static_cast<long long>(p.n_qt) * BH;
    if (blocks > 0x7FFFFFFFLL) return PMKL_ERR_INVALID_SHAPE;
    kernel<<<static_cast<unsigned>(blocks), tc::kThreads, C::kSmemBytes, stream>>>(tq, tk, tv, to, p);
    return launch_status();
}

int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 148;
    }
    return n;
}

// The persistent kernel re-splits its registers between warpgroups with
// setmaxnreg; the split only fits when the kernel was built with exactly
// pp::kLaunchRegs registers per thread.  Checked once per process.
template <int D, bool BF16, bool DELTA = false>
bool pp_launchable() {
    static int ok = -1;
    if (ok < 0) {
        cudaFuncAttributes attr;
        ok = (cudaFuncGetAttributes(&attr, pp::attn_fwd_pp_kernel<D, BF16, PMKL_PP_NPOLY, DELTA>) == cudaSuccess &&
              attr.numRegs == pp::kLaunchRegs)
                 ? 1
                 : 0;
        cudaGetLastError();
    }
    return ok == 1;
}

// Backward's use of the persistent forward: instead of O, m, l it writes the
// row statistics (b, delta) from dO and the caller's m~, l~.
struct DeltaArgs {
    const void *dout;
    long long do_s[3];  // element strides of dout (batch, head, row)
    const void *m_given;
    const void *l_given;
    float2 *rowstat;
    int S_pad;
};

template <int D, bool BF16>
int launch_pp(const void *q, const void *k, const void *v, void *o, void *m, void *l, int S, int BH, int causal,
              float scale, int dtype, int out_dtype, const AttnLayout &lay, cudaStream_t stream,
              const DeltaArgs *delta = nullptr) {
    using C = pp::Cfg<D>;
    static std::once_flag smem_once[kMaxDevices];
    static std::once_flag smem_once_delta[kMaxDevices];
    auto kernel = delta ? pp::attn_fwd_pp_kernel<D, BF16, PMKL_PP_NPOLY, true> : pp::attn_fwd_pp_kernel<D, BF16>;
    if (!ensure_smem(kernel, C::kSmemBytes, delta ? smem_once_delta : smem_once)) return PMKL_ERR_LAUNCH;
    CUtensorMap tq, tk, tv, to;
    const bool o16 = out_dtype != PMKL_DTYPE_F32;
    const int B = BH / lay.H, Hkv = lay.H / lay.kv_group;
    if (!make_tile_map_4d(&tq, q, dtype, D, S, lay.H, B, lay.q) ||
        !make_tile_map_4d(&tk, k, dtype, D, S, Hkv, B, lay.k) ||
        !make_tile_map_4d(&tv, v, dtype, D, S, Hkv, B, lay.v) ||
        !make_tile_map_4d(&to, o16 ? o : q, dtype, D, S, lay.H, B, o16 ? lay.o : lay.q))
        return PMKL_ERR_LAUNCH;
    pp::Params p;
    p.S = S;
    p.BH = BH;
    p.H = lay.H;
    p.kv_group = lay.kv_group;
    p.o_sb = lay.o[0];
    p.o_sh = lay.o[1];
    p.o_ss = lay.o[2];
    const int n_qt = (S + 127) / 128;
    p.n_pairs = (n_qt + 1) / 2;
    const long long units = static_cast<long long>(p.n_pairs) * BH;
    if (units > 0x7FFFFFFFLL) return PMKL_ERR_INVALID_SHAPE;
    p.n_units = static_cast<int>(units);
    // Slices per scheduling group: K and V of a group stay within
    // PMKL_PP_GROUP_BYTES of the 126 MB L2, at least one slice.
    const long long kv_bytes = 2LL * S * D * 2;
    long long grp = PMKL_PP_GROUP_BYTES / (kv_bytes > 0 ? kv_bytes : 1);
    if (grp < 1) grp = 1;
    // Small problems (all slices' K and V within about one and a half L2s, as a
    // GPU's shard of config 3 on 8 GPUs): one longest-first list over every
    // slice balances the SMs better than L2-sized groups, whose repeated
    // long-to-short runs leave SMs idle at the end (B200, 64 slices of config
    // 3: 851 vs 779 TFLOP/s; at 128 slices the groups still win, 875 vs 827).
    if (kv_bytes * BH <= 8LL * PMKL_PP_GROUP_BYTES) grp = BH;
    if (grp > BH) grp = BH;
    p.group = static_cast<int>(grp);
    // One longest-first list: hand out odd rounds in reverse CTA order; L2
    // groups: alternate the direction of consecutive groups instead (B200,
    // simulated max / mean CTA load, config 3: 1.025 -> 1.016; config 4:
    // 1.106 -> 1.030; a 64-slice shard of config 3: 1.132 -> 1.020).
    p.snake = grp == BH ? 1 : 0;
    p.flip = grp == BH ? 0 : 1;
    p.causal = causal;
    p.out_dtype = out_dtype;
    p.scale = scale;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.o_f32 = o;
    p.m_out = m;
    p.l_out = l;
    pp::DeltaParams dp{};
    if (delta) {
        dp.S_pad = delta->S_pad;
        dp.dout = delta->dout;
        for (int i = 0; i < 3; ++i) dp.do_s[i] = delta->do_s[i];
        dp.m_given = delta->m_given;
        dp.l_given = delta->l_given;
        dp.rowstat = delta->rowstat;
    }
    const int grid = static_cast<int>(units < sm_count() ? units : sm_count());
    p.n_rounds = static_cast<int>((units + grid - 1) / grid);
    kernel<<<grid, pp::kThreads, C::kSmemBytes, stream>>>(tq, tk, tv, to, p, dp);
    return launch_status();
}

template <typename T, int DMAX>
int launch_simt_t(const void *q, const void *k, const void *v, void *o, void *m, void *l, int S, int D, int BH,
                  int causal, float scale, int out_dtype, const AttnLayout &lay, cudaStream_t stream) {
    static std::once_flag smem_once[kMaxDevices];
    auto kernel = simt::attn_fwd_simt_kernel<T, DMAX>;
    constexpr int smem = simt::smem_bytes<DMAX>();
    if (!ensure_smem(kernel, smem, smem_once)) return PMKL_ERR_LAUNCH;
    const int n_qt = (S + simt::kBM - 1) / simt::kBM;
    const long long blocks = static_cast<long long>(n_qt) * BH;
    if (blocks > 0x7FFFFFFFLL) return PMKL_ERR_INVALID_SHAPE;
    kernel<<<static_cast<unsigned>(blocks), simt::kThreads, smem, stream>>>(
        static_cast<const T *>(q), static_cast<const T *>(k), static_cast<const T *>(v), o, m, l, S, D, BH, n_qt,
        causal, scale, out_dtype, lay);
    return launch_status();
}

template <typename T>
int launch_simt(const void *q, const void *k, const void *v, void *o, void *m, void *l, int S, int D, int BH,
                int causal, float scale, int out_dtype, const AttnLayout &lay, cudaStream_t stream) {
    if (D <= 32) return launch_simt_t<T, 32>(q, k, v, o, m, l, S, D, BH, causal, scale, out_dtype, lay, stream);
    if (D <= 64) return launch_simt_t<T, 64>(q, k, v, o, m, l, S, D, BH, causal, scale, out_dtype, lay, stream);
    if (D <= 128) return launch_simt_t<T, 128>(q, k, v, o, m, l, S, D, BH, causal, scale, out_dtype, lay, stream);
    return launch_simt_t<T, 256>(q, k, v, o, m, l, S, D, BH, causal, scale, out_dtype, lay, stream);
}

// The tensor-core kernels read q, k, v (and write a 16-bit o) through TMA:
// 16-byte aligned bases and strides that are multiples of 16 bytes; an fp32 o
// is written with 16-byte vector stores.
bool strides_ok(const long long (&s)[3], int elems_per_16b) {
    for (long long x : s)
        if (x < 0 || x % elems_per_16b != 0 || x >= (1LL << 38)) return false;
    return true;
}

bool tc_applies(const void *q, const void *k, const void *v, const void *o, int D, int dtype, int out_dtype,
                const AttnLayout &lay) {
    if (dtype != PMKL_DTYPE_F16 && dtype != PMKL_DTYPE_BF16) return false;
    if (D != 64 && D != 128) return false;
    if (out_dtype != dtype && out_dtype != PMKL_DTYPE_F32) return false;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return false;
    if (!strides_ok(lay.q, 8) || !strides_ok(lay.k, 8) || !strides_ok(lay.v, 8)) return false;
    if (!strides_ok(lay.o, out_dtype == PMKL_DTYPE_F32 ? 4 : 8)) return false;
    return true;
}

// Which kernel runs: the persistent tensor-core kernel when it applies (and
// its register split is available), the one-tile tensor-core kernel when
// asked for or as the fallback, else the CUDA-core kernel.
int select_kernel(const void *q, const void *k, const void *v, const void *o, int hidden, int S, int dtype,
                  int out_dtype, int kernel, const AttnLayout &lay) {
    const bool tc_ok = tc_applies(q, k, v, o, hidden, dtype, out_dtype, lay);
    // The one-tile kernel reads contiguous [B*H, S, D] tensors only.
    const bool simple_ok = tc_ok && layout_contiguous(lay, S, hidden);
    if ((kernel == PMKL_ATTN_TCGEN05 || kernel == PMKL_ATTN_TCGEN05_SIMPLE) && !tc_ok) return PMKL_ERR_UNSUPPORTED;
    if (kernel == PMKL_ATTN_TCGEN05_SIMPLE && !simple_ok) return PMKL_ERR_UNSUPPORTED;
    if (kernel == PMKL_ATTN_SIMT || !tc_ok) return PMKL_ATTN_SIMT;
    if (kernel == PMKL_ATTN_TCGEN05_SIMPLE) return PMKL_ATTN_TCGEN05_SIMPLE;
    const bool bf = dtype == PMKL_DTYPE_BF16;
    const bool ready = hidden == 64 ? (bf ? pp_launchable<64, true>() : pp_launchable<64, false>())
                                    : (bf ? pp_launchable<128, true>() : pp_launchable<128, false>());
    if (ready) return PMKL_ATTN_TCGEN05;
    // Only a build whose persistent kernel did not get its launch register
    // count lands here; say so once, since the fallback costs ~40 %.
    static std::once_flag warned;
    std::call_once(warned, []() {
        std::fprintf(stderr,
                     "pmkl_b200: the persistent tensor-core attention kernel cannot take its register split in "
                     "this build; falling back to a slower kernel (pmkl_attention_selected_kernel reports which)\n");
    });
    return simple_ok ? PMKL_ATTN_TCGEN05_SIMPLE : PMKL_ATTN_SIMT;
}

int attention_impl(const void *q, const void *k, const void *v, void *o, void *m, void *l, int batch, int heads,
                   int seq, int hidden, int dtype, int out_dtype, int is_causal, float scale, int kernel,
                   void *stream_, const AttnLayout *layout = nullptr) {
    if (batch < 0 || heads < 0 || seq < 0 || hidden < 0) return PMKL_ERR_INVALID_SHAPE;
    if (!dtype_valid(dtype) || !dtype_valid(out_dtype)) return PMKL_ERR_INVALID_DTYPE;
    if (out_dtype != dtype && out_dtype != PMKL_DTYPE_F32) return PMKL_ERR_INVALID_DTYPE;
    if (kernel != PMKL_ATTN_AUTO && kernel != PMKL_ATTN_SIMT && kernel != PMKL_ATTN_TCGEN05 &&
        kernel != PMKL_ATTN_TCGEN05_SIMPLE)
        return PMKL_ERR_UNSUPPORTED;
    const long long BH = static_cast<long long>(batch) * heads;
    if (BH == 0 || seq == 0 || hidden == 0) return PMKL_OK;  // causal_attention.h:270
    if (hidden > 256) return PMKL_ERR_UNSUPPORTED;
    if (BH > 0x7FFFFFFFLL) return PMKL_ERR_INVALID_SHAPE;
    if (!q || !k || !v || !o || !m || !l) return PMKL_ERR_NULL_POINTER;
    const int dev_rc = current_device_ok();
    if (dev_rc != PMKL_OK) return dev_rc;
    const float sc = (scale > 0.f) ? scale : 1.0f / sqrtf(static_cast<float>(hidden));
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const int causal = is_causal ? 1 : 0;
    const AttnLayout lay = layout ? *layout : contiguous_layout(heads, seq, hidden);
    const int chosen = select_kernel(q, k, v, o, hidden, seq, dtype, out_dtype, kernel, lay);
    if (chosen < 0) return chosen;
    if (chosen == PMKL_ATTN_TCGEN05) {
        const int bh = static_cast<int>(BH);
        if (dtype == PMKL_DTYPE_BF16)
            return hidden == 64
                       ? launch_pp<64, true>(q, k, v, o, m, l, seq, bh, causal, sc, dtype, out_dtype, lay, stream)
                       : launch_pp<128, true>(q, k, v, o, m, l, seq, bh, causal, sc, dtype, out_dtype, lay, stream);
        return hidden == 64
                   ? launch_pp<64, false>(q, k, v, o, m, l, seq, bh, causal, sc, dtype, out_dtype, lay, stream)
                   : launch_pp<128, false>(q, k, v, o, m, l, seq, bh, causal, sc, dtype, out_dtype, lay, stream);
    }
    if (chosen == PMKL_ATTN_TCGEN05_SIMPLE) {
        const int bh = static_cast<int>(BH);
        if (dtype == PMKL_DTYPE_BF16)
            return hidden == 64 ? launch_tc<64, true>(q, k, v, o, m, l, seq, bh, causal, sc, dtype, out_dtype, stream)
                                : launch_tc<128, true>(q, k, v, o, m, l, seq, bh, causal, sc, dtype, out_dtype, stream);
        return hidden == 64 ? launch_tc<64, false>(q, k, v, o, m, l, seq, bh, causal, sc, dtype, out_dtype, stream)
                            : launch_tc<128, false>(q, k, v, o, m, l, seq, bh, causal, sc, dtype, out_dtype, stream);
    }
    const int bh = static_cast<int>(BH);
    if (dtype == PMKL_DTYPE_F32)
        return launch_simt<float>(q, k, v, o, m, l, seq, hidden, bh, causal, sc, out_dtype, lay, stream);
    if (dtype == PMKL_DTYPE_F16)
        return launch_simt<__half>(q, k, v, o, m, l, seq, hidden, bh, causal, sc, out_dtype, lay, stream);
    return launch_simt<__nv_bfloat16>(q, k, v, o, m, l, seq, hidden, bh, causal, sc, out_dtype, lay, stream);
}

// ------------------------------------------------------------------ backward
size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace of the tensor-core backward: the per-row (b, delta) pairs at a
// row pitch of S rounded up to 128 come first -- the fused route (delta from
// the persistent forward's epilogue) needs nothing else -- followed by the
// fp32 O, m, l that only the long route (a forward with fp32 outputs, then the
// row-statistics kernel) writes.
struct BwdLayout {
    size_t rowstat, o, m, l;
    size_t fused_total;  // bytes the fused route needs
    size_t total;        // bytes the long route needs
    int S_pad;
};

BwdLayout bwd_layout_tc(long long BH, int S, int D) {
    BwdLayout L;
    L.S_pad = ((S + 127) / 128) * 128;
    size_t off = 0;
    L.rowstat = off;
    off = align256(off + static_cast<size_t>(BH) * L.S_pad * 8);
    L.fused_total = off;
    L.o = off;
    off = align256(off + static_cast<size_t>(BH) * S * D * 4);
    L.m = off;
    off = align256(off + static_cast<size_t>(BH) * S * 4);
    L.l = off;
    off = align256(off + static_cast<size_t>(BH) * S * 4);
    L.total = off;
    return L;
}

// Workspace of the CUDA-core backward: delta per row.
size_t bwd_ws_simt(long long BH, int S) { return align256(static_cast<size_t>(BH) * S * 4); }

bool bwd_tc_applies(const void *const (&ptrs)[9], int D, int dtype, const AttnBwdLayout &lay) {
    if (dtype != PMKL_DTYPE_F16 && dtype != PMKL_DTYPE_BF16) return false;
    if (D != 64 && D != 128) return false;
    for (const void *p : ptrs)
        if (!aligned16(p)) return false;
    // TMA: every stride a multiple of 16 bytes.
    for (const auto *st : {&lay.dout, &lay.q, &lay.k, &lay.v, &lay.dq, &lay.dk, &lay.dv})
        if (!strides_ok(*st, 8)) return false;
    return true;
}

template <typename T>
int launch_bwd_rowstat(const void *dout, const float *o32, const float *m32, const float *l32, const void *m_in,
                       const void *l_in, float2 *rowstat, int S, int S_pad, int D, long long BH,
                       cudaStream_t stream) {
    const long long n_rows = BH * S_pad;
    long long blocks = (n_rows + 7) / 8;
    const long long cap = static_cast<long long>(sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    bwd::bwd_rowstat_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T *>(dout), o32, m32, l32, m_in, l_in, rowstat, S, S_pad, D, n_rows);
    return launch_status();
}

template <int D, bool BF16>
int launch_bwd_tc(const void *dout, const void *q, const void *k, const void *v, void *dq, void *dk, void *dv, int S,
                  int BH, int causal, float scale, int dtype, const float2 *rowstat, int S_pad,
                  const AttnBwdLayout &lay, cudaStream_t stream) {
    static std::once_flag once_q[kMaxDevices], once_kv[kMaxDevices];
    auto kq = bwd::attn_bwd_dq_kernel<D, BF16>;
    auto kkv = bwd::attn_bwd_dkv_kernel<D, BF16>;
    constexpr int smem_q = bwd::CfgQ<D>::kSmemBytes;
    constexpr int smem_kv = bwd::CfgKV<D>::kSmemBytes;
    if (!ensure_smem(kq, smem_q, once_q) || !ensure_smem(kkv, smem_kv, once_kv)) return PMKL_ERR_LAUNCH;
    const int B = BH / lay.H, Hkv = lay.H / lay.kv_group;
    CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
    if (!make_tile_map_4d(&tq, q, dtype, D, S, lay.H, B, lay.q) ||
        !make_tile_map_4d(&tk, k, dtype, D, S, Hkv, B, lay.k) ||
        !make_tile_map_4d(&tv, v, dtype, D, S, Hkv, B, lay.v) ||
        !make_tile_map_4d(&tdo, dout, dtype, D, S, lay.H, B, lay.dout) ||
        !make_tile_map_4d(&tdq, dq, dtype, D, S, lay.H, B, lay.dq) ||
        !make_tile_map_4d(&tdk, dk, dtype, D, S, Hkv, B, lay.dk) ||
        !make_tile_map_4d(&tdv, dv, dtype, D, S, Hkv, B, lay.dv))
        return PMKL_ERR_LAUNCH;
    bwd::Params p;
    p.S = S;
    p.S_pad = S_pad;
    p.BH = BH;
    p.H = lay.H;
    p.kv_group = lay.kv_group;
    p.BHkv = B * Hkv;
    p.n_qt = (S + 127) / 128;
    p.causal = causal;
    p.scale = scale;
    p.scale_log2 = scale * bwd::kLog2e;
    p.rowstat = rowstat;
    const long long blocks_q = static_cast<long long>(p.n_qt) * BH;
    const long long blocks_kv = static_cast<long long>(p.n_qt) * p.BHkv;
    if (blocks_q > 0x7FFFFFFFLL) return PMKL_ERR_INVALID_SHAPE;
    kq<<<static_cast<unsigned>(blocks_q), bwd::kThreads, smem_q, stream>>>(tq, tk, tv, tdo, tdq, p);
    const int rc = launch_status();
    if (rc != PMKL_OK) return rc;
    kkv<<<static_cast<unsigned>(blocks_kv), bwd::kThreads, smem_kv, stream>>>(tq, tk, tv, tdo, tdk, tdv, p);
    return launch_status();
}

template <typename T, int DMAX>
int launch_bwd_simt_t(const void *dout, const void *q, const void *k, const void *v, const void *m, const void *l,
                      void *dq, void *dk, void *dv, float *delta, int S, int D, int BH, int causal, float scale,
                      const AttnBwdLayout &lay, cudaStream_t stream) {
    static std::once_flag once_q[kMaxDevices], once_kv[kMaxDevices];
    auto kq = simt::attn_bwd_simt_q_kernel<T, DMAX>;
    auto kkv = simt::attn_bwd_simt_kv_kernel<T, DMAX>;
    constexpr int smem = simt::bwd_smem_bytes<DMAX>();
    if (!ensure_smem(kq, smem, once_q) || !ensure_smem(kkv, smem, once_kv)) return PMKL_ERR_LAUNCH;
    const int n_t = (S + 31) / 32;
    const int BHkv = BH / lay.kv_group;
    const long long blocks = static_cast<long long>(n_t) * BH;
    const long long blocks_kv = static_cast<long long>(n_t) * BHkv;
    if (blocks > 0x7FFFFFFFLL) return PMKL_ERR_INVALID_SHAPE;
    const T *tdo = static_cast<const T *>(dout), *tq = static_cast<const T *>(q), *tk = static_cast<const T *>(k),
            *tv = static_cast<const T *>(v), *tm = static_cast<const T *>(m), *tl = static_cast<const T *>(l);
    kq<<<static_cast<unsigned>(blocks), simt::kThreads, smem, stream>>>(tdo, tq, tk, tv, tm, tl, static_cast<T *>(dq),
                                                                        delta, S, D, BH, n_t, causal, scale, lay);
    const int rc = launch_status();
    if (rc != PMKL_OK) return rc;
    kkv<<<static_cast<unsigned>(blocks_kv), simt::kThreads, smem, stream>>>(
        tdo, tq, tk, tv, tm, tl, delta, static_cast<T *>(dk), static_cast<T *>(dv), S, D, BHkv, causal, scale, lay);
    return launch_status();
}

template <typename T>
int launch_bwd_simt(const void *dout, const void *q, const void *k, const void *v, const void *m, const void *l,
                    void *dq, void *dk, void *dv, float *delta, int S, int D, int BH, int causal, float scale,
                    const AttnBwdLayout &lay, cudaStream_t stream) {
    if (D <= 32)
        return launch_bwd_simt_t<T, 32>(dout, q, k, v, m, l, dq, dk, dv, delta, S, D, BH, causal, scale, lay, stream);
    if (D <= 64)
        return launch_bwd_simt_t<T, 64>(dout, q, k, v, m, l, dq, dk, dv, delta, S, D, BH, causal, scale, lay, stream);
    if (D <= 128)
        return launch_bwd_simt_t<T, 128>(dout, q, k, v, m, l, dq, dk, dv, delta, S, D, BH, causal, scale, lay, stream);
    return launch_bwd_simt_t<T, 256>(dout, q, k, v, m, l, dq, dk, dv, delta, S, D, BH, causal, scale, lay, stream);
}

AttnBwdLayout contiguous_bwd_layout(int H, int S, int D) {
    AttnBwdLayout L;
    L.H = H;
    L.kv_group = 1;
    const long long s3[3] = {static_cast<long long>(H) * S * D, static_cast<long long>(S) * D, D};
    for (int i = 0; i < 3; ++i) L.dout[i] = L.q[i] = L.k[i] = L.v[i] = L.dq[i] = L.dk[i] = L.dv[i] = s3[i];
    return L;
}

bool bwd_layout_contiguous(const AttnBwdLayout &L, int S, int D) {
    const AttnBwdLayout c = contiguous_bwd_layout(L.H, S, D);
    for (int i = 0; i < 3; ++i)
        if (L.dout[i] != c.dout[i] || L.q[i] != c.q[i] || L.k[i] != c.k[i] || L.v[i] != c.v[i] ||
            L.dq[i] != c.dq[i] || L.dk[i] != c.dk[i] || L.dv[i] != c.dv[i])
            return false;
    return L.kv_group == 1;
}

// Scratch of pmkl_causal_attention_bwd_static: static device memory of this
// module, never allocated or freed by a call.  Every device on which the
// module is loaded holds it, whichever entry points the caller uses.
__device__ __align__(256) uint8_t g_bwd_static_scratch[PMKL_BWD_STATIC_SCRATCH_BYTES];

// Address of the scratch on each device, looked up with that device current.
// Only a successful lookup is kept: a failed one is tried again next call.
std::atomic<void *> g_static_scratch[kMaxDevices];

void *static_scratch() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return nullptr;
    }
    void *p = g_static_scratch[dev].load(std::memory_order_acquire);
    if (p) return p;
    if (cudaGetSymbolAddress(&p, g_bwd_static_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return nullptr;
    }
    g_static_scratch[dev].store(p, std::memory_order_release);
    return p;
}

// Workspace bytes of the backward route that `kernel` selects for these sizes:
// the fused tensor-core route (AUTO, TCGEN05) needs the row statistics only,
// the long route (TCGEN05_SIMPLE) also the forward's fp32 O, m, l, and the
// CUDA-core route one fp32 delta per row.
size_t bwd_workspace_size(long long BH, int S, int D, int dtype, int kernel) {
    const bool tc_shape = (dtype == PMKL_DTYPE_F16 || dtype == PMKL_DTYPE_BF16) && (D == 64 || D == 128);
    const size_t simt_bytes = bwd_ws_simt(BH, S);
    if (!tc_shape || kernel == PMKL_ATTN_SIMT) return simt_bytes;
    const BwdLayout L = bwd_layout_tc(BH, S, D);
    const size_t tc_bytes = kernel == PMKL_ATTN_TCGEN05_SIMPLE ? L.total : L.fused_total;
    return tc_bytes > simt_bytes ? tc_bytes : simt_bytes;
}

int attention_bwd_impl(const void *dout, const void *q, const void *k, const void *v, const void *m, const void *l,
                       void *dq, void *dk, void *dv, int batch, int heads, int seq, int hidden, int dtype,
                       int is_causal, float scale, void *workspace, size_t workspace_bytes, int kernel,
                       void *stream_, const AttnBwdLayout *layout = nullptr) {
    if (batch < 0 || heads < 0 || seq < 0 || hidden < 0) return PMKL_ERR_INVALID_SHAPE;
    if (!dtype_valid(dtype)) return PMKL_ERR_INVALID_DTYPE;
    if (kernel != PMKL_ATTN_AUTO && kernel != PMKL_ATTN_SIMT && kernel != PMKL_ATTN_TCGEN05 &&
        kernel != PMKL_ATTN_TCGEN05_SIMPLE)
        return PMKL_ERR_UNSUPPORTED;
    const long long BH = static_cast<long long>(batch) * heads;
    if (BH == 0 || seq == 0 || hidden == 0) return PMKL_OK;
    if (hidden > 256) return PMKL_ERR_UNSUPPORTED;
    if (BH > 0x7FFFFFFFLL) return PMKL_ERR_INVALID_SHAPE;
    if (!dout || !q || !k || !v || !m || !l || !dq || !dk || !dv || !workspace) return PMKL_ERR_NULL_POINTER;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return PMKL_ERR_MISALIGNED;
    const int dev_rc = current_device_ok();
    if (dev_rc != PMKL_OK) return dev_rc;
    const float sc = (scale > 0.f) ? scale : 1.0f / sqrtf(static_cast<float>(hidden));
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const int causal = is_causal ? 1 : 0;
    const int bh = static_cast<int>(BH);
    const AttnBwdLayout lay = layout ? *layout : contiguous_bwd_layout(heads, seq, hidden);
    const bool contiguous = bwd_layout_contiguous(lay, seq, hidden);
    const void *const ptrs[9] = {dout, q, k, v, m, l, dq, dk, dv};
    const bool tc_ok = bwd_tc_applies(ptrs, hidden, dtype, lay);
    if ((kernel == PMKL_ATTN_TCGEN05 || kernel == PMKL_ATTN_TCGEN05_SIMPLE) && !tc_ok) return PMKL_ERR_UNSUPPORTED;
    // The long route's forward and row-statistics kernel read contiguous,
    // equal-head tensors only.
    if (kernel == PMKL_ATTN_TCGEN05_SIMPLE && !contiguous) return PMKL_ERR_UNSUPPORTED;
    const bool bf = dtype == PMKL_DTYPE_BF16;
    // delta = sum_j p dP comes from this library's forward through dO . O: the
    // persistent kernel forms it in its epilogue (O never leaves tensor
    // memory; the fused route); otherwise a forward with fp32 O, m, l and the
    // row-statistics kernel (the long route, which needs the larger workspace).
    const bool fused = tc_ok && kernel != PMKL_ATTN_TCGEN05_SIMPLE && kernel != PMKL_ATTN_SIMT &&
                       (hidden == 64 ? (bf ? pp_launchable<64, true, true>() : pp_launchable<64, false, true>())
                                     : (bf ? pp_launchable<128, true, true>() : pp_launchable<128, false, true>()));
    const BwdLayout L = bwd_layout_tc(BH, seq, hidden);
    // Without the fused route (a build whose persistent kernel cannot take its
    // register split) the automatic choice takes the long route when the
    // workspace holds it and the CUDA-core route otherwise, so that the size
    // pmkl_causal_attention_bwd_workspace_size reports always suffices.
    const bool tc_route = tc_ok && kernel != PMKL_ATTN_SIMT &&
                          (fused || (contiguous && (kernel != PMKL_ATTN_AUTO || workspace_bytes >= L.total)));
    if (kernel == PMKL_ATTN_TCGEN05 && !tc_route) return PMKL_ERR_UNSUPPORTED;
    if (tc_route) {
        if (workspace_bytes < (fused ? L.fused_total : L.total)) return PMKL_ERR_WORKSPACE;
        uint8_t *ws = static_cast<uint8_t *>(workspace);
        float2 *rowstat = reinterpret_cast<float2 *>(ws + L.rowstat);
        int rc;
        if (fused) {
            const DeltaArgs da{dout, {lay.dout[0], lay.dout[1], lay.dout[2]}, m, l, rowstat, L.S_pad};
            // The forward reads q, k, v through their strides; it writes no O.
            AttnLayout fl;
            fl.H = lay.H;
            fl.kv_group = lay.kv_group;
            for (int i = 0; i < 3; ++i) {
                fl.q[i] = fl.o[i] = lay.q[i];
                fl.k[i] = lay.k[i];
                fl.v[i] = lay.v[i];
            }
            rc = hidden == 64
                     ? (bf ? launch_pp<64, true>(q, k, v, const_cast<void *>(q), nullptr, nullptr, seq, bh, causal, sc,
                                                 dtype, dtype, fl, stream, &da)
                           : launch_pp<64, false>(q, k, v, const_cast<void *>(q), nullptr, nullptr, seq, bh, causal, sc,
                                                  dtype, dtype, fl, stream, &da))
                     : (bf ? launch_pp<128, true>(q, k, v, const_cast<void *>(q), nullptr, nullptr, seq, bh, causal, sc,
                                                  dtype, dtype, fl, stream, &da)
                           : launch_pp<128, false>(q, k, v, const_cast<void *>(q), nullptr, nullptr, seq, bh, causal,
                                                   sc, dtype, dtype, fl, stream, &da));
        } else {
            float *o32 = reinterpret_cast<float *>(ws + L.o);
            float *m32 = reinterpret_cast<float *>(ws + L.m);
            float *l32 = reinterpret_cast<float *>(ws + L.l);
            rc = attention_impl(q, k, v, o32, m32, l32, batch, heads, seq, hidden, dtype, PMKL_DTYPE_F32, causal, sc,
                                kernel == PMKL_ATTN_TCGEN05_SIMPLE ? PMKL_ATTN_TCGEN05_SIMPLE : PMKL_ATTN_AUTO,
                                stream_);
            if (rc != PMKL_OK) return rc;
            rc = bf ? launch_bwd_rowstat<__nv_bfloat16>(dout, o32, m32, l32, m, l, rowstat, seq, L.S_pad, hidden, BH,
                                                        stream)
                    : launch_bwd_rowstat<__half>(dout, o32, m32, l32, m, l, rowstat, seq, L.S_pad, hidden, BH, stream);
        }
        if (rc != PMKL_OK) return rc;
        if (dtype == PMKL_DTYPE_BF16)
            return hidden == 64 ? launch_bwd_tc<64, true>(dout, q, k, v, dq, dk, dv, seq, bh, causal, sc, dtype,
                                                          rowstat, L.S_pad, lay, stream)
                                : launch_bwd_tc<128, true>(dout, q, k, v, dq, dk, dv, seq, bh, causal, sc, dtype,
                                                           rowstat, L.S_pad, lay, stream);
        return hidden == 64 ? launch_bwd_tc<64, false>(dout, q, k, v, dq, dk, dv, seq, bh, causal, sc, dtype, rowstat,
                                                       L.S_pad, lay, stream)
                            : launch_bwd_tc<128, false>(dout, q, k, v, dq, dk, dv, seq, bh, causal, sc, dtype, rowstat,
                                                        L.S_pad, lay, stream);
    }
    if (workspace_bytes < bwd_ws_simt(BH, seq)) return PMKL_ERR_WORKSPACE;
    float *delta = static_cast<float *>(workspace);
    if (dtype == PMKL_DTYPE_F32)
        return launch_bwd_simt<float>(dout, q, k, v, m, l, dq, dk, dv, delta, seq, hidden, bh, causal, sc, lay, stream);
    if (dtype == PMKL_DTYPE_F16)
        return launch_bwd_simt<__half>(dout, q, k, v, m, l, dq, dk, dv, delta, seq, hidden, bh, causal, sc, lay,
                                       stream);
    return launch_bwd_simt<__nv_bfloat16>(dout, q, k, v, m, l, dq, dk, dv, delta, seq, hidden, bh, causal, sc, lay,
                                          stream);
}

// ------------------------------------------------------------------ softmax launchers
template <bool LOG>
int launch_softmax_vec(float *dst, const float *src, int elements, int stride, int rows, cudaStream_t stream) {
    const int vpl = (elements + 127) / 128;
    const unsigned blocks = static_cast<unsigned>((rows + softmax::kThreads / 32 - 1) / (softmax::kThreads / 32));
#define PMKL_SOFTMAX_VEC_CASE(N)                                                                     \
    case N:                                                                                          \
        softmax::softmax_vec_kernel<N, LOG><<<blocks, softmax::kThreads, 0, stream>>>(dst, src, elements, \
                                                                                      stride, rows); \
        break;
    switch (vpl) {
        PMKL_SOFTMAX_VEC_CASE(1)
        PMKL_SOFTMAX_VEC_CASE(2)
        PMKL_SOFTMAX_VEC_CASE(3)
        PMKL_SOFTMAX_VEC_CASE(4)
        PMKL_SOFTMAX_VEC_CASE(5)
        PMKL_SOFTMAX_VEC_CASE(6)
        PMKL_SOFTMAX_VEC_CASE(7)
        PMKL_SOFTMAX_VEC_CASE(8)
        default:
            return PMKL_ERR_INVALID_SHAPE;
    }
#undef PMKL_SOFTMAX_VEC_CASE
    return launch_status();
}

template <typename TI, typename TO, bool LOG>
int launch_softmax_vec8_t(void *dst, const void *src, int elements, int stride, int rows, cudaStream_t stream) {
    const int v8 = (elements + 255) / 256;
    const unsigned blocks = static_cast<unsigned>((rows + softmax::kThreads / 32 - 1) / (softmax::kThreads / 32));
    TO *d = static_cast<TO *>(dst);
    const TI *s = static_cast<const TI *>(src);
    switch (v8) {
        case 1:
            softmax::softmax_vec8_kernel<TI, TO, 1, LOG><<<blocks, softmax::kThreads, 0, stream>>>(d, s, elements, stride, rows);
            break;
        case 2:
            softmax::softmax_vec8_kernel<TI, TO, 2, LOG><<<blocks, softmax::kThreads, 0, stream>>>(d, s, elements, stride, rows);
            break;
        case 3:
            softmax::softmax_vec8_kernel<TI, TO, 3, LOG><<<blocks, softmax::kThreads, 0, stream>>>(d, s, elements, stride, rows);
            break;
        case 4:
            softmax::softmax_vec8_kernel<TI, TO, 4, LOG><<<blocks, softmax::kThreads, 0, stream>>>(d, s, elements, stride, rows);
            break;
        default:
            return PMKL_ERR_INVALID_SHAPE;
    }
    return launch_status();
}

template <typename TI, bool LOG>
int launch_softmax_vec8_out(void *dst, const void *src, int elements, int stride, int rows, int out_dtype,
                            cudaStream_t stream) {
    if (out_dtype == PMKL_DTYPE_F32) return launch_softmax_vec8_t<TI, float, LOG>(dst, src, elements, stride, rows, stream);
    if (out_dtype == PMKL_DTYPE_F16) return launch_softmax_vec8_t<TI, __half, LOG>(dst, src, elements, stride, rows, stream);
    return launch_softmax_vec8_t<TI, __nv_bfloat16, LOG>(dst, src, elements, stride, rows, stream);
}

template <bool LOG>
int launch_softmax_vec8(void *dst, const void *src, int elements, int stride, int rows, int in_dtype, int out_dtype,
                        cudaStream_t stream) {
    if (in_dtype == PMKL_DTYPE_F32)
        return launch_softmax_vec8_out<float, LOG>(dst, src, elements, stride, rows, out_dtype, stream);
    if (in_dtype == PMKL_DTYPE_F16)
        return launch_softmax_vec8_out<__half, LOG>(dst, src, elements, stride, rows, out_dtype, stream);
    return launch_softmax_vec8_out<__nv_bfloat16, LOG>(dst, src, elements, stride, rows, out_dtype, stream);
}

template <bool LOG>
int launch_softmax_gen(void *dst, const void *src, int elements, int stride, int rows, int in_dtype, int out_dtype,
                       cudaStream_t stream) {
    int l2e = 0;
    while ((1 << l2e) < elements) ++l2e;  // log2_ceil, warp_softmax.h:25-29
    const int lanes = (1 << l2e) < 32 ? (1 << l2e) : 32;
    const long long rows_per_block = static_cast<long long>(softmax::kThreads / 32) * (32 / lanes);
    const unsigned blocks = static_cast<unsigned>((rows + rows_per_block - 1) / rows_per_block);
#define PMKL_SOFTMAX_GEN_CASE(L)                                                                           \
    case L:                                                                                                \
        softmax::softmax_gen_kernel<L, LOG><<<blocks, softmax::kThreads, 0, stream>>>(dst, src, elements, \
                                                                                      stride, rows, in_dtype, \
                                                                                      out_dtype);        \
        break;
    switch (l2e) {
        PMKL_SOFTMAX_GEN_CASE(0)
        PMKL_SOFTMAX_GEN_CASE(1)
        PMKL_SOFTMAX_GEN_CASE(2)
        PMKL_SOFTMAX_GEN_CASE(3)
        PMKL_SOFTMAX_GEN_CASE(4)
        PMKL_SOFTMAX_GEN_CASE(5)
        PMKL_SOFTMAX_GEN_CASE(6)
        PMKL_SOFTMAX_GEN_CASE(7)
        PMKL_SOFTMAX_GEN_CASE(8)
        PMKL_SOFTMAX_GEN_CASE(9)
        PMKL_SOFTMAX_GEN_CASE(10)
        default:
            return PMKL_ERR_INVALID_SHAPE;
    }
#undef PMKL_SOFTMAX_GEN_CASE
    return launch_status();
}

}  // namespace
}  // namespace pmkl_b200

using namespace pmkl_b200;

extern "C" {

int pmkl_causal_attention_fwd(const void *q, const void *k, const void *v, void *o, void *m, void *l, int batch,
                              int heads, int seq, int hidden, int dtype, int out_dtype, int is_causal, float scale,
                              void *stream) {
    return attention_impl(q, k, v, o, m, l, batch, heads, seq, hidden, dtype, out_dtype, is_causal, scale,
                          PMKL_ATTN_AUTO, stream);
}

int pmkl_causal_attention_fwd_ex(const void *q, const void *k, const void *v, void *o, void *m, void *l, int batch,
                                 int heads, int seq, int hidden, int dtype, int out_dtype, int is_causal, float scale,
                                 int kernel, void *stream) {
    return attention_impl(q, k, v, o, m, l, batch, heads, seq, hidden, dtype, out_dtype, is_causal, scale, kernel,
                          stream);
}

int pmkl_causal_attention_bwd(const void *dout, const void *q, const void *k, const void *v, const void *m,
                              const void *l, void *dq, void *dk, void *dv, int batch, int heads, int seq,
                              int hidden, int dtype, int is_causal, float scale, void *workspace,
                              size_t workspace_bytes, void *stream) {
    return attention_bwd_impl(dout, q, k, v, m, l, dq, dk, dv, batch, heads, seq, hidden, dtype, is_causal, scale,
                              workspace, workspace_bytes, PMKL_ATTN_AUTO, stream);
}

int pmkl_causal_attention_bwd_ex(const void *dout, const void *q, const void *k, const void *v, const void *m,
                                 const void *l, void *dq, void *dk, void *dv, int batch, int heads, int seq,
                                 int hidden, int dtype, int is_causal, float scale, void *workspace,
                                 size_t workspace_bytes, int kernel, void *stream) {
    return attention_bwd_impl(dout, q, k, v, m, l, dq, dk, dv, batch, heads, seq, hidden, dtype, is_causal, scale,
                              workspace, workspace_bytes, kernel, stream);
}

int pmkl_causal_attention_bwd_strided(const void *dout, const void *q, const void *k, const void *v, const void *m,
                                      const void *l, void *dq, void *dk, void *dv, int batch, int heads, int kv_heads,
                                      int seq, int hidden, const int64_t *dout_strides, const int64_t *q_strides,
                                      const int64_t *k_strides, const int64_t *v_strides, const int64_t *dq_strides,
                                      const int64_t *dk_strides, const int64_t *dv_strides, int dtype, int is_causal,
                                      float scale, void *workspace, size_t workspace_bytes, int kernel,
                                      void *stream) {
    if (batch < 0 || heads < 0 || seq < 0 || hidden < 0 || kv_heads < 0) return PMKL_ERR_INVALID_SHAPE;
    if (heads > 0 && (kv_heads == 0 || heads % kv_heads != 0)) return PMKL_ERR_INVALID_SHAPE;
    AttnBwdLayout lay = contiguous_bwd_layout(heads > 0 ? heads : 1, seq, hidden);
    lay.kv_group = (heads > 0 && kv_heads > 0) ? heads / kv_heads : 1;
    const long long Hkv = kv_heads > 0 ? kv_heads : 1;
    const long long kv_contig[3] = {Hkv * seq * hidden, static_cast<long long>(seq) * hidden, hidden};
    const int64_t *given[7] = {dout_strides, q_strides, k_strides, v_strides, dq_strides, dk_strides, dv_strides};
    long long *dst[7] = {lay.dout, lay.q, lay.k, lay.v, lay.dq, lay.dk, lay.dv};
    for (int t = 0; t < 7; ++t) {
        const bool kv_shaped = t == 2 || t == 3 || t == 5 || t == 6;
        const long long extent[3] = {batch, kv_shaped ? Hkv : heads, seq};
        for (int i = 0; i < 3; ++i) {
            if (given[t]) {
                if (given[t][i] < 0) return PMKL_ERR_INVALID_SHAPE;
                // A dimension of extent 1 is never stepped: its stride does not matter.
                dst[t][i] = extent[i] == 1 ? 0 : given[t][i];
            } else if (kv_shaped) {
                dst[t][i] = kv_contig[i];
            }
        }
    }
    return attention_bwd_impl(dout, q, k, v, m, l, dq, dk, dv, batch, heads, seq, hidden, dtype, is_causal, scale,
                              workspace, workspace_bytes, kernel, stream, &lay);
}

int pmkl_causal_attention_bwd_static(const void *dout, const void *q, const void *k, const void *v, const void *m,
                                     const void *l, void *dq, void *dk, void *dv, int batch, int heads, int seq,
                                     int hidden, int dtype, int is_causal, float scale, void *stream) {
    // Argument errors and empty problems first, as the workspace entry reports them.
    if (batch < 0 || heads < 0 || seq < 0 || hidden < 0) return PMKL_ERR_INVALID_SHAPE;
    if (!dtype_valid(dtype)) return PMKL_ERR_INVALID_DTYPE;
    if (static_cast<long long>(batch) * heads == 0 || seq == 0 || hidden == 0) return PMKL_OK;
    if (hidden > 256) return PMKL_ERR_UNSUPPORTED;
    const int dev_rc = current_device_ok();
    if (dev_rc != PMKL_OK) return dev_rc;
    void *ws = static_scratch();
    if (!ws) return PMKL_ERR_LAUNCH;
    return attention_bwd_impl(dout, q, k, v, m, l, dq, dk, dv, batch, heads, seq, hidden, dtype, is_causal, scale, ws,
                              PMKL_BWD_STATIC_SCRATCH_BYTES, PMKL_ATTN_AUTO, stream);
}

size_t pmkl_causal_attention_bwd_workspace_size(int batch, int heads, int seq, int hidden, int dtype) {
    return pmkl_causal_attention_bwd_workspace_size_ex(batch, heads, seq, hidden, dtype, PMKL_ATTN_AUTO);
}

size_t pmkl_causal_attention_bwd_workspace_size_ex(int batch, int heads, int seq, int hidden, int dtype,
                                                   int kernel) {
    if (batch <= 0 || heads <= 0 || seq <= 0 || hidden <= 0 || !dtype_valid(dtype)) return 0;
    if (kernel != PMKL_ATTN_AUTO && kernel != PMKL_ATTN_SIMT && kernel != PMKL_ATTN_TCGEN05 &&
        kernel != PMKL_ATTN_TCGEN05_SIMPLE)
        return 0;
    return bwd_workspace_size(static_cast<long long>(batch) * heads, seq, hidden, dtype, kernel);
}

int pmkl_causal_attention_fwd_strided(const void *q, const void *k, const void *v, void *o, void *m, void *l,
                                      int batch, int heads, int kv_heads, int seq, int hidden,
                                      const int64_t *q_strides, const int64_t *k_strides, const int64_t *v_strides,
                                      const int64_t *o_strides, int dtype, int out_dtype, int is_causal, float scale,
                                      int kernel, void *stream) {
    if (batch < 0 || heads < 0 || seq < 0 || hidden < 0 || kv_heads < 0) return PMKL_ERR_INVALID_SHAPE;
    if (heads > 0 && (kv_heads == 0 || heads % kv_heads != 0)) return PMKL_ERR_INVALID_SHAPE;
    AttnLayout lay = contiguous_layout(heads > 0 ? heads : 1, seq, hidden);
    lay.kv_group = (heads > 0 && kv_heads > 0) ? heads / kv_heads : 1;
    const long long Hkv = kv_heads > 0 ? kv_heads : 1;
    const long long kv_contig[3] = {Hkv * seq * hidden, static_cast<long long>(seq) * hidden, hidden};
    const int64_t *given[4] = {q_strides, k_strides, v_strides, o_strides};
    long long *dst[4] = {lay.q, lay.k, lay.v, lay.o};
    for (int t = 0; t < 4; ++t) {
        const long long extent[3] = {batch, (t == 1 || t == 2) ? Hkv : heads, seq};
        for (int i = 0; i < 3; ++i) {
            if (given[t]) {
                if (given[t][i] < 0) return PMKL_ERR_INVALID_SHAPE;
                // A dimension of extent 1 is never stepped: its stride does not matter.
                dst[t][i] = extent[i] == 1 ? 0 : given[t][i];
            } else if (t == 1 || t == 2) {
                dst[t][i] = kv_contig[i];
            }
        }
    }
    return attention_impl(q, k, v, o, m, l, batch, heads, seq, hidden, dtype, out_dtype, is_causal, scale, kernel,
                          stream, &lay);
}

int pmkl_attention_selected_kernel(const void *q, const void *k, const void *v, const void *o, int hidden, int dtype,
                                   int out_dtype, int kernel) {
    if (!dtype_valid(dtype) || !dtype_valid(out_dtype)) return PMKL_ERR_INVALID_DTYPE;
    if (kernel != PMKL_ATTN_AUTO && kernel != PMKL_ATTN_SIMT && kernel != PMKL_ATTN_TCGEN05 &&
        kernel != PMKL_ATTN_TCGEN05_SIMPLE)
        return PMKL_ERR_UNSUPPORTED;
    const int dev_rc = current_device_ok();
    if (dev_rc != PMKL_OK) return dev_rc;
    const AttnLayout lay = contiguous_layout(1, 128, hidden > 0 ? hidden : 1);
    return select_kernel(q, k, v, o, hidden, 128, dtype, out_dtype, kernel, lay);
}

int pmkl_warp_softmax_fwd(void *dst, const void *src, int elements, int stride, int rows, int in_dtype,
                          int out_dtype, int is_log, void *stream_) {
    if (elements < 0 || elements > 1024) return PMKL_ERR_INVALID_SHAPE;  // warp_softmax.h:162
    if (rows < 0 || stride < elements) return PMKL_ERR_INVALID_SHAPE;
    if (!dtype_valid(in_dtype) || !dtype_valid(out_dtype)) return PMKL_ERR_INVALID_DTYPE;
    if (elements == 0 || rows == 0) return PMKL_OK;  // warp_softmax.h:163-164
    if (!dst || !src) return PMKL_ERR_NULL_POINTER;
    const int dev_rc = current_device_ok();
    if (dev_rc != PMKL_OK) return dev_rc;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const bool vec = in_dtype == PMKL_DTYPE_F32 && out_dtype == PMKL_DTYPE_F32 && (elements % 4) == 0 &&
                     (stride % 4) == 0 && aligned16(dst) && aligned16(src);
    if (vec) {
        return is_log ? launch_softmax_vec<true>(static_cast<float *>(dst), static_cast<const float *>(src), elements,
                                                 stride, rows, stream)
                      : launch_softmax_vec<false>(static_cast<float *>(dst), static_cast<const float *>(src),
                                                  elements, stride, rows, stream);
    }
    // Other dtype pairs: 8-element vectors when rows allow them.
    const bool vec8 = (elements % 8) == 0 && (stride % 8) == 0 && aligned16(dst) && aligned16(src);
    if (vec8)
        return is_log ? launch_softmax_vec8<true>(dst, src, elements, stride, rows, in_dtype, out_dtype, stream)
                      : launch_softmax_vec8<false>(dst, src, elements, stride, rows, in_dtype, out_dtype, stream);
    return is_log ? launch_softmax_gen<true>(dst, src, elements, stride, rows, in_dtype, out_dtype, stream)
                  : launch_softmax_gen<false>(dst, src, elements, stride, rows, in_dtype, out_dtype, stream);
}

const char *pmkl_status_string(int status) {
    switch (status) {
        case PMKL_OK:
            return "PMKL_OK";
        case PMKL_ERR_INVALID_SHAPE:
            return "PMKL_ERR_INVALID_SHAPE: invalid or unsupported sizes";
        case PMKL_ERR_INVALID_DTYPE:
            return "PMKL_ERR_INVALID_DTYPE: unsupported dtype";
        case PMKL_ERR_NULL_POINTER:
            return "PMKL_ERR_NULL_POINTER: null pointer for a non-empty problem";
        case PMKL_ERR_MISALIGNED:
            return "PMKL_ERR_MISALIGNED: pointer alignment";
        case PMKL_ERR_UNSUPPORTED:
            return "PMKL_ERR_UNSUPPORTED: no kernel for these arguments";
        case PMKL_ERR_NO_DEVICE:
            return "PMKL_ERR_NO_DEVICE: no sm_100 CUDA device is current";
        case PMKL_ERR_LAUNCH:
            return "PMKL_ERR_LAUNCH: CUDA launch failed";
        case PMKL_ERR_DEVICE_TIMEOUT:
            return "PMKL_ERR_DEVICE_TIMEOUT: a kernel abandoned a bounded wait";
        case PMKL_ERR_WORKSPACE:
            return "PMKL_ERR_WORKSPACE: workspace too small";
        default:
            return "PMKL_ERR_UNKNOWN";
    }
}

int pmkl_version(void) { return PMKL_B200_VERSION; }

int pmkl_stream_synchronize(void *stream) {
    return cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) == cudaSuccess ? PMKL_OK : PMKL_ERR_LAUNCH;
}

int pmkl_device_error(int clear) {
    const int dev_rc = current_device_ok();
    if (dev_rc != PMKL_OK) return dev_rc;
    if (cudaDeviceSynchronize() != cudaSuccess) return PMKL_ERR_LAUNCH;
    unsigned int word = 0;
    if (cudaMemcpyFromSymbol(&word, g_device_error, sizeof(word)) != cudaSuccess) return PMKL_ERR_LAUNCH;
    if (word != 0 && clear) {
        const unsigned int zero = 0;
        if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)) != cudaSuccess) return PMKL_ERR_LAUNCH;
    }
    return word ? PMKL_ERR_DEVICE_TIMEOUT : PMKL_OK;
}

int pmkl_wait_selftest(int ctas, unsigned long long limit_ns, unsigned long long *out, void *stream) {
    if (ctas < 1 || ctas > 1024) return PMKL_ERR_INVALID_SHAPE;
    if (limit_ns < 100000ull || limit_ns > ptx::kWaitTimeoutNs) return PMKL_ERR_INVALID_SHAPE;
    if (!out) return PMKL_ERR_NULL_POINTER;
    if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return PMKL_ERR_MISALIGNED;
    const int dev_rc = current_device_ok();
    if (dev_rc != PMKL_OK) return dev_rc;
    diag::wait_selftest_kernel<<<ctas, 128, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, out);
    return launch_status();
}

int pmkl_tc_selftest(int which, const void *a, const void *b, float *c, int hidden, int dtype, void *stream_) {
    if (which != 0 && which != 1) return PMKL_ERR_UNSUPPORTED;
    if (hidden != 64 && hidden != 128) return PMKL_ERR_UNSUPPORTED;
    if (dtype != PMKL_DTYPE_F16 && dtype != PMKL_DTYPE_BF16) return PMKL_ERR_INVALID_DTYPE;
    if (!a || !b || !c) return PMKL_ERR_NULL_POINTER;
    if (!aligned16(a) || !aligned16(b)) return PMKL_ERR_MISALIGNED;
    const int dev_rc = current_device_ok();
    if (dev_rc != PMKL_OK) return dev_rc;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    CUtensorMap ta, tb;
    if (!make_tile_map(&ta, a, dtype, which == 0 ? hidden : 128, 128, 1) ||
        !make_tile_map(&tb, b, dtype, hidden, 128, 1))
        return PMKL_ERR_LAUNCH;
    constexpr int smem = 4 * tc::kBoxBytes + 1024 + 64;
    const bool bf = dtype == PMKL_DTYPE_BF16;
    auto run = [&](auto kernel) -> int {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return PMKL_ERR_LAUNCH;
        kernel<<<1, 128, smem, stream>>>(ta, tb, static_cast<const uint16_t *>(a), c, which);
        return launch_status();
    };
    if (hidden == 64) return bf ? run(tc::tc_selftest_kernel<64, true>) : run(tc::tc_selftest_kernel<64, false>);
    return bf ? run(tc::tc_selftest_kernel<128, true>) : run(tc::tc_selftest_kernel<128, false>);
}

}  // extern "C"
