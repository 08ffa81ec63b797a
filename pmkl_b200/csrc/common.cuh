// common.cuh -- element-type helpers and the device error word shared by the
// kernels of libpmkl_b200.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "pmkl_b200.h"

namespace pmkl_b200 {

// Bit 0: a kernel abandoned a bounded wait (PMKL_DEVERR_TIMEOUT).
constexpr unsigned int PMKL_DEVERR_TIMEOUT = 1u;

// Read and cleared by pmkl_device_error().  The library is one translation
// unit (pmkl_b200.cu includes every kernel header), so this is its only copy.
__device__ unsigned int g_device_error = 0;

__device__ __forceinline__ void report_device_error(unsigned int bits) { atomicOr(&g_device_error, bits); }

template <typename T>
struct Elem;

template <>
struct Elem<float> {
    static constexpr int kDtype = PMKL_DTYPE_F32;
    __device__ __forceinline__ static float load(const float *p) { return *p; }
    __device__ __forceinline__ static float to_float(float v) { return v; }
    __device__ __forceinline__ static float from_float(float v) { return v; }
};

template <>
struct Elem<__half> {
    static constexpr int kDtype = PMKL_DTYPE_F16;
    __device__ __forceinline__ static float to_float(__half v) { return __half2float(v); }
    __device__ __forceinline__ static __half from_float(float v) { return __float2half_rn(v); }
};

template <>
struct Elem<__nv_bfloat16> {
    static constexpr int kDtype = PMKL_DTYPE_BF16;
    __device__ __forceinline__ static float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
    __device__ __forceinline__ static __nv_bfloat16 from_float(float v) { return __float2bfloat16_rn(v); }
};

// Element strides of the attention tensors.  q, k, v, o are [batch][head]
// [row][head_size] with the head-size dimension contiguous; k and v have
// H / kv_group heads, query head h reading K/V head h / kv_group.  m and l
// are always contiguous [batch * H][rows].
struct AttnLayout {
    int H;
    int kv_group;
    long long q[3], k[3], v[3], o[3];  // (batch, head, row)
};

// Element strides of the backward's tensors (batch, head, row) with the
// head-size dimension contiguous.  q, dout, dq have H heads; k, v, dk, dv have
// H / kv_group heads, query head h reading K/V head h / kv_group.  m, l and
// the per-row terms are contiguous [batch * H][rows].
struct AttnBwdLayout {
    int H;
    int kv_group;
    long long dout[3], q[3], k[3], v[3], dq[3], dk[3], dv[3];
};

__host__ __device__ __forceinline__ long long elem_off(const long long (&st)[3], long long b, long long h,
                                                        long long row) {
    return b * st[0] + h * st[1] + row * st[2];
}

// Stores one fp32 value as out_dtype.
__device__ __forceinline__ void store_as(void *base, size_t idx, int out_dtype, float v) {
    if (out_dtype == PMKL_DTYPE_F32)
        static_cast<float *>(base)[idx] = v;
    else if (out_dtype == PMKL_DTYPE_F16)
        static_cast<__half *>(base)[idx] = __float2half_rn(v);
    else
        static_cast<__nv_bfloat16 *>(base)[idx] = __float2bfloat16_rn(v);
}

inline size_t dtype_size(int dtype) { return dtype == PMKL_DTYPE_F32 ? 4 : 2; }

inline bool dtype_valid(int dtype) {
    return dtype == PMKL_DTYPE_F32 || dtype == PMKL_DTYPE_F16 || dtype == PMKL_DTYPE_BF16;
}

}  // namespace pmkl_b200
