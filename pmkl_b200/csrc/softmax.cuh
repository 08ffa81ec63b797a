// softmax.cuh -- row-wise softmax / log-softmax, fp32 accumulation.
//
// Replaces pmkl::norm::warp_softmax_forward_impl (pmkl/norm/warp_softmax.h:
// 74-157).  The reference loads one 4-byte element per lane per iteration and
// ends each of its two warp reductions with __syncthreads and a shared-memory
// broadcast.  Here:
//   * vector path (fp32 in/out, 16-byte aligned rows, elements % 4 == 0):
//     one warp per row, every lane loads its share of the row with 16-byte
//     non-caching loads (a row of 1024 floats = 8 float4 per lane, all in
//     flight at once), max and sum are butterfly shuffles that leave the
//     result in every lane (no shared memory, no block barrier), and the
//     results go out with 16-byte streaming stores.  Bandwidth-bound: one
//     read and one write of every element.
//   * 8-element vector path (any dtype pair; elements and stride multiples of
//     8, 16-byte aligned rows): the same with 16-byte loads of eight 16-bit
//     values, converted to fp32 in registers and back on the store.
//   * general path (any dtype pair, any stride/alignment): the reference's
//     shape -- 2^L elements per row padded with -inf, min(2^L, 32) lanes per
//     row, coalesced scalar loads -- with shuffle-only reductions.
// Results: dst = exp(x - max) / sum, or x - max - log(sum) for log-softmax;
// a row whose sum is 0 yields NaN (warp_softmax.h:147-148).
#pragma once

#include "common.cuh"

namespace pmkl_b200 {
namespace softmax {

constexpr int kThreads = 256;  // 8 warps per block

template <int LANES>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
    for (int o = LANES / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int LANES>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = LANES / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float4 ld_stream(const float4 *p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void st_stream(float4 *p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// VPL = float4 vectors per lane (elements <= 128 * VPL).
template <int VPL, bool LOG>
__global__ void __launch_bounds__(kThreads)
    softmax_vec_kernel(float *__restrict__ dst, const float *__restrict__ src, int elements, long long stride,
                       int rows) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long row = static_cast<long long>(blockIdx.x) * (kThreads / 32) + warp;
    if (row >= rows) return;
    const float4 *s4 = reinterpret_cast<const float4 *>(src + row * stride);
    float4 *d4 = reinterpret_cast<float4 *>(dst + row * stride);
    const int n4 = elements >> 2;
    float4 x[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int idx = lane + 32 * i;
        x[i] = (idx < n4) ? ld_stream(s4 + idx) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPL; ++i) mx = fmaxf(fmaxf(mx, fmaxf(x[i].x, x[i].y)), fmaxf(x[i].z, x[i].w));
    mx = group_max<32>(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        float4 e = make_float4(expf(x[i].x - mx), expf(x[i].y - mx), expf(x[i].z - mx), expf(x[i].w - mx));
        sum += (e.x + e.y) + (e.z + e.w);
        if (!LOG) x[i] = e;
    }
    sum = group_sum<32>(sum);
    if (LOG) {
        const float sub = mx + logf(sum);
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int idx = lane + 32 * i;
            if (idx < n4) st_stream(d4 + idx, make_float4(x[i].x - sub, x[i].y - sub, x[i].z - sub, x[i].w - sub));
        }
    } else {
        const float inv = (sum == 0.f) ? __int_as_float(0x7fc00000) : 1.f / sum;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int idx = lane + 32 * i;
            if (idx < n4) st_stream(d4 + idx, make_float4(x[i].x * inv, x[i].y * inv, x[i].z * inv, x[i].w * inv));
        }
    }
}

__device__ __forceinline__ float ptx_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Eight consecutive elements of a row as fp32: one 16-byte load for 16-bit
// types, two for fp32 (non-caching, the row is read once).
template <typename T>
__device__ __forceinline__ void load8(const T *p, float (&v)[8]) {
    if constexpr (sizeof(T) == 4) {
        const float4 a = ld_stream(reinterpret_cast<const float4 *>(p));
        const float4 b = ld_stream(reinterpret_cast<const float4 *>(p) + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
        uint32_t w[4];
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                     : "l"(p));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float lo, hi;
            if constexpr (std::is_same<T, __half>::value) {
                const __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
                lo = __low2float(h), hi = __high2float(h);
            } else {
                lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xffff0000u);
            }
            v[2 * i] = lo, v[2 * i + 1] = hi;
        }
    }
}

// Eight fp32 values stored as T (round to nearest), streaming stores.
template <typename T>
__device__ __forceinline__ void store8(T *p, const float (&v)[8]) {
    if constexpr (sizeof(T) == 4) {
        st_stream(reinterpret_cast<float4 *>(p), make_float4(v[0], v[1], v[2], v[3]));
        st_stream(reinterpret_cast<float4 *>(p) + 1, make_float4(v[4], v[5], v[6], v[7]));
    } else {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (std::is_same<T, __half>::value) {
                const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t *>(&h);
            } else {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                w[i] = *reinterpret_cast<const uint32_t *>(&h);
            }
        }
        asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                     "r"(w[3])
                     : "memory");
    }
}

// Vector path for any dtype pair: one warp per row, 8-element vectors (16 bytes
// of 16-bit data), V8 vectors per lane (elements <= 256 * V8, a multiple of 8;
// 16-byte aligned rows), fp32 accumulation, shuffle-only reductions.
template <typename TI, typename TO, int V8, bool LOG>
__global__ void __launch_bounds__(kThreads)
    softmax_vec8_kernel(TO *__restrict__ dst, const TI *__restrict__ src, int elements, long long stride, int rows) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long row = static_cast<long long>(blockIdx.x) * (kThreads / 32) + warp;
    if (row >= rows) return;
    const TI *s = src + row * stride;
    TO *d = dst + row * stride;
    const int n8 = elements >> 3;
    float x[V8][8];
#pragma unroll
    for (int i = 0; i < V8; ++i) {
        const int idx = lane + 32 * i;
        if (idx < n8) {
            load8(s + 8 * idx, x[i]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) x[i][e] = -INFINITY;
        }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < V8; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) mx = fmaxf(mx, x[i][e]);
    mx = group_max<32>(mx);
    // With a 16-bit output the hardware exp2 on (x - max) log2 e is far more
    // precise than the stored value (2^-9 / 2^-12 relative); fp32 outputs keep
    // the accurate expf of the reference's fp32 path.
    constexpr bool kFastExp = sizeof(TO) == 2;
    constexpr float kLog2e = 1.4426950408889634f;
    const float mxl = mx * kLog2e;
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < V8; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float ev = kFastExp ? ptx_ex2(fmaf(x[i][e], kLog2e, -mxl)) : expf(x[i][e] - mx);
            sum += ev;
            if (!LOG) x[i][e] = ev;
        }
    sum = group_sum<32>(sum);
    const float sub = LOG ? mx + logf(sum) : 0.f;
    const float inv = (sum == 0.f) ? __int_as_float(0x7fc00000) : 1.f / sum;
#pragma unroll
    for (int i = 0; i < V8; ++i) {
        const int idx = lane + 32 * i;
        if (idx < n8) {
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = LOG ? x[i][e] - sub : x[i][e] * inv;
            store8(d + 8 * idx, y);
        }
    }
}

__device__ __forceinline__ float load_elem(const void *p, long long i, int dtype) {
    if (dtype == PMKL_DTYPE_F32) return static_cast<const float *>(p)[i];
    if (dtype == PMKL_DTYPE_F16) return __half2float(static_cast<const __half *>(p)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
}

// 2^L2E padded elements per row; LANES = min(2^L2E, 32) lanes per row.
template <int L2E, bool LOG>
__global__ void __launch_bounds__(kThreads)
    softmax_gen_kernel(void *__restrict__ dst, const void *__restrict__ src, int elements, long long stride, int rows,
                       int in_dtype, int out_dtype) {
    constexpr int P2 = 1 << L2E;
    constexpr int LANES = P2 < 32 ? P2 : 32;
    constexpr int ITERS = P2 / LANES;
    constexpr int ROWS_PER_WARP = 32 / LANES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane / LANES, li = lane % LANES;
    const long long row =
        (static_cast<long long>(blockIdx.x) * (kThreads / 32) + warp) * ROWS_PER_WARP + sub;
    const bool active = row < rows;
    const long long rb = active ? row * stride : 0;
    float x[ITERS];
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int c = li + it * LANES;
        x[it] = (active && c < elements) ? load_elem(src, rb + c, in_dtype) : -INFINITY;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) mx = fmaxf(mx, x[it]);
    mx = group_max<LANES>(mx);
    float sum = 0.f;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const float e = expf(x[it] - mx);
        // Padding lanes hold -inf: exp(-inf - mx) = 0 for finite mx.
        sum += (li + it * LANES < elements) ? e : 0.f;
        if (!LOG) x[it] = e;
    }
    sum = group_sum<LANES>(sum);
    if (!active) return;
    const float lg = LOG ? logf(sum) : 0.f;
    const float inv = (sum == 0.f) ? __int_as_float(0x7fc00000) : 1.f / sum;
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int c = li + it * LANES;
        if (c < elements) store_as(dst, rb + c, out_dtype, LOG ? (x[it] - mx - lg) : x[it] * inv);
    }
}

}  // namespace softmax
}  // namespace pmkl_b200
