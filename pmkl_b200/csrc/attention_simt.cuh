// attention_simt.cuh -- generic CUDA-core flash attention forward.
//
// Covers every case the tensor-core kernel does not: fp32 inputs (which the
// reference's own GPU kernel handles, pmkl/nlp/causal_attention.h:258), any
// head size 1..256, 16-bit inputs with other head sizes, and unaligned
// pointers.  fp32 arithmetic throughout with accurate expf, so that fp32
// results stay within the reference's all_close tolerance (1e-5 absolute +
// relative, pmkl/core/utils/measure.h:10-12).
//
// Block = 4 warps on a 32-row query tile; each warp owns 8 query rows.  Key
// tiles of 32 rows are staged in shared memory as fp32; lane j scores key j
// against the warp's rows, a warp shuffle gives row max and sum, and each lane
// accumulates output columns lane, lane + 32, ... for the warp's rows.  Key
// tiles above the diagonal are skipped in causal mode.
#pragma once

#include "common.cuh"

namespace pmkl_b200 {
namespace simt {

constexpr int kBM = 32;
constexpr int kBN = 32;
constexpr int kRowsPerWarp = 8;
constexpr int kThreads = 128;

template <int DMAX>
constexpr int smem_bytes() {
    return (kBM * DMAX + kBN * (DMAX + 1) + kBN * DMAX) * 4;
}

template <typename T>
__device__ __forceinline__ float ld_f(const T *p) {
    return Elem<T>::to_float(*p);
}
template <>
__device__ __forceinline__ float ld_f<float>(const float *p) {
    return *p;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T, int DMAX>
__global__ void __launch_bounds__(kThreads)
    attn_fwd_simt_kernel(const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v, void *__restrict__ o,
                         void *__restrict__ m_out, void *__restrict__ l_out, int S, int D, int BH, int n_qt, int causal,
                         float scale, int out_dtype, const AttnLayout lay) {
    extern __shared__ float smem_f[];
    float *Qs = smem_f;                      // [kBM][DMAX]
    float *Ks = Qs + kBM * DMAX;             // [kBN][DMAX + 1]
    float *Vs = Ks + kBN * (DMAX + 1);       // [kBN][DMAX]
    constexpr int KS = DMAX + 1;
    constexpr int CPL = DMAX / 32;           // output columns per lane

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int bid = blockIdx.x;
    const int qt = causal ? (n_qt - 1 - bid / BH) : (bid / BH);
    const int bh = bid % BH;
    const int bb = bh / lay.H, hh = bh % lay.H, hk = hh / lay.kv_group;
    const long long qb = bb * lay.q[0] + hh * lay.q[1];
    const long long kb0 = bb * lay.k[0] + hk * lay.k[1];
    const long long vb0 = bb * lay.v[0] + hk * lay.v[1];
    const long long ob0 = bb * lay.o[0] + hh * lay.o[1];
    const int row0 = qt * kBM;

    for (int idx = threadIdx.x; idx < kBM * DMAX; idx += kThreads) {
        const int r = idx / DMAX, d = idx % DMAX;
        const int row = row0 + r;
        Qs[idx] = (row < S && d < D) ? ld_f(q + qb + row * lay.q[2] + d) : 0.f;
    }

    float mrow[kRowsPerWarp], lrow[kRowsPerWarp], acc[kRowsPerWarp][CPL];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        mrow[i] = -INFINITY;
        lrow[i] = 0.f;
#pragma unroll
        for (int t = 0; t < CPL; ++t) acc[i][t] = 0.f;
    }

    const int kv_end = causal ? min(S, row0 + kBM) : S;
    for (int kb = 0; kb < kv_end; kb += kBN) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < kBN * DMAX; idx += kThreads) {
            const int r = idx / DMAX, d = idx % DMAX;
            const int key = kb + r;
            const bool in = key < S && d < D;
            Ks[r * KS + d] = in ? ld_f(k + kb0 + key * lay.k[2] + d) : 0.f;
            Vs[idx] = in ? ld_f(v + vb0 + key * lay.v[2] + d) : 0.f;
        }
        __syncthreads();

        const int key = kb + lane;
        float s[kRowsPerWarp];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) s[i] = 0.f;
        for (int d = 0; d < D; ++d) {
            const float kd = Ks[lane * KS + d];
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i) s[i] = fmaf(Qs[(warp * kRowsPerWarp + i) * DMAX + d], kd, s[i]);
        }
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            const int row = row0 + warp * kRowsPerWarp + i;
            const bool valid = key < S && (!causal || key <= row);
            const float si = valid ? s[i] * scale : -INFINITY;
            const float mx = warp_max(si);
            const float m_new = fmaxf(mrow[i], mx);
            const float corr = (mrow[i] == -INFINITY) ? 0.f : expf(mrow[i] - m_new);
            const float pi = (m_new == -INFINITY) ? 0.f : expf(si - m_new);
            lrow[i] = lrow[i] * corr + warp_sum(pi);
            mrow[i] = m_new;
#pragma unroll
            for (int t = 0; t < CPL; ++t) acc[i][t] *= corr;
#pragma unroll 8
            for (int jj = 0; jj < kBN; ++jj) {
                const float pj = __shfl_sync(0xffffffffu, pi, jj);
#pragma unroll
                for (int t = 0; t < CPL; ++t) acc[i][t] = fmaf(pj, Vs[jj * DMAX + lane + 32 * t], acc[i][t]);
            }
        }
    }

#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int row = row0 + warp * kRowsPerWarp + i;
        if (row >= S) continue;
        const float inv = 1.f / lrow[i];
        const long long ob = ob0 + row * lay.o[2];
#pragma unroll
        for (int t = 0; t < CPL; ++t) {
            const int d = lane + 32 * t;
            if (d < D) store_as(o, ob + d, out_dtype, acc[i][t] * inv);
        }
        if (lane == 0) {
            const size_t mi = static_cast<size_t>(bh) * S + row;
            store_as(m_out, mi, out_dtype, mrow[i]);
            store_as(l_out, mi, out_dtype, lrow[i]);
        }
    }
}

}  // namespace simt
}  // namespace pmkl_b200
