// attention_bwd_simt.cuh -- generic CUDA-core backward of the fused causal
// self-attention: fp32 inputs (the reference's own test runs the backward in
// fp32, pmkl_pytorch_ext/test/test_fused_self_attention.py:21-38), every head
// size 1..256, 16-bit inputs with other head sizes, unaligned pointers.
//
// Same gradient as fused_self_attention.cpp:66-135, fp32 arithmetic with
// accurate expf:  p = exp(scale q.k - m~) / l~ (masked: 0), dP = dO . v,
// delta = sum_j p dP, dS = p (dP - delta), dQ = scale dS K, dK = scale dS^T Q,
// dV = P^T dO.  Two launches:
//   attn_bwd_simt_q_kernel   32-row query tiles, 4 warps x 8 rows; a first pass
//                            over the key tiles forms delta, a second forms dQ
//                            (lane j scores key j; each lane accumulates dQ
//                            columns lane, lane + 32, ...).  Writes delta.
//   attn_bwd_simt_kv_kernel  32-row key tiles of one K/V head, 4 warps x 8
//                            rows; for every query head reading that K/V head
//                            (grouped-query attention) and every 32-query
//                            tile, lane j scores query j, each lane
//                            accumulates dK/dV columns lane, lane + 32, ...
// Tensors are addressed through the caller's strides (AttnBwdLayout).
#pragma once

#include "attention_simt.cuh"

namespace pmkl_b200 {
namespace simt {

template <int DMAX>
constexpr int bwd_smem_bytes() {
    return (2 * 32 * DMAX + 2 * 32 * (DMAX + 1) + 3 * 32) * 4;
}

template <typename T, int DMAX>
__global__ void __launch_bounds__(kThreads)
    attn_bwd_simt_q_kernel(const T *__restrict__ dout, const T *__restrict__ q, const T *__restrict__ k,
                           const T *__restrict__ v, const T *__restrict__ m_in, const T *__restrict__ l_in,
                           T *__restrict__ dq, float *__restrict__ delta_out, int S, int D, int BH, int n_qt,
                           int causal, float scale, const AttnBwdLayout L) {
    extern __shared__ float smem_f[];
    constexpr int KS = DMAX + 1;
    constexpr int CPL = DMAX / 32;
    float *Qs = smem_f;              // [32][DMAX]
    float *DOs = Qs + 32 * DMAX;     // [32][DMAX]
    float *Ks = DOs + 32 * DMAX;     // [32][DMAX + 1]
    float *Vs = Ks + 32 * KS;        // [32][DMAX + 1]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int bid = blockIdx.x;
    const int qt = causal ? (n_qt - 1 - bid / BH) : (bid / BH);
    const int bh = bid % BH;
    const int bb = bh / L.H, hh = bh - bb * L.H, hkv = hh / L.kv_group;
    const int row0 = qt * 32;

    for (int idx = threadIdx.x; idx < 32 * DMAX; idx += kThreads) {
        const int r = idx / DMAX, d = idx % DMAX;
        const int row = row0 + r;
        const bool in = row < S && d < D;
        Qs[idx] = in ? ld_f(q + elem_off(L.q, bb, hh, row) + d) : 0.f;
        DOs[idx] = in ? ld_f(dout + elem_off(L.dout, bb, hh, row) + d) : 0.f;
    }
    float mr[kRowsPerWarp], lr[kRowsPerWarp], part[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int row = row0 + warp * kRowsPerWarp + i;
        mr[i] = row < S ? ld_f(m_in + static_cast<size_t>(bh) * S + row) : 0.f;
        lr[i] = row < S ? ld_f(l_in + static_cast<size_t>(bh) * S + row) : 1.f;
        part[i] = 0.f;
    }
    const int kv_end = causal ? min(S, row0 + 32) : S;

    // Scores and dP of the warp's rows against key kb + lane.
    auto tile_p_dp = [&](int kb, float (&pr)[kRowsPerWarp], float (&dp)[kRowsPerWarp]) {
        const int key = kb + lane;
        float s[kRowsPerWarp];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) s[i] = dp[i] = 0.f;
        for (int d = 0; d < D; ++d) {
            const float kd = Ks[lane * KS + d], vd = Vs[lane * KS + d];
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i) {
                s[i] = fmaf(Qs[(warp * kRowsPerWarp + i) * DMAX + d], kd, s[i]);
                dp[i] = fmaf(DOs[(warp * kRowsPerWarp + i) * DMAX + d], vd, dp[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            const int row = row0 + warp * kRowsPerWarp + i;
            const bool valid = key < S && row < S && (!causal || key <= row);
            pr[i] = valid ? expf(s[i] * scale - mr[i]) / lr[i] : 0.f;
        }
    };
    auto load_kv = [&](int kb) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < 32 * DMAX; idx += kThreads) {
            const int r = idx / DMAX, d = idx % DMAX;
            const int key = kb + r;
            const bool in = key < S && d < D;
            Ks[r * KS + d] = in ? ld_f(k + elem_off(L.k, bb, hkv, key) + d) : 0.f;
            Vs[r * KS + d] = in ? ld_f(v + elem_off(L.v, bb, hkv, key) + d) : 0.f;
        }
        __syncthreads();
    };

    // Pass 1: delta.
    for (int kb = 0; kb < kv_end; kb += 32) {
        load_kv(kb);
        float pr[kRowsPerWarp], dp[kRowsPerWarp];
        tile_p_dp(kb, pr, dp);
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) part[i] = fmaf(pr[i], dp[i], part[i]);
    }
    float delta[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) delta[i] = warp_sum(part[i]);

    // Pass 2: dQ.
    float acc[kRowsPerWarp][CPL];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
        for (int t = 0; t < CPL; ++t) acc[i][t] = 0.f;
    for (int kb = 0; kb < kv_end; kb += 32) {
        load_kv(kb);
        float pr[kRowsPerWarp], dp[kRowsPerWarp];
        tile_p_dp(kb, pr, dp);
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            const float ds = pr[i] * (dp[i] - delta[i]);
#pragma unroll 8
            for (int jj = 0; jj < 32; ++jj) {
                const float dsj = __shfl_sync(0xffffffffu, ds, jj);
#pragma unroll
                for (int t = 0; t < CPL; ++t) acc[i][t] = fmaf(dsj, Ks[jj * KS + lane + 32 * t], acc[i][t]);
            }
        }
    }

#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int row = row0 + warp * kRowsPerWarp + i;
        if (row >= S) continue;
        const long long ob = elem_off(L.dq, bb, hh, row);
#pragma unroll
        for (int t = 0; t < CPL; ++t) {
            const int d = lane + 32 * t;
            if (d < D) dq[ob + d] = Elem<T>::from_float(acc[i][t] * scale);
        }
        if (lane == 0) delta_out[static_cast<size_t>(bh) * S + row] = delta[i];
    }
}

template <typename T, int DMAX>
__global__ void __launch_bounds__(kThreads)
    attn_bwd_simt_kv_kernel(const T *__restrict__ dout, const T *__restrict__ q, const T *__restrict__ k,
                            const T *__restrict__ v, const T *__restrict__ m_in, const T *__restrict__ l_in,
                            const float *__restrict__ delta_in, T *__restrict__ dk, T *__restrict__ dv, int S, int D,
                            int BHkv, int causal, float scale, const AttnBwdLayout L) {
    extern __shared__ float smem_f[];
    constexpr int QS = DMAX + 1;
    constexpr int CPL = DMAX / 32;
    float *Ks = smem_f;              // [32][DMAX]   this block's key rows
    float *Vs = Ks + 32 * DMAX;      // [32][DMAX]
    float *Qs = Vs + 32 * DMAX;      // [32][DMAX + 1]   one query tile
    float *DOs = Qs + 32 * QS;       // [32][DMAX + 1]
    float *Ms = DOs + 32 * QS;       // [32] m~, l~, delta of the query tile
    float *Ls = Ms + 32;
    float *Dl = Ls + 32;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int kt = blockIdx.x / BHkv;  // causal: ascending = most query tiles first
    const int bkv = blockIdx.x % BHkv;
    const int Hkv = L.H / L.kv_group;
    const int bb = bkv / Hkv, hkv = bkv - bb * Hkv;
    const int key0 = kt * 32;

    for (int idx = threadIdx.x; idx < 32 * DMAX; idx += kThreads) {
        const int r = idx / DMAX, d = idx % DMAX;
        const int key = key0 + r;
        const bool in = key < S && d < D;
        Ks[idx] = in ? ld_f(k + elem_off(L.k, bb, hkv, key) + d) : 0.f;
        Vs[idx] = in ? ld_f(v + elem_off(L.v, bb, hkv, key) + d) : 0.f;
    }
    float acc_k[kRowsPerWarp][CPL], acc_v[kRowsPerWarp][CPL];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
        for (int t = 0; t < CPL; ++t) acc_k[i][t] = acc_v[i][t] = 0.f;

    // Every query head of the group, each over its query tiles (the sum over
    // the group is the gradient of the shared K/V head).
    const int n_qb = (S - (causal ? key0 : 0) + 31) / 32;
    for (int step = 0; step < L.kv_group * n_qb; ++step) {
        const int g = step / n_qb;
        const int qb = (causal ? key0 : 0) + (step - g * n_qb) * 32;
        const int hh = hkv * L.kv_group + g;
        const long long bh = static_cast<long long>(bb) * L.H + hh;
        __syncthreads();
        for (int idx = threadIdx.x; idx < 32 * DMAX; idx += kThreads) {
            const int r = idx / DMAX, d = idx % DMAX;
            const int qr = qb + r;
            const bool in = qr < S && d < D;
            Qs[r * QS + d] = in ? ld_f(q + elem_off(L.q, bb, hh, qr) + d) : 0.f;
            DOs[r * QS + d] = in ? ld_f(dout + elem_off(L.dout, bb, hh, qr) + d) : 0.f;
        }
        if (threadIdx.x < 32) {
            const int qr = qb + threadIdx.x;
            const size_t si = static_cast<size_t>(bh) * S + qr;
            Ms[threadIdx.x] = qr < S ? ld_f(m_in + si) : 0.f;
            Ls[threadIdx.x] = qr < S ? ld_f(l_in + si) : 1.f;
            Dl[threadIdx.x] = qr < S ? delta_in[si] : 0.f;
        }
        __syncthreads();

        const int qr = qb + lane;  // this lane's query
        float s[kRowsPerWarp], dp[kRowsPerWarp];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) s[i] = dp[i] = 0.f;
        for (int d = 0; d < D; ++d) {
            const float qd = Qs[lane * QS + d], gd = DOs[lane * QS + d];
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i) {
                s[i] = fmaf(Ks[(warp * kRowsPerWarp + i) * DMAX + d], qd, s[i]);
                dp[i] = fmaf(Vs[(warp * kRowsPerWarp + i) * DMAX + d], gd, dp[i]);
            }
        }
        const float mq = Ms[lane], lq = Ls[lane], dq_ = Dl[lane];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            const int key = key0 + warp * kRowsPerWarp + i;
            const bool valid = qr < S && key < S && (!causal || key <= qr);
            const float pr = valid ? expf(s[i] * scale - mq) / lq : 0.f;
            const float ds = pr * (dp[i] - dq_);
#pragma unroll 8
            for (int jj = 0; jj < 32; ++jj) {
                const float pj = __shfl_sync(0xffffffffu, pr, jj);
                const float dsj = __shfl_sync(0xffffffffu, ds, jj);
#pragma unroll
                for (int t = 0; t < CPL; ++t) {
                    acc_v[i][t] = fmaf(pj, DOs[jj * QS + lane + 32 * t], acc_v[i][t]);
                    acc_k[i][t] = fmaf(dsj, Qs[jj * QS + lane + 32 * t], acc_k[i][t]);
                }
            }
        }
    }

#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int key = key0 + warp * kRowsPerWarp + i;
        if (key >= S) continue;
        const long long okk = elem_off(L.dk, bb, hkv, key), ovv = elem_off(L.dv, bb, hkv, key);
#pragma unroll
        for (int t = 0; t < CPL; ++t) {
            const int d = lane + 32 * t;
            if (d < D) {
                dk[okk + d] = Elem<T>::from_float(acc_k[i][t] * scale);
                dv[ovv + d] = Elem<T>::from_float(acc_v[i][t]);
            }
        }
    }
}

}  // namespace simt
}  // namespace pmkl_b200
