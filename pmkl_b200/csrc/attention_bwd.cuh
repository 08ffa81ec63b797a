// attention_bwd.cuh -- tensor-core (tcgen05) backward of the fused causal
// self-attention for sm_100a, fp16/bf16 inputs, head size 64 or 128.
//
// Gradients of what fused_self_attention_bw computes
// (pmkl_pytorch_ext/fused_self_attention.cpp:66-135), given dO, Q, K, V and
// the forward's row statistics m~, l~ as the caller passes them:
//   p_nj  = exp(s_nj - m~_n) / l~_n,   s = scale Q K^T (masked: p = 0)
//   dP_nj = dO_n . V_j,   delta_n = sum_j p_nj dP_nj
//   dS_nj = p_nj (dP_nj - delta_n)
//   dQ = scale dS K,   dK = scale dS^T Q,   dV = P^T dO
// (the reference's innermost loop, :99-121, sums exactly scale p_nm (dP_nm -
// delta_n) for each (n, m)).  Three steps, no atomics, deterministic:
//   1. per query row, b_n = m~_n log2 e + log2 l~_n (so that p = 2^(s c2 - b_n)
//      with c2 = scale log2 e) and delta_n, from this library's own forward:
//        sum_j p_nj dP_nj = exp(m_n - m~_n) (l_n / l~_n) (dO_n . O_n),
//      exact algebra, because the reference backward takes no O.  The
//      persistent forward forms them in its epilogue (attention_pp.cuh,
//      DeltaParams); otherwise a forward writes fp32 O, m, l and
//      bwd_rowstat_kernel forms them.
//   2. attn_bwd_dq_kernel: one CTA per (slice, 128-row query tile); per key
//      tile S = Q K^T and dP = dO V^T into tensor memory, dS (16-bit) back
//      into tensor memory, dQ += dS K.
//   3. attn_bwd_dkv_kernel: one CTA per (K/V slice, 128-row key tile); per
//      query tile of every query head that reads this K/V head (grouped-query
//      attention: kv_group heads, one after the other) S^T = K Q^T and
//      dP^T = V dO^T, P^T and dS^T (16-bit) back into tensor memory,
//      dV += P^T dO and dK += dS^T Q, summed over the group in tensor memory.
// Every tensor is addressed through 4-D maps {D, S, heads, batch} with the
// caller's strides, so views are read and written in place.
// Both gradient kernels: warps 0-7 are the elementwise warps (two per tile
// row -- one per half of the columns; the backward's elementwise work has no
// row reduction), warp 8 issues TMA loads, warp 9 (one thread) issues
// tcgen05.mma.  Every wait is bounded (sm100_ptx.cuh).
#pragma once

#include "attention_tc.cuh"

namespace pmkl_b200 {
namespace bwd {

using tc::kBoxBytes;
using tc::kBoxCols;

// Warps 0-7 are the elementwise warps: warp w serves tensor-memory lanes
// 32 (w % 4) .. + 31 (tile rows) and the column half w / 4 (keys or queries
// 64 (w / 4) .. + 63), so each sub-partition runs two of them.  Warp 8 issues
// TMA loads, warp 9 (one thread) tcgen05.mma.
constexpr int kElemWarps = 8;
constexpr int kThreads = 32 * (kElemWarps + 2);
constexpr int kWarpTma = kElemWarps;
constexpr int kWarpMma = kElemWarps + 1;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;      // S or S^T (fp32); the 16-bit P / dS packed into its first 64 columns
constexpr uint32_t kColDP = 128;   // dP or dP^T (fp32); the 16-bit dS^T packed into its first 64 columns
constexpr uint32_t kColAcc = 256;  // dQ; or dV at kColAcc and dK at kColAcc + D
// The elementwise warps pack their 16-bit results (P, dS) into the first half
// of the column range they read: keys 0..63 -> columns 0..31, keys 64..127 ->
// columns 64..95.  K-step kk (16 keys) of a product reading them from tensor
// memory therefore starts at this column.
__host__ __device__ constexpr uint32_t packed_col(int kk) { return (kk >> 2) * 64 + (kk & 3) * 8; }
// The dQ kernel's second S buffer (after dQ): S(t) lives in buffer t % 2.
template <int D>
__host__ __device__ constexpr uint32_t col_sbuf(int b) { return b ? kColAcc + D : kColS; }
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kStatBytes = 128 * 8;  // (b, delta) of one 128-row query tile

struct Params {
    int S;
    int S_pad;   // row pitch of the row statistics (a multiple of 128)
    int BH;      // query slices: batch x heads
    int H;       // query heads; slice bh = b H + h
    int kv_group;  // query heads per K/V head: query head h reads K/V head h / kv_group
    int BHkv;    // K/V slices: batch x heads / kv_group
    int n_qt;    // 128-row tiles per slice
    int causal;
    float scale;
    float scale_log2;
    const float2 *rowstat;  // [BH][S_pad]: (b_n, delta_n)
};

template <typename T>
__device__ __forceinline__ float load_f(const void *base, size_t idx) {
    return Elem<T>::to_float(static_cast<const T *>(base)[idx]);
}
template <>
__device__ __forceinline__ float load_f<float>(const void *base, size_t idx) {
    return static_cast<const float *>(base)[idx];
}

// One warp per row of the padded [BH][S_pad] grid.
template <typename T>
__global__ void __launch_bounds__(256)
    bwd_rowstat_kernel(const T *__restrict__ dout, const float *__restrict__ o32, const float *__restrict__ m32,
                       const float *__restrict__ l32, const void *__restrict__ m_in, const void *__restrict__ l_in,
                       float2 *__restrict__ rowstat, int S, int S_pad, int D, long long n_rows) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    for (long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n_rows;
         r += warps) {
        const long long bh = r / S_pad;
        const int n = static_cast<int>(r - bh * S_pad);
        if (n >= S) {
            if (lane == 0) rowstat[r] = make_float2(0.f, 0.f);
            continue;
        }
        const size_t row = static_cast<size_t>(bh) * S + n;
        const T *dr = dout + row * D;
        const float *orow = o32 + row * D;
        float acc = 0.f;
        for (int d = lane; d < D; d += 32) acc = fmaf(Elem<T>::to_float(dr[d]), orow[d], acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            const float mt = load_f<T>(m_in, row);
            const float lt = load_f<T>(l_in, row);
            const float f = expf(m32[row] - mt) * (l32[row] / lt);
            rowstat[r] = make_float2(mt * kLog2e + log2f(lt), f * acc);
        }
    }
}

// Writes 32 fp32 columns (times `mul`) of one tile row as 16-bit values into a
// [128 rows][D] tile laid out as the TMA tensor map's 128-byte-swizzled boxes.
template <bool BF16>
__device__ __forceinline__ void stage_row32(uint8_t *tile, int row, int cc, const uint32_t (&o)[32], float mul) {
    uint32_t pk[16];
#pragma unroll
    for (int t = 0; t < 16; ++t)
        pk[t] = ptx::pack2<BF16>(__uint_as_float(o[2 * t]) * mul, __uint_as_float(o[2 * t + 1]) * mul);
    uint8_t *box = tile + (cc >> 1) * kBoxBytes + row * 128;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
        const int chunk = (cc & 1) * 4 + q4;
        *reinterpret_cast<uint4 *>(box + ((chunk ^ (row & 7)) * 16)) =
            make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
    }
}

// ============================================================== dQ kernel
template <int D>
struct CfgQ {
    static_assert(D == 64 || D == 128, "head size 64 or 128");
    static constexpr int kBoxes = D / kBoxCols;
    static constexpr int kTile = kBoxes * kBoxBytes;
    // K(t) is read by S(t), issued one key tile ahead, and by dQ(t): three K
    // tiles are live at once; V(t) only by dP(t).
    static constexpr int kKStages = (D == 64) ? 4 : 3;
    static constexpr int kVStages = (D == 64) ? 4 : 2;
    static constexpr int kOffQ = 0;
    static constexpr int kOffDO = kTile;
    static constexpr int kOffK = 2 * kTile;
    static constexpr int kOffV = kOffK + kKStages * kTile;
    static constexpr int kOffBars = kOffV + kVStages * kTile;
    static constexpr int kNumBars = 1 + 2 * kKStages + 2 * kVStages + 7;
    static constexpr int kSmemBytes = kOffBars + kNumBars * 8 + 16 + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dq, const Params p) {
    using namespace ptx;
    using C = CfgQ<D>;
    constexpr int KS = C::kKStages;
    constexpr int VS = C::kVStages;
    constexpr int TILE = C::kTile;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t *sQ = smem + C::kOffQ;
    uint8_t *sDO = smem + C::kOffDO;
    uint8_t *sK = smem + C::kOffK;  // [KS][TILE]
    uint8_t *sV = smem + C::kOffV;  // [VS][TILE]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kOffBars);
    uint64_t *qd_full = bars;
    uint64_t *k_full = bars + 1;       // [KS]
    uint64_t *k_empty = k_full + KS;   // [KS]
    uint64_t *v_full = k_empty + KS;   // [VS]
    uint64_t *v_empty = v_full + VS;   // [VS]
    uint64_t *s_full = v_empty + VS;   // [2]: S(t) in S buffer t % 2
    uint64_t *dp_full = s_full + 2;    // dP(t) in the dP buffer
    uint64_t *p_full = dp_full + 1;    // dS(t) packed (S(t) and dP(t) read)
    uint64_t *acc_full = p_full + 1;
    uint64_t *mma_done = acc_full + 1;
    uint64_t *staged = mma_done + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(staged + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int bid = blockIdx.x;
    const int qt = p.causal ? (p.n_qt - 1 - bid / p.BH) : (bid / p.BH);  // heaviest tiles first
    const int bh = bid % p.BH;
    const int bb = bh / p.H, hh = bh - bb * p.H, hkv = hh / p.kv_group;
    const int n_kv = p.causal ? qt + 1 : p.n_qt;

    if (threadIdx.x == 0) {
        mbar_init(qd_full, 1);
        for (int s = 0; s < KS; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < VS; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(dp_full, 1);
        mbar_init(p_full, kElemWarps);
        mbar_init(acc_full, 1);
        mbar_init(mma_done, 1);
        mbar_init(staged, kElemWarps);
        *abort_flag = (*reinterpret_cast<volatile unsigned int *>(&g_device_error) != 0u) ? 1 : 0;
        fence_mbarrier_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool skip = *abort_flag != 0;

    if (skip) {
        // fall through to the teardown
    } else if (warp == kWarpTma) {
        if (lane == 0) {
            tma_prefetch_desc(&tm_q);
            tma_prefetch_desc(&tm_k);
            tma_prefetch_desc(&tm_v);
            tma_prefetch_desc(&tm_do);
            mbar_arrive_expect_tx(qd_full, 2 * TILE);
            for (int b = 0; b < C::kBoxes; ++b) {
                tma_load_4d(sQ + b * kBoxBytes, &tm_q, qd_full, b * kBoxCols, qt * 128, hh, bb);
                tma_load_4d(sDO + b * kBoxBytes, &tm_do, qd_full, b * kBoxCols, qt * 128, hh, bb);
            }
            int issued = 0;
            for (int t = 0; t < n_kv; ++t) {
                const int sk = t % KS, sv = t % VS;
                if (t >= KS && !mbar_wait(&k_empty[sk], ((t / KS) - 1) & 1, abort_flag)) break;
                mbar_arrive_expect_tx(&k_full[sk], TILE);
                for (int b = 0; b < C::kBoxes; ++b)
                    tma_load_4d(sK + sk * TILE + b * kBoxBytes, &tm_k, &k_full[sk], b * kBoxCols, t * 128, hkv, bb);
                if (t >= VS && !mbar_wait(&v_empty[sv], ((t / VS) - 1) & 1, abort_flag)) {
                    issued = -(t + 1);  // K(t) issued, V(t) not
                    break;
                }
                mbar_arrive_expect_tx(&v_full[sv], TILE);
                for (int b = 0; b < C::kBoxes; ++b)
                    tma_load_4d(sV + sv * TILE + b * kBoxBytes, &tm_v, &v_full[sv], b * kBoxCols, t * 128, hkv, bb);
                issued = t + 1;
            }
            if (*abort_flag) {
                // Let the copies already issued land before shared memory is released.
                volatile int never = 0;
                mbar_wait(qd_full, 0, &never);
                const int nk = issued < 0 ? -issued : issued;  // K tiles issued
                const int nv = issued < 0 ? -issued - 1 : issued;
                for (int i = max(0, nk - KS); i < nk; ++i) mbar_wait(&k_full[i % KS], (i / KS) & 1, &never);
                for (int i = max(0, nv - VS); i < nv; ++i) mbar_wait(&v_full[i % VS], (i / VS) & 1, &never);
            }
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t kIdS = idesc_f16(128, 128, BF16 ? 1 : 0, 0, 0);
            constexpr uint32_t kIdAcc = idesc_f16(128, D, BF16 ? 1 : 0, 0, 1);
            const uint32_t q_addr = smem_u32(sQ);
            const uint32_t do_addr = smem_u32(sDO);
            // dQ += dS(t) K_t: dS from tensor memory, K_t (keys x D, D contiguous) as an MN-major B.
            auto issue_dq = [&](int t) {
                const uint32_t k_addr = smem_u32(sK + (t % KS) * TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts(tmem + kColAcc, tmem + col_sbuf<D>(t & 1) + packed_col(kk),
                           smem_desc_sw128(k_addr + kk * 2048, kBoxBytes, 1024), kIdAcc, (t > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&k_empty[t % KS]);
            };
            auto issue_s = [&](int t) {
                const uint32_t k_addr = smem_u32(sK + (t % KS) * TILE);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
                    mma_ss(tmem + col_sbuf<D>(t & 1), smem_desc_sw128(q_addr + off, 16, 1024),
                           smem_desc_sw128(k_addr + off, 16, 1024), kIdS, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[t & 1]);
            };
            auto issue_dp = [&](int t) {
                const uint32_t v_addr = smem_u32(sV + (t % VS) * TILE);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
                    mma_ss(tmem + kColDP, smem_desc_sw128(do_addr + off, 16, 1024),
                           smem_desc_sw128(v_addr + off, 16, 1024), kIdS, kk > 0 ? 1u : 0u);
                }
                mma_commit(dp_full);
                mma_commit(&v_empty[t % VS]);
            };
            auto wait_k = [&](int t) { return mbar_wait(&k_full[t % KS], (t / KS) & 1, abort_flag); };
            auto wait_v = [&](int t) { return mbar_wait(&v_full[t % VS], (t / VS) & 1, abort_flag); };
            // Key tile t: S(t+1) goes out as soon as dQ(t-1) (the last reader of
            // its buffer) has been issued, so the elementwise warps' exps of
            // tile t+1 start right after they finish tile t; dP(t+1) waits for
            // them to have read dP(t); dQ(t) last.
            bool ok = mbar_wait(qd_full, 0, abort_flag) && wait_k(0) && wait_v(0);
            if (ok) {
                tc_fence_after();
                issue_s(0);
                issue_dp(0);
            }
            for (int t = 0; ok && t < n_kv; ++t) {
                if (t + 1 < n_kv) {
                    if (!(ok = wait_k(t + 1))) break;
                    tc_fence_after();
                    issue_s(t + 1);
                }
                if (!(ok = mbar_wait(p_full, t & 1, abort_flag))) break;
                tc_fence_after();
                if (t + 1 < n_kv) {
                    if (!(ok = wait_v(t + 1))) break;
                    tc_fence_after();
                    issue_dp(t + 1);
                }
                issue_dq(t);
            }
            if (ok) mma_commit(acc_full);
            mma_commit(mma_done);
            volatile int never = 0;
            mbar_wait(mma_done, 0, &never);
        }
    } else {
        // ------------------------------------------------------------ elementwise warps
        const int quarter = warp & 3, half = warp >> 2;
        const int r = quarter * 32 + lane;  // tile row == tensor-memory lane
        const int row = qt * 128 + r;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        float b = 0.f, delta = 0.f;
        if (row < p.S) {
            const float2 st = p.rowstat[static_cast<size_t>(bh) * p.S_pad + row];
            b = st.x;
            delta = st.y;
        }
        const float c2 = p.scale_log2;
        const float2 nd2 = make_float2(-delta, -delta);
        bool ok = true;
        for (int t = 0; t < n_kv; ++t) {
            int lim = p.S - t * 128;  // keys [lim, 128) of this tile are masked for this row
            if (p.causal) lim = min(lim, row - t * 128 + 1);
            const bool masked = __any_sync(0xffffffffu, lim < 128);
            const uint32_t sbuf = lane_base + col_sbuf<D>(t & 1);
            // Phase 1: e = 2^(S c2 - b) for this warp's 64 keys.
            if (!(ok = mbar_wait_warp(&s_full[t & 1], (t >> 1) & 1, abort_flag))) break;
            tc_fence_after();
            float ev[64];
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c = 2 * half + cc;  // 32-key chunk
                uint32_t sv[32];
                tmem_ld32(sbuf + c * 32, sv);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float s0 = __uint_as_float(sv[i]);
                    if (masked && c * 32 + i >= lim) s0 = -INFINITY;
                    ev[cc * 32 + i] = ex2_approx(fmaf(s0, c2, -b));
                }
            }
            // Phase 2: dS = e (dP - delta), packed into the S buffer's columns
            // this warp has read.
            if (!(ok = mbar_wait_warp(dp_full, t & 1, abort_flag))) break;
            tc_fence_after();
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c = 2 * half + cc;
                uint32_t dv[32];
                tmem_ld32(lane_base + kColDP + c * 32, dv);
                tmem_wait_ld();
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float2 g = mul2(make_float2(ev[cc * 32 + 2 * i], ev[cc * 32 + 2 * i + 1]),
                                          add2(make_float2(__uint_as_float(dv[2 * i]), __uint_as_float(dv[2 * i + 1])),
                                               nd2));
                    w[i] = pack2<BF16>(g.x, g.y);
                }
                tmem_st16(sbuf + half * 64 + cc * 16, w);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok) ok = mbar_wait_warp(acc_full, 0, abort_flag);
        if (ok) {
            tc_fence_after();
            // Every MMA has completed: Q's shared memory stages the dQ tile.
#pragma unroll
            for (int i = 0; i < D / 64; ++i) {
                const int cc = half * (D / 64) + i;  // 32-column chunk of dQ
                uint32_t o[32];
                tmem_ld32(lane_base + kColAcc + cc * 32, o);
                tmem_wait_ld();
                stage_row32<BF16>(sQ, r, cc, o, p.scale);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(staged);
            if (threadIdx.x == 0 && mbar_wait(staged, 0, abort_flag)) {
                for (int bx = 0; bx < C::kBoxes; ++bx)
                    tma_store_4d(&tm_dq, sQ + bx * kBoxBytes, bx * kBoxCols, qt * 128, hh, bb);
                tma_store_commit();
                tma_store_wait_read0();
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && *abort_flag && !skip) report_device_error(PMKL_DEVERR_TIMEOUT);
}

// ============================================================== dK, dV kernel
template <int D>
struct CfgKV {
    static_assert(D == 64 || D == 128, "head size 64 or 128");
    static constexpr int kBoxes = D / kBoxCols;
    static constexpr int kTile = kBoxes * kBoxBytes;
    static constexpr int kStages = (D == 64) ? 4 : 2;    // (Q, dO, row stats) in flight
    static constexpr int kStage = 2 * kTile + kStatBytes;  // a multiple of 1024
    static constexpr int kOffK = 0;
    static constexpr int kOffV = kTile;
    static constexpr int kOffRing = 2 * kTile;
    static constexpr int kOffBars = kOffRing + kStages * kStage;
    static constexpr int kNumBars = 1 + 2 * kStages + 7;
    static constexpr int kSmemBytes = kOffBars + kNumBars * 8 + 16 + 1024;
    static_assert(kStage % 1024 == 0, "stage alignment");
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                        const __grid_constant__ CUtensorMap tm_dk, const __grid_constant__ CUtensorMap tm_dv,
                        const Params p) {
    using namespace ptx;
    using C = CfgKV<D>;
    constexpr int NS = C::kStages;
    constexpr int TILE = C::kTile;
    constexpr int STAGE = C::kStage;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t *sK = smem + C::kOffK;
    uint8_t *sV = smem + C::kOffV;
    uint8_t *sRing = smem + C::kOffRing;  // stage s: Q, dO, (b, delta)[128]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kOffBars);
    uint64_t *kv_full = bars;
    uint64_t *qd_full = bars + 1;       // [NS]
    uint64_t *qd_empty = qd_full + NS;  // [NS]
    uint64_t *s_full = qd_empty + NS;   // S^T(x) in tensor memory
    uint64_t *dp_full = s_full + 1;     // dP^T(x) in tensor memory
    uint64_t *p1_full = dp_full + 1;    // P^T(x) packed (S^T read)
    uint64_t *p2_full = p1_full + 1;    // dS^T(x) packed (dP^T read)
    uint64_t *acc_full = p2_full + 1;
    uint64_t *mma_done = acc_full + 1;
    uint64_t *staged = mma_done + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(staged + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int bid = blockIdx.x;
    const int kt = bid / p.BHkv;  // causal: key tile 0 meets every query tile, so ascending = heaviest first
    const int bkv = bid % p.BHkv;
    const int Hkv = p.H / p.kv_group;
    const int bb = bkv / Hkv, hkv = bkv - bb * Hkv;
    const int i0 = p.causal ? kt : 0;
    const int n_q = p.n_qt - i0;     // query tiles per query head
    const int n_x = n_q * p.kv_group;  // (query head of the group, query tile) steps

    if (threadIdx.x == 0) {
        mbar_init(kv_full, 1);
        for (int s = 0; s < NS; ++s) {
            mbar_init(&qd_full[s], 1);
            mbar_init(&qd_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(dp_full, 1);
        mbar_init(p1_full, kElemWarps);
        mbar_init(p2_full, kElemWarps);
        mbar_init(acc_full, 1);
        mbar_init(mma_done, 1);
        mbar_init(staged, kElemWarps);
        *abort_flag = (*reinterpret_cast<volatile unsigned int *>(&g_device_error) != 0u) ? 1 : 0;
        fence_mbarrier_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool skip = *abort_flag != 0;

    if (skip) {
        // fall through to the teardown
    } else if (warp == kWarpTma) {
        if (lane == 0) {
            tma_prefetch_desc(&tm_q);
            tma_prefetch_desc(&tm_k);
            tma_prefetch_desc(&tm_v);
            tma_prefetch_desc(&tm_do);
            mbar_arrive_expect_tx(kv_full, 2 * TILE);
            for (int b = 0; b < C::kBoxes; ++b) {
                tma_load_4d(sK + b * kBoxBytes, &tm_k, kv_full, b * kBoxCols, kt * 128, hkv, bb);
                tma_load_4d(sV + b * kBoxBytes, &tm_v, kv_full, b * kBoxCols, kt * 128, hkv, bb);
            }
            int issued = 0;
            for (int x = 0; x < n_x; ++x) {
                const int s = x % NS;
                const int g = x / n_q;
                const int i = i0 + (x - g * n_q);
                const int hh = hkv * p.kv_group + g;  // query head
                if (x >= NS && !mbar_wait(&qd_empty[s], ((x / NS) - 1) & 1, abort_flag)) break;
                uint8_t *st = sRing + s * STAGE;
                mbar_arrive_expect_tx(&qd_full[s], 2 * TILE + kStatBytes);
                for (int b = 0; b < C::kBoxes; ++b) {
                    tma_load_4d(st + b * kBoxBytes, &tm_q, &qd_full[s], b * kBoxCols, i * 128, hh, bb);
                    tma_load_4d(st + TILE + b * kBoxBytes, &tm_do, &qd_full[s], b * kBoxCols, i * 128, hh, bb);
                }
                bulk_load(st + 2 * TILE,
                          p.rowstat + static_cast<size_t>(bb * p.H + hh) * p.S_pad + static_cast<size_t>(i) * 128,
                          kStatBytes, &qd_full[s]);
                issued = x + 1;
            }
            if (*abort_flag) {
                volatile int never = 0;
                mbar_wait(kv_full, 0, &never);
                for (int x = max(0, issued - NS); x < issued; ++x) mbar_wait(&qd_full[x % NS], (x / NS) & 1, &never);
            }
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            constexpr uint32_t kIdS = idesc_f16(128, 128, BF16 ? 1 : 0, 0, 0);
            constexpr uint32_t kIdAcc = idesc_f16(128, D, BF16 ? 1 : 0, 0, 1);
            const uint32_t k_addr = smem_u32(sK);
            const uint32_t v_addr = smem_u32(sV);
            // Two chains per query tile x, each hidden behind the other's
            // elementwise phase:
            //   phase 1 (S^T -> P^T) -> dV(x) += P^T dO_x -> S^T(x+1)  (S buffer)
            //   phase 2 (dP^T -> dS^T) -> dK(x) += dS^T Q_x -> dP^T(x+1)  (dP buffer)
            // Each buffer is overwritten only after the product that reads its
            // packed 16-bit half (one thread's MMAs execute in order).
            auto stage_addr = [&](int x) { return smem_u32(sRing + (x % NS) * STAGE); };
            auto issue_s = [&](int x) {
                const uint32_t q_addr = stage_addr(x);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
                    mma_ss(tmem + kColS, smem_desc_sw128(k_addr + off, 16, 1024),
                           smem_desc_sw128(q_addr + off, 16, 1024), kIdS, kk > 0 ? 1u : 0u);
                }
                mma_commit(s_full);
            };
            auto issue_dp = [&](int x) {
                const uint32_t do_addr = stage_addr(x) + TILE;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
                    mma_ss(tmem + kColDP, smem_desc_sw128(v_addr + off, 16, 1024),
                           smem_desc_sw128(do_addr + off, 16, 1024), kIdS, kk > 0 ? 1u : 0u);
                }
                mma_commit(dp_full);
            };
            // The query-tile operands (queries x D, D contiguous) as MN-major B.
            auto issue_dv = [&](int x) {
                const uint32_t do_addr = stage_addr(x) + TILE;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts(tmem + kColAcc, tmem + kColS + packed_col(kk),
                           smem_desc_sw128(do_addr + kk * 2048, kBoxBytes, 1024), kIdAcc, (x > 0 || kk > 0) ? 1u : 0u);
            };
            auto issue_dk = [&](int x) {
                const uint32_t q_addr = stage_addr(x);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts(tmem + kColAcc + D, tmem + kColDP + packed_col(kk),
                           smem_desc_sw128(q_addr + kk * 2048, kBoxBytes, 1024), kIdAcc, (x > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&qd_empty[x % NS]);  // the last product reading stage x % NS
            };
            bool ok = mbar_wait(kv_full, 0, abort_flag) && mbar_wait(&qd_full[0], 0, abort_flag);
            if (ok) {
                tc_fence_after();
                issue_s(0);
                issue_dp(0);
            }
            for (int x = 0; ok && x < n_x; ++x) {
                if (!(ok = mbar_wait(p1_full, x & 1, abort_flag))) break;
                tc_fence_after();
                issue_dv(x);
                if (x + 1 < n_x) {
                    if (!(ok = mbar_wait(&qd_full[(x + 1) % NS], ((x + 1) / NS) & 1, abort_flag))) break;
                    tc_fence_after();
                    issue_s(x + 1);
                }
                if (!(ok = mbar_wait(p2_full, x & 1, abort_flag))) break;
                tc_fence_after();
                issue_dk(x);
                if (x + 1 < n_x) issue_dp(x + 1);
            }
            if (ok) mma_commit(acc_full);
            mma_commit(mma_done);
            volatile int never = 0;
            mbar_wait(mma_done, 0, &never);
        }
    } else {
        // ------------------------------------------------------------ elementwise warps
        const int quarter = warp & 3, half = warp >> 2;
        const int r = quarter * 32 + lane;  // key row of the tile == tensor-memory lane
        const int key = kt * 128 + r;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        const float c2 = p.scale_log2;
        bool ok = true;
        for (int x = 0; x < n_x; ++x) {
            const float4 *st = reinterpret_cast<const float4 *>(sRing + (x % NS) * STAGE + 2 * TILE);
            const int qbase = (i0 + x % n_q) * 128;
            const int lo = p.causal ? key - qbase : 0;  // queries [0, lo) precede this key
            const int hi = p.S - qbase;                  // queries [hi, 128) are past the end
            const bool masked = __any_sync(0xffffffffu, lo > 0 || hi < 128);
            // Phase 1: P^T = 2^(S^T c2 - b) for this warp's 64 queries, kept in
            // fp32 for phase 2 and packed to 16 bits for dV.
            if (!(ok = mbar_wait_warp(s_full, x & 1, abort_flag))) break;
            tc_fence_after();
            float pv[64];
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c = 2 * half + cc;  // 32-query chunk
                uint32_t sv[32];
                tmem_ld32(lane_base + kColS + c * 32, sv);
                tmem_wait_ld();
                uint32_t wp[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n0 = c * 32 + 2 * i;
                    const float4 bd = st[n0 >> 1];  // (b, delta) of queries n0, n0 + 1
                    float s0 = __uint_as_float(sv[2 * i]), s1 = __uint_as_float(sv[2 * i + 1]);
                    if (masked) {
                        if (n0 < lo || n0 >= hi) s0 = -INFINITY;
                        if (n0 + 1 < lo || n0 + 1 >= hi) s1 = -INFINITY;
                    }
                    pv[cc * 32 + 2 * i] = ex2_approx(fmaf(s0, c2, -bd.x));
                    pv[cc * 32 + 2 * i + 1] = ex2_approx(fmaf(s1, c2, -bd.z));
                    wp[i] = pack2<BF16>(pv[cc * 32 + 2 * i], pv[cc * 32 + 2 * i + 1]);
                }
                tmem_st16(lane_base + kColS + half * 64 + cc * 16, wp);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p1_full);
            // Phase 2: dS^T = P^T (dP^T - delta), packed to 16 bits for dK.
            if (!(ok = mbar_wait_warp(dp_full, x & 1, abort_flag))) break;
            tc_fence_after();
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int c = 2 * half + cc;
                uint32_t dv[32];
                tmem_ld32(lane_base + kColDP + c * 32, dv);
                tmem_wait_ld();
                uint32_t wd[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n0 = c * 32 + 2 * i;
                    const float4 bd = st[n0 >> 1];
                    const float2 g =
                        mul2(make_float2(pv[cc * 32 + 2 * i], pv[cc * 32 + 2 * i + 1]),
                             add2(make_float2(__uint_as_float(dv[2 * i]), __uint_as_float(dv[2 * i + 1])),
                                  make_float2(-bd.y, -bd.w)));
                    wd[i] = pack2<BF16>(g.x, g.y);
                }
                tmem_st16(lane_base + kColDP + half * 64 + cc * 16, wd);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p2_full);
        }
        if (ok) ok = mbar_wait_warp(acc_full, 0, abort_flag);
        if (ok) {
            tc_fence_after();
            // Every MMA has completed: K's and V's shared memory stage dV and dK.
#pragma unroll
            for (int i = 0; i < D / 64; ++i) {
                const int cc = half * (D / 64) + i;  // 32-column chunk of dV and dK
                uint32_t o[32];
                tmem_ld32(lane_base + kColAcc + cc * 32, o);
                tmem_wait_ld();
                stage_row32<BF16>(sK, r, cc, o, 1.f);
                tmem_ld32(lane_base + kColAcc + D + cc * 32, o);
                tmem_wait_ld();
                stage_row32<BF16>(sV, r, cc, o, p.scale);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(staged);
            if (threadIdx.x == 0 && mbar_wait(staged, 0, abort_flag)) {
                for (int bx = 0; bx < C::kBoxes; ++bx) {
                    tma_store_4d(&tm_dv, sK + bx * kBoxBytes, bx * kBoxCols, kt * 128, hkv, bb);
                    tma_store_4d(&tm_dk, sV + bx * kBoxBytes, bx * kBoxCols, kt * 128, hkv, bb);
                }
                tma_store_commit();
                tma_store_wait_read0();
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && *abort_flag && !skip) report_device_error(PMKL_DEVERR_TIMEOUT);
}

}  // namespace bwd
}  // namespace pmkl_b200
