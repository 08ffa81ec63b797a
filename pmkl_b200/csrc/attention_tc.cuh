// attention_tc.cuh -- tensor-core (tcgen05) flash attention forward for
// sm_100a, fp16/bf16 inputs, head size 64 or 128.
//
// Computes what pmkl::nlp::causal_attention_forward computes
// (pmkl/nlp/causal_attention.h:145-256): per (batch*head, 128-row query tile)
// an online softmax over key tiles, writing O (already normalised), the row
// max m of the scaled scores and the exp-sum l.  The reference walks every
// key tile with fp32 CUDA-core dot products and masks with -1e20; here
//   * one warp issues TMA loads: Q once, K and V through an NST-stage ring;
//   * one thread issues tcgen05.mma: S = Q K^T into tensor memory (two S
//     buffers, so S(j+1) is computed while the softmax reads S(j)), then
//     O += P V with P read from tensor memory;
//   * four warps (one per tensor-memory lane quarter, one thread per query
//     row) run the online softmax on S in registers: row max, exp2 with the
//     scale folded in, row sum, P packed to 16-bit into tensor memory, and the
//     O rescale, done only when the running max grew by more than 2^8
//     (otherwise the stale max stays the reference point and the final m/l
//     are corrected once in the epilogue);
//   * key tiles wholly above the diagonal are never loaded (causal skip); only
//     the diagonal tile and a ragged last tile are masked;
//   * the epilogue normalises O by 1/l, stages it in shared memory and writes
//     it with a TMA store (rows past seq are clipped by the tensor map).
//
// Precision: when every row of a tile sees at most 128 keys (causal query
// tile 0, or seq <= 128), P is split into hi + lo 16-bit parts and both are
// multiplied with V, so that O keeps fp32-level accuracy on rows with few
// keys, where a single rounding of P to bf16 (2^-9 relative) would show.
#pragma once

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace pmkl_b200 {
namespace tc {

constexpr int kBM = 128;                   // query rows per tile (MMA M)
constexpr int kBN = 128;                   // keys per tile
constexpr int kBoxCols = 64;               // elements per 128-byte swizzle row
constexpr int kBoxBytes = 128 * 128;       // one TMA box: 128 rows x 128 bytes
constexpr int kThreads = 192;              // 4 softmax warps + TMA warp + MMA warp
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColP = 256, kColPlo = 320, kColO = 384;

template <int D>
struct Cfg {
    static_assert(D == 64 || D == 128, "tcgen05 path supports head size 64 or 128");
    static constexpr int kBoxes = D / kBoxCols;
    static constexpr int kTileBytes = kBoxes * kBoxBytes;  // 128 rows x D x 2 bytes
    static constexpr int kStages = (D == 64) ? 4 : 3;
    static constexpr int kNumBars = 1 + 3 * kStages + 2 + 2 + 1 + 1 + 1;
    static constexpr int kSmemBytes = kTileBytes * (1 + 2 * kStages) + 256 + 1024;  // + barriers, + align slack
};

struct Params {
    int S;
    int BH;
    int n_qt;       // query tiles per (batch, head)
    int causal;
    int out_dtype;  // PMKL_DTYPE_*; 16-bit outputs go through the TMA store
    float scale;        // natural-log score scale (for m)
    float scale_log2;   // scale * log2(e)
    void *o_f32;    // O when out_dtype == F32 (plain stores)
    void *m_out;
    void *l_out;
};

template <bool BF16>
__device__ __forceinline__ void unpack2(uint32_t u, float &lo, float &hi) {
    if (BF16) {
        lo = __uint_as_float(u << 16);
        hi = __uint_as_float(u & 0xFFFF0000u);
    } else {
        __half2 h = *reinterpret_cast<__half2 *>(&u);
        lo = __low2float(h);
        hi = __high2float(h);
    }
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                       const Params p) {
    using namespace ptx;
    using C = Cfg<D>;
    constexpr int NST = C::kStages;
    constexpr int TILE = C::kTileBytes;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t *sQ = smem;
    uint8_t *sK0 = smem + TILE;
    uint8_t *sV0 = smem + TILE * (1 + NST);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + TILE * (1 + 2 * NST));
    uint64_t *bar_q = bars;
    uint64_t *bar_kfull = bars + 1;
    uint64_t *bar_vfull = bar_kfull + NST;
    uint64_t *bar_kvempty = bar_vfull + NST;
    uint64_t *bar_sfull = bar_kvempty + NST;  // [2]
    uint64_t *bar_sfree = bar_sfull + 2;      // [2]
    uint64_t *bar_pfull = bar_sfree + 2;
    uint64_t *bar_odone = bar_pfull + 1;
    uint64_t *bar_final = bar_odone + 1;
    uint64_t *bar_ostage = bar_final + 1;  // softmax warps -> store thread: O tile staged
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_ostage + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Heaviest query tiles first (causal work grows with the tile index).
    const int bid = blockIdx.x;
    const int qt = p.causal ? (p.n_qt - 1 - bid / p.BH) : (bid / p.BH);
    const int bh = bid % p.BH;
    const int n_kv_all = (p.S + kBN - 1) / kBN;
    const int n_kv = p.causal ? min(qt + 1, n_kv_all) : n_kv_all;
    const bool hilo = (n_kv == 1) && (p.causal ? (qt == 0) : true);

    if (threadIdx.x == 0) {
        mbar_init(bar_q, 1);
        for (int s = 0; s < NST; ++s) {
            mbar_init(&bar_kfull[s], 1);
            mbar_init(&bar_vfull[s], 1);
            mbar_init(&bar_kvempty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bar_sfull[b], 1);
            mbar_init(&bar_sfree[b], 4);
        }
        mbar_init(bar_pfull, 4);
        mbar_init(bar_odone, 1);
        mbar_init(bar_final, 1);
        mbar_init(bar_ostage, 4);
        // Fast fail: once any CTA has abandoned a wait (the device error word
        // is set), later CTAs skip their work instead of each timing out.
        *abort_flag = (*reinterpret_cast<volatile unsigned int *>(&g_device_error) != 0u) ? 1 : 0;
        fence_mbarrier_init();
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool skip = *abort_flag != 0;

    if (skip) {
        // nothing: fall through to the teardown
    } else if (warp == 4) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tm_q);
            tma_prefetch_desc(&tm_k);
            tma_prefetch_desc(&tm_v);
            mbar_arrive_expect_tx(bar_q, TILE);
            for (int b = 0; b < C::kBoxes; ++b) tma_load_3d(sQ + b * kBoxBytes, &tm_q, bar_q, b * kBoxCols, qt * kBM, bh);
            int issued = 0;
            for (int j = 0; j < n_kv; ++j) {
                const int s = j % NST;
                const int u = j / NST;
                if (u > 0 && !mbar_wait(&bar_kvempty[s], (u - 1) & 1, abort_flag)) break;
                uint8_t *sk = sK0 + s * TILE;
                uint8_t *sv = sV0 + s * TILE;
                mbar_arrive_expect_tx(&bar_kfull[s], TILE);
                for (int b = 0; b < C::kBoxes; ++b)
                    tma_load_3d(sk + b * kBoxBytes, &tm_k, &bar_kfull[s], b * kBoxCols, j * kBN, bh);
                mbar_arrive_expect_tx(&bar_vfull[s], TILE);
                for (int b = 0; b < C::kBoxes; ++b)
                    tma_load_3d(sv + b * kBoxBytes, &tm_v, &bar_vfull[s], b * kBoxCols, j * kBN, bh);
                issued = j + 1;
            }
            if (*abort_flag) {
                // Let the copies already issued land before shared memory is released.
                volatile int never = 0;
                mbar_wait(bar_q, 0, &never);
                for (int j = max(0, issued - NST); j < issued; ++j) {
                    mbar_wait(&bar_kfull[j % NST], (j / NST) & 1, &never);
                    mbar_wait(&bar_vfull[j % NST], (j / NST) & 1, &never);
                }
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t kIdescS = idesc_f16(kBM, kBN, BF16 ? 1 : 0, 0, 0);
            constexpr uint32_t kIdescO = idesc_f16(kBM, D, BF16 ? 1 : 0, 0, 1);
            const uint32_t q_addr = smem_u32(sQ);
            bool ok = mbar_wait(bar_q, 0, abort_flag);
            for (int j = 0; ok && j <= n_kv; ++j) {
                if (j < n_kv) {
                    const int s = j % NST;
                    const int sb = j & 1;
                    if (!mbar_wait(&bar_kfull[s], (j / NST) & 1, abort_flag)) break;
                    if (j >= 2 && !mbar_wait(&bar_sfree[sb], ((j >> 1) - 1) & 1, abort_flag)) break;
                    tc_fence_after();
                    const uint32_t k_addr = smem_u32(sK0 + s * TILE);
                    const uint32_t d_tmem = tmem + (sb ? kColS1 : kColS0);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
                        const uint64_t a = smem_desc_sw128(q_addr + off, 16, 1024);
                        const uint64_t b = smem_desc_sw128(k_addr + off, 16, 1024);
                        mma_ss(d_tmem, a, b, kIdescS, kk > 0 ? 1u : 0u);
                    }
                    mma_commit(&bar_sfull[sb]);
                }
                if (j >= 1) {
                    const int i = j - 1;
                    const int s = i % NST;
                    if (!mbar_wait(bar_pfull, i & 1, abort_flag)) break;
                    if (!mbar_wait(&bar_vfull[s], (i / NST) & 1, abort_flag)) break;
                    tc_fence_after();
                    const uint32_t v_addr = smem_u32(sV0 + s * TILE);
#pragma unroll
                    for (int kk = 0; kk < kBN / 16; ++kk) {
                        // V tile rows are keys (K of this product), D is contiguous (MN-major B):
                        // 16 keys = 2048 bytes, next 64-column box at +16 KB (LBO), 8-key groups at 1 KB (SBO).
                        const uint64_t b = smem_desc_sw128(v_addr + kk * 16 * 128, kBoxBytes, 1024);
                        mma_ts(tmem + kColO, tmem + kColP + kk * 8, b, kIdescO, (i > 0 || kk > 0) ? 1u : 0u);
                    }
                    if (hilo) {
#pragma unroll
                        for (int kk = 0; kk < kBN / 16; ++kk) {
                            const uint64_t b = smem_desc_sw128(v_addr + kk * 16 * 128, kBoxBytes, 1024);
                            mma_ts(tmem + kColO, tmem + kColPlo + kk * 8, b, kIdescO, 1u);
                        }
                    }
                    mma_commit(bar_odone);
                    mma_commit(&bar_kvempty[s]);
                }
            }
            // Drain every MMA issued before tensor memory is released.
            mma_commit(bar_final);
            volatile int never = 0;
            mbar_wait(bar_final, 0, &never);
        }
    } else {
        // ------------------------------------------------------------ softmax + epilogue
        const int row_local = warp * 32 + lane;  // == tensor-memory lane
        const int row = qt * kBM + row_local;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        const float c2 = p.scale_log2;
        float m_used = -INFINITY;  // reference point of the exp2 (raw score units)
        float m_true = -INFINITY;  // exact running max (raw score units)
        float l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int sb = j & 1;
            if (!mbar_wait_warp(&bar_sfull[sb], (j >> 1) & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            uint32_t sr[128];
            {
                uint32_t(&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[0]);
                uint32_t(&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[32]);
                uint32_t(&r2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[64]);
                uint32_t(&r3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sr[96]);
                const uint32_t sa = lane_base + (sb ? kColS1 : kColS0);
                tmem_ld32(sa + 0, r0);
                tmem_ld32(sa + 32, r1);
                tmem_ld32(sa + 64, r2);
                tmem_ld32(sa + 96, r3);
                tmem_wait_ld();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_sfree[sb]);

            float s[128];
#pragma unroll
            for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(sr[c]);
            const int kbase = j * kBN;
            int lim = p.S - kbase;  // valid columns of this tile for this row
            if (p.causal) lim = min(lim, row - kbase + 1);
            if (lim < kBN) {
#pragma unroll
                for (int c = 0; c < 128; ++c)
                    if (c >= lim) s[c] = -INFINITY;
            }
            float mx = s[0];
#pragma unroll
            for (int c = 1; c < 128; ++c) mx = fmaxf(mx, s[c]);
            m_true = fmaxf(m_true, mx);
            // Move the reference point only when the max grew by more than 2^8.
            const bool resc = (m_used == -INFINITY) ? (m_true != -INFINITY) : ((m_true - m_used) * c2 > 8.0f);
            const float m_new = resc ? m_true : m_used;
            const float fac = (resc && m_used != -INFINITY) ? ex2_approx((m_used - m_new) * c2) : (resc ? 0.f : 1.f);
            const float mref = (m_new == -INFINITY) ? 0.f : m_new * c2;

            uint32_t ph[64];
            uint32_t pl[64];
            float rs = 0.f;
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                const float p0 = ex2_approx(fmaf(s[2 * c], c2, -mref));
                const float p1 = ex2_approx(fmaf(s[2 * c + 1], c2, -mref));
                rs += p0 + p1;
                ph[c] = ptx::pack2<BF16>(p0, p1);
                if (hilo) {
                    float h0, h1;
                    unpack2<BF16>(ph[c], h0, h1);
                    pl[c] = ptx::pack2<BF16>(p0 - h0, p1 - h1);
                }
            }
            l = l * fac + rs;
            m_used = m_new;

            // O and the P slot are free once PV(j-1) has completed.
            if (j >= 1) {
                if (!mbar_wait_warp(bar_odone, (j - 1) & 1, abort_flag)) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, resc)) {
#pragma unroll
                    for (int cc = 0; cc < D / 32; ++cc) {
                        uint32_t o[32];
                        tmem_ld32(lane_base + kColO + cc * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * fac);
                        tmem_st32(lane_base + kColO + cc * 32, o);
                    }
                }
            }
            tmem_st32(lane_base + kColP, *reinterpret_cast<uint32_t(*)[32]>(&ph[0]));
            tmem_st32(lane_base + kColP + 32, *reinterpret_cast<uint32_t(*)[32]>(&ph[32]));
            if (hilo) {
                tmem_st32(lane_base + kColPlo, *reinterpret_cast<uint32_t(*)[32]>(&pl[0]));
                tmem_st32(lane_base + kColPlo + 32, *reinterpret_cast<uint32_t(*)[32]>(&pl[32]));
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_pfull);
        }

        if (ok && n_kv > 0) ok = mbar_wait_warp(bar_odone, (n_kv - 1) & 1, abort_flag);
        if (ok) {
            tc_fence_after();
            const float inv_l = 1.f / l;
            if (p.out_dtype == PMKL_DTYPE_F32) {
                float *orow = static_cast<float *>(p.o_f32) + (static_cast<size_t>(bh) * p.S + row) * D;
#pragma unroll
                for (int cc = 0; cc < D / 32; ++cc) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + kColO + cc * 32, o);
                    tmem_wait_ld();
                    if (row < p.S) {
#pragma unroll
                        for (int t = 0; t < 32; t += 4) {
                            float4 v4 = make_float4(__uint_as_float(o[t]) * inv_l, __uint_as_float(o[t + 1]) * inv_l,
                                                    __uint_as_float(o[t + 2]) * inv_l,
                                                    __uint_as_float(o[t + 3]) * inv_l);
                            *reinterpret_cast<float4 *>(orow + cc * 32 + t) = v4;
                        }
                    }
                }
            } else {
                // Stage the 16-bit O tile in the (now idle) Q buffer using the
                // same 128-byte swizzle as the tensor map, then TMA-store it.
#pragma unroll
                for (int cc = 0; cc < D / 32; ++cc) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + kColO + cc * 32, o);
                    tmem_wait_ld();
                    uint32_t pk[16];
#pragma unroll
                    for (int t = 0; t < 16; ++t)
                        pk[t] = ptx::pack2<BF16>(__uint_as_float(o[2 * t]) * inv_l, __uint_as_float(o[2 * t + 1]) * inv_l);
                    uint8_t *box = sQ + (cc >> 1) * kBoxBytes + row_local * 128;
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int chunk = (cc & 1) * 4 + q4;  // 16-byte chunk within the 128-byte row
                        uint4 v = make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
                        *reinterpret_cast<uint4 *>(box + ((chunk ^ (row_local & 7)) * 16)) = v;
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_ostage);
                // Bounded wait (not a named barrier): a warp that gave up earlier
                // never arrives, and the store thread then gives up too.
                if (threadIdx.x == 0 && mbar_wait(bar_ostage, 0, abort_flag)) {
#pragma unroll
                    for (int b = 0; b < C::kBoxes; ++b) tma_store_3d(&tm_o, sQ + b * kBoxBytes, b * kBoxCols, qt * kBM, bh);
                    tma_store_commit();
                    tma_store_wait_read0();
                }
            }
            if (row < p.S) {
                const size_t idx = static_cast<size_t>(bh) * p.S + row;
                const float m_nat = m_true * p.scale;
                const float l_true = (m_true == -INFINITY) ? 0.f : l * ex2_approx((m_used - m_true) * c2);
                store_as(p.m_out, idx, p.out_dtype, m_nat);
                store_as(p.l_out, idx, p.out_dtype, l_true);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && *abort_flag && !skip) report_device_error(PMKL_DEVERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// Self-test kernel: one CTA, exercises the same descriptors and tensor-memory
// layouts as the attention kernel on a single tile.
//   which 0: C[128 x 128] = A[128 x D] * B[128 x D]^T   (SS, both K-major)
//   which 1: C[128 x D]   = A[128 x 128] * B[128 x D]   (A via tensor memory, B MN-major)
template <int D, bool BF16>
__global__ void __launch_bounds__(128, 1)
    tc_selftest_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                       const uint16_t *__restrict__ a_raw, float *__restrict__ c, int which) {
    using namespace ptx;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t *sA = smem;                       // up to 2 boxes
    uint8_t *sB = smem + 2 * kBoxBytes;       // up to 2 boxes
    uint64_t *bar_ld = reinterpret_cast<uint64_t *>(smem + 4 * kBoxBytes);
    uint64_t *bar_mma = bar_ld + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_mma + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(bar_ld, 1);
        mbar_init(bar_mma, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int a_boxes = (which == 0) ? D / 64 : 2;
    const int b_boxes = D / 64;
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(bar_ld, (which == 0 ? a_boxes : 0) * kBoxBytes + b_boxes * kBoxBytes);
        if (which == 0)
            for (int b = 0; b < a_boxes; ++b) tma_load_3d(sA + b * kBoxBytes, &tm_a, bar_ld, b * 64, 0, 0);
        for (int b = 0; b < b_boxes; ++b) tma_load_3d(sB + b * kBoxBytes, &tm_b, bar_ld, b * 64, 0, 0);
    }
    if (which == 1) {
        // Thread r writes row r of A (128 x 128 16-bit) into tensor memory at kColP.
        const int r = threadIdx.x;
        const uint32_t base = tmem + (static_cast<uint32_t>(warp * 32) << 16) + kColP;
        for (int cc = 0; cc < 2; ++cc) {
            uint32_t w[32];
            for (int t = 0; t < 32; ++t)
                w[t] = static_cast<uint32_t>(a_raw[r * 128 + cc * 64 + 2 * t]) |
                       (static_cast<uint32_t>(a_raw[r * 128 + cc * 64 + 2 * t + 1]) << 16);
            tmem_st32(base + cc * 32, w);
        }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    bool ok = true;
    if (threadIdx.x == 0) {
        ok = mbar_wait(bar_ld, 0, abort_flag);
        if (ok) {
            tc_fence_after();
            if (which == 0) {
                constexpr uint32_t idesc = idesc_f16(128, 128, BF16 ? 1 : 0, 0, 0);
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
                    mma_ss(tmem + kColS0, smem_desc_sw128(smem_u32(sA) + off, 16, 1024),
                           smem_desc_sw128(smem_u32(sB) + off, 16, 1024), idesc, kk > 0);
                }
            } else {
                constexpr uint32_t idesc = idesc_f16(128, D, BF16 ? 1 : 0, 0, 1);
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts(tmem + kColO, tmem + kColP + kk * 8,
                           smem_desc_sw128(smem_u32(sB) + kk * 16 * 128, kBoxBytes, 1024), idesc, kk > 0);
            }
            mma_commit(bar_mma);
        }
    }
    ok = mbar_wait_warp(bar_mma, 0, abort_flag) && ok;
    if (ok) {
        tc_fence_after();
        const int r = threadIdx.x;
        const int ncols = (which == 0) ? 128 : D;
        const uint32_t base = tmem + (static_cast<uint32_t>(warp * 32) << 16) + (which == 0 ? kColS0 : kColO);
        for (int cc = 0; cc < ncols / 32; ++cc) {
            uint32_t o[32];
            tmem_ld32(base + cc * 32, o);
            tmem_wait_ld();
            for (int t = 0; t < 32; ++t) c[r * ncols + cc * 32 + t] = __uint_as_float(o[t]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && *abort_flag) report_device_error(PMKL_DEVERR_TIMEOUT);
}

}  // namespace tc
}  // namespace pmkl_b200
