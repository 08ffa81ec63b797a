// attention_kv64.cuh -- persistent two-query-tile tcgen05 flash attention
// forward for sm_100a with 64-key tiles and double-buffered scores:
// fp16/bf16 inputs, head size 64 or 128.
//
// Same results as pmkl::nlp::causal_attention_forward
// (pmkl/nlp/causal_attention.h:145-256): O (normalised), m = row max of the
// scaled masked scores, l = sum exp(s - m).
//
// Why 64-key tiles.  With 128-key tiles, two query tiles fill all 512
// tensor-memory columns (S and O of each), P has to live inside S's columns,
// and the next S of a query tile can only be computed after P.V has read P:
// every query tile then runs the chain softmax -> P.V -> next S -> softmax
// serially, and the softmax and the tensor pipe wait on each other.  With
// 64-key tiles each query tile holds two 64-column score buffers plus its O
// (2 x (64 + 64 + 128) = 512 columns at D = 128), so S(j+1) is computed while
// the softmax works on S(j), and S(j+2) is issued as soon as P.V(j) is:
// the softmax of a query tile runs from one key tile to the next without
// waiting for its own products.
//
//   * persistent grid (one CTA per SM); a work unit is a pair of adjacent
//     128-row query tiles A, B of one (batch*head) slice, taken round-robin
//     from the longest-first, L2-grouped order of the ping-pong kernel.
//   * warp roles (16 warps): WG0 / WG1 softmax of tile A / B (one thread per
//     query row = tensor-memory lane); WG2 epilogue; warp 12 TMA loads
//     (Q_A, Q_B per unit; 64-row K and V tiles through a ring in the order
//     K0, K1, V0, K2, V1, K3, ...); warp 13 issues tcgen05.mma.
//   * tensor memory: S_A0 [0,64) S_A1 [64,128) S_B0 [128,192) S_B1 [192,256)
//     O_A [256,256+D) O_B [384,384+D).  P (16-bit, 64 keys = 32 columns) goes
//     into the first 32 columns of its score buffer; for tiles whose rows see
//     at most 128 keys, the low part of a hi/lo split into the next 32.
//   * MMA issue per key tile j: PV_A(j), S_A(j+2), PV_B(j), S_B(j+2).  S_X(j+2)
//     reuses the buffer of S_X(j) and runs after PV_X(j) (one thread's
//     tcgen05.mma operations execute in order).  Each P.V is followed by a
//     commit to pv_done[X]; the softmax waits on it only when it has to
//     rescale O (its running maximum grew by more than 2^8), because P.V(j-1)
//     can still be running when the softmax of key tile j starts.
//   * every wait is bounded (sm100_ptx.cuh); on expiry the CTA drains its own
//     copies and MMAs, frees tensor memory and reports PMKL_DEVERR_TIMEOUT.
#pragma once

#include "attention_pp.cuh"

namespace pmkl_b200 {
namespace kv64 {

using pp::DeltaParams;
using pp::Params;
using tc::kBoxBytes;  // Q / O box: 128 rows x 128 bytes
using tc::kBoxCols;

constexpr int kBN = 64;                  // keys per key tile
constexpr int kKVBoxBytes = kBN * 128;   // K / V box: 64 rows x 128 bytes
constexpr int kThreads = 512;
constexpr int kWarpTma = 12;
constexpr int kWarpMma = 13;
constexpr uint32_t kTmemCols = 512;
__host__ __device__ constexpr uint32_t col_s(int x, int b) { return static_cast<uint32_t>(x * 128 + b * 64); }
__host__ __device__ constexpr uint32_t col_o(int x) { return x ? 384u : 256u; }
constexpr uint32_t kPHi = 0;   // P (hi) columns inside a score buffer
constexpr uint32_t kPLo = 32;  // P (lo) columns inside a score buffer

constexpr uint32_t kRegSoftmax = pp::kRegSoftmax;
constexpr uint32_t kRegEpilogue = pp::kRegEpilogue;
constexpr uint32_t kRegProducer = pp::kRegProducer;
constexpr int kLaunchRegs = pp::kLaunchRegs;

template <int D>
struct Cfg {
    static_assert(D == 64 || D == 128, "head size 64 or 128");
    static constexpr int kBoxes = D / kBoxCols;
    static constexpr int kQTile = kBoxes * kBoxBytes;     // 128 rows x D x 2 bytes
    static constexpr int kKVTile = kBoxes * kKVBoxBytes;  // 64 rows x D x 2 bytes
    static constexpr int kStages = (D == 64) ? 16 : 8;    // ring of K and V tiles
    static constexpr int kOffQ = 0;                        // Q_A, Q_B
    static constexpr int kOffStage = 2 * kQTile;           // epilogue staging, one 128 x 64 box
    static constexpr int kOffRing = kOffStage + kBoxBytes;
    static constexpr int kOffStats = kOffRing + kStages * kKVTile;  // [2][3][128] {m_used, m_true, l}
    static constexpr int kOffBars = kOffStats + 2 * 128 * 3 * 4;
    static constexpr int kNumBars = 2 + 2 + 2 * kStages + 4 + 4 + 2 + 2 + 2 + 2 + 2 + 3;
    static constexpr int kSmemBytes = kOffBars + kNumBars * 8 + 16 + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    static_assert(kKVTile % 1024 == 0 && kQTile % 1024 == 0, "tiles keep the 1024-byte swizzle alignment");
};

struct Unit {
    int bh;
    int row0;     // first row of tile A
    bool act[2];  // tile active (row0 of the tile < S)
    int n[2];     // 64-key tiles per query tile
    int n_max;
    bool hilo[2];  // every row of the tile sees at most 128 keys
};

// The ping-pong kernel's work order (pp::decode) with key tiles of 64.
__device__ __forceinline__ Unit unit_at(const Params &p, int u) {
    Unit w;
    const int n_kv_all = (p.S + kBN - 1) / kBN;
    const int per_group = p.n_pairs * p.group;
    const int g = u / per_group;
    const int within = u - g * per_group;
    const int g_slices = min(p.group, p.BH - g * p.group);
    const int rank = within / g_slices;
    const int pair = p.causal ? (p.n_pairs - 1 - rank) : rank;
    w.bh = g * p.group + (within - rank * g_slices);
    w.row0 = pair * 256;
    for (int x = 0; x < 2; ++x) {
        const int r0 = w.row0 + 128 * x;
        w.act[x] = r0 < p.S;
        w.n[x] = !w.act[x] ? 0 : (p.causal ? min((r0 + 128) / kBN, n_kv_all) : n_kv_all);
        w.hilo[x] = w.act[x] && (p.causal ? (r0 == 0) : (p.S <= 128));
    }
    w.n_max = max(w.n[0], w.n[1]);
    return w;
}

// p = 2^(s * c2 - mref) for the 32-key chunks [C0, C1) of a 64-score row,
// packed to 16-bit pairs into the P (hi) columns of the row's score buffer
// (HILO: the rounding remainder into the P (lo) columns).  TRACK gathers the
// row maximum of these scores in four running maxima alongside.  Returns the
// partial row sum as a pair.
template <bool BF16, bool HILO, int C0, int C1, bool TRACK>
__device__ __forceinline__ float2 exp_chunks(const float (&s)[64], float2 c22, float2 nm2, uint32_t sa,
                                             float (&mx)[4]) {
    using namespace ptx;
    float2 rs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int c0 = C0; c0 < C1; c0 += 32) {
        uint32_t ph[16];
        uint32_t pl[HILO ? 16 : 1];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float s0 = s[c0 + 2 * i], s1 = s[c0 + 2 * i + 1];
            if constexpr (TRACK) mx[i & 3] = fmax3(mx[i & 3], s0, s1);
            const float2 a = fma2(make_float2(s0, s1), c22, nm2);
            const float2 e = make_float2(ex2_approx(a.x), ex2_approx(a.y));
            rs2[i & 1] = add2(rs2[i & 1], e);
            ph[i] = pack2<BF16>(e.x, e.y);
            if constexpr (HILO) {
                float h0, h1;
                tc::unpack2<BF16>(ph[i], h0, h1);
                pl[i] = pack2<BF16>(e.x - h0, e.y - h1);
            }
        }
        tmem_st16(sa + kPHi + c0 / 2, ph);
        if constexpr (HILO) tmem_st16(sa + kPLo + c0 / 2, pl);
    }
    return add2(rs2[0], rs2[1]);
}

// DELTA: the backward's instantiation, writing the row statistics (b, delta)
// instead of O, m, l (pp::DeltaParams).
template <int D, bool BF16, bool DELTA = false>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kv64_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                         const Params p, const DeltaParams dpar) {
    using namespace ptx;
    using C = Cfg<D>;
    constexpr int NS = C::kStages;
    constexpr int QTILE = C::kQTile;
    constexpr int KVTILE = C::kKVTile;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t *sQ = smem + C::kOffQ;  // [2][QTILE]
    uint8_t *sStage = smem + C::kOffStage;
    uint8_t *sRing = smem + C::kOffRing;  // [NS][KVTILE]
    float *sStats = reinterpret_cast<float *>(smem + C::kOffStats);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kOffBars);
    uint64_t *q_full = bars;              // [2]
    uint64_t *q_empty = bars + 2;         // [2]
    uint64_t *kv_full = bars + 4;         // [NS]
    uint64_t *kv_empty = kv_full + NS;    // [NS]
    uint64_t *s_full = kv_empty + NS;     // [2 tiles][2 buffers]
    uint64_t *p_full = s_full + 4;        // [2 tiles][2 buffers]
    uint64_t *pv_done = p_full + 4;       // [2]
    uint64_t *o_full = pv_done + 2;       // [2]
    uint64_t *o_empty = o_full + 2;       // [2]
    uint64_t *st_full = o_empty + 2;      // [2]
    uint64_t *st_empty = st_full + 2;     // [2]
    uint64_t *mma_done = st_empty + 2;
    uint64_t *stg_written = mma_done + 1;  // epilogue warps -> store thread
    uint64_t *stg_free = stg_written + 1;  // store thread -> epilogue warps
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(stg_free + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int wg = warp >> 2;

    if (threadIdx.x == 0) {
        for (int x = 0; x < 2; ++x) {
            mbar_init(&q_full[x], 1);
            mbar_init(&q_empty[x], 1);
            mbar_init(&pv_done[x], 1);
            mbar_init(&o_full[x], 1);
            mbar_init(&o_empty[x], 4);
            mbar_init(&st_full[x], 4);
            mbar_init(&st_empty[x], 4);
        }
        for (int i = 0; i < 4; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
        }
        for (int s = 0; s < NS; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(mma_done, 1);
        mbar_init(stg_written, 4);
        mbar_init(stg_free, 1);
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

    if (wg == 3) {
        reg_dealloc<kRegProducer>();
        if (!skip && warp == kWarpTma && lane == 0) {
            // ------------------------------------------------------------ TMA producer
            tma_prefetch_desc(&tm_q);
            tma_prefetch_desc(&tm_k);
            tma_prefetch_desc(&tm_v);
            uint32_t qc0 = 0, qc1 = 0;
            int kvc = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                const int bb = w.bh / p.H;
                const int hh = w.bh - bb * p.H;
                const int hkv = hh / p.kv_group;
                auto load_q = [&](const int x, uint32_t &qcx) {
                    if (!ok) return;
                    if (qcx > 0 && !(ok = mbar_wait(&q_empty[x], (qcx - 1) & 1, abort_flag))) return;
                    mbar_arrive_expect_tx(&q_full[x], QTILE);
#pragma unroll
                    for (int b = 0; b < C::kBoxes; ++b)
                        tma_load_4d(sQ + x * QTILE + b * kBoxBytes, &tm_q, &q_full[x], b * kBoxCols, w.row0 + 128 * x,
                                    hh, bb);
                    ++qcx;
                };
                // One 64-row K or V tile into the next ring stage.
                auto load_kv = [&](const bool is_v, const int jt) {
                    if (!ok) return;
                    const int s = kvc % NS;
                    if (kvc >= NS && !(ok = mbar_wait(&kv_empty[s], ((kvc / NS) - 1) & 1, abort_flag))) return;
                    mbar_arrive_expect_tx(&kv_full[s], KVTILE);
                    const CUtensorMap *map = is_v ? &tm_v : &tm_k;
#pragma unroll
                    for (int b = 0; b < C::kBoxes; ++b)
                        tma_load_4d(sRing + s * KVTILE + b * kKVBoxBytes, map, &kv_full[s], b * kBoxCols, jt * kBN,
                                    hkv, bb);
                    ++kvc;
                };
                if (w.act[0]) load_q(0, qc0);
                if (w.act[1]) load_q(1, qc1);
                // The MMA issuer's order: K0, K1, then V(j) and K(j+2) per key tile.
                load_kv(false, 0);
                if (w.n_max > 1) load_kv(false, 1);
                for (int j = 0; ok && j < w.n_max; ++j) {
                    load_kv(true, j);
                    if (j + 2 < w.n_max) load_kv(false, j + 2);
                }
            }
            if (*abort_flag) {
                // Let issued copies land before shared memory is released.
                volatile int never = 0;
                for (int i = max(0, kvc - NS); i < kvc; ++i) mbar_wait(&kv_full[i % NS], (i / NS) & 1, &never);
                if (qc0 > 0) mbar_wait(&q_full[0], (qc0 - 1) & 1, &never);
                if (qc1 > 0) mbar_wait(&q_full[1], (qc1 - 1) & 1, &never);
            }
        } else if (!skip && warp == kWarpMma && lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            constexpr uint32_t kIdescS = idesc_f16(128, kBN, BF16 ? 1 : 0, 0, 0);
            constexpr uint32_t kIdescO = idesc_f16(128, D, BF16 ? 1 : 0, 0, 1);
            uint32_t qc0 = 0, qc1 = 0, oc0 = 0, oc1 = 0;
            int g0 = 0, g1 = 0;  // key tiles issued so far per query tile (buffer = step & 1)
            int kvc = 0;
            bool ok = true;
            // Descriptors are built once; each operand slice is the base
            // descriptor's low word plus a constant added to its start-address
            // field (addresses stay below 256 KB, so it never carries).
            const uint64_t dq0 = smem_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t dk0 = smem_desc_sw128(smem_u32(sRing), 16, 1024);           // K view of stage 0
            const uint64_t dv0 = smem_desc_sw128(smem_u32(sRing), kKVBoxBytes, 1024);  // V view of stage 0
            const uint32_t q_lo = static_cast<uint32_t>(dq0), qk_hi = static_cast<uint32_t>(dq0 >> 32);
            const uint32_t k_lo = static_cast<uint32_t>(dk0);
            const uint32_t v_lo = static_cast<uint32_t>(dv0), v_hi = static_cast<uint32_t>(dv0 >> 32);
            auto issue_s = [&](int x, int buf, int stage) {
                const uint32_t a0 = q_lo + static_cast<uint32_t>(x * (QTILE >> 4));
                const uint32_t b0 = k_lo + static_cast<uint32_t>(stage * (KVTILE >> 4));
                const uint32_t d = tmem + col_s(x, buf);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t oa = static_cast<uint32_t>(((kk >> 2) * kBoxBytes + (kk & 3) * 32) >> 4);
                    const uint32_t ob = static_cast<uint32_t>(((kk >> 2) * kKVBoxBytes + (kk & 3) * 32) >> 4);
                    mma_ss_h(d, a0 + oa, qk_hi, b0 + ob, qk_hi, kIdescS, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[x * 2 + buf]);
            };
            auto issue_pv = [&](int x, int buf, int stage, bool first, bool hilo) {
                const uint32_t b0 = v_lo + static_cast<uint32_t>(stage * (KVTILE >> 4));
                const uint32_t d = tmem + col_o(x);
                const uint32_t a = tmem + col_s(x, buf);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk)
                    mma_ts_h(d, a + kPHi + kk * 8, b0 + static_cast<uint32_t>(kk * 128), v_hi, kIdescO,
                             (!first || kk > 0) ? 1u : 0u);
                if (hilo) {
#pragma unroll
                    for (int kk = 0; kk < kBN / 16; ++kk)
                        mma_ts_h(d, a + kPLo + kk * 8, b0 + static_cast<uint32_t>(kk * 128), v_hi, kIdescO, 1u);
                }
                mma_commit(&pv_done[x]);
            };
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                const int n0 = w.n[0], n1 = w.n[1];
                const bool hl0 = w.hilo[0], hl1 = w.hilo[1];
                if (w.act[0]) {
                    ok = mbar_wait(&q_full[0], qc0 & 1, abort_flag);
                    ++qc0;
                }
                if (ok && w.act[1]) {
                    ok = mbar_wait(&q_full[1], qc1 & 1, abort_flag);
                    ++qc1;
                }
                if (!ok) break;
                // K0 -> S_A(0), S_B(0); K1 -> S_A(1), S_B(1).
                for (int jt = 0; jt < 2 && jt < w.n_max; ++jt) {
                    const int sK = kvc % NS;
                    if (!(ok = mbar_wait(&kv_full[sK], (kvc / NS) & 1, abort_flag))) break;
                    ++kvc;
                    tc_fence_after();
                    if (jt < n0) {
                        issue_s(0, (g0 + jt) & 1, sK);
                        if (jt + 1 == n0) mma_commit(&q_empty[0]);
                    }
                    if (jt < n1) {
                        issue_s(1, (g1 + jt) & 1, sK);
                        if (jt + 1 == n1) mma_commit(&q_empty[1]);
                    }
                    mma_commit(&kv_empty[sK]);
                }
                if (!ok) break;
                for (int j = 0; ok && j < w.n_max; ++j) {
                    const int sV = kvc % NS;
                    if (!(ok = mbar_wait(&kv_full[sV], (kvc / NS) & 1, abort_flag))) break;
                    ++kvc;
                    const bool has_k = j + 2 < w.n_max;
                    const int kvc_k = kvc;
                    const int sK = kvc % NS;
                    if (has_k) ++kvc;
                    bool k_ready = false;
                    auto tile = [&](const int x, const int nx, const int gx, const bool hlx, uint32_t &ocx) {
                        if (!ok || j >= nx) return;
                        const int G = gx + j;
                        const int buf = G & 1;
                        if (!(ok = pp::wait_p_ready(&p_full[x * 2 + buf], (G >> 1) & 1, abort_flag))) return;
                        if (j == 0 && ocx > 0 && !(ok = mbar_wait(&o_empty[x], (ocx - 1) & 1, abort_flag))) return;
                        tc_fence_after();
                        issue_pv(x, buf, sV, j == 0, hlx);
                        if (j + 2 < nx) {
                            if (!k_ready) {
                                if (!(ok = mbar_wait(&kv_full[sK], (kvc_k / NS) & 1, abort_flag))) return;
                                k_ready = true;
                                tc_fence_after();
                            }
                            issue_s(x, buf, sK);
                            if (j + 3 == nx) mma_commit(&q_empty[x]);
                        }
                        if (j + 1 == nx) {
                            mma_commit(&o_full[x]);
                            ++ocx;
                        }
                    };
                    tile(0, n0, g0, hl0, oc0);
                    tile(1, n1, g1, hl1, oc1);
                    if (!ok) break;
                    mma_commit(&kv_empty[sV]);
                    if (has_k) mma_commit(&kv_empty[sK]);
                }
                g0 += n0;
                g1 += n1;
            }
            // Drain every MMA issued before tensor memory is released.
            mma_commit(mma_done);
            volatile int never = 0;
            mbar_wait(mma_done, 0, &never);
        }
    } else if (wg < 2) {
        reg_alloc<kRegSoftmax>();
        if (!skip) {
            // ------------------------------------------------------------ softmax of tile x = wg
            const int x = wg;
            const int r_local = (warp & 3) * 32 + lane;  // == tensor-memory lane
            const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
            const float c2 = p.scale_log2;
            const float2 c22 = make_float2(c2, c2);
            int gx = 0, uc = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                const bool actx = x ? w.act[1] : w.act[0];
                const int nx = x ? w.n[1] : w.n[0];
                const bool hilox = x ? w.hilo[1] : w.hilo[0];
                if (!actx) continue;
                const int row = w.row0 + 128 * x + r_local;
                float m_used = -INFINITY, m_true = -INFINITY, l = 0.f;
                for (int j = 0; j < nx; ++j) {
                    const int G = gx + j;
                    const int buf = G & 1;
                    const uint32_t sa = lane_base + col_s(x, buf);
                    const int kbase = j * kBN;
                    int lim = p.S - kbase;
                    if (p.causal) lim = min(lim, row - kbase + 1);
                    const bool masked = __any_sync(0xffffffffu, lim < kBN);
                    float s[64];
                    uint32_t *sr = reinterpret_cast<uint32_t *>(s);
                    auto mask_half = [&](const int h) {
                        if (masked) {
#pragma unroll
                            for (int c = 32 * h; c < 32 * h + 32; ++c)
                                if (c >= lim) s[c] = -INFINITY;
                        }
                    };
                    if (!(ok = pp::wait_s_ready(&s_full[x * 2 + buf], (G >> 1) & 1, abort_flag))) break;
                    tc_fence_after();
                    float m_new, fac, rsum;
                    bool any_fac;
                    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                    if (j == 0 || hilox) {
                        // Exact form: the tile maximum comes first.  Used for a
                        // row's first key tile and for the (rare) hi/lo tiles.
                        tmem_ld32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
                        tmem_ld32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
                        tmem_wait_ld();
                        mask_half(0);
                        mask_half(1);
#pragma unroll
                        for (int c = 0; c < 64; c += 8)
#pragma unroll
                            for (int t = 0; t < 4; ++t) mx[t] = fmax3(mx[t], s[c + t], s[c + 4 + t]);
                        m_true = fmaxf(m_true, fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]));
                        m_new = m_true;
                        const float mref = (m_new == -INFINITY) ? 0.f : m_new * c2;
                        const float2 nm2 = make_float2(-mref, -mref);
                        float2 r;
                        if (hilox)
                            r = exp_chunks<BF16, true, 0, 64, false>(s, c22, nm2, sa, mx);
                        else
                            r = exp_chunks<BF16, false, 0, 64, false>(s, c22, nm2, sa, mx);
                        rsum = r.x + r.y;
                        if (j == 0) {
                            fac = 0.f;  // l and O hold nothing yet
                            any_fac = false;
                        } else {
                            fac = (m_new == m_used) ? 1.f : ex2_approx((m_used - m_new) * c2);
                            any_fac = __any_sync(0xffffffffu, m_new != m_used);
                        }
                    } else {
                        // Later key tiles: exps against a reference taken from
                        // earlier tiles while this tile's maximum is gathered
                        // alongside.  A reference more than 2^8 below the running
                        // maximum is moved up first; a tile whose own maximum is
                        // more than 2^kSpec above the reference is redone.
                        m_new = ((m_true - m_used) * c2 > 8.0f) ? m_true : m_used;
                        float2 nm2 = make_float2(-m_new * c2, -m_new * c2);
                        tmem_ld32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
                        tmem_wait_ld();
                        tmem_ld32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
                        mask_half(0);
                        float2 r = exp_chunks<BF16, false, 0, 32, true>(s, c22, nm2, sa, mx);
                        tmem_wait_ld();
                        mask_half(1);
                        r = add2(r, exp_chunks<BF16, false, 32, 64, true>(s, c22, nm2, sa, mx));
                        m_true = fmaxf(m_true, fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]));
                        constexpr float kSpec = BF16 ? 30.0f : 15.0f;
                        const bool redo = (m_true - m_new) * c2 > kSpec;
                        if (__any_sync(0xffffffffu, redo)) {
                            // Rare: all 64 scores are still in registers.
                            if (redo) m_new = m_true;
                            nm2 = make_float2(-m_new * c2, -m_new * c2);
                            tmem_wait_st();
                            r = exp_chunks<BF16, false, 0, 64, false>(s, c22, nm2, sa, mx);
                        }
                        rsum = r.x + r.y;
                        fac = (m_new == m_used) ? 1.f : ex2_approx((m_used - m_new) * c2);
                        any_fac = __any_sync(0xffffffffu, m_new != m_used);
                    }
                    if (any_fac) {
                        // P.V(j-1) may still be adding into O_X: wait for it.
                        if (!(ok = mbar_wait_warp(&pv_done[x], (G - 1) & 1, abort_flag))) break;
                        tc_fence_after();
#pragma unroll
                        for (int cc = 0; cc < D / 32; ++cc) {
                            uint32_t o[32];
                            tmem_ld32(lane_base + col_o(x) + cc * 32, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * fac);
                            tmem_st32(lane_base + col_o(x) + cc * 32, o);
                        }
                    }
                    l = l * fac + rsum;
                    m_used = m_new;
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&p_full[x * 2 + buf]);
                }
                if (!ok) break;
                gx += nx;
                // Row statistics for the epilogue.
                if (uc > 0 && !(ok = mbar_wait_warp(&st_empty[x], (uc - 1) & 1, abort_flag))) break;
                sStats[(x * 3 + 0) * 128 + r_local] = m_used;
                sStats[(x * 3 + 1) * 128 + r_local] = m_true;
                sStats[(x * 3 + 2) * 128 + r_local] = l;
                __syncwarp();
                if (lane == 0) mbar_arrive(&st_full[x]);
                ++uc;
            }
        }
    } else {
        reg_dealloc<kRegEpilogue>();
        if (!skip) {
            // ------------------------------------------------------------ epilogue (WG2)
            const int r_local = (warp & 3) * 32 + lane;
            const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
            const bool lead = (warp == 8 && lane == 0);
            const float c2 = p.scale_log2;
            uint32_t oc0 = 0, oc1 = 0;
            int nb = 0;  // staging boxes used so far
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                for (int x = 0; x < 2 && ok; ++x) {
                    if (!(x ? w.act[1] : w.act[0])) continue;
                    const uint32_t ocx = x ? oc1 : oc0;
                    if (!(ok = mbar_wait_warp(&o_full[x], ocx & 1, abort_flag))) break;
                    if (!(ok = mbar_wait_warp(&st_full[x], ocx & 1, abort_flag))) break;
                    if (x) ++oc1; else ++oc0;
                    tc_fence_after();
                    const float m_used = sStats[(x * 3 + 0) * 128 + r_local];
                    const float m_true = sStats[(x * 3 + 1) * 128 + r_local];
                    const float l = sStats[(x * 3 + 2) * 128 + r_local];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&st_empty[x]);
                    const float inv_l = 1.f / l;
                    const int row = w.row0 + 128 * x + r_local;
                    const uint32_t oa = lane_base + col_o(x);
                    const int bb = w.bh / p.H;
                    const int hh = w.bh - bb * p.H;
                    if constexpr (DELTA) {
                        using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
                        const size_t ridx = static_cast<size_t>(w.bh) * p.S + row;
                        const uint4 *drow = reinterpret_cast<const uint4 *>(static_cast<const T *>(dpar.dout) + ridx * D);
                        float dot = 0.f;
#pragma unroll
                        for (int cc = 0; cc < D / 32; ++cc) {
                            uint32_t o[32];
                            tmem_ld32(oa + cc * 32, o);
                            tmem_wait_ld();
                            if (cc == D / 32 - 1) {
                                tc_fence_before();
                                __syncwarp();
                                if (lane == 0) mbar_arrive(&o_empty[x]);
                            }
                            if (row < p.S) {
#pragma unroll
                                for (int q4 = 0; q4 < 4; ++q4) {
                                    const uint4 dv = __ldg(drow + cc * 4 + q4);
                                    const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
                                    for (int e = 0; e < 4; ++e) {
                                        float d0, d1;
                                        tc::unpack2<BF16>(dw[e], d0, d1);
                                        dot = fmaf(__uint_as_float(o[q4 * 8 + 2 * e]), d0, dot);
                                        dot = fmaf(__uint_as_float(o[q4 * 8 + 2 * e + 1]), d1, dot);
                                    }
                                }
                            }
                        }
                        float2 rs = make_float2(0.f, 0.f);
                        if (row < p.S) {
                            const float mg = Elem<T>::to_float(static_cast<const T *>(dpar.m_given)[ridx]);
                            const float lg = Elem<T>::to_float(static_cast<const T *>(dpar.l_given)[ridx]);
                            const float l_true = (m_true == -INFINITY) ? 0.f : l * ex2_approx((m_used - m_true) * c2);
                            const float f = expf(m_true * p.scale - mg) * (l_true / lg);
                            rs = make_float2(mg * 1.4426950408889634f + log2f(lg), f * dot * inv_l);
                        }
                        dpar.rowstat[static_cast<size_t>(w.bh) * dpar.S_pad + row] = rs;
                        continue;
                    }
                    if (p.out_dtype == PMKL_DTYPE_F32) {
                        float *orow = static_cast<float *>(p.o_f32) + bb * p.o_sb + hh * p.o_sh + row * p.o_ss;
#pragma unroll
                        for (int cc = 0; cc < D / 32; ++cc) {
                            uint32_t o[32];
                            tmem_ld32(oa + cc * 32, o);
                            tmem_wait_ld();
                            if (cc == D / 32 - 1) {
                                tc_fence_before();
                                __syncwarp();
                                if (lane == 0) mbar_arrive(&o_empty[x]);
                            }
                            if (row < p.S) {
#pragma unroll
                                for (int t = 0; t < 32; t += 4)
                                    *reinterpret_cast<float4 *>(orow + cc * 32 + t) =
                                        make_float4(__uint_as_float(o[t]) * inv_l, __uint_as_float(o[t + 1]) * inv_l,
                                                    __uint_as_float(o[t + 2]) * inv_l,
                                                    __uint_as_float(o[t + 3]) * inv_l);
                            }
                        }
                    } else {
#pragma unroll
                        for (int b = 0; b < C::kBoxes; ++b) {
                            // The staging box is free once the previous TMA store has read it.
                            if (nb > 0 && !(ok = mbar_wait_warp(stg_free, (nb - 1) & 1, abort_flag))) break;
                            uint8_t *box = sStage + r_local * 128;
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                uint32_t o[32];
                                tmem_ld32(oa + b * 64 + h * 32, o);
                                tmem_wait_ld();
                                if (b == C::kBoxes - 1 && h == 1) {
                                    tc_fence_before();
                                    __syncwarp();
                                    if (lane == 0) mbar_arrive(&o_empty[x]);
                                }
                                uint32_t pk[16];
#pragma unroll
                                for (int t = 0; t < 16; ++t)
                                    pk[t] = pack2<BF16>(__uint_as_float(o[2 * t]) * inv_l,
                                                        __uint_as_float(o[2 * t + 1]) * inv_l);
#pragma unroll
                                for (int q4 = 0; q4 < 4; ++q4) {
                                    const int chunk = h * 4 + q4;
                                    *reinterpret_cast<uint4 *>(box + ((chunk ^ (r_local & 7)) * 16)) =
                                        make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
                                }
                            }
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(stg_written);
                            if (lead) {
                                // Once all four warps have written their rows of this box,
                                // store it and hand the buffer back when the store has read it.
                                if ((ok = mbar_wait(stg_written, nb & 1, abort_flag))) {
                                    tma_store_4d(&tm_o, sStage, b * kBoxCols, w.row0 + 128 * x, hh, bb);
                                    tma_store_commit();
                                    tma_store_wait_read0();
                                }
                                mbar_arrive(stg_free);
                            }
                            ++nb;
                            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                            if (!ok) break;
                        }
                        if (!ok) break;
                    }
                    if (row < p.S) {
                        const size_t idx = static_cast<size_t>(w.bh) * p.S + row;
                        store_as(p.m_out, idx, p.out_dtype, m_true * p.scale);
                        store_as(p.l_out, idx, p.out_dtype,
                                 (m_true == -INFINITY) ? 0.f : l * ex2_approx((m_used - m_true) * c2));
                    }
                }
            }
            if (lead) tma_store_wait0();
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

}  // namespace kv64
}  // namespace pmkl_b200
