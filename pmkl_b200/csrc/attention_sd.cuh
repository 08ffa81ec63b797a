// attention_sd.cuh -- persistent tcgen05 flash attention forward for sm_100a
// with one query tile per work unit and double-buffered scores and P:
// fp16/bf16 inputs, head size 64 or 128.
//
// Same results as pmkl::nlp::causal_attention_forward
// (pmkl/nlp/causal_attention.h:145-256): O (normalised), m = row max of the
// scaled masked scores, l = sum exp(s - m).
//
// Why one tile.  Two query tiles per CTA (attention_pp.cuh) fill the 512
// tensor-memory columns with their S and O, so P must live inside S and each
// tile's next S waits for its P.V: softmax -> P.V -> next S -> softmax is a
// serial chain, and the two tiles' softmax phases end up sharing the MUFU unit.
// One tile leaves room for two S buffers and two P buffers:
//   S0 [0,128)  S1 [128,256)  O [256,256+D)  P0 [384,448)  P1 [448,512)
// so S(j+1) is ready before the softmax finishes S(j), and the softmax runs
// from one key tile to the next without waiting for its own products; the
// tensor pipe does P.V(j) and S(j+2) meanwhile.
//
//   * persistent grid (one CTA per SM); a work unit is one 128-row query tile
//     of one (batch*head) slice, taken round-robin from a list ordered
//     longest-first inside groups of slices whose K and V fit in L2.
//   * warp roles (16 warps): WG0 and WG1 run the softmax of the even and the
//     odd key tiles of the unit (one thread per query row = tensor-memory
//     lane; thread i of both warpgroups owns row i); WG2 epilogue; warp 12
//     TMA loads (Q double buffered per unit; K and V through a ring in the
//     order K0, K1, V0, K2, V1, K3, ...); warp 13 issues tcgen05.mma.
//   * exp reference.  Both warpgroups add into one O, so every key tile j has
//     a reference r_j that both can compute without waiting for each other:
//     r_j = f(r_(j-1), M_(j-2)), where M_k is the row maximum over key tiles
//     <= k and f moves the reference up to M only when M lies more than 2^8
//     above it.  After its exps each warpgroup publishes its tile maximum and
//     final reference r'_j (r_j, or the tile's own maximum when the tile
//     lies so far above r_j that P could overflow and is redone) in shared
//     memory slots indexed by the global key-tile number modulo 4; the other
//     warpgroup reads them one key tile later (for M and for the O rescale
//     from r'_(j-1) to r'_j, rare).  A writer cannot lap its reader: writing
//     tile j + 4 needs P.V(j + 2), which the issuer starts only after P(j + 1),
//     which the reader releases after reading tile j.  Each warpgroup keeps its
//     row sum at its own last reference; the epilogue combines the two.
//   * MMA issue per key tile j: P.V(j) (P from buffer j & 1), then S(j+2)
//     into the S buffer of S(j), which the softmax has finished reading.
//     Each P.V commits to pv_done[j & 1]; the softmax waits on it before
//     reusing that P buffer (two key tiles later) and before the rare O
//     rescale.
//   * tiles whose rows see at most 128 keys also multiply the low part of a
//     hi/lo split of P, kept in the other (unused) S buffer.
//   * every wait is bounded (sm100_ptx.cuh); on expiry the CTA drains its own
//     copies and MMAs, frees tensor memory and reports PMKL_DEVERR_TIMEOUT.
#pragma once

#include "attention_pp.cuh"

namespace pmkl_b200 {
namespace sd {

using pp::DeltaParams;
using tc::kBoxBytes;
using tc::kBoxCols;

constexpr int kThreads = 512;
constexpr int kWarpTma = 12;
constexpr int kWarpMma = 13;
constexpr uint32_t kTmemCols = 512;
__host__ __device__ constexpr uint32_t col_s(int b) { return b ? 128u : 0u; }
__host__ __device__ constexpr uint32_t col_p(int b) { return b ? 448u : 384u; }
constexpr uint32_t kColO = 256;

// Register budget per warpgroup after the split (launch: 512 x 128 = 65536).
constexpr uint32_t kRegSoftmax = 184;
constexpr uint32_t kRegEpilogue = 64;
constexpr uint32_t kRegProducer = 80;
static_assert(128 * (2 * kRegSoftmax + kRegEpilogue + kRegProducer) <= 65536, "register split exceeds the pool");
constexpr int kLaunchRegs = 128;

template <int D>
struct Cfg {
    static_assert(D == 64 || D == 128, "head size 64 or 128");
    static constexpr int kBoxes = D / kBoxCols;
    static constexpr int kTile = kBoxes * kBoxBytes;     // 128 rows x D x 2 bytes
    static constexpr int kStages = (D == 64) ? 8 : 4;    // K/V ring
    static constexpr int kOffQ = 0;                       // two Q slots
    static constexpr int kOffStage = 2 * kTile;           // epilogue staging, one 128 x 64 box
    static constexpr int kOffRing = kOffStage + kBoxBytes;
    static constexpr int kOffStats = kOffRing + kStages * kTile;  // [2 warpgroups][3][128] {ref, max, l}
    static constexpr int kOffPub = kOffStats + 2 * 3 * 128 * 4;     // [4 slots][2][128] {tile max, ref}
    static constexpr int kOffBars = kOffPub + 4 * 2 * 128 * 4;
    static constexpr int kNumBars = 2 + 2 + 2 * kStages + 2 + 2 + 2 + 1 + 1 + 1 + 1 + 3 + 4;
    static constexpr int kSmemBytes = kOffBars + kNumBars * 8 + 16 + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// Same fields as pp::Params; n_units = n_qt * BH here.
struct Params {
    int S;
    int BH;
    int H;
    int kv_group;
    long long o_sb, o_sh, o_ss;
    int n_qt;
    int n_units;
    int group;
    int causal;
    int out_dtype;
    float scale;
    float scale_log2;
    void *o_f32;
    void *m_out;
    void *l_out;
};

struct Unit {
    int bh;
    int row0;
    int n;      // key tiles
    bool hilo;  // every row sees at most 128 keys
};

// Slices are taken in groups of p.group (b, h) slices whose K and V fit in
// L2; inside a group the query tiles go longest first, so all tiles of a
// slice run close together in time and re-read its K/V from L2.
__device__ __forceinline__ Unit unit_at(const Params &p, int u) {
    Unit w;
    const int n_kv_all = (p.S + 127) / 128;
    const int per_group = p.n_qt * p.group;
    const int g = u / per_group;
    const int within = u - g * per_group;
    const int g_slices = min(p.group, p.BH - g * p.group);
    const int rank = within / g_slices;
    const int qt = p.causal ? (p.n_qt - 1 - rank) : rank;
    w.bh = g * p.group + (within - rank * g_slices);
    w.row0 = qt * 128;
    w.n = p.causal ? min(qt + 1, n_kv_all) : n_kv_all;
    w.hilo = (w.n == 1) && (p.causal ? (qt == 0) : true);
    return w;
}

// p = 2^(s * c2 - mref) for the 32-key chunks [C0, C1) of a 128-score row,
// packed to 16-bit pairs into P buffer `pa` (HILO: the rounding remainder into
// `pl`).  TRACK gathers the row maximum of these scores in four running maxima
// alongside.  Returns the partial row sum as a pair.
template <bool BF16, bool HILO, int C0, int C1, bool TRACK>
__device__ __forceinline__ float2 exp_chunks(const float (&s)[128], float2 c22, float2 nm2, uint32_t pa, uint32_t pl,
                                             float (&mx)[4]) {
    using namespace ptx;
    float2 rs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int c0 = C0; c0 < C1; c0 += 32) {
        uint32_t ph[16];
        uint32_t plo[HILO ? 16 : 1];
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
                plo[i] = pack2<BF16>(e.x - h0, e.y - h1);
            }
        }
        tmem_st16(pa + c0 / 2, ph);
        if constexpr (HILO) tmem_st16(pl + c0 / 2, plo);
    }
    return add2(rs2[0], rs2[1]);
}

// DELTA: the backward's instantiation, writing the row statistics (b, delta)
// instead of O, m, l (pp::DeltaParams).
template <int D, bool BF16, bool DELTA = false>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                       const Params p, const DeltaParams dpar) {
    using namespace ptx;
    using C = Cfg<D>;
    constexpr int NS = C::kStages;
    constexpr int TILE = C::kTile;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t *sQ = smem + C::kOffQ;  // [2][TILE]
    uint8_t *sStage = smem + C::kOffStage;
    uint8_t *sRing = smem + C::kOffRing;  // [NS][TILE]
    float *sStats = reinterpret_cast<float *>(smem + C::kOffStats);  // [2][3][128]
    float *sPub = reinterpret_cast<float *>(smem + C::kOffPub);      // [4][2][128]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kOffBars);
    uint64_t *q_full = bars;            // [2]
    uint64_t *q_empty = bars + 2;       // [2]
    uint64_t *kv_full = bars + 4;       // [NS]
    uint64_t *kv_empty = kv_full + NS;  // [NS]
    uint64_t *s_full = kv_empty + NS;   // [2] per S buffer
    uint64_t *p_full = s_full + 2;      // [2] per P buffer
    uint64_t *pv_done = p_full + 2;     // [2] per P buffer
    uint64_t *o_full = pv_done + 2;
    uint64_t *o_empty = o_full + 1;
    uint64_t *st_full = o_empty + 1;
    uint64_t *st_empty = st_full + 1;
    uint64_t *mma_done = st_empty + 1;
    uint64_t *stg_written = mma_done + 1;  // epilogue warps -> store thread
    uint64_t *stg_free = stg_written + 1;  // store thread -> epilogue warps
    uint64_t *pub_full = stg_free + 1;     // [4] publication slots, one writer warpgroup each time
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pub_full + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int wg = warp >> 2;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(&q_full[b], 1);
            mbar_init(&q_empty[b], 1);
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 4);
            mbar_init(&pv_done[b], 1);
        }
        for (int s = 0; s < NS; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(o_full, 1);
        mbar_init(o_empty, 4);
        mbar_init(st_full, 8);
        for (int i = 0; i < 4; ++i) mbar_init(&pub_full[i], 4);
        mbar_init(st_empty, 4);
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
            int uq = 0, kvc = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                const int bb = w.bh / p.H;
                const int hh = w.bh - bb * p.H;
                const int hkv = hh / p.kv_group;
                const int qb = uq & 1;
                if (uq >= 2 && !(ok = mbar_wait(&q_empty[qb], ((uq >> 1) - 1) & 1, abort_flag))) break;
                mbar_arrive_expect_tx(&q_full[qb], TILE);
#pragma unroll
                for (int b = 0; b < C::kBoxes; ++b)
                    tma_load_4d(sQ + qb * TILE + b * kBoxBytes, &tm_q, &q_full[qb], b * kBoxCols, w.row0, hh, bb);
                ++uq;
                auto load_kv = [&](const bool is_v, const int jt) {
                    if (!ok) return;
                    const int s = kvc % NS;
                    if (kvc >= NS && !(ok = mbar_wait(&kv_empty[s], ((kvc / NS) - 1) & 1, abort_flag))) return;
                    mbar_arrive_expect_tx(&kv_full[s], TILE);
                    const CUtensorMap *map = is_v ? &tm_v : &tm_k;
#pragma unroll
                    for (int b = 0; b < C::kBoxes; ++b)
                        tma_load_4d(sRing + s * TILE + b * kBoxBytes, map, &kv_full[s], b * kBoxCols, jt * 128, hkv, bb);
                    ++kvc;
                };
                // The MMA issuer's order: K0, K1, then V(j) and K(j+2) per key tile.
                load_kv(false, 0);
                if (w.n > 1) load_kv(false, 1);
                for (int j = 0; ok && j < w.n; ++j) {
                    load_kv(true, j);
                    if (j + 2 < w.n) load_kv(false, j + 2);
                }
            }
            if (*abort_flag) {
                // Let issued copies land before shared memory is released.
                volatile int never = 0;
                for (int i = max(0, kvc - NS); i < kvc; ++i) mbar_wait(&kv_full[i % NS], (i / NS) & 1, &never);
                for (int i = max(0, uq - 2); i < uq; ++i) mbar_wait(&q_full[i & 1], (i >> 1) & 1, &never);
            }
        } else if (!skip && warp == kWarpMma && lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            constexpr uint32_t kIdescS = idesc_f16(128, 128, BF16 ? 1 : 0, 0, 0);
            constexpr uint32_t kIdescO = idesc_f16(128, D, BF16 ? 1 : 0, 0, 1);
            int uq = 0, kvc = 0, g = 0;
            uint32_t oc = 0;
            bool ok = true;
            // Descriptors are built once; each operand slice is the base
            // descriptor's low word plus a constant added to its start-address
            // field (addresses stay below 256 KB, so it never carries).
            const uint64_t dq0 = smem_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t dk0 = smem_desc_sw128(smem_u32(sRing), 16, 1024);
            const uint64_t dv0 = smem_desc_sw128(smem_u32(sRing), kBoxBytes, 1024);
            const uint32_t q_lo = static_cast<uint32_t>(dq0), qk_hi = static_cast<uint32_t>(dq0 >> 32);
            const uint32_t k_lo = static_cast<uint32_t>(dk0);
            const uint32_t v_lo = static_cast<uint32_t>(dv0), v_hi = static_cast<uint32_t>(dv0 >> 32);
            auto issue_s = [&](int qb, int buf, int stage) {
                const uint32_t a0 = q_lo + static_cast<uint32_t>(qb * (TILE >> 4));
                const uint32_t b0 = k_lo + static_cast<uint32_t>(stage * (TILE >> 4));
                const uint32_t d = tmem + col_s(buf);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = static_cast<uint32_t>(((kk >> 2) * kBoxBytes + (kk & 3) * 32) >> 4);
                    mma_ss_h(d, a0 + off, qk_hi, b0 + off, qk_hi, kIdescS, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[buf]);
            };
            auto issue_pv = [&](int buf, int stage, bool first, bool hilo) {
                const uint32_t b0 = v_lo + static_cast<uint32_t>(stage * (TILE >> 4));
                const uint32_t d = tmem + kColO;
                const uint32_t a = tmem + col_p(buf);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts_h(d, a + kk * 8, b0 + static_cast<uint32_t>(kk * 128), v_hi, kIdescO,
                             (!first || kk > 0) ? 1u : 0u);
                if (hilo) {
                    const uint32_t al = tmem + col_s(buf ^ 1);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_ts_h(d, al + kk * 8, b0 + static_cast<uint32_t>(kk * 128), v_hi, kIdescO, 1u);
                }
                mma_commit(&pv_done[buf]);
            };
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                const int n = w.n;
                const int qb = uq & 1;
                if (!(ok = mbar_wait(&q_full[qb], (uq >> 1) & 1, abort_flag))) break;
                ++uq;
                // K0 -> S(0), K1 -> S(1).
                for (int jt = 0; jt < 2 && jt < n; ++jt) {
                    const int sK = kvc % NS;
                    if (!(ok = mbar_wait(&kv_full[sK], (kvc / NS) & 1, abort_flag))) break;
                    ++kvc;
                    tc_fence_after();
                    issue_s(qb, (g + jt) & 1, sK);
                    if (jt + 1 == n) mma_commit(&q_empty[qb]);
                    mma_commit(&kv_empty[sK]);
                }
                if (!ok) break;
                for (int j = 0; j < n; ++j) {
                    const int G = g + j;
                    const int buf = G & 1;
                    const int sV = kvc % NS;
                    if (!(ok = mbar_wait(&kv_full[sV], (kvc / NS) & 1, abort_flag))) break;
                    ++kvc;
                    if (!(ok = mbar_wait(&p_full[buf], (G >> 1) & 1, abort_flag))) break;
                    if (j == 0 && oc > 0 && !(ok = mbar_wait(o_empty, (oc - 1) & 1, abort_flag))) break;
                    tc_fence_after();
                    issue_pv(buf, sV, j == 0, w.hilo);
                    mma_commit(&kv_empty[sV]);
                    if (j + 2 < n) {
                        const int sK = kvc % NS;
                        if (!(ok = mbar_wait(&kv_full[sK], (kvc / NS) & 1, abort_flag))) break;
                        ++kvc;
                        tc_fence_after();
                        issue_s(qb, buf, sK);
                        if (j + 3 == n) mma_commit(&q_empty[qb]);
                        mma_commit(&kv_empty[sK]);
                    }
                    if (j + 1 == n) {
                        mma_commit(o_full);
                        ++oc;
                    }
                }
                g += n;
            }
            // Drain every MMA issued before tensor memory is released.
            mma_commit(mma_done);
            volatile int never = 0;
            mbar_wait(mma_done, 0, &never);
        }
    } else if (wg < 2) {
        reg_alloc<kRegSoftmax>();
        if (!skip) {
            // ------------------------------------------------------------ softmax of key tiles j = x, x + 2, ...
            const int x = wg;
            const int r_local = (warp & 3) * 32 + lane;  // == tensor-memory lane
            const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
            const float c2 = p.scale_log2;
            const float2 c22 = make_float2(c2, c2);
            // The reference moves up to a lagged maximum only when it lies more than 2^8 above.
            auto move_ref = [&](float r, float M) { return (M != -INFINITY && M * c2 - r > 8.0f) ? M * c2 : r; };
            auto publish = [&](int G, float tmax, float rfin) {
                float *slot = sPub + (G & 3) * 256;
                slot[r_local] = tmax;
                slot[128 + r_local] = rfin;
                __syncwarp();
                if (lane == 0) mbar_arrive(&pub_full[G & 3]);
            };
            int g = 0, uc = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                const int row = w.row0 + r_local;
                float l = 0.f, lref = 0.f;  // this warpgroup's row sum and the reference it is held at
                float m_own = -INFINITY;    // maximum over this warpgroup's key tiles
                float Ma = -INFINITY, Mb = -INFINITY;  // M_(j-3), M_(j-2) at the start of own tile j
                float ra = 0.f;                        // r_(j-2)
                for (int j = x; j < w.n; j += 2) {
                    const int G = g + j;
                    const int buf = G & 1;
                    const uint32_t sa = lane_base + col_s(buf);
                    const uint32_t pa = lane_base + col_p(buf);
                    const uint32_t pl = lane_base + col_s(buf ^ 1);  // hi/lo tiles only
                    const int kbase = j * 128;
                    int lim = p.S - kbase;
                    if (p.causal) lim = min(lim, row - kbase + 1);
                    const bool masked = __any_sync(0xffffffffu, lim < 128);
                    float s[128];
                    uint32_t *sr = reinterpret_cast<uint32_t *>(s);
                    auto mask_half = [&](const int h) {
                        if (masked) {
#pragma unroll
                            for (int c = 64 * h; c < 64 * h + 64; ++c)
                                if (c >= lim) s[c] = -INFINITY;
                        }
                    };
                    if (!(ok = mbar_wait_warp(&s_full[buf], (G >> 1) & 1, abort_flag))) break;
                    // P buffer `buf` is free once P.V two key tiles back has read it.
                    if (G >= 2 && !(ok = mbar_wait_warp(&pv_done[buf], ((G >> 1) - 1) & 1, abort_flag))) break;
                    tc_fence_after();
                    float tmax = -INFINITY, rj, rfin, rsum;
                    float tprev = -INFINITY, rprev = 0.f;  // the other warpgroup's tile j - 1
                    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                    if (j == 0) {
                        // First key tile of the unit: the maximum comes first and is
                        // published at once (the other warpgroup starts from it).
                        tmem_ld32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
                        tmem_ld32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
                        tmem_ld32(sa + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
                        tmem_ld32(sa + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
                        tmem_wait_ld();
                        mask_half(0);
                        mask_half(1);
                        float mx8[8];
#pragma unroll
                        for (int t = 0; t < 8; ++t) mx8[t] = fmax3(s[t], s[t + 8], s[t + 16]);
#pragma unroll
                        for (int c = 24; c < 120; c += 16)
#pragma unroll
                            for (int t = 0; t < 8; ++t) mx8[t] = fmax3(mx8[t], s[c + t], s[c + 8 + t]);
#pragma unroll
                        for (int t = 0; t < 8; ++t) mx8[t] = fmaxf(mx8[t], s[120 + t]);
                        tmax = fmaxf(fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), mx8[6]),
                                     mx8[7]);
                        rj = (tmax == -INFINITY) ? 0.f : tmax * c2;
                        rfin = rj;
                        publish(G, tmax, rfin);
                        const float2 nm2 = make_float2(-rj, -rj);
                        float2 r;
                        if (w.hilo)
                            r = exp_chunks<BF16, true, 0, 128, false>(s, c22, nm2, pa, pl, mx);
                        else
                            r = exp_chunks<BF16, false, 0, 128, false>(s, c22, nm2, pa, pl, mx);
                        rsum = r.x + r.y;
                    } else {
                        if (j == 1) {
                            // r_1 = r_0, the other warpgroup's first reference.
                            if (!(ok = mbar_wait_warp(&pub_full[(G - 1) & 3], ((G - 1) >> 2) & 1, abort_flag))) break;
                            tprev = sPub[((G - 1) & 3) * 256 + r_local];
                            rprev = sPub[((G - 1) & 3) * 256 + 128 + r_local];
                            rj = rprev;
                        } else {
                            rj = move_ref(move_ref(ra, Ma), Mb);  // r_j from r_(j-2) via r_(j-1)
                        }
                        float2 nm2 = make_float2(-rj, -rj);
                        tmem_ld32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
                        tmem_ld32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
                        tmem_wait_ld();
                        tmem_ld32(sa + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
                        tmem_ld32(sa + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
                        mask_half(0);
                        float2 r = exp_chunks<BF16, false, 0, 64, true>(s, c22, nm2, pa, pl, mx);
                        tmem_wait_ld();
                        mask_half(1);
                        r = add2(r, exp_chunks<BF16, false, 64, 128, true>(s, c22, nm2, pa, pl, mx));
                        tmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]);
                        // A tile whose maximum lies more than 2^kSpec above its reference
                        // (P could overflow the 16-bit type) is redone against that maximum.
                        constexpr float kSpec = BF16 ? 30.0f : 15.0f;
                        const bool redo = tmax * c2 - rj > kSpec;
                        rfin = redo ? tmax * c2 : rj;
                        if (__any_sync(0xffffffffu, redo)) {
                            nm2 = make_float2(-rfin, -rfin);
                            tmem_wait_st();
                            r = exp_chunks<BF16, false, 0, 128, false>(s, c22, nm2, pa, pl, mx);
                        }
                        rsum = r.x + r.y;
                        publish(G, tmax, rfin);
                        if (j > 1) {
                            if (!(ok = mbar_wait_warp(&pub_full[(G - 1) & 3], ((G - 1) >> 2) & 1, abort_flag))) break;
                            tprev = sPub[((G - 1) & 3) * 256 + r_local];
                            rprev = sPub[((G - 1) & 3) * 256 + 128 + r_local];
                        }
                        // O holds key tiles < j at reference r'_(j-1); bring it to r'_j.
                        if (__any_sync(0xffffffffu, rprev != rfin)) {
                            if (!(ok = mbar_wait_warp(&pv_done[buf ^ 1], ((G - 1) >> 1) & 1, abort_flag))) break;
                            tc_fence_after();
                            const float fac = (rprev == rfin) ? 1.f : ex2_approx(rprev - rfin);
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
                    l = (j == x) ? rsum : l * ex2_approx(lref - rfin) + rsum;
                    lref = rfin;
                    m_own = fmaxf(m_own, tmax);
                    const float Mjm1 = fmaxf(Mb, tprev);  // M_(j-1)
                    Ma = Mjm1;
                    Mb = fmaxf(Mjm1, tmax);  // M_j
                    ra = rj;
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&p_full[buf]);
                }
                if (!ok) break;
                g += w.n;
                // Row statistics for the epilogue (a warpgroup without key tiles reports l = 0).
                if (uc > 0 && !(ok = mbar_wait_warp(st_empty, (uc - 1) & 1, abort_flag))) break;
                sStats[(x * 3 + 0) * 128 + r_local] = lref;
                sStats[(x * 3 + 1) * 128 + r_local] = m_own;
                sStats[(x * 3 + 2) * 128 + r_local] = (x < w.n) ? l : 0.f;
                __syncwarp();
                if (lane == 0) mbar_arrive(st_full);
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
            uint32_t oc = 0;
            int nb = 0;  // staging boxes used so far
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.n_units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                if (!(ok = mbar_wait_warp(o_full, oc & 1, abort_flag))) break;
                if (!(ok = mbar_wait_warp(st_full, oc & 1, abort_flag))) break;
                ++oc;
                tc_fence_after();
                // O is held at the reference of the unit's last key tile.
                const int xl = (w.n - 1) & 1;
                const float R = sStats[(xl * 3 + 0) * 128 + r_local];
                float l = 0.f;
#pragma unroll
                for (int xx = 0; xx < 2; ++xx) {
                    const float lx = sStats[(xx * 3 + 2) * 128 + r_local];
                    if (lx > 0.f) l += lx * ex2_approx(sStats[(xx * 3 + 0) * 128 + r_local] - R);
                }
                const float m_true = fmaxf(sStats[1 * 128 + r_local], sStats[4 * 128 + r_local]);
                __syncwarp();
                if (lane == 0) mbar_arrive(st_empty);
                const float inv_l = 1.f / l;
                // l at the row maximum m_true (the reference of the m, l outputs).
                const float l_true = (m_true == -INFINITY) ? 0.f : l * ex2_approx(R - m_true * c2);
                const int row = w.row0 + r_local;
                const uint32_t oa = lane_base + kColO;
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
                            if (lane == 0) mbar_arrive(o_empty);
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
                            if (lane == 0) mbar_arrive(o_empty);
                        }
                        if (row < p.S) {
#pragma unroll
                            for (int t = 0; t < 32; t += 4)
                                *reinterpret_cast<float4 *>(orow + cc * 32 + t) =
                                    make_float4(__uint_as_float(o[t]) * inv_l, __uint_as_float(o[t + 1]) * inv_l,
                                                __uint_as_float(o[t + 2]) * inv_l, __uint_as_float(o[t + 3]) * inv_l);
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
                                if (lane == 0) mbar_arrive(o_empty);
                            }
                            uint32_t pk[16];
#pragma unroll
                            for (int t = 0; t < 16; ++t)
                                pk[t] = pack2<BF16>(__uint_as_float(o[2 * t]) * inv_l, __uint_as_float(o[2 * t + 1]) * inv_l);
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
                                tma_store_4d(&tm_o, sStage, b * kBoxCols, w.row0, hh, bb);
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
                    store_as(p.l_out, idx, p.out_dtype, l_true);
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

}  // namespace sd
}  // namespace pmkl_b200
