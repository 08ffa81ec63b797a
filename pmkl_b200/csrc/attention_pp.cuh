// attention_pp.cuh -- persistent, two-query-tile ("ping-pong") tcgen05 flash
// attention forward for sm_100a: fp16/bf16 inputs, head size 64 or 128.
//
// Same results as pmkl::nlp::causal_attention_forward
// (pmkl/nlp/causal_attention.h:145-256): O (normalised), m = row max of the
// scaled masked scores, l = sum exp(s - m).  Organisation:
//
//   * persistent grid (one CTA per SM); a work unit is a pair of adjacent
//     128-row query tiles A, B of one (batch*head) slice.  Units are taken
//     round-robin from a list sorted by decreasing causal work (longest first).
//   * warp roles (16 warps, 4 warpgroups):
//       WG0  softmax of tile A        WG1  softmax of tile B
//       WG2  epilogue (O/l -> 16-bit -> shared -> TMA store; m, l stores)
//       WG3  warp 12: TMA loads (Q_A, Q_B per unit; K, V through a ring)
//            warp 13: tcgen05.mma issue (one thread)
//   * tensor memory: S_A [0,128) S_B [128,256) O_A [256,256+D) O_B [384,384+D).
//     The softmax writes P (16-bit) into the lower half of its S buffer and,
//     for tiles whose rows see at most 128 keys, the low part of a hi/lo split
//     into the upper half; O += P V reads P from tensor memory.
//   * the MMA thread issues, per key tile j:  PV_A(j), S_A(j+1), PV_B(j),
//     S_B(j+1).  tcgen05.mma operations of one thread execute in issue order,
//     so S_X(j+1) (which overwrites P_X(j)) runs after PV_X(j) has read it, and
//     the commit that announces S_X(j+1) also proves PV_X(j) complete, which
//     frees O_X for the softmax's rescale.  While softmax A works on S_A(j+1)
//     the tensor pipe runs PV_B(j) and S_B(j+1), and the other way round.
//   * the O rescale after a max change is skipped unless the running max grew
//     by more than 2^8 (the stale max stays the exp2 reference point; the
//     epilogue corrects m and l once).  After a row's first key tile the exps
//     do not wait for the tile's own maximum: they run against the reference
//     of the earlier tiles while the maximum is gathered alongside, and the
//     rare tile whose maximum lands far above that reference is redone.
//   * hand-offs are kept short on each tile's chain: every softmax and epilogue
//     thread arrives on the barriers it signals (no warp barrier and lane-0
//     branch), warp-wide waits are tested by all 32 lanes (a vote, no
//     broadcast from lane 0), the row-sum bookkeeping follows P's release,
//     and at head size 128 the exps start once scores 0-31 are loaded.
//   * the TMA warp pulls the next unit's Q and first K/V tiles into L2 a unit
//     ahead (PMKL_PP_PREFETCH_NEXT).
//   * every wait is bounded (sm100_ptx.cuh); on expiry the CTA drains its own
//     copies and MMAs, frees tensor memory and reports PMKL_DEVERR_TIMEOUT.
#pragma once

#include "attention_tc.cuh"

namespace pmkl_b200 {
namespace pp {

using tc::kBoxBytes;
using tc::kBoxCols;

constexpr int kThreads = 512;
constexpr int kWarpTma = 12;
constexpr int kWarpMma = 13;
constexpr uint32_t kTmemCols = 512;
__host__ __device__ constexpr uint32_t col_s(int x) { return x ? 128u : 0u; }  // S_A, S_B
__host__ __device__ constexpr uint32_t col_o(int x) { return x ? 384u : 256u; }  // O_A, O_B
// P (hi) lives in the lower half of its S buffer: the columns of scores 0-63,
// which the softmax has read before it stores the first P chunk, so the load
// of scores 64-127 can still be in flight while P of keys 0-63 is stored, and
// scores 64-127 stay intact in tensor memory until the next S.
constexpr uint32_t kPHi = 0;   // P (hi) columns inside an S buffer
constexpr uint32_t kPLo = 64;  // P (lo) columns inside an S buffer
// Head size 64: O takes 64 columns, which leaves room for a P buffer of its
// own per query tile (P_A [320,384), P_B [448,512)).  P then never aliases S,
// so a tile's next S is issued as soon as the softmax has read S, without
// waiting for P.V: the softmax packs P in registers, signals "S read", waits
// for the previous P.V to have read the P buffer and stores P.
__host__ __device__ constexpr uint32_t col_p64(int x) { return x ? 448u : 320u; }

// Register budget per warpgroup after the split (launch: 512 x 128 = 65536).
// The softmax warpgroups hold a 128-score row each; 184 keeps their loop
// almost free of spills (168 spilled ~76 bytes per thread, measured with
// -Xptxas -v), paid for by the epilogue and producer warpgroups.
#ifndef PMKL_PP_REG_SOFTMAX
#define PMKL_PP_REG_SOFTMAX 184
#define PMKL_PP_REG_EPILOGUE 64
#define PMKL_PP_REG_PRODUCER 80
#endif
constexpr uint32_t kRegSoftmax = PMKL_PP_REG_SOFTMAX;
constexpr uint32_t kRegEpilogue = PMKL_PP_REG_EPILOGUE;
constexpr uint32_t kRegProducer = PMKL_PP_REG_PRODUCER;
static_assert(128 * (2 * kRegSoftmax + kRegEpilogue + kRegProducer) <= 65536, "register split exceeds the pool");
constexpr int kLaunchRegs = 128;

template <int D>
struct Cfg {
    static_assert(D == 64 || D == 128, "head size 64 or 128");
    static constexpr int kBoxes = D / kBoxCols;
    static constexpr int kTile = kBoxes * kBoxBytes;       // 128 rows x D x 2 bytes
    static constexpr int kStages = (D == 64) ? 8 : 4;      // K/V ring (K and V alternate)
    static constexpr int kOffQ = 0;                         // Q_A, Q_B
    static constexpr int kOffStage = 2 * kTile;             // epilogue staging, one 128 x 64 box
    static constexpr int kOffRing = kOffStage + kBoxBytes;
    static constexpr int kOffStats = kOffRing + kStages * kTile;  // [2][128] x {m_used, m_true, l}
    static constexpr int kOffBars = kOffStats + 2 * 128 * 3 * 4;
    static constexpr int kNumBars = 4 + 2 * kStages + 2 + 2 + 2 + 2 + 2 + 2 + 3 + 4;
    static constexpr int kSmemBytes = kOffBars + kNumBars * 8 + 16 + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Params {
    int S;
    int BH;
    int H;         // query heads per batch entry (slice bh = b * H + h)
    int kv_group;  // query heads per K/V head: slice (b, h) reads K/V head h / kv_group
    long long o_sb, o_sh, o_ss;  // element strides of O (batch, head, row) for fp32 output
    int n_pairs;     // ceil(n_qt / 2)
    int n_units;     // n_pairs * BH
    int n_rounds;    // ceil(n_units / gridDim.x)
    int group;       // (b, h) slices per scheduling group
    int snake;       // odd rounds go to the CTAs in reverse order
    int flip;        // odd groups run their pairs shortest first
    int causal;
    int out_dtype;
    float scale;
    float scale_log2;
    void *o_f32;
    void *m_out;
    void *l_out;
};

// The backward's instantiation writes row statistics instead of O, m, l: for
// each query row, b = m~ log2 e + log2 l~ and delta = exp(m - m~) (l / l~)
// (dO . O), with m~, l~ the caller's statistics (input dtype) and m, l, O this
// kernel's own; rows in [S, S_pad) get (0, 0).
struct DeltaParams {
    int S_pad;
    const void *dout;      // [B][H][S][D], input dtype, element strides do_s (batch, head, row)
    long long do_s[3];
    const void *m_given;   // [BH][S]
    const void *l_given;
    float2 *rowstat;       // [BH][S_pad]
};

struct Unit {
    int bh;
    int row0;     // first row of tile A
    bool act[2];  // tile active (row0 of the tile < S)
    int n[2];     // key tiles per query tile
    int n_max;
    bool hilo[2];
};

// Work order: slices are taken in groups of p.group (b, h) slices whose K and
// V together fit in L2, and inside a group the query-tile pairs go longest
// first (with p.flip, every other group shortest first, so that a CTA that
// drew long pairs in one group draws short ones in the next).  All pairs of a
// slice then run close together in time and re-read that slice's K/V from L2
// instead of HBM.
__device__ __forceinline__ Unit decode(const Params &p, int u) {
    Unit w;
    const int n_kv_all = (p.S + 127) / 128;
    const int per_group = p.n_pairs * p.group;
    const int g = u / per_group;
    const int within = u - g * per_group;
    const int g_slices = min(p.group, p.BH - g * p.group);
    const int rank0 = within / g_slices;
    const int rank = (p.flip && (g & 1)) ? (p.n_pairs - 1 - rank0) : rank0;
    const int pair = p.causal ? (p.n_pairs - 1 - rank) : rank;
    w.bh = g * p.group + (within - rank0 * g_slices);
    w.row0 = pair * 256;
    for (int x = 0; x < 2; ++x) {
        const int r0 = w.row0 + 128 * x;
        w.act[x] = r0 < p.S;
        w.n[x] = !w.act[x] ? 0 : (p.causal ? min(r0 / 128 + 1, n_kv_all) : n_kv_all);
        w.hilo[x] = w.act[x] && w.n[x] == 1 && (p.causal ? (r0 == 0) : true);
    }
    w.n_max = max(w.n[0], w.n[1]);
    return w;
}

// The list entry a CTA takes in round k: rounds of gridDim.x consecutive
// entries, one per CTA; with p.snake, odd rounds hand them out in reverse CTA
// order, so that over a longest-first list every CTA alternates between the
// long and the short end of a round.  Returns n_units or more for a CTA that
// has no entry in the (last, partial) round.
__device__ __forceinline__ int unit_of(const Params &p, int k) {
    const int b = (p.snake && (k & 1)) ? static_cast<int>(gridDim.x - 1 - blockIdx.x) : static_cast<int>(blockIdx.x);
    return k * static_cast<int>(gridDim.x) + b;
}

// 2^x for x <= 0 on the FMA pipe, two lanes per instruction, to take load off
// the MUFU unit (16 ex2 per clock per SM, which otherwise caps the softmax):
//   x = n + f with n = round(x) (read from the low mantissa bits of
//   x + 1.5*2^23) and f in [-1/2, 1/2];
//   2^f by a degree-3 polynomial, a Chebyshev-node least-squares fit refined
//   towards minimax (Lawson iterations), max relative error 7.5e-5 -- below
//   the 2^-9 rounding that P gets anyway;
//   2^n by adding n to the exponent field.
// x is clamped to -125 so the result stays a normal number.
__device__ __forceinline__ float2 exp2_poly(float2 x) {
    using namespace ptx;
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    x.x = fmaxf(x.x, -125.0f);
    x.y = fmaxf(x.y, -125.0f);
    const float2 r = add2(x, make_float2(kMagic, kMagic));
    const float2 n = add2(r, make_float2(-kMagic, -kMagic));
    const float2 f = fma2(n, make_float2(-1.0f, -1.0f), x);
    float2 p = fma2(f, make_float2(0.0551716648f, 0.0551716648f), make_float2(0.2426111251f, 0.2426111251f));
    p = fma2(p, f, make_float2(0.6932609677f, 0.6932609677f));
    p = fma2(p, f, make_float2(0.9999280572f, 0.9999280572f));
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(r.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(r.y) << 23)));
}

// p = 2^(s * c2 - mref) for one 128-key score row, packed to 16-bit pairs and
// stored into the P (hi) columns of the row's S buffer (and, with HILO, the
// rounding remainder into the P (lo) columns).  With `poly`, the first NPOLY
// pairs of each 32-key chunk go through exp2_poly, the rest through
// ex2.approx.  Returns the fp32 row sum.  The kernel calls the HILO form (rare:
// tiles whose rows see at most 128 keys) and the plain form from one place
// each, so that only one copy of the hot loop competes for the instruction
// cache with the MMA-issuing warp.
// DEFER: P (hi) goes to `pbuf` (32-bit words, two keys each) instead of
// tensor memory; the caller stores it later.
template <bool BF16, bool HILO, int NPOLY, bool DEFER = false>
__device__ __forceinline__ float exp_pack_store(const float (&s)[128], float c2, float mref, uint32_t sa, bool poly,
                                                uint32_t (&pbuf)[64]) {
    using namespace ptx;
    float2 rs2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    const float2 c22 = make_float2(c2, c2);
    const float2 nm2 = make_float2(-mref, -mref);
#pragma unroll
    for (int c0 = 0; c0 < 128; c0 += 32) {
        uint32_t ph[16];
        uint32_t pl[HILO ? 16 : 1];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float2 a = fma2(make_float2(s[c0 + 2 * i], s[c0 + 2 * i + 1]), c22, nm2);
            const float2 e =
                (!HILO && i < NPOLY && poly) ? exp2_poly(a) : make_float2(ex2_approx(a.x), ex2_approx(a.y));
            rs2[i & 3] = add2(rs2[i & 3], e);
            ph[i] = pack2<BF16>(e.x, e.y);
            if constexpr (HILO) {
                float h0, h1;
                tc::unpack2<BF16>(ph[i], h0, h1);
                pl[i] = pack2<BF16>(e.x - h0, e.y - h1);
            }
        }
        if constexpr (DEFER) {
#pragma unroll
            for (int i = 0; i < 16; ++i) pbuf[c0 / 2 + i] = ph[i];
        } else {
            tmem_st16(sa + kPHi + c0 / 2, ph);
        }
        if constexpr (HILO) tmem_st16(sa + kPLo + c0 / 2, pl);
    }
    const float2 rr = add2(add2(rs2[0], rs2[1]), add2(rs2[2], rs2[3]));
    return rr.x + rr.y;
}

// The speculative form used after a row's first key tile: exps of the 32-key
// chunks [C0, C1) against a reference taken from earlier tiles, P stored as
// above, and (TRACK) the row maximum of these scores gathered on the side in
// four running maxima, so that the maximum is off the path from S to P.
// Returns the partial row sum as a pair.
template <bool BF16, int NPOLY, int C0, int C1, bool TRACK, bool DEFER = false>
__device__ __forceinline__ float2 exp_chunks(const float (&s)[128], float2 c22, float2 nm2, uint32_t sa, bool poly,
                                             float (&mx)[4], uint32_t (&pbuf)[64]) {
    using namespace ptx;
    float2 rs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int c0 = C0; c0 < C1; c0 += 32) {
        uint32_t ph[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float s0 = s[c0 + 2 * i], s1 = s[c0 + 2 * i + 1];
            if constexpr (TRACK) mx[i & 3] = fmax3(mx[i & 3], s0, s1);
            const float2 a = fma2(make_float2(s0, s1), c22, nm2);
            const float2 e = (i < NPOLY && poly) ? exp2_poly(a) : make_float2(ex2_approx(a.x), ex2_approx(a.y));
            rs2[i & 1] = add2(rs2[i & 1], e);
            ph[i] = pack2<BF16>(e.x, e.y);
        }
        if constexpr (DEFER) {
#pragma unroll
            for (int i = 0; i < 16; ++i) pbuf[c0 / 2 + i] = ph[i];
        } else {
            tmem_st16(sa + kPHi + c0 / 2, ph);
        }
    }
    return add2(rs2[0], rs2[1]);
}

// Pairs per 32-key chunk whose exp2 runs on the FMA pipe (0..16); the rest
// use the MUFU unit.  A build-time knob, tuned on B200.
#ifndef PMKL_PP_PREFETCH_NEXT
#define PMKL_PP_PREFETCH_NEXT 1
#endif
#ifndef PMKL_PP_NPOLY
#define PMKL_PP_NPOLY 0
#endif

// DELTA: the backward's instantiation, writing the row statistics (b, delta)
// instead of O, m, l (DeltaParams).
template <int D, bool BF16, int NPOLY = PMKL_PP_NPOLY, bool DELTA = false>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_pp_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
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
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kOffBars);
    uint64_t *q_full = bars;             // [2]
    uint64_t *q_empty = bars + 2;        // [2]
    uint64_t *kv_full = bars + 4;        // [NS]
    uint64_t *kv_empty = kv_full + NS;   // [NS]
    uint64_t *s_full = kv_empty + NS;    // [2]
    uint64_t *p_full = s_full + 2;       // [2]
    uint64_t *o_full = p_full + 2;       // [2]
    uint64_t *o_empty = o_full + 2;      // [2]
    uint64_t *st_full = o_empty + 2;     // [2]
    uint64_t *st_empty = st_full + 2;    // [2]
    uint64_t *mma_done = st_empty + 2;
    uint64_t *stg_written = mma_done + 1;  // epilogue warps -> store thread
    uint64_t *stg_free = stg_written + 1;  // store thread -> epilogue warps
    uint64_t *s_read = stg_free + 1;       // [2] head size 64: the softmax has read S_X
    uint64_t *pv_done = s_read + 2;        // [2] head size 64: P.V of tile X complete
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pv_done + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int wg = warp >> 2;
    // Warp-wide waits (softmax and epilogue warps): every lane tests the
    // barrier and the warp agrees by vote, with no single-lane wait and
    // broadcast on a tile's chain (B200, config 3: 994 -> 1054 TFLOP/s).  Head
    // size 128 parks the warp with suspend-hinted tests; head size 64 polls
    // (parking measured 2-4 % slower there, polling 4-8 % faster).
    auto wait_warp = [&](uint64_t *bar, uint32_t parity) -> bool {
        if constexpr (D == 128)
            return mbar_wait_warp_all(bar, parity, abort_flag);
        else
            return mbar_wait_warp_poll(bar, parity, abort_flag);
    };

    if (threadIdx.x == 0) {
        for (int x = 0; x < 2; ++x) {
            mbar_init(&q_full[x], 1);
            mbar_init(&q_empty[x], 1);
            mbar_init(&s_full[x], 1);
            mbar_init(&p_full[x], 128);  // every softmax thread releases its own P row
            mbar_init(&o_full[x], 1);
            mbar_init(&o_empty[x], 128);  // hand-offs between warpgroups: one arrival per thread
            mbar_init(&st_full[x], 128);
            mbar_init(&st_empty[x], 128);
            mbar_init(&s_read[x], 4);
            mbar_init(&pv_done[x], 1);
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
            // Per-tile counters are separate scalars (not arrays indexed by a
            // run-time tile number), so that they stay in registers.
            uint32_t qc0 = 0, qc1 = 0;
            int kvc = 0;
            bool ok = true;
            for (int k = 0; ok && k < p.n_rounds; ++k) {
                const int u = unit_of(p, k);
                if (u >= p.n_units) continue;
                const Unit w = decode(p, u);
                const int bb = w.bh / p.H;
                const int hh = w.bh - bb * p.H;
                const int hkv = hh / p.kv_group;
                auto load_q = [&](const int x, uint32_t &qcx) {
                    if (!ok) return;
                    if (qcx > 0 && !(ok = mbar_wait(&q_empty[x], (qcx - 1) & 1, abort_flag))) return;
                    mbar_arrive_expect_tx(&q_full[x], TILE);
#pragma unroll
                    for (int b = 0; b < C::kBoxes; ++b)
                        tma_load_4d(sQ + x * TILE + b * kBoxBytes, &tm_q, &q_full[x], b * kBoxCols, w.row0 + 128 * x,
                                    hh, bb);
                    ++qcx;
                };
                if (w.act[0]) load_q(0, qc0);
                if (w.act[1]) load_q(1, qc1);
#if PMKL_PP_PREFETCH_NEXT
                // The next unit's Q tiles (read once, from HBM) and its first K
                // and V tiles are pulled into L2 now, a unit ahead, so that the
                // loads at the unit boundary are served from L2.
                if (k + 1 < p.n_rounds) {
                    const int un = unit_of(p, k + 1);
                    if (un < p.n_units) {
                        const Unit wn = decode(p, un);
                        const int bn = wn.bh / p.H;
                        const int hn = wn.bh - bn * p.H;
#pragma unroll
                        for (int b = 0; b < C::kBoxes; ++b) {
                            tma_prefetch_l2_4d(&tm_q, b * kBoxCols, wn.row0, hn, bn);
                            if (wn.act[1]) tma_prefetch_l2_4d(&tm_q, b * kBoxCols, wn.row0 + 128, hn, bn);
                            tma_prefetch_l2_4d(&tm_k, b * kBoxCols, 0, hn / p.kv_group, bn);
                            tma_prefetch_l2_4d(&tm_v, b * kBoxCols, 0, hn / p.kv_group, bn);
                        }
                    }
                }
#endif
                // One K or V tile into the next ring stage.
                auto load_kv = [&](const int kv, const int jt) {
                    if (!ok) return;
                    const int s = kvc % NS;
                    if (kvc >= NS && !(ok = mbar_wait(&kv_empty[s], ((kvc / NS) - 1) & 1, abort_flag))) return;
                    mbar_arrive_expect_tx(&kv_full[s], TILE);
                    const CUtensorMap *map = kv ? &tm_v : &tm_k;
                    for (int b = 0; b < C::kBoxes; ++b)
                        tma_load_4d(sRing + s * TILE + b * kBoxBytes, map, &kv_full[s], b * kBoxCols, jt * 128, hkv, bb);
                    ++kvc;
                };
                if constexpr (D == 64) {
                    // The issuer's order here: K0, then K(j+1) and V(j) per key tile.
                    load_kv(0, 0);
                    for (int j = 0; ok && j < w.n_max; ++j) {
                        if (j + 1 < w.n_max) load_kv(0, j + 1);
                        load_kv(1, j);
                    }
                } else {
                    for (int j = 0; ok && j < w.n_max; ++j) {
                        load_kv(0, j);
                        load_kv(1, j);
                    }
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
            constexpr uint32_t kIdescS = idesc_f16(128, 128, BF16 ? 1 : 0, 0, 0);
            constexpr uint32_t kIdescO = idesc_f16(128, D, BF16 ? 1 : 0, 0, 1);
            uint32_t qc0 = 0, qc1 = 0, pc0 = 0, pc1 = 0, oc0 = 0, oc1 = 0, rc0 = 0, rc1 = 0;
            int kvc = 0;
            bool ok = true;
            // Descriptors are built once; every operand slice is then the base
            // descriptor's low word plus a constant added to its 14-bit
            // start-address field (addresses stay below 256 KB, so the field
            // never carries into the high word).
            const uint64_t dq0 = smem_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t dk0 = smem_desc_sw128(smem_u32(sRing), 16, 1024);         // K view of stage 0
            const uint64_t dv0 = smem_desc_sw128(smem_u32(sRing), kBoxBytes, 1024);  // V view of stage 0
            const uint32_t q_lo = static_cast<uint32_t>(dq0), qk_hi = static_cast<uint32_t>(dq0 >> 32);
            const uint32_t k_lo = static_cast<uint32_t>(dk0);
            const uint32_t v_lo = static_cast<uint32_t>(dv0), v_hi = static_cast<uint32_t>(dv0 >> 32);
            auto issue_s = [&](int x, int stage) {
                const uint32_t a0 = q_lo + static_cast<uint32_t>(x * (TILE >> 4));
                const uint32_t b0 = k_lo + static_cast<uint32_t>(stage * (TILE >> 4));
                const uint32_t d = tmem + col_s(x);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = static_cast<uint32_t>(((kk >> 2) * kBoxBytes + (kk & 3) * 32) >> 4);
                    mma_ss_h(d, a0 + off, qk_hi, b0 + off, qk_hi, kIdescS, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[x]);
            };
            auto issue_pv = [&](int x, int stage, bool first, bool hilo) {
                const uint32_t b0 = v_lo + static_cast<uint32_t>(stage * (TILE >> 4));
                const uint32_t d = tmem + col_o(x);
                const uint32_t a = tmem + col_s(x);
                const uint32_t ahi = (D == 64) ? tmem + col_p64(x) : a + kPHi;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts_h(d, ahi + kk * 8, b0 + static_cast<uint32_t>(kk * 128), v_hi, kIdescO,
                             (!first || kk > 0) ? 1u : 0u);
                if (hilo) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_ts_h(d, a + kPLo + kk * 8, b0 + static_cast<uint32_t>(kk * 128), v_hi, kIdescO, 1u);
                }
            };
            for (int k = 0; ok && k < p.n_rounds; ++k) {
                const int u = unit_of(p, k);
                if (u >= p.n_units) continue;
                const Unit w = decode(p, u);
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
                // K_0 -> S_A(0), S_B(0)
                int sK = kvc % NS;
                if (!(ok = mbar_wait(&kv_full[sK], (kvc / NS) & 1, abort_flag))) break;
                ++kvc;
                tc_fence_after();
                if (w.act[0]) {
                    issue_s(0, sK);
                    if (n0 == 1) mma_commit(&q_empty[0]);
                }
                if (w.act[1]) {
                    issue_s(1, sK);
                    if (n1 == 1) mma_commit(&q_empty[1]);
                }
                mma_commit(&kv_empty[sK]);
                if constexpr (D == 64) {
                    // Per key tile j and query tile X: S_X(j+1) once the softmax has
                    // read S_X(j), then P.V_X(j) once P_X(j) is stored.
                    for (int j = 0; ok && j < w.n_max; ++j) {
                        const bool has_next = j + 1 < w.n_max;
                        if (has_next) {
                            sK = kvc % NS;
                            if (!(ok = mbar_wait(&kv_full[sK], (kvc / NS) & 1, abort_flag))) break;
                            ++kvc;
                        }
                        const int sV = kvc % NS;
                        if (!(ok = mbar_wait(&kv_full[sV], (kvc / NS) & 1, abort_flag))) break;
                        ++kvc;
                        auto tile64 = [&](const int x, const int nx, const bool hlx, uint32_t &rcx, uint32_t &pcx,
                                          uint32_t &ocx) {
                            if (!ok || j >= nx) return;
                            if (!(ok = mbar_wait(&s_read[x], rcx & 1, abort_flag))) return;
                            ++rcx;
                            if (j + 1 < nx) {
                                tc_fence_after();
                                issue_s(x, sK);
                                if (j + 2 == nx) mma_commit(&q_empty[x]);
                            }
                            if (!(ok = mbar_wait(&p_full[x], pcx & 1, abort_flag))) return;
                            ++pcx;
                            if (j == 0 && ocx > 0 && !(ok = mbar_wait(&o_empty[x], (ocx - 1) & 1, abort_flag)))
                                return;
                            tc_fence_after();
                            issue_pv(x, sV, j == 0, hlx);
                            mma_commit(&pv_done[x]);
                            if (j + 1 == nx) {
                                mma_commit(&o_full[x]);
                                ++ocx;
                            }
                        };
                        tile64(0, n0, hl0, rc0, pc0, oc0);
                        tile64(1, n1, hl1, rc1, pc1, oc1);
                        if (!ok) break;
                        if (has_next) mma_commit(&kv_empty[sK]);
                        mma_commit(&kv_empty[sV]);
                    }
                } else {
                    for (int j = 0; ok && j < w.n_max; ++j) {
                        const int sV = kvc % NS;
                        if (!(ok = mbar_wait(&kv_full[sV], (kvc / NS) & 1, abort_flag))) break;
                        ++kvc;
                        const bool has_next = j + 1 < w.n_max;
                        const int kvc_next = kvc;
                        if (has_next) {
                            sK = kvc % NS;
                            ++kvc;
                        }
                        bool k_ready = false;
                        auto tile = [&](const int x, const int nx, const bool hlx, uint32_t &pcx, uint32_t &ocx) {
                            if (!ok || j >= nx) return;
                            if (!(ok = mbar_wait(&p_full[x], pcx & 1, abort_flag))) return;
                            ++pcx;
                            if (j == 0 && ocx > 0 && !(ok = mbar_wait(&o_empty[x], (ocx - 1) & 1, abort_flag))) return;
                            tc_fence_after();
                            issue_pv(x, sV, j == 0, hlx);
                            if (j + 1 < nx) {
                                if (!k_ready) {
                                    if (!(ok = mbar_wait(&kv_full[sK], (kvc_next / NS) & 1, abort_flag))) return;
                                    k_ready = true;
                                    tc_fence_after();
                                }
                                issue_s(x, sK);
                                if (j + 2 == nx) mma_commit(&q_empty[x]);
                            } else {
                                mma_commit(&o_full[x]);
                                ++ocx;
                            }
                        };
                        tile(0, n0, hl0, pc0, oc0);
                        tile(1, n1, hl1, pc1, oc1);
                        if (!ok) break;
                        mma_commit(&kv_empty[sV]);
                        if (has_next) mma_commit(&kv_empty[sK]);
                    }
                }
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
            const uint32_t sa = lane_base + col_s(x);
            const float c2 = p.scale_log2;
            int sc = 0, uc = 0;
            uint32_t pvc = 0;  // head size 64: P tiles stored so far (one P.V each)
            bool ok = true;
            for (int k = 0; ok && k < p.n_rounds; ++k) {
                const int u = unit_of(p, k);
                if (u >= p.n_units) continue;
                const Unit w = decode(p, u);
                // This warpgroup's tile, picked by value (no run-time array index).
                const bool actx = x ? w.act[1] : w.act[0];
                const int nx = x ? w.n[1] : w.n[0];
                const bool hilox = x ? w.hilo[1] : w.hilo[0];
                if (!actx) continue;
                const int row = w.row0 + 128 * x + r_local;
                float m_used = -INFINITY, m_true = -INFINITY, l = 0.f;
                for (int j = 0; j < nx; ++j) {
                    const int kbase = j * 128;
                    int lim = p.S - kbase;
                    if (p.causal) lim = min(lim, row - kbase + 1);
                    const bool masked = __any_sync(0xffffffffu, lim < 128);
                    float s[128];
                    uint32_t pbuf[64];  // head size 64: P (hi) until the P buffer is free
                    uint32_t *sr = reinterpret_cast<uint32_t *>(s);
                    auto mask_range = [&](const int c0, const int c1) {
                        if (masked) {
#pragma unroll
                            for (int c = c0; c < c1; ++c)
                                if (c >= lim) s[c] = -INFINITY;
                        }
                    };
                    auto mask_half = [&](const int h) {
                        if (masked) {
#pragma unroll
                            for (int c = 64 * h; c < 64 * h + 64; ++c)
                                if (c >= lim) s[c] = -INFINITY;
                        }
                    };
                    float m_new, fac, rsum;
                    bool any_fac;
                    if (j == 0) {
                        // First key tile of the row: the maximum comes first.
                        if (!(ok = wait_warp(&s_full[x], sc & 1))) break;
                        ++sc;
                        tc_fence_after();
                        float mx8[8];
                        tmem_ld32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
                        tmem_ld32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
                        tmem_wait_ld();
                        tmem_ld32(sa + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
                        tmem_ld32(sa + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
                        mask_half(0);
#pragma unroll
                        for (int t = 0; t < 8; ++t) mx8[t] = fmax3(s[t], s[t + 8], s[t + 16]);
#pragma unroll
                        for (int t = 0; t < 8; ++t) mx8[t] = fmax3(mx8[t], s[t + 24], s[t + 32]);
#pragma unroll
                        for (int t = 0; t < 8; ++t) mx8[t] = fmax3(mx8[t], s[t + 40], s[t + 48]);
#pragma unroll
                        for (int t = 0; t < 8; ++t) mx8[t] = fmaxf(mx8[t], s[t + 56]);
                        tmem_wait_ld();
                        mask_half(1);
#pragma unroll
                        for (int c = 64; c < 128; c += 16)
#pragma unroll
                            for (int t = 0; t < 8; ++t) mx8[t] = fmax3(mx8[t], s[c + t], s[c + 8 + t]);
                        m_true = fmaxf(fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), mx8[6]),
                                       mx8[7]);
                        m_new = m_true;
                        const float mref = (m_new == -INFINITY) ? 0.f : m_new * c2;
                        if (hilox)
                            rsum = exp_pack_store<BF16, true, 0, D == 64>(s, c2, mref, sa, false, pbuf);
                        else
                            rsum = exp_pack_store<BF16, false, NPOLY, D == 64>(s, c2, mref, sa, !masked, pbuf);
                        fac = 0.f;  // l and O hold nothing yet
                        any_fac = false;
                    } else {
                        // Later key tiles: the exps run against a reference taken
                        // from earlier tiles (known before S arrives) while this
                        // tile's maximum is gathered alongside.  A reference more
                        // than 2^8 below the running maximum is moved up first.
                        // A tile whose own maximum is more than 2^kSpec above the
                        // reference (P could then overflow the 16-bit type, or
                        // lose the row's scale) is redone against its maximum.
                        m_new = ((m_true - m_used) * c2 > 8.0f) ? m_true : m_used;
                        const float2 c22 = make_float2(c2, c2);
                        float2 nm2 = make_float2(-m_new * c2, -m_new * c2);
                        // Whether O and l move to a new reference this step is
                        // known before S arrives; the vote is off the path from
                        // the last exp to P's release.
                        any_fac = __any_sync(0xffffffffu, m_new != m_used);
                        if (!(ok = wait_warp(&s_full[x], sc & 1))) break;
                        ++sc;
                        tc_fence_after();
                        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                        float2 r;
                        if constexpr (D == 128) {
                            // The exps start once scores 0-31 are in registers;
                            // the other 96 load meanwhile.  P of keys 0-31 goes to
                            // columns whose scores have been read.
                            tmem_ld32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
                            tmem_wait_ld();
                            tmem_ld32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
                            tmem_ld32(sa + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
                            tmem_ld32(sa + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
                            mask_range(0, 32);
                            r = exp_chunks<BF16, NPOLY, 0, 32, true, false>(s, c22, nm2, sa, !masked, mx, pbuf);
                            tmem_wait_ld();
                            mask_range(32, 128);
                            r = add2(r, exp_chunks<BF16, NPOLY, 32, 128, true, false>(s, c22, nm2, sa, !masked, mx, pbuf));
                        } else {
                            tmem_ld32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
                            tmem_ld32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
                            tmem_wait_ld();
                            tmem_ld32(sa + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
                            tmem_ld32(sa + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
                            mask_half(0);
                            r = exp_chunks<BF16, NPOLY, 0, 64, true, true>(s, c22, nm2, sa, !masked, mx, pbuf);
                            tmem_wait_ld();
                            mask_half(1);
                            r = add2(r, exp_chunks<BF16, NPOLY, 64, 128, true, true>(s, c22, nm2, sa, !masked, mx, pbuf));
                        }
                        m_true = fmaxf(m_true, fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]));
                        constexpr float kSpec = BF16 ? 30.0f : 15.0f;
                        const bool redo = (m_true - m_new) * c2 > kSpec;
                        if (__any_sync(0xffffffffu, redo)) {
                            if (redo) m_new = m_true;
                            any_fac = __any_sync(0xffffffffu, m_new != m_used);
                            nm2 = make_float2(-m_new * c2, -m_new * c2);
                            float unused[4];
                            if constexpr (D == 64) {
                                // Rare.  S is untouched by P here (P waits in
                                // registers): stream the scores back 32 at a
                                // time into the deferred P words, so that the
                                // path needs no more registers than the common one.
                                r = make_float2(0.f, 0.f);
#pragma unroll
                                for (int c0 = 0; c0 < 128; c0 += 32) {
                                    uint32_t w[32];
                                    tmem_ld32(sa + c0, w);
                                    tmem_wait_ld();
                                    uint32_t ph[16];
#pragma unroll
                                    for (int i = 0; i < 16; ++i) {
                                        float s0 = __uint_as_float(w[2 * i]), s1 = __uint_as_float(w[2 * i + 1]);
                                        if (masked && c0 + 2 * i >= lim) s0 = -INFINITY;
                                        if (masked && c0 + 2 * i + 1 >= lim) s1 = -INFINITY;
                                        const float2 a = fma2(make_float2(s0, s1), c22, nm2);
                                        const float2 e = make_float2(ex2_approx(a.x), ex2_approx(a.y));
                                        r = add2(r, e);
                                        ph[i] = pack2<BF16>(e.x, e.y);
                                    }
#pragma unroll
                                    for (int i = 0; i < 16; ++i) pbuf[c0 / 2 + i] = ph[i];
                                }
                            } else {
                                // Rare: scores 64-127 are reloaded (P went to the
                                // columns of scores 0-63), scores 0-63 are still in
                                // registers.
                                tmem_ld32(sa + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
                                tmem_ld32(sa + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
                                tmem_wait_ld();
                                mask_half(1);
                                tmem_wait_st();
                                r = exp_chunks<BF16, 0, 0, 128, false, false>(s, c22, nm2, sa, false, unused, pbuf);
                            }
                        }
                        rsum = r.x + r.y;
                        fac = 1.f;  // the rare rescale below sets the factor
                    }
                    if constexpr (D == 64) {
                        // S_X may be overwritten from here on; P goes to its own
                        // buffer once P.V of the previous key tile has read it
                        // (which also leaves O_X idle for the rescale below).
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&s_read[x]);
                        if (pvc > 0 && !(ok = wait_warp(&pv_done[x], (pvc - 1) & 1))) break;
                        ++pvc;
                        tc_fence_after();
                        tmem_st32(lane_base + col_p64(x), *reinterpret_cast<uint32_t(*)[32]>(pbuf));
                        tmem_st32(lane_base + col_p64(x) + 32, *reinterpret_cast<uint32_t(*)[32]>(pbuf + 32));
                    }
                    // O_X is idle here (head size 128: S_X(j) was issued after PV_X(j-1),
                    // and its commit covers every earlier MMA).
                    if (any_fac) {
                        fac = (m_new == m_used) ? 1.f : ex2_approx((m_used - m_new) * c2);
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
                    // Every thread releases its own row (its release covers its own
                    // P stores), so no warp barrier or single-lane branch sits
                    // between the last P store and the arrive.
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(&p_full[x]);
                    // Row-sum bookkeeping after P is released.
                    l = l * fac + rsum;
                    m_used = m_new;
                }
                if (!ok) break;
                // Row statistics for the epilogue.
                if (uc > 0 && !(ok = wait_warp(&st_empty[x], (uc - 1) & 1))) break;
                sStats[(x * 3 + 0) * 128 + r_local] = m_used;
                sStats[(x * 3 + 1) * 128 + r_local] = m_true;
                sStats[(x * 3 + 2) * 128 + r_local] = l;
                mbar_arrive(&st_full[x]);
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
            for (int k = 0; ok && k < p.n_rounds; ++k) {
                const int u = unit_of(p, k);
                if (u >= p.n_units) continue;
                const Unit w = decode(p, u);
                for (int x = 0; x < 2 && ok; ++x) {
                    if (!(x ? w.act[1] : w.act[0])) continue;
                    const uint32_t ocx = x ? oc1 : oc0;
                    if (!(ok = wait_warp(&o_full[x], ocx & 1))) break;
                    if (!(ok = wait_warp(&st_full[x], ocx & 1))) break;
                    if (x) ++oc1; else ++oc0;
                    tc_fence_after();
                    const float m_used = sStats[(x * 3 + 0) * 128 + r_local];
                    const float m_true = sStats[(x * 3 + 1) * 128 + r_local];
                    const float l = sStats[(x * 3 + 2) * 128 + r_local];
                    mbar_arrive(&st_empty[x]);
                    const float inv_l = 1.f / l;
                    const int row = w.row0 + 128 * x + r_local;
                    const uint32_t oa = lane_base + col_o(x);
                    const int bb = w.bh / p.H;
                    const int hh = w.bh - bb * p.H;
                    if constexpr (DELTA) {
                        using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
                        const size_t ridx = static_cast<size_t>(w.bh) * p.S + row;
                        const uint4 *drow = reinterpret_cast<const uint4 *>(
                            static_cast<const T *>(dpar.dout) + bb * dpar.do_s[0] + hh * dpar.do_s[1] +
                            static_cast<long long>(row) * dpar.do_s[2]);
                        float dot = 0.f;
#pragma unroll
                        for (int cc = 0; cc < D / 32; ++cc) {
                            uint32_t o[32];
                            tmem_ld32(oa + cc * 32, o);
                            tmem_wait_ld();
                            if (cc == D / 32 - 1) {
                                tc_fence_before();
                                mbar_arrive(&o_empty[x]);
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
                                mbar_arrive(&o_empty[x]);
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
                            if (nb > 0 && !(ok = wait_warp(stg_free, (nb - 1) & 1))) break;
                            uint8_t *box = sStage + r_local * 128;
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                uint32_t o[32];
                                tmem_ld32(oa + b * 64 + h * 32, o);
                                tmem_wait_ld();
                                if (b == C::kBoxes - 1 && h == 1) {
                                    tc_fence_before();
                                    mbar_arrive(&o_empty[x]);
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

}  // namespace pp
}  // namespace pmkl_b200
