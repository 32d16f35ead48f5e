// Paged multi-query attention on tcgen05 for head_dim 128 with 128-key tiles
// (chunked prefill and long verify chains; the packed query tile has >= 64
// rows).  The tensor pipe's cost per kind::f16 MMA (M 128, K 16) is about the
// same for every N up to 128, so both products here run at N = 128: the score
// MMA over 128 keys and the PV MMA over the 128 head-dim columns.
//
// One CTA owns (sequence b, KV head h, one query tile of kTcRows = 128 packed
// rows: row r is token t0 + r / G, query head h*G + r % G).  Twelve warps:
//
//   producer warps: TMA loads of K(i), V(i) (eight 16-token pool blocks each,
//                   128-byte column halves, 128-byte swizzle) into a ring of
//                   five 32 KB slots, in the order the MMAs read them; three
//                   warps issue them (one TMA instruction costs its issuing
//                   thread ~100 cycles, so one thread cannot keep up);
//   MMA warp      : one thread issues S(i) = Q K(i)^T into TMEM buffer i % 2
//                   (Q read from TMEM) and O += P(i) V(i) into TMEM, in the
//                   order S(0), S(1), PV(0), S(2), PV(1), S(3), ...: while the
//                   softmax works on S(i), the tensor pipe runs PV(i-1) and
//                   S(i+1);
//   warps 0-7     : softmax in two warpgroups, thread (c, r) owning key columns
//                   [64 c, 64 c + 64) of row r (TMEM lane r): its 64 S values
//                   in registers, causal / sliding-window mask on edge tiles
//                   only, the row max shared with the other half through
//                   shared memory, running max and a per-half denominator
//                   (summed in the epilogue), lazy O rescale
//                   (only when a row max grows by more than 2^8; a stale max is
//                   exact after the final division), bf16 P into shared memory
//                   (swizzled K-major) once PV(i-1) has completed (it runs
//                   right after S(i), so the wait is normally over already).
//
// TMEM columns: S buffers [0, 128) and [128, 256), O [256, 384), Q as bf16
// pairs [384, 448).  Every wait
// is bounded; on a timeout the CTA raises CX_DEV_WAIT_TIMEOUT, drains its own
// copies and MMAs, frees its TMEM and returns.  tcgen05.ld / tcgen05.st are
// warp-collective, so every branch around them is decided warp-uniformly.
#pragma once
#include "attn_prefill_tc.cuh"

namespace cx {

constexpr int kT128Keys = 128;   // keys per key tile (S: N, PV: K)

// Block ids outside the pool.  The producers load block 0 in place of such an
// id, so the softmax leaves the block's keys out (probability 0; block 0's
// data is finite, so the PV product adds exactly 0).  Each softmax warp scans
// the sequence's ids once before its key loop (tc_seq_has_bad); only when one
// is bad does it look up each tile's 8 ids (tc_bad_mask: bit k for block k of
// the tile).  The kernels instantiate their key loop with and without the
// masking: masking code in the one shared loop changed how the whole softmax
// was compiled (146 instead of 168 registers) and cost the prefill 14 %
// (820 -> 705 TFLOP/s at head_dim 128), even with no bad id present.
__device__ __forceinline__ bool tc_seq_has_bad(const int32_t* tab, int kb0, int nblk_seq,
                                               int n_blocks, int lane) {
    bool bad = false;
#pragma unroll 4
    for (int blk = kb0 + lane; blk < nblk_seq; blk += 32) {
        const int id = tab[blk];
        bad |= id < 0 || id >= n_blocks;
    }
    return __any_sync(0xffffffffu, bad);
}

__device__ __forceinline__ unsigned tc_bad_mask(const int32_t* tab, int kb0, int ti, int nblk_seq,
                                                int n_blocks, int lane) {
    const int blk = kb0 + ti * (kT128Keys / kBlockTok) + lane;
    const int id = (lane < kT128Keys / kBlockTok && blk < nblk_seq) ? tab[blk] : 0;
    return __ballot_sync(0xffffffffu, id < 0 || id >= n_blocks) & 0xffu;
}
constexpr int kT128Slots = 5;    // ring slots, one K or V tile each

// Ring item q (the order the MMA thread reads them: K(0), K(1), V(0), K(2),
// V(1), K(3), ..., V(n-2), V(n-1)) -> V or K, key tile i.
__device__ __forceinline__ void t128_item(int q, int n, bool& is_v, int& i) {
    if (n == 1) {
        is_v = q == 1;
        i = 0;
    } else if (q < 2) {
        is_v = false;
        i = q;
    } else if (q - 2 < 2 * (n - 2)) {
        const int r = q - 2;
        is_v = (r & 1) == 0;
        i = is_v ? r >> 1 : (r >> 1) + 2;
    } else {
        is_v = true;
        i = n - 2 + (q - 2 - 2 * (n - 2));
    }
}

// TMA producer of the 128-key kernels (run by each of NPROD warps): ring items
// (K or V tiles of eight 16-token pool blocks, HALVES 128-byte swizzled 64-dim
// column halves each: 16 KB per half) in the order t128_item gives, key tile i + rot (mod
// n_tiles) for item tile i.  Producer pw loads blocks pw, pw + NPROD, ... of
// each item.  The warps decide together at named barrier 1 whether an item goes
// ahead, so an item is issued by all of them or by none and `s_issued` stays
// exact for the teardown drain.
template <int SLOTS, int NPROD, int HALVES>
__device__ __forceinline__ void t128_produce(const CUtensorMap* tmk, const CUtensorMap* tmv,
                                             const TcParams& p, int b, int h, int kb0,
                                             int nblk_seq, int n_tiles, int rot, int pw, int lane,
                                             unsigned char* ring, uint64_t* full, uint64_t* empty,
                                             volatile int* s_abort, volatile int* s_issued) {
    constexpr int BPT = kT128Keys / kBlockTok;              // 8 pool blocks per key tile
    constexpr int KV_HALF = kT128Keys * 128;                // one 64-dim half of a tile
    constexpr int SLOT = KV_HALF * HALVES;
    const int32_t* tab = p.tables + (int64_t)b * p.table_stride;
    const int first_id = kb0 < nblk_seq ? tab[kb0] : 0;
    int my_blocks = 0;
    for (int k = pw; k < BPT; k += NPROD) ++my_blocks;
    // block ids of four key tiles, one per lane, for the K and the V stream
    int ids_k = 0, ids_v = 0;
    for (int q = 0; q < 2 * n_tiles; ++q) {
        bool is_v;
        int i;
        t128_item(q, n_tiles, is_v, i);
        i += rot;                                           // key tile actually read
        if (i >= n_tiles) i -= n_tiles;
        if ((i * BPT) % 32 == 0 || q < 2 || (is_v && q < 4)) {
            // first tile of a stream, or a new group of four tiles
            const int blk = kb0 + (i & ~3) * BPT + lane;
            int id = blk < nblk_seq ? tab[blk] : first_id;
            if (id < 0 || id >= p.n_blocks) {
                raise_flag(CX_DEV_BAD_BLOCK);
                id = 0;
            }
            if (is_v) ids_v = id; else ids_k = id;
        }
        const int ids = is_v ? ids_v : ids_k;
        const int s = q % SLOTS;
        const int use = q / SLOTS;
        bool go = true;
        if (lane == 0 && use > 0 &&
            !mbar_wait_bounded(&empty[s], (use - 1) & 1, s_abort, kWaitLimitNs))
            go = false;
        go = __shfl_sync(0xffffffffu, go, 0) && !*s_abort;
        if (!bar_red_and(1, 32 * NPROD, go)) {
            if (lane == 0) {
                *s_abort = 1;
                raise_flag(CX_DEV_WAIT_TIMEOUT);
            }
            break;
        }
        if (lane == 0) mbar_arrive_expect_tx(&full[s], my_blocks * (SLOT / BPT));
        unsigned char* dst = ring + s * SLOT;
        for (int k = pw; k < BPT; k += NPROD) {
            const int id = __shfl_sync(0xffffffffu, ids, (i * BPT + k) & 31);
            if (lane == 0) {
                const int z = (p.layer * p.n_blocks + id) * p.hk + h;
#pragma unroll
                for (int hf = 0; hf < HALVES; ++hf)
                    tma_load_3d(dst + hf * KV_HALF + k * 2048, is_v ? tmv : tmk, &full[s],
                                hf * 64, 0, z);
            }
        }
        if (pw == 0 && lane == 0) *s_issued = q + 1;
    }
}

// tcgen05.mma with the A operand (M x 16, bf16 pairs per 32-bit column, row i
// in lane i) read from TMEM.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15])
        : "memory");
}

struct T128Cfg {
    static constexpr int D = 128;
    static constexpr int KV_HALF = kT128Keys * 128;         // 16 KB: 128 keys x 128 B
    static constexpr int SLOT = 2 * KV_HALF;                // one K or V tile
    static constexpr int P_HALF = kTcRows * 128;            // 64-key half of P
    static constexpr int P_BYTES = 2 * P_HALF;
    static constexpr int OFF_RING = 0;
    static constexpr int OFF_P = OFF_RING + kT128Slots * SLOT;
    static constexpr int OFF_BAR = OFF_P + P_BYTES;
    static constexpr int OFF_RED = OFF_BAR + 256;               // row-max exchange [2][2][128]
    static constexpr int SMEM = OFF_RED + 2 * 2 * kTcRows * 4 + 1024;   // + alignment slack
    static constexpr int TMEM_COLS = 512;                       // 448 used
    static constexpr int TM_O = 2 * kT128Keys;                  // O columns
    static constexpr int TM_Q = TM_O + D;                       // Q columns (bf16 pairs)
    static constexpr int N_PRODUCERS = 3;
    static constexpr int THREADS = 384;                 // softmax x 8, producers x 3, MMA
    static constexpr int PRODUCER_WARP = 8;             // first producer warp
    static constexpr int MMA_WARP = 11;
};
static_assert(T128Cfg::SMEM <= 232448, "shared memory above the per-CTA limit");

template <typename QT>
__global__ void __launch_bounds__(T128Cfg::THREADS, 1)
    paged_attn_tc128_kernel(const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv, const TcParams p) {
    using C = T128Cfg;
    constexpr int D = C::D;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* ring = sm + C::OFF_RING;
    unsigned char* sp = sm + C::OFF_P;
    float* s_red = reinterpret_cast<float*>(sm + C::OFF_RED);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
    uint64_t* full = bars;                     // [kT128Slots] slot loaded
    uint64_t* empty = bars + kT128Slots;       // [kT128Slots] slot read by its MMAs
    uint64_t* s_full = bars + 2 * kT128Slots;  // [2] S buffer ready in TMEM
    uint64_t* s_free = s_full + 2;             // [2] S buffer read into registers
    uint64_t* p_full = s_full + 4;             // P(i) written, O rescaled
    uint64_t* o_done = s_full + 5;             // PV(i) completed
    uint64_t* mma_drain = s_full + 6;          // last commit of the MMA thread
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_full + 7);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
    volatile int* s_issued = s_abort + 1;      // ring items whose TMA loads were issued

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = (int)(blockIdx.x / p.n_ctiles);
    const int ctile = p.n_ctiles - 1 - (int)(blockIdx.x % p.n_ctiles);  // longest first
    const int b = bh / p.hk, h = bh % p.hk;
    const int G = p.group, tpt = p.tpt;

    const int qs = p.q_start ? p.q_start[b] : b;
    const int T = p.q_start ? p.q_start[b + 1] - qs : 1;
    const int t0 = ctile * tpt;                // first token of the query tile
    if (t0 >= T) return;
    const int t_end = min(T, t0 + tpt);
    const int cap = (int)(p.table_stride * kBlockTok);
    const int ctx = min(max(p.ctx_lens[b], 0), cap);
    const int pos0 = ctx - T;                  // position of query token 0
    const int key_hi = min(pos0 + t_end - 1, ctx - 1);
    int key_lo = 0;
    if (p.window > 0) key_lo = max(0, pos0 + t0 - p.window + 1);
    const int kb0 = key_lo / kBlockTok;
    const int n_tiles = key_hi >= key_lo ? (key_hi - kb0 * kBlockTok) / kT128Keys + 1 : 0;
    const int nblk_seq = (ctx + kBlockTok - 1) / kBlockTok;
    // a negative scale is folded into Q, so the softmax always sees scale >= 0
    const bool neg = p.scale_log2 < 0.f;
    // Key tiles are visited from `rot` upwards, wrapping around (the online
    // softmax does not depend on the order): the query tiles of one (sequence,
    // KV head) run at the same time and read the same K/V, and starting them at
    // different tiles spreads their concurrent reads over different L2 lines.
    const int rot = n_tiles > 0 ? ctile % n_tiles : 0;

    // This thread's 64 Q values (row tid % 128, dims [64 c, 64 c + 64) for
    // warpgroup c) are loaded first, 16 bytes at a time, so their memory
    // latency overlaps the barrier set-up and the TMEM allocation.
    constexpr int QV = 64 * (int)sizeof(QT) / 16;          // 16-byte vectors per half row
    uint4 qv[QV];
    if (warp < 8) {
        const int r = tid & 127;
        const int t = t0 + r / G;
        const QT* src = static_cast<const QT*>(p.q) +
                        ((int64_t)(qs + t) * p.hq + h * G + r % G) * D + (warp >> 2) * 64;
        const bool ok = t < t_end;
        if ((reinterpret_cast<uintptr_t>(p.q) & 15) == 0) {
#pragma unroll
            for (int v = 0; v < QV; ++v)
                qv[v] = ok ? __ldg(reinterpret_cast<const uint4*>(src) + v) : make_uint4(0, 0, 0, 0);
        } else {
            // unaligned Q: element loads into the same vectors
#pragma unroll
            for (int v = 0; v < QV; ++v) {
                QT e[16 / sizeof(QT)];
#pragma unroll
                for (int k = 0; k < 16 / (int)sizeof(QT); ++k)
                    e[k] = ok ? src[v * (16 / sizeof(QT)) + k] : Conv<QT>::from_f(0.f);
                memcpy(&qv[v], e, 16);
            }
        }
    }

    if (tid == 0) {
        for (int s = 0; s < kT128Slots; ++s) {
            mbar_init(&full[s], C::N_PRODUCERS);
            mbar_init(&empty[s], 1);
        }
        for (int u = 0; u < 2; ++u) {
            mbar_init(&s_full[u], 1);
            mbar_init(&s_free[u], 256);
        }
        mbar_init(p_full, 256);
        mbar_init(o_done, 1);
        mbar_init(mma_drain, 1);
        *s_abort = 0;
        *s_issued = 0;
        fence_mbar_init();
    }
    if (warp == C::MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(s_tmem)),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    // Q tile -> TMEM as bf16 pairs (row r in lane r; rows past the chunk are
    // zero).  Only the MMA warp waits for it (named barrier 3): the producers
    // start loading K and V at once.
    if (warp < 8) {
        uint32_t wv[32];
        if constexpr (sizeof(QT) == 2) {
#pragma unroll
            for (int v = 0; v < QV; ++v) {
                wv[4 * v] = qv[v].x;
                wv[4 * v + 1] = qv[v].y;
                wv[4 * v + 2] = qv[v].z;
                wv[4 * v + 3] = qv[v].w;
            }
        } else {
#pragma unroll
            for (int v = 0; v < QV; ++v) {
                wv[2 * v] = pack_bf16(__uint_as_float(qv[v].x), __uint_as_float(qv[v].y));
                wv[2 * v + 1] = pack_bf16(__uint_as_float(qv[v].z), __uint_as_float(qv[v].w));
            }
        }
        if (neg) {
#pragma unroll
            for (int k = 0; k < 32; ++k) wv[k] ^= 0x80008000u;      // negate both halves
        }
        const uint32_t tm_q = tmem + C::TM_Q + (warp >> 2) * 32 + ((uint32_t)((warp & 3) * 32) << 16);
        tc_st16(tm_q, &wv[0]);
        tc_st16(tm_q + 16, &wv[16]);
        tc_wait_st();
        tc_fence_before();
        named_bar_arrive(3, 256 + 32);
    }

    if (warp >= C::PRODUCER_WARP && warp < C::PRODUCER_WARP + C::N_PRODUCERS) {
        t128_produce<kT128Slots, C::N_PRODUCERS, 2>(&tmk, &tmv, p, b, h, kb0, nblk_seq, n_tiles, rot,
                                                 warp - C::PRODUCER_WARP, lane, ring, full,
                                                 empty, s_abort, s_issued);
    } else if (warp == C::MMA_WARP) {
        // ---------------- MMA issuer ----------------
        named_bar_sync(3, 256 + 32);                   // Q is in TMEM
        tc_fence_after();
        if (lane == 0) {
            constexpr uint32_t idesc_s = tc_idesc(kTcRows, kT128Keys, 0);
            constexpr uint32_t idesc_o = tc_idesc(kTcRows, D, 1);
            const uint32_t p_base = smem_addr(sp);
            const uint32_t r_base = smem_addr(ring);
            bool ok = true;
            int q = 0;                                 // next ring item
            auto wait_item = [&]() {
                const bool r = mbar_wait_bounded(&full[q % kT128Slots], (q / kT128Slots) & 1,
                                                 s_abort, kWaitLimitNs);
                if (r) tc_fence_after();
                return r;
            };
            auto wait_bar = [&](uint64_t* bar, int parity) {
                const bool r = mbar_wait_bounded(bar, parity & 1, s_abort, kWaitLimitNs);
                if (r) tc_fence_after();
                return r;
            };
            // S(i) = Q K(i)^T into buffer i % 2: K = D in steps of 16 dims
            // (8 TMEM columns of Q per step)
            auto issue_s = [&](int i) {
                const uint32_t k_base = r_base + (q % kT128Slots) * C::SLOT;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    tc_mma_ts(tmem + (i & 1) * kT128Keys, tmem + C::TM_Q + kk * 8,
                              tc_sdesc(k_base + (kk >> 2) * C::KV_HALF + (kk & 3) * 32, 16, 1024),
                              idesc_s, kk > 0);
                tc_commit(&s_full[i & 1]);
                tc_commit(&empty[q % kT128Slots]);
                ++q;
            };
            // O += P(i) V(i): K = 128 keys in steps of 16; P K-major (64-key
            // halves P_HALF apart), V MN-major (64-dim halves KV_HALF apart,
            // 8-key groups 1 KB apart)
            auto issue_pv = [&](int i) {
                const uint32_t v_base = r_base + (q % kT128Slots) * C::SLOT;
#pragma unroll
                for (int kk = 0; kk < kT128Keys / 16; ++kk)
                    tc_mma(tmem + C::TM_O,
                           tc_sdesc(p_base + (kk >> 2) * C::P_HALF + (kk & 3) * 32, 16, 1024),
                           tc_sdesc(v_base + kk * 2048, C::KV_HALF, 1024), idesc_o,
                           (i > 0 || kk > 0) ? 1u : 0u);
                tc_commit(o_done);
                tc_commit(&empty[q % kT128Slots]);
                ++q;
            };
            // ring items are read in the order t128_item gives
            for (int i = 0; ok && i < 2 && i < n_tiles; ++i) {
                if (!(ok = wait_item())) break;
                issue_s(i);
            }
            for (int i = 0; ok && i < n_tiles; ++i) {
                if (!(ok = wait_item())) break;
                if (!(ok = wait_bar(p_full, i))) break;
                issue_pv(i);
                if (i + 2 < n_tiles) {
                    if (!(ok = wait_item())) break;
                    if (!(ok = wait_bar(&s_free[i & 1], i >> 1))) break;
                    issue_s(i + 2);
                }
            }
            if (!ok) {
                *s_abort = 1;
                raise_flag(CX_DEV_WAIT_TIMEOUT);
            }
            tc_commit(mma_drain);   // completes once every MMA issued above has
        }
    } else {
        // ---------------- softmax / correction / epilogue (warps 0-7) ----------------
        const int r = tid & 127, c = warp >> 2;          // row, key / output-column half
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tm_o = tmem + C::TM_O + c * 64 + lane_off;
        const int t = t0 + r / G;
        const int pos = pos0 + t;
        const int pos_lo = pos0 + t0, pos_hi = pos0 + max(t_end, t0 + 1) - 1;
        const int win = p.window;
        const float sl2 = fabsf(p.scale_log2);
        constexpr int HK = kT128Keys / 2;                // keys per half
        const int32_t* tab = p.tables + (int64_t)b * p.table_stride;
        const bool any_bad = tc_seq_has_bad(tab, kb0, nblk_seq, p.n_blocks, lane);
        float m = -INFINITY, l = 0.f;
        // `ok` turns false (warp-uniformly) when a bounded wait gives up; the
        // warp then skips its waits, TMEM and P work but keeps meeting the
        // named barrier of the two halves, so the other warps never wait forever.
        bool ok = true;
        // The key loop is instantiated twice: without bad-id masking (the
        // normal case, code identical to a kernel that has none) and with it.
        auto key_loop = [&](auto bad_tag) {
        constexpr bool BAD = decltype(bad_tag)::value;
        for (int i = 0; i < n_tiles; ++i) {
            const int u = i & 1;
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&s_full[u], (i >> 1) & 1,
                                                                  s_abort, kWaitLimitNs));
            float sv[HK];
            if (ok) {
                tc_fence_after();
                const uint32_t tm_s = tmem + u * kT128Keys + c * HK + lane_off;
                tc_ld32(tm_s, &sv[0]);
                tc_ld32(tm_s + 32, &sv[32]);
                tc_wait_ld();
            } else {
#pragma unroll
                for (int j = 0; j < HK; ++j) sv[j] = -INFINITY;
            }
            tc_fence_before();
            mbar_arrive(&s_free[u]);                   // S buffer u may be overwritten now
            const int ti = i + rot < n_tiles ? i + rot : i + rot - n_tiles;
            // bad block ids of this tile's half (4 blocks)
            const unsigned badh =
                BAD ? (tc_bad_mask(tab, kb0, ti, nblk_seq, p.n_blocks, lane) >> (c * 4)) & 0xfu
                    : 0u;
            const int kbase = kb0 * kBlockTok + ti * kT128Keys + c * HK;
            const bool edge = (kbase + HK - 1 > pos_lo) ||
                              (win > 0 && kbase <= pos_hi - win) || (kbase + HK > ctx) ||
                              (BAD && badh != 0);
            float mx[8];
#pragma unroll
            for (int a = 0; a < 8; ++a) mx[a] = -INFINITY;
            if (edge) {
#pragma unroll
                for (int j = 0; j < HK; ++j) {
                    const int key = kbase + j;
                    const bool keep = key <= pos && key < ctx && (win <= 0 || key > pos - win) &&
                                      (!BAD || !((badh >> (j >> 4)) & 1u));
                    sv[j] = keep ? sv[j] : -INFINITY;
                    mx[j & 7] = fmaxf(mx[j & 7], sv[j]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < HK; ++j) mx[j & 7] = fmaxf(mx[j & 7], sv[j]);
            }
            // row max over both halves: s_red[tile parity][half][row]
            float* red = s_red + u * 2 * kTcRows;
            red[c * kTcRows + r] = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                         fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            named_bar_sync(2, 256);
            const float mr = fmaxf(red[r], red[kTcRows + r]);
            // scaled row max of this tile; -inf when every key of the row is masked
            const float mt = mr == -INFINITY ? -INFINITY : mr * sl2;
            // lazy rescale: keep the reference max unless the row max grew by > 2^8
            const bool grow = mt > m + kTcRescaleLog2 || (m == -INFINITY && mt > -INFINITY);
            const float m_new = grow ? mt : m;
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = grow ? exp2f(m - m_use) : 1.f;
            float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (edge) {
#pragma unroll
                for (int j = 0; j < HK; ++j) {
                    const float e = sv[j] == -INFINITY ? 0.f : ex2_sfu(fmaf(sv[j], sl2, -m_use));
                    sv[j] = e;
                    ps[j & 7] += e;
                }
            } else {
#pragma unroll
                for (int j = 0; j < HK; ++j) {
                    sv[j] = ex2_sfu(fmaf(sv[j], sl2, -m_use));
                    ps[j & 7] += sv[j];
                }
            }
            l = l * alpha +
                (((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7])));
            m = m_new;
            // P and O are busy until PV(i-1) has completed
            if (i > 0 && ok) {
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(o_done, (i - 1) & 1, s_abort,
                                                                kWaitLimitNs));
                if (ok) tc_fence_after();
            }
            if (ok && i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                for (int q = 0; q < 2; ++q) {
                    float ov[32];
                    tc_ld32(tm_o + q * 32, ov);
                    tc_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] *= alpha;
                    tc_st32(tm_o + q * 32, ov);
                }
                tc_wait_st();
            }
            if (ok) {
#pragma unroll
                for (int q = 0; q < HK / 8; ++q) {
                    const uint4 v4 = make_uint4(pack_bf16(sv[q * 8 + 0], sv[q * 8 + 1]),
                                                pack_bf16(sv[q * 8 + 2], sv[q * 8 + 3]),
                                                pack_bf16(sv[q * 8 + 4], sv[q * 8 + 5]),
                                                pack_bf16(sv[q * 8 + 6], sv[q * 8 + 7]));
                    *reinterpret_cast<uint4*>(sp + tc_swz(r, c * HK + q * 8, kTcRows)) = v4;
                }
                fence_async_smem();
            }
            tc_fence_before();
            mbar_arrive(p_full);
        }
        };
        if (any_bad)
            key_loop(std::true_type{});
        else
            key_loop(std::false_type{});
        // epilogue: row sum over both halves, then this half's 64 output columns
        // (the buffer the last tile did not use: its last readers passed the
        // last exchange barrier before this write)
        float* lred = s_red + (n_tiles & 1) * 2 * kTcRows;
        lred[c * kTcRows + r] = l;
        named_bar_sync(2, 256);
        const float lt = lred[r] + lred[kTcRows + r];
        const bool row_ok = t < t_end;
        float* dst = p.out + ((int64_t)(qs + t) * p.hq + h * G + r % G) * D + c * 64;
        if (n_tiles == 0) {
            if (row_ok)
                for (int d = 0; d < 64; d += 4)
                    *reinterpret_cast<float4*>(dst + d) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else if (__all_sync(0xffffffffu,
                              ok && mbar_wait_bounded(o_done, (n_tiles - 1) & 1, s_abort,
                                                      kWaitLimitNs))) {
            tc_fence_after();
            const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll 1
            for (int q = 0; q < 2; ++q) {
                float ov[32];
                tc_ld32(tm_o + q * 32, ov);
                tc_wait_ld();
                if (row_ok) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(dst + q * 32 + e) =
                            make_float4(ov[e] * inv, ov[e + 1] * inv, ov[e + 2] * inv,
                                        ov[e + 3] * inv);
                }
            }
        } else {
            ok = false;
        }
        if (!ok) {
            *s_abort = 1;
            raise_flag(CX_DEV_WAIT_TIMEOUT);
        }
    }

    // ---- teardown: drain this CTA's own copies and MMAs, then free TMEM ----
    tc_fence_before();
    __syncthreads();
    if (*s_abort && tid == 0) {
        const int issued = *s_issued;
        for (int s = 0; s < kT128Slots; ++s) {
            const int uses = issued > s ? (issued - 1 - s) / kT128Slots + 1 : 0;
            if (uses > 0) mbar_wait_bounded(&full[s], (uses - 1) & 1, nullptr, kWaitLimitNs);
        }
    }
    if (tid == C::MMA_WARP * 32) mbar_wait_bounded(mma_drain, 0, nullptr, kWaitLimitNs);
    __syncthreads();
    tc_fence_after();
    if (warp == C::MMA_WARP)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(C::TMEM_COLS)
                     : "memory");
}

template <typename QT>
static int launch_tc128(const CUtensorMap& tk, const CUtensorMap& tv, const TcParams& p,
                        cudaStream_t st) {
    using C = T128Cfg;
    auto kern = paged_attn_tc128_kernel<QT>;
    CX_CUDA_CHECK(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    const int64_t grid = (int64_t)p.n_ctiles * p.batch * p.hk;
    if (grid <= 0) return CX_OK;
    if (grid > INT32_MAX) return fail(CX_ERR_UNSUPPORTED, "paged attention: grid too large");
    kern<<<(unsigned)grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);
    return check_launch("paged_attn_tc128_kernel");
}

}  // namespace cx
