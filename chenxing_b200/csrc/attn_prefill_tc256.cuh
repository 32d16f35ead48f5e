// Paged multi-query attention on tcgen05 for head_dim 64 or 128: two query
// tiles per CTA and 128-key tiles (chunked prefill and long verify chains; used when a
// sequence's packed query rows fill at least one 128-row tile).
//
// A K or V tile of 128 keys is read once for 256 query rows, half the load
// traffic per FLOP of a one-tile CTA: the per-SM TMA issue rate (about 100
// cycles per 2 KB box of the paged layout) is what bounds one tile per CTA.
// Every MMA runs at N = 128 (the tensor pipe's cost per kind::f16 MMA is about
// the same for any N up to 128).
//
// One CTA owns (sequence b, KV head h) and query tiles w = 0, 1 of kTcRows =
// 128 packed rows each (row r of tile w: token t0 + w * tpt + r / G, query head
// h * G + r % G).  Twelve warps:
//
//   producer warps : t128_produce, three warps, a 160 KB ring of K or V tiles
//                    (five slots of 32 KB at head_dim 128, ten of 16 KB at
//                    64) loaded in the order K(0), K(1), V(0), K(2), V(1), ...;
//   MMA warp       : one thread issues S_w(i) = Q_w K(i)^T into TMEM
//                    [128 w, 128 w + 128) and O_w += P_w(i) V(i) into TMEM
//                    [256 + D w, ...) with P_w read from TMEM, in the order
//                    PV_0(i), S_0(i+1), PV_1(i), S_1(i+1): while one tile's
//                    softmax runs, the tensor pipe works on the other tile;
//   warpgroup w    : softmax of query tile w, thread r owning row r (TMEM lane
//                    r), in two passes over its 128 S columns (row max, then
//                    exponentials) so no thread holds the whole row; bf16 P_w
//                    is written back over the first 64 columns of S_w (keys
//                    2c, 2c + 1 in column c: keys 0-63 only after S columns
//                    0-63 were read, keys 64-127 after the rest); lazy O
//                    rescale (only when a row max grows by more than 2^8; a
//                    stale max is exact after the final division); fp32 output
//                    rows in the epilogue.
//
// The MMAs of one thread complete in issue order, so S_w(i) being ready means
// PV_w(i-1) has read P_w(i-1) and finished accumulating O_w: the softmax needs
// no other wait before rescaling O_w or writing P_w(i), and S_w(i+1), issued
// after PV_w(i), never overwrites a P that is still to be read.
//
// Q_0, Q_1 live in shared memory (D / 4 KB each).  Every wait is
// bounded; on a timeout the CTA raises CX_DEV_WAIT_TIMEOUT, drains its own
// copies and MMAs, frees its TMEM and returns.  tcgen05.ld / tcgen05.st are
// warp-collective, so every branch around them is decided warp-uniformly.
#pragma once
#include "attn_prefill_tc128.cuh"

namespace cx {


// Ring position of K(j) and V(j) among n key tiles (the order t128_item gives).
__device__ __forceinline__ int t128_pos_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int t128_pos_v(int j, int n) {
    return n == 1 ? 1 : (j == n - 1 ? 2 * n - 1 : 2 * j + 2);
}

template <int D_>
struct T256Cfg {
    static constexpr int D = D_;
    static constexpr int HALVES = D / 64;                   // 128-byte column halves
    static constexpr int Q_HALF = kTcRows * 128;            // 16 KB: 128 rows x 128 B
    static constexpr int Q_BYTES = HALVES * Q_HALF;         // one query tile
    static constexpr int KV_HALF = kT128Keys * 128;         // 16 KB: 128 keys x 128 B
    static constexpr int SLOT = HALVES * KV_HALF;           // one K or V tile
    static constexpr int SLOTS = 160 * 1024 / SLOT;         // ring of 160 KB
    static constexpr int OFF_Q = 0;                         // Q_0, Q_1
    static constexpr int OFF_RING = OFF_Q + 2 * Q_BYTES;
    static constexpr int OFF_BAR = OFF_RING + SLOTS * SLOT;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;       // + 1 KB alignment slack
    // S_0 / P_0, S_1 / P_1, O_0, O_1 (256 + 2 D columns, allocated as 512)
    static constexpr int TMEM_COLS = 512;
    static constexpr int N_PRODUCERS = 3;
    static constexpr int THREADS = 384;                     // softmax 2 x 4, producers 3, MMA
    static constexpr int PRODUCER_WARP = 8;                 // first producer warp
    static constexpr int MMA_WARP = 11;
};
static_assert(T256Cfg<128>::SMEM <= 232448 && T256Cfg<64>::SMEM <= 232448,
              "shared memory above the per-CTA limit");
static_assert(T256Cfg<64>::SMEM > 232448 / 2, "one CTA per SM: its TMEM takes 512 columns");
static_assert(T256Cfg<128>::SLOTS == 5 && T256Cfg<64>::SLOTS == 10, "ring depth");

template <int DH, typename QT>
__global__ void __launch_bounds__(T256Cfg<DH>::THREADS, 1)
    paged_attn_tc256_kernel(const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv, const TcParams p) {
    using C = T256Cfg<DH>;
    constexpr int D = C::D;
    constexpr int kT256Slots = C::SLOTS;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sq = sm + C::OFF_Q;
    unsigned char* ring = sm + C::OFF_RING;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
    uint64_t* full = bars;                     // [kT256Slots] slot loaded
    uint64_t* empty = bars + kT256Slots;       // [kT256Slots] slot read by its MMAs
    uint64_t* s_full = bars + 2 * kT256Slots;  // [2] S_w ready in TMEM
    uint64_t* p_full = s_full + 4;             // [2] P_w written, O_w rescaled
    uint64_t* o_done = s_full + 6;             // [2] PV_w completed
    uint64_t* mma_drain = s_full + 8;          // last commit of the MMA thread
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_full + 9);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
    volatile int* s_issued = s_abort + 1;      // ring items whose TMA loads were issued

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = (int)(blockIdx.x / p.n_ctiles);
    const int ctile = p.n_ctiles - 1 - (int)(blockIdx.x % p.n_ctiles);  // longest first
    const int b = bh / p.hk, h = bh % p.hk;
    const int G = p.group, tpt = p.tpt;

    const int qs = p.q_start ? p.q_start[b] : b;
    const int T = p.q_start ? p.q_start[b + 1] - qs : 1;
    const int t0 = ctile * 2 * tpt;            // first token of query tile 0
    if (t0 >= T) return;
    const int nq = t0 + tpt < T ? 2 : 1;        // query tiles with valid rows
    const int t_end = min(T, t0 + nq * tpt);
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
    // key tiles are visited from `rot` upwards, wrapping around (the online
    // softmax does not depend on the order), to spread the concurrent reads of
    // the CTAs that share this (sequence, KV head)
    const int rot = n_tiles > 0 ? ctile % n_tiles : 0;

    if (tid == 0) {
        for (int s = 0; s < kT256Slots; ++s) {
            mbar_init(&full[s], C::N_PRODUCERS);
            mbar_init(&empty[s], 1);
        }
        for (int w = 0; w < 2; ++w) {
            mbar_init(&s_full[w], 1);
            mbar_init(&p_full[w], 128);
            mbar_init(&o_done[w], 1);
        }
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
    // Q tiles -> shared memory (bf16, swizzled K-major; rows past the chunk are
    // zero), 16-byte loads all in flight at once.  Only the MMA warp waits for
    // them (named barrier 3): the producers start loading K and V at once.
    if (warp < 8) {
        const int w = warp >> 2, r = tid & 127;
        const int t = t0 + w * tpt + r / G;
        const bool ok = t < t_end;
        const QT* src =
            static_cast<const QT*>(p.q) + ((int64_t)(qs + t) * p.hq + h * G + r % G) * D;
        unsigned char* qdst = sq + w * C::Q_BYTES;
        const bool vec = (reinterpret_cast<uintptr_t>(p.q) & 15) == 0;
        constexpr int EPV = 16 / (int)sizeof(QT);              // elements per 16-byte vector
        constexpr int NV = D * (int)sizeof(QT) / 16;
        uint4 raw[NV];
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            if (!ok) {
                raw[v] = make_uint4(0, 0, 0, 0);
            } else if (vec) {
                raw[v] = __ldg(reinterpret_cast<const uint4*>(src) + v);
            } else {
                QT e[EPV];
#pragma unroll
                for (int k = 0; k < EPV; ++k) e[k] = src[v * EPV + k];
                memcpy(&raw[v], e, 16);
            }
        }
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {                      // 8 dims per 16-byte chunk
            uint4 w4;
            if constexpr (sizeof(QT) == 2) {
                w4 = raw[c];
            } else {
                const uint4 a0 = raw[2 * c], a1 = raw[2 * c + 1];
                w4 = make_uint4(pack_bf16(__uint_as_float(a0.x), __uint_as_float(a0.y)),
                                pack_bf16(__uint_as_float(a0.z), __uint_as_float(a0.w)),
                                pack_bf16(__uint_as_float(a1.x), __uint_as_float(a1.y)),
                                pack_bf16(__uint_as_float(a1.z), __uint_as_float(a1.w)));
            }
            if (neg) {
                w4.x ^= 0x80008000u;                           // negate both bf16 halves
                w4.y ^= 0x80008000u;
                w4.z ^= 0x80008000u;
                w4.w ^= 0x80008000u;
            }
            *reinterpret_cast<uint4*>(qdst + tc_swz(r, c * 8, kTcRows)) = w4;
        }
        fence_async_smem();
        named_bar_arrive(3, 256 + 32);
    }

    if (warp >= C::PRODUCER_WARP && warp < C::PRODUCER_WARP + C::N_PRODUCERS) {
        t128_produce<kT256Slots, C::N_PRODUCERS, C::HALVES>(&tmk, &tmv, p, b, h, kb0, nblk_seq, n_tiles, rot,
                                                 warp - C::PRODUCER_WARP, lane, ring, full,
                                                 empty, s_abort, s_issued);
    } else if (warp == C::MMA_WARP) {
        // ---------------- MMA issuer ----------------
        named_bar_sync(3, 256 + 32);                   // Q_0, Q_1 are in shared memory
        if (lane == 0) {
            constexpr uint32_t idesc_s = tc_idesc(kTcRows, kT128Keys, 0);
            constexpr uint32_t idesc_o = tc_idesc(kTcRows, D, 1);
            const uint32_t q_base = smem_addr(sq);
            const uint32_t r_base = smem_addr(ring);
            bool ok = true;
            // wait for the ring item at position `pos`; returns its slot or -1
            auto wait_pos = [&](int pos) {
                const bool r = mbar_wait_bounded(&full[pos % kT256Slots],
                                                 (pos / kT256Slots) & 1, s_abort, kWaitLimitNs);
                if (r) tc_fence_after();
                return r ? pos % kT256Slots : -1;
            };
            auto wait_bar = [&](uint64_t* bar, int parity) {
                const bool r = mbar_wait_bounded(bar, parity & 1, s_abort, kWaitLimitNs);
                if (r) tc_fence_after();
                return r;
            };
            // S_w = Q_w K^T from the K tile in `slot`: K = D in steps of 16 dims
            auto issue_s = [&](int w, int slot) {
                const uint32_t k_base = r_base + slot * C::SLOT;
                const uint32_t qw = q_base + w * C::Q_BYTES;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    tc_mma(tmem + w * kT128Keys,
                           tc_sdesc(qw + (kk >> 2) * C::Q_HALF + (kk & 3) * 32, 16, 1024),
                           tc_sdesc(k_base + (kk >> 2) * C::KV_HALF + (kk & 3) * 32, 16, 1024),
                           idesc_s, kk > 0);
                tc_commit(&s_full[w]);
            };
            // O_w += P_w V from the V tile in `slot`: K = 128 keys in steps of 16;
            // P_w from TMEM (8 columns of bf16 pairs per step), V MN-major
            // (64-dim halves KV_HALF apart, 8-key groups 1 KB apart)
            auto issue_pv = [&](int w, int slot, bool acc) {
                const uint32_t v_base = r_base + slot * C::SLOT;
#pragma unroll
                for (int kk = 0; kk < kT128Keys / 16; ++kk)
                    tc_mma_ts(tmem + 2 * kT128Keys + w * D, tmem + w * kT128Keys + kk * 8,
                              tc_sdesc(v_base + kk * 2048, C::KV_HALF, 1024), idesc_o,
                              (acc || kk > 0) ? 1u : 0u);
                tc_commit(&o_done[w]);
            };
            if (n_tiles > 0) {
                const int ks = wait_pos(t128_pos_k(0));
                ok = ks >= 0;
                if (ok) {
                    issue_s(0, ks);
                    if (nq == 2) issue_s(1, ks);
                    tc_commit(&empty[ks]);
                }
            }
            for (int i = 0; ok && i < n_tiles; ++i) {
                const bool next = i + 1 < n_tiles;
                const int vs = wait_pos(t128_pos_v(i, n_tiles));
                ok = vs >= 0;
                if (!ok) break;
                int ks = 0;
                if (next) {
                    ks = wait_pos(t128_pos_k(i + 1));
                    ok = ks >= 0;
                    if (!ok) break;
                }
                for (int w = 0; ok && w < nq; ++w) {
                    if (!(ok = wait_bar(&p_full[w], i))) break;
                    issue_pv(w, vs, i > 0);
                    if (next) issue_s(w, ks);          // after PV_w(i) has been issued
                }
                if (!ok) break;
                tc_commit(&empty[vs]);
                if (next) tc_commit(&empty[ks]);
            }
            if (!ok) {
                *s_abort = 1;
                raise_flag(CX_DEV_WAIT_TIMEOUT);
            }
            tc_commit(mma_drain);   // completes once every MMA issued above has
        }
    } else if (warp < 4 * nq) {
        // ---------------- softmax / correction / epilogue (warpgroup w) ----------------
        const int w = warp >> 2, r = tid & 127;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tm_s = tmem + w * kT128Keys + lane_off;
        const uint32_t tm_o = tmem + 2 * kT128Keys + w * D + lane_off;
        const int tw0 = t0 + w * tpt;                            // first token of this tile
        const int tw1 = min(t_end, tw0 + tpt);
        const int t = tw0 + r / G;
        const int pos = pos0 + t;
        const int pos_lo = pos0 + tw0, pos_hi = pos0 + max(tw1, tw0 + 1) - 1;
        const int win = p.window;
        const float sl2 = fabsf(p.scale_log2);
        const int32_t* tab = p.tables + (int64_t)b * p.table_stride;
        const bool any_bad = tc_seq_has_bad(tab, kb0, nblk_seq, p.n_blocks, lane);
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        // The key loop is instantiated twice: without bad-id masking (the
        // normal case, code identical to a kernel that has none) and with it.
        auto key_loop = [&](auto bad_tag) {
        constexpr bool BAD = decltype(bad_tag)::value;
        for (int i = 0; i < n_tiles; ++i) {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[w], i & 1, s_abort,
                                                            kWaitLimitNs))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int ti = i + rot < n_tiles ? i + rot : i + rot - n_tiles;
            // bad block ids of this tile (8 blocks)
            const unsigned bad8 =
                BAD ? tc_bad_mask(tab, kb0, ti, nblk_seq, p.n_blocks, lane) : 0u;
            const int kbase = kb0 * kBlockTok + ti * kT128Keys;
            const bool edge = (kbase + kT128Keys - 1 > pos_lo) ||
                              (win > 0 && kbase <= pos_hi - win) || (kbase + kT128Keys > ctx) ||
                              (BAD && bad8 != 0);
            auto keep = [&](int key) {
                return key <= pos && key < ctx && (win <= 0 || key > pos - win) &&
                       (!BAD || !((bad8 >> ((key - kbase) >> 4)) & 1u));
            };
            // pass 1: row max over the 128 columns, 64 at a time
            float mx[8];
#pragma unroll
            for (int a = 0; a < 8; ++a) mx[a] = -INFINITY;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float v[64];
                tc_ld32(tm_s + hh * 64, &v[0]);
                tc_ld32(tm_s + hh * 64 + 32, &v[32]);
                tc_wait_ld();
                if (edge) {
#pragma unroll
                    for (int j = 0; j < 64; ++j)
                        mx[j & 7] = fmaxf(mx[j & 7], keep(kbase + hh * 64 + j) ? v[j] : -INFINITY);
                } else {
#pragma unroll
                    for (int j = 0; j < 64; ++j) mx[j & 7] = fmaxf(mx[j & 7], v[j]);
                }
            }
            const float mr = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                   fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            // scaled row max of this tile; -inf when every key of the row is masked
            const float mt = mr == -INFINITY ? -INFINITY : mr * sl2;
            // lazy rescale: keep the reference max unless the row max grew by > 2^8
            const bool grow = mt > m + kTcRescaleLog2 || (m == -INFINITY && mt > -INFINITY);
            const float m_new = grow ? mt : m;
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = grow ? exp2f(m - m_use) : 1.f;
            m = m_new;
            // O_w holds PV_w(0 .. i-1): S_w(i) was issued after PV_w(i-1)
            if (i > 0) {
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                    for (int c = 0; c < D / 32; ++c) {
                        float ov[32];
                        tc_ld32(tm_o + c * 32, ov);
                        tc_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) ov[e] *= alpha;
                        tc_st32(tm_o + c * 32, ov);
                    }
                    tc_wait_st();
                }
            }
            // pass 2: p = 2^(s * scale - m), 64 columns at a time, bf16 pairs
            // written back over S_w columns [32 hh, 32 hh + 32)
            float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float v[64];
                tc_ld32(tm_s + hh * 64, &v[0]);
                tc_ld32(tm_s + hh * 64 + 32, &v[32]);
                tc_wait_ld();
                if (edge) {
#pragma unroll
                    for (int j = 0; j < 64; ++j) {
                        const float e = keep(kbase + hh * 64 + j)
                                            ? ex2_sfu(fmaf(v[j], sl2, -m_use)) : 0.f;
                        v[j] = e;
                        ps[j & 7] += e;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 64; ++j) {
                        v[j] = ex2_sfu(fmaf(v[j], sl2, -m_use));
                        ps[j & 7] += v[j];
                    }
                }
                float pk[32];
#pragma unroll
                for (int c = 0; c < 32; ++c)
                    pk[c] = __uint_as_float(pack_bf16(v[2 * c], v[2 * c + 1]));
                tc_st32(tm_s + hh * 32, pk);
            }
            l = l * alpha +
                (((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7])));
            tc_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[w]);
        }
        };
        if (any_bad)
            key_loop(std::true_type{});
        else
            key_loop(std::false_type{});
        // epilogue
        const bool row_ok = t < tw1;
        float* dst = p.out + ((int64_t)(qs + t) * p.hq + h * G + r % G) * D;
        if (n_tiles == 0) {
            if (row_ok)
                for (int d = 0; d < D; d += 4)
                    *reinterpret_cast<float4*>(dst + d) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else if (__all_sync(0xffffffffu,
                              ok && mbar_wait_bounded(&o_done[w], (n_tiles - 1) & 1, s_abort,
                                                      kWaitLimitNs))) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                float ov[32];
                tc_ld32(tm_o + c * 32, ov);
                tc_wait_ld();
                if (row_ok) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(dst + c * 32 + e) =
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
        for (int s = 0; s < kT256Slots; ++s) {
            const int uses = issued > s ? (issued - 1 - s) / kT256Slots + 1 : 0;
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

template <int DH, typename QT>
static int launch_tc256(const CUtensorMap& tk, const CUtensorMap& tv, const TcParams& p,
                        cudaStream_t st) {
    using C = T256Cfg<DH>;
    auto kern = paged_attn_tc256_kernel<DH, QT>;
    CX_CUDA_CHECK(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    const int64_t grid = (int64_t)p.n_ctiles * p.batch * p.hk;
    if (grid <= 0) return CX_OK;
    if (grid > INT32_MAX) return fail(CX_ERR_UNSUPPORTED, "paged attention: grid too large");
    kern<<<(unsigned)grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);
    return check_launch("paged_attn_tc256_kernel");
}

}  // namespace cx
