// Paged multi-query attention on tcgen05 for head_dim 128: two query tiles per
// CTA and 128-key tiles (chunked prefill and long verify chains; used when a
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
//   producer warps : t128_produce, three warps, a ring of three 32 KB slots
//                    holding K(0), K(1), V(0), K(2), V(1), ... ;
//   MMA warp       : one thread issues S_w(i) = Q_w K(i)^T into TMEM
//                    [128 w, 128 w + 128) and O_w += P_w(i) V(i) into TMEM
//                    [256 + 128 w, ...), in the order S_0(i+1), PV_0(i),
//                    S_1(i+1), PV_1(i): the next scores of a tile are computed
//                    while its softmax finishes and the other tile's runs;
//   warpgroup w    : softmax of query tile w, thread r owning row r (TMEM lane
//                    r), in two passes over its 128 S columns (row max, then
//                    exponentials) so no thread holds the whole row; S_w is
//                    released after the second pass's TMEM reads, bf16 P_w goes
//                    to shared memory (swizzled K-major) once PV_w(i-1) has
//                    completed; lazy O rescale (only when a row max grows by
//                    more than 2^8; a stale max is exact after the final
//                    division); fp32 output rows in the epilogue.
//
// Q_0, Q_1 and P_0, P_1 live in shared memory (32 KB each).  Every wait is
// bounded; on a timeout the CTA raises CX_DEV_WAIT_TIMEOUT, drains its own
// copies and MMAs, frees its TMEM and returns.  tcgen05.ld / tcgen05.st are
// warp-collective, so every branch around them is decided warp-uniformly.
#pragma once
#include "attn_prefill_tc128.cuh"

namespace cx {

constexpr int kT256Slots = 3;    // ring slots, one K or V tile each

struct T256Cfg {
    static constexpr int D = 128;
    static constexpr int Q_HALF = kTcRows * 128;            // 16 KB: 128 rows x 128 B
    static constexpr int Q_BYTES = 2 * Q_HALF;              // one query tile
    static constexpr int KV_HALF = kT128Keys * 128;         // 16 KB: 128 keys x 128 B
    static constexpr int SLOT = 2 * KV_HALF;                // one K or V tile
    static constexpr int P_HALF = kTcRows * 128;            // 64-key half of P
    static constexpr int P_BYTES = 2 * P_HALF;              // one P tile
    static constexpr int OFF_Q = 0;                         // Q_0, Q_1
    static constexpr int OFF_P = OFF_Q + 2 * Q_BYTES;       // P_0, P_1
    static constexpr int OFF_RING = OFF_P + 2 * P_BYTES;
    static constexpr int OFF_BAR = OFF_RING + kT256Slots * SLOT;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;       // + 1 KB alignment slack
    static constexpr int TMEM_COLS = 512;                   // S_0, S_1, O_0, O_1
    static constexpr int N_PRODUCERS = 3;
    static constexpr int THREADS = 384;                     // softmax 2 x 4, producers 3, MMA
    static constexpr int PRODUCER_WARP = 8;                 // first producer warp
    static constexpr int MMA_WARP = 11;
};
static_assert(T256Cfg::SMEM <= 232448, "shared memory above the per-CTA limit");

template <typename QT>
__global__ void __launch_bounds__(T256Cfg::THREADS, 1)
    paged_attn_tc256_kernel(const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv, const TcParams p) {
    using C = T256Cfg;
    constexpr int D = C::D;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sq = sm + C::OFF_Q;
    unsigned char* sp = sm + C::OFF_P;
    unsigned char* ring = sm + C::OFF_RING;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
    uint64_t* full = bars;                     // [kT256Slots] slot loaded
    uint64_t* empty = bars + kT256Slots;       // [kT256Slots] slot read by its MMAs
    uint64_t* s_full = bars + 2 * kT256Slots;  // [2] S_w ready in TMEM
    uint64_t* s_free = s_full + 2;             // [2] S_w read by its softmax
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
            mbar_init(&s_free[w], 128);
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
        t128_produce<kT256Slots, C::N_PRODUCERS>(&tmk, &tmv, p, b, h, kb0, nblk_seq, n_tiles, rot,
                                                 warp - C::PRODUCER_WARP, lane, ring, full,
                                                 empty, s_abort, s_issued);
    } else if (warp == C::MMA_WARP) {
        // ---------------- MMA issuer ----------------
        named_bar_sync(3, 256 + 32);                   // Q_0, Q_1 are in shared memory
        if (lane == 0) {
            constexpr uint32_t idesc_s = tc_idesc(kTcRows, kT128Keys, 0);
            constexpr uint32_t idesc_o = tc_idesc(kTcRows, D, 1);
            const uint32_t q_base = smem_addr(sq), p_base = smem_addr(sp);
            const uint32_t r_base = smem_addr(ring);
            bool ok = true;
            int q = 0;                                 // next ring item (t128_item order)
            auto wait_item = [&]() {
                const bool r = mbar_wait_bounded(&full[q % kT256Slots], (q / kT256Slots) & 1,
                                                 s_abort, kWaitLimitNs);
                if (r) tc_fence_after();
                return r;
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
            // P K-major (64-key halves P_HALF apart), V MN-major (64-dim halves
            // KV_HALF apart, 8-key groups 1 KB apart)
            auto issue_pv = [&](int w, int slot, bool acc) {
                const uint32_t v_base = r_base + slot * C::SLOT;
                const uint32_t pw = p_base + w * C::P_BYTES;
#pragma unroll
                for (int kk = 0; kk < kT128Keys / 16; ++kk)
                    tc_mma(tmem + 2 * kT128Keys + w * D,
                           tc_sdesc(pw + (kk >> 2) * C::P_HALF + (kk & 3) * 32, 16, 1024),
                           tc_sdesc(v_base + kk * 2048, C::KV_HALF, 1024), idesc_o,
                           (acc || kk > 0) ? 1u : 0u);
                tc_commit(&o_done[w]);
            };
            if (n_tiles > 0) {
                ok = wait_item();                      // K(0)
                if (ok) {
                    const int ks = q % kT256Slots;
                    ++q;
                    issue_s(0, ks);
                    if (nq == 2) issue_s(1, ks);
                    tc_commit(&empty[ks]);
                }
            }
            for (int i = 0; ok && i < n_tiles; ++i) {
                const bool next = i + 1 < n_tiles;
                int ks = 0;
                if (next) {                            // K(i+1) comes before V(i) in the ring
                    if (!(ok = wait_item())) break;
                    ks = q % kT256Slots;
                    ++q;
                }
                if (!(ok = wait_item())) break;        // V(i)
                const int vs = q % kT256Slots;
                ++q;
                for (int w = 0; ok && w < nq; ++w) {
                    if (next) {
                        if (!(ok = wait_bar(&s_free[w], i))) break;
                        issue_s(w, ks);
                    }
                    if (!(ok = wait_bar(&p_full[w], i))) break;
                    issue_pv(w, vs, i > 0);
                }
                if (!ok) break;
                if (next) tc_commit(&empty[ks]);
                tc_commit(&empty[vs]);
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
        unsigned char* pw = sp + w * C::P_BYTES;
        const int tw0 = t0 + w * tpt;                            // first token of this tile
        const int tw1 = min(t_end, tw0 + tpt);
        const int t = tw0 + r / G;
        const int pos = pos0 + t;
        const int pos_lo = pos0 + tw0, pos_hi = pos0 + max(tw1, tw0 + 1) - 1;
        const int win = p.window;
        const float sl2 = fabsf(p.scale_log2);
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int i = 0; i < n_tiles; ++i) {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[w], i & 1, s_abort,
                                                            kWaitLimitNs))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int ti = i + rot < n_tiles ? i + rot : i + rot - n_tiles;
            const int kbase = kb0 * kBlockTok + ti * kT128Keys;
            const bool edge = (kbase + kT128Keys - 1 > pos_lo) ||
                              (win > 0 && kbase <= pos_hi - win) || (kbase + kT128Keys > ctx);
            auto keep = [&](int key) {
                return key <= pos && key < ctx && (win <= 0 || key > pos - win);
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
            if (i > 0) {
                // P_w and O_w are busy until PV_w(i-1) has completed
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_done[w], (i - 1) & 1,
                                                                s_abort, kWaitLimitNs))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
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
            // pass 2: p = 2^(s * scale - m), 64 columns at a time, bf16 P row
            // into shared memory; S_w is released after the last TMEM read
            float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float v[64];
                tc_ld32(tm_s + hh * 64, &v[0]);
                tc_ld32(tm_s + hh * 64 + 32, &v[32]);
                tc_wait_ld();
                if (hh == 1) {
                    tc_fence_before();
                    mbar_arrive(&s_free[w]);           // S_w may be overwritten now
                }
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
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint4 v4 = make_uint4(pack_bf16(v[c * 8 + 0], v[c * 8 + 1]),
                                                pack_bf16(v[c * 8 + 2], v[c * 8 + 3]),
                                                pack_bf16(v[c * 8 + 4], v[c * 8 + 5]),
                                                pack_bf16(v[c * 8 + 6], v[c * 8 + 7]));
                    *reinterpret_cast<uint4*>(pw + tc_swz(r, hh * 64 + c * 8, kTcRows)) = v4;
                }
            }
            l = l * alpha +
                (((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7])));
            fence_async_smem();
            tc_fence_before();
            mbar_arrive(&p_full[w]);
        }
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

template <typename QT>
static int launch_tc256(const CUtensorMap& tk, const CUtensorMap& tv, const TcParams& p,
                        cudaStream_t st) {
    using C = T256Cfg;
    auto kern = paged_attn_tc256_kernel<QT>;
    CX_CUDA_CHECK(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    const int64_t grid = (int64_t)p.n_ctiles * p.batch * p.hk;
    if (grid <= 0) return CX_OK;
    if (grid > INT32_MAX) return fail(CX_ERR_UNSUPPORTED, "paged attention: grid too large");
    kern<<<(unsigned)grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);
    return check_launch("paged_attn_tc256_kernel");
}

}  // namespace cx
