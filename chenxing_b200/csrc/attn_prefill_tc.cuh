// Paged multi-query attention on the 5th-generation tensor cores (sm_100a):
// chunked prefill and long speculative-verify chains, used when the packed
// query tile reaches 64 rows (rows = query tokens x GQA group).
//
// One CTA owns (sequence b, KV head h, query tile): kTcRows = 128 packed rows,
// row r = (token t0 + r / G, query head h*G + r % G), so every row of the tile
// reads the same K/V head and the tile is a dense M = 128 operand.  Keys are
// walked in tiles of kTcKeys = 128 (eight 16-token pool blocks):
//
//   producer warp  : TMA loads of the eight blocks' K and V tiles (two
//                    128-byte column halves each, 128-byte swizzle) into a
//                    2-stage ring, completing on mbarriers;
//   MMA warp       : one elected thread issues S = Q K^T (tcgen05.mma,
//                    kind::f16, bf16 x bf16 -> fp32, M 128, N 128, K = D) into
//                    TMEM, then O += P V (K = 128 keys) into a second TMEM
//                    region, and signals completion with tcgen05.commit;
//   softmax warps  : 4 warps = 128 threads = the 128 TMEM lanes, so thread r
//                    owns row r: it reads its S row with tcgen05.ld, applies
//                    the causal / sliding-window mask, keeps the running max
//                    and denominator in registers (no shuffles: the whole row
//                    is in one thread), rescales its O row in TMEM when the
//                    max moves, and writes P (bf16) to shared memory in the
//                    swizzled K-major layout the next MMA reads.
//
// Q is staged once per CTA (bf16, same swizzled layout).  The epilogue reads
// O from TMEM, divides by the denominator and writes fp32 rows.  Every wait
// is bounded; on a timeout the CTA raises CX_DEV_WAIT_TIMEOUT, drains its own
// outstanding copies and MMAs, frees its TMEM and returns.
#pragma once
#include "cx_common.cuh"

namespace cx {

constexpr int kTcRows = 128;   // packed query rows per CTA (MMA M)
constexpr int kTcKeys = 128;   // keys per tile (S: N, PV: K)
constexpr int kTcStages = 2;

struct TcParams {
    const int32_t* tables;
    int64_t table_stride;
    const int32_t* ctx_lens;
    const int32_t* q_start;  // NULL: one query row per sequence
    int32_t batch, hk, hq, group, tpt, n_qtiles, n_blocks, layer, window;
    float scale_log2;
    const void* q;
    float* out;
};

template <int D>
struct TcCfg {
    static constexpr int HALVES = D / 64;                   // 128-byte column halves
    static constexpr int HALF_ROWS128 = 128 * 128;          // one half of a 128-row tile
    static constexpr int Q_BYTES = kTcRows * D * 2;
    static constexpr int KT_BYTES = kTcKeys * D * 2;        // one K (or V) tile
    static constexpr int STAGE = 2 * KT_BYTES;
    static constexpr int P_BYTES = kTcRows * kTcKeys * 2;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_KV = OFF_Q + Q_BYTES;
    static constexpr int OFF_P = OFF_KV + kTcStages * STAGE;
    static constexpr int OFF_BAR = OFF_P + P_BYTES;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;       // + 1 KB alignment slack
    // S uses columns [0, 128), O [128, 128 + D); the whole 512-column TMEM is
    // taken (one CTA per SM: shared memory allows no second one)
    static constexpr int TMEM_COLS = 512;
    static constexpr int THREADS = 192;                     // softmax x4, producer, MMA
    static constexpr int PRODUCER_WARP = 4;
    static constexpr int MMA_WARP = 5;
};

// ---- tcgen05 helpers ------------------------------------------------------
// Shared-memory matrix descriptor (tcgen05 format): start address, leading
// and stride byte offsets (16-byte units), descriptor version 1, 128-byte
// swizzle.  Operand tiles are 1024-byte aligned, so the base offset is 0.
__device__ __forceinline__ uint64_t tc_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B,
// A K-major, B K-major (b_mn = 0) or MN-major (b_mn = 1), shape M x N.
__host__ __device__ constexpr uint32_t tc_idesc(int m, int n, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_st32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Byte offset of element (row, col) of a K-major bf16 tile with 128 rows and
// 128-byte swizzle: column halves of 64 elements are separate 16 KB regions;
// inside one, row r is the 128-byte line r and its 16-byte chunk c sits at
// chunk c ^ (r & 7).
__device__ __forceinline__ uint32_t tc_swz(int row, int col) {
    return (uint32_t)((col >> 6) * (128 * 128) + row * 128 +
                      ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

template <int D, typename QT>
__global__ void __launch_bounds__(TcCfg<D>::THREADS, 1)
    paged_attn_tc_kernel(const __grid_constant__ CUtensorMap tmk,
                         const __grid_constant__ CUtensorMap tmv, const TcParams p) {
    using C = TcCfg<D>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sq = sm + C::OFF_Q;
    unsigned char* skv = sm + C::OFF_KV;
    unsigned char* sp = sm + C::OFF_P;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
    uint64_t* kv_full = bars;                 // [kTcStages]
    uint64_t* kv_empty = bars + kTcStages;    // [kTcStages]
    uint64_t* s_full = bars + 2 * kTcStages;
    uint64_t* p_full = s_full + 1;
    uint64_t* o_done = s_full + 2;
    uint64_t* mma_drain = s_full + 3;          // last commit of the MMA thread
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_full + 4);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
    volatile int* s_issued = s_abort + 1;      // key tiles whose TMA loads were issued
    volatile int* s_pv = s_abort + 2;          // key tiles whose P V was committed

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int BH = p.batch * p.hk;
    const int qtile = p.n_qtiles - 1 - (int)(blockIdx.x / BH);  // longest key ranges first
    const int rem = (int)(blockIdx.x % BH);
    const int b = rem / p.hk, h = rem % p.hk;
    const int G = p.group;

    const int qs = p.q_start ? p.q_start[b] : b;
    const int T = p.q_start ? p.q_start[b + 1] - qs : 1;
    const int t0 = qtile * p.tpt;
    if (t0 >= T) return;
    const int t1 = min(T, t0 + p.tpt);
    const int cap = (int)(p.table_stride * kBlockTok);
    const int ctx = min(max(p.ctx_lens[b], 0), cap);
    const int pos0 = ctx - T;                  // position of query token 0
    const int pos_lo = pos0 + t0, pos_hi = pos0 + t1 - 1;
    const int key_hi = min(pos_hi, ctx - 1);
    int key_lo = 0;
    if (p.window > 0) key_lo = max(0, pos_lo - p.window + 1);
    const int kb0 = key_lo / kBlockTok;
    const int n_tiles = key_hi >= key_lo ? (key_hi - kb0 * kBlockTok) / kTcKeys + 1 : 0;
    const int nblk_seq = (ctx + kBlockTok - 1) / kBlockTok;

    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(p_full, 128);
        mbar_init(o_done, 1);
        mbar_init(mma_drain, 1);
        *s_abort = 0;
        *s_issued = 0;
        *s_pv = 0;
        fence_mbar_init();
    }
    // TMEM: S in columns [0, 128), O in [128, 128 + D)
    if (warp == C::MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(s_tmem)),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Q tile -> shared memory (bf16, swizzled K-major), rows past the chunk zeroed
    if (warp < 4) {
        const int r = tid;
        const int t = t0 + r / G;
        const int head = h * G + r % G;
        const bool ok = t < t1;
        const QT* src = static_cast<const QT*>(p.q) + ((int64_t)(qs + t) * p.hq + head) * D;
#pragma unroll 4
        for (int c = 0; c < D / 8; ++c) {
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            if (ok) {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    w[e] = pack_bf16(Conv<QT>::to_f(src[c * 8 + 2 * e]),
                                     Conv<QT>::to_f(src[c * 8 + 2 * e + 1]));
            }
            *reinterpret_cast<uint4*>(sq + tc_swz(r, c * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    const uint32_t tm_s = tmem, tm_o = tmem + 128;

    if (warp == C::PRODUCER_WARP) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const int32_t* tab = p.tables + (int64_t)b * p.table_stride;
            const int first_id = kb0 < nblk_seq ? tab[kb0] : 0;
            for (int i = 0; i < n_tiles; ++i) {
                const int s = i % kTcStages;
                const int use = i / kTcStages;
                if (use > 0 && !mbar_wait_bounded(&kv_empty[s], (use - 1) & 1, s_abort,
                                                  kWaitLimitNs)) {
                    *s_abort = 1;
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                    break;
                }
                if (*s_abort) break;
                mbar_arrive_expect_tx(&kv_full[s], C::STAGE);
                unsigned char* kd = skv + s * C::STAGE;
                unsigned char* vd = kd + C::KT_BYTES;
#pragma unroll 1
                for (int j = 0; j < kTcKeys / kBlockTok; ++j) {
                    const int blk = kb0 + i * (kTcKeys / kBlockTok) + j;
                    int id = blk < nblk_seq ? tab[blk] : first_id;
                    if (id < 0 || id >= p.n_blocks) {
                        raise_flag(CX_DEV_BAD_BLOCK);
                        id = 0;
                    }
                    const int z = (p.layer * p.n_blocks + id) * p.hk + h;
#pragma unroll
                    for (int hf = 0; hf < C::HALVES; ++hf) {
                        tma_load_3d(kd + hf * C::HALF_ROWS128 + j * 2048, &tmk, &kv_full[s],
                                    hf * 64, 0, z);
                        tma_load_3d(vd + hf * C::HALF_ROWS128 + j * 2048, &tmv, &kv_full[s],
                                    hf * 64, 0, z);
                    }
                }
                *s_issued = i + 1;
            }
        }
    } else if (warp == C::MMA_WARP) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc_s = tc_idesc(kTcRows, kTcKeys, 0);
            constexpr uint32_t idesc_o = tc_idesc(kTcRows, D, 1);
            const uint32_t q_base = smem_addr(sq), p_base = smem_addr(sp);
            for (int i = 0; i < n_tiles; ++i) {
                const int s = i % kTcStages;
                if (!mbar_wait_bounded(&kv_full[s], (i / kTcStages) & 1, s_abort,
                                       kWaitLimitNs)) {
                    *s_abort = 1;
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t k_base = smem_addr(skv + s * C::STAGE);
                const uint32_t v_base = k_base + C::KT_BYTES;
                // S = Q K^T : K = D in steps of 16 (32 bytes inside a 128-byte row)
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * C::HALF_ROWS128 + (kk & 3) * 32;
                    tc_mma(tm_s, tc_sdesc(q_base + off, 16, 1024),
                           tc_sdesc(k_base + off, 16, 1024), idesc_s, kk > 0);
                }
                tc_commit(s_full);
                if (!mbar_wait_bounded(p_full, i & 1, s_abort, kWaitLimitNs)) {
                    *s_abort = 1;
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                    break;
                }
                tc_fence_after();
                // O += P V : K = 128 keys in steps of 16 (P: K-major, V: MN-major,
                // 64-column halves of V 16 KB apart, 8-key groups 1 KB apart)
#pragma unroll
                for (int kk = 0; kk < kTcKeys / 16; ++kk) {
                    const uint32_t poff = (kk >> 2) * C::HALF_ROWS128 + (kk & 3) * 32;
                    tc_mma(tm_o, tc_sdesc(p_base + poff, 16, 1024),
                           tc_sdesc(v_base + kk * 2048, C::HALF_ROWS128, 1024), idesc_o,
                           (i > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(o_done);
                tc_commit(&kv_empty[s]);
                *s_pv = i + 1;
            }
            tc_commit(mma_drain);   // completes once every MMA issued above has
        }
    } else {
        // ---------------- softmax / correction / epilogue (warps 0-3) ----------------
        const int r = tid;                      // TMEM lane = packed row
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const int t = t0 + r / G;
        const int pos = pos0 + t;
        const int win = p.window;
        const float sl2 = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        // tcgen05.ld / tcgen05.st are warp-collective (.sync.aligned): every
        // branch around them below is decided warp-uniformly (__all_sync /
        // __any_sync), including the give-up paths of the bounded waits.
        for (int i = 0; i < n_tiles; ++i) {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(s_full, i & 1, s_abort,
                                                            kWaitLimitNs))) {
                *s_abort = 1;
                raise_flag(CX_DEV_WAIT_TIMEOUT);
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[kTcKeys];
#pragma unroll
            for (int c = 0; c < kTcKeys / 32; ++c)
                tc_ld32(tm_s + lane_off + c * 32, &sv[c * 32]);
            tc_wait_ld();
            const int kbase = kb0 * kBlockTok + i * kTcKeys;
            const bool edge = (kbase + kTcKeys - 1 > pos_lo) ||
                              (win > 0 && kbase <= pos_hi - win) || (kbase + kTcKeys > ctx);
            float mt = -INFINITY;
            if (edge) {
#pragma unroll
                for (int j = 0; j < kTcKeys; ++j) {
                    const int key = kbase + j;
                    const bool keep = key <= pos && key < ctx && (win <= 0 || key > pos - win);
                    sv[j] = keep ? sv[j] * sl2 : -INFINITY;
                    mt = fmaxf(mt, sv[j]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < kTcKeys; ++j) {
                    sv[j] *= sl2;
                    mt = fmaxf(mt, sv[j]);
                }
            }
            const float m_new = fmaxf(m, mt);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = exp2f(m - m_use);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < kTcKeys; ++j) {
                sv[j] = exp2f(sv[j] - m_use);
                sum += sv[j];
            }
            l = l * alpha + sum;
            m = m_new;
            if (i > 0) {
                // P and O are busy until the previous P V has completed
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(o_done, (i - 1) & 1, s_abort,
                                                                kWaitLimitNs))) {
                    *s_abort = 1;
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                    for (int c = 0; c < D / 32; ++c) {
                        float ov[32];
                        tc_ld32(tm_o + lane_off + c * 32, ov);
                        tc_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) ov[e] *= alpha;
                        tc_st32(tm_o + lane_off + c * 32, ov);
                    }
                    tc_wait_st();
                }
            }
#pragma unroll
            for (int c = 0; c < kTcKeys / 8; ++c) {
                const uint4 w = make_uint4(pack_bf16(sv[c * 8 + 0], sv[c * 8 + 1]),
                                           pack_bf16(sv[c * 8 + 2], sv[c * 8 + 3]),
                                           pack_bf16(sv[c * 8 + 4], sv[c * 8 + 5]),
                                           pack_bf16(sv[c * 8 + 6], sv[c * 8 + 7]));
                *reinterpret_cast<uint4*>(sp + tc_swz(r, c * 8)) = w;
            }
            fence_async_smem();
            tc_fence_before();
            mbar_arrive(p_full);
        }
        // epilogue
        const bool row_ok = t < t1;
        float* dst = p.out + ((int64_t)(qs + t) * p.hq + h * G + r % G) * D;
        if (n_tiles == 0) {
            if (row_ok)
                for (int d = 0; d < D; d += 4)
                    *reinterpret_cast<float4*>(dst + d) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else if (__all_sync(0xffffffffu,
                              ok && mbar_wait_bounded(o_done, (n_tiles - 1) & 1, s_abort,
                                                      kWaitLimitNs))) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                float ov[32];
                tc_ld32(tm_o + lane_off + c * 32, ov);
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
            *s_abort = 1;
            raise_flag(CX_DEV_WAIT_TIMEOUT);
        }
    }

    // ---- teardown: drain this CTA's own copies and MMAs, then free TMEM ----
    tc_fence_before();
    __syncthreads();
    if (*s_abort && tid == 0) {
        // wait (bounded) for the loads and MMAs this CTA issued
        const int issued = *s_issued, pv = *s_pv;
        for (int s = 0; s < kTcStages; ++s) {
            const int uses = issued > s ? (issued - 1 - s) / kTcStages + 1 : 0;
            if (uses > 0) mbar_wait_bounded(&kv_full[s], (uses - 1) & 1, nullptr, kWaitLimitNs);
        }
        (void)pv;
    }
    if (tid == C::MMA_WARP * 32) mbar_wait_bounded(mma_drain, 0, nullptr, kWaitLimitNs);
    __syncthreads();
    tc_fence_after();
    if (warp == C::MMA_WARP)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(C::TMEM_COLS)
                     : "memory");
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Same 3-D pool view as the decode kernel, box of one head: 64 x 16 x 1.
static bool tc_eligible(const cx_pool* pool, const cx_attn_batch* b, int32_t q_dtype) {
    const int64_t G = b->n_q_heads / pool->n_kv_heads;
    const int64_t rows = G * b->max_q_len;
    const int64_t tiles = pool->n_layers * pool->n_blocks * pool->n_kv_heads;
    const uintptr_t a = reinterpret_cast<uintptr_t>(pool->k) | reinterpret_cast<uintptr_t>(pool->v);
    return pool->dtype == CX_BF16 && pool->block_size == kBlockTok &&
           (pool->head_dim == 64 || pool->head_dim == 128) && rows >= 64 && G <= kTcRows &&
           kTcRows % G == 0 && (q_dtype == CX_F32 || q_dtype == CX_BF16) &&
           tiles < (1ll << 31) && (a & 15) == 0 && b->max_q_len < (1 << 24);
}

template <int D, typename QT>
static int launch_tc(const CUtensorMap& tk, const CUtensorMap& tv, const TcParams& p,
                     cudaStream_t st) {
    using C = TcCfg<D>;
    auto kern = paged_attn_tc_kernel<D, QT>;
    CX_CUDA_CHECK(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    const int64_t grid = (int64_t)p.n_qtiles * p.batch * p.hk;
    if (grid <= 0) return CX_OK;
    if (grid > INT32_MAX) return fail(CX_ERR_UNSUPPORTED, "paged attention: grid too large");
    kern<<<(unsigned)grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);
    return check_launch("paged_attn_tc_kernel");
}

}  // namespace cx
