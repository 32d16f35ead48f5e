// Paged multi-query attention on the 5th-generation tensor cores (sm_100a):
// chunked prefill and long speculative-verify chains, used when the packed
// query tile reaches 64 rows (rows = query tokens x GQA group).
//
// One CTA owns (sequence b, KV head h) and two query tiles of kTcRows = 128
// packed rows each; row r of tile w is (token t0 + w*tpt + r / G, query head
// h*G + r % G), so every row shares the K/V head and a tile is a dense
// M = 128 operand even for GQA.  Keys are walked in tiles of kTcKeys = 64
// (four 16-token pool blocks):
//
//   producer warps : TMA loads of the four blocks' K and V tiles (128-byte
//                    column halves, 128-byte swizzle) into a 4-stage ring,
//                    issued from three warps (one TMA instruction costs its
//                    issuing thread ~100 cycles, so one thread alone cannot
//                    keep up with the tensor pipe);
//   MMA warp       : one thread issues tcgen05.mma (kind::f16, bf16 x bf16 ->
//                    fp32) S_w = Q_w K^T into TMEM and O_w += P_w V into TMEM
//                    for both query tiles w = 0, 1: the next tile's scores
//                    S_w(i+1) as soon as warpgroup w has read S_w(i) into
//                    registers, PV_w(i) once P_w(i) is written, so the tensor
//                    pipe computes scores while the softmax runs;
//   grid           : the query tiles of one (sequence, KV head) are adjacent
//                    block indices (longest key range first), so the CTAs
//                    resident at a time share their K/V through L2;
//   softmax warps  : one warpgroup per query tile, 128 threads = the 128 TMEM
//                    lanes, thread r owning row r: tcgen05.ld of its S row,
//                    causal / sliding-window mask on edge tiles only, running
//                    max and denominator in registers (no shuffles), lazy O
//                    rescale in TMEM (only when a row max grows by more than
//                    2^8; a stale max is exact after the final division by
//                    the denominator), bf16 P into shared memory in the
//                    swizzled K-major layout the PV MMA reads.
//
// Q is staged once per CTA (bf16, same layout).  The epilogue reads O from
// TMEM, divides by the denominator and writes fp32 rows.  Every wait is
// bounded; on a timeout the CTA raises CX_DEV_WAIT_TIMEOUT, drains its own
// copies and MMAs, frees its TMEM and returns.  tcgen05.ld / tcgen05.st are
// warp-collective, so every branch around them is decided warp-uniformly.
#pragma once
#include "cx_common.cuh"

namespace cx {

constexpr int kTcRows = 128;    // packed query rows per query tile (MMA M)
constexpr int kTcKeys = 64;     // keys per key tile (S: N, PV: K)
constexpr int kTcStages = 4;
constexpr float kTcRescaleLog2 = 8.f;   // rescale O only when a row max grows by > 2^8

struct TcParams {
    const int32_t* tables;
    int64_t table_stride;
    const int32_t* ctx_lens;
    const int32_t* q_start;  // NULL: one query row per sequence
    int32_t batch, hk, hq, group, tpt, n_ctiles, n_blocks, layer, window;
    float scale_log2;
    const void* q;
    float* out;
};

template <int D>
struct TcCfg {
    static constexpr int HALVES = D / 64;                    // 128-byte column halves
    static constexpr int Q_HALF = kTcRows * 128;             // 16 KB: 128 rows x 128 B
    static constexpr int Q_BYTES = kTcRows * D * 2;
    static constexpr int KV_HALF = kTcKeys * 128;            // 8 KB: 64 keys x 128 B
    static constexpr int KT_BYTES = kTcKeys * D * 2;         // one K (or V) tile
    static constexpr int STAGE = 2 * KT_BYTES;
    static constexpr int P_BYTES = kTcRows * kTcKeys * 2;    // 16 KB
    static constexpr int OFF_Q = 0;                          // 2 query tiles
    static constexpr int OFF_KV = OFF_Q + 2 * Q_BYTES;
    static constexpr int OFF_P = OFF_KV + kTcStages * STAGE; // 2 P tiles
    static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;        // + 1 KB alignment slack
    // TMEM columns: S_0 [0, 64), S_1 [64, 128), O_0 [128, 128 + D),
    // O_1 [256, 256 + D); all 512 are taken (one CTA per SM by shared memory)
    static constexpr int TMEM_COLS = 512;
    static constexpr int N_PRODUCERS = 3;
    static constexpr int THREADS = 384;                      // 2 x 4 softmax, 3 producers, MMA
    static constexpr int PRODUCER_WARP = 8;                  // first producer warp
    static constexpr int MMA_WARP = 11;
};

// AND of `pred` over the `nthreads` threads that meet at named barrier `id`.
__device__ __forceinline__ bool bar_red_and(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %3, 0;\n\t"
        "bar.red.and.pred p, %1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(id), "r"(nthreads), "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

// 2^x as one special-function-unit instruction (ex2.approx.ftz: relative error
// about 2^-22, far below the bf16 rounding of P; 2^-inf = +0 and results below
// the normal range flush to 0, which is what masked keys need).
__device__ __forceinline__ float ex2_sfu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

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

// Byte offset of element (row, col) of a K-major bf16 operand tile with
// 128-byte swizzle: column halves of 64 elements are separate regions of
// `rows` 128-byte lines; inside one, row r is line r and its 16-byte chunk c
// sits at chunk c ^ (r & 7).
__device__ __forceinline__ uint32_t tc_swz(int row, int col, int rows) {
    return (uint32_t)((col >> 6) * (rows * 128) + row * 128 +
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
    uint64_t* kv_full = bars;                  // [kTcStages]
    uint64_t* kv_empty = bars + kTcStages;     // [kTcStages]
    uint64_t* s_full = bars + 2 * kTcStages;   // [2] S_w ready in TMEM
    uint64_t* p_full = s_full + 2;             // [2] P_w in smem, O_w rescaled
    uint64_t* o_done = s_full + 4;             // [2] PV_w completed
    uint64_t* s_free = s_full + 6;             // [2] S_w read into registers
    uint64_t* mma_drain = s_full + 8;          // last commit of the MMA thread
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_full + 9);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
    volatile int* s_issued = s_abort + 1;      // key tiles whose TMA loads were issued

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
    const int n_tiles = key_hi >= key_lo ? (key_hi - kb0 * kBlockTok) / kTcKeys + 1 : 0;
    const int nblk_seq = (ctx + kBlockTok - 1) / kBlockTok;

    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&kv_full[s], C::N_PRODUCERS);
            mbar_init(&kv_empty[s], 1);
        }
        for (int w = 0; w < 2; ++w) {
            mbar_init(&s_full[w], 1);
            mbar_init(&p_full[w], 128);
            mbar_init(&o_done[w], 1);
            mbar_init(&s_free[w], 128);
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
        const int head = h * G + r % G;
        const bool ok = t < t_end;
        const QT* src = static_cast<const QT*>(p.q) + ((int64_t)(qs + t) * p.hq + head) * D;
        unsigned char* qdst = sq + w * C::Q_BYTES;
        const bool vec = (reinterpret_cast<uintptr_t>(p.q) & 15) == 0;
        constexpr int EPV = 16 / (int)sizeof(QT);            // elements per 16-byte vector
        uint4 raw[D * (int)sizeof(QT) / 16];
#pragma unroll
        for (int v = 0; v < D * (int)sizeof(QT) / 16; ++v) {
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
            *reinterpret_cast<uint4*>(qdst + tc_swz(r, c * 8, kTcRows)) = w4;
        }
        fence_async_smem();
        named_bar_arrive(3, 256 + 32);
    }

    if (warp >= C::PRODUCER_WARP && warp < C::PRODUCER_WARP + C::N_PRODUCERS) {
        // ---------------- TMA producers ----------------
        // Producer pw issues the (block j, K or V) pairs pw, pw + 3, ... of each
        // stage.  The three warps decide together at a named barrier whether a
        // stage goes ahead, so a stage is issued by all of them or by none and
        // `s_issued` stays exact for the teardown drain.
        const int pw = warp - C::PRODUCER_WARP;
        constexpr int PAIRS = 2 * (kTcKeys / kBlockTok);       // (block, K or V) per stage
        constexpr int PAIR_BYTES = kBlockTok * D * 2;
        int my_pairs = 0;
        for (int q = pw; q < PAIRS; q += C::N_PRODUCERS) ++my_pairs;
        const int32_t* tab = p.tables + (int64_t)b * p.table_stride;
        const int first_id = kb0 < nblk_seq ? tab[kb0] : 0;
        int ids = 0;                                           // 32 block ids, one per lane
        for (int i = 0; i < n_tiles; ++i) {
            const int s = i % kTcStages;
            const int use = i / kTcStages;
            if ((i * (kTcKeys / kBlockTok)) % 32 == 0) {
                const int blk = kb0 + i * (kTcKeys / kBlockTok) + lane;
                ids = blk < nblk_seq ? tab[blk] : first_id;
                if (ids < 0 || ids >= p.n_blocks) {
                    raise_flag(CX_DEV_BAD_BLOCK);
                    ids = 0;
                }
            }
            bool go = true;
            if (lane == 0 && use > 0 &&
                !mbar_wait_bounded(&kv_empty[s], (use - 1) & 1, s_abort, kWaitLimitNs))
                go = false;
            go = __shfl_sync(0xffffffffu, go, 0) && !*s_abort;
            if (!bar_red_and(1, 32 * C::N_PRODUCERS, go)) {
                if (lane == 0) {
                    *s_abort = 1;
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                }
                break;
            }
            unsigned char* kd = skv + s * C::STAGE;
            if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], my_pairs * PAIR_BYTES);
            for (int q = pw; q < PAIRS; q += C::N_PRODUCERS) {
                const int j = q >> 1;                          // block of the stage
                const int id = __shfl_sync(0xffffffffu, ids,
                                           (i * (kTcKeys / kBlockTok) + j) & 31);
                if (lane == 0) {
                    const int z = (p.layer * p.n_blocks + id) * p.hk + h;
                    unsigned char* dst = kd + (q & 1) * C::KT_BYTES + j * 2048;
#pragma unroll
                    for (int hf = 0; hf < C::HALVES; ++hf)
                        tma_load_3d(dst + hf * C::KV_HALF, (q & 1) ? &tmv : &tmk, &kv_full[s],
                                    hf * 64, 0, z);
                }
            }
            if (pw == 0 && lane == 0) *s_issued = i + 1;
        }
    } else if (warp == C::MMA_WARP) {
        // ---------------- MMA issuer ----------------
        named_bar_sync(3, 256 + 32);                   // Q is in shared memory
        if (lane == 0) {
            constexpr uint32_t idesc_s = tc_idesc(kTcRows, kTcKeys, 0);
            constexpr uint32_t idesc_o = tc_idesc(kTcRows, D, 1);
            const uint32_t q_base = smem_addr(sq), p_base = smem_addr(sp);
            bool ok = true;
            // S_w(i) = Q_w K(i)^T : K = D in steps of 16 (32 bytes of a 128-byte line)
            auto issue_s = [&](int w, int i) {
                const uint32_t k_base = smem_addr(skv + (i % kTcStages) * C::STAGE);
                const uint32_t qw = q_base + w * C::Q_BYTES;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    tc_mma(tmem + w * kTcKeys,
                           tc_sdesc(qw + (kk >> 2) * C::Q_HALF + (kk & 3) * 32, 16, 1024),
                           tc_sdesc(k_base + (kk >> 2) * C::KV_HALF + (kk & 3) * 32, 16, 1024),
                           idesc_s, kk > 0);
                }
                tc_commit(&s_full[w]);
            };
            // O_w += P_w V(i) : K = 64 keys in steps of 16; P K-major, V MN-major
            // (64-column halves of V KV_HALF apart, 8-key groups 1 KB apart)
            auto issue_pv = [&](int w, int i) {
                const uint32_t v_base =
                    smem_addr(skv + (i % kTcStages) * C::STAGE) + C::KT_BYTES;
                const uint32_t pw = p_base + w * C::P_BYTES;
#pragma unroll
                for (int kk = 0; kk < kTcKeys / 16; ++kk) {
                    tc_mma(tmem + 128 + w * 128, tc_sdesc(pw + kk * 32, 16, 1024),
                           tc_sdesc(v_base + kk * 2048, C::KV_HALF, 1024), idesc_o,
                           (i > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(&o_done[w]);
            };
            auto wait_kv = [&](int i) {
                const bool r = mbar_wait_bounded(&kv_full[i % kTcStages],
                                                 (i / kTcStages) & 1, s_abort, kWaitLimitNs);
                if (r) tc_fence_after();
                return r;
            };
            auto wait_p = [&](int w, int i) {
                const bool r = mbar_wait_bounded(&p_full[w], i & 1, s_abort, kWaitLimitNs);
                if (r) tc_fence_after();
                return r;
            };
            auto wait_sfree = [&](int w, int i) {
                const bool r = mbar_wait_bounded(&s_free[w], i & 1, s_abort, kWaitLimitNs);
                if (r) tc_fence_after();
                return r;
            };
            // Order per key tile i: S_0(i+1), S_1(i+1) as soon as each softmax
            // warpgroup has read S(i) into registers, then PV_0(i), PV_1(i) as
            // soon as P(i) is written: the next scores are computed while the
            // softmax of this tile runs.
            if (n_tiles > 0) {
                ok = wait_kv(0);
                if (ok) {
                    issue_s(0, 0);
                    if (nq == 2) issue_s(1, 0);
                }
            }
            for (int i = 0; ok && i < n_tiles; ++i) {
                if (i + 1 < n_tiles) {
                    if (!(ok = wait_kv(i + 1))) break;
                    if (!(ok = wait_sfree(0, i))) break;
                    issue_s(0, i + 1);
                    if (nq == 2) {
                        if (!(ok = wait_sfree(1, i))) break;
                        issue_s(1, i + 1);
                    }
                }
                if (!(ok = wait_p(0, i))) break;
                issue_pv(0, i);
                if (nq == 2) {
                    if (!(ok = wait_p(1, i))) break;
                    issue_pv(1, i);
                }
                tc_commit(&kv_empty[i % kTcStages]);
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
        const uint32_t tm_s = tmem + w * kTcKeys + lane_off;
        const uint32_t tm_o = tmem + 128 + w * 128 + lane_off;
        unsigned char* pw = sp + w * C::P_BYTES;
        const int tw0 = t0 + w * tpt;                            // first token of this tile
        const int tw1 = min(t_end, tw0 + tpt);
        const int t = tw0 + r / G;
        const int pos = pos0 + t;
        const int pos_lo = pos0 + tw0, pos_hi = pos0 + max(tw1, tw0 + 1) - 1;
        const int win = p.window;
        const float sl2 = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int i = 0; i < n_tiles; ++i) {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[w], i & 1, s_abort,
                                                            kWaitLimitNs))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[kTcKeys];
            tc_ld32(tm_s, &sv[0]);
            tc_ld32(tm_s + 32, &sv[32]);
            tc_wait_ld();
            tc_fence_before();
            mbar_arrive(&s_free[w]);                   // S_w may be overwritten now
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
            // lazy rescale: keep the reference max unless the row max grew by > 2^8
            const bool grow = mt > m + kTcRescaleLog2 || (m == -INFINITY && mt > -INFINITY);
            const float m_new = grow ? mt : m;
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = grow ? exp2f(m - m_use) : 1.f;
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < kTcKeys; ++j) {
                sv[j] = ex2_sfu(sv[j] - m_use);
                sum += sv[j];
            }
            l = l * alpha + sum;
            m = m_new;
            if (i > 0) {
                // P_w and O_w are busy until the previous PV_w has completed
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
#pragma unroll
            for (int c = 0; c < kTcKeys / 8; ++c) {
                const uint4 v4 = make_uint4(pack_bf16(sv[c * 8 + 0], sv[c * 8 + 1]),
                                            pack_bf16(sv[c * 8 + 2], sv[c * 8 + 3]),
                                            pack_bf16(sv[c * 8 + 4], sv[c * 8 + 5]),
                                            pack_bf16(sv[c * 8 + 6], sv[c * 8 + 7]));
                *reinterpret_cast<uint4*>(pw + tc_swz(r, c * 8, kTcRows)) = v4;
            }
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
        for (int s = 0; s < kTcStages; ++s) {
            const int uses = issued > s ? (issued - 1 - s) / kTcStages + 1 : 0;
            if (uses > 0) mbar_wait_bounded(&kv_full[s], (uses - 1) & 1, nullptr, kWaitLimitNs);
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

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
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
    const int64_t grid = (int64_t)p.n_ctiles * p.batch * p.hk;
    if (grid <= 0) return CX_OK;
    if (grid > INT32_MAX) return fail(CX_ERR_UNSUPPORTED, "paged attention: grid too large");
    kern<<<(unsigned)grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);
    return check_launch("paged_attn_tc_kernel");
}

}  // namespace cx
