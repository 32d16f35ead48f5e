// Paged flash-decode / multi-query verify over a bf16 pool with 16-token
// blocks and head_dim 64 or 128 (sm_100a).
//
// Work decomposition ("units"): one unit = one 16-token block of one KV head
// of one sequence.  All units of a call are laid out as
//     for b in sequences: for h in kv heads: for j in the sequence's blocks
// and split into equal contiguous chunks, one chunk per persistent CTA, so
// every SM streams the same number of bytes whatever the context-length mix.
// A chunk may start or end inside a (sequence, head) range; such a range is
// finished by whichever CTA arrives last at its counter (atomic ticket, no
// waiting), which merges the per-CTA partial softmax states from the
// workspace (log-sum-exp merge) and writes the final row.
//
// Inside a CTA: warp NCW is the producer.  Its lanes fetch 32 block ids of
// the table at a time; lane 0 issues, per unit, TMA tile loads (no multicast)
// of the 16 x D K tile and V tile into a STAGES-deep shared-memory ring,
// completing on a per-stage mbarrier.  The TMA writes the 128-byte swizzled
// layout, so the ldmatrix reads below are bank-conflict free.  Consumer
// warps are indexed (mt, ks): mt picks 16 packed query rows (row = query
// token * G + head-in-group), ks picks every KS-th unit.  Per unit a consumer
// computes S = Q K^T and O += P V with mma.sync m16n8k16 (bf16 in, fp32
// accumulate) and keeps the online softmax (running max m, denominator l,
// rescaled O) in registers, reducing row maxima across each lane quad with
// warp shuffles.  At the end of a (sequence, head) range the KS states are
// merged through shared memory.  Every wait is bounded (CX_DEV_WAIT_TIMEOUT).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "cx_common.cuh"  // unity build: included from cxkv.cu

namespace cx {

constexpr int kBlockTok = 16;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait
constexpr int kPlanMagic = 0x43584b56;                       // "CXKV"
constexpr int kMinUnitsPerCta = 8;

struct MmaParams {
    const int32_t* tables;
    int64_t table_stride;
    const int32_t* ctx_lens;
    const int32_t* q_start;  // NULL: decode, one query row per sequence
    int32_t batch, hk, hq, group, max_q, rows;
    int32_t n_blocks, layer, window;
    float scale_log2;
    const void* q;
    float* out;
    int32_t* plan;       // [16] header: W, chunk, P_eff, magic, batch, hk
    int32_t* seq_start;  // [batch + 1] first unit of each sequence
    int32_t* blk_lo;     // [batch] first block attended (sliding window)
    int32_t* counters;   // [batch * hk] merge tickets, zero between calls
    float* partials;     // [(P + batch*hk)][rows][D + 2]
};

// ---------------------------------------------------------------------------
// plan: unit prefix sums and the chunking (one CTA of 1024 threads)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) paged_plan_kernel(MmaParams p, int grid) {
    __shared__ long long s_part[1024];
    const int t = threadIdx.x, B = p.batch;
    const int per = (B + 1023) / 1024;
    const int b0 = t * per, b1 = min(B, b0 + per);
    long long local = 0;
    for (int b = b0; b < b1; ++b) {
        int ctx = p.ctx_lens[b];
        const int sq = p.q_start ? p.q_start[b + 1] - p.q_start[b] : 1;
        const long long cap = p.table_stride * (long long)kBlockTok;
        if (ctx < 0) ctx = 0;
        if (ctx > cap) {
            raise_flag(CX_DEV_TABLE_OVERRUN);
            ctx = (int)cap;
        }
        // an empty sequence (ctx == 0) is allowed and yields zero rows
        if (sq > p.max_q || sq < 0 || (ctx > 0 && sq > ctx)) raise_flag(CX_DEV_BAD_QLEN);
        int lo_tok = 0;
        if (p.window > 0) lo_tok = max(0, ctx - sq - p.window + 1);
        const int lo = lo_tok / kBlockTok;
        const int hi = (ctx + kBlockTok - 1) / kBlockTok;
        p.blk_lo[b] = lo;
        local += (ctx > 0 && hi > lo) ? (long long)(hi - lo) * p.hk : 0;
    }
    s_part[t] = local;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {  // Hillis-Steele inclusive scan
        long long v = t >= off ? s_part[t - off] : 0;
        __syncthreads();
        s_part[t] += v;
        __syncthreads();
    }
    long long run = s_part[t] - local;  // exclusive prefix
    for (int b = b0; b < b1; ++b) {
        p.seq_start[b] = (int)run;
        int ctx = min(max(p.ctx_lens[b], 0), (int)(p.table_stride * kBlockTok));
        const int hi = (ctx + kBlockTok - 1) / kBlockTok;
        run += (ctx > 0 && hi > p.blk_lo[b]) ? (long long)(hi - p.blk_lo[b]) * p.hk : 0;
    }
    for (int i = t; i < B * p.hk; i += 1024) p.counters[i] = 0;
    if (t == 1023) {
        long long W = s_part[1023];
        if (W > (1ll << 30)) {
            raise_flag(CX_DEV_TABLE_OVERRUN);
            W = 0;
        }
        p.seq_start[B] = (int)W;
        long long want = (W + kMinUnitsPerCta - 1) / kMinUnitsPerCta;
        long long pe = want < grid ? want : grid;
        if (pe < 1) pe = 1;
        const long long chunk = W > 0 ? (W + pe - 1) / pe : 1;
        p.plan[0] = (int)W;
        p.plan[1] = (int)chunk;
        p.plan[2] = W > 0 ? (int)((W + chunk - 1) / chunk) : 0;
        p.plan[4] = B;
        p.plan[5] = p.hk;
        __threadfence();
        p.plan[3] = kPlanMagic;
    }
}

// ---------------------------------------------------------------------------
// main kernel
// ---------------------------------------------------------------------------
struct Seg {
    int b, h, j0, cnt, nb;
    bool whole;
};

// Walks the (sequence, head) ranges covered by the CTA's unit interval.
struct SegCursor {
    int u, u_end, b, batch, hk;
    const int32_t* seq_start;
    const int32_t* blk_lo;
    __device__ void init(int u0, int u1, const MmaParams& p) {
        u = u0;
        u_end = u1;
        batch = p.batch;
        hk = p.hk;
        seq_start = p.seq_start;
        blk_lo = p.blk_lo;
        int lo = 0, hi = batch;  // largest b with seq_start[b] <= u0
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (seq_start[mid] <= u0) lo = mid; else hi = mid - 1;
        }
        b = lo;
    }
    __device__ bool next(Seg& s) {
        if (u >= u_end) return false;
        while (b < batch && seq_start[b + 1] <= u) ++b;
        if (b >= batch) return false;
        const int n_units = seq_start[b + 1] - seq_start[b];
        const int nb = n_units / hk;
        const int local = u - seq_start[b];
        s.b = b;
        s.h = local / nb;
        const int jo = local - s.h * nb;
        s.cnt = min(nb - jo, u_end - u);
        s.j0 = blk_lo[b] + jo;
        s.nb = nb;
        s.whole = (jo == 0 && s.cnt == nb);
        u += s.cnt;
        return true;
    }
};

template <int D>
__device__ __forceinline__ uint32_t swz(int t, int d) {
    // byte offset of (token t, dim d [multiple of 8]) in a TMA SWIZZLE_128B
    // tile made of D/64 boxes of 16 rows x 128 bytes
    return (uint32_t)((d >> 6) * (kBlockTok * 128) + t * 128 + ((((d & 63) >> 3) ^ (t & 7)) << 4));
}

template <typename QT> struct QLoad;
template <> struct QLoad<float> {
    __device__ __forceinline__ static float2 two(const float* q, int64_t i) {
        return *reinterpret_cast<const float2*>(q + i);
    }
};
template <> struct QLoad<__nv_bfloat16> {
    __device__ __forceinline__ static float2 two(const __nv_bfloat16* q, int64_t i) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(q + i));
    }
};

template <int D, int MT, int KS, int STAGES>
struct MmaCfg {
    static constexpr int NCW = MT * KS;             // consumer warps
    static constexpr int THREADS = (NCW + 1) * 32;  // + producer warp
    static constexpr int TILE = kBlockTok * D * 2;  // bytes of one K (or V) tile
    static constexpr int STAGE = 2 * TILE;
    static constexpr int NT = D / 8;    // n-tiles of the output
    static constexpr int KSTEP = D / 16;
    static size_t smem_bytes(int rows) {
        return 1024 + (size_t)STAGES * STAGE + 2 * STAGES * sizeof(uint64_t) +
               (size_t)KS * rows * (D + 2) * sizeof(float) + 64;
    }
};

template <int D, int MT, int KS, int STAGES, typename QT>
__global__ void __launch_bounds__(MmaCfg<D, MT, KS, STAGES>::THREADS, 1)
    paged_attn_mma_kernel(const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const MmaParams p) {
    using C = MmaCfg<D, MT, KS, STAGES>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* ring = smem;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(ring + STAGES * C::STAGE);
    uint64_t* empty_bar = full_bar + STAGES;
    float* merge = reinterpret_cast<float*>(empty_bar + STAGES);
    int* s_flags = reinterpret_cast<int*>(merge + KS * p.rows * (D + 2));
    volatile int* s_abort = s_flags;
    int* s_last = s_flags + 1;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int B = p.batch, Hq = p.hq, G = p.group;

    // The plan must come from paged_plan_kernel for this batch shape.
    if (p.plan[3] != kPlanMagic || p.plan[4] != B || p.plan[5] != p.hk) {
        if (tid == 0 && blockIdx.x == 0) raise_flag(CX_DEV_BAD_QLEN);
        return;
    }
    // Sequences with no cached token produce zero rows.
    for (int b = blockIdx.x; b < B; b += gridDim.x) {
        if (p.seq_start[b + 1] != p.seq_start[b]) continue;
        const int sq = p.q_start ? p.q_start[b + 1] - p.q_start[b] : 1;
        const int64_t r0 = p.q_start ? p.q_start[b] : b;
        for (int64_t e = tid; e < (int64_t)sq * Hq * D; e += blockDim.x)
            p.out[r0 * Hq * D + e] = 0.f;
    }
    const int W = p.plan[0], chunk = p.plan[1], P_eff = p.plan[2];
    if ((int)blockIdx.x >= P_eff) return;
    const int u0 = blockIdx.x * chunk;
    const int u1 = min(W, u0 + chunk);

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], MT);
        }
        s_flags[0] = 0;
        s_flags[1] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    SegCursor cur;
    cur.init(u0, u1, p);
    Seg seg;

    if (warp == C::NCW) {
        // ------------------------------ producer ------------------------------
        int i = 0, issued = 0;
        bool aborted = false;
        while (cur.next(seg)) {
            const int32_t* bt = p.tables + (int64_t)seg.b * p.table_stride;
            for (int k0 = 0; k0 < seg.cnt; k0 += 32) {
                const int n = min(32, seg.cnt - k0);
                int bid = -1;
                if (lane < n) {
                    const int jj = seg.j0 + k0 + lane;
                    bid = jj < p.table_stride ? bt[jj] : -1;
                    if (bid < 0 || bid >= p.n_blocks) {
                        raise_flag(CX_DEV_BAD_BLOCK);
                        bid = -1;
                    }
                }
                for (int k = 0; k < n; ++k, ++i) {
                    const int bk = __shfl_sync(0xffffffffu, bid, k);
                    if (lane == 0 && !aborted) {
                        const int s = i % STAGES;
                        const uint32_t par = ((i / STAGES) & 1) ^ 1;
                        if (!mbar_wait_bounded(&empty_bar[s], par, s_abort, kWaitLimitNs)) {
                            aborted = true;
                            *s_abort = 1;
                            raise_flag(CX_DEV_WAIT_TIMEOUT);
                        } else if (bk >= 0) {
                            mbar_arrive_expect_tx(&full_bar[s], C::STAGE);
                            const int z = (p.layer * p.n_blocks + bk) * p.hk + seg.h;
                            unsigned char* kd = ring + s * C::STAGE;
#pragma unroll
                            for (int bx = 0; bx < D / 64; ++bx) {
                                tma_load_3d(kd + bx * (kBlockTok * 128), &tmk, &full_bar[s], bx * 64, 0, z);
                                tma_load_3d(kd + C::TILE + bx * (kBlockTok * 128), &tmv, &full_bar[s],
                                            bx * 64, 0, z);
                            }
                        } else {
                            mbar_arrive(&full_bar[s]);  // bad id: release the slot, data unused
                        }
                        if (!aborted) ++issued;
                    }
                    __syncwarp();
                }
            }
        }
        // Do not leave the CTA with tile copies still landing in its smem.
        if (lane == 0) {
            const int first = issued > STAGES ? issued - STAGES : 0;
            for (int t = first; t < issued; ++t) {
                if (!mbar_wait_bounded(&full_bar[t % STAGES], (t / STAGES) & 1, nullptr,
                                       kWaitLimitNs)) {
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                    break;
                }
            }
        }
        return;
    }

    // ------------------------------- consumers -------------------------------
    const int mt = warp / KS, ks = warp % KS;
    const int NCT = C::NCW * 32;
    const int ctid = tid;  // consumer threads are 0..NCT-1
    // per-lane ldmatrix coordinates
    const int k_tok = (lane & 7) + 8 * (lane >> 4), k_dsub = 8 * ((lane >> 3) & 1);
    const int v_tok = (lane & 7) + 8 * ((lane >> 3) & 1), v_dsub = 8 * (lane >> 4);
    const int qr0 = lane >> 2, qc = 2 * (lane & 3);
    const int R0 = mt * 16 + qr0, R1 = R0 + 8;  // packed rows this lane owns
    const QT* qbase = static_cast<const QT*>(p.q);

    int ibase = 0;
    while (cur.next(seg)) {
        const int b = seg.b, h = seg.h;
        const int ctx = min(p.ctx_lens[b], (int)(p.table_stride * kBlockTok));
        const int sq = p.q_start ? p.q_start[b + 1] - p.q_start[b] : 1;
        const int64_t qs = p.q_start ? p.q_start[b] : b;
        const int rows_b = G * sq;
        const int pos0 = ctx - sq;  // position of query row 0
        const int rpos0 = R0 < rows_b ? pos0 + R0 / G : -1;
        const int rpos1 = R1 < rows_b ? pos0 + R1 / G : -1;

        // Q fragments (bf16, A operand of m16n8k16), zero for padding rows
        uint32_t qa[C::KSTEP][4];
#pragma unroll
        for (int kk = 0; kk < C::KSTEP; ++kk) {
            float2 a = make_float2(0.f, 0.f), bq = a, c = a, d = a;
            const int col = kk * 16 + qc;
            if (R0 < rows_b) {
                const int64_t row = ((qs + R0 / G) * Hq + (int64_t)h * G + R0 % G) * D;
                a = QLoad<QT>::two(qbase, row + col);
                c = QLoad<QT>::two(qbase, row + col + 8);
            }
            if (R1 < rows_b) {
                const int64_t row = ((qs + R1 / G) * Hq + (int64_t)h * G + R1 % G) * D;
                bq = QLoad<QT>::two(qbase, row + col);
                d = QLoad<QT>::two(qbase, row + col + 8);
            }
            qa[kk][0] = pack_bf16(a.x, a.y);
            qa[kk][1] = pack_bf16(bq.x, bq.y);
            qa[kk][2] = pack_bf16(c.x, c.y);
            qa[kk][3] = pack_bf16(d.x, d.y);
        }

        float o[C::NT][4];
#pragma unroll
        for (int n = 0; n < C::NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

        for (int k = ((ks - ibase) % KS + KS) % KS; k < seg.cnt; k += KS) {
            const int i = ibase + k;
            const int s = i % STAGES;
            bool ok = !*s_abort;
            if (ok) ok = mbar_wait_bounded(&full_bar[s], (i / STAGES) & 1, s_abort, kWaitLimitNs);
            // mma.sync / ldmatrix need the whole warp: agree on one outcome
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !*s_abort) {
                    *s_abort = 1;
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                }
            } else {
                const uint32_t kb = smem_addr(ring + s * C::STAGE);
                const uint32_t vb = kb + C::TILE;
                float sa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                float sb[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
                for (int kk = 0; kk < C::KSTEP; ++kk) {
                    uint32_t f[4];
                    ldmatrix_x4(f, kb + swz<D>(k_tok, kk * 16 + k_dsub));
                    if (kk & 1) {
                        mma_bf16_16816(sb[0], qa[kk], f[0], f[1]);
                        mma_bf16_16816(sb[1], qa[kk], f[2], f[3]);
                    } else {
                        mma_bf16_16816(sa[0], qa[kk], f[0], f[1]);
                        mma_bf16_16816(sa[1], qa[kk], f[2], f[3]);
                    }
                }
                float x[2][4];
#pragma unroll
                for (int n = 0; n < 2; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e) x[n][e] = (sa[n][e] + sb[n][e]) * p.scale_log2;
                const int j = seg.j0 + k;
                const int t0 = j * kBlockTok;
                const bool edge = (t0 + kBlockTok - 1 > pos0) ||
                                  (p.window > 0 && t0 <= ctx - 1 - p.window);
                if (edge) {
#pragma unroll
                    for (int n = 0; n < 2; ++n)
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int tok = t0 + n * 8 + qc + (e & 1);
                            const int rp = (e < 2) ? rpos0 : rpos1;
                            const bool ok_t = tok <= rp && (p.window <= 0 || tok > rp - p.window);
                            if (!ok_t) x[n][e] = -INFINITY;
                        }
                }
                float mx0 = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
                float mx1 = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
                const float base0 = mn0 == -INFINITY ? 0.f : mn0;
                const float base1 = mn1 == -INFINITY ? 0.f : mn1;
                const float a0 = exp2f(m0 - base0), a1 = exp2f(m1 - base1);
                float pr[2][4];
#pragma unroll
                for (int n = 0; n < 2; ++n) {
                    pr[n][0] = exp2f(x[n][0] - base0);
                    pr[n][1] = exp2f(x[n][1] - base0);
                    pr[n][2] = exp2f(x[n][2] - base1);
                    pr[n][3] = exp2f(x[n][3] - base1);
                }
                l0 = l0 * a0 + (pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1]);
                l1 = l1 * a1 + (pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3]);
                m0 = mn0;
                m1 = mn1;
#pragma unroll
                for (int n = 0; n < C::NT; ++n) {
                    o[n][0] *= a0;
                    o[n][1] *= a0;
                    o[n][2] *= a1;
                    o[n][3] *= a1;
                }
                uint32_t pa[4];
                pa[0] = pack_bf16(pr[0][0], pr[0][1]);
                pa[1] = pack_bf16(pr[0][2], pr[0][3]);
                pa[2] = pack_bf16(pr[1][0], pr[1][1]);
                pa[3] = pack_bf16(pr[1][2], pr[1][3]);
#pragma unroll
                for (int np = 0; np < C::KSTEP; ++np) {
                    uint32_t f[4];
                    ldmatrix_x4_trans(f, vb + swz<D>(v_tok, np * 16 + v_dsub));
                    mma_bf16_16816(o[2 * np], pa, f[0], f[1]);
                    mma_bf16_16816(o[2 * np + 1], pa, f[2], f[3]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[s]);
        }
        ibase += seg.cnt;

        // ---- merge the KS key slices of this (sequence, head) range ----
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        {
            float* mrow = merge + (size_t)ks * p.rows * (D + 2);
            if (R0 < rows_b) {
                float* r = mrow + (size_t)R0 * (D + 2);
#pragma unroll
                for (int n = 0; n < C::NT; ++n) {
                    r[n * 8 + qc] = o[n][0];
                    r[n * 8 + qc + 1] = o[n][1];
                }
                if ((lane & 3) == 0) {
                    r[D] = m0;
                    r[D + 1] = l0;
                }
            }
            if (R1 < rows_b) {
                float* r = mrow + (size_t)R1 * (D + 2);
#pragma unroll
                for (int n = 0; n < C::NT; ++n) {
                    r[n * 8 + qc] = o[n][2];
                    r[n * 8 + qc + 1] = o[n][3];
                }
                if ((lane & 3) == 0) {
                    r[D] = m1;
                    r[D + 1] = l1;
                }
            }
        }
        named_bar_sync(1, NCT);
        const int bh = b * p.hk + h;
        float* slot = p.partials + (size_t)(blockIdx.x + bh) * p.rows * (D + 2);
        for (int e = ctid; e < rows_b * D; e += NCT) {
            const int R = e / D, d = e - R * D;
            float M = -INFINITY;
#pragma unroll
            for (int s2 = 0; s2 < KS; ++s2)
                M = fmaxf(M, merge[((size_t)s2 * p.rows + R) * (D + 2) + D]);
            float L = 0.f, O = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int s2 = 0; s2 < KS; ++s2) {
                    const float* r = merge + ((size_t)s2 * p.rows + R) * (D + 2);
                    const float wgt = exp2f(r[D] - M);
                    L += r[D + 1] * wgt;
                    O += r[d] * wgt;
                }
            }
            if (seg.whole) {
                const int64_t orow = (qs + R / G) * Hq + (int64_t)h * G + R % G;
                p.out[orow * D + d] = L > 0.f ? O / L : 0.f;
            } else {
                slot[(size_t)R * (D + 2) + d] = O;
                if (d == 0) {
                    slot[(size_t)R * (D + 2) + D] = M;
                    slot[(size_t)R * (D + 2) + D + 1] = L;
                }
            }
        }
        if (!seg.whole) {
            __threadfence();
            named_bar_sync(1, NCT);
            if (ctid == 0) {
                const int first_u = p.seq_start[b] + h * seg.nb;
                const int pf = first_u / chunk, pl = (first_u + seg.nb - 1) / chunk;
                const int prev = atomicAdd(&p.counters[bh], 1);
                *s_last = (prev == pl - pf) ? (pf | (pl << 16)) + 1 : 0;
            }
            named_bar_sync(1, NCT);
            const int last = *s_last;
            if (last) {
                __threadfence();
                const int pf = (last - 1) & 0xffff, pl = (last - 1) >> 16;
                for (int e = ctid; e < rows_b * D; e += NCT) {
                    const int R = e / D, d = e - R * D;
                    float M = -INFINITY;
                    for (int pp = pf; pp <= pl; ++pp) {
                        const float* r = p.partials + (size_t)(pp + bh) * p.rows * (D + 2) +
                                         (size_t)R * (D + 2);
                        M = fmaxf(M, __ldcg(r + D));
                    }
                    float L = 0.f, O = 0.f;
                    if (M != -INFINITY) {
                        for (int pp = pf; pp <= pl; ++pp) {
                            const float* r = p.partials + (size_t)(pp + bh) * p.rows * (D + 2) +
                                             (size_t)R * (D + 2);
                            const float wgt = exp2f(__ldcg(r + D) - M);
                            L += __ldcg(r + D + 1) * wgt;
                            O += __ldcg(r + d) * wgt;
                        }
                    }
                    const int64_t orow = (qs + R / G) * Hq + (int64_t)h * G + R % G;
                    p.out[orow * D + d] = L > 0.f ? O / L : 0.f;
                }
                if (ctid == 0) p.counters[bh] = 0;
            }
        }
        named_bar_sync(1, NCT);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// 3-D view of a bf16 pool: (head_dim, 16 slots, layers*blocks*heads tiles),
// box 64 x 16 x 1 with 128-byte swizzle.
static int make_pool_tmap(CUtensorMap* m, void* base, const cx_pool* p) {
    auto enc = tmap_encoder();
    if (!enc) return fail(CX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[3] = {(cuuint64_t)p->head_dim, (cuuint64_t)p->block_size,
                                (cuuint64_t)(p->n_layers * p->n_blocks * p->n_kv_heads)};
    const cuuint64_t strides[2] = {(cuuint64_t)p->head_dim * 2,
                                   (cuuint64_t)(p->block_size * p->head_dim * 2)};
    const cuuint32_t box[3] = {64, (cuuint32_t)p->block_size, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CX_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    return CX_OK;
}

constexpr int kStages = 16;

struct WsLayout {
    size_t plan, seq, lo, cnt, part, total;
};

static int mt_for_rows(int64_t rows) { return (int)((rows + 15) / 16); }
static int ks_for_mt(int mt) { return mt == 1 ? 8 : (mt == 2 ? 4 : 2); }

static WsLayout ws_layout(int64_t batch, int64_t hk, int64_t rows, int64_t d, int64_t grid) {
    auto up = [](size_t x, size_t a) { return (x + a - 1) / a * a; };
    WsLayout w{};
    w.plan = 0;
    w.seq = 64;
    w.lo = up(w.seq + (batch + 1) * 4, 16);
    w.cnt = up(w.lo + batch * 4, 16);
    w.part = up(w.cnt + batch * hk * 4, 256);
    w.total = w.part + (size_t)(grid + batch * hk) * rows * (d + 2) * 4;
    return w;
}

template <int D, int MT, typename QT>
static int launch_mma_cfg(const CUtensorMap& tk, const CUtensorMap& tv, const MmaParams& p,
                          cudaStream_t st, int grid) {
    constexpr int KS = MT == 1 ? 8 : (MT == 2 ? 4 : 2);
    using C = MmaCfg<D, MT, KS, kStages>;
    auto kern = paged_attn_mma_kernel<D, MT, KS, kStages, QT>;
    const size_t smem = C::smem_bytes(p.rows);
    CX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, C::THREADS, smem, st>>>(tk, tv, p);
    return check_launch("paged_attn_mma_kernel");
}

template <int D, typename QT>
static int launch_mma_d(int mt, const CUtensorMap& tk, const CUtensorMap& tv, const MmaParams& p,
                        cudaStream_t st, int grid) {
    switch (mt) {
        case 1: return launch_mma_cfg<D, 1, QT>(tk, tv, p, st, grid);
        case 2: return launch_mma_cfg<D, 2, QT>(tk, tv, p, st, grid);
        case 3: return launch_mma_cfg<D, 3, QT>(tk, tv, p, st, grid);
        case 4: return launch_mma_cfg<D, 4, QT>(tk, tv, p, st, grid);
        default: return fail(CX_ERR_UNSUPPORTED, "paged attention: more than 64 packed rows");
    }
}

static bool mma_eligible(const cx_pool* pool, const cx_attn_batch* b, int32_t q_dtype) {
    const int64_t G = b->n_q_heads / pool->n_kv_heads;
    const int64_t rows = G * b->max_q_len;
    const int64_t tiles = pool->n_layers * pool->n_blocks * pool->n_kv_heads;
    const uintptr_t a = reinterpret_cast<uintptr_t>(pool->k) | reinterpret_cast<uintptr_t>(pool->v);
    return pool->dtype == CX_BF16 && pool->block_size == kBlockTok &&
           (pool->head_dim == 64 || pool->head_dim == 128) && rows >= 1 && rows <= 64 &&
           (q_dtype == CX_F32 || q_dtype == CX_BF16) && tiles < (1ll << 31) && (a & 15) == 0 &&
           b->batch < (1 << 24) && pool->n_kv_heads * b->batch < (1 << 24);
}

static int grid_size() { return num_sms(); }

static int paged_attention(const cx_pool* pool, int64_t layer, const cx_attn_batch* bt,
                           const void* q, int32_t q_dtype, float* out, void* ws,
                           size_t ws_bytes, int32_t replan, void* stream, bool verify) {
    int rc = check_pool(pool);
    if (rc) return rc;
    if (!bt) return fail(CX_ERR_SHAPE, "paged attention: batch is NULL");
    if (layer < 0 || layer >= pool->n_layers)
        return fail(CX_ERR_RANGE, "paged attention: layer out of range");
    if (bt->batch < 0 || bt->n_q_heads <= 0 || bt->n_q_heads % pool->n_kv_heads != 0)
        return fail(CX_ERR_SHAPE, "paged attention: n_q_heads must be a multiple of n_kv_heads");
    if (verify ? (bt->max_q_len < 1 || !bt->q_start) : bt->q_start != nullptr)
        return fail(CX_ERR_SHAPE, verify ? "cx_paged_verify: q_start and max_q_len >= 1 required"
                                         : "cx_paged_decode: q_start must be NULL");
    if (pool->head_dim > 256) return fail(CX_ERR_UNSUPPORTED, "paged attention: head_dim > 256");
    if (bt->batch == 0) return CX_OK;
    if (!bt->block_tables || !bt->ctx_lens || !q || !out || bt->table_stride <= 0)
        return fail(CX_ERR_SHAPE, "paged attention: NULL array or empty table");
    const int64_t max_q = verify ? bt->max_q_len : 1;
    const float scale =
        isnan(bt->scale) ? 1.0f / sqrtf((float)pool->head_dim) : bt->scale;
    cudaStream_t st = as_stream(stream);
    cx_attn_batch b = *bt;
    b.max_q_len = max_q;

    if (!mma_eligible(pool, &b, q_dtype)) {
        GenericParams g{};
        g.q = q;
        g.out = out;
        g.batch = b.batch;
        g.hq = b.n_q_heads;
        g.hk = pool->n_kv_heads;
        g.d = g.dv = pool->head_dim;
        g.max_q = max_q;
        g.scale = scale;
        g.mask_kind = 1;
        g.window = b.window;
        g.kp = pool->k;
        g.vp = pool->v;
        g.n_layers = pool->n_layers;
        g.n_blocks = pool->n_blocks;
        g.block_size = pool->block_size;
        g.layer = layer;
        g.tables = b.block_tables;
        g.table_stride = b.table_stride;
        g.ctx_lens = b.ctx_lens;
        g.q_start = b.q_start;
        return launch_generic<true>(q_dtype, pool->dtype, g, st);
    }

    const int64_t G = b.n_q_heads / pool->n_kv_heads;
    const int64_t rows = G * max_q;
    const int grid = grid_size();
    const WsLayout wl = ws_layout(b.batch, pool->n_kv_heads, rows, pool->head_dim, grid);
    if (!ws || ws_bytes < wl.total)
        return fail(CX_ERR_WORKSPACE, "paged attention: workspace missing or too small");
    if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
        return fail(CX_ERR_WORKSPACE, "paged attention: workspace must be 256-byte aligned");
    if (b.window > (1ll << 30) || b.table_stride > (1ll << 26))
        return fail(CX_ERR_UNSUPPORTED, "paged attention: window or table too large");

    char* w = static_cast<char*>(ws);
    MmaParams p{};
    p.tables = b.block_tables;
    p.table_stride = b.table_stride;
    p.ctx_lens = b.ctx_lens;
    p.q_start = b.q_start;
    p.batch = (int)b.batch;
    p.hk = (int)pool->n_kv_heads;
    p.hq = (int)b.n_q_heads;
    p.group = (int)G;
    p.max_q = (int)max_q;
    p.rows = (int)rows;
    p.n_blocks = (int)pool->n_blocks;
    p.layer = (int)layer;
    p.window = b.window > 0 ? (int)b.window : 0;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.q = q;
    p.out = out;
    p.plan = reinterpret_cast<int32_t*>(w + wl.plan);
    p.seq_start = reinterpret_cast<int32_t*>(w + wl.seq);
    p.blk_lo = reinterpret_cast<int32_t*>(w + wl.lo);
    p.counters = reinterpret_cast<int32_t*>(w + wl.cnt);
    p.partials = reinterpret_cast<float*>(w + wl.part);

    if (replan) {
        paged_plan_kernel<<<1, 1024, 0, st>>>(p, grid);
        rc = check_launch("paged_plan_kernel");
        if (rc) return rc;
    }
    CUtensorMap tk, tv;
    rc = make_pool_tmap(&tk, pool->k, pool);
    if (rc) return rc;
    rc = make_pool_tmap(&tv, pool->v, pool);
    if (rc) return rc;
    const int mt = mt_for_rows(rows);
    if (pool->head_dim == 128)
        return q_dtype == CX_F32 ? launch_mma_d<128, float>(mt, tk, tv, p, st, grid)
                                 : launch_mma_d<128, __nv_bfloat16>(mt, tk, tv, p, st, grid);
    return q_dtype == CX_F32 ? launch_mma_d<64, float>(mt, tk, tv, p, st, grid)
                             : launch_mma_d<64, __nv_bfloat16>(mt, tk, tv, p, st, grid);
}

}  // namespace cx

extern "C" {

size_t cx_paged_workspace_bytes(const cx_pool* pool, const cx_attn_batch* b) {
    using namespace cx;
    if (!pool || !b || pool->n_kv_heads <= 0 || b->n_q_heads <= 0 || b->batch < 0) return 0;
    const int64_t G = b->n_q_heads / pool->n_kv_heads;
    const int64_t max_q = b->q_start ? (b->max_q_len > 0 ? b->max_q_len : 1) : 1;
    return ws_layout(b->batch, pool->n_kv_heads, G * max_q, pool->head_dim, grid_size()).total;
}

int cx_paged_decode(const cx_pool* pool, int64_t layer, const cx_attn_batch* batch, const void* q,
                    int32_t q_dtype, float* out, void* workspace, size_t workspace_bytes,
                    int32_t replan, void* stream) {
    return cx::paged_attention(pool, layer, batch, q, q_dtype, out, workspace, workspace_bytes,
                               replan, stream, false);
}

int cx_paged_verify(const cx_pool* pool, int64_t layer, const cx_attn_batch* batch, const void* q,
                    int32_t q_dtype, float* out, void* workspace, size_t workspace_bytes,
                    int32_t replan, void* stream) {
    return cx::paged_attention(pool, layer, batch, q, q_dtype, out, workspace, workspace_bytes,
                               replan, stream, true);
}

}  // extern "C"
