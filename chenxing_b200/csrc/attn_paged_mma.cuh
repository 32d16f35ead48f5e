// Paged flash-decode / multi-query verify over a bf16 pool with 16-token
// blocks and head_dim 64 or 128 (sm_100a).
//
// Work decomposition ("units"): one unit = one 16-token block of a group of
// HG consecutive KV heads of one sequence.  Because the pool stores the
// heads of a block next to each other ([layer][block][head][16][D]), the K
// (and the V) data of a unit is one contiguous HG x 4 KB run, fetched by two
// TMA tile loads (the two 128-byte column halves, 128-byte swizzle).  All
// units of a call are laid out as
//     for b in sequences: for g in head groups: for j in the sequence's blocks
// and split into equal contiguous chunks, one per persistent CTA, so every SM
// streams the same number of bytes whatever the context-length mix.  A chunk
// may start or end inside a (sequence, head group) range; such a range is
// finished by whichever CTA arrives last at its counter (atomic ticket, no
// waiting), which merges the per-CTA partial softmax states from the
// workspace (log-sum-exp merge, one pass over the partials) and writes the
// final rows.
//
// Inside a CTA: the last warp is the producer.  Its lanes fetch 32 block ids
// of the table at a time; lane 0 issues the TMA loads (CTA-local destination) of each
// unit into a ring of shared-memory stages, completing on per-stage
// mbarriers.  Consumer warps are indexed (hh, mt, ks): head hh of the group,
// 16 packed query rows mt (row = query token * G + head-in-group), and key
// slice ks (every KS-th unit).  Per unit a consumer computes S = Q K^T and
// O += P V with mma.sync m16n8k16 (bf16 in, fp32 accumulate) and keeps the
// online softmax (running max m, denominator l, rescaled O) in registers,
// reducing row maxima across each lane quad with warp shuffles.  Where the
// registers allow (MmaCfg::U), a consumer takes two of its units per
// iteration for more independent MMAs between waits; at two row tiles, and at
// three row tiles of 4 heads (12 consumer warps), the Q fragments sit in
// per-lane shared-memory slots (MmaCfg::QSM) instead of registers.  Key slices
// (KS > 1) are merged through shared memory at the end of a range.  Every
// wait is bounded and reports CX_DEV_WAIT_TIMEOUT instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "cx_common.cuh"  // unity build: included from cxkv.cu

namespace cx {

constexpr int kBlockTok = 16;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait

// Limit of the decode / verify pipeline waits (default kWaitLimitNs).  A test
// shortens it (cx_set_wait_limit_ns) to make the waits run out on purpose and
// check that the kernel returns with CX_DEV_WAIT_TIMEOUT raised.
static std::atomic<unsigned long long> g_wait_limit_ns{kWaitLimitNs};
constexpr int kPlanMagic = 0x43584b56;                       // "CXKV"
constexpr int kMinUnitsPerCta = 4;
constexpr int kConsumerWarps = 8;
constexpr size_t kSmemBudget = 227 * 1024;

struct MmaParams {
    const int32_t* tables;
    int64_t table_stride;
    const int32_t* ctx_lens;
    const int32_t* q_start;  // NULL: decode, one query row per sequence
    int32_t batch, hk, hq, group, max_q, rows;
    int32_t hg, n_groups;    // heads per unit, head groups per sequence
    int32_t n_blocks, layer, window;
    int32_t stages, stage_bytes;
    float scale_log2;
    uint64_t wait_ns;    // limit of every pipeline wait (cx_set_wait_limit_ns)
    int32_t ks, mt;      // fp32 kernel: key slices and row tiles (runtime)
    int32_t q_bf16;      // fp32 kernel: q is bf16 (else fp32)
    const void* q;
    float* out;
    int32_t* plan;       // [16] header: W, chunk, P_eff, magic, batch, n_groups
    int32_t* seq_start;  // [batch + 1] first unit of each sequence
    int32_t* blk_lo;     // [batch] first block attended (sliding window)
    int32_t* counters;   // [batch * n_groups] merge tickets, zero between calls
    float* partials;     // [(P + batch*n_groups)][hg][rows][D + 2]
};

// ---------------------------------------------------------------------------
// plan: unit prefix sums and the chunking (one CTA of 1024 threads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int plan_units(const MmaParams& p, int b, int* lo_out) {
    int ctx = p.ctx_lens[b];
    const int sq = p.q_start ? p.q_start[b + 1] - p.q_start[b] : 1;
    const int cap = (int)(p.table_stride * kBlockTok);
    ctx = min(max(ctx, 0), cap);
    int lo_tok = 0;
    if (p.window > 0) lo_tok = max(0, ctx - sq - p.window + 1);
    const int lo = lo_tok / kBlockTok;
    const int hi = (ctx + kBlockTok - 1) / kBlockTok;
    *lo_out = lo;
    return (ctx > 0 && hi > lo) ? (hi - lo) : 0;
}

__global__ void __launch_bounds__(1024) paged_plan_kernel(MmaParams p, int grid) {
    __shared__ long long s_warp[32];
    __shared__ long long s_total;
    const int t = threadIdx.x, B = p.batch;
    const int lane = t & 31, wid = t >> 5;
    const int per = (B + 1023) / 1024;
    const int b0 = t * per, b1 = min(B, b0 + per);
    long long local = 0;
    for (int b = b0; b < b1; ++b) {
        const int ctx = p.ctx_lens[b];
        const int sq = p.q_start ? p.q_start[b + 1] - p.q_start[b] : 1;
        if (ctx > p.table_stride * kBlockTok) raise_flag(CX_DEV_TABLE_OVERRUN);
        // an empty sequence (ctx == 0) is allowed and yields zero rows
        if (sq > p.max_q || sq < 0 || (ctx > 0 && sq > ctx)) raise_flag(CX_DEV_BAD_QLEN);
        int lo;
        local += (long long)plan_units(p, b, &lo) * p.n_groups;
        p.blk_lo[b] = lo;
    }
    // block-wide exclusive scan of the per-thread unit counts: shuffle scans
    // within each warp, then over the 32 warp totals (two block barriers)
    long long inc = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const long long v = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += v;
    }
    if (lane == 31) s_warp[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        long long w = s_warp[lane];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const long long v = __shfl_up_sync(0xffffffffu, w, off);
            if (lane >= off) w += v;
        }
        s_warp[lane] = w - s_warp[lane];       // exclusive prefix of warp totals
        if (lane == 31) s_total = w;
    }
    __syncthreads();
    long long run = s_warp[wid] + inc - local;  // exclusive prefix of this thread
    for (int b = b0; b < b1; ++b) {
        p.seq_start[b] = (int)run;
        int lo;
        run += (long long)plan_units(p, b, &lo) * p.n_groups;
    }
    for (int i = t; i < B * p.n_groups; i += 1024) p.counters[i] = 0;
    if (t == 1023) {
        long long W = s_total;
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
        p.plan[5] = p.n_groups;
        __threadfence();
        p.plan[3] = kPlanMagic;
    }
}

// ---------------------------------------------------------------------------
// main kernel
// ---------------------------------------------------------------------------
struct Seg {
    int b, g, j0, cnt, nb;
    bool whole;
};

// Walks the (sequence, head group) ranges covered by the CTA's unit interval.
struct SegCursor {
    int u, u_end, b, batch, ng;
    const int32_t* seq_start;
    const int32_t* blk_lo;
    __device__ void init(int u0, int u1, const MmaParams& p) {
        u = u0;
        u_end = u1;
        batch = p.batch;
        ng = p.n_groups;
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
        const int nb = (seq_start[b + 1] - seq_start[b]) / ng;
        const int local = u - seq_start[b];
        s.b = b;
        s.g = local / nb;
        const int jo = local - s.g * nb;
        s.cnt = min(nb - jo, u_end - u);
        s.j0 = blk_lo[b] + jo;
        s.nb = nb;
        s.whole = (jo == 0 && s.cnt == nb);
        u += s.cnt;
        return true;
    }
};

// ---------------------------------------------------------------------------
// TMA producer (the last warp of a decode / verify CTA), shared by the bf16
// mma.sync kernel and the fp32 FMA kernel: for every unit of the CTA's chunk,
// in order, wait for its ring stage to be free, then load the unit's K and V
// (HG heads x 16 tokens x head_dim) as NBOX column boxes of 128 bytes each
// (BOX_COLS elements, 128-byte swizzle) with 3-D TMA tile loads into this
// CTA's own shared memory; a block id outside the pool loads nothing and
// marks the stage bad.  Lanes fetch 32 block ids of the table per load; lane
// 0 issues.  Every wait is bounded; after a give-up (own or a consumer's) no
// stage is re-armed, and before returning the producer waits for its own
// copies still in flight.
// ---------------------------------------------------------------------------
template <int NBOX, int BOX_COLS, int BOX_BYTES, int TILES, int STAGE>
__device__ __forceinline__ void produce_units(const CUtensorMap* tmk, const CUtensorMap* tmv,
                                              const MmaParams& p, SegCursor cur, int HG,
                                              unsigned char* ring, uint64_t* full_bar,
                                              uint64_t* empty_bar, volatile int* s_abort,
                                              volatile unsigned char* s_bad, int lane) {
    const int STAGES = p.stages;
    Seg seg;
    int i = 0, issued = 0;
    bool aborted = false;
    while (cur.next(seg)) {
        const int32_t* bt = p.tables + (int64_t)seg.b * p.table_stride;
        const int zh = seg.g * HG;
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
                    if (!mbar_wait_bounded(&empty_bar[s], par, s_abort, p.wait_ns)) {
                        aborted = true;
                        *s_abort = 1;
                        raise_flag(CX_DEV_WAIT_TIMEOUT);
                    } else if (*s_abort) {
                        // A consumer gave up and released this stage without
                        // waiting for its previous fill, whose bytes may still
                        // be landing: never re-arm it.
                        aborted = true;
                    } else if (bk >= 0) {
                        s_bad[s] = 0;
                        mbar_arrive_expect_tx(&full_bar[s], STAGE);
                        const int z = (p.layer * p.n_blocks + bk) * p.hk + zh;
                        unsigned char* kd = ring + (size_t)s * STAGE;
#pragma unroll
                        for (int c = 0; c < NBOX; ++c) {
                            tma_load_3d(kd + c * BOX_BYTES, tmk, &full_bar[s], c * BOX_COLS, 0, z);
                            tma_load_3d(kd + TILES + c * BOX_BYTES, tmv, &full_bar[s],
                                        c * BOX_COLS, 0, z);
                        }
                    } else {
                        // bad id: nothing is loaded; the consumers see the flag
                        // and leave the stage's keys out
                        s_bad[s] = 1;
                        mbar_arrive(&full_bar[s]);
                    }
                    if (!aborted) ++issued;
                }
                __syncwarp();
            }
        }
    }
    // Do not leave the CTA with tile copies still landing in its smem (a fixed
    // limit: the copies land within microseconds unless the GPU is broken, and
    // a short test limit must not cut this wait).
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
}

// ---------------------------------------------------------------------------
// End of a (sequence, head group) range, shared by the decode / verify
// kernels.  Partial softmax states are rows of D + 2 floats: the unnormalised
// O, the running max m (base-2 domain) and the denominator l.
// ---------------------------------------------------------------------------
// Merge the KS key slices of the CTA from shared memory (`merge`,
// [KS][HG][p.rows][D + 2], filled by every consumer warp) into the final rows
// (a range wholly inside this CTA) or into the CTA's workspace slot.
template <int D, int HG>
__device__ __forceinline__ void ks_merge(const MmaParams& p, const float* merge, float* slot,
                                         const Seg& seg, int64_t qs, int rows_b, int ctid,
                                         int NCT, int KS) {
    const int G = p.group, Hq = p.hq;
    named_bar_sync(1, NCT);
    for (int e = ctid; e < HG * rows_b * D; e += NCT) {
        const int d = e % D;
        const int R = (e / D) % rows_b;
        const int eh = e / (D * rows_b);
        float M = -INFINITY;
#pragma unroll 4
        for (int s2 = 0; s2 < KS; ++s2)
            M = fmaxf(M, merge[(((size_t)s2 * HG + eh) * p.rows + R) * (D + 2) + D]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll 4
            for (int s2 = 0; s2 < KS; ++s2) {
                const float* r = merge + (((size_t)s2 * HG + eh) * p.rows + R) * (D + 2);
                const float wgt = exp2f(r[D] - M);
                L += r[D + 1] * wgt;
                O += r[d] * wgt;
            }
        }
        if (seg.whole) {
            const int64_t orow = (qs + R / G) * Hq + (int64_t)(seg.g * HG + eh) * G + R % G;
            p.out[orow * D + d] = L > 0.f ? O / L : 0.f;
        } else {
            float* r = slot + ((size_t)eh * p.rows + R) * (D + 2);
            r[d] = O;
            if (d == 0) {
                r[D] = M;
                r[D + 1] = L;
            }
        }
    }
}

// A range cut by a chunk boundary: every CTA holding part of it takes an
// atomic ticket after writing its slot; the last one merges all partials of
// the range in one pass (log-sum-exp) and writes the final rows.  No waiting.
template <int D, int HG>
__device__ __forceinline__ void ticket_merge(const MmaParams& p, const Seg& seg, int b,
                                             int64_t qs, int rows_b, int ctid, int NCT,
                                             int chunk, int* s_last) {
    const int G = p.group, Hq = p.hq;
    const int bg = b * p.n_groups + seg.g;
    const size_t slot_floats = (size_t)HG * p.rows * (D + 2);
    __threadfence();
    named_bar_sync(1, NCT);
    if (ctid == 0) {
        const int first_u = p.seq_start[b] + seg.g * seg.nb;
        const int pf = first_u / chunk, pl = (first_u + seg.nb - 1) / chunk;
        const int prev = atomicAdd(&p.counters[bg], 1);
        *s_last = (prev == pl - pf) ? (pf | (pl << 16)) + 1 : 0;
    }
    named_bar_sync(1, NCT);
    const int last = *s_last;
    if (!last) return;
    __threadfence();
    const int pf = (last - 1) & 0xffff, pl = (last - 1) >> 16;
    // one pass over the partials, two columns per thread: the loads of every
    // partial are independent of the running merge, so they overlap instead
    // of costing an L2 round trip each
    constexpr int D2 = D / 2;
    for (int e = ctid; e < HG * rows_b * D2; e += NCT) {
        const int d = 2 * (e % D2);
        const int R = (e / D2) % rows_b;
        const int eh = e / (D2 * rows_b);
        const float* r0 = p.partials + (size_t)(pf + bg) * slot_floats +
                          ((size_t)eh * p.rows + R) * (D + 2);
        float M = -INFINITY, L = 0.f, Ox = 0.f, Oy = 0.f;
#pragma unroll 4
        for (int pp = 0; pp <= pl - pf; ++pp) {
            const float* r = r0 + (size_t)pp * slot_floats;
            const float m = __ldcg(r + D), l = __ldcg(r + D + 1);
            const float2 o = __ldcg(reinterpret_cast<const float2*>(r + d));
            if (m == -INFINITY) continue;  // a partial that saw no key
            const float Mn = fmaxf(M, m);
            const float a = exp2f(M - Mn), w = exp2f(m - Mn);
            L = L * a + l * w;
            Ox = Ox * a + o.x * w;
            Oy = Oy * a + o.y * w;
            M = Mn;
        }
        const int64_t orow = (qs + R / G) * Hq + (int64_t)(seg.g * HG + eh) * G + R % G;
        const float inv = L > 0.f ? 1.f / L : 0.f;
        *reinterpret_cast<float2*>(p.out + orow * D + d) =
            L > 0.f ? make_float2(Ox * inv, Oy * inv) : make_float2(0.f, 0.f);
    }
    if (ctid == 0) p.counters[bg] = 0;
}

// The plan must come from paged_plan_kernel for this batch shape (else the
// flag is raised and the CTA returns false); sequences with no cached token
// get zero rows (naive_attention semantics for rows with no key).
template <int D>
__device__ __forceinline__ bool plan_ok_zero_empty(const MmaParams& p) {
    const int B = p.batch, Hq = p.hq, tid = threadIdx.x;
    if (p.plan[3] != kPlanMagic || p.plan[4] != B || p.plan[5] != p.n_groups) {
        if (tid == 0 && blockIdx.x == 0) raise_flag(CX_DEV_BAD_QLEN);
        return false;
    }
    for (int b = blockIdx.x; b < B; b += gridDim.x) {
        if (p.seq_start[b + 1] != p.seq_start[b]) continue;
        const int sq = p.q_start ? p.q_start[b + 1] - p.q_start[b] : 1;
        const int64_t r0 = p.q_start ? p.q_start[b] : b;
        for (int64_t e = tid; e < (int64_t)sq * Hq * D; e += blockDim.x)
            p.out[r0 * Hq * D + e] = 0.f;
    }
    return true;
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

// Rescale O only when a row max grows by more than 2^8 (see the consumer loop).
constexpr float kMmaRescaleLog2 = 8.f;

// 2^x as one special-function-unit instruction (ex2.approx.ftz: relative error
// about 2^-22, far below the bf16 rounding of P; 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int D, int MT, int HG>
struct MmaCfg {
    static constexpr int KS = (HG * MT >= kConsumerWarps) ? 1 : kConsumerWarps / (HG * MT);
    static constexpr int NCW = HG * MT * KS;           // consumer warps
    static constexpr int THREADS = (NCW + 1) * 32;     // + producer warp
    // Q fragments in shared memory (one 16-byte slot per lane and k-step,
    // reloaded per block) instead of registers: lets 12 consumer warps (13
    // warps, 128 registers a thread) run without spilling, and frees the
    // registers for two blocks per iteration at two row tiles.  Decode (one
    // row tile) keeps Q in registers: the slots would cost it two ring stages.
    static constexpr bool QSM = NCW + 1 > 12 || MT == 2;
    // blocks per consumer iteration: 2 when the block has at most 8 warps (two
    // per SM sub-partition, so up to 255 registers a thread) or Q sits in
    // shared memory at two row tiles, else 1
    static constexpr int U = (NCW + 1 <= 8 || MT == 2) ? 2 : 1;
    static constexpr size_t QSM_BYTES = QSM ? (size_t)NCW * (D / 16) * 32 * 16 : 0;
    static constexpr int HALF_BOX = kBlockTok * 128;   // one head, 16 rows x 128 B
    static constexpr int TILES = HG * kBlockTok * D * 2;  // K (or V) bytes of a unit
    static constexpr int STAGE = 2 * TILES;
    static constexpr int NT = D / 8;     // n-tiles of the output
    static constexpr int KSTEP = D / 16;
    // byte offset of (head hh, token t, dim d [multiple of 8]) inside a K or V
    // region: D/64 column halves, each HG heads x 16 rows x 128 B, swizzled
    __device__ __forceinline__ static uint32_t swz(int hh, int t, int d) {
        return (uint32_t)((d >> 6) * (HG * HALF_BOX) + hh * HALF_BOX + t * 128 +
                          ((((d & 63) >> 3) ^ (t & 7)) << 4));
    }
    __host__ __device__ static size_t merge_bytes(int rows) {
        return KS > 1 ? (size_t)KS * HG * rows * (D + 2) * sizeof(float) : 0;
    }
    static int stages_for(int rows) {
        const size_t fixed = 1024 + merge_bytes(rows) + 64 + QSM_BYTES;
        const size_t avail = kSmemBudget > fixed ? kSmemBudget - fixed : 0;
        int s = (int)(avail / (STAGE + 2 * sizeof(uint64_t)));
        s = s > 32 ? 32 : s;
        // The KS consumer warps of one (head, row tile) share each stage;
        // mbarrier parity is derived from (iteration / STAGES), so a ring
        // whose length is not a multiple of KS would let two consumers wait
        // on the same barrier phase for different fills.
        return (s / KS) * KS;
    }
    static size_t smem_bytes(int rows, int stages) {
        return 1024 + (size_t)stages * STAGE + 2 * stages * sizeof(uint64_t) + merge_bytes(rows) +
               64 + QSM_BYTES;
    }
};

template <int D, int MT, int HG, typename QT>
__global__ void __launch_bounds__(MmaCfg<D, MT, HG>::THREADS, 1)
    paged_attn_mma_kernel(const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const MmaParams p) {
    using C = MmaCfg<D, MT, HG>;
    constexpr int KS = C::KS;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* ring = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int STAGES = p.stages;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(ring + (size_t)STAGES * C::STAGE);
    uint64_t* empty_bar = full_bar + STAGES;
    float* merge = reinterpret_cast<float*>(empty_bar + STAGES);
    int* s_flags = reinterpret_cast<int*>(reinterpret_cast<unsigned char*>(merge) +
                                          C::merge_bytes(p.rows));
    volatile int* s_abort = s_flags;
    int* s_last = s_flags + 1;
    // per ring stage: 1 when its block id was outside the pool (nothing loaded)
    volatile unsigned char* s_bad = reinterpret_cast<unsigned char*>(s_flags + 4);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int B = p.batch, Hq = p.hq, G = p.group;
    // A warp taking two units holds the first while it waits for the second
    // (KS units later); the producer can fill that one only if the ring has
    // more than KS stages.
    if (STAGES < 2 || STAGES % KS != 0 || (C::U == 2 && STAGES < 2 * KS)) {
        if (tid == 0 && blockIdx.x == 0) raise_flag(CX_DEV_BAD_QLEN);
        return;
    }

    if (!plan_ok_zero_empty<D>(p)) return;
    const int W = p.plan[0], chunk = p.plan[1], P_eff = p.plan[2];
    if ((int)blockIdx.x >= P_eff) return;
    const int u0 = blockIdx.x * chunk;
    const int u1 = min(W, u0 + chunk);

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], HG * MT);
        }
        s_flags[0] = 0;
        s_flags[1] = 0;
        s_flags[2] = 0;   // verify: some block id of this CTA is outside the pool
        fence_mbar_init();
    }
    __syncthreads();

    SegCursor cur;
    cur.init(u0, u1, p);
    Seg seg;

    if (warp == C::NCW) {
        produce_units<D / 64, 64, HG * C::HALF_BOX, C::TILES, C::STAGE>(
            &tmk, &tmv, p, cur, HG, ring, full_bar, empty_bar, s_abort, s_bad, lane);
        return;
    }

    // ------------------------------- consumers -------------------------------
    const int hh = warp % HG, mt = (warp / HG) % MT, ks = warp / (HG * MT);
    const int NCT = C::NCW * 32;
    const int ctid = tid;  // consumer threads are 0..NCT-1
    // per-lane ldmatrix coordinates
    const int k_tok = (lane & 7) + 8 * (lane >> 4), k_dsub = 8 * ((lane >> 3) & 1);
    const int v_tok = (lane & 7) + 8 * ((lane >> 3) & 1), v_dsub = 8 * (lane >> 4);
    const int qr0 = lane >> 2, qc = 2 * (lane & 3);
    const int R0 = mt * 16 + qr0, R1 = R0 + 8;  // packed rows this lane owns
    const QT* qbase = static_cast<const QT*>(p.q);
    // this lane's Q slots when C::QSM: [warp][k-step][lane] x 16 B after the flags
    const uint32_t q_slot = smem_addr(reinterpret_cast<unsigned char*>(s_flags) + 64) +
                            (uint32_t)((warp * C::KSTEP * 32 + lane) * 16);
    const size_t slot_floats = (size_t)HG * p.rows * (D + 2);

    // Verify (MT > 1): block ids outside the pool anywhere in this CTA's
    // units.  The consumer warps scan them together (warp w takes every NCW-th
    // run of 32 ids) and combine the result at one named barrier, while the
    // first stage is still loading.  The unit loop then exists in two
    // instantiations: without bad-id handling (the normal case) and with it
    // (read each stage's flag, leave its keys out).  Reading the flag per unit
    // cost verify 3 % at gamma 4; each warp scanning every id itself cost 3-6 %.
    // Decode (MT 1) keeps the one loop that reads the flag: it measured no
    // slower, and two instantiations made it spill.
    bool any_bad = true;
    if constexpr (MT > 1) {
        SegCursor c2 = cur;
        Seg s2;
        bool bad = false;
        while (c2.next(s2)) {
            const int32_t* bt = p.tables + (int64_t)s2.b * p.table_stride;
            for (int k = warp * 32 + lane; k < s2.cnt; k += C::NCW * 32) {
                const int jj = s2.j0 + k;
                const int bid = jj < p.table_stride ? bt[jj] : -1;
                bad |= bid < 0 || bid >= p.n_blocks;
            }
        }
        if (__any_sync(0xffffffffu, bad) && lane == 0) s_flags[2] = 1;
        named_bar_sync(1, NCT);
        any_bad = *reinterpret_cast<volatile int*>(s_flags + 2) != 0;
    }

    int ibase = 0;
    while (cur.next(seg)) {
        const int b = seg.b, h = seg.g * HG + hh;
        const int ctx = min(p.ctx_lens[b], (int)(p.table_stride * kBlockTok));
        // clamped: a query run longer than max_q_len (flagged by the plan) must
        // not index rows past the partial / merge rows the call was sized for
        const int sq = p.q_start ? min(max(p.q_start[b + 1] - p.q_start[b], 0), p.max_q) : 1;
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
        if constexpr (C::QSM) {
            // each lane writes and later reads only its own slots
#pragma unroll
            for (int kk = 0; kk < C::KSTEP; ++kk)
                st_shared_v4(q_slot + kk * 32 * 16, qa[kk]);
        }

        float o[C::NT][4];
#pragma unroll
        for (int n = 0; n < C::NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

        // U == 2: a warp takes two of its units per iteration (keys k and
        // k + KS): twice the independent MMAs between waits and one softmax
        // round (max, shuffles, vote) per 32 keys.
        constexpr int U = C::U;
        auto unit_loop = [&](auto bad_tag) {
        constexpr bool BAD = decltype(bad_tag)::value;
        for (int k = ((ks - ibase) % KS + KS) % KS; k < seg.cnt; k += U * KS) {
            const bool two = U == 2 && k + KS < seg.cnt;  // warp-uniform
            int su[U];
#pragma unroll
            for (int u = 0; u < U; ++u) su[u] = (ibase + k + u * KS) % STAGES;
            bool ok = !*s_abort;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = ibase + k + u * KS;
                if (ok && (u == 0 || two))
                    ok = mbar_wait_bounded(&full_bar[su[u]], (i / STAGES) & 1, s_abort,
                                           p.wait_ns);
            }
            // mma.sync / ldmatrix need the whole warp: agree on one outcome
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !*s_abort) {
                    *s_abort = 1;
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                }
            } else {
                // a stage whose block id was bad holds no data: its keys are
                // left out (scores -inf, no PV product), as the generic kernel
                // skips them (the flag is per stage, so warp-uniform)
                bool bad[U];
#pragma unroll
                for (int u = 0; u < U; ++u) bad[u] = BAD && (u == 0 || two) && s_bad[su[u]] != 0;
                float x[U][2][4];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if ((u > 0 && !two) || bad[u]) {
#pragma unroll
                        for (int n = 0; n < 2; ++n)
#pragma unroll
                            for (int e = 0; e < 4; ++e) x[u][n][e] = -INFINITY;
                        continue;
                    }
                    const uint32_t kb = smem_addr(ring + (size_t)su[u] * C::STAGE);
                    float sa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                    float sb[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
                    for (int kk = 0; kk < C::KSTEP; ++kk) {
                        uint32_t f[4];
                        ldmatrix_x4(f, kb + C::swz(hh, k_tok, kk * 16 + k_dsub));
                        uint32_t qk[4];
                        if constexpr (C::QSM) {
                            ld_shared_v4(qk, q_slot + kk * 32 * 16);
                        } else {
                            qk[0] = qa[kk][0];
                            qk[1] = qa[kk][1];
                            qk[2] = qa[kk][2];
                            qk[3] = qa[kk][3];
                        }
                        if (kk & 1) {
                            mma_bf16_16816(sb[0], qk, f[0], f[1]);
                            mma_bf16_16816(sb[1], qk, f[2], f[3]);
                        } else {
                            mma_bf16_16816(sa[0], qk, f[0], f[1]);
                            mma_bf16_16816(sa[1], qk, f[2], f[3]);
                        }
                    }
#pragma unroll
                    for (int n = 0; n < 2; ++n)
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            x[u][n][e] = (sa[n][e] + sb[n][e]) * p.scale_log2;
                    const int t0 = (seg.j0 + k + u * KS) * kBlockTok;
                    const bool edge = (t0 + kBlockTok - 1 > pos0) ||
                                      (p.window > 0 && t0 <= ctx - 1 - p.window);
                    if (edge) {
#pragma unroll
                        for (int n = 0; n < 2; ++n)
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int tok = t0 + n * 8 + qc + (e & 1);
                                const int rp = (e < 2) ? rpos0 : rpos1;
                                const bool ok_t =
                                    tok <= rp && (p.window <= 0 || tok > rp - p.window);
                                if (!ok_t) x[u][n][e] = -INFINITY;
                            }
                    }
                }
                float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    mx0 = fmaxf(mx0, fmaxf(fmaxf(x[u][0][0], x[u][0][1]),
                                           fmaxf(x[u][1][0], x[u][1][1])));
                    mx1 = fmaxf(mx1, fmaxf(fmaxf(x[u][0][2], x[u][0][3]),
                                           fmaxf(x[u][1][2], x[u][1][3])));
                }
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                // lazy rescale: a row keeps its reference max until its block
                // max exceeds it by more than 2^8 (p <= 256 meanwhile; the
                // final division, and the split-K merge, which uses each
                // partial's own m, make a stale max exact)
                const bool g0 = mx0 > m0 + kMmaRescaleLog2 || (m0 == -INFINITY && mx0 > -INFINITY);
                const bool g1 = mx1 > m1 + kMmaRescaleLog2 || (m1 == -INFINITY && mx1 > -INFINITY);
                const float mn0 = g0 ? mx0 : m0, mn1 = g1 ? mx1 : m1;
                const float base0 = mn0 == -INFINITY ? 0.f : mn0;
                const float base1 = mn1 == -INFINITY ? 0.f : mn1;
                const float a0 = g0 ? exp2f(m0 - base0) : 1.f, a1 = g1 ? exp2f(m1 - base1) : 1.f;
                float pr[U][2][4];
                float r0, r1;
#pragma unroll
                for (int u = 0; u < U; ++u) {
#pragma unroll
                    for (int n = 0; n < 2; ++n) {
                        pr[u][n][0] = ex2_approx(x[u][n][0] - base0);
                        pr[u][n][1] = ex2_approx(x[u][n][1] - base0);
                        pr[u][n][2] = ex2_approx(x[u][n][2] - base1);
                        pr[u][n][3] = ex2_approx(x[u][n][3] - base1);
                    }
                    const float q0 = pr[u][0][0] + pr[u][0][1] + pr[u][1][0] + pr[u][1][1];
                    const float q1 = pr[u][0][2] + pr[u][0][3] + pr[u][1][2] + pr[u][1][3];
                    r0 = u == 0 ? q0 : r0 + q0;
                    r1 = u == 0 ? q1 : r1 + q1;
                }
                l0 = l0 * a0 + r0;
                l1 = l1 * a1 + r1;
                m0 = mn0;
                m1 = mn1;
                if (__any_sync(0xffffffffu, g0 || g1)) {
#pragma unroll
                    for (int n = 0; n < C::NT; ++n) {
                        o[n][0] *= a0;
                        o[n][1] *= a0;
                        o[n][2] *= a1;
                        o[n][3] *= a1;
                    }
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if ((u > 0 && !two) || bad[u]) continue;
                    const uint32_t vb = smem_addr(ring + (size_t)su[u] * C::STAGE) + C::TILES;
                    uint32_t pa[4];
                    pa[0] = pack_bf16(pr[u][0][0], pr[u][0][1]);
                    pa[1] = pack_bf16(pr[u][0][2], pr[u][0][3]);
                    pa[2] = pack_bf16(pr[u][1][0], pr[u][1][1]);
                    pa[3] = pack_bf16(pr[u][1][2], pr[u][1][3]);
#pragma unroll
                    for (int np = 0; np < C::KSTEP; ++np) {
                        uint32_t f[4];
                        ldmatrix_x4_trans(f, vb + C::swz(hh, v_tok, np * 16 + v_dsub));
                        mma_bf16_16816(o[2 * np], pa, f[0], f[1]);
                        mma_bf16_16816(o[2 * np + 1], pa, f[2], f[3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty_bar[su[0]]);
                if (two) mbar_arrive(&empty_bar[su[U - 1]]);
            }
        }
        };
        if constexpr (MT == 1) {
            unit_loop(std::true_type{});
        } else {
            if (any_bad)
                unit_loop(std::true_type{});
            else
                unit_loop(std::false_type{});
        }
        ibase += seg.cnt;

        // ---- finish this (sequence, head group) range ----
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        const int bg = b * p.n_groups + seg.g;
        float* slot = p.partials + (size_t)(blockIdx.x + bg) * slot_floats;
        if (KS == 1) {
            // each warp owns complete rows: write straight from registers
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int R = half ? R1 : R0;
                if (R >= rows_b) continue;
                const float mm = half ? m1 : m0, ll = half ? l1 : l0;
                if (seg.whole) {
                    const float inv = ll > 0.f ? 1.f / ll : 0.f;
                    const int64_t orow = (qs + R / G) * Hq + (int64_t)h * G + R % G;
                    float* dst = p.out + orow * D;
#pragma unroll
                    for (int n = 0; n < C::NT; ++n) {
                        *reinterpret_cast<float2*>(dst + n * 8 + qc) =
                            make_float2(o[n][2 * half] * inv, o[n][2 * half + 1] * inv);
                    }
                } else {
                    float* r = slot + ((size_t)hh * p.rows + R) * (D + 2);
#pragma unroll
                    for (int n = 0; n < C::NT; ++n)
                        *reinterpret_cast<float2*>(r + n * 8 + qc) =
                            make_float2(o[n][2 * half], o[n][2 * half + 1]);
                    if ((lane & 3) == 0) {
                        r[D] = mm;
                        r[D + 1] = ll;
                    }
                }
            }
        } else {
            // merge the KS key slices through shared memory
            {
                float* mrow = merge + ((size_t)ks * HG + hh) * p.rows * (D + 2);
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int R = half ? R1 : R0;
                    if (R >= rows_b) continue;
                    float* r = mrow + (size_t)R * (D + 2);
#pragma unroll
                    for (int n = 0; n < C::NT; ++n) {
                        r[n * 8 + qc] = o[n][2 * half];
                        r[n * 8 + qc + 1] = o[n][2 * half + 1];
                    }
                    if ((lane & 3) == 0) {
                        r[D] = half ? m1 : m0;
                        r[D + 1] = half ? l1 : l0;
                    }
                }
            }
            ks_merge<D, HG>(p, merge, slot, seg, qs, rows_b, ctid, NCT, KS);
        }
        if (!seg.whole)
            ticket_merge<D, HG>(p, seg, b, qs, rows_b, ctid, NCT, chunk, s_last);
        named_bar_sync(1, NCT);
    }
}

}  // namespace cx

#include "attn_paged_f32.cuh"
#include "attn_prefill_tc.cuh"
#include "attn_prefill_tc128.cuh"
#include "attn_prefill_tc256.cuh"

namespace cx {

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

// 3-D view of a bf16 or fp32 pool: (head_dim, 16 slots, layers*blocks*heads
// tiles), box of one 128-byte column (64 bf16 or 32 fp32 values) x 16 x hg
// (hg consecutive heads of one block) with 128-byte swizzle.
static int make_pool_tmap(CUtensorMap* m, void* base, const cx_pool* p, int hg) {
    auto enc = tmap_encoder();
    if (!enc) return fail(CX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const bool f32 = p->dtype == CX_F32;
    const cuuint64_t e = f32 ? 4 : 2;
    const cuuint64_t dims[3] = {(cuuint64_t)p->head_dim, (cuuint64_t)p->block_size,
                                (cuuint64_t)(p->n_layers * p->n_blocks * p->n_kv_heads)};
    const cuuint64_t strides[2] = {(cuuint64_t)p->head_dim * e,
                                   (cuuint64_t)(p->block_size * p->head_dim * e)};
    const cuuint32_t box[3] = {(cuuint32_t)(128 / e), (cuuint32_t)p->block_size, (cuuint32_t)hg};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                     3, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CX_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    return CX_OK;
}

struct MmaShape {
    int mt, hg, ks, n_groups;
};

// Heads per unit: a power of two dividing the KV head count, at most 4 (one
// to three row tiles) or 2 (four): 4 heads keep a unit's 16-token stage at
// 32 KB (8 KB TMA boxes), so the ring has six stages and frees them in finer
// steps; 8 heads (64 KB stages, three of them) measured 2.7 % slower at
// decode, 2 heads (4 KB boxes) 16 % slower.  The row-tile warps are then
// split over the unit's blocks (ks) up to 8 consumer warps; three row tiles
// of 4 heads run 12 consumer warps with Q in shared memory (MmaCfg::QSM).
static MmaShape mma_shape(int64_t hk, int64_t rows) {
    MmaShape s{};
    s.mt = (int)((rows + 15) / 16);
    const int cap = s.mt <= 3 ? 4 : 2;
    s.hg = 1;
    while (s.hg * 2 <= cap && hk % (s.hg * 2) == 0) s.hg *= 2;
    s.ks = s.hg * s.mt >= kConsumerWarps ? 1 : kConsumerWarps / (s.hg * s.mt);
    s.n_groups = (int)(hk / s.hg);
    return s;
}

// fp32 pools: heads per unit and row tiles of RT = 4, 8 or 16 rows.  One
// head's K (or V) of a unit is 4 KB (head_dim 64) or 8 KB (128) of fp32, and
// each TMA box covers a 128-byte column of hg heads (hg x 2 KB): a single
// issuing thread keeps up with HBM only from about 4 KB a box, so hg is 2 or 4
// where the KV head count allows (stage = hg x 16 KB or hg x 32 KB).  The key
// slices (ks) are chosen at launch from the ring length.
static int f32_rt(int64_t rows) { return rows <= 4 ? 4 : rows <= 8 ? 8 : 16; }

static MmaShape f32_shape(int64_t hk, int64_t rows, int64_t d) {
    MmaShape s{};
    const int rt = f32_rt(rows);
    s.mt = (int)((rows + rt - 1) / rt);
    const int cap = d == 64 ? 4 : 2;
    // consumer warps available: 7 for the wide row tiles (F32Cfg::MAX_CONSUMERS)
    const int warps = (rt == 16 || (rt == 8 && d == 128)) ? 7 : kConsumerWarps;
    s.hg = 1;
    while (s.hg * 2 <= cap && hk % (s.hg * 2) == 0 && s.hg * 2 * s.mt <= warps) s.hg *= 2;
    s.ks = 0;
    s.n_groups = (int)(hk / s.hg);
    return s;
}

static MmaShape unit_shape(const cx_pool* pool, int64_t rows) {
    return pool->dtype == CX_F32 ? f32_shape(pool->n_kv_heads, rows, pool->head_dim)
                                 : mma_shape(pool->n_kv_heads, rows);
}

struct WsLayout {
    size_t plan, seq, lo, cnt, part, total;
};

static WsLayout ws_layout(int64_t batch, const MmaShape& sh, int64_t rows, int64_t d,
                          int64_t grid) {
    auto up = [](size_t x, size_t a) { return (x + a - 1) / a * a; };
    WsLayout w{};
    w.plan = 0;
    w.seq = 64;
    w.lo = up(w.seq + (batch + 1) * 4, 16);
    w.cnt = up(w.lo + batch * 4, 16);
    w.part = up(w.cnt + batch * sh.n_groups * 4, 256);
    w.total = w.part + (size_t)(grid + batch * sh.n_groups) * sh.hg * rows * (d + 2) * 4;
    return w;
}

template <int D, int MT, int HG, typename QT>
static int launch_mma_cfg(const CUtensorMap& tk, const CUtensorMap& tv, MmaParams p,
                          cudaStream_t st, int grid) {
    using C = MmaCfg<D, MT, HG>;
    auto kern = paged_attn_mma_kernel<D, MT, HG, QT>;
    p.stages = C::stages_for(p.rows);
    p.stage_bytes = C::STAGE;
    if (p.stages < 2 || p.stages % C::KS != 0 || (C::U == 2 && p.stages < 2 * C::KS))
        return fail(CX_ERR_UNSUPPORTED, "paged attention: shared memory too small");
    const size_t smem = C::smem_bytes(p.rows, p.stages);
    CX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, C::THREADS, smem, st>>>(tk, tv, p);
    return check_launch("paged_attn_mma_kernel");
}

template <int D, typename QT>
static int launch_mma_d(const MmaShape& sh, const CUtensorMap& tk, const CUtensorMap& tv,
                        const MmaParams& p, cudaStream_t st, int grid) {
#define CX_CASE(MT_, HG_) \
    if (sh.mt == MT_ && sh.hg == HG_) return launch_mma_cfg<D, MT_, HG_, QT>(tk, tv, p, st, grid);
    CX_CASE(1, 8) CX_CASE(1, 4) CX_CASE(1, 2) CX_CASE(1, 1)
    CX_CASE(2, 4) CX_CASE(2, 2) CX_CASE(2, 1)
    CX_CASE(3, 4) CX_CASE(3, 2) CX_CASE(3, 1)
    CX_CASE(4, 2) CX_CASE(4, 1)
#undef CX_CASE
    return fail(CX_ERR_UNSUPPORTED, "paged attention: no kernel for this row/head shape");
}

template <int D, int HG, int RT>
static int launch_f32_cfg(const CUtensorMap& tk, const CUtensorMap& tv, MmaParams p,
                          cudaStream_t st, int grid) {
    using C = F32Cfg<D, HG, RT>;
    auto kern = paged_attn_f32_kernel<D, HG, RT>;
    // key slices: the ring length must be a multiple of them (each stage is
    // always consumed by the same slice).  Take the most consumer warps whose
    // ring still holds at least 4 stages and 3/4 of the longest ring: one warp
    // per head walks its units serially (a 4-unit chunk at 1 slice measured
    // 33 us for cfg1, the SMs busy 14 % of it), while a ring shortened from 6
    // to 4 stages of 32 KB costs more than the third and fourth slice give.
    const int max_ks = C::MAX_CONSUMERS / (HG * p.mt);
    int stg_of[kConsumerWarps + 1] = {};
    int longest = 0;
    for (int ks = 1; ks <= max_ks; ++ks) {
        stg_of[ks] = (C::raw_stages(p.rows, p.mt, ks) / ks) * ks;
        longest = stg_of[ks] > longest ? stg_of[ks] : longest;
    }
    int best_ks = 0, best_st = 0;
    for (int ks = 1; ks <= max_ks; ++ks) {
        const int stg = stg_of[ks];
        if (stg >= 2 && (best_ks == 0 || (stg >= 4 && 4 * stg >= 3 * longest))) {
            best_st = stg;
            best_ks = ks;
        }
    }
    if (!best_ks) return fail(CX_ERR_UNSUPPORTED, "paged attention: shared memory too small");
    p.ks = best_ks;
    p.stages = best_st;
    p.stage_bytes = C::STAGE;
    const size_t smem = C::smem_bytes(p.rows, p.mt, p.ks, p.stages);
    const int threads = (HG * p.mt * p.ks + 1) * 32;
    CX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, threads, smem, st>>>(tk, tv, p);
    return check_launch("paged_attn_f32_kernel");
}

template <int D>
static int launch_f32_d(const MmaShape& sh, const CUtensorMap& tk, const CUtensorMap& tv,
                        const MmaParams& p, cudaStream_t st, int grid) {
    const int rt = f32_rt(p.rows);
#define CX_CASE(HG_, RT_) \
    if (sh.hg == HG_ && rt == RT_) return launch_f32_cfg<D, HG_, RT_>(tk, tv, p, st, grid);
    CX_CASE(1, 4) CX_CASE(1, 8) CX_CASE(1, 16)
    CX_CASE(2, 4) CX_CASE(2, 8) CX_CASE(2, 16)
    if constexpr (D == 64) {
        CX_CASE(4, 4) CX_CASE(4, 8) CX_CASE(4, 16)
    }
#undef CX_CASE
    return fail(CX_ERR_UNSUPPORTED, "paged attention: no fp32 kernel for this row/head shape");
}

// fp32 pool, 16-token blocks, head_dim 64 / 128, at most 64 packed query rows
// per KV head: the TMA + FMA kernel (attn_paged_f32.cuh)
static bool f32_eligible(const cx_pool* pool, const cx_attn_batch* b, int32_t q_dtype) {
    const int64_t G = b->n_q_heads / pool->n_kv_heads;
    const int64_t rows = G * b->max_q_len;
    const int64_t tiles = pool->n_layers * pool->n_blocks * pool->n_kv_heads;
    const uintptr_t a = reinterpret_cast<uintptr_t>(pool->k) | reinterpret_cast<uintptr_t>(pool->v);
    return pool->dtype == CX_F32 && pool->block_size == kBlockTok &&
           (pool->head_dim == 64 || pool->head_dim == 128) && rows >= 1 && rows <= 64 &&
           (q_dtype == CX_F32 || q_dtype == CX_BF16) && tiles < (1ll << 31) && (a & 15) == 0 &&
           b->batch < (1 << 24) && pool->n_kv_heads * b->batch < (1 << 24);
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

// Scratch bytes a decode (verify = false) or verify call will use: the plan /
// split-K workspace of the mma.sync and fp32 FMA kernels; none for the
// tcgen05 and generic kernels.  Same kernel choice as paged_attention.
static size_t paged_scratch_need(const cx_pool* pool, const cx_attn_batch* bt, const void* q,
                                 int32_t q_dtype, const float* out, bool verify) {
    if (!pool || !bt || pool->n_kv_heads <= 0 || bt->n_q_heads <= 0 || bt->batch <= 0) return 0;
    cx_attn_batch b = *bt;
    b.max_q_len = verify ? (bt->max_q_len > 0 ? bt->max_q_len : 1) : 1;
    const bool vec_ok =
        ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    if (vec_ok && tc_eligible(pool, &b, q_dtype)) return 0;
    const bool use_f32 = vec_ok && f32_eligible(pool, &b, q_dtype);
    if (!use_f32 && (!vec_ok || !mma_eligible(pool, &b, q_dtype))) return 0;
    const int64_t rows = (b.n_q_heads / pool->n_kv_heads) * b.max_q_len;
    return ws_layout(b.batch, unit_shape(pool, rows), rows, pool->head_dim, grid_size()).total;
}

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

    // The tensor-core kernels move Q and the output rows with 8- and 16-byte
    // vector accesses; other pointers take the element-wise generic kernel.
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    if (vec_ok && tc_eligible(pool, &b, q_dtype)) {
        // packed query tile >= 64 rows: tcgen05 kernel, no workspace
        const int G = (int)(b.n_q_heads / pool->n_kv_heads);
        TcParams t{};
        t.tables = b.block_tables;
        t.table_stride = b.table_stride;
        t.ctx_lens = b.ctx_lens;
        t.q_start = b.q_start;
        t.batch = (int)b.batch;
        t.hk = (int)pool->n_kv_heads;
        t.hq = (int)b.n_q_heads;
        t.group = G;
        t.tpt = kTcRows / G;
        // head_dim 128: one query tile per CTA when no sequence has more than
        // one (short verify chains), else two; head_dim 64: two
        const int64_t q_tiles = (max_q + t.tpt - 1) / t.tpt;
        const int tiles_per_cta = pool->head_dim == 128 && q_tiles == 1 ? 1 : 2;
        t.n_ctiles = (int)((max_q + tiles_per_cta * t.tpt - 1) / (tiles_per_cta * t.tpt));
        t.n_blocks = (int)pool->n_blocks;
        t.layer = (int)layer;
        t.window = b.window > 0 ? (int)(b.window < (1ll << 30) ? b.window : (1ll << 30)) : 0;
        t.scale_log2 = scale * 1.4426950408889634f;
        t.q = q;
        t.out = out;
        if (b.table_stride > (1ll << 26) || pool->n_blocks > INT32_MAX / pool->n_kv_heads ||
            (int64_t)pool->n_layers * pool->n_blocks * pool->n_kv_heads > INT32_MAX)
            return fail(CX_ERR_UNSUPPORTED, "paged attention: pool or table too large");
        CUtensorMap tk, tv;
        rc = make_pool_tmap(&tk, pool->k, pool, 1);
        if (rc) return rc;
        rc = make_pool_tmap(&tv, pool->v, pool, 1);
        if (rc) return rc;
        if (pool->head_dim == 128)
            return tiles_per_cta == 1
                       ? (q_dtype == CX_F32 ? launch_tc128<float>(tk, tv, t, st)
                                            : launch_tc128<__nv_bfloat16>(tk, tv, t, st))
                       : (q_dtype == CX_F32 ? launch_tc256<128, float>(tk, tv, t, st)
                                            : launch_tc256<128, __nv_bfloat16>(tk, tv, t, st));
        return q_dtype == CX_F32 ? launch_tc256<64, float>(tk, tv, t, st)
                                 : launch_tc256<64, __nv_bfloat16>(tk, tv, t, st);
    }

    const bool use_f32 = vec_ok && f32_eligible(pool, &b, q_dtype);
    if (!use_f32 && (!vec_ok || !mma_eligible(pool, &b, q_dtype))) {
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
    const MmaShape sh = unit_shape(pool, rows);
    const int grid = grid_size();
    const WsLayout wl = ws_layout(b.batch, sh, rows, pool->head_dim, grid);
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
    p.hg = sh.hg;
    p.n_groups = sh.n_groups;
    p.mt = sh.mt;
    p.q_bf16 = q_dtype == CX_BF16;
    p.n_blocks = (int)pool->n_blocks;
    p.layer = (int)layer;
    p.window = b.window > 0 ? (int)b.window : 0;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.wait_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
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
    rc = make_pool_tmap(&tk, pool->k, pool, sh.hg);
    if (rc) return rc;
    rc = make_pool_tmap(&tv, pool->v, pool, sh.hg);
    if (rc) return rc;
    if (use_f32)
        return pool->head_dim == 128 ? launch_f32_d<128>(sh, tk, tv, p, st, grid)
                                     : launch_f32_d<64>(sh, tk, tv, p, st, grid);
    if (pool->head_dim == 128)
        return q_dtype == CX_F32 ? launch_mma_d<128, float>(sh, tk, tv, p, st, grid)
                                 : launch_mma_d<128, __nv_bfloat16>(sh, tk, tv, p, st, grid);
    return q_dtype == CX_F32 ? launch_mma_d<64, float>(sh, tk, tv, p, st, grid)
                             : launch_mma_d<64, __nv_bfloat16>(sh, tk, tv, p, st, grid);
}

}  // namespace cx

extern "C" {

size_t cx_paged_workspace_bytes(const cx_pool* pool, const cx_attn_batch* b) {
    using namespace cx;
    if (!pool || !b || pool->n_kv_heads <= 0 || b->n_q_heads <= 0 || b->batch < 0) return 0;
    const int64_t G = b->n_q_heads / pool->n_kv_heads;
    const int64_t max_q = b->q_start ? (b->max_q_len > 0 ? b->max_q_len : 1) : 1;
    return ws_layout(b->batch, unit_shape(pool, G * max_q), G * max_q, pool->head_dim,
                     grid_size()).total;
}

int cx_paged_kernel_kind(const cx_pool* pool, const cx_attn_batch* batch, int32_t q_dtype,
                         int32_t verify) {
    using namespace cx;
    if (!pool || !batch || pool->n_kv_heads <= 0) return CX_KERNEL_GENERIC;
    cx_attn_batch b = *batch;
    b.max_q_len = verify ? (b.max_q_len > 0 ? b.max_q_len : 1) : 1;
    if (tc_eligible(pool, &b, q_dtype)) return CX_KERNEL_TCGEN05;
    if (mma_eligible(pool, &b, q_dtype)) return CX_KERNEL_MMA;
    if (f32_eligible(pool, &b, q_dtype)) return CX_KERNEL_FMA;
    return CX_KERNEL_GENERIC;
}

void cx_set_wait_limit_ns(uint64_t ns) {
    cx::g_wait_limit_ns.store(ns ? ns : cx::kWaitLimitNs, std::memory_order_relaxed);
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
