// Paged flash-decode / multi-query verify over an fp32 pool with 16-token
// blocks and head_dim 64 or 128 (sm_100a): the reference's own precision
// (chenxing/core/attention.py:95-115 computes in fp32 throughout), so the math
// runs on the FP32 pipe with fused multiply-adds, not on tensor cores (TF32
// would miss the 1e-5 parity bar by two orders of magnitude).
//
// Work decomposition, plan, TMA producer and range merge are the bf16
// kernel's (attn_paged_mma.cuh): units of one 16-token block x HG KV heads,
// equal contiguous chunks of units per persistent CTA, atomic-ticket merge of
// ranges cut by a chunk boundary.  A unit's K (and V) arrive as D/32 column
// boxes of 32 floats (128 bytes, 128-byte swizzle) x 16 tokens x HG heads.
//
// Consumer warps are indexed (hh, mt, ks): head hh of the group, row tile mt
// (RT packed rows, row = query token * G + head-in-group) and key slice ks
// (every KS-th unit; KS is chosen on the host so that the ring length is a
// multiple of it).  Per unit a warp
//   * S phase: lane (t = lane % 16, parity = lane / 16) computes the scores of
//     key t against rows parity, parity + 2, ...: 16-byte K chunks from the
//     swizzled stage (conflict-free), Q chunks broadcast from a padded
//     shared-memory copy of the group's query rows;
//   * softmax: row maxima over the 16 keys by xor shuffles, exchanged between
//     the two half-warps so every lane holds every row's running max; the
//     accumulator is rescaled lazily (only when a row max grows by more than
//     2^8, exact after the final division);
//   * PV phase: P goes through a per-warp shared-memory tile, and lane owns
//     D/32 consecutive output columns of every row: O[r][:] += p[r][t] V[t][:].
#pragma once

namespace cx {

template <int D, int HG, int RT>
struct F32Cfg {
    // at most 8 warps (7 consumers + producer) for the wide row tiles: two
    // warps per SM sub-partition leave 255 registers a thread, enough for
    // their accumulators without spilling
    static constexpr bool WIDE = RT == 16 || (RT == 8 && D == 128);
    static constexpr int MAX_CONSUMERS = WIDE ? 7 : kConsumerWarps;
    static constexpr int MAX_THREADS = (MAX_CONSUMERS + 1) * 32;
    static constexpr int RPL = RT / 2;                  // rows per lane in the S phase
    static constexpr int BOX = HG * kBlockTok * 128;    // one 32-column box of HG heads
    static constexpr int NBOX = D / 32;
    static constexpr int TILES = HG * kBlockTok * D * 4;  // K (or V) bytes of a unit
    static constexpr int STAGE = 2 * TILES;
    static constexpr int QROW = D + 4;                  // padded shared-memory Q row (floats)
    static constexpr int DPL = D / 32;                  // output columns per lane
    // byte offset of (head hh, token t, 16-byte chunk c of the row) in a K or V
    // region: box c / 8, then the 128-byte swizzle of chunk c % 8 by t % 8
    __device__ __forceinline__ static uint32_t off(int hh, int t, int c) {
        return (uint32_t)((c >> 3) * BOX + hh * (kBlockTok * 128) + t * 128 +
                          ((((c & 7) ^ (t & 7))) << 4));
    }
    __host__ __device__ static size_t merge_bytes(int rows, int ks) {
        return ((size_t)ks * HG * rows * (D + 2) * sizeof(float) + 15) / 16 * 16;
    }
    __host__ __device__ static size_t q_bytes(int mt) { return (size_t)HG * mt * RT * QROW * 4; }
    __host__ __device__ static size_t p_bytes(int ncw) { return (size_t)ncw * RT * 16 * 4; }
    __host__ __device__ static size_t fixed_bytes(int rows, int mt, int ks) {
        return 1024 + merge_bytes(rows, ks) + 64 + q_bytes(mt) + p_bytes(HG * mt * ks);
    }
    static int raw_stages(int rows, int mt, int ks) {
        const size_t fixed = fixed_bytes(rows, mt, ks);
        const size_t avail = kSmemBudget > fixed ? kSmemBudget - fixed : 0;
        const int s = (int)(avail / (STAGE + 2 * sizeof(uint64_t)));
        return s > 32 ? 32 : s;
    }
    static size_t smem_bytes(int rows, int mt, int ks, int stages) {
        return fixed_bytes(rows, mt, ks) + (size_t)stages * (STAGE + 2 * sizeof(uint64_t));
    }
};

template <int D, int HG, int RT>
__global__ void __launch_bounds__(F32Cfg<D, HG, RT>::MAX_THREADS, 1)
    paged_attn_f32_kernel(const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const MmaParams p) {
    using C = F32Cfg<D, HG, RT>;
    constexpr int RPL = C::RPL, DPL = C::DPL;
    const int KS = p.ks, MT = p.mt;
    const int NCW = HG * MT * KS;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* ring = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int STAGES = p.stages;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(ring + (size_t)STAGES * C::STAGE);
    uint64_t* empty_bar = full_bar + STAGES;
    float* merge = reinterpret_cast<float*>(empty_bar + STAGES);
    int* s_flags = reinterpret_cast<int*>(reinterpret_cast<unsigned char*>(merge) +
                                          C::merge_bytes(p.rows, KS));
    volatile int* s_abort = s_flags;
    int* s_last = s_flags + 1;
    volatile unsigned char* s_bad = reinterpret_cast<unsigned char*>(s_flags + 4);
    float* s_q = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(s_flags) + 64);
    float* s_p = s_q + (size_t)HG * MT * RT * C::QROW;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Hq = p.hq, G = p.group;
    if (STAGES < 1 || KS < 1 || STAGES % KS != 0 || (int)blockDim.x != (NCW + 1) * 32) {
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
        fence_mbar_init();
    }
    __syncthreads();

    SegCursor cur;
    cur.init(u0, u1, p);
    if (warp == NCW) {
        produce_units<C::NBOX, 32, C::BOX, C::TILES, C::STAGE>(
            &tmk, &tmv, p, cur, HG, ring, full_bar, empty_bar, s_abort, s_bad, lane);
        return;
    }

    // ------------------------------- consumers -------------------------------
    const int hh = warp % HG, mt = (warp / HG) % MT, ks = warp / (HG * MT);
    const int NCT = NCW * 32, ctid = tid;
    const int t = lane & 15, rh = lane >> 4;
    const float* qw = s_q + (size_t)(hh + HG * mt) * RT * C::QROW;  // this warp's Q rows
    float* pw = s_p + (size_t)warp * RT * 16;                       // this warp's P tile
    const int d0 = lane * DPL;                                      // output columns
    // V chunk of this lane's columns: 16-byte chunk d0 / 4, byte offset inside it
    const int v_chunk = d0 >> 2, v_byte = (d0 & 3) * 4;
    const size_t slot_floats = (size_t)HG * p.rows * (D + 2);

    Seg seg;
    int ibase = 0;
    while (cur.next(seg)) {
        const int b = seg.b;
        const int ctx = min(p.ctx_lens[b], (int)(p.table_stride * kBlockTok));
        // clamped: a query run longer than max_q_len (flagged by the plan) must
        // not index rows past the partial / merge rows the call was sized for
        const int sq = p.q_start ? min(max(p.q_start[b + 1] - p.q_start[b], 0), p.max_q) : 1;
        const int64_t qs = p.q_start ? p.q_start[b] : b;
        const int rows_b = G * sq;
        const int pos0 = ctx - sq;  // position of query row 0

        // stage the group's query rows (fp32, zero padding rows): tile
        // (hh2, mt2) row r is packed row mt2 * RT + r of head seg.g * HG + hh2
        for (int e = ctid; e < HG * MT * RT * D; e += NCT) {
            const int d = e % D, r = (e / D) % RT, tile = e / (D * RT);
            const int hh2 = tile % HG, R = (tile / HG) * RT + r;
            float v = 0.f;
            if (R < rows_b) {
                const int64_t qi =
                    ((qs + R / G) * Hq + (int64_t)(seg.g * HG + hh2) * G + R % G) * D + d;
                v = p.q_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.q)[qi])
                             : static_cast<const float*>(p.q)[qi];
            }
            s_q[(size_t)tile * RT * C::QROW + r * C::QROW + d] = v;
        }
        named_bar_sync(1, NCT);

        int rpos[RPL];  // positions of this lane's S-phase rows (-1: padding)
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
            const int R = mt * RT + rh + 2 * i;
            rpos[i] = R < rows_b ? pos0 + R / G : -1;
        }
        float o[RT][DPL];
        float m[RT];
#pragma unroll
        for (int r = 0; r < RT; ++r) {
            m[r] = -INFINITY;
#pragma unroll
            for (int j = 0; j < DPL; ++j) o[r][j] = 0.f;
        }
        float l[RPL];
#pragma unroll
        for (int i = 0; i < RPL; ++i) l[i] = 0.f;

        for (int k = ((ks - ibase) % KS + KS) % KS; k < seg.cnt; k += KS) {
            const int it = ibase + k;
            const int st = it % STAGES;
            bool ok = !*s_abort;
            if (ok) ok = mbar_wait_bounded(&full_bar[st], (it / STAGES) & 1, s_abort, p.wait_ns);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !*s_abort) {
                    *s_abort = 1;
                    raise_flag(CX_DEV_WAIT_TIMEOUT);
                }
            } else if (!s_bad[st]) {  // a bad block id: its keys are left out
                const unsigned char* kb = ring + (size_t)st * C::STAGE;
                // ---- S = Q K^T for key t, rows rh + 2 i ----
                float sa[RPL], sb[RPL];
#pragma unroll
                for (int i = 0; i < RPL; ++i) sa[i] = sb[i] = 0.f;
#pragma unroll
                for (int c = 0; c < D / 4; ++c) {
                    const float4 kv = *reinterpret_cast<const float4*>(kb + C::off(hh, t, c));
#pragma unroll
                    for (int i = 0; i < RPL; ++i) {
                        const float4 qv =
                            *reinterpret_cast<const float4*>(qw + (rh + 2 * i) * C::QROW + 4 * c);
                        float& acc = (c & 1) ? sb[i] : sa[i];
                        acc = fmaf(qv.x, kv.x, acc);
                        acc = fmaf(qv.y, kv.y, acc);
                        acc = fmaf(qv.z, kv.z, acc);
                        acc = fmaf(qv.w, kv.w, acc);
                    }
                }
                const int t0 = (seg.j0 + k) * kBlockTok;
                const bool edge =
                    (t0 + kBlockTok - 1 > pos0) || (p.window > 0 && t0 <= ctx - 1 - p.window);
                float x[RPL], mx[RPL];
#pragma unroll
                for (int i = 0; i < RPL; ++i) {
                    x[i] = (sa[i] + sb[i]) * p.scale_log2;
                    if (edge) {
                        const int tok = t0 + t;
                        if (!(tok <= rpos[i] && (p.window <= 0 || tok > rpos[i] - p.window)))
                            x[i] = -INFINITY;
                    }
                    float v = x[i];
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
                    mx[i] = v;
                }
                // every row's block max in every lane: row 2 i + h comes from half h
                float a[RT];
                bool grow = false;
#pragma unroll
                for (int i = 0; i < RPL; ++i) {
                    const float other = __shfl_xor_sync(0xffffffffu, mx[i], 16);
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        const int r = 2 * i + h2;
                        const float bm = (h2 == rh) ? mx[i] : other;
                        const bool g = bm > m[r] + kMmaRescaleLog2 ||
                                       (m[r] == -INFINITY && bm > -INFINITY);
                        const float mn = g ? bm : m[r];
                        a[r] = g ? exp2f(m[r] - (mn == -INFINITY ? 0.f : mn)) : 1.f;
                        m[r] = mn;
                        grow |= g;
                    }
                }
#pragma unroll
                for (int i = 0; i < RPL; ++i) {
                    const float mo = rh ? m[2 * i + 1] : m[2 * i];
                    const float ao = rh ? a[2 * i + 1] : a[2 * i];
                    const float pr = ex2_approx(x[i] - (mo == -INFINITY ? 0.f : mo));
                    l[i] = l[i] * ao + pr;
                    pw[(rh + 2 * i) * 16 + t] = pr;
                }
                if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                    for (int r = 0; r < RT; ++r)
#pragma unroll
                        for (int j = 0; j < DPL; ++j) o[r][j] *= a[r];
                }
                __syncwarp();
                // ---- O += P V over the 16 keys of the unit ----
                const unsigned char* vb = kb + C::TILES;
#pragma unroll
                for (int t4 = 0; t4 < kBlockTok; t4 += 4) {
                    float4 pr[RT];
#pragma unroll
                    for (int r = 0; r < RT; ++r)
                        pr[r] = *reinterpret_cast<const float4*>(pw + r * 16 + t4);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        float vv[DPL];
                        const unsigned char* va = vb + C::off(hh, t4 + u, v_chunk) + v_byte;
                        if constexpr (DPL == 4) {
                            const float4 w = *reinterpret_cast<const float4*>(va);
                            vv[0] = w.x; vv[1] = w.y; vv[2] = w.z; vv[3] = w.w;
                        } else {
                            const float2 w = *reinterpret_cast<const float2*>(va);
                            vv[0] = w.x; vv[1] = w.y;
                        }
#pragma unroll
                        for (int r = 0; r < RT; ++r) {
                            const float pu = u == 0 ? pr[r].x : u == 1 ? pr[r].y
                                           : u == 2 ? pr[r].z : pr[r].w;
#pragma unroll
                            for (int j = 0; j < DPL; ++j) o[r][j] = fmaf(pu, vv[j], o[r][j]);
                        }
                    }
                }
                __syncwarp();  // P read before the next unit overwrites it
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[st]);
        }
        ibase += seg.cnt;

        // ---- finish this (sequence, head group) range ----
        // row denominators: sum the 16 keys' partial sums of each half, then
        // every row in every lane
        float la[RT];
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
            float v = l[i];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            const float other = __shfl_xor_sync(0xffffffffu, v, 16);
            la[2 * i] = rh ? other : v;
            la[2 * i + 1] = rh ? v : other;
        }
        float* mrow = merge + ((size_t)ks * HG + hh) * p.rows * (D + 2);
#pragma unroll
        for (int r = 0; r < RT; ++r) {
            const int R = mt * RT + r;
            if (R >= rows_b) continue;
            float* rr = mrow + (size_t)R * (D + 2);
#pragma unroll
            for (int j = 0; j < DPL; j += 2)
                *reinterpret_cast<float2*>(rr + d0 + j) = make_float2(o[r][j], o[r][j + 1]);
            if (lane == 0) {
                rr[D] = m[r];
                rr[D + 1] = la[r];
            }
        }
        const int bg = b * p.n_groups + seg.g;
        float* slot = p.partials + (size_t)(blockIdx.x + bg) * slot_floats;
        ks_merge<D, HG>(p, merge, slot, seg, qs, rows_b, ctid, NCT, KS);
        if (!seg.whole) ticket_merge<D, HG>(p, seg, b, qs, rows_b, ctid, NCT, chunk, s_last);
        named_bar_sync(1, NCT);
    }
}

}  // namespace cx
