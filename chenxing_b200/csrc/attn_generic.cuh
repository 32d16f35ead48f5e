// Generic exact-fp32 attention over a paged pool or dense K/V arrays: the
// path for fp16 pools, block sizes other than 16, head dims other than 64 /
// 128 (up to 256, also dv != d), fp32 verify chains beyond 64 packed rows,
// explicit boolean masks and the dense flash_attention API.  bf16 and fp32
// pools with 16-token blocks and head_dim 64 / 128 take the TMA kernels of
// attn_paged_mma.cuh / attn_paged_f32.cuh instead.
//
// One CTA per (sequence, KV head, tile of up to 8 packed rows; row = query
// token * G + head-in-group, so the G query heads of a KV head share every
// K/V read), four warps that split the key range into 16-key tiles (warp w
// takes tiles w, w + 4, ...).  Per tile a warp stages K and V (converted to
// fp32) in its own shared-memory buffers with coalesced loads, then
//   * lane (key j = lane % 16, parity = lane / 16) scores key j against rows
//     parity, parity + 2, ... (query rows broadcast from shared memory);
//   * row maxima over the 16 keys by xor shuffles, exchanged between the two
//     half-warps, and an online softmax with expf (running max m, running
//     denominator l, rescaled accumulator);
//   * lane owns output columns lane, lane + 32, ...: acc[r] += p[r][j] V[j].
// The four warps' partial states are merged through shared memory at the end
// (log-sum-exp), in a fixed order.
#include <math.h>

#include "cx_common.cuh"  // unity build: included from cxkv.cu

namespace cx {

struct GenericParams {
    // queries / output
    const void* q;
    float* out;
    int64_t batch, hq, hk, d, dv;
    int64_t max_q;  // rows per (b, head): sq for dense, max_q_len for paged
    float scale;
    int32_t mask_kind;  // 0 none, 1 causal(+window), 2 explicit
    int64_t window;     // <= 0: none
    const uint8_t* mask;  // [sq][sk] for mask_kind 2
    // dense K/V
    const void* k;
    const void* v;
    int64_t sk;
    // paged K/V
    const void* kp;
    const void* vp;
    int64_t n_layers, n_blocks, block_size, layer;
    const int32_t* tables;
    int64_t table_stride;
    const int32_t* ctx_lens;
    const int32_t* q_start;  // NULL: one query per sequence
};

constexpr int kGenRows = 8;     // packed rows per CTA
constexpr int kGenWarps = 4;    // key-splitting warps per CTA
constexpr int kGenKeys = 16;    // keys per tile
constexpr int kGenMaxE = 8;     // output columns per lane (dv <= 256)

// Shared memory of one CTA (floats): query rows [8][qs], then per warp a K
// tile [16][ks] and a V tile [16][dv] and a P tile [8][16]; the merge area
// [4][8][dv + 2] reuses the warps' buffers after the key loop.
struct GenSmem {
    int qs, ks, per_warp;
    bool v4;  // head_dim % 4 == 0: 16-byte rows, scores read as float4
    __host__ __device__ static GenSmem of(int64_t d, int64_t dv) {
        GenSmem g;
        g.v4 = d % 4 == 0;
        // Row strides that keep the reads of a key tile conflict-free (lanes j =
        // 0..7 of a phase read 16-byte chunk c of rows j: stride / 4 odd puts
        // them in distinct 16-byte bank groups; scalar reads need an odd
        // stride) and the two half-warps' broadcast query rows apart.
        g.qs = g.v4 ? (int)(d + (d % 8 == 0 ? 4 : 8)) : (int)(d % 2 == 0 ? d + 1 : d);
        g.ks = g.qs;
        g.per_warp = (kGenKeys * g.ks + kGenKeys * (int)dv + kGenRows * kGenKeys + 3) / 4 * 4;
        return g;
    }
    __host__ __device__ size_t bytes(int64_t dv) const {
        const size_t tiles = (size_t)kGenRows * qs + (size_t)kGenWarps * per_warp;
        const size_t merge = (size_t)kGenWarps * kGenRows * (dv + 2);
        return 4 * (tiles > merge + (size_t)kGenRows * qs ? tiles : merge + (size_t)kGenRows * qs);
    }
};

template <typename QT, typename KT, bool PAGED>
__global__ void __launch_bounds__(kGenWarps * 32) attn_generic_kernel(GenericParams p) {
    extern __shared__ float gsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t b = blockIdx.x / p.hk, kh = blockIdx.x % p.hk;
    const int G = (int)(p.hq / p.hk);
    const int D = (int)p.d, DV = (int)p.dv;
    const GenSmem L = GenSmem::of(p.d, p.dv);

    int64_t sq, sk, q0;
    if (PAGED) {
        sk = p.ctx_lens[b];
        q0 = p.q_start ? p.q_start[b] : b;
        sq = p.q_start ? (p.q_start[b + 1] - q0) : 1;
        if (sk > p.table_stride * p.block_size) {
            if (threadIdx.x == 0 && blockIdx.y == 0) raise_flag(CX_DEV_TABLE_OVERRUN);
            sk = p.table_stride * p.block_size;
        }
        if (((sk > 0 && sq > sk) || sq > p.max_q) && threadIdx.x == 0 && blockIdx.y == 0)
            raise_flag(CX_DEV_BAD_QLEN);
        if (sq > p.max_q) sq = p.max_q;
        if (sq < 0) sq = 0;
    } else {
        sk = p.sk;
        sq = p.max_q;
        q0 = 0;
    }
    const int64_t rows = sq * G;
    const int64_t r0 = (int64_t)blockIdx.y * kGenRows;
    if (r0 >= rows) return;
    const int nr = (int)min((int64_t)kGenRows, rows - r0);   // rows of this CTA
    const QT* qb = static_cast<const QT*>(p.q);
    const int32_t* table = PAGED ? p.tables + b * p.table_stride : nullptr;

    // ---- query rows (fp32, zero padding) and each row's attendable range ----
    float* s_q = gsm;
    for (int e = threadIdx.x; e < kGenRows * D; e += blockDim.x) {
        const int r = e / D, d = e % D;
        float v = 0.f;
        if (r < nr) {
            const int64_t R = r0 + r, i = R / G, h = kh * G + R % G;
            const int64_t qoff = PAGED ? ((q0 + i) * p.hq + h) * p.d
                                       : ((b * p.hq + h) * sq + i) * p.d;
            v = Conv<QT>::to_f(qb[qoff + d]);
        }
        s_q[r * L.qs + d] = v;
    }
    // key range over all rows of the CTA: [lo_all, hi_all]
    int64_t lo_all = sk, hi_all = -1;
    for (int r = 0; r < nr; ++r) {
        const int64_t i = (r0 + r) / G, pos = sk - sq + i;
        int64_t lo = 0, hi = sk - 1;
        if (p.mask_kind == 1) {
            hi = pos < hi ? pos : hi;
            if (p.window > 0) lo = pos - p.window + 1 > 0 ? pos - p.window + 1 : 0;
        }
        if (hi >= lo) {
            lo_all = lo < lo_all ? lo : lo_all;
            hi_all = hi > hi_all ? hi : hi_all;
        }
    }
    __syncthreads();

    // 16-byte row copies: rows a multiple of 16 bytes on 16-byte-aligned bases
    constexpr int kEPC = 16 / (int)sizeof(KT);
    const uintptr_t kv_al = reinterpret_cast<uintptr_t>(PAGED ? p.kp : p.k) |
                            reinterpret_cast<uintptr_t>(PAGED ? p.vp : p.v);
    const bool vec_rows = L.v4 && D % kEPC == 0 && DV % kEPC == 0 && (kv_al & 15) == 0;
    float* s_k = gsm + kGenRows * L.qs + (size_t)warp * L.per_warp;
    float* s_v = s_k + kGenKeys * L.ks;
    float* s_p = s_v + kGenKeys * DV;
    const int j = lane & 15, rh = lane >> 4;

    float m[kGenRows], l[kGenRows / 2], acc[kGenRows][kGenMaxE];
#pragma unroll
    for (int r = 0; r < kGenRows; ++r) {
        m[r] = -INFINITY;
#pragma unroll
        for (int e = 0; e < kGenMaxE; ++e) acc[r][e] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < kGenRows / 2; ++i) l[i] = 0.f;

    const int64_t t_first = hi_all >= lo_all ? lo_all / kGenKeys : 0;
    const int64_t t_end = hi_all >= lo_all ? hi_all / kGenKeys + 1 : 0;
    for (int64_t t = t_first + warp; t < t_end; t += kGenWarps) {
        const int64_t k0 = t * kGenKeys;
        // ---- stage K and V of keys k0 .. k0 + 15 (fp32; keys outside [0, sk)
        // or in a bad block: zeros, and marked invalid).  Lane jj < 16 finds
        // key k0 + jj's row offset (one table lookup a key); the rows are then
        // copied by all lanes, 16 bytes a load where the rows allow. ----
        int64_t my_off = -1;
        if (lane < kGenKeys) {
            const int64_t key = k0 + lane;
            if (key < sk) {
                if (PAGED) {
                    // 32-bit division: contexts and block sizes are below 2^31
                    const uint32_t kq = (uint32_t)key / (uint32_t)p.block_size;
                    const uint32_t kr = (uint32_t)key - kq * (uint32_t)p.block_size;
                    const int64_t blk = table[kq];
                    if (blk < 0 || blk >= p.n_blocks)
                        raise_flag(CX_DEV_BAD_BLOCK);
                    else
                        my_off = (((p.layer * p.n_blocks + blk) * p.hk + kh) * p.block_size +
                                  kr) * p.d;
                } else {
                    my_off = (b * p.hk + kh) * sk + key;   // row index (times d or dv below)
                }
            }
        }
        const unsigned valid = __ballot_sync(0xffffffffu, my_off >= 0) & 0xffffu;
        const KT* kbase = static_cast<const KT*>(PAGED ? p.kp : p.k);
        const KT* vbase = static_cast<const KT*>(PAGED ? p.vp : p.v);
        if (vec_rows) {
            constexpr int EPC = 16 / (int)sizeof(KT);
            const int cpk = D / EPC, cpv = DV / EPC;
            const int n_chunks = kGenKeys * (cpk + cpv);
            // a warp-uniform trip count: the shuffle below needs every lane
            for (int c0 = 0; c0 < n_chunks; c0 += 32) {
                const int c = c0 + lane;
                const bool act = c < n_chunks;
                const bool is_v = c >= kGenKeys * cpk;
                const int cc = is_v ? c - kGenKeys * cpk : c;
                const int cpr = is_v ? cpv : cpk;
                const int jj = act ? cc / cpr : 0, ch = cc - jj * cpr;
                const int64_t off = __shfl_sync(0xffffffffu, my_off, jj);
                if (!act) continue;
                float x[EPC];
                if (off >= 0) {
                    const KT* src = is_v ? vbase + (PAGED ? off : off * p.dv)
                                         : kbase + (PAGED ? off : off * p.d);
                    const uint4 raw = *reinterpret_cast<const uint4*>(src + ch * EPC);
                    const KT* e = reinterpret_cast<const KT*>(&raw);
#pragma unroll
                    for (int q2 = 0; q2 < EPC; ++q2) x[q2] = Conv<KT>::to_f(e[q2]);
                } else {
#pragma unroll
                    for (int q2 = 0; q2 < EPC; ++q2) x[q2] = 0.f;
                }
                float* dst = is_v ? s_v + jj * DV + ch * EPC : s_k + jj * L.ks + ch * EPC;
#pragma unroll
                for (int q2 = 0; q2 < EPC; ++q2) dst[q2] = x[q2];
            }
        } else {
            for (int jj = 0; jj < kGenKeys; ++jj) {
                const int64_t off = __shfl_sync(0xffffffffu, my_off, jj);
                const KT* kr = off >= 0 ? kbase + (PAGED ? off : off * p.d) : nullptr;
                const KT* vr = off >= 0 ? vbase + (PAGED ? off : off * p.dv) : nullptr;
                for (int d = lane; d < D; d += 32) s_k[jj * L.ks + d] = kr ? Conv<KT>::to_f(kr[d]) : 0.f;
                for (int d = lane; d < DV; d += 32) s_v[jj * DV + d] = vr ? Conv<KT>::to_f(vr[d]) : 0.f;
            }
        }
        __syncwarp();
        // ---- scores of key j against rows rh, rh + 2, ... ----
        const int64_t key = k0 + j;
        float dot[kGenRows / 2];
#pragma unroll
        for (int i = 0; i < kGenRows / 2; ++i) dot[i] = 0.f;
        {
            const float* krow = s_k + j * L.ks;
            const float* qrow = s_q + rh * L.qs;
            if (L.v4) {
#pragma unroll 4
                for (int d = 0; d < D; d += 4) {
                    const float4 kv = *reinterpret_cast<const float4*>(krow + d);
#pragma unroll
                    for (int i = 0; i < kGenRows / 2; ++i) {
                        const float4 qv =
                            *reinterpret_cast<const float4*>(qrow + 2 * i * L.qs + d);
                        dot[i] = fmaf(qv.x, kv.x, dot[i]);
                        dot[i] = fmaf(qv.y, kv.y, dot[i]);
                        dot[i] = fmaf(qv.z, kv.z, dot[i]);
                        dot[i] = fmaf(qv.w, kv.w, dot[i]);
                    }
                }
            } else {
#pragma unroll 4
                for (int d = 0; d < D; ++d) {
                    const float kd = krow[d];
#pragma unroll
                    for (int i = 0; i < kGenRows / 2; ++i)
                        dot[i] = fmaf(qrow[2 * i * L.qs + d], kd, dot[i]);
                }
            }
        }
        float x[kGenRows / 2];
#pragma unroll
        for (int i = 0; i < kGenRows / 2; ++i) {
            const int r = rh + 2 * i;
            float sc = dot[i] * p.scale;
            bool ok = r < nr && ((valid >> j) & 1u);
            if (ok) {
                const int64_t iq = (r0 + r) / G, pos = sk - sq + iq;
                if (p.mask_kind == 1)
                    ok = key <= pos && (p.window <= 0 || key > pos - p.window);
                else if (p.mask_kind == 2)
                    ok = p.mask[iq * sk + key] != 0;
            }
            x[i] = ok ? sc : -INFINITY;
        }
        // ---- online softmax: row maxima over the tile, every row in every lane ----
        float bm[kGenRows];
#pragma unroll
        for (int i = 0; i < kGenRows / 2; ++i) {
            float v = x[i];
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
            const float o = __shfl_xor_sync(0xffffffffu, v, 16);
            bm[2 * i] = rh ? o : v;
            bm[2 * i + 1] = rh ? v : o;
        }
        float corr[kGenRows];
#pragma unroll
        for (int r = 0; r < kGenRows; ++r) {
            const float mn = fmaxf(m[r], bm[r]);
            corr[r] = mn == -INFINITY ? 1.f : expf(m[r] - mn);
            m[r] = mn;
        }
#pragma unroll
        for (int i = 0; i < kGenRows / 2; ++i) {
            const float mo = rh ? m[2 * i + 1] : m[2 * i];
            const float co = rh ? corr[2 * i + 1] : corr[2 * i];
            const float pr = x[i] == -INFINITY ? 0.f : expf(x[i] - mo);
            l[i] = l[i] * co + pr;
            s_p[(rh + 2 * i) * kGenKeys + j] = pr;
        }
        __syncwarp();
        // ---- acc[r] = acc[r] * corr[r] + sum_j p[r][j] V[j] ----
#pragma unroll
        for (int r = 0; r < kGenRows; ++r)
#pragma unroll
            for (int e = 0; e < kGenMaxE; ++e) acc[r][e] *= corr[r];
        for (int jj = 0; jj < kGenKeys; ++jj) {
            if (!((valid >> jj) & 1u)) continue;
            float vv[kGenMaxE];
#pragma unroll
            for (int e = 0; e < kGenMaxE; ++e) {
                const int d = lane + 32 * e;
                vv[e] = d < DV ? s_v[jj * DV + d] : 0.f;
            }
#pragma unroll
            for (int r = 0; r < kGenRows; ++r) {
                const float pr = s_p[r * kGenKeys + jj];
#pragma unroll
                for (int e = 0; e < kGenMaxE; ++e) acc[r][e] = fmaf(pr, vv[e], acc[r][e]);
            }
        }
        __syncwarp();
    }
    // ---- row denominators, then the four warps' states merged in order ----
    float la[kGenRows];
#pragma unroll
    for (int i = 0; i < kGenRows / 2; ++i) {
        float v = l[i];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        const float o = __shfl_xor_sync(0xffffffffu, v, 16);
        la[2 * i] = rh ? o : v;
        la[2 * i + 1] = rh ? v : o;
    }
    __syncthreads();                                   // tiles no longer read
    float* s_m = gsm + kGenRows * L.qs;                // [warp][row][dv + 2]
    const int mrow = DV + 2;
#pragma unroll
    for (int r = 0; r < kGenRows; ++r) {
        float* dst = s_m + ((size_t)warp * kGenRows + r) * mrow;
#pragma unroll
        for (int e = 0; e < kGenMaxE; ++e) {
            const int d = lane + 32 * e;
            if (d < DV) dst[d] = acc[r][e];
        }
        if (lane == 0) {
            dst[DV] = m[r];
            dst[DV + 1] = la[r];
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nr * DV; e += blockDim.x) {
        const int r = e / DV, d = e % DV;
        float M = -INFINITY;
        for (int w = 0; w < kGenWarps; ++w) M = fmaxf(M, s_m[((size_t)w * kGenRows + r) * mrow + DV]);
        float Lsum = 0.f, O = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < kGenWarps; ++w) {
                const float* src = s_m + ((size_t)w * kGenRows + r) * mrow;
                const float wgt = expf(src[DV] - M);
                Lsum += src[DV + 1] * wgt;
                O += src[d] * wgt;
            }
        }
        const int64_t R = r0 + r, i = R / G, h = kh * G + R % G;
        const int64_t ooff = PAGED ? ((q0 + i) * p.hq + h) * p.dv : ((b * p.hq + h) * sq + i) * p.dv;
        p.out[ooff + d] = Lsum > 0.f ? O / Lsum : 0.f;
    }
}

template <bool PAGED, typename QT>
static int launch_generic_kv(int32_t kvdt, const GenericParams& p, dim3 grid, size_t smem,
                             cudaStream_t st) {
    switch (kvdt) {
        case CX_F32: {
            auto k = attn_generic_kernel<QT, float, PAGED>;
            CX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            k<<<grid, kGenWarps * 32, smem, st>>>(p);
            break;
        }
        case CX_BF16: {
            auto k = attn_generic_kernel<QT, __nv_bfloat16, PAGED>;
            CX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            k<<<grid, kGenWarps * 32, smem, st>>>(p);
            break;
        }
        case CX_F16: {
            auto k = attn_generic_kernel<QT, __half, PAGED>;
            CX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            k<<<grid, kGenWarps * 32, smem, st>>>(p);
            break;
        }
        default: return fail(CX_ERR_DTYPE, "attention: unknown K/V dtype");
    }
    return check_launch("attn_generic_kernel");
}

template <bool PAGED>
static int launch_generic(int32_t qdt, int32_t kvdt, const GenericParams& p, cudaStream_t st) {
    const int64_t G = p.hq / p.hk;
    const int64_t rows = G * p.max_q;
    const int64_t gy = (rows + kGenRows - 1) / kGenRows;
    if (p.batch * p.hk > 0x7fffffff || gy > 65535)
        return fail(CX_ERR_UNSUPPORTED, "attention: grid too large for the generic kernel");
    if (gy == 0) return CX_OK;
    const size_t smem = GenSmem::of(p.d, p.dv).bytes(p.dv);
    dim3 grid((unsigned)(p.batch * p.hk), (unsigned)gy);
    switch (qdt) {
        case CX_F32: return launch_generic_kv<PAGED, float>(kvdt, p, grid, smem, st);
        case CX_BF16: return launch_generic_kv<PAGED, __nv_bfloat16>(kvdt, p, grid, smem, st);
        case CX_F16: return launch_generic_kv<PAGED, __half>(kvdt, p, grid, smem, st);
        default: return fail(CX_ERR_DTYPE, "attention: unknown query dtype");
    }
}

}  // namespace cx

extern "C" int cx_attention_dense(const void* q, int32_t q_dtype, const void* k, const void* v,
                                  int32_t kv_dtype, int64_t b, int64_t hq, int64_t sq, int64_t hk,
                                  int64_t sk, int64_t d, int64_t dv, int32_t mask_kind,
                                  int64_t window, const uint8_t* mask, float scale, float* out,
                                  void* stream) {
    using namespace cx;
    if (b < 0 || sq < 0 || sk < 0) return fail(CX_ERR_SHAPE, "cx_attention_dense: negative size");
    if (hq <= 0 || hk <= 0 || d <= 0 || dv <= 0)
        return fail(CX_ERR_SHAPE, "cx_attention_dense: sizes must be positive");
    if (hq % hk != 0)
        return fail(CX_ERR_SHAPE, "cx_attention_dense: GQA requires hq % hk == 0");
    if (d > 256 || dv > 256)
        return fail(CX_ERR_UNSUPPORTED, "cx_attention_dense: head_dim above 256");
    if (mask_kind < 0 || mask_kind > 2) return fail(CX_ERR_SHAPE, "cx_attention_dense: mask_kind");
    if (mask_kind == 2 && !mask && sq * sk > 0)
        return fail(CX_ERR_SHAPE, "cx_attention_dense: explicit mask is NULL");
    if (b == 0 || sq == 0) return CX_OK;
    if (!q || !out || (sk > 0 && (!k || !v))) return fail(CX_ERR_SHAPE, "cx_attention_dense: NULL");
    GenericParams p{};
    p.q = q;
    p.out = out;
    p.batch = b;
    p.hq = hq;
    p.hk = hk;
    p.d = d;
    p.dv = dv;
    p.max_q = sq;
    p.scale = isnan(scale) ? 1.0f / sqrtf((float)d) : scale;
    p.mask_kind = mask_kind;
    p.window = window;
    p.mask = mask;
    p.k = k;
    p.v = v;
    p.sk = sk;
    return launch_generic<false>(q_dtype, kv_dtype, p, as_stream(stream));
}
