// Generic exact-fp32 attention over a paged pool or dense K/V arrays.
//
// One warp owns one query row (query token i of sequence b, query head hq)
// and streams its attendable keys with a per-key online softmax (running max
// m, running denominator l, rescaled accumulator acc), accumulating in fp32
// with expf.  This is the path for fp32 / fp16 pools, head dims up to 256,
// any block size, explicit boolean masks and the dense flash_attention API;
// bf16 pools with 16-token blocks and head_dim 64/128 take the tensor-core
// kernel in attn_paged_mma.cuh instead.
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

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

template <typename QT, typename KT, bool PAGED>
__global__ void __launch_bounds__(128) attn_generic_kernel(GenericParams p) {
    constexpr int MAXE = 8;  // head_dim <= 256
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t b = blockIdx.x / p.hk, kh = blockIdx.x % p.hk;
    const int64_t G = p.hq / p.hk;

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
    } else {
        sk = p.sk;
        sq = p.max_q;
        q0 = 0;
    }
    const int64_t rows = sq * G;
    const int64_t rows_per_cta = 4 * 4;
    const QT* qb = static_cast<const QT*>(p.q);
    const int32_t* table = PAGED ? p.tables + b * p.table_stride : nullptr;

    for (int64_t r = blockIdx.y * rows_per_cta + warp; r < rows && r < (blockIdx.y + 1) * rows_per_cta;
         r += 4) {
        const int64_t i = r / G, g = r % G, h = kh * G + g;
        // query / output row offsets (elements)
        int64_t qoff, ooff;
        if (PAGED) {
            qoff = ((q0 + i) * p.hq + h) * p.d;
            ooff = ((q0 + i) * p.hq + h) * p.dv;
        } else {
            qoff = ((b * p.hq + h) * sq + i) * p.d;
            ooff = ((b * p.hq + h) * sq + i) * p.dv;
        }
        float qv[MAXE], acc[MAXE];
#pragma unroll
        for (int e = 0; e < MAXE; ++e) {
            const int64_t dd = lane + 32 * e;
            qv[e] = dd < p.d ? Conv<QT>::to_f(qb[qoff + dd]) : 0.f;
            acc[e] = 0.f;
        }
        // attendable key range for this row
        const int64_t pos = sk - sq + i;
        int64_t lo = 0, hi = sk - 1;
        if (p.mask_kind == 1) {
            hi = pos < hi ? pos : hi;
            if (p.window > 0) {
                const int64_t w0 = pos - p.window + 1;
                lo = w0 > 0 ? w0 : 0;
            }
        }
        float m = -INFINITY, l = 0.f;
        for (int64_t j = lo; j <= hi; ++j) {
            if (p.mask_kind == 2 && !p.mask[i * sk + j]) continue;
            const KT* kr;
            const KT* vr;
            if (PAGED) {
                const int64_t blk = table[j / p.block_size];
                if (blk < 0 || blk >= p.n_blocks) {
                    if (lane == 0) raise_flag(CX_DEV_BAD_BLOCK);
                    continue;
                }
                const int64_t off =
                    ((((p.layer * p.n_blocks + blk) * p.hk + kh) * p.block_size) +
                     (j % p.block_size)) * p.d;
                kr = static_cast<const KT*>(p.kp) + off;
                vr = static_cast<const KT*>(p.vp) + off;
            } else {
                kr = static_cast<const KT*>(p.k) + ((b * p.hk + kh) * sk + j) * p.d;
                vr = static_cast<const KT*>(p.v) + ((b * p.hk + kh) * sk + j) * p.dv;
            }
            float dot = 0.f;
#pragma unroll
            for (int e = 0; e < MAXE; ++e) {
                const int64_t dd = lane + 32 * e;
                if (dd < p.d) dot = fmaf(qv[e], Conv<KT>::to_f(kr[dd]), dot);
            }
            const float s = warp_sum(dot) * p.scale;
            const float m_new = fmaxf(m, s);
            const float corr = expf(m - m_new);
            const float pr = expf(s - m_new);
            l = l * corr + pr;
#pragma unroll
            for (int e = 0; e < MAXE; ++e) {
                const int64_t dd = lane + 32 * e;
                if (dd < p.dv) acc[e] = fmaf(pr, Conv<KT>::to_f(vr[dd]), acc[e] * corr);
            }
            m = m_new;
        }
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int e = 0; e < MAXE; ++e) {
            const int64_t dd = lane + 32 * e;
            if (dd < p.dv) p.out[ooff + dd] = acc[e] * inv;
        }
    }
}

template <bool PAGED, typename QT>
static int launch_generic_kv(int32_t kvdt, const GenericParams& p, dim3 grid, cudaStream_t st) {
    switch (kvdt) {
        case CX_F32: attn_generic_kernel<QT, float, PAGED><<<grid, 128, 0, st>>>(p); break;
        case CX_BF16: attn_generic_kernel<QT, __nv_bfloat16, PAGED><<<grid, 128, 0, st>>>(p); break;
        case CX_F16: attn_generic_kernel<QT, __half, PAGED><<<grid, 128, 0, st>>>(p); break;
        default: return fail(CX_ERR_DTYPE, "attention: unknown K/V dtype");
    }
    return check_launch("attn_generic_kernel");
}

template <bool PAGED>
static int launch_generic(int32_t qdt, int32_t kvdt, const GenericParams& p, cudaStream_t st) {
    const int64_t G = p.hq / p.hk;
    const int64_t rows = G * p.max_q;
    const int64_t gy = (rows + 15) / 16;
    if (p.batch * p.hk > 0x7fffffff || gy > 65535)
        return fail(CX_ERR_UNSUPPORTED, "attention: grid too large for the generic kernel");
    dim3 grid((unsigned)(p.batch * p.hk), (unsigned)gy);
    switch (qdt) {
        case CX_F32: return launch_generic_kv<PAGED, float>(kvdt, p, grid, st);
        case CX_BF16: return launch_generic_kv<PAGED, __nv_bfloat16>(kvdt, p, grid, st);
        case CX_F16: return launch_generic_kv<PAGED, __half>(kvdt, p, grid, st);
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
