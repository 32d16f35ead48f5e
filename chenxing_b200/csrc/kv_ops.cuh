// KV pool data movement: slot-mapped append (+ copy-on-write of shared tail
// blocks), the read_layer gather, and whole/partial block copies.
// Pool layout: [n_layers][n_blocks][n_kv_heads][block_size][head_dim].
#include <type_traits>

#include "cx_common.cuh"  // unity build: included from cxkv.cu

namespace cx {

struct PoolGeom {
    int64_t n_layers, n_blocks, block_size, n_kv_heads, head_dim;
    // element offset of (layer, block, head, slot 0, dim 0)
    __host__ __device__ __forceinline__ int64_t tile(int64_t layer, int64_t block,
                                                     int64_t head) const {
        return (((layer * n_blocks + block) * n_kv_heads + head) * block_size) * head_dim;
    }
};

inline PoolGeom geom_of(const cx_pool* p) {
    return PoolGeom{p->n_layers, p->n_blocks, p->block_size, p->n_kv_heads, p->head_dim};
}

// Cooperative byte copy over `n` threads (thread index `i`), widest vector
// the alignment of both pointers and the length allow.
__device__ __forceinline__ void copy_bytes(char* dst, const char* src, int64_t nbytes, int i,
                                          int n) {
    uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
                  static_cast<uintptr_t>(nbytes);
    if ((a & 15) == 0) {
        const uint4* s = reinterpret_cast<const uint4*>(src);
        uint4* d = reinterpret_cast<uint4*>(dst);
        for (int64_t k = i; k < nbytes / 16; k += n) d[k] = s[k];
    } else if ((a & 3) == 0) {
        const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
        uint32_t* d = reinterpret_cast<uint32_t*>(dst);
        for (int64_t k = i; k < nbytes / 4; k += n) d[k] = s[k];
    } else {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
        uint16_t* d = reinterpret_cast<uint16_t*>(dst);
        for (int64_t k = i; k < nbytes / 2; k += n) d[k] = s[k];
    }
}

// One warp per job.  Jobs [0, n_tok*H) store token rows; jobs
// [n_tok*H, (n_tok+n_cow)*H) copy the valid prefix of a shared tail block.
template <typename S, typename P>
__global__ void __launch_bounds__(256) kv_append_kernel(
    P* __restrict__ kp, P* __restrict__ vp, PoolGeom g, int64_t layer,
    const S* __restrict__ kn, const S* __restrict__ vn, const int64_t* __restrict__ slots,
    int64_t n_tok, const int32_t* __restrict__ cow_src, const int32_t* __restrict__ cow_dst,
    const int32_t* __restrict__ cow_nv, int64_t n_cow) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t H = g.n_kv_heads, D = g.head_dim;
    const int64_t n_jobs = (n_tok + n_cow) * H;
    for (int64_t job = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); job < n_jobs;
         job += warps) {
        const int64_t h = job % H;
        const int64_t t = job / H;
        if (t < n_tok) {
            const int64_t slot = slots[t];
            if (slot < 0) continue;  // padding token
            if (slot >= g.n_blocks * g.block_size) {
                if (lane == 0) raise_flag(CX_DEV_BAD_SLOT);
                continue;
            }
            const int64_t blk = slot / g.block_size, off = slot % g.block_size;
            const int64_t dst = g.tile(layer, blk, h) + off * D;
            const int64_t src = (t * H + h) * D;
            for (int64_t d = lane; d < D; d += 32) {
                kp[dst + d] = Conv<P>::from_f(Conv<S>::to_f(kn[src + d]));
                vp[dst + d] = Conv<P>::from_f(Conv<S>::to_f(vn[src + d]));
            }
        } else {
            const int64_t c = t - n_tok;
            const int64_t sb = cow_src[c], db = cow_dst[c], nv = cow_nv[c];
            if (sb < 0 || sb >= g.n_blocks || db < 0 || db >= g.n_blocks || nv < 0 ||
                nv > g.block_size) {
                if (lane == 0) raise_flag(CX_DEV_BAD_BLOCK);
                continue;
            }
            const int64_t nbytes = nv * D * (int64_t)sizeof(P);
            copy_bytes(reinterpret_cast<char*>(kp + g.tile(layer, db, h)),
                       reinterpret_cast<const char*>(kp + g.tile(layer, sb, h)), nbytes, lane, 32);
            copy_bytes(reinterpret_cast<char*>(vp + g.tile(layer, db, h)),
                       reinterpret_cast<const char*>(vp + g.tile(layer, sb, h)), nbytes, lane, 32);
        }
    }
}

// 8 consecutive elements, loaded / converted / stored as 16-byte (32 for
// fp32) vectors.  Both pointers are 16-byte aligned (checked on the host).
template <typename T> struct Vec8;
template <> struct Vec8<float> {
    __device__ __forceinline__ static void load(const float* p, float (&x)[8]) {
        const float4 a = reinterpret_cast<const float4*>(p)[0];
        const float4 b = reinterpret_cast<const float4*>(p)[1];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    __device__ __forceinline__ static void store(float* p, const float (&x)[8]) {
        reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
    }
};
template <typename H> struct Vec8Half {
    __device__ __forceinline__ static void load(const H* p, float (&x)[8]) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const H* e = reinterpret_cast<const H*>(&u);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = Conv<H>::to_f(e[i]);
    }
    __device__ __forceinline__ static void store(H* p, const float (&x)[8]) {
        uint4 u;
        H* e = reinterpret_cast<H*>(&u);
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = Conv<H>::from_f(x[i]);
        *reinterpret_cast<uint4*>(p) = u;
    }
};
template <> struct Vec8<__nv_bfloat16> : Vec8Half<__nv_bfloat16> {};
template <> struct Vec8<__half> : Vec8Half<__half> {};

// Vector form of kv_append_kernel.  Copy-on-write jobs (the first nv slots
// of block cow_src[c] into block cow_dst[c], every head, K and V) run first,
// one warp per (job, head, K|V) region as 16-byte words; they touch slots
// [0, nv) of the destination block, and every token slot the same launch
// writes into that block is >= nv (checked on the host by the callers that
// build the slots), so the two never overlap.
// A CTA walks tokens t = blockIdx.x, blockIdx.x + gridDim.x, ...; its threads
// own fixed 8-element chunks of a token's rows (ordered head, K|V, chunk, so
// a warp writes whole contiguous rows), and each thread keeps kUnroll tokens'
// loads in flight before storing.  Same rounding as the scalar kernel (to
// float, then round-to-nearest-even to the pool type).  The host guarantees
// n_blocks * block_size < 2^31 (32-bit slot arithmetic).
template <typename S, typename P>
__global__ void __launch_bounds__(256) kv_append_vec_kernel(
    P* __restrict__ kp, P* __restrict__ vp, PoolGeom g, int64_t layer,
    const S* __restrict__ kn, const S* __restrict__ vn, const int64_t* __restrict__ slots,
    int64_t n_tok, const int32_t* __restrict__ cow_src, const int32_t* __restrict__ cow_dst,
    const int32_t* __restrict__ cow_nv, int64_t n_cow) {
    // same element type: move raw 16-byte words (no conversion, fewer
    // registers, more tokens in flight); otherwise convert through float
    constexpr bool kRaw = std::is_same<S, P>::value && sizeof(S) == 2;
    constexpr int kUnroll = kRaw ? 8 : 4;
    const int H = (int)g.n_kv_heads, D = (int)g.head_dim;
    if (n_cow > 0) {
        const int lane = threadIdx.x & 31;
        const int64_t wpb = blockDim.x >> 5;
        const int64_t regions = n_cow * H * 2;
        for (int64_t j = blockIdx.x * wpb + (threadIdx.x >> 5); j < regions;
             j += (int64_t)gridDim.x * wpb) {
            const int64_t c = j / (2 * H);
            const int h = (int)((j >> 1) % H);
            const int64_t sb = cow_src[c], db = cow_dst[c], nv = cow_nv[c];
            if (sb < 0 || sb >= g.n_blocks || db < 0 || db >= g.n_blocks || nv < 0 ||
                nv > g.block_size) {
                if (lane == 0) raise_flag(CX_DEV_BAD_BLOCK);
                continue;
            }
            P* base = (j & 1) ? vp : kp;
            const uint4* sw = reinterpret_cast<const uint4*>(base + g.tile(layer, sb, h));
            uint4* dw = reinterpret_cast<uint4*>(base + g.tile(layer, db, h));
            const int words = (int)(nv * D * (int64_t)sizeof(P) / 16);
            for (int w = lane; w < words; w += 32) dw[w] = sw[w];
        }
    }
    const int cpr = D / 8;                              // chunks per row
    const int per_tok = H * 2 * cpr;
    const uint32_t bs = (uint32_t)g.block_size;
    const int64_t cap = g.n_blocks * g.block_size;
    for (int c0 = threadIdx.x; c0 < per_tok; c0 += blockDim.x) {
        const int h = c0 / (2 * cpr);
        const int r = c0 - h * 2 * cpr;
        const bool is_v = r >= cpr;
        const int c = is_v ? r - cpr : r;
        const S* src = (is_v ? vn : kn) + (int64_t)h * D + c * 8;
        P* dstp = (is_v ? vp : kp) + g.tile(layer, 0, h) + c * 8;
        const int64_t blk_stride = g.n_kv_heads * g.block_size * g.head_dim;
        for (int64_t t0 = blockIdx.x; t0 < n_tok; t0 += (int64_t)gridDim.x * kUnroll) {
            float x[kRaw ? 1 : kUnroll][8];
            uint4 raw[kRaw ? kUnroll : 1];
            int64_t slot[kUnroll];
            // the row loads do not wait for the slot loads (a skipped token's
            // source row is still valid memory), so all of them are in flight
            // together
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int64_t t = t0 + (int64_t)u * gridDim.x;
                slot[u] = -1;
                if (t < n_tok) {
                    slot[u] = slots[t];
                    if constexpr (kRaw)
                        raw[u] = *reinterpret_cast<const uint4*>(src + t * H * D);
                    else
                        Vec8<S>::load(src + t * H * D, x[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                if (slot[u] >= cap) {
                    if (c0 == 0) raise_flag(CX_DEV_BAD_SLOT);
                    continue;
                }
                if (slot[u] < 0) continue;
                const uint32_t blk = (uint32_t)slot[u] / bs;
                const uint32_t off = (uint32_t)slot[u] - blk * bs;
                const int64_t dst = (int64_t)blk * blk_stride + (int64_t)off * D;
                if constexpr (kRaw)
                    *reinterpret_cast<uint4*>(dstp + dst) = raw[u];
                else
                    Vec8<P>::store(dstp + dst, x[u]);
            }
        }
    }
}

// RoPE + append: one thread per rotation pair of one row of one token; a
// token's rows are [Q heads | K heads | V heads].  Pair j is (j, j + D/2)
// (half-split) or (2j, 2j + 1) (interleaved).  Products and sums use the
// _rn intrinsics so no multiply-add is contracted: each output is the fp32
// value the reference's NumPy expression produces.
__device__ __forceinline__ void rope_pair(float a, float b, const float* c, const float* s,
                                          int j, int half, bool inter, float& oa, float& ob) {
    if (inter) {
        oa = __fsub_rn(__fmul_rn(a, c[j]), __fmul_rn(b, s[j]));
        ob = __fadd_rn(__fmul_rn(a, s[j]), __fmul_rn(b, c[j]));
    } else {
        oa = __fadd_rn(__fmul_rn(a, c[j]), __fmul_rn(-b, s[j]));
        ob = __fadd_rn(__fmul_rn(b, c[j + half]), __fmul_rn(a, s[j + half]));
    }
}

template <typename S, typename P, typename QO>
__global__ void __launch_bounds__(256) kv_append_rope_kernel(
    P* __restrict__ kp, P* __restrict__ vp, PoolGeom g, int64_t layer,
    const S* __restrict__ kn, const S* __restrict__ vn, const int64_t* __restrict__ slots,
    const int64_t* __restrict__ positions, int64_t n_tok, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, int64_t rows, int inter, const S* __restrict__ q,
    int hq, QO* __restrict__ q_out) {
    const int H = (int)g.n_kv_heads, D = (int)g.head_dim, half = D / 2;
    const int rows_tok = hq + 2 * H;
    const int64_t per_tok = (int64_t)rows_tok * half;
    const int64_t total = n_tok * per_tok;
    const int64_t cap = g.n_blocks * g.block_size;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        // token and item within it: a 32-bit division where the item count
        // allows (the 64-bit one is a long emulated sequence per item)
        int64_t t;
        int rem;
        if (total <= 0xffffffffll) {
            const uint32_t iu = (uint32_t)i, tu = iu / (uint32_t)per_tok;
            t = tu;
            rem = (int)(iu - tu * (uint32_t)per_tok);
        } else {
            t = i / per_tok;
            rem = (int)(i - t * per_tok);
        }
        const int row = rem / half, j = rem - row * half;
        const int64_t pos = positions[t];
        if (pos < 0 || pos >= rows) {
            if (rem == 0) raise_flag(CX_DEV_BAD_POSITION);
            continue;
        }
        const int ia = inter ? 2 * j : j, ib = inter ? 2 * j + 1 : j + half;
        if (row < hq) {                                   // Q -> q_out
            const S* x = q + (t * hq + row) * D;
            float oa, ob;
            rope_pair(Conv<S>::to_f(x[ia]), Conv<S>::to_f(x[ib]), cos_t + pos * D,
                      sin_t + pos * D, j, half, inter, oa, ob);
            QO* y = q_out + (t * hq + row) * D;
            y[ia] = Conv<QO>::from_f(oa);
            y[ib] = Conv<QO>::from_f(ob);
            continue;
        }
        const int64_t slot = slots[t];
        if (slot < 0) continue;                           // padding token
        if (slot >= cap) {
            if (rem == 0) raise_flag(CX_DEV_BAD_SLOT);
            continue;
        }
        const bool is_v = row >= hq + H;
        const int h = row - hq - (is_v ? H : 0);
        const int64_t dst = g.tile(layer, slot / g.block_size, h) + (slot % g.block_size) * D;
        const S* x = (is_v ? vn : kn) + (t * H + h) * D;
        const float a = Conv<S>::to_f(x[ia]), b = Conv<S>::to_f(x[ib]);
        P* y = (is_v ? vp : kp) + dst;
        if (is_v) {
            y[ia] = Conv<P>::from_f(a);
            y[ib] = Conv<P>::from_f(b);
        } else {
            float oa, ob;
            rope_pair(a, b, cos_t + pos * D, sin_t + pos * D, j, half, inter, oa, ob);
            y[ia] = Conv<P>::from_f(oa);
            y[ib] = Conv<P>::from_f(ob);
        }
    }
}

// Vector form of kv_append_rope_kernel: one thread per 8 rotation pairs of one
// row (pairs p .. p+7: elements p.. and p+half.. half-split, 2p .. 2p+15
// interleaved), 8-element vector accesses.  The position, slot and row loads
// are all issued before any of them is checked, so their latencies overlap;
// the cos / sin rows (shared by every row of the token, so cache hits) follow.
// The same _rn products and sums as rope_pair, so the same bits.  The host
// guarantees head_dim % 16 == 0, 16-byte aligned buffers and n_blocks *
// block_size < 2^31.
template <typename S, typename P, typename QO>
__global__ void __launch_bounds__(256) kv_append_rope_vec_kernel(
    P* __restrict__ kp, P* __restrict__ vp, PoolGeom g, int64_t layer,
    const S* __restrict__ kn, const S* __restrict__ vn, const int64_t* __restrict__ slots,
    const int64_t* __restrict__ positions, int64_t n_tok, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, int64_t rows, int inter, const S* __restrict__ q,
    int hq, QO* __restrict__ q_out) {
    const int H = (int)g.n_kv_heads, D = (int)g.head_dim, half = D / 2;
    const int gpr = half / 8;                             // 8-pair groups per row
    const int per_tok = (hq + 2 * H) * gpr;
    const int64_t total = n_tok * per_tok;
    const int64_t cap = g.n_blocks * g.block_size;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        // token and item within it: a 32-bit division where the item count
        // allows (the 64-bit one is a long emulated sequence per item)
        int64_t t;
        int rem;
        if (total <= 0xffffffffll) {
            const uint32_t iu = (uint32_t)i, tu = iu / (uint32_t)per_tok;
            t = tu;
            rem = (int)(iu - tu * (uint32_t)per_tok);
        } else {
            t = i / per_tok;
            rem = (int)(i - t * per_tok);
        }
        const int row = rem / gpr, p0 = (rem - row * gpr) * 8;
        const bool is_q = row < hq;
        const bool is_v = row >= hq + H;
        const int h = row - hq - (is_v ? H : 0);
        const int ea = inter ? 2 * p0 : p0, eb = inter ? 2 * p0 + 8 : p0 + half;
        const S* x = is_q ? q + (t * hq + row) * D : (is_v ? vn : kn) + (t * H + h) * D;
        // every load of this item first
        const int64_t pos = positions[t];
        const int64_t slot = is_q ? 0 : slots[t];
        float fa[8], fb[8];
        Vec8<S>::load(x + ea, fa);
        Vec8<S>::load(x + eb, fb);
        if (pos < 0 || pos >= rows) {
            if (rem == 0) raise_flag(CX_DEV_BAD_POSITION);
            continue;
        }
        int64_t dst = 0;
        if (!is_q) {
            if (slot < 0) continue;                       // padding token
            if (slot >= cap) {
                if (rem == 0) raise_flag(CX_DEV_BAD_SLOT);
                continue;
            }
            const uint32_t blk = (uint32_t)slot / (uint32_t)g.block_size;
            const uint32_t off = (uint32_t)slot - blk * (uint32_t)g.block_size;
            dst = g.tile(layer, blk, h) + (int64_t)off * D;
        }
        float a[8], b[8];
        if (inter) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                a[k] = fa[2 * k];
                b[k] = fa[2 * k + 1];
                a[k + 4] = fb[2 * k];
                b[k + 4] = fb[2 * k + 1];
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                a[k] = fa[k];
                b[k] = fb[k];
            }
        }
        float oa[8], ob[8];
        if (is_v) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                oa[k] = a[k];
                ob[k] = b[k];
            }
        } else {
            const float* cr = cos_t + pos * D;
            const float* sr = sin_t + pos * D;
            float c0[8], s0[8];
            Vec8<float>::load(cr + p0, c0);
            Vec8<float>::load(sr + p0, s0);
            if (inter) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    oa[k] = __fsub_rn(__fmul_rn(a[k], c0[k]), __fmul_rn(b[k], s0[k]));
                    ob[k] = __fadd_rn(__fmul_rn(a[k], s0[k]), __fmul_rn(b[k], c0[k]));
                }
            } else {
                float c1[8], s1[8];
                Vec8<float>::load(cr + p0 + half, c1);
                Vec8<float>::load(sr + p0 + half, s1);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    oa[k] = __fadd_rn(__fmul_rn(a[k], c0[k]), __fmul_rn(-b[k], s0[k]));
                    ob[k] = __fadd_rn(__fmul_rn(b[k], c1[k]), __fmul_rn(a[k], s1[k]));
                }
            }
        }
        auto put = [&](auto* y) {
            using T = typename std::remove_pointer<decltype(y)>::type;
            if (inter) {
                float e0[8], e1[8];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    e0[2 * k] = oa[k];
                    e0[2 * k + 1] = ob[k];
                    e1[2 * k] = oa[k + 4];
                    e1[2 * k + 1] = ob[k + 4];
                }
                Vec8<T>::store(y + ea, e0);
                Vec8<T>::store(y + eb, e1);
            } else {
                Vec8<T>::store(y + ea, oa);
                Vec8<T>::store(y + eb, ob);
            }
        };
        if (is_q)
            put(q_out + (t * hq + row) * D);
        else
            put((is_v ? vp : kp) + dst);
    }
}

// One warp per (token, head) row of the output.
__global__ void __launch_bounds__(256) kv_gather_kernel(
    const char* __restrict__ kp, const char* __restrict__ vp, PoolGeom g, int64_t layer,
    int eb, const int32_t* __restrict__ table, int64_t n_tok, char* __restrict__ ko,
    char* __restrict__ vo) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t H = g.n_kv_heads, D = g.head_dim;
    const int64_t row_bytes = D * eb;
    for (int64_t job = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
         job < n_tok * H; job += warps) {
        const int64_t h = job % H, t = job / H;
        const int64_t blk = table[t / g.block_size];
        if (blk < 0 || blk >= g.n_blocks) {
            if (lane == 0) raise_flag(CX_DEV_BAD_BLOCK);
            continue;
        }
        const int64_t src = (g.tile(layer, blk, h) + (t % g.block_size) * D) * eb;
        copy_bytes(ko + job * row_bytes, kp + src, row_bytes, lane, 32);
        copy_bytes(vo + job * row_bytes, vp + src, row_bytes, lane, 32);
    }
}

// One CTA per job = (pair, layer, head, K|V): slots [0, n_slots) of a tile.
__global__ void __launch_bounds__(256) block_copy_kernel(
    char* __restrict__ kp, char* __restrict__ vp, PoolGeom g, int eb,
    const int32_t* __restrict__ src, const int32_t* __restrict__ dst, int64_t n,
    int64_t n_slots) {
    const int64_t H = g.n_kv_heads;
    const int64_t n_jobs = n * g.n_layers * H * 2;
    const int64_t nbytes = n_slots * g.head_dim * eb;
    for (int64_t job = blockIdx.x; job < n_jobs; job += gridDim.x) {
        int64_t r = job;
        const int kv = (int)(r & 1);
        r >>= 1;
        const int64_t h = r % H;
        r /= H;
        const int64_t layer = r % g.n_layers;
        const int64_t i = r / g.n_layers;
        const int64_t sb = src[i], db = dst[i];
        if (sb < 0 || sb >= g.n_blocks || db < 0 || db >= g.n_blocks) {
            if (threadIdx.x == 0) raise_flag(CX_DEV_BAD_BLOCK);
            continue;
        }
        char* base = kv ? vp : kp;
        copy_bytes(base + g.tile(layer, db, h) * eb, base + g.tile(layer, sb, h) * eb, nbytes,
                   threadIdx.x, blockDim.x);
    }
}

// 16-byte variants of the two movers above (rows a multiple of 16 bytes,
// 16-byte aligned buffers).  A pool block's K (or V) rows of all heads are one
// contiguous region [H][block_size][D], so a job is a whole region where it
// can be: each thread keeps kMoveUnroll 16-byte loads of it in flight before
// its stores, and one block-id load serves the whole region.
constexpr int kMoveUnroll = 8;

// Block copy: job = (pair i, layer, head group, K|V) of `hj` heads' first
// n_slots rows; `hj` = H when whole blocks move (one contiguous region),
// else 1 (a partial tail per head).  `cj` = 16-byte chunks per job.
__global__ void __launch_bounds__(256) block_copy_vec_kernel(
    uint4* __restrict__ kp, uint4* __restrict__ vp, PoolGeom g, int eb,
    const int32_t* __restrict__ src, const int32_t* __restrict__ dst, int64_t n, int hj,
    int cj) {
    const uint32_t groups = (uint32_t)(g.n_kv_heads / hj);
    const int64_t n_jobs = n * g.n_layers * groups * 2;
    for (int64_t job = blockIdx.x; job < n_jobs; job += gridDim.x) {
        // 32-bit index math (the host guarantees n_jobs < 2^31)
        uint32_t r = (uint32_t)job >> 1;
        const uint32_t hg = r % groups;
        r /= groups;
        const uint32_t layer = r % (uint32_t)g.n_layers;
        const uint32_t i = r / (uint32_t)g.n_layers;
        const int64_t sb = src[i], db = dst[i];
        if (sb < 0 || sb >= g.n_blocks || db < 0 || db >= g.n_blocks) {
            if (threadIdx.x == 0) raise_flag(CX_DEV_BAD_BLOCK);
            continue;
        }
        uint4* base = (job & 1) ? vp : kp;
        const uint4* s = base + g.tile(layer, sb, (int64_t)hg * hj) * eb / 16;
        uint4* d = base + g.tile(layer, db, (int64_t)hg * hj) * eb / 16;
        // a head group's rows: hj tiles of cj / hj chunks, tile stride = a full tile
        const int per_tile = cj / hj;
        const int tile_chunks = (int)(g.block_size * g.head_dim * eb / 16);
        for (int k0 = threadIdx.x; k0 < cj; k0 += blockDim.x * kMoveUnroll) {
            uint4 buf[kMoveUnroll];
            int off[kMoveUnroll];
#pragma unroll
            for (int u = 0; u < kMoveUnroll; ++u) {
                const int k = k0 + u * blockDim.x;
                off[u] = -1;
                if (k < cj) {
                    const int tt = k / per_tile;
                    off[u] = tt * tile_chunks + (k - tt * per_tile);
                    buf[u] = s[off[u]];
                }
            }
#pragma unroll
            for (int u = 0; u < kMoveUnroll; ++u)
                if (off[u] >= 0) d[off[u]] = buf[u];
        }
    }
}

// read_layer gather: job = (table block jb, K|V): the block's contiguous
// [H][block_size][D] region is read in order and written to token rows
// [jb * block_size + slot][head][D] (rows past n_tok are skipped).
__global__ void __launch_bounds__(256) kv_gather_vec_kernel(
    const uint4* __restrict__ kp, const uint4* __restrict__ vp, PoolGeom g, int64_t layer,
    int eb, const int32_t* __restrict__ table, int64_t n_tok, uint4* __restrict__ ko,
    uint4* __restrict__ vo) {
    const int H = (int)g.n_kv_heads;
    const int bs = (int)g.block_size;
    const int cpr = (int)(g.head_dim * eb / 16);          // chunks per row
    const int cj = H * bs * cpr;                          // chunks per region
    const int64_t n_blk = (n_tok + bs - 1) / bs;
    for (int64_t job = blockIdx.x; job < 2 * n_blk; job += gridDim.x) {
        const int64_t jb = job >> 1;
        const int64_t blk = table[jb];
        if (blk < 0 || blk >= g.n_blocks) {
            if (threadIdx.x == 0) raise_flag(CX_DEV_BAD_BLOCK);
            continue;
        }
        const bool is_v = job & 1;
        const uint4* s = (is_v ? vp : kp) + g.tile(layer, blk, 0) * eb / 16;
        uint4* o = is_v ? vo : ko;
        const int rows = (int)min((int64_t)bs, n_tok - jb * bs);   // valid slots
        for (int k0 = threadIdx.x; k0 < cj; k0 += blockDim.x * kMoveUnroll) {
            uint4 buf[kMoveUnroll];
            int64_t dst[kMoveUnroll];
#pragma unroll
            for (int u = 0; u < kMoveUnroll; ++u) {
                const int k = k0 + u * blockDim.x;
                dst[u] = -1;
                if (k < cj) {
                    const int h = k / (bs * cpr);
                    const int rem = k - h * bs * cpr;
                    const int slot = rem / cpr, c = rem - slot * cpr;
                    if (slot < rows) {
                        dst[u] = ((jb * bs + slot) * H + h) * cpr + c;
                        buf[u] = s[k];
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < kMoveUnroll; ++u)
                if (dst[u] >= 0) o[dst[u]] = buf[u];
        }
    }
}

static int check_pool(const cx_pool* p) {
    if (!p) return fail(CX_ERR_SHAPE, "pool is NULL");
    if (!p->k || !p->v) return fail(CX_ERR_SHAPE, "pool buffers are NULL");
    if (p->n_layers <= 0 || p->n_blocks <= 0 || p->block_size <= 0 || p->n_kv_heads <= 0 ||
        p->head_dim <= 0)
        return fail(CX_ERR_SHAPE, "pool sizes must be positive");
    if (elem_bytes(p->dtype) == 0) return fail(CX_ERR_DTYPE, "unknown pool dtype");
    return CX_OK;
}

static int grid_for(int64_t work_items, int per_block) {
    int64_t b = (work_items + per_block - 1) / per_block;
    int64_t cap = (int64_t)num_sms() * 16;
    if (cap <= 0) cap = 2048;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

template <typename S, typename P>
static void launch_append(const cx_pool* p, int64_t layer, const void* k, const void* v,
                          const int64_t* slots, int64_t n_tok, const int32_t* cs,
                          const int32_t* cd, const int32_t* cn, int64_t n_cow, cudaStream_t st) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                         reinterpret_cast<uintptr_t>(p->k) | reinterpret_cast<uintptr_t>(p->v);
    if (p->head_dim % 8 == 0 && (al & 15) == 0 && p->n_blocks * p->block_size < (1ll << 31) &&
        p->n_kv_heads * 2 * (p->head_dim / 8) <= (1 << 20)) {
        const int64_t cap = (int64_t)num_sms() * 16;
        int64_t blocks = n_tok > n_cow * p->n_kv_heads / 4 ? n_tok : n_cow * p->n_kv_heads / 4;
        blocks = blocks < cap ? blocks : cap;
        if (blocks < 1) blocks = 1;
        kv_append_vec_kernel<S, P><<<(unsigned)blocks, 256, 0, st>>>(
            static_cast<P*>(p->k), static_cast<P*>(p->v), geom_of(p), layer,
            static_cast<const S*>(k), static_cast<const S*>(v), slots, n_tok, cs, cd, cn, n_cow);
        return;
    }
    const int64_t jobs = (n_tok + n_cow) * p->n_kv_heads;
    kv_append_kernel<S, P><<<grid_for(jobs, 8), 256, 0, st>>>(
        static_cast<P*>(p->k), static_cast<P*>(p->v), geom_of(p), layer,
        static_cast<const S*>(k), static_cast<const S*>(v), slots, n_tok, cs, cd, cn, n_cow);
}

template <typename P>
static int dispatch_append_src(int32_t sdt, const cx_pool* p, int64_t layer, const void* k,
                               const void* v, const int64_t* slots, int64_t n_tok,
                               const int32_t* cs, const int32_t* cd, const int32_t* cn,
                               int64_t n_cow, cudaStream_t st) {
    switch (sdt) {
        case CX_F32: launch_append<float, P>(p, layer, k, v, slots, n_tok, cs, cd, cn, n_cow, st); break;
        case CX_BF16: launch_append<__nv_bfloat16, P>(p, layer, k, v, slots, n_tok, cs, cd, cn, n_cow, st); break;
        case CX_F16: launch_append<__half, P>(p, layer, k, v, slots, n_tok, cs, cd, cn, n_cow, st); break;
        default: return fail(CX_ERR_DTYPE, "cx_kv_append: unknown source dtype");
    }
    return check_launch("kv_append_kernel");
}

}  // namespace cx

extern "C" {

int cx_kv_append(const cx_pool* pool, int64_t layer, const void* k_new, const void* v_new,
                 int32_t src_dtype, const int64_t* slot_mapping, int64_t n_tokens,
                 const int32_t* cow_src, const int32_t* cow_dst, const int32_t* cow_n_valid,
                 int64_t n_cow, void* stream) {
    using namespace cx;
    int rc = check_pool(pool);
    if (rc) return rc;
    if (layer < 0 || layer >= pool->n_layers)
        return fail(CX_ERR_RANGE, "cx_kv_append: layer out of range");
    if (n_tokens < 0 || n_cow < 0) return fail(CX_ERR_SHAPE, "cx_kv_append: negative count");
    if (n_tokens > 0 && (!k_new || !v_new || !slot_mapping))
        return fail(CX_ERR_SHAPE, "cx_kv_append: NULL token arrays");
    if (n_cow > 0 && (!cow_src || !cow_dst || !cow_n_valid))
        return fail(CX_ERR_SHAPE, "cx_kv_append: NULL copy-on-write arrays");
    if (n_tokens == 0 && n_cow == 0) return CX_OK;
    cudaStream_t st = as_stream(stream);
    switch (pool->dtype) {
        case CX_F32: return dispatch_append_src<float>(src_dtype, pool, layer, k_new, v_new, slot_mapping, n_tokens, cow_src, cow_dst, cow_n_valid, n_cow, st);
        case CX_BF16: return dispatch_append_src<__nv_bfloat16>(src_dtype, pool, layer, k_new, v_new, slot_mapping, n_tokens, cow_src, cow_dst, cow_n_valid, n_cow, st);
        case CX_F16: return dispatch_append_src<__half>(src_dtype, pool, layer, k_new, v_new, slot_mapping, n_tokens, cow_src, cow_dst, cow_n_valid, n_cow, st);
        default: return fail(CX_ERR_DTYPE, "cx_kv_append: unknown pool dtype");
    }
}

int cx_kv_append_rope(const cx_pool* pool, int64_t layer, const void* k_new, const void* v_new,
                      int32_t src_dtype, const int64_t* slot_mapping, const int64_t* positions,
                      int64_t n_tokens, const float* cos_table, const float* sin_table,
                      int64_t table_rows, int32_t interleaved, const void* q,
                      int64_t n_q_heads, void* q_out, int32_t q_out_dtype, void* stream) {
    using namespace cx;
    int rc = check_pool(pool);
    if (rc) return rc;
    if (layer < 0 || layer >= pool->n_layers)
        return fail(CX_ERR_RANGE, "cx_kv_append_rope: layer out of range");
    if (n_tokens < 0 || n_q_heads < 0 || table_rows < 0)
        return fail(CX_ERR_SHAPE, "cx_kv_append_rope: negative count");
    if (pool->head_dim % 2 != 0)
        return fail(CX_ERR_SHAPE, "cx_kv_append_rope: head_dim must be even");
    if (n_tokens == 0) return CX_OK;
    if (!k_new || !v_new || !slot_mapping || !positions || !cos_table || !sin_table)
        return fail(CX_ERR_SHAPE, "cx_kv_append_rope: NULL array");
    if (n_q_heads > 0 && (!q || !q_out))
        return fail(CX_ERR_SHAPE, "cx_kv_append_rope: n_q_heads > 0 needs q and q_out");
    if (n_q_heads > (1 << 20) || pool->n_kv_heads > (1 << 20))
        return fail(CX_ERR_UNSUPPORTED, "cx_kv_append_rope: too many heads");
    if (src_dtype != CX_F32 && src_dtype != CX_BF16)
        return fail(CX_ERR_DTYPE, "cx_kv_append_rope: source must be CX_F32 or CX_BF16");
    if (n_q_heads > 0 && q_out_dtype != CX_F32 && q_out_dtype != CX_BF16)
        return fail(CX_ERR_DTYPE, "cx_kv_append_rope: q_out must be CX_F32 or CX_BF16");
    const int64_t work = n_tokens * (n_q_heads + 2 * pool->n_kv_heads) * (pool->head_dim / 2);
    const int grid = grid_for(work, 256);
    cudaStream_t st = as_stream(stream);
    const int hq = (int)n_q_heads;
    auto go = [&](auto s_tag, auto p_tag, auto q_tag) {
        using S = decltype(s_tag);
        using P = decltype(p_tag);
        using QO = decltype(q_tag);
        const uintptr_t al = reinterpret_cast<uintptr_t>(pool->k) |
                             reinterpret_cast<uintptr_t>(pool->v) |
                             reinterpret_cast<uintptr_t>(k_new) |
                             reinterpret_cast<uintptr_t>(v_new) |
                             reinterpret_cast<uintptr_t>(cos_table) |
                             reinterpret_cast<uintptr_t>(sin_table) |
                             reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(q_out);
        if (pool->head_dim % 16 == 0 && (al & 15) == 0 &&
            pool->n_blocks * pool->block_size < (1ll << 31)) {
            kv_append_rope_vec_kernel<S, P, QO><<<grid_for(work / 8, 256), 256, 0, st>>>(
                static_cast<P*>(pool->k), static_cast<P*>(pool->v), geom_of(pool), layer,
                static_cast<const S*>(k_new), static_cast<const S*>(v_new), slot_mapping,
                positions, n_tokens, cos_table, sin_table, table_rows, interleaved ? 1 : 0,
                static_cast<const S*>(q), hq, static_cast<QO*>(q_out));
            return check_launch("kv_append_rope_vec_kernel");
        }
        kv_append_rope_kernel<S, P, QO><<<grid, 256, 0, st>>>(
            static_cast<P*>(pool->k), static_cast<P*>(pool->v), geom_of(pool), layer,
            static_cast<const S*>(k_new), static_cast<const S*>(v_new), slot_mapping, positions,
            n_tokens, cos_table, sin_table, table_rows, interleaved ? 1 : 0,
            static_cast<const S*>(q), hq, static_cast<QO*>(q_out));
        return check_launch("kv_append_rope_kernel");
    };
    auto with_q = [&](auto s_tag, auto p_tag) {
        return q_out_dtype == CX_BF16 ? go(s_tag, p_tag, __nv_bfloat16{}) : go(s_tag, p_tag, 0.f);
    };
    auto with_p = [&](auto s_tag) {
        switch (pool->dtype) {
            case CX_F32: return with_q(s_tag, 0.f);
            case CX_BF16: return with_q(s_tag, __nv_bfloat16{});
            case CX_F16: return with_q(s_tag, __half{});
            default: return fail(CX_ERR_DTYPE, "cx_kv_append_rope: unknown pool dtype");
        }
    };
    return src_dtype == CX_BF16 ? with_p(__nv_bfloat16{}) : with_p(0.f);
}

int cx_kv_gather(const cx_pool* pool, int64_t layer, const int32_t* block_table,
                 int64_t n_tokens, void* k_out, void* v_out, void* stream) {
    using namespace cx;
    int rc = check_pool(pool);
    if (rc) return rc;
    if (layer < 0 || layer >= pool->n_layers)
        return fail(CX_ERR_RANGE, "cx_kv_gather: layer out of range");
    if (n_tokens < 0) return fail(CX_ERR_SHAPE, "cx_kv_gather: negative n_tokens");
    if (n_tokens == 0) return CX_OK;
    if (!block_table || !k_out || !v_out) return fail(CX_ERR_SHAPE, "cx_kv_gather: NULL array");
    const int eb = elem_bytes(pool->dtype);
    const uintptr_t al = reinterpret_cast<uintptr_t>(pool->k) | reinterpret_cast<uintptr_t>(pool->v) |
                         reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out);
    if ((pool->head_dim * eb) % 16 == 0 && (al & 15) == 0 && n_tokens < (1ll << 31) &&
        pool->n_kv_heads * pool->block_size * (pool->head_dim * eb / 16) < (1ll << 30)) {
        const int64_t jobs = 2 * ((n_tokens + pool->block_size - 1) / pool->block_size);
        kv_gather_vec_kernel<<<grid_for(jobs, 1), 256, 0, as_stream(stream)>>>(
            static_cast<const uint4*>(pool->k), static_cast<const uint4*>(pool->v),
            geom_of(pool), layer, eb, block_table, n_tokens, static_cast<uint4*>(k_out),
            static_cast<uint4*>(v_out));
        return check_launch("kv_gather_vec_kernel");
    }
    kv_gather_kernel<<<grid_for(n_tokens * pool->n_kv_heads, 8), 256, 0, as_stream(stream)>>>(
        static_cast<const char*>(pool->k), static_cast<const char*>(pool->v), geom_of(pool), layer,
        eb, block_table, n_tokens, static_cast<char*>(k_out), static_cast<char*>(v_out));
    return check_launch("kv_gather_kernel");
}

int cx_block_copy(const cx_pool* pool, const int32_t* src, const int32_t* dst, int64_t n,
                  int64_t n_slots, void* stream) {
    using namespace cx;
    int rc = check_pool(pool);
    if (rc) return rc;
    if (n < 0 || n_slots < 0 || n_slots > pool->block_size)
        return fail(CX_ERR_SHAPE, "cx_block_copy: bad n or n_slots");
    if (n == 0 || n_slots == 0) return CX_OK;
    if (!src || !dst) return fail(CX_ERR_SHAPE, "cx_block_copy: NULL id arrays");
    const int64_t jobs = n * pool->n_layers * pool->n_kv_heads * 2;
    const int eb = elem_bytes(pool->dtype);
    const uintptr_t al = reinterpret_cast<uintptr_t>(pool->k) | reinterpret_cast<uintptr_t>(pool->v);
    const int64_t region = pool->n_kv_heads * pool->block_size * pool->head_dim * eb / 16;
    if ((pool->head_dim * eb) % 16 == 0 && (al & 15) == 0 && jobs < (1ll << 31) &&
        region < (1ll << 30)) {
        // whole blocks: one contiguous region per (pair, layer, K|V); a partial
        // tail: per head
        const int hj = n_slots == pool->block_size ? (int)pool->n_kv_heads : 1;
        const int cj = (int)(hj * n_slots * pool->head_dim * eb / 16);
        const int64_t vjobs = n * pool->n_layers * (pool->n_kv_heads / hj) * 2;
        block_copy_vec_kernel<<<grid_for(vjobs, 1), 256, 0, as_stream(stream)>>>(
            static_cast<uint4*>(pool->k), static_cast<uint4*>(pool->v), geom_of(pool), eb, src,
            dst, n, hj, cj);
        return check_launch("block_copy_vec_kernel");
    }
    block_copy_kernel<<<grid_for(jobs, 1), 256, 0, as_stream(stream)>>>(
        static_cast<char*>(pool->k), static_cast<char*>(pool->v), geom_of(pool),
        elem_bytes(pool->dtype), src, dst, n, n_slots);
    return check_launch("block_copy_kernel");
}

}  // extern "C"
