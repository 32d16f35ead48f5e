// Shared pieces of the tcgen05 paged-attention kernels (chunked prefill and
// long speculative-verify chains, used when the packed query tile reaches 64
// rows = query tokens x GQA group): launch parameters, the eligibility test,
// the tcgen05 / TMEM / shared-memory-descriptor helpers and two small device
// utilities.  The kernels are attn_prefill_tc256.cuh (two 128-row query tiles
// per CTA, head_dim 64 or 128) and attn_prefill_tc128.cuh (one query tile per
// CTA, head_dim 128, when every sequence fits in one tile).
#pragma once
#include <type_traits>

#include "cx_common.cuh"

namespace cx {

constexpr int kTcRows = 128;    // packed query rows per query tile (MMA M)
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


}  // namespace cx
