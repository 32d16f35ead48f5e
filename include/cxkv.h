/*
 * cxkv.h — C ABI of libcxkv.so, the B200 (sm_100a) KV-cache hot path of
 * Chenxing: the physical block pool of RadixPagedKVCache and the paged
 * attention that reads it.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * handle (cudaStream_t passed as void*; NULL = legacy default stream), runs
 * asynchronously on that stream and returns a cx_status.  Nothing here
 * allocates device memory: callers own the pools, the metadata arrays and the
 * attention workspace.  Host-side argument checks return an error code before
 * any launch; device-side range checks (block ids, slots, table overruns)
 * skip the offending access and raise a bit in a per-library device flag word
 * that cx_device_error() reads back.
 *
 * Physical pool layout (one allocation each for K and V):
 *     [n_layers][n_blocks][n_kv_heads][block_size][head_dim]
 * i.e. one (block, head) is a contiguous block_size x head_dim tile.  The
 * reference's view (n_layers, n_blocks, block_size, n_kv_heads, head_dim)
 * (chenxing/engine/radix_kv.py:87) is the same storage with axes 2 and 3
 * swapped.
 */
#ifndef CXKV_H
#define CXKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
    CX_OK = 0,
    CX_ERR_RANGE = 1,        /* index outside the pool / table              */
    CX_ERR_SHAPE = 2,        /* inconsistent sizes                          */
    CX_ERR_CUDA = 3,         /* a CUDA runtime call failed                  */
    CX_ERR_DTYPE = 4,        /* unsupported element type                    */
    CX_ERR_UNSUPPORTED = 5,  /* valid request this build does not handle    */
    CX_ERR_WORKSPACE = 6     /* workspace missing or too small              */
};

/* ---- element types ----------------------------------------------------- */
enum { CX_F32 = 0, CX_BF16 = 1, CX_F16 = 2 };

/* ---- device-side error flag bits (cx_device_error) --------------------- */
enum {
    CX_DEV_BAD_SLOT = 1u << 0,     /* append slot outside n_blocks*block_size */
    CX_DEV_BAD_BLOCK = 1u << 1,    /* block id outside [0, n_blocks)          */
    CX_DEV_TABLE_OVERRUN = 1u << 2,/* context longer than its block table     */
    CX_DEV_WAIT_TIMEOUT = 1u << 3, /* a bounded pipeline wait gave up         */
    CX_DEV_BAD_QLEN = 1u << 4,     /* query length > context or > max_q_len   */
    CX_DEV_BAD_POSITION = 1u << 5  /* RoPE position outside the cos/sin table */
};

/* A block pool: K and V device buffers plus their shape. */
typedef struct cx_pool {
    void* k;
    void* v;
    int64_t n_layers;
    int64_t n_blocks;
    int64_t block_size;
    int64_t n_kv_heads;
    int64_t head_dim;
    int32_t dtype;           /* CX_F32 / CX_BF16 / CX_F16 */
    int32_t reserved;
} cx_pool;

/* A batch of sequences to attend over the pool (all arrays on the device). */
typedef struct cx_attn_batch {
    const int32_t* block_tables; /* [batch][table_stride] physical block ids     */
    int64_t table_stride;
    const int32_t* ctx_lens;     /* [batch] cached tokens, INCLUDING the new     */
                                 /* query tokens already appended                */
    const int32_t* q_start;      /* [batch+1] query-row prefix sums; NULL means  */
                                 /* one query token per sequence (decode)        */
    int64_t batch;
    int64_t max_q_len;           /* >= every q_start[b+1]-q_start[b]; 1 for decode */
    int64_t n_q_heads;           /* multiple of n_kv_heads (GQA)                 */
    float scale;                 /* NaN selects 1/sqrt(head_dim); any other     */
                                 /* value (also 0 or negative) is used as given  */
    int32_t reserved;
    int64_t window;              /* <= 0: plain causal; else sliding window w    */
} cx_attn_batch;

const char* cx_version(void);
/* Message for the most recent non-OK status returned on this host thread. */
const char* cx_last_error(void);
/* Synchronises `stream`, stores the device flag word in *flags, clears it
 * when `clear` != 0. */
int cx_device_error(void* stream, int clear, uint32_t* flags);

/* KV append — replaces RadixPagedKVCache.write_layer
 * (chenxing/engine/radix_kv.py:113-128), batched over sequences.
 * Token t (k_new/v_new row t, shape [n_tokens][n_kv_heads][head_dim] of
 * src_dtype) is stored at slot slot_mapping[t] = block*block_size + offset of
 * `layer`; a negative slot skips the token.  Values are rounded to the pool
 * type with round-to-nearest-even.  In the same launch, for c < n_cow the
 * first cow_n_valid[c] slots of block cow_src[c] are copied into block
 * cow_dst[c] for this layer (copy-on-write of a shared partial tail block; the
 * reference has no counterpart, it shares whole blocks only, radix_kv.py:16-21).
 * The copies and the token stores run concurrently: every slot the call
 * writes in a block cow_dst[c] must be at offset >= cow_n_valid[c] (the
 * Python layer checks this before the launch).  cow_* may be NULL when
 * n_cow == 0. */
int cx_kv_append(const cx_pool* pool, int64_t layer,
                 const void* k_new, const void* v_new, int32_t src_dtype,
                 const int64_t* slot_mapping, int64_t n_tokens,
                 const int32_t* cow_src, const int32_t* cow_dst,
                 const int32_t* cow_n_valid, int64_t n_cow, void* stream);

/* RoPE fused into the KV append — replaces apply_rope on Q and K followed by
 * write_layer (chenxing/model/transformer.py:84-87, chenxing/core/tensor.py:
 * 129-180, radix_kv.py:113-128).  Token t sits at absolute position
 * positions[t] (0 <= position < table_rows); cos_table / sin_table are the
 * float32 [table_rows][head_dim] tables of build_rope_cache
 * (tensor.py:80-121).  K rows are rotated and scattered like cx_kv_append
 * (negative slot = skip, no copy-on-write), V rows are copied, and when
 * n_q_heads > 0 the Q rows q [n_tokens][n_q_heads][head_dim] (src_dtype) are
 * rotated into q_out (q_out_dtype CX_F32 or CX_BF16).  interleaved != 0 pairs
 * elements (2j, 2j+1), else (j, j + head_dim/2).  Each rotated element is the
 * fp32 expression the reference evaluates (two products, one sum, no fused
 * multiply-add), then rounded to the destination type.  head_dim must be
 * even; a position outside the table raises CX_DEV_BAD_POSITION and skips
 * the token. */
int cx_kv_append_rope(const cx_pool* pool, int64_t layer, const void* k_new, const void* v_new,
                      int32_t src_dtype, const int64_t* slot_mapping, const int64_t* positions,
                      int64_t n_tokens, const float* cos_table, const float* sin_table,
                      int64_t table_rows, int32_t interleaved, const void* q,
                      int64_t n_q_heads, void* q_out, int32_t q_out_dtype, void* stream);

/* KV gather — replaces RadixPagedKVCache.read_layer
 * (chenxing/engine/radix_kv.py:130-144): k_out/v_out [n_tokens][n_kv_heads]
 * [head_dim] (pool dtype) receive the first n_tokens positions of the
 * sequence whose table is block_table[ceil(n_tokens/block_size)]. */
int cx_kv_gather(const cx_pool* pool, int64_t layer, const int32_t* block_table,
                 int64_t n_tokens, void* k_out, void* v_out, void* stream);

/* Block copy — eviction compaction and prefix forking over all layers and
 * both K and V: for i < n, slots [0, n_slots) of block dst[i] := block src[i].
 * No reference counterpart: the reference aliases shared blocks
 * (radix_kv.py:172) and only relabels evicted ids (radix_kv.py:232-233). */
int cx_block_copy(const cx_pool* pool, const int32_t* src, const int32_t* dst,
                  int64_t n, int64_t n_slots, void* stream);

/* Workspace bytes cx_paged_decode / cx_paged_verify need for `batch` on the
 * current device (plan, split-K partials and merge counters). */
size_t cx_paged_workspace_bytes(const cx_pool* pool, const cx_attn_batch* batch);

/* Paged decode — replaces, per layer, read_layer + flash_attention with
 * sq = 1 and CausalMask(sliding_window) (chenxing/model/transformer.py:88-94,
 * chenxing/core/attention.py:43-116).  q: [batch][n_q_heads][head_dim] of
 * q_dtype; out: float32 [batch][n_q_heads][head_dim].  Query head h reads KV
 * head h / (n_q_heads / n_kv_heads) (attention.py:30-40).  The workspace must
 * be zero-filled once after allocation; calls leave it reusable.  `replan`
 * != 0 rebuilds the split plan from ctx_lens (once per step; the plan stays
 * valid for every layer of the step while ctx_lens is unchanged).  A row with
 * no attendable key yields zeros (naive_attention semantics,
 * attention.py:146-147). */
int cx_paged_decode(const cx_pool* pool, int64_t layer, const cx_attn_batch* batch,
                    const void* q, int32_t q_dtype, float* out,
                    void* workspace, size_t workspace_bytes, int32_t replan,
                    void* stream);

/* Paged multi-query attention for speculative verification and chunked
 * prefill — the reference's forward_ids with T = gamma+1 or a prompt chunk
 * (chenxing/engine/speculative.py:141-143, chenxing/engine/engine.py:149-151)
 * through transformer.py:88-94.  Query rows of sequence b are
 * q[q_start[b] .. q_start[b+1]) ([rows][n_q_heads][head_dim]); row i sits at
 * position ctx_lens[b] - q_len + i (attention.py:76) and sees keys
 * j <= pos with j > pos - window when window > 0 (attention.py:78-79).
 * out: float32 [q_start[batch]][n_q_heads][head_dim]. */
int cx_paged_verify(const cx_pool* pool, int64_t layer, const cx_attn_batch* batch,
                    const void* q, int32_t q_dtype, float* out,
                    void* workspace, size_t workspace_bytes, int32_t replan,
                    void* stream);

/* Paged decode that allocates nothing — no counterpart in the reference (its
 * NumPy path needs no device memory at all).  Same inputs, outputs and
 * results as cx_paged_decode, but the plan / split-K partials / merge tickets
 * live in a scratch array compiled into this library (8 MiB per device,
 * resident on every GPU that loads the library until the process exits), for
 * callers that cannot allocate device memory: a serving process whose HBM is
 * already fully reserved by the block pool and its own allocator, or a host
 * runtime behind a plain C FFI with no device allocator to give us.
 * - Rejects, with CX_ERR_WORKSPACE and a message, any batch whose scratch
 *   need (cx_paged_workspace_bytes, for the split-K kernels; batches that take
 *   the generic kernel need none) exceeds 8 MiB; it never calls cudaMalloc,
 *   cudaFree or any allocating library routine.
 * - The first call on a device resolves the scratch address with
 *   cudaGetSymbolAddress (that device must be current); make that first call
 *   before any stream capture.  The address is cached per device index for
 *   the life of the process: after cudaDeviceReset on a device it is stale,
 *   so do not call this entry point on that device again in the process.
 * - Every call re-plans and zeroes the merge tickets itself.  All calls on a
 *   device share the one scratch array, which keeps the last call's contents:
 *   calls that overlap on the GPU (different streams, no ordering between
 *   them) race on it and must be serialised by the caller. */
int cx_paged_decode_static(const cx_pool* pool, int64_t layer, const cx_attn_batch* batch,
                           const void* q, int32_t q_dtype, float* out, void* stream);

/* Limit, in nanoseconds, of every pipeline wait inside the decode / verify
 * kernels of later calls in this process (0 restores the default, 2 s).  A
 * wait that runs out makes its CTA stop, wait (with the default limit) for its
 * own copies in flight, raise CX_DEV_WAIT_TIMEOUT and return; that call's
 * output is then undefined and the device stays usable.  Meant for tests of
 * that failure path (a limit of a few nanoseconds makes the waits run out);
 * no counterpart in the reference, which has no device waits. */
void cx_set_wait_limit_ns(uint64_t ns);

/* Which kernel cx_paged_decode (verify = 0) or cx_paged_verify (verify = 1)
 * runs for this pool, batch shape and query type — diagnostics, no
 * counterpart in the reference: CX_KERNEL_GENERIC (fp16 pools, other block
 * sizes or head dims, fp32 pools beyond 64 packed rows: exact CUDA-core
 * kernel), CX_KERNEL_MMA (bf16 pool, packed query tile of 1..63 rows: TMA +
 * mma.sync split-K kernel), CX_KERNEL_TCGEN05 (bf16 pool, packed tile of 64
 * rows or more: TMA + tcgen05 / TMEM kernel) or CX_KERNEL_FMA (fp32 pool,
 * 16-token blocks, head_dim 64 / 128, up to 64 packed rows per KV head: TMA +
 * fp32 FMA split-K kernel).  Packed rows = (n_q_heads / n_kv_heads) x
 * max_q_len.  Reads only the host fields of `batch` and assumes
 * 16-byte-aligned q and out pointers: the decode / verify calls run the
 * generic kernel for q or out pointers that are not 16-byte aligned. */
enum { CX_KERNEL_GENERIC = 0, CX_KERNEL_MMA = 1, CX_KERNEL_TCGEN05 = 2, CX_KERNEL_FMA = 3 };
int cx_paged_kernel_kind(const cx_pool* pool, const cx_attn_batch* batch, int32_t q_dtype,
                         int32_t verify);

/* Dense attention — replaces flash_attention / naive_attention on contiguous
 * arrays (chenxing/core/attention.py:43-148): q [b][hq][sq][d],
 * k [b][hk][sk][d], v [b][hk][sk][dv] (kv_dtype), out float32 [b][hq][sq][dv].
 * mask_kind 0 = none, 1 = causal with query offset sk - sq and optional
 * window (> 0), 2 = explicit boolean mask [sq][sk] (nonzero = attend).
 * scale NaN selects 1/sqrt(d). */
int cx_attention_dense(const void* q, int32_t q_dtype, const void* k, const void* v,
                       int32_t kv_dtype, int64_t b, int64_t hq, int64_t sq,
                       int64_t hk, int64_t sk, int64_t d, int64_t dv,
                       int32_t mask_kind, int64_t window, const uint8_t* mask,
                       float scale, float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CXKV_H */
