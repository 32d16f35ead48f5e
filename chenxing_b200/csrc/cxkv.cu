// libcxkv.so — single translation unit of the C ABI declared in
// include/cxkv.h (one TU so every kernel shares the device flag word without
// relocatable device code).
#include "capi.cuh"
#include "kv_ops.cuh"
#include "attn_generic.cuh"
#include "attn_paged_mma.cuh"

// ---------------------------------------------------------------------------
// Paged decode that allocates nothing.
//
// Some callers cannot hand this library a workspace: a serving process that
// has already reserved its HBM (the block pool takes ~90 % and its own
// caching allocator owns the rest) and forbids further device allocations,
// or a host runtime reached over a plain C FFI that has no device allocator
// to offer.  cx_paged_decode_static serves them with a fixed scratch area
// that lives in the library itself: kScratchBytes per device, held by every
// GPU that loads the library until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace cx {

constexpr size_t kScratchBytes = 8u << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_static_scratch[kScratchBytes];

// The host-side name g_static_scratch is only a stand-in for the device
// array; the device address comes from cudaGetSymbolAddress, resolved once
// per device while that device is current and cached here.
static void* static_scratch_ptr(int* rc_out) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void* ptrs[kMaxDevices] = {};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *rc_out = cuda_fail(e, "cudaGetDevice");
        return nullptr;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        *rc_out = fail(CX_ERR_UNSUPPORTED, "cx_paged_decode_static: device index above 63");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(mu);
    if (!ptrs[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || !p) {
            *rc_out = cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
            return nullptr;
        }
        ptrs[dev] = p;
    }
    *rc_out = CX_OK;
    return ptrs[dev];
}

}  // namespace cx

extern "C" int cx_paged_decode_static(const cx_pool* pool, int64_t layer,
                                      const cx_attn_batch* batch, const void* q,
                                      int32_t q_dtype, float* out, void* stream) {
    using namespace cx;
    if (!pool || !batch) return fail(CX_ERR_SHAPE, "cx_paged_decode_static: NULL pool or batch");
    // only the split-K kernels use scratch (the generic kernel needs none)
    const size_t need = paged_scratch_need(pool, batch, q, q_dtype, out, false);
    if (need > kScratchBytes)
        return fail(CX_ERR_WORKSPACE,
                    "cx_paged_decode_static: this batch needs " + std::to_string(need) +
                        " bytes of scratch, the static area holds " +
                        std::to_string(kScratchBytes) +
                        "; use cx_paged_decode with a caller workspace");
    int rc = CX_OK;
    void* ws = static_scratch_ptr(&rc);
    if (!ws) return rc;
    // Always re-plan: the scratch is shared by every call, so the plan and
    // merge tickets of a previous call (other batch, other stream) must not be
    // reused; the plan kernel rewrites the plan and zeroes the tickets.
    return paged_attention(pool, layer, batch, q, q_dtype, out, ws, kScratchBytes, 1, stream,
                           false);
}
