// libcxkv.so — single translation unit of the C ABI declared in
// include/cxkv.h (one TU so every kernel shares the device flag word without
// relocatable device code).
#include "capi.cuh"
#include "kv_ops.cuh"
#include "attn_generic.cuh"
#include "attn_paged_mma.cuh"
