// Library-wide pieces of the C ABI: version, per-thread error text, the
// device flag word and the per-device SM count cache.
#include <mutex>
#include <string>
#include <vector>

#include "cx_common.cuh"  // unity build: included from cxkv.cu

namespace cx {

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
    t_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return CX_ERR_CUDA;
}

int num_sms() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace cx

extern "C" {

const char* cx_version(void) { return "cxkv 0.1 sm_100a"; }

const char* cx_last_error(void) { return cx::t_last_error.c_str(); }

int cx_device_error(void* stream, int clear, uint32_t* flags) {
    if (!flags) return cx::fail(CX_ERR_SHAPE, "cx_device_error: flags is NULL");
    cudaStream_t s = cx::as_stream(stream);
    unsigned int v = 0;
    CX_CUDA_CHECK(cudaMemcpyFromSymbolAsync(&v, cx::g_dev_flags, sizeof(v), 0,
                                            cudaMemcpyDeviceToHost, s));
    CX_CUDA_CHECK(cudaStreamSynchronize(s));
    if (clear) {
        unsigned int z = 0;
        CX_CUDA_CHECK(cudaMemcpyToSymbolAsync(cx::g_dev_flags, &z, sizeof(z), 0,
                                              cudaMemcpyHostToDevice, s));
        CX_CUDA_CHECK(cudaStreamSynchronize(s));
    }
    *flags = v;
    return CX_OK;
}

}  // extern "C"
