/*
 * status.cpp -- error reporting and per-device launch geometry.
 */
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg)
{
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what)
{
    g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                   cudaGetErrorString(e) + ")";
    return DIA_ERR_CUDA;
}

int num_sms()
{
    static std::mutex mu;
    static std::unordered_map<int, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(dev);
    if (it != cache.end()) return it->second;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0)
        sms = 148;
    cache[dev] = sms;
    return sms;
}

/* Blocks for a persistent launch: every SM filled to the kernel's occupancy. */
int persistent_blocks(const void* kernel, int smem_bytes)
{
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kBlock, smem_bytes) !=
            cudaSuccess ||
        per_sm <= 0)
        per_sm = 1;
    return per_sm * num_sms();
}

}  // namespace dia

extern "C" const char* dia_last_error(void) { return dia::g_last_error.c_str(); }

extern "C" int dia_version(void) { return 100; }
