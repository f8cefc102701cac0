/*
 * synth.cu -- counter-based generator for the synthetic benchmark matrices.
 *
 * value(seed, d, i) is a hash of (seed, diagonal offset, global row), so any
 * rank generates its own row block of a partitioned matrix without
 * communication and the result does not depend on the partition or on the
 * diagonal order.  Arithmetic is integer plus separately rounded fp32 ops,
 * so the host restatement in the oracle reproduces it bit for bit.
 */
#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float synth_value(uint64_t seed, int d, long long row, int kind,
                                             float base, float lo, float hi)
{
    uint64_t h = mix64(mix64(seed ^ ((uint64_t)(uint32_t)d * 0xD6E8FEB86659FD93ull)) ^
                       (uint64_t)row);
    if (kind == 0) {
        const float u = __fmul_rn((float)(uint32_t)(h >> 40), 1.0f / 16777216.0f);
        return __fadd_rn(base, __fadd_rn(lo, __fmul_rn(__fsub_rn(hi, lo), u)));
    }
    long long s = 0;
    for (int r = 0; r < 12; ++r) {
        s += (long long)(h >> 40);
        h = mix64(h);
    }
    s -= 6LL * 16777216;
    const float z = __fmul_rn(__ll2float_rn(s), 1.0f / 16777216.0f);
    return __fadd_rn(base, __fmul_rn(hi, z));
}

__global__ void synth_rows_kernel(uint64_t seed, long long n_rows, long long n_cols, int K,
                                  const int* off, const float* base, int kind, float lo,
                                  float hi, long long row0, long long nrows, long long stride,
                                  float* vals)
{
    const long long total = (long long)K * stride;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int k = (int)(e / stride);
        const long long i = e - (long long)k * stride;
        const long long g = row0 + i;
        const int d = off[k];
        const long long c = g + d;
        float v = 0.0f;
        if (i < nrows && g < n_rows && c >= 0 && c < n_cols)
            v = synth_value(seed, d, g, kind, base ? base[k] : 0.0f, lo, hi);
        vals[e] = v;
    }
}

__global__ void synth_vector_kernel(uint64_t seed, long long i0, long long len, float lo,
                                    float hi, float* out)
{
    for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < len;
         j += (long long)gridDim.x * blockDim.x)
        out[j] = synth_value(seed, 0x7fffffff, i0 + j, 0, 0.0f, lo, hi);
}

}  // namespace dia

using namespace dia;

extern "C" int dia_synth_rows(uint64_t seed, int64_t n_rows, int64_t n_cols, int K,
                              const int* d_offsets, const float* d_base, int kind, float lo,
                              float hi, int64_t row0, int64_t nrows, int64_t stride,
                              float* d_vals, cudaStream_t stream)
{
    if (K < 0 || stride < 0 || nrows < 0 || nrows > stride || (kind != 0 && kind != 1))
        return fail(DIA_ERR_INVALID, "dia_synth_rows: bad size or kind");
    if (K == 0 || stride == 0) return DIA_OK;
    if (!d_offsets || !d_vals) return fail(DIA_ERR_INVALID, "dia_synth_rows: null pointer");
    synth_rows_kernel<<<num_sms() * 8, kBlock, 0, stream>>>(seed, n_rows, n_cols, K, d_offsets,
                                                           d_base, kind, lo, hi, row0, nrows,
                                                           stride, d_vals);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}

extern "C" int dia_synth_vector(uint64_t seed, int64_t i0, int64_t len, float lo, float hi,
                                float* d_out, cudaStream_t stream)
{
    if (len < 0) return fail(DIA_ERR_INVALID, "dia_synth_vector: negative length");
    if (len == 0) return DIA_OK;
    if (!d_out) return fail(DIA_ERR_INVALID, "dia_synth_vector: null pointer");
    synth_vector_kernel<<<num_sms() * 8, kBlock, 0, stream>>>(seed, i0, len, lo, hi, d_out);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}
