// pn_act.cu -- per-token absmax int8 activation quantiser.
//
// The reference's int8 line quantises with one absmax scale for the whole
// tensor (penta_avx2_wrapper.py:130-131): s = max|x| / 127,
// xq = clamp(round(x / s), -128, 127).  Here the same two formulas run per
// token (row), with IEEE division and round-half-even; an all-zero row gets
// s = 1.  The output rows are padded with zeros to a pitch the tensor-core
// kernel loads in 32-byte slabs, and the row sums feed its unsigned-code
// correction (sum_k xq*(c-2) = sum_k xq*c - 2*sum_k xq).
#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

constexpr int kActThreads = 256;

int64_t act_i8_pitch(int64_t K) { return (K + 31) / 32 * 32; }

template <typename T>
__device__ __forceinline__ float ld_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, int64_t i) {
    return p[i];
}
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}

template <typename T>
__global__ void __launch_bounds__(kActThreads) quant_act_i8_kernel(const T* __restrict__ x, int64_t K,
                                                                   int8_t* __restrict__ xq, int64_t pitch,
                                                                   float* __restrict__ s_x,
                                                                   int32_t* __restrict__ rowsum) {
    __shared__ float red_f[kActThreads / 32];
    __shared__ int red_i[kActThreads / 32];
    const int64_t m = blockIdx.x;
    const T* row = x + m * K;
    float amax = 0.0f;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(ld_f(row, k)));
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red_f[threadIdx.x >> 5] = amax;
    __syncthreads();
    float a = red_f[0];
#pragma unroll
    for (int i = 1; i < kActThreads / 32; ++i) a = fmaxf(a, red_f[i]);
    float s = __fdiv_rn(a, 127.0f);
    if (!(s > 0.0f)) s = 1.0f;
    int8_t* qrow = xq + m * pitch;
    int sum = 0;
    for (int64_t k = threadIdx.x; k < pitch; k += blockDim.x) {
        int q = 0;
        if (k < K) {
            float r = rintf(__fdiv_rn(ld_f(row, k), s));
            r = fminf(fmaxf(r, -128.0f), 127.0f);
            q = (int)r;
        }
        qrow[k] = (int8_t)q;
        sum += q;
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 31) == 0) red_i[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
#pragma unroll
        for (int i = 0; i < kActThreads / 32; ++i) t += red_i[i];
        rowsum[m] = t;
        s_x[m] = s;
    }
}

cudaError_t launch_quant_act_i8(const void* x, int x_dtype, int64_t M, int64_t K, int8_t* xq, int64_t pitch,
                                float* s_x, int32_t* rowsum, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (x_dtype == PN_F32)
        quant_act_i8_kernel<float><<<(unsigned)M, kActThreads, 0, s>>>(static_cast<const float*>(x), K, xq, pitch,
                                                                        s_x, rowsum);
    else
        quant_act_i8_kernel<__nv_bfloat16><<<(unsigned)M, kActThreads, 0, s>>>(
            static_cast<const __nv_bfloat16*>(x), K, xq, pitch, s_x, rowsum);
    return cudaGetLastError();
}

}  // namespace pn
