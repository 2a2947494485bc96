// pn_pack.cu -- absmean scale, quantise+pack and unpack kernels.
//
// Byte-for-byte the packed format of quantize_and_pack (penta_kernel.py:42-78):
// gamma = max(mean|W|, 1e-8) (:57), q = clamp(round_half_even(W / gamma), -2, 2)
// with IEEE float division (:60), code = q + 2 (:70), word |= code << 3i (:74-76),
// K padded with code 2 (:62-65).  All three kernels are HBM-bound streams.
#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

constexpr int kAbsBlocks = 512;   // fixed partial count: the reduction order never depends on the device
constexpr int kAbsThreads = 512;

template <typename T>
__device__ __forceinline__ float load_as_float(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_as_float<float>(const float* p, int64_t i) {
    return __ldg(p + i);
}
template <>
__device__ __forceinline__ float load_as_float<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}

// Pass 1: block b sums |w| over the contiguous range [b*chunk, (b+1)*chunk) in
// double, threads striding by blockDim, then a fixed-shape tree.
template <typename T>
__global__ void __launch_bounds__(kAbsThreads) absmean_partial_kernel(const T* __restrict__ w, int64_t n,
                                                                      double* __restrict__ partial) {
    __shared__ double red[kAbsThreads / 32];
    const int64_t chunk = (n + kAbsBlocks - 1) / kAbsBlocks;
    const int64_t begin = (int64_t)blockIdx.x * chunk;
    const int64_t end = begin + chunk < n ? begin + chunk : n;
    double s = 0.0;
    for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) s += fabs((double)load_as_float(w, i));
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < kAbsThreads / 32 ? red[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) partial[blockIdx.x] = t;
    }
}

// Pass 2: one block folds the partials in a fixed order and writes gamma.
__global__ void __launch_bounds__(kAbsBlocks) absmean_final_kernel(const double* __restrict__ partial, int64_t n,
                                                                   float* __restrict__ scale) {
    __shared__ double red[kAbsBlocks / 32];
    double s = partial[threadIdx.x];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < kAbsBlocks / 32 ? red[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) {
            float mean = n > 0 ? (float)(t / (double)n) : 0.0f;
            *scale = mean > 1e-8f ? mean : 1e-8f;  // .clamp(min=1e-8)
        }
    }
}

// round_half_even(v / gamma) clamped to [-qmax, qmax], as a code.  v times
// the correctly rounded reciprocal is within ~2 ulp of the IEEE quotient, so
// it rounds to the same integer unless the quotient lies within 1e-4 of a
// half-integer (the only place where the clamped code can differ: |t| is at
// most ~qmax + 0.5 there, so 2 ulp is far below 1e-4); there, and for NaN or
// infinite products, the IEEE division decides.  NaN quantises to 0 (the
// reference leaves it platform-defined); +-inf saturate to +-qmax like clamp.
__device__ __forceinline__ uint32_t quant_code(float v, float gamma, float rg, float qmax) {
    float t = v * rg;
    float r = rintf(t);  // round half to even
    if (!(fabsf(fabsf(t - r) - 0.5f) >= 1e-4f)) {
        t = __fdiv_rn(v, gamma);
        r = rintf(t);
    }
    r = fminf(fmaxf(r, -qmax), qmax);
    return (t != t) ? 2u : (uint32_t)((int)r + 2);
}

// One thread per packed word (its ten weights are 40 contiguous bytes, so a
// warp's loads cover 1280 contiguous bytes that L1 serves after the first).
// A tiled variant staging 256-word row tiles through shared memory was
// slower (314-334 us against 273 us for a 940 MB fp32 matrix).
//
// qmax 2: pentanary (penta_kernel.py:60); qmax 1: the ternary (BitNet) rule
// of the reference's QuantLinear (train_pentagpt.py:33-36) in the same codes.
template <typename T>
__global__ void __launch_bounds__(256) quantize_pack_kernel(const T* __restrict__ w, int64_t N, int64_t K,
                                                            int64_t KP, const float* __restrict__ d_scale,
                                                            int32_t* __restrict__ packed, float qmax) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= N * KP) return;
    const float gamma = __ldg(d_scale);
    const float rg = __frcp_rn(gamma);
    const int64_t n = idx / KP;
    const int64_t g = idx - n * KP;
    const T* row = w + n * K;
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < kPerWord; ++i) {
        const int64_t k = g * kPerWord + i;
        const uint32_t code = k < K ? quant_code(load_as_float(row, k), gamma, rg, qmax) : 2u;
        word |= code << (3 * i);
    }
    packed[idx] = (int32_t)word;
}

// One thread per packed word: ten int8 values, cropped at K_orig.
__global__ void __launch_bounds__(256) unpack_kernel(const int32_t* __restrict__ packed, int64_t N, int64_t KP,
                                                     int64_t K, int8_t* __restrict__ out) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= N * KP) return;
    const int64_t n = idx / KP;
    const int64_t g = idx - n * KP;
    const uint32_t p = (uint32_t)__ldg(packed + idx);
    int8_t* row = out + n * K;
#pragma unroll
    for (int i = 0; i < kPerWord; ++i) {
        const int64_t k = g * kPerWord + i;
        if (k < K) row[k] = (int8_t)((int)((p >> (3 * i)) & 7u) - 2);
    }
}

size_t absmean_workspace_bytes() { return sizeof(double) * kAbsBlocks; }

cudaError_t launch_absmean(const void* w, int dtype, int64_t n, float* d_scale, void* ws, cudaStream_t s) {
    double* partial = static_cast<double*>(ws);
    if (dtype == PN_F32)
        absmean_partial_kernel<float><<<kAbsBlocks, kAbsThreads, 0, s>>>(static_cast<const float*>(w), n, partial);
    else
        absmean_partial_kernel<__nv_bfloat16>
            <<<kAbsBlocks, kAbsThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(w), n, partial);
    absmean_final_kernel<<<1, kAbsBlocks, 0, s>>>(partial, n, d_scale);
    return cudaGetLastError();
}

cudaError_t launch_quantize_pack(const void* w, int dtype, int64_t N, int64_t K, const float* d_scale,
                                 int32_t* packed, int qmax, cudaStream_t s) {
    const int64_t KP = (K + kPerWord - 1) / kPerWord;
    const int64_t total = N * KP;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    if (dtype == PN_F32)
        quantize_pack_kernel<float>
            <<<blocks, 256, 0, s>>>(static_cast<const float*>(w), N, K, KP, d_scale, packed, (float)qmax);
    else
        quantize_pack_kernel<__nv_bfloat16>
            <<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), N, K, KP, d_scale, packed, (float)qmax);
    return cudaGetLastError();
}

cudaError_t launch_unpack(const int32_t* packed, int64_t N, int64_t KP, int64_t K, int8_t* out, cudaStream_t s) {
    const int64_t total = N * KP;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    unpack_kernel<<<blocks, 256, 0, s>>>(packed, N, KP, K, out);
    return cudaGetLastError();
}

}  // namespace pn
