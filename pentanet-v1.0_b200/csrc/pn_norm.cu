// pn_norm.cu -- LayerNorm over the last dimension with the output written in
// the projection's input type.
//
// The reference GPT normalises before every projection (ln_1, ln_2, ln_f;
// nn.LayerNorm without bias, train_pentagpt.py:94-96,113,127) under bf16 autocast,
// where torch runs each call as three passes over the activations: a cast of
// the bf16 input to fp32, an fp32 layer_norm, and a cast of its fp32 output
// to bf16 in front of the projection.  Here one pass reads the bf16 (or fp32)
// row, takes fp32 statistics (mean, then the mean squared deviation from it:
// the biased variance), and writes (x - mean) * rsqrt(var + eps) * w + b
// rounded once to bf16 (or as fp32).
#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

constexpr int kNormWarps = 8;  // one warp per row

template <typename T>
struct Vec8;  // eight consecutive elements as fp32
template <>
struct Vec8<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[8]) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
};
template <>
struct Vec8<float> {
    static __device__ __forceinline__ void load(const float* p, float (&v)[8]) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        const float4 b = *reinterpret_cast<const float4*>(p + 4);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    }
};

// Eight consecutive row elements kept in their storage type (4 registers
// for bf16), converted to fp32 on each use.
template <typename T>
struct RowVec8;
template <>
struct RowVec8<__nv_bfloat16> {
    uint32_t w[4];
    __device__ __forceinline__ void load(const __nv_bfloat16* p) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        w[0] = u.x, w[1] = u.y, w[2] = u.z, w[3] = u.w;
    }
    __device__ __forceinline__ float get(int j) const {
        return __uint_as_float((j & 1) ? (w[j >> 1] & 0xFFFF0000u) : (w[j >> 1] << 16));
    }
};
template <>
struct RowVec8<float> {
    float f[8];
    __device__ __forceinline__ void load(const float* p) { Vec8<float>::load(p, f); }
    __device__ __forceinline__ float get(int j) const { return f[j]; }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Rows of C <= 256 * V elements (C % 8 == 0, 16-byte aligned rows, weight
// and bias 16-byte aligned), held in registers: lane l owns the 8-element
// vectors l, l + 32, ...  Five blocks per SM: the register cap keeps 40 warps
// resident so enough loads are in flight.
template <typename T, int V>
__global__ void __launch_bounds__(kNormWarps * 32, 5) layer_norm_reg_kernel(const T* __restrict__ x, int64_t M, int C,
                                                                         const float* __restrict__ w,
                                                                         const float* __restrict__ b, float eps,
                                                                         void* __restrict__ y, int y_f32) {
    // The product that reads this output may start its prologue and weight
    // streaming now (it waits for this grid before reading the output).
    asm volatile("griddepcontrol.launch_dependents;");
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= M) return;
    const T* xr = x + row * C;
    RowVec8<T> v[V];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = (i * 32 + lane) * 8;
        if (c < C) {
            v[i].load(xr + c);
#pragma unroll
            for (int j = 0; j < 8; ++j) s += v[i].get(j);
        }
    }
    const float mean = __fdiv_rn(warp_sum(s), (float)C);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        if ((i * 32 + lane) * 8 < C) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float d = v[i].get(j) - mean;
                q = fmaf(d, d, q);
            }
        }
    }
    const float rstd = rsqrtf(__fdiv_rn(warp_sum(q), (float)C) + eps);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = (i * 32 + lane) * 8;
        if (c >= C) continue;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (v[i].get(j) - mean) * rstd;
        if (w) {
            float wv[8];
            Vec8<float>::load(w + c, wv);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] *= wv[j];
        }
        if (b) {
            float bv[8];
            Vec8<float>::load(b + c, bv);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] += bv[j];
        }
        if (y_f32) {
            float* yr = static_cast<float*>(y) + row * C + c;
            *reinterpret_cast<float4*>(yr) = make_float4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<float4*>(yr + 4) = make_float4(o[4], o[5], o[6], o[7]);
        } else {
            uint32_t u[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * k], o[2 * k + 1]);
                u[k] = *reinterpret_cast<const uint32_t*>(&h);
            }
            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(y) + row * C + c) = make_uint4(u[0], u[1], u[2], u[3]);
        }
    }
}

template <typename T>
__device__ __forceinline__ float ld_elem(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_elem<float>(const float* p, int64_t i) {
    return p[i];
}
template <>
__device__ __forceinline__ float ld_elem<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}

// Any C: the same arithmetic, three strided passes over the row.
template <typename T>
__global__ void __launch_bounds__(kNormWarps * 32) layer_norm_any_kernel(const T* __restrict__ x, int64_t M, int64_t C,
                                                                         const float* __restrict__ w,
                                                                         const float* __restrict__ b, float eps,
                                                                         void* __restrict__ y, int y_f32) {
    // The product that reads this output may start its prologue and weight
    // streaming now (it waits for this grid before reading the output).
    asm volatile("griddepcontrol.launch_dependents;");
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= M) return;
    const T* xr = x + row * C;
    float s = 0.0f;
    for (int64_t c = lane; c < C; c += 32) s += ld_elem(xr, c);
    const float mean = __fdiv_rn(warp_sum(s), (float)C);
    float q = 0.0f;
    for (int64_t c = lane; c < C; c += 32) {
        const float d = ld_elem(xr, c) - mean;
        q = fmaf(d, d, q);
    }
    const float rstd = rsqrtf(__fdiv_rn(warp_sum(q), (float)C) + eps);
    for (int64_t c = lane; c < C; c += 32) {
        float t = (ld_elem(xr, c) - mean) * rstd;
        if (w) t *= __ldg(w + c);
        if (b) t += __ldg(b + c);
        if (y_f32)
            static_cast<float*>(y)[row * C + c] = t;
        else
            static_cast<__nv_bfloat16*>(y)[row * C + c] = __float2bfloat16_rn(t);
    }
}

template <typename T>
static cudaError_t launch_norm_t(const T* x, int64_t M, int64_t C, const float* w, const float* b, float eps, void* y,
                                 int y_f32, cudaStream_t s) {
    const unsigned blocks = (unsigned)((M + kNormWarps - 1) / kNormWarps);
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) % 16) == 0; };
    const bool vec = C % 8 == 0 && a16(x) && a16(y) && a16(w) && a16(b);
    const int c = (int)C;
    // Register-held rows up to the width that compiles without spills at five
    // blocks per SM: 1024 bf16 / 512 fp32 elements; wider rows take the
    // strided kernel.
    constexpr int kMaxC = sizeof(T) == 2 ? 1024 : 512;
    if (vec && C <= 256)
        layer_norm_reg_kernel<T, 1><<<blocks, kNormWarps * 32, 0, s>>>(x, M, c, w, b, eps, y, y_f32);
    else if (vec && C <= 512)
        layer_norm_reg_kernel<T, 2><<<blocks, kNormWarps * 32, 0, s>>>(x, M, c, w, b, eps, y, y_f32);
    else if (vec && C <= 768 && C <= kMaxC)
        layer_norm_reg_kernel<T, sizeof(T) == 2 ? 3 : 2><<<blocks, kNormWarps * 32, 0, s>>>(x, M, c, w, b, eps, y, y_f32);
    else if (vec && C <= kMaxC)
        layer_norm_reg_kernel<T, sizeof(T) == 2 ? 4 : 2><<<blocks, kNormWarps * 32, 0, s>>>(x, M, c, w, b, eps, y, y_f32);
    else
        layer_norm_any_kernel<T><<<blocks, kNormWarps * 32, 0, s>>>(x, M, C, w, b, eps, y, y_f32);
    return cudaGetLastError();
}

cudaError_t launch_layer_norm(const void* x, int x_dtype, int64_t M, int64_t C, const float* w, const float* b,
                              float eps, void* y, int y_dtype, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (x_dtype == PN_F32)
        return launch_norm_t(static_cast<const float*>(x), M, C, w, b, eps, y, y_dtype == PN_F32, s);
    return launch_norm_t(static_cast<const __nv_bfloat16*>(x), M, C, w, b, eps, y, y_dtype == PN_F32, s);
}

}  // namespace pn
