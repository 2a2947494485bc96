// pn_simt.cu -- CUDA-core dequant-matmul for bf16 activations whose row pitch
// is not a multiple of 8 elements (the tensor-core kernel loads activations
// by TMA, which needs 16-byte row pitches).  Same result contract as the
// tensor-core path: fp32 accumulation of bf16 x times exact {-2..2} weights,
// then * scale, bias and bf16 rounding as penta_kernel.py:221-224,275-276.
#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

constexpr int kSimtTok = 8;  // tokens per pass

// One warp per weight row; lanes stride over the row's packed words.
__global__ void __launch_bounds__(256) simt_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int64_t K,
                                                        const int32_t* __restrict__ packed, int64_t ld, int64_t N,
                                                        int64_t KP,
                                                        float scale, const __nv_bfloat16* __restrict__ bias,
                                                        const __nv_bfloat16* residual, int64_t ld_res, int act,
                                                        void* __restrict__ y, int y_f32) {
    const int64_t n = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    const int32_t* prow = packed + n * ld;
    const float bias_f = bias ? __bfloat162float(bias[n]) : 0.0f;
    for (int64_t m0 = 0; m0 < M; m0 += kSimtTok) {
        float acc[kSimtTok];
#pragma unroll
        for (int j = 0; j < kSimtTok; ++j) acc[j] = 0.0f;
        for (int64_t g = lane; g < KP; g += 32) {
            const uint32_t p = (uint32_t)__ldg(prow + g);
#pragma unroll
            for (int i = 0; i < kPerWord; ++i) {
                const int64_t k = g * kPerWord + i;
                if (k >= K) break;
                const float w = (float)((int)((p >> (3 * i)) & 7u) - 2);
#pragma unroll
                for (int j = 0; j < kSimtTok; ++j)
                    if (m0 + j < M) acc[j] = fmaf(w, __bfloat162float(x[(m0 + j) * K + k]), acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < kSimtTok; ++j)
            for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < kSimtTok; ++j) {
                const int64_t m = m0 + j;
                if (m >= M) break;
                const float yv = __fmul_rn(acc[j], scale);
                const __nv_bfloat16* res = residual ? residual + m * ld_res + n : nullptr;
                if (y_f32)
                    static_cast<float*>(y)[m * N + n] = epilogue_f32(yv, bias, bias_f, act, res);
                else
                    static_cast<__nv_bfloat16*>(y)[m * N + n] = epilogue_bf16(yv, bias, bias_f, act, res);
            }
        }
    }
}

cudaError_t launch_linear_simt_bf16(const LinearArgs& a, cudaStream_t s) {
    if (a.M == 0 || a.N == 0) return cudaSuccess;
    const int warps = 8;
    const unsigned blocks = (unsigned)((a.N + warps - 1) / warps);
    simt_bf16_kernel<<<blocks, warps * 32, 0, s>>>(static_cast<const __nv_bfloat16*>(a.x), a.M, a.K, a.packed, a.packed_ld, a.N,
                                                   a.KP, a.scale, static_cast<const __nv_bfloat16*>(a.bias),
                                                   static_cast<const __nv_bfloat16*>(a.residual), a.ld_res, a.act,
                                                   a.y, a.y_dtype == PN_F32);
    return cudaGetLastError();
}

}  // namespace pn
