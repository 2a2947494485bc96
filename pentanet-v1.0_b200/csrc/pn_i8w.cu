// pn_i8w.cu -- the reference's CPU matmul ABI on the GPU: fp32 activations
// times pre-unpacked int8 weights in {-2..+2}, out = scale * x . w^T in fp32
// (penta_matmul_avx2, penta_avx2.c:87-171, which the reference calls after
// penta_unpack_3bit, penta_avx2_wrapper.py:42-90).  A compatibility entry for
// callers that already hold the unpacked int8 matrix; the packed products
// (pn_linear_bf16 and friends) read 3.2 bits per weight instead of 8.
//
// CUDA cores, one warp per weight row: lanes stride over the row 16 weights at
// a time (one 16-byte load when the row is 16-byte aligned, else byte loads),
// each weight converted to fp32 and multiplied into up to kI8wTok tokens'
// fp32 sums (the products are exact: |w| <= 2); the 32 lane sums are added in
// a fixed shuffle tree and the total is multiplied by scale once, as the
// reference does.
#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

constexpr int kI8wTok = 8;  // tokens per pass over a weight row

__global__ void __launch_bounds__(256) matmul_i8w_kernel(const float* __restrict__ x, const int8_t* __restrict__ w,
                                                         float* __restrict__ out, int64_t M, int64_t N, int64_t K,
                                                         float scale) {
    const int64_t n = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    const int8_t* wrow = w + n * K;
    const bool vec = (reinterpret_cast<uintptr_t>(wrow) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                     (K & 3) == 0;
    const int64_t K16 = vec ? (K & ~int64_t(15)) : 0;
    for (int64_t m0 = 0; m0 < M; m0 += kI8wTok) {
        const int nt = M - m0 < kI8wTok ? (int)(M - m0) : kI8wTok;
        float acc[kI8wTok];
#pragma unroll
        for (int j = 0; j < kI8wTok; ++j) acc[j] = 0.0f;
        for (int64_t k = (int64_t)lane * 16; k < K16; k += 32 * 16) {
            const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wrow + k));
            const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
            float wf[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) wf[i] = (float)(int8_t)(wr[i >> 2] >> (8 * (i & 3)));
#pragma unroll
            for (int j = 0; j < kI8wTok; ++j) {
                if (j >= nt) break;
                const float4* xr = reinterpret_cast<const float4*>(x + (m0 + j) * K + k);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 xv = __ldg(xr + q);
                    acc[j] = __fmaf_rn(xv.x, wf[4 * q + 0], acc[j]);
                    acc[j] = __fmaf_rn(xv.y, wf[4 * q + 1], acc[j]);
                    acc[j] = __fmaf_rn(xv.z, wf[4 * q + 2], acc[j]);
                    acc[j] = __fmaf_rn(xv.w, wf[4 * q + 3], acc[j]);
                }
            }
        }
        // the rest of the row (or all of it when unaligned), one weight per lane
        for (int64_t k = K16 + lane; k < K; k += 32) {
            const float wf = (float)__ldg(wrow + k);
#pragma unroll
            for (int j = 0; j < kI8wTok; ++j) {
                if (j >= nt) break;
                acc[j] = __fmaf_rn(__ldg(x + (m0 + j) * K + k), wf, acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < kI8wTok; ++j) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[j] = __fadd_rn(acc[j], __shfl_xor_sync(0xffffffffu, acc[j], o));
        }
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < kI8wTok; ++j)
                if (j < nt) out[(m0 + j) * N + n] = __fmul_rn(acc[j], scale);
        }
    }
}

}  // namespace pn

extern "C" int pn_matmul_i8w(const float* x, const int8_t* w, float* out, int64_t M, int64_t N, int64_t K,
                             float scale, void* stream) {
    if ((M > 0 && K > 0 && !x) || (N > 0 && K > 0 && !w) || (M > 0 && N > 0 && !out))
        return fail(PN_ERR_ARG, "pn_matmul_i8w: null pointer");
    if (M < 0 || N < 0 || K < 0)
        return fail(PN_ERR_SHAPE, "pn_matmul_i8w: M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
    if (!aligned(x, 4) || !aligned(out, 4)) return fail(PN_ERR_ALIGN, "pn_matmul_i8w: x and out need 4-byte alignment");
    if (int st = check_device()) return st;
    if (M == 0 || N == 0) return ok();
    if (K == 0) {
        const cudaError_t e = cudaMemsetAsync(out, 0, (size_t)M * N * sizeof(float), (cudaStream_t)stream);
        return e == cudaSuccess ? ok() : cuda_fail(e, "pn_matmul_i8w");
    }
    const int64_t blocks = (N + 7) / 8;  // 8 warps per block, one row each
    if (blocks > 0x7fffffff) return fail(PN_ERR_SHAPE, "pn_matmul_i8w: N=%lld too large", (long long)N);
    pn::matmul_i8w_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, w, out, M, N, K, scale);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_matmul_i8w");
}
