// pn_ternary2.cu -- the ternary (BitNet) weights in a 2-bit format: sixteen
// codes per int32, code = q + 1 in {0, 1, 2} at bits 2j..2j+1 for k = 16g + j
// of word g, rows of ceil(K / 16) words, padding code 1 (q = 0).  The rule is
// QuantLinear's bitnet mode (train_pentagpt.py:33-36): q = clamp(round(w /
// gamma), -1, 1), gamma = mean|W| clamped to 1e-8 (pn_absmean_scale), the
// same quotient rounding as the 3-bit packer.  2 bits per weight against the
// 3.2 of the 3-bit format (which holds the same ternary codes through
// pn_quantize_pack_ternary).
//
// The product runs on CUDA cores (one warp per weight row, 16 weights per
// packed word, fp32 sums, then the reference's scale / bias / bf16 rounding
// as penta_linear does): the format path, not a tuned decode kernel.  A code
// 3 (never written by the packer) reads as q = 2.
#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

constexpr int kPerWord2 = 16;

template <typename T>
__global__ void __launch_bounds__(256) quantize_pack_2bit_kernel(const T* __restrict__ w, int64_t N, int64_t K,
                                                                 int64_t KW, const float* __restrict__ d_scale,
                                                                 int32_t* __restrict__ packed) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= N * KW) return;
    const float gamma = __ldg(d_scale);
    const float rg = __frcp_rn(gamma);
    const int64_t n = idx / KW;
    const int64_t g = idx - n * KW;
    const T* row = w + n * K;
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < kPerWord2; ++i) {
        const int64_t k = g * kPerWord2 + i;
        // quant_code gives q + 2 for |q| <= 1
        const uint32_t code = k < K ? quant_code(load_as_float(row, k), gamma, rg, 1.0f) - 1u : 1u;
        word |= code << (2 * i);
    }
    packed[idx] = (int32_t)word;
}

__global__ void __launch_bounds__(256) unpack_2bit_kernel(const int32_t* __restrict__ packed, int64_t N, int64_t KW,
                                                          int64_t K, int8_t* __restrict__ out) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= N * KW) return;
    const int64_t n = idx / KW;
    const int64_t g = idx - n * KW;
    const uint32_t p = (uint32_t)__ldg(packed + idx);
#pragma unroll
    for (int i = 0; i < kPerWord2; ++i) {
        const int64_t k = g * kPerWord2 + i;
        if (k < K) out[n * K + k] = (int8_t)((int)((p >> (2 * i)) & 3u) - 1);
    }
}

constexpr int kT2Tok = 8;  // tokens per pass over a weight row

__global__ void __launch_bounds__(256) linear_2bit_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int64_t K,
                                                          const int32_t* __restrict__ packed, int64_t N, int64_t KW,
                                                          float scale, const __nv_bfloat16* __restrict__ bias,
                                                          void* __restrict__ y, int y_f32) {
    const int64_t n = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    const int32_t* prow = packed + n * KW;
    const float bias_f = bias ? __bfloat162float(bias[n]) : 0.0f;
    // 16-byte activation loads when every row of x is 16-byte aligned
    const bool vec = (K & 7) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    for (int64_t m0 = 0; m0 < M; m0 += kT2Tok) {
        const int nt = M - m0 < kT2Tok ? (int)(M - m0) : kT2Tok;
        float acc[kT2Tok];
#pragma unroll
        for (int j = 0; j < kT2Tok; ++j) acc[j] = 0.0f;
        for (int64_t g = lane; g < KW; g += 32) {
            const uint32_t p = (uint32_t)__ldg(prow + g);
            float q[kPerWord2];
#pragma unroll
            for (int i = 0; i < kPerWord2; ++i) q[i] = (float)((int)((p >> (2 * i)) & 3u) - 1);
            const int64_t k0 = g * kPerWord2;
            if (vec && k0 + kPerWord2 <= K) {
#pragma unroll
                for (int j = 0; j < kT2Tok; ++j) {
                    if (j >= nt) break;
                    const uint4* xr = reinterpret_cast<const uint4*>(x + (m0 + j) * K + k0);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint4 v = __ldg(xr + h);
                        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            acc[j] = fmaf(q[8 * h + 2 * e], __uint_as_float(u[e] << 16), acc[j]);
                            acc[j] = fmaf(q[8 * h + 2 * e + 1], __uint_as_float(u[e] & 0xFFFF0000u), acc[j]);
                        }
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < kPerWord2; ++i) {
                    const int64_t k = k0 + i;
                    if (k >= K) break;
#pragma unroll
                    for (int j = 0; j < kT2Tok; ++j)
                        if (j < nt) acc[j] = fmaf(q[i], __bfloat162float(x[(m0 + j) * K + k]), acc[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kT2Tok; ++j)
            for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < kT2Tok; ++j) {
                if (j >= nt) break;
                const int64_t m = m0 + j;
                const float yv = __fmul_rn(acc[j], scale);
                if (y_f32)
                    static_cast<float*>(y)[m * N + n] = epilogue_f32(yv, bias, bias_f, kActNone, nullptr);
                else
                    static_cast<__nv_bfloat16*>(y)[m * N + n] = epilogue_bf16(yv, bias, bias_f, kActNone, nullptr);
            }
        }
    }
}

}  // namespace pn

namespace {
int64_t words_2bit(int64_t K) { return (K + pn::kPerWord2 - 1) / pn::kPerWord2; }
unsigned grid_for(int64_t threads) { return (unsigned)((threads + 255) / 256); }
}  // namespace

extern "C" {

int64_t pn_words_2bit(int64_t K) { return K <= 0 ? 0 : words_2bit(K); }

int pn_quantize_pack_2bit(const void* w, int w_dtype, int64_t N, int64_t K, const float* d_scale, int32_t* packed,
                          void* stream) {
    if (!d_scale || ((!w || !packed) && N > 0)) return fail(PN_ERR_ARG, "pn_quantize_pack_2bit: null pointer");
    if (w_dtype != PN_F32 && w_dtype != PN_BF16) return fail(PN_ERR_DTYPE, "pn_quantize_pack_2bit: dtype %d", w_dtype);
    if (N < 0 || K < 1) return fail(PN_ERR_SHAPE, "pn_quantize_pack_2bit: N=%lld K=%lld", (long long)N, (long long)K);
    if (!aligned(w, w_dtype == PN_F32 ? 4 : 2) || !aligned(packed, 4) || !aligned(d_scale, 4))
        return fail(PN_ERR_ALIGN, "pn_quantize_pack_2bit: misaligned pointer");
    if (int st = check_device()) return st;
    if (N == 0) return ok();
    const int64_t KW = words_2bit(K);
    if (N * KW > (int64_t)0xffffffff * 256) return fail(PN_ERR_SHAPE, "pn_quantize_pack_2bit: too large");
    cudaStream_t s = (cudaStream_t)stream;
    if (w_dtype == PN_F32)
        pn::quantize_pack_2bit_kernel<float><<<grid_for(N * KW), 256, 0, s>>>(static_cast<const float*>(w), N, K, KW,
                                                                            d_scale, packed);
    else
        pn::quantize_pack_2bit_kernel<__nv_bfloat16><<<grid_for(N * KW), 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(w), N, K, KW, d_scale, packed);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_quantize_pack_2bit");
}

int pn_unpack_2bit(const int32_t* packed, int64_t N, int64_t K_words, int64_t K_orig, int8_t* out, void* stream) {
    if ((!packed || !out) && N > 0) return fail(PN_ERR_ARG, "pn_unpack_2bit: null pointer");
    if (N < 0 || K_words < 0 || K_orig < 0 || K_orig > K_words * pn::kPerWord2)
        return fail(PN_ERR_SHAPE, "pn_unpack_2bit: N=%lld K_words=%lld K_orig=%lld", (long long)N,
                    (long long)K_words, (long long)K_orig);
    if (!aligned(packed, 4)) return fail(PN_ERR_ALIGN, "pn_unpack_2bit: packed not 4-byte aligned");
    if (int st = check_device()) return st;
    if (N == 0 || K_words == 0) return ok();
    pn::unpack_2bit_kernel<<<grid_for(N * K_words), 256, 0, (cudaStream_t)stream>>>(packed, N, K_words, K_orig, out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_unpack_2bit");
}

int pn_linear_bf16_2bit(const void* x, int64_t M, int64_t K, const int32_t* packed, int64_t N, int64_t K_words,
                        float scale, const void* bias, void* y, int y_dtype, void* stream) {
    if ((!x && M > 0) || (!packed && N > 0) || (!y && M > 0 && N > 0))
        return fail(PN_ERR_ARG, "pn_linear_bf16_2bit: null pointer");
    if (y_dtype != PN_BF16 && y_dtype != PN_F32) return fail(PN_ERR_DTYPE, "pn_linear_bf16_2bit: y_dtype %d", y_dtype);
    if (M < 0 || N < 0 || K < 1 || N > (int64_t)0x7fffffff * 8)
        return fail(PN_ERR_SHAPE, "pn_linear_bf16_2bit: M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
    if (K_words != words_2bit(K))
        return fail(PN_ERR_SHAPE, "pn_linear_bf16_2bit: activation K=%lld needs K_words=%lld, got %lld",
                    (long long)K, (long long)words_2bit(K), (long long)K_words);
    if (!aligned(x, 2) || !aligned(packed, 4) || !aligned(y, y_dtype == PN_F32 ? 4 : 2) || !aligned(bias, 2))
        return fail(PN_ERR_ALIGN, "pn_linear_bf16_2bit: misaligned pointer");
    if (int st = check_device()) return st;
    if (M == 0 || N == 0) return ok();
    pn::linear_2bit_kernel<<<(unsigned)((N + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const __nv_bfloat16*>(x), M, K, packed, N, K_words, scale,
        static_cast<const __nv_bfloat16*>(bias), y, y_dtype == PN_F32);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_linear_bf16_2bit");
}

}  // extern "C"
