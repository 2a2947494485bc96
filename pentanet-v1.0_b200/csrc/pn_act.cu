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
    // The product that reads this output may start its prologue and weight
    // streaming now (it waits for this grid before reading the output).
    asm volatile("griddepcontrol.launch_dependents;");
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

// bf16 rows with K % 8 == 0 and 16-byte aligned rows.  TPT threads per token
// (8 to 256, the fewest that hold the row in at most 16 pieces each, so that
// every thread has as many loads in flight as possible); each keeps its
// 16-byte pieces of the row in registers between the absmax and the quantise
// pass (one read of x) and writes 8 quantised bytes per piece.
//
// Same results as quant_act_i8_kernel, bit for bit.  rint(x / s) needs the
// correctly rounded quotient only where rounding to an integer can depend
// on it: q = x * (1/s) (reciprocal correctly rounded) is within 2 ulp of
// x / s, so unless q lies within 2^-14 of a half-integer (>= 16 ulp for
// |q| < 128) both round to the same integer.  q is rounded with the
// 1.5 * 2^23 addition (round to nearest, ties to even, for |q| < 2^22; the
// integer is then the low bits of the sum), all in FMA-pipe arithmetic.  The
// rare elements near a half-integer, and NaN, take the exact division.
// 16-byte pieces per thread: 8 (64 bf16) for rows up to 256 * 64 elements,
// 16 for rows up to twice that.  Sixteen pieces hold 64 registers of data
// (80+ per thread, two blocks per SM), which made the 4096 x 4096 case
// 1.5x slower than eight pieces with the same output.
constexpr int kActVecPiecesSmall = 8;
constexpr int kActVecPiecesLarge = 16;
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ int quant1(float xv, float s, float rs) {
    const float q = __fmul_rn(xv, rs);
    const float t = __fadd_rn(q, kRoundMagic);
    const float d = fabsf(__fsub_rn(q, __fsub_rn(t, kRoundMagic)));  // distance to the nearest integer
    if (d <= 0.5f - 0x1p-14f) return min(max(__float_as_int(t) - __float_as_int(kRoundMagic), -128), 127);
    float r = rintf(__fdiv_rn(xv, s));
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    return (int)r;
}

template <int TPT, int kActVecPieces>
__global__ void __launch_bounds__(kActThreads) quant_act_i8_vec_kernel(const uint4* __restrict__ x, int64_t M,
                                                                       int64_t K, int8_t* __restrict__ xq,
                                                                       int64_t pitch, float* __restrict__ s_x,
                                                                       int32_t* __restrict__ rowsum) {
    // The product that reads this output may start its prologue and weight
    // streaming now (it waits for this grid before reading the output).
    asm volatile("griddepcontrol.launch_dependents;");
    constexpr int kTokens = kActThreads / TPT;  // tokens per block
    constexpr int kWarpsPerToken = TPT / 32;     // 0 when a warp holds several tokens
    constexpr int kShfl = TPT < 32 ? TPT : 32;   // lanes of one token inside a warp
    __shared__ float red_f[kActThreads / 32];
    __shared__ int red_i[kActThreads / 32];
    const int t = threadIdx.x % TPT;
    const int64_t m = (int64_t)blockIdx.x * kTokens + threadIdx.x / TPT;
    const bool live = m < M;
    const int pieces = (int)(K / 8);          // 8 bf16 per piece
    const int out_pieces = (int)(pitch / 8);  // 8 int8 per output piece
    const uint4* row = x + (live ? m : 0) * pieces;
    uint4 v[kActVecPieces];
    uint32_t amax2 = 0;  // bf16x2 running max of |x|
#pragma unroll
    for (int i = 0; i < kActVecPieces; ++i) {
        const int c = t + i * TPT;
        v[i] = live && c < pieces ? __ldg(row + c) : make_uint4(0, 0, 0, 0);
        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t a;
            asm("abs.bf16x2 %0, %1;" : "=r"(a) : "r"(w[j]));
            asm("max.bf16x2 %0, %1, %2;" : "=r"(amax2) : "r"(amax2), "r"(a));
        }
    }
    float amax = fmaxf(__uint_as_float(amax2 << 16), __uint_as_float(amax2 & 0xFFFF0000u));
    for (int o = kShfl / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if constexpr (kWarpsPerToken > 1) {
        if ((threadIdx.x & 31) == 0) red_f[threadIdx.x >> 5] = amax;
        __syncthreads();
        const int w0 = (threadIdx.x / TPT) * kWarpsPerToken;  // this token's first warp
        amax = red_f[w0];
#pragma unroll
        for (int i = 1; i < kWarpsPerToken; ++i) amax = fmaxf(amax, red_f[w0 + i]);
    }
    float s = __fdiv_rn(amax, 127.0f);
    if (!(s > 0.0f)) s = 1.0f;
    const float rs = __frcp_rn(s);
    uint2* qrow = reinterpret_cast<uint2*>(xq + (live ? m : 0) * pitch);
    int sum = 0;
#pragma unroll
    for (int i = 0; i < kActVecPieces; ++i) {
        const int c = t + i * TPT;
        if (!live || c >= out_pieces) break;
        uint2 o = make_uint2(0, 0);
        if (c < pieces) {
            const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
            uint32_t b[2] = {0, 0};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int q0 = quant1(__uint_as_float(w[j] << 16), s, rs);
                const int q1 = quant1(__uint_as_float(w[j] & 0xFFFF0000u), s, rs);
                sum += q0 + q1;
                b[j >> 1] |= (((uint32_t)q0 & 0xFFu) | (((uint32_t)q1 & 0xFFu) << 8)) << (16 * (j & 1));
            }
            o = make_uint2(b[0], b[1]);
        }
        qrow[c] = o;
    }
    for (int o = kShfl / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if constexpr (kWarpsPerToken > 1) {
        if ((threadIdx.x & 31) == 0) red_i[threadIdx.x >> 5] = sum;
        __syncthreads();
        const int w0 = (threadIdx.x / TPT) * kWarpsPerToken;
        sum = 0;
#pragma unroll
        for (int i = 0; i < kWarpsPerToken; ++i) sum += red_i[w0 + i];
    }
    if (live && t == 0) {
        rowsum[m] = sum;
        s_x[m] = s;
    }
}

cudaError_t launch_quant_act_i8(const void* x, int x_dtype, int64_t M, int64_t K, int8_t* xq, int64_t pitch,
                                float* s_x, int32_t* rowsum, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    const bool vec = x_dtype == PN_BF16 && K % 8 == 0 && pitch % 8 == 0 &&
                     reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(xq) % 8 == 0;
    // pieces per thread: the fewer that lets kActThreads threads cover the row
    const int pieces_pt = pitch <= (int64_t)kActThreads * 8 * kActVecPiecesSmall ? kActVecPiecesSmall
                                                                                 : kActVecPiecesLarge;
    // threads per token: the fewest covering the row's output pieces, doubled
    // while the grid would have fewer than ~2 blocks per SM
    int tpt = 8;
    while (tpt < kActThreads && (int64_t)tpt * 8 * pieces_pt < pitch) tpt *= 2;
    const int64_t min_blocks = 2 * (int64_t)(device_sm_count() > 0 ? device_sm_count() : 148);
    while (tpt < kActThreads && M * tpt / kActThreads < min_blocks) tpt *= 2;
    if (vec && (int64_t)tpt * 8 * pieces_pt >= pitch) {
        const int tokens = kActThreads / tpt;
        const unsigned blocks = (unsigned)((M + tokens - 1) / tokens);
        const uint4* xv = static_cast<const uint4*>(x);
        auto go = [&](auto pc) {
            constexpr int PC = decltype(pc)::value;
            switch (tpt) {
                case 8: quant_act_i8_vec_kernel<8, PC><<<blocks, kActThreads, 0, s>>>(xv, M, K, xq, pitch, s_x, rowsum); break;
                case 16: quant_act_i8_vec_kernel<16, PC><<<blocks, kActThreads, 0, s>>>(xv, M, K, xq, pitch, s_x, rowsum); break;
                case 32: quant_act_i8_vec_kernel<32, PC><<<blocks, kActThreads, 0, s>>>(xv, M, K, xq, pitch, s_x, rowsum); break;
                case 64: quant_act_i8_vec_kernel<64, PC><<<blocks, kActThreads, 0, s>>>(xv, M, K, xq, pitch, s_x, rowsum); break;
                case 128: quant_act_i8_vec_kernel<128, PC><<<blocks, kActThreads, 0, s>>>(xv, M, K, xq, pitch, s_x, rowsum); break;
                default: quant_act_i8_vec_kernel<256, PC><<<blocks, kActThreads, 0, s>>>(xv, M, K, xq, pitch, s_x, rowsum); break;
            }
        };
        if (pieces_pt == kActVecPiecesSmall)
            go(std::integral_constant<int, kActVecPiecesSmall>{});
        else
            go(std::integral_constant<int, kActVecPiecesLarge>{});
    } else if (x_dtype == PN_F32)
        quant_act_i8_kernel<float><<<(unsigned)M, kActThreads, 0, s>>>(static_cast<const float*>(x), K, xq, pitch,
                                                                        s_x, rowsum);
    else
        quant_act_i8_kernel<__nv_bfloat16><<<(unsigned)M, kActThreads, 0, s>>>(
            static_cast<const __nv_bfloat16*>(x), K, xq, pitch, s_x, rowsum);
    return cudaGetLastError();
}

}  // namespace pn
