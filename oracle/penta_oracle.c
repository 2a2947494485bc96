/*
 * penta_oracle.c -- CPU restatement of PentaNet's packed pentanary path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against; nothing in the shipped library links, loads or calls it.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it.
 *
 * Every function restates one step of the reference implementation
 * (Kyworn/PentaNet-v1.0) and cites the file:line it follows.  It is written
 * in plain C without -ffast-math so that float division, round-half-even and
 * the accumulation order are the IEEE operations the reference performs on
 * the CPU.
 *
 * Encoding (penta_kernel.py:7-20): weight q in {-2,-1,0,+1,+2} is stored as
 * the 3-bit code q+2; weight k = 10*g + i of a row lives in bits [3i+2:3i] of
 * word g; bits 31:30 are zero; K is padded to a multiple of 10 with code 2.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define PNO_PER_WORD 10

int64_t pno_k_packs(int64_t K) { return (K + PNO_PER_WORD - 1) / PNO_PER_WORD; }

/* Sum of |w| in double, sequential order.  The reference computes
 * weight.float().abs().mean() (penta_kernel.py:57); a double sum of float
 * magnitudes rounds to the same float mean except in pathological cases, and
 * the golden fixtures pin the two against each other. */
double pno_abs_sum_f64(const float *w, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += fabs((double)w[i]);
    return s;
}

/* gamma = max(mean|W|, 1e-8) as a float (penta_kernel.py:57). */
float pno_absmean_scale(const float *w, int64_t n) {
    if (n <= 0) return 1e-8f;
    float mean = (float)(pno_abs_sum_f64(w, n) / (double)n);
    const float floor_v = 1e-8f;
    return mean > floor_v ? mean : floor_v;
}

/* Quantise one element: clamp(round_half_even(w / gamma), -2, 2)
 * (penta_kernel.py:60).  NaN has no defined result in the reference (its
 * int32 cast is platform dependent); it is mapped to 0 here and in the
 * CUDA kernel. */
static inline int pno_quant1(float w, float gamma, float qmax) {
    float t = w / gamma;                 /* IEEE float division */
    if (t != t) return 0;                /* NaN */
    float r = nearbyintf(t);             /* round half to even */
    if (r < -qmax) r = -qmax;
    if (r > qmax) r = qmax;
    return (int)r;
}

/* quantize_and_pack body for a given gamma (penta_kernel.py:60-78):
 * code = q + 2 (:70), packed |= code << 3i (:74-76), pad with code 2 (:62-65). */
static void pno_quantize_pack_q(const float *w, int64_t N, int64_t K, float gamma,
                                int32_t *packed, float qmax) {
    const int64_t KP = pno_k_packs(K);
    for (int64_t n = 0; n < N; ++n) {
        const float *row = w + n * K;
        for (int64_t g = 0; g < KP; ++g) {
            uint32_t word = 0;
            for (int i = 0; i < PNO_PER_WORD; ++i) {
                int64_t k = g * PNO_PER_WORD + i;
                uint32_t code = (k < K) ? (uint32_t)(pno_quant1(row[k], gamma, qmax) + 2) : 2u;
                word |= code << (3 * i);
            }
            packed[n * KP + g] = (int32_t)word;
        }
    }
}

void pno_quantize_pack(const float *w, int64_t N, int64_t K, float gamma, int32_t *packed) {
    pno_quantize_pack_q(w, N, K, gamma, packed, 2.0f);
}

/* The ternary (BitNet) mode of the reference's QuantLinear
 * (train_pentagpt.py:33-36): clamp(round(w / gamma), -1, 1), same absmean
 * gamma, stored in the same 3-bit codes (q + 2 in {1, 2, 3}). */
void pno_quantize_pack_ternary(const float *w, int64_t N, int64_t K, float gamma, int32_t *packed) {
    pno_quantize_pack_q(w, N, K, gamma, packed, 1.0f);
}

/* unpack_weights / penta_unpack_3bit (penta_kernel.py:81-90,
 * penta_avx2.c:41-59): ((p >> 3i) & 7) - 2, cropped to K_orig. */
void pno_unpack(const int32_t *packed, int64_t N, int64_t KP, int64_t K,
                int8_t *out) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t g = 0; g < KP; ++g) {
            uint32_t p = (uint32_t)packed[n * KP + g];
            for (int i = 0; i < PNO_PER_WORD; ++i) {
                int64_t k = g * PNO_PER_WORD + i;
                if (k < K) out[n * K + k] = (int8_t)((int)((p >> (3 * i)) & 7u) - 2);
            }
        }
}

/* Zero-multiplier fp32 matmul of the numba kernel (penta_kernel_cpu.py:35-60):
 * per (m, n) a float accumulator walks k in order and adds/subtracts x or
 * x + x by the weight value; the result is multiplied by gamma afterwards
 * (penta_kernel_cpu.py:97, penta_avx2.c:168).  Weights outside {-2..2}
 * contribute nothing, as in the numba branch chain. */
void pno_matmul_f32(const float *x, const int8_t *w, float *out, int64_t M,
                    int64_t N, int64_t K, float gamma) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            const float *xr = x + m * K;
            const int8_t *wr = w + n * K;
            float acc = 0.0f;
            for (int64_t k = 0; k < K; ++k) {
                float xk = xr[k];
                switch (wr[k]) {
                    case 1: acc += xk; break;
                    case -1: acc -= xk; break;
                    case 2: acc += xk + xk; break;
                    case -2: acc -= xk + xk; break;
                    default: break;
                }
            }
            out[m * N + n] = acc * gamma;
        }
}

/* Per-token int8 activation quantiser.  The reference's int8 line
 * (penta_avx2_wrapper.py:130-131) uses one absmax scale for the whole tensor:
 * s = absmax/127, xq = clamp(round(x/s), -128, 127).  Applied here row by row
 * (per token).  An all-zero row has no defined scale in the reference
 * (0/0); it is given s = 1 and a zero row. */
void pno_quant_act_i8(const float *x, int64_t M, int64_t K, int8_t *xq,
                      float *sx) {
    for (int64_t m = 0; m < M; ++m) {
        const float *xr = x + m * K;
        float amax = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            float a = fabsf(xr[k]);
            if (a > amax) amax = a;
        }
        float s = amax / 127.0f;
        if (!(s > 0.0f)) s = 1.0f;
        sx[m] = s;
        for (int64_t k = 0; k < K; ++k) {
            float r = nearbyintf(xr[k] / s);
            if (r < -128.0f) r = -128.0f;
            if (r > 127.0f) r = 127.0f;
            xq[m * K + k] = (int8_t)r;
        }
    }
}

/* torch._int_mm(xq, wq.T) (penta_avx2_wrapper.py:137): exact int32 dot
 * products, accumulated in int64 and narrowed (no overflow is possible for
 * |xq| <= 128, |w| <= 2, K < 2^22). */
void pno_matmul_i8(const int8_t *xq, const int8_t *w, int32_t *acc, int64_t M,
                   int64_t N, int64_t K) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            int64_t s = 0;
            const int8_t *xr = xq + m * K;
            const int8_t *wr = w + n * K;
            for (int64_t k = 0; k < K; ++k) s += (int64_t)xr[k] * (int64_t)wr[k];
            acc[m * N + n] = (int32_t)s;
        }
}

/* Int8 epilogue (penta_avx2_wrapper.py:147): y = float(acc) * (gamma * s_x),
 * with gamma * s_x formed in float, per token. */
void pno_dequant_i8(const int32_t *acc, const float *sx, int64_t M, int64_t N,
                    float gamma, float *y) {
    for (int64_t m = 0; m < M; ++m) {
        float f = gamma * sx[m];
        for (int64_t n = 0; n < N; ++n) y[m * N + n] = (float)acc[m * N + n] * f;
    }
}
