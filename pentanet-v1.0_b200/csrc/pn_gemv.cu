// pn_gemv.cu -- decode GEMV for a few tokens on the CUDA cores.
//
// The same product as the tensor-core kernel (y = scale * x . w, w in {-2..2}
// packed ten 3-bit codes per int32, penta_kernel.py:111-224) for decode
// batches of a few tokens, where a tensor-core tile computes 16 token columns
// for one or two real ones and its operand pipeline, not HBM, bounds the time.
//
// Each weight enters an FMA with one logical AND and no conversion: the float
// whose bit pattern is the packed word masked to one code, `p & (7 << 3j)`, is
// the fp32 subnormal c * 2^(3j - 149) (c = q + 2, the stored code).  Codes
// 7..9 sit at bits 21-29, beyond the 23-bit mantissa, so they are taken from
// p >> 9 (bit positions 12, 15, 18).  The activation pre-pass stores, per
// token t, ten planes j of x[10w + j] * 2^(100 - E_t - e_j) (e_j the code's
// bit position in its masked word, E_t = floor(log2 max|x_t|)), so every
// product is c * x * 2^(-49 - E_t): exact, normal for |x| >= 2^(E_t - 77),
// and the sum over a row stays far from overflow.  The codes carry the +2
// offset of the packed format, so the pre-pass also sums 2 x_k in the same
// units, and the epilogue subtracts that sum, rescales by 2^(49 + E_t)
// (exact) and applies the tensor-core path's epilogue (scale, bias with the
// reference's double rounding, optional GELU / residual, bf16 or fp32 out).
// The pairs of an FMA are two adjacent words of one row (packed fp32x2 FMA:
// one instruction, two products), which the plane layout makes adjacent
// floats of one 16-byte shared-memory load.
//
// Kernel layout: one persistent CTA per SM, one producer warp and eight
// consumer warps.  The producer streams weight boxes (RT rows x 256 words,
// TMA, no swizzle) into a ring of shared-memory stages and, once, copies the
// activation planes of the CTA's K window into shared memory (bulk copies);
// in-flight bytes live in shared memory, not registers.  In a stage, warp w
// takes words [32 (w mod 8), +32) of one half of the rows (w / 8); lane l
// takes four words (l mod 8) of the rows l/8 + 4i of that half.  The CTAs split K into windows whose activations fit in
// shared memory (one window for the 70B-class decode shapes up to 4 tokens)
// and the output rows into ranges of whole row tiles; with several windows
// each writes fp32 partial sums that a second kernel adds in window order.
// Every sum has a fixed order, so results are deterministic.
#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

constexpr int kGvSlices = 8;                          // 32-word slices of a box row
constexpr int kGvConsumers = 16;                      // consumer warps: slice x row half
constexpr int kGvThreads = 32 * (kGvConsumers + 1);   // + one producer warp
constexpr int kGvBoxWords = 256;                      // words per row of a weight box
constexpr int kGvPrepWords = 256;                     // words per pre-pass block
constexpr int kGvSmemBudget = 227 * 1024;

__host__ __device__ constexpr int gv_code_exp(int j) { return j <= 6 ? 3 * j : 3 * j - 9; }
__host__ __device__ constexpr int64_t gv_round4(int64_t v) { return (v + 3) & ~int64_t(3); }

// Pre-pass, grid (ceil(KP / 256), M): planes[t][j][w] = x[t][10w + j] *
// 2^(100 - E_t - e_j) (zero for k >= K and for KP <= w < round4(KP)),
// E[t] = E_t, off_part[t][b] = block b's sum of 2 x_k 2^(-49 - E_t).
__global__ void __launch_bounds__(256) gemv_xprep_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int K,
                                                         int KP, float* __restrict__ planes,
                                                         int* __restrict__ E_out, float* __restrict__ off_part) {
    // x may be the previous product's output and the planes its workspace: wait for it.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ float red[8];
    const int t = blockIdx.y;
    const int KP4 = (int)gv_round4(KP);
    const __nv_bfloat16* xr = x + (int64_t)t * ldx;
    float mx = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(__bfloat162float(xr[k])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
    const int E = (mx > 0.0f && isfinite(mx)) ? ilogbf(mx) : 0;
    if (blockIdx.x == 0 && threadIdx.x == 0) E_out[t] = E;
    const int w0 = blockIdx.x * kGvPrepWords;
    float osum = 0.0f;
    float* pl = planes + (int64_t)t * kPerWord * KP4;
    for (int i = threadIdx.x; i < kGvPrepWords * kPerWord; i += blockDim.x) {
        const int j = i / kGvPrepWords;          // plane
        const int w = w0 + i % kGvPrepWords;     // word (consecutive threads: consecutive words)
        if (w >= KP4) continue;
        const int k = w * kPerWord + j;
        float v = 0.0f;
        if (w < KP && k < K) {
            const float xv = __bfloat162float(xr[k]);
            v = ldexpf(xv, 100 - E - gv_code_exp(j));
            osum += ldexpf(xv, -48 - E);
        }
        pl[(int64_t)j * KP4 + w] = v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) osum += __shfl_xor_sync(0xffffffffu, osum, o);
    __syncthreads();  // red is reused
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = osum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) s += red[i];
        off_part[(int64_t)t * gridDim.x + blockIdx.x] = s;
    }
}

struct GemvParams {
    int64_t N;
    int KP, KP4, M;
    int KW;              // words per K window (multiple of 256)
    int nwin, groups;    // grid = nwin x groups
    int ntile;           // row tiles of RT rows
    const float* planes; // pre-pass output
    const int* E;
    const float* off_part;
    int n_off_part;
    float* partial;      // [nwin][M][N] fp32 when nwin > 1
    float scale;
    const __nv_bfloat16* bias;
    const __nv_bfloat16* residual;
    int64_t ld_res;
    int act;
    void* y_out[8];
    int n_out;
    int64_t ld_y, y_col0;
    int y_f32;
};

__device__ __forceinline__ uint4 lds128_u(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 lds128_f(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// acc.{x,y} += {a, b} * {xa, xb} as one packed fp32 FMA (a, b: masked words,
// i.e. fp32 subnormals; no flush to zero).
__device__ __forceinline__ void fma2(float2& acc, uint32_t a, uint32_t b, float xa, float xb) {
    unsigned long long av, xv, cv;
    asm("mov.b64 %0, {%1, %2};" : "=l"(av) : "r"(a), "r"(b));
    asm("mov.b64 %0, {%1, %2};" : "=l"(xv) : "f"(xa), "f"(xb));
    asm("mov.b64 %0, {%1, %2};" : "=l"(cv) : "f"(acc.x), "f"(acc.y));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(cv) : "l"(av), "l"(xv));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(acc.x), "=f"(acc.y) : "l"(cv));
}

// The output of one (row, token) sum: offset, rescale, the shared epilogue,
// stores into every output buffer.
__device__ __forceinline__ void gemv_store(const GemvParams& p, int64_t n, int t, float sum) {
    float off = 0.0f;
    for (int b = 0; b < p.n_off_part; ++b) off += p.off_part[(int64_t)t * p.n_off_part + b];
    const float v = ldexpf(__fsub_rn(sum, off), 49 + p.E[t]);  // exact: back from units of 2^(-49 - E_t)
    const float yv = __fmul_rn(v, p.scale);
    const float bias_f = p.bias ? __bfloat162float(p.bias[n]) : 0.0f;
    const __nv_bfloat16* res = p.residual ? p.residual + (int64_t)t * p.ld_res + n : nullptr;
    const int64_t at = (int64_t)t * p.ld_y + p.y_col0 + n;
    if (p.y_f32) {
        const float o = epilogue_f32(yv, p.bias, bias_f, p.act, res);
        for (int d = 0; d < p.n_out; ++d) static_cast<float*>(p.y_out[d])[at] = o;
    } else {
        const __nv_bfloat16 o = epilogue_bf16(yv, p.bias, bias_f, p.act, res);
        for (int d = 0; d < p.n_out; ++d) static_cast<__nv_bfloat16*>(p.y_out[d])[at] = o;
    }
}

}  // namespace pn

namespace pn {

// Rows per lane (RPL) and ring depth by token count: one or two tokens keep
// four rows per lane (16-row boxes, 16 KB stages), more tokens two.
template <int MT>
struct GvCfg {
    static constexpr int RPL = MT <= 2 ? 4 : 2;
    static constexpr int RT = 4 * RPL;                      // rows per tile / box
    static constexpr int kStageBytes = RT * kGvBoxWords * 4;
    static constexpr int S = MT <= 2 ? 6 : 8;               // ring stages
    static constexpr int RH = RPL / 2;                      // rows per lane in a warp's half
    static constexpr int kRedBytes = 2 * kGvSlices * RT * MT * 4;  // double-buffered
    static constexpr int kFixed = S * kStageBytes + kRedBytes + (2 * S + 1) * 8 + 16 + 1024;
};

template <int MT>
__global__ void __launch_bounds__(kGvThreads, 1)
    gemv_kernel(const __grid_constant__ CUtensorMap wmap, const GemvParams p) {
    using C = GvCfg<MT>;
    constexpr int RH = C::RH;
    constexpr int RT = C::RT;
    constexpr int S = C::S;
    // The next product's pre-pass may be scheduled now (it waits for this grid
    // before it touches memory).
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint32_t* stages = reinterpret_cast<uint32_t*>(smem);
    float* xsm = reinterpret_cast<float*>(smem + S * C::kStageBytes);
    float* red = xsm + (size_t)MT * kPerWord * p.KW;
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kGvSlices * RT * MT);
    uint64_t* empty = full + S;
    uint64_t* xbar = empty + S;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(xbar + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int win = blockIdx.x / p.groups;
    const int grp = blockIdx.x % p.groups;
    const int kw0 = win * p.KW;
    const int kw1 = min(p.KP, kw0 + p.KW);
    const int nkb = (kw1 - kw0 + kGvBoxWords - 1) / kGvBoxWords;
    const int tile0 = (int)((int64_t)grp * p.ntile / p.groups);
    const int tile1 = (int)((int64_t)(grp + 1) * p.ntile / p.groups);
    const uint32_t total = (uint32_t)(tile1 - tile0) * (uint32_t)nkb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGvConsumers);
        }
        mbar_init(xbar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kGvConsumers) {
        // ------------------------------------------------------ producer ----
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            bool ok = true, xissued = false;
            uint32_t it = 0;
            auto issue = [&](uint32_t i) -> bool {
                const int s = (int)(i % S);
                if (!mbar_wait(&empty[s], ((i / S) & 1) ^ 1, abort_flag)) return false;
                mbar_arrive_expect_tx(&full[s], C::kStageBytes);
                tma_load_2d(stages + s * (C::kStageBytes / 4), &wmap, &full[s],
                            kw0 + (int)(i % nkb) * kGvBoxWords, (tile0 + (int)(i / nkb)) * RT);
                return true;
            };
            // weights first (they do not depend on the pre-pass) ...
            for (; it < total && it < (uint32_t)S && ok; ++it) ok = issue(it);
            // ... then the activation planes of this window, written by the pre-pass
            asm volatile("griddepcontrol.wait;" ::: "memory");
            if (ok) {
                const int len4 = (int)gv_round4(kw1 - kw0);
                mbar_arrive_expect_tx(xbar, (uint32_t)(MT * kPerWord * len4 * 4));
                for (int t = 0; t < MT; ++t)
                    for (int j = 0; j < kPerWord; ++j)
                        bulk_load(xsm + (size_t)(t * kPerWord + j) * p.KW,
                                  p.planes + ((int64_t)t * kPerWord + j) * p.KP4 + kw0, (uint32_t)(len4 * 4), xbar);
                xissued = true;
            }
            for (; it < total && ok; ++it) ok = issue(it);
            if (!ok) {
                // let every issued copy land before the CTA exits
                for (uint32_t j = it > (uint32_t)S ? it - S : 0u; j < it; ++j)
                    mbar_wait_drain(&full[j % S], (j / S) & 1);
                if (xissued) mbar_wait_drain(xbar, 0);
            }
        }
    } else {
        // ----------------------------------------------------- consumers ----
        const int slice = warp % kGvSlices;  // 32-word slice of the box row
        const int half = warp / kGvSlices;   // half of the tile's rows
        const int wq = lane & 7;             // which four words of the slice
        const int rl = half * (RT / 2) + (lane >> 3);  // first row of the lane (then rl + 4, ...)
        const uint32_t stage0 = smem_u32(stages) + (uint32_t)((rl * kGvBoxWords + 32 * slice + 4 * wq) * 4);
        const uint32_t x0 = smem_u32(xsm);
        // the epilogue reads the pre-pass's per-token exponents and offsets
        asm volatile("griddepcontrol.wait;" ::: "memory");
        bool ok = warp_wait(xbar, 0, abort_flag);
        uint32_t st = 0;
        int parity = 0;
        for (int tile = tile0; tile < tile1; ++tile, parity ^= 1) {
            float2 acc[RH][MT][2];
#pragma unroll
            for (int r = 0; r < RH; ++r)
#pragma unroll
                for (int t = 0; t < MT; ++t) acc[r][t][0] = acc[r][t][1] = make_float2(0.0f, 0.0f);
            for (int kb = 0; kb < nkb; ++kb, ++st) {
                const int s = (int)(st % S);
                // after an abort the loop still runs (no waits, no work) so that
                // every consumer warp reaches the same named barriers
                if (ok) ok = warp_wait(&full[s], (st / S) & 1, abort_flag);
                const int wl = kb * kGvBoxWords + 32 * slice + 4 * wq;  // word offset in the window
                if (ok && kw0 + wl < kw1) {
                    const uint32_t sa = stage0 + (uint32_t)(s * C::kStageBytes);
                    uint4 P[RH], Q[RH];
#pragma unroll
                    for (int r = 0; r < RH; ++r) {
                        P[r] = lds128_u(sa + (uint32_t)(4 * r * kGvBoxWords * 4));
                        Q[r] = make_uint4(P[r].x >> 9, P[r].y >> 9, P[r].z >> 9, P[r].w >> 9);
                    }
#pragma unroll
                    for (int j = 0; j < kPerWord; ++j) {
                        float4 X[MT];
#pragma unroll
                        for (int t = 0; t < MT; ++t)
                            X[t] = lds128_f(x0 + (uint32_t)((((t * kPerWord + j) * p.KW) + wl) * 4));
                        constexpr uint32_t kMask[kPerWord] = {7u,       7u << 3,  7u << 6,  7u << 9,  7u << 12,
                                                              7u << 15, 7u << 18, 7u << 12, 7u << 15, 7u << 18};
#pragma unroll
                        for (int r = 0; r < RH; ++r) {
                            const uint4 src = j <= 6 ? P[r] : Q[r];
                            const uint32_t a0 = src.x & kMask[j], a1 = src.y & kMask[j];
                            const uint32_t a2 = src.z & kMask[j], a3 = src.w & kMask[j];
#pragma unroll
                            for (int t = 0; t < MT; ++t) {
                                fma2(acc[r][t][0], a0, a1, X[t].x, X[t].y);
                                fma2(acc[r][t][1], a2, a3, X[t].z, X[t].w);
                            }
                        }
                    }
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(&empty[s]);
            }
            // the tile's sums: the 8 lanes of a row, then the 8 slices (fixed order)
#pragma unroll
            for (int r = 0; r < RH; ++r)
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    float v = (acc[r][t][0].x + acc[r][t][0].y) + (acc[r][t][1].x + acc[r][t][1].y);
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    v += __shfl_xor_sync(0xffffffffu, v, 4);
                    if (wq == 0) red[((parity * kGvSlices + slice) * RT + rl + 4 * r) * MT + t] = v;
                }
            // One barrier per tile: red is double-buffered by tile parity, and the
            // next barrier orders this tile's reads before the buffer's reuse.
            asm volatile("bar.sync 1, %0;" ::"n"(kGvConsumers * 32) : "memory");
            for (int i = threadIdx.x; i < RT * MT; i += kGvConsumers * 32) {
                const int64_t n = (int64_t)tile * RT + i / MT;
                const int t = i % MT;
                if (n >= p.N || !ok) continue;
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < kGvSlices; ++w) sum += red[(parity * kGvSlices + w) * RT * MT + i];
                if (p.nwin == 1)
                    gemv_store(p, n, t, sum);
                else
                    p.partial[((int64_t)win * p.M + t) * p.N + n] = sum;
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kGvConsumers * 32) : "memory");
        if (p.n_out > 1 && p.nwin == 1 && threadIdx.x == 0) __threadfence_system();  // peer stores, then the barrier kernel
    }
}

// Several K windows: out = sum of the windows' partials in window order.
__global__ void __launch_bounds__(256) gemv_finish_kernel(const GemvParams p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int64_t total = (int64_t)p.M * p.N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / p.N);
        const int64_t n = i - (int64_t)t * p.N;
        float sum = 0.0f;
        for (int w = 0; w < p.nwin; ++w) sum += p.partial[((int64_t)w * p.M + t) * p.N + n];
        gemv_store(p, n, t, sum);
    }
    if (p.n_out > 1) {
        __syncthreads();
        if (threadIdx.x == 0) __threadfence_system();
    }
}

}  // namespace pn

namespace pn {

namespace {
int g_gemv_max_tokens = kGemvMaxTokensDefault;

size_t gv_align(size_t b) { return (b + 255) & ~size_t(255); }
int gv_prep_blocks(int64_t KP) { return (int)((KP + kGvPrepWords - 1) / kGvPrepWords); }

struct GvPlan {
    int KW = 0, nwin = 0;
    size_t smem = 0;
};

template <int MT>
GvPlan gv_plan_mt(int64_t KP) {
    using C = GvCfg<MT>;
    GvPlan g;
    const int64_t budget = (int64_t)kGvSmemBudget - C::kFixed;
    int64_t kw = budget / ((int64_t)MT * kPerWord * 4) / kGvBoxWords * kGvBoxWords;
    if (kw < kGvBoxWords) return g;
    const int64_t nwin = (KP + kw - 1) / kw;
    // equal windows, each a whole number of boxes
    kw = ((KP + nwin - 1) / nwin + kGvBoxWords - 1) / kGvBoxWords * kGvBoxWords;
    g.KW = (int)kw;
    g.nwin = (int)((KP + kw - 1) / kw);
    g.smem = (size_t)C::kFixed + (size_t)MT * kPerWord * kw * 4;
    return g;
}

GvPlan gv_plan(int64_t M, int64_t KP) {
    switch (M) {
        case 1: return gv_plan_mt<1>(KP);
        case 2: return gv_plan_mt<2>(KP);
        case 3: return gv_plan_mt<3>(KP);
        case 4: return gv_plan_mt<4>(KP);
        case 5: return gv_plan_mt<5>(KP);
        case 6: return gv_plan_mt<6>(KP);
        case 7: return gv_plan_mt<7>(KP);
        default: return gv_plan_mt<8>(KP);
    }
}

struct GvLayout {
    size_t planes, E, off, partial, total;
};
GvLayout gv_layout(int64_t M, int64_t N, int64_t KP, const GvPlan& g) {
    GvLayout L;
    L.planes = 0;
    L.E = gv_align((size_t)M * kPerWord * gv_round4(KP) * sizeof(float));
    L.off = L.E + gv_align((size_t)M * sizeof(int));
    L.partial = L.off + gv_align((size_t)M * gv_prep_blocks(KP) * sizeof(float));
    L.total = L.partial + (g.nwin > 1 ? gv_align((size_t)g.nwin * M * N * sizeof(float)) : 0);
    return L;
}

template <int MT>
cudaError_t gemv_launch_mt(const CUtensorMap& wmap, const GemvParams& prm, size_t smem, cudaStream_t s) {
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kGvSmemBudget);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(prm.nwin * prm.groups));
    cfg.blockDim = dim3(kGvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    // Programmatic dependent of the pre-pass: weight streaming starts before
    // griddepcontrol.wait; the activation planes are copied after it.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<MT>, wmap, prm);
}
}  // namespace

int gemv_max_tokens() { return g_gemv_max_tokens; }
void set_gemv_max_tokens(int m) { g_gemv_max_tokens = m < 0 ? 0 : (m > kGemvMaxTokens ? kGemvMaxTokens : m); }

size_t gemv_workspace_bytes(int64_t M, int64_t N, int64_t KP) {
    if (M < 1 || M > kGemvMaxTokens || N < 1) return 0;
    const GvPlan g = gv_plan(M, KP);
    if (g.nwin == 0) return 0;
    return gv_layout(M, N, KP, g).total;
}

bool gemv_takes(const LinearArgs& a) {
    if (a.kind != PN_BF16 || a.M < 1 || a.M > g_gemv_max_tokens || a.N < 1) return false;
    if (a.packed_ld % 4 != 0 || a.KP > 0x3fffffff || a.K > 0x7fffffff || a.N > 0x7fffffff) return false;
    const GvPlan g = gv_plan(a.M, a.KP);
    if (g.nwin == 0) return false;
    return a.workspace != nullptr && reinterpret_cast<uintptr_t>(a.workspace) % 256 == 0 &&
           a.workspace_bytes >= gv_layout(a.M, a.N, a.KP, g).total;
}

cudaError_t launch_gemv(const LinearArgs& a, cudaStream_t s) {
    const GvPlan g = gv_plan(a.M, a.KP);
    const GvLayout L = gv_layout(a.M, a.N, a.KP, g);
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    float* planes = reinterpret_cast<float*>(ws + L.planes);
    int* E = reinterpret_cast<int*>(ws + L.E);
    float* off = reinterpret_cast<float*>(ws + L.off);
    const int nb = gv_prep_blocks(a.KP);
    gemv_xprep_kernel<<<dim3(nb, (unsigned)a.M), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(a.x), a.x_pitch,
                                                               (int)a.K, (int)a.KP, planes, E, off);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    const int RT = a.M <= 2 ? 16 : 8;  // GvCfg<MT>::RT
    EncodeTiledFn encode = get_encode_fn();
    if (!encode) return cudaErrorNotSupported;
    CUtensorMap wmap;
    {
        cuuint64_t dims[2] = {(cuuint64_t)a.KP, (cuuint64_t)a.N};
        cuuint64_t strides[1] = {(cuuint64_t)(a.packed_ld * 4)};
        cuuint32_t box[2] = {(cuuint32_t)kGvBoxWords, (cuuint32_t)RT};
        cuuint32_t estr[2] = {1, 1};
        if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(a.packed), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    GemvParams prm{};
    prm.N = a.N;
    prm.KP = (int)a.KP;
    prm.KP4 = (int)gv_round4(a.KP);
    prm.M = (int)a.M;
    prm.KW = g.KW;
    prm.nwin = g.nwin;
    prm.ntile = (int)((a.N + RT - 1) / RT);
    const int sms = device_sm_count() > 0 ? device_sm_count() : 148;
    int groups = sms / g.nwin > 0 ? sms / g.nwin : 1;
    if (groups > prm.ntile) groups = prm.ntile;
    prm.groups = groups;
    prm.planes = planes;
    prm.E = E;
    prm.off_part = off;
    prm.n_off_part = nb;
    prm.partial = g.nwin > 1 ? reinterpret_cast<float*>(ws + L.partial) : nullptr;
    prm.scale = a.scale;
    prm.bias = static_cast<const __nv_bfloat16*>(a.bias);
    prm.residual = static_cast<const __nv_bfloat16*>(a.residual);
    prm.ld_res = a.ld_res;
    prm.act = a.act;
    if (a.n_peers > 0) {
        prm.n_out = a.n_peers;
        for (int r = 0; r < 8; ++r) prm.y_out[r] = r < a.n_peers ? a.y_peers[r] : nullptr;
        prm.ld_y = a.ld_y;
        prm.y_col0 = a.y_col0;
    } else {
        prm.n_out = 1;
        prm.y_out[0] = a.y;
        prm.ld_y = a.N;
        prm.y_col0 = 0;
    }
    prm.y_f32 = a.y_dtype == PN_F32;
    switch (a.M) {
        case 1: e = gemv_launch_mt<1>(wmap, prm, g.smem, s); break;
        case 2: e = gemv_launch_mt<2>(wmap, prm, g.smem, s); break;
        case 3: e = gemv_launch_mt<3>(wmap, prm, g.smem, s); break;
        case 4: e = gemv_launch_mt<4>(wmap, prm, g.smem, s); break;
        case 5: e = gemv_launch_mt<5>(wmap, prm, g.smem, s); break;
        case 6: e = gemv_launch_mt<6>(wmap, prm, g.smem, s); break;
        case 7: e = gemv_launch_mt<7>(wmap, prm, g.smem, s); break;
        default: e = gemv_launch_mt<8>(wmap, prm, g.smem, s); break;
    }
    if (e != cudaSuccess || g.nwin == 1) return e;
    cudaLaunchConfig_t cfg = {};
    const int64_t total = a.M * a.N;
    cfg.gridDim = dim3((unsigned)((total + 255) / 256 < 2048 ? (total + 255) / 256 : 2048));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_finish_kernel, prm);
}

}  // namespace pn
