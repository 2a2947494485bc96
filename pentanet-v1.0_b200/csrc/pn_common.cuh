// pn_common.cuh -- shared device helpers for the PentaNet sm_100a kernels.
//
// Inline-PTX wrappers for mbarriers (every wait is bounded by a wall-clock
// limit and reports a status instead of spinning forever), TMA tensor loads,
// cp.async staging and the tcgen05 tensor-memory / MMA instructions.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "pentanet_b200.h"

namespace pn {

// 3-bit encoding (penta_kernel.py:7-20): code = q + 2, ten codes per int32.
constexpr int kPerWord = 10;
// A word holding ten zero weights (code 2 everywhere).
constexpr uint32_t kZeroWord = 0x12492492u;

// Device-side status word: kernels that give up on a bounded wait record the
// reason here (first writer wins); the host reads it with pn_device_status().
__device__ int g_device_status = 0;

// Epilogue activations (pn_act_code in the C header).
constexpr int kActNone = 0;
constexpr int kActGelu = 1;

// GELU, erf form, in fp32 with torch's operation order for bf16 tensors
// (x * 0.5 * (1 + erf(x * sqrt(1/2))), the approximate='none' nn.GELU of the
// GPT's MLP, train_pentagpt.py:80,86); erff is CUDA's.
__device__ __forceinline__ float gelu_erf(float v) {
    return __fmul_rn(__fmul_rn(v, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn(v, 0.7071067811865476f))));
}

// The epilogue after the product's bf16 rounding, in the order the reference
// model applies the separate ops: + bias (bf16(t + bf16 bias),
// penta_kernel.py:275-276), the activation (bf16(gelu(t))), then the residual
// stream (bf16(res + t), train_pentagpt.py:100-101).
__device__ __forceinline__ __nv_bfloat16 epilogue_bf16(float yv, const __nv_bfloat16* bias_n, float bias_f, int act,
                                                       const __nv_bfloat16* res) {
    __nv_bfloat16 t = __float2bfloat16_rn(yv);
    if (bias_n) t = __float2bfloat16_rn(__fadd_rn(__bfloat162float(t), bias_f));
    if (act == kActGelu) t = __float2bfloat16_rn(gelu_erf(__bfloat162float(t)));
    if (res) t = __float2bfloat16_rn(__fadd_rn(__bfloat162float(*res), __bfloat162float(t)));
    return t;
}
// The fp32-output form: no intermediate rounding.
__device__ __forceinline__ float epilogue_f32(float yv, const __nv_bfloat16* bias_n, float bias_f, int act,
                                             const __nv_bfloat16* res) {
    if (bias_n) yv = __fadd_rn(yv, bias_f);
    if (act == kActGelu) yv = gelu_erf(yv);
    if (res) yv = __fadd_rn(__bfloat162float(*res), yv);
    return yv;
}

__device__ __forceinline__ void record_status(int code) {
    atomicCAS(&g_device_status, 0, code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------ mbarrier ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// Limit of one barrier wait, in SM clock cycles (2^32 cycles: 2.2 s at the
// 1965 MHz boost clock, longer at lower clocks).  Healthy waits last
// microseconds; a wait that reaches the limit means a producer is gone.
constexpr long long kWaitLimitCycles = 1ll << 32;

// Bounded wait.  Returns false (and records PN_ERR_TIMEOUT) when the limit is
// reached or another thread of the CTA has already aborted (*abort != 0).
// A wait that does not complete at once backs off with nanosleep (8 ns doubling
// to 256 ns) so that waiting warps leave the issue slots to working ones.
// Non-blocking probe of a phase: cheaper than try_wait when the phase has
// already completed (~20-30 cycles against ~50-70 on B200), which is the
// common case for well-fed pipeline stages.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_test_wait(bar, parity)) return true;
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    uint32_t ns = 8;
    while (true) {
        __nanosleep(ns);
        if (mbar_try_wait(bar, parity)) return true;
        if (ns < 256) ns <<= 1;
        if (*abort) return false;
        if (clock64() - t0 > kWaitLimitCycles) {
            *abort = 1;
            record_status(PN_ERR_TIMEOUT);
            return false;
        }
    }
}

// Warp-uniform bounded wait: every lane waits (and so acquires the barrier's
// data), and the warp agrees on the outcome so that no .sync.aligned
// instruction afterwards sees a diverged warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const bool ok = mbar_wait(bar, parity, abort);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------- cp.async -----
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src)
                 : "memory");
}
// Arrive on `bar` once all cp.async issued so far by this thread have landed.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------- TMA -----
// Plain (non-multicast) tiled 2D TMA load into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
// Non-tensor bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------ tcgen05 -----
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Signal `bar` when every tcgen05 operation issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem]; kind::f16 (bf16 operands, fp32 accumulate).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The same MMAs issued from a converged warp: elect.sync picks one lane to
// issue.  Operands computed by the whole warp are warp-uniform, which lets
// the issue path skip the per-instruction uniformisation a single-lane branch
// needs (measured on B200: ~42 cycles per MMA issue against ~77).
__device__ __forceinline__ void mma_f16_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_i8_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Five MMAs over consecutive K-steps from a converged warp with one election:
// A at TMEM columns a, a+8, ..., a+32; B descriptors given as 32-bit halves
// (lo: start address and leading offset, hi: stride offset, version and
// layout), so that the issuing warp spends almost no integer instructions per
// MMA (it shares its SM sub-partition with the ALU-bound unpack warps).  The
// first MMA accumulates iff acc0 != 0, the others always.
template <bool I8>
__device__ __forceinline__ void mma5_ts_warp(uint32_t d_tmem, uint32_t a_tmem, const uint32_t (&lo)[5],
                                             const uint32_t (&hi)[5], uint32_t idesc, uint32_t acc0) {
    if constexpr (I8) {
        asm volatile(
            "{\n\t.reg .pred p, e;\n\t.reg .b32 r, a1, a2, a3, a4;\n\t.reg .b64 b0, b1, b2, b3, b4;\n\t"
            "setp.ne.b32 p, %13, 0;\n\t"
            "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\tadd.u32 a4, %1, 32;\n\t"
            "mov.b64 b0, {%2, %7};\n\tmov.b64 b1, {%3, %8};\n\tmov.b64 b2, {%4, %9};\n\t"
            "mov.b64 b3, {%5, %10};\n\tmov.b64 b4, {%6, %11};\n\t"
            "elect.sync r|e, 0xffffffff;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], b0, %12, p;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], [a1], b1, %12, 1;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], [a2], b2, %12, 1;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], [a3], b3, %12, 1;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::i8 [%0], [a4], b4, %12, 1;\n\t}" ::"r"(d_tmem),
            "r"(a_tmem), "r"(lo[0]), "r"(lo[1]), "r"(lo[2]), "r"(lo[3]), "r"(lo[4]), "r"(hi[0]), "r"(hi[1]),
            "r"(hi[2]), "r"(hi[3]), "r"(hi[4]), "r"(idesc), "r"(acc0)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p, e;\n\t.reg .b32 r, a1, a2, a3, a4;\n\t.reg .b64 b0, b1, b2, b3, b4;\n\t"
            "setp.ne.b32 p, %13, 0;\n\t"
            "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\tadd.u32 a4, %1, 32;\n\t"
            "mov.b64 b0, {%2, %7};\n\tmov.b64 b1, {%3, %8};\n\tmov.b64 b2, {%4, %9};\n\t"
            "mov.b64 b3, {%5, %10};\n\tmov.b64 b4, {%6, %11};\n\t"
            "elect.sync r|e, 0xffffffff;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], b0, %12, p;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %12, 1;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %12, 1;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %12, 1;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], b4, %12, 1;\n\t}" ::"r"(d_tmem),
            "r"(a_tmem), "r"(lo[0]), "r"(lo[1]), "r"(lo[2]), "r"(lo[3]), "r"(lo[4]), "r"(hi[0]), "r"(hi[1]),
            "r"(hi[2]), "r"(hi[3]), "r"(hi[4]), "r"(idesc), "r"(acc0)
            : "memory");
    }
}
// High words of the shared-memory descriptors above (stride offset, version 1, layout).
constexpr uint32_t kDescHiSW32 = (256u >> 4) | (1u << 14) | (6u << 29);
constexpr uint32_t kDescHiSW64 = (512u >> 4) | (1u << 14) | (4u << 29);
constexpr uint32_t kDescHiSW128 = (1024u >> 4) | (1u << 14) | (2u << 29);

// mma5_ts_warp (kind::f16) followed by a sixth MMA under the same election:
// A at TMEM column a6, B at the 32-byte-swizzled slab whose descriptor low
// word is lo6 (accumulating).
__device__ __forceinline__ void mma5c_ts_warp(uint32_t d_tmem, uint32_t a_tmem, const uint32_t (&lo)[5],
                                              const uint32_t (&hi)[5], uint32_t a6, uint32_t lo6, uint32_t idesc,
                                              uint32_t acc0) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r, a1, a2, a3, a4;\n\t.reg .b64 b0, b1, b2, b3, b4, b5;\n\t"
        "setp.ne.b32 p, %13, 0;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\tadd.u32 a4, %1, 32;\n\t"
        "mov.b64 b0, {%2, %7};\n\tmov.b64 b1, {%3, %8};\n\tmov.b64 b2, {%4, %9};\n\t"
        "mov.b64 b3, {%5, %10};\n\tmov.b64 b4, {%6, %11};\n\tmov.b64 b5, {%15, %16};\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], b0, %12, p;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %12, 1;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %12, 1;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %12, 1;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], b4, %12, 1;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%14], b5, %12, 1;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "r"(lo[0]), "r"(lo[1]), "r"(lo[2]), "r"(lo[3]), "r"(lo[4]), "r"(hi[0]), "r"(hi[1]),
        "r"(hi[2]), "r"(hi[3]), "r"(hi[4]), "r"(idesc), "r"(acc0), "r"(a6), "r"(lo6), "r"(kDescHiSW32)
        : "memory");
}

// tcgen05.commit from a converged warp (one elected lane).
__device__ __forceinline__ void tc_commit_warp(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

// kind::i8 (8-bit integer operands, int32 accumulate).
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Each thread of a warp stores 8 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3])
                 : "memory");
}
__device__ __forceinline__ void tmem_st2(uint32_t taddr, const uint32_t (&v)[2]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(v[0]), "r"(v[1])
                 : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
// Each thread loads 16 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor (tcgen05 format, version 1) for a K-major
// operand stored in 32-byte swizzled slabs: 8-row groups of 32-byte rows, one
// slab per MMA K-step, slab base 256-byte aligned.
__device__ __forceinline__ uint64_t smem_desc_sw32(const void* slab) {
    const uint64_t addr = smem_u32(slab);
    uint64_t d = (addr >> 4) & 0x3FFFull;  // start address
    d |= 1ull << 16;                       // leading byte offset (unused for swizzled K-major)
    d |= (256ull >> 4) << 32;              // stride byte offset: 8 rows x 32 B
    d |= 1ull << 46;                       // descriptor version (sm_100)
    d |= 6ull << 61;                       // layout: SWIZZLE_32B
    return d;
}

// The same for K-major operands in 128- and 64-byte swizzled boxes (8-row
// groups of 128- or 64-byte rows, box base aligned to the 8-row group).  An
// MMA K-step inside a swizzled row starts at the row's start plus its byte
// offset; the swizzle is applied to the computed addresses, so the offset
// is simply added to the start address.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* start) {
    const uint64_t addr = smem_u32(start);
    uint64_t d = (addr >> 4) & 0x3FFFull;
    d |= 1ull << 16;
    d |= (1024ull >> 4) << 32;  // stride byte offset: 8 rows x 128 B
    d |= 1ull << 46;
    d |= 2ull << 61;            // layout: SWIZZLE_128B
    return d;
}
__device__ __forceinline__ uint64_t smem_desc_sw64(const void* start) {
    const uint64_t addr = smem_u32(start);
    uint64_t d = (addr >> 4) & 0x3FFFull;
    d |= 1ull << 16;
    d |= (512ull >> 4) << 32;   // stride byte offset: 8 rows x 64 B
    d |= 1ull << 46;
    d |= 4ull << 61;            // layout: SWIZZLE_64B
    return d;
}

__device__ __forceinline__ uint32_t elect_lane0() { return (threadIdx.x & 31) == 0; }

}  // namespace pn
