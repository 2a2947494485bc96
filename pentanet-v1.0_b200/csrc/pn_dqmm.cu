// pn_dqmm.cu -- fused pentanary dequant-matmul on the sm_100a tensor cores.
//
// Computes Y[m, n] = scale * sum_k X[m, k] * w[n, k] for packed 3-bit weights
// (the op of _penta_matmul_kernel, penta_kernel.py:111-224) as a swap-AB
// tcgen05 GEMM: the weight tile is the MMA's A operand (128 weight rows = the
// 128 TMEM lanes) and the activations are the B operand (BT tokens).
//
//   * Weights are streamed from HBM exactly once per (row tile, token tile):
//     a loader warp stages 16 packed words (160 k) of each of the 128 rows per
//     k-block into shared memory with cp.async; four unpack warps (one weight
//     row per thread) turn their row's words into MMA operands in registers and
//     write them straight into tensor memory with tcgen05.st -- the A operand
//     never touches shared memory.
//       kind::f16: exact bf16 weights c-2 (mantissa trick + one bf16x2 subtract)
//       kind::i8 : the unsigned codes c in {0..4}; the -2 offset is applied in
//                  the epilogue as -2 * rowsum(xq) (exact integer algebra).
//   * Activations arrive by TMA (no multicast) in 32-byte swizzled slabs, one
//     slab per MMA K-step.
//   * One thread issues the MMAs; the fp32/int32 accumulator lives in TMEM and
//     is read back by the unpack warps for the fused epilogue (scale, per-token
//     activation scale, bias, bf16 rounding as the reference does it).
//
// Every barrier wait is bounded (pn_common.cuh); a CTA that gives up drains
// its in-flight copies and MMAs, frees its tensor memory and exits, leaving
// PN_ERR_TIMEOUT in the device status word.
#include "pn_common.cuh"
#include "pn_internal.h"

#include <cstring>
#include <mutex>
#include <type_traits>

namespace pn {

constexpr int kRows = 128;         // weight rows per tile (MMA M, TMEM lanes)
constexpr int kWordsPerKB = 16;    // packed words per row per k-block (160 k)
constexpr int kKB = kWordsPerKB * kPerWord;
constexpr int kWStageWords = 2 * kWordsPerKB;           // one weight stage = 2 k-blocks = 128 bytes per row
constexpr int kWStageBytes = kRows * kWStageWords * 4;  // 16 KB, one 128B-swizzled TMA box
constexpr int kUnpackWarps = 16;   // warps 0-15: unpack + epilogue (four per TMEM lane quarter)
constexpr int kUnpackGroups = kUnpackWarps / 4;  // warps per lane quarter; they take turns on k-blocks
constexpr int kLoadWarp = kUnpackWarps;       // weight staging, even stages
constexpr int kLoadWarp2 = kUnpackWarps + 1;  // weight staging, odd stages
constexpr int kXLoadWarp = kUnpackWarps + 2;  // activation staging
constexpr int kMmaWarp = kUnpackWarps + 3;    // TMEM allocation + MMA issue; warps kMmaWarp.. issue MMAs
constexpr int kMaxIssuers = 4;
constexpr int kThreads = 32 * (kUnpackWarps + 3 + kMaxIssuers);
constexpr int kTmemCols = 512;

// F16: bf16 activations, kind::f16 MMAs.  I8: int8 activations (per-token
// absmax quantised), kind::i8.  L8: bf16 activations of a decode batch (at
// most 16 tokens) as four int8 limbs of a per-token 32-bit fixed-point
// integer, kind::i8 (see limb_x_kernel).
enum class Kind { F16, I8, L8 };

template <Kind KIND>
struct KindT;
template <>
struct KindT<Kind::F16> {
    static constexpr int kXElem = 2;       // bytes per activation element
    static constexpr int kSlabElems = 16;  // elements per 32-byte slab = MMA K
    static constexpr int kSteps = 10;      // MMAs per k-block
    static constexpr int kACols = 80;      // TMEM columns of A per k-block (2 bf16 per column)
    static constexpr int kAPerKB = 2;      // TMEM operand stages per k-block (8 words / 5 MMAs each)
};
template <>
struct KindT<Kind::I8> {
    static constexpr int kXElem = 1;
    static constexpr int kSlabElems = 32;
    static constexpr int kSteps = 5;
    static constexpr int kACols = 40;      // 4 codes per column
    static constexpr int kAPerKB = 1;
};
template <>
struct KindT<Kind::L8> : KindT<Kind::I8> {};

// Limb decode (Kind::L8): a token occupies four accumulator columns (its
// four limbs), so a 16-column epilogue chunk holds 4 tokens.
constexpr int kL8Cols = 4;
constexpr int kL8MaxTokens = 16;
// Default limit of pn_set_limb_max_tokens: the limb path is faster than the
// kind::f16 decode kernel on the compact 8-column tile (1-2 tokens: 30.0 vs
// 33.8 us per 94 MB product on B200) and slower on the wider tiles.
constexpr int kL8DefaultTokens = 2;
constexpr int kL8MaxK = 65536;  // keeps every limb accumulator inside int32 (|A| <= 224, |limb| <= 128)
constexpr int kL8NonFinite = -0x7fffffff - 1;  // lx_shift of a token holding an inf or NaN

// v * 2^e for e in [-252, 254], as at most two products by normal powers of
// two (exact unless the result is subnormal).
__device__ __forceinline__ float scale_pow2(float v, int e) {
    if (e < -126) {
        v = __fmul_rn(v, 0x1p-126f);
        e += 126;
    } else if (e > 127) {
        v = __fmul_rn(v, 0x1p127f);
        e -= 127;
    }
    return __fmul_rn(v, __int_as_float((127 + e) << 23));
}

template <Kind KIND, int BT>
struct Cfg {
    using T = KindT<KIND>;
    // Small token tiles (decode) run several MMA-issuing warps, each taking
    // every kIssuers-th k-block into its own accumulator: one warp issues an
    // MMA only every ~40-80 cycles, which the short MMAs of a 16- or 32-token
    // tile (8-16 tensor cycles) cannot hide.  A 64-token MMA takes ~32 tensor
    // cycles, so two issuers keep the tensor pipe busy; large tiles use one.
    static constexpr bool kXTma = BT >= 128;
    // bf16 decode tiles use the permuted unpack; their activations come
    // pre-arranged (permute_x_kernel / limb_x_kernel) and are staged with one
    // bulk copy per k-block.
    static constexpr bool kL8 = KIND == Kind::L8;
    static constexpr bool kPerm = (KIND == Kind::F16 && BT <= 64) || kL8;
    // kind::f16 decode tiles add the code offset through one extra MMA per
    // k-block (constant A columns x a correction slab); limb tiles subtract it
    // in the epilogue.
    static constexpr bool kCorr = KIND == Kind::F16 && kPerm;
    // accumulator columns per token: BT counts columns, BT / kCPT tokens
    static constexpr int kCPT = kL8 ? kL8Cols : 1;
    static constexpr int kIssuers = BT <= 32 ? 4 : (BT <= 64 ? 2 : 1);
    // MMA N.  The 8-token decode tile (bf16, up to 8 tokens) runs N = 16 MMAs
    // over a compact activation image: each slab holds only 8 rows (256 bytes,
    // one 8-row core-matrix group), so the MMA's second group (rows 8-15, one
    // stride offset = 256 bytes further) reads the next slab; it feeds
    // accumulator columns 8-15, which are never read.  Half the bytes per
    // k-block of the 16-token image, and twice the ring depth.
    static constexpr int kMmaN = BT < 16 ? 16 : BT;
    static constexpr int kSlabBytes = BT * 32;
    // Activation stage: the k-block's BT rows x kRowBytes.  Staged by TMA as
    // kWide boxes of 128-byte rows (128-byte swizzle) and one box of the
    // remaining kTail bytes per row (32- or 64-byte swizzle), each box BT rows;
    // the MMA for K-step j reads bytes [32j, 32j + 32) of every row.  Bulk-copied
    // decode stages are kSteps 32-byte-swizzled slabs instead.
    static constexpr int kRowBytes = kKB * T::kXElem;
    static constexpr int kWide = kRowBytes / 128;
    static constexpr int kTail = kRowBytes % 128;
    // Decode stages carry one more slab: the k-block's offset correction (see
    // permute_x_kernel), multiplied by constant A columns in one extra MMA.
    static constexpr int kXSlabs = kCorr ? T::kSteps + 1 : T::kSteps;
    static constexpr int kXDataBytes = kSlabBytes * kXSlabs;
    // (+ the 256 bytes the last slab's second row group reads in a compact image)
    static constexpr int kXStageBytes = (kXDataBytes + (BT < 16 ? 256 : 0) + 1023) / 1024 * 1024;
    static constexpr int kChunksPerRow = kKB * T::kXElem / 16;      // 16-byte pieces of one row per k-block
    static constexpr int kDCols = kIssuers * kMmaN;               // accumulators D_0..D_{kIssuers-1}
    static constexpr int kA0 = kDCols < 32 ? 32 : kDCols;         // first A column
    // Ring depths.  Waiters that take turns on k-blocks (unpack groups on the
    // TMEM operand ring and the weight ring, MMA issuers on the operand and
    // activation rings) must each see every phase of the slots they use, in
    // order; otherwise a parity wait can pass on a phase two rounds old.  So
    // each ring depth is a multiple of the number of parties taking turns on it.
    // TMEM operand stages: 40 columns each (half a bf16 k-block, a whole int8
    // one), so that an unpack group fills one stage while the MMAs read its other.
    static constexpr int kAStageCols = T::kACols / T::kAPerKB;
    static constexpr int kStepsPerA = T::kSteps / T::kAPerKB;
    static_assert(kStepsPerA == 5, "five MMAs per operand stage");
    static constexpr int kAParties = kUnpackGroups * T::kAPerKB;  // stage uses per round of groups
    static constexpr int kSAfit = (kTmemCols - kA0) / kAStageCols;
    static constexpr int kSA = (kSAfit >= 8 ? 8 : kSAfit) / kAParties * kAParties;
    static constexpr int kBudget = 218 * 1024;
    static constexpr int kSW = kXStageBytes >= 40 * 1024 ? 4 : (kXStageBytes >= 20 * 1024 ? 6 : 8);
    static constexpr int kSXfit = (kBudget - kSW * kWStageBytes) / kXStageBytes;
    // Up to three activation stages per issuer: a copy is issued when the
    // stage's use kSX k-blocks earlier is done, so deeper rings hide its latency.
    static constexpr int kSXcap = (BT < 16 ? 6 : 3) * kIssuers;
    static constexpr int kSX = (kSXfit > kSXcap ? kSXcap : (kSXfit > 8 ? 8 : kSXfit)) / kIssuers * kIssuers;
    // 8-token decode tiles: the activation loader copies the activations of
    // the CTA's first kSX k-blocks (use 0 of every activation stage, as soon
    // as the pre-pass is done); every later use is copied by the weight
    // loaders, each weight stage's two k-blocks just before its weight box in
    // the same TMA queue, so they land ahead of the weights they meet (a
    // separate loader, queued behind the 16 KB weight boxes, issued one copy
    // per weight box and fell behind the MMAs).  This needs an activation
    // ring that outlasts the weight ring's lead (kSX >= 2 kSW + 4: the stage a
    // weight loader refills was released long before), and a stage's later
    // uses all fall to one weight-loader warp (kSX / 2 even), which then waits
    // for every release of that stage in order.  Larger tiles keep the
    // activation loader for all k-blocks.
    static constexpr bool kXByWLoader = kPerm && kSX >= 2 * kSW + 4 && (kSX / 2) % 2 == 0;
    static constexpr int kActEarly = kXByWLoader ? kSX : 0;
    static constexpr int kBarOff = kSX * kXStageBytes + kSW * kWStageBytes;
    // TMEM columns holding the constant A operand of the correction MMA (decode)
    static constexpr int kConstCol = kA0 + kSA * kAStageCols;
    static constexpr int kNumBars = 2 * kSW + 2 * kSX + 2 * kSA + 4 + kIssuers;
    static constexpr int kSmem = kBarOff + kNumBars * 8 + 16 + 1024;  // + tmem slot, abort and last-arriver flags + align slack
    static_assert(kSX >= 2 && kSX % kIssuers == 0, "activation ring");
    static_assert(!kXByWLoader || kActEarly % 2 == 0, "activation copies by whole weight stages");
    static_assert(kSA >= kAParties && kSA % kAParties == 0 && kSA % (kIssuers * T::kAPerKB) == 0, "TMEM operand ring");
    static_assert(kSW % 2 == 0, "weight ring: two producers, two k-blocks per stage");
    static_assert((kSX * kXStageBytes) % 1024 == 0, "weight stages must stay 1024-byte aligned (128B swizzle)");
    static_assert(kA0 + kSA * kAStageCols + (kCorr ? 8 : 0) <= kTmemCols, "TMEM over-subscribed");
    static_assert((BT % 16 == 0 && BT >= 16 && BT <= 256) || (BT == 8 && kPerm), "token tile");
    static_assert(!kL8 || BT <= 64, "limb tiles: at most 16 tokens");
    static_assert(kSmem <= 227 * 1024, "shared memory per block");
    static_assert(kTail == 32 || kTail == 64, "activation tail box");
};

struct DqmmParams {
    int64_t N, KP;
    int M;
    int n_row_tiles, n_items, n_kb;
    int64_t total_pairs;   // n_items * (n_kb / 2): the flattened (tile, k-block pair) work
    uint32_t units;        // total_pairs / unit
    int unit;              // pairs per indivisible unit: 1 (tiles may split) or n_kb / 2 (whole tiles)
    // Split tiles.  16-token tiles: one sum buffer per split tile,
    // [gridDim.x][acc_cols][128] int64 fixed point (bf16 path) / int32,
    // added with atomics.  Larger tiles: per-CTA partials
    // [gridDim.x][2][BT/4][128][4] (groups of 4 columns, row-major inside a
    // group, so a warp's 16-byte accesses are contiguous), summed by the
    // last contributor.
    void* accbuf;
    int acc_cols;          // columns of a 16-token tile's sum buffer: min(16, M)
    int* counters;         // [n_items][16 unpack warps] arrival counters of split tiles (zeroed by the host)
    const uint8_t* xperm;  // permuted activation slabs (bf16 decode tiles)
    float scale;
    const __nv_bfloat16* bias;
    const __nv_bfloat16* residual;  // (M, ld_res) bf16 added after the activation, or null
    int64_t ld_res;
    int act;               // kActNone / kActGelu
    void* y_out[8];        // output buffers (one, or one per GPU of an output-sharded layer)
    int n_out;
    int64_t ld_y, y_col0;  // row stride of the outputs and this shard's first column
    int y_f32;
    int32_t* acc_out;
    const float* s_x;
    const int32_t* rowsum;
    // limb decode (Kind::L8), written by limb_x_kernel: per token its
    // fixed-point exponent S (kL8NonFinite when a value is inf or NaN) and
    // the partial sums of its offset correction, lx_chunks per token
    const int* lx_shift;
    const long long* lx_corr;
    int lx_chunks;
};

// (a & M) | C as one LOP3.  Written out because the compiler otherwise emits
// an AND and an OR when both M and C are immediates, which costs the unpack
// loops a third of their integer-pipe throughput.
template <uint32_t M, uint32_t C>
__device__ __forceinline__ uint32_t and_or(uint32_t a) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "n"(M), "n"(C));
    return r;
}
// (a & M) | c for a register c.
template <uint32_t M>
__device__ __forceinline__ uint32_t and_or_r(uint32_t a, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "n"(M), "r"(c));
    return r;
}

// bf16 weights of one packed word: five bf16x2 registers, natural k order
// (register j holds k = 2j in the low half and k = 2j+1 in the high half).
// (128 + c) is built in the mantissa of a bf16 with exponent 2^7, then 130 is
// subtracted: exact c - 2 for every code.
__device__ __forceinline__ uint32_t bf16_pair(uint32_t lo_src, uint32_t hi_src) {
    const uint32_t t = and_or_r<0x00070000u>(hi_src, and_or<0x00000007u, 0x43004300u>(lo_src));
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(t), "r"(0x43024302u));
    return r;
}
__device__ __forceinline__ void unpack_word_bf16(uint32_t p, uint32_t* r) {
    r[0] = bf16_pair(p, p << 13);
    r[1] = bf16_pair(p >> 6, p << 7);
    r[2] = bf16_pair(p >> 12, p << 1);
    r[3] = bf16_pair(p >> 18, p >> 5);
    r[4] = bf16_pair(p >> 24, p >> 11);
}

// Decode variant: five bf16x2 registers per word in a permuted k order, each
// half a bf16 subnormal c * 2^(j-133) holding the raw code c = q + 2 at
// mantissa bit j -- two right shifts, one left shift (an IMAD, off the ALU
// pipe) and five masks, 0.8 instructions per weight with no floating-point
// work.  Register r holds codes r (low half) and r+5 (high half): position 2r
// <- code r, position 2r+1 <- code r+5 of the word, and the value stored at
// position q is c * 2^(kPermExp(q) - 133).  The activations are permuted to
// match and scaled by 2^(66 - kPermExp(q)) (permute_x_kernel), so every
// product is c * x * 2^-67 (exact: tcgen05 keeps bf16 subnormal operands),
// and the offset of the code, sum_k -2 x_k per k-block, enters the
// accumulator through one extra MMA per k-block (constant A columns times a
// correction slab written by the pre-pass).
__host__ __device__ constexpr int perm_src(int q) { return (q & 1) ? (q >> 1) + 5 : (q >> 1); }
__host__ __device__ constexpr int perm_exp(int q) {
    return (int)((0x3401340101ull >> (4 * q)) & 0xF);  // {1,0,1,0,4,3,1,0,4,3}
}
// Decode products accumulate in units of 2^-67 (the scales above).
constexpr int kPermUnitExp = 67;
__device__ __forceinline__ void unpack_word_bf16_perm(uint32_t p, uint32_t* r) {
    const uint32_t l1 = p * 2u;  // IMAD, not a shift
    const uint32_t r2 = p >> 2;
    const uint32_t r8 = p >> 8;
    r[0] = l1 & 0x0007000Eu;  // code 0 at bit 1, code 5 at bit 16
    r[1] = r2 & 0x0007000Eu;  // code 1 at bit 1, code 6 at bit 16
    r[2] = r2 & 0x00380070u;  // code 2 at bit 4, code 7 at bit 19
    r[3] = r8 & 0x0007000Eu;  // code 3 at bit 1, code 8 at bit 16
    r[4] = r8 & 0x00380070u;  // code 4 at bit 4, code 9 at bit 19
}

// Limb decode (Kind::L8): unsigned 8-bit A operands of two packed words (20
// weights) in five registers, one mask per four codes.  Each byte holds one
// code c in place, shifted left by t = (its bit offset in the word) minus
// (the byte's offset), so the byte's value is c * 2^t (t <= 5: at most 224
// for a 3-bit field).  Register 0 (word p): codes 0, 3, 6, 8 with t = 0, 1,
// 2, 0; register 1: codes 1, 4, 7, 9 with t = 3, 4, 5, 3; registers 2-3 the
// same for word q; register 4: codes 2 and 5 of p, then of q, t = 0, 1, 0, 1.
// MMA position r (0..19) of the pair therefore multiplies the weight at k
// offset l8_src(r) (0-9 in p, 10-19 in q) by 2^l8_shift(r); limb_x_kernel
// scales that activation by 2^-l8_shift(r) to match.
__host__ __device__ constexpr int l8_src(int r) {
    // {0,3,6,8, 1,4,7,9, 10,13,16,18, 11,14,17,19, 2,5,12,15}
    return r < 16 ? (r & 8 ? 10 : 0) + ((r & 4) ? (int)((0x9741u >> (4 * (r & 3))) & 0xF)
                                               : (int)((0x8630u >> (4 * (r & 3))) & 0xF))
                  : (int)((0xFC52u >> (4 * (r - 16))) & 0xF);
}
__host__ __device__ constexpr int l8_shift(int r) {
    // {0,1,2,0, 3,4,5,3, 0,1,2,0, 3,4,5,3, 0,1,0,1}
    return r < 16 ? ((r & 4) ? (int)((0x3543u >> (4 * (r & 3))) & 0xF) : (int)((0x0210u >> (4 * (r & 3))) & 0xF))
                  : (r & 1);
}
__device__ __forceinline__ void unpack_pair_l8(uint32_t p, uint32_t q, uint32_t* r) {
    r[0] = p & 0x071C0E07u;
    r[1] = p & 0x38E07038u;
    r[2] = q & 0x071C0E07u;
    r[3] = q & 0x38E07038u;
    // (p >> 6): code 2 -> bits 0-2, code 5 -> bits 9-11; (q << 10): code 2 ->
    // bits 16-18, code 5 -> bits 25-27; the left shift as a multiply (FMA pipe)
    r[4] = and_or_r<0x00000E07u>(p >> 6, (q * 1024u) & 0x0E070000u);
}

// Unsigned codes of two packed words (20 weights) as five int8x4 registers in
// natural k order.  Four codes at stride 3 are spread to stride 8 with two
// carry-free multiplies (even and odd codes separately).
__device__ __forceinline__ uint32_t spread4(uint32_t t) {
    const uint32_t e = t & 0x1C7u;  // codes 0 and 2
    const uint32_t o = t & 0xE38u;  // codes 1 and 3
    return and_or_r<0x00070007u>(e * 0x401u, (o * 0x8020u) & 0x07000700u);
}
__device__ __forceinline__ void unpack_pair_u8(uint32_t p0, uint32_t p1, uint32_t* r) {
    const uint32_t lo = p0 | (p1 << 30);
    const uint32_t hi = p1 >> 2;
    r[0] = spread4(lo);
    r[1] = spread4(lo >> 12);
    r[2] = spread4(__funnelshift_r(lo, hi, 24));
    r[3] = spread4(hi >> 4);
    r[4] = spread4(hi >> 16);
}

// Bounded wait used while draining after an abort (ignores the abort flag).
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitLimitCycles) {
            record_status(PN_ERR_TIMEOUT);
            return;
        }
    }
}

// Work split (stream-K style): the flattened (tile, k-block pair) space is cut
// into gridDim.x equal contiguous ranges of units, one per CTA; a unit is one
// k-block pair (tiles may split) or one whole tile.  A CTA walks its range as
// segments -- a whole tile, or the k-block range of one tile that its range
// covers.  Tiles split over several CTAs are finished by the last one to
// arrive, which sums the partials in CTA order (deterministic).
struct Seg {
    int tile;
    int kb0, kb1;   // k-blocks [kb0, kb1), both even
    bool whole;
};
// All in 32-bit unsigned arithmetic (the host checks that units * (grid + 1)
// fits): these run at the start of every role and segment, and 64-bit
// divisions cost hundreds of cycles there.
__device__ __forceinline__ int64_t range_begin(const DqmmParams& p, int c) {
    const uint32_t units = p.units;
    return (int64_t)((uint32_t)c * units / gridDim.x) * p.unit;
}
// CTA whose range holds pair u.
__device__ __forceinline__ int owner_of(const DqmmParams& p, int64_t u) {
    const uint32_t units = p.units;
    return (int)((((uint32_t)u / (uint32_t)p.unit + 1u) * gridDim.x - 1u) / units);
}
__device__ __forceinline__ Seg segment_at(const DqmmParams& p, int64_t u, int64_t u_end) {
    const int P = p.n_kb / 2;
    Seg g;
    g.tile = (int)((uint32_t)u / (uint32_t)P);
    const int pb = (int)(u - (int64_t)g.tile * P);
    const int64_t left = u_end - u;
    const int pe = (int64_t)(P - pb) < left ? P : (int)(pb + left);
    g.kb0 = 2 * pb;
    g.kb1 = 2 * pe;
    g.whole = pb == 0 && pe == P;
    return g;
}

// Split 16-token tiles are summed with integer atomics, so the result does not
// depend on the order in which contributors arrive: int32 accumulators add exactly,
// and fp32 partials are added as 64-bit fixed point with 2^-24 resolution
// (exact for every partial of magnitude >= 2^-1, error <= 2^-25 otherwise;
// range +-2^39).  The sum is converted back with one rounding to fp32.
constexpr float kFixScale = 16777216.0f;  // 2^24
__device__ __forceinline__ void red_add(long long* p, long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_add(int* p, int v) {
    asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// EPI: the instance that also fuses an activation and a residual add into
// the epilogue (separate instances keep the plain products' register
// allocation untouched; the extra epilogue code costs registers at the
// 80-per-thread budget).
template <Kind KIND, int BT, bool EPI>
__global__ void __launch_bounds__(kThreads, 1)
    dqmm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xmap_tail,
                const __grid_constant__ CUtensorMap wmap, const DqmmParams p) {
    using C = Cfg<KIND, BT>;
    using T = typename C::T;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_x = smem;
    uint32_t* smem_w = reinterpret_cast<uint32_t*>(smem + C::kSX * C::kXStageBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* full_w = bars;
    uint64_t* empty_w = full_w + C::kSW;
    uint64_t* full_x = empty_w + C::kSW;
    uint64_t* empty_x = full_x + C::kSX;
    uint64_t* full_a = empty_x + C::kSX;
    uint64_t* empty_a = full_a + C::kSA;
    uint64_t* acc_full = empty_a + C::kSA;
    uint64_t* acc_empty = acc_full + 1;
    uint64_t* drain = acc_empty + 1;  // one per issuer
    uint64_t* const_bar = drain + C::kIssuers;  // decode: constant A columns written
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // The next product on the stream (its decode pre-pass, launched as a
    // programmatic dependent) may be scheduled now: it waits for this grid's
    // completion before it touches memory, and the GEMM after it starts its
    // prologue and weight streaming on the SMs this grid frees.
    asm volatile("griddepcontrol.launch_dependents;");

    // Barrier setup spread over warp 0's lanes (one thread initialising the
    // ~90 barriers serially took ~2000 cycles before the first weight load).
    if (warp == 0) {
        for (int s = lane; s < C::kSW; s += 32) {
            mbar_init(&full_w[s], 1);
            mbar_init(&empty_w[s], 8);  // 2 k-blocks x 4 lane quarters
        }
        for (int s = lane; s < C::kSX; s += 32) {
            mbar_init(&full_x[s], 1);
            mbar_init(&empty_x[s], 1);
        }
        for (int s = lane; s < C::kSA; s += 32) {
            mbar_init(&full_a[s], 4);
            mbar_init(&empty_a[s], 1);
        }
        if (lane < C::kIssuers) mbar_init(&drain[lane], 1);
        if (lane == 0) {
            mbar_init(acc_full, C::kIssuers);
            mbar_init(acc_empty, kUnpackWarps);
            mbar_init(const_bar, 4);
            *abort_flag = 0;
        }
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    if ((warp == kLoadWarp || warp == kLoadWarp2) && lane == 0) tma_prefetch_desc(&wmap);
    if (warp == kXLoadWarp && lane == 0 && !C::kPerm) {
        tma_prefetch_desc(&xmap);
        tma_prefetch_desc(&xmap_tail);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kLoadWarp || warp == kLoadWarp2) {
        // ------------------------------------------------ weight loaders ----
        // One TMA box per stage: 128 rows x 32 words (2 k-blocks), 128-byte
        // swizzled; words >= K_packs and rows >= N are zero-filled.  The two
        // loader warps take alternate stages.
        const int producer = warp - kLoadWarp;
        uint32_t st = 0;  // global stage counter
        uint32_t x_first = 0, x_end = 0;  // activation copies this warp issued: CTA k-blocks [x_first, x_end)
        bool ok = true, x_waited = false;
        const int64_t u_end = range_begin(p, blockIdx.x + 1);
        for (int64_t u = range_begin(p, blockIdx.x); u < u_end && ok;) {
            const Seg g = segment_at(p, u, u_end);
            u += (g.kb1 - g.kb0) / 2;
            const int n0 = (g.tile % p.n_row_tiles) * kRows;
            for (int ws = g.kb0 / 2; ws < g.kb1 / 2; ++ws, ++st) {
                if ((int)(st & 1) != producer) continue;
                const int sw = st % C::kSW;
                if constexpr (C::kXByWLoader) {
                    if (2 * st >= (uint32_t)C::kActEarly) {
                        // the two k-blocks' activations (the pre-pass's output)
                        if (!x_waited) {
                            asm volatile("griddepcontrol.wait;" ::: "memory");
                            x_waited = true;
                            x_first = 2 * st;
                        }
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const uint32_t c = 2 * st + h;
                            const int sx = c % C::kSX;
                            if (!warp_wait(&empty_x[sx], ((c / C::kSX) & 1) ^ 1, abort_flag)) { ok = false; break; }
                            if (lane == 0) {
                                mbar_arrive_expect_tx(&full_x[sx], C::kXDataBytes);
                                bulk_load(smem_x + sx * C::kXStageBytes, p.xperm + (size_t)(2 * ws + h) * C::kXDataBytes,
                                          C::kXDataBytes, &full_x[sx]);
                            }
                            x_end = c + 1;
                        }
                        if (!ok) break;
                    }
                }
                if (!warp_wait(&empty_w[sw], ((st / C::kSW) & 1) ^ 1, abort_flag)) { ok = false; break; }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full_w[sw], kWStageBytes);
                    tma_load_2d(smem_w + sw * (kWStageBytes / 4), &wmap, &full_w[sw], ws * kWStageWords, n0);
                }
                __syncwarp();
            }
        }
        if (!ok && lane == 0) {
            // Let every issued copy land before the CTA can exit.
            for (uint32_t j = (st > (uint32_t)C::kSW ? st - C::kSW : 0u); j < st; ++j)
                if ((int)(j & 1) == producer) mbar_wait_drain(&full_w[j % C::kSW], (j / C::kSW) & 1);
            // this warp's activation copies: its stages' k-blocks among the last kSX
            for (uint32_t c = (x_end > (uint32_t)C::kSX && x_end - C::kSX > x_first) ? x_end - C::kSX : x_first;
                 c < x_end; ++c)
                if ((int)((c >> 1) & 1) == producer) mbar_wait_drain(&full_x[c % C::kSX], (c / C::kSX) & 1);
        }
    } else if (warp == kXLoadWarp) {
        // -------------------------------------------- activation loader ----
        // One lane serves every issuer's activation stages.  Stage s belongs
        // to issuer s mod kIssuers (k-block c of this CTA uses stage c mod kSX
        // and issuer c mod kIssuers), and each issuer's stages are refilled as
        // soon as its own MMAs release them: a slow issuer never holds back
        // the copies of the others.
        if (lane == 0) {
            // The activations are the previous grid's output (the decode
            // pre-pass, the int8 quantiser or whatever produced x): every
            // GEMM is a programmatic dependent, so wait for that grid.
            asm volatile("griddepcontrol.wait;" ::: "memory");
            const int64_t u_begin = range_begin(p, blockIdx.x);
            uint32_t total = (uint32_t)(2 * (range_begin(p, blockIdx.x + 1) - u_begin));
            if (C::kXByWLoader && total > (uint32_t)C::kActEarly) total = C::kActEarly;  // the rest: weight loaders
            const uint32_t P = (uint32_t)(p.n_kb / 2);
            uint32_t cur[C::kIssuers];  // next k-block of each issuer
#pragma unroll
            for (int i = 0; i < C::kIssuers; ++i) cur[i] = i;
            bool ok = true;
            long long t_idle = clock64();
            while (true) {
                bool left = false, moved = false;
#pragma unroll
                for (int i = 0; i < C::kIssuers; ++i) {
                    const uint32_t c = cur[i];
                    if (c >= total) continue;
                    left = true;
                    const int sx = c % C::kSX;
                    if (!mbar_test_wait(&empty_x[sx], ((c / C::kSX) & 1) ^ 1)) continue;
                    // k-block c of the CTA's range: pair u, its tile and k-block index
                    const uint32_t u = (uint32_t)u_begin + (c >> 1);
                    const uint32_t tile = u / P;
                    const int kb = (int)(2 * (u - tile * P) + (c & 1));
                    uint8_t* xs = smem_x + sx * C::kXStageBytes;
                    mbar_arrive_expect_tx(&full_x[sx], C::kXDataBytes);
                    if constexpr (C::kPerm) {
                        bulk_load(xs, p.xperm + (size_t)kb * C::kXDataBytes, C::kXDataBytes, &full_x[sx]);
                    } else {
                        const int m0 = (int)(tile / (uint32_t)p.n_row_tiles) * BT;
                        const int k0 = kb * kKB;
#pragma unroll
                        for (int b = 0; b < C::kWide; ++b)
                            tma_load_2d(xs + b * BT * 128, &xmap, &full_x[sx], k0 + b * (128 / T::kXElem), m0);
                        tma_load_2d(xs + C::kWide * BT * 128, &xmap_tail, &full_x[sx],
                                    k0 + C::kWide * (128 / T::kXElem), m0);
                    }
                    cur[i] = c + C::kIssuers;
                    moved = true;
                }
                if (!left) break;
                if (moved) {
                    t_idle = clock64();
                    continue;
                }
                if (*abort_flag) {
                    ok = false;
                    break;
                }
                if (clock64() - t_idle > kWaitLimitCycles) {
                    *abort_flag = 1;
                    record_status(PN_ERR_TIMEOUT);
                    ok = false;
                    break;
                }
                // Nothing free: sleep on the stage of the oldest pending k-block
                // (the next one the MMAs release) instead of polling, which would
                // take issue slots from the unpack warps of this sub-partition.
                uint32_t oldest = 0xffffffffu;
#pragma unroll
                for (int i = 0; i < C::kIssuers; ++i)
                    if (cur[i] < total && cur[i] < oldest) oldest = cur[i];
                mbar_try_wait(&empty_x[oldest % C::kSX], ((oldest / C::kSX) & 1) ^ 1);
            }
            if (!ok) {
                // Let every issued copy land before the CTA can exit: an issuer's
                // copies in flight are its last kSX / kIssuers ones.
#pragma unroll 1
                for (int i = 0; i < C::kIssuers; ++i)
                    for (uint32_t c = cur[i] >= (uint32_t)C::kSX ? cur[i] - C::kSX : (uint32_t)i; c < cur[i];
                         c += C::kIssuers)
                        mbar_wait_drain(&full_x[c % C::kSX], (c / C::kSX) & 1);
            }
        }
    } else if (warp >= kMmaWarp) {
        // --------------------------------------------------------- MMAs ----
        // Issuer i (warp kMmaWarp + i, converged; one elected lane issues)
        // takes the k-blocks with global index it % kIssuers == i and
        // accumulates into D_i.
        const int issuer = warp - kMmaWarp;
        if (issuer < C::kIssuers) {
            uint32_t idesc;
            if constexpr (KIND == Kind::F16)
                idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(C::kMmaN >> 3) << 17) | ((128u >> 4) << 24);
            else  // A = unsigned 8-bit codes, B = signed int8, D = s32
                idesc = (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(C::kMmaN >> 3) << 17) | ((128u >> 4) << 24);
            const uint32_t d_tmem = tmem_base + issuer * C::kMmaN;
            uint32_t it = 0, n_local = 0;
            bool ok = true;
            if constexpr (C::kCorr) {
                ok = warp_wait(const_bar, 0, abort_flag);
                tc_fence_after();
            }
            const int64_t u_end = range_begin(p, blockIdx.x + 1);
            for (int64_t u = range_begin(p, blockIdx.x); u < u_end && ok; ++n_local) {
                const Seg g = segment_at(p, u, u_end);
                u += (g.kb1 - g.kb0) / 2;
                if (!warp_wait(acc_empty, (n_local & 1) ^ 1, abort_flag)) break;
                tc_fence_after();
                bool first = true;
                // this issuer's k-blocks of the segment: global index == issuer (mod kIssuers)
                const uint32_t it0 = it;
                const int nkb = g.kb1 - g.kb0;
                for (int j = (int)((issuer - it0) & (C::kIssuers - 1)); j < nkb; j += C::kIssuers) {
                    const uint32_t ik = it0 + j;
                    const int sx = ik % C::kSX;
                    if (!warp_wait(&full_x[sx], (ik / C::kSX) & 1, abort_flag)) { ok = false; break; }
                    // descriptor low word of the stage: start address >> 4, leading offset 1
                    const uint32_t xs_lo = (smem_u32(smem_x + sx * C::kXStageBytes) >> 4) + (1u << 16);
#pragma unroll
                    for (int hh = 0; hh < T::kAPerKB; ++hh) {
                        const uint32_t ua = ik * T::kAPerKB + hh;  // operand stage use
                        const int sa = ua % C::kSA;
                        if (!warp_wait(&full_a[sa], (ua / C::kSA) & 1, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t a_col = tmem_base + C::kA0 + sa * C::kAStageCols;
                        uint32_t lo[5], hi[5];
#pragma unroll
                        for (int j = 0; j < 5; ++j) {
                            const int step = hh * C::kStepsPerA + j;
                            if constexpr (C::kPerm) {
                                lo[j] = xs_lo + ((step * C::kSlabBytes) >> 4);
                                hi[j] = kDescHiSW32;
                            } else if (step * 32 < C::kWide * 128) {
                                // inside a 128-byte-swizzled box: the start advances 32 bytes per step
                                lo[j] = xs_lo + (((step * 32 / 128) * BT * 128 + (step * 32) % 128) >> 4);
                                hi[j] = kDescHiSW128;
                            } else if constexpr (C::kTail == 32) {
                                lo[j] = xs_lo + ((C::kWide * BT * 128) >> 4);
                                hi[j] = kDescHiSW32;
                            } else {
                                lo[j] = xs_lo + ((C::kWide * BT * 128 + (step * 32 - C::kWide * 128)) >> 4);
                                hi[j] = kDescHiSW64;
                            }
                        }
                        if (C::kCorr && hh == T::kAPerKB - 1) {
                            // + the k-block's offset correction: constant A columns x slab kSteps
                            mma5c_ts_warp(d_tmem, a_col, lo, hi, tmem_base + C::kConstCol,
                                          xs_lo + ((T::kSteps * C::kSlabBytes) >> 4), idesc, first ? 0u : 1u);
                        } else {
                            mma5_ts_warp<KIND != Kind::F16>(d_tmem, a_col, lo, hi, idesc, first ? 0u : 1u);
                        }
                        first = false;
                        // the stage is free for its group once these MMAs are done
                        tc_commit_warp(&empty_a[sa]);
                    }
                    if (!ok) break;
                    tc_commit_warp(&empty_x[sx]);
                }
                it = it0 + nkb;
                if (!ok) break;
                if (first) {
                    // no k-block of this segment: D_i unused (the epilogue skips it)
                    if (lane == 0) mbar_arrive(acc_full);
                    __syncwarp();
                } else {
                    tc_commit_warp(acc_full);
                }
            }
            // Every MMA this warp issued completes before tensor memory is freed.
            tc_commit_warp(&drain[issuer]);
            if (lane == 0) mbar_wait_drain(&drain[issuer], 0);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------- unpack + epilogue ----
        // Warps q, q+4, q+8, q+12 share TMEM lane quarter q (rows 32q..32q+31)
        // and take turns: warp group h unpacks the k-blocks with global index
        // it % kUnpackGroups == h, all 16 words of its rows.
        const int quarter = warp & 3;
        const int half = warp >> 2;  // warp group within the quarter
        const int row = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        if constexpr (C::kCorr) {
            // Constant A operand of the correction MMA: 1.0 at K positions 0-2
            // of every row (bf16 pairs: column 0 = (1, 1), column 1 = (1, 0)).
            if (half == 0) {
                const uint32_t one[8] = {0x3F803F80u, 0x00003F80u, 0u, 0u, 0u, 0u, 0u, 0u};
                tmem_st8(tmem_base + lane_base + C::kConstCol, one);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(const_bar);
            }
        }
        uint32_t it = 0, n_local = 0;
        bool ok = true;
        const int64_t u_begin = range_begin(p, blockIdx.x);
        const int64_t u_end = range_begin(p, blockIdx.x + 1);
        const int my_first_tile = (int)(u_begin / (p.n_kb / 2));
        // single-output destination (n_out == 1: row stride N, first column 0)
        float* const y0f = static_cast<float*>(p.y_out[0]);
        __nv_bfloat16* const y0h = static_cast<__nv_bfloat16*>(p.y_out[0]);
        for (int64_t u = u_begin; u < u_end && ok; ++n_local) {
            const Seg g = segment_at(p, u, u_end);
            u += (g.kb1 - g.kb0) / 2;
            const int64_t n0 = (int64_t)(g.tile % p.n_row_tiles) * kRows;
            // first token of the tile, and the tile's accumulator columns that
            // carry tokens (kCPT columns per token)
            const int m0 = (g.tile / p.n_row_tiles) * (BT / C::kCPT);
            const int ncol = (p.M - m0) * C::kCPT < BT ? (p.M - m0) * C::kCPT : BT;
            const uint32_t it_item = it;
            // this group's k-blocks of the segment: global index == half (mod 4)
            const int nkb = g.kb1 - g.kb0;
            for (int j = (int)((half - it_item) & (kUnpackGroups - 1)); j < nkb; j += kUnpackGroups) {
                const uint32_t ik = it_item + j;
                // Weight stages hold 2 k-blocks: global k-block `ik` is half (ik & 1)
                // of global stage ik / 2 (every item has an even k-block count).
                const uint32_t wst = ik >> 1;
                const int sw = wst % C::kSW;
                if (!warp_wait(&full_w[sw], (wst / C::kSW) & 1, abort_flag)) { ok = false; break; }
                // 128-byte swizzle: 16-byte chunk q of row r sits at chunk q ^ (r & 7).
                const uint4* rowp = reinterpret_cast<const uint4*>(smem_w + sw * (kWStageBytes / 4) + row * kWStageWords);
                auto load8 = [&](int hh, uint32_t (&wv)[8]) {
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const uint4 v = rowp[(4 * (ik & 1) + 2 * hh + q) ^ (row & 7)];
                        wv[4 * q + 0] = v.x;
                        wv[4 * q + 1] = v.y;
                        wv[4 * q + 2] = v.z;
                        wv[4 * q + 3] = v.w;
                    }
                };
#pragma unroll
                for (int hh = 0; hh < T::kAPerKB; ++hh) {
                    // Words are read from shared memory only when needed (8 per bf16
                    // half, all 16 for int8), which keeps register pressure down; the
                    // weight stage is released right after the last read.
                    uint32_t wa[8], wb[8];
                    if constexpr (KIND == Kind::F16) {
                        load8(hh, wa);
                    } else {
                        load8(0, wa);
                        load8(1, wb);
                    }
                    if (hh == T::kAPerKB - 1) {
                        // The k-block's words are in registers: its half of the
                        // weight stage is free for the loader now.
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty_w[sw]);
                    }
                    const uint32_t ua = ik * T::kAPerKB + hh;  // operand stage use
                    const int sa = ua % C::kSA;
                    const uint32_t a_addr = tmem_base + lane_base + C::kA0 + sa * C::kAStageCols;
                    uint32_t cols[40];
                    if constexpr (KIND == Kind::F16) {
                        // 8 words (half the k-block) -> 40 columns
#pragma unroll
                        for (int w = 0; w < 8; ++w) {
                            if constexpr (C::kPerm)
                                unpack_word_bf16_perm(wa[w], &cols[5 * w]);
                            else
                                unpack_word_bf16(wa[w], &cols[5 * w]);
                        }
                    } else {
                        // 8 word pairs -> 40 columns
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            if constexpr (C::kL8) {
                                unpack_pair_l8(wa[2 * w], wa[2 * w + 1], &cols[5 * w]);
                                unpack_pair_l8(wb[2 * w], wb[2 * w + 1], &cols[20 + 5 * w]);
                            } else {
                                unpack_pair_u8(wa[2 * w], wa[2 * w + 1], &cols[5 * w]);
                                unpack_pair_u8(wb[2 * w], wb[2 * w + 1], &cols[20 + 5 * w]);
                            }
                        }
                    }
                    // The stage is free once the MMAs of its previous use are done
                    // (waited after the unpack, so that the ALU work overlaps them).
                    // Every stage belongs to one group (stage = 2 * (k-block mod 4) + half
                    // for bf16, k-block mod 8 for int8), so the group sees each of its
                    // phases in order.
                    if (!warp_wait(&empty_a[sa], ((ua / C::kSA) & 1) ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < 5; ++c) {
                        uint32_t v8[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) v8[i] = cols[8 * c + i];
                        tmem_st8(a_addr + 8 * c, v8);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full_a[sa]);
                }
                if (!ok) break;
            }
            it = it_item + nkb;
            if (!ok) break;

            // ------------------------------------------------- epilogue ----
            // The epilogue reads what the previous grid wrote (split-tile
            // counters zeroed by the decode pre-pass, per-token scales and row
            // sums of the quantiser, a residual) and writes outputs it may
            // still read: wait for that grid.
            asm volatile("griddepcontrol.wait;" ::: "memory");
            // Issuer (it_item + a) % kIssuers accumulated k-blocks of this segment
            // iff a < its k-block count (segments are at least 2 k-blocks long).
            if (!warp_wait(acc_full, n_local & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const int64_t n = n0 + row;
            float bias_f = 0.0f;
            if (p.bias != nullptr && n < p.N) bias_f = __bfloat162float(p.bias[n]);
            // bf16 products: decode accumulators are in units of 2^-67; the
            // power-of-two rescale is exact, so acc * scale is rounded once.
            auto f16_out = [&](uint32_t a) {
                float v = __uint_as_float(a);
                if constexpr (C::kPerm) v = __fmul_rn(v, 0x1p67f);
                return __fmul_rn(v, p.scale);
            };
            // Fixed-point unit of the split-tile sums (2^-24 of an output unit).
            constexpr float kFix = C::kCorr ? 0x1p91f : kFixScale;
            // Final epilogue of 16 accumulator columns starting at c0.
            // MULTI: output-sharded layers store into every GPU's buffer; the
            // common single-output case is compiled separately.
            auto finish_t = [&](auto multi, int c0, const uint32_t (&acc)[16]) {
                constexpr bool MULTI = decltype(multi)::value;
                if (n >= p.N) return;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = m0 + c0 + j;
                    if (m >= p.M) break;
                    float yv;
                    if constexpr (KIND == Kind::F16) {
                        yv = f16_out(acc[j]);
                    } else {
                        const int acc_i = (int)acc[j] - 2 * __ldg(p.rowsum + m);
                        if (p.acc_out) p.acc_out[(int64_t)m * p.N + n] = acc_i;
                        const float f = __fmul_rn(p.scale, __ldg(p.s_x + m));
                        yv = __fmul_rn((float)acc_i, f);
                    }
                    if (p.n_out > 0) {
                        const __nv_bfloat16* res = nullptr;
                        int act = kActNone;
                        if constexpr (EPI) {
                            if (p.residual) res = p.residual + (int64_t)m * p.ld_res + n;
                            act = p.act;
                        }
                        if (p.y_f32) {
                            yv = epilogue_f32(yv, p.bias, bias_f, act, res);
                            if constexpr (MULTI) {
                                const int64_t off = (int64_t)m * p.ld_y + p.y_col0 + n;
                                for (int r = 0; r < p.n_out; ++r) static_cast<float*>(p.y_out[r])[off] = yv;
                            } else {
                                y0f[(int64_t)m * p.N + n] = yv;
                            }
                        } else {
                            const __nv_bfloat16 t = epilogue_bf16(yv, p.bias, bias_f, act, res);
                            if constexpr (MULTI) {
                                const int64_t off = (int64_t)m * p.ld_y + p.y_col0 + n;
                                for (int r = 0; r < p.n_out; ++r) static_cast<__nv_bfloat16*>(p.y_out[r])[off] = t;
                            } else {
                                y0h[(int64_t)m * p.N + n] = t;
                            }
                        }
                    }
                }
            };
            // Common case in one straight pass: one bf16 output, no bias, no
            // accumulator copy, all 16 tokens of the chunk present.
            auto finish_fast = [&](int c0, const uint32_t (&acc)[16]) {
                if (n >= p.N) return;
                __nv_bfloat16* yp = y0h + (int64_t)(m0 + c0) * p.N + n;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    float yv;
                    if constexpr (KIND == Kind::F16) {
                        yv = f16_out(acc[j]);
                    } else {
                        const int m = m0 + c0 + j;
                        const int acc_i = (int)acc[j] - 2 * __ldg(p.rowsum + m);
                        yv = __fmul_rn((float)acc_i, __fmul_rn(p.scale, __ldg(p.s_x + m)));
                    }
                    yp[(int64_t)j * p.N] = __float2bfloat16_rn(yv);
                }
            };
            // The same for output-sharded products: the 16 values are computed
            // once, then each output buffer gets one straight run of stores.
            auto finish_fast_multi = [&](int c0, const uint32_t (&acc)[16]) {
                if (n >= p.N) return;
                __nv_bfloat16 v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    float yv;
                    if constexpr (KIND == Kind::F16) {
                        yv = f16_out(acc[j]);
                    } else {
                        const int m = m0 + c0 + j;
                        const int acc_i = (int)acc[j] - 2 * __ldg(p.rowsum + m);
                        yv = __fmul_rn((float)acc_i, __fmul_rn(p.scale, __ldg(p.s_x + m)));
                    }
                    v[j] = __float2bfloat16_rn(yv);
                }
                const int64_t off = (int64_t)(m0 + c0) * p.ld_y + p.y_col0 + n;
                for (int r = 0; r < p.n_out; ++r) {
                    __nv_bfloat16* yp = static_cast<__nv_bfloat16*>(p.y_out[r]) + off;
#pragma unroll
                    for (int j = 0; j < 16; ++j) yp[(int64_t)j * p.ld_y] = v[j];
                }
            };
            // One bf16 output with a bias, an activation or a residual: the
            // same straight pass with the fused epilogue ops.
            auto finish_epi = [&](int c0, const uint32_t (&acc)[16]) {
                if (n >= p.N) return;
                __nv_bfloat16* yp = y0h + (int64_t)(m0 + c0) * p.N + n;
                const __nv_bfloat16* rp = p.residual + (int64_t)(m0 + c0) * p.ld_res + n;
                // Residual values are loaded eight at a time ahead of their
                // stores: the residual may be the output itself, so the compiler
                // cannot move a load above an earlier store, and interleaved they
                // would cost one memory round trip per value.
#pragma unroll
                for (int j0 = 0; j0 < 16; j0 += 8) {
                    __nv_bfloat16 rv[8];
                    if (p.residual) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) rv[j] = rp[(int64_t)(j0 + j) * p.ld_res];
                    }
#pragma unroll
                    for (int j = j0; j < j0 + 8; ++j) {
                        float yv;
                        if constexpr (KIND == Kind::F16) {
                            yv = f16_out(acc[j]);
                        } else {
                            const int m = m0 + c0 + j;
                            const int acc_i = (int)acc[j] - 2 * __ldg(p.rowsum + m);
                            yv = __fmul_rn((float)acc_i, __fmul_rn(p.scale, __ldg(p.s_x + m)));
                        }
                        yp[(int64_t)j * p.N] =
                            epilogue_bf16(yv, p.bias, bias_f, p.act, p.residual ? &rv[j - j0] : nullptr);
                    }
                }
            };
            const bool plain_out = !p.y_f32 && p.bias == nullptr && p.acc_out == nullptr &&
                                   (!EPI || (p.residual == nullptr && p.act == kActNone));
            const bool fast_out = p.n_out == 1 && plain_out;
            const bool epi_out = EPI && p.n_out == 1 && !p.y_f32 && p.acc_out == nullptr && !plain_out;
            // Limb decode: a chunk holds 4 tokens; token j's limb sums D0..D3
            // (columns 4j..4j+3) combine exactly as D0 + 2^8 D1 + 2^16 D2 +
            // 2^24 D3 in 64 bits, minus twice its offset correction; then one
            // conversion to fp32, the exact power-of-two rescale 2^-S and the
            // weight scale.
            auto finish_l8 = [&](int c0, const uint32_t (&acc)[16]) {
                if (n >= p.N) return;
#pragma unroll
                for (int j = 0; j < 16 / kL8Cols; ++j) {
                    const int m = m0 + c0 / kL8Cols + j;
                    if (m >= p.M) break;
                    const int sh = __ldcg(p.lx_shift + m);
                    float yv;
                    if (sh == kL8NonFinite) {
                        yv = __int_as_float(0x7fc00000);
                    } else {
                        long long corr = 0;
                        for (int c = 0; c < p.lx_chunks; ++c) corr += __ldcg(p.lx_corr + (size_t)m * p.lx_chunks + c);
                        const long long r = (long long)(int)acc[kL8Cols * j] +
                                            (long long)(int)acc[kL8Cols * j + 1] * 256 +
                                            (long long)(int)acc[kL8Cols * j + 2] * 65536 +
                                            (long long)(int)acc[kL8Cols * j + 3] * 16777216 - 2 * corr;
                        yv = __fmul_rn(scale_pow2(__ll2float_rn(r), -sh), p.scale);
                    }
                    if (p.n_out == 0) continue;
                    const __nv_bfloat16* res = nullptr;
                    int act = kActNone;
                    if constexpr (EPI) {
                        if (p.residual) res = p.residual + (int64_t)m * p.ld_res + n;
                        act = p.act;
                    }
                    const int64_t off = (int64_t)m * p.ld_y + p.y_col0 + n;
                    if (p.y_f32) {
                        yv = epilogue_f32(yv, p.bias, bias_f, act, res);
                        for (int r = 0; r < p.n_out; ++r) static_cast<float*>(p.y_out[r])[off] = yv;
                    } else {
                        const __nv_bfloat16 t = epilogue_bf16(yv, p.bias, bias_f, act, res);
                        for (int r = 0; r < p.n_out; ++r) static_cast<__nv_bfloat16*>(p.y_out[r])[off] = t;
                    }
                }
            };
            auto finish = [&](int c0, const uint32_t (&acc)[16]) {
                if constexpr (C::kL8) {
                    finish_l8(c0, acc);
                } else {
                    if constexpr (EPI) {
                        if (epi_out && m0 + c0 + 16 <= p.M) {
                            finish_epi(c0, acc);
                            return;
                        }
                    }
                    if (fast_out && m0 + c0 + 16 <= p.M)
                        finish_fast(c0, acc);
                    else if (p.n_out > 1 && plain_out && m0 + c0 + 16 <= p.M)
                        finish_fast_multi(c0, acc);
                    else if (p.n_out > 1)
                        finish_t(std::true_type{}, c0, acc);
                    else
                        finish_t(std::false_type{}, c0, acc);
                }
            };
            auto add_into = [&](uint32_t& d, uint32_t v) {
                if constexpr (KIND == Kind::F16)
                    d = __float_as_uint(__fadd_rn(__uint_as_float(d), __uint_as_float(v)));
                else
                    d = (uint32_t)((int)d + (int)v);
            };
            // Split tiles: 16-token tiles add into the sum buffer of the tile's
            // first contributor (each CTA is the first contributor of at most
            // one split tile); larger tiles publish partials to this CTA's
            // slot 0 (its first tile) or 1.
            constexpr bool kRedSum = BT <= 16;
            const int Pp = p.n_kb / 2;
            const int c_first = g.whole ? 0 : owner_of(p, (int64_t)g.tile * Pp);
            // sum (row, c) of the split tile at acc_base + c * kRows: a warp's lanes are contiguous
            const size_t acc_base = (size_t)c_first * kRows * p.acc_cols + row;
            const int slot = g.tile == my_first_tile ? 0 : 1;
            // partial (row, c) at part[(c / 4) * 512 + c % 4]
            uint32_t* part = static_cast<uint32_t*>(p.accbuf) + (size_t)(blockIdx.x * 2 + slot) * kRows * BT + row * 4;
            // This thread's accumulator columns: chunks c0 = 16*half + 64*i.
#pragma unroll 1
            for (int c0 = 16 * half; c0 < BT; c0 += 16 * kUnpackGroups) {
                if (c0 >= ncol) break;  // warp-uniform
                uint32_t acc[16], v[16];
                tmem_ld16(tmem_base + lane_base + (it_item % C::kIssuers) * C::kMmaN + c0, acc);
                tmem_wait_ld();
                for (int a = 1; a < C::kIssuers && a < g.kb1 - g.kb0; ++a) {
                    tmem_ld16(tmem_base + lane_base + ((it_item + a) % C::kIssuers) * C::kMmaN + c0, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) add_into(acc[j], v[j]);
                }
                if (g.whole) {
                    finish(c0, acc);
                } else if constexpr (kRedSum) {
                    // (griddepcontrol.wait above: the decode pre-pass zeroed the sums)
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (c0 + j >= ncol) break;
                        if constexpr (KIND == Kind::F16)
                            red_add(static_cast<long long*>(p.accbuf) + acc_base + (size_t)(c0 + j) * kRows,
                                    __float2ll_rn(__uint_as_float(acc[j]) * kFix));
                        else
                            red_add(static_cast<int*>(p.accbuf) + acc_base + (size_t)(c0 + j) * kRows, (int)acc[j]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<uint4*>(part + (c0 + j) * kRows) =
                            make_uint4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                }
            }
            // TMEM is free for the next segment.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);

            if (!g.whole) {
                // Each warp owns a fixed slice of the tile (its 32 rows x its
                // column chunks) in every contributing CTA, so arrivals are
                // counted per (tile, warp): the last warp to add (or publish)
                // its slice turns that slice of the sum into outputs.
                const int c_last = owner_of(p, (int64_t)g.tile * Pp + Pp - 1);
                __threadfence();
                __syncwarp();
                int last = 0;
                if (lane == 0) {
                    int* ctr = p.counters + (size_t)g.tile * kUnpackWarps + warp;
                    last = atomicAdd(ctr, 1) == c_last - c_first;
                    if (last) *ctr = 0;  // ready for the next launch
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
#pragma unroll 1
                    for (int c0 = 16 * half; c0 < BT; c0 += 16 * kUnpackGroups) {
                        if (c0 >= ncol) break;
                        uint32_t acc[16];
                        if constexpr (kRedSum) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                acc[j] = 0;
                                if (c0 + j < ncol) {
                                    if constexpr (KIND == Kind::F16) {
                                        const long long v =
                                            __ldcg(static_cast<const long long*>(p.accbuf) + acc_base + (size_t)(c0 + j) * kRows);
                                        acc[j] = __float_as_uint(__ll2float_rn(v) * (1.0f / kFix));
                                    } else {
                                        acc[j] = (uint32_t)__ldcg(static_cast<const int*>(p.accbuf) + acc_base + (size_t)(c0 + j) * kRows);
                                    }
                                }
                            }
                        } else {
                            // CTA c's partials sit in its slot 0 when the tile is its
                            // first one, else in slot 1; summed in CTA order.
                            for (int c = c_first; c <= c_last; ++c) {
                                const int slot_c = g.tile == (int)(range_begin(p, c) / Pp) ? 0 : 1;
                                const uint32_t* pc = static_cast<const uint32_t*>(p.accbuf) +
                                                     (size_t)(c * 2 + slot_c) * kRows * BT + row * 4 + c0 * kRows;
#pragma unroll
                                for (int j = 0; j < 16; j += 4) {
                                    const uint4 q4 = __ldcg(reinterpret_cast<const uint4*>(pc + j * kRows));
                                    if (c == c_first) {
                                        acc[j] = q4.x;
                                        acc[j + 1] = q4.y;
                                        acc[j + 2] = q4.z;
                                        acc[j + 3] = q4.w;
                                    } else {
                                        add_into(acc[j], q4.x);
                                        add_into(acc[j + 1], q4.y);
                                        add_into(acc[j + 2], q4.z);
                                        add_into(acc[j + 3], q4.w);
                                    }
                                }
                            }
                        }
                        finish(c0, acc);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Outputs written into other GPUs' memory are ordered before this grid's
    // completion, which the cross-GPU barrier after the product relies on:
    // one system-scope fence per CTA, after the CTA barrier that orders every
    // thread's stores before it (a fence in each storing thread cost ~10 us
    // per launch).
    if (p.n_out > 1 && threadIdx.x == 0) __threadfence_system();
    if (warp == kMmaWarp) tmem_dealloc(tmem_base, kTmemCols);
}

// Writes the activations of a bf16 decode tile as the GEMM kernel's shared-
// memory image of its B operand: per k-block 10 slabs (MMA K-steps) of BT rows
// x 32 bytes, 32-byte swizzled, each 10-group of k permuted by perm_src and
// scaled by 2^(133 - 67 - perm_exp) (exact), then an 11th slab holding the
// k-block's offset correction: the weights enter the MMAs as their codes
// c = q + 2, so sum_k q x = sum_k c x - 2 sum_k x, and per token the value
// t = -2 * 2^-67 * sum_k x (the sum over the k-block, in fp32, in a fixed
// order) is stored as three bf16 pieces (t = p1 + p2 + p3 exactly) at K
// positions 0-2, which the kernel multiplies by constant 1.0 A columns.
// Positions past K are zero; rows >= M are not written (their accumulator
// columns are never read back).
//
// One block per (group of kPermTok tokens, k-block) at a time, one thread per
// position of the k-block (160 threads, five warps): every thread loads,
// scales and stores the value of each of the group's tokens (independent
// loads in flight together), and each token's k-block sum is a fixed-order
// reduction (a shuffle tree per warp, then the five warp sums in order), so
// the result is deterministic.
constexpr int kPermThreads = kKB;
constexpr int kPermTok = 4;
template <int BT>
__global__ void __launch_bounds__(kPermThreads) permute_x_kernel(const __nv_bfloat16* __restrict__ x, int M, int64_t K,
                                                        int n_kb, uint8_t* __restrict__ out, uint4* __restrict__ zero,
                                                        int64_t n_zero16) {
    // The GEMM launched after this kernel (programmatic dependent launch) may
    // start its prologue and weight streaming now; it waits for this grid's
    // results before it reads them.
    asm volatile("griddepcontrol.launch_dependents;");
    // the GEMM's split-tile counters and sums start at zero
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_zero16; i += (int64_t)gridDim.x * blockDim.x)
        zero[i] = make_uint4(0, 0, 0, 0);
    constexpr int kStage = BT * 32 * 11;
    __shared__ float warp_sum[kPermTok][kPermThreads / 32];
    const uint32_t e = threadIdx.x;  // position in the k-block
    const uint32_t grp = e / kPerWord;
    const int q = (int)(e - grp * kPerWord);
    const uint32_t src = grp * kPerWord + perm_src(q);
    const uint32_t j = e >> 4, ee = e & 15;
    // * 2^(133 - 67 - perm_exp(q)), exact
    const float vscale = __int_as_float((127 + 133 - kPermUnitExp - perm_exp(q)) << 23);
    // 32-bit index arithmetic (the host checks M * n_kb * 160 < 2^31)
    const uint32_t groups = ((uint32_t)M + kPermTok - 1) / kPermTok;
    const uint32_t pairs = groups * (uint32_t)n_kb;
    for (uint32_t mk = blockIdx.x; mk < pairs; mk += gridDim.x) {
        const uint32_t mg = mk / (uint32_t)n_kb;
        const uint32_t kb = mk - mg * (uint32_t)n_kb;
        const uint32_t ksrc = kb * kKB + src;
        float v[kPermTok];
#pragma unroll
        for (int t = 0; t < kPermTok; ++t) {
            const uint32_t m = mg * kPermTok + t;
            v[t] = (m < (uint32_t)M && ksrc < (uint64_t)K) ? __bfloat162float(x[(size_t)m * K + ksrc]) : 0.0f;
        }
#pragma unroll
        for (int t = 0; t < kPermTok; ++t) {
            const uint32_t m = mg * kPermTok + t;
            if (m < (uint32_t)M) {
                uint8_t* const kbase = out + (size_t)kb * kStage + m * 32;
                const uint32_t flip = (m >> 2) & 1;  // 32-byte swizzle: 16-byte halves swap every 4 rows
                *reinterpret_cast<__nv_bfloat16*>(kbase + j * (BT * 32) + (((ee >> 3) ^ flip) << 4) + (ee & 7) * 2) =
                    __float2bfloat16_rn(__fmul_rn(v[t], vscale));
            }
            float sum = v[t];
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 16));
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 8));
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 4));
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
            sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
            if ((e & 31) == 0) warp_sum[t][e >> 5] = sum;
        }
        __syncthreads();
        if (e < kPermTok && mg * kPermTok + e < (uint32_t)M) {
            const uint32_t m = mg * kPermTok + e;
            uint8_t* const kbase = out + (size_t)kb * kStage + m * 32;
            const uint32_t flip = (m >> 2) & 1;
            float t = warp_sum[e][0];
#pragma unroll
            for (int w = 1; w < kPermThreads / 32; ++w) t = __fadd_rn(t, warp_sum[e][w]);
            t = __fmul_rn(t, -0x1p-66f);  // -2 * 2^-67 * sum, exact
            const __nv_bfloat16 p1 = __float2bfloat16_rn(t);
            const float r1 = __fsub_rn(t, __bfloat162float(p1));
            const __nv_bfloat16 p2 = __float2bfloat16_rn(r1);
            const __nv_bfloat16 p3 = __float2bfloat16_rn(__fsub_rn(r1, __bfloat162float(p2)));
            const uint32_t w01 = (uint32_t)__bfloat16_as_ushort(p1) | ((uint32_t)__bfloat16_as_ushort(p2) << 16);
            const uint32_t w23 = (uint32_t)__bfloat16_as_ushort(p3);
            uint8_t* const slab = kbase + 10 * (BT * 32);
            *reinterpret_cast<uint4*>(slab + (flip << 4)) = make_uint4(w01, w23, 0u, 0u);       // K 0-7
            *reinterpret_cast<uint4*>(slab + ((flip ^ 1) << 4)) = make_uint4(0u, 0u, 0u, 0u);  // K 8-15
        }
        __syncthreads();  // warp_sum is reused by the next pair
    }
}

// Limb decode pre-pass: writes a decode batch's bf16 activations as the GEMM
// kernel's shared-memory image of its int8 B operand.
//
// Per token m: E with max|x_m| < 2^E (from the largest bf16 magnitude), the
// fixed-point exponent S = 30 - E, and for every k the integer
// X_k = round_half_even(x_k * 2^(S - t_k)), |X_k| <= 2^30, where t_k is the
// shift its weight carries in the A operand (unpack_pair_l8).  X_k is split
// into balanced base-256 limbs X = L0 + 2^8 L1 + 2^16 L2 + 2^24 L3, each in
// [-128, 127], stored in the B rows (accumulator columns) 4m .. 4m+3; the MMAs
// then sum c_k 2^t_k L_l,k exactly in int32 per limb.  The code offset enters
// as corr_m = sum_k 2^t_k X_k (exact, int64), from which the epilogue forms
// sum_k (c_k - 2) 2^t_k X_k = sum_k q_k x~_k 2^S, x~_k being x_k rounded to a
// multiple of 2^(t_k - S) <= 2^(E - 25): at most 2^-25 max|x_m| away, and
// exact for every element within a factor 2^17 of the row's largest magnitude.
//
// Layout: per k-block 5 slabs (MMA K-steps of 32 k) of BT rows x 32 bytes,
// 32-byte swizzled; MMA position r of a k-block holds k = 20 (r / 20) +
// l8_src(r % 20).  Rows of tokens >= M are not written (their accumulator
// columns are never read back).
//
// Grid (chunks + zeroing blocks, M); each chunk block reduces the token's
// whole row for max|x| (the row is in L2: the redundant reads are cheap at
// decode sizes), then writes kb_per_chunk k-blocks, one thread per 4 MMA
// positions, and its partial correction to lx_corr[m][chunk].
constexpr int kLimbThreads = 256;
template <int BT>
__global__ void __launch_bounds__(kLimbThreads) limb_x_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                                                               int n_kb, int kb_per_chunk, int n_chunks,
                                                               uint8_t* __restrict__ out, int* __restrict__ lx_shift,
                                                               long long* __restrict__ lx_corr,
                                                               uint4* __restrict__ zero, int64_t n_zero16) {
    asm volatile("griddepcontrol.launch_dependents;");
    // the GEMM's split-tile counters and sums start at zero
    {
        const int64_t b = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
        const int64_t nthr = (int64_t)gridDim.x * gridDim.y * kLimbThreads;
        for (int64_t i = b * kLimbThreads + threadIdx.x; i < n_zero16; i += nthr) zero[i] = make_uint4(0, 0, 0, 0);
    }
    const int ch = blockIdx.x;
    if (ch >= n_chunks) return;  // zeroing-only block
    const int m = blockIdx.y;
    const __nv_bfloat16* xr = x + (size_t)m * K;
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(xr);

    // max |x| of the row as bf16 magnitude bits (ordered like the values;
    // 0x7F80 and above: inf or NaN)
    uint32_t mx = 0;
    if ((reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
        const int nv = K >> 3;
        const uint4* xv = reinterpret_cast<const uint4*>(xr);
        for (int i = threadIdx.x; i < nv; i += kLimbThreads) {
            const uint4 v = __ldg(xv + i);
            uint32_t t = __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                                  __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
            t = max(t & 0xFFFFu, t >> 16);
            mx = max(mx, t);
        }
        for (int k = (nv << 3) + threadIdx.x; k < K; k += kLimbThreads) mx = max(mx, (uint32_t)(__ldg(xs + k) & 0x7FFFu));
    } else {
        for (int k = threadIdx.x; k < K; k += kLimbThreads) mx = max(mx, (uint32_t)(__ldg(xs + k) & 0x7FFFu));
    }
    __shared__ uint32_t red_u[kLimbThreads / 32];
    __shared__ long long red_ll[kLimbThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red_u[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red_u[0];
#pragma unroll
    for (int w = 1; w < kLimbThreads / 32; ++w) mx = max(mx, red_u[w]);

    const bool finite = mx < 0x7F80u;
    // max|x| < 2^E; E = -126 covers zero and subnormal maxima
    const int ebits = (int)(mx >> 7);
    const int E = ebits == 0 ? -126 : ebits - 126;
    const int S = 30 - E;
    if (ch == 0 && threadIdx.x == 0) lx_shift[m] = finite ? S : kL8NonFinite;

    constexpr int kSlab = BT * 32;
    constexpr int kStage = 5 * kSlab;
    const uint32_t flip = (uint32_t)(m & 1) << 4;  // 32-byte swizzle: rows 4m..4m+3 share (row >> 2) & 1 = m & 1
    uint8_t* const rows = out + (size_t)m * 4 * 32;
    long long corr = 0;
    const int kb0 = ch * kb_per_chunk;
    const int kb1 = min(n_kb, kb0 + kb_per_chunk);
    const int nq = (kb1 - kb0) * (kKB / 4);  // 40 quads of MMA positions per k-block
    for (int qi = threadIdx.x; qi < nq; qi += kLimbThreads) {
        const int kb = kb0 + qi / (kKB / 4);
        const int qk = qi - (kb - kb0) * (kKB / 4);  // quad within the k-block
        uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = 4 * qk + i;          // MMA position in the k-block
            const int pr = r / 20, rr = r - 20 * (r / 20);
            const int t = l8_shift(rr);
            const int k = kb * kKB + 20 * pr + l8_src(rr);
            int X = 0;
            if (finite && k < K) {
                const float xf = __uint_as_float((uint32_t)__ldg(xs + k) << 16);
                X = __float2int_rn(scale_pow2(xf, S - t));
            }
            corr += (long long)X * (1 << t);
            const int l0 = (int)(int8_t)X;
            const int x1 = (X - l0) >> 8;
            const int l1 = (int)(int8_t)x1;
            const int x2 = (x1 - l1) >> 8;
            const int l2 = (int)(int8_t)x2;
            const int l3 = (x2 - l2) >> 8;
            w0 |= (uint32_t)(l0 & 0xFF) << (8 * i);
            w1 |= (uint32_t)(l1 & 0xFF) << (8 * i);
            w2 |= (uint32_t)(l2 & 0xFF) << (8 * i);
            w3 |= (uint32_t)(l3 & 0xFF) << (8 * i);
        }
        // slab qk / 8, bytes 4 (qk % 8) .. +3 of each limb row
        const uint32_t b = 4u * (uint32_t)(qk & 7);
        uint8_t* const dst = rows + (size_t)kb * kStage + (qk >> 3) * kSlab + ((((b >> 4) << 4) ^ flip) | (b & 15));
        *reinterpret_cast<uint32_t*>(dst) = w0;
        *reinterpret_cast<uint32_t*>(dst + 32) = w1;
        *reinterpret_cast<uint32_t*>(dst + 64) = w2;
        *reinterpret_cast<uint32_t*>(dst + 96) = w3;
    }
    // the block's correction partial (integer sums: order-independent)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) corr += __shfl_xor_sync(0xffffffffu, corr, o);
    if ((threadIdx.x & 31) == 0) red_ll[threadIdx.x >> 5] = corr;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long t = 0;
#pragma unroll
        for (int w = 0; w < kLimbThreads / 32; ++w) t += red_ll[w];
        lx_corr[(size_t)m * n_chunks + ch] = t;
    }
}

// ------------------------------------------------------------------ host ----

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

int device_sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    return n;
}

// Limb decode (Kind::L8) takes bf16 products of at most g_l8_max_tokens
// tokens (settable, 0 = off) with K <= kL8MaxK.
static int g_l8_max_tokens = kL8DefaultTokens;
int l8_max_tokens() { return g_l8_max_tokens; }
void set_l8_max_tokens(int m) { g_l8_max_tokens = m < 0 ? 0 : (m > kL8MaxTokens ? kL8MaxTokens : m); }
static bool l8_shape(int kind, int64_t M, int64_t K) {
    return kind == PN_BF16 && M >= 1 && M <= kL8MaxTokens && K <= kL8MaxK;
}
static bool l8_takes(int kind, int64_t M, int64_t K) { return l8_shape(kind, M, K) && M <= g_l8_max_tokens; }
// accumulator columns of a limb tile: 4 per token
static int l8_tile(int64_t M) { return M <= 2 ? 8 : (M <= 4 ? 16 : (M <= 8 ? 32 : 64)); }
constexpr int kL8KbPerChunk = 16;  // k-blocks per limb_x_kernel block

// k-blocks per item: enough to cover the packed words, rounded up to even so
// that weight stages (2 k-blocks each) never straddle items.  The padding block
// multiplies zero activations (past K) by zero-filled weights.
static int n_kblocks(int64_t KP) {
    const int64_t n = (KP * kPerWord + kKB - 1) / kKB;
    return (int)((n + 1) & ~int64_t(1));
}

static size_t round256(size_t b) { return (b + 255) & ~size_t(255); }
static int64_t w_pitch(int64_t KP) { return (KP + 3) & ~int64_t(3); }

// Token tile for a call: the kernel instantiation launch_kind picks.
static int token_tile(int kind, int64_t M) {
    if (kind == PN_BF16 && M <= 8) return 8;
    if (M <= 16) return 16;
    if (M <= 32) return 32;
    if (M <= 64) return 64;
    if (kind == PN_BF16 || M <= 128) return 128;
    return 256;
}

// Workspace sections, each 256-byte aligned:
//   [decode activation slabs (bf16, M <= 64)]
//   [weights re-pitched to 16-byte rows (K_packs % 4 != 0)]
//   [split-tile arrival counters: one int per tile and unpack warp]
//   [split-tile sums (16-token tiles): grid x 128 x min(16, M), int64 (bf16) /
//    int32 (int8) -- zeroed with the counters in one pass -- or partials
//    (larger tiles): grid x 2 x 128 x BT x 4 bytes]
// Tiles split across CTAs only while there are few of them per SM; with many
// tiles whole-tile ranges already balance to within one tile.
struct WsLayout {
    size_t xperm, wpitch, counters, accbuf, zero_bytes, total, lx_shift, lx_corr;
    int64_t n_items, total_pairs;
    int grid, bt, n_kb, unit, acc_cols, n_chunks;
};
// repitch: the packed rows are not 16 bytes apart (packed_ld % 4 != 0), so a
// 16-byte-pitch copy of the whole matrix is part of the workspace.
// l8: the limb decode layout (limb image, per-token exponents and correction
// partials; BT counts accumulator columns, four per token).
static WsLayout ws_layout_ex(int kind, int64_t M, int64_t N, int64_t K, bool allow_split, bool repitch, bool l8) {
    WsLayout w{};
    const int64_t KP = (K + kPerWord - 1) / kPerWord;
    w.bt = l8 ? l8_tile(M) : token_tile(kind, M);
    const int cpt = l8 ? kL8Cols : 1;
    w.n_kb = n_kblocks(KP);
    w.n_chunks = l8 ? (w.n_kb + kL8KbPerChunk - 1) / kL8KbPerChunk : 0;
    w.n_items = ((N + kRows - 1) / kRows) * ((M * cpt + w.bt - 1) / w.bt);
    w.total_pairs = w.n_items * (w.n_kb / 2);
    int sms = device_sm_count();
    if (sms <= 0) sms = 148;
    const bool split = allow_split && w.n_items % sms != 0 && w.n_items < 8 * (int64_t)sms;
    w.unit = split ? 1 : w.n_kb / 2;
    const int64_t units = w.total_pairs / w.unit;
    w.grid = (int)(units < sms ? units : sms);
    size_t off = 0;
    w.xperm = off;
    if (l8) {
        off += round256((size_t)w.n_kb * w.bt * 32 * 5);
        w.lx_shift = off;
        off += round256((size_t)M * 4);
        w.lx_corr = off;
        off += round256((size_t)M * w.n_chunks * 8);
    } else if (kind == PN_BF16 && M >= 1 && M <= 64) {
        off += round256((size_t)w.n_kb * w.bt * 32 * 11);
    }
    w.wpitch = off;
    if (repitch) off += round256((size_t)N * w_pitch(KP) * 4);
    w.acc_cols = (int)(M * cpt < 16 ? M * cpt : 16);
    w.counters = off;
    w.accbuf = off;
    w.zero_bytes = 0;
    if (split) {
        off += round256((size_t)w.n_items * kUnpackWarps * 4);
        w.accbuf = off;
        if (w.bt <= 16) {
            off += round256((size_t)w.grid * kRows * w.acc_cols * (kind == PN_BF16 && !l8 ? 8 : 4));
            w.zero_bytes = off - w.counters;  // counters and sums
        } else {
            w.zero_bytes = off - w.counters;  // counters only
            off += round256((size_t)w.grid * 2 * kRows * w.bt * 4);
        }
    }
    w.total = off;
    return w;
}
static WsLayout ws_layout(int kind, int64_t M, int64_t N, int64_t K, bool allow_split, bool repitch) {
    return ws_layout_ex(kind, M, N, K, allow_split, repitch, l8_takes(kind, M, K));
}
size_t linear_workspace_bytes(int kind, int64_t M, int64_t N, int64_t K, int64_t packed_ld) {
    if (M <= 0 || N <= 0) return 0;
    size_t tc = ws_layout_ex(kind, M, N, K, true, packed_ld % 4 != 0, false).total;
    // enough for either tensor-core decode path, whichever pn_set_limb_max_tokens selects
    if (l8_shape(kind, M, K)) {
        const size_t t8 = ws_layout_ex(kind, M, N, K, true, packed_ld % 4 != 0, true).total;
        if (t8 > tc) tc = t8;
    }
    // bf16 decode batches may run on the CUDA-core GEMV instead (pn_gemv.cu)
    const size_t gv = kind == PN_BF16 ? gemv_workspace_bytes(M, N, (K + kPerWord - 1) / kPerWord) : 0;
    return tc > gv ? tc : gv;
}
size_t linear_workspace_min_bytes(int kind, int64_t M, int64_t N, int64_t K, int64_t packed_ld) {
    if (M <= 0 || N <= 0) return 0;
    return ws_layout(kind, M, N, K, false, packed_ld % 4 != 0).total;
}

// Copies packed rows (src_ld words apart) into a 16-byte pitch so that TMA
// can address them.
__global__ void __launch_bounds__(256) repitch_kernel(const int32_t* __restrict__ src, int64_t src_ld, int64_t N,
                                                      int64_t KP, int64_t pitch, int32_t* __restrict__ dst) {
    const int64_t total = N * KP;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / KP;
        const int64_t w = i - n * KP;
        dst[n * pitch + w] = __ldg(src + n * src_ld + w);
    }
}

template <Kind KIND, int BT, bool EPI>
static int launch_bt(const LinearArgs& a, cudaStream_t s, cudaError_t* err, const char** why) {
    using C = Cfg<KIND, BT>;
    using T = typename C::T;
    EncodeTiledFn encode = get_encode_fn();
    if (!encode) {
        *why = "cuTensorMapEncodeTiled unavailable";
        return PN_ERR_CUDA;
    }
    const int64_t pitch_bytes = a.x_pitch * T::kXElem;
    const CUtensorMapDataType xdt = KIND == Kind::F16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    cuuint32_t estr[3] = {1, 1, 1};
    // Activations: two 2D maps over the (M, K) rows, one with a box of 128-byte
    // rows (128-byte swizzle) and one with a box of the k-block's remaining
    // 32 or 64 bytes per row (matching swizzle).  Columns >= K and rows >= M
    // are zero-filled.  Decode tiles stage pre-arranged slabs without a map.
    CUtensorMap xmap, xmap_tail;
    std::memset(&xmap, 0, sizeof(xmap));
    std::memset(&xmap_tail, 0, sizeof(xmap_tail));
    if (!C::kPerm) {
        cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
        cuuint64_t strides[1] = {(cuuint64_t)pitch_bytes};
        cuuint32_t box[2] = {(cuuint32_t)(128 / T::kXElem), (cuuint32_t)BT};
        cuuint32_t box_tail[2] = {(cuuint32_t)(C::kTail / T::kXElem), (cuuint32_t)BT};
        if (encode(&xmap, xdt, 2, const_cast<void*>(a.x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
            encode(&xmap_tail, xdt, 2, const_cast<void*>(a.x), dims, strides, box_tail, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   C::kTail == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            *why = "cuTensorMapEncodeTiled rejected the activation layout";
            return PN_ERR_ALIGN;
        }
    }
    // Packed weights: one 128-byte-swizzled TMA box per weight stage (128 rows
    // x 32 words).  TMA needs 16-byte row pitches; other shapes are first copied
    // into the workspace with the pitch rounded up.
    // The full layout when the workspace holds it, else whole tiles per CTA.
    // TMA reads the rows in place when they are 16 bytes apart (a multiple of
    // 4 words: K_packs % 4 == 0, or rows stored at a padded stride); other
    // layouts are first copied into the workspace at a 16-byte pitch.
    const bool repitch = a.packed_ld % 4 != 0;
    WsLayout L = ws_layout(a.kind, a.M, a.N, a.K, true, repitch);
    if (a.workspace_bytes < L.total) L = ws_layout(a.kind, a.M, a.N, a.K, false, repitch);
    if (L.bt != BT) {
        *why = "internal: token tile mismatch";
        return PN_ERR_ARG;
    }
    if ((L.total > 0 && a.workspace == nullptr) || a.workspace_bytes < L.total ||
        reinterpret_cast<uintptr_t>(a.workspace) % 256) {
        *why = "workspace missing, too small or not 256-byte aligned";
        return PN_ERR_WORKSPACE;
    }
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    const int64_t pitch = repitch ? w_pitch(a.KP) : a.packed_ld;
    const int32_t* wsrc = a.packed;
    if (repitch) {
        int32_t* dst = reinterpret_cast<int32_t*>(ws + L.wpitch);
        const int64_t total = a.N * a.KP;
        const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
        repitch_kernel<<<blocks, 256, 0, s>>>(a.packed, a.packed_ld, a.N, a.KP, pitch, dst);
        wsrc = dst;
    }
    CUtensorMap wmap;
    {
        cuuint64_t dims[2] = {(cuuint64_t)a.KP, (cuuint64_t)a.N};
        cuuint64_t strides[1] = {(cuuint64_t)(pitch * 4)};
        cuuint32_t box[2] = {(cuuint32_t)kWStageWords, (cuuint32_t)kRows};
        if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<int32_t*>(wsrc), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            *why = "cuTensorMapEncodeTiled rejected the packed-weight layout";
            return PN_ERR_ALIGN;
        }
    }
    DqmmParams prm;
    prm.N = a.N;
    prm.KP = a.KP;
    prm.M = (int)a.M;
    prm.n_row_tiles = (int)((a.N + kRows - 1) / kRows);
    const int n_tok_tiles = (int)((a.M + BT - 1) / BT);
    prm.n_items = prm.n_row_tiles * n_tok_tiles;
    prm.total_pairs = L.total_pairs;
    {
        const int64_t units = L.total_pairs / L.unit;
        if (units * (int64_t)(L.grid + 1) >= (int64_t)1 << 32 || L.total_pairs >= (int64_t)1 << 32) {
            *why = "work split exceeds 32-bit indexing (shape too large)";
            return PN_ERR_UNSUPPORTED;
        }
        prm.units = (uint32_t)units;
    }
    prm.unit = L.unit;
    prm.accbuf = ws + L.accbuf;
    prm.acc_cols = L.acc_cols;
    prm.counters = reinterpret_cast<int*>(ws + L.counters);
    prm.n_kb = n_kblocks(a.KP);
    prm.xperm = ws + L.xperm;
    // split-tile counters start at zero (the decode pre-pass zeroes them, else a memset)
    const int64_t n_zero16 = L.unit == 1 ? (int64_t)(L.zero_bytes / 16) : 0;
    prm.lx_shift = reinterpret_cast<const int*>(ws + L.lx_shift);
    prm.lx_corr = reinterpret_cast<const long long*>(ws + L.lx_corr);
    prm.lx_chunks = L.n_chunks;
    if constexpr (C::kL8) {
        if (a.M * kL8Cols > BT || a.K > kL8MaxK) {
            *why = "internal: limb tile too small for the batch";
            return PN_ERR_ARG;
        }
        // chunk blocks per token, plus zeroing-only blocks when the split-tile
        // sums need them (~4 zeroing stores per thread)
        int64_t gx = L.n_chunks;
        const int64_t zx = (n_zero16 / (4 * kLimbThreads) + a.M - 1) / a.M;
        if (zx > gx) gx = zx < 4096 ? zx : 4096;
        const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(a.x);
        uint4* zero = reinterpret_cast<uint4*>(ws + L.counters);
        // A plain launch, like the bf16 decode pre-pass below; the GEMM is its
        // programmatic dependent.
        limb_x_kernel<BT><<<dim3((unsigned)gx, (unsigned)a.M), kLimbThreads, 0, s>>>(
            xb, (int)a.M, (int)a.K, prm.n_kb, kL8KbPerChunk, L.n_chunks, ws + L.xperm,
            reinterpret_cast<int*>(ws + L.lx_shift), reinterpret_cast<long long*>(ws + L.lx_corr), zero, n_zero16);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            *err = e;
            *why = "limb activation pre-pass launch";
            return PN_ERR_CUDA;
        }
    } else if (C::kPerm) {
        const int64_t total = a.M * (int64_t)prm.n_kb * kKB;
        if (total >= (int64_t)1 << 31) {
            *why = "activation re-layout exceeds 32-bit indexing (K too large)";
            return PN_ERR_UNSUPPORTED;
        }
        // one block per (token group, k-block); extra blocks when the zeroing needs them
        int64_t want = ((a.M + kPermTok - 1) / kPermTok) * (int64_t)prm.n_kb;
        if (n_zero16 / (4 * kPermThreads) > want) want = n_zero16 / (4 * kPermThreads);  // ~4 zeroing stores per thread
        const int blocks = (int)(want < 4096 ? (want > 0 ? want : 1) : 4096);
        const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(a.x);
        uint4* zero = reinterpret_cast<uint4*>(ws + L.counters);
        // A plain launch: it runs once everything before it on the stream is
        // done (its x may be the previous product's output, and its workspace
        // the previous product's), on SMs no GEMM occupies yet, so it is short;
        // the GEMM after it is its programmatic dependent.
        permute_x_kernel<BT><<<blocks, kPermThreads, 0, s>>>(xb, (int)a.M, a.K, prm.n_kb, ws + L.xperm, zero, n_zero16);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            *err = e;
            *why = "activation re-layout launch";
            return PN_ERR_CUDA;
        }
    } else if (n_zero16 > 0) {
        cudaError_t e = cudaMemsetAsync(ws + L.counters, 0, L.zero_bytes, s);
        if (e != cudaSuccess) {
            *err = e;
            *why = "cudaMemsetAsync of the split-tile counters";
            return PN_ERR_CUDA;
        }
    }
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
        prm.n_out = a.y != nullptr ? 1 : 0;
        for (int r = 0; r < 8; ++r) prm.y_out[r] = r == 0 ? a.y : nullptr;
        prm.ld_y = a.N;
        prm.y_col0 = 0;
    }
    prm.y_f32 = a.y_dtype == PN_F32;
    prm.acc_out = a.acc_out;
    prm.s_x = a.s_x;
    prm.rowsum = a.rowsum;

    auto kern = dqmm_kernel<KIND, BT, EPI>;
    static bool attr_done[64] = {};  // per instantiation and device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) {
            *err = e;
            *why = "cudaFuncSetAttribute";
            return PN_ERR_CUDA;
        }
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    const int grid = L.grid;
    cudaError_t e;
    {
        // Programmatic dependent launch: the GEMM's prologue, TMEM allocation
        // and weight streaming overlap the grid before it (the decode
        // pre-pass, the int8 quantiser, a LayerNorm: kernels that let their
        // dependents start early); the threads that read that grid's results
        // wait for it (griddepcontrol.wait).  After a kernel that does not
        // trigger early it simply starts when that kernel ends.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = C::kSmem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kern, xmap, xmap_tail, wmap, prm);
    }
    if (e != cudaSuccess) {
        *err = e;
        *why = "kernel launch";
        return PN_ERR_CUDA;
    }
    return PN_OK;
}

template <Kind KIND, bool EPI>
static int launch_kind(const LinearArgs& a, cudaStream_t s, cudaError_t* err, const char** why) {
    if constexpr (KIND == Kind::L8) {
        // accumulator columns: four per token
        if (a.M <= 2) return launch_bt<KIND, 8, EPI>(a, s, err, why);
        if (a.M <= 4) return launch_bt<KIND, 16, EPI>(a, s, err, why);
        if (a.M <= 8) return launch_bt<KIND, 32, EPI>(a, s, err, why);
        return launch_bt<KIND, 64, EPI>(a, s, err, why);
    } else {
        if constexpr (KIND == Kind::F16) {
            if (a.M <= 8) return launch_bt<KIND, 8, EPI>(a, s, err, why);
        }
        if (a.M <= 16) return launch_bt<KIND, 16, EPI>(a, s, err, why);
        if (a.M <= 32) return launch_bt<KIND, 32, EPI>(a, s, err, why);
        if (a.M <= 64) return launch_bt<KIND, 64, EPI>(a, s, err, why);
        if constexpr (KIND == Kind::F16) {
            // bf16 operands of a 256-token tile leave TMEM room for only 3 operand stages
            return launch_bt<KIND, 128, EPI>(a, s, err, why);
        } else {
            if (a.M <= 128) return launch_bt<KIND, 128, EPI>(a, s, err, why);
            return launch_bt<KIND, 256, EPI>(a, s, err, why);
        }
    }
}

int launch_linear(const LinearArgs& a, cudaStream_t s, cudaError_t* err, const char** why) {
    *err = cudaSuccess;
    *why = "";
    if (a.M == 0 || a.N == 0) return PN_OK;
    const bool epi = a.act != kActNone || a.residual != nullptr;
    if (l8_takes(a.kind, a.M, a.K))
        return epi ? launch_kind<Kind::L8, true>(a, s, err, why) : launch_kind<Kind::L8, false>(a, s, err, why);
    if (a.kind == PN_BF16)
        return epi ? launch_kind<Kind::F16, true>(a, s, err, why) : launch_kind<Kind::F16, false>(a, s, err, why);
    return epi ? launch_kind<Kind::I8, true>(a, s, err, why) : launch_kind<Kind::I8, false>(a, s, err, why);
}

}  // namespace pn
