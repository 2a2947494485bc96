// pn_static_ws.cu -- pn_linear_bf16 for callers that cannot allocate device memory.
//
// pn_linear_bf16 takes a caller-provided scratch workspace: for batches of up
// to 64 tokens it holds the activations re-laid-out for the decode kernel,
// for every batch the partial sums of output tiles split across SMs, and,
// when the packed rows are not 16 bytes apart, a re-pitched copy of the whole
// weight matrix.  Some callers have no way to provide it: code that runs where
// no allocator may be called (a host callback, a signal-safe or real-time
// path, an embedding that hands the library only raw input/output pointers,
// or a process whose device memory is fully reserved up front).
// pn_linear_bf16_nows serves them from one fixed scratch array that lives in
// this file as a __device__ variable: every GPU that loads the library holds
// kStaticScratchBytes of it until the process exits, and no call allocates or
// frees anything.
//
// Limits and sharing:
//   * the least scratch a call runs with must be <= kStaticScratchBytes
//     (4 MiB).  That is the decode activation image for M <= 64
//     (ceil(ceil(K/10)/16) rounded up to even x tile x 352 bytes, tile = 8,
//     16, 32 or 64 tokens: 4.06 MB at K = 28672 and 64 tokens), plus
//     N * round4(K_packs) * 4 bytes when the rows are not 16 bytes apart
//     (packed_ld % 4 != 0) -- far more than 4 MiB for most layers, so callers
//     store their weights at the pn_packed_ld(K_packs) stride.  Larger
//     requests are rejected with PN_ERR_WORKSPACE before anything is
//     enqueued.  When the array also holds the split-tile partial sums the
//     kernel uses them, else it gives each SM whole tiles;
//   * all calls on a device share the one array and it keeps the last call's
//     contents.  Each call sets every byte it later reads (the split-tile
//     counters by a memset or the decode pre-pass on its stream), so nothing
//     needs clearing between calls -- but calls that can overlap on the GPU
//     (different streams without ordering between them) race on the array and
//     must be serialised by the caller;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make that
//     first call before any stream capture on the device.  The cached address
//     belongs to the device's primary context: do not use this entry point
//     across a cudaDeviceReset of that device.
#include <mutex>

#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device (host code cannot
// use the symbol itself: on the host it names a stand-in, not device memory).
int static_scratch(void** out, const char** why) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *why = "no usable current device";
        return PN_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || p == nullptr) {
            *why = "cudaGetSymbolAddress of the static scratch array failed";
            return PN_ERR_CUDA;
        }
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return PN_OK;
}
}  // namespace
}  // namespace pn

extern "C" int pn_linear_bf16_nows(const void* x, int64_t M, int64_t K, const int32_t* packed, int64_t N,
                                   int64_t K_packs, int64_t packed_ld, float scale, const void* bias, void* y,
                                   int y_dtype, void* stream) {
    // The shape first, so that a bad shape reports PN_ERR_SHAPE rather than a
    // scratch size computed from it; pn_linear_bf16_ld repeats every check.
    if (M < 0 || N < 0 || K < 1 || M > 0x7fffffff || N > 0x7fffffff || K_packs != k_packs(K) || packed_ld < K_packs)
        return fail(PN_ERR_SHAPE, "pn_linear_bf16_nows: M=%lld N=%lld K=%lld K_packs=%lld packed_ld=%lld",
                    (long long)M, (long long)N, (long long)K, (long long)K_packs, (long long)packed_ld);
    const size_t need = pn::linear_workspace_min_bytes(PN_BF16, M, N, K, packed_ld);
    if (need > pn::kStaticScratchBytes) {
        if (packed_ld % 4 != 0)
            return fail(PN_ERR_WORKSPACE,
                        "pn_linear_bf16_nows: this shape needs %zu bytes of scratch, most of it a 16-byte-pitch copy "
                        "of the weights (packed_ld %% 4 != 0); the static array holds %zu: store the packed rows at "
                        "pn_packed_ld(K_packs) = %lld words",
                        need, pn::kStaticScratchBytes, (long long)pn_packed_ld(K_packs));
        return fail(PN_ERR_WORKSPACE,
                    "pn_linear_bf16_nows: this shape needs %zu bytes of scratch; the static array holds %zu "
                    "(use pn_linear_bf16 with a caller-provided workspace)",
                    need, pn::kStaticScratchBytes);
    }
    void* ws = nullptr;
    const char* why = "";
    if (const int st = pn::static_scratch(&ws, &why)) return fail(st, "pn_linear_bf16_nows: %s", why);
    return pn_linear_bf16_ld(x, M, K, packed, N, K_packs, packed_ld, scale, bias, y, y_dtype, ws,
                             pn::kStaticScratchBytes, stream);
}
