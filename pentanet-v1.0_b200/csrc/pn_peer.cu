// pn_peer.cu -- output-sharded layers across the GPUs of one node.
//
// A layer whose output rows are split over P GPUs needs every rank to end up
// with the whole (M, N) output.  Instead of a separate all-gather, the GEMM's
// epilogue stores each output value into the full-output buffer of every GPU
// (peer memory over NVLink, plain stores), and a one-warp cross-GPU barrier
// after the GEMM tells each rank that all shards have landed.  The buffers
// are ordinary cudaMalloc memory (e.g. PyTorch tensors) shared through CUDA
// IPC handles.
#include "pn_common.cuh"
#include "pn_internal.h"

namespace pn {

// Cross-GPU barrier.  Rank r writes the new generation into slot r of every
// rank's flag array (system-scope release), then waits until every slot of
// its own array holds at least that generation (system-scope acquire).  The
// generation counter lives in device memory, so a captured CUDA graph replays
// correctly.  Waits are bounded (wait_ns of the global nanosecond timer): on
// timeout the device status word records PN_ERR_TIMEOUT and the kernel
// returns.  After a timeout the ranks' generations are out of step; every
// rank must then re-zero its flag array and generation (with no barrier in
// flight anywhere) before the next barrier.
struct PeerFlags {
    int* flags[8];  // flags[r] = rank r's array of `world` ints (peer pointers)
};

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(PeerFlags f, int world, int rank, int* gen,
                                                          uint64_t wait_ns) {
    // The next product's pre-pass (a programmatic dependent) may be scheduled
    // during the exchange: it waits for this grid's completion before it
    // touches memory, and the GEMM after it starts streaming weights.
    asm volatile("griddepcontrol.launch_dependents;");
    // This kernel is itself a programmatic dependent of the GEMM before it
    // (so that the chain GEMM -> barrier -> next pre-pass -> next GEMM can
    // overlap the next GEMM's prologue with this one's tail): nothing is
    // posted before that grid has completed and its stores are visible.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x;
    int g = 0;
    if (lane == 0) {
        g = *gen + 1;
        *gen = g;
    }
    g = __shfl_sync(0xffffffffu, g, 0);
    if (lane < world) {
        // everything this GPU wrote before (the GEMM's peer stores) is
        // visible system-wide before the flag
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f.flags[lane] + rank), "r"(g) : "memory");
    }
    if (lane < world) {
        const int* mine = f.flags[rank] + lane;
        const uint64_t t0 = global_ns();
        while (true) {
            int v;
            asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if (v - g >= 0) break;
            if (global_ns() - t0 > wait_ns) {
                record_status(PN_ERR_TIMEOUT);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();
}

}  // namespace pn

namespace {
// Default wait of the cross-GPU barrier: long enough for any product the
// ranks run between two barriers, short enough that a missing rank surfaces
// as PN_ERR_TIMEOUT within seconds.
constexpr uint64_t kPeerWaitDefaultNs = 2000000000ull;

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
GetAddressRangeFn address_range_fn() {
    static GetAddressRangeFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<GetAddressRangeFn>(f);
    }();
    return fn;
}
}  // namespace

// IPC handles name whole allocations; *offset_out is ptr's offset inside its
// allocation (so buffers carved out of a larger allocation, e.g. by PyTorch's
// caching allocator, can be shared too).
extern "C" int pn_ipc_handle(const void* ptr, void* handle_out, size_t* offset_out) {
    if (!ptr || !handle_out || !offset_out) return fail(PN_ERR_ARG, "pn_ipc_handle: null pointer");
    GetAddressRangeFn range = address_range_fn();
    if (!range) return fail(PN_ERR_CUDA, "pn_ipc_handle: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t bytes = 0;
    if (range(&base, &bytes, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return fail(PN_ERR_ARG, "pn_ipc_handle: not a device allocation");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_fail(e, "pn_ipc_handle");
    std::memcpy(handle_out, &h, sizeof(h));
    *offset_out = (size_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return ok();
}

extern "C" int pn_ipc_open(const void* handle, void** ptr_out) {
    if (!handle || !ptr_out) return fail(PN_ERR_ARG, "pn_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_ipc_open");
}

extern "C" int pn_ipc_close(void* ptr) {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_ipc_close");
}

extern "C" int pn_peer_barrier(int* const* flags, int world, int rank, int* gen, void* stream) {
    return pn_peer_barrier_wait(flags, world, rank, gen, 0, stream);
}

extern "C" int pn_peer_barrier_wait(int* const* flags, int world, int rank, int* gen, int64_t wait_ns,
                                    void* stream) {
    if (wait_ns < 0) return fail(PN_ERR_ARG, "pn_peer_barrier_wait: wait_ns=%lld", (long long)wait_ns);
    const uint64_t limit = wait_ns == 0 ? kPeerWaitDefaultNs : (uint64_t)wait_ns;
    if (world < 1 || world > 8 || rank < 0 || rank >= world || !flags || !gen)
        return fail(PN_ERR_ARG, "pn_peer_barrier: world=%d rank=%d", world, rank);
    pn::PeerFlags f{};
    for (int r = 0; r < world; ++r) {
        if (!flags[r] || !aligned(flags[r], 4)) return fail(PN_ERR_ARG, "pn_peer_barrier: flag array %d", r);
        f.flags[r] = flags[r];
    }
    if (int st = check_device()) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, pn::peer_barrier_kernel, f, world, rank, gen, limit);
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_peer_barrier");
}

extern "C" int pn_linear_bf16_peers(const void* x, int64_t M, int64_t K, const int32_t* packed, int64_t N,
                                    int64_t K_packs, float scale, const void* bias, void* const* y_peers,
                                    int n_peers, int64_t ld_y, int64_t y_col0, int y_dtype, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (n_peers < 1 || n_peers > 8 || !y_peers) return fail(PN_ERR_ARG, "pn_linear_bf16_peers: n_peers=%d", n_peers);
    if (y_dtype != PN_BF16 && y_dtype != PN_F32) return fail(PN_ERR_DTYPE, "pn_linear_bf16_peers: y_dtype %d", y_dtype);
    if (y_col0 < 0 || ld_y < y_col0 + N)
        return fail(PN_ERR_SHAPE, "pn_linear_bf16_peers: ld_y=%lld y_col0=%lld N=%lld", (long long)ld_y,
                    (long long)y_col0, (long long)N);
    for (int r = 0; r < n_peers; ++r)
        if (!y_peers[r] || !aligned(y_peers[r], y_dtype == PN_F32 ? 4 : 2))
            return fail(PN_ERR_ALIGN, "pn_linear_bf16_peers: output %d", r);
    if (M > 64 && (K % 8 != 0 || !aligned(x, 16)))
        return fail(PN_ERR_UNSUPPORTED, "pn_linear_bf16_peers: M > 64 needs K %% 8 == 0 and 16-byte aligned x");
    return linear_bf16_impl(x, M, K, packed, N, K_packs, K_packs, scale, bias, nullptr, 0, PN_ACT_NONE, nullptr,
                            y_dtype, workspace, workspace_bytes, stream, y_peers, n_peers, ld_y, y_col0,
                            "pn_linear_bf16_peers");
}
