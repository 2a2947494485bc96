// pn_capi.cu -- the extern "C" boundary (include/pentanet_b200.h).
//
// Validates every argument on the host before anything is enqueued and turns
// failures into status codes plus a per-thread message, the C-ABI form of the
// reference's AssertionErrors (penta_kernel.py:249-257).
#include <cstdio>
#include <cstring>

#include "pn_common.cuh"
#include "pn_internal.h"

namespace {

thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}

int ok() {
    g_msg[0] = '\0';
    return PN_OK;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(PN_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

// The tensor-core kernels use sm_100a instructions (tcgen05, TMA).
int check_device() {
    static int checked[64] = {};  // 0 unknown, 1 ok, 2 unsupported
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev >= 0 && dev < 64 && checked[dev] == 1) return PN_OK;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0) {
        if (dev >= 0 && dev < 64) checked[dev] = 2;
        return fail(PN_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", dev, major, minor);
    }
    if (dev >= 0 && dev < 64) checked[dev] = 1;
    return PN_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int64_t k_packs(int64_t K) { return (K + pn::kPerWord - 1) / pn::kPerWord; }

// Fused epilogue arguments shared by the bf16 and int8 products.
int check_epilogue(const void* residual, int64_t ld_res, int act, int64_t N, const void* y, int n_peers,
                   const char* name) {
    if (act != PN_ACT_NONE && act != PN_ACT_GELU) return fail(PN_ERR_ARG, "%s: act %d", name, act);
    if (!residual) return PN_OK;
    if (n_peers > 0) return fail(PN_ERR_UNSUPPORTED, "%s: no residual for output-sharded products", name);
    if (ld_res < N) return fail(PN_ERR_SHAPE, "%s: ld_res=%lld < N=%lld", name, (long long)ld_res, (long long)N);
    if (residual == y && ld_res != N)
        return fail(PN_ERR_SHAPE, "%s: an in-place residual needs ld_res == N", name);
    if (!aligned(residual, 2)) return fail(PN_ERR_ALIGN, "%s: misaligned residual", name);
    return PN_OK;
}

}  // namespace

extern "C" {

int pn_abi_version(void) { return 1; }

const char* pn_status_string(int status) {
    switch (status) {
        case PN_OK: return "ok";
        case PN_ERR_ARG: return "invalid argument";
        case PN_ERR_SHAPE: return "invalid shape";
        case PN_ERR_ALIGN: return "misaligned pointer or pitch";
        case PN_ERR_DTYPE: return "unsupported dtype";
        case PN_ERR_CUDA: return "CUDA error";
        case PN_ERR_UNSUPPORTED: return "unsupported device";
        case PN_ERR_TIMEOUT: return "device-side wait timed out";
        case PN_ERR_WORKSPACE: return "workspace missing or too small";
        default: return "unknown status";
    }
}

const char* pn_last_error(void) { return g_msg; }

int pn_device_status(int reset, int* status_out) {
    if (!status_out) return fail(PN_ERR_ARG, "pn_device_status: status_out is NULL");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "pn_device_status: cudaDeviceSynchronize");
    int v = 0;
    e = cudaMemcpyFromSymbol(&v, pn::g_device_status, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "pn_device_status: read");
    if (reset) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(pn::g_device_status, &zero, sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e, "pn_device_status: reset");
    }
    *status_out = v;
    return ok();
}

int pn_device_sm_count(int* count_out) {
    if (!count_out) return fail(PN_ERR_ARG, "pn_device_sm_count: count_out is NULL");
    const int n = pn::device_sm_count();
    if (n <= 0) return fail(PN_ERR_CUDA, "pn_device_sm_count: no current device");
    *count_out = n;
    return ok();
}

size_t pn_absmean_workspace_size(void) { return pn::absmean_workspace_bytes(); }

int pn_absmean_scale(const void* w, int w_dtype, int64_t n_elems, float* d_scale, void* workspace,
                     size_t workspace_bytes, void* stream) {
    if (!d_scale || (!w && n_elems > 0)) return fail(PN_ERR_ARG, "pn_absmean_scale: null pointer");
    if (w_dtype != PN_F32 && w_dtype != PN_BF16) return fail(PN_ERR_DTYPE, "pn_absmean_scale: dtype %d", w_dtype);
    if (n_elems < 0) return fail(PN_ERR_SHAPE, "pn_absmean_scale: n_elems=%lld", (long long)n_elems);
    if (!workspace || workspace_bytes < pn::absmean_workspace_bytes())
        return fail(PN_ERR_WORKSPACE, "pn_absmean_scale: workspace needs %zu bytes", pn::absmean_workspace_bytes());
    if (!aligned(workspace, 8) || !aligned(w, w_dtype == PN_F32 ? 4 : 2) || !aligned(d_scale, 4))
        return fail(PN_ERR_ALIGN, "pn_absmean_scale: misaligned pointer");
    if (int st = check_device()) return st;
    cudaError_t e = pn::launch_absmean(w, w_dtype, n_elems, d_scale, workspace, (cudaStream_t)stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_absmean_scale");
}

static int quantize_pack_impl(const void* w, int w_dtype, int64_t N, int64_t K, const float* d_scale,
                              int32_t* packed, int qmax, void* stream) {
    if (!d_scale || ((!w || !packed) && N > 0)) return fail(PN_ERR_ARG, "pn_quantize_pack: null pointer");
    if (w_dtype != PN_F32 && w_dtype != PN_BF16) return fail(PN_ERR_DTYPE, "pn_quantize_pack: dtype %d", w_dtype);
    if (N < 0 || K < 1) return fail(PN_ERR_SHAPE, "pn_quantize_pack: N=%lld K=%lld", (long long)N, (long long)K);
    if (!aligned(w, w_dtype == PN_F32 ? 4 : 2) || !aligned(packed, 4) || !aligned(d_scale, 4))
        return fail(PN_ERR_ALIGN, "pn_quantize_pack: misaligned pointer");
    if (int st = check_device()) return st;
    if (N == 0) return ok();
    cudaError_t e = pn::launch_quantize_pack(w, w_dtype, N, K, d_scale, packed, qmax, (cudaStream_t)stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_quantize_pack");
}

int pn_quantize_pack(const void* w, int w_dtype, int64_t N, int64_t K, const float* d_scale, int32_t* packed,
                     void* stream) {
    return quantize_pack_impl(w, w_dtype, N, K, d_scale, packed, 2, stream);
}

int pn_quantize_pack_ternary(const void* w, int w_dtype, int64_t N, int64_t K, const float* d_scale,
                             int32_t* packed, void* stream) {
    return quantize_pack_impl(w, w_dtype, N, K, d_scale, packed, 1, stream);
}

int pn_unpack(const int32_t* packed, int64_t N, int64_t K_packs, int64_t K_orig, int8_t* out, void* stream) {
    if ((!packed || !out) && N > 0) return fail(PN_ERR_ARG, "pn_unpack: null pointer");
    if (N < 0 || K_packs < 0 || K_orig < 0 || K_orig > K_packs * pn::kPerWord)
        return fail(PN_ERR_SHAPE, "pn_unpack: N=%lld K_packs=%lld K_orig=%lld", (long long)N, (long long)K_packs,
                    (long long)K_orig);
    if (!aligned(packed, 4)) return fail(PN_ERR_ALIGN, "pn_unpack: packed not 4-byte aligned");
    if (int st = check_device()) return st;
    if (N == 0 || K_packs == 0) return ok();
    cudaError_t e = pn::launch_unpack(packed, N, K_packs, K_orig, out, (cudaStream_t)stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_unpack");
}

int pn_set_gemv_max_tokens(int max_tokens) {
    const int prev = pn::gemv_max_tokens();
    if (max_tokens >= 0) pn::set_gemv_max_tokens(max_tokens);
    return prev;
}

int pn_set_limb_max_tokens(int max_tokens) {
    const int prev = pn::l8_max_tokens();
    if (max_tokens >= 0) pn::set_l8_max_tokens(max_tokens);
    return prev;
}

size_t pn_linear_workspace_size(int kind, int64_t M, int64_t N, int64_t K) {
    return pn::linear_workspace_bytes(kind, M, N, K, k_packs(K));
}

size_t pn_linear_workspace_min_size(int kind, int64_t M, int64_t N, int64_t K) {
    return pn::linear_workspace_min_bytes(kind, M, N, K, k_packs(K));
}

}  // extern "C"

namespace {
// pn_linear_bf16 and its output-sharded form share validation and launch.
int linear_bf16_impl(const void* x, int64_t M, int64_t K, const int32_t* packed, int64_t N, int64_t K_packs,
                     int64_t packed_ld, float scale, const void* bias, const void* residual, int64_t ld_res, int act,
                     void* y, int y_dtype, void* workspace, size_t workspace_bytes, void* stream,
                     void* const* y_peers, int n_peers, int64_t ld_y, int64_t y_col0, const char* name) {
    if ((!x && M > 0) || (!packed && N > 0) || (!y && n_peers == 0 && M > 0 && N > 0))
        return fail(PN_ERR_ARG, "%s: null pointer", name);
    if (y_dtype != PN_BF16 && y_dtype != PN_F32) return fail(PN_ERR_DTYPE, "%s: y_dtype %d", name, y_dtype);
    if (M < 0 || N < 0 || K < 1 || M > 0x7fffffff || N > 0x7fffffff)
        return fail(PN_ERR_SHAPE, "%s: M=%lld N=%lld K=%lld", name, (long long)M, (long long)N, (long long)K);
    if (K_packs != k_packs(K))
        return fail(PN_ERR_SHAPE, "%s: activation K=%lld needs K_packs=%lld, got %lld", name, (long long)K,
                    (long long)k_packs(K), (long long)K_packs);
    if (packed_ld < K_packs)
        return fail(PN_ERR_SHAPE, "%s: packed_ld=%lld < K_packs=%lld", name, (long long)packed_ld, (long long)K_packs);
    if (!aligned(x, 2) || !aligned(packed, 16) || !aligned(y, y_dtype == PN_F32 ? 4 : 2) || !aligned(bias, 2))
        return fail(PN_ERR_ALIGN, "%s: misaligned pointer (packed weights need 16-byte alignment)", name);
    if (int st = check_epilogue(residual, ld_res, act, N, y, n_peers, name)) return st;
    const size_t need = pn::linear_workspace_min_bytes(PN_BF16, M, N, K, packed_ld);
    if (need > 0 && (!workspace || workspace_bytes < need))
        return fail(PN_ERR_WORKSPACE, "%s: workspace needs at least %zu bytes (%zu recommended)", name, need,
                    pn::linear_workspace_bytes(PN_BF16, M, N, K, packed_ld));
    if (int st = check_device()) return st;
    if (M == 0 || N == 0) return ok();
    pn::LinearArgs a{};
    a.kind = PN_BF16;
    a.x = x;
    a.x_pitch = K;
    a.M = M;
    a.K = K;
    a.N = N;
    a.KP = K_packs;
    a.packed = packed;
    a.packed_ld = packed_ld;
    a.scale = scale;
    a.bias = bias;
    a.residual = residual;
    a.ld_res = ld_res;
    a.act = act;
    a.y = y;
    a.y_dtype = y_dtype;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes;
    a.n_peers = n_peers;
    for (int r = 0; r < n_peers && r < 8; ++r) a.y_peers[r] = y_peers[r];
    a.ld_y = ld_y;
    a.y_col0 = y_col0;
    // Decode-sized M reads x with plain loads (any K); larger M loads it by TMA,
    // which needs 16-byte rows.
    if (M > 64 && (K % 8 != 0 || !aligned(x, 16))) {
        cudaError_t e = pn::launch_linear_simt_bf16(a, (cudaStream_t)stream);
        return e == cudaSuccess ? ok() : cuda_fail(e, "pn_linear_bf16 (cuda-core)");
    }
    if (pn::gemv_takes(a)) {
        cudaError_t e = pn::launch_gemv(a, (cudaStream_t)stream);
        return e == cudaSuccess ? ok() : cuda_fail(e, "pn_linear_bf16 (decode GEMV)");
    }
    cudaError_t ce;
    const char* why;
    const int st = pn::launch_linear(a, (cudaStream_t)stream, &ce, &why);
    if (st == PN_ERR_CUDA) return cuda_fail(ce, why);
    if (st != PN_OK) return fail(st, "%s: %s", name, why);
    return ok();
}
}  // namespace

extern "C" {

int pn_linear_bf16(const void* x, int64_t M, int64_t K, const int32_t* packed, int64_t N, int64_t K_packs,
                   float scale, const void* bias, void* y, int y_dtype, void* workspace, size_t workspace_bytes,
                   void* stream) {
    return linear_bf16_impl(x, M, K, packed, N, K_packs, K_packs, scale, bias, nullptr, 0, PN_ACT_NONE, y, y_dtype,
                            workspace, workspace_bytes, stream, nullptr, 0, 0, 0, "pn_linear_bf16");
}

int64_t pn_packed_ld(int64_t K_packs) { return K_packs <= 0 ? 0 : (K_packs + 3) / 4 * 4; }

int pn_linear_bf16_ld(const void* x, int64_t M, int64_t K, const int32_t* packed, int64_t N, int64_t K_packs,
                      int64_t packed_ld, float scale, const void* bias, void* y, int y_dtype, void* workspace,
                      size_t workspace_bytes, void* stream) {
    return linear_bf16_impl(x, M, K, packed, N, K_packs, packed_ld, scale, bias, nullptr, 0, PN_ACT_NONE, y, y_dtype,
                            workspace, workspace_bytes, stream, nullptr, 0, 0, 0, "pn_linear_bf16_ld");
}

int pn_linear_bf16_epi(const void* x, int64_t M, int64_t K, const int32_t* packed, int64_t N, int64_t K_packs,
                       int64_t packed_ld, float scale, const void* bias, int act, const void* residual,
                       int64_t ld_res, void* y, int y_dtype, void* workspace, size_t workspace_bytes, void* stream) {
    return linear_bf16_impl(x, M, K, packed, N, K_packs, packed_ld, scale, bias, residual, ld_res, act, y, y_dtype,
                            workspace, workspace_bytes, stream, nullptr, 0, 0, 0, "pn_linear_bf16_epi");
}

int pn_layer_norm(const void* x, int x_dtype, int64_t M, int64_t C, const float* weight, const float* bias, float eps,
                  void* y, int y_dtype, void* stream) {
    if (M > 0 && (!x || !y)) return fail(PN_ERR_ARG, "pn_layer_norm: null pointer");
    if ((x_dtype != PN_F32 && x_dtype != PN_BF16) || (y_dtype != PN_F32 && y_dtype != PN_BF16))
        return fail(PN_ERR_DTYPE, "pn_layer_norm: x_dtype %d y_dtype %d", x_dtype, y_dtype);
    if (M < 0 || C < 1 || C > 0x7fffffff || !(eps >= 0.0f))
        return fail(PN_ERR_SHAPE, "pn_layer_norm: M=%lld C=%lld eps=%g", (long long)M, (long long)C, (double)eps);
    if (!aligned(x, x_dtype == PN_F32 ? 4 : 2) || !aligned(y, y_dtype == PN_F32 ? 4 : 2) || !aligned(weight, 4) ||
        !aligned(bias, 4))
        return fail(PN_ERR_ALIGN, "pn_layer_norm: misaligned pointer");
    if (x == y && x_dtype != y_dtype) return fail(PN_ERR_ARG, "pn_layer_norm: in place needs x_dtype == y_dtype");
    if (int st = check_device()) return st;
    cudaError_t e = pn::launch_layer_norm(x, x_dtype, M, C, weight, bias, eps, y, y_dtype, (cudaStream_t)stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_layer_norm");
}

int64_t pn_act_i8_pitch(int64_t K) { return pn::act_i8_pitch(K); }

int pn_quant_act_i8(const void* x, int x_dtype, int64_t M, int64_t K, int8_t* xq, int64_t xq_pitch, float* s_x,
                    int32_t* rowsum, void* stream) {
    if (M > 0 && (!x || !xq || !s_x || !rowsum)) return fail(PN_ERR_ARG, "pn_quant_act_i8: null pointer");
    if (x_dtype != PN_F32 && x_dtype != PN_BF16) return fail(PN_ERR_DTYPE, "pn_quant_act_i8: dtype %d", x_dtype);
    if (M < 0 || K < 1 || M > 0x7fffffff || xq_pitch < K || xq_pitch % 16 != 0)
        return fail(PN_ERR_SHAPE, "pn_quant_act_i8: M=%lld K=%lld pitch=%lld (pitch must be >= K, multiple of 16)",
                    (long long)M, (long long)K, (long long)xq_pitch);
    if (!aligned(x, x_dtype == PN_F32 ? 4 : 2) || !aligned(xq, 16) || !aligned(s_x, 4) || !aligned(rowsum, 4))
        return fail(PN_ERR_ALIGN, "pn_quant_act_i8: misaligned pointer");
    if (int st = check_device()) return st;
    cudaError_t e = pn::launch_quant_act_i8(x, x_dtype, M, K, xq, xq_pitch, s_x, rowsum, (cudaStream_t)stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "pn_quant_act_i8");
}

static int linear_i8_impl(const int8_t* xq, int64_t xq_pitch, const float* s_x, const int32_t* rowsum, int64_t M,
                          int64_t K, const int32_t* packed, int64_t N, int64_t K_packs, int64_t packed_ld, float scale,
                          const void* bias, const void* residual, int64_t ld_res, int act, void* y, int y_dtype,
                          int32_t* acc_out, void* workspace, size_t workspace_bytes, void* stream) {
    if (M > 0 && N > 0 && (!xq || !s_x || !rowsum || !packed || (!y && !acc_out)))
        return fail(PN_ERR_ARG, "pn_linear_i8: null pointer");
    if (y && y_dtype != PN_BF16 && y_dtype != PN_F32) return fail(PN_ERR_DTYPE, "pn_linear_i8: y_dtype %d", y_dtype);
    if (M < 0 || N < 0 || K < 1 || M > 0x7fffffff || N > 0x7fffffff || xq_pitch < K || xq_pitch % 16 != 0)
        return fail(PN_ERR_SHAPE, "pn_linear_i8: M=%lld N=%lld K=%lld pitch=%lld", (long long)M, (long long)N,
                    (long long)K, (long long)xq_pitch);
    if (K_packs != k_packs(K))
        return fail(PN_ERR_SHAPE, "pn_linear_i8: K=%lld needs K_packs=%lld, got %lld", (long long)K,
                    (long long)k_packs(K), (long long)K_packs);
    if (packed_ld < K_packs)
        return fail(PN_ERR_SHAPE, "pn_linear_i8: packed_ld=%lld < K_packs=%lld", (long long)packed_ld,
                    (long long)K_packs);
    if (!aligned(xq, 16) || !aligned(packed, 16) || !aligned(s_x, 4) || !aligned(rowsum, 4) || !aligned(acc_out, 4) ||
        !aligned(y, y_dtype == PN_F32 ? 4 : 2) || !aligned(bias, 2))
        return fail(PN_ERR_ALIGN, "pn_linear_i8: misaligned pointer");
    if ((residual || act != PN_ACT_NONE) && !y) return fail(PN_ERR_ARG, "pn_linear_i8: epilogue ops need y");
    if (int st = check_epilogue(residual, ld_res, act, N, y, 0, "pn_linear_i8")) return st;
    const size_t need = pn::linear_workspace_min_bytes(PN_I8, M, N, K, packed_ld);
    if (need > 0 && (!workspace || workspace_bytes < need))
        return fail(PN_ERR_WORKSPACE, "pn_linear_i8: workspace needs at least %zu bytes (%zu recommended)", need,
                    pn::linear_workspace_bytes(PN_I8, M, N, K, packed_ld));
    if (int st = check_device()) return st;
    if (M == 0 || N == 0) return ok();
    pn::LinearArgs a{};
    a.kind = PN_I8;
    a.x = xq;
    a.x_pitch = xq_pitch;
    a.M = M;
    a.K = K;
    a.N = N;
    a.KP = K_packs;
    a.packed = packed;
    a.packed_ld = packed_ld;
    a.scale = scale;
    a.bias = bias;
    a.residual = residual;
    a.ld_res = ld_res;
    a.act = act;
    a.y = y;
    a.y_dtype = y_dtype;
    a.acc_out = acc_out;
    a.s_x = s_x;
    a.rowsum = rowsum;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes;
    cudaError_t ce;
    const char* why;
    const int st = pn::launch_linear(a, (cudaStream_t)stream, &ce, &why);
    if (st == PN_ERR_CUDA) return cuda_fail(ce, why);
    if (st != PN_OK) return fail(st, "pn_linear_i8: %s", why);
    return ok();
}

int pn_linear_i8(const int8_t* xq, int64_t xq_pitch, const float* s_x, const int32_t* rowsum, int64_t M, int64_t K,
                 const int32_t* packed, int64_t N, int64_t K_packs, float scale, const void* bias, void* y,
                 int y_dtype, int32_t* acc_out, void* workspace, size_t workspace_bytes, void* stream) {
    return linear_i8_impl(xq, xq_pitch, s_x, rowsum, M, K, packed, N, K_packs, K_packs, scale, bias, nullptr, 0,
                          PN_ACT_NONE, y, y_dtype, acc_out, workspace, workspace_bytes, stream);
}

int pn_linear_i8_ld(const int8_t* xq, int64_t xq_pitch, const float* s_x, const int32_t* rowsum, int64_t M,
                    int64_t K, const int32_t* packed, int64_t N, int64_t K_packs, int64_t packed_ld, float scale,
                    const void* bias, void* y, int y_dtype, int32_t* acc_out, void* workspace,
                    size_t workspace_bytes, void* stream) {
    return linear_i8_impl(xq, xq_pitch, s_x, rowsum, M, K, packed, N, K_packs, packed_ld, scale, bias, nullptr, 0,
                          PN_ACT_NONE, y, y_dtype, acc_out, workspace, workspace_bytes, stream);
}

int pn_linear_i8_epi(const int8_t* xq, int64_t xq_pitch, const float* s_x, const int32_t* rowsum, int64_t M,
                     int64_t K, const int32_t* packed, int64_t N, int64_t K_packs, int64_t packed_ld, float scale,
                     const void* bias, int act, const void* residual, int64_t ld_res, void* y, int y_dtype,
                     int32_t* acc_out, void* workspace, size_t workspace_bytes, void* stream) {
    return linear_i8_impl(xq, xq_pitch, s_x, rowsum, M, K, packed, N, K_packs, packed_ld, scale, bias, residual, ld_res,
                          act, y, y_dtype, acc_out, workspace, workspace_bytes, stream);
}

}  // extern "C"
