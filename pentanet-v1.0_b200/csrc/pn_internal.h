// pn_internal.h -- launchers shared between the kernel files and the C ABI.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace pn {

size_t absmean_workspace_bytes();
cudaError_t launch_absmean(const void* w, int dtype, int64_t n, float* d_scale, void* ws, cudaStream_t s);
cudaError_t launch_quantize_pack(const void* w, int dtype, int64_t N, int64_t K, const float* d_scale,
                                 int32_t* packed, int qmax, cudaStream_t s);
cudaError_t launch_unpack(const int32_t* packed, int64_t N, int64_t KP, int64_t K, int8_t* out, cudaStream_t s);

int64_t act_i8_pitch(int64_t K);
cudaError_t launch_quant_act_i8(const void* x, int x_dtype, int64_t M, int64_t K, int8_t* xq, int64_t pitch,
                                float* s_x, int32_t* rowsum, cudaStream_t s);

// LayerNorm over the last dimension (C) of M rows; w, b: NULL or C fp32 values.
cudaError_t launch_layer_norm(const void* x, int x_dtype, int64_t M, int64_t C, const float* w, const float* b,
                              float eps, void* y, int y_dtype, cudaStream_t s);

// Fused dequant-matmul on the tensor cores (tcgen05, A operand in TMEM).
struct LinearArgs {
    int kind;                 // PN_BF16 (kind::f16) or PN_I8 (kind::i8)
    const void* x;            // bf16 X (M, K) or int8 Xq (M, pitch)
    int64_t x_pitch;          // elements per X row
    int64_t M, K, N, KP;
    const int32_t* packed;
    int64_t packed_ld;        // int32 words between packed rows (>= KP)
    float scale;
    const void* bias;         // bf16 (N) or null
    const void* residual;     // bf16 (M, ld_res) added after the activation, or null
    int64_t ld_res;
    int act;                  // PN_ACT_NONE / PN_ACT_GELU
    void* y;                  // (M, N) or null (int8 path only)
    int y_dtype;              // PN_BF16 / PN_F32
    // Output-sharded layers: when n_peers > 0 the outputs go to every buffer
    // in y_peers (this GPU's and its peers', row stride ld_y elements, this
    // shard's columns starting at y_col0) instead of y.
    void* y_peers[8];
    int n_peers;
    int64_t ld_y, y_col0;
    int32_t* acc_out;         // int8 path: (M, N) int32 or null
    const float* s_x;         // int8 path
    const int32_t* rowsum;    // int8 path
    void* workspace;
    size_t workspace_bytes;
};
// Workspace that lets tiles split across SMs (recommended), and the least the
// kernel runs with (whole tiles per SM), for packed rows packed_ld words apart
// (a re-pitched copy of the weights is included when packed_ld % 4 != 0).
size_t linear_workspace_bytes(int kind, int64_t M, int64_t N, int64_t K, int64_t packed_ld);
size_t linear_workspace_min_bytes(int kind, int64_t M, int64_t N, int64_t K, int64_t packed_ld);
// Returns a pn_status_code; CUDA errors are reported through *cuda_err.
int launch_linear(const LinearArgs& a, cudaStream_t s, cudaError_t* cuda_err, const char** why);

// CUDA-core path for shapes the tensor-core kernel does not take (bf16 X whose
// row pitch is not a multiple of 16 elements).
cudaError_t launch_linear_simt_bf16(const LinearArgs& a, cudaStream_t s);

int device_sm_count();

// Limb decode (bf16 products of at most l8_max_tokens() tokens, 0..16) on the
// kind::i8 tensor cores; set_l8_max_tokens clamps to that range.
int l8_max_tokens();
void set_l8_max_tokens(int m);

// CUDA-core decode GEMV (pn_gemv.cu) for bf16 products of at most
// gemv_max_tokens() tokens (settable up to kGemvMaxTokens) whose packed rows
// sit at a 16-byte pitch; its workspace is gemv_workspace_bytes(M, N, KP).
constexpr int kGemvMaxTokens = 8;
constexpr int kGemvMaxTokensDefault = 0;
int gemv_max_tokens();
void set_gemv_max_tokens(int m);
size_t gemv_workspace_bytes(int64_t M, int64_t N, int64_t KP);
bool gemv_takes(const LinearArgs& a);
cudaError_t launch_gemv(const LinearArgs& a, cudaStream_t s);

}  // namespace pn
