/*
 * pentanet_b200.h -- C ABI of the B200 (sm_100a) PentaNet packed-weight path.
 *
 * Plain pointers and sizes only.  Every function returns an int status
 * (PN_OK = 0).  All device pointers are caller-allocated; no entry point
 * allocates memory.  Work is enqueued on the given CUDA stream (a cudaStream_t
 * passed as void*, NULL = legacy default stream) and is asynchronous to the
 * host unless stated otherwise.
 *
 * Packed weight format (penta_kernel.py:7-20, identical bytes): an (N, K_packs)
 * row-major int32 array, K_packs = ceil(K/10); weight k = 10g+i of row n is the
 * 3-bit code q+2 (q in {-2..2}) in bits [3i+2:3i] of word (n, g); bits 31:30
 * are zero; K is padded with code 2.
 */
#ifndef PENTANET_B200_H
#define PENTANET_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum pn_status_code {
    PN_OK = 0,
    PN_ERR_ARG = 1,         /* null pointer / invalid enum                     */
    PN_ERR_SHAPE = 2,       /* dimension out of range or inconsistent          */
    PN_ERR_ALIGN = 3,       /* pointer or row pitch not aligned as required    */
    PN_ERR_DTYPE = 4,       /* unsupported element type                        */
    PN_ERR_CUDA = 5,        /* a CUDA runtime/driver call failed               */
    PN_ERR_UNSUPPORTED = 6, /* device is not sm_100                            */
    PN_ERR_TIMEOUT = 7,     /* a kernel gave up on a bounded wait (device side)*/
    PN_ERR_WORKSPACE = 8    /* workspace missing or too small                  */
};

/* ---- element types -------------------------------------------------------- */
enum pn_dtype { PN_F32 = 0, PN_BF16 = 1, PN_I8 = 2, PN_I32 = 3 };

/* Activation fused into a product's epilogue (pn_linear_bf16_epi / _i8_epi). */
enum pn_act_code { PN_ACT_NONE = 0, PN_ACT_GELU = 1 };

/* ABI version of this header (bumped on any signature change). */
int pn_abi_version(void);
/* Static text for a status code. */
const char *pn_status_string(int status);
/* Message of the last failing call on this host thread ("" if none). */
const char *pn_last_error(void);
/* Device-side status word of the current device: a kernel that abandons a
 * bounded wait records PN_ERR_TIMEOUT there.  Synchronises the device.  When
 * reset != 0 the word is cleared after reading. */
int pn_device_status(int reset, int *status_out);

/* ---- packing: replaces quantize_and_pack (penta_kernel.py:42-78) ---------- */

/* Bytes of workspace pn_absmean_scale needs. */
size_t pn_absmean_workspace_size(void);

/* gamma = max(mean|W|, 1e-8) as a float written to d_scale (device pointer):
 * penta_kernel.py:57.  W has n_elems elements of w_dtype (PN_F32 or PN_BF16).
 * The sum of |W| is accumulated in double in a fixed order, so the result is
 * deterministic.
 * Stated deviation: gamma is the correctly rounded mean (double sum, one
 * rounding to float).  The reference's torch fp32 CPU mean is not always
 * correctly rounded; in 10 of the 17 reference fixtures the two differ by one
 * float ulp.  The packed bytes were identical in every fixture.  A W/gamma
 * quotient lying within about one ulp of a half-integer could round the
 * other way under the reference's gamma.  Callers that must reproduce the
 * reference's gamma exactly pass their own scale to pn_quantize_pack
 * (quantize_and_pack(w, scale=...)). */
int pn_absmean_scale(const void *w, int w_dtype, int64_t n_elems, float *d_scale, void *workspace,
                     size_t workspace_bytes, void *stream);

/* Quantise with the device-resident scale and pack (penta_kernel.py:60-78):
 * q = clamp(round_half_even(W / gamma), -2, 2) with IEEE float division,
 * code = q + 2, ten codes per word, K padded with code 2.  W is (N, K)
 * row-major, packed is (N, ceil(K/10)) int32. */
int pn_quantize_pack(const void *w, int w_dtype, int64_t N, int64_t K, const float *d_scale,
                     int32_t *packed, void *stream);

/* The ternary (BitNet) rule of the reference's QuantLinear(mode='bitnet')
 * (train_pentagpt.py:33-36): q = clamp(round_half_even(W / gamma), -1, 1)
 * with the same absmean gamma, stored in the same 3-bit codes (q + 2), so
 * every product entry point runs ternary layers unchanged. */
int pn_quantize_pack_ternary(const void *w, int w_dtype, int64_t N, int64_t K, const float *d_scale,
                             int32_t *packed, void *stream);

/* ---- unpack: replaces unpack_weights (penta_kernel.py:81-90) and the C
 *      penta_unpack_3bit (penta_avx2.c:41-59) ------------------------------- */

/* out[n, k] = ((packed[n, k/10] >> 3*(k%10)) & 7) - 2 as int8, k < K_orig. */
int pn_unpack(const int32_t *packed, int64_t N, int64_t K_packs, int64_t K_orig, int8_t *out, void *stream);

/* ---- ternary weights in 2 bits (no counterpart in the reference's packed
 *      format; the rule is QuantLinear's bitnet mode, train_pentagpt.py:33-36).
 * Sixteen codes per int32, code = q + 1 in {0, 1, 2} at bits 2j..2j+1 for
 * k = 16g + j of word g, rows of pn_words_2bit(K) = ceil(K/16) words,
 * padding code 1 (q = 0); q = clamp(round_half_even(w / gamma), -1, 1) with
 * gamma from pn_absmean_scale (device pointer), rounded as pn_quantize_pack.
 * pn_linear_bf16_2bit: y = x . q^T * scale (+ bias) with fp32 sums and the
 * output rounding of pn_linear_bf16, on CUDA cores (a format path: 2 bits
 * per weight read, not tuned); a code 3 reads as q = 2. */
int64_t pn_words_2bit(int64_t K);
int pn_quantize_pack_2bit(const void *w, int w_dtype, int64_t N, int64_t K, const float *d_scale, int32_t *packed,
                          void *stream);
int pn_unpack_2bit(const int32_t *packed, int64_t N, int64_t K_words, int64_t K_orig, int8_t *out, void *stream);
int pn_linear_bf16_2bit(const void *x, int64_t M, int64_t K, const int32_t *packed, int64_t N, int64_t K_words,
                        float scale, const void *bias, void *y, int y_dtype, void *stream);

/* The reference's CPU matmul on the GPU: out (M, N) fp32 = scale * x . w^T
 * for fp32 x (M, K) and unpacked int8 weights w (N, K) in {-2..+2} (from
 * pn_unpack), both row-major contiguous; replaces penta_matmul_avx2
 * (penta_avx2.c:87-95, bound by penta_avx2_wrapper.py:27-34) with the same
 * argument order plus a stream and a status.  fp32 sums of exact products,
 * multiplied by scale once; within fp32 rounding of the reference's result
 * (the summation order differs).  Reads 8 bits per weight: the packed
 * entry points below are the fast path. */
int pn_matmul_i8w(const float *x, const int8_t *w, float *out, int64_t M, int64_t N, int64_t K, float scale,
                  void *stream);

/* ---- fused dequant-matmul: replaces penta_linear / _penta_matmul_kernel
 *      (penta_kernel.py:111-278) ------------------------------------------- */

/* bf16 products of at most this many tokens (0..8; default 0) whose packed
 * rows sit at a 16-byte pitch run on the CUDA-core decode GEMV (fp32 FMAs of
 * the masked codes, no tensor cores); larger ones on the tensor-core kernel.
 * Both compute the same fp32-accumulated product (results may differ in the
 * last bf16 bit, the summation order being different).  Sets the limit when
 * max_tokens >= 0 and returns the previous one.  Process-wide.  No
 * counterpart in the reference. */
int pn_set_gemv_max_tokens(int max_tokens);

/* bf16 products of at most this many tokens (0..16; default 2) with
 * K <= 65536 run on the limb decode kernel: each token's activations become
 * 32-bit fixed-point integers (x within 2^-25 max|x| of itself, exact for
 * every element within a factor 2^17 of the row's largest), split into four
 * int8 limbs, and the packed codes meet them in kind::i8 MMAs whose int32
 * sums combine exactly; one fp32 rounding at the end.  Larger batches use the kind::f16 kernel
 * (bf16 products accumulated in fp32).  A token holding an inf or NaN gives
 * NaN outputs on the limb path.  Sets the limit when max_tokens >= 0 and
 * returns the previous one.  Process-wide.  No counterpart in the
 * reference. */
int pn_set_limb_max_tokens(int max_tokens);

/* Recommended workspace bytes for pn_linear_bf16 / pn_linear_i8 at this shape
 * (0 allowed when the result is 0).  kind: PN_BF16 or PN_I8.  With this much
 * the kernel may split one output tile's K range over several SMs when there
 * are few tiles per SM (the partial sums live in the workspace).  A smaller
 * workspace is accepted down to pn_linear_workspace_min_size; the call then
 * gives each SM whole tiles. */
size_t pn_linear_workspace_size(int kind, int64_t M, int64_t N, int64_t K);

/* The least workspace pn_linear_bf16 / pn_linear_i8 accept at this shape
 * (whole output tiles per SM).  No reference counterpart. */
size_t pn_linear_workspace_min_size(int kind, int64_t M, int64_t N, int64_t K);

/* Y[M, N] = (X[M, K] . unpack(packed)^T) * scale (+ bias), fp32 accumulation.
 * X: bf16 row-major (row pitch K elements).  packed: (N, K_packs) int32,
 * 16-byte aligned.
 * bias: NULL or N bf16 values.  y_dtype PN_BF16 reproduces the reference's
 * rounding (bf16(acc*scale), then bf16(. + bf16(bias)), penta_kernel.py:224,
 * :275-276); PN_F32 returns the unrounded fp32 value acc*scale + bias.
 * Workspace: pn_linear_workspace_size(PN_BF16, M, N, K) bytes, 256-byte
 * aligned, contents need no initialisation (each call sets what it reads, on
 * its stream).  It holds the activations re-laid out for the decode kernel
 * (M <= 64), a copy of the packed rows at a 16-byte pitch when
 * K_packs % 4 != 0, and the partial sums of split tiles. */
int pn_linear_bf16(const void *x, int64_t M, int64_t K, const int32_t *packed, int64_t N, int64_t K_packs,
                   float scale, const void *bias, void *y, int y_dtype, void *workspace,
                   size_t workspace_bytes, void *stream);

/* pn_linear_bf16 with the packed rows packed_ld int32 words apart
 * (packed_ld >= K_packs; the (N, K_packs) tensor may be a view of a wider
 * buffer).  With packed_ld % 4 == 0 the rows are 16 bytes apart and are read
 * in place; pn_linear_bf16 (packed_ld = K_packs) otherwise copies them into the
 * workspace at a 16-byte pitch on every call, so callers that keep weights
 * resident store them at pn_packed_ld(K_packs).  Replaces penta_linear
 * (penta_kernel.py:229-278) for such stored weights. */
int pn_linear_bf16_ld(const void *x, int64_t M, int64_t K, const int32_t *packed, int64_t N, int64_t K_packs,
                      int64_t packed_ld, float scale, const void *bias, void *y, int y_dtype, void *workspace,
                      size_t workspace_bytes, void *stream);

/* pn_linear_bf16_ld with the elementwise ops that follow a projection in the
 * reference's GPT block fused into the epilogue, each rounded to bf16 as the
 * separate torch ops round it (fp32 output: no intermediate rounding):
 *   t = bf16(acc * scale); t = bf16(t + bf16(bias))       (bias != NULL)
 *   t = bf16(gelu(t))      (act == PN_ACT_GELU; erf form, nn.GELU(),
 *                           train_pentagpt.py:80,86)
 *   y = bf16(residual + t) (residual != NULL; x + attn(..) / x + mlp(..),
 *                           train_pentagpt.py:100-101)
 * residual: NULL or (M, ld_res) bf16, ld_res >= N; it may be y itself (then
 * ld_res == N), each element being read before its output is written.  No
 * reference counterpart: the reference runs these as separate torch ops. */
int pn_linear_bf16_epi(const void *x, int64_t M, int64_t K, const int32_t *packed, int64_t N, int64_t K_packs,
                       int64_t packed_ld, float scale, const void *bias, int act, const void *residual,
                       int64_t ld_res, void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                       void *stream);

/* The packed row stride (int32 words) that lets the GEMM read weights in
 * place: K_packs rounded up to a multiple of 4. */
int64_t pn_packed_ld(int64_t K_packs);

/* pn_linear_bf16_ld without a workspace argument, for callers that cannot
 * allocate device memory (code where no allocator may run, or embeddings that
 * hand the library only raw input/output pointers).  No counterpart in the
 * reference (its wrapper allocates with torch.empty, penta_kernel.py:259).
 * Scratch comes from one static 4 MiB device array per GPU (held until the
 * process exits).  A call needs the decode activation slab for M <= 64
 * (3.7 MB at K = 28672 and 64 tokens) plus, when packed_ld % 4 != 0, a
 * 16-byte-pitch copy of the weights (N * pn_packed_ld(K_packs) * 4 bytes,
 * beyond the array for most layers): store the rows at pn_packed_ld(K_packs).
 * Shapes needing more return PN_ERR_WORKSPACE before anything is enqueued.
 * Calls that overlap on the GPU share the array and race: serialise them.
 * The first call on a device looks up the array's address; make it before
 * any stream capture, and do not use this entry point across a
 * cudaDeviceReset.  Allocates and frees nothing. */
int pn_linear_bf16_nows(const void *x, int64_t M, int64_t K, const int32_t *packed, int64_t N, int64_t K_packs,
                        int64_t packed_ld, float scale, const void *bias, void *y, int y_dtype, void *stream);

/* ---- int8 activation path: replaces the int8 line of the reference
 *      benchmark (penta_avx2_wrapper.py:130-131,137,147), per token --------- */

/* Row pitch (bytes) of the quantised-activation buffer for a given K. */
int64_t pn_act_i8_pitch(int64_t K);

/* Per-token absmax int8 quantiser: s_x[m] = max|X[m,:]| / 127 (1 for an
 * all-zero row), xq = clamp(round_half_even(X / s_x), -128, 127).  xq is
 * (M, pitch) int8 with pitch = pn_act_i8_pitch(K); bytes k >= K are written
 * as 0.  rowsum[m] = sum_k xq[m, k] (int32).  X is bf16 or fp32 (x_dtype). */
int pn_quant_act_i8(const void *x, int x_dtype, int64_t M, int64_t K, int8_t *xq, int64_t xq_pitch, float *s_x,
                    int32_t *rowsum, void *stream);

/* acc[m, n] = sum_k xq[m, k] * w[n, k] (exact int32, = torch._int_mm(xq, w^T));
 * Y = float(acc) * float(scale * s_x[m]) (+ bias).  acc_out: NULL or (M, N)
 * int32 to receive the accumulators.  y: NULL or (M, N) of y_dtype
 * (PN_BF16 / PN_F32).  xq/s_x/rowsum as produced by pn_quant_act_i8. */
int pn_linear_i8(const int8_t *xq, int64_t xq_pitch, const float *s_x, const int32_t *rowsum, int64_t M,
                 int64_t K, const int32_t *packed, int64_t N, int64_t K_packs, float scale, const void *bias,
                 void *y, int y_dtype, int32_t *acc_out, void *workspace, size_t workspace_bytes,
                 void *stream);

/* pn_linear_i8 with the packed rows packed_ld int32 words apart (as
 * pn_linear_bf16_ld). */
int pn_linear_i8_ld(const int8_t *xq, int64_t xq_pitch, const float *s_x, const int32_t *rowsum, int64_t M,
                    int64_t K, const int32_t *packed, int64_t N, int64_t K_packs, int64_t packed_ld, float scale,
                    const void *bias, void *y, int y_dtype, int32_t *acc_out, void *workspace,
                    size_t workspace_bytes, void *stream);

/* pn_linear_i8_ld with the fused epilogue ops of pn_linear_bf16_epi (y must
 * not be NULL when act or residual is given). */
int pn_linear_i8_epi(const int8_t *xq, int64_t xq_pitch, const float *s_x, const int32_t *rowsum, int64_t M,
                     int64_t K, const int32_t *packed, int64_t N, int64_t K_packs, int64_t packed_ld, float scale,
                     const void *bias, int act, const void *residual, int64_t ld_res, void *y, int y_dtype,
                     int32_t *acc_out, void *workspace, size_t workspace_bytes, void *stream);

/* LayerNorm over the last dimension: y[m, :] = (x[m, :] - mean) *
 * rsqrt(var + eps) * weight + bias with fp32 mean and biased variance of the
 * row; x and y PN_BF16 or PN_F32 (row-major, C elements per row), weight and
 * bias NULL or C fp32 values, y rounded once.  Replaces the three kernels
 * torch runs for nn.LayerNorm under bf16 autocast in the reference GPT (fp32
 * cast, layer_norm, bf16 cast of the output; train_pentagpt.py:94-96,113,
 * 100-101,127).  In place (y == x) when the dtypes match. */
int pn_layer_norm(const void *x, int x_dtype, int64_t M, int64_t C, const float *weight, const float *bias,
                  float eps, void *y, int y_dtype, void *stream);

/* Number of SMs of the current device (used to size launches and shards). */
int pn_device_sm_count(int *count_out);

/* ---- output-sharded layers over the GPUs of one node (the reference has no
 *      multi-GPU path; replaces "GEMV + NCCL all-gather") ------------------- */

/* CUDA IPC: 64-byte handle of the allocation holding ptr (any cudaMalloc
 * memory, e.g. a PyTorch tensor) and ptr's offset in it; map / unmap a peer's
 * allocation (add the offset to the mapped base). */
int pn_ipc_handle(const void *ptr, void *handle_out, size_t *offset_out);
int pn_ipc_open(const void *handle, void **ptr_out);
int pn_ipc_close(void *ptr);

/* pn_linear_bf16 on this GPU's output rows [y_col0, y_col0 + N) of a layer,
 * storing every output into each of the n_peers (<= 8) full-output buffers
 * y_peers[r] (row stride ld_y elements; this GPU's and its peers'), so that
 * after pn_peer_barrier every GPU holds the whole output.  M > 64 requires
 * K % 8 == 0 and 16-byte aligned x. */
int pn_linear_bf16_peers(const void *x, int64_t M, int64_t K, const int32_t *packed, int64_t N,
                         int64_t K_packs, float scale, const void *bias, void *const *y_peers, int n_peers,
                         int64_t ld_y, int64_t y_col0, int y_dtype, void *workspace, size_t workspace_bytes,
                         void *stream);

/* Cross-GPU barrier on `stream`: flags[r] is rank r's array of `world` ints
 * (peer-mapped), gen this GPU's generation counter (device int, zero at
 * start).  Returns once every rank has reached the same barrier; waits are
 * bounded (PN_ERR_TIMEOUT in the device status word). */
int pn_peer_barrier(int *const *flags, int world, int rank, int *gen, void *stream);

/* pn_peer_barrier with an explicit wait limit: each rank's wait ends after
 * wait_ns nanoseconds (0 = the default of 2 s) with PN_ERR_TIMEOUT recorded
 * in the device status word, and the kernel returns.  After a timeout the
 * generations are out of step: with no barrier in flight on any rank, every
 * rank zeroes its flag array and gen before the next barrier
 * (penta_dist.PeerGroup.reset).  No counterpart in the reference, which has
 * no multi-GPU code. */
int pn_peer_barrier_wait(int *const *flags, int world, int rank, int *gen, int64_t wait_ns, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* PENTANET_B200_H */
