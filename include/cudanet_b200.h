/* The C ABI of libcudanet_b200.so, the B200 (sm_100a) evaluator of MayFly's network.
 *
 * The first seven entry points are the reference backend's C ABI, same names, arguments, meaning and error
 * behaviour: mayfly/chess/cudanet/cudanet_capi.h:15-37 (implementation cudanet/cudanet_capi.cpp:31-124). A
 * caller of cudanet.dll (cudanet/cudanet_py.py, cudanet/cudanet_backend.cpp) binds these unchanged. Everything
 * after them is additive.
 *
 * Conventions (as in the reference): C++ exceptions never cross this boundary; a failing call returns NULL or
 * -1 and writes a NUL-terminated reason, cut to err_len bytes, into err. The caller owns every host buffer; the
 * library copies inputs into its own pinned staging and copies outputs out before returning. A handle owns
 * the weights, buffers, stream and CUDA graphs on one device. Calls on one handle are serialised by a mutex;
 * any thread may call (the device is made current on each call).
 *
 * Sizes: B positions (1..max_batch), wide legal-move slots per row (1..256). ids [B*64] piece ids 0..12 in
 * the side to move's frame, cast [B*4], hm [B] halfmove bucket 0..101, ep [B] en passant square + 1 or 0,
 * I [B*wide] policy indices 0..4161 of the legal moves, M [B*wide] nonzero on legal slots. Outputs: pol
 * [B*wide] raw policy logits at the legal moves (0 on padding), val [B] in [-1, 1], qv [B*wide] 2*sigmoid(q)-1
 * (0 on padding).
 */
#ifndef CUDANET_B200_H
#define CUDANET_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define CUDANET_API __attribute__((visibility("default")))
#else
#define CUDANET_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- the reference's ABI (cudanet_capi.h) */

/* cudanet_capi.h:16. Load a weight file (MFCNW001: version 1 with f16 matrices, or version 2 with bf16
 * matrices) onto `device`. Returns a handle, or NULL with the reason in err. The largest batch is 1024, or env
 * MAYFLY_CUDANET_MAX_BATCH (1..16384) read here. */
CUDANET_API void* cudanet_create(const char* weights_path, int device, char* err, int err_len);

/* cudanet_capi.h:20-22. One batch, synchronous. Returns 0, or -1 with the reason in err. */
CUDANET_API int cudanet_evaluate(void* handle, int B, int wide, const int64_t* ids, const float* cast,
                                 const int64_t* hm, const int64_t* ep, const int64_t* I, const uint8_t* M,
                                 float* pol, float* val, float* qv, char* err, int err_len);

/* cudanet_capi.h:25. The weight file's fingerprint (mcts_cpp.fingerprint of the model), copied into buf.
 * Returns its length, or -1 on a null handle. */
CUDANET_API int cudanet_fingerprint(void* handle, char* buf, int buf_len);

/* cudanet_capi.h:28. The largest B the handle takes, -1 on a null handle. */
CUDANET_API int cudanet_max_batch(void* handle);

/* cudanet_capi.h:32. Milliseconds a pass takes by step at batch B (the mean of reps eager passes with an
 * event after each step, every row an empty board), then last the whole pass as a CUDA graph, into ms (n
 * slots). Returns how many were written, or -1 with the reason in err. */
CUDANET_API int cudanet_profile(void* handle, int B, int reps, double* ms, int n, char* err, int err_len);

/* cudanet_capi.h:35. The step names of cudanet_profile, comma separated, copied into buf. Returns their
 * length. */
CUDANET_API int cudanet_profile_names(char* buf, int buf_len);

/* cudanet_capi.h:37. Never fails; a null handle is ignored. */
CUDANET_API void cudanet_destroy(void* handle);

/* ---------------------------------------------------------------- additive entry points */

/* cudanet_evaluate, and also the full logits [B * 2*4162] f32 (policy logits, then qvalue logits) of every
 * row, for parity tests against the reference model's raw heads. */
CUDANET_API int cudanet_evaluate_logits(void* handle, int B, int wide, const int64_t* ids, const float* cast,
                                        const int64_t* hm, const int64_t* ep, const int64_t* I,
                                        const uint8_t* M, float* pol, float* val, float* qv, float* logits,
                                        char* err, int err_len);

/* The reference CudaNet::begin / CudaNet::end pair (cudanet/cudanet.h:31-37): begin copies the inputs and
 * queues the whole pass, end waits for the oldest batch begun and copies its outputs out. At most two batches
 * are in flight. Both return 0, or -1 with the reason in err. */
CUDANET_API int cudanet_begin(void* handle, int B, int wide, const int64_t* ids, const float* cast,
                              const int64_t* hm, const int64_t* ep, const int64_t* I, const uint8_t* M,
                              char* err, int err_len);
CUDANET_API int cudanet_end(void* handle, float* pol, float* val, float* qv, char* err, int err_len);

/* Positions as transposition keys instead of encoded inputs (no counterpart in the C ABI; the reference's
 * encoder is mayfly/chess/encode.py:73-100 encode_keys, which MCTS._prepare runs on the host before
 * CudaNet.evaluate). Per board: keys[10 b .. 10 b + 9] = pawns, knights, bishops, rooks, queens, kings, white,
 * black (64-bit boards, a1 = bit 0), turn (nonzero: white to move), clean castling rights, i.e.
 * Board._transposition_key()[0:10]; ep_sq[b] the key's legal en passant square, negative for None; clock[b] the
 * halfmove clock. 96 bytes a board cross PCIe instead of 548; the GPU encodes them (encode_keys_kernel) into the
 * inputs cudanet_evaluate takes, with encode_keys' exact values, then runs the same pass. I, M and the outputs
 * are cudanet_evaluate's. Returns 0, or -1 with the reason in err. */
CUDANET_API int cudanet_evaluate_keys(void* handle, int B, int wide, const uint64_t* keys, const int64_t* ep_sq,
                                      const int64_t* clock, const int64_t* I, const uint8_t* M, float* pol,
                                      float* val, float* qv, char* err, int err_len);
/* cudanet_begin from transposition keys (finish with cudanet_end). */
CUDANET_API int cudanet_begin_keys(void* handle, int B, int wide, const uint64_t* keys, const int64_t* ep_sq,
                                   const int64_t* clock, const int64_t* I, const uint8_t* M, char* err,
                                   int err_len);
/* The encoder alone, on device memory and a caller stream (NULL: the default stream): keys, ep_sq and clock as
 * above (B boards) to ids [B * 64] int64, cast [B * 4] f32, hm [B] int64, ep [B] int64, exactly what
 * encode.py:73-100 encode_keys returns. Asynchronous on `stream`; returns 0, or -1 with the reason in err. */
CUDANET_API int cudanet_encode_keys(const uint64_t* keys, const int64_t* ep_sq, const int64_t* clock, int B,
                                    int64_t* ids, float* cast, int64_t* hm, int64_t* ep, void* stream, char* err,
                                    int err_len);

/* The arithmetic the handle runs its products in: "f16", "bf16" or "e4m3" (the layer products on e4m3
 * operands, the heads in bf16). Returns the length, -1 on a null handle. */
CUDANET_API int cudanet_precision(void* handle, char* buf, int buf_len);

/* One batch whose inputs and outputs are already in device memory of the handle's device, queued on `stream`
 * (a cudaStream_t, NULL for the legacy default stream) without waiting for it. The arrays are as for
 * cudanet_evaluate. Device-side failures (a bounded wait that timed out) are reported by the next
 * cudanet_check. Returns 0, or -1 with the reason in err. */
CUDANET_API int cudanet_evaluate_device(void* handle, int B, int wide, const int64_t* ids, const float* cast,
                                        const int64_t* hm, const int64_t* ep, const int64_t* I,
                                        const uint8_t* M, float* pol, float* val, float* qv, void* stream,
                                        char* err, int err_len);

/* Wait for the handle's work, including work queued by cudanet_evaluate_device on `stream`, and report a
 * device-side failure recorded since the last check. Returns 0, or -1 with the reason in err. */
CUDANET_API int cudanet_check(void* handle, void* stream, char* err, int err_len);

/* Runs the handle's 16-bit pass on B positions (ids, cast, hm, ep as for cudanet_evaluate) and writes, per
 * layer i, max |.| of the inputs of its four products to amax[4i + 0..3] (qkv, out, ff1, ff2): the ranges an
 * e4m3 weight file's static input scales are set from. amax holds n floats, at least 4 * layers. Returns the
 * count written, or -1 with the reason in err (also for an e4m3 handle). No counterpart in the reference,
 * whose FP8 path was a simulation (mayfly/docs/cuda_backend.md:150-152). */
CUDANET_API int cudanet_calibrate(void* handle, int B, const int64_t* ids, const float* cast, const int64_t* hm,
                                  const int64_t* ep, float* amax, int n, char* err, int err_len);

/* ---------------------------------------------------------------- single kernels, for unit tests
 * Device pointers on the current device, queued on `stream`, synchronous (the call waits for the stream).
 * dtype: 0 = f16, 1 = bf16. */

/* C = A[M, K] * W[N, K]^T + epilogue, with epi 0: C 16-bit = acc + bias; 1: C 16-bit = gelu(acc + bias);
 * 2: C f32 += acc + bias; 3: C f32 = acc + bias. C has leading dimension ldc (elements); C's row length and
 * pitch in bytes must be multiples of 16. K must be a multiple of 64 and A's, W's row pitch K elements. bn 0
 * picks the tile, 64, 128 or 256 ask for single-CTA tiles of that width, 2 for CTA-pair 256 x 256 tiles. */
CUDANET_API int cudanet_k_gemm(int dtype, int epi, int bn, const void* A, const void* W, const float* bias,
                               void* C, int M, int N, int K, int ldc, void* stream, char* err, int err_len);

/* The same product as cudanet_k_gemm, for callers that cannot call cudaMalloc (a process whose GPU memory is
 * all reserved up front, or a search thread that must not take the device-wide synchronisation an allocation
 * costs while other batches are in flight). No counterpart in the reference. It allocates nothing: its only
 * scratch, the kernel's 4-byte error word, lives in a static 256-byte device array that every GPU loading the
 * library holds until exit. The first call on a device looks up that array's address (cudaGetSymbolAddress);
 * make that first call before any stream capture. The address is kept for the life of the process, so do not
 * call this on a device after resetting it (cudaDeviceReset). Like the other single-kernel entry points the
 * call is synchronous: it reads the error word back and returns once the product has completed. Calls share
 * the array and it keeps the last call's word (each call clears it first, in stream order), so calls that
 * overlap on the GPU race on it. It takes and rejects exactly what cudanet_k_gemm does (ldc < N included).
 * Any M, N, K that cudanet_k_gemm takes fits: the scratch need does not grow with the product. */
CUDANET_API int cudanet_k_gemm_noalloc(int dtype, int epi, int bn, const void* A, const void* W, const float* bias,
                                       void* C, int M, int N, int K, int ldc, void* stream, char* err, int err_len);

/* X[M, N] += A[M, K] * W[N, K]^T + bias (f32, in place), then H[M, N] = LayerNorm(X) * g + b (16-bit, eps 1e-5):
 * the residual product fused with the LayerNorm after it. N must be 256, 512 or 1024. */
CUDANET_API int cudanet_k_gemm_resln(int dtype, const void* A, const void* W, const float* bias, float* X,
                                     const float* g, const float* b, void* H, int M, int N, int K, void* stream,
                                     char* err, int err_len);

/* att[rows, d] = per (board, head) softmax(q k^T / sqrt(d/heads)) v over the 65 tokens of each board, qkv
 * [B*65, 3d]. */
CUDANET_API int cudanet_k_attention(int dtype, const void* qkv, void* att, int B, int d, int heads, void* stream,
                                    char* err, int err_len);

/* cudanet_k_attention on the two-group tensor-memory kernel (tcgen05 products, head width 64 only). */
CUDANET_API int cudanet_k_attention_tc(int dtype, const void* qkv, void* att, int B, int d, int heads, void* stream,
                                       char* err, int err_len);
/* One attention launch on a chosen kernel: kernel 0 the mma.sync kernel, 1 the two-group and 4 the four-group
 * tensor-memory kernels (head width 64), -1 the evaluator's choice; e4m3_out writes e4m3 of att * mul (bf16
 * qkv only), else att in the qkv type. For tests of every kernel on every output type. */
CUDANET_API int cudanet_k_attention_kernel(int dtype, int e4m3_out, int kernel, const void* qkv, void* att, int B,
                                           int d, int heads, float mul, void* stream, char* err, int err_len);

/* att[b, :] = the attention output of board b's CLS query only (token 0 of each board), att dense [B, d]: what
 * the last layer needs, since the heads read the CLS row alone. No counterpart in the reference. */
CUDANET_API int cudanet_k_attention_cls(int dtype, const void* qkv, void* att, int B, int d, int heads, void* stream,
                                        char* err, int err_len);

/* h[i] = LayerNorm(x[i * row_stride]) (f32 in, 16-bit out), i < n, eps 1e-5. */
CUDANET_API int cudanet_k_layernorm(int dtype, const float* x, const float* g, const float* b, void* h, int n,
                                    int d, int row_stride, void* stream, char* err, int err_len);

/* The FP8 pieces (no counterpart in the reference). A[M, K] and W[N, K] are e4m3 bytes, K a multiple of 128;
 * v = acc * colscale[n] + bias[n] with epi 0: C bf16 = v; 2: C f32 += v; 3: C f32 = v; 4: C e4m3 =
 * gelu(v) * out_scale_inv (round to nearest even, saturating at +-448); 5: C bf16 = bf16(C + bf16(v)) (v rounded
 * to bf16, then added into C by a bf16 reduction in memory). bn as for cudanet_k_gemm. */
CUDANET_API int cudanet_k_gemm_f8(int epi, int bn, const void* A, const void* W, const float* colscale,
                                  const float* bias, float out_scale_inv, void* C, int M, int N, int K, int ldc,
                                  void* stream, char* err, int err_len);

/* cudanet_k_attention on bf16 qkv with e4m3 output: att = e4m3(attention * mul). */
CUDANET_API int cudanet_k_attention_f8(const void* qkv, void* att, int B, int d, int heads, float mul, void* stream,
                                       char* err, int err_len);

/* cudanet_k_layernorm with e4m3 output: h[i] = e4m3(LayerNorm(x[i * row_stride]) * mul), x f32 (x_dtype 0)
 * or bf16 (x_dtype 1, the FP8 path's residual stream). */
CUDANET_API int cudanet_k_layernorm_f8(int x_dtype, const void* x, const float* g, const float* b, void* h, int n,
                                       int d, int row_stride, float mul, void* stream, char* err, int err_len);

#ifdef __cplusplus
}
#endif

#endif /* CUDANET_B200_H */
