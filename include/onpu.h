/*
 * libonpu for NVIDIA B200 (sm_100a): the C ABI of OpenNPU's int4 weight-only matmul path.
 *
 * Part 1 keeps the reference library's exported names, signatures, argument meaning and error
 * behaviour (NULL handle / 0 return = "not supported, fall back"), so the reference's ctypes
 * binding (opennpu/native/npu4/model.py:281-335) and its callers load this library unchanged.
 * Every declaration cites the reference definition it replaces (llama/ggml-opennpu/...).
 * Buffers passed as float* / int32_t* are HOST memory, fp32, row-major, contiguous, as in the
 * reference; the library copies them to the GPU and back. Outputs are overwritten.
 *
 * Part 2 adds B200-specific entry points (device pointers + CUDA streams, packed-int4 ingest,
 * error reporting). They have no counterpart in the reference.
 *
 * Errors never throw across the ABI. A failing call records a message readable with
 * onpu_last_error() and, for calls that return a value, returns NULL / 0 / a negative code.
 */
#ifndef ONPU_H
#define ONPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ======================================================================== part 1: reference ABI */

/* 1 when a CUDA device is usable (reference: NPU device found, onpu_api.cpp:59). */
int onpu_ok(void);
/* 1 when the batched (multi-token) path is available (onpu_api.cpp:60). Always equal to onpu_ok():
 * the GPU kernels take 1..any tokens per weight pass. */
int onpu_batched_ok(void);
/* Kernel launches so far and host seconds spent waiting for them (onpu_api.cpp:72-80). */
void onpu_stats(int64_t *calls, double *wait_s);
/* 1 if a device shape exists (onpu_api.cpp:82-84). The GPU kernels are shape-generic: 1 whenever
 * onpu_ok(). */
int onpu_has_shape(int tiles, int kc, int batched);

/* R, S, tiles, kc, ks, rows_col, cb, nbytes of an [N, K] matrix on ncols columns; all 0 when
 * there is no geometry (onpu_api.cpp:64-69). Identical arithmetic: these sizes define the upload
 * buffers below, and opennpu/native/npu4/model.py:353-360 checks them against its own Mat. */
void onpu_geometry2(int64_t N, int64_t K, int ncols, int sym, int64_t *out);
void onpu_geometry(int64_t N, int64_t K, int ncols, int64_t *out);

/* ---- dense matrices (onpu_api.cpp:87-156) */
/* New [N, K] matrix; sym 0 = q4nx (bf16 scale+min per 32), 1 = q4s (bf16 scale). NULL when the
 * shape has no 8-column geometry or no device (onpu_api.cpp:87-101). */
void *onpu_dense_new2(int64_t N, int64_t K, int sym);
void *onpu_dense_new(int64_t N, int64_t K);                 /* onpu_api.cpp:102 */
/* Host buffer of onpu_dense_bytes() bytes for the caller to fill with the stream-order packets
 * of opennpu_core.hpp:178-254 (onpu_api.cpp:103-104). */
uint8_t *onpu_dense_buf(void *h);
int64_t onpu_dense_bytes(void *h);
/* Upload the buffer and convert it to the GPU layout (onpu_api.cpp:106-114). */
void onpu_dense_sync(void *h);
/* y[rows][N] = x[rows][K] . W^T; x rounded to bf16 first, fp32 accumulate, fp32 y
 * (onpu_api.cpp:119-156). */
void onpu_dense_mv(void *h, const float *x, int64_t rows, float *y);
void onpu_dense_free(void *h);                              /* onpu_api.cpp:116 */

/* ---- expert banks: E experts of [N, K], expert e's packets at e * expert_bytes (onpu_api.cpp:159-250) */
void *onpu_bank_new2(int64_t N, int64_t K, int64_t E, int ncols, int sym);
void *onpu_bank_new(int64_t N, int64_t K, int64_t E, int ncols);   /* onpu_api.cpp:168 */
uint8_t *onpu_bank_buf(void *h);                           /* onpu_api.cpp:169 */
int64_t onpu_bank_expert_bytes(void *h);                   /* onpu_api.cpp:170 */
void onpu_bank_sync(void *h);                              /* onpu_api.cpp:171-174 */
/* y[T][k][N]: token t, slot j -> expert ids[t*k+j] applied to x[t] (x_per_slot == 0) or
 * x[t][j] (x_per_slot != 0) (onpu_api.cpp:177-250). */
void onpu_bank_run(void *h, const float *x, int x_per_slot, int64_t T, const int32_t *ids, int k, float *y);
void onpu_bank_free(void *h);                              /* onpu_api.cpp:175 */

/* ---- MoE glue (onpu_api.cpp:252-278, onpu_cpu.cpp:231-274) */
/* y[T][Nd] = sum_j w[t][j] * (dn_e . act(gu_e . x_t + gu_bias[e]) + dn_bias[e]); act 0:
 * silu(h[:I]) * h[I:]; act 1: gpt-oss interleaved clamped gate (alpha, limit). */
void onpu_moe_ffn(void *gu, void *dn, const float *x, int64_t T, const int32_t *ids, int k, const float *w, int act,
                  float alpha, float limit, const float *gu_bias, const float *dn_bias, float *y);
/* Host CPU helpers with the reference's semantics (onpu_cpu.cpp:233-274). */
void onpu_moe_act(const float *h, int64_t rows, int64_t Ng, const int32_t *ids, const float *gu_bias, int act,
                  float alpha, float limit, float *a);
void onpu_moe_sum(const float *o, int64_t T, int k, int64_t N, const int32_t *ids, const float *w, const float *bias,
                  float *y);
/* One decode token of softmax attention (onpu_cpu.cpp:173-229, same arguments): q [Hq][D] fp32;
 * K, V: Hkv heads of S rows of D values (fp32, or bf16 for *_bf16), head stride hs and row stride
 * rs in elements; mask [S] additive or NULL; sinks [Hq] extra logits or NULL; out [Hq][D] fp32.
 * Host pointers, as in the reference; runs on the GPU (the cache rows are copied up each call).
 * Needs Hq % Hkv == 0 with Hq / Hkv <= 16 and D <= 256 with D * (4 or 2) % 16 == 0; otherwise
 * out is untouched and onpu_last_error() says why. */
void onpu_attn_step(const float *q, int Hq, int D, const float *K, const float *V, int Hkv, int64_t S, int64_t hs,
                    int64_t rs, const float *mask, const float *sinks, float scale, float *out);
void onpu_attn_step_bf16(const float *q, int Hq, int D, const uint16_t *K, const uint16_t *V, int Hkv, int64_t S,
                         int64_t hs, int64_t rs, const float *mask, const float *sinks, float scale, float *out);

/* ---- fused routed-expert FFN (onpu_api.cpp:292-496) */
void *onpu_ffn_new(int64_t Ng, int64_t Kg, int64_t Nd, int64_t Kd, int64_t E, int sym);
void *onpu_ffn_gu(void *h);                                /* onpu_api.cpp:326 */
void *onpu_ffn_dn(void *h);                                /* onpu_api.cpp:327 */
int onpu_ffn_fused(void *h);                               /* onpu_api.cpp:328 */
/* packed gate_up row r holds original row perm[r] (onpu_api.cpp:329-332). Identity here: the GPU
 * interleaves gate/up rows itself when it converts the upload. */
void onpu_ffn_perm(void *h, int32_t *out);
/* one token: y[Nd] = sum_j w[j] * FFN_{ids[j]}(x); 1 = done (onpu_api.cpp:423-446) */
int onpu_ffn_run(void *h, const float *x, const int32_t *ids, int k, const float *w, float *y);
/* T tokens: y[T][Nd] (onpu_api.cpp:451-496) */
int onpu_ffn_run_many(void *h, const float *x, int64_t T, const int32_t *ids, int k, const float *w, float *y);
void onpu_ffn_free(void *h);                               /* onpu_api.cpp:333-339 */

/* ---- codec (onpu_api.cpp:499-529): host CPU, load time */
int64_t onpu_pack(const float *W, int64_t N, int64_t K, int ncols, int sym, uint8_t *out, int threads);
void onpu_quant_dequant(const float *W, int64_t N, int64_t K, int sym, float *out, int threads);

/* ======================================================================== part 2: B200 additions */
/* No counterpart in the reference. */

/* Weight formats of the GPU layout. */
#define ONPU_FMT_Q4NX 0   /* q*s + m, bf16 s, m  (reference sym = 0)           */
#define ONPU_FMT_Q4S 1    /* (q-8)*d, bf16 d     (reference sym = 1)           */
#define ONPU_FMT_Q4F16 2  /* v*s, int4 v in [-8,7] packed along K, fp16 s      */

/* Output epilogues of the device-pointer GEMV. */
#define ONPU_EPI_F32 0    /* y fp32                                                    */
#define ONPU_EPI_BF16 1   /* y bf16                                                    */
#define ONPU_EPI_SWIGLU 2 /* y[i] = bf16(silu(acc[gate i]) * acc[up i]); needs a gate/up */
                          /* matrix created with onpu_dense_new_int4(..., gateup = 1)     */
#define ONPU_EPI_PAIRSUM 3 /* y[i] = acc[row i] + acc[residual of row i], fp32; needs a    */
                           /* matrix from onpu_dense_new_residual_f32_dev                 */
#define ONPU_EPI_SWIGLU_F32 5 /* as ONPU_EPI_SWIGLU with fp32 y: the activation keeps full     */
                              /* precision for an fp32-input down projection (onpu_dense_mv_f32_dev) */

/* Last error message of this thread (NULL if the last failing-capable call succeeded). */
const char *onpu_last_error(void);
/* Device-side status: 0 ok, else a kernel reported a timed-out wait (then reset). Synchronises. */
int onpu_check_device(void);

/* A dense [N, K] matrix filled from int4 packed along K: qk[N][K/2] (two's complement, element
 * 2j in the low nibble of byte j) and fp16 scales s[N][K/32]. Any K % 32 == 0 (no geometry
 * limit). gateup != 0: rows [0, N/2) are gate, [N/2, N) up, stored interleaved so that
 * ONPU_EPI_SWIGLU can fuse the activation (N/2 % 8 == 0). */
void *onpu_dense_new_int4(int64_t N, int64_t K, int gateup);
/* Fill from host (on_device = 0) or device (on_device = 1) arrays; 0 ok, < 0 error. */
int onpu_dense_load_int4(void *h, const uint8_t *qk, const uint16_t *scales, int on_device, void *stream);
/* GGUF weights as they lie in a llama.cpp checkpoint (ggml type ids): rows of blocks, row stride
 * K/32 * 18 bytes (Q4_0) or K/256 * 144 bytes (Q4_K).
 * Q4_0: blocks of 32 = fp16 d + 16 bytes (element j in the low nibble of byte j, j + 16 in the
 *   high one), w = (q - 8) d: the BASELINE int4 + fp16 format, ingested exactly (ONPU_FMT_Q4F16),
 *   no requantisation (the reference dequantises and requantises every non-Q4_K type,
 *   llama/ggml-opennpu/ggml-opennpu.cpp:183-207).
 * Q4_K: super-blocks of 256 = fp16 d, fp16 dmin, 12 bytes of 6-bit scales / mins, 128 bytes of
 *   codes; transcoded into q4nx (ONPU_FMT_Q4NX) as the reference's q4k_codes does
 *   (ggml-opennpu.cpp:100-143): the codes exactly, each 32-group's scale d * sc and min -dmin * m
 *   as the bf16 pair among their 3 x 3 bf16 neighbours closest (least squares) to the exact
 *   weights. The transcode runs on the GPU. */
#define ONPU_GGML_Q4_0 2
#define ONPU_GGML_Q4_K 12
/* GGUF rows (device) -> codes q [rows][K] (0..15), 16-bit scales [rows][K/32] (fp16 bits for Q4_0,
 * bf16 for Q4_K) and, for Q4_K, bf16 mins [rows][K/32] (device). Asynchronous. 0 ok, < 0 error. */
int onpu_gguf_codes_dev(int type, const void *src, int64_t rows, int64_t K, uint8_t *q, uint16_t *scales,
                        uint16_t *mins, void *stream);
/* A dense [N, K] handle from N GGUF rows on the host (on_device = 0) or device (1); gateup as in
 * onpu_dense_new_int4. Synchronous; NULL on error. */
void *onpu_dense_new_gguf(int64_t N, int64_t K, int type, const void *data, int on_device, int gateup, void *stream);
/* An expert bank [E][N, K] from E x N GGUF rows (a ggml [K, N, E] expert tensor), as
 * onpu_bank_new_int4 for int4. Synchronous; NULL on error. */
void *onpu_bank_new_gguf(int64_t N, int64_t K, int64_t E, int type, const void *data, int on_device, int gateup,
                         void *stream);
/* The load-time search quantisers on the GPU: W fp32 [N][ldw] (device, 16-byte
 * aligned, ldw % 4 == 0, K % 32 == 0) -> codes q [N][K] (0..15), 16-bit (bf16) scales [N][K/32] and,
 * for q4nx (sym = 0), mins [N][K/32]; bit-exact with onpu_pack's quantisers
 * (opennpu_core.hpp:103-169, which the reference runs on the host at load time). Asynchronous. */
int onpu_quantize_dev(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, uint8_t *q, uint16_t *scales,
                      uint16_t *mins, void *stream);
/* A dense handle quantised on the GPU from fp32 weights (q4s when sym != 0, else q4nx): the same
 * codes and scales onpu_pack + onpu_dense_sync produce, without the host pass. gateup as in
 * onpu_dense_new_int4. Synchronous; NULL on error. */
void *onpu_dense_new_f32_dev(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, int gateup, void *stream);
/* The two-pass (~8-bit) mode of the reference's NPULinearGroup(residual=True)
 * (opennpu/native/npu4/model.py:793-833): rows [W; W - quant_dequant(W)], each pass quantised with
 * the search quantiser, the two halves added after the product. Here both halves are quantised on
 * the GPU from fp32 W [N][ldw] (N % 8 == 0) and stored interleaved per 16-row strip, so one GEMV
 * launch with ONPU_EPI_PAIRSUM (onpu_dense_mv_dev, output [rows][N] fp32) streams both and adds
 * them in its epilogue. Synchronous; NULL on error. */
void *onpu_dense_new_residual_f32_dev(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, void *stream);
/* Format, N, K, bytes of the GPU-layout matrix. */
int onpu_dense_info(void *h, int64_t *out4);
/* y = x . W^T on the GPU, asynchronous on `stream` (NULL: the legacy default stream).
 * x: bf16 [rows][ldx] device, 16-byte aligned rows (ldx % 8 == 0); y: [rows][ldy] fp32 or bf16
 * device (by epi). A first call for a given row count allocates (call it outside stream capture);
 * later calls with that row count allocate nothing. 0 ok, < 0 error. */
int onpu_dense_mv_dev(void *h, const void *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi, void *stream);
/* onpu_dense_mv_dev with fp32 activations x [rows][ldx] (device, 16-byte aligned rows, ldx % 4 ==
 * 0), rows <= 8: each value is staged as two fp16 halves (x rounded, then its rounding error) on
 * two tensor-core columns whose products are added, so the products keep ~22 bits of x instead of
 * bf16's 8: the down projection of a decode MLP can take ONPU_EPI_SWIGLU_F32's output and match
 * the reference's fp32 dequantise-then-matmul path (opennpu/native/reference.py:55-57, :84)
 * without rounding the activation. Same epilogues, outputs and allocation rule. 0 ok, < 0 error. */
int onpu_dense_mv_f32_dev(void *h, const float *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi,
                          void *stream);
/* The most rows (0..8) onpu_dense_mv_f32_dev takes for this matrix: each CTA keeps its part of
 * the two fp16 rows per token in shared memory (e.g. 3 for a 4096 x 12288 down projection on one
 * B200, 8 for its tensor-parallel shards). 0 without a usable device. */
int onpu_dense_max_f32_rows(void *h);
/* Y = X . W^T for many tokens (prefill) on the tensor cores (tcgen05, fp32 accumulators in tensor
 * memory); same arguments as onpu_dense_mv_dev, any rows >= 1. The weights are dequantised to
 * fp16 (one rounding per weight) and the activations copied to fp16 first (a token beyond the fp16
 * range is scaled by a power of two). Replaces the reference's multi-token device path
 * (opennpu/native/npu4/kernels/gemm8.cc:33-139, one 8-token pass per 8 tokens). Asynchronous;
 * allocates its fp16 activation copy on first use of a larger row count. 0 ok, < 0 error. */
int onpu_dense_mm_dev(void *h, const void *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi, void *stream);
/* Prepare (allocate descriptors and scratch for) `rows`-row calls without running one. */
int onpu_dense_prepare(void *h, int64_t rows);
/* ---- device-resident MoE layer (config 4's routed experts, every buffer on the GPU)
 * Router: logits = h . Wr^T (bf16 h [T][ldh], bf16 Wr [E][H], fp32 sums), probabilities softmax,
 * the k largest (descending; equal probabilities: lower expert id first), weights renormalised over
 * the k when norm != 0. Replaces the reference's CPU router (opennpu/native/reference.py:71-76,
 * opennpu/native/moe_runtime.py:333-341). ids int32 [T][k], w fp32 [T][k], logits fp32
 * [T][E] or NULL. 1 <= k <= 16, k <= E <= 256, H % 8 == 0, 16-byte aligned rows. Asynchronous. */
int onpu_route_dev(const void *h, int64_t ldh, int64_t T, const void *wr, int64_t E, int64_t H, int k, int norm,
                   int32_t *ids, float *w, float *logits, void *stream);
/* An expert bank of E [N, K] matrices filled from int4 packed along K (the layout of
 * onpu_dense_new_int4, experts back to back: qk[E][N][K/2], scales[E][N][K/32]). gateup != 0
 * stores gate/up rows interleaved for the fused SwiGLU. The int4 counterpart of onpu_bank_new2
 * (llama/ggml-opennpu/onpu_api.cpp:159-167) for checkpoints that are already group-32 int4. */
void *onpu_bank_new_int4(int64_t N, int64_t K, int64_t E, int gateup);
int onpu_bank_load_int4(void *h, const uint8_t *qk, const uint16_t *scales, int on_device, void *stream);
/* A routed-expert FFN (gate_up [E][Ng][Kg] with Ng = 2 * Kd, down [E][Nd][Kd]) of int4 banks; fill
 * them with onpu_bank_load_int4 on onpu_ffn_gu / onpu_ffn_dn. The int4 counterpart of onpu_ffn_new
 * (llama/ggml-opennpu/onpu_api.cpp:292-309). */
void *onpu_ffn_new_int4(int64_t Ng, int64_t Kg, int64_t Nd, int64_t Kd, int64_t E);
/* y[t] = sum_j w[t][j] * down_e(silu(gate_e . x_t) * (up_e . x_t)), e = ids[t][j], on the GPU:
 * x bf16 [T][ldx], ids/w from onpu_route_dev (device), y fp32 [T][ldy]. Four launches on `stream`,
 * no host synchronisation (capturable in a CUDA graph once a first call has sized the scratch):
 * the token-sorted expert jobs are built on the device from the ids, then gate_up (fused SwiGLU,
 * fp32 activation), down (the activation staged as two fp16 halves per value, so it is not
 * rounded to 16 bits) and the weighted combine. An id outside [0, E) drops that (token, slot)
 * pair and sets the device status (onpu_check_device reports it). At most 2048 experts. Replaces
 * opennpu/native/reference.py:77-84 and the device part of onpu_moe_ffn
 * (llama/ggml-opennpu/onpu_api.cpp:261-278). 0 ok, < 0 error. */
int onpu_moe_ffn_dev(void *ffn, const void *x, int64_t ldx, int64_t T, const int32_t *ids, const float *w, int k,
                     float *y, int64_t ldy, void *stream);
/* How onpu_moe_ffn_dev, onpu_moe_ffn_dev_ep and onpu_moe_layer_dev run the expert FFN (no
 * reference counterpart; the reference's onpu_ffn_run is one NPU dispatch, onpu_api.cpp:423-496):
 * 1 (default) as ONE persistent launch (gate_up + SwiGLU, down and the combine, grid barriers
 * between them) whenever both banks share a format; 0 as three launches (gate_up grouped GEMV with
 * SwiGLU, down grouped GEMV, combine). Both compute the same exact products in fp32; where the
 * three-launch form splits a row group between CTAs its sums may differ from the persistent
 * kernel's in the last bits. Returns the previous mode, or -1 for a mode other than 0 or 1. */
int onpu_moe_set_fused(int mode);
/* The whole MoE layer: the router (bf16 wr [E][H], H = the FFN's hidden size; k, norm as in
 * onpu_route_dev) writes ids [T][k] / w [T][k] and, in its last CTA, the expert job lists; then
 * the expert FFN as onpu_moe_ffn_dev. Same results as onpu_route_dev followed by
 * onpu_moe_ffn_dev (reference.py:71-84), one launch fewer. 0 ok, < 0 error. */
int onpu_moe_layer_dev(void *ffn, const void *wr, const void *x, int64_t ldx, int64_t T, int k, int norm, int32_t *ids,
                       float *w, float *y, int64_t ldy, void *stream);
/* Expert parallelism: the same layer when this FFN holds only experts e0 .. e0 + E - 1 of a larger
 * pool. ids are global; slots routed to other experts are skipped, so y[t] is this rank's share of
 * the sum (the ranks' shares add up to onpu_moe_ffn_dev's y). No reference counterpart (the
 * reference has no multi-device path). 0 ok, < 0 error. */
int onpu_moe_ffn_dev_ep(void *ffn, const void *x, int64_t ldx, int64_t T, const int32_t *ids, const float *w, int k,
                        int64_t e0, float *y, int64_t ldy, void *stream);
/* ---- one-shot all-reduce over NVLink peer memory (tensor-parallel decode; no reference
 * counterpart). One handle per rank (one process per GPU): onpu_comm_new allocates this rank's
 * buffer for vectors of up to cap floats, onpu_comm_ipc_handle writes its 64-byte CUDA IPC handle,
 * the caller exchanges the handles (e.g. an all-gather on the host) and passes all world of them,
 * in rank order, to onpu_comm_open. onpu_comm_allreduce: the sum over ranks of src (n floats) into
 * dst (fp32, may be src) and / or dst_bf16 (bf16; either may be NULL), one launch on `stream`:
 * every rank stores each value, paired with the call number in one 8-byte word, into every peer's
 * buffer, then reads the world words of each element until they carry this call's number and
 * adds them in rank order (identical sums on every rank). Every rank must make the same sequence
 * of calls; capturable in a CUDA graph. A peer that does not arrive within 2 s sets the device
 * status (onpu_check_device). */
void *onpu_comm_new(int rank, int world, int64_t cap_floats);
int onpu_comm_ipc_handle(void *comm, void *out64);
int onpu_comm_open(void *comm, const void *handles);
int onpu_comm_allreduce(void *comm, const float *src, float *dst, void *dst_bf16, int64_t n, void *stream);
void onpu_comm_free(void *comm);
/* How long a kernel waits for another rank's words (the fused all-reduce GEMV and
 * onpu_comm_allreduce) before it gives up, sets the device status (onpu_check_device reports
 * an all-reduce timeout) and returns with the values as found: 2 s unless set; later launches use
 * the new limit. 0 ok, < 0 error. */
int onpu_comm_set_wait(double seconds);
/* The row-parallel projection and its all-reduce fused in one launch (no reference counterpart):
 * y / y_bf16 (either may be NULL) = the sum over ranks of x . W_rank^T, rows x N fp32 / bf16,
 * where W_rank is this rank's K block (dense handle h, no gate/up or residual rows) and comm an
 * opened onpu_comm handle with cap >= rows x N. The GEMV's epilogue stores every finished output,
 * paired with the call number in one 8-byte word, straight into every rank's buffer over NVLink
 * while the rest of the matrix is still streaming; after its range each CTA waits (bounded) for
 * every rank's words of the rows it finished, adds them in rank order (the same sums on every
 * rank) and writes them. The rows each CTA sums follow from the shape, so every call on one
 * communicator must have the same matrix shape, row count and activation type (use one
 * communicator per call site, e.g. one for o and one for down), and no onpu_comm_allreduce on it;
 * every rank makes the same sequence of calls. 0 ok, < 0 error. */
int onpu_dense_mv_allreduce_dev(void *h, void *comm, const void *x, int64_t ldx, int64_t rows, float *y,
                                void *y_bf16, void *stream);
/* The same with fp32 activations (rows <= 8, staged as in onpu_dense_mv_f32_dev). */
int onpu_dense_mv_allreduce_f32_dev(void *h, void *comm, const float *x, int64_t ldx, int64_t rows, float *y,
                                    void *y_bf16, void *stream);
/* ---- GEMV chains: a decode step's dense GEMVs recorded once on fixed device buffers and run as
 * ONE persistent launch (the GPU analogue of the reference's instruction stream per call,
 * llama/ggml-opennpu/opennpu_core.hpp:418-505, and of onpu_ffn_run's gate_up -> act -> down
 * sequence, onpu_api.cpp:423-446). Links run in order; a link whose x or y overlaps the y (or,
 * for y, the x) of an earlier link waits on the device until that link is finished everywhere.
 * Runs of one chain must be ordered on one stream. */
void *onpu_chain_new(void);
/* Append y = x . W^T (dense handle h, 1..16 rows; pointer rules of onpu_dense_mv_dev). dep: an
 * earlier link this one must also wait for (-1: data overlaps only). The link index, < 0 on
 * error. All links of a chain share one weight format. */
int onpu_chain_add(void *chain, void *h, const void *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi,
                   int dep);
/* links, CTAs, shared memory per CTA, MMA n-tiles (CTAs and shared memory after prepare) */
int onpu_chain_info(void *chain, int64_t *out4);
/* the link a link waits for (-1 none; -2 bad index) */
int onpu_chain_link_dep(void *chain, int link);
/* Allocate the chain's scratch and upload its links (the first run does it when needed: call
 * this outside stream capture). 0 ok. */
int onpu_chain_prepare(void *chain);
/* One launch on `stream`, asynchronous. 0 ok. */
int onpu_chain_run(void *chain, void *stream);
/* Tracing: later runs write %globaltimer stamps (ns) to the device buffer `stamps`
 * [CTAs][links][8]: consumer start, dependency met, activations staged, math done, link counted,
 * producer first copy, producer last copy, then the nanoseconds consumer warp 0 waited for weights
 * during the link. NULL turns it off. CTAs from onpu_chain_info. */
int onpu_chain_trace(void *chain, uint64_t *stamps);
void onpu_chain_free(void *chain);
/* Tracing of the GEMV kernels (dense and expert launches through this library): later launches
 * with at most `ctas` CTAs write 12 values per CTA to the device buffer `stamps` [ctas][12]:
 * %globaltimer stamps (ns) of entry, producer's first copy issued, consumers past
 * griddepcontrol.wait, activations staged, first weights arrived, last stage consumed, range
 * flushed; the nanoseconds the consumers waited for weights; then for a split row group the stamp
 * of this CTA's partial sums published (as a later contributor), the stamp of its partners' flags
 * seen and their count (as the first contributor), and the stamp of their partial sums read. Slots
 * a launch does not reach keep their value; each launch overwrites the same slots. NULL turns it
 * off. */
int onpu_gemv_trace(uint64_t *stamps, int64_t ctas);

/* onpu_dense_mv_dev with no allocation in the call: no reference counterpart (the NPU library
 * has no device scratch). Same arguments, epilogues (ONPU_EPI_PAIRSUM and ONPU_EPI_SWIGLU_F32
 * included) and bit-identical results as onpu_dense_mv_dev (the same grid, so the same summation
 * order), but the split-row scratch and descriptors live in one static device array shared by
 * every call on a device, for callers that cannot let the library allocate (all free HBM handed to
 * their own pool, or a fixed device footprint). rows <= 256 per call, else -1 with an error
 * message. The descriptors are written on the device by a small kernel on `stream` before the
 * GEMV. The first call on a device looks up the array (cudaGetSymbolAddress) and clears it; make
 * that first call before any stream capture. Overlapping calls race: order them on one stream. */
int onpu_dense_mv_dev_noalloc(void *h, const void *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi,
                              void *stream);
/* GPU layout -> plain codes q[N][K] (0..15), scales[N][K/32] (and mins for q4nx), device pointers;
 * for bit-exact verification. */
int onpu_dense_unpack_dev(void *h, uint8_t *q, uint16_t *scales, uint16_t *mins, void *stream);

/* ---- the ggml-opennpu backend's operator layer (llama/ggml-opennpu/ggml-opennpu.cpp:270-539,
 * 703-753) over this library: which MUL_MAT / MUL_MAT_ID nodes it takes, their tensor layouts,
 * and the learned sibling fusion. Tensors are described by the ggml_tensor fields the layer
 * reads; the ggml_backend_* registration around it is llama.cpp code (it needs llama.cpp's
 * headers) and calls these entry points from its supports_op and graph_compute callbacks. */
typedef struct onpu_ggml_tensor {
    int32_t type;            /* ggml type id: F32 0, F16 1, Q4_0 2, Q4_K 12, I32 26, BF16 30 */
    int32_t weights;         /* non-zero: the tensor lives in a weights buffer */
    int64_t ne[4];           /* elements per dimension, innermost first (ggml ne) */
    int64_t nb[4];           /* byte strides per dimension (ggml nb) */
    void *data;              /* host memory */
    const char *name;        /* "blk.<i>.<what>.weight" for weights (sibling fusion groups by block) */
} onpu_ggml_tensor;
#define ONPU_GGML_OP_VIEW 0        /* NONE / RESHAPE / VIEW / PERMUTE / TRANSPOSE: no work */
#define ONPU_GGML_OP_MUL_MAT 1     /* dst[N, M...] = w[K, N] x[K, M...]                      */
#define ONPU_GGML_OP_MUL_MAT_ID 2  /* dst[N, n_used, T] = w[K, N, E] experts ids[n_used, T] of x[K, n_used|1, T] */
/* 1 when the node runs here (opennpu_supports): MUL_MAT of a contiguous weight (F32, F16, BF16,
 * Q4_0, Q4_K; K % 32 == 0, Q4_K K % 256 == 0) with ne2 == ne3 == 1 over F32 rows, not a Hadamard
 * hint, N x K >= OPENNPU_MIN_PARAMS (default 2^20); MUL_MAT_ID of Q4_0 / Q4_K experts with I32 ids
 * and N x K >= 2^17; view ops; never a weight named by an OPENNPU_CPU_TENSORS prefix. */
int onpu_ggml_supports(int op, const onpu_ggml_tensor *dst, const onpu_ggml_tensor *w, const onpu_ggml_tensor *x,
                       const onpu_ggml_tensor *ids, int hadamard_hint);
void *onpu_ggml_new(void);
/* Record a node before any runs (the backend's supports_op sees every node while llama.cpp
 * reserves its graphs): weights reading the same input, in the same block and with the same K,
 * become one fused group (at most 4) on the first compute; OPENNPU_FUSE=0 turns fusion off. */
void onpu_ggml_note(void *ctx, int op, const onpu_ggml_tensor *w, const onpu_ggml_tensor *x,
                    const onpu_ggml_tensor *ids);
/* Run a node, writing dst (host). A fused group's first member computes every member; the others
 * copy their waiting slice when their input (pointer and contents) and ids are unchanged. Weights
 * become GPU handles on first use. 0 ok, < 0 error (onpu_last_error). */
int onpu_ggml_compute(void *ctx, int op, const onpu_ggml_tensor *dst, const onpu_ggml_tensor *w,
                      const onpu_ggml_tensor *x, const onpu_ggml_tensor *ids);
/* fused slices used, fused slices discarded, groups, weight handles */
void onpu_ggml_stats(void *ctx, int64_t *out4);
void onpu_ggml_free(void *ctx);

/* onpu_attn_step on device pointers (a KV cache resident in HBM), asynchronous on `stream`:
 * kv_bf16 selects a bf16 cache. K, V 16-byte aligned with hs and rs multiples of 16 bytes.
 * 0 ok, < 0 error. Split-KV: each CTA streams a range of one kv head's rows once for all the
 * query heads that share it; a second kernel merges the ranges. */
int onpu_attn_step_dev(const float *q, int Hq, int D, const void *K, const void *V, int Hkv, int64_t S, int64_t hs,
                       int64_t rs, const float *mask, const float *sinks, float scale, float *out, int kv_bf16,
                       void *stream);

/* ---- weight blobs: the GPU layout on disk (replaces what the reference's PackCache stores,
 * npu4/model.py:712-759: the packed upload bytes of one NPU buffer, so a second model load skips
 * reading and quantising the checkpoint). A blob is self-describing: a 64-byte header (magic
 * "ONPUB2GL", onpu_layout_version(), kind, matrix count), then per matrix a 64-byte header
 * (N, K, E, format, flags) and its GPU-layout bytes as they lie in HBM, padded to 64 bytes.
 * A second load of a blob is one host->device copy per matrix: no quantisation, no repack.
 *
 * *_export: dst NULL returns the blob's size; else writes it to host memory dst (cap bytes) and
 * returns its size, or -1 (cap too small, K % 32 != 0, weights never loaded). Synchronises the
 * device first (weights loaded asynchronously are complete).
 * *_import: a new handle (free it with the matching *_free) from a blob in host memory; NULL with
 * an error message if the magic, the layout version, the kind, a shape or the size does not
 * match (checked before any device call). Imported dense handles run on every dense entry point
 * (host and device); like onpu_dense_new_int4 handles they have no stream-order upload buffer. */
int onpu_layout_version(void);
int64_t onpu_dense_export(void *h, void *dst, int64_t cap);
void *onpu_dense_import(const void *src, int64_t nbytes);
int64_t onpu_bank_export(void *h, void *dst, int64_t cap);
void *onpu_bank_import(const void *src, int64_t nbytes);
/* both banks of a routed-expert FFN (gate_up, then down) in one blob */
int64_t onpu_ffn_export(void *h, void *dst, int64_t cap);
void *onpu_ffn_import(const void *src, int64_t nbytes);

#ifdef __cplusplus
}
#endif
#endif /* ONPU_H */
