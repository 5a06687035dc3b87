// Host-callable launchers of libonpu's CUDA kernels (no torch types; plain pointers + streams).
#pragma once
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "gpu_layout.cuh"

namespace onpu_b200 {

// ---- GEMV (gemv.cu)
// Activations of a single-job launch stay resident in shared memory when they take at most this
// many bytes (tokens x padded K x 2 B); otherwise every stage carries its own slice.
constexpr int64_t kResidentXBudget = 40 * 1024;
// A one-job launch whose rows do not fit that budget (5..16 rows of a long K) may instead run one
// CTA per SM with up to this many bytes of resident rows (the ring takes the rest of the 227 KB)
constexpr int64_t kWideResidentXBudget = 136 * 1024;

struct GemvLayout {
    int xres;          // activations resident
    int xstride;       // resident: bytes per activation row (padded)
    int ctab_off;      // resident: offset of the per-group offset table in the activation region
    int wchunks;       // resident: 64-K chunks per row (all of K, or a CTA's window of it)
    int xslots;        // per-stage: token slots per chunk (max tokens + 1 zero slot)
    int off_bar;       // byte offset of the mbarriers in shared memory
    int smem;          // dynamic shared memory per CTA
};
// mrows: activation rows of the largest job (twice its tokens for fp32 split activations);
// wchunks: chunks of K each resident row holds (0 = all of K)
GemvLayout gemv_layout(int fmt, int mrows, int64_t K, int wchunks = 0, int64_t budget = kResidentXBudget);
// true when jobs of up to mrows activation rows stay resident (fp16 path) for this K
bool gemv_resident(int mrows, int64_t K);
int gemv_ctas_per_sm(int fmt, int ntiles, int smem);
int gemv_chunks_per_stage();
int64_t gemv_part_floats_per_worker(int ntiles);
cudaError_t gemv_launch(int fmt, int ntiles, int epi, const GemvParams &p, int smem, cudaStream_t stream, bool pdl);

// ---- GEMV chain (chain.cu): a sequence of dense GEMVs in one persistent launch
// Rows per link: up to two MMA n-tiles of 8 tokens.
constexpr int kChainMaxRows = 16;
struct ChainLayout {
    int ns;            // ring stages
    int off_x;         // activation region
    int off_comb;      // buffer in which the consumer warps combine a row group's partial sums
    int off_bar;       // mbarriers
    int smem;          // dynamic shared memory per CTA
};
// shared memory for a chain whose largest activation region (rows, offset table) is xregion_bytes
ChainLayout chain_layout(int fmt, int ntiles, int64_t xregion_bytes, int ns);
// activation region of one link (m rows of K), its row stride and offset-table position
int64_t chain_xregion_bytes(int64_t m, int64_t K, int ntiles, int *xstride, int *ctab_off);
int chain_ctas_per_sm(int fmt, int ntiles, int smem);        // 0: does not fit
int64_t chain_part_floats_per_slot();
cudaError_t chain_launch(int fmt, int ntiles, const ChainParams &p, int smem, cudaStream_t stream);

// ---- prefill dequant-GEMM (dqgemm.cu): tcgen05 tensor cores, fp16 operands, fp32 accumulators
// x (bf16 [M][ldx]) -> xh (fp16 [M][K], scaled per token when |x| > 2^15) and tscale[M]
cudaError_t x_to_f16_launch(const uint16_t *x, int64_t ldx, int M, int K, uint16_t *xh, float *tscale,
                            cudaStream_t stream);
// Y = Xh . W^T with the dequantised weights; grid of 128-token x 256-row tiles
cudaError_t dqgemm_launch(int fmt, int epi, const uint16_t *xh, const DqGemmParams &p, cudaStream_t stream);
int dqgemm_tile_tokens();

// ---- load-time search quantisers (quant.cu): W fp32 [N][ldw] -> codes [N][K], 16-bit scales and
// mins [N][K/32] (mins may be null; q4s writes none), bit-exact with host_codec's quant_q4s32 /
// quant_q4nx32. ldw % 4 == 0, W 16-byte aligned, K % 32 == 0.
cudaError_t quant_launch(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, uint8_t *q, uint16_t *scales,
                         uint16_t *mins, cudaStream_t stream);
// R [N][K] = W - the dequantised codes (the host's rounding), for the two-pass residual rows
cudaError_t residual_launch(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, const uint8_t *q,
                            const uint16_t *scales, const uint16_t *mins, float *R, cudaStream_t stream);

// ---- one-shot all-reduce over NVLink peer memory (comm.cu)
constexpr int kCommCtas = 16;
constexpr int kCommMaxRanks = kPeerMaxRanks;
// where a fused row-parallel GEMV sends its outputs: every rank's all-reduce buffer
struct PeerOut {
    void *bufs[kCommMaxRanks];
    int rank, world;
    int64_t cap;
    void *y_bf16 = nullptr;    // the summed rows also as bf16
};
// the receive half of comm_allreduce_launch: wait for every rank's words of this call (the senders
// were the GEMV's kEpiPeer epilogues) and add them in rank order into dst / dst_bf16
cudaError_t comm_reduce_launch(void *const *bufs, int rank, int world, int64_t cap, float *dst, void *dst_bf16,
                               int64_t n, int *err, uint64_t wait_ns, cudaStream_t stream);
// bytes of one rank's buffer: two slot sets of world x cap 8-byte words, per-CTA call counters
// (the comm kernel's kCommCtas, then kPeerCtaCounters of the GEMV CTAs that sum rows)
int64_t comm_buffer_bytes(int world, int64_t cap);
// bufs[r]: rank r's buffer as mapped in this process (own at [rank]); dst (fp32) and / or dst_bf16
// = the sum over ranks of src, added in rank order
cudaError_t comm_allreduce_launch(void *const *bufs, int rank, int world, int64_t cap, const float *src, float *dst,
                                  void *dst_bf16, int64_t n, int *err, uint64_t wait_ns, cudaStream_t stream);

// ---- MoE router (router.cu): softmax(h . Wr^T) -> top-k -> renormalise, one CTA per token
constexpr int kMaxRouteExperts = 256;
constexpr int kMaxRouteK = 16;
constexpr int kMaxJobExperts = 2048;    // expert_jobs_kernel keeps 4 ints per expert in shared memory

// Device-side grouping of routed (token, slot) pairs into the GEMV jobs of two expert banks.
struct ExpertJobsParams {
    const int32_t *ids;        // [TK] expert per (token, slot)
    int64_t TK;                // tokens * k
    int k, E;
    int per_job;               // tokens per job at most (1..16)
    const uint8_t *w0;         // bank 0 (gate_up): expert e at w0 + e * bytes0; jobs read token rows
    int64_t bytes0;
    const uint8_t *w1;         // bank 1 (down): jobs read per-slot rows
    int64_t bytes1;
    GemvJob *jobs0, *jobs1;    // capacity min(E, TK) + TK / per_job each
    int *njobs;                // out: jobs in each list
    int *order;                // scratch [TK]
    int *err;                  // bit 8: an id outside [0, E) (that pair is dropped)
    int id_base;               // the bank holds experts id_base .. id_base + E - 1
    int skip_foreign;          // 1: ids outside that range belong to other ranks (skipped, no error)
};
cudaError_t expert_jobs_launch(const ExpertJobsParams &p, cudaStream_t stream);

// The routed-expert FFN in one persistent launch (moe_ffn.cu): gate/up + SwiGLU (fp32), down and
// the weighted combine over the job lists the router kernel built. One resident wave of CTAs.
struct MoeFfnFused {
    int fmt;                          // kFmtQ4S / kFmtQ4F16 / kFmtQ4NX (both banks)
    const GemvJob *jobs_gu, *jobs_dn; // device job lists (expert_jobs_launch / route_launch)
    const int *njobs;                 // device: jobs in each list
    int rg_gu, ch_gu, N_gu, K_gu;     // gate/up bank: row groups, 64-K chunks, rows, K
    int rg_dn, ch_dn, N_dn, K_dn;     // down bank
    const uint16_t *x;                // bf16 token rows
    int64_t ldx;
    float *af;                        // [T*k][K_dn] SwiGLU outputs (scratch)
    float *o;                         // [T*k][N_dn] expert outputs (scratch)
    const int32_t *ids;               // [T][k] expert ids
    const float *w;                   // [T][k] routing weights
    int64_t T;
    int k;
    int id_lo, id_hi;                 // slots whose expert id lies in [id_lo, id_hi) are combined
    float *y;                         // [T][N_dn] fp32, row stride ldy
    int64_t ldy;
    unsigned *bar;                    // 3 counters, zero before the first launch (left zero)
    int *err;
    int workers;                      // CTAs: one resident wave
    int mslots_gu, mslots_dn;         // staged rows: tokens per job, twice that (fp32 halves)
    int xstride_gu, xstride_dn;       // resident activation row strides
    int off_bar;                      // shared-memory offset of the mbarriers
    uint32_t mul[4];                  // 2^28, 2^24, 2^20, 2^16 (as in GemvParams)
    uint32_t unpk[3];                 // 0x000F000F, 0x00F000F0, 0x64006400
};
// dynamic shared memory of the fused FFN kernel, and its layout (mbarrier offset, row strides)
int moe_ffn_fused_smem(int fmt, int mslots_gu, int K_gu, int mslots_dn, int K_dn, int *off_bar, int *xstride_gu,
                       int *xstride_dn);
int moe_ffn_fused_ctas_per_sm(int fmt, int smem);
cudaError_t moe_ffn_fused_launch(const MoeFfnFused &p, int smem, cudaStream_t stream);

// logits: fp32 [T][E] (output or scratch); counters: route_counter_slots(T) words, zero before the
// first launch and left zero by every launch
// jobs (optional): the last token block to finish also builds the expert job lists (as
// expert_jobs_launch would, from the ids just written), in the same launch
cudaError_t route_launch(const uint16_t *h, int64_t ldh, int64_t T, const uint16_t *wr, int E, int H, int k, int norm,
                         int32_t *ids, float *w, float *logits, unsigned *counters, cudaStream_t stream,
                         const ExpertJobsParams *jobs = nullptr);
int64_t route_counter_slots(int64_t T);

// ---- GGUF block formats (gguf.cu): ggml rows of Q4_0 / Q4_K blocks -> plain codes q [rows][K]
// (0..15), 16-bit scales [rows][K/32] (fp16 for Q4_0, bf16 for Q4_K) and bf16 mins (Q4_K)
constexpr int kGgmlQ4_0 = 2;
constexpr int kGgmlQ4_K = 12;
int64_t gguf_row_bytes(int type, int64_t K);                // -1: type or K not supported
cudaError_t gguf_codes_launch(int type, const uint8_t *src, int64_t rows, int64_t K, uint8_t *q, uint16_t *scales,
                              uint16_t *mins, cudaStream_t stream);

// ---- layout conversion (repack.cu)
// Where the codes of the matrix come from.
enum RepackSource : int {
    kSrcStream = 0,     // the reference's stream-order packets (onpu_*_buf upload format)
    kSrcInt4K = 1,      // int4 two's complement packed 2/byte along K (low nibble first) + fp16 scales
    kSrcCodes = 2,      // plain codes q [N][K] (0..15) + 16-bit scales/mins [N][K/32]
};

struct RepackParams {
    int src_kind;
    const uint8_t *src;        // stream bytes / packed int4 / codes
    const uint16_t *scales;    // kSrcInt4K, kSrcCodes
    const uint16_t *mins;      // kSrcCodes (q4nx)
    const int *src_row;        // optional: GPU row -> source row (row interleaving), null = identity
    int64_t N, K;              // logical matrix
    int fmt;                   // GPU format (decides symmetric padding and the mins section)
    // reference stream-order geometry (kSrcStream)
    int R, S, tiles, kc;
    int64_t ks, rows_col, cb;
    int pkt;
    uint8_t *dst;              // GPU layout, make_gpu_matrix(N, K, fmt).bytes
};
cudaError_t repack_launch(const RepackParams &p, cudaStream_t stream);

// GPU layout -> plain codes (q [N][K], scales [N][K/32], mins) for bit-exact checks.
cudaError_t unpack_gpu_launch(const uint8_t *src, int64_t N, int64_t K, int fmt, uint8_t *q, uint16_t *s,
                              uint16_t *m, cudaStream_t stream);

// ---- small elementwise kernels (misc.cu)
// jobs[0 .. ceil(rows / 16)) = the descriptors of a dense GEMV over rows consecutive rows of weights
// w (16 rows per job), and flags[0 .. nflags) = 0; one small launch
cudaError_t dense_jobs_launch(GemvJob *jobs, const uint8_t *w, int rows, unsigned *flags, int nflags,
                              cudaStream_t stream);
// fp32 -> bf16 bits with the reference's rounding (RNE; NaN -> quiet NaN), rows x cols with strides.
cudaError_t f32_to_bf16_launch(const float *x, int64_t rows, int64_t cols, int64_t ldx, uint16_t *out, int64_t ldo,
                               cudaStream_t stream);
// a[r][i] = act(h[r] + gu_bias[ids[r]]) in fp32 (the reference's moe_act output type), act 0 =
// silu(gate) * up, 1 = gpt-oss clamped gate.
cudaError_t moe_act_f32_launch(const float *h, int64_t ldh, int64_t rows, int64_t Ng, const int32_t *ids,
                               const float *gu_bias, int act, float alpha, float limit, float *a, int64_t lda,
                               cudaStream_t stream);
// y[t][n] = sum_j w[t][j] * (o[(t*k + j)][n] + bias[ids[t*k+j]][n]) in slot order.
// Only slots whose expert id lies in [id_lo, id_hi) contribute (expert parallelism: this rank's
// experts); the default range takes every slot.
cudaError_t moe_combine_launch(const float *o, int64_t ldo, int64_t T, int k, int64_t N, const int32_t *ids,
                               const float *w, const float *bias, float *y, int64_t ldy, cudaStream_t stream,
                               int id_lo = INT32_MIN, int id_hi = INT32_MAX);

// ---- decode attention (attn.cu)
struct AttnParams {
    const float *q;                   // [Hq][D]
    const void *k, *v;                // fp32 or bf16 cache: head kh, row j at kh * hs + j * rs (elements)
    const float *mask, *sinks;        // [S] additive / [Hq] extra logits, or null
    float *out;                       // [Hq][D]
    int Hq, D, Hkv;
    int64_t S, hs, rs;
    float scale;
    int tile_rows, rows_per_split, splits;
    float *part_ml, *part_o;          // [Hq][splits][2] (max, sum), [Hq][splits][D] (16-byte aligned)
};
// tensor-core form (bf16 cache, D 64 / 128, <= 8 query heads per kv head): each CTA of
// attn_tc_warps() warps covers rows_per_split rows (a multiple of warps * attn_tc_rows())
bool attn_use_tc(int D, int rep, bool bf16);
int attn_tc_warps();
int attn_tc_rows();
int attn_ctas_per_sm(int D, int rep, bool bf16);
int attn_tile_rows(int D, bool bf16);
int attn_smem_bytes(int D, int rep, int R, bool bf16);
cudaError_t attn_launch(const AttnParams &p, bool bf16, cudaStream_t stream);

}  // namespace onpu_b200
