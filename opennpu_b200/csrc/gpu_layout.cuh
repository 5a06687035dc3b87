// The int4 weight layout libonpu keeps in B200 HBM, and the descriptors the kernels share.
//
// A matrix W [N][K] (K % 32 == 0; one 16-bit scale, and for q4nx one 16-bit min, per 32 weights
// along K) is stored as row groups of 64 rows; each row group as chunks of 64 along K; each chunk
// as 4 "strips" of 16 rows:
//
//   matrix  = [ceil(N/64) row groups][ceil(K/64) chunks][4 strips][strip bytes]
//   strip   = 512 B codes | 64 B scales | (q4nx) 64 B mins         (576 or 640 B)
//
// so a chunk is 2304 B (q4s / int4-fp16) or 2560 B (q4nx), and any run of chunks in a row group
// (or across row groups) is one contiguous byte range: the GEMV streams it with 1-D bulk copies.
//
// Inside a strip the 512 code bytes are 32 lanes x 16 B: lane L = 4r + t (r = L/4, t = L%4) owns
// the codes its mma.sync.m16n8k16 A fragments need for strip rows r and r+8, K offsets
// 8t .. 8t+7 of both 32-groups of the chunk. Word w = 2*gi + j (gi = group in the chunk, j = k16
// step) holds 8 codes at bits 4p, p = i + 4h, for A register i (0..3) and half h (0/1):
//     strip row  = r + 8*(i & 1)
//     K in group = 8t + 4j + 2*(i >> 1) + h
// so (w >> 4i) & 0x000F000F puts the two codes of A register i into its two 16-bit halves, and
// OR-ing 0x43004300 makes them the exact bf16 values 128 + q. Because every lane's 8 K offsets of
// a group are contiguous, its B fragments (activations) are one 16-B load per group.
// Scales: [r 0..7][gi 0..1][h 0..1] 16-bit values, the scale of strip row r + 8h in group gi;
// a lane loads its 4 with one 8-B load. Mins (q4nx) use the same order.
//
// Codes are always q in 0..15: q4nx w = q*s + m (bf16 s, m); q4s w = (q-8)*d (bf16 d); the
// int4/fp16 format (int4 v in [-8, 7], fp16 scale) stores q = v + 8, w = (q-8)*s. Padding rows
// or columns carry q = 8 (symmetric) or 0 (q4nx) with zero scale/min, and contribute 0.
#pragma once
#include <cstdint>

namespace onpu_b200 {

enum WeightFormat : int {
    kFmtQ4NX = 0,   // asymmetric, bf16 scale + bf16 min      (reference "q4nx", sym = 0)
    kFmtQ4S = 1,    // symmetric, bf16 scale                  (reference "q4s", sym = 1)
    kFmtQ4F16 = 2,  // symmetric int4 [-8, 7], fp16 scale     (packed-along-K int4 + fp16 ingest)
};

// Version of the weights' device layout below (row groups, chunks, strips, code and scale order).
// Saved weight blobs (onpu_dense_export and friends) carry it; a blob of another version is refused.
constexpr int kGpuLayoutVersion = 1;

constexpr int kRowGroup = 64;
constexpr int kStripRows = 16;
constexpr int kChunkK = 64;
constexpr int kCodeBytes = 512;
constexpr int kScaleBytes = 64;
constexpr int kMaxTokensPerJob = 16;   // two n8 MMA tiles

__host__ __device__ constexpr int strip_bytes(int fmt) { return fmt == kFmtQ4NX ? 640 : 576; }
__host__ __device__ constexpr int chunk_bytes(int fmt) { return 4 * strip_bytes(fmt); }

struct GpuMatrix {
    int64_t N = 0, K = 0;
    int fmt = kFmtQ4S;
    int row_groups = 0, chunks = 0;    // ceil(N/64), ceil(K/64)
    int64_t bytes = 0;
};

inline GpuMatrix make_gpu_matrix(int64_t N, int64_t K, int fmt) {
    GpuMatrix g;
    g.N = N;
    g.K = K;
    g.fmt = fmt;
    g.row_groups = static_cast<int>((N + kRowGroup - 1) / kRowGroup);
    g.chunks = static_cast<int>((K + kChunkK - 1) / kChunkK);
    g.bytes = static_cast<int64_t>(g.row_groups) * g.chunks * chunk_bytes(fmt);
    return g;
}

// One GEMV job: up to 16 activation rows against one matrix (an expert, or the dense matrix).
struct GemvJob {
    const uint8_t *w;                  // GPU-layout matrix
    int m;                             // tokens in this job (1..16)
    int pad_;
    int xrow[kMaxTokensPerJob];        // activation row of token n
    int yrow[kMaxTokensPerJob];        // output row of token n
};

enum GemvEpilogue : int {
    kEpiF32 = 0,      // y[yrow][n] = acc (fp32)
    kEpiBF16 = 1,     // y[yrow][n] = bf16(acc)
    kEpiSwiGLU = 2,   // strip rows 0-7 gate, 8-15 up: y[yrow][i] = bf16(silu(gate_i) * up_i) (fp32 with yf32)
    kEpiPairSum = 3,  // strip rows 0-7 a row, 8-15 its residual: y[yrow][i] = row_i + residual_i (fp32)
    kEpiPeer = 4,     // row-parallel projection + all-reduce: each finished output goes to every rank's
                      // buffer as an 8-byte {value, call} word; after its range, a CTA waits for every
                      // rank's words of the rows it finished and writes their sum (fp32 y, bf16 y_bf16)
};

// GEMV tracing: per CTA, ns stamps of kernel entry, producer's first copy issued, consumers past
// griddepcontrol.wait, activations staged, first weight stage arrived, last stage consumed, range
// flushed (split row groups closed), and the ns the consumers waited for weights in total
constexpr int kGemvTrace = 12;

constexpr int kPeerMaxRanks = 8;       // ranks of the peer-memory all-reduce (comm.cu)
constexpr int kPeerCtaCounters = 1024; // call counters of the GEMV CTAs that sum rows (kEpiPeer)

struct GemvParams {
    const GemvJob *jobs;
    int njobs;
    int N, K;                          // every job's matrix shape (logical)
    int row_groups, chunks;            // of one job
    int total_chunks;                  // njobs * row_groups * chunks
    int workers;                       // CTAs sharing the chunk sequence (at most one resident wave)
    const uint16_t *x;                 // bf16 activations, row stride ldx (elements)
    int64_t ldx;
    void *y;                           // output rows, stride ldy (elements of the output type)
    int64_t ldy;
    const int *row_map;                // optional: GPU row -> output column (fp32/bf16 epilogues)
    float *part;                       // split row groups: head partial sums, [workers][4][8][2][16]
    unsigned *counters;                // [workers] partial-ready flags, zero between launches
    int *err;                          // set non-zero on a timed-out wait
    int jobs_ready;                    // job list not written by the previous kernel in the stream
    const int *njobs_dev;              // non-null: the job count lives on the device (written by the
                                       // previous kernel); njobs / total_chunks are upper bounds
    unsigned long long *trace;         // non-null: %globaltimer stamps, kGemvTrace per CTA
    uint32_t mul[4];                   // 2^28, 2^24, 2^20, 2^16: shift multipliers the compiler cannot fold
    uint32_t unpk[3];                  // 0x000F000F, 0x00F000F0, 0x64006400 (fp16 code unpacking)
    int xslots;                        // per-stage activations: slots per chunk (max tokens + 1 zero slot)
    int xres;                          // activations resident in shared memory (single job)
    int xstride;                       // resident: bytes per token row
    int ctab_off;                      // resident: offset table position in the activation region
    int off_bar;                       // shared-memory offset of the mbarriers
    int wchunks;                       // resident: 64-K chunks the activation region holds per row
    int kwin;                          // resident, one job: each CTA stages only its own chunk range's
                                       // part of K (every range is at most wchunks long)
    int xsplit;                        // resident: activations are fp32 (xf); token n is staged as two fp16
                                       // rows (x rounded, and the rounding error) whose sums are added at
                                       // the store; jobs hold at most 8 tokens
    const float *xf;                   // xsplit: fp32 activations, row stride ldx (elements)
    int yf32;                          // kEpiSwiGLU: fp32 outputs instead of bf16
    // kEpiPeer: every output value goes, with the all-reduce call number, into slot [parity][rank]
    // of each rank's buffer (comm.cu layout); CTA i's call number is peer_calls[i] + 1 (one counter
    // per CTA in this rank's buffer, advanced by the CTA when its rows are summed)
    void *peer[kPeerMaxRanks];
    int peer_rank, peer_world;
    int64_t peer_cap;
    uint32_t *peer_calls;
    void *y_bf16;                      // kEpiPeer: the summed rows also as bf16 (may be null)
    uint64_t peer_wait_ns;             // kEpiPeer: how long a CTA waits for a peer rank's words
};

// One link of a GEMV chain: y = x . W^T for m consecutive activation rows, run inside one
// persistent launch together with the other links (chain.cu).
struct ChainOp {
    const uint8_t *w;                  // GPU-layout matrix
    const uint16_t *x;                 // bf16 activations, rows 0..m-1, stride ldx (elements)
    void *y;                           // output rows 0..m-1, stride ldy (elements of the output type)
    const int *row_map;                // optional: GPU row -> output column (fp32/bf16 epilogues)
    int64_t ldx, ldy;
    int N, K;                          // logical shape
    int row_groups, chunks;            // GPU layout
    int epi;                           // GemvEpilogue
    int dep;                           // last earlier link whose outputs/inputs overlap this one (-1: none)
    int m;                             // tokens (1..16)
    int xstride;                       // bytes per resident activation row in shared memory
    int ctab_off;                      // offset table position in the activation region
    int pad_;
};

struct ChainParams {
    const ChainOp *ops;
    int nops;
    int workers;                       // CTAs (one resident wave); every link is split over all of them
    float *part;                       // [kChainRing][workers][2][slot] partial sums of split row groups
    unsigned *flags;                   // [kChainRing][workers][2] slot in use (zero at rest)
    unsigned *rgcnt;                   // [nops][workers] arrivals per split row group (by first contributor)
    unsigned *done;                    // [nops] workers finished per link, then one exit counter
    int *err;
    uint32_t mul[4];
    uint32_t unpk[3];                  // 0x000F000F, 0x00F000F0, 0x64006400 (fp16 code unpacking)
    int ns;                            // ring stages
    int off_x, off_comb, off_bar;      // shared memory: activation region, combine buffer, mbarriers
    unsigned long long *trace;         // optional: [workers][nops][kChainTrace] global-timer stamps
};

// Prefill dequant-GEMM (dqgemm.cu): Y[M][N] = X[M][K] . W^T for many tokens.
struct DqGemmParams {
    const uint8_t *w;                  // GPU-layout matrix
    int N, K;                          // logical shape (K a multiple of 32)
    int row_groups, chunks;            // GPU layout
    int M;                             // tokens
    void *y;                           // [M][ldy] fp32 / bf16 (or bf16 [M][N/2] for SwiGLU)
    int64_t ldy;
    const int *row_map;                // optional: GPU row -> output column (fp32/bf16 epilogues)
    const float *tscale;               // [M] per-token scale of the fp16 activation copy
    int *err;
    uint32_t unpk[3];                  // 0x000F000F, 0x00F000F0, 0x64006400
};

constexpr int kChainRing = 4;          // links whose split-row partials may be outstanding at once
// trace stamps per (CTA, link): consumer start, dependency met, activations staged, math done,
// link counted; producer first copy issued, last copy issued; then the nanoseconds consumer
// warp 0 spent waiting for weight stages during the link
constexpr int kChainTrace = 8;

}  // namespace onpu_b200
