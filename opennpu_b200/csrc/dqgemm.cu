// int4 group-32 dequant-GEMM for prefill (many tokens per weight pass) on the 5th-generation
// tensor cores: Y[M][N] = X[M][K] . W^T, W in the GPU layout (int4 codes + per-32 scales).
//
// Replaces the reference's multi-token NPU path (the 8-token GEMM opennpu/native/npu4/kernels/
// gemm8.cc:33-139 run ceil(M/8) times, and the MLIR-AIR prefill devices cited in
// opennpu/native/prefill.py:107-256 for shapes only). Arithmetic contract as the reference's
// dequantise-then-matmul (reference.py:24-28): W dequantised per 32 along K, fp32 accumulation.
// Here the dequantised weight is rounded once to fp16 and the activations are fp16 (exact for
// bf16 inputs in the fp16 range; a token beyond it is scaled by a power of two and unscaled in
// the epilogue): both tensor-core operands must have one type, and bf16 weights would round
// 8x coarser.
//
// Persistent CTAs (one per SM) walk 256 (tokens) x 128 (weight rows) tiles; the fp32 accumulators
// of a tile (two 128-token halves sharing each dequantised weight tile) live in tensor memory,
// double-buffered so that one tile's epilogue overlaps the next tile's main loop. Warp roles:
//  * warp 0: one thread issues the copies: the fp16 activation tile of each 64-K stage through a
//    128-byte-swizzled tensor map (TMA, no multicast), and the int4 chunks of the tile's two row
//    groups as 1-D bulk copies into a raw ring.
//  * warp 1: allocates tensor memory; one thread issues tcgen05.mma kind::f16 (M128 N128 K16,
//    eight per stage: two token halves x four K steps) from shared-memory descriptors and commits
//    each stage's completion to the mbarrier that frees the stage.
//  * warps 2-9: dequantise each raw chunk into the stage's fp16 B tile in the canonical K-major
//    128-byte-swizzled layout (a lane's 16 bytes of codes are two 8-K runs of two rows: one LOP3,
//    one f16x2 subtract and one f16x2 multiply per pair of weights, 16-byte stores).
//  * warps 10-13: read a finished tile's accumulators with tcgen05.ld (each warp its 32 lanes),
//    apply the epilogue and store, then hand the buffer back to warp 1.
// Every wait is bounded (2 s of global time) and reports through the error word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdio>

#include "gpu_layout.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

constexpr int kTM = 256, kTN = 128, kTK = 64;           // CTA tile: tokens, weight rows, K per stage
constexpr int kMmaM = 128;                              // one MMA: 128 tokens x kTN rows x 16 K
constexpr int kOpStages = 4, kRawStages = 4;
constexpr int kXTile = kTM * kTK * 2;                   // 32 KB fp16 activations (256 rows of 128 B)
constexpr int kWTile = kTN * kTK * 2;                   // 16 KB fp16 weights
constexpr int kRawMax = 2 * 2560;                       // two row groups' chunk (q4nx is largest)
constexpr int kDqWarps = 8, kEpiWarps = 4;              // warps 2..9 dequantise, 10..13 store
constexpr int kGThreads = (2 + kDqWarps + kEpiWarps) * 32;
constexpr int kAccCols = 2 * kTN;                       // one tile's accumulators: 2 x 128 tokens
constexpr int kTmemCols = 2 * kAccCols;                 // double-buffered: 512 columns (all of it)
constexpr uint64_t kWaitNs = 2000000000ull;

constexpr int smem_bytes() {
    return 1024 /* alignment slack */ + kOpStages * (kXTile + kWTile) + kRawStages * kRawMax +
           (2 * kOpStages + 2 * kRawStages + 4) * 8 + 16;
}

// ---------------------------------------------------------------- tcgen05 / TMA
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B in 8-row atoms 1024 B
// apart (stride byte offset), start address in 16-byte units; version 1 (Blackwell). The tile
// base is 1024-aligned, so the base offset is 0.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused when swizzled)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset
    d |= static_cast<uint64_t>(1) << 46;                  // descriptor version
    d |= static_cast<uint64_t>(2) << 61;                  // SWIZZLE_128B
    return d;
}

// Instruction descriptor for kind::f16: fp32 accumulator, fp16 A and B, both K-major, N and M.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(kTN >> 3) << 17) |
                            (static_cast<uint32_t>(kMmaM >> 4) << 24);

// byte offset of 16-byte chunk c (0..7, 8 fp16 along K) of row n in a K-major 128-byte-swizzled tile
__device__ __forceinline__ uint32_t swz(int n, int c) {
    return static_cast<uint32_t>((n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4));
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 16-bit scale (fp16, or bf16 for the reference formats) -> fp16 bits
template <int FMT>
__device__ __forceinline__ uint32_t to_f16_bits(uint32_t v16) {
    if constexpr (FMT == kFmtQ4F16) return v16;
    return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(__uint_as_float(v16 << 16))));
}

// The epilogue of one accumulator chunk: 32 outputs (columns nb..nb+31) of token `row`.
template <int EPI>
__device__ __forceinline__ void store_chunk(const DqGemmParams &p, int row, int nb, float tsc, bool vec_ok,
                                            const uint32_t (&v)[32]) {
    if constexpr (EPI == kEpiSwiGLU) {
        // columns are GPU rows: strip rows 0-7 gate, 8-15 up of output 8 * strip + r; a full
        // strip's 8 outputs go out as one 16-byte store when the row allows it
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int strip = (nb >> 4) + h;
            if (strip * 16 >= p.N) continue;
            __nv_bfloat16 *out = reinterpret_cast<__nv_bfloat16 *>(p.y) + static_cast<int64_t>(row) * p.ldy + strip * 8;
            uint32_t pk[4];
#pragma unroll
            for (int r8 = 0; r8 < 8; r8 += 2) {
                float o2[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float gte = __uint_as_float(v[h * 16 + r8 + e]) * tsc;
                    const float up = __uint_as_float(v[h * 16 + 8 + r8 + e]) * tsc;
                    o2[e] = __fdividef(gte, 1.0f + __expf(-gte)) * up;
                }
                pk[r8 / 2] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(o2[0]))) |
                             (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(o2[1]))) << 16);
            }
            if (vec_ok && strip * 8 + 8 <= p.N / 2) {
                *reinterpret_cast<uint4 *>(out) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            } else {
#pragma unroll
                for (int r8 = 0; r8 < 8; ++r8)
                    if (strip * 8 + r8 < p.N / 2)
                        reinterpret_cast<uint16_t *>(out)[r8] = static_cast<uint16_t>(pk[r8 / 2] >> (16 * (r8 & 1)));
            }
        }
    } else if (vec_ok && !p.row_map && nb + 32 <= p.N) {
        // 32 consecutive outputs of this token: 16-byte stores
        if constexpr (EPI == kEpiF32) {
            float4 *out = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.y) + static_cast<int64_t>(row) * p.ldy + nb);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                out[j] = make_float4(__uint_as_float(v[4 * j]) * tsc, __uint_as_float(v[4 * j + 1]) * tsc,
                                     __uint_as_float(v[4 * j + 2]) * tsc, __uint_as_float(v[4 * j + 3]) * tsc);
        } else {
            uint4 *out = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.y) + static_cast<int64_t>(row) * p.ldy + nb);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t pk[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    pk[e] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[8 * j + 2 * e]) * tsc))) |
                            (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[8 * j + 2 * e + 1]) * tsc))) << 16);
                out[j] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int n = nb + j;
            if (n >= p.N) break;
            const int col = p.row_map ? p.row_map[n] : n;
            const float val = __uint_as_float(v[j]) * tsc;
            const int64_t o = static_cast<int64_t>(row) * p.ldy + col;
            if constexpr (EPI == kEpiF32) reinterpret_cast<float *>(p.y)[o] = val;
            else reinterpret_cast<__nv_bfloat16 *>(p.y)[o] = __float2bfloat16_rn(val);
        }
    }
}

// Persistent: CTA c takes tiles c, c + gridDim.x, ... (tokens fastest, so the CTAs running at one
// time share weight tiles through L2); every role walks the same tile sequence and the stage rings
// run on across tiles. Tensor memory holds two tiles' accumulators, so the epilogue warps drain
// one tile while the next one accumulates.
template <int FMT, int EPI>
__global__ void __launch_bounds__(kGThreads, 1)
    dqgemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ DqGemmParams p) {
    constexpr int CB = chunk_bytes(FMT), SB = strip_bytes(FMT);
    extern __shared__ uint8_t smem_raw[];
    const uint32_t s0 = smem_u32(smem_raw), sb = (s0 + 1023u) & ~1023u;
    uint8_t *base = smem_raw + (sb - s0);
    const uint32_t xs = sb, ws = xs + kOpStages * kXTile, raw = ws + kOpStages * kWTile;
    const uint32_t bars = raw + kRawStages * kRawMax;
    const uint32_t op_full = bars, op_empty = op_full + kOpStages * 8, raw_full = op_empty + kOpStages * 8,
                   raw_empty = raw_full + kRawStages * 8, acc_full = raw_empty + kRawStages * 8,
                   acc_empty = acc_full + 2 * 8;
    const uint32_t tmem_slot = acc_empty + 2 * 8;
    volatile uint32_t *tmem_slot_p = reinterpret_cast<volatile uint32_t *>(base + (tmem_slot - sb));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mtiles = (p.M + kTM - 1) / kTM, ntiles = (p.N + kTN - 1) / kTN, tiles = mtiles * ntiles;
    const int nk = p.chunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kOpStages; ++s) {
            mbar_init(op_full + s * 8, 1 + kDqWarps);      // producer (with the copy bytes) + the dequant warps
            mbar_init(op_empty + s * 8, 1);                // tcgen05.commit
        }
        for (int r = 0; r < kRawStages; ++r) {
            mbar_init(raw_full + r * 8, 1);
            mbar_init(raw_empty + r * 8, kDqWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b * 8, 1);                // tcgen05.commit after a tile's last MMA
            mbar_init(acc_empty + b * 8, kEpiWarps);       // the epilogue warps have read the buffer
        }
        mbar_init_fence();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot_p;

    if (warp == 0) {
        // ============================================================ copies
        if (lane == 0) {
            bool failed = false;
            int stage = 0;
            for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
                const int m0 = (t % mtiles) * kTM, g0 = (t / mtiles) * (kTN / kRowGroup);
                const int nvalid = (g0 < p.row_groups) + (g0 + 1 < p.row_groups);
                for (int kt = 0; kt < nk; ++kt, ++stage) {
                    const int r = stage % kRawStages, rr = stage / kRawStages;
                    if (rr > 0 && !mbar_wait_bounded(raw_empty + r * 8, (rr - 1) & 1, kWaitNs)) {
                        failed = true;
                        break;
                    }
                    mbar_arrive_expect_tx(raw_full + r * 8, static_cast<uint32_t>(nvalid * CB));
                    for (int gg = 0; gg < 2; ++gg)
                        if (g0 + gg < p.row_groups)
                            bulk_g2s(raw + r * kRawMax + gg * CB,
                                     p.w + (static_cast<int64_t>(g0 + gg) * p.chunks + kt) * CB, CB, raw_full + r * 8);
                    const int s = stage % kOpStages, sr = stage / kOpStages;
                    if (sr > 0 && !mbar_wait_bounded(op_empty + s * 8, (sr - 1) & 1, kWaitNs)) {
                        failed = true;
                        break;
                    }
                    mbar_arrive_expect_tx(op_full + s * 8, kXTile);
                    tma_load_2d(xs + s * kXTile, &tmap_x, kt * kTK, m0, op_full + s * 8);
                }
            }
            if (failed) atomicOr(p.err, 64);
        }
    } else if (warp == 1) {
        // ============================================================ tensor-core issue
        if (lane == 0) {
            bool failed = false;
            int stage = 0, li = 0;
            for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++li) {
                const int b = li & 1, use = li >> 1;
                if (!failed && use > 0 && !mbar_wait_bounded(acc_empty + b * 8, (use - 1) & 1, kWaitNs)) failed = true;
                tc_fence_after();
                const uint32_t d0 = tmem + b * kAccCols, d1 = d0 + kTN;
                for (int kt = 0; kt < nk; ++kt, ++stage) {
                    const int s = stage % kOpStages, sr = stage / kOpStages;
                    if (!failed && !mbar_wait_bounded(op_full + s * 8, sr & 1, kWaitNs)) failed = true;
                    tc_fence_after();
                    if (!failed) {
                        const uint32_t xa = xs + s * kXTile, wb = ws + s * kWTile;
#pragma unroll
                        for (int kk = 0; kk < kTK / 16; ++kk) {
                            const uint64_t bdesc = sw128_desc(wb + kk * 32);
                            const uint32_t acc = (kt | kk) != 0 ? 1u : 0u;
                            tc_mma_f16(d0, sw128_desc(xa + kk * 32), bdesc, kIdesc, acc);
                            tc_mma_f16(d1, sw128_desc(xa + kMmaM * 128 + kk * 32), bdesc, kIdesc, acc);
                        }
                    }
                    tc_commit(op_empty + s * 8);           // also after a failure: keeps the rings moving
                }
                tc_commit(acc_full + b * 8);               // arrives once the tile's MMAs have completed
            }
            if (failed) atomicOr(p.err, 128);
        }
    } else if (warp < 2 + kDqWarps) {
        // ============================================================ dequantise
        const int dt = threadIdx.x - 64;                   // one 16-byte code block per thread and stage
        const int gg = dt >> 7, st = (dt >> 5) & 3, L = dt & 31, rq = L >> 2, tq = L & 3;
        const uint32_t mlo = p.unpk[0], magic = p.unpk[2];
        const uint32_t c_off = FMT == kFmtQ4NX ? 0x64006400u : 0x64086408u;   // 1024 / 1032 in f16x2
        const int nlo = gg * kRowGroup + st * kStripRows + rq, nhi = nlo + 8;
        bool failed = false;
        int stage = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            const int g0 = (t / mtiles) * (kTN / kRowGroup);
            const bool valid = g0 + gg < p.row_groups;
            for (int kt = 0; kt < nk; ++kt, ++stage) {
                const int r = stage % kRawStages, rr = stage / kRawStages, s = stage % kOpStages, sr = stage / kOpStages;
                if (!failed && !mbar_wait_bounded(raw_full + r * 8, rr & 1, kWaitNs)) failed = true;
                if (!failed && sr > 0 && !mbar_wait_bounded(op_empty + s * 8, (sr - 1) & 1, kWaitNs)) failed = true;
                if (!failed && valid) {
                    const uint32_t sbase = raw + r * kRawMax + gg * CB + st * SB;
                    uint8_t *wtile = base + (ws + s * kWTile - sb);
                    const uint4 code = lds_v4(sbase + L * 16);
                    const uint2 sc = lds_v2(sbase + kCodeBytes + rq * 8);
                    uint2 mn = make_uint2(0, 0);
                    if constexpr (FMT == kFmtQ4NX) mn = lds_v2(sbase + kCodeBytes + kScaleBytes + rq * 8);
                    // lanes of odd rows take the groups in the other order: within each 8-lane
                    // phase of a 16-byte store, rows rq and rq^1 then hit eight different 16-byte
                    // units of the swizzled row (no shared-memory bank conflicts)
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const int gi = k ^ (rq & 1);
                        const uint32_t sp = gi ? sc.y : sc.x;
                        const uint32_t slo = to_f16_bits<FMT>(sp & 0xffffu), shi = to_f16_bits<FMT>(sp >> 16);
                        const uint32_t slo2 = slo | (slo << 16), shi2 = shi | (shi << 16);
                        uint32_t mlo2 = 0, mhi2 = 0;
                        if constexpr (FMT == kFmtQ4NX) {
                            const uint32_t mp = gi ? mn.y : mn.x;
                            const uint32_t ma = to_f16_bits<FMT>(mp & 0xffffu), mb = to_f16_bits<FMT>(mp >> 16);
                            mlo2 = ma | (ma << 16);
                            mhi2 = mb | (mb << 16);
                        }
                        uint32_t rlo[4], rhi[4];
#pragma unroll
                        for (int j = 0; j < 2; ++j) {
                            const uint32_t w = gi ? (j ? code.w : code.z) : (j ? code.y : code.x);
                            uint32_t a4[4];
                            a4[0] = lop3_and_or(w, mlo, magic);
                            a4[1] = lop3_and_or(w >> 4, mlo, magic);
                            a4[2] = lop3_and_or(w >> 8, mlo, magic);
                            a4[3] = lop3_and_or(w >> 12, mlo, magic);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t q = hsub2(a4[i], c_off);         // exact: q - 8 (q4nx: q)
                                if constexpr (FMT == kFmtQ4NX) a4[i] = hfma2(q, (i & 1) ? shi2 : slo2, (i & 1) ? mhi2 : mlo2);
                                else a4[i] = hmul2(q, (i & 1) ? shi2 : slo2);
                            }
                            rlo[2 * j] = a4[0];
                            rlo[2 * j + 1] = a4[2];
                            rhi[2 * j] = a4[1];
                            rhi[2 * j + 1] = a4[3];
                        }
                        *reinterpret_cast<uint4 *>(wtile + swz(nlo, gi * 4 + tq)) = make_uint4(rlo[0], rlo[1], rlo[2], rlo[3]);
                        *reinterpret_cast<uint4 *>(wtile + swz(nhi, gi * 4 + tq)) = make_uint4(rhi[0], rhi[1], rhi[2], rhi[3]);
                    }
                    fence_proxy_async_smem();              // generic stores -> tensor-core reads
                }
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(op_full + s * 8);
                    mbar_arrive(raw_empty + r * 8);
                }
            }
        }
        if (failed && lane == 0) atomicOr(p.err, 256);
    } else {
        // ============================================================ epilogue
        // warp w reads tensor-memory lanes 32 (w % 4) .. +31 of both accumulators of a tile
        const int quarter = warp & 3;
        constexpr int kOutBytes = EPI == kEpiF32 ? 4 : 2;
        const bool vec_ok = (reinterpret_cast<uintptr_t>(p.y) & 15) == 0 && (p.ldy * kOutBytes) % 16 == 0;
        bool failed = false;
        int li = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++li) {
            const int b = li & 1, use = li >> 1;
            const bool ok = !failed && mbar_wait_bounded(acc_full + b * 8, use & 1, kWaitNs);
            if (!ok) failed = true;
            tc_fence_after();
            const int m0 = (t % mtiles) * kTM, n0 = (t / mtiles) * kTN;
#pragma unroll 1
            for (int a = 0; a < 2; ++a) {
                const int row = m0 + a * kMmaM + quarter * 32 + lane;
                const float tsc = row < p.M ? p.tscale[row] : 0.f;
#pragma unroll 1
                for (int c = 0; c < kTN / 32; ++c) {
                    uint32_t v[32];
                    __syncwarp();                          // tcgen05.ld is warp-collective
                    tc_ld_32x32b_x32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + b * kAccCols + a * kTN + c * 32, v);
                    if (ok && row < p.M) store_chunk<EPI>(p, row, n0 + c * 32, tsc, vec_ok, v);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + b * 8);
        }
        if (failed && lane == 0) atomicOr(p.err, 512);
    }

    // ---- teardown: the epilogue has waited for every tile's MMAs, so tensor memory is idle
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// One CTA per token row: fp16 copy of the row, scaled by 2^-e when max |x| > 2^15 (tscale = 2^e).
__global__ void __launch_bounds__(256) x_to_f16_kernel(const uint16_t *x, int64_t ldx, int K, uint16_t *xh,
                                                       float *tscale) {
    __shared__ float red[8];
    const int row = blockIdx.x;
    const uint16_t *src = x + static_cast<int64_t>(row) * ldx;
    uint16_t *dst = xh + static_cast<int64_t>(row) * K;
    float mx = 0.f;
    for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
        const uint4 v = ld_nc_v4(src + k);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(w4[i] << 16)), fabsf(__uint_as_float(w4[i] & 0xffff0000u))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
    const float e = mx > 32768.0f ? ceilf(log2f(mx * (1.0f / 32768.0f))) : 0.0f;
    const float inv = exp2f(-e);
    for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
        const uint4 v = ld_nc_v4(src + k);
        uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float lo = __uint_as_float(w4[i] << 16) * inv, hi = __uint_as_float(w4[i] & 0xffff0000u) * inv;
            w4[i] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(lo))) |
                    (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(hi))) << 16);
        }
        *reinterpret_cast<uint4 *>(dst + k) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
    if (threadIdx.x == 0) tscale[row] = exp2f(e);
}

template <int FMT, int EPI>
cudaError_t launch_t(const CUtensorMap &map, const DqGemmParams &p, cudaStream_t s) {
    static bool attr = false;
    if (!attr) {
        attr = true;
        cudaFuncSetAttribute(dqgemm_kernel<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes());
    }
    static int nsm = 0;
    if (!nsm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if (nsm <= 0) nsm = 1;
    }
    const int tiles = ((p.M + kTM - 1) / kTM) * ((p.N + kTN - 1) / kTN);
    dqgemm_kernel<FMT, EPI><<<tiles < nsm ? tiles : nsm, kGThreads, smem_bytes(), s>>>(map, p);
    return cudaGetLastError();
}

template <int FMT>
cudaError_t launch_fmt(int epi, const CUtensorMap &map, const DqGemmParams &p, cudaStream_t s) {
    switch (epi) {
        case kEpiF32: return launch_t<FMT, kEpiF32>(map, p, s);
        case kEpiBF16: return launch_t<FMT, kEpiBF16>(map, p, s);
        case kEpiSwiGLU: return launch_t<FMT, kEpiSwiGLU>(map, p, s);
        default: return cudaErrorInvalidValue;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

}  // namespace

int dqgemm_tile_tokens() { return kTM; }

cudaError_t x_to_f16_launch(const uint16_t *x, int64_t ldx, int M, int K, uint16_t *xh, float *tscale,
                            cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    x_to_f16_kernel<<<M, 256, 0, stream>>>(x, ldx, K, xh, tscale);
    return cudaGetLastError();
}

cudaError_t dqgemm_launch(int fmt, int epi, const uint16_t *xh, const DqGemmParams &p, cudaStream_t stream) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    CUtensorMap map;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.K), static_cast<cuuint64_t>(p.M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.K) * 2};
    const cuuint32_t box[2] = {kTK, kTM}, estr[2] = {1, 1};
    if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t *>(xh), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    switch (fmt) {
        case kFmtQ4NX: return launch_fmt<kFmtQ4NX>(epi, map, p, stream);
        case kFmtQ4S: return launch_fmt<kFmtQ4S>(epi, map, p, stream);
        case kFmtQ4F16: return launch_fmt<kFmtQ4F16>(epi, map, p, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace onpu_b200
