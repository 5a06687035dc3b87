// int4 group-32 weight-only GEMV for B200 (decode: 1..16 activation rows per weight pass).
//
// Replaces the reference's NPU GEMV (opennpu/native/npu4/kernels/gemv_any.cc:63-149, gv_acc /
// gv_flush, driven by llama/ggml-opennpu/opennpu_core.hpp:418-505) and its 8-token variant
// (gemm8.cc:58-139). Same arithmetic contract: y = x . W^T with W dequantised per 32 along K and
// fp32 accumulation; unlike the NPU it neither rounds the dequantised weight nor the K-slice
// partial sums to bf16, so it is closer to the reference's CPU path (reference.py:24-28, :55-57).
//
// Design (HBM-bound: 0.5625 B per weight, read once):
//  * Work = the chunk sequence of all jobs ([job][row group][64-K chunk], 2304 or 2560 B each,
//    contiguous per job). The grid is at most one resident wave of CTAs; CTA i owns an equal
//    contiguous range of chunks.
//  * Per CTA, one producer warp and four consumer warps. The producer streams the range
//    HBM -> shared memory with 1-D bulk copies (cp.async.bulk, mbarrier transaction counts, no
//    multicast), NS stages of CPS chunks, recycled through "empty" mbarriers.
//  * Activations: a single-job launch whose tokens fit keeps them resident in shared memory
//    (loaded once by the consumers after griddepcontrol.wait), so the copy engine only carries
//    weights; otherwise each stage also carries one 128-B copy per token per chunk.
//  * Consumer warp s owns strip s (16 rows) of every chunk. Codes become exact bf16 values
//    (128 + q) with one LOP3 per code pair (the shifts run on the FMA pipe as mul.hi by opaque
//    powers of two), minus the offset in one bf16x2 op, and the dot products run on the tensor
//    cores (mma.sync m16n8k16, bf16 x bf16 -> fp32) with tokens on the MMA's N axis; then
//    acc += scale * D per 32-group in fp32. Weights are never rounded.
//  * A row group split between CTAs is the tail segment of its first contributor and the head
//    segment of each later one. Later contributors store their head partial sums and raise a flag
//    (release store, no waiting); the first contributor, at the end of its range, waits for those
//    flags (bounded) and adds the partials to its registers in CTA order - deterministic. Waits
//    only point at higher-numbered CTAs and the grid is one resident wave, so they terminate.
//  * Programmatic dependent launch: the weight prefetch (constant data) is issued before
//    griddepcontrol.wait, so a kernel's weight stream overlaps the previous kernel's tail.
//  * Every wait is bounded (2 s of global time); a timed-out wait sets the error word and the
//    warp keeps draining the pipeline without computing, so no copy is left in flight at exit.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gpu_layout.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

constexpr int kConsumers = 4;                      // one warp per 16-row strip
constexpr int kThreads = (kConsumers + 1) * 32;    // + the producer warp
constexpr int kCPS = 4, kNS = 8;                   // chunks per stage, stages
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // a copy that has not landed in 2 s is a fault
constexpr int kSlotFloats = 4 * 8 * 2 * 16;        // [strip][r][h][token] head partial sums of a CTA
constexpr int kXSlot = 192;                        // per-stage activation slot: 128 B + 64 B pad

__host__ __device__ constexpr int stage_w_bytes(int fmt) { return kCPS * chunk_bytes(fmt); }

// two 16-bit scale/min values (strip rows r, r+8) -> fp32; mul[3] = 2^16 (an FMA-pipe shift)
template <int FMT>
__device__ __forceinline__ void decode_pair(uint32_t w, const uint32_t (&mul)[4], float &lo, float &hi) {
    if constexpr (FMT == kFmtQ4F16) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w));
        lo = f.x;
        hi = f.y;
    } else {
        lo = __uint_as_float(w * mul[3]);
        hi = __uint_as_float(w & 0xffff0000u);
    }
}

// Codes of one packed word -> the four bf16x2 A registers (128 + q). The right shifts are
// mul.hi by 2^28 / 2^24 / 2^20 passed in as kernel parameters: they run on the FMA pipe instead
// of the half-rate integer pipe, which the mask-and-OR (LOP3) already keeps busy.
__device__ __forceinline__ void codes_to_a(uint32_t w, const uint32_t (&mul)[4], uint32_t (&a)[4]) {
    a[0] = (w & 0x000F000Fu) | 0x43004300u;
    a[1] = (__umulhi(w, mul[0]) & 0x000F000Fu) | 0x43004300u;
    a[2] = (__umulhi(w, mul[1]) & 0x000F000Fu) | 0x43004300u;
    a[3] = (__umulhi(w, mul[2]) & 0x000F000Fu) | 0x43004300u;
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                         const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

__device__ __forceinline__ int worker_of(int c, int W, int T) {
    return static_cast<int>((static_cast<int64_t>(c + 1) * W - 1) / T);
}

// One strip (16 rows) x one chunk (2 groups of 32 along K) into acc. wsb: the strip's bytes in
// shared memory; xa[nt]: shared address of this lane's 8 activations of the chunk's first group
// for n-tile nt (the second group is 64 B further; absent tokens read zeros).
// Without a table (CI false): symmetric codes (128+q) - 136 = q - 8 exactly in bf16,
// D = sum((q-8) x), acc += s * D; q4nx (128+q) - 128 = q, acc += s * sum(q x) + m * sum(x), with
// sum(x) from an MMA against ones. With a table (CI true, resident activations): the MMA starts
// from c * sum(x) read from shared memory at ca (+ gi * 8 * MT; c = -136 symmetric, -128 q4nx),
// so the 128 + q codes go into the MMA as they are.
template <int FMT, int NT, bool CI>
__device__ __forceinline__ void strip_chunk(uint32_t wsb, const uint32_t (&xa)[NT], uint32_t ca, int lane, int r,
                                            const uint32_t (&mul)[4], float (&acc)[NT][4]) {
    const uint32_t off = FMT == kFmtQ4NX ? 0x43004300u : 0x43084308u;   // bf16x2 (128) / (136)
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t bx[2][NT][4];
#pragma unroll
    for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint4 v = lds_v4(xa[nt] + gi * 64);
            bx[gi][nt][0] = v.x; bx[gi][nt][1] = v.y; bx[gi][nt][2] = v.z; bx[gi][nt][3] = v.w;
        }
    const uint4 code = lds_v4(wsb + lane * 16);
    const uint2 sc = lds_v2(wsb + kCodeBytes + r * 8);
    uint2 mn = make_uint2(0, 0);
    if constexpr (FMT == kFmtQ4NX) mn = lds_v2(wsb + kCodeBytes + kScaleBytes + r * 8);
    constexpr int MT = 8 * NT;
    float cinit[2][NT][4];
    if constexpr (CI) {
#pragma unroll
        for (int gi = 0; gi < 2; ++gi)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint2 c2 = lds_v2(ca + (gi * MT + nt * 8) * 4);
                cinit[gi][nt][0] = cinit[gi][nt][2] = __uint_as_float(c2.x);
                cinit[gi][nt][1] = cinit[gi][nt][3] = __uint_as_float(c2.y);
            }
    }
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
        uint32_t a0[4], a1[4];
        codes_to_a(gi ? code.z : code.x, mul, a0);
        codes_to_a(gi ? code.w : code.y, mul, a1);
        if constexpr (!CI) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a0[i] = bf16x2_sub(a0[i], off);
                a1[i] = bf16x2_sub(a1[i], off);
            }
        }
        float s_lo, s_hi;
        decode_pair<FMT>(gi ? sc.y : sc.x, mul, s_lo, s_hi);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float d[4];
            if constexpr (CI) mma16816(d, a0, bx[gi][nt][0], bx[gi][nt][1], cinit[gi][nt]);
            else mma16816(d, a0, bx[gi][nt][0], bx[gi][nt][1], zero4);
            mma16816(d, a1, bx[gi][nt][2], bx[gi][nt][3], d);
            acc[nt][0] = fmaf(s_lo, d[0], acc[nt][0]);
            acc[nt][1] = fmaf(s_lo, d[1], acc[nt][1]);
            acc[nt][2] = fmaf(s_hi, d[2], acc[nt][2]);
            acc[nt][3] = fmaf(s_hi, d[3], acc[nt][3]);
            if constexpr (FMT == kFmtQ4NX && CI) {
                float m_lo, m_hi;
                decode_pair<FMT>(gi ? mn.y : mn.x, mul, m_lo, m_hi);
                m_lo *= -0.0078125f;                       // cinit = -128 sum(x): m * sum(x)
                m_hi *= -0.0078125f;
                acc[nt][0] = fmaf(m_lo, cinit[gi][nt][0], acc[nt][0]);
                acc[nt][1] = fmaf(m_lo, cinit[gi][nt][1], acc[nt][1]);
                acc[nt][2] = fmaf(m_hi, cinit[gi][nt][2], acc[nt][2]);
                acc[nt][3] = fmaf(m_hi, cinit[gi][nt][3], acc[nt][3]);
            }
            if constexpr (FMT == kFmtQ4NX && !CI) {
                float m_lo, m_hi, xs[4];
                decode_pair<FMT>(gi ? mn.y : mn.x, mul, m_lo, m_hi);
                const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
                mma16816(xs, ones, bx[gi][nt][0], bx[gi][nt][1], zero4);
                mma16816(xs, ones, bx[gi][nt][2], bx[gi][nt][3], xs);
                acc[nt][0] = fmaf(m_lo, xs[0], acc[nt][0]);
                acc[nt][1] = fmaf(m_lo, xs[1], acc[nt][1]);
                acc[nt][2] = fmaf(m_hi, xs[2], acc[nt][2]);
                acc[nt][3] = fmaf(m_hi, xs[3], acc[nt][3]);
            }
        }
    }
}

// Store the finished sums of strip rows r (v_lo) and r+8 (v_hi) of one token (output row yr).
template <int EPI>
__device__ __forceinline__ void store_pair(const GemvParams &p, int g, int s, int r, int yr, float v_lo, float v_hi) {
    if (yr < 0) return;
    if constexpr (EPI == kEpiSwiGLU) {
        const int i = g * (kRowGroup / 2) + s * 8 + r;       // gate row r, up row r+8 of the strip
        if (i < p.N / 2)
            reinterpret_cast<__nv_bfloat16 *>(p.y)[static_cast<int64_t>(yr) * p.ldy + i] =
                __float2bfloat16_rn(silu_f(v_lo) * v_hi);
    } else {
        const int row = g * kRowGroup + s * kStripRows + r;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int rr = row + 8 * h;
            if (rr < p.N) {
                const int col = p.row_map ? p.row_map[rr] : rr;
                const int64_t o = static_cast<int64_t>(yr) * p.ldy + col;
                const float v = h ? v_hi : v_lo;
                if constexpr (EPI == kEpiF32) reinterpret_cast<float *>(p.y)[o] = v;
                else reinterpret_cast<__nv_bfloat16 *>(p.y)[o] = __float2bfloat16_rn(v);
            }
        }
    }
}

template <int FMT, int NT, int EPI, bool CI>
__global__ void __launch_bounds__(kThreads, 2) gemv_int4_kernel(const GemvParams p) {
    constexpr int CB = chunk_bytes(FMT), SB = strip_bytes(FMT), STAGE_W = stage_w_bytes(FMT);
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int W = p.workers, T = p.total_chunks, cta = blockIdx.x;
    const int lo = static_cast<int>(static_cast<int64_t>(cta) * T / W);
    const int hi = static_cast<int>(static_cast<int64_t>(cta + 1) * T / W);
    const int nst = (hi - lo + kCPS - 1) / kCPS;
    const int per_job = p.row_groups * p.chunks;
    constexpr bool xres = CI;                         // resident activations carry the offset table
    const int xchunk = p.xslots * kXSlot, stage_x = kCPS * xchunk;   // per-stage activation layout
    const uint32_t sbase = smem_u32(smem);
    const uint32_t wring = sbase, xregion = sbase + kNS * STAGE_W;
    const uint32_t full = sbase + p.off_bar, empty = full + kNS * 8;

    if (!xres)   // the zero slot is never written; a chunk half past K gets a 64-B copy only
        for (int e = threadIdx.x; e < kNS * stage_x / 16; e += blockDim.x)
            *reinterpret_cast<uint4 *>(smem + kNS * STAGE_W + e * 16) = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kNS; ++s) {
            mbar_init(full + s * 8, xres ? 1 : 2);   // weights arrival (+ activations arrival)
            mbar_init(empty + s * 8, kConsumers);
        }
        mbar_init_fence();
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ============================================================ producer
        int wj = lo / per_job;                        // weight cursor: job of the next chunk
        const uint8_t *wbase = p.jobs_ready ? p.jobs[wj].w : nullptr;
        auto issue_weights = [&](int st) {            // lane 0 only
            const int c0 = lo + st * kCPS, c1 = min(hi, c0 + kCPS);
            const uint32_t bar = full + (st % kNS) * 8;
            mbar_arrive_expect_tx(bar, static_cast<uint32_t>((c1 - c0) * CB));
            uint32_t dst = wring + (st % kNS) * STAGE_W;
            int c = c0;
            while (c < c1) {                          // one copy per run of chunks within a job
                if (c >= (wj + 1) * per_job) wbase = p.jobs[++wj].w;
                const int run_end = min(c1, (wj + 1) * per_job);
                bulk_g2s(dst, wbase + static_cast<int64_t>(c - wj * per_job) * CB,
                         static_cast<uint32_t>((run_end - c) * CB), bar);
                dst += (run_end - c) * CB;
                c = run_end;
            }
        };
        const int npro = min(kNS, nst);
        if (lane == 0 && p.jobs_ready)
            for (int st = 0; st < npro; ++st) issue_weights(st);
        pdl_launch_dependents();
        pdl_wait_prerequisites();                     // activations may come from the previous kernel
        if (lane == 0 && !p.jobs_ready) {
            wbase = p.jobs[wj].w;
            for (int st = 0; st < npro; ++st) issue_weights(st);
        }
        __syncwarp();

        // activation cursor (per-stage mode): chunk -> (job, k chunk); lane holds xrow[lane & 15]
        int cj = lo / per_job, ckc = (lo - cj * per_job) % p.chunks;
        int xm = p.jobs[cj].m, xrow = p.jobs[cj].xrow[lane & 15];
        bool failed = false;
        for (int st = 0; st < nst; ++st) {
            const int slot = st % kNS;
            if (st >= kNS) {
                if (!failed && !mbar_wait_bounded(empty + slot * 8, ((st / kNS) - 1) & 1, kWaitLimitNs)) {
                    failed = true;
                    if (lane == 0) atomicOr(p.err, 2);
                }
                __syncwarp();
                if (lane == 0) issue_weights(st);
            }
            if (xres) continue;
            // activations of this stage: per chunk one 128-B copy per token (64 B when the chunk's
            // second group lies past K); the byte total is announced first
            const int c0 = lo + st * kCPS, c1 = min(hi, c0 + kCPS);
            uint32_t xbytes = 0;
            {
                int jj = cj, kk = ckc, mm = xm;
                for (int c = c0; c < c1; ++c) {
                    xbytes += static_cast<uint32_t>(mm * min(128, 2 * (p.K - kk * kChunkK)));
                    if (++kk == p.chunks) {
                        kk = 0;
                        if ((c + 1) % per_job == 0 && c + 1 < hi) mm = p.jobs[++jj].m;
                    }
                }
            }
            if (lane == 0) mbar_arrive_expect_tx(full + slot * 8, xbytes);
            __syncwarp();
            for (int c = c0; c < c1; ++c) {
                const int k0 = ckc * kChunkK;
                const uint32_t nb = static_cast<uint32_t>(min(128, 2 * (p.K - k0)));
                if (lane < xm)
                    bulk_g2s(xregion + slot * stage_x + (c - c0) * xchunk + lane * kXSlot,
                             p.x + static_cast<int64_t>(xrow) * p.ldx + k0, nb, full + slot * 8);
                if (++ckc == p.chunks) {
                    ckc = 0;
                    if ((c + 1) % per_job == 0 && c + 1 < hi) {
                        ++cj;
                        xm = p.jobs[cj].m;
                        xrow = p.jobs[cj].xrow[lane & 15];
                    }
                }
            }
        }
        return;
    }

    // ================================================================ consumers (strip s = warp)
    const int s = warp, r = lane >> 2, t = lane & 3;
    volatile int *flag = reinterpret_cast<volatile int *>(smem + p.off_bar + 2 * kNS * 8);
    pdl_launch_dependents();
    pdl_wait_prerequisites();                         // x / outputs / scratch may belong to the previous kernel

    int j = lo / per_job;
    int g = (lo - j * per_job) / p.chunks;
    int kc = lo - j * per_job - g * p.chunks;
    int seg = lo;
    int m = p.jobs[j].m;

    if (xres) {
        // resident activations: token rows of xstride bytes, then one zero block of 128 B
        const int n16 = p.K / 8, row16 = p.xstride / 16;   // 16-B pieces: data, row incl. zero pad
        for (int e = threadIdx.x; e < m * row16; e += kConsumers * 32) {
            const int n = e / row16, q = e - n * row16;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (q < n16) v = ld_nc_v4(p.x + static_cast<int64_t>(p.jobs[j].xrow[n]) * p.ldx + q * 8);
            *reinterpret_cast<uint4 *>(smem + kNS * STAGE_W + n * p.xstride + q * 16) = v;
        }
        if (threadIdx.x < 8)
            *reinterpret_cast<uint4 *>(smem + kNS * STAGE_W + m * p.xstride + threadIdx.x * 16) = make_uint4(0, 0, 0, 0);
        named_bar_sync(1, kConsumers * 32);
        // offset table [k chunk][group][token slot] = c * sum of the token's 32 activations
        constexpr int MT = 8 * NT;
        const float c = FMT == kFmtQ4NX ? -128.0f : -136.0f;
        float *tab = reinterpret_cast<float *>(smem + kNS * STAGE_W + p.ctab_off);
        for (int e = threadIdx.x; e < p.chunks * 2 * MT; e += kConsumers * 32) {
            const int tok = e % MT, grp = e / MT;             // grp = k chunk * 2 + group
            float sum = 0.f;
            if (tok < m && grp * 32 < p.K) {
                const uint8_t *row = smem + kNS * STAGE_W + tok * p.xstride + grp * 64;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(row + q * 16);
                    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) sum += __uint_as_float(w4[i] << 16) + __uint_as_float(w4[i] & 0xffff0000u);
                }
            }
            tab[e] = c * sum;
        }
        named_bar_sync(1, kConsumers * 32);
    }

    int yr[NT][2];
    uint32_t xrb[NT], xkm[NT];                        // activation base and per-chunk stride of this lane
    auto load_rows = [&]() {
        m = p.jobs[j].m;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int tok = nt * 8 + r;
            if (xres) {
                xrb[nt] = xregion + (tok < m ? tok * p.xstride : m * p.xstride) + t * 16;
                xkm[nt] = tok < m ? 128u : 0u;        // absent tokens stay on the zero block
            } else {
                xrb[nt] = xregion + (tok < m ? tok : p.xslots - 1) * kXSlot + t * 16;
                xkm[nt] = 0u;
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int tk = nt * 8 + 2 * t + h;
                yr[nt][h] = tk < m ? p.jobs[j].yrow[tk] : -1;
            }
        }
    };
    load_rows();

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int f = 0; f < 4; ++f) acc[nt][f] = 0.f;

    // Close segment [a, b) of row group (j, g) for this strip.
    auto flush = [&](int a, int b) {
        const int gstart = (j * p.row_groups + g) * p.chunks;
        if (a == gstart && b == gstart + p.chunks) {          // the whole row group is here
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int h = 0; h < 2; ++h) store_pair<EPI>(p, g, s, r, yr[nt][h], acc[nt][h], acc[nt][2 + h]);
            return;
        }
        const int cf = worker_of(gstart, W, T), cl = worker_of(gstart + p.chunks - 1, W, T);
        if (cta != cf) {
            // head segment of a later contributor: publish the partial sums
            float *slot = p.part + static_cast<int64_t>(cta) * kSlotFloats;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int f = 0; f < 4; ++f) {
                    const int tok = nt * 8 + 2 * t + (f & 1);
                    if (tok < m) slot[((s * 8 + r) * 2 + (f >> 1)) * 16 + tok] = acc[nt][f];
                }
            named_bar_sync(1, kConsumers * 32);
            if (threadIdx.x == 0) st_release_gpu(p.counters + cta, 1u);
            return;
        }
        // tail segment of the first contributor: collect cf+1 .. cl (bounded wait on their flags)
        if (warp == 0) {
            for (int w2 = cf + 1 + lane; w2 <= cl; w2 += 32) {
                const uint64_t t0 = global_timer_ns();
                while (ld_acquire_gpu(p.counters + w2) == 0u) {
                    __nanosleep(256);
                    if (global_timer_ns() - t0 > kWaitLimitNs) {
                        atomicOr(p.err, 4);
                        break;
                    }
                }
                p.counters[w2] = 0u;                          // consumed: ready for the next launch
            }
        }
        named_bar_sync(1, kConsumers * 32);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int f = 0; f < 4; ++f) {
                const int tok = nt * 8 + 2 * t + (f & 1);
                if (tok < m) {
                    float v = acc[nt][f];
                    const int e = ((s * 8 + r) * 2 + (f >> 1)) * 16 + tok;
#pragma unroll 4
                    for (int w2 = cf + 1; w2 <= cl; ++w2) v += __ldcg(p.part + static_cast<int64_t>(w2) * kSlotFloats + e);
                    acc[nt][f] = v;
                }
            }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) store_pair<EPI>(p, g, s, r, yr[nt][h], acc[nt][h], acc[nt][2 + h]);
    };
    (void)flag;

    const uint32_t mul[4] = {p.mul[0], p.mul[1], p.mul[2], p.mul[3]};
    auto advance = [&](int c) {                       // chunk c finished: close its row group?
        if (++kc == p.chunks) {
            flush(seg, c + 1);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int f = 0; f < 4; ++f) acc[nt][f] = 0.f;
            seg = c + 1;
            kc = 0;
            if (++g == p.row_groups) {
                g = 0;
                ++j;
                if (c + 1 < hi) load_rows();
            }
        }
    };
    // this lane's activation addresses for chunk ci of the current stage (k chunk kcc)
    auto xaddr = [&](uint32_t (&xa)[NT], uint32_t xstage, int ci, int kcc) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) xa[nt] = xrb[nt] + (xres ? kcc * xkm[nt] : xstage + ci * xchunk);
    };
    // offset-table address of this lane's tokens 2t, 2t+1 for k chunk kcc (resident mode)
    const uint32_t ctab = xregion + p.ctab_off + t * 8;
    auto caddr = [&](int kcc) { return ctab + kcc * (2 * 8 * NT * 4); };

    bool failed = false;
    for (int st = 0; st < nst; ++st) {
        const int slot = st % kNS;
        if (!failed && !mbar_wait_bounded(full + slot * 8, (st / kNS) & 1, kWaitLimitNs)) {
            failed = true;
            if (lane == 0) atomicOr(p.err, 1);
        }
        const int c0 = lo + st * kCPS, n = min(hi - c0, kCPS);
        const uint32_t wsb = wring + slot * STAGE_W + s * SB, xstage = slot * stage_x;
        if (failed) {
            // drain only: keep the barriers moving, skip the math and the outputs
        } else if (n == kCPS && kc + kCPS < p.chunks) {
            // the common case: a full stage inside one row group
#pragma unroll
            for (int ci = 0; ci < kCPS; ++ci) {
                uint32_t xa[NT];
                xaddr(xa, xstage, ci, kc + ci);
                strip_chunk<FMT, NT, CI>(wsb + ci * CB, xa, caddr(kc + ci), lane, r, mul, acc);
            }
            kc += kCPS;
        } else {
            for (int ci = 0; ci < n; ++ci) {
                uint32_t xa[NT];
                xaddr(xa, xstage, ci, kc);
                strip_chunk<FMT, NT, CI>(wsb + ci * CB, xa, caddr(kc), lane, r, mul, acc);
                advance(c0 + ci);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot * 8);
    }
    if (!failed && seg < hi) flush(seg, hi);
}

template <int FMT, int NT, int EPI, bool CI>
struct GemvKernel {
    static void prepare() {
        static bool done = false;
        if (!done) {
            done = true;
            cudaFuncSetAttribute(gemv_int4_kernel<FMT, NT, EPI, CI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 227 * 1024);
        }
    }
    static int occupancy(int smem) {
        prepare();
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, gemv_int4_kernel<FMT, NT, EPI, CI>, kThreads, smem) !=
            cudaSuccess)
            o = 1;
        return o > 0 ? o : 1;
    }
    static cudaError_t launch(const GemvParams &p, int smem, cudaStream_t stream, bool pdl) {
        prepare();
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(p.workers);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, gemv_int4_kernel<FMT, NT, EPI, CI>, p);
    }
};

template <int FMT, int NT, bool CI>
cudaError_t dispatch_epi_ci(int epi, const GemvParams &p, int smem, cudaStream_t s, bool pdl) {
    switch (epi) {
        case kEpiF32: return GemvKernel<FMT, NT, kEpiF32, CI>::launch(p, smem, s, pdl);
        case kEpiBF16: return GemvKernel<FMT, NT, kEpiBF16, CI>::launch(p, smem, s, pdl);
        case kEpiSwiGLU: return GemvKernel<FMT, NT, kEpiSwiGLU, CI>::launch(p, smem, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

template <int FMT, int NT>
cudaError_t dispatch_epi(int epi, const GemvParams &p, int smem, cudaStream_t s, bool pdl) {
    return p.xres ? dispatch_epi_ci<FMT, NT, true>(epi, p, smem, s, pdl)
                  : dispatch_epi_ci<FMT, NT, false>(epi, p, smem, s, pdl);
}

template <int FMT>
cudaError_t dispatch_nt(int nt, int epi, const GemvParams &p, int smem, cudaStream_t s, bool pdl) {
    return nt == 1 ? dispatch_epi<FMT, 1>(epi, p, smem, s, pdl) : dispatch_epi<FMT, 2>(epi, p, smem, s, pdl);
}

template <int FMT>
int occ_fmt(int nt, int smem) {
    return nt == 1 ? GemvKernel<FMT, 1, kEpiF32, true>::occupancy(smem) : GemvKernel<FMT, 2, kEpiF32, true>::occupancy(smem);
}

}  // namespace

GemvLayout gemv_layout(int fmt, int njobs, int mmax, int64_t K) {
    GemvLayout L{};
    const int64_t xstride = (K * 2 + 127) / 128 * 128 + 64;   // rows 64 B off mod 128: conflict-free
    const int64_t mt = mmax > 8 ? 16 : 8;
    const int64_t chunks = (K + kChunkK - 1) / kChunkK;
    const int64_t res_bytes = mmax * xstride + 128 + chunks * 2 * mt * 4;   // rows, zero block, offset table
    L.xres = njobs == 1 && res_bytes <= kResidentXBudget;
    L.xstride = static_cast<int>(xstride);
    L.ctab_off = static_cast<int>(mmax * xstride + 128);
    L.xslots = mmax + 1;
    const int64_t xbytes = L.xres ? res_bytes : static_cast<int64_t>(kNS) * kCPS * L.xslots * kXSlot;
    L.off_bar = static_cast<int>(kNS * stage_w_bytes(fmt) + (xbytes + 15) / 16 * 16);
    L.smem = L.off_bar + 2 * kNS * 8 + 16;
    return L;
}

int gemv_ctas_per_sm(int fmt, int ntiles, int smem) {
    if (fmt == kFmtQ4NX) return occ_fmt<kFmtQ4NX>(ntiles, smem);
    if (fmt == kFmtQ4S) return occ_fmt<kFmtQ4S>(ntiles, smem);
    return occ_fmt<kFmtQ4F16>(ntiles, smem);
}

int gemv_chunks_per_stage() { return kCPS; }

int64_t gemv_part_floats_per_worker(int ntiles) {
    (void)ntiles;
    return kSlotFloats;
}

cudaError_t gemv_launch(int fmt, int ntiles, int epi, const GemvParams &p, int smem, cudaStream_t stream, bool pdl) {
    switch (fmt) {
        case kFmtQ4NX: return dispatch_nt<kFmtQ4NX>(ntiles, epi, p, smem, stream, pdl);
        case kFmtQ4S: return dispatch_nt<kFmtQ4S>(ntiles, epi, p, smem, stream, pdl);
        case kFmtQ4F16: return dispatch_nt<kFmtQ4F16>(ntiles, epi, p, smem, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace onpu_b200
