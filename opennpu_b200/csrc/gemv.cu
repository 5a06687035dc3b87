// int4 group-32 weight-only GEMV for B200 (decode: 1..16 activation rows per weight pass).
//
// Replaces the reference's NPU GEMV (opennpu/native/npu4/kernels/gemv_any.cc:63-149, gv_acc /
// gv_flush, driven by llama/ggml-opennpu/opennpu_core.hpp:418-505) and its 8-token variant
// (gemm8.cc:58-139). Same arithmetic contract: y = x . W^T with W dequantised per 32 along K and
// fp32 accumulation; unlike the NPU it neither rounds the dequantised weight nor the K-slice
// partial sums to bf16, so it is closer to the reference's CPU path (reference.py:24-28, :55-57).
//
// Design (HBM-bound; ~0.56 B of weights per MAC pair at M=1):
//  * Work = the chunk sequence of all jobs ([job][row group][64-K chunk], 2304/2560 B each,
//    contiguous per job). Every warp is an independent worker owning an equal contiguous range
//    (split evenly over the grid, which is sized to whole waves of the 148 SMs).
//  * Each warp streams its range HBM -> its own shared-memory ring with 1-D bulk copies
//    (cp.async.bulk, mbarrier transaction counts, NS stages of CPS chunks) and consumes it with
//    128-bit shared loads.
//  * Codes become exact bf16 values 128+q with one LOP3 per code pair; the dot products run on
//    the tensor cores (mma.sync m16n8k16, bf16 x bf16 -> fp32), tokens on the MMA's N axis. The
//    offset is removed without per-code work: the accumulator of each 32-group starts at
//    c * sum(x) (c = -136 for symmetric codes, -128 for q4nx) from one extra MMA against a
//    constant A, so D = sum((q - 8) x) (or sum(q x)), then acc += scale * D in fp32 (+ min *
//    sum(x) for q4nx). Only the 16-bit scale multiplies per group; the weights are never rounded.
//  * A row group split between warps is finished by the last of its warps to arrive (atomic
//    counter): partial sums go to a scratch slot per warp, the last arriver adds them in worker
//    order, so the result is deterministic.
//  * Programmatic dependent launch: the weight prefetch (which depends on nothing) is issued
//    before griddepcontrol.wait, so a kernel's stream overlaps the previous kernel's tail.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gpu_layout.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

constexpr int kWarps = 4;                         // warps (workers) per CTA
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: a bulk copy that never lands is a fault

template <int FMT, int NT, int CPS, int NS>
struct Cfg {
    static constexpr int SB = strip_bytes(FMT);
    static constexpr int CB = chunk_bytes(FMT);
    static constexpr int STAGE = CPS * CB;
    static constexpr int RING = NS * STAGE;
    static constexpr int SMEM = kWarps * RING + kWarps * NS * 8;
};

// two 16-bit scale/min values (strip rows r, r+8) -> fp32
template <int FMT>
__device__ __forceinline__ void decode_pair(uint32_t w, float &lo, float &hi) {
    if constexpr (FMT == kFmtQ4F16) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w));
        lo = f.x;
        hi = f.y;
    } else {
        lo = __uint_as_float(w << 16);
        hi = __uint_as_float(w & 0xffff0000u);
    }
}

__device__ __forceinline__ void codes_to_a(uint32_t w, uint32_t (&a)[4]) {
    a[0] = (w & 0x000F000Fu) | 0x43004300u;
    a[1] = ((w >> 4) & 0x000F000Fu) | 0x43004300u;
    a[2] = ((w >> 8) & 0x000F000Fu) | 0x43004300u;
    a[3] = ((w >> 12) & 0x000F000Fu) | 0x43004300u;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

__device__ __forceinline__ int worker_of(int c, int W, int T) {
    return static_cast<int>((static_cast<int64_t>(c + 1) * W - 1) / T);
}

template <int NT>
struct JobRegs {
    const uint16_t *xp[NT];   // activation row of token (8*nt + r), or null
    int yr[NT][2];            // output rows of tokens 8*nt + 2t, +1 (-1: none)
    int m;
};

template <int NT>
__device__ __forceinline__ void load_job(const GemvParams &p, int j, int r, int t, JobRegs<NT> &jr) {
    const GemvJob &job = p.jobs[j];
    jr.m = job.m;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int n = nt * 8 + r;
        jr.xp[nt] = n < jr.m ? p.x + static_cast<int64_t>(job.xrow[n]) * p.ldx : nullptr;
        const int t0 = nt * 8 + 2 * t;
        jr.yr[nt][0] = t0 < jr.m ? job.yrow[t0] : -1;
        jr.yr[nt][1] = t0 + 1 < jr.m ? job.yrow[t0 + 1] : -1;
    }
}

// Write one row group's finished sums (vals[strip][ntile][frag]) through the epilogue.
template <int EPI, int NT>
__device__ __forceinline__ void epilogue(const GemvParams &p, int g, int r, const JobRegs<NT> &jr,
                                         const float (&vals)[4][NT][4]) {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            if constexpr (EPI == kEpiSwiGLU) {
                const int i = g * (kRowGroup / 2) + s * 8 + r;   // strip rows r (gate), r+8 (up)
                if (i < p.N / 2) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int yr = jr.yr[nt][h];
                        if (yr >= 0) {
                            const float a = silu_f(vals[s][nt][h]) * vals[s][nt][2 + h];
                            reinterpret_cast<__nv_bfloat16 *>(p.y)[static_cast<int64_t>(yr) * p.ldy + i] =
                                __float2bfloat16_rn(a);
                        }
                    }
                }
            } else {
#pragma unroll
                for (int f = 0; f < 4; ++f) {
                    const int row = g * kRowGroup + s * kStripRows + r + 8 * (f >> 1);
                    const int yr = jr.yr[nt][f & 1];
                    if (row < p.N && yr >= 0) {
                        const int col = p.row_map ? p.row_map[row] : row;
                        const int64_t o = static_cast<int64_t>(yr) * p.ldy + col;
                        if constexpr (EPI == kEpiF32) reinterpret_cast<float *>(p.y)[o] = vals[s][nt][f];
                        else reinterpret_cast<__nv_bfloat16 *>(p.y)[o] = __float2bfloat16_rn(vals[s][nt][f]);
                    }
                }
            }
        }
    }
}

// partial-sum slot layout: [strip][ntile][token in tile (8)][strip row (16)] floats
__device__ __forceinline__ int part_index(int s, int nt, int NT, int tok, int row) {
    return ((s * NT + nt) * 8 + tok) * 16 + row;
}

template <int FMT, int NT, int EPI, int CPS, int NS>
__global__ void __launch_bounds__(kWarps * 32) gemv_int4_kernel(const GemvParams p) {
    using C = Cfg<FMT, NT, CPS, NS>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, t = lane & 3;
    const int wid = blockIdx.x * kWarps + warp;
    const int W = p.workers, T = p.total_chunks;
    const bool active = wid < W;
    const int lo = active ? static_cast<int>(static_cast<int64_t>(wid) * T / W) : 0;
    const int hi = active ? static_cast<int>(static_cast<int64_t>(wid + 1) * T / W) : 0;
    const int nst = (hi - lo + CPS - 1) / CPS;
    const int per_job = p.row_groups * p.chunks;
    const uint32_t ring = smem_u32(smem + warp * C::RING);
    const uint32_t bars = smem_u32(smem + kWarps * C::RING) + warp * NS * 8;

    auto issue = [&](int st) {   // lane 0: bulk-copy the chunks of stage st into its ring slot
        const int c0 = lo + st * CPS, c1 = min(hi, c0 + CPS);
        const uint32_t bar = bars + (st % NS) * 8;
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>((c1 - c0) * C::CB));
        uint32_t dst = ring + (st % NS) * C::STAGE;
        for (int c = c0; c < c1; ++c) {
            const int j = c / per_job;
            const uint8_t *src = p.jobs[j].w + static_cast<int64_t>(c - j * per_job) * C::CB;
            bulk_g2s(dst, src, C::CB, bar);
            dst += C::CB;
        }
    };

    if (active && lane == 0) {
        for (int s = 0; s < NS; ++s) mbar_init(bars + s * 8, 1);
        mbar_init_fence();
        // Weights are written before any launch that reads them; when the job list is too
        // (jobs_ready), the weight prefetch starts before the previous kernel has finished.
        if (p.jobs_ready)
            for (int st = 0; st < min(NS, nst); ++st) issue(st);
    }
    __syncwarp();
    pdl_launch_dependents();
    pdl_wait_prerequisites();   // activations / outputs / scratch may belong to the previous kernel
    if (!active) return;
    if (!p.jobs_ready && lane == 0)
        for (int st = 0; st < min(NS, nst); ++st) issue(st);
    __syncwarp();

    const uint32_t cA = FMT == kFmtQ4NX ? 0xC300C300u : 0xC308C308u;   // bf16x2 (-128) / (-136)
    const uint32_t constA[4] = {cA, cA, cA, cA};

    int j = lo / per_job;
    int g = (lo - j * per_job) / p.chunks;
    int kc = lo - j * per_job - g * p.chunks;
    int seg = lo;                                  // first chunk of the open segment
    JobRegs<NT> jr;
    load_job<NT>(p, j, r, t, jr);

    float acc[4][NT][4];
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int f = 0; f < 4; ++f) acc[s][nt][f] = 0.f;

    // Close segment [a, b) of row group (j, g): direct epilogue when this warp holds the whole
    // row group, else a partial slot; the last of the row group's warps adds them up.
    auto flush = [&](int a, int b) {
        const int gstart = (j * p.row_groups + g) * p.chunks;
        if (a == gstart && b == gstart + p.chunks) {
            epilogue<EPI, NT>(p, g, r, jr, acc);
            return;
        }
        float *slot = p.part + static_cast<int64_t>(wid * 2 + (a == lo ? 0 : 1)) * (4 * NT * 8 * 16);
#pragma unroll
        for (int s = 0; s < 4; ++s)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int f = 0; f < 4; ++f) {
                    const int tok = 2 * t + (f & 1);
                    if (nt * 8 + tok < jr.m) slot[part_index(s, nt, NT, tok, r + 8 * (f >> 1))] = acc[s][nt][f];
                }
        __threadfence();
        __syncwarp();
        unsigned old = 0;
        const int ctr = j * p.row_groups + g;
        if (lane == 0) old = atomicAdd(p.counters + ctr, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        const int wf = worker_of(gstart, W, T), wl = worker_of(gstart + p.chunks - 1, W, T);
        if (old != static_cast<unsigned>(wl - wf)) return;
        __threadfence();
        float red[4][NT][4];
#pragma unroll
        for (int s = 0; s < 4; ++s)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int f = 0; f < 4; ++f) red[s][nt][f] = 0.f;
        for (int w2 = wf; w2 <= wl; ++w2) {
            const int lo2 = static_cast<int>(static_cast<int64_t>(w2) * T / W);
            const float *src = p.part + static_cast<int64_t>(w2 * 2 + (lo2 >= gstart ? 0 : 1)) * (4 * NT * 8 * 16);
#pragma unroll
            for (int s = 0; s < 4; ++s)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        const int tok = 2 * t + (f & 1);
                        if (nt * 8 + tok < jr.m)
                            red[s][nt][f] += __ldcg(src + part_index(s, nt, NT, tok, r + 8 * (f >> 1)));
                    }
        }
        epilogue<EPI, NT>(p, g, r, jr, red);
        if (lane == 0) atomicExch(p.counters + ctr, 0u);
    };

    bool failed = false;
    int st = 0;
    for (; st < nst; ++st) {
        const int slot = st % NS;
        if (!mbar_wait_bounded(bars + slot * 8, (st / NS) & 1, kWaitLimitNs)) {
            failed = true;
            break;
        }
        const int c0 = lo + st * CPS, c1 = min(hi, c0 + CPS);
        for (int c = c0; c < c1; ++c) {
            const uint32_t cbase = ring + slot * C::STAGE + (c - c0) * C::CB;
            // B fragments for both 32-groups of this chunk and the offset-carrying accumulators
            uint32_t bx[2][NT][4];
            float ci[2][NT][4];
#pragma unroll
            for (int gi = 0; gi < 2; ++gi) {
                const int k0 = kc * kChunkK + gi * 32 + 8 * t;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    uint4 v = make_uint4(0, 0, 0, 0);
                    if (jr.xp[nt] != nullptr && k0 < p.K) v = ld_nc_v4(jr.xp[nt] + k0);
                    bx[gi][nt][0] = v.x; bx[gi][nt][1] = v.y; bx[gi][nt][2] = v.z; bx[gi][nt][3] = v.w;
                    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
                    mma_bf16_m16n8k16(ci[gi][nt], constA, v.x, v.y, zero);
                    mma_bf16_m16n8k16(ci[gi][nt], constA, v.z, v.w, ci[gi][nt]);
                }
            }
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t sb = cbase + s * C::SB;
                const uint4 code = lds_v4(sb + lane * 16);
                const uint2 sc = lds_v2(sb + kCodeBytes + r * 8);
                uint2 mn = make_uint2(0, 0);
                if constexpr (FMT == kFmtQ4NX) mn = lds_v2(sb + kCodeBytes + kScaleBytes + r * 8);
#pragma unroll
                for (int gi = 0; gi < 2; ++gi) {
                    uint32_t a0[4], a1[4];
                    codes_to_a(gi ? code.z : code.x, a0);
                    codes_to_a(gi ? code.w : code.y, a1);
                    float s_lo, s_hi;
                    decode_pair<FMT>(gi ? sc.y : sc.x, s_lo, s_hi);
                    float m_lo = 0.f, m_hi = 0.f;
                    if constexpr (FMT == kFmtQ4NX) {
                        decode_pair<FMT>(gi ? mn.y : mn.x, m_lo, m_hi);
                        m_lo *= -0.0078125f;   // the accumulator offset is -128 sum(x)
                        m_hi *= -0.0078125f;
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        float d[4];
                        mma_bf16_m16n8k16(d, a0, bx[gi][nt][0], bx[gi][nt][1], ci[gi][nt]);
                        mma_bf16_m16n8k16(d, a1, bx[gi][nt][2], bx[gi][nt][3], d);
                        acc[s][nt][0] = fmaf(s_lo, d[0], acc[s][nt][0]);
                        acc[s][nt][1] = fmaf(s_lo, d[1], acc[s][nt][1]);
                        acc[s][nt][2] = fmaf(s_hi, d[2], acc[s][nt][2]);
                        acc[s][nt][3] = fmaf(s_hi, d[3], acc[s][nt][3]);
                        if constexpr (FMT == kFmtQ4NX) {
                            acc[s][nt][0] = fmaf(m_lo, ci[gi][nt][0], acc[s][nt][0]);
                            acc[s][nt][1] = fmaf(m_lo, ci[gi][nt][1], acc[s][nt][1]);
                            acc[s][nt][2] = fmaf(m_hi, ci[gi][nt][2], acc[s][nt][2]);
                            acc[s][nt][3] = fmaf(m_hi, ci[gi][nt][3], acc[s][nt][3]);
                        }
                    }
                }
            }
            // advance to the next chunk; a finished row group closes its segment
            if (++kc == p.chunks) {
                flush(seg, c + 1);
#pragma unroll
                for (int s = 0; s < 4; ++s)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int f = 0; f < 4; ++f) acc[s][nt][f] = 0.f;
                seg = c + 1;
                kc = 0;
                if (++g == p.row_groups) {
                    g = 0;
                    ++j;
                    if (c + 1 < hi) load_job<NT>(p, j, r, t, jr);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && st + NS < nst) {
            fence_proxy_async_smem();   // this stage's shared reads are done before it is refilled
            issue(st + NS);
        }
    }
    if (failed) {
        if (lane == 0) atomicOr(p.err, 1);
        // copies still in flight must land before the CTA's shared memory is released
        for (int s2 = st; s2 < min(nst, st + NS); ++s2)
            (void)mbar_wait_bounded(bars + (s2 % NS) * 8, (s2 / NS) & 1, kWaitLimitNs);
        return;
    }
    if (seg < hi) flush(seg, hi);
}

template <int FMT, int NT, int EPI>
struct GemvKernel {
    static constexpr int CPS = 2, NS = 4;
    using C = Cfg<FMT, NT, CPS, NS>;
    static int occupancy() {
        static int occ = -1;
        if (occ < 0) {
            auto k = gemv_int4_kernel<FMT, NT, EPI, CPS, NS>;
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
            int o = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k, kWarps * 32, C::SMEM) != cudaSuccess) o = 1;
            occ = o > 0 ? o : 1;
        }
        return occ;
    }
    static cudaError_t launch(const GemvParams &p, cudaStream_t stream, bool pdl) {
        auto k = gemv_int4_kernel<FMT, NT, EPI, CPS, NS>;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((p.workers + kWarps - 1) / kWarps);
        cfg.blockDim = dim3(kWarps * 32);
        cfg.dynamicSmemBytes = C::SMEM;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, k, p);
    }
};

template <int FMT, int NT>
cudaError_t dispatch_epi(int epi, const GemvParams &p, cudaStream_t s, bool pdl) {
    switch (epi) {
        case kEpiF32: return GemvKernel<FMT, NT, kEpiF32>::launch(p, s, pdl);
        case kEpiBF16: return GemvKernel<FMT, NT, kEpiBF16>::launch(p, s, pdl);
        case kEpiSwiGLU: return GemvKernel<FMT, NT, kEpiSwiGLU>::launch(p, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

template <int FMT>
cudaError_t dispatch_nt(int nt, int epi, const GemvParams &p, cudaStream_t s, bool pdl) {
    return nt == 1 ? dispatch_epi<FMT, 1>(epi, p, s, pdl) : dispatch_epi<FMT, 2>(epi, p, s, pdl);
}

}  // namespace

int gemv_ctas_per_sm(int fmt, int ntiles) {
    // occupancy does not depend on the epilogue (same shared memory); query one instantiation
    if (fmt == kFmtQ4NX) return ntiles == 1 ? GemvKernel<kFmtQ4NX, 1, kEpiF32>::occupancy() : GemvKernel<kFmtQ4NX, 2, kEpiF32>::occupancy();
    if (fmt == kFmtQ4S) return ntiles == 1 ? GemvKernel<kFmtQ4S, 1, kEpiF32>::occupancy() : GemvKernel<kFmtQ4S, 2, kEpiF32>::occupancy();
    return ntiles == 1 ? GemvKernel<kFmtQ4F16, 1, kEpiF32>::occupancy() : GemvKernel<kFmtQ4F16, 2, kEpiF32>::occupancy();
}

int gemv_warps_per_cta() { return kWarps; }

int64_t gemv_part_floats_per_worker(int ntiles) { return 2LL * 4 * ntiles * 8 * 16; }

cudaError_t gemv_launch(int fmt, int ntiles, int epi, const GemvParams &p, cudaStream_t stream, bool pdl) {
    // every instantiation must have had its shared-memory limit raised before its first launch
    (void)gemv_ctas_per_sm(fmt, ntiles);
    auto raise = [](auto kern, int smem) { cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); };
    static bool raised[3][2][3] = {};
    if (!raised[fmt][ntiles - 1][epi]) {
        raised[fmt][ntiles - 1][epi] = true;
#define ONPU_RAISE(F, N, E) if (fmt == F && ntiles == N && epi == E) raise(gemv_int4_kernel<F, N, E, 2, 4>, Cfg<F, N, 2, 4>::SMEM)
        ONPU_RAISE(kFmtQ4NX, 1, kEpiF32); ONPU_RAISE(kFmtQ4NX, 1, kEpiBF16); ONPU_RAISE(kFmtQ4NX, 1, kEpiSwiGLU);
        ONPU_RAISE(kFmtQ4NX, 2, kEpiF32); ONPU_RAISE(kFmtQ4NX, 2, kEpiBF16); ONPU_RAISE(kFmtQ4NX, 2, kEpiSwiGLU);
        ONPU_RAISE(kFmtQ4S, 1, kEpiF32); ONPU_RAISE(kFmtQ4S, 1, kEpiBF16); ONPU_RAISE(kFmtQ4S, 1, kEpiSwiGLU);
        ONPU_RAISE(kFmtQ4S, 2, kEpiF32); ONPU_RAISE(kFmtQ4S, 2, kEpiBF16); ONPU_RAISE(kFmtQ4S, 2, kEpiSwiGLU);
        ONPU_RAISE(kFmtQ4F16, 1, kEpiF32); ONPU_RAISE(kFmtQ4F16, 1, kEpiBF16); ONPU_RAISE(kFmtQ4F16, 1, kEpiSwiGLU);
        ONPU_RAISE(kFmtQ4F16, 2, kEpiF32); ONPU_RAISE(kFmtQ4F16, 2, kEpiBF16); ONPU_RAISE(kFmtQ4F16, 2, kEpiSwiGLU);
#undef ONPU_RAISE
    }
    switch (fmt) {
        case kFmtQ4NX: return dispatch_nt<kFmtQ4NX>(ntiles, epi, p, stream, pdl);
        case kFmtQ4S: return dispatch_nt<kFmtQ4S>(ntiles, epi, p, stream, pdl);
        case kFmtQ4F16: return dispatch_nt<kFmtQ4F16>(ntiles, epi, p, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace onpu_b200
