// The routed-expert FFN of one MoE layer as ONE persistent launch: gate/up GEMV with the SwiGLU
// epilogue, down GEMV and the weighted combine, for every expert the router selected. This is the
// GPU form of the reference's onpu_ffn_run / onpu_ffn_run_many (llama/ggml-opennpu/
// onpu_api.cpp:423-496: gate_up -> act -> down of the routed experts in one NPU dispatch); the
// arithmetic is that of the grouped GEMV path (gemv.cu + moe_combine_kernel), so both agree.
//
// Design (one resident wave of CTAs, each one producer warp + four consumer warps):
//  * Work items are whole row groups (job, row group): 64 output rows over all of K, so no row
//    group is split between CTAs and no partial sums cross CTAs. CTA w takes an equal contiguous
//    range of the gate/up items, then of the down items (consecutive items share a job, so its
//    activations are staged once); the job lists and their count come from the router kernel that
//    runs before, on the device: no host round trip, capturable in a CUDA graph.
//  * The producer streams every item's chunks, gate/up items then down items, through one ring of
//    shared-memory stages (cp.async.bulk, no multicast, L2 evict-first): the weights do not
//    depend on activations, so the down weights stream in while the gate/up phase finishes.
//  * Consumers stage a job's activations when their item changes job: gate/up reads the bf16
//    token rows (fp16 in shared memory with the offset table), down reads the fp32 SwiGLU rows
//    that gate/up wrote in this launch (L2 loads, two fp16 halves per value). Between the phases
//    every CTA arrives at a grid barrier (release/acquire counters) and waits for all of them.
//  * After a second barrier every CTA combines a slice of the [T, N] output in slot order.
//  * The counters are left at zero by the last CTA out, so CUDA-graph replays need no host reset.
// Every wait is bounded (2 s of global time); a timeout sets the error word and the kernel drains.
// The grid never exceeds one resident wave (every CTA waited for is running).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <type_traits>

#include "gemv_core.cuh"
#include "gpu_layout.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

using namespace gemv_core;

constexpr int kCombineThreads = kConsumers * 32;
constexpr int kBarRegion = 2 * kNS * 8;             // full + empty mbarriers of the finest ring
constexpr int64_t kWideStageSlots = 128;            // routed slots (T * k) from which stages hold 8 chunks

// bounded wait until the barrier counter reaches `target`; false (and err |= 4) after the limit
__device__ __forceinline__ bool grid_wait(const unsigned *ctr, unsigned target, int *err) {
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_gpu(ctr) < target) {
        __nanosleep(64);
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicOr(err, 4);
            return false;
        }
    }
    return true;
}

// Every item of one phase for this CTA's consumers. NT n-tiles of 8 MMA columns; SPLIT: fp32
// activations staged as two fp16 rows per token (down), else bf16 (gate/up). st: the ring stage
// counter, shared with the producer's order. EPI_SWIGLU: out[yrow][g*32 + s*8 + r] =
// silu(rows r) * rows r+8 (the interleaved gate/up layout); else out[yrow][row].
template <int FMT, int NT, bool SPLIT, bool SWIGLU, int CPS>
__device__ __forceinline__ void consume_phase(const MoeFfnFused &p, uint8_t *smem, int nj, int &st, bool &failed) {
    constexpr int CB = chunk_bytes(FMT), SB = strip_bytes(FMT), STAGE_W = CPS * CB;
    constexpr int NS = kCPS * kNS / CPS;              // ring stages: the same 32 chunks either way
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, s = warp, r = lane >> 2, t = lane & 3;
    const int W = p.workers;
    const GemvJob *jobs = SWIGLU ? p.jobs_gu : p.jobs_dn;
    const int rg = SWIGLU ? p.rg_gu : p.rg_dn, ch = SWIGLU ? p.ch_gu : p.ch_dn;
    const int K = SWIGLU ? p.K_gu : p.K_dn, N = SWIGLU ? p.N_gu : p.N_dn;
    const int mslots = SWIGLU ? p.mslots_gu : p.mslots_dn, xstride = SWIGLU ? p.xstride_gu : p.xstride_dn;
    float *out = SWIGLU ? p.af : p.o;
    const int64_t ldo = SWIGLU ? p.K_dn : p.N_dn;
    const uint32_t sbase = smem_u32(smem), wring = sbase, xregion = sbase + NS * STAGE_W;
    const uint32_t full = sbase + p.off_bar, empty = full + NS * 8;
    int *s_xrow = reinterpret_cast<int *>(smem + p.off_bar + kBarRegion);
    const uint32_t mul[4] = {p.mul[0], p.mul[1], p.mul[2], p.mul[3]};
    const Unpack u{p.unpk[0], p.unpk[1], p.unpk[2]};
    const uint32_t ctab = xregion + mslots * xstride + 128 + t * 8;
    const float *tscale = reinterpret_cast<const float *>(smem + NS * STAGE_W + mslots * xstride + 128 +
                                                          ch * tab_chunk_bytes(NT));
    int cur = -1, m = 0;
    uint32_t xrb[NT], xkm[NT];
    int yr[NT][2];
    const int n_items = nj * rg;
    const int lo = static_cast<int>(static_cast<int64_t>(blockIdx.x) * n_items / W);
    const int hi = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * n_items / W);
    for (int it = lo; it < hi; ++it) {
        const int j = it / rg, g = it - j * rg;
        if (j != cur) {
            // a new job: every consumer is done with the previous activations, then stage this one's
            named_bar_sync(1, kConsumers * 32);
            const int mt = jobs[j].m;
            if (threadIdx.x < kMaxTokensPerJob) s_xrow[threadIdx.x] = jobs[j].xrow[threadIdx.x];
            auto row_of = [s_xrow](int n) { return s_xrow[n]; };
            if constexpr (SPLIT)
                stage_activations<FMT, NT, true, true, 1>(p.af, p.K_dn, row_of, mt, mslots, K, 0, ch, ch, xstride,
                                                          smem + NS * STAGE_W, threadIdx.x, kConsumers * 32);
            else
                stage_activations<FMT, NT, false, false, 4>(p.x, p.ldx, row_of, mt, mslots, K, 0, ch, ch, xstride,
                                                            smem + NS * STAGE_W, threadIdx.x, kConsumers * 32);
            m = SPLIT ? 2 * mt : mt;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int tok = nt * 8 + r;
                xrb[nt] = xregion + (tok < m ? tok * xstride : mslots * xstride) + t * 16;
                xkm[nt] = tok < m ? 128u : 0u;                  // absent tokens stay on the zero block
                if constexpr (SPLIT) {
                    const int tk = nt * 4 + t;
                    yr[nt][0] = tk < mt ? jobs[j].yrow[tk] : -1;
                    yr[nt][1] = -1;
                } else {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int tk = nt * 8 + 2 * t + h;
                        yr[nt][h] = tk < mt ? jobs[j].yrow[tk] : -1;
                    }
                }
            }
            cur = j;
        }
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int f = 0; f < 4; ++f) acc[nt][f] = 0.f;
        for (int c0 = 0; c0 < ch; c0 += CPS, ++st) {
            const int slot = st % NS, n = min(CPS, ch - c0);
            if (!failed && !mbar_wait_bounded(full + slot * 8, (st / NS) & 1, kWaitLimitNs)) {
                failed = true;
                if (lane == 0) atomicOr(p.err, 1);
            }
            if (!failed) {
                const uint32_t wsb = wring + slot * STAGE_W + s * SB;
                auto chunk = [&](int ci) {
                    const int kcc = c0 + ci;
                    uint32_t xa[NT];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) xa[nt] = xrb[nt] + kcc * xkm[nt];
                    strip_chunk_h<FMT, NT>(wsb + ci * CB, xa, ctab + kcc * tab_chunk_bytes(NT), lane, r, mul, u, acc);
                };
                if (n == CPS) {                      // a full stage: unrolled, so the chunks' chains overlap
#pragma unroll
                    for (int ci = 0; ci < CPS; ++ci) chunk(ci);
                } else {
                    for (int ci = 0; ci < n; ++ci) chunk(ci);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + slot * 8);
        }
        finish_rows<NT>(acc, tscale, t);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int h = 0; h < (SPLIT ? 1 : 2); ++h) {
                const int y = yr[nt][h];
                if (y < 0) continue;
                const float lo = SPLIT ? acc[nt][0] + acc[nt][1] : acc[nt][h];
                const float hi = SPLIT ? acc[nt][2] + acc[nt][3] : acc[nt][2 + h];
                if constexpr (SWIGLU) {
                    const int i = g * (kRowGroup / 2) + s * 8 + r;
                    if (i < N / 2) out[static_cast<int64_t>(y) * ldo + i] = silu_f(lo) * hi;
                } else {
                    const int row = g * kRowGroup + s * kStripRows + r;
                    if (row < N) out[static_cast<int64_t>(y) * ldo + row] = lo;
                    if (row + 8 < N) out[static_cast<int64_t>(y) * ldo + row + 8] = hi;
                }
            }
        }
    }
}

template <int FMT, int CPS>
__global__ void __launch_bounds__(kThreads, 2) moe_ffn_kernel(const MoeFfnFused p) {
    constexpr int CB = chunk_bytes(FMT), STAGE_W = CPS * CB;
    constexpr int NS = kCPS * kNS / CPS;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int W = p.workers, cta = blockIdx.x;
    const uint32_t sbase = smem_u32(smem), wring = sbase;
    const uint32_t full = sbase + p.off_bar, empty = full + NS * 8;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full + s * 8, 1);
            mbar_init(empty + s * 8, kConsumers);
        }
        mbar_init_fence();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait_prerequisites();                          // the job lists come from the router kernel
    const int nj = __ldcg(p.njobs);

    if (warp == kConsumers) {
        // ============================================================ producer (lane 0)
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();   // expert weights are read once
            int st = 0;
            bool failed = false;
            for (int ph = 0; ph < 2; ++ph) {
                const GemvJob *jobs = ph ? p.jobs_dn : p.jobs_gu;
                const int rg = ph ? p.rg_dn : p.rg_gu, ch = ph ? p.ch_dn : p.ch_gu;
                const int n_items = nj * rg;
                const int lo = static_cast<int>(static_cast<int64_t>(cta) * n_items / W);
                const int hi = static_cast<int>(static_cast<int64_t>(cta + 1) * n_items / W);
                for (int it = lo; it < hi; ++it) {
                    const int j = it / rg, g = it - j * rg;
                    const uint8_t *base = jobs[j].w + static_cast<int64_t>(g) * ch * CB;
                    for (int c0 = 0; c0 < ch; c0 += CPS, ++st) {
                        const int slot = st % NS, n = min(CPS, ch - c0);
                        if (st >= NS && !failed &&
                            !mbar_wait_bounded(empty + slot * 8, ((st / NS) - 1) & 1, kWaitLimitNs)) {
                            failed = true;
                            atomicOr(p.err, 2);
                        }
                        mbar_arrive_expect_tx(full + slot * 8, static_cast<uint32_t>(n * CB));
                        bulk_g2s_hint(wring + slot * STAGE_W, base + static_cast<int64_t>(c0) * CB,
                                      static_cast<uint32_t>(n * CB), full + slot * 8, pol);
                    }
                }
            }
        }
        return;
    }

    // ================================================================ consumers
    int st = 0;
    bool failed = false;
    consume_phase<FMT, 1, false, true, CPS>(p, smem, nj, st, failed);
    // grid barrier 0: every CTA's gate/up outputs are stored before any down activations are read
    named_bar_sync(1, kConsumers * 32);
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_add_gpu(p.bar, 1u);
        grid_wait(p.bar, static_cast<unsigned>(W), p.err);
    }
    named_bar_sync(1, kConsumers * 32);
    consume_phase<FMT, 2, true, false, CPS>(p, smem, nj, st, failed);
    // grid barrier 1: every expert output is stored before the combine reads it
    named_bar_sync(1, kConsumers * 32);
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_add_gpu(p.bar + 1, 1u);
        grid_wait(p.bar + 1, static_cast<unsigned>(W), p.err);
    }
    named_bar_sync(1, kConsumers * 32);
    // y[t][n] = sum_j w[t][j] * o[t*k + j][n] in slot order (moe_combine_kernel's sum); slots
    // whose expert id is outside [id_lo, id_hi) (another rank's expert, or an id the job builder
    // dropped) add nothing
    const int64_t total = p.T * p.N_dn;
    for (int64_t i = static_cast<int64_t>(cta) * kCombineThreads + threadIdx.x; i < total;
         i += static_cast<int64_t>(W) * kCombineThreads) {
        const int64_t tk = i / p.N_dn, c = i - tk * p.N_dn;
        float acc = 0.f;
        for (int j = 0; j < p.k; ++j) {
            const int64_t slot = tk * p.k + j;
            const int id = p.ids[slot];
            if (id < p.id_lo || id >= p.id_hi) continue;
            acc += p.w[slot] * __ldcg(p.o + slot * p.N_dn + c);
        }
        p.y[tk * p.ldy + c] = acc;
    }
    // leave: the last CTA out returns the counters to zero for the next launch (every CTA has
    // passed both barriers before it counts itself out)
    named_bar_sync(1, kConsumers * 32);
    if (threadIdx.x == 0) {
        const unsigned left = atom_add_acqrel_gpu(p.bar + 2, 1u);
        if (left == static_cast<unsigned>(W) - 1u) {
            p.bar[0] = 0u;
            p.bar[1] = 0u;
            p.bar[2] = 0u;
        }
    }
}

template <int FMT, int CPS>
struct MoeFfnKernel {
    static void prepare() {
        static bool done = false;
        if (!done) {
            done = true;
            cudaFuncSetAttribute(moe_ffn_kernel<FMT, CPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        }
    }
    static cudaError_t launch(const MoeFfnFused &p, int smem, cudaStream_t stream) {
        prepare();
        return launch_pdl(moe_ffn_kernel<FMT, CPS>, dim3(static_cast<unsigned>(p.workers)), dim3(kThreads), smem,
                          stream, p);
    }
};

}  // namespace

int moe_ffn_fused_smem(int fmt, int mslots_gu, int K_gu, int mslots_dn, int K_dn, int *off_bar, int *xstride_gu,
                       int *xstride_dn) {
    const int64_t xs_gu = xres_stride(K_gu), xs_dn = xres_stride(K_dn);
    const int64_t x_gu = xres_bytes(mslots_gu, K_gu, 1, xs_gu), x_dn = xres_bytes(mslots_dn, K_dn, 2, xs_dn);
    const int64_t xbytes = x_gu > x_dn ? x_gu : x_dn;
    const int ob = static_cast<int>(kNS * stage_w_bytes(fmt) + (xbytes + 15) / 16 * 16);
    if (off_bar) *off_bar = ob;
    if (xstride_gu) *xstride_gu = static_cast<int>(xs_gu);
    if (xstride_dn) *xstride_dn = static_cast<int>(xs_dn);
    return ob + 2 * kNS * 8 + kMaxTokensPerJob * 4;
}

int moe_ffn_fused_ctas_per_sm(int fmt, int smem) {
    int o = 0;
    if (fmt == kFmtQ4S) {
        MoeFfnKernel<kFmtQ4S, kCPS>::prepare();
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, moe_ffn_kernel<kFmtQ4S, kCPS>, kThreads, smem);
    } else if (fmt == kFmtQ4F16) {
        MoeFfnKernel<kFmtQ4F16, kCPS>::prepare();
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, moe_ffn_kernel<kFmtQ4F16, kCPS>, kThreads, smem);
    } else {
        MoeFfnKernel<kFmtQ4NX, kCPS>::prepare();
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, moe_ffn_kernel<kFmtQ4NX, kCPS>, kThreads, smem);
    }
    return o;
}

// 8-chunk stages when the layer routes many slots (each CTA then streams several row groups:
// longer unrolled chunk runs between ring waits), 4-chunk stages for few (one row group a CTA)
cudaError_t moe_ffn_fused_launch(const MoeFfnFused &p, int smem, cudaStream_t stream) {
    const bool wide = p.T * p.k >= kWideStageSlots;
    switch (p.fmt) {
        case kFmtQ4S:
            return wide ? MoeFfnKernel<kFmtQ4S, 2 * kCPS>::launch(p, smem, stream)
                        : MoeFfnKernel<kFmtQ4S, kCPS>::launch(p, smem, stream);
        case kFmtQ4F16:
            return wide ? MoeFfnKernel<kFmtQ4F16, 2 * kCPS>::launch(p, smem, stream)
                        : MoeFfnKernel<kFmtQ4F16, kCPS>::launch(p, smem, stream);
        case kFmtQ4NX:
            return wide ? MoeFfnKernel<kFmtQ4NX, 2 * kCPS>::launch(p, smem, stream)
                        : MoeFfnKernel<kFmtQ4NX, kCPS>::launch(p, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace onpu_b200
