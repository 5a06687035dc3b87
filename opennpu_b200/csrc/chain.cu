// A chain of int4 GEMVs in one persistent launch: a decode step's projections (q/k/v, gate_up,
// down, layer after layer) without a kernel boundary between them.
//
// The reference drives a sequence of GEMVs as one NPU instruction stream per call
// (llama/ggml-opennpu/opennpu_core.hpp:418-505 builds it; onpu_api.cpp:292-496 chains gate_up ->
// act -> down the same way). On B200 a separate launch per matrix costs a launch ramp of a few
// microseconds each (the grid fills, the first weight bytes arrive, the split-row tails drain),
// comparable to a whole 14 MB GEMV at HBM speed. Here one wave of CTAs walks all links in order:
//  * Every link's chunk sequence is split evenly over all CTAs (the single-matrix kernel's
//    stream-K partition, per link). CTA w's producer warp streams its range of link 0, then of
//    link 1, ... through one ring of shared-memory stages; weights are constant, so it never
//    waits for anything but free stages and runs ahead across link boundaries.
//  * The consumer warps take the links in the same order. At the start of a link they wait, if
//    the link reads (or overwrites) another link's data, until every CTA has finished that link
//    (a per-link counter reaching the CTA count), then load the link's activations into shared
//    memory (L2 loads: they may have been written in this launch) with their offset table.
//    Counters only grow within a launch and every CTA finishes links in order, so waiting for
//    the latest conflicting link covers all earlier ones.
//  * Split row groups are reduced as in the single-matrix kernel, with the partial slots and
//    flags in a ring of kChainRing links; a later contributor whose slot still holds an
//    unconsumed partial from kChainRing links back waits for it (bounded).
//  * The last CTA to finish resets the counters, so the next launch starts from zero.
// Every wait is bounded (2 s); a timeout sets the error word and the CTA drains its pipeline.
// The grid never exceeds one resident wave, so every CTA that is waited for is running.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gemv_core.cuh"
#include "gpu_layout.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

using namespace gemv_core;

__device__ __forceinline__ void chain_store(const ChainOp &op, int g, int s, int r, int yr, float v_lo, float v_hi) {
    if (yr < 0) return;
    if (op.epi == kEpiSwiGLU) {
        const int i = g * (kRowGroup / 2) + s * 8 + r;       // gate row r, up row r+8 of the strip
        if (i < op.N / 2)
            reinterpret_cast<__nv_bfloat16 *>(op.y)[static_cast<int64_t>(yr) * op.ldy + i] =
                __float2bfloat16_rn(silu_f(v_lo) * v_hi);
        return;
    }
    const int row = g * kRowGroup + s * kStripRows + r;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int rr = row + 8 * h;
        if (rr < op.N) {
            const int col = op.row_map ? op.row_map[rr] : rr;
            const int64_t o = static_cast<int64_t>(yr) * op.ldy + col;
            const float v = h ? v_hi : v_lo;
            if (op.epi == kEpiF32) reinterpret_cast<float *>(op.y)[o] = v;
            else reinterpret_cast<__nv_bfloat16 *>(op.y)[o] = __float2bfloat16_rn(v);
        }
    }
}

// bounded spin until *f satisfies pred; false (and err |= code) after the limit
template <typename Pred>
__device__ __forceinline__ bool spin_until(const unsigned *f, Pred pred, int *err, int code) {
    const uint64_t t0 = global_timer_ns();
    while (!pred(ld_acquire_gpu(f))) {
        __nanosleep(128);
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicOr(err, code);
            return false;
        }
    }
    return true;
}

// Finish segment [a, b) of row group g of link i: the consumer warps' partial sums are in the
// combine buffer (finished rows, token scales applied). Warp s takes strip s. A whole row group
// is stored; a split one is published and the last contributor to arrive adds all partials in
// contributor order and stores. Called by every consumer thread; returns true after a timed-out
// wait. Kept out of line so that the math loop keeps its registers.
template <int NT>
__device__ __noinline__ bool chain_flush(const ChainParams &p, const ChainOp *op, int i, int g, int a, int b, int m,
                                         const float4 *comb, volatile int *last_arrival, bool failed) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 2, t = lane & 3, cw = warp;
    const int W = p.workers, w = blockIdx.x, T = op->row_groups * op->chunks, ring = i % kChainRing;
    int yr[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int tk = nt * 8 + 2 * t + h;
            yr[nt][h] = tk < m ? tk : -1;
        }
    const int s = cw;                      // this warp's strip from here on
    float sa[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        float4 v = comb[((0 * 4 + s) * 32 + lane) * NT + nt];
#pragma unroll
        for (int w2 = 1; w2 < 4; ++w2) {
            const float4 q = comb[((w2 * 4 + s) * 32 + lane) * NT + nt];
            v.x += q.x; v.y += q.y; v.z += q.z; v.w += q.w;
        }
        sa[nt][0] = v.x; sa[nt][1] = v.y; sa[nt][2] = v.z; sa[nt][3] = v.w;
    }
    named_bar_sync(1, kConsumers * 32);   // the buffer is free again
    const int gstart = g * op->chunks;
    auto store_all = [&]() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) chain_store(*op, g, s, r, yr[nt][h], sa[nt][h], sa[nt][2 + h]);
    };
    if (a == gstart && b == gstart + op->chunks) {
        store_all();
        return failed;
    }
    // split row group: every contributor publishes its partial and counts itself in;
    // the last to arrive adds all partials in contributor order (deterministic) and
    // stores. Nobody waits for another CTA here.
    const int cf = worker_of(gstart, W, T), cl = worker_of(gstart + op->chunks - 1, W, T);
    // contributors: every CTA cf..cl when each CTA holds at least one chunk (T >= W); with fewer
    // chunks than CTAs each CTA holds at most one, so they are the owners of the row group's chunks
    const int ncontrib = T >= W ? cl - cf + 1 : op->chunks;
    auto contributor = [&](int k) { return T >= W ? cf + k : worker_of(gstart + k, W, T); };
    const int which = a == gstart ? 1 : 0;               // tail of cf / head of a later CTA
    const int idx = (ring * W + w) * 2 + which;
    if (threadIdx.x == 0 && !failed)                     // the slot's previous partial was consumed
        if (!spin_until(p.flags + idx, [](unsigned v) { return v == 0u; }, p.err, 16)) failed = true;
    named_bar_sync(1, kConsumers * 32);
    float *pslot = p.part + static_cast<int64_t>(idx) * kSlotFloats;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            const int tok = nt * 8 + 2 * t + (f & 1);
            if (tok < m) pslot[((s * 8 + r) * 2 + (f >> 1)) * 16 + tok] = sa[nt][f];
        }
    named_bar_sync(1, kConsumers * 32);
    if (threadIdx.x == 0) {
        __threadfence();
        p.flags[idx] = 1u;
        const unsigned prev = atomicAdd(p.rgcnt + static_cast<int64_t>(i) * W + cf, 1u);
        __threadfence();
        *last_arrival = prev == static_cast<unsigned>(ncontrib - 1) ? 1 : 0;
    }
    named_bar_sync(1, kConsumers * 32);
    if (!*last_arrival) return failed;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            const int tok = nt * 8 + 2 * t + (f & 1);
            if (tok < m) {
                const int e = ((s * 8 + r) * 2 + (f >> 1)) * 16 + tok;
                float v = 0.f;
                for (int k = 0; k < ncontrib; ++k) {
                    const int w2 = contributor(k);
                    v += w2 == w ? sa[nt][f]
                                 : __ldcg(p.part + static_cast<int64_t>((ring * W + w2) * 2 + (w2 == cf)) *
                                                       kSlotFloats + e);
                }
                sa[nt][f] = v;
            }
        }
    store_all();
    named_bar_sync(1, kConsumers * 32);   // every partial is read: the slots may be reused
    for (int k = threadIdx.x; k < ncontrib; k += kConsumers * 32) {
        const int w2 = contributor(k);
        st_release_gpu(p.flags + (ring * W + w2) * 2 + (w2 == cf), 0u);
    }
    if (threadIdx.x == 0) p.rgcnt[static_cast<int64_t>(i) * W + cf] = 0u;
    return failed;
}

template <int FMT, int NT>
__global__ void __launch_bounds__(kThreads, 2) gemv_chain_kernel(const __grid_constant__ ChainParams p) {
    constexpr int CB = chunk_bytes(FMT), STAGE_W = stage_w_bytes(FMT);
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int W = p.workers, w = blockIdx.x, NS = p.ns;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t wring = sbase, xregion = sbase + p.off_x;
    const uint32_t full = sbase + p.off_bar, empty = full + NS * 8;
    volatile int *last_arrival = reinterpret_cast<volatile int *>(smem + p.off_bar + 2 * NS * 8);

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full + s * 8, 1);
            mbar_init(empty + s * 8, kConsumers);
        }
        mbar_init_fence();
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ============================================================ producer
        pdl_launch_dependents();
        pdl_wait_prerequisites();
        int slot = 0, round = 0;                      // ring position of the next stage
        bool failed = false;
        for (int i = 0; i < p.nops; ++i) {
            const ChainOp *opp = p.ops + i;
            const uint8_t *wb = opp->w;
            const int T = opp->row_groups * opp->chunks;
            const int lo = static_cast<int>(static_cast<int64_t>(w) * T / W);
            const int hi = static_cast<int>(static_cast<int64_t>(w + 1) * T / W);
            unsigned long long *trace =
                p.trace && lane == 0 ? p.trace + (static_cast<int64_t>(w) * p.nops + i) * kChainTrace : nullptr;
            for (int c0 = lo; c0 < hi; c0 += kCPS) {
                if (round > 0 && !failed && !mbar_wait_bounded(empty + slot * 8, (round - 1) & 1, kWaitLimitNs)) {
                    failed = true;
                    if (lane == 0) atomicOr(p.err, 2);
                }
                __syncwarp();
                if (lane == 0) {
                    const uint32_t nb = static_cast<uint32_t>(min(kCPS, hi - c0) * CB);
                    mbar_arrive_expect_tx(full + slot * 8, nb);
                    bulk_g2s(wring + slot * STAGE_W, wb + static_cast<int64_t>(c0) * CB, nb, full + slot * 8);
                    if (trace && c0 == lo) trace[5] = global_timer_ns();
                    if (trace && c0 + kCPS >= hi) trace[6] = global_timer_ns();
                }
                if (++slot == NS) {
                    slot = 0;
                    ++round;
                }
            }
        }
        return;
    }

    // ================================================================ consumers
    // warp cw computes chunk cw of every stage for all 4 strips; at a row-group end the warps
    // combine, and warp s finishes strip s
    const int cw = warp, r = lane >> 2, t = lane & 3;
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const uint32_t mul[4] = {p.mul[0], p.mul[1], p.mul[2], p.mul[3]};
    const Unpack u{p.unpk[0], p.unpk[1], p.unpk[2]};
    float4 *comb = reinterpret_cast<float4 *>(smem + p.off_comb);
    int slot = 0, round = 0;
    bool failed = false;

    for (int i = 0; i < p.nops; ++i) {
        const ChainOp *opp = p.ops + i;
        const int chunks = opp->chunks, T = opp->row_groups * chunks;
        const int lo = static_cast<int>(static_cast<int64_t>(w) * T / W);
        const int hi = static_cast<int>(static_cast<int64_t>(w + 1) * T / W);
        unsigned long long *trace =
            p.trace && threadIdx.x == 0 ? p.trace + (static_cast<int64_t>(w) * p.nops + i) * kChainTrace : nullptr;
        if (trace) trace[0] = global_timer_ns();
        if (lo < hi) {
            // ---- wait for the link this one depends on, then stage its activations
            if (opp->dep >= 0 && threadIdx.x == 0 && !failed)
                if (!spin_until(p.done + opp->dep, [W](unsigned v) { return v >= static_cast<unsigned>(W); }, p.err, 8))
                    failed = true;
            named_bar_sync(1, kConsumers * 32);       // also: every warp is done with the previous link's x
            if (trace) trace[1] = global_timer_ns();
            const int m = opp->m, xstride = opp->xstride, ctab_off = opp->ctab_off;
            stage_activations<FMT, NT, true, false, 4>(opp->x, opp->ldx, [](int n) { return n; }, m, m, opp->K, 0,
                                                       chunks, chunks, xstride, smem + p.off_x, threadIdx.x,
                                                       kConsumers * 32);
            if (trace) trace[2] = global_timer_ns();

            // ---- this lane's activation rows, output rows
            uint32_t xrb[NT], xkm[NT];
            int yr[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int tok = nt * 8 + r;
                xrb[nt] = xregion + (tok < m ? tok * xstride : m * xstride) + t * 16;
                xkm[nt] = tok < m ? 128u : 0u;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int tk = nt * 8 + 2 * t + h;
                    yr[nt][h] = tk < m ? tk : -1;
                }
            }
            const uint32_t ctab = xregion + ctab_off + t * 8;
            const float *tscale = reinterpret_cast<const float *>(smem + p.off_x + ctab_off +
                                                                  chunks * tab_chunk_bytes(NT));
            const int ring = i % kChainRing;
            int g = lo / chunks, seg = lo;
            float acc[4][NT][4];
#pragma unroll
            for (int s = 0; s < 4; ++s)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int f = 0; f < 4; ++f) acc[s][nt][f] = 0.f;

            // close segment [a, b) of row group g: combine the warps, warp s finishes strip s
            auto flush = [&](int a, int b) {
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    finish_rows<NT>(acc[s], tscale, t);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        comb[((cw * 4 + s) * 32 + lane) * NT + nt] =
                            make_float4(acc[s][nt][0], acc[s][nt][1], acc[s][nt][2], acc[s][nt][3]);
                }
                named_bar_sync(1, kConsumers * 32);
                if (chain_flush<NT>(p, opp, i, g, a, b, m, comb, last_arrival, failed)) failed = true;
            };

            unsigned long long waited = 0;
            auto wait_stage = [&]() {
                const unsigned long long tw = trace ? global_timer_ns() : 0ull;
                if (!failed && !mbar_wait_bounded(full + slot * 8, round & 1, kWaitLimitNs)) {
                    failed = true;
                    if (lane == 0) atomicOr(p.err, 1);
                }
                if (trace) waited += global_timer_ns() - tw;
            };
            auto release_stage = [&]() {
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + slot * 8);
                if (++slot == NS) {
                    slot = 0;
                    ++round;
                }
            };
            int c0 = lo;
            while (c0 < hi) {
                // full stages that end before the row group does: one chunk per warp, nothing else
                const int gend = (g + 1) * chunks;
                const int nfast = (min(hi, gend - 1) - c0) / kCPS;   // c0 + 4 <= min(hi, gend - 1)
                if (nfast > 0) {
                    int kc = c0 - g * chunks + cw;
                    uint32_t xa[NT];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) xa[nt] = xrb[nt] + kc * xkm[nt];
                    uint32_t ca = ctab + kc * tab_chunk_bytes(NT);
                    for (int k = 0; k < nfast; ++k) {
                        wait_stage();
                        if (!failed)
                            chunk_h<FMT, NT>(wring + slot * STAGE_W + cw * CB, xa, ca, lane, r, mul, u, acc);
                        release_stage();
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) xa[nt] += kCPS * xkm[nt];
                        ca += kCPS * tab_chunk_bytes(NT);
                    }
                    c0 += nfast * kCPS;
                    continue;
                }
                // a stage that reaches or crosses a row-group end (or the range end): in segments;
                // after a timed-out wait only the math is skipped, the barriers in flush() stay uniform
                wait_stage();
                const int c1 = min(hi, c0 + kCPS), c = c0 + cw;   // this warp's chunk of the stage
                const uint32_t sw = wring + slot * STAGE_W;
                int a = c0;
                while (a < c1) {
                    const int ge = (g + 1) * chunks, b = min(c1, ge);
                    if (!failed && c >= a && c < b) {
                        const int kc = c - g * chunks;
                        uint32_t xa[NT];
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) xa[nt] = xrb[nt] + kc * xkm[nt];
                        chunk_h<FMT, NT>(sw + (c - c0) * CB, xa, ctab + kc * tab_chunk_bytes(NT), lane, r, mul, u,
                                         acc);
                    }
                    if (b == ge) {
                        flush(seg, ge);
#pragma unroll
                        for (int s = 0; s < 4; ++s)
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                                for (int f = 0; f < 4; ++f) acc[s][nt][f] = 0.f;
                        seg = ge;
                        ++g;
                    }
                    a = b;
                }
                release_stage();
                c0 = c1;
            }
            if (trace) {
                trace[3] = global_timer_ns();
                trace[7] = waited;
            }
            if (seg < hi) flush(seg, hi);
        }
        // ---- link i is finished here (outputs stored): count this CTA
        named_bar_sync(1, kConsumers * 32);
        if (threadIdx.x == 0) {
            __threadfence();
            red_release_add_gpu(p.done + i, 1u);
        }
        if (trace) trace[4] = global_timer_ns();
    }
    // the last CTA out resets the counters for the next launch (nobody waits on them any more)
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(p.done + p.nops, 1u);
        if (prev == static_cast<unsigned>(W - 1)) {
            for (int i = 0; i < p.nops; ++i) p.done[i] = 0u;
            p.done[p.nops] = 0u;
            __threadfence();
        }
    }
}

template <int FMT, int NT>
struct ChainKernel {
    static void prepare() {
        static bool done = false;
        if (!done) {
            done = true;
            cudaFuncSetAttribute(gemv_chain_kernel<FMT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        }
    }
    static int occupancy(int smem) {
        prepare();
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, gemv_chain_kernel<FMT, NT>, kThreads, smem) != cudaSuccess)
            o = 0;
        return o;
    }
    // cooperative: the runtime guarantees every CTA is resident at once (CTAs wait on each other)
    static cudaError_t launch(const ChainParams &p, int smem, cudaStream_t stream) {
        prepare();
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(p.workers);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, gemv_chain_kernel<FMT, NT>, p);
    }
};

template <int FMT>
int chain_occ(int nt, int smem) {
    return nt == 1 ? ChainKernel<FMT, 1>::occupancy(smem) : ChainKernel<FMT, 2>::occupancy(smem);
}
template <int FMT>
cudaError_t chain_launch_fmt(int nt, const ChainParams &p, int smem, cudaStream_t s) {
    return nt == 1 ? ChainKernel<FMT, 1>::launch(p, smem, s) : ChainKernel<FMT, 2>::launch(p, smem, s);
}

}  // namespace

ChainLayout chain_layout(int fmt, int ntiles, int64_t xregion_bytes, int ns) {
    ChainLayout L{};
    L.ns = ns;
    L.off_x = ns * stage_w_bytes(fmt);
    L.off_comb = static_cast<int>(L.off_x + (xregion_bytes + 127) / 128 * 128);
    L.off_bar = L.off_comb + combine_bytes(ntiles);
    L.smem = L.off_bar + 2 * ns * 8 + 16;         // full[ns], empty[ns], last-arrival word
    return L;
}

int64_t chain_xregion_bytes(int64_t m, int64_t K, int ntiles, int *xstride, int *ctab_off) {
    const int64_t xs = xres_stride(K);
    if (xstride) *xstride = static_cast<int>(xs);
    if (ctab_off) *ctab_off = static_cast<int>(m * xs + 128);
    return xres_bytes(m, K, ntiles, xs);
}

int chain_ctas_per_sm(int fmt, int ntiles, int smem) {
    if (fmt == kFmtQ4NX) return chain_occ<kFmtQ4NX>(ntiles, smem);
    if (fmt == kFmtQ4S) return chain_occ<kFmtQ4S>(ntiles, smem);
    return chain_occ<kFmtQ4F16>(ntiles, smem);
}

int64_t chain_part_floats_per_slot() { return kSlotFloats; }

cudaError_t chain_launch(int fmt, int ntiles, const ChainParams &p, int smem, cudaStream_t stream) {
    switch (fmt) {
        case kFmtQ4NX: return chain_launch_fmt<kFmtQ4NX>(ntiles, p, smem, stream);
        case kFmtQ4S: return chain_launch_fmt<kFmtQ4S>(ntiles, p, smem, stream);
        case kFmtQ4F16: return chain_launch_fmt<kFmtQ4F16>(ntiles, p, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace onpu_b200
