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
//    multicast, an L2 evict-first policy: weights are read once), NS stages of CPS chunks,
//    recycled through "empty" mbarriers.
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
//  * Programmatic dependent launch: the weight prefetch (constant data) and host-written job
//    descriptors are read before griddepcontrol.wait, so a kernel's weight stream overlaps the
//    previous kernel's tail and its activation staging starts with the activation loads.
//  * Every wait is bounded (2 s of global time); a timed-out wait sets the error word and the
//    warp keeps draining the pipeline without computing, so no copy is left in flight at exit.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "gemv_core.cuh"
#include "gpu_layout.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

using namespace gemv_core;

constexpr int kBarRegion = 2 * kNS * 8;          // full + empty mbarriers of the finest ring (4-chunk stages)
constexpr int kWideStageChunks = 32;             // chunks per CTA from which a launch takes 8-chunk stages


// Store the finished sums of strip rows r (v_lo) and r+8 (v_hi) of one token (output row yr).
// call: kEpiPeer's all-reduce call number of this CTA.
template <int EPI>
__device__ __forceinline__ void store_pair(const GemvParams &p, int g, int s, int r, int yr, float v_lo, float v_hi,
                                           uint32_t call) {
    if (yr < 0) return;
    if constexpr (EPI == kEpiSwiGLU || EPI == kEpiPairSum) {
        const int i = g * (kRowGroup / 2) + s * 8 + r;       // row r and row r+8 of the strip pair up
        if (i < p.N / 2) {
            const int64_t o = static_cast<int64_t>(yr) * p.ldy + i;
            if constexpr (EPI == kEpiSwiGLU) {
                const float a = silu_f(v_lo) * v_hi;
                if (p.yf32) reinterpret_cast<float *>(p.y)[o] = a;
                else reinterpret_cast<__nv_bfloat16 *>(p.y)[o] = __float2bfloat16_rn(a);
            } else {
                reinterpret_cast<float *>(p.y)[o] = v_lo + v_hi;
            }
        }
    } else if constexpr (EPI == kEpiPeer) {
        // row-parallel projection: each finished value goes straight to every rank's all-reduce
        // buffer as one 8-byte {value, call number} word (the receive side waits on the number)
        const int64_t set = static_cast<int64_t>(call & 1u) * p.peer_world;
        const int row = g * kRowGroup + s * kStripRows + r;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int rr = row + 8 * h;
            if (rr < p.N) {
                const int64_t e = static_cast<int64_t>(yr) * p.ldy + rr;
                const uint32_t v = __float_as_uint(h ? v_hi : v_lo);
                for (int d = 0; d < p.peer_world; ++d)
                    st_word(static_cast<uint2 *>(p.peer[d]) + (set + p.peer_rank) * p.peer_cap + e, v, call);
            }
        }
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

// kEpiPeer, after the CTA's range: the rows this CTA finished (row groups whose first chunk lies in
// [lo, hi): it summed their split parts) were sent to every rank; the same CTA index of every rank
// finished the same rows (same shape, same grid), so wait for each rank's word of each of them
// carrying this call's number, add the ranks' values in rank order (the same float sum on every
// rank) and write the sum. Waits are bounded (peer_wait_ns, 2 s by default; then the error word and
// the value as found).
__device__ void peer_receive(const GemvParams &p, int lo, int hi, uint32_t call, int tid, int nthr) {
    const int rg0 = (lo + p.chunks - 1) / p.chunks, rg1 = (hi + p.chunks - 1) / p.chunks;   // one job
    const int mt = p.jobs[0].m;
    const int64_t n_el = static_cast<int64_t>(rg1 - rg0) * kRowGroup * mt;
    const int64_t set = static_cast<int64_t>(call & 1u) * p.peer_world;
    const uint2 *own = static_cast<const uint2 *>(p.peer[p.peer_rank]);
    for (int64_t i = tid; i < n_el; i += nthr) {
        const int tok = static_cast<int>(i % mt);
        const int64_t rr = static_cast<int64_t>(rg0) * kRowGroup + i / mt;
        if (rr >= p.N) continue;
        const int yr = p.jobs[0].yrow[tok];
        const int64_t e = static_cast<int64_t>(yr) * p.ldy + rr;
        const float acc = recv_words_sum<kPeerMaxRanks>(own + set * p.peer_cap + e, p.peer_cap, p.peer_world, call,
                                                         p.peer_wait_ns, p.err);
        if (p.y) reinterpret_cast<float *>(p.y)[e] = acc;
        if (p.y_bf16) reinterpret_cast<__nv_bfloat16 *>(p.y_bf16)[e] = __float2bfloat16_rn(acc);
    }
}

// XS: fp32 activations staged as two fp16 rows per token (resident only); a template parameter so
// the bf16 kernels keep their register allocation
template <int FMT, int NT, int EPI, bool CI, bool XS, int CPS>
__global__ void __launch_bounds__(kThreads, 2) gemv_int4_kernel(const GemvParams p) {
    constexpr int CB = chunk_bytes(FMT), SB = strip_bytes(FMT), STAGE_W = CPS * CB;
    constexpr int NS = kCPS * kNS / CPS;              // ring stages: the same 32 chunks either way
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int W = p.workers, cta = blockIdx.x;
    unsigned long long *trace = p.trace ? p.trace + static_cast<int64_t>(cta) * kGemvTrace : nullptr;
    if (trace && threadIdx.x == 0) trace[0] = global_timer_ns();
    int T = p.total_chunks;
    if (p.njobs_dev) {                                // jobs built on the device by the previous kernel
        pdl_wait_prerequisites();
        T = __ldcg(p.njobs_dev) * p.row_groups * p.chunks;
    }
    const int lo = static_cast<int>(static_cast<int64_t>(cta) * T / W);
    const int hi = static_cast<int>(static_cast<int64_t>(cta + 1) * T / W);
    if (lo >= hi) return;      // no chunks (a device-side job count below the grid, or zero jobs)
    const int nst = (hi - lo + CPS - 1) / CPS;
    const int per_job = p.row_groups * p.chunks;
    constexpr bool xres = CI;                         // resident activations carry the offset table
    const int xchunk = p.xslots * kXSlot, xstage_bytes = CPS * xchunk;   // per-stage activation layout
    const uint32_t sbase = smem_u32(smem);
    const uint32_t wring = sbase, xregion = sbase + NS * STAGE_W;
    const uint32_t full = sbase + p.off_bar, empty = full + NS * 8;

    if (!xres)   // the zero slot is never written; a chunk half past K gets a 64-B copy only
        for (int e = threadIdx.x; e < NS * xstage_bytes / 16; e += blockDim.x)
            *reinterpret_cast<uint4 *>(smem + NS * STAGE_W + e * 16) = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
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
        const uint64_t wpol = l2_evict_first_policy();   // weights are read once per launch
        auto issue_weights = [&](int st) {            // lane 0 only
            const int c0 = lo + st * CPS, c1 = min(hi, c0 + CPS);
            const uint32_t bar = full + (st % NS) * 8;
            mbar_arrive_expect_tx(bar, static_cast<uint32_t>((c1 - c0) * CB));
            uint32_t dst = wring + (st % NS) * STAGE_W;
            int c = c0;
            while (c < c1) {                          // one copy per run of chunks within a job
                if (c >= (wj + 1) * per_job) wbase = p.jobs[++wj].w;
                const int run_end = min(c1, (wj + 1) * per_job);
                bulk_g2s_hint(dst, wbase + static_cast<int64_t>(c - wj * per_job) * CB,
                              static_cast<uint32_t>((run_end - c) * CB), bar, wpol);
                dst += (run_end - c) * CB;
                c = run_end;
            }
        };
        const int npro = min(NS, nst);
        if (lane == 0 && p.jobs_ready)
            for (int st = 0; st < npro; ++st) issue_weights(st);
        if (trace && lane == 0) trace[1] = global_timer_ns();
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
            const int slot = st % NS;
            if (st >= NS) {
                if (!failed && !mbar_wait_bounded(empty + slot * 8, ((st / NS) - 1) & 1, kWaitLimitNs)) {
                    failed = true;
                    if (lane == 0) atomicOr(p.err, 2);
                }
                __syncwarp();
                if (lane == 0) issue_weights(st);
            }
            if (xres) continue;
            // activations of this stage: per chunk one 128-B copy per token (64 B when the chunk's
            // second group lies past K); the byte total is announced first
            const int c0 = lo + st * CPS, c1 = min(hi, c0 + CPS);
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
                    bulk_g2s(xregion + slot * xstage_bytes + (c - c0) * xchunk + lane * kXSlot,
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
    volatile int *flag = reinterpret_cast<volatile int *>(smem + p.off_bar + kBarRegion);
    int *s_xrow = reinterpret_cast<int *>(smem + p.off_bar + kBarRegion + 16);   // the staged job's rows
    int j = lo / per_job;
    int g = (lo - j * per_job) / p.chunks;
    int kc = lo - j * per_job - g * p.chunks;
    int seg = lo;
    int m = 0;
    // descriptors the host wrote are read before griddepcontrol.wait (they are not the previous
    // kernel's output), so staging starts with the activation loads themselves
    auto load_job = [&]() {
        m = p.jobs[j].m;
        if (threadIdx.x < kMaxTokensPerJob) s_xrow[threadIdx.x] = p.jobs[j].xrow[threadIdx.x];
    };
    if (p.jobs_ready) load_job();
    pdl_launch_dependents();
    pdl_wait_prerequisites();                         // x / outputs / scratch may belong to the previous kernel
    if (!p.jobs_ready) load_job();
    const bool tr = trace && threadIdx.x == 0;
    if (tr) trace[2] = global_timer_ns();
    uint32_t call = 0;                                // kEpiPeer: this CTA's all-reduce call number
    if constexpr (EPI == kEpiPeer) call = *reinterpret_cast<volatile uint32_t *>(p.peer_calls + cta) + 1u;

    const int mslots = p.xslots - 1;                  // rows the activation region is laid out for
    // resident activations: fp16 rows, a zero block, the offset table, token scales; staged
    // again (after every consumer is done with them) when the range enters the next job.
    // kwin (one job): only this CTA's part of K, window chunk i = the range's i-th chunk
    const bool win = xres && p.kwin;
    const int kc0 = win ? lo % p.chunks : 0, nch = win ? hi - lo : p.chunks;
    constexpr bool split = XS;
    // s_xrow holds job jj's rows and mj its token count; stage_activations' first barrier
    // publishes s_xrow to every consumer thread before any activation load
    auto row_of = [s_xrow](int n) { return s_xrow[n]; };
    auto stage = [&](int mj, auto su) {
        constexpr int SU = decltype(su)::value;
        if constexpr (XS)
            stage_activations<FMT, NT, false, true, SU>(p.xf, p.ldx, row_of, mj, mslots, p.K, kc0, nch, p.wchunks,
                                                        p.xstride, smem + NS * STAGE_W, threadIdx.x, kConsumers * 32);
        else
            stage_activations<FMT, NT, false, false, SU>(p.x, p.ldx, row_of, mj, mslots, p.K, kc0, nch, p.wchunks,
                                                         p.xstride, smem + NS * STAGE_W, threadIdx.x, kConsumers * 32);
    };
    if (xres) stage(m, std::integral_constant<int, 4>{});
    if (tr) trace[3] = global_timer_ns();
    uint64_t waited = 0;
    // the next job (every consumer is past the previous one's activations); inside the chunk
    // loop, so fewer loads in flight per thread and the loop keeps its registers
    auto restage = [&](int jj) {
        if (threadIdx.x < kMaxTokensPerJob) s_xrow[threadIdx.x] = p.jobs[jj].xrow[threadIdx.x];
        stage(p.jobs[jj].m, std::integral_constant<int, 1>{});
    };
    const float *tscale = reinterpret_cast<const float *>(smem + NS * STAGE_W + p.ctab_off +
                                                          p.wchunks * tab_chunk_bytes(NT));

    // m counts activation rows (MMA columns): the job's tokens, twice that when split (rows 2n and
    // 2n + 1 carry token n, so lane t's two columns are one token's halves)
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int f = 0; f < 4; ++f) acc[nt][f] = 0.f;
    int yr[NT][2];
    uint32_t xrb[NT], xkm[NT];                        // activation base and per-chunk stride of this lane
    auto load_rows = [&]() {
        const int mt = p.jobs[j].m;
        m = split ? 2 * mt : mt;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int tok = nt * 8 + r;
            if (xres) {
                xrb[nt] = xregion + (tok < m ? tok * p.xstride : mslots * p.xstride) + t * 16;
                xkm[nt] = tok < m ? 128u : 0u;        // absent tokens stay on the zero block
            } else {
                xrb[nt] = xregion + (tok < m ? tok : p.xslots - 1) * kXSlot + t * 16;
                xkm[nt] = 0u;
            }
            if (split) {
                const int tk = nt * 4 + t;
                yr[nt][0] = tk < mt ? p.jobs[j].yrow[tk] : -1;
                yr[nt][1] = -1;
            } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int tk = nt * 8 + 2 * t + h;
                    yr[nt][h] = tk < mt ? p.jobs[j].yrow[tk] : -1;
                }
            }
        }
    };
    // the finished sums of this lane's rows r, r + 8 (split: one token's two halves added)
    auto store_rows = [&]() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            if (split) {
                store_pair<EPI>(p, g, s, r, yr[nt][0], acc[nt][0] + acc[nt][1], acc[nt][2] + acc[nt][3], call);
            } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) store_pair<EPI>(p, g, s, r, yr[nt][h], acc[nt][h], acc[nt][2 + h], call);
            }
        }
    };
    load_rows();

    // Close segment [a, b) of row group (j, g) for this strip.
    auto flush = [&](int a, int b) {
        if (xres) finish_rows<NT>(acc, tscale, t);
        const int gstart = (j * p.row_groups + g) * p.chunks;
        if (a == gstart && b == gstart + p.chunks) {          // the whole row group is here
            store_rows();
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
            if (tr) trace[8] = global_timer_ns();
            return;
        }
        // tail segment of the first contributor: collect cf+1 .. cl (bounded wait on their flags)
        if (warp == 0) {
            for (int w2 = cf + 1 + lane; w2 <= cl; w2 += 32) {
                if (range_empty(w2, W, T)) continue;          // fewer chunks than CTAs: no partials
                const uint64_t t0 = global_timer_ns();
                while (ld_acquire_gpu(p.counters + w2) == 0u) {
                    __nanosleep(32);
                    if (global_timer_ns() - t0 > kWaitLimitNs) {
                        atomicOr(p.err, 4);
                        break;
                    }
                }
                p.counters[w2] = 0u;                          // consumed: ready for the next launch
            }
        }
        named_bar_sync(1, kConsumers * 32);
        if (tr) {
            trace[9] = global_timer_ns();
            trace[10] = static_cast<unsigned long long>(cl - cf);
        }
        // the partners' partial sums, kPartBatch partners' loads in flight before the first add
        // (one L2 round trip per batch, not per partner), added in partner order (deterministic)
        for (int w0 = cf + 1; w0 <= cl; w0 += kPartBatch) {
            float pv[kPartBatch][NT][4];
            bool has[kPartBatch];
#pragma unroll
            for (int q = 0; q < kPartBatch; ++q) {
                has[q] = w0 + q <= cl && !range_empty(w0 + q, W, T);
                const float *src = p.part + static_cast<int64_t>(w0 + q) * kSlotFloats;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        const int tok = nt * 8 + 2 * t + (f & 1);
                        pv[q][nt][f] = has[q] && tok < m ? __ldcg(src + ((s * 8 + r) * 2 + (f >> 1)) * 16 + tok) : 0.f;
                    }
            }
#pragma unroll
            for (int q = 0; q < kPartBatch; ++q)
                if (has[q])
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int f = 0; f < 4; ++f)
                            if (nt * 8 + 2 * t + (f & 1) < m) acc[nt][f] += pv[q][nt][f];
        }
        if (tr) trace[11] = global_timer_ns();
        store_rows();
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
                if (c + 1 < hi) {
                    if (xres) {
                        named_bar_sync(1, kConsumers * 32);       // every warp is done with job j - 1
                        restage(j);
                    }
                    load_rows();
                }
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
    auto caddr = [&](int kcc) { return ctab + kcc * tab_chunk_bytes(NT); };
    const Unpack u{p.unpk[0], p.unpk[1], p.unpk[2]};
    // resident activations take the fp16 path, per-stage slices the bf16 one
    auto chunk_math = [&](uint32_t wsc, const uint32_t (&xa)[NT], int kcc) {
        if constexpr (CI) strip_chunk_h<FMT, NT>(wsc, xa, caddr(kcc), lane, r, mul, u, acc);
        else strip_chunk<FMT, NT, false>(wsc, xa, 0u, lane, r, mul, acc);
    };

    bool failed = false;
    for (int st = 0; st < nst; ++st) {
        const int slot = st % NS;
        const uint64_t tw = tr ? global_timer_ns() : 0;
        if (!failed && !mbar_wait_bounded(full + slot * 8, (st / NS) & 1, kWaitLimitNs)) {
            failed = true;
            if (lane == 0) atomicOr(p.err, 1);
        }
        if (tr) {
            const uint64_t now = global_timer_ns();
            waited += now - tw;
            if (st == 0) trace[4] = now;
        }
        const int c0 = lo + st * CPS, n = min(hi - c0, CPS);
        const uint32_t wsb = wring + slot * STAGE_W + s * SB, xstage = slot * xstage_bytes;
        // after a timed-out wait (failed is per thread) only the math is skipped: the bookkeeping
        // and every named barrier in flush() stay the same in all consumer threads
        // resident activations of chunk c sit at window chunk c - lo (kwin) or at its k chunk
        if (n == CPS && kc + CPS < p.chunks) {
            // the common case: a full stage inside one row group
            if (!failed) {
                const int xb = win ? c0 - lo : kc;
#pragma unroll
                for (int ci = 0; ci < CPS; ++ci) {
                    uint32_t xa[NT];
                    xaddr(xa, xstage, ci, xb + ci);
                    chunk_math(wsb + ci * CB, xa, xb + ci);
                }
            }
            kc += CPS;
        } else {
            for (int ci = 0; ci < n; ++ci) {
                if (!failed) {
                    const int xb = win ? c0 + ci - lo : kc;
                    uint32_t xa[NT];
                    xaddr(xa, xstage, ci, xb);
                    chunk_math(wsb + ci * CB, xa, xb);
                }
                advance(c0 + ci);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot * 8);
    }
    if (tr) trace[5] = global_timer_ns();
    if (seg < hi) flush(seg, hi);
    if constexpr (EPI == kEpiPeer) {
        __threadfence();                               // this CTA's own words, before other threads read them
        named_bar_sync(1, kConsumers * 32);
        peer_receive(p, lo, hi, call, threadIdx.x, kConsumers * 32);
        named_bar_sync(1, kConsumers * 32);
        if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t *>(p.peer_calls + cta) = call;
    }
    if (tr) {
        trace[6] = global_timer_ns();
        trace[7] = waited;
    }
}

template <int FMT, int NT, int EPI, bool CI, bool XS, int CPS>
struct GemvKernel {
    static void prepare() {
        static bool done = false;
        if (!done) {
            done = true;
            cudaFuncSetAttribute(gemv_int4_kernel<FMT, NT, EPI, CI, XS, CPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 227 * 1024);
        }
    }
    static int occupancy(int smem) {
        prepare();
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, gemv_int4_kernel<FMT, NT, EPI, CI, XS, CPS>, kThreads,
                                                          smem) != cudaSuccess)
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
        return cudaLaunchKernelEx(&cfg, gemv_int4_kernel<FMT, NT, EPI, CI, XS, CPS>, p);
    }
};

template <int FMT, int NT, bool CI, int CPS>
cudaError_t dispatch_epi_ci(int epi, const GemvParams &p, int smem, cudaStream_t s, bool pdl) {
    switch (epi) {
        case kEpiF32: return GemvKernel<FMT, NT, kEpiF32, CI, false, CPS>::launch(p, smem, s, pdl);
        case kEpiBF16: return GemvKernel<FMT, NT, kEpiBF16, CI, false, CPS>::launch(p, smem, s, pdl);
        case kEpiSwiGLU: return GemvKernel<FMT, NT, kEpiSwiGLU, CI, false, CPS>::launch(p, smem, s, pdl);
        case kEpiPairSum: return GemvKernel<FMT, NT, kEpiPairSum, CI, false, CPS>::launch(p, smem, s, pdl);
        case kEpiPeer: return GemvKernel<FMT, NT, kEpiPeer, CI, false, CPS>::launch(p, smem, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

// fp32 (split) activations: the epilogues of the projections that take them (a down or o
// projection, a gate/up fed by one, a row-parallel projection); resident activations only
template <int FMT, int NT, int CPS>
cudaError_t dispatch_split(int epi, const GemvParams &p, int smem, cudaStream_t s, bool pdl) {
    switch (epi) {
        case kEpiF32: return GemvKernel<FMT, NT, kEpiF32, true, true, CPS>::launch(p, smem, s, pdl);
        case kEpiSwiGLU: return GemvKernel<FMT, NT, kEpiSwiGLU, true, true, CPS>::launch(p, smem, s, pdl);
        case kEpiPeer: return GemvKernel<FMT, NT, kEpiPeer, true, true, CPS>::launch(p, smem, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

template <int FMT, int NT, int CPS>
cudaError_t dispatch_epi(int epi, const GemvParams &p, int smem, cudaStream_t s, bool pdl) {
    if (p.xsplit) return p.xres ? dispatch_split<FMT, NT, CPS>(epi, p, smem, s, pdl) : cudaErrorInvalidValue;
    return p.xres ? dispatch_epi_ci<FMT, NT, true, CPS>(epi, p, smem, s, pdl)
                  : dispatch_epi_ci<FMT, NT, false, CPS>(epi, p, smem, s, pdl);
}

// Stages of 8 chunks for launches whose CTAs stream long ranges (more independent chunk chains
// per consumer warp between ring waits: the 32B gate/up launch 3826 -> 4233 GB/s), of 4 chunks for
// short ranges and device-counted (expert) launches, whose ring fills and drains dominate
template <int FMT>
cudaError_t dispatch_nt(int nt, int epi, const GemvParams &p, int smem, cudaStream_t s, bool pdl) {
    const bool wide = !p.njobs_dev && p.workers > 0 && (p.total_chunks + p.workers - 1) / p.workers >= kWideStageChunks;
    if (wide)
        return nt == 1 ? dispatch_epi<FMT, 1, 2 * kCPS>(epi, p, smem, s, pdl)
                       : dispatch_epi<FMT, 2, 2 * kCPS>(epi, p, smem, s, pdl);
    return nt == 1 ? dispatch_epi<FMT, 1, kCPS>(epi, p, smem, s, pdl) : dispatch_epi<FMT, 2, kCPS>(epi, p, smem, s, pdl);
}

template <int FMT>
int occ_fmt(int nt, int smem) {
    return nt == 1 ? GemvKernel<FMT, 1, kEpiF32, true, false, kCPS>::occupancy(smem)
                   : GemvKernel<FMT, 2, kEpiF32, true, false, kCPS>::occupancy(smem);
}

}  // namespace

GemvLayout gemv_layout(int fmt, int mrows, int64_t K, int wchunks, int64_t budget) {
    GemvLayout L{};
    const int chunks = static_cast<int>((K + kChunkK - 1) / kChunkK);
    if (wchunks <= 0 || wchunks > chunks) wchunks = chunks;
    const int64_t xstride = xres_stride(static_cast<int64_t>(wchunks) * kChunkK);
    // rows, zero block, table, scales
    const int64_t res_bytes = xres_bytes(mrows, static_cast<int64_t>(wchunks) * kChunkK, mrows > 8 ? 2 : 1, xstride);
    L.xres = res_bytes <= budget;                 // several jobs: staged again per job
    L.wchunks = wchunks;
    L.xstride = static_cast<int>(xstride);
    L.ctab_off = static_cast<int>(mrows * xstride + 128);
    L.xslots = mrows + 1;
    const int64_t xbytes = L.xres ? res_bytes : static_cast<int64_t>(kNS) * kCPS * L.xslots * kXSlot;
    L.off_bar = static_cast<int>(kNS * stage_w_bytes(fmt) + (xbytes + 15) / 16 * 16);
    L.smem = L.off_bar + kBarRegion + 16 + kMaxTokensPerJob * 4;   // mbarriers, flag, staged job's rows
    return L;
}

bool gemv_resident(int mrows, int64_t K) {
    return xres_bytes(mrows, K, mrows > 8 ? 2 : 1, xres_stride(K)) <= kResidentXBudget;
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
