// MoE router on the GPU: logits = h . Wr^T, softmax over the experts, top-k, renormalise.
//
// Replaces the reference's CPU router (opennpu/native/reference.py:71-76;
// opennpu/native/moe_runtime.py:333-341): probabilities softmax(h Wr^T), the k largest in descending order (on
// equal probabilities the lower expert id first, as a stable argsort of -p), weights renormalised
// over the k when norm_topk_prob is set. bf16 h and Wr, fp32 logits (sums of exact products).
// The logits are spread over a grid of 8-expert x 8-token CTAs (a 1-token call reads the router
// matrix with E/8 CTAs instead of one); the last CTA of each token block does the softmax and the
// top-k by k rounds of a warp argmax. Renormalising divides by the selected sum, so the softmax
// denominator cancels; without renormalisation it is kept.
#include <cuda_runtime.h>

#include <cfloat>

#include "gpu_layout.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

constexpr int kRouterThreads = 256;
constexpr int kRouteExperts = 8;     // experts per CTA: one per warp
constexpr int kRouteTokens = 8;      // tokens per CTA

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float dot8(const uint4 a, const uint4 b, float acc) {
    acc = fmaf(bf16_lo(a.x), bf16_lo(b.x), acc);
    acc = fmaf(bf16_hi(a.x), bf16_hi(b.x), acc);
    acc = fmaf(bf16_lo(a.y), bf16_lo(b.y), acc);
    acc = fmaf(bf16_hi(a.y), bf16_hi(b.y), acc);
    acc = fmaf(bf16_lo(a.z), bf16_lo(b.z), acc);
    acc = fmaf(bf16_hi(a.z), bf16_hi(b.z), acc);
    acc = fmaf(bf16_lo(a.w), bf16_lo(b.w), acc);
    return fmaf(bf16_hi(a.w), bf16_hi(b.w), acc);
}

constexpr int kJobThreads = 1024;
constexpr int64_t kJobSmemInts = 11776;          // dynamic shared memory of the job builder: <= 46 KB

// the slot order goes to shared memory when it fits beside the 4 ints per expert (+1)
__host__ __device__ inline bool order_in_smem(const ExpertJobsParams &p) {
    return 4 * static_cast<int64_t>(p.E) + 1 + p.TK <= kJobSmemInts;
}

// exclusive block-wide scan of one int per thread (any block of whole warps, <= 1024 threads);
// returns the block total
__device__ int block_exclusive_scan(int v, int &total, int *warp_sums) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? warp_sums[lane] : 0, wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += n;
        }
        warp_sums[lane] = wi - w;                       // exclusive prefix of the warp totals
        if (lane == 31) warp_sums[32] = wi;
    }
    __syncthreads();
    const int r = warp_sums[warp] + incl - v;
    total = warp_sums[32];
    __syncthreads();
    return r;
}

// Routed (token, slot) pairs grouped by expert into GEMV jobs of <= per_job tokens, on the device:
// the grouping of the host builder (ascending expert id, slots in arrival order), so the whole MoE
// layer runs without a host round trip. One CTA. jobs0 read token rows (slot / k) against bank 0
// (gate_up), jobs1 read the per-slot activation rows against bank 1 (down); both write per slot.
// js: 4E + 1 ints of shared memory; the whole block calls this. ids are read through L2 (the router
// may have written them earlier in the same launch).
__device__ void build_jobs(const ExpertJobsParams &p, int *js, int *warp_sums) {
    int *cnt = js, *start = cnt + p.E, *jstart = start + p.E, *cursor = jstart + p.E + 1;
    // the slot order stays in shared memory when it fits (read back 16 at a time per job)
    int *order = order_in_smem(p) ? cursor + p.E : p.order;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nwarps = nthr >> 5;
    for (int e = tid; e < p.E; e += nthr) {
        cnt[e] = 0;
        cursor[e] = 0;
    }
    __syncthreads();
    for (int64_t i = tid; i < p.TK; i += nthr) {
        const int e = __ldcg(p.ids + i) - p.id_base;
        if (e >= 0 && e < p.E) atomicAdd(&cnt[e], 1);
        else if (!p.skip_foreign) atomicOr(p.err, 8);
    }
    __syncthreads();
    // slot offsets and job offsets per expert (E may exceed the block: scan in pieces)
    int base_s = 0, base_j = 0;
    for (int e0 = 0; e0 < p.E; e0 += nthr) {
        const int e = e0 + tid;
        const int c = e < p.E ? cnt[e] : 0, nj = (c + p.per_job - 1) / p.per_job;
        int ts, tj;
        const int xs = block_exclusive_scan(c, ts, warp_sums);
        const int xj = block_exclusive_scan(nj, tj, warp_sums);
        if (e < p.E) {
            start[e] = base_s + xs;
            jstart[e] = base_j + xj;
        }
        base_s += ts;
        base_j += tj;
    }
    if (tid == 0) jstart[p.E] = base_j;
    __syncthreads();
    // stable placement: warps in turn claim consecutive places per expert
    for (int64_t b = 0; b < p.TK; b += nthr) {
        const int64_t i = b + tid;
        const int e = i < p.TK ? __ldcg(p.ids + i) - p.id_base : -1;
        const bool ok = e >= 0 && e < p.E;
        const unsigned grp = __match_any_sync(0xffffffffu, ok ? e : -1);
        const int rank = __popc(grp & ((1u << lane) - 1u)), leader = __ffs(grp) - 1;
        for (int w = 0; w < nwarps; ++w) {
            if (warp == w && ok) {
                int pos = 0;
                if (lane == leader) {
                    pos = cursor[e];
                    cursor[e] = pos + __popc(grp);
                }
                pos = __shfl_sync(grp, pos, leader);
                order[start[e] + pos + rank] = static_cast<int>(i);
            }
            __syncthreads();
        }
    }
    const int NJ = jstart[p.E];
    for (int jb = tid; jb < NJ; jb += nthr) {
        int lo = 0, hi = p.E;                             // expert e with jstart[e] <= jb < jstart[e + 1]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (jstart[mid] <= jb) lo = mid;
            else hi = mid;
        }
        const int e = lo, part = jb - jstart[e], a = start[e] + part * p.per_job;
        const int m = min(p.per_job, cnt[e] - part * p.per_job);
        GemvJob *j0 = p.jobs0 + jb, *j1 = p.jobs1 + jb;
        j0->w = p.w0 + static_cast<int64_t>(e) * p.bytes0;
        j1->w = p.w1 + static_cast<int64_t>(e) * p.bytes1;
        j0->m = j1->m = m;
        for (int n = 0; n < kMaxTokensPerJob; ++n) {
            const int slot = n < m ? order[a + n] : 0;
            j0->xrow[n] = slot / p.k;
            j0->yrow[n] = j1->xrow[n] = j1->yrow[n] = slot;
        }
    }
    if (tid == 0) *p.njobs = NJ;
}


__global__ void __launch_bounds__(kJobThreads) expert_jobs_kernel(const ExpertJobsParams p) {
    extern __shared__ int js[];
    __shared__ int warp_sums[33];
    pdl_wait_prerequisites();                              // the routed ids
    pdl_launch_dependents();
    build_jobs(p, js, warp_sums);
}

// softmax and top-k of token t, by one warp, from its E logits
__device__ __forceinline__ void select_top_k(const float *lg, int64_t t, int E, int k, int norm, int32_t *ids, float *w,
                                             int lane) {
    const float *row = lg + t * E;
    float v[kMaxRouteExperts / 32];
    float mx = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < kMaxRouteExperts / 32; ++i) {
        const int x = lane + 32 * i;
        v[i] = x < E ? __ldcg(row + x) : -FLT_MAX;
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxRouteExperts / 32; ++i) {
        v[i] = lane + 32 * i < E ? __expf(v[i] - mx) : -3.f;   // probabilities up to the common factor
        total += fmaxf(v[i], 0.f);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    float sel_sum = 0.f, mine = 0.f;                          // lane j keeps the j-th selected value
    for (int j = 0; j < k; ++j) {                             // absent -3 < taken -2 < start < any p >= 0
        float bv = -1.5f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kMaxRouteExperts / 32; ++i)
            if (v[i] > bv) {                                  // ascending ids: ties keep the lower one
                bv = v[i];
                bi = lane + 32 * i;
            }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 31) == lane) {
#pragma unroll
            for (int i = 0; i < kMaxRouteExperts / 32; ++i)
                if (lane + 32 * i == bi) v[i] = -2.f;         // taken
        }
        if (lane == 0) ids[t * k + j] = bi;
        if (lane == j) mine = bv;
        sel_sum += bv;
    }
    const float denom = norm ? sel_sum : total;
    if (lane < k) w[t * k + lane] = mine / denom;
}

// Grid (experts / 8, tokens / 8): each CTA computes the logits of 8 experts x 8 tokens, its warps
// splitting K (see the loop below). The last CTA of a token block to finish
// (counter per token block, reset by that CTA) runs the softmax and top-k of its 8 tokens, one
// warp per token, with the E probabilities in registers (E <= 256: 8 per lane).
__global__ void __launch_bounds__(kRouterThreads) route_kernel(const uint16_t *h, int64_t ldh, int64_t T,
                                                               const uint16_t *wr, int E, int H, int k, int norm,
                                                               int32_t *ids, float *w, float *lg, unsigned *counters,
                                                               const ExpertJobsParams jp) {
    __shared__ int last;
    __shared__ int warp_sums[33];
    extern __shared__ int js[];
    pdl_wait_prerequisites();                              // h (and the counters) of earlier kernels
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * kRouteTokens;
    const int nt = T - t0 < kRouteTokens ? static_cast<int>(T - t0) : kRouteTokens;
    // Warp w takes the K slices w, w + 8, ... of 256 elements; lane L the 8 elements at 8L of a
    // slice, for all 8 experts and 8 tokens of the CTA (16 independent 16-byte loads per slice, so
    // a lane's loads are all in flight together), 64 partial sums per lane.
    __shared__ float red[kRouterThreads / 32][kRouteExperts * kRouteTokens];
    const int e0 = blockIdx.x * kRouteExperts;
    float acc[kRouteExperts * kRouteTokens];
#pragma unroll
    for (int q = 0; q < kRouteExperts * kRouteTokens; ++q) acc[q] = 0.f;
    for (int d = (warp * 32 + lane) * 8; d < H; d += kRouterThreads * 8) {
        uint4 b[kRouteExperts], a[kRouteTokens];
#pragma unroll
        for (int x = 0; x < kRouteExperts; ++x)
            b[x] = e0 + x < E ? ld_nc_v4(wr + static_cast<int64_t>(e0 + x) * H + d) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int n = 0; n < kRouteTokens; ++n)
            a[n] = n < nt ? ld_nc_v4(h + (t0 + n) * ldh + d) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int x = 0; x < kRouteExperts; ++x)
#pragma unroll
            for (int n = 0; n < kRouteTokens; ++n) acc[x * kRouteTokens + n] = dot8(a[n], b[x], acc[x * kRouteTokens + n]);
    }
    // reduce the 64 sums over the warp's lanes by halving exchanges: after the offsets 16, 8, 4,
    // 2, 1, lane L holds the complete warp sums of pairs 2L and 2L + 1 (pair = expert * 8 + token)
#pragma unroll
    for (int o = 16, half = 32; o; o >>= 1, half >>= 1) {
        const bool up = lane & o;
#pragma unroll
        for (int q = 0; q < 32; ++q) {
            if (q < half) {
                const float send = up ? acc[q] : acc[q + half];
                const float keep = up ? acc[q + half] : acc[q];
                acc[q] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
    }
    red[warp][2 * lane] = acc[0];
    red[warp][2 * lane + 1] = acc[1];
    __syncthreads();
    if (threadIdx.x < kRouteExperts * kRouteTokens) {
        const int x = threadIdx.x / kRouteTokens, n = threadIdx.x % kRouteTokens;
        float v = red[0][threadIdx.x];
#pragma unroll
        for (int ww = 1; ww < kRouterThreads / 32; ++ww) v += red[ww][threadIdx.x];   // warps in order
        if (e0 + x < E && n < nt) lg[(t0 + n) * E + e0 + x] = v;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(counters + blockIdx.y, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (threadIdx.x == 0) counters[blockIdx.y] = 0u;          // ready for the next launch
    if (warp < nt) select_top_k(lg, t0 + warp, E, k, norm, ids, w, lane);
    if (jp.TK <= 0) return;
    // the job lists too: the last token block to finish groups every slot by expert
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        last = atomicAdd(counters + gridDim.y, 1u) == gridDim.y - 1;
        if (last) counters[gridDim.y] = 0u;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    build_jobs(jp, js, warp_sums);
}

// 4 ints per expert (+1), and the slot order when it fits
size_t job_smem_bytes(const ExpertJobsParams &p) {
    return sizeof(int) * (4 * static_cast<size_t>(p.E) + 1 + (order_in_smem(p) ? p.TK : 0));
}

}  // namespace

cudaError_t expert_jobs_launch(const ExpertJobsParams &p, cudaStream_t stream) {
    if (p.TK <= 0) return cudaSuccess;
    return launch_pdl(expert_jobs_kernel, dim3(1), dim3(kJobThreads), job_smem_bytes(p), stream, p);
}

cudaError_t route_launch(const uint16_t *h, int64_t ldh, int64_t T, const uint16_t *wr, int E, int H, int k, int norm,
                         int32_t *ids, float *w, float *logits, unsigned *counters, cudaStream_t stream,
                         const ExpertJobsParams *jobs) {
    if (T <= 0) return cudaSuccess;
    const dim3 grid((E + kRouteExperts - 1) / kRouteExperts, static_cast<unsigned>((T + kRouteTokens - 1) / kRouteTokens));
    ExpertJobsParams jp{};
    size_t smem = 0;
    if (jobs) {
        jp = *jobs;
        smem = job_smem_bytes(jp);
    }
    return launch_pdl(route_kernel, grid, dim3(kRouterThreads), smem, stream, h, ldh, T, wr, E, H, k, norm, ids, w,
                      logits, counters, jp);
}

// a counter per 8-token block, and one for the blocks that finished (job building)
int64_t route_counter_slots(int64_t T) { return (T + kRouteTokens - 1) / kRouteTokens + 1; }

}  // namespace onpu_b200
