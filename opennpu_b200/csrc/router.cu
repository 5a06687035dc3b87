// MoE router on the GPU: logits = h . Wr^T, softmax over the experts, top-k, renormalise.
//
// Replaces the reference's CPU router (opennpu/native/reference.py:71-76;
// opennpu/native/moe_runtime.py:333-341): probabilities softmax(h Wr^T), the k largest in descending order (on
// equal probabilities the lower expert id first, as a stable argsort of -p), weights renormalised
// over the k when norm_topk_prob is set. bf16 h and Wr, fp32 logits (sums of exact products).
// One CTA per token: eight warps compute the E logits (one dot product per warp and expert,
// 16-byte loads, a warp reduction), warp 0 does the softmax and the top-k by k rounds of a warp
// argmax. Renormalising divides by the selected sum, so the softmax denominator cancels; without
// renormalisation it is kept.
#include <cuda_runtime.h>

#include <cfloat>

#include "gpu_layout.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

constexpr int kRouterThreads = 256;

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__global__ void __launch_bounds__(kRouterThreads) route_kernel(const uint16_t *h, int64_t ldh, const uint16_t *wr, int E,
                                                               int H, int k, int norm, int32_t *ids, float *w,
                                                               float *logits) {
    extern __shared__ float sm[];                    // [E] logits, then [E] exp(logit - max)
    float *lg = sm, *ex = sm + E;
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint16_t *hr = h + static_cast<int64_t>(t) * ldh;
    for (int e = warp; e < E; e += kRouterThreads / 32) {
        const uint16_t *wrow = wr + static_cast<int64_t>(e) * H;
        float acc = 0.f;
        for (int d = lane * 8; d < H; d += 32 * 8) {
            const uint4 a = ld_nc_v4(hr + d), b = ld_nc_v4(wrow + d);
            acc = fmaf(bf16_lo(a.x), bf16_lo(b.x), acc);
            acc = fmaf(bf16_hi(a.x), bf16_hi(b.x), acc);
            acc = fmaf(bf16_lo(a.y), bf16_lo(b.y), acc);
            acc = fmaf(bf16_hi(a.y), bf16_hi(b.y), acc);
            acc = fmaf(bf16_lo(a.z), bf16_lo(b.z), acc);
            acc = fmaf(bf16_hi(a.z), bf16_hi(b.z), acc);
            acc = fmaf(bf16_lo(a.w), bf16_lo(b.w), acc);
            acc = fmaf(bf16_hi(a.w), bf16_hi(b.w), acc);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) lg[e] = acc;
    }
    __syncthreads();
    if (warp != 0) return;
    float mx = -FLT_MAX;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[e]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float total = 0.f;
    for (int e = lane; e < E; e += 32) {
        const float v = __expf(lg[e] - mx);
        ex[e] = v;
        total += v;
        if (logits) logits[static_cast<int64_t>(t) * E + e] = lg[e];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    __syncwarp();
    float sel_sum = 0.f, mine = 0.f;                 // lane j keeps the j-th selected value
    for (int j = 0; j < k; ++j) {
        float bv = -1.f;
        int bi = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            const float v = ex[e];
            if (v > bv || (v == bv && e < bi)) {
                bv = v;
                bi = e;
            }
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
        if (lane == 0) {
            ids[static_cast<int64_t>(t) * k + j] = bi;
            ex[bi] = -2.f;                           // taken
        }
        if (lane == j) mine = bv;
        sel_sum += bv;
        __syncwarp();
    }
    const float denom = norm ? sel_sum : total;
    if (lane < k) w[static_cast<int64_t>(t) * k + lane] = mine / denom;
}

constexpr int kJobThreads = 1024;

// exclusive block-wide scan of one int per thread (kJobThreads threads); returns the block total
__device__ int block_exclusive_scan(int v, int &total, int *warp_sums) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = warp_sums[lane], wi = w;
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

// Routed (token, slot) pairs grouped by expert into GEMV jobs of <= 16 tokens, on the device: the
// grouping of the host builder (ascending expert id, slots in arrival order), so the whole MoE
// layer runs without a host round trip. One CTA. jobs0 read token rows (slot / k) against bank 0
// (gate_up), jobs1 read the per-slot activation rows against bank 1 (down); both write per slot.
__global__ void __launch_bounds__(kJobThreads) expert_jobs_kernel(const ExpertJobsParams p) {
    extern __shared__ int js[];
    int *cnt = js, *start = cnt + p.E, *jstart = start + p.E, *cursor = jstart + p.E + 1;
    __shared__ int warp_sums[33];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < p.E; e += kJobThreads) {
        cnt[e] = 0;
        cursor[e] = 0;
    }
    __syncthreads();
    for (int64_t i = tid; i < p.TK; i += kJobThreads) {
        const int e = p.ids[i];
        if (e >= 0 && e < p.E) atomicAdd(&cnt[e], 1);
        else atomicOr(p.err, 8);
    }
    __syncthreads();
    // slot offsets and job offsets per expert (E may exceed the block: scan in pieces)
    int base_s = 0, base_j = 0;
    for (int e0 = 0; e0 < p.E; e0 += kJobThreads) {
        const int e = e0 + tid;
        const int c = e < p.E ? cnt[e] : 0, nj = (c + kMaxTokensPerJob - 1) / kMaxTokensPerJob;
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
    for (int64_t b = 0; b < p.TK; b += kJobThreads) {
        const int64_t i = b + tid;
        const int e = i < p.TK ? p.ids[i] : -1;
        const bool ok = e >= 0 && e < p.E;
        const unsigned grp = __match_any_sync(0xffffffffu, ok ? e : -1);
        const int rank = __popc(grp & ((1u << lane) - 1u)), leader = __ffs(grp) - 1;
        for (int w = 0; w < kJobThreads / 32; ++w) {
            if (warp == w && ok) {
                int pos = 0;
                if (lane == leader) {
                    pos = cursor[e];
                    cursor[e] = pos + __popc(grp);
                }
                pos = __shfl_sync(grp, pos, leader);
                p.order[start[e] + pos + rank] = static_cast<int>(i);
            }
            __syncthreads();
        }
    }
    const int NJ = jstart[p.E];
    for (int jb = tid; jb < NJ; jb += kJobThreads) {
        int lo = 0, hi = p.E;                             // expert e with jstart[e] <= jb < jstart[e + 1]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (jstart[mid] <= jb) lo = mid;
            else hi = mid;
        }
        const int e = lo, part = jb - jstart[e], a = start[e] + part * kMaxTokensPerJob;
        const int m = min(kMaxTokensPerJob, cnt[e] - part * kMaxTokensPerJob);
        GemvJob j0{}, j1{};
        j0.w = p.w0 + static_cast<int64_t>(e) * p.bytes0;
        j1.w = p.w1 + static_cast<int64_t>(e) * p.bytes1;
        j0.m = j1.m = m;
        for (int n = 0; n < m; ++n) {
            const int slot = p.order[a + n];
            j0.xrow[n] = slot / p.k;
            j0.yrow[n] = j1.xrow[n] = j1.yrow[n] = slot;
        }
        p.jobs0[jb] = j0;
        p.jobs1[jb] = j1;
    }
    if (tid == 0) *p.njobs = NJ;
}

}  // namespace

cudaError_t expert_jobs_launch(const ExpertJobsParams &p, cudaStream_t stream) {
    if (p.TK <= 0) return cudaSuccess;
    const size_t smem = sizeof(int) * (3 * static_cast<size_t>(p.E) + 1 + p.E);
    expert_jobs_kernel<<<1, kJobThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t route_launch(const uint16_t *h, int64_t ldh, int64_t T, const uint16_t *wr, int E, int H, int k, int norm,
                         int32_t *ids, float *w, float *logits, cudaStream_t stream) {
    if (T <= 0) return cudaSuccess;
    route_kernel<<<static_cast<unsigned>(T), kRouterThreads, 2 * E * sizeof(float), stream>>>(h, ldh, wr, E, H, k, norm,
                                                                                              ids, w, logits);
    return cudaGetLastError();
}

}  // namespace onpu_b200
