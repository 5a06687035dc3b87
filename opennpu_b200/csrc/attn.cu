// One decode token of softmax attention over a KV cache (any GQA model), the step between the
// projections in decode: out[h] = softmax(scale * q[h] . K^T + mask, with an optional per-head
// sink logit that takes probability mass but has no value) . V, K and V the cache of kv head
// h / (Hq / Hkv). Follows onpu_attn_step / onpu_attn_step_bf16 (llama/ggml-opennpu/
// onpu_cpu.cpp:173-229): fp32 arithmetic, the cache fp32 or bf16, head stride hs and row stride
// rs in elements, mask [S] additive or null, sinks [Hq] or null.
//
// HBM-bound on the cache: 2 * Hkv * S * D * elt bytes per call. Split-KV: CTA (split, kv head)
// streams its rows of K and V once through shared memory (cp.async, two tiles in flight) for all
// Hq / Hkv query heads that share the kv head, keeping a running max, sum and unnormalised output
// per head (online softmax); a second kernel merges the splits and the sink per query head.
// Edge cases as the reference: S = 0 gives zeros; a cache whose every score is -inf, with no
// sink, gives NaN (exp(-inf - -inf)); with a sink it gives zeros.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kernels.h"

namespace onpu_b200 {
namespace {

constexpr int kAttnThreads = 256;

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// 16 bytes of cache -> floats: 4 fp32 or 8 bf16
template <bool BF16>
struct Chunk;
template <>
struct Chunk<false> {
    using T = float;
    static constexpr int kN = 4;
    __device__ static void get(const float *p, float (&f)[4]) {
        const float4 v = *reinterpret_cast<const float4 *>(p);
        f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
    }
    __device__ static float2 two(const float *p) { return *reinterpret_cast<const float2 *>(p); }
};
template <>
struct Chunk<true> {
    using T = uint16_t;
    static constexpr int kN = 8;
    __device__ static void get(const uint16_t *p, float (&f)[8]) {
        const uint4 v = *reinterpret_cast<const uint4 *>(p);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    __device__ static float2 two(const uint16_t *p) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    }
};

// DC: the head size as a compile-time constant (64, 128, 256), or 0 for any other (read from p)
template <bool BF16, int DC>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const AttnParams p) {
    using C = Chunk<BF16>;
    using T = typename C::T;
    constexpr int kN = C::kN;
    extern __shared__ __align__(16) uint8_t smem[];
    const int D = DC ? DC : p.D, rep = p.Hq / p.Hkv, R = p.tile_rows, cpr = D / kN;   // 16-byte chunks per row
    const int kh = blockIdx.y, split = blockIdx.x, tid = threadIdx.x;
    const int64_t j0 = static_cast<int64_t>(split) * p.rows_per_split;
    const int64_t j1 = min(p.S, j0 + p.rows_per_split);
    const int64_t tile_elems = static_cast<int64_t>(R) * D;
    T *tiles = reinterpret_cast<T *>(smem);                              // [2 buffers][K, V][R][D]
    float *qs = reinterpret_cast<float *>(smem + 4 * tile_elems * sizeof(T));
    float *os = qs + rep * D;                                            // running outputs [rep][D]
    float *sc = os + rep * D;                                            // scores / weights [rep][R]
    float *mrun = sc + rep * R, *lrun = mrun + rep, *alpha = lrun + rep;
    const T *Kb = static_cast<const T *>(p.k) + static_cast<int64_t>(kh) * p.hs;
    const T *Vb = static_cast<const T *>(p.v) + static_cast<int64_t>(kh) * p.hs;

    auto issue = [&](int64_t t0, int buf) {                              // rows t0 .. of K and V
        const int rows = static_cast<int>(min(static_cast<int64_t>(R), j1 - t0));
        T *kt = tiles + buf * 2 * tile_elems, *vt = kt + tile_elems;
        for (int c = tid; c < rows * cpr; c += kAttnThreads) {
            const int r = c / cpr, q = c - r * cpr;
            const int64_t go = (t0 + r) * p.rs + q * kN;
            cp_async16(kt + r * D + q * kN, Kb + go);
            cp_async16(vt + r * D + q * kN, Vb + go);
        }
        cp_async_commit();
    };
    const int ntiles = static_cast<int>((j1 - j0 + R - 1) / R);
    if (ntiles > 0) issue(j0, 0);
    for (int i = tid; i < rep * D; i += kAttnThreads) {
        qs[i] = p.q[static_cast<int64_t>(kh) * rep * D + i];
        os[i] = 0.f;
    }
    if (tid < rep) {
        mrun[tid] = -INFINITY;
        lrun[tid] = 0.f;
    }
    const int warp = tid >> 5, lane = tid & 31;
    for (int t = 0; t < ntiles; ++t) {
        const int64_t t0 = j0 + static_cast<int64_t>(t) * R;
        const int rows = static_cast<int>(min(static_cast<int64_t>(R), j1 - t0));
        if (t + 1 < ntiles) {
            issue(t0 + R, (t + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const T *kt = tiles + (t & 1) * 2 * tile_elems, *vt = kt + tile_elems;
        // scores: one (head, row) per thread; each row's chunks start at a rotated index so the
        // rows read by one warp fall in different banks
        for (int i = tid; i < rep * R; i += kAttnThreads) {
            const int h = i / R, r = i - h * R;
            float s = -INFINITY;
            if (r < rows) {
                const float *qh = qs + h * D;
                const T *kr = kt + r * D;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};        // independent chains
                const int rot = r % cpr;                      // once per score, not per chunk
#pragma unroll(DC ? DC / kN : 1)
                for (int c0 = 0; c0 < cpr; ++c0) {
                    int c = c0 + rot;
                    c -= c >= cpr ? cpr : 0;
                    float f[kN];
                    C::get(kr + c * kN, f);
#pragma unroll
                    for (int e = 0; e < kN; e += 4) {
                        const float4 qv = *reinterpret_cast<const float4 *>(qh + c * kN + e);
                        acc[0] = fmaf(qv.x, f[e], acc[0]);
                        acc[1] = fmaf(qv.y, f[e + 1], acc[1]);
                        acc[2] = fmaf(qv.z, f[e + 2], acc[2]);
                        acc[3] = fmaf(qv.w, f[e + 3], acc[3]);
                    }
                }
                s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) * p.scale + (p.mask ? p.mask[t0 + r] : 0.f);
            }
            sc[i] = s;
        }
        __syncthreads();
        // online softmax, one warp per head
        for (int h = warp; h < rep; h += kAttnThreads / 32) {
            float mx = -INFINITY;
            for (int r = lane; r < R; r += 32) mx = fmaxf(mx, sc[h * R + r]);
            mx = warp_max(mx);
            const float mold = mrun[h], mnew = fmaxf(mold, mx);
            float sum = 0.f;
            for (int r = lane; r < R; r += 32) {
                const float e = mnew == -INFINITY ? 0.f : expf(sc[h * R + r] - mnew);
                sc[h * R + r] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float a = mold == -INFINITY ? 0.f : expf(mold - mnew);
                alpha[h] = a;
                lrun[h] = lrun[h] * a + sum;
                mrun[h] = mnew;
            }
        }
        __syncthreads();
        // outputs: two adjacent (head, d) per thread, rescaled by the new max, plus this tile's
        // p . V (even and odd rows in separate sums)
        for (int i = tid; i < rep * D / 2; i += kAttnThreads) {
            const int h = (2 * i) / D, d = 2 * i - h * D;
            const float *ph = sc + h * R;
            float2 ev = make_float2(0.f, 0.f), od = make_float2(0.f, 0.f);
            int r = 0;
            for (; r + 1 < rows; r += 2) {
                const float2 v0 = C::two(vt + r * D + d), v1 = C::two(vt + (r + 1) * D + d);
                const float p0 = ph[r], p1 = ph[r + 1];
                ev.x = fmaf(p0, v0.x, ev.x);
                ev.y = fmaf(p0, v0.y, ev.y);
                od.x = fmaf(p1, v1.x, od.x);
                od.y = fmaf(p1, v1.y, od.y);
            }
            if (r < rows) {
                const float2 v0 = C::two(vt + r * D + d);
                ev.x = fmaf(ph[r], v0.x, ev.x);
                ev.y = fmaf(ph[r], v0.y, ev.y);
            }
            float2 *o = reinterpret_cast<float2 *>(os + h * D + d);
            const float a = alpha[h];
            *o = make_float2(fmaf(o->x, a, ev.x + od.x), fmaf(o->y, a, ev.y + od.y));
        }
        __syncthreads();        // the buffer read here is refilled by the next iteration's issue
    }
    const int splits = p.splits;
    for (int i = tid; i < rep * D; i += kAttnThreads) {
        const int h = i / D, d = i - h * D, hq = kh * rep + h;
        p.part_o[(static_cast<int64_t>(hq) * splits + split) * D + d] = os[i];
    }
    if (tid < rep) {
        const int hq = kh * rep + tid;
        p.part_ml[(static_cast<int64_t>(hq) * splits + split) * 2] = mrun[tid];
        p.part_ml[(static_cast<int64_t>(hq) * splits + split) * 2 + 1] = lrun[tid];
    }
}

// per query head: merge the splits' (max, sum, output) and the sink. The splits' weights
// exp(m_s - m) go to shared memory once; each warp then sums a share of the splits for 128
// outputs at a time (4 per lane, float4 loads all in flight), and the warps' sums are added
// in shared memory.
constexpr int kCombineThreads = 256, kCombineWarps = kCombineThreads / 32;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float *red) {
    v = is_max ? warp_max(v) : warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();                      // red is reused between calls
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < kCombineWarps; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
    return r;
}

__global__ void __launch_bounds__(kCombineThreads) attn_combine_kernel(const AttnParams p) {
    extern __shared__ float wsm[];        // [splits] weights
    __shared__ float red[kCombineWarps];
    __shared__ float4 acc[kCombineWarps][32];
    const int h = blockIdx.x, D = p.D, splits = p.splits, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float *ml = p.part_ml + static_cast<int64_t>(h) * splits * 2;
    const float *po = p.part_o + static_cast<int64_t>(h) * splits * D;
    float *out = p.out + static_cast<int64_t>(h) * D;
    if (p.S == 0) {                       // no rows: the reference's output stays zero
        for (int d = tid; d < D; d += kCombineThreads) out[d] = 0.f;
        return;
    }
    const float sink = p.sinks ? p.sinks[h] : -INFINITY;
    float m = -INFINITY;
    for (int s = tid; s < splits; s += kCombineThreads) m = fmaxf(m, ml[2 * s]);
    m = fmaxf(block_reduce(m, true, red), sink);
    if (m == -INFINITY) {                 // every score -inf and no sink: exp(-inf - -inf) in the reference
        for (int d = tid; d < D; d += kCombineThreads) out[d] = NAN;
        return;
    }
    float l = 0.f;
    for (int s = tid; s < splits; s += kCombineThreads) {
        const float ms = ml[2 * s], w = ms == -INFINITY ? 0.f : expf(ms - m);
        wsm[s] = w;
        l = fmaf(ml[2 * s + 1], w, l);
    }
    l = block_reduce(l, false, red) + (p.sinks ? expf(sink - m) : 0.f);   // also publishes wsm
    const float inv = 1.0f / l;
    for (int d0 = 0; d0 < D; d0 += 128) {                 // D % 4 == 0
        const int d = d0 + 4 * lane;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (d < D) {
#pragma unroll 4
            for (int s = warp; s < splits; s += kCombineWarps) {
                const float4 v = *reinterpret_cast<const float4 *>(po + static_cast<int64_t>(s) * D + d);
                const float w = wsm[s];
                o.x = fmaf(v.x, w, o.x);
                o.y = fmaf(v.y, w, o.y);
                o.z = fmaf(v.z, w, o.z);
                o.w = fmaf(v.w, w, o.w);
            }
        }
        acc[warp][lane] = o;
        __syncthreads();
        if (warp == 0 && d < D) {
            float4 t = acc[0][lane];
            for (int w = 1; w < kCombineWarps; ++w) {
                const float4 u = acc[w][lane];
                t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
            }
            out[d] = t.x * inv;           // scalar stores: out is only 4-byte aligned
            out[d + 1] = t.y * inv;
            out[d + 2] = t.z * inv;
            out[d + 3] = t.w * inv;
        }
        __syncthreads();
    }
}

}  // namespace

int attn_tile_rows(int D, bool bf16) {
    const int row = D * (bf16 ? 2 : 4);
    const int r = 8192 / row / 8 * 8;     // four tiles (two buffers of K and V) in <= 32 KB: ~6 CTAs per SM
    return r < 8 ? 8 : (r > 64 ? 64 : r);
}

int attn_smem_bytes(int D, int rep, int R, bool bf16) {
    return 4 * R * D * (bf16 ? 2 : 4) + (2 * rep * D + rep * R + 3 * rep) * 4;
}

cudaError_t attn_launch(const AttnParams &p, bool bf16, cudaStream_t stream) {
    const int rep = p.Hq / p.Hkv, smem = attn_smem_bytes(p.D, rep, p.tile_rows, bf16);
    if (p.S > 0) {
        const dim3 grid(p.splits, p.Hkv);
        cudaError_t e;
        void (*k)(AttnParams) = nullptr;
        switch (p.D) {
            case 64: k = bf16 ? attn_split_kernel<true, 64> : attn_split_kernel<false, 64>; break;
            case 128: k = bf16 ? attn_split_kernel<true, 128> : attn_split_kernel<false, 128>; break;
            case 256: k = bf16 ? attn_split_kernel<true, 256> : attn_split_kernel<false, 256>; break;
            default: k = bf16 ? attn_split_kernel<true, 0> : attn_split_kernel<false, 0>; break;
        }
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        k<<<grid, kAttnThreads, smem, stream>>>(p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    attn_combine_kernel<<<p.Hq, kCombineThreads, p.splits * sizeof(float), stream>>>(p);
    return cudaGetLastError();
}

}  // namespace onpu_b200
