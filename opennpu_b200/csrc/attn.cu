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
    __device__ static float one(const float *p) { return *p; }
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
    __device__ static float one(const uint16_t *p) { return __uint_as_float(static_cast<uint32_t>(*p) << 16); }
};

template <bool BF16>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const AttnParams p) {
    using C = Chunk<BF16>;
    using T = typename C::T;
    constexpr int kN = C::kN;
    extern __shared__ __align__(16) uint8_t smem[];
    const int D = p.D, rep = p.Hq / p.Hkv, R = p.tile_rows, cpr = D / kN;   // 16-byte chunks per row
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
                float acc = 0.f;
                for (int c0 = 0; c0 < cpr; ++c0) {
                    const int c = (c0 + r) % cpr;
                    float f[kN];
                    C::get(kr + c * kN, f);
#pragma unroll
                    for (int e = 0; e < kN; ++e) acc = fmaf(qh[c * kN + e], f[e], acc);
                }
                s = acc * p.scale + (p.mask ? p.mask[t0 + r] : 0.f);
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
        // outputs: one (head, d) per thread, rescaled by the new max, plus this tile's p . V
        for (int i = tid; i < rep * D; i += kAttnThreads) {
            const int h = i / D, d = i - h * D;
            const float *ph = sc + h * R;
            float o = os[i] * alpha[h];
            for (int r = 0; r < rows; ++r) o = fmaf(ph[r], C::one(vt + r * D + d), o);
            os[i] = o;
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

// per query head: merge the splits' (max, sum, output) and the sink
__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnParams p) {
    const int h = blockIdx.x, D = p.D, splits = p.splits;
    const float *ml = p.part_ml + static_cast<int64_t>(h) * splits * 2;
    const float *po = p.part_o + static_cast<int64_t>(h) * splits * D;
    float *out = p.out + static_cast<int64_t>(h) * D;
    if (p.S == 0) {                       // no rows: the reference's output stays zero
        for (int d = threadIdx.x; d < D; d += blockDim.x) out[d] = 0.f;
        return;
    }
    const float sink = p.sinks ? p.sinks[h] : -INFINITY;
    float m = sink;
    for (int s = 0; s < splits; ++s) m = fmaxf(m, ml[2 * s]);
    if (m == -INFINITY) {                 // every score -inf and no sink: exp(-inf - -inf) in the reference
        for (int d = threadIdx.x; d < D; d += blockDim.x) out[d] = NAN;
        return;
    }
    float l = p.sinks ? expf(sink - m) : 0.f;
    for (int s = 0; s < splits; ++s) {
        const float ms = ml[2 * s];
        if (ms != -INFINITY) l += ml[2 * s + 1] * expf(ms - m);
    }
    const float inv = 1.0f / l;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float o = 0.f;
        for (int s = 0; s < splits; ++s) {
            const float ms = ml[2 * s];
            if (ms != -INFINITY) o = fmaf(po[static_cast<int64_t>(s) * D + d], expf(ms - m), o);
        }
        out[d] = o * inv;
    }
}

}  // namespace

int attn_tile_rows(int D, bool bf16) {
    const int row = D * (bf16 ? 2 : 4);
    const int r = 16384 / row / 8 * 8;    // four tiles (two buffers of K and V) in <= 64 KB
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
        if (bf16) {
            e = cudaFuncSetAttribute(attn_split_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
            attn_split_kernel<true><<<grid, kAttnThreads, smem, stream>>>(p);
        } else {
            e = cudaFuncSetAttribute(attn_split_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
            attn_split_kernel<false><<<grid, kAttnThreads, smem, stream>>>(p);
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    attn_combine_kernel<<<p.Hq, 128, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace onpu_b200
