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
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

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
    pdl_launch_dependents();              // the combine may launch now; it waits for this grid's end
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

// ---------------------------------------------------------------- tensor-core form (bf16 cache)
// For a bf16 cache with D = 64 or 128 and at most 8 query heads per kv head. Each warp is its own
// sub-split: it streams 16-row blocks of K and V through its shared memory (cp.async, two blocks
// in flight, 16-byte chunks swizzled by row so ldmatrix reads are conflict-free) and runs
//   scores[r][h] = K[r][:] . q[h][:]          mma m16n8k16: A = 16 rows of K, B = q^T (heads as n)
//   O^T[d][h]  += V^T[d][r] . P^T[r][h]        A = V^T (ldmatrix.trans), B = P^T
// with q and P each split into three bf16 parts (q = q1 + q2 + q3 exactly), so every product is
// exact in fp32 and the sums are fp32: the accuracy of the fp32 CUDA-core form, at a fraction of
// its instructions. The warp keeps its running max and sum per head in registers; the CTA's four
// warps merge theirs in shared memory and write one partial (max, sum, output) per CTA, which
// the combine kernel merges with the other splits'.
constexpr int kTcWarps = 4, kTcRows = 16;

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}
// x = p1 + p2 + p3 with each part a bf16 (the rounding residuals); exact for finite fp32 x
__device__ __forceinline__ void split3(float x, float &p1, float &p2, float &p3) {
    p1 = __bfloat162float(__float2bfloat16_rn(x));
    const float r1 = x - p1;
    p2 = __bfloat162float(__float2bfloat16_rn(r1));
    p3 = r1 - p2;
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

template <int D>
__global__ void __launch_bounds__(kTcWarps * 32) attn_split_tc_kernel(const AttnParams p) {
    constexpr int CPR = D / 8;                      // 16-byte chunks per row (8 or 16)
    constexpr int KS = D / 16;                      // k-steps of the score MMA, m-blocks of P . V
    constexpr int BLK = kTcRows * D;                // elements of one 16-row block
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_launch_dependents();              // the combine may launch now; it waits for this grid's end
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int rep = p.Hq / p.Hkv, kh = blockIdx.y, split = blockIdx.x;
    // per warp: [2 stages][K, V][16 rows][D] bf16, then a 8 x 16 float transpose buffer
    uint16_t *wbuf = reinterpret_cast<uint16_t *>(smem) + warp * (4 * BLK + 8 * kTcRows * 2);
    float *pbuf = reinterpret_cast<float *>(wbuf + 4 * BLK);
    const uint32_t wbase = static_cast<uint32_t>(__cvta_generic_to_shared(wbuf));

    // this warp's rows: the CTA's range cut in four, each a whole number of 16-row blocks
    const int64_t c0 = static_cast<int64_t>(split) * p.rows_per_split, c1 = min(p.S, c0 + p.rows_per_split);
    const int64_t per = ((c1 - c0 + kTcWarps * kTcRows - 1) / (kTcWarps * kTcRows)) * kTcRows;
    const int64_t j0 = min(c1, c0 + warp * per), j1 = min(c1, j0 + per);
    const int nblk = static_cast<int>((j1 - j0 + kTcRows - 1) / kTcRows);
    const uint16_t *Kb = static_cast<const uint16_t *>(p.k) + static_cast<int64_t>(kh) * p.hs;
    const uint16_t *Vb = static_cast<const uint16_t *>(p.v) + static_cast<int64_t>(kh) * p.hs;

    auto issue = [&](int b, int stage) {            // block b of this warp's rows into a stage
        const int64_t r0 = j0 + static_cast<int64_t>(b) * kTcRows;
        const int valid = static_cast<int>(min(static_cast<int64_t>(kTcRows), j1 - r0));
        uint16_t *ks = wbuf + stage * 2 * BLK, *vs = ks + BLK;
#pragma unroll
        for (int k = 0; k < kTcRows * CPR / 32; ++k) {
            const int idx = lane + 32 * k, r = idx / CPR, c = idx % CPR;
            const int off = r * D + ((c ^ (r & 7)) * 8);
            if (r < valid) {
                const int64_t go = (r0 + r) * p.rs + c * 8;
                cp_async16(ks + off, Kb + go);
                cp_async16(vs + off, Vb + go);
            } else {                                // rows past the range: zeros (never NaN garbage)
                *reinterpret_cast<uint4 *>(ks + off) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4 *>(vs + off) = make_uint4(0, 0, 0, 0);
            }
        }
        cp_async_commit();
    };
    if (nblk > 0) issue(0, 0);

    // q^T as B fragments, three bf16 parts: b0 = q[h=g][16k + 2t, +1], b1 = q[g][16k + 2t + 8, +9]
    uint32_t qb[3][KS][2];
    {
        const bool hv = g < rep;
        const float *qh = p.q + (static_cast<int64_t>(kh) * rep + (hv ? g : 0)) * D;
#pragma unroll
        for (int k = 0; k < KS; ++k)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int d = 16 * k + 2 * t + 8 * hh;
                const float x0 = hv ? qh[d] : 0.f, x1 = hv ? qh[d + 1] : 0.f;
                float a1, a2, a3, b1, b2, b3;
                split3(x0, a1, a2, a3);
                split3(x1, b1, b2, b3);
                qb[0][k][hh] = pack_bf16(a1, b1);
                qb[1][k][hh] = pack_bf16(a2, b2);
                qb[2][k][hh] = pack_bf16(a3, b3);
            }
    }
    float o[KS][4];
#pragma unroll
    for (int m = 0; m < KS; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.f;
    float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.f, 0.f};   // heads 2t, 2t+1
    const bool hv0 = 2 * t < rep, hv1 = 2 * t + 1 < rep;

    for (int b = 0; b < nblk; ++b) {
        const int stage = b & 1;
        __syncwarp();                               // every lane is past its reads of the stage refilled here
        if (b + 1 < nblk) {
            issue(b + 1, stage ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncwarp();
        const int64_t r0 = j0 + static_cast<int64_t>(b) * kTcRows;
        const uint32_t kbase = wbase + stage * 2 * BLK * 2, vbase = kbase + BLK * 2;
        // scores: rows g, g+8 of the block for heads 2t, 2t+1
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < KS; ++k) {
            const int mi = lane >> 3, row = (lane & 7) + (mi & 1) * 8, ch = 2 * k + (mi >> 1);
            uint32_t a[4];
            ldsm_x4(a, kbase + (row * D + ((ch ^ (row & 7)) * 8)) * 2);
            mma_bf16(sc, a, qb[0][k][0], qb[0][k][1]);
            mma_bf16(sc, a, qb[1][k][0], qb[1][k][1]);
            mma_bf16(sc, a, qb[2][k][0], qb[2][k][1]);
        }
        const bool rv0 = r0 + g < j1, rv1 = r0 + g + 8 < j1;
        const float mk0 = rv0 && p.mask ? p.mask[r0 + g] : 0.f, mk1 = rv1 && p.mask ? p.mask[r0 + g + 8] : 0.f;
        float s[4];
        s[0] = rv0 && hv0 ? sc[0] * p.scale + mk0 : -INFINITY;
        s[1] = rv0 && hv1 ? sc[1] * p.scale + mk0 : -INFINITY;
        s[2] = rv1 && hv0 ? sc[2] * p.scale + mk1 : -INFINITY;
        s[3] = rv1 && hv1 ? sc[3] * p.scale + mk1 : -INFINITY;
        float alpha[2], pr[4];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {            // head 2t + hh: its 16 rows sit on the 8 lanes of this t
            float mx = fmaxf(s[hh], s[hh + 2]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mnew = fmaxf(mrun[hh], mx);
            pr[hh] = mnew == -INFINITY ? 0.f : expf(s[hh] - mnew);
            pr[hh + 2] = mnew == -INFINITY ? 0.f : expf(s[hh + 2] - mnew);
            float sum = pr[hh] + pr[hh + 2];
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            sum += __shfl_xor_sync(0xffffffffu, sum, 8);
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            alpha[hh] = mrun[hh] == -INFINITY ? 0.f : expf(mrun[hh] - mnew);
            lrun[hh] = lrun[hh] * alpha[hh] + sum;
            mrun[hh] = mnew;
        }
        // P^T as B fragments: lane (g, t) needs P[h = g][r = 2t, 2t+1] and [2t+8, 2t+9]
        pbuf[(2 * t) * kTcRows + g] = pr[0];
        pbuf[(2 * t + 1) * kTcRows + g] = pr[1];
        pbuf[(2 * t) * kTcRows + g + 8] = pr[2];
        pbuf[(2 * t + 1) * kTcRows + g + 8] = pr[3];
        __syncwarp();
        uint32_t pb[3][2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const float2 v = *reinterpret_cast<const float2 *>(pbuf + g * kTcRows + 2 * t + 8 * hh);
            float a1, a2, a3, b1, b2, b3;
            split3(v.x, a1, a2, a3);
            split3(v.y, b1, b2, b3);
            pb[0][hh] = pack_bf16(a1, b1);
            pb[1][hh] = pack_bf16(a2, b2);
            pb[2][hh] = pack_bf16(a3, b3);
        }
        __syncwarp();                               // pbuf and this stage are reused next block
#pragma unroll
        for (int m = 0; m < KS; ++m) {
            o[m][0] *= alpha[0];
            o[m][1] *= alpha[1];
            o[m][2] *= alpha[0];
            o[m][3] *= alpha[1];
            // A = V^T (d 16m .. 16m+15 x rows 0..15): source matrices rows 0-7 / 8-15 at chunks 2m, 2m+1
            const int mi = lane >> 3, row = (lane & 7) + (mi >> 1) * 8, ch = 2 * m + (mi & 1);
            uint32_t a[4];
            ldsm_x4_t(a, vbase + (row * D + ((ch ^ (row & 7)) * 8)) * 2);
            mma_bf16(o[m], a, pb[0][0], pb[0][1]);
            mma_bf16(o[m], a, pb[1][0], pb[1][1]);
            mma_bf16(o[m], a, pb[2][0], pb[2][1]);
        }
    }
    // merge the four warps' partials in shared memory (the stage buffers are free: every warp
    // drained its copies with cp.async.wait_group 0), then write one partial per CTA.
    // o[m] holds O^T[d = 16m + g (+8)][h = 2t, 2t+1].
    __syncthreads();
    float *msm = reinterpret_cast<float *>(smem);                 // [warps][8 heads][max, sum]
    float *osm = msm + kTcWarps * 16;                             // [warps][8 heads][D]
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int h = 2 * t + hh;
        if (g == 0) {
            msm[(warp * 8 + h) * 2] = mrun[hh];
            msm[(warp * 8 + h) * 2 + 1] = lrun[hh];
        }
#pragma unroll
        for (int m = 0; m < KS; ++m) {
            osm[(warp * 8 + h) * D + 16 * m + g] = o[m][hh];
            osm[(warp * 8 + h) * D + 16 * m + g + 8] = o[m][hh + 2];
        }
    }
    __syncthreads();
    const int splits = p.splits;
    for (int i = threadIdx.x; i < rep * D; i += kTcWarps * 32) {
        const int h = i / D, d = i - h * D;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) mx = fmaxf(mx, msm[(w * 8 + h) * 2]);
        float ov = 0.f, lv = 0.f;
        if (mx != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kTcWarps; ++w) {
                const float mw = msm[(w * 8 + h) * 2];
                if (mw == -INFINITY) continue;
                const float e = expf(mw - mx);
                ov = fmaf(osm[(w * 8 + h) * D + d], e, ov);
                lv = fmaf(msm[(w * 8 + h) * 2 + 1], e, lv);
            }
        }
        const int64_t hq = static_cast<int64_t>(kh) * rep + h;
        p.part_o[(hq * splits + split) * D + d] = ov;
        if (d == 0) {
            p.part_ml[(hq * splits + split) * 2] = mx;
            p.part_ml[(hq * splits + split) * 2 + 1] = lv;
        }
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
    pdl_wait_prerequisites();             // launched early (programmatic dependent launch): wait for the partials
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

bool attn_use_tc(int D, int rep, bool bf16) { return bf16 && (D == 64 || D == 128) && rep <= 8; }
int attn_tc_warps() { return kTcWarps; }

// CTAs of the split kernel resident per SM (the host sizes the grid to one wave of them)
int attn_ctas_per_sm(int D, int rep, bool bf16) {
    if (!attn_use_tc(D, rep, bf16)) return 4;
    static int cached[2] = {0, 0};                   // D = 64, 128
    int &n = cached[D == 128];
    if (!n) {
        const int tsm = kTcWarps * (4 * kTcRows * D * 2 + 8 * kTcRows * 2 * 4);
        void (*k)(AttnParams) = D == 64 ? attn_split_tc_kernel<64> : attn_split_tc_kernel<128>;
        int blocks = 0;
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, tsm) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, kTcWarps * 32, tsm) != cudaSuccess)
            blocks = 0;
        n = blocks > 0 ? blocks : 1;
    }
    return n;
}
int attn_tc_rows() { return kTcRows; }

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
    if (p.S > 0 && attn_use_tc(p.D, rep, bf16)) {
        const dim3 grid(p.splits, p.Hkv);
        const int tsm = kTcWarps * (4 * kTcRows * p.D * 2 + 8 * kTcRows * 2 * 4);
        void (*k)(AttnParams) = p.D == 64 ? attn_split_tc_kernel<64> : attn_split_tc_kernel<128>;
        static bool attr[2] = {false, false};       // set once per kernel (no call during a graph capture)
        if (!attr[p.D == 128]) {
            const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, tsm);
            if (e != cudaSuccess) return e;
            attr[p.D == 128] = true;
        }
        k<<<grid, kTcWarps * 32, tsm, stream>>>(p);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    } else if (p.S > 0) {
        const dim3 grid(p.splits, p.Hkv);
        cudaError_t e;
        void (*k)(AttnParams) = nullptr;
        int slot = 0;
        switch (p.D) {
            case 64: k = bf16 ? attn_split_kernel<true, 64> : attn_split_kernel<false, 64>; slot = 0; break;
            case 128: k = bf16 ? attn_split_kernel<true, 128> : attn_split_kernel<false, 128>; slot = 1; break;
            case 256: k = bf16 ? attn_split_kernel<true, 256> : attn_split_kernel<false, 256>; slot = 2; break;
            default: k = bf16 ? attn_split_kernel<true, 0> : attn_split_kernel<false, 0>; slot = 3; break;
        }
        // set once per kernel, to the most any head size and head grouping it serves can use
        static bool attr[2][4] = {};
        if (!attr[bf16][slot]) {
            const int dmax = slot == 0 ? 64 : slot == 1 ? 128 : 256;
            e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     attn_smem_bytes(dmax, 16, attn_tile_rows(dmax, bf16), bf16));
            if (e != cudaSuccess) return e;
            attr[bf16][slot] = true;
        }
        k<<<grid, kAttnThreads, smem, stream>>>(p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(attn_combine_kernel, dim3(p.Hq), dim3(kCombineThreads), p.splits * sizeof(float), stream, p);
}

}  // namespace onpu_b200
