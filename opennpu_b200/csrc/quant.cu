// The load-time search quantisers on the GPU, bit-exact with the host ones.
//
// Restates, one thread per 32-group, the two searches of the reference's packer
// (llama/ggml-opennpu/opennpu_core.hpp:103-169, the same as host_codec.cpp here):
//  * q4nx (asymmetric, w = q·s + m): 21 stretches of the min..max grid; for each, the least-squares
//    (scale, min) of the codes it assigns, rounded to bf16, scored by the squared error of
//    re-quantising with them; the best (first on ties) wins; constant groups get s = 1, m = the
//    value;
//  * q4s (symmetric, w = (q - 8)·d): 16 divisors of the signed peak, least-squares d rounded to
//    bf16, same scoring; an all-zero group gets d = 1, codes 8.
// Every operation is an explicitly rounded fp32 operation in the host's order (no contraction
// into FMAs: the host is built with -ffp-contract=off), divisions are IEEE, rounding to integers is
// to nearest even (std::nearbyint), and min/max/clamp follow std::min/std::max, so NaN inputs take
// the same branches as on the host.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace onpu_b200 {

namespace {

__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float smin(float a, float b) { return b < a ? b : a; }       // std::min(a, b)
__device__ __forceinline__ float smax(float a, float b) { return a < b ? b : a; }       // std::max(a, b)
__device__ __forceinline__ float clamp_code(float v, float lo, float hi) { return smin(hi, smax(lo, v)); }

__device__ __forceinline__ uint16_t to_bf16(float f) {
    const uint32_t bits = __float_as_uint(f);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((bits >> 16) | 0x40u);
    const uint32_t lsb = (bits >> 16) & 1u;
    return static_cast<uint16_t>((bits + 0x7fffu + lsb) >> 16);
}
__device__ __forceinline__ float from_bf16(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }
__device__ __forceinline__ float bf16_round(float v) { return from_bf16(to_bf16(v)); }

__device__ void quant_asym(const float *x, uint8_t *q, uint16_t &s_bf, uint16_t &m_bf) {
    float lo = x[0], hi = x[0];
    for (int i = 1; i < 32; ++i) {
        lo = smin(lo, x[i]);
        hi = smax(hi, x[i]);
    }
    const float range = sub(hi, lo);
    if (!(range > 0)) {
        s_bf = to_bf16(1.0f);
        m_bf = to_bf16(lo);
        for (int i = 0; i < 32; ++i) q[i] = 0;
        return;
    }
    float best_err = __int_as_float(0x7f800000), best_s = __fdiv_rn(range, 15.0f), best_m = lo;
    for (int stretch = 0; stretch <= 20; ++stretch) {
        const float inv = __fdiv_rn(add(add(-1.0f, mul(0.1f, static_cast<float>(stretch))), 15.0f), range);
        float sum_l = 0, sum_ll = 0, sum_x = 0, sum_lx = 0;
        for (int i = 0; i < 32; ++i) {
            const float l = clamp_code(rintf(mul(inv, sub(x[i], lo))), 0.0f, 15.0f);
            sum_l = add(sum_l, l);
            sum_ll = add(sum_ll, mul(l, l));
            sum_x = add(sum_x, x[i]);
            sum_lx = add(sum_lx, mul(l, x[i]));
        }
        const float det = sub(mul(32.0f, sum_ll), mul(sum_l, sum_l));
        float sc = __fdiv_rn(range, 15.0f), mn = lo;
        if (det > 0) {
            sc = __fdiv_rn(sub(mul(32.0f, sum_lx), mul(sum_l, sum_x)), det);
            mn = __fdiv_rn(sub(mul(sum_ll, sum_x), mul(sum_l, sum_lx)), det);
        }
        sc = bf16_round(sc);
        mn = bf16_round(mn);
        if (!(sc > 0)) continue;
        float err = 0;
        for (int i = 0; i < 32; ++i) {
            const float l = clamp_code(rintf(__fdiv_rn(sub(x[i], mn), sc)), 0.0f, 15.0f);
            const float d = sub(add(mul(l, sc), mn), x[i]);
            err = add(err, mul(d, d));
        }
        if (err < best_err) {
            best_err = err;
            best_s = sc;
            best_m = mn;
        }
    }
    best_s = bf16_round(best_s);
    best_m = bf16_round(best_m);
    for (int i = 0; i < 32; ++i)
        q[i] = static_cast<uint8_t>(clamp_code(rintf(__fdiv_rn(sub(x[i], best_m), best_s)), 0.0f, 15.0f));
    s_bf = to_bf16(best_s);
    m_bf = to_bf16(best_m);
}

__device__ void quant_sym(const float *x, uint8_t *q, uint16_t &d_bf) {
    float peak = 0;
    for (int i = 0; i < 32; ++i)
        if (fabsf(x[i]) > fabsf(peak)) peak = x[i];
    if (peak == 0) {
        d_bf = to_bf16(1.0f);
        for (int i = 0; i < 32; ++i) q[i] = 8;
        return;
    }
    float best_err = __int_as_float(0x7f800000), best_d = __fdiv_rn(peak, -8.0f);
    for (int cand = 0; cand < 16; ++cand) {
        const float div = cand < 8 ? add(-9.0f, __fdiv_rn(mul(2.5f, static_cast<float>(cand)), 7.0f))
                                   : add(6.5f, __fdiv_rn(mul(1.5f, static_cast<float>(cand - 8)), 7.0f));
        const float d0 = __fdiv_rn(peak, div);
        float sum_vv = 0, sum_vx = 0;
        for (int i = 0; i < 32; ++i) {
            const float v = clamp_code(rintf(__fdiv_rn(x[i], d0)), -8.0f, 7.0f);
            sum_vv = add(sum_vv, mul(v, v));
            sum_vx = add(sum_vx, mul(v, x[i]));
        }
        float d = sum_vv > 0 ? __fdiv_rn(sum_vx, sum_vv) : d0;
        d = bf16_round(d);
        if (d == 0) continue;
        float err = 0;
        for (int i = 0; i < 32; ++i) {
            const float v = clamp_code(rintf(__fdiv_rn(x[i], d)), -8.0f, 7.0f);
            const float r = sub(mul(v, d), x[i]);
            err = add(err, mul(r, r));
        }
        if (err < best_err) {
            best_err = err;
            best_d = d;
        }
    }
    for (int i = 0; i < 32; ++i)
        q[i] = static_cast<uint8_t>(add(clamp_code(rintf(__fdiv_rn(x[i], best_d)), -8.0f, 7.0f), 8.0f));
    d_bf = to_bf16(best_d);
}

// one thread per 32-group of one row: W [N][ldw] fp32 -> codes q [N][K], scales / mins [N][K/32]
__global__ void __launch_bounds__(128) quant_kernel(const float *W, int64_t ldw, int64_t N, int64_t K, int sym,
                                                    uint8_t *q, uint16_t *scales, uint16_t *mins) {
    const int64_t G = K / 32;
    const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gid >= N * G) return;
    const int64_t row = gid / G, g = gid - row * G;
    float x[32];
    const float4 *src = reinterpret_cast<const float4 *>(W + row * ldw + g * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = src[i];
        x[4 * i] = v.x;
        x[4 * i + 1] = v.y;
        x[4 * i + 2] = v.z;
        x[4 * i + 3] = v.w;
    }
    uint8_t qc[32];
    uint16_t s = 0, m = 0;
    if (sym) quant_sym(x, qc, s);
    else quant_asym(x, qc, s, m);
    uint32_t *dst = reinterpret_cast<uint32_t *>(q + row * K + g * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        dst[i] = qc[4 * i] | (qc[4 * i + 1] << 8) | (qc[4 * i + 2] << 16) | (static_cast<uint32_t>(qc[4 * i + 3]) << 24);
    scales[row * G + g] = s;
    if (mins) mins[row * G + g] = sym ? uint16_t{0} : m;
}

// R = W - dequant(codes) with the host's rounding: (q - 8) * d, or q * s + m (a product then a sum,
// not contracted), then one subtraction - the residual rows of the two-pass (~8-bit) mode
__global__ void residual_kernel(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, const uint8_t *q,
                                const uint16_t *scales, const uint16_t *mins, float *R) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= N * K) return;
    const int64_t row = i / K, col = i - row * K, gidx = row * (K / 32) + col / 32;
    const float qf = static_cast<float>(q[i]);
    const float dq = sym ? mul(sub(qf, 8.0f), from_bf16(scales[gidx]))
                         : add(mul(qf, from_bf16(scales[gidx])), from_bf16(mins[gidx]));
    R[i] = sub(W[row * ldw + col], dq);
}

}  // namespace

cudaError_t residual_launch(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, const uint8_t *q,
                            const uint16_t *scales, const uint16_t *mins, float *R, cudaStream_t stream) {
    const int64_t n = N * K;
    if (n <= 0) return cudaSuccess;
    residual_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(W, ldw, N, K, sym, q, scales, mins, R);
    return cudaGetLastError();
}

cudaError_t quant_launch(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, uint8_t *q, uint16_t *scales,
                         uint16_t *mins, cudaStream_t stream) {
    const int64_t groups = N * (K / 32);
    if (groups <= 0) return cudaSuccess;
    quant_kernel<<<static_cast<unsigned>((groups + 127) / 128), 128, 0, stream>>>(W, ldw, N, K, sym, q, scales, mins);
    return cudaGetLastError();
}

}  // namespace onpu_b200
