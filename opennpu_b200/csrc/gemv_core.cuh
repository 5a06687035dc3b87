// Device building blocks shared by the int4 GEMV kernels (gemv.cu: one matrix per launch;
// chain.cu: a sequence of matrices per launch): pipeline constants, code unpacking, the
// tensor-core strip x chunk product.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gpu_layout.cuh"
#include "ptx.cuh"

namespace onpu_b200 {
namespace gemv_core {

constexpr int kConsumers = 4;                      // one warp per 16-row strip
constexpr int kThreads = (kConsumers + 1) * 32;    // + the producer warp
constexpr int kCPS = 4, kNS = 8;                   // chunks per stage, stages
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // a copy that has not landed in 2 s is a fault
constexpr int kSlotFloats = 4 * 8 * 2 * 16;        // [strip][r][h][token] head partial sums of a CTA
constexpr int kPartBatch = 4;                       // partners whose partial sums are loaded at once
constexpr int kXSlot = 192;                        // per-stage activation slot: 128 B + 64 B pad

__host__ __device__ constexpr int stage_w_bytes(int fmt) { return kCPS * chunk_bytes(fmt); }

// two 16-bit scale/min values (strip rows r, r+8) -> fp32; mul[3] = 2^16 (an FMA-pipe shift)
template <int FMT>
__device__ __forceinline__ void decode_pair(uint32_t w, const uint32_t (&mul)[4], float &lo, float &hi) {
    if constexpr (FMT == kFmtQ4F16) {
        lo = __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
        hi = __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
    } else {
        lo = __uint_as_float(w * mul[3]);
        hi = __uint_as_float(w & 0xffff0000u);
    }
}

// Codes of one packed word -> the four bf16x2 A registers (128 + q). The right shifts are
// mul.hi by 2^28 / 2^24 / 2^20 passed in as kernel parameters: they run on the FMA pipe instead
// of the half-rate integer pipe, which the mask-and-OR (LOP3) already keeps busy.
__device__ __forceinline__ void codes_to_a(uint32_t w, const uint32_t (&mul)[4], uint32_t (&a)[4]) {
    a[0] = (w & 0x000F000Fu) | 0x43004300u;
    a[1] = (__umulhi(w, mul[0]) & 0x000F000Fu) | 0x43004300u;
    a[2] = (__umulhi(w, mul[1]) & 0x000F000Fu) | 0x43004300u;
    a[3] = (__umulhi(w, mul[2]) & 0x000F000Fu) | 0x43004300u;
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                         const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

__device__ __forceinline__ int worker_of(int c, int W, int T) {
    return static_cast<int>((static_cast<int64_t>(c + 1) * W - 1) / T);
}

// CTA w of W owns chunks [w*T/W, (w+1)*T/W): empty when there are fewer chunks than CTAs
__device__ __forceinline__ bool range_empty(int w, int W, int T) {
    return static_cast<int64_t>(w) * T / W == static_cast<int64_t>(w + 1) * T / W;
}

// One strip (16 rows) x one chunk (2 groups of 32 along K) into acc. wsb: the strip's bytes in
// shared memory; xa[nt]: shared address of this lane's 8 activations of the chunk's first group
// for n-tile nt (the second group is 64 B further; absent tokens read zeros).
// Without a table (CI false): symmetric codes (128+q) - 136 = q - 8 exactly in bf16,
// D = sum((q-8) x), acc += s * D; q4nx (128+q) - 128 = q, acc += s * sum(q x) + m * sum(x), with
// sum(x) from an MMA against ones. With a table (CI true, resident activations): the MMA starts
// from c * sum(x) read from shared memory at ca (+ gi * 8 * MT; c = -136 symmetric, -128 q4nx),
// so the 128 + q codes go into the MMA as they are.
template <int FMT, int NT, bool CI>
__device__ __forceinline__ void strip_chunk(uint32_t wsb, const uint32_t (&xa)[NT], uint32_t ca, int lane, int r,
                                            const uint32_t (&mul)[4], float (&acc)[NT][4]) {
    const uint32_t off = FMT == kFmtQ4NX ? 0x43004300u : 0x43084308u;   // bf16x2 (128) / (136)
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t bx[2][NT][4];
#pragma unroll
    for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint4 v = lds_v4(xa[nt] + gi * 64);
            bx[gi][nt][0] = v.x; bx[gi][nt][1] = v.y; bx[gi][nt][2] = v.z; bx[gi][nt][3] = v.w;
        }
    const uint4 code = lds_v4(wsb + lane * 16);
    const uint2 sc = lds_v2(wsb + kCodeBytes + r * 8);
    uint2 mn = make_uint2(0, 0);
    if constexpr (FMT == kFmtQ4NX) mn = lds_v2(wsb + kCodeBytes + kScaleBytes + r * 8);
    constexpr int MT = 8 * NT;
    float cinit[2][NT][4];
    if constexpr (CI) {
#pragma unroll
        for (int gi = 0; gi < 2; ++gi)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint2 c2 = lds_v2(ca + (gi * MT + nt * 8) * 4);
                cinit[gi][nt][0] = cinit[gi][nt][2] = __uint_as_float(c2.x);
                cinit[gi][nt][1] = cinit[gi][nt][3] = __uint_as_float(c2.y);
            }
    }
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
        uint32_t a0[4], a1[4];
        codes_to_a(gi ? code.z : code.x, mul, a0);
        codes_to_a(gi ? code.w : code.y, mul, a1);
        if constexpr (!CI) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a0[i] = bf16x2_sub(a0[i], off);
                a1[i] = bf16x2_sub(a1[i], off);
            }
        }
        float s_lo, s_hi;
        decode_pair<FMT>(gi ? sc.y : sc.x, mul, s_lo, s_hi);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float d[4];
            if constexpr (CI) mma16816(d, a0, bx[gi][nt][0], bx[gi][nt][1], cinit[gi][nt]);
            else mma16816(d, a0, bx[gi][nt][0], bx[gi][nt][1], zero4);
            mma16816(d, a1, bx[gi][nt][2], bx[gi][nt][3], d);
            acc[nt][0] = fmaf(s_lo, d[0], acc[nt][0]);
            acc[nt][1] = fmaf(s_lo, d[1], acc[nt][1]);
            acc[nt][2] = fmaf(s_hi, d[2], acc[nt][2]);
            acc[nt][3] = fmaf(s_hi, d[3], acc[nt][3]);
            if constexpr (FMT == kFmtQ4NX && CI) {
                float m_lo, m_hi;
                decode_pair<FMT>(gi ? mn.y : mn.x, mul, m_lo, m_hi);
                m_lo *= -0.0078125f;                       // cinit = -128 sum(x): m * sum(x)
                m_hi *= -0.0078125f;
                acc[nt][0] = fmaf(m_lo, cinit[gi][nt][0], acc[nt][0]);
                acc[nt][1] = fmaf(m_lo, cinit[gi][nt][1], acc[nt][1]);
                acc[nt][2] = fmaf(m_hi, cinit[gi][nt][2], acc[nt][2]);
                acc[nt][3] = fmaf(m_hi, cinit[gi][nt][3], acc[nt][3]);
            }
            if constexpr (FMT == kFmtQ4NX && !CI) {
                float m_lo, m_hi, xs[4];
                decode_pair<FMT>(gi ? mn.y : mn.x, mul, m_lo, m_hi);
                const uint32_t ones[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
                mma16816(xs, ones, bx[gi][nt][0], bx[gi][nt][1], zero4);
                mma16816(xs, ones, bx[gi][nt][2], bx[gi][nt][3], xs);
                acc[nt][0] = fmaf(m_lo, xs[0], acc[nt][0]);
                acc[nt][1] = fmaf(m_lo, xs[1], acc[nt][1]);
                acc[nt][2] = fmaf(m_hi, xs[2], acc[nt][2]);
                acc[nt][3] = fmaf(m_hi, xs[3], acc[nt][3]);
            }
        }
    }
}

// ================================================================ fp16 path (resident activations)
// The resident kernels feed the tensor cores fp16 subnormals: a code q masked into the low
// mantissa bits with a zero exponent is the fp16 value q * 2^-24 exactly. Strip rows r take
// mask 0x000F000F (q * 2^-24), rows r+8 mask 0x00F000F0 (16 q * 2^-24), one AND each from the
// packed word or the word >> 8: 5 instructions per 8 codes, no bias to remove. Symmetric formats
// start each group's MMA from -8 * 2^-24 * sum(x) (x 16 on rows r+8), read from a table of group
// sums written at staging; this offset is of the size of the products' sum (q in 0..15 against
// 8), so the fp32 accumulation keeps its precision (a 1024 + q encoding with the offset applied
// the same way cancels ~1000x larger partial sums). q4nx starts from 0 and adds m * sum(x) * 2^-24
// from the same table. The factors 2^-24 and 16 are removed exactly (powers of two) at the end of
// a segment (finish_rows). The activations are staged as fp16 (scaled per token by a power of
// two when |x| would leave the fp16 range). The weights are never rounded.
struct Unpack {
    uint32_t mlo, mhi, magic;      // 0x000F000F, 0x00F000F0, 0x64006400 (kernel parameters: kept in registers;
                                   // the fp16 path uses the two masks)
};

// 8 codes -> the A registers as exact fp16 subnormals: rows r hold q * 2^-24, rows r+8
// 16 q * 2^-24 (nibbles 0/4 and 1/5 of w, 2/6 and 3/7 of w >> 8)
__device__ __forceinline__ void codes_to_a_h(uint32_t w, const Unpack &u, uint32_t (&a)[4]) {
    const uint32_t s = w >> 8;
    a[0] = w & u.mlo;
    a[1] = w & u.mhi;
    a[2] = s & u.mlo;
    a[3] = s & u.mhi;
}

// Group-sum table entry per fp32 sum of a group's fp16 activations: the MMA's starting value on
// rows r for the symmetric formats (-8 * 2^-24), the min term's factor for q4nx (2^-24)
template <int FMT>
__host__ __device__ constexpr float tab_factor() { return FMT == kFmtQ4NX ? 0x1p-24f : -0x1p-21f; }

__device__ __forceinline__ void mma16816_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// the same from C = {c0, c1, c2, c3}
__device__ __forceinline__ void mma16816_f16_c(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                               float c0, float c1, float c2, float c3) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

// the same with C = 0 (a fresh per-group sum: no register copies of zeros)
__device__ __forceinline__ void mma16816_f16_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// offset table bytes per 64-K chunk: [group][n-tile][t][2 floats] = sum(x) of tokens 2t, 2t+1
__host__ __device__ constexpr int tab_chunk_bytes(int nt) { return 2 * nt * 4 * 8; }

// One strip x one chunk, fp16 path. xa[nt]: this lane's fp16 activations of the chunk's first
// group (second group 64 B further); ca: this lane's offset-table entry of the chunk (t * 8 in).
template <int FMT, int NT>
__device__ __forceinline__ void strip_chunk_h(uint32_t wsb, const uint32_t (&xa)[NT], uint32_t ca, int lane, int r,
                                              const uint32_t (&mul)[4], const Unpack &u, float (&acc)[NT][4]) {
    uint32_t bx[2][NT][4];
#pragma unroll
    for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint4 v = lds_v4(xa[nt] + gi * 64);
            bx[gi][nt][0] = v.x; bx[gi][nt][1] = v.y; bx[gi][nt][2] = v.z; bx[gi][nt][3] = v.w;
        }
    const uint4 code = lds_v4(wsb + lane * 16);
    const uint2 sc = lds_v2(wsb + kCodeBytes + r * 8);
    uint2 mn = make_uint2(0, 0);
    if constexpr (FMT == kFmtQ4NX) mn = lds_v2(wsb + kCodeBytes + kScaleBytes + r * 8);
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
        uint32_t a0[4], a1[4];
        codes_to_a_h(gi ? code.z : code.x, u, a0);
        codes_to_a_h(gi ? code.w : code.y, u, a1);
        float s_lo, s_hi;
        decode_pair<FMT>(gi ? sc.y : sc.x, mul, s_lo, s_hi);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint2 c2 = lds_v2(ca + (gi * NT + nt) * 32);
            const float x0 = __uint_as_float(c2.x), x1 = __uint_as_float(c2.y);
            float d[4];
            if constexpr (FMT == kFmtQ4NX) mma16816_f16_z(d, a0, bx[gi][nt][0], bx[gi][nt][1]);
            else mma16816_f16_c(d, a0, bx[gi][nt][0], bx[gi][nt][1], x0, x1, 16.0f * x0, 16.0f * x1);
            mma16816_f16(d, a1, bx[gi][nt][2], bx[gi][nt][3]);
            acc[nt][0] = fmaf(s_lo, d[0], acc[nt][0]);
            acc[nt][1] = fmaf(s_lo, d[1], acc[nt][1]);
            acc[nt][2] = fmaf(s_hi, d[2], acc[nt][2]);
            acc[nt][3] = fmaf(s_hi, d[3], acc[nt][3]);
            if constexpr (FMT == kFmtQ4NX) {
                // + m * sum(x) on rows r, 16 m * sum(x) on rows r+8
                float m_lo, m_hi;
                decode_pair<FMT>(gi ? mn.y : mn.x, mul, m_lo, m_hi);
                m_hi *= 16.0f;
                acc[nt][0] = fmaf(m_lo, x0, acc[nt][0]);
                acc[nt][1] = fmaf(m_lo, x1, acc[nt][1]);
                acc[nt][2] = fmaf(m_hi, x0, acc[nt][2]);
                acc[nt][3] = fmaf(m_hi, x1, acc[nt][3]);
            }
        }
    }
}

// One whole chunk (all 4 strips) by one warp, fp16 path: the activations (and for q4nx their
// group sums) are read once per chunk and shared by the strips. wcb: the chunk in shared
// memory; xa/ca as in strip_chunk_h; acc[strip][n-tile][4].
template <int FMT, int NT>
__device__ __forceinline__ void chunk_h(uint32_t wcb, const uint32_t (&xa)[NT], uint32_t ca, int lane, int r,
                                        const uint32_t (&mul)[4], const Unpack &u, float (&acc)[4][NT][4]) {
    constexpr int SB = strip_bytes(FMT);
    uint32_t bx[2][NT][4];
    float xs[2][NT][2];
#pragma unroll
    for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint4 v = lds_v4(xa[nt] + gi * 64);
            bx[gi][nt][0] = v.x; bx[gi][nt][1] = v.y; bx[gi][nt][2] = v.z; bx[gi][nt][3] = v.w;
            const uint2 c2 = lds_v2(ca + (gi * NT + nt) * 32);
            xs[gi][nt][0] = __uint_as_float(c2.x);
            xs[gi][nt][1] = __uint_as_float(c2.y);
        }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const uint4 code = lds_v4(wcb + s * SB + lane * 16);
        const uint2 sc = lds_v2(wcb + s * SB + kCodeBytes + r * 8);
        uint2 mn = make_uint2(0, 0);
        if constexpr (FMT == kFmtQ4NX) mn = lds_v2(wcb + s * SB + kCodeBytes + kScaleBytes + r * 8);
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            uint32_t a0[4], a1[4];
            codes_to_a_h(gi ? code.z : code.x, u, a0);
            codes_to_a_h(gi ? code.w : code.y, u, a1);
            float s_lo, s_hi;
            decode_pair<FMT>(gi ? sc.y : sc.x, mul, s_lo, s_hi);
            float m_lo = 0.f, m_hi = 0.f;
            if constexpr (FMT == kFmtQ4NX) {
                decode_pair<FMT>(gi ? mn.y : mn.x, mul, m_lo, m_hi);
                m_hi *= 16.0f;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float x0 = xs[gi][nt][0], x1 = xs[gi][nt][1];
                float d[4];
                if constexpr (FMT == kFmtQ4NX) mma16816_f16_z(d, a0, bx[gi][nt][0], bx[gi][nt][1]);
                else mma16816_f16_c(d, a0, bx[gi][nt][0], bx[gi][nt][1], x0, x1, 16.0f * x0, 16.0f * x1);
                mma16816_f16(d, a1, bx[gi][nt][2], bx[gi][nt][3]);
                acc[s][nt][0] = fmaf(s_lo, d[0], acc[s][nt][0]);
                acc[s][nt][1] = fmaf(s_lo, d[1], acc[s][nt][1]);
                acc[s][nt][2] = fmaf(s_hi, d[2], acc[s][nt][2]);
                acc[s][nt][3] = fmaf(s_hi, d[3], acc[s][nt][3]);
                if constexpr (FMT == kFmtQ4NX) {
                    acc[s][nt][0] = fmaf(m_lo, x0, acc[s][nt][0]);
                    acc[s][nt][1] = fmaf(m_lo, x1, acc[s][nt][1]);
                    acc[s][nt][2] = fmaf(m_hi, x0, acc[s][nt][2]);
                    acc[s][nt][3] = fmaf(m_hi, x1, acc[s][nt][3]);
                }
            }
        }
    }
}

// Bytes of the buffer in which the 4 consumer warps combine their per-strip partial sums:
// [warp][strip][lane][n-tile * 4 floats]
__host__ __device__ constexpr int combine_bytes(int nt) { return 4 * 4 * 32 * nt * 16; }

// Resident activation region: m rows of xstride bytes (fp16), a 128-B zero block, the offset table
// (chunks * tab_chunk_bytes), then 16 token scales (float) and 16 token maxima (uint).
__host__ __device__ inline int64_t xres_bytes(int64_t m, int64_t K, int nt, int64_t xstride) {
    const int64_t chunks = (K + kChunkK - 1) / kChunkK;
    return m * xstride + 128 + chunks * tab_chunk_bytes(nt) + 128;
}
__host__ __device__ inline int64_t xres_stride(int64_t K) { return (K * 2 + 127) / 128 * 128 + 64; }   // 64 B off mod 128

// Convert 32 bf16 activations (4 x 16 B) to fp16, returning their fp16-rounded sum and max |x|
// (as fp32 bits); inv scales them first (a power of two).
// SUM: also return the group's sum (the fp16 path's table of group sums); the pair conversion is
// one packed cvt, so staging is not held up by the conversion unit
template <bool SUM>
__device__ __forceinline__ float group_to_f16(uint4 (&v)[4], float inv, uint32_t &mx) {
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t w4[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float lo = __uint_as_float(w4[k] << 16) * inv, hi = __uint_as_float(w4[k] & 0xffff0000u) * inv;
            mx = max(mx, max(__float_as_uint(fabsf(lo)), __float_as_uint(fabsf(hi))));
            const __half2 h2 = __floats2half2_rn(lo, hi);          // .x = lo (low half), .y = hi
            if constexpr (SUM) {
                const float2 f = __half22float2(h2);
                sum += f.x + f.y;
            }
            w4[k] = *reinterpret_cast<const uint32_t *>(&h2);
        }
        v[q] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
    return sum;
}

// 8 fp32 activations (2 x 16 B) -> 16 B of each fp16 row: h = fp16(x * inv), l = fp16(x * inv - h),
// so h + l carries x to ~22 significant bits; sh / sl accumulate their fp32 sums, mx the max
// |x * inv| (fp32 bits)
__device__ __forceinline__ void split8_f16(const uint4 &a4, const uint4 &b4, float inv, uint32_t &mx, uint4 &h,
                                           uint4 &l, float &sh, float &sl) {
    const float f[8] = {__uint_as_float(a4.x), __uint_as_float(a4.y), __uint_as_float(a4.z), __uint_as_float(a4.w),
                        __uint_as_float(b4.x), __uint_as_float(b4.y), __uint_as_float(b4.z), __uint_as_float(b4.w)};
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float a = f[2 * k] * inv, b = f[2 * k + 1] * inv;
        mx = max(mx, max(__float_as_uint(fabsf(a)), __float_as_uint(fabsf(b))));
        const __half2 h2 = __floats2half2_rn(a, b);
        const float2 hf = __half22float2(h2);
        const __half2 l2 = __floats2half2_rn(a - hf.x, b - hf.y);      // exact differences
        const float2 lf = __half22float2(l2);
        sh += hf.x + hf.y;
        sl += lf.x + lf.y;
        hw[k] = *reinterpret_cast<const uint32_t *>(&h2);
        lw[k] = *reinterpret_cast<const uint32_t *>(&l2);
    }
    h = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    l = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// Stage m tokens' activations as fp16 rows + the offset table, by the nthr consumer threads (every
// one must call this; named barrier 1 synchronises them). Only a window of the K axis is staged:
// window chunk i (0 <= i < nch) holds K chunk (kc0 + i) mod chunks, so a CTA whose chunk range
// covers part of a row group stages just that part (its chunk at range position i sits at window
// chunk i); kc0 = 0, nch = chunks stages all of K. The region is laid out for mslots >= rows rows
// and a table of tabch >= nch chunks: rows, a 128-B zero block at mslots * xstride, the table, the
// token scales. Token n is x + row_of(n) * ldx (16-byte aligned). CG: load through L2 only (rows
// written earlier in the same launch).
// SPLIT false: x is bf16, token n is row n. SPLIT true: x is fp32 and token n becomes rows 2n
// (fp16(x)) and 2n + 1 (fp16(x - fp16(x))): a lane's two MMA columns hold the halves of one token,
// whose products are added when the segment is stored (2m <= mslots).
// The (token, 32-group) items are spread evenly over the threads; each thread issues the loads of
// kSU groups before converting, stores fp16 and writes the group sums. A token whose |x| exceeds
// 2^15 is redone scaled by 2^-e (rare) and the scale of its rows is 2^e.
template <int FMT, int NT, bool CG, bool SPLIT, int kSU, typename RowOf>
__device__ void stage_activations(const void *xv, int64_t ldx, RowOf row_of, int m, int mslots, int K, int kc0,
                                  int nch, int tabch, int xstride, uint8_t *xs, int tid, int nthr) {
    constexpr int MT = 8 * NT;
    constexpr int LQ = SPLIT ? 8 : 4;                   // 16-B loads per (token, group)
    constexpr int SU = SPLIT ? 1 : kSU;                 // fp32 groups: 128 B of loads each
    const int chunks = (K + kChunkK - 1) / kChunkK, G = K / 32, GW = 2 * nch;
    const int mv = SPLIT ? 2 * m : m;                   // rows
    float *tab = reinterpret_cast<float *>(xs + mslots * xstride + 128);
    float *tscale = reinterpret_cast<float *>(xs + mslots * xstride + 128 + tabch * tab_chunk_bytes(NT));
    unsigned *tmax = reinterpret_cast<unsigned *>(tscale + 16);
    auto tab_at = [&](int grp, int row) -> float & {
        return tab[((grp * NT + row / 8) * 4 + (row % 8) / 2) * 2 + (row & 1)];
    };
    auto kgroup = [&](int gw) {                         // window group -> K group (>= G: past K)
        int kc = kc0 + (gw >> 1);
        if (kc >= chunks) kc -= chunks;
        return 2 * kc + (gw & 1);
    };
    auto src_of = [&](int n, int gk) {
        const uint8_t *b = static_cast<const uint8_t *>(xv);
        return reinterpret_cast<const uint4 *>(b + (static_cast<int64_t>(row_of(n)) * ldx + gk * 32) * (SPLIT ? 4 : 2));
    };
    // the zero block (absent tokens) and the table entries of absent rows
    if (tid < 8) *reinterpret_cast<uint4 *>(xs + mslots * xstride + tid * 16) = make_uint4(0, 0, 0, 0);
    for (int e = tid; e < nch * 2 * MT; e += nthr) {
        const int row = e % MT, grp = e / MT;
        if (row >= mv) tab_at(grp, row) = 0.f;
    }
    if (tid < 16) tmax[tid] = 0u;
    named_bar_sync(1, nthr);
    const uint4 z4 = make_uint4(0, 0, 0, 0);
    // convert one (token, window group) and store it with its table entries
    auto convert = [&](uint4 (&v)[LQ], float inv, uint32_t &mx, int n, int gw) {
        if constexpr (SPLIT) {
            uint4 *rh = reinterpret_cast<uint4 *>(xs + 2 * n * xstride + gw * 64);
            uint4 *rl = reinterpret_cast<uint4 *>(xs + (2 * n + 1) * xstride + gw * 64);
            float sh = 0.f, sl = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 h, l;
                split8_f16(v[2 * q], v[2 * q + 1], inv, mx, h, l, sh, sl);
                rh[q] = h;
                rl[q] = l;
            }
            tab_at(gw, 2 * n) = sh * tab_factor<FMT>();
            tab_at(gw, 2 * n + 1) = sl * tab_factor<FMT>();
        } else {
            const float sum = group_to_f16<true>(v, inv, mx);
            uint4 *row = reinterpret_cast<uint4 *>(xs + n * xstride + gw * 64);
#pragma unroll
            for (int q = 0; q < 4; ++q) row[q] = v[q];
            tab_at(gw, n) = sum * tab_factor<FMT>();
        }
    };
    auto zero = [&](int n, int gw) {                    // the half chunk past K
#pragma unroll
        for (int h = 0; h < (SPLIT ? 2 : 1); ++h) {
            const int row = SPLIT ? 2 * n + h : n;
            uint4 *r = reinterpret_cast<uint4 *>(xs + row * xstride + gw * 64);
#pragma unroll
            for (int q = 0; q < 4; ++q) r[q] = z4;
            tab_at(gw, row) = 0.f;
        }
    };
    const int items = m * GW;
    for (int e0 = 0; e0 < items; e0 += nthr * SU) {
        uint4 v[SU][LQ];
#pragma unroll
        for (int u = 0; u < SU; ++u) {
            const int e = e0 + u * nthr + tid;
            if (e < items) {
                const int n = e / GW, gk = kgroup(e - n * GW);
                if (gk < G) {
                    const uint4 *src = src_of(n, gk);
#pragma unroll
                    for (int q = 0; q < LQ; ++q) v[u][q] = CG ? ld_cg_v4(src + q) : ld_nc_v4(src + q);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < SU; ++u) {
            const int e = e0 + u * nthr + tid;
            if (e < items) {
                const int n = e / GW, gw = e - n * GW;
                if (kgroup(gw) < G) {
                    uint32_t mx = 0;
                    convert(v[u], 1.0f, mx, n, gw);
                    if (mx > 0x47000000u) atomicMax(tmax + n, mx);      // only values above 2^15 matter
                } else {
                    zero(n, gw);
                }
            }
        }
    }
    named_bar_sync(1, nthr);
    bool big = false;
#pragma unroll 1
    for (int n = 0; n < m; ++n) big |= tmax[n] != 0u;
    if (big) {   // rare: redo the tokens beyond the fp16 range, scaled by 2^-e
        for (int e = tid; e < items; e += nthr) {
            const int n = e / GW, gw = e - n * GW, gk = kgroup(gw);
            if (tmax[n] == 0u || gk >= G) continue;
            const float inv = exp2f(-ceilf(log2f(__uint_as_float(tmax[n]) * (1.0f / 32768.0f))));
            const uint4 *src = src_of(n, gk);
            uint4 v[LQ];
#pragma unroll
            for (int q = 0; q < LQ; ++q) v[q] = CG ? ld_cg_v4(src + q) : ld_nc_v4(src + q);
            uint32_t mx = 0;
            convert(v, inv, mx, n, gw);
        }
    }
    if (tid < 16) {
        const unsigned tm = tmax[SPLIT ? tid >> 1 : tid];
        tscale[tid] = tid < mv && tm ? exp2f(ceilf(log2f(__uint_as_float(tm) * (1.0f / 32768.0f)))) : 1.0f;
    }
    named_bar_sync(1, nthr);
}

// End of a segment (fp16 path): the sums lose the codes' factor 2^-24 (rows r+8 also their
// factor 16), tokens their staging scale; all powers of two, so exact.
template <int NT>
__device__ __forceinline__ void finish_rows(float (&acc)[NT][4], const float *tscale, int t) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            const float sc = tscale[nt * 8 + 2 * t + (f & 1)];
            acc[nt][f] *= f >= 2 ? sc * 0x1p20f : sc * 0x1p24f;
        }
}

}  // namespace gemv_core
}  // namespace onpu_b200
