// GGUF (ggml) block formats -> plain codes q [rows][K] (0..15) and 16-bit scales (and mins)
// [rows][K/32], which repack.cu (kSrcCodes) turns into the GPU layout. Load time only.
//
// Q4_0 (ggml type 2): blocks of 32 weights, 18 bytes: fp16 d, then 16 bytes whose low nibbles are
//   elements 0..15 and high nibbles elements 16..31; w = (q - 8) * d. This is the int4 + fp16
//   format exactly (q = v + 8, fp16 scale): codes and scale are copied, nothing is rounded.
// Q4_K (ggml type 12): super-blocks of 256 weights, 144 bytes: fp16 d, fp16 dmin, 12 bytes of
//   6-bit sub-block scales and mins, 128 bytes of codes (bytes 32j..32j+31 hold sub-block 2j in
//   their low nibbles and 2j+1 in their high ones); sub-block b is w = q * (d * sc_b) - dmin * m_b.
//   That is q4nx (w = q * s + m) exactly except that s and m are bf16 here: the transcode keeps
//   the codes and takes, among the bf16 values next to d * sc_b and -dmin * m_b (3 x 3 pairs), the
//   pair whose weights are closest (least squares over the 32 weights) to the exact ones. This is
//   the reference's transcode (llama/ggml-opennpu/ggml-opennpu.cpp:100-143, q4k_codes / bf_step),
//   restated: the same float operations in the same order, each rounded separately (no FMA), so
//   the scales and mins are bit-identical to a host run of the same steps.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace onpu_b200 {

namespace {

// fp32 -> bf16 bits, round to nearest even, NaN keeps its top bits with the quiet bit set
__device__ __forceinline__ uint16_t f2bf(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 64u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}
__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

// the bf16 value next to h, upwards (dir > 0) or downwards in value; from zero the smallest
// subnormal of that sign
__device__ __forceinline__ uint16_t bf_step(uint16_t h, int dir) {
    const float f = bf2f(h);
    if (f == 0.0f) return dir > 0 ? static_cast<uint16_t>(0x0001) : static_cast<uint16_t>(0x8001);
    return static_cast<uint16_t>(((f > 0.0f) == (dir > 0)) ? h + 1 : h - 1);
}

__global__ void q4_0_codes_kernel(const uint8_t *src, int64_t rows, int64_t K, int64_t row_bytes, uint8_t *q,
                                  uint16_t *s) {
    const int64_t G = K / 32, total = rows * G;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / G, g = i - r * G;
        const uint8_t *b = src + r * row_bytes + g * 18;
        s[i] = static_cast<uint16_t>(b[0] | (b[1] << 8));
        uint8_t *o = q + r * K + g * 32;
#pragma unroll 4
        for (int j = 0; j < 16; ++j) {
            const uint8_t v = b[2 + j];
            o[j] = v & 0xF;
            o[j + 16] = v >> 4;
        }
    }
}

__global__ void q4k_codes_kernel(const uint8_t *src, int64_t rows, int64_t K, int64_t row_bytes, uint8_t *q,
                                 uint16_t *s_out, uint16_t *m_out) {
    const int64_t G = K / 32, total = rows * G;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / G, gc = (i - r * G) * 32;
        const uint8_t *b = src + r * row_bytes + (gc / 256) * 144;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(b[0] | (b[1] << 8))));
        const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(b[2] | (b[3] << 8))));
        const uint8_t *sc = b + 4, *qs = b + 16;
        const int sub = static_cast<int>((gc % 256) / 32);
        int sv, mv;
        if (sub < 4) {
            sv = sc[sub] & 63;
            mv = sc[sub + 4] & 63;
        } else {
            sv = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4);
            mv = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
        }
        const uint8_t *qq = qs + (sub / 2) * 32;
        float qf[32];
        uint8_t *o = q + r * K + gc;
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            const int c = (sub & 1) ? (qq[l] >> 4) : (qq[l] & 0xF);
            o[l] = static_cast<uint8_t>(c);
            qf[l] = static_cast<float>(c);
        }
        const float S = __fmul_rn(d, static_cast<float>(sv)), M = __fmul_rn(-dmin, static_cast<float>(mv));
        const uint16_t s0 = f2bf(S), m0 = f2bf(M);
        float best = __int_as_float(0x7f800000);
        uint16_t bs = s0, bm = m0;
        for (int ds = -1; ds <= 1; ++ds)
            for (int dm = -1; dm <= 1; ++dm) {
                const uint16_t sc_ = ds ? bf_step(s0, ds) : s0, mn_ = dm ? bf_step(m0, dm) : m0;
                const float sf = bf2f(sc_), mf = bf2f(mn_);
                float e = 0.0f;
#pragma unroll
                for (int l = 0; l < 32; ++l) {
                    const float x = __fsub_rn(__fadd_rn(__fmul_rn(qf[l], sf), mf), __fadd_rn(__fmul_rn(qf[l], S), M));
                    e = __fadd_rn(e, __fmul_rn(x, x));
                }
                if (e < best) {
                    best = e;
                    bs = sc_;
                    bm = mn_;
                }
            }
        s_out[i] = bs;
        m_out[i] = bm;
    }
}

unsigned grid_for(int64_t n) {
    const int64_t g = (n + 255) / 256;
    return static_cast<unsigned>(g < 65535 * 8 ? (g > 0 ? g : 1) : 65535 * 8);
}

}  // namespace

int64_t gguf_row_bytes(int type, int64_t K) {
    if (type == kGgmlQ4_0 && K % 32 == 0) return K / 32 * 18;
    if (type == kGgmlQ4_K && K % 256 == 0) return K / 256 * 144;
    return -1;
}

cudaError_t gguf_codes_launch(int type, const uint8_t *src, int64_t rows, int64_t K, uint8_t *q, uint16_t *scales,
                              uint16_t *mins, cudaStream_t stream) {
    const int64_t rb = gguf_row_bytes(type, K);
    if (rb < 0 || rows <= 0 || (type == kGgmlQ4_K && !mins)) return cudaErrorInvalidValue;
    const int64_t groups = rows * (K / 32);
    if (type == kGgmlQ4_0)
        q4_0_codes_kernel<<<grid_for(groups), 256, 0, stream>>>(src, rows, K, rb, q, scales);
    else
        q4k_codes_kernel<<<grid_for(groups), 256, 0, stream>>>(src, rows, K, rb, q, scales, mins);
    return cudaGetLastError();
}

}  // namespace onpu_b200
