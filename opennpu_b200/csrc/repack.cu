// Load-time layout conversion into the GPU layout of gpu_layout.cuh, on the GPU.
//
// Sources:
//  * the reference's stream-order packets, the bytes a caller writes into onpu_dense_buf /
//    onpu_bank_buf (layout: llama/ggml-opennpu/opennpu_core.hpp:178-219, column blocks :236-254;
//    opennpu/native/npu4/gemv_device.py:160-185);
//  * int4 packed along K (two's complement, low nibble = even column) with fp16 scales per 32;
//  * plain codes + 16-bit scales (+ mins).
// One thread writes one lane's 16 code bytes of one strip-chunk and, for t == 0, that lane's
// scale (and min) entries, so every GPU byte is written exactly once.
#include <cuda_runtime.h>

#include "gpu_layout.cuh"
#include "kernels.h"

namespace onpu_b200 {

namespace {

struct Code {
    uint8_t q;
    bool valid;
};

// reference stream order: byte offset of packet (row, col) and position inside it
__device__ __forceinline__ int64_t stream_packet(const RepackParams &p, int64_t row, int64_t col, int &n_in, int &kq) {
    const int rb = static_cast<int>(row / p.rows_col);
    const int64_t rin = row - rb * p.rows_col;
    const int64_t core_rows = static_cast<int64_t>(p.tiles) * 64;
    const int cr = static_cast<int>(rin / core_rows);
    const int64_t rem = rin - cr * core_rows;
    const int tile = static_cast<int>(rem / 64);
    n_in = static_cast<int>(rem - tile * 64);
    const int sl = static_cast<int>(col / p.ks);
    const int64_t kin = col - sl * p.ks;
    const int kp = static_cast<int>(kin / 256);
    kq = static_cast<int>(kin - kp * 256);
    return static_cast<int64_t>(rb * p.S + sl) * p.cb + ((static_cast<int64_t>(tile) * p.kc + kp) * 4 + cr) * p.pkt;
}

__device__ __forceinline__ uint8_t src_code(const RepackParams &p, int64_t row, int64_t col) {
    switch (p.src_kind) {
        case kSrcStream: {
            int n_in, kq;
            const uint8_t *pk = p.src + stream_packet(p, row, col, n_in, kq);
            const uint8_t b = pk[((static_cast<int64_t>(n_in >> 3) * 32 + (kq >> 3)) * 8 + (kq & 7)) * 4 + ((n_in & 7) >> 1)];
            return (n_in & 1) ? static_cast<uint8_t>(b >> 4) : static_cast<uint8_t>(b & 15);
        }
        case kSrcInt4K: {
            const uint8_t b = p.src[row * (p.K / 2) + (col >> 1)];
            const uint8_t u = (col & 1) ? static_cast<uint8_t>(b >> 4) : static_cast<uint8_t>(b & 15);
            return static_cast<uint8_t>(u ^ 8u);   // two's complement v -> offset code v + 8
        }
        default:
            return p.src[row * p.K + col];
    }
}

// 16-bit scale (which = 0) or min (which = 1) of (row, group)
__device__ __forceinline__ uint16_t src_param(const RepackParams &p, int64_t row, int64_t grp, int which) {
    switch (p.src_kind) {
        case kSrcStream: {
            int n_in, kq;
            const uint8_t *pk = p.src + stream_packet(p, row, grp * 32, n_in, kq);
            const uint8_t *e = pk + 64 * 256 / 2 + which * (256 / 32) * 64 * 2 + ((kq >> 5) * 64 + n_in) * 2;
            return static_cast<uint16_t>(e[0] | (e[1] << 8));
        }
        case kSrcInt4K:
            return which ? uint16_t{0} : p.scales[row * (p.K / 32) + grp];
        default:
            return (which ? p.mins : p.scales)[row * (p.K / 32) + grp];
    }
}

__global__ void repack_kernel(const RepackParams p, int row_groups, int chunks) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t total = static_cast<int64_t>(row_groups) * chunks * 4 * 32;
    if (tid >= total) return;
    const int lane = static_cast<int>(tid & 31);
    const int strip = static_cast<int>((tid >> 5) & 3);
    const int64_t blk = tid >> 7;                      // (row group, chunk)
    const int g = static_cast<int>(blk / chunks), c = static_cast<int>(blk - static_cast<int64_t>(g) * chunks);
    const int r = lane >> 2, t = lane & 3;
    const bool sym = p.fmt != kFmtQ4NX;
    const int SB = strip_bytes(p.fmt);
    uint8_t *out = p.dst + blk * chunk_bytes(p.fmt) + strip * SB;
    const int64_t row_base = static_cast<int64_t>(g) * kRowGroup + strip * kStripRows;

    uint32_t words[4];
    for (int gi = 0; gi < 2; ++gi)
        for (int jstep = 0; jstep < 2; ++jstep) {
            uint32_t w = 0;
            for (int pnib = 0; pnib < 8; ++pnib) {
                const int i = pnib & 3, h = pnib >> 2;
                const int64_t grow = row_base + r + 8 * (i & 1);
                const int64_t col = static_cast<int64_t>(c) * kChunkK + gi * 32 + 8 * t + 4 * jstep + 2 * (i >> 1) + h;
                uint32_t q = sym ? 8u : 0u;
                if (grow < p.N && col < p.K) {
                    const int64_t srow = p.src_row ? p.src_row[grow] : grow;
                    if (srow >= 0) q = src_code(p, srow, col);
                }
                w |= (q & 15u) << (4 * pnib);
            }
            words[gi * 2 + jstep] = w;
        }
    reinterpret_cast<uint4 *>(out)[lane] = make_uint4(words[0], words[1], words[2], words[3]);

    if (t == 0) {   // this lane's row pair (r, r+8): scales (and mins) of both groups
        for (int which = 0; which < (sym ? 1 : 2); ++which) {
            uint16_t v[4];
            for (int gi = 0; gi < 2; ++gi)
                for (int h = 0; h < 2; ++h) {
                    const int64_t grow = row_base + r + 8 * h;
                    const int64_t grp = static_cast<int64_t>(c) * 2 + gi;
                    uint16_t s = 0;
                    if (grow < p.N && grp * 32 < p.K) {
                        const int64_t srow = p.src_row ? p.src_row[grow] : grow;
                        if (srow >= 0) s = src_param(p, srow, grp, which);
                    }
                    v[gi * 2 + h] = s;
                }
            uint16_t *dstp = reinterpret_cast<uint16_t *>(out + kCodeBytes + which * kScaleBytes) + r * 4;
            for (int e = 0; e < 4; ++e) dstp[e] = v[e];
        }
    }
}

__global__ void unpack_gpu_kernel(const uint8_t *src, int64_t N, int64_t K, int fmt, int row_groups, int chunks,
                                  uint8_t *q, uint16_t *s, uint16_t *m) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t total = static_cast<int64_t>(row_groups) * chunks * 4 * 32;
    if (tid >= total) return;
    const int lane = static_cast<int>(tid & 31);
    const int strip = static_cast<int>((tid >> 5) & 3);
    const int64_t blk = tid >> 7;
    const int g = static_cast<int>(blk / chunks), c = static_cast<int>(blk - static_cast<int64_t>(g) * chunks);
    const int r = lane >> 2, t = lane & 3;
    const uint8_t *in = src + blk * chunk_bytes(fmt) + strip * strip_bytes(fmt);
    const uint4 wv = reinterpret_cast<const uint4 *>(in)[lane];
    const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
    const int64_t row_base = static_cast<int64_t>(g) * kRowGroup + strip * kStripRows;
    for (int gi = 0; gi < 2; ++gi)
        for (int jstep = 0; jstep < 2; ++jstep)
            for (int pnib = 0; pnib < 8; ++pnib) {
                const int i = pnib & 3, h = pnib >> 2;
                const int64_t row = row_base + r + 8 * (i & 1);
                const int64_t col = static_cast<int64_t>(c) * kChunkK + gi * 32 + 8 * t + 4 * jstep + 2 * (i >> 1) + h;
                if (row < N && col < K) q[row * K + col] = static_cast<uint8_t>((words[gi * 2 + jstep] >> (4 * pnib)) & 15u);
            }
    if (t == 0) {
        for (int which = 0; which < (fmt == kFmtQ4NX ? 2 : 1); ++which) {
            const uint16_t *e = reinterpret_cast<const uint16_t *>(in + kCodeBytes + which * kScaleBytes) + r * 4;
            uint16_t *dst = which ? m : s;
            for (int gi = 0; gi < 2; ++gi)
                for (int h = 0; h < 2; ++h) {
                    const int64_t row = row_base + r + 8 * h, grp = static_cast<int64_t>(c) * 2 + gi;
                    if (row < N && grp * 32 < K) dst[row * (K / 32) + grp] = e[gi * 2 + h];
                }
        }
    }
}

}  // namespace

cudaError_t repack_launch(const RepackParams &p, cudaStream_t stream) {
    const GpuMatrix gm = make_gpu_matrix(p.N, p.K, p.fmt);
    const int64_t threads = static_cast<int64_t>(gm.row_groups) * gm.chunks * 4 * 32;
    if (threads == 0) return cudaSuccess;
    const int block = 256;
    repack_kernel<<<static_cast<unsigned>((threads + block - 1) / block), block, 0, stream>>>(p, gm.row_groups, gm.chunks);
    return cudaGetLastError();
}

cudaError_t unpack_gpu_launch(const uint8_t *src, int64_t N, int64_t K, int fmt, uint8_t *q, uint16_t *s,
                              uint16_t *m, cudaStream_t stream) {
    const GpuMatrix gm = make_gpu_matrix(N, K, fmt);
    const int64_t threads = static_cast<int64_t>(gm.row_groups) * gm.chunks * 4 * 32;
    if (threads == 0) return cudaSuccess;
    const int block = 256;
    unpack_gpu_kernel<<<static_cast<unsigned>((threads + block - 1) / block), block, 0, stream>>>(
        src, N, K, fmt, gm.row_groups, gm.chunks, q, s, m);
    return cudaGetLastError();
}

}  // namespace onpu_b200
