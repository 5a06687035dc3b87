// Host side of libonpu for B200: the reference's matrix geometry (the packed-buffer contract the
// Python engine checks with onpu_geometry2), its two 4-bit search quantisers, and its stream-order
// packet layout. These run at load time on the CPU; the per-token path is all CUDA.
//
// Contract with the reference (paths relative to its project root):
//   Geometry        llama/ggml-opennpu/opennpu_core.hpp:65-97  (npu4/model.py:151-190 checks it)
//   quant_q4nx32    llama/ggml-opennpu/opennpu_core.hpp:103-138
//   quant_q4s32     llama/ggml-opennpu/opennpu_core.hpp:142-169
//   stream order    llama/ggml-opennpu/opennpu_core.hpp:178-254
#pragma once
#include <cstddef>
#include <cstdint>

namespace onpu_b200 {

// Packet constants of the reference's stream order (its NPU device's tile shape). They only
// define the upload format of onpu_*_buf; the GPU layout is different (gpu_layout.cuh).
constexpr int kNC = 8, kNR = 4, kGN = 64, kGK = 256, kKMAX = 2048;
constexpr int kPktQ4NX = kGN * kGK / 2 + 2 * 2 * (kGK / 32) * kGN;  // 10240 B
constexpr int kPktQ4S = kGN * kGK / 2 + 2 * (kGK / 32) * kGN;       // 9216 B

uint16_t f32_to_bf16(float f);   // RNE; NaN -> quiet NaN with the top bits kept
float bf16_to_f32(uint16_t h);
float f16_to_f32(uint16_t h);

// R row blocks x S K-slices over ncols columns, every block (tiles, kc) packets; ok == false when
// no split keeps K / S <= 2048. Same arithmetic as the reference, so buffer sizes agree byte for
// byte.
struct Geometry {
    int64_t N = 0, K = 0;
    int ncols = 0, R = 0, S = 0, tiles = 0, kc = 0;
    int64_t ks = 0, rows_col = 0, cb = 0, nbytes = 0;
    bool ok = false, sym = false;
    Geometry() = default;
    Geometry(int64_t n, int64_t k, int nc, bool sy);
    int pkt() const { return sym ? kPktQ4S : kPktQ4NX; }
};

// 32 weights -> codes (0..15) and bf16 scale (+ min for q4nx), the reference's search quantisers.
void quant_q4nx32(const float *x, uint8_t *q, uint16_t &s_bf, uint16_t &m_bf);
void quant_q4s32(const float *x, uint8_t *q, uint16_t &d_bf);

// Quantise W [N][K] (row stride K) and write the stream-order bytes of geometry g (g.nbytes).
// Work split over `threads` host threads by column block.
void pack_stream(const Geometry &g, const float *W, uint8_t *out, int threads);

// Each 32-group quantised as pack_stream would, then dequantised (K % 32 == 0).
void quant_dequant(const float *W, int64_t N, int64_t K, bool sym, float *out, int threads);

}  // namespace onpu_b200
