// Small elementwise kernels of libonpu: input rounding to bf16 and the MoE weighted combine.
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

// fp32 -> bf16 exactly as the reference's host converts NPU inputs (opennpu_core.hpp:50-56):
// round to nearest even, NaN -> top bits with the quiet bit set.
__device__ __forceinline__ uint16_t to_bf16_bits(float f) {
    const uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
    return static_cast<uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

__global__ void f32_to_bf16_kernel(const float *x, int64_t rows, int64_t cols, int64_t ldx, uint16_t *out,
                                   int64_t ldo) {
    const int64_t n = rows * cols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t rr = i / cols, cc = i - rr * cols;
        out[rr * ldo + cc] = to_bf16_bits(x[rr * ldx + cc]);
    }
}

// Weighted sum of a token's expert outputs in slot order (onpu_cpu.cpp:259-274 semantics):
// deterministic, one thread per output element.
__global__ void moe_combine_kernel(const float *o, int64_t ldo, int64_t T, int k, int64_t N, const int32_t *ids,
                                   const float *w, const float *bias, float *y, int64_t ldy, int id_lo, int id_hi) {
    pdl_wait_prerequisites();                              // the expert outputs
    pdl_launch_dependents();
    const int64_t n = T * N;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / N, c = i - t * N;
        float acc = 0.f;
        for (int j = 0; j < k; ++j) {
            const int64_t slot = t * k + j;
            if (ids[slot] < id_lo || ids[slot] >= id_hi) continue;
            float v = o[slot * ldo + c];
            if (bias) v += bias[static_cast<int64_t>(ids[slot]) * N + c];
            acc += w[slot] * v;
        }
        y[t * ldy + c] = acc;
    }
}

// a[r][i] = act(h[r] + gu_bias[ids[r]]) in fp32 (onpu_cpu.cpp:233-256 semantics): act 0
// silu(h[:I]) * h[I:]; act 1 (gpt-oss) interleaved gate/up, gate <= limit, |up| <= limit,
// (up + 1) * gate * sigmoid(alpha * gate).
__global__ void moe_act_kernel(const float *h, int64_t ldh, int64_t rows, int64_t Ng, const int32_t *ids,
                               const float *gu_bias, int act, float alpha, float limit, float *a, int64_t lda) {
    const int64_t I = Ng / 2, n = rows * I;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < n;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = idx / I, i = idx - r * I;
        const float *hr = h + r * ldh;
        const float *b = gu_bias ? gu_bias + static_cast<int64_t>(ids[r]) * Ng : nullptr;
        float out;
        if (act == 1) {
            float g = hr[2 * i] + (b ? b[2 * i] : 0.f), u = hr[2 * i + 1] + (b ? b[2 * i + 1] : 0.f);
            g = fminf(g, limit);
            u = fmaxf(-limit, fminf(u, limit));
            out = (u + 1.f) * g / (1.f + expf(-alpha * g));
        } else {
            const float g = hr[i] + (b ? b[i] : 0.f), u = hr[I + i] + (b ? b[I + i] : 0.f);
            out = g / (1.f + expf(-g)) * u;
        }
        a[r * lda + i] = out;
    }
}

// GEMV descriptors of a dense call (jobs of 16 consecutive rows) written on the device, and the
// split-row ready flags of the launch cleared: the arguments travel by value in the launch.
__global__ void dense_jobs_kernel(GemvJob *jobs, const uint8_t *w, int rows, unsigned *flags, int nflags) {
    const int njobs = (rows + kMaxTokensPerJob - 1) / kMaxTokensPerJob;
    for (int i = threadIdx.x; i < njobs * kMaxTokensPerJob; i += blockDim.x) {
        const int j = i / kMaxTokensPerJob, n = i - j * kMaxTokensPerJob;
        GemvJob &jb = jobs[j];
        const int m = min(kMaxTokensPerJob, rows - j * kMaxTokensPerJob);
        if (n == 0) {
            jb.w = w;
            jb.m = m;
            jb.pad_ = 0;
        }
        jb.xrow[n] = jb.yrow[n] = n < m ? j * kMaxTokensPerJob + n : 0;
    }
    for (int i = threadIdx.x; i < nflags; i += blockDim.x) flags[i] = 0u;
}

unsigned grid_for(int64_t n, int block) {
    const int64_t g = (n + block - 1) / block;
    return static_cast<unsigned>(g < 65535 * 8 ? (g > 0 ? g : 1) : 65535 * 8);
}

}  // namespace

cudaError_t moe_act_f32_launch(const float *h, int64_t ldh, int64_t rows, int64_t Ng, const int32_t *ids,
                               const float *gu_bias, int act, float alpha, float limit, float *a, int64_t lda,
                               cudaStream_t stream) {
    if (rows * (Ng / 2) == 0) return cudaSuccess;
    moe_act_kernel<<<grid_for(rows * (Ng / 2), 256), 256, 0, stream>>>(h, ldh, rows, Ng, ids, gu_bias, act, alpha,
                                                                        limit, a, lda);
    return cudaGetLastError();
}

cudaError_t dense_jobs_launch(GemvJob *jobs, const uint8_t *w, int rows, unsigned *flags, int nflags,
                              cudaStream_t stream) {
    dense_jobs_kernel<<<1, 256, 0, stream>>>(jobs, w, rows, flags, nflags);
    return cudaGetLastError();
}

cudaError_t f32_to_bf16_launch(const float *x, int64_t rows, int64_t cols, int64_t ldx, uint16_t *out, int64_t ldo,
                               cudaStream_t stream) {
    if (rows * cols == 0) return cudaSuccess;
    f32_to_bf16_kernel<<<grid_for(rows * cols, 256), 256, 0, stream>>>(x, rows, cols, ldx, out, ldo);
    return cudaGetLastError();
}

cudaError_t moe_combine_launch(const float *o, int64_t ldo, int64_t T, int k, int64_t N, const int32_t *ids,
                               const float *w, const float *bias, float *y, int64_t ldy, cudaStream_t stream,
                               int id_lo, int id_hi) {
    if (T * N == 0) return cudaSuccess;
    return launch_pdl(moe_combine_kernel, dim3(grid_for(T * N, 256)), dim3(256), 0, stream, o, ldo, T, k, N, ids, w,
                      bias, y, ldy, id_lo, id_hi);
}

}  // namespace onpu_b200
