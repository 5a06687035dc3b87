// One-shot all-reduce of small fp32 vectors between the GPUs of one node over NVLink peer memory
// (tensor-parallel decode: the [M, hidden] partial outputs of the row-parallel o and down
// projections, 20-160 KB), with the sum also written as bf16 (the next projection's input).
// The send half can instead be the row-parallel GEMV's own epilogue (gemv.cu, kEpiPeer): its
// finished rows go to the peers while the rest of the matrix is still streaming, and this kernel
// only receives and adds (comm_reduce_launch).
//
// Every rank owns one buffer (cudaMalloc, shared with the peers through CUDA IPC handles):
//   slots[2][world][cap] of 8-byte words {fp32 value, call number} | calls[kCommCtas] u32
//   | the call counters of the row-parallel GEMV's CTAs (kEpiPeer, gemv.cu) [kPeerCtaCounters] u32
// A call is one launch of kCommCtas CTAs; CTA b owns elements [b * per, (b + 1) * per):
//  1. every thread stores its elements of the local partial, each paired with the call number in
//     one 8-byte store, into slot [parity][rank] of every rank's buffer (peer stores over NVLink);
//  2. it then reads slot [parity][s][i] of its own buffer for every rank s (all ranks' loads in
//     flight at once), until the word carries this call's number (an 8-byte store lands whole, so
//     value and number arrive together: no fence, no separate flag), and adds the values in rank
//     order (the same float sum on every rank). Waits are bounded (2 s by default, then the error
//     word is set and the word's value is used).
// The call number is kept per CTA in the owner's buffer, so CUDA-graph replays need no host
// state. Two slot sets by call parity: a rank can be at most one call ahead of a peer that is
// still reading (it cannot finish call c+1 without that peer's words of call c+1).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

namespace onpu_b200 {

namespace {

constexpr int kCommThreads = 256;

struct CommParams {
    uint2 *bufs[kCommMaxRanks];      // every rank's buffer (this rank's own at [rank])
    int rank, world;
    int64_t cap;                     // words per slot
    const float *src;                // this rank's partial [n]
    float *dst;                      // the sum [n] (may alias src; may be null)
    __nv_bfloat16 *dst_bf16;         // the sum as bf16 [n] (may be null)
    int64_t n;
    int *err;
    int send;                        // 0: the values were sent by a GEMV epilogue; only receive
    uint64_t wait_ns;                // how long a thread waits for a peer's word
};

__global__ void __launch_bounds__(kCommThreads) comm_allreduce_kernel(const CommParams p) {
    const int b = blockIdx.x;
    const int64_t per = (p.n + kCommCtas - 1) / kCommCtas;
    const int64_t lo = b * per, hi = lo + per < p.n ? lo + per : p.n;
    uint2 *own = p.bufs[p.rank];
    uint32_t *calls = reinterpret_cast<uint32_t *>(own + 2 * static_cast<int64_t>(p.world) * p.cap);
    __shared__ uint32_t call;
    if (threadIdx.x == 0) call = calls[b] + 1u;
    __syncthreads();
    const uint32_t c = call;
    const int64_t set = static_cast<int64_t>(c & 1u) * p.world;
    if (p.send)
        for (int64_t i = lo + threadIdx.x; i < hi; i += kCommThreads) {
            const uint32_t v = __float_as_uint(p.src[i]);
            for (int d = 0; d < p.world; ++d) st_word(p.bufs[d] + (set + p.rank) * p.cap + i, v, c);
        }
    for (int64_t i = lo + threadIdx.x; i < hi; i += kCommThreads) {
        const float acc = recv_words_sum<kCommMaxRanks>(own + set * p.cap + i, p.cap, p.world, c, p.wait_ns, p.err);
        if (p.dst) p.dst[i] = acc;
        if (p.dst_bf16) p.dst_bf16[i] = __float2bfloat16_rn(acc);
    }
    __syncthreads();
    if (threadIdx.x == 0) calls[b] = c;
}

}  // namespace

int64_t comm_buffer_bytes(int world, int64_t cap) {
    return 2 * static_cast<int64_t>(world) * cap * 8 + (kCommCtas + kPeerCtaCounters) * 4;
}

cudaError_t comm_allreduce_launch(void *const *bufs, int rank, int world, int64_t cap, const float *src, float *dst,
                                  void *dst_bf16, int64_t n, int *err, uint64_t wait_ns, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if (world < 1 || world > kCommMaxRanks || n > cap) return cudaErrorInvalidValue;
    CommParams p{};
    for (int r = 0; r < world; ++r) p.bufs[r] = static_cast<uint2 *>(bufs[r]);
    p.rank = rank;
    p.world = world;
    p.cap = cap;
    p.src = src;
    p.dst = dst;
    p.dst_bf16 = static_cast<__nv_bfloat16 *>(dst_bf16);
    p.n = n;
    p.err = err;
    p.send = 1;
    p.wait_ns = wait_ns;
    comm_allreduce_kernel<<<kCommCtas, kCommThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t comm_reduce_launch(void *const *bufs, int rank, int world, int64_t cap, float *dst, void *dst_bf16,
                               int64_t n, int *err, uint64_t wait_ns, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if (world < 1 || world > kCommMaxRanks || n > cap) return cudaErrorInvalidValue;
    CommParams p{};
    for (int r = 0; r < world; ++r) p.bufs[r] = static_cast<uint2 *>(bufs[r]);
    p.rank = rank;
    p.world = world;
    p.cap = cap;
    p.dst = dst;
    p.dst_bf16 = static_cast<__nv_bfloat16 *>(dst_bf16);
    p.n = n;
    p.err = err;
    p.send = 0;
    p.wait_ns = wait_ns;
    comm_allreduce_kernel<<<kCommCtas, kCommThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace onpu_b200
