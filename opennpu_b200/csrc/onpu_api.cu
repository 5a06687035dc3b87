// libonpu for B200: the reference's C ABI (llama/ggml-opennpu/onpu_api.cpp, onpu_cpu.cpp) backed
// by CUDA, plus device-pointer additions. See include/onpu.h for the per-function contract.
//
// Runtime model: one process per GPU; the library uses the CUDA device that is current when it is
// first called. Host-pointer calls (the reference ABI) are serialised by one process-wide mutex
// like the reference's g_mu (onpu_api.cpp:53) and run on the library's own stream; each copies its
// inputs in, launches, copies out and waits. Device-pointer calls (_dev) are asynchronous on the
// caller's stream and must be stream-ordered with respect to each other (they share the GEMV's
// split-row scratch).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "gpu_layout.cuh"
#include "host_codec.hpp"
#include "kernels.h"
#include "onpu.h"

using namespace onpu_b200;

namespace {

// ------------------------------------------------------------------ errors
thread_local std::string t_err;
thread_local bool t_has_err = false;

void set_err(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    t_has_err = true;
    if (std::getenv("ONPU_DEBUG")) fprintf(stderr, "onpu: %s\n", buf);
}
void clear_err() { t_has_err = false; }

#define ONPU_CUDA(expr, ret)                                                               \
    do {                                                                                   \
        cudaError_t e_ = (expr);                                                           \
        if (e_ != cudaSuccess) {                                                           \
            set_err("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__); \
            return ret;                                                                    \
        }                                                                                  \
    } while (0)

std::mutex g_mu;

// ------------------------------------------------------------------ device context
template <typename T>
bool grow(T *&p, int64_t &cap, int64_t n, bool zero = false) {
    if (n <= cap) return true;
    if (p) {
        cudaDeviceSynchronize();   // the old buffer may still be in use by queued kernels
        cudaFree(p);
    }
    p = nullptr;
    cap = 0;
    cudaError_t e = cudaMalloc(reinterpret_cast<void **>(&p), static_cast<size_t>(n) * sizeof(T));
    if (e != cudaSuccess) {
        set_err("cudaMalloc(%lld bytes): %s", static_cast<long long>(n * sizeof(T)), cudaGetErrorString(e));
        p = nullptr;
        return false;
    }
    if (zero && cudaMemset(p, 0, static_cast<size_t>(n) * sizeof(T)) != cudaSuccess) return false;
    cap = n;
    return true;
}

struct Ctx {
    bool tried = false, ok = false;
    int device = 0, nsm = 0;
    cudaStream_t stream = nullptr;
    int *d_err = nullptr;
    float *d_part = nullptr;
    int64_t part_cap = 0;
    unsigned *d_cnt = nullptr;
    int64_t cnt_cap = 0;
    // staging for host-pointer calls
    float *d_in = nullptr;
    int64_t in_cap = 0;
    uint16_t *d_x = nullptr;
    int64_t x_cap = 0;
    float *d_h = nullptr;
    int64_t h_cap = 0;
    uint16_t *d_a = nullptr;
    int64_t a_cap = 0;
    float *d_af = nullptr;              // MoE: the fp32 activation between the projections
    int64_t af_cap = 0;
    float *d_o = nullptr;
    int64_t o_cap = 0;
    float *d_y = nullptr;
    int64_t y_cap = 0;
    GemvJob *d_jobs = nullptr;
    int64_t jobs_cap = 0;
    int32_t *d_ids = nullptr;
    int64_t ids_cap = 0;
    float *d_w = nullptr;
    int64_t w_cap = 0;
    float *d_gb = nullptr;
    int64_t gb_cap = 0;
    float *d_db = nullptr;
    int64_t db_cap = 0;
    std::vector<GemvJob> h_jobs;
    unsigned *d_rcnt = nullptr;         // router: per-token-block arrival counters (kept zero)
    int64_t rcnt_cap = 0;
    float *d_rlg = nullptr;             // router: logits scratch when the caller wants none
    int64_t rlg_cap = 0;
    int32_t *d_order = nullptr;         // device MoE layer: slots sorted by expert
    int64_t order_cap = 0;
    int *d_njobs = nullptr;             // and the job count of its job lists
    int64_t njobs_cap = 0;
    unsigned *d_ffnbar = nullptr;       // fused expert FFN: grid-barrier counters (kept zero)
    int64_t ffnbar_cap = 0;
    int moe_fused = 1;                  // onpu_moe_set_fused: 1 the persistent expert FFN, 0 three launches
    uint16_t *d_xh = nullptr;           // prefill GEMM: fp16 copy of the activations
    int64_t xh_cap = 0;
    float *d_ts = nullptr;              // and their per-token scales
    int64_t ts_cap = 0;
    int64_t calls = 0;
    double wait_s = 0;
    uint64_t peer_wait_ns = 2000000000ull;   // bounded waits on other ranks' words (onpu_comm_set_wait)
    unsigned long long *gemv_trace = nullptr;   // onpu_gemv_trace: stamps of later GEMV launches
    int64_t gemv_trace_ctas = 0;
};

Ctx &ctx() {
    static Ctx c;
    if (!c.tried) {
        c.tried = true;
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
            cudaGetLastError();
            return c;
        }
        if (cudaGetDevice(&c.device) != cudaSuccess) return c;
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, c.device) != cudaSuccess) return c;
        c.nsm = prop.multiProcessorCount;
        if (prop.major < 10) {
            fprintf(stderr, "onpu: %s (sm_%d%d) is not a B200-class GPU; libonpu targets sm_100a\n", prop.name,
                    prop.major, prop.minor);
            return c;
        }
        if (cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking) != cudaSuccess) return c;
        if (cudaMalloc(&c.d_err, sizeof(int)) != cudaSuccess) return c;
        cudaMemset(c.d_err, 0, sizeof(int));
        c.ok = true;
    }
    return c;
}

// ------------------------------------------------------------------ matrices on the GPU
struct GpuMat {
    GpuMatrix gm;                 // one matrix (expert)
    int64_t E = 1;
    uint8_t *d_w = nullptr;       // E * gm.bytes
    int *d_row_map = nullptr;     // GPU row -> original row (interleaved gate/up), null = identity
    std::vector<int> src_row;     // host copy of the same map
    ~GpuMat() {
        if (d_w) cudaFree(d_w);
        if (d_row_map) cudaFree(d_row_map);
    }
};

// ONPU_PDL=0 turns programmatic dependent launch off (a diagnostic switch; on by default)
bool pdl_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("ONPU_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

bool alloc_mat(GpuMat &m, int64_t N, int64_t K, int fmt, int64_t E) {
    m.gm = make_gpu_matrix(N, round_up(K, 32), fmt);
    m.E = E;
    cudaError_t e = cudaMalloc(&m.d_w, static_cast<size_t>(m.gm.bytes * E));
    if (e != cudaSuccess) {
        set_err("cudaMalloc of %lld weight bytes: %s", static_cast<long long>(m.gm.bytes * E), cudaGetErrorString(e));
        m.d_w = nullptr;
        return false;
    }
    return true;
}

// gate rows [0, N/2) and up rows [N/2, N) interleaved per 16-row strip: strip rows 0-7 gate
// 8s..8s+7, rows 8-15 up 8s..8s+7, so the GEMV epilogue sees gate_i and up_i in one lane
bool set_gateup_interleave(GpuMat &m) {
    const int64_t N = m.gm.N, I = N / 2;
    if (N % 2 || I % 8) return false;
    m.src_row.resize(static_cast<size_t>(N));
    for (int64_t rho = 0; rho < N; ++rho) {
        const int64_t strip = rho / 16, rr = rho % 16;
        m.src_row[rho] = static_cast<int>(rr < 8 ? 8 * strip + rr : I + 8 * strip + rr - 8);
    }
    if (cudaMalloc(&m.d_row_map, sizeof(int) * N) != cudaSuccess) return false;
    return cudaMemcpy(m.d_row_map, m.src_row.data(), sizeof(int) * N, cudaMemcpyHostToDevice) == cudaSuccess;
}

// ------------------------------------------------------------------ GEMV driver
int choose_workers(const Ctx &c, int fmt, int ntiles, int T, int smem) {
    // at most one resident wave (every SM the same number of CTAs), each with >= 1 full stage
    const int full = c.nsm * gemv_ctas_per_sm(fmt, ntiles, smem), cps = gemv_chunks_per_stage();
    if (T >= full * cps) return full;
    return std::max(1, std::min(full, (T + cps - 1) / cps));
}

// With a job count known on the host and at least one CTA per row group, trim the wave to a whole
// number of CTAs per row group: every row group is then split into the same number of equal chunk
// ranges, so no CTA straddles two row groups and the split-row reductions are spread evenly. The
// trim is taken only while it keeps at least 6/7 of the wave; deeper trims lose more streaming
// CTAs than the alignment gains. Measured on a B200: 4096 x 4096 launches 15 % faster
// (296 -> 256 CTAs), the Qwen3-8B decode step 4.4 %; Qwen2.5-32B's 224- and 240-CTA trims 4 % slower.
int align_workers(int W, int njobs, int row_groups) {
    const int units = njobs * row_groups;
    if (units <= 0 || units > W) return W;
    const int trimmed = W / units * units;
    return 7 * trimmed >= 6 * W ? trimmed : W;
}

bool ensure_scratch(Ctx &c, int workers, int ntiles, int counters) {
    const int64_t pf = static_cast<int64_t>(workers) * gemv_part_floats_per_worker(ntiles);
    if (!grow(c.d_part, c.part_cap, pf)) return false;
    if (!grow(c.d_cnt, c.cnt_cap, std::max<int64_t>(counters, 1024), true)) return false;
    return true;
}

// Activation and output forms of a GEMV launch beyond bf16 in / the epilogue's own type.
struct GemvOpts {
    const float *xf = nullptr;    // fp32 activations (row stride ldx), staged as two fp16 halves
                                  // per value; jobs of at most 8 tokens, resident only
    bool yf32 = false;            // kEpiSwiGLU: fp32 outputs
};

constexpr int kMaxCtasPerRowGroup = 4;
constexpr int kCapBelowChunks = 16;     // ... when the CTAs would get fewer chunks than this

// The resident activation layout of a launch of T chunks, and its CTA count: one resident wave,
// trimmed to whole CTAs per row group (host-known job count). A one-job launch whose CTAs each
// cover less than a row group stages only its own part of K (kwin) when that layout keeps the wave
// resident.
struct GemvPlan {
    GemvLayout lay;
    int workers = 0, ntiles = 1;
    bool kwin = false;
};
GemvPlan plan_gemv(const Ctx &c, const GpuMatrix &gm, int njobs, int mrows, bool device_count) {
    GemvPlan pl;
    const int T = njobs * gm.row_groups * gm.chunks;
    pl.ntiles = mrows > 8 ? 2 : 1;
    pl.lay = gemv_layout(gm.fmt, mrows, gm.K);
    int W = choose_workers(c, gm.fmt, pl.ntiles, T, pl.lay.smem);
    if (!device_count) W = align_workers(W, njobs, gm.row_groups);
    // a small matrix with few row groups (a tensor-parallel shard) would otherwise split each row
    // group over many CTAs of a few chunks each, and its first CTA waits for and adds every
    // partner's partial sums: then at most kMaxCtasPerRowGroup CTAs per row group (such a matrix
    // is latency-, not bandwidth-bound)
    if (!device_count && njobs == 1 && (T + W - 1) / W < kCapBelowChunks && W > gm.row_groups * kMaxCtasPerRowGroup)
        W = gm.row_groups * kMaxCtasPerRowGroup;
    pl.workers = W;
    if (njobs == 1 && !device_count && W > 0) {
        const int len = (T + W - 1) / W;
        if (len < gm.chunks) {
            const GemvLayout lw = gemv_layout(gm.fmt, mrows, gm.K, len);
            if (lw.xres && c.nsm * gemv_ctas_per_sm(gm.fmt, pl.ntiles, lw.smem) >= W) {
                pl.lay = lw;
                pl.kwin = true;
            }
        }
    }
    if (njobs == 1 && !device_count && !pl.lay.xres) {
        // the rows do not fit beside two CTAs' rings (5..16 rows of a long K): one CTA per SM with
        // the rows resident (all of K, or the CTA's window of it) instead of a slice of every row
        // per stage. The tokens already share each MMA's 8 (16) columns, so the math per chunk is
        // the one-row launch's; the staged rows are what grows.
        for (int per_sm = 2; per_sm >= 1; --per_sm) {
            const int Wb = align_workers(std::min(c.nsm * per_sm, T), 1, gm.row_groups);
            const int len = (T + Wb - 1) / Wb;
            const GemvLayout lw =
                gemv_layout(gm.fmt, mrows, gm.K, len < gm.chunks ? len : 0, kWideResidentXBudget);
            if (lw.xres && c.nsm * gemv_ctas_per_sm(gm.fmt, pl.ntiles, lw.smem) >= Wb) {
                pl.lay = lw;
                pl.kwin = len < gm.chunks;
                pl.workers = Wb;
                break;
            }
        }
    }
    return pl;
}

// mmax: the largest token count of any job (the kernel sizes its activation slots by it)
// d_njobs: the job count is written on the device by the previous kernel (njobs is its bound)
int run_gemv(Ctx &c, const GpuMat &m, const GemvJob *d_jobs, int njobs, int mmax, int epi, const uint16_t *x,
             int64_t ldx, void *y, int64_t ldy, cudaStream_t s, bool pdl, const int *d_njobs = nullptr,
             const PeerOut *peer = nullptr, const GemvOpts &o = GemvOpts{}) {
    const int T = njobs * m.gm.row_groups * m.gm.chunks;
    if (T == 0) return 0;
    const bool split = o.xf != nullptr;
    const GemvPlan pl = plan_gemv(c, m.gm, njobs, split ? 2 * mmax : mmax, d_njobs != nullptr);
    const GemvLayout &lay = pl.lay;
    const int W = pl.workers, ntiles = pl.ntiles;
    if (split && epi != kEpiF32 && epi != kEpiSwiGLU && epi != kEpiPeer) {
        set_err("fp32 activations take the fp32, SwiGLU and peer epilogues (epilogue %d given)", epi);
        return -1;
    }
    if (split && (!lay.xres || mmax > 8)) {
        set_err("fp32 activations need jobs of at most 8 tokens whose rows fit in shared memory (K = %lld)",
                static_cast<long long>(m.gm.K));
        return -1;
    }
    if (!ensure_scratch(c, W, ntiles, W)) return -1;
    GemvParams p{};
    p.jobs = d_jobs;
    p.njobs = njobs;
    p.N = static_cast<int>(m.gm.N);
    p.K = static_cast<int>(m.gm.K);
    p.row_groups = m.gm.row_groups;
    p.chunks = m.gm.chunks;
    p.total_chunks = T;
    p.workers = W;
    p.x = x;
    p.ldx = ldx;
    p.y = y;
    p.ldy = ldy;
    p.row_map = epi == kEpiSwiGLU || epi == kEpiPairSum ? nullptr : m.d_row_map;
    p.wchunks = lay.wchunks;
    p.kwin = pl.kwin ? 1 : 0;
    p.xsplit = split ? 1 : 0;
    p.xf = o.xf;
    p.yf32 = o.yf32 ? 1 : 0;
    p.part = c.d_part;
    p.counters = c.d_cnt;
    p.err = c.d_err;
    p.jobs_ready = d_njobs ? 0 : 1;
    p.njobs_dev = d_njobs;
    p.trace = c.gemv_trace && W <= c.gemv_trace_ctas ? c.gemv_trace : nullptr;
    if (peer) {
        for (int r = 0; r < peer->world; ++r) p.peer[r] = peer->bufs[r];
        p.peer_rank = peer->rank;
        p.peer_world = peer->world;
        p.peer_cap = peer->cap;
        p.peer_calls = reinterpret_cast<uint32_t *>(static_cast<uint2 *>(peer->bufs[peer->rank]) +
                                                    2 * static_cast<int64_t>(peer->world) * peer->cap) +
                       kCommCtas;
        p.y_bf16 = peer->y_bf16;
        p.peer_wait_ns = c.peer_wait_ns;
        if (W > kPeerCtaCounters) {
            set_err("the all-reduce GEMV's %d CTAs exceed the communicator's %d call counters", W, kPeerCtaCounters);
            return -1;
        }
    }
    p.mul[0] = 1u << 28;
    p.mul[1] = 1u << 24;
    p.mul[2] = 1u << 20;
    p.mul[3] = 1u << 16;
    p.unpk[0] = 0x000F000Fu;
    p.unpk[1] = 0x00F000F0u;
    p.unpk[2] = 0x64006400u;
    p.xslots = lay.xslots;
    p.xres = lay.xres;
    p.xstride = lay.xstride;
    p.ctab_off = lay.ctab_off;
    p.off_bar = lay.off_bar;
    ONPU_CUDA(gemv_launch(m.gm.fmt, ntiles, epi, p, lay.smem, s, pdl), -1);
    ++c.calls;
    return 0;
}

// The deepest ring (8 .. 4 stages) that still gives two CTAs per SM, else one CTA per SM; false if
// the activation region does not fit at all.
bool choose_chain_layout(int fmt, int ntiles, int64_t xregion, ChainLayout &lay, int &occ) {
    occ = 0;
    for (int want = 2; want >= 1; --want)
        for (int ns = 8; ns >= 4; --ns) {
            lay = chain_layout(fmt, ntiles, xregion, ns);
            occ = lay.smem <= 227 * 1024 ? chain_ctas_per_sm(fmt, ntiles, lay.smem) : 0;
            if (occ >= want) return true;
        }
    return false;
}

void reset_chains_after_error();   // GEMV chains: clear their counters (defined with the chains)

// after a synchronising host call: surface device-side timeouts and reset the split-row counters
int check_device_err(Ctx &c) {
    int h = 0;
    if (cudaMemcpy(&h, c.d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        set_err("reading the device status failed: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    if (h) {
        cudaMemset(c.d_err, 0, sizeof(int));
        if (c.d_cnt) cudaMemset(c.d_cnt, 0, sizeof(unsigned) * c.cnt_cap);
        if (c.d_ffnbar) cudaMemset(c.d_ffnbar, 0, sizeof(unsigned) * c.ffnbar_cap);   // counters a timed-out wait left
        reset_chains_after_error();
        if (h & 16)
            set_err("an all-reduce timed out waiting for a peer rank (device status %d)", h);
        else if (h & 8)
            set_err("an expert id was out of range [0, E) in a routed job list; those (token, slot) pairs were "
                    "dropped (device status %d)", h);
        else
            set_err("a GEMV kernel timed out waiting for its weight copies (device status %d)", h);
        return -2;
    }
    return 0;
}

// stage host fp32 rows [rows][K] -> bf16 [rows][Kp] (zero past K) on the library stream
bool stage_x(Ctx &c, const float *x, int64_t rows, int64_t K, int64_t Kp) {
    if (!grow(c.d_in, c.in_cap, rows * K) || !grow(c.d_x, c.x_cap, rows * Kp)) return false;
    if (cudaMemcpyAsync(c.d_in, x, sizeof(float) * rows * K, cudaMemcpyHostToDevice, c.stream) != cudaSuccess) return false;
    if (Kp != K && cudaMemsetAsync(c.d_x, 0, sizeof(uint16_t) * rows * Kp, c.stream) != cudaSuccess) return false;
    return f32_to_bf16_launch(c.d_in, rows, K, K, c.d_x, Kp, c.stream) == cudaSuccess;
}

bool finish(Ctx &c) {
    const auto t0 = std::chrono::steady_clock::now();
    cudaError_t e = cudaStreamSynchronize(c.stream);
    c.wait_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (e != cudaSuccess) {
        set_err("kernel failed: %s", cudaGetErrorString(e));
        return false;
    }
    return check_device_err(c) == 0;
}

// (token, slot) pairs grouped by expert (ascending id, then arrival order), <= per_job per job
void build_expert_jobs(const GpuMat &m, const int32_t *ids, int64_t T, int k, bool x_per_slot, bool x_by_slot,
                       std::vector<GemvJob> &jobs, int &mmax, int per_job = kMaxTokensPerJob) {
    jobs.clear();
    mmax = 1;
    std::vector<int64_t> count(static_cast<size_t>(m.E) + 1, 0);
    for (int64_t i = 0; i < T * k; ++i) ++count[ids[i] + 1];
    for (int64_t e = 0; e < m.E; ++e) count[e + 1] += count[e];
    std::vector<int64_t> order(static_cast<size_t>(T * k));
    std::vector<int64_t> pos(count.begin(), count.end() - 1);
    for (int64_t i = 0; i < T * k; ++i) order[pos[ids[i]]++] = i;
    for (int64_t e = 0; e < m.E; ++e) {
        for (int64_t a = count[e]; a < count[e + 1]; a += per_job) {
            GemvJob jb{};
            jb.w = m.d_w + e * m.gm.bytes;
            jb.m = static_cast<int>(std::min<int64_t>(per_job, count[e + 1] - a));
            for (int n = 0; n < jb.m; ++n) {
                const int64_t slot = order[a + n];
                jb.xrow[n] = static_cast<int>(x_by_slot ? slot : (x_per_slot ? slot : slot / k));
                jb.yrow[n] = static_cast<int>(slot);
            }
            mmax = std::max(mmax, jb.m);
            jobs.push_back(jb);
        }
    }
}

bool upload_jobs(Ctx &c, const std::vector<GemvJob> &jobs) {
    if (!grow(c.d_jobs, c.jobs_cap, static_cast<int64_t>(jobs.size()))) return false;
    return cudaMemcpyAsync(c.d_jobs, jobs.data(), sizeof(GemvJob) * jobs.size(), cudaMemcpyHostToDevice, c.stream) ==
           cudaSuccess;
}

// ------------------------------------------------------------------ handles
struct JobSet {
    GemvJob *d = nullptr;
    int n = 0, ntiles = 1, mmax = 1;
};

struct DenseH {
    Geometry geo;                 // reference upload geometry (8 columns); !ok for int4 ingest
    int fmt = kFmtQ4S;
    GpuMat mat;
    uint8_t *h_buf = nullptr;     // pinned stream-order upload buffer
    bool gateup = false;
    bool residual = false;        // rows [W; W - dequant(W)] interleaved per strip (two-pass mode)
    std::map<int64_t, JobSet> jobs;
    ~DenseH() {
        if (h_buf) cudaFreeHost(h_buf);
        for (auto &kv : jobs) cudaFree(kv.second.d);
    }
};

struct BankH {
    Geometry geo;
    int fmt = kFmtQ4S;
    GpuMat mat;
    uint8_t *h_buf = nullptr;     // E * geo.nbytes
    bool owns_buf = true;
    ~BankH() {
        if (h_buf && owns_buf) cudaFreeHost(h_buf);
    }
};

struct FfnH {
    BankH *gu = nullptr, *dn = nullptr;
    bool fused = false;           // gate/up interleaved on the GPU: SwiGLU fused into the GEMV
    ~FfnH() {
        delete gu;
        delete dn;
    }
};

JobSet *dense_jobs(DenseH *d, int64_t rows) {
    auto it = d->jobs.find(rows);
    if (it != d->jobs.end()) return &it->second;
    JobSet js;
    js.n = static_cast<int>((rows + kMaxTokensPerJob - 1) / kMaxTokensPerJob);
    std::vector<GemvJob> h(static_cast<size_t>(js.n));
    for (int j = 0; j < js.n; ++j) {
        GemvJob &jb = h[j];
        jb.w = d->mat.d_w;
        jb.m = static_cast<int>(std::min<int64_t>(kMaxTokensPerJob, rows - static_cast<int64_t>(j) * kMaxTokensPerJob));
        for (int n = 0; n < jb.m; ++n) jb.xrow[n] = jb.yrow[n] = j * kMaxTokensPerJob + n;
        if (jb.m > 8) js.ntiles = 2;
        js.mmax = std::max(js.mmax, jb.m);
    }
    if (cudaMalloc(&js.d, sizeof(GemvJob) * js.n) != cudaSuccess ||
        cudaMemcpy(js.d, h.data(), sizeof(GemvJob) * js.n, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_err("allocating GEMV descriptors failed");
        return nullptr;
    }
    return &(d->jobs[rows] = js);
}

// stream-order upload (device copy at d_src) -> GPU layout of expert/matrix at dst
cudaError_t repack_stream(const Geometry &g, const GpuMat &m, const uint8_t *d_src, uint8_t *dst, cudaStream_t s) {
    RepackParams p{};
    p.src_kind = kSrcStream;
    p.src = d_src;
    p.src_row = nullptr;
    p.N = g.N;
    p.K = m.gm.K;            // padded to 32; the stream buffer holds the quantised padding
    p.fmt = m.gm.fmt;
    p.R = g.R;
    p.S = g.S;
    p.tiles = g.tiles;
    p.kc = g.kc;
    p.ks = g.ks;
    p.rows_col = g.rows_col;
    p.cb = g.cb;
    p.pkt = g.pkt();
    p.dst = dst;
    if (!m.src_row.empty()) {
        // the interleave map is also the row_map on the device
        p.src_row = m.d_row_map;
    }
    return repack_launch(p, s);
}

BankH *new_bank(int64_t N, int64_t K, int64_t E, int ncols, int sym) {
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    Geometry g(N, K, ncols, sym != 0);
    if (!g.ok || E <= 0) {
        set_err("no %d-column geometry for [%lld, %lld]", ncols, static_cast<long long>(N), static_cast<long long>(K));
        return nullptr;
    }
    auto *b = new BankH;
    b->geo = g;
    b->fmt = sym ? kFmtQ4S : kFmtQ4NX;
    if (!alloc_mat(b->mat, N, K, b->fmt, E)) {
        delete b;
        return nullptr;
    }
    if (cudaHostAlloc(&b->h_buf, static_cast<size_t>(g.nbytes * E), cudaHostAllocDefault) != cudaSuccess) {
        set_err("pinned host buffer of %lld bytes", static_cast<long long>(g.nbytes * E));
        delete b;
        return nullptr;
    }
    std::memset(b->h_buf, 0, static_cast<size_t>(g.nbytes * E));
    return b;
}

bool sync_bank(BankH *b) {
    if (!b->h_buf) return true;   // int4 banks are loaded by onpu_bank_load_int4
    Ctx &c = ctx();
    const int64_t per = b->geo.nbytes;
    const int64_t batch = std::max<int64_t>(1, std::min<int64_t>(b->mat.E, (256LL << 20) / std::max<int64_t>(per, 1)));
    uint8_t *tmp = nullptr;
    ONPU_CUDA(cudaMalloc(&tmp, static_cast<size_t>(per * batch)), false);
    bool ok = true;
    for (int64_t e0 = 0; e0 < b->mat.E && ok; e0 += batch) {
        const int64_t n = std::min(batch, b->mat.E - e0);
        ok = cudaMemcpyAsync(tmp, b->h_buf + e0 * per, static_cast<size_t>(per * n), cudaMemcpyHostToDevice, c.stream) ==
             cudaSuccess;
        for (int64_t e = 0; e < n && ok; ++e)
            ok = repack_stream(b->geo, b->mat, tmp + e * per, b->mat.d_w + (e0 + e) * b->mat.gm.bytes, c.stream) ==
                 cudaSuccess;
        ok = ok && cudaStreamSynchronize(c.stream) == cudaSuccess;
    }
    cudaFree(tmp);
    if (!ok) set_err("bank upload failed: %s", cudaGetErrorString(cudaGetLastError()));
    return ok;
}

bool valid_ids(const int32_t *ids, int64_t n, int64_t E) {
    for (int64_t i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= E) {
            set_err("expert id %d out of range [0, %lld)", ids[i], static_cast<long long>(E));
            return false;
        }
    return true;
}

// routed-expert FFN on the device; inputs already validated. fused: gate_up bank interleaved,
// SwiGLU in the GEMV epilogue (act 0 and no biases only). The activation between the projections
// stays fp32 (the reference's moe_act output, onpu_cpu.cpp:233-256): the down GEMV stages it as
// two fp16 halves per value, so its products keep ~22 bits of the activation.
bool moe_ffn_impl(BankH *gu, BankH *dn, const float *x, int64_t T, const int32_t *ids, int k, const float *w, int act,
                  float alpha, float limit, const float *gu_bias, const float *dn_bias, float *y, bool fused) {
    Ctx &c = ctx();
    const int64_t Ng = gu->geo.N, I = Ng / 2, Nd = dn->geo.N, Kg = gu->geo.K, Kgp = gu->mat.gm.K;
    const int64_t Kdp = dn->mat.gm.K, TK = T * k;
    if (dn->geo.K != I) {
        set_err("down bank K (%lld) != gate_up N/2 (%lld)", static_cast<long long>(dn->geo.K), static_cast<long long>(I));
        return false;
    }
    // down jobs: the most tokens (<= 8) whose two fp16 rows each stay resident
    int dn_per_job = 8;
    while (dn_per_job > 1 && !gemv_resident(2 * dn_per_job, Kdp)) dn_per_job /= 2;
    if (!gemv_resident(2 * dn_per_job, Kdp)) {
        set_err("down projection K = %lld is too long for one resident fp32 activation row", static_cast<long long>(Kdp));
        return false;
    }
    if (!stage_x(c, x, T, Kg, Kgp)) return false;
    std::vector<GemvJob> jg, jd;
    int mg = 1, md = 1;
    build_expert_jobs(gu->mat, ids, T, k, false, false, jg, mg);
    build_expert_jobs(dn->mat, ids, T, k, false, true, jd, md, dn_per_job);
    std::vector<GemvJob> all(jg);
    all.insert(all.end(), jd.begin(), jd.end());
    if (!upload_jobs(c, all)) return false;
    if (!grow(c.d_af, c.af_cap, TK * Kdp) || !grow(c.d_o, c.o_cap, TK * Nd) || !grow(c.d_y, c.y_cap, T * Nd) ||
        !grow(c.d_ids, c.ids_cap, TK) || !grow(c.d_w, c.w_cap, TK))
        return false;
    ONPU_CUDA(cudaMemcpyAsync(c.d_ids, ids, sizeof(int32_t) * TK, cudaMemcpyHostToDevice, c.stream), false);
    ONPU_CUDA(cudaMemcpyAsync(c.d_w, w, sizeof(float) * TK, cudaMemcpyHostToDevice, c.stream), false);
    if (Kdp != I) ONPU_CUDA(cudaMemsetAsync(c.d_af, 0, sizeof(float) * TK * Kdp, c.stream), false);
    const float *d_gb = nullptr, *d_db = nullptr;
    if (gu_bias) {
        if (!grow(c.d_gb, c.gb_cap, gu->mat.E * Ng)) return false;
        ONPU_CUDA(cudaMemcpyAsync(c.d_gb, gu_bias, sizeof(float) * gu->mat.E * Ng, cudaMemcpyHostToDevice, c.stream), false);
        d_gb = c.d_gb;
    }
    if (dn_bias) {
        if (!grow(c.d_db, c.db_cap, dn->mat.E * Nd)) return false;
        ONPU_CUDA(cudaMemcpyAsync(c.d_db, dn_bias, sizeof(float) * dn->mat.E * Nd, cudaMemcpyHostToDevice, c.stream), false);
        d_db = c.d_db;
    }
    if (fused && act == 0 && !gu_bias) {
        GemvOpts o;
        o.yf32 = true;
        if (run_gemv(c, gu->mat, c.d_jobs, static_cast<int>(jg.size()), mg, kEpiSwiGLU, c.d_x, Kgp, c.d_af, Kdp,
                     c.stream, false, nullptr, nullptr, o))
            return false;
    } else {
        if (!grow(c.d_h, c.h_cap, TK * Ng)) return false;
        if (run_gemv(c, gu->mat, c.d_jobs, static_cast<int>(jg.size()), mg, kEpiF32, c.d_x, Kgp, c.d_h, Ng, c.stream,
                     false))
            return false;
        ONPU_CUDA(moe_act_f32_launch(c.d_h, Ng, TK, Ng, c.d_ids, d_gb, act, alpha, limit, c.d_af, Kdp, c.stream), false);
    }
    GemvOpts od;
    od.xf = c.d_af;
    if (run_gemv(c, dn->mat, c.d_jobs + jg.size(), static_cast<int>(jd.size()), md, kEpiF32, nullptr, Kdp, c.d_o, Nd,
                 c.stream, false, nullptr, nullptr, od))
        return false;
    ONPU_CUDA(moe_combine_launch(c.d_o, Nd, T, k, Nd, c.d_ids, c.d_w, d_db, c.d_y, Nd, c.stream), false);
    ONPU_CUDA(cudaMemcpyAsync(y, c.d_y, sizeof(float) * T * Nd, cudaMemcpyDeviceToHost, c.stream), false);
    return finish(c);
}

}  // namespace

// ======================================================================== part 1
extern "C" {

int onpu_ok(void) { return ctx().ok ? 1 : 0; }
int onpu_batched_ok(void) { return onpu_ok(); }

void onpu_stats(int64_t *calls, double *wait_s) {
    Ctx &c = ctx();
    *calls = c.calls;
    *wait_s = c.wait_s;
}

int onpu_has_shape(int tiles, int kc, int batched) {
    (void)tiles;
    (void)kc;
    (void)batched;
    return onpu_ok();
}

void onpu_geometry2(int64_t N, int64_t K, int ncols, int sym, int64_t *out) {
    const Geometry g(N, K, ncols, sym != 0);
    const int64_t v[8] = {g.R, g.S, g.tiles, g.kc, g.ks, g.rows_col, g.cb, g.nbytes};
    for (int i = 0; i < 8; ++i) out[i] = g.ok ? v[i] : 0;
}

void onpu_geometry(int64_t N, int64_t K, int ncols, int64_t *out) { onpu_geometry2(N, K, ncols, 0, out); }

// ---- dense
void *onpu_dense_new2(int64_t N, int64_t K, int sym) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    Geometry g(N, K, kNC, sym != 0);
    if (!g.ok) {
        set_err("no 8-column geometry for [%lld, %lld]", static_cast<long long>(N), static_cast<long long>(K));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    auto *d = new DenseH;
    d->geo = g;
    d->fmt = sym ? kFmtQ4S : kFmtQ4NX;
    if (!alloc_mat(d->mat, N, K, d->fmt, 1) ||
        cudaHostAlloc(&d->h_buf, static_cast<size_t>(g.nbytes), cudaHostAllocDefault) != cudaSuccess) {
        if (!t_has_err) set_err("pinned host buffer of %lld bytes", static_cast<long long>(g.nbytes));
        delete d;
        return nullptr;
    }
    std::memset(d->h_buf, 0, static_cast<size_t>(g.nbytes));
    return d;
}

void *onpu_dense_new(int64_t N, int64_t K) { return onpu_dense_new2(N, K, 0); }
uint8_t *onpu_dense_buf(void *h) { return static_cast<DenseH *>(h)->h_buf; }
int64_t onpu_dense_bytes(void *h) { return static_cast<DenseH *>(h)->geo.nbytes; }

void onpu_dense_sync(void *h) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    if (!d->h_buf) {
        set_err("onpu_dense_sync: this matrix takes int4 uploads (onpu_dense_load_int4)");
        return;
    }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    uint8_t *tmp = nullptr;
    ONPU_CUDA(cudaMalloc(&tmp, static_cast<size_t>(d->geo.nbytes)), );
    cudaError_t e = cudaMemcpyAsync(tmp, d->h_buf, static_cast<size_t>(d->geo.nbytes), cudaMemcpyHostToDevice, c.stream);
    if (e == cudaSuccess) e = repack_stream(d->geo, d->mat, tmp, d->mat.d_w, c.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c.stream);
    cudaFree(tmp);
    if (e != cudaSuccess) set_err("onpu_dense_sync: %s", cudaGetErrorString(e));
}

void onpu_dense_mv(void *h, const float *x, int64_t rows, float *y) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    if (rows <= 0) return;
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    const int64_t K = d->mat.gm.K, N = d->mat.gm.N;
    const int64_t Kin = d->geo.ok ? d->geo.K : K;
    JobSet *js = dense_jobs(d, rows);
    if (!js || !grow(c.d_y, c.y_cap, rows * N)) return;
    // up to 8 rows whose fp32 values fit in shared memory: staged exactly (two fp16 halves per
    // value); otherwise rounded to bf16, as the reference's device path rounds its inputs
    const bool exact = Kin == K && rows <= 8 && plan_gemv(c, d->mat.gm, 1, 2 * static_cast<int>(rows), false).lay.xres;
    if (exact) {
        if (!grow(c.d_in, c.in_cap, rows * K)) return;
        ONPU_CUDA(cudaMemcpyAsync(c.d_in, x, sizeof(float) * rows * K, cudaMemcpyHostToDevice, c.stream), );
        GemvOpts o;
        o.xf = c.d_in;
        if (run_gemv(c, d->mat, js->d, js->n, js->mmax, kEpiF32, nullptr, K, c.d_y, N, c.stream, false, nullptr,
                     nullptr, o))
            return;
    } else {
        if (!stage_x(c, x, rows, Kin, K)) return;
        if (run_gemv(c, d->mat, js->d, js->n, js->mmax, kEpiF32, c.d_x, K, c.d_y, N, c.stream, false)) return;
    }
    ONPU_CUDA(cudaMemcpyAsync(y, c.d_y, sizeof(float) * rows * N, cudaMemcpyDeviceToHost, c.stream), );
    finish(c);
}

void onpu_dense_free(void *h) {
    std::lock_guard<std::mutex> lk(g_mu);
    cudaDeviceSynchronize();
    delete static_cast<DenseH *>(h);
}

// ---- banks
void *onpu_bank_new2(int64_t N, int64_t K, int64_t E, int ncols, int sym) {
    clear_err();
    std::lock_guard<std::mutex> lk(g_mu);
    return new_bank(N, K, E, ncols, sym);
}
void *onpu_bank_new(int64_t N, int64_t K, int64_t E, int ncols) { return onpu_bank_new2(N, K, E, ncols, 0); }
uint8_t *onpu_bank_buf(void *h) { return static_cast<BankH *>(h)->h_buf; }
int64_t onpu_bank_expert_bytes(void *h) { return static_cast<BankH *>(h)->geo.nbytes; }

void onpu_bank_sync(void *h) {
    clear_err();
    std::lock_guard<std::mutex> lk(g_mu);
    sync_bank(static_cast<BankH *>(h));
}

void onpu_bank_free(void *h) {
    std::lock_guard<std::mutex> lk(g_mu);
    cudaDeviceSynchronize();
    delete static_cast<BankH *>(h);
}

void onpu_bank_run(void *h, const float *x, int x_per_slot, int64_t T, const int32_t *ids, int k, float *y) {
    clear_err();
    auto *b = static_cast<BankH *>(h);
    if (T <= 0 || k <= 0) return;
    if (!valid_ids(ids, T * k, b->mat.E)) return;
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    const int64_t N = b->geo.N, Kp = b->mat.gm.K;
    const int64_t xrows = x_per_slot ? T * k : T;
    std::vector<GemvJob> jobs;
    int mm = 1;
    // fp32 inputs staged exactly (two fp16 halves, jobs of 8) when those rows fit in shared
    // memory; otherwise rounded to bf16 (the reference's device rounding)
    const bool exact = b->geo.K == Kp && gemv_resident(16, Kp);
    if (exact) {
        if (!grow(c.d_in, c.in_cap, xrows * Kp)) return;
        ONPU_CUDA(cudaMemcpyAsync(c.d_in, x, sizeof(float) * xrows * Kp, cudaMemcpyHostToDevice, c.stream), );
    } else if (!stage_x(c, x, xrows, b->geo.K, Kp)) {
        return;
    }
    build_expert_jobs(b->mat, ids, T, k, x_per_slot != 0, false, jobs, mm, exact ? 8 : kMaxTokensPerJob);
    if (!upload_jobs(c, jobs) || !grow(c.d_y, c.y_cap, T * k * N)) return;
    GemvOpts o;
    if (exact) o.xf = c.d_in;
    if (run_gemv(c, b->mat, c.d_jobs, static_cast<int>(jobs.size()), mm, kEpiF32, exact ? nullptr : c.d_x, Kp, c.d_y, N,
                 c.stream, false, nullptr, nullptr, o))
        return;
    ONPU_CUDA(cudaMemcpyAsync(y, c.d_y, sizeof(float) * T * k * N, cudaMemcpyDeviceToHost, c.stream), );
    finish(c);
}

// ---- MoE
void onpu_moe_ffn(void *gu, void *dn, const float *x, int64_t T, const int32_t *ids, int k, const float *w, int act,
                  float alpha, float limit, const float *gu_bias, const float *dn_bias, float *y) {
    clear_err();
    auto *g = static_cast<BankH *>(gu);
    auto *d = static_cast<BankH *>(dn);
    if (T <= 0) return;
    if (!valid_ids(ids, T * k, std::min(g->mat.E, d->mat.E))) return;
    std::lock_guard<std::mutex> lk(g_mu);
    moe_ffn_impl(g, d, x, T, ids, k, w, act, alpha, limit, gu_bias, dn_bias, y, !g->mat.src_row.empty());
}

void onpu_moe_act(const float *h, int64_t rows, int64_t Ng, const int32_t *ids, const float *gu_bias, int act,
                  float alpha, float limit, float *a) {
    const int64_t I = Ng / 2;
    std::vector<float> tmp(static_cast<size_t>(Ng));
    for (int64_t r = 0; r < rows; ++r) {
        const float *hr = h + r * Ng;
        if (gu_bias) {
            const float *b = gu_bias + static_cast<int64_t>(ids[r]) * Ng;
            for (int64_t i = 0; i < Ng; ++i) tmp[i] = hr[i] + b[i];
            hr = tmp.data();
        }
        float *ar = a + r * I;
        for (int64_t i = 0; i < I; ++i) {
            if (act == 1) {
                const float gt = std::min(hr[2 * i], limit);
                const float up = std::max(-limit, std::min(hr[2 * i + 1], limit));
                ar[i] = (up + 1.f) * gt / (1.f + std::exp(-alpha * gt));
            } else {
                ar[i] = hr[i] / (1.f + std::exp(-hr[i])) * hr[I + i];
            }
        }
    }
}

void onpu_moe_sum(const float *o, int64_t T, int k, int64_t N, const int32_t *ids, const float *w, const float *bias,
                  float *y) {
    for (int64_t t = 0; t < T; ++t) {
        float *yt = y + t * N;
        std::fill(yt, yt + N, 0.f);
        for (int j = 0; j < k; ++j) {
            const int64_t r = t * k + j;
            const float wr = w[r], *orow = o + r * N;
            const float *b = bias ? bias + static_cast<int64_t>(ids[r]) * N : nullptr;
            for (int64_t i = 0; i < N; ++i) yt[i] += wr * (orow[i] + (b ? b[i] : 0.f));
        }
    }
}

// ---- fused FFN
void *onpu_ffn_new(int64_t Ng, int64_t Kg, int64_t Nd, int64_t Kd, int64_t E, int sym) {
    clear_err();
    std::lock_guard<std::mutex> lk(g_mu);
    auto *f = new FfnH;
    f->gu = new_bank(Ng, Kg, E, 1, sym);
    f->dn = f->gu ? new_bank(Nd, Kd, E, 1, sym) : nullptr;
    if (!f->gu || !f->dn) {
        delete f;
        return nullptr;
    }
    f->fused = Kd == Ng / 2 && set_gateup_interleave(f->gu->mat);
    return f;
}
void *onpu_ffn_gu(void *h) { return static_cast<FfnH *>(h)->gu; }
void *onpu_ffn_dn(void *h) { return static_cast<FfnH *>(h)->dn; }
int onpu_ffn_fused(void *h) { return static_cast<FfnH *>(h)->fused ? 1 : 0; }
void onpu_ffn_perm(void *h, int32_t *out) {
    const int64_t n = static_cast<FfnH *>(h)->gu->geo.N;
    for (int64_t r = 0; r < n; ++r) out[r] = static_cast<int32_t>(r);
}
void onpu_ffn_free(void *h) {
    std::lock_guard<std::mutex> lk(g_mu);
    cudaDeviceSynchronize();
    delete static_cast<FfnH *>(h);
}

int onpu_ffn_run(void *h, const float *x, const int32_t *ids, int k, const float *w, float *y) {
    return onpu_ffn_run_many(h, x, 1, ids, k, w, y);
}

int onpu_ffn_run_many(void *h, const float *x, int64_t T, const int32_t *ids, int k, const float *w, float *y) {
    clear_err();
    auto *f = static_cast<FfnH *>(h);
    if (T <= 0) return 1;
    if (!valid_ids(ids, T * k, f->gu->mat.E)) return 0;
    std::lock_guard<std::mutex> lk(g_mu);
    return moe_ffn_impl(f->gu, f->dn, x, T, ids, k, w, 0, 0.f, 0.f, nullptr, nullptr, y, f->fused) ? 1 : 0;
}

// ---- codec
int64_t onpu_pack(const float *W, int64_t N, int64_t K, int ncols, int sym, uint8_t *out, int threads) {
    const Geometry g(N, K, ncols, sym != 0);
    if (!g.ok) return 0;
    pack_stream(g, W, out, threads);
    return g.nbytes;
}

void onpu_quant_dequant(const float *W, int64_t N, int64_t K, int sym, float *out, int threads) {
    quant_dequant(W, N, K, sym != 0, out, threads);
}

// ======================================================================== part 2
const char *onpu_last_error(void) { return t_has_err ? t_err.c_str() : nullptr; }

int onpu_check_device(void) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return -1;
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        set_err("device error: %s", cudaGetErrorString(e));
        return -1;
    }
    return check_device_err(c);
}

void *onpu_dense_new_int4(int64_t N, int64_t K, int gateup) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    if (N <= 0 || K <= 0 || K % 32) {
        set_err("onpu_dense_new_int4: need N > 0 and K %% 32 == 0 (got %lld, %lld)", static_cast<long long>(N),
                static_cast<long long>(K));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    auto *d = new DenseH;
    d->fmt = kFmtQ4F16;
    d->gateup = gateup != 0;
    if (!alloc_mat(d->mat, N, K, d->fmt, 1)) {
        delete d;
        return nullptr;
    }
    if (d->gateup && !set_gateup_interleave(d->mat)) {
        set_err("onpu_dense_new_int4: gate/up matrix needs N/2 %% 8 == 0");
        delete d;
        return nullptr;
    }
    return d;
}

}  // extern "C"

namespace {
// E matrices of GGUF rows (device bytes, E * N rows of row_bytes) -> the GPU layout of m (one
// matrix after the other): codes, scales and mins on the device, then the codes repack. Caller
// holds g_mu.
bool gguf_to_mat(GpuMat &m, int type, const uint8_t *d_src, int64_t N, int64_t K, int64_t E, cudaStream_t s,
                 const char *who) {
    const int64_t rb = gguf_row_bytes(type, K);
    uint8_t *q = nullptr;
    uint16_t *sc = nullptr, *mn = nullptr;
    const size_t nq = static_cast<size_t>(N * K), ns = static_cast<size_t>(N * (K / 32));
    cudaError_t e = cudaMalloc(&q, nq);
    if (e == cudaSuccess) e = cudaMalloc(&sc, ns * 2);
    if (e == cudaSuccess) e = cudaMalloc(&mn, ns * 2);
    for (int64_t x = 0; x < E && e == cudaSuccess; ++x) {
        e = gguf_codes_launch(type, d_src + x * N * rb, N, K, q, sc, mn, s);
        RepackParams p{};
        p.src_kind = kSrcCodes;
        p.src = q;
        p.scales = sc;
        p.mins = type == kGgmlQ4_K ? mn : nullptr;
        p.src_row = m.d_row_map;
        p.N = N;
        p.K = K;
        p.fmt = m.gm.fmt;
        p.dst = m.d_w + x * m.gm.bytes;
        if (e == cudaSuccess) e = repack_launch(p, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);     // q / sc / mn are reused
    }
    cudaFree(q);
    cudaFree(sc);
    cudaFree(mn);
    if (e != cudaSuccess) {
        set_err("%s: %s", who, cudaGetErrorString(e));
        return false;
    }
    return true;
}

// GGUF bytes of E matrices on the device (a copy when they are on the host); nullptr on error
const uint8_t *gguf_device_bytes(const void *data, int on_device, int64_t bytes, uint8_t *&owned, cudaStream_t s,
                                 const char *who) {
    owned = nullptr;
    if (on_device) return static_cast<const uint8_t *>(data);
    cudaError_t e = cudaMalloc(&owned, static_cast<size_t>(bytes));
    if (e == cudaSuccess) e = cudaMemcpyAsync(owned, data, static_cast<size_t>(bytes), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
        set_err("%s: %s", who, cudaGetErrorString(e));
        cudaFree(owned);
        owned = nullptr;
        return nullptr;
    }
    return owned;
}
}  // namespace

extern "C" {

int onpu_gguf_codes_dev(int type, const void *src, int64_t rows, int64_t K, uint8_t *q, uint16_t *scales,
                        uint16_t *mins, void *stream) {
    clear_err();
    if (gguf_row_bytes(type, K) < 0 || rows <= 0 || (type == kGgmlQ4_K && !mins)) {
        set_err("onpu_gguf_codes_dev: type %d with K = %lld is not a supported GGUF layout (Q4_0: K %% 32 == 0, "
                "Q4_K: K %% 256 == 0 and a mins output)", type, static_cast<long long>(K));
        return -1;
    }
    ONPU_CUDA(gguf_codes_launch(type, static_cast<const uint8_t *>(src), rows, K, q, scales, mins,
                                static_cast<cudaStream_t>(stream)),
              -1);
    return 0;
}

void *onpu_dense_new_gguf(int64_t N, int64_t K, int type, const void *data, int on_device, int gateup, void *stream) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    const int64_t rb = gguf_row_bytes(type, K);
    if (N <= 0 || rb < 0 || !data) {
        set_err("onpu_dense_new_gguf: type %d with K = %lld is not a supported GGUF layout (Q4_0: K %% 32 == 0, "
                "Q4_K: K %% 256 == 0)", type, static_cast<long long>(K));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c.stream;
    auto *d = new DenseH;
    d->fmt = type == kGgmlQ4_K ? kFmtQ4NX : kFmtQ4F16;
    d->gateup = gateup != 0;
    uint8_t *owned = nullptr;
    bool ok = alloc_mat(d->mat, N, K, d->fmt, 1);
    if (ok && d->gateup && !set_gateup_interleave(d->mat)) {
        set_err("onpu_dense_new_gguf: gate/up matrix needs N/2 %% 8 == 0");
        ok = false;
    }
    const uint8_t *src = ok ? gguf_device_bytes(data, on_device, N * rb, owned, s, "onpu_dense_new_gguf") : nullptr;
    ok = ok && src && gguf_to_mat(d->mat, type, src, N, K, 1, s, "onpu_dense_new_gguf");
    cudaFree(owned);
    if (!ok) {
        delete d;
        return nullptr;
    }
    return d;
}

void *onpu_bank_new_gguf(int64_t N, int64_t K, int64_t E, int type, const void *data, int on_device, int gateup,
                         void *stream) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    const int64_t rb = gguf_row_bytes(type, K);
    if (N <= 0 || E <= 0 || rb < 0 || !data) {
        set_err("onpu_bank_new_gguf: type %d with K = %lld is not a supported GGUF layout (Q4_0: K %% 32 == 0, "
                "Q4_K: K %% 256 == 0)", type, static_cast<long long>(K));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c.stream;
    auto *b = new BankH;
    b->fmt = type == kGgmlQ4_K ? kFmtQ4NX : kFmtQ4F16;
    b->owns_buf = false;
    b->geo.N = N;                 // no stream-order geometry: the weights arrive as GGUF blocks
    b->geo.K = K;
    uint8_t *owned = nullptr;
    bool ok = alloc_mat(b->mat, N, K, b->fmt, E);
    if (ok && gateup && !set_gateup_interleave(b->mat)) {
        set_err("onpu_bank_new_gguf: gate/up rows need N %% 2 == 0 and N/2 %% 8 == 0");
        ok = false;
    }
    const uint8_t *src = ok ? gguf_device_bytes(data, on_device, E * N * rb, owned, s, "onpu_bank_new_gguf") : nullptr;
    ok = ok && src && gguf_to_mat(b->mat, type, src, N, K, E, s, "onpu_bank_new_gguf");
    cudaFree(owned);
    if (!ok) {
        delete b;
        return nullptr;
    }
    return b;
}

int onpu_quantize_dev(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, uint8_t *q, uint16_t *scales,
                      uint16_t *mins, void *stream) {
    clear_err();
    if (N <= 0 || K <= 0 || K % 32 || ldw < K || ldw % 4 || (reinterpret_cast<uintptr_t>(W) & 15) ||
        (reinterpret_cast<uintptr_t>(q) & 3)) {
        set_err("onpu_quantize_dev: need K %% 32 == 0, ldw >= K with ldw %% 4 == 0, 16-byte aligned W, 4-byte aligned q");
        return -1;
    }
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return -1;
    }
    ONPU_CUDA(quant_launch(W, ldw, N, K, sym, q, scales, mins, static_cast<cudaStream_t>(stream)), -1);
    return 0;
}

void *onpu_dense_new_f32_dev(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, int gateup, void *stream) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    if (N <= 0 || K <= 0 || K % 32) {
        set_err("onpu_dense_new_f32_dev: need N > 0 and K %% 32 == 0");
        return nullptr;
    }
    auto s = static_cast<cudaStream_t>(stream);
    uint8_t *q = nullptr;
    uint16_t *sc = nullptr, *mn = nullptr;
    const size_t nq = static_cast<size_t>(N * K), ns = static_cast<size_t>(N * (K / 32));
    if (cudaMalloc(&q, nq) != cudaSuccess || cudaMalloc(&sc, ns * 2) != cudaSuccess ||
        cudaMalloc(&mn, ns * 2) != cudaSuccess) {
        set_err("onpu_dense_new_f32_dev: %s", cudaGetErrorString(cudaGetLastError()));
        cudaFree(q);
        cudaFree(sc);
        return nullptr;
    }
    DenseH *d = nullptr;
    if (onpu_quantize_dev(W, ldw, N, K, sym, q, sc, mn, stream) == 0) {
        std::lock_guard<std::mutex> lk(g_mu);
        d = new DenseH;
        d->fmt = sym ? kFmtQ4S : kFmtQ4NX;
        d->gateup = gateup != 0;
        bool ok = alloc_mat(d->mat, N, K, d->fmt, 1);
        if (ok && d->gateup && !set_gateup_interleave(d->mat)) {
            set_err("onpu_dense_new_f32_dev: gate/up matrix needs N/2 %% 8 == 0");
            ok = false;
        }
        if (ok) {
            RepackParams p{};
            p.src_kind = kSrcCodes;
            p.src = q;
            p.scales = sc;
            p.mins = mn;
            p.src_row = d->mat.d_row_map;
            p.N = N;
            p.K = K;
            p.fmt = d->fmt;
            p.dst = d->mat.d_w;
            cudaError_t e = repack_launch(p, s);
            if (e == cudaSuccess) e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) {
                set_err("onpu_dense_new_f32_dev: %s", cudaGetErrorString(e));
                ok = false;
            }
        }
        if (!ok) {
            delete d;
            d = nullptr;
        }
    }
    cudaFree(q);
    cudaFree(sc);
    cudaFree(mn);
    return d;
}

void *onpu_dense_new_residual_f32_dev(const float *W, int64_t ldw, int64_t N, int64_t K, int sym, void *stream) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    if (N <= 0 || N % 8 || K <= 0 || K % 32 || ldw < K || ldw % 4 || (reinterpret_cast<uintptr_t>(W) & 15)) {
        set_err("onpu_dense_new_residual_f32_dev: need N %% 8 == 0, K %% 32 == 0, ldw >= K with ldw %% 4 == 0, "
                "16-byte aligned W");
        return nullptr;
    }
    auto s = static_cast<cudaStream_t>(stream);
    const int64_t G = K / 32;
    uint8_t *q = nullptr;
    uint16_t *sc = nullptr, *mn = nullptr;
    float *R = nullptr;
    DenseH *d = nullptr;
    cudaError_t e = cudaMalloc(&q, static_cast<size_t>(2 * N * K));
    if (e == cudaSuccess) e = cudaMalloc(&sc, static_cast<size_t>(2 * N * G) * 2);
    if (e == cudaSuccess) e = cudaMalloc(&mn, static_cast<size_t>(2 * N * G) * 2);
    if (e == cudaSuccess) e = cudaMalloc(&R, static_cast<size_t>(N * K) * 4);
    // pass 1: W; residual R = W - what pass 1 makes of W; pass 2: R (rows N .. 2N - 1 of the codes)
    if (e == cudaSuccess) e = quant_launch(W, ldw, N, K, sym, q, sc, mn, s);
    if (e == cudaSuccess) e = residual_launch(W, ldw, N, K, sym, q, sc, mn, R, s);
    if (e == cudaSuccess) e = quant_launch(R, K, N, K, sym, q + N * K, sc + N * G, mn + N * G, s);
    if (e == cudaSuccess) {
        std::lock_guard<std::mutex> lk(g_mu);
        d = new DenseH;
        d->fmt = sym ? kFmtQ4S : kFmtQ4NX;
        d->residual = true;
        // GPU strip rows 0-7: rows 8s..8s+7 of W, rows 8-15: the same rows of R (as gate/up pairs)
        if (!alloc_mat(d->mat, 2 * N, K, d->fmt, 1) || !set_gateup_interleave(d->mat)) {
            if (!onpu_last_error()) set_err("onpu_dense_new_residual_f32_dev: allocation failed");
            delete d;
            d = nullptr;
        } else {
            RepackParams p{};
            p.src_kind = kSrcCodes;
            p.src = q;
            p.scales = sc;
            p.mins = mn;
            p.src_row = d->mat.d_row_map;
            p.N = 2 * N;
            p.K = K;
            p.fmt = d->fmt;
            p.dst = d->mat.d_w;
            e = repack_launch(p, s);
        }
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(q);
    cudaFree(sc);
    cudaFree(mn);
    cudaFree(R);
    if (e != cudaSuccess) {
        set_err("onpu_dense_new_residual_f32_dev: %s", cudaGetErrorString(e));
        delete d;
        return nullptr;
    }
    return d;
}

int onpu_dense_load_int4(void *h, const uint8_t *qk, const uint16_t *scales, int on_device, void *stream) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    if (d->fmt != kFmtQ4F16) {
        set_err("onpu_dense_load_int4: matrix was not created by onpu_dense_new_int4");
        return -1;
    }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    const int64_t N = d->mat.gm.N, K = d->mat.gm.K;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c.stream;
    uint8_t *tq = nullptr;
    uint16_t *ts = nullptr;
    const uint8_t *sq = qk;
    const uint16_t *ss = scales;
    if (!on_device) {
        ONPU_CUDA(cudaMalloc(&tq, static_cast<size_t>(N * K / 2)), -1);
        ONPU_CUDA(cudaMalloc(&ts, static_cast<size_t>(N * K / 32) * 2), -1);
        ONPU_CUDA(cudaMemcpyAsync(tq, qk, static_cast<size_t>(N * K / 2), cudaMemcpyHostToDevice, s), -1);
        ONPU_CUDA(cudaMemcpyAsync(ts, scales, static_cast<size_t>(N * K / 32) * 2, cudaMemcpyHostToDevice, s), -1);
        sq = tq;
        ss = ts;
    }
    RepackParams p{};
    p.src_kind = kSrcInt4K;
    p.src = sq;
    p.scales = ss;
    p.src_row = d->mat.d_row_map;
    p.N = N;
    p.K = K;
    p.fmt = kFmtQ4F16;
    p.dst = d->mat.d_w;
    cudaError_t e = repack_launch(p, s);
    if (e == cudaSuccess && (!on_device || !stream)) e = cudaStreamSynchronize(s);
    if (tq) cudaFree(tq);
    if (ts) cudaFree(ts);
    if (e != cudaSuccess) {
        set_err("onpu_dense_load_int4: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

int onpu_dense_info(void *h, int64_t *out4) {
    auto *d = static_cast<DenseH *>(h);
    out4[0] = d->fmt;
    out4[1] = d->mat.gm.N;
    out4[2] = d->mat.gm.K;
    out4[3] = d->mat.gm.bytes;
    return 0;
}

int onpu_dense_prepare(void *h, int64_t rows) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    JobSet *js = dense_jobs(d, rows);
    if (!js) return -1;
    // the larger of the bf16 and the fp32 (split) activation plans
    const GemvPlan a = plan_gemv(c, d->mat.gm, js->n, js->mmax, false);
    const GemvPlan b = plan_gemv(c, d->mat.gm, js->n, 2 * js->mmax, false);
    const int W = std::max(a.workers, b.workers);
    return ensure_scratch(c, W, 2, W) ? 0 : -1;
}

}  // extern "C"

namespace {
// onpu_dense_mv_dev / onpu_dense_mv_f32_dev: x is bf16, or fp32 when xf32 (at most 8 rows)
int dense_mv_dev_impl(const char *who, void *h, const void *x, bool xf32, int64_t ldx, int64_t rows, void *y,
                      int64_t ldy, int epi, void *stream) {
    auto *d = static_cast<DenseH *>(h);
    if (rows <= 0) return 0;
    const bool yf32 = epi == ONPU_EPI_SWIGLU_F32;
    if (yf32) epi = kEpiSwiGLU;
    if (epi < kEpiF32 || epi > kEpiPairSum || (epi == kEpiSwiGLU && !d->gateup) ||
        (epi == kEpiPairSum && !d->residual)) {
        set_err("%s: bad epilogue %d for this matrix", who, yf32 ? ONPU_EPI_SWIGLU_F32 : epi);
        return -1;
    }
    if (d->geo.ok && d->geo.K != d->mat.gm.K) {
        set_err("%s: K must be a multiple of 32", who);
        return -1;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx & (xf32 ? 3 : 7)) || ldx < d->mat.gm.K) {
        set_err("%s: x rows must be 16-byte aligned (ldx a multiple of 16 bytes) with ldx >= K", who);
        return -1;
    }
    if (xf32 && rows > 8) {
        set_err("%s: fp32 activations take at most 8 rows per call (%lld given)", who, static_cast<long long>(rows));
        return -1;
    }
    if (ldy < (epi >= kEpiSwiGLU ? d->mat.gm.N / 2 : d->mat.gm.N) || (reinterpret_cast<uintptr_t>(y) & 3)) {
        set_err("%s: y row stride %lld is shorter than the output row", who, static_cast<long long>(ldy));
        return -1;
    }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    JobSet *js = dense_jobs(d, rows);
    if (!js) return -1;
    GemvOpts o;
    o.yf32 = yf32;
    if (xf32) o.xf = static_cast<const float *>(x);
    return run_gemv(c, d->mat, js->d, js->n, js->mmax, epi, xf32 ? nullptr : static_cast<const uint16_t *>(x), ldx, y,
                    ldy, static_cast<cudaStream_t>(stream), pdl_enabled(), nullptr, nullptr, o);
}
}  // namespace

extern "C" {

int onpu_dense_mv_dev(void *h, const void *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi, void *stream) {
    clear_err();
    return dense_mv_dev_impl("onpu_dense_mv_dev", h, x, false, ldx, rows, y, ldy, epi, stream);
}

int onpu_dense_mv_f32_dev(void *h, const float *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi,
                          void *stream) {
    clear_err();
    return dense_mv_dev_impl("onpu_dense_mv_f32_dev", h, x, true, ldx, rows, y, ldy, epi, stream);
}

int onpu_dense_max_f32_rows(void *h) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    Ctx &c = ctx();
    if (!d || !c.ok) return 0;
    std::lock_guard<std::mutex> lk(g_mu);
    for (int rows = 8; rows >= 1; --rows)
        if (plan_gemv(c, d->mat.gm, 1, 2 * rows, false).lay.xres) return rows;
    return 0;
}

int onpu_dense_mm_dev(void *h, const void *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi, void *stream) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    if (rows <= 0) return 0;
    if (rows > (int64_t{1} << 30)) {
        set_err("onpu_dense_mm_dev: %lld rows is too many", static_cast<long long>(rows));
        return -1;
    }
    if (epi < kEpiF32 || epi > kEpiSwiGLU || (epi == kEpiSwiGLU && !d->gateup)) {
        set_err("onpu_dense_mm_dev: bad epilogue %d for this matrix", epi);
        return -1;
    }
    if (d->geo.ok && d->geo.K != d->mat.gm.K) {
        set_err("onpu_dense_mm_dev: K must be a multiple of 32");
        return -1;
    }
    const int64_t K = d->mat.gm.K, N = d->mat.gm.N;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx & 7) || ldx < K) {
        set_err("onpu_dense_mm_dev: x rows must be 16-byte aligned with ldx %% 8 == 0 and ldx >= K");
        return -1;
    }
    if (ldy < (epi == kEpiSwiGLU ? N / 2 : N) || (reinterpret_cast<uintptr_t>(y) & 3)) {
        set_err("onpu_dense_mm_dev: y row stride %lld is shorter than the output row", static_cast<long long>(ldy));
        return -1;
    }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    if (!grow(c.d_xh, c.xh_cap, rows * K) || !grow(c.d_ts, c.ts_cap, rows)) return -1;
    auto s = static_cast<cudaStream_t>(stream);
    ONPU_CUDA(x_to_f16_launch(static_cast<const uint16_t *>(x), ldx, static_cast<int>(rows), static_cast<int>(K), c.d_xh,
                              c.d_ts, s),
              -1);
    DqGemmParams p{};
    p.w = d->mat.d_w;
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.row_groups = d->mat.gm.row_groups;
    p.chunks = d->mat.gm.chunks;
    p.M = static_cast<int>(rows);
    p.y = y;
    p.ldy = ldy;
    p.row_map = epi == kEpiSwiGLU ? nullptr : d->mat.d_row_map;
    p.tscale = c.d_ts;
    p.err = c.d_err;
    p.unpk[0] = 0x000F000Fu;
    p.unpk[1] = 0x00F000F0u;
    p.unpk[2] = 0x64006400u;
    ONPU_CUDA(dqgemm_launch(d->mat.gm.fmt, epi, c.d_xh, p, s), -1);
    ++c.calls;
    return 0;
}

int onpu_route_dev(const void *h, int64_t ldh, int64_t T, const void *wr, int64_t E, int64_t H, int k, int norm,
                   int32_t *ids, float *w, float *logits, void *stream) {
    clear_err();
    if (T <= 0) return 0;
    if (k < 1 || k > 16 || E < k || E > 256) {
        set_err("onpu_route_dev: need 1 <= k <= 16 and k <= E <= 256 (k %d, E %lld)", k, static_cast<long long>(E));
        return -1;
    }
    if (H <= 0 || H % 8 || ldh < H || ldh % 8 || (reinterpret_cast<uintptr_t>(h) & 15) ||
        (reinterpret_cast<uintptr_t>(wr) & 15)) {
        set_err("onpu_route_dev: h and Wr rows must be 16-byte aligned bf16 with H %% 8 == 0 and ldh >= H, ldh %% 8 == 0");
        return -1;
    }
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return -1;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!grow(c.d_rcnt, c.rcnt_cap, route_counter_slots(T), true) || (!logits && !grow(c.d_rlg, c.rlg_cap, T * E)))
        return -1;
    ONPU_CUDA(route_launch(static_cast<const uint16_t *>(h), ldh, T, static_cast<const uint16_t *>(wr),
                           static_cast<int>(E), static_cast<int>(H), k, norm, ids, w, logits ? logits : c.d_rlg,
                           c.d_rcnt, static_cast<cudaStream_t>(stream)),
              -1);
    return 0;
}

void *onpu_bank_new_int4(int64_t N, int64_t K, int64_t E, int gateup) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    if (N <= 0 || K <= 0 || K % 32 || E <= 0) {
        set_err("onpu_bank_new_int4: need N > 0, K %% 32 == 0, E > 0");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    auto *b = new BankH;
    b->fmt = kFmtQ4F16;
    b->owns_buf = false;
    b->geo.N = N;                 // no stream-order geometry: the weights arrive as int4 + fp16 scales
    b->geo.K = K;
    if (!alloc_mat(b->mat, N, K, kFmtQ4F16, E) || (gateup && !set_gateup_interleave(b->mat))) {
        if (gateup) set_err("onpu_bank_new_int4: gate/up rows need N %% 2 == 0 and N/2 %% 8 == 0");
        delete b;
        return nullptr;
    }
    return b;
}

int onpu_bank_load_int4(void *h, const uint8_t *qk, const uint16_t *scales, int on_device, void *stream) {
    clear_err();
    auto *b = static_cast<BankH *>(h);
    if (b->fmt != kFmtQ4F16 || b->h_buf) {
        set_err("onpu_bank_load_int4: bank was not created by onpu_bank_new_int4");
        return -1;
    }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    const int64_t N = b->mat.gm.N, K = b->mat.gm.K, E = b->mat.E;
    const int64_t qb = N * K / 2, sb = N * (K / 32);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c.stream;
    uint8_t *tq = nullptr;
    uint16_t *ts = nullptr;
    if (!on_device) {
        ONPU_CUDA(cudaMalloc(&tq, static_cast<size_t>(qb)), -1);
        ONPU_CUDA(cudaMalloc(&ts, static_cast<size_t>(sb) * 2), -1);
    }
    cudaError_t e = cudaSuccess;
    for (int64_t x = 0; x < E && e == cudaSuccess; ++x) {
        const uint8_t *sq = qk + x * qb;
        const uint16_t *ss = scales + x * sb;
        if (!on_device) {
            e = cudaMemcpyAsync(tq, sq, static_cast<size_t>(qb), cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess) e = cudaMemcpyAsync(ts, ss, static_cast<size_t>(sb) * 2, cudaMemcpyHostToDevice, s);
            sq = tq;
            ss = ts;
        }
        RepackParams p{};
        p.src_kind = kSrcInt4K;
        p.src = sq;
        p.scales = ss;
        p.src_row = b->mat.d_row_map;
        p.N = N;
        p.K = K;
        p.fmt = kFmtQ4F16;
        p.dst = b->mat.d_w + x * b->mat.gm.bytes;
        if (e == cudaSuccess) e = repack_launch(p, s);
        if (e == cudaSuccess && !on_device) e = cudaStreamSynchronize(s);   // the staging buffers are reused
    }
    if (e == cudaSuccess && (!on_device || !stream)) e = cudaStreamSynchronize(s);
    if (tq) cudaFree(tq);
    if (ts) cudaFree(ts);
    if (e != cudaSuccess) {
        set_err("onpu_bank_load_int4: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

void *onpu_ffn_new_int4(int64_t Ng, int64_t Kg, int64_t Nd, int64_t Kd, int64_t E) {
    clear_err();
    if (Kd * 2 != Ng) {
        set_err("onpu_ffn_new_int4: down K (%lld) must be gate_up N / 2 (%lld)", static_cast<long long>(Kd),
                static_cast<long long>(Ng / 2));
        return nullptr;
    }
    auto *gu = static_cast<BankH *>(onpu_bank_new_int4(Ng, Kg, E, 1));
    if (!gu) return nullptr;
    auto *dn = static_cast<BankH *>(onpu_bank_new_int4(Nd, Kd, E, 0));
    if (!dn) {
        delete gu;
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    auto *f = new FfnH;
    f->gu = gu;
    f->dn = dn;
    f->fused = true;
    return f;
}

namespace {
// e0 >= 0: expert parallelism, the FFN holds experts e0 .. e0 + E - 1 and the other ids are
// skipped (their slots contribute nothing to y)
// route: the router runs first, in the same stream, writing ids / w and building the job lists
// in its last CTA (one launch fewer than routing and expert_jobs_launch separately)
struct RouteSpec {
    const uint16_t *wr;
    int H, norm;
};

// Whether a layer's expert FFN runs as one persistent launch (moe_ffn.cu) instead of gate/up,
// down and combine launches: both banks in one format and the kernel's layout resident. Measured
// on a B200 at config 4's shapes (48 layers, CUDA graph): 35.4 -> 29.4 us a layer at T = 1,
// 98.8 -> 88.9 at T = 16, 144.7 -> 136.0 at T = 64.
bool moe_fused_path(Ctx &c, const GpuMat &gu, const GpuMat &dn, int per_job) {
    if (c.moe_fused == 0 || gu.gm.fmt != dn.gm.fmt) return false;
    const int smem = moe_ffn_fused_smem(gu.gm.fmt, per_job, static_cast<int>(gu.gm.K), 2 * per_job,
                                        static_cast<int>(dn.gm.K), nullptr, nullptr, nullptr);
    if (smem > 227 * 1024 || moe_ffn_fused_ctas_per_sm(gu.gm.fmt, smem) < 1) return false;
    return grow(c.d_ffnbar, c.ffnbar_cap, 4, true);
}

int moe_ffn_dev_impl(void *ffn, const void *x, int64_t ldx, int64_t T, const int32_t *ids, const float *w, int k,
                     int64_t e0, float *y, int64_t ldy, void *stream, const RouteSpec *route = nullptr) {
    auto *f = static_cast<FfnH *>(ffn);
    if (T <= 0) return 0;
    if (!f || !f->fused || k < 1) {
        set_err("onpu_moe_ffn_dev: needs an FFN handle with interleaved gate/up (onpu_ffn_new_int4) and k >= 1");
        return -1;
    }
    BankH *gu = f->gu, *dn = f->dn;
    const int64_t Kg = gu->mat.gm.K, Kd = dn->mat.gm.K, Nd = dn->mat.gm.N, TK = T * k, E = gu->mat.E;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx & 7) || ldx < Kg) {
        set_err("onpu_moe_ffn_dev: x rows must be 16-byte aligned with ldx %% 8 == 0 and ldx >= K");
        return -1;
    }
    if (ldy < Nd || (reinterpret_cast<uintptr_t>(y) & 3)) {
        set_err("onpu_moe_ffn_dev: y row stride %lld is shorter than the output row", static_cast<long long>(ldy));
        return -1;
    }
    if (E > kMaxJobExperts || dn->mat.E != E || TK > (int64_t{1} << 30)) {
        set_err("onpu_moe_ffn_dev: at most %d experts (the same in both banks) and 2^30 routed slots", kMaxJobExperts);
        return -1;
    }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    auto s = static_cast<cudaStream_t>(stream);
    // job lists are built on the device from the routed ids: no host round trip, capturable.
    // Tokens per job: the most (<= 8) for which gate_up's bf16 rows and down's fp32 activations
    // (two fp16 rows per token) both stay resident in shared memory (one staging per job)
    int per_job = 8;
    while (per_job > 1 && !(gemv_resident(per_job, Kg) && gemv_resident(2 * per_job, Kd))) per_job /= 2;
    if (!gemv_resident(per_job, Kg) || !gemv_resident(2 * per_job, Kd)) {
        set_err("onpu_moe_ffn_dev: K = %lld / %lld is too long for resident activation rows",
                static_cast<long long>(Kg), static_cast<long long>(Kd));
        return -1;
    }
    const int64_t njmax = std::min(E, TK) + TK / per_job;
    if (!grow(c.d_jobs, c.jobs_cap, 2 * njmax) || !grow(c.d_order, c.order_cap, TK) ||
        !grow(c.d_njobs, c.njobs_cap, 1) || !grow(c.d_af, c.af_cap, TK * Kd) || !grow(c.d_o, c.o_cap, TK * Nd))
        return -1;
    ExpertJobsParams jp{};
    jp.ids = ids;
    jp.TK = TK;
    jp.k = k;
    jp.E = static_cast<int>(E);
    jp.per_job = per_job;
    jp.w0 = gu->mat.d_w;
    jp.bytes0 = gu->mat.gm.bytes;
    jp.w1 = dn->mat.d_w;
    jp.bytes1 = dn->mat.gm.bytes;
    jp.jobs0 = c.d_jobs;
    jp.jobs1 = c.d_jobs + njmax;
    jp.njobs = c.d_njobs;
    jp.order = c.d_order;
    jp.err = c.d_err;
    jp.id_base = e0 >= 0 ? static_cast<int>(e0) : 0;
    jp.skip_foreign = e0 >= 0 ? 1 : 0;
    if (route) {
        if (!grow(c.d_rcnt, c.rcnt_cap, route_counter_slots(T), true) || !grow(c.d_rlg, c.rlg_cap, T * E)) return -1;
        ONPU_CUDA(route_launch(static_cast<const uint16_t *>(x), ldx, T, route->wr, static_cast<int>(E), route->H, k,
                               route->norm, const_cast<int32_t *>(ids), const_cast<float *>(w), c.d_rlg, c.d_rcnt, s,
                               &jp),
                  -1);
    } else {
        ONPU_CUDA(expert_jobs_launch(jp, s), -1);
    }
    if (moe_fused_path(c, gu->mat, dn->mat, per_job)) {
        // the expert FFN in one persistent launch (moe_ffn.cu) over the same job lists
        MoeFfnFused fp{};
        fp.fmt = gu->mat.gm.fmt;
        fp.jobs_gu = jp.jobs0;
        fp.jobs_dn = jp.jobs1;
        fp.njobs = c.d_njobs;
        fp.rg_gu = gu->mat.gm.row_groups;
        fp.ch_gu = gu->mat.gm.chunks;
        fp.N_gu = static_cast<int>(gu->mat.gm.N);
        fp.K_gu = static_cast<int>(Kg);
        fp.rg_dn = dn->mat.gm.row_groups;
        fp.ch_dn = dn->mat.gm.chunks;
        fp.N_dn = static_cast<int>(Nd);
        fp.K_dn = static_cast<int>(Kd);
        fp.x = static_cast<const uint16_t *>(x);
        fp.ldx = ldx;
        fp.af = c.d_af;
        fp.o = c.d_o;
        fp.ids = ids;
        fp.w = w;
        fp.T = T;
        fp.k = k;
        fp.id_lo = e0 >= 0 ? static_cast<int>(e0) : 0;      // expert parallelism: this rank's experts
        fp.id_hi = static_cast<int>(fp.id_lo + E);
        fp.y = y;
        fp.ldy = ldy;
        fp.bar = c.d_ffnbar;
        fp.err = c.d_err;
        fp.mslots_gu = per_job;
        fp.mslots_dn = 2 * per_job;
        const int smem = moe_ffn_fused_smem(fp.fmt, fp.mslots_gu, fp.K_gu, fp.mslots_dn, fp.K_dn, &fp.off_bar,
                                            &fp.xstride_gu, &fp.xstride_dn);
        fp.workers = c.nsm * moe_ffn_fused_ctas_per_sm(fp.fmt, smem);
        fp.mul[0] = 1u << 28;
        fp.mul[1] = 1u << 24;
        fp.mul[2] = 1u << 20;
        fp.mul[3] = 1u << 16;
        fp.unpk[0] = 0x000F000Fu;
        fp.unpk[1] = 0x00F000F0u;
        fp.unpk[2] = 0x64006400u;
        ONPU_CUDA(moe_ffn_fused_launch(fp, smem, s), -1);
        return 0;
    }
    const int mmax = static_cast<int>(std::min<int64_t>(T, per_job));
    // an expert sees each token at most once (the k experts of a token are distinct); the down
    // projection's jobs hold the same slots, so both lists share the bound. The activation between
    // the projections stays fp32 (SwiGLU epilogue -> fp32, staged by down as two fp16 halves)
    GemvOpts og, od;
    og.yf32 = true;
    od.xf = c.d_af;
    if (run_gemv(c, gu->mat, jp.jobs0, static_cast<int>(njmax), mmax, kEpiSwiGLU, static_cast<const uint16_t *>(x), ldx,
                 c.d_af, Kd, s, true, c.d_njobs, nullptr, og))
        return -1;
    if (run_gemv(c, dn->mat, jp.jobs1, static_cast<int>(njmax), mmax, kEpiF32, nullptr, Kd, c.d_o, Nd, s, true,
                 c.d_njobs, nullptr, od))
        return -1;
    if (e0 >= 0)
        ONPU_CUDA(moe_combine_launch(c.d_o, Nd, T, k, Nd, ids, w, nullptr, y, ldy, s, static_cast<int>(e0),
                                     static_cast<int>(e0 + E)),
                  -1);
    else
        ONPU_CUDA(moe_combine_launch(c.d_o, Nd, T, k, Nd, ids, w, nullptr, y, ldy, s), -1);
    return 0;
}
}  // namespace

int onpu_moe_ffn_dev(void *ffn, const void *x, int64_t ldx, int64_t T, const int32_t *ids, const float *w, int k,
                     float *y, int64_t ldy, void *stream) {
    clear_err();
    return moe_ffn_dev_impl(ffn, x, ldx, T, ids, w, k, -1, y, ldy, stream);
}

int onpu_moe_layer_dev(void *ffn, const void *wr, const void *x, int64_t ldx, int64_t T, int k, int norm, int32_t *ids,
                       float *w, float *y, int64_t ldy, void *stream) {
    clear_err();
    auto *f = static_cast<FfnH *>(ffn);
    if (T <= 0) return 0;
    if (!f || !f->gu) {
        set_err("onpu_moe_layer_dev: no FFN handle");
        return -1;
    }
    const int64_t E = f->gu->mat.E, H = f->gu->mat.gm.K;
    if (k < 1 || k > kMaxRouteK || E < k || E > kMaxRouteExperts || H % 8 || (reinterpret_cast<uintptr_t>(wr) & 15)) {
        set_err("onpu_moe_layer_dev: the router needs 1 <= k <= %d, k <= E <= %d, a 16-byte aligned bf16 [E][H] "
                "matrix", kMaxRouteK, kMaxRouteExperts);
        return -1;
    }
    const RouteSpec rs{static_cast<const uint16_t *>(wr), static_cast<int>(H), norm};
    return moe_ffn_dev_impl(ffn, x, ldx, T, ids, w, k, -1, y, ldy, stream, &rs);
}

int onpu_moe_set_fused(int mode) {
    clear_err();
    if (mode < 0 || mode > 1) {
        set_err("onpu_moe_set_fused: mode %d is not 0 or 1", mode);
        return -1;
    }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    const int prev = c.moe_fused;
    c.moe_fused = mode;
    return prev;
}

int onpu_moe_ffn_dev_ep(void *ffn, const void *x, int64_t ldx, int64_t T, const int32_t *ids, const float *w, int k,
                        int64_t e0, float *y, int64_t ldy, void *stream) {
    clear_err();
    if (e0 < 0 || e0 > INT32_MAX / 2) {
        set_err("onpu_moe_ffn_dev_ep: first expert id %lld out of range", static_cast<long long>(e0));
        return -1;
    }
    return moe_ffn_dev_impl(ffn, x, ldx, T, ids, w, k, e0, y, ldy, stream);
}

int onpu_dense_unpack_dev(void *h, uint8_t *q, uint16_t *scales, uint16_t *mins, void *stream) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    ONPU_CUDA(unpack_gpu_launch(d->mat.d_w, d->mat.gm.N, d->mat.gm.K, d->mat.gm.fmt, q, scales, mins,
                                static_cast<cudaStream_t>(stream)),
              -1);
    return 0;
}

}  // extern "C"

// ------------------------------------------------------------------ no-allocation entry point
// onpu_dense_mv_dev_noalloc: onpu_dense_mv_dev whose split-row scratch (partial-sum slots, ready
// flags) and GEMV descriptors live in one file-scope __device__ array instead of buffers that the
// library grows with cudaMalloc on first use. For callers that cannot let a library allocate in
// their decode loop: engines that hand all free HBM to their own pool at start-up (a serving
// engine's KV-cache reservation leaves nothing for a lazy cudaMalloc, which then fails mid-run),
// and callers with a fixed, pre-planned device footprint. The regular path's first call for a new
// row count allocates descriptors, and its scratch growth synchronises the whole device first
// (grow() above), a stall such callers cannot take inside a step either.
//
// Limits: rows <= kStaticMaxRows (descriptors for kStaticMaxRows / 16 jobs), at most
// kStaticWorkers CTAs (the launch uses min(chosen, kStaticWorkers)). The array is
// kStaticWorkers * 4 KB + 4 KB of flags + descriptors (~4.1 MB), device memory the driver
// reserves when this translation unit's device image is loaded.
//
// Every call on a device shares the one array: calls must be ordered on one stream (overlapping
// calls race on the flags, slots and descriptors). Each call clears the flags it uses on its
// stream before the launch, so a call never reads state left by an earlier one.
namespace {

constexpr int kStaticWorkers = 1024;
constexpr int kStaticSlotFloats = 1024;                       // gemv_part_floats_per_worker
constexpr int kStaticMaxRows = 256;
constexpr int kStaticMaxJobs = kStaticMaxRows / kMaxTokensPerJob;
constexpr size_t kStaticPartBytes = size_t(kStaticWorkers) * kStaticSlotFloats * sizeof(float);
constexpr size_t kStaticFlagBytes = size_t(kStaticWorkers) * sizeof(unsigned);
constexpr size_t kStaticJobBytes = size_t(kStaticMaxJobs) * sizeof(GemvJob);
constexpr size_t kStaticBytes = kStaticPartBytes + kStaticFlagBytes + kStaticJobBytes;
static_assert(kStaticPartBytes % 256 == 0 && kStaticFlagBytes % 256 == 0, "scratch sections stay aligned");

__device__ __align__(256) unsigned char g_static_scratch[kStaticBytes];

constexpr int kMaxDevices = 64;
unsigned char *g_static_ptr[kMaxDevices] = {};

// once per device, with that device current; the first call on a device does it, so on each
// device that first call should come before any stream capture. Caller holds g_mu.
unsigned char *static_scratch(int dev) {
    if (dev < 0 || dev >= kMaxDevices) {
        set_err("onpu_dense_mv_dev_noalloc: device ordinal %d out of range", dev);
        return nullptr;
    }
    if (g_static_ptr[dev]) return g_static_ptr[dev];
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
        set_err("onpu_dense_mv_dev_noalloc: cudaGetSymbolAddress of the static scratch failed: %s",
                cudaGetErrorString(e));
        return nullptr;
    }
    e = cudaMemset(static_cast<unsigned char *>(ptr) + kStaticPartBytes, 0, kStaticFlagBytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        set_err("onpu_dense_mv_dev_noalloc: clearing the static scratch failed: %s", cudaGetErrorString(e));
        return nullptr;
    }
    g_static_ptr[dev] = static_cast<unsigned char *>(ptr);
    return g_static_ptr[dev];
}

}  // namespace

extern "C" {

int onpu_dense_mv_dev_noalloc(void *h, const void *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi,
                              void *stream) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    if (!d) {
        set_err("onpu_dense_mv_dev_noalloc: null matrix handle");
        return -1;
    }
    if (rows <= 0) return 0;
    if (rows > kStaticMaxRows) {
        set_err("onpu_dense_mv_dev_noalloc: %lld rows exceed the static scratch limit of %d rows per call",
                static_cast<long long>(rows), kStaticMaxRows);
        return -1;
    }
    const bool yf32 = epi == ONPU_EPI_SWIGLU_F32;
    if (yf32) epi = kEpiSwiGLU;
    if (epi < kEpiF32 || epi > kEpiPairSum || (epi == kEpiSwiGLU && !d->gateup) ||
        (epi == kEpiPairSum && !d->residual)) {
        set_err("onpu_dense_mv_dev_noalloc: bad epilogue %d for this matrix", yf32 ? ONPU_EPI_SWIGLU_F32 : epi);
        return -1;
    }
    if (d->geo.ok && d->geo.K != d->mat.gm.K) {
        set_err("onpu_dense_mv_dev_noalloc: K must be a multiple of 32");
        return -1;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx & 7) || ldx < d->mat.gm.K) {
        set_err("onpu_dense_mv_dev_noalloc: x rows must be 16-byte aligned with ldx %% 8 == 0 and ldx >= K");
        return -1;
    }
    if (ldy < (epi >= kEpiSwiGLU ? d->mat.gm.N / 2 : d->mat.gm.N) || (reinterpret_cast<uintptr_t>(y) & 3)) {
        set_err("onpu_dense_mv_dev_noalloc: y row stride %lld is shorter than the output row",
                static_cast<long long>(ldy));
        return -1;
    }
    if (gemv_part_floats_per_worker(2) > kStaticSlotFloats) {
        set_err("onpu_dense_mv_dev_noalloc: GEMV slot size exceeds the static scratch layout");
        return -1;
    }
    // the handle exists, so the library context (device, stream, status word) is already set up
    Ctx &c = ctx();
    int dev = -1;
    ONPU_CUDA(cudaGetDevice(&dev), -1);
    if (dev != c.device) {
        set_err("onpu_dense_mv_dev_noalloc: current device %d is not the library's device %d", dev, c.device);
        return -1;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    unsigned char *base = static_scratch(dev);
    if (!base) return -1;
    float *part = reinterpret_cast<float *>(base);
    unsigned *flags = reinterpret_cast<unsigned *>(base + kStaticPartBytes);
    GemvJob *d_jobs = reinterpret_cast<GemvJob *>(base + kStaticPartBytes + kStaticFlagBytes);

    // the same launch plan (grid, activation window) as onpu_dense_mv_dev for this row count, so
    // both entries add the split rows in the same order and agree bit for bit
    const int njobs = static_cast<int>((rows + kMaxTokensPerJob - 1) / kMaxTokensPerJob);
    const int mmax = static_cast<int>(std::min<int64_t>(rows, kMaxTokensPerJob));
    const int T = njobs * d->mat.gm.row_groups * d->mat.gm.chunks;
    if (T == 0) return 0;
    const GemvPlan pl = plan_gemv(c, d->mat.gm, njobs, mmax, false);
    const GemvLayout &lay = pl.lay;
    const int W = pl.workers;
    if (W > kStaticWorkers) {
        set_err("onpu_dense_mv_dev_noalloc: %d CTAs exceed the static scratch's %d", W, kStaticWorkers);
        return -1;
    }
    auto s = static_cast<cudaStream_t>(stream);
    // descriptors written and the flags this launch uses cleared by a small kernel on the caller's
    // stream: every argument is passed by value, nothing is read from host memory
    ONPU_CUDA(dense_jobs_launch(d_jobs, d->mat.d_w, static_cast<int>(rows), flags, W, s), -1);

    GemvParams p{};
    p.jobs = d_jobs;
    p.njobs = njobs;
    p.N = static_cast<int>(d->mat.gm.N);
    p.K = static_cast<int>(d->mat.gm.K);
    p.row_groups = d->mat.gm.row_groups;
    p.chunks = d->mat.gm.chunks;
    p.total_chunks = T;
    p.workers = W;
    p.x = static_cast<const uint16_t *>(x);
    p.ldx = ldx;
    p.y = y;
    p.ldy = ldy;
    p.row_map = epi == kEpiSwiGLU || epi == kEpiPairSum ? nullptr : d->mat.d_row_map;
    p.part = part;
    p.counters = flags;
    p.err = c.d_err;
    p.jobs_ready = 1;
    p.mul[0] = 1u << 28;
    p.mul[1] = 1u << 24;
    p.mul[2] = 1u << 20;
    p.mul[3] = 1u << 16;
    p.unpk[0] = 0x000F000Fu;
    p.unpk[1] = 0x00F000F0u;
    p.unpk[2] = 0x64006400u;
    p.xslots = lay.xslots;
    p.xres = lay.xres;
    p.xstride = lay.xstride;
    p.ctab_off = lay.ctab_off;
    p.off_bar = lay.off_bar;
    p.wchunks = lay.wchunks;
    p.kwin = pl.kwin ? 1 : 0;
    p.yf32 = yf32 ? 1 : 0;
    ONPU_CUDA(gemv_launch(d->mat.gm.fmt, pl.ntiles, epi, p, lay.smem, s, false), -1);
    ++c.calls;
    return 0;
}

}  // extern "C"

// ------------------------------------------------------------------ GEMV chains
// A decode step's dense GEMVs recorded once on fixed device buffers and run as one persistent
// launch (chain.cu). Links keep their order; a link that reads or overwrites memory an earlier
// link writes (or reads, for an overwrite) waits on the device until every CTA has finished the
// latest such link. Runs of one chain must be ordered on one stream (its counters and partial
// slots are shared by its runs).
namespace {

struct ChainH {
    std::vector<ChainOp> ops;
    std::vector<uintptr_t> xr, yr;    // per link: [x0, x1), [y0, y1) byte ranges
    int fmt = -1, ntiles = 1;
    bool ready = false;
    ChainOp *d_ops = nullptr;
    float *d_part = nullptr;
    unsigned *d_flags = nullptr, *d_done = nullptr, *d_rgcnt = nullptr;
    int W = 0, smem = 0;
    ChainLayout lay{};
    unsigned long long *trace = nullptr;   // caller's device buffer, or null
    void release() {
        if (d_ops) cudaFree(d_ops);
        if (d_part) cudaFree(d_part);
        if (d_flags) cudaFree(d_flags);
        if (d_done) cudaFree(d_done);
        if (d_rgcnt) cudaFree(d_rgcnt);
        d_ops = nullptr;
        d_part = nullptr;
        d_flags = d_done = d_rgcnt = nullptr;
        ready = false;
    }
    ChainH();
    ~ChainH();
};

std::set<ChainH *> g_chains;           // live chains (guarded by g_mu)
ChainH::ChainH() { g_chains.insert(this); }
ChainH::~ChainH() {
    g_chains.erase(this);
    release();
}

// a timed-out wait can leave a chain's counters or flags raised: clear them (device is idle here)
void reset_chains_after_error() {
    for (ChainH *ch : g_chains) {
        if (ch->d_flags) cudaMemset(ch->d_flags, 0, sizeof(unsigned) * kChainRing * ch->W * 2);
        if (ch->d_rgcnt) cudaMemset(ch->d_rgcnt, 0, sizeof(unsigned) * ch->ops.size() * ch->W);
        if (ch->d_done) cudaMemset(ch->d_done, 0, sizeof(unsigned) * (ch->ops.size() + 1));
    }
}

bool overlap(uintptr_t a0, uintptr_t a1, uintptr_t b0, uintptr_t b1) { return a0 < b1 && b0 < a1; }

int chain_prepare(Ctx &c, ChainH *ch) {
    if (ch->ready) return 0;
    if (ch->ops.empty()) {
        set_err("onpu_chain: the chain has no links");
        return -1;
    }
    cudaDeviceSynchronize();              // a previous run may still use the old buffers
    ch->release();
    int64_t xregion = 0;
    for (auto &op : ch->ops) {
        const int64_t b = chain_xregion_bytes(op.m, op.K, ch->ntiles, &op.xstride, &op.ctab_off);
        xregion = std::max(xregion, b);
    }
    ChainLayout lay{};
    int occ = 0;
    if (!choose_chain_layout(ch->fmt, ch->ntiles, xregion, lay, occ)) {
        set_err("onpu_chain: the largest link's activations (%lld bytes) do not fit in shared memory",
                static_cast<long long>(xregion));
        return -1;
    }
    ch->W = c.nsm * occ;
    ch->smem = lay.smem;
    ch->lay = lay;
    const size_t nops = ch->ops.size();
    const size_t part = static_cast<size_t>(kChainRing) * ch->W * 2 * chain_part_floats_per_slot();
    const size_t nflags = static_cast<size_t>(kChainRing) * ch->W * 2, nrg = nops * ch->W;
    ONPU_CUDA(cudaMalloc(&ch->d_ops, sizeof(ChainOp) * nops), -1);
    ONPU_CUDA(cudaMalloc(&ch->d_part, sizeof(float) * part), -1);
    ONPU_CUDA(cudaMalloc(&ch->d_flags, sizeof(unsigned) * nflags), -1);
    ONPU_CUDA(cudaMalloc(&ch->d_rgcnt, sizeof(unsigned) * nrg), -1);
    ONPU_CUDA(cudaMalloc(&ch->d_done, sizeof(unsigned) * (nops + 1)), -1);
    ONPU_CUDA(cudaMemset(ch->d_flags, 0, sizeof(unsigned) * nflags), -1);
    ONPU_CUDA(cudaMemset(ch->d_rgcnt, 0, sizeof(unsigned) * nrg), -1);
    ONPU_CUDA(cudaMemset(ch->d_done, 0, sizeof(unsigned) * (nops + 1)), -1);
    ONPU_CUDA(cudaMemcpy(ch->d_ops, ch->ops.data(), sizeof(ChainOp) * nops, cudaMemcpyHostToDevice), -1);
    ch->ready = true;
    return 0;
}

}  // namespace

extern "C" {

void *onpu_chain_new(void) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    return new ChainH();
}

int onpu_chain_add(void *chain, void *h, const void *x, int64_t ldx, int64_t rows, void *y, int64_t ldy, int epi,
                   int dep) {
    clear_err();
    auto *ch = static_cast<ChainH *>(chain);
    auto *d = static_cast<DenseH *>(h);
    if (!ch || !d) {
        set_err("onpu_chain_add: null handle");
        return -1;
    }
    if (rows < 1 || rows > kChainMaxRows) {
        set_err("onpu_chain_add: rows must be 1..%d (got %lld)", kChainMaxRows, static_cast<long long>(rows));
        return -1;
    }
    if (epi < kEpiF32 || epi > kEpiSwiGLU || (epi == kEpiSwiGLU && !d->gateup)) {
        set_err("onpu_chain_add: bad epilogue %d for this matrix", epi);
        return -1;
    }
    if (d->geo.ok && d->geo.K != d->mat.gm.K) {
        set_err("onpu_chain_add: K must be a multiple of 32");
        return -1;
    }
    const int64_t K = d->mat.gm.K, ncol = epi == kEpiSwiGLU ? d->mat.gm.N / 2 : d->mat.gm.N;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx & 7) || ldx < K) {
        set_err("onpu_chain_add: x rows must be 16-byte aligned with ldx %% 8 == 0 and ldx >= K");
        return -1;
    }
    if (ldy < ncol || (reinterpret_cast<uintptr_t>(y) & 3)) {
        set_err("onpu_chain_add: y row stride %lld is shorter than the output row", static_cast<long long>(ldy));
        return -1;
    }
    if (ch->fmt >= 0 && ch->fmt != d->mat.gm.fmt) {
        set_err("onpu_chain_add: every link of a chain must use the same weight format");
        return -1;
    }
    const int idx = static_cast<int>(ch->ops.size());
    if (dep >= idx) {
        set_err("onpu_chain_add: dep %d does not name an earlier link", dep);
        return -1;
    }
    const int esz = epi == kEpiF32 ? 4 : 2;
    const uintptr_t x0 = reinterpret_cast<uintptr_t>(x), x1 = x0 + ((rows - 1) * ldx + K) * 2;
    const uintptr_t y0 = reinterpret_cast<uintptr_t>(y), y1 = y0 + ((rows - 1) * ldy + ncol) * esz;
    int d_auto = -1;
    for (int i = idx - 1; i >= 0 && d_auto < 0; --i)
        if (overlap(x0, x1, ch->yr[2 * i], ch->yr[2 * i + 1]) || overlap(y0, y1, ch->xr[2 * i], ch->xr[2 * i + 1]) ||
            overlap(y0, y1, ch->yr[2 * i], ch->yr[2 * i + 1]))
            d_auto = i;
    ChainOp op{};
    op.w = d->mat.d_w;
    op.x = static_cast<const uint16_t *>(x);
    op.y = y;
    op.row_map = epi == kEpiSwiGLU ? nullptr : d->mat.d_row_map;
    op.ldx = ldx;
    op.ldy = ldy;
    op.N = static_cast<int>(d->mat.gm.N);
    op.K = static_cast<int>(K);
    op.row_groups = d->mat.gm.row_groups;
    op.chunks = d->mat.gm.chunks;
    op.epi = epi;
    op.dep = std::max(dep, d_auto);
    op.m = static_cast<int>(rows);
    ch->ops.push_back(op);
    ch->xr.push_back(x0);
    ch->xr.push_back(x1);
    ch->yr.push_back(y0);
    ch->yr.push_back(y1);
    ch->fmt = d->mat.gm.fmt;
    if (rows > 8) ch->ntiles = 2;
    ch->ready = false;
    return idx;
}

int onpu_chain_info(void *chain, int64_t *out4) {
    auto *ch = static_cast<ChainH *>(chain);
    out4[0] = static_cast<int64_t>(ch->ops.size());
    out4[1] = ch->W;
    out4[2] = ch->smem;
    out4[3] = ch->ntiles;
    return 0;
}

int onpu_chain_link_dep(void *chain, int link) {
    auto *ch = static_cast<ChainH *>(chain);
    if (link < 0 || link >= static_cast<int>(ch->ops.size())) return -2;
    return ch->ops[link].dep;
}

int onpu_chain_prepare(void *chain) {
    clear_err();
    std::lock_guard<std::mutex> lk(g_mu);
    return chain_prepare(ctx(), static_cast<ChainH *>(chain));
}

int onpu_chain_run(void *chain, void *stream) {
    clear_err();
    auto *ch = static_cast<ChainH *>(chain);
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    if (chain_prepare(c, ch)) return -1;
    ChainParams p{};
    p.ops = ch->d_ops;
    p.nops = static_cast<int>(ch->ops.size());
    p.workers = ch->W;
    p.part = ch->d_part;
    p.flags = ch->d_flags;
    p.rgcnt = ch->d_rgcnt;
    p.done = ch->d_done;
    p.err = c.d_err;
    p.mul[0] = 1u << 28;
    p.mul[1] = 1u << 24;
    p.mul[2] = 1u << 20;
    p.mul[3] = 1u << 16;
    p.unpk[0] = 0x000F000Fu;
    p.unpk[1] = 0x00F000F0u;
    p.unpk[2] = 0x64006400u;
    p.ns = ch->lay.ns;
    p.off_x = ch->lay.off_x;
    p.off_comb = ch->lay.off_comb;
    p.off_bar = ch->lay.off_bar;
    p.trace = ch->trace;
    ONPU_CUDA(chain_launch(ch->fmt, ch->ntiles, p, ch->smem, static_cast<cudaStream_t>(stream)), -1);
    ++c.calls;
    return 0;
}

// ---- one-shot all-reduce between the ranks of one node (tensor-parallel decode)
struct CommH {
    int rank = 0, world = 1, device = -1;
    int64_t cap = 0;
    void *buf = nullptr;                        // this rank's buffer
    void *bufs[kCommMaxRanks] = {};             // every rank's buffer, mapped here
    bool mapped[kCommMaxRanks] = {};
    ~CommH() {
        for (int r = 0; r < kCommMaxRanks; ++r)
            if (mapped[r]) cudaIpcCloseMemHandle(bufs[r]);
        if (buf) cudaFree(buf);
    }
};

void *onpu_comm_new(int rank, int world, int64_t cap_floats) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    if (world < 1 || world > kCommMaxRanks || rank < 0 || rank >= world || cap_floats <= 0) {
        set_err("onpu_comm_new: need 1 <= world <= %d, 0 <= rank < world, cap > 0", kCommMaxRanks);
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    auto *h = new CommH;
    h->rank = rank;
    h->world = world;
    h->cap = (cap_floats + 3) / 4 * 4;
    cudaGetDevice(&h->device);
    const int64_t bytes = comm_buffer_bytes(world, h->cap);
    if (cudaMalloc(&h->buf, static_cast<size_t>(bytes)) != cudaSuccess ||
        cudaMemset(h->buf, 0, static_cast<size_t>(bytes)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        set_err("onpu_comm_new: %s", cudaGetErrorString(cudaGetLastError()));
        delete h;
        return nullptr;
    }
    h->bufs[rank] = h->buf;
    return h;
}

int onpu_comm_ipc_handle(void *comm, void *out) {
    clear_err();
    auto *h = static_cast<CommH *>(comm);
    cudaIpcMemHandle_t ih;
    ONPU_CUDA(cudaIpcGetMemHandle(&ih, h->buf), -1);
    std::memcpy(out, &ih, sizeof(ih));
    return static_cast<int>(sizeof(ih));
}

int onpu_comm_open(void *comm, const void *handles) {
    clear_err();
    auto *h = static_cast<CommH *>(comm);
    std::lock_guard<std::mutex> lk(g_mu);
    const auto *hb = static_cast<const unsigned char *>(handles);
    for (int r = 0; r < h->world; ++r) {
        if (r == h->rank || h->mapped[r]) continue;
        cudaIpcMemHandle_t ih;
        std::memcpy(&ih, hb + r * sizeof(ih), sizeof(ih));
        void *ptr = nullptr;
        ONPU_CUDA(cudaIpcOpenMemHandle(&ptr, ih, cudaIpcMemLazyEnablePeerAccess), -1);
        h->bufs[r] = ptr;
        h->mapped[r] = true;
    }
    return 0;
}

}  // extern "C"

namespace {
// onpu_dense_mv_allreduce(_f32)_dev: x bf16, or fp32 (at most 8 rows) when xf32
int mv_allreduce_impl(const char *who, void *h, void *comm, const void *x, bool xf32, int64_t ldx, int64_t rows,
                      float *y, void *y_bf16, void *stream) {
    auto *d = static_cast<DenseH *>(h);
    auto *cm = static_cast<CommH *>(comm);
    if (rows <= 0) return 0;
    if (d->gateup || d->residual || (d->geo.ok && d->geo.K != d->mat.gm.K)) {
        set_err("%s: needs a plain matrix (no gate/up or residual rows, K %% 32 == 0)", who);
        return -1;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx & (xf32 ? 3 : 7)) || ldx < d->mat.gm.K) {
        set_err("%s: x rows must be 16-byte aligned (ldx a multiple of 16 bytes) with ldx >= K", who);
        return -1;
    }
    if (xf32 && rows > 8) {
        set_err("%s: fp32 activations take at most 8 rows per call", who);
        return -1;
    }
    const int64_t n = rows * d->mat.gm.N;
    if (n > cm->cap || (!y && !y_bf16) || (y_bf16 && (reinterpret_cast<uintptr_t>(y_bf16) & 1))) {
        set_err("%s: rows x N = %lld exceeds the all-reduce buffer (%lld) or no output", who,
                static_cast<long long>(n), static_cast<long long>(cm->cap));
        return -1;
    }
    for (int r = 0; r < cm->world; ++r)
        if (!cm->bufs[r]) {
            set_err("%s: rank %d's buffer is not mapped (onpu_comm_open)", who, r);
            return -1;
        }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    JobSet *js = dense_jobs(d, rows);
    if (!js) return -1;
    PeerOut po{};
    for (int r = 0; r < cm->world; ++r) po.bufs[r] = cm->bufs[r];
    po.rank = cm->rank;
    po.world = cm->world;
    po.cap = cm->cap;
    auto s = static_cast<cudaStream_t>(stream);
    po.y_bf16 = y_bf16;
    GemvOpts o;
    if (xf32) o.xf = static_cast<const float *>(x);
    // one launch: the epilogue sends each finished row to every rank, and each CTA then sums every
    // rank's words of the rows it finished into y / y_bf16
    return run_gemv(c, d->mat, js->d, js->n, js->mmax, kEpiPeer, xf32 ? nullptr : static_cast<const uint16_t *>(x),
                    ldx, y, d->mat.gm.N, s, pdl_enabled(), nullptr, &po, o);
}
}  // namespace

extern "C" {

int onpu_dense_mv_allreduce_dev(void *h, void *comm, const void *x, int64_t ldx, int64_t rows, float *y,
                                void *y_bf16, void *stream) {
    clear_err();
    return mv_allreduce_impl("onpu_dense_mv_allreduce_dev", h, comm, x, false, ldx, rows, y, y_bf16, stream);
}

int onpu_dense_mv_allreduce_f32_dev(void *h, void *comm, const float *x, int64_t ldx, int64_t rows, float *y,
                                    void *y_bf16, void *stream) {
    clear_err();
    return mv_allreduce_impl("onpu_dense_mv_allreduce_f32_dev", h, comm, x, true, ldx, rows, y, y_bf16, stream);
}


int onpu_comm_allreduce(void *comm, const float *src, float *dst, void *dst_bf16, int64_t n, void *stream) {
    clear_err();
    auto *h = static_cast<CommH *>(comm);
    if ((!dst && !dst_bf16) || (dst_bf16 && (reinterpret_cast<uintptr_t>(dst_bf16) & 1))) {
        set_err("onpu_comm_allreduce: needs an fp32 and / or an aligned bf16 output");
        return -1;
    }
    if (n > h->cap || n < 0) {
        set_err("onpu_comm_allreduce: %lld floats exceed the buffer's %lld", static_cast<long long>(n),
                static_cast<long long>(h->cap));
        return -1;
    }
    for (int r = 0; r < h->world; ++r)
        if (!h->bufs[r]) {
            set_err("onpu_comm_allreduce: rank %d's buffer is not mapped (onpu_comm_open)", r);
            return -1;
        }
    Ctx &c = ctx();
    ONPU_CUDA(comm_allreduce_launch(h->bufs, h->rank, h->world, h->cap, src, dst, dst_bf16, n, c.d_err, c.peer_wait_ns,
                                    static_cast<cudaStream_t>(stream)),
              -1);
    return 0;
}

int onpu_comm_set_wait(double seconds) {
    clear_err();
    if (!(seconds > 0.0) || seconds > 60.0) {
        set_err("onpu_comm_set_wait: the limit must be in (0, 60] seconds");
        return -1;
    }
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    c.peer_wait_ns = static_cast<uint64_t>(seconds * 1e9);
    return 0;
}

void onpu_comm_free(void *comm) {
    std::lock_guard<std::mutex> lk(g_mu);
    cudaDeviceSynchronize();
    delete static_cast<CommH *>(comm);
}

int onpu_gemv_trace(uint64_t *stamps, int64_t ctas) {
    Ctx &c = ctx();
    std::lock_guard<std::mutex> lk(g_mu);
    c.gemv_trace = reinterpret_cast<unsigned long long *>(stamps);
    c.gemv_trace_ctas = stamps ? ctas : 0;
    return 0;
}

int onpu_chain_trace(void *chain, uint64_t *stamps) {
    auto *ch = static_cast<ChainH *>(chain);
    ch->trace = reinterpret_cast<unsigned long long *>(stamps);
    return 0;
}

void onpu_chain_free(void *chain) {
    std::lock_guard<std::mutex> lk(g_mu);
    delete static_cast<ChainH *>(chain);
}

}  // extern "C"

// ------------------------------------------------------------------ weight blobs (the pack cache)
// A blob is a 64-byte header (magic, layout version, kind, matrix count) and per matrix a 64-byte
// section header (N, K, E, format, flags, payload bytes) followed by the GPU-layout bytes exactly
// as they lie in HBM, padded to 64 bytes. Everything is validated before any device call, so a
// truncated or foreign file is refused with a message instead of being copied.
namespace {
constexpr char kBlobMagic[8] = {'O', 'N', 'P', 'U', 'B', '2', 'G', 'L'};
constexpr uint32_t kBlobDense = 1, kBlobBank = 2, kBlobFfn = 3;
constexpr uint32_t kMatGateUp = 1, kMatResidual = 2;   // gate/up strip interleave; two-pass pairs

struct BlobHead {
    char magic[8];
    uint32_t version, kind, nmats, pad;
    uint8_t rsv[40];
};
struct MatHead {
    int64_t N, K, E;
    int32_t fmt;
    uint32_t flags;
    int64_t bytes;
    uint8_t rsv[24];
};
static_assert(sizeof(BlobHead) == 64 && sizeof(MatHead) == 64, "blob headers are 64 bytes");

int64_t section_bytes(const GpuMat &m) { return static_cast<int64_t>(sizeof(MatHead)) + round_up(m.gm.bytes * m.E, 64); }

// K of a handle made through the reference upload path must be the GPU layout's K
bool exportable(const Geometry &geo, const GpuMat &m, const char *who) {
    if (!m.d_w || (geo.ok && geo.K != m.gm.K)) {
        set_err("%s: only matrices with K %% 32 == 0 and loaded weights can be exported", who);
        return false;
    }
    return true;
}

bool write_section(const GpuMat &m, uint32_t flags, uint8_t *dst) {
    MatHead h{};
    h.N = m.gm.N;
    h.K = m.gm.K;
    h.E = m.E;
    h.fmt = m.gm.fmt;
    h.flags = flags;
    h.bytes = m.gm.bytes * m.E;
    std::memcpy(dst, &h, sizeof h);
    const cudaError_t e = cudaMemcpy(dst + sizeof h, m.d_w, static_cast<size_t>(h.bytes), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        set_err("weight export: %s", cudaGetErrorString(e));
        return false;
    }
    std::memset(dst + sizeof h + h.bytes, 0, static_cast<size_t>(round_up(h.bytes, 64) - h.bytes));
    return true;
}

// Validates the blob header; out: the matrix sections' headers and payload pointers.
bool parse_blob(const void *src, int64_t nbytes, uint32_t kind, uint32_t nmats, MatHead *heads,
                const uint8_t **payloads, const char *who) {
    if (!src || nbytes < static_cast<int64_t>(sizeof(BlobHead))) {
        set_err("%s: blob of %lld bytes is shorter than its header", who, static_cast<long long>(nbytes));
        return false;
    }
    const auto *p = static_cast<const uint8_t *>(src), *end = p + nbytes;
    BlobHead bh;
    std::memcpy(&bh, p, sizeof bh);
    if (std::memcmp(bh.magic, kBlobMagic, sizeof kBlobMagic) != 0) {
        set_err("%s: not a weight blob (bad magic)", who);
        return false;
    }
    if (bh.version != static_cast<uint32_t>(kGpuLayoutVersion)) {
        set_err("%s: blob of layout version %u, this library writes version %d", who, bh.version, kGpuLayoutVersion);
        return false;
    }
    if (bh.kind != kind || bh.nmats != nmats) {
        set_err("%s: blob holds kind %u with %u matrices, expected kind %u with %u", who, bh.kind, bh.nmats, kind,
                nmats);
        return false;
    }
    p += sizeof bh;
    for (uint32_t i = 0; i < nmats; ++i) {
        MatHead h;
        if (end - p < static_cast<int64_t>(sizeof h)) {
            set_err("%s: blob truncated in matrix %u's header", who, i);
            return false;
        }
        std::memcpy(&h, p, sizeof h);
        p += sizeof h;
        if (h.N <= 0 || h.N > (int64_t{1} << 30) || h.K <= 0 || h.K > (int64_t{1} << 30) || h.K % 32 || h.E <= 0 ||
            h.E > (int64_t{1} << 16) || h.fmt < kFmtQ4NX || h.fmt > kFmtQ4F16 || (h.flags & ~(kMatGateUp | kMatResidual))) {
            set_err("%s: matrix %u has an invalid header (N %lld, K %lld, E %lld, format %d, flags %u)", who, i,
                    static_cast<long long>(h.N), static_cast<long long>(h.K), static_cast<long long>(h.E), h.fmt,
                    h.flags);
            return false;
        }
        const GpuMatrix g = make_gpu_matrix(h.N, h.K, h.fmt);
        if (g.bytes > (int64_t{1} << 40) / h.E || h.bytes != g.bytes * h.E) {
            set_err("%s: matrix %u declares %lld payload bytes, its shape needs %lld", who, i,
                    static_cast<long long>(h.bytes), static_cast<long long>(g.bytes * h.E));
            return false;
        }
        if (end - p < round_up(h.bytes, 64)) {
            set_err("%s: blob truncated in matrix %u's weights", who, i);
            return false;
        }
        heads[i] = h;
        payloads[i] = p;
        p += round_up(h.bytes, 64);
    }
    if (p != end) {
        set_err("%s: %lld bytes after the last matrix", who, static_cast<long long>(end - p));
        return false;
    }
    return true;
}

bool load_section(GpuMat &m, const MatHead &h, const uint8_t *payload, const char *who) {
    if (!alloc_mat(m, h.N, h.K, h.fmt, h.E)) return false;
    if ((h.flags & (kMatGateUp | kMatResidual)) && !set_gateup_interleave(m)) {
        set_err("%s: interleaved rows need N %% 2 == 0 and N/2 %% 8 == 0", who);
        return false;
    }
    const cudaError_t e = cudaMemcpy(m.d_w, payload, static_cast<size_t>(h.bytes), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        set_err("%s: %s", who, cudaGetErrorString(e));
        return false;
    }
    return true;
}

int64_t write_blob(uint32_t kind, const GpuMat *const *mats, const uint32_t *flags, int n, void *dst, int64_t cap,
                   const char *who) {
    int64_t total = sizeof(BlobHead);
    for (int i = 0; i < n; ++i) total += section_bytes(*mats[i]);
    if (!dst) return total;
    if (cap < total) {
        set_err("%s: the blob needs %lld bytes, the buffer holds %lld", who, static_cast<long long>(total),
                static_cast<long long>(cap));
        return -1;
    }
    const cudaError_t e = cudaDeviceSynchronize();     // weights loaded on any stream are complete
    if (e != cudaSuccess) {
        set_err("%s: %s", who, cudaGetErrorString(e));
        return -1;
    }
    BlobHead bh{};
    std::memcpy(bh.magic, kBlobMagic, sizeof kBlobMagic);
    bh.version = kGpuLayoutVersion;
    bh.kind = kind;
    bh.nmats = static_cast<uint32_t>(n);
    auto *p = static_cast<uint8_t *>(dst);
    std::memcpy(p, &bh, sizeof bh);
    p += sizeof bh;
    for (int i = 0; i < n; ++i) {
        if (!write_section(*mats[i], flags[i], p)) return -1;
        p += section_bytes(*mats[i]);
    }
    return total;
}

BankH *bank_from_section(const MatHead &h, const uint8_t *payload, const char *who) {
    auto *b = new BankH;
    b->fmt = h.fmt;
    b->owns_buf = false;
    b->geo.N = h.N;
    b->geo.K = h.K;
    if (!load_section(b->mat, h, payload, who)) {
        delete b;
        return nullptr;
    }
    return b;
}
}  // namespace

// ------------------------------------------------------------------ decode attention
namespace {
struct AttnScratch {
    float *part = nullptr;
    int64_t part_cap = 0;
    float *host_in = nullptr;         // staging of host-pointer calls (q, mask, sinks, K, V)
    int64_t host_cap = 0;
    float *host_out = nullptr;
    int64_t out_cap = 0;
};
AttnScratch &attn_scratch() {
    static AttnScratch a;
    return a;
}

int attn_dev(const float *q, int Hq, int D, const void *K, const void *V, int Hkv, int64_t S, int64_t hs, int64_t rs,
             const float *mask, const float *sinks, float scale, float *out, bool bf16, cudaStream_t s) {
    const int elt = bf16 ? 2 : 4;
    if (Hq <= 0 || Hkv <= 0 || Hq % Hkv || Hq / Hkv > 16 || D <= 0 || D > 256 || (D * elt) % 16 || S < 0 ||
        S > (int64_t{1} << 31)) {
        set_err("onpu_attn_step: need Hq %% Hkv == 0 with Hq / Hkv <= 16, 0 < D <= 256 with D * %d %% 16 == 0, "
                "0 <= S < 2^31 (got Hq %d, Hkv %d, D %d, S %lld)", elt, Hq, Hkv, D, static_cast<long long>(S));
        return -1;
    }
    if (S > 0 && ((reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(V)) & 15 || (hs * elt) % 16 ||
                  (rs * elt) % 16 || rs < D)) {
        set_err("onpu_attn_step: K and V must be 16-byte aligned with hs and rs multiples of 16 bytes and rs >= D");
        return -1;
    }
    Ctx &c = ctx();
    AttnScratch &a = attn_scratch();
    AttnParams p{};
    p.q = q;
    p.k = K;
    p.v = V;
    p.mask = mask;
    p.sinks = sinks;
    p.out = out;
    p.Hq = Hq;
    p.D = D;
    p.Hkv = Hkv;
    p.S = S;
    p.hs = hs;
    p.rs = rs;
    p.scale = scale;
    const bool tc = attn_use_tc(D, Hq / Hkv, bf16);
    p.tile_rows = tc ? attn_tc_warps() * attn_tc_rows() : attn_tile_rows(D, bf16);
    // one wave of resident CTAs over all kv heads, each split a whole number of tiles
    // (tensor-core form: of 16-row blocks for each of its warps)
    const int64_t target = static_cast<int64_t>(attn_ctas_per_sm(D, Hq / Hkv, bf16)) * c.nsm;
    int64_t rows = (S * Hkv + target - 1) / target;
    rows = std::max<int64_t>(p.tile_rows, (rows + p.tile_rows - 1) / p.tile_rows * p.tile_rows);
    p.rows_per_split = static_cast<int>(std::min<int64_t>(rows, int64_t{1} << 30));
    p.splits = S > 0 ? static_cast<int>((S + rows - 1) / rows) : 1;
    const int64_t nml = round_up(static_cast<int64_t>(Hq) * p.splits * 2, 4);   // keeps part_o 16-byte aligned
    if (!grow(a.part, a.part_cap, nml + static_cast<int64_t>(Hq) * p.splits * D)) return -1;
    p.part_ml = a.part;
    p.part_o = a.part + nml;
    ONPU_CUDA(attn_launch(p, bf16, s), -1);
    return 0;
}

// host-pointer form: stage q, mask, sinks and the cache rows [Hkv][S][D] on the device
void attn_host(const float *q, int Hq, int D, const void *K, const void *V, int Hkv, int64_t S, int64_t hs, int64_t rs,
               const float *mask, const float *sinks, float scale, float *out, bool bf16) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return;
    }
    if (Hq <= 0 || D <= 0 || S < 0 || Hkv <= 0 || (S > 0 && rs < D)) {
        set_err("onpu_attn_step: bad sizes (Hq %d, D %d, Hkv %d, S %lld, rs %lld)", Hq, D, Hkv,
                static_cast<long long>(S), static_cast<long long>(rs));
        return;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    AttnScratch &a = attn_scratch();
    const int elt = bf16 ? 2 : 4;
    const int64_t nq = static_cast<int64_t>(Hq) * D, nkv = (static_cast<int64_t>(Hkv) * S * D * elt + 15) / 16 * 4;
    const int64_t total = nq + (mask ? S : 0) + (sinks ? Hq : 0) + 2 * nkv + 16;
    if (!grow(a.host_in, a.host_cap, total) || !grow(a.host_out, a.out_cap, nq)) return;
    float *dq = a.host_in, *dm = dq + nq, *dsk = dm + (mask ? S : 0);
    float *dk = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(dsk + (sinks ? Hq : 0)) + 15) & ~uintptr_t{15});
    float *dv = dk + nkv;
    cudaStream_t s = c.stream;
    ONPU_CUDA(cudaMemcpyAsync(dq, q, nq * 4, cudaMemcpyHostToDevice, s), );
    if (mask) ONPU_CUDA(cudaMemcpyAsync(dm, mask, S * 4, cudaMemcpyHostToDevice, s), );
    if (sinks) ONPU_CUDA(cudaMemcpyAsync(dsk, sinks, Hq * 4, cudaMemcpyHostToDevice, s), );
    const size_t row = static_cast<size_t>(D) * elt;
    for (int kh = 0; kh < Hkv && S > 0; ++kh) {        // one strided copy per kv head and tensor
        const auto *ks = static_cast<const uint8_t *>(K) + static_cast<int64_t>(kh) * hs * elt;
        const auto *vs = static_cast<const uint8_t *>(V) + static_cast<int64_t>(kh) * hs * elt;
        auto *kd = reinterpret_cast<uint8_t *>(dk) + static_cast<int64_t>(kh) * S * row;
        auto *vd = reinterpret_cast<uint8_t *>(dv) + static_cast<int64_t>(kh) * S * row;
        ONPU_CUDA(cudaMemcpy2DAsync(kd, row, ks, static_cast<size_t>(rs) * elt, row, static_cast<size_t>(S),
                                    cudaMemcpyHostToDevice, s), );
        ONPU_CUDA(cudaMemcpy2DAsync(vd, row, vs, static_cast<size_t>(rs) * elt, row, static_cast<size_t>(S),
                                    cudaMemcpyHostToDevice, s), );
    }
    if (attn_dev(dq, Hq, D, dk, dv, Hkv, S, S * D, D, mask ? dm : nullptr, sinks ? dsk : nullptr, scale, a.host_out,
                 bf16, s) != 0)
        return;
    ONPU_CUDA(cudaMemcpyAsync(out, a.host_out, nq * 4, cudaMemcpyDeviceToHost, s), );
    ONPU_CUDA(cudaStreamSynchronize(s), );
}
}  // namespace

extern "C" {

void onpu_attn_step(const float *q, int Hq, int D, const float *K, const float *V, int Hkv, int64_t S, int64_t hs,
                    int64_t rs, const float *mask, const float *sinks, float scale, float *out) {
    attn_host(q, Hq, D, K, V, Hkv, S, hs, rs, mask, sinks, scale, out, false);
}

void onpu_attn_step_bf16(const float *q, int Hq, int D, const uint16_t *K, const uint16_t *V, int Hkv, int64_t S,
                         int64_t hs, int64_t rs, const float *mask, const float *sinks, float scale, float *out) {
    attn_host(q, Hq, D, K, V, Hkv, S, hs, rs, mask, sinks, scale, out, true);
}

int onpu_attn_step_dev(const float *q, int Hq, int D, const void *K, const void *V, int Hkv, int64_t S, int64_t hs,
                       int64_t rs, const float *mask, const float *sinks, float scale, float *out, int kv_bf16,
                       void *stream) {
    clear_err();
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return -1;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    return attn_dev(q, Hq, D, K, V, Hkv, S, hs, rs, mask, sinks, scale, out, kv_bf16 != 0,
                    static_cast<cudaStream_t>(stream));
}

int onpu_layout_version(void) { return kGpuLayoutVersion; }

int64_t onpu_dense_export(void *h, void *dst, int64_t cap) {
    clear_err();
    auto *d = static_cast<DenseH *>(h);
    if (!d || !exportable(d->geo, d->mat, "onpu_dense_export")) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    const GpuMat *mats[1] = {&d->mat};
    const uint32_t flags[1] = {(d->gateup ? kMatGateUp : 0u) | (d->residual ? kMatResidual : 0u)};
    return write_blob(kBlobDense, mats, flags, 1, dst, cap, "onpu_dense_export");
}

void *onpu_dense_import(const void *src, int64_t nbytes) {
    clear_err();
    MatHead h[1];
    const uint8_t *pl[1];
    if (!parse_blob(src, nbytes, kBlobDense, 1, h, pl, "onpu_dense_import")) return nullptr;
    if (h[0].E != 1 || (h[0].flags == (kMatGateUp | kMatResidual))) {
        set_err("onpu_dense_import: a dense blob holds one matrix, gate/up or two-pass, not both");
        return nullptr;
    }
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    auto *d = new DenseH;
    d->fmt = h[0].fmt;
    d->gateup = h[0].flags == kMatGateUp;
    d->residual = h[0].flags == kMatResidual;
    if (!load_section(d->mat, h[0], pl[0], "onpu_dense_import")) {
        delete d;
        return nullptr;
    }
    return d;
}

int64_t onpu_bank_export(void *h, void *dst, int64_t cap) {
    clear_err();
    auto *b = static_cast<BankH *>(h);
    if (!b || !exportable(b->geo, b->mat, "onpu_bank_export")) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    const GpuMat *mats[1] = {&b->mat};
    const uint32_t flags[1] = {b->mat.d_row_map ? kMatGateUp : 0u};
    return write_blob(kBlobBank, mats, flags, 1, dst, cap, "onpu_bank_export");
}

void *onpu_bank_import(const void *src, int64_t nbytes) {
    clear_err();
    MatHead h[1];
    const uint8_t *pl[1];
    if (!parse_blob(src, nbytes, kBlobBank, 1, h, pl, "onpu_bank_import")) return nullptr;
    if (h[0].flags & kMatResidual) {
        set_err("onpu_bank_import: expert banks have no two-pass form");
        return nullptr;
    }
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    return bank_from_section(h[0], pl[0], "onpu_bank_import");
}

int64_t onpu_ffn_export(void *h, void *dst, int64_t cap) {
    clear_err();
    auto *f = static_cast<FfnH *>(h);
    if (!f || !exportable(f->gu->geo, f->gu->mat, "onpu_ffn_export") ||
        !exportable(f->dn->geo, f->dn->mat, "onpu_ffn_export"))
        return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    const GpuMat *mats[2] = {&f->gu->mat, &f->dn->mat};
    const uint32_t flags[2] = {f->gu->mat.d_row_map ? kMatGateUp : 0u, f->dn->mat.d_row_map ? kMatGateUp : 0u};
    return write_blob(kBlobFfn, mats, flags, 2, dst, cap, "onpu_ffn_export");
}

void *onpu_ffn_import(const void *src, int64_t nbytes) {
    clear_err();
    MatHead h[2];
    const uint8_t *pl[2];
    if (!parse_blob(src, nbytes, kBlobFfn, 2, h, pl, "onpu_ffn_import")) return nullptr;
    if (((h[0].flags | h[1].flags) & kMatResidual) || h[0].E != h[1].E) {
        set_err("onpu_ffn_import: gate_up and down banks need the same expert count and no two-pass form");
        return nullptr;
    }
    Ctx &c = ctx();
    if (!c.ok) {
        set_err("no usable CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    auto *f = new FfnH;
    f->gu = bank_from_section(h[0], pl[0], "onpu_ffn_import");
    f->dn = f->gu ? bank_from_section(h[1], pl[1], "onpu_ffn_import") : nullptr;
    if (!f->gu || !f->dn) {
        delete f;
        return nullptr;
    }
    f->fused = (h[0].flags & kMatGateUp) && h[1].K * 2 == h[0].N;
    return f;
}

}  // extern "C"
