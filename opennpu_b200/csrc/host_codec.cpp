// Load-time host codec of libonpu for B200 (see host_codec.hpp for the reference contract).
//
// The quantisers must reproduce the reference's codes bit for bit (a model packed by either
// library has to dequantise identically), so the float expressions below evaluate in the same
// order as opennpu_core.hpp:103-169 and this file is compiled with -ffp-contract=off.
#include "host_codec.hpp"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace onpu_b200 {

uint16_t f32_to_bf16(float f) {
    uint32_t bits;
    std::memcpy(&bits, &f, sizeof bits);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((bits >> 16) | 0x40u);
    const uint32_t lsb = (bits >> 16) & 1u;
    return static_cast<uint16_t>((bits + 0x7fffu + lsb) >> 16);
}

float bf16_to_f32(uint16_t h) {
    const uint32_t bits = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &bits, sizeof f);
    return f;
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (h & 0x8000u) ? 0x80000000u : 0u;
    const int e = (h >> 10) & 0x1f;
    const uint32_t mant = h & 0x3ffu;
    float mag;
    if (e == 0) mag = std::ldexp(static_cast<float>(mant), -24);
    else if (e == 31) mag = mant ? NAN : INFINITY;
    else mag = std::ldexp(static_cast<float>(mant | 0x400u), e - 25);
    uint32_t bits;
    std::memcpy(&bits, &mag, sizeof bits);
    bits |= sign;
    std::memcpy(&mag, &bits, sizeof mag);
    return mag;
}

static inline float bf16_round(float v) { return bf16_to_f32(f32_to_bf16(v)); }
static inline float clamp_code(float v, float lo, float hi) { return std::min(hi, std::max(lo, v)); }

// ------------------------------------------------------------------ geometry
Geometry::Geometry(int64_t n, int64_t k, int nc, bool sy) : N(n), K(k), ncols(nc), sym(sy) {
    // Candidate split: S K-slices of ceil(K / (S*256)) packets, R = ncols / S row blocks of
    // ceil(N / (R*256)) 64-row tiles per core row; tiles*kc must be even. Cost = packets streamed
    // with a 3% penalty per extra slice (host sums); first minimum wins.
    double best_cost = -1.0;
    for (int s = 1; s <= nc; ++s) {
        if (nc % s != 0) continue;
        const int64_t slice = static_cast<int64_t>(s) * kGK;
        int kcs = static_cast<int>((k + slice - 1) / slice);
        if (kcs > kKMAX / kGK) continue;
        const int r = nc / s;
        const int64_t rows = static_cast<int64_t>(r) * kNR * kGN;
        int tl = static_cast<int>((n + rows - 1) / rows);
        if ((tl * kcs) % 2 != 0) {
            const bool widen_k = kcs + 1 <= kKMAX / kGK &&
                                 static_cast<int64_t>(tl) * (kcs + 1) < static_cast<int64_t>(tl + 1) * kcs;
            if (widen_k) ++kcs;
            else ++tl;
        }
        const double cost = static_cast<double>(r) * s * tl * kcs * (1 + 0.03 * (s - 1));
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            R = r; S = s; tiles = tl; kc = kcs;
        }
    }
    if (best_cost < 0) return;
    ks = static_cast<int64_t>(kc) * kGK;
    rows_col = static_cast<int64_t>(kNR) * tiles * kGN;
    cb = static_cast<int64_t>(tiles) * kc * kNR * pkt();
    nbytes = static_cast<int64_t>(R) * S * cb;
    ok = true;
}

// ------------------------------------------------------------------ quantisers
void quant_q4nx32(const float *x, uint8_t *q, uint16_t &s_bf, uint16_t &m_bf) {
    float lo = x[0], hi = x[0];
    for (int i = 1; i < 32; ++i) {
        lo = std::min(lo, x[i]);
        hi = std::max(hi, x[i]);
    }
    const float range = hi - lo;
    if (!(range > 0)) {                       // constant (or NaN) group
        s_bf = f32_to_bf16(1.0f);
        m_bf = f32_to_bf16(lo);
        std::fill(q, q + 32, uint8_t{0});
        return;
    }
    float best_err = INFINITY, best_s = range / 15, best_m = lo;
    for (int stretch = 0; stretch <= 20; ++stretch) {
        const float inv = (-1.0f + 0.1f * stretch + 15.0f) / range;
        // least-squares (scale, min) for the codes this stretch assigns
        float sum_l = 0, sum_ll = 0, sum_x = 0, sum_lx = 0;
        for (int i = 0; i < 32; ++i) {
            const float l = clamp_code(std::nearbyint(inv * (x[i] - lo)), 0.0f, 15.0f);
            sum_l += l;
            sum_ll += l * l;
            sum_x += x[i];
            sum_lx += l * x[i];
        }
        const float det = 32 * sum_ll - sum_l * sum_l;
        float sc = range / 15, mn = lo;
        if (det > 0) {
            sc = (32 * sum_lx - sum_l * sum_x) / det;
            mn = (sum_ll * sum_x - sum_l * sum_lx) / det;
        }
        sc = bf16_round(sc);
        mn = bf16_round(mn);
        if (!(sc > 0)) continue;
        float err = 0;
        for (int i = 0; i < 32; ++i) {
            const float l = clamp_code(std::nearbyint((x[i] - mn) / sc), 0.0f, 15.0f);
            const float d = l * sc + mn - x[i];
            err += d * d;
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
        q[i] = static_cast<uint8_t>(clamp_code(std::nearbyint((x[i] - best_m) / best_s), 0.0f, 15.0f));
    s_bf = f32_to_bf16(best_s);
    m_bf = f32_to_bf16(best_m);
}

void quant_q4s32(const float *x, uint8_t *q, uint16_t &d_bf) {
    float peak = 0;                           // the signed value of largest magnitude (first wins)
    for (int i = 0; i < 32; ++i)
        if (std::fabs(x[i]) > std::fabs(peak)) peak = x[i];
    if (peak == 0) {
        d_bf = f32_to_bf16(1.0f);
        std::fill(q, q + 32, uint8_t{8});
        return;
    }
    float best_err = INFINITY, best_d = peak / -8.0f;
    for (int cand = 0; cand < 16; ++cand) {
        // divisors: 8 spread over [-9, -6.5], then 8 over [6.5, 8]
        const float div = cand < 8 ? -9.0f + 2.5f * cand / 7 : 6.5f + 1.5f * (cand - 8) / 7;
        const float d0 = peak / div;
        float sum_vv = 0, sum_vx = 0;
        for (int i = 0; i < 32; ++i) {
            const float v = clamp_code(std::nearbyint(x[i] / d0), -8.0f, 7.0f);
            sum_vv += v * v;
            sum_vx += v * x[i];
        }
        float d = sum_vv > 0 ? sum_vx / sum_vv : d0;
        d = bf16_round(d);
        if (d == 0) continue;
        float err = 0;
        for (int i = 0; i < 32; ++i) {
            const float v = clamp_code(std::nearbyint(x[i] / d), -8.0f, 7.0f);
            const float r = v * d - x[i];
            err += r * r;
        }
        if (err < best_err) {
            best_err = err;
            best_d = d;
        }
    }
    for (int i = 0; i < 32; ++i)
        q[i] = static_cast<uint8_t>(clamp_code(std::nearbyint(x[i] / best_d), -8.0f, 7.0f) + 8);
    d_bf = f32_to_bf16(best_d);
}

// ------------------------------------------------------------------ stream order
namespace {

// One column block: rows [r0, r1) x cols [k0, k1) of W, quantised, written as tiles*kc*NR packets
// in the order [tile][k packet][core row]; rows/cols past the block are padding (code 0 for
// q4nx, 8 for q4s; zero scale/min).
void pack_block(const Geometry &g, const float *W, int64_t r0, int64_t r1, int64_t k0, int64_t k1,
                uint8_t *out) {
    const int64_t rows = g.rows_col, kpad = g.ks, groups = kpad / 32;
    std::vector<uint8_t> code(static_cast<size_t>(rows * kpad), g.sym ? 8 : 0);
    std::vector<uint16_t> scale(static_cast<size_t>(rows * groups), 0), minv(scale.size(), 0);
    float grp[32];
    for (int64_t r = 0; r < rows && r0 + r < r1; ++r)
        for (int64_t gi = 0; gi < groups && k0 + gi * 32 < k1; ++gi) {
            const int64_t col = k0 + gi * 32;
            for (int i = 0; i < 32; ++i) grp[i] = col + i < k1 ? W[(r0 + r) * g.K + col + i] : 0.0f;
            uint8_t *qg = &code[r * kpad + gi * 32];
            if (g.sym) quant_q4s32(grp, qg, scale[r * groups + gi]);
            else quant_q4nx32(grp, qg, scale[r * groups + gi], minv[r * groups + gi]);
        }
    uint8_t *o = out;
    for (int t = 0; t < g.tiles; ++t)
        for (int kp = 0; kp < g.kc; ++kp)
            for (int cr = 0; cr < kNR; ++cr) {
                const int64_t row0 = static_cast<int64_t>(cr) * g.tiles * kGN + static_cast<int64_t>(t) * kGN;
                const int64_t col0 = static_cast<int64_t>(kp) * kGK;
                // nibbles: [8-row band][8-col band][col in band][row pair] -> low nibble = even row
                for (int rb = 0; rb < kGN / 8; ++rb)
                    for (int cband = 0; cband < kGK / 8; ++cband)
                        for (int cc = 0; cc < 8; ++cc) {
                            const int64_t col = col0 + cband * 8 + cc;
                            for (int rp = 0; rp < 8; rp += 2) {
                                const int64_t ra = row0 + rb * 8 + rp;
                                *o++ = static_cast<uint8_t>(code[ra * kpad + col] | (code[(ra + 1) * kpad + col] << 4));
                            }
                        }
                // bf16 scales then mins, [group of 32][row] little endian
                for (int pass = 0; pass < (g.sym ? 1 : 2); ++pass) {
                    const std::vector<uint16_t> &src = pass ? minv : scale;
                    for (int gi = 0; gi < kGK / 32; ++gi)
                        for (int n = 0; n < kGN; ++n) {
                            const uint16_t v = src[(row0 + n) * groups + col0 / 32 + gi];
                            *o++ = static_cast<uint8_t>(v & 0xffu);
                            *o++ = static_cast<uint8_t>(v >> 8);
                        }
                }
            }
}

template <typename F>
void parallel_for(int64_t n, int threads, F &&fn) {
    if (threads <= 1 || n <= 1) {
        for (int64_t i = 0; i < n; ++i) fn(i);
        return;
    }
    std::atomic<int64_t> next{0};
    std::vector<std::thread> pool;
    const int nt = static_cast<int>(std::min<int64_t>(threads, n));
    for (int t = 0; t < nt; ++t)
        pool.emplace_back([&] {
            for (int64_t i; (i = next.fetch_add(1)) < n;) fn(i);
        });
    for (auto &th : pool) th.join();
}

}  // namespace

void pack_stream(const Geometry &g, const float *W, uint8_t *out, int threads) {
    parallel_for(static_cast<int64_t>(g.R) * g.S, threads, [&](int64_t c) {
        const int64_t r = c / g.S, s = c % g.S;
        const int64_t r0 = r * g.rows_col, r1 = std::min(g.N, (r + 1) * g.rows_col);
        const int64_t k0 = s * g.ks, k1 = std::min(g.K, (s + 1) * g.ks);
        uint8_t *dst = out + c * g.cb;
        if (r1 > r0 && k1 > k0) pack_block(g, W, r0, r1, k0, k1, dst);
        else std::memset(dst, 0, static_cast<size_t>(g.cb));   // a block wholly outside the matrix
    });
}

void quant_dequant(const float *W, int64_t N, int64_t K, bool sym, float *out, int threads) {
    const int64_t chunks = std::max<int64_t>(1, std::min<int64_t>(threads, N / 64 + 1));
    parallel_for(chunks, threads, [&](int64_t part) {
        uint8_t q[32];
        for (int64_t r = N * part / chunks; r < N * (part + 1) / chunks; ++r)
            for (int64_t c = 0; c < K; c += 32) {
                const float *x = W + r * K + c;
                float *o = out + r * K + c;
                uint16_t s = 0, m = 0;
                if (sym) {
                    quant_q4s32(x, q, s);
                    for (int i = 0; i < 32; ++i) o[i] = (static_cast<float>(q[i]) - 8.0f) * bf16_to_f32(s);
                } else {
                    quant_q4nx32(x, q, s, m);
                    for (int i = 0; i < 32; ++i) o[i] = static_cast<float>(q[i]) * bf16_to_f32(s) + bf16_to_f32(m);
                }
            }
    });
}

}  // namespace onpu_b200
