// The ggml-opennpu backend's operator layer over this library's C ABI: which MUL_MAT /
// MUL_MAT_ID nodes it takes (opennpu_supports, llama/ggml-opennpu/ggml-opennpu.cpp:703-753),
// how their tensors are laid out (input rows, expert ids, outputs: :270-277, :317-385, :467-539),
// and the learned sibling fusion (:387-465): weights that read the same input in the same block
// run as one stacked matrix, the first sibling's call computes all of them and the others find
// their slice waiting (checked against their input before use).
//
// The tensors arrive as onpu_ggml_tensor descriptors (the ggml_tensor fields the logic reads), so
// the layer builds and is tested without ggml; the backend glue (ggml_backend_* registration,
// buffer types) needs llama.cpp's headers and is the only part left to the integration.
//
// Weights become libonpu handles on first use, cached by their data pointer:
//  - Q4_0 / Q4_K rows go to the GPU as they are (onpu_dense_new_gguf / onpu_bank_new_gguf: Q4_0
//    exactly, Q4_K transcoded to q4nx on the device as the reference transcodes it);
//  - F32 / F16 / BF16 (and groups mixing formats) are widened to fp32 on the host and quantised on
//    the GPU with the reference's q4nx search quantiser (onpu_dense_new_f32_dev), where the
//    reference dequantises every format through ggml's to_float and packs with the same search.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "onpu.h"

namespace {

constexpr int kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ4_K = 12, kI32 = 26, kBF16 = 30;
constexpr int64_t kMinParams = int64_t{1} << 20;     // the reference's MIN_PARAMS
constexpr size_t kMaxGroup = 4;                      // siblings per fused dispatch (:438)

// bytes of one row of K elements, -1 for a type this layer does not take
int64_t row_bytes(int type, int64_t K) {
    switch (type) {
        case kF32: return K * 4;
        case kF16: case kBF16: return K * 2;
        case kQ4_0: return K % 32 ? -1 : K / 32 * 18;
        case kQ4_K: return K % 256 ? -1 : K / 256 * 144;
        default: return -1;
    }
}
int64_t elt_bytes(int type) { return type == kF32 || type == kI32 ? 4 : (type == kF16 || type == kBF16 ? 2 : 0); }
bool quantized(int type) { return type == kQ4_0 || type == kQ4_K; }

float half_to_float(uint16_t h) {
    const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 31u, m = h & 1023u;
    float v;
    if (e == 0) v = std::ldexp(static_cast<float>(m), -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = std::ldexp(static_cast<float>(m | 1024u), static_cast<int>(e) - 25);
    return s ? -v : v;
}

// one row of K weights of `type` -> fp32 (Q4_0: (q - 8) d; Q4_K: q (d sc) - dmin m per 32)
void row_to_f32(int type, const uint8_t *src, int64_t K, float *out) {
    if (type == kF32) {
        std::memcpy(out, src, K * 4);
    } else if (type == kF16) {
        for (int64_t i = 0; i < K; ++i) out[i] = half_to_float(static_cast<uint16_t>(src[2 * i] | (src[2 * i + 1] << 8)));
    } else if (type == kBF16) {
        for (int64_t i = 0; i < K; ++i) {
            const uint32_t u = static_cast<uint32_t>(src[2 * i] | (src[2 * i + 1] << 8)) << 16;
            std::memcpy(out + i, &u, 4);
        }
    } else if (type == kQ4_0) {
        for (int64_t b = 0; b < K / 32; ++b) {
            const uint8_t *p = src + b * 18;
            const float d = half_to_float(static_cast<uint16_t>(p[0] | (p[1] << 8)));
            for (int j = 0; j < 16; ++j) {
                out[b * 32 + j] = static_cast<float>((p[2 + j] & 15) - 8) * d;
                out[b * 32 + j + 16] = static_cast<float>((p[2 + j] >> 4) - 8) * d;
            }
        }
    } else {   // Q4_K
        for (int64_t b = 0; b < K / 256; ++b) {
            const uint8_t *p = src + b * 144, *sc = p + 4, *qs = p + 16;
            const float d = half_to_float(static_cast<uint16_t>(p[0] | (p[1] << 8)));
            const float dmin = half_to_float(static_cast<uint16_t>(p[2] | (p[3] << 8)));
            for (int sub = 0; sub < 8; ++sub) {
                int sv, mv;
                if (sub < 4) {
                    sv = sc[sub] & 63;
                    mv = sc[sub + 4] & 63;
                } else {
                    sv = (sc[sub + 4] & 0xF) | ((sc[sub - 4] >> 6) << 4);
                    mv = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
                }
                const float S = d * static_cast<float>(sv), dm = dmin * static_cast<float>(mv);
                const uint8_t *qq = qs + (sub / 2) * 32;
                for (int l = 0; l < 32; ++l) {
                    const int q = (sub & 1) ? (qq[l] >> 4) : (qq[l] & 15);
                    out[b * 256 + sub * 32 + l] = static_cast<float>(q) * S - dm;
                }
            }
        }
    }
}

bool contiguous(const onpu_ggml_tensor *t) {
    const int64_t rb = row_bytes(t->type, t->ne[0]);
    if (rb < 0) return false;
    if (!quantized(t->type) && t->nb[0] != elt_bytes(t->type)) return false;
    return t->nb[1] == rb && t->nb[2] == t->nb[1] * t->ne[1] && t->nb[3] == t->nb[2] * t->ne[2];
}

// OPENNPU_CPU_TENSORS: comma-separated name prefixes kept on the CPU (:703-717)
bool keep_on_cpu(const onpu_ggml_tensor *w) {
    static const std::vector<std::string> prefixes = [] {
        std::vector<std::string> v;
        const char *e = std::getenv("OPENNPU_CPU_TENSORS");
        std::string cur;
        for (const char *c = e ? e : "";; ++c) {
            if (*c == ',' || *c == 0) {
                if (!cur.empty()) v.push_back(cur);
                cur.clear();
                if (!*c) break;
            } else {
                cur += *c;
            }
        }
        return v;
    }();
    if (!w->name) return false;
    for (const auto &p : prefixes)
        if (std::strncmp(w->name, p.c_str(), p.size()) == 0) return true;
    return false;
}

int64_t min_params() {
    static const int64_t v = [] {
        const char *e = std::getenv("OPENNPU_MIN_PARAMS");
        return e ? std::atoll(e) : kMinParams;
    }();
    return v;
}

bool weight_ok(const onpu_ggml_tensor *w) {
    return w && w->weights && w->data && w->ne[0] % 32 == 0 && row_bytes(w->type, w->ne[0]) > 0 && contiguous(w);
}

std::string blk_of(const char *name) {              // "blk.12." of "blk.12.attn_q.weight"
    const std::string n(name ? name : "");
    const size_t a = n.find('.'), b = a == std::string::npos ? a : n.find('.', a + 1);
    return b == std::string::npos ? n : n.substr(0, b + 1);
}

// the input's rows in (i3, i2, i1) order (:270-277)
std::vector<const float *> input_rows(const onpu_ggml_tensor *x) {
    std::vector<const float *> r;
    for (int64_t i3 = 0; i3 < x->ne[3]; ++i3)
        for (int64_t i2 = 0; i2 < x->ne[2]; ++i2)
            for (int64_t i1 = 0; i1 < x->ne[1]; ++i1)
                r.push_back(reinterpret_cast<const float *>(static_cast<const char *>(x->data) + i1 * x->nb[1] +
                                                            i2 * x->nb[2] + i3 * x->nb[3]));
    return r;
}

// A weight as the layer remembers it (descriptors are not kept by the caller).
struct WeightInfo {
    int type = 0;
    int64_t ne[4] = {0, 0, 0, 0}, nb[4] = {0, 0, 0, 0};
    const void *data = nullptr;
    std::string name;
};
WeightInfo info_of(const onpu_ggml_tensor *w) {
    WeightInfo i;
    i.type = w->type;
    std::memcpy(i.ne, w->ne, sizeof i.ne);
    std::memcpy(i.nb, w->nb, sizeof i.nb);
    i.data = w->data;
    i.name = w->name ? w->name : "";
    return i;
}

using Group = std::vector<const void *>;            // weight data pointers, the first one leads

struct Pending {                                     // a sibling's output, computed with its group
    const void *x_data = nullptr;
    std::vector<float> x;                            // the input it was computed for
    std::vector<int32_t> ids;
    std::vector<float> out;                          // [rows or (t, slot)] x N
};

struct Ctx {
    std::mutex mu;
    std::map<const void *, WeightInfo> weights;                 // every weight noted or computed
    std::map<const void *, std::vector<const void *>> by_input; // input data -> weights reading it
    std::map<const void *, Group> group_of;                     // leader -> its group
    std::map<const void *, const void *> leader;                // non-leading member -> leader
    bool grouped = false;
    std::map<const void *, void *> dense, banks;                // leader -> libonpu handle
    std::map<const void *, Pending> pend;
    int64_t hits = 0, misses = 0;
    std::vector<float> xs, ys;
    std::vector<int32_t> ids;
    ~Ctx() {
        for (auto &kv : dense) onpu_dense_free(kv.second);
        for (auto &kv : banks) onpu_bank_free(kv.second);
    }
};

std::vector<float> input_copy(const onpu_ggml_tensor *x) {
    std::vector<float> v;
    for (const float *r : input_rows(x)) v.insert(v.end(), r, r + x->ne[0]);
    return v;
}
std::vector<int32_t> ids_copy(const onpu_ggml_tensor *ids) {
    std::vector<int32_t> v;
    if (!ids) return v;
    for (int64_t t = 0; t < ids->ne[1]; ++t) {
        const auto *id = reinterpret_cast<const int32_t *>(static_cast<const char *>(ids->data) + t * ids->nb[1]);
        v.insert(v.end(), id, id + ids->ne[0]);
    }
    return v;
}

// groups from the noted siblings: same block, same K, same expert count, at most kMaxGroup,
// each weight in one group only (:433-465)
void finalize_groups(Ctx &c) {
    static const bool off = std::getenv("OPENNPU_FUSE") && std::string(std::getenv("OPENNPU_FUSE")) == "0";
    if (off) return;
    for (auto &kv : c.by_input) {
        const auto &v = kv.second;
        if (v.size() < 2) continue;
        const WeightInfo &w0 = c.weights[v[0]];
        Group g{v[0]};
        for (size_t i = 1; i < v.size() && g.size() < kMaxGroup; ++i) {
            const WeightInfo &w = c.weights[v[i]];
            if (w.ne[0] == w0.ne[0] && w.ne[2] == w0.ne[2] && blk_of(w.name.c_str()) == blk_of(w0.name.c_str()))
                g.push_back(v[i]);
        }
        if (g.size() < 2) continue;
        bool clash = false;
        for (const void *m : g) clash |= c.group_of.count(m) || c.leader.count(m);
        if (clash) continue;
        c.group_of[g[0]] = g;
        for (size_t i = 1; i < g.size(); ++i) c.leader[g[i]] = g[0];
    }
}

int64_t group_rows(Ctx &c, const Group &g) {
    int64_t n = 0;
    for (const void *w : g) n += c.weights[w].ne[1];
    return n;
}

// the group's matrices stacked by rows (expert e: every member's rows of expert e), as GGUF bytes
// when they share a quantised type, else as fp32
bool stack_group(Ctx &c, const Group &g, int64_t E, int &type, std::vector<uint8_t> &bytes, std::vector<float> &f32) {
    const WeightInfo &w0 = c.weights[g[0]];
    const int64_t K = w0.ne[0], N = group_rows(c, g);
    type = w0.type;
    for (const void *w : g) type = c.weights[w].type == type ? type : -1;
    if (type >= 0 && quantized(type)) {
        const int64_t rb = row_bytes(type, K);
        bytes.resize(static_cast<size_t>(E * N * rb));
        uint8_t *o = bytes.data();
        for (int64_t e = 0; e < E; ++e)
            for (const void *wp : g) {
                const WeightInfo &w = c.weights[wp];
                const size_t n = static_cast<size_t>(w.ne[1] * rb);
                std::memcpy(o, static_cast<const uint8_t *>(w.data) + e * w.nb[2], n);
                o += n;
            }
        return true;
    }
    type = kF32;
    f32.resize(static_cast<size_t>(E * N * K));
    float *o = f32.data();
    for (int64_t e = 0; e < E; ++e)
        for (const void *wp : g) {
            const WeightInfo &w = c.weights[wp];
            for (int64_t r = 0; r < w.ne[1]; ++r, o += K)
                row_to_f32(w.type, static_cast<const uint8_t *>(w.data) + e * w.nb[2] + r * w.nb[1], K, o);
        }
    return true;
}

void *dense_handle(Ctx &c, const Group &g) {
    auto it = c.dense.find(g[0]);
    if (it != c.dense.end()) return it->second;
    const int64_t K = c.weights[g[0]].ne[0], N = group_rows(c, g);
    int type = 0;
    std::vector<uint8_t> bytes;
    std::vector<float> f32;
    stack_group(c, g, 1, type, bytes, f32);
    void *h = nullptr;
    if (type != kF32) {
        h = onpu_dense_new_gguf(N, K, type, bytes.data(), 0, 0, nullptr);
    } else {
        float *dW = nullptr;
        if (cudaMalloc(&dW, f32.size() * sizeof(float)) == cudaSuccess &&
            cudaMemcpy(dW, f32.data(), f32.size() * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess)
            h = onpu_dense_new_f32_dev(dW, K, N, K, 0, 0, nullptr);     // q4nx, the reference's default
        cudaFree(dW);
    }
    if (h) c.dense[g[0]] = h;
    return h;
}

void *bank_handle(Ctx &c, const Group &g) {
    auto it = c.banks.find(g[0]);
    if (it != c.banks.end()) return it->second;
    const WeightInfo &w0 = c.weights[g[0]];
    const int64_t K = w0.ne[0], N = group_rows(c, g), E = w0.ne[2];
    int type = 0;
    std::vector<uint8_t> bytes;
    std::vector<float> f32;
    stack_group(c, g, E, type, bytes, f32);
    if (type == kF32) return nullptr;               // expert banks take Q4_0 or Q4_K (onpu_ggml_supports)
    void *h = onpu_bank_new_gguf(N, K, E, type, bytes.data(), 0, 0, nullptr);
    if (h) c.banks[g[0]] = h;
    return h;
}

// an output row of the node: MUL_MAT row r of the input's (i3, i2, i1) order; MUL_MAT_ID (token,
// slot) = dst + slot * nb1 + token * nb2
char *dst_row(const onpu_ggml_tensor *dst, const onpu_ggml_tensor *x, bool ex, int64_t row, int64_t slot) {
    char *base = static_cast<char *>(dst->data);
    if (ex) return base + slot * dst->nb[1] + row * dst->nb[2];
    const int64_t i1 = row % x->ne[1], i2 = (row / x->ne[1]) % x->ne[2], i3 = row / (x->ne[1] * x->ne[2]);
    return base + i1 * dst->nb[1] + i2 * dst->nb[2] + i3 * dst->nb[3];
}

int compute(Ctx &c, int op, const onpu_ggml_tensor *dst, const onpu_ggml_tensor *w, const onpu_ggml_tensor *x,
            const onpu_ggml_tensor *ids) {
    const bool ex = op == ONPU_GGML_OP_MUL_MAT_ID;
    if (!c.weights.count(w->data)) c.weights[w->data] = info_of(w);
    if (!c.grouped) {
        finalize_groups(c);
        c.grouped = true;
    }
    const int64_t N = w->ne[1], K = w->ne[0];
    // a sibling whose output its group's leader computed
    auto pit = c.pend.find(w->data);
    if (pit != c.pend.end()) {
        Pending &p = pit->second;
        if (p.x_data == x->data && p.x == input_copy(x) && p.ids == ids_copy(ids)) {
            if (!ex) {
                const int64_t R = x->ne[1] * x->ne[2] * x->ne[3];
                for (int64_t r = 0; r < R; ++r) std::memcpy(dst_row(dst, x, false, r, 0), p.out.data() + r * N, N * 4);
            } else {
                for (int64_t t = 0; t < ids->ne[1]; ++t)
                    for (int64_t j = 0; j < ids->ne[0]; ++j)
                        std::memcpy(dst_row(dst, x, true, t, j), p.out.data() + (t * ids->ne[0] + j) * N, N * 4);
            }
            c.pend.erase(pit);
            ++c.hits;
            return 0;
        }
        ++c.misses;
        c.pend.erase(pit);
    }
    Group g{w->data};                                // a member whose slice is not waiting runs on its own
    auto git = c.group_of.find(w->data);
    if (git != c.group_of.end()) g = git->second;
    const int64_t Ntot = group_rows(c, g);
    // run the (stacked) matrix
    if (!ex) {
        const std::vector<const float *> rows = input_rows(x);
        const int64_t R = static_cast<int64_t>(rows.size());
        c.xs.resize(static_cast<size_t>(R * K));
        for (int64_t r = 0; r < R; ++r) std::memcpy(c.xs.data() + r * K, rows[r], K * 4);
        c.ys.resize(static_cast<size_t>(R * Ntot));
        void *h = dense_handle(c, g);
        if (!h) return -1;
        onpu_dense_mv(h, c.xs.data(), R, c.ys.data());
        if (onpu_last_error()) return -1;
    } else {
        const int64_t T = ids->ne[1], k = ids->ne[0], xr = x->ne[1];
        c.xs.resize(static_cast<size_t>(T * xr * K));
        for (int64_t t = 0; t < T; ++t)
            for (int64_t j = 0; j < xr; ++j)
                std::memcpy(c.xs.data() + (t * xr + j) * K,
                            static_cast<const char *>(x->data) + j * x->nb[1] + t * x->nb[2], K * 4);
        c.ids = ids_copy(ids);
        c.ys.resize(static_cast<size_t>(T * k * Ntot));
        void *h = bank_handle(c, g);
        if (!h) return -1;
        onpu_bank_run(h, c.xs.data(), xr == 1 ? 0 : 1, T, c.ids.data(), static_cast<int>(k), c.ys.data());
        if (onpu_last_error()) return -1;
    }
    // member 0's slice to this node, the others' slices waiting for their nodes
    const int64_t nrows = ex ? ids->ne[1] * ids->ne[0] : x->ne[1] * x->ne[2] * x->ne[3];
    std::vector<Pending *> pp(g.size(), nullptr);
    if (g.size() > 1) {
        const std::vector<float> xc = input_copy(x);
        const std::vector<int32_t> ic = ids_copy(ids);
        for (size_t i = 1; i < g.size(); ++i) {
            Pending &p = c.pend[g[i]];
            p.x_data = x->data;
            p.x = xc;
            p.ids = ic;
            p.out.assign(static_cast<size_t>(nrows * c.weights[g[i]].ne[1]), 0.0f);
            pp[i] = &p;
        }
    }
    for (int64_t r = 0; r < nrows; ++r) {
        const float *y = c.ys.data() + r * Ntot;
        int64_t o = 0;
        for (size_t i = 0; i < g.size(); ++i) {
            const int64_t n = c.weights[g[i]].ne[1];
            if (i == 0) {
                const int64_t row = ex ? r / ids->ne[0] : r, slot = ex ? r % ids->ne[0] : 0;
                std::memcpy(dst_row(dst, x, ex, row, slot), y + o, n * 4);
            } else {
                std::memcpy(pp[i]->out.data() + r * n, y + o, n * 4);
            }
            o += n;
        }
    }
    return 0;
}

}  // namespace

extern "C" {

int onpu_ggml_supports(int op, const onpu_ggml_tensor *dst, const onpu_ggml_tensor *w, const onpu_ggml_tensor *x,
                       const onpu_ggml_tensor *ids, int hadamard_hint) {
    if (op == ONPU_GGML_OP_VIEW) return 1;
    if (op != ONPU_GGML_OP_MUL_MAT && op != ONPU_GGML_OP_MUL_MAT_ID) return 0;
    if (!w || !x || !dst || keep_on_cpu(w) || !weight_ok(w)) return 0;
    if (x->type != kF32 || x->nb[0] != 4 || dst->nb[0] != 4) return 0;
    if (op == ONPU_GGML_OP_MUL_MAT) {
        if (hadamard_hint || w->ne[2] != 1 || w->ne[3] != 1) return 0;
        return w->ne[0] * w->ne[1] >= min_params() ? 1 : 0;
    }
    if (!ids || ids->type != kI32 || !quantized(w->type)) return 0;
    return w->ne[0] * w->ne[1] >= kMinParams / 8 ? 1 : 0;
}

void *onpu_ggml_new(void) { return new Ctx; }

void onpu_ggml_note(void *ctx, int op, const onpu_ggml_tensor *w, const onpu_ggml_tensor *x,
                    const onpu_ggml_tensor *ids) {
    (void)ids;
    auto &c = *static_cast<Ctx *>(ctx);
    std::lock_guard<std::mutex> lk(c.mu);
    if ((op != ONPU_GGML_OP_MUL_MAT && op != ONPU_GGML_OP_MUL_MAT_ID) || !w || !x) return;
    c.weights[w->data] = info_of(w);
    auto &v = c.by_input[x->data];
    if (std::find(v.begin(), v.end(), w->data) == v.end()) v.push_back(w->data);
}

int onpu_ggml_compute(void *ctx, int op, const onpu_ggml_tensor *dst, const onpu_ggml_tensor *w,
                      const onpu_ggml_tensor *x, const onpu_ggml_tensor *ids) {
    auto &c = *static_cast<Ctx *>(ctx);
    std::lock_guard<std::mutex> lk(c.mu);
    if (op == ONPU_GGML_OP_VIEW) return 0;
    if (!onpu_ggml_supports(op, dst, w, x, ids, 0)) return -1;
    return compute(c, op, dst, w, x, ids);
}

void onpu_ggml_stats(void *ctx, int64_t *out4) {
    auto &c = *static_cast<Ctx *>(ctx);
    std::lock_guard<std::mutex> lk(c.mu);
    out4[0] = c.hits;
    out4[1] = c.misses;
    out4[2] = static_cast<int64_t>(c.group_of.size());
    out4[3] = static_cast<int64_t>(c.dense.size() + c.banks.size());
}

void onpu_ggml_free(void *ctx) { delete static_cast<Ctx *>(ctx); }

}  // extern "C"
