// TEST INFRASTRUCTURE ONLY - extern "C" entry points over the vastloom reference library itself,
// which oracle/Makefile compiles from the reference's own sources into oracle/_ref/. Used by the
// tests to pin the C restatement (vlb_oracle.c) and by bench.py's reference/cpu_baseline legs.
//
// Everything arithmetic here is the reference's own code (matvec_*_f32, dequantize_*,
// deepseek_v4_route_*_logits, deepseek_v4_rms_norm). The only restated piece is the MoE layer
// loop, which is file-static in the reference (deepseek_v4_graph.cpp:1826-2274 execute_expert /
// moe_forward; olmoe_runtime.cpp:1119-1290); vlr_moe_forward below follows that loop order
// exactly and calls the reference's public kernels for every product.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <span>
#include <string>
#include <vector>

#include "vastloom/inference/deepseek_v4_reference.hpp"
#include "vastloom/inference/ggml_quantization.hpp"
#include "vastloom/inference/qwen3_8_flash_next_reference.hpp"

namespace vi = vastloom::inference;

extern "C" {

struct vlr_matrix {
    uint32_t type;
    size_t rows;
    size_t cols;
    const uint8_t* data;
};

struct vlr_moe_layer {
    size_t hidden, intermediate, experts, top_k;
    int score;  // 0 sqrt_softplus, 1 sigmoid (no reference router: unsupported here), 2 softmax
    int hash_routing;
    int weight_after_down;
    float route_scale, routed_swiglu_limit, shared_swiglu_limit;
    const float* router;
    const float* bias;
    const uint32_t* tid2eid;
    size_t vocab;
    const vlr_matrix* w1;
    const vlr_matrix* w3;
    const vlr_matrix* w2;
    const vlr_matrix* shared_w1;
    const vlr_matrix* shared_w3;
    const vlr_matrix* shared_w2;
};

static std::span<const std::byte> bytes_of(const vlr_matrix& m, size_t nbytes) {
    return {reinterpret_cast<const std::byte*>(m.data), nbytes};
}

static size_t matrix_bytes(uint32_t type, size_t rows, size_t cols) {
    auto b = vi::ggml_storage_bytes(type, rows, cols, vi::QuantizedKernelLimits{1ull << 40, 1});
    return b ? b.value() : 0;
}

// Copies a reference codebook (iq*_grid_table) into caller storage; returns its byte size.
size_t vlr_grid(uint32_t type, void* out, size_t cap) {
    std::span<const std::byte> g;
    if (type == vi::kGgmlTypeIq1S) g = std::as_bytes(vi::iq1_s_grid_table());
    else if (type == vi::kGgmlTypeIq2Xxs) g = std::as_bytes(vi::iq2_xxs_grid_table());
    else if (type == vi::kGgmlTypeIq3Xxs) g = std::as_bytes(vi::iq3_xxs_grid_table());
    else if (type == vi::kGgmlTypeIq2S) g = std::as_bytes(vi::iq2_s_grid_table());
    else return 0;
    if (out && cap >= g.size()) std::memcpy(out, g.data(), g.size());
    return g.size();
}

int vlr_dequantize(uint32_t type, const uint8_t* enc, size_t nbytes, float* out, size_t n) {
    std::span<const std::byte> e(reinterpret_cast<const std::byte*>(enc), nbytes);
    std::span<float> o(out, n);
    vi::QuantizedKernelLimits lim{1ull << 40, 1};
    vastloom::Result<void> r;
    switch (type) {
        case vi::kGgmlTypeQ8_0: r = vi::dequantize_q8_0(e, o, lim); break;
        case vi::kGgmlTypeIq2Xxs: r = vi::dequantize_iq2_xxs(e, o, lim); break;
        case vi::kGgmlTypeIq3Xxs: r = vi::dequantize_iq3_xxs(e, o, lim); break;
        case vi::kGgmlTypeIq1S: r = vi::dequantize_iq1_s(e, o, lim); break;
        case vi::kGgmlTypeQ4K: r = vi::dequantize_q4_k(e, o, lim); break;
        case vi::kGgmlTypeQ5K: r = vi::dequantize_q5_k(e, o, lim); break;
        case vi::kGgmlTypeQ6K: r = vi::dequantize_q6_k(e, o, lim); break;
        case vi::kGgmlTypeIq2S: r = vi::dequantize_iq2_s(e, o, lim); break;
        case vi::kGgmlTypeMxfp4: r = vi::dequantize_mxfp4(e, o, lim); break;
        default: return -2;
    }
    return r ? 0 : -1;
}

int vlr_matvec(uint32_t type, const uint8_t* enc, size_t rows, size_t cols, const float* x,
               float* y, unsigned threads) {
    const size_t nb = matrix_bytes(type, rows, cols);
    if (nb == 0) return -2;
    std::span<const std::byte> e(reinterpret_cast<const std::byte*>(enc), nb);
    std::vector<float> scratch(rows);
    vi::QuantizedKernelLimits lim{1ull << 40, threads == 0 ? 1u : threads};
    auto r = vi::matvec_ggml_f32_transactional(type, e, rows, cols, {x, cols}, scratch,
                                               {y, rows}, lim);
    return r ? 0 : -1;
}

int vlr_quantize_q8_0(const float* m, size_t rows, size_t lc, size_t sc, uint8_t* out) {
    auto r = vi::quantize_q8_0_reference({m, rows * lc}, rows, lc, sc);
    if (!r) return -1;
    std::memcpy(out, r.value().data(), r.value().size());
    return 0;
}

static int copy_route(const vastloom::Result<vi::DeepseekV4RouteResult>& r, uint32_t* idx,
                      float* w) {
    if (!r) return -1;
    std::memcpy(idx, r.value().indices.data(), r.value().indices.size() * sizeof(uint32_t));
    std::memcpy(w, r.value().weights.data(), r.value().weights.size() * sizeof(float));
    return 0;
}

int vlr_route_learned(const float* logits, const float* bias, size_t T, size_t E, size_t k,
                      float route_scale, uint32_t* idx, float* w) {
    return copy_route(vi::deepseek_v4_route_learned_logits({logits, T * E}, {bias, E}, T, E, k,
                                                           route_scale),
                      idx, w);
}

int vlr_route_hash(const float* logits, const uint32_t* token_ids, const uint32_t* table,
                   size_t T, size_t V, size_t E, size_t k, float route_scale, uint32_t* idx,
                   float* w) {
    return copy_route(vi::deepseek_v4_route_hash_logits({logits, T * E}, {token_ids, T},
                                                        {table, V * k}, T, V, E, k,
                                                        route_scale),
                      idx, w);
}

int vlr_rms_norm(const float* x, const float* w, size_t rows, size_t width, float eps,
                 float* out) {
    auto r = vi::deepseek_v4_rms_norm({x, rows * width}, {w, width}, rows, width, eps);
    if (!r) return -1;
    std::memcpy(out, r.value().data(), rows * width * sizeof(float));
    return 0;
}

static void copy_split(const vi::DeepseekV4HyperConnectionSplit& s, float* pre, float* post, float* comb) {
    std::memcpy(pre, s.pre.data(), s.pre.size() * sizeof(float));
    std::memcpy(post, s.post.data(), s.post.size() * sizeof(float));
    std::memcpy(comb, s.combination.data(), s.combination.size() * sizeof(float));
}

int vlr_hc_split_sinkhorn(const float* mixes, const float* scale, const float* base, size_t T, size_t m,
                          size_t iters, float eps, float* pre, float* post, float* comb) {
    auto r = vi::deepseek_v4_hc_split_sinkhorn({mixes, T * (2 + m) * m}, {scale, 3}, {base, (2 + m) * m}, T, m,
                                               iters, eps);
    if (!r) return -1;
    copy_split(r.value(), pre, post, comb);
    return 0;
}

int vlr_hc_pre(const float* x, const float* fn, const float* scale, const float* base, size_t T, size_t m,
               size_t W, size_t iters, float norm_eps, float hc_eps, float* reduced, float* pre, float* post,
               float* comb) {
    const size_t mw = (2 + m) * m;
    auto r = vi::deepseek_v4_hc_pre({x, T * m * W}, {fn, mw * m * W}, {scale, 3}, {base, mw}, T, m, W, iters,
                                    norm_eps, hc_eps);
    if (!r) return -1;
    std::memcpy(reduced, r.value().reduced.data(), T * W * sizeof(float));
    copy_split(r.value().split, pre, post, comb);
    return 0;
}

int vlr_hc_post(const float* sub, const float* residual, const float* post, const float* comb, size_t T,
                size_t m, size_t W, float* out) {
    vi::DeepseekV4HyperConnectionSplit split;
    split.token_count = T;
    split.multiplier = m;
    split.pre.assign(T * m, 1.0f);
    split.post.assign(post, post + T * m);
    split.combination.assign(comb, comb + T * m * m);
    auto r = vi::deepseek_v4_hc_post({sub, T * W}, {residual, T * m * W}, split, W);
    if (!r) return -1;
    std::memcpy(out, r.value().data(), T * m * W * sizeof(float));
    return 0;
}

// qwen38_moe_route (qwen3_8_flash_next_reference.cpp:1186-1239) for T tokens: hidden [T x H],
// router [E x H]; logits [T x E] (may be null), idx / w [T x k].
int vlr_qwen_route(const float* hidden, const float* router, size_t T, size_t H, size_t E, size_t k,
                   int norm, float* logits, uint32_t* idx, float* w) {
    for (size_t t = 0; t < T; ++t) {
        auto r = vi::qwen38_moe_route({hidden + t * H, H}, {router, E * H}, static_cast<uint32_t>(E),
                                      static_cast<uint32_t>(k), norm != 0);
        if (!r) return -1;
        if (logits) std::memcpy(logits + t * E, r.value().logits.data(), E * sizeof(float));
        std::memcpy(idx + t * k, r.value().indices.data(), k * sizeof(uint32_t));
        std::memcpy(w + t * k, r.value().weights.data(), k * sizeof(float));
    }
    return 0;
}

// deepseek_v4_expert_swiglu (deepseek_v4_reference.cpp:309-385); routing_weights may be null.
int vlr_expert_swiglu(const float* x, const float* gate_w, const float* down_w, const float* up_w,
                      const float* routing_weights, size_t T, size_t width, size_t inter, float limit,
                      float* out) {
    auto r = vi::deepseek_v4_expert_swiglu({x, T * width}, {gate_w, inter * width}, {down_w, width * inter},
                                           {up_w, inter * width},
                                           routing_weights ? std::span<const float>(routing_weights, T)
                                                           : std::span<const float>(),
                                           T, width, inter, limit);
    if (!r) return -1;
    std::memcpy(out, r.value().data(), T * width * sizeof(float));
    return 0;
}

// Router projection as the reference graph computes it (linear, deepseek_v4_graph.cpp:735-767).
static std::vector<float> router_logits(const vlr_moe_layer& L, const float* x, size_t T) {
    std::vector<float> logits(T * L.experts);
    for (size_t t = 0; t < T; ++t)
        for (size_t e = 0; e < L.experts; ++e) {
            double s = 0.0;
            for (size_t c = 0; c < L.hidden; ++c)
                s += static_cast<double>(x[t * L.hidden + c]) *
                     static_cast<double>(L.router[e * L.hidden + c]);
            logits[t * L.experts + e] = static_cast<float>(s);
        }
    return logits;
}

static int mv(const vlr_matrix& m, const float* x, float* y, std::vector<float>& scratch,
              unsigned threads) {
    const size_t nb = matrix_bytes(m.type, m.rows, m.cols);
    scratch.resize(m.rows);
    vi::QuantizedKernelLimits lim{1ull << 40, threads == 0 ? 1u : threads};
    auto r = vi::matvec_ggml_f32_transactional(m.type, bytes_of(m, nb), m.rows, m.cols,
                                               {x, m.cols}, scratch, {y, m.rows}, lim);
    return r ? 0 : -1;
}

// The layer loop of moe_forward/execute_expert (DeepSeek V4) or of the OLMoE forward, with the
// reference's own products. threads = QuantizedKernelLimits::max_threads for every matvec (the
// reference's RowWorkPool row split, bit-identical to serial). Optional logits_in replaces the
// router projection. Returns 0 on success.
int vlr_moe_forward(const vlr_moe_layer* Lp, const float* x, const uint32_t* token_ids,
                    size_t T, const float* logits_in, float* out, uint32_t* idx, float* weights,
                    unsigned threads) {
    const auto& L = *Lp;
    const size_t H = L.hidden, I = L.intermediate, E = L.experts, k = L.top_k;
    std::vector<float> logits = logits_in ? std::vector<float>(logits_in, logits_in + T * E)
                                          : router_logits(L, x, T);
    std::vector<float> gate(I), up(I), act(I), eo(H), scratch;
    if (L.score == 2) {
        // OLMoE router and combine, olmoe_runtime.cpp:1120-1137 and :1276-1286.
        std::vector<float> p(E);
        std::vector<uint32_t> order(E);
        for (size_t t = 0; t < T; ++t) {
            const float* l = logits.data() + t * E;
            float mx = l[0];
            for (size_t e = 1; e < E; ++e) mx = std::max(mx, l[e]);
            double den = 0.0;
            for (size_t e = 0; e < E; ++e) {
                p[e] = std::exp(l[e] - mx);
                den += static_cast<double>(p[e]);
                order[e] = static_cast<uint32_t>(e);
            }
            for (auto& v : p) v /= static_cast<float>(den);
            std::partial_sort(order.begin(), order.begin() + static_cast<std::ptrdiff_t>(k),
                              order.end(), [&](uint32_t a, uint32_t b) {
                                  if (p[a] != p[b]) return p[a] > p[b];
                                  return a < b;
                              });
            for (size_t s = 0; s < k; ++s) {
                idx[t * k + s] = order[s];
                weights[t * k + s] = p[order[s]];
            }
        }
        std::memset(out, 0, T * H * sizeof(float));
        for (size_t t = 0; t < T; ++t)
            for (size_t s = 0; s < k; ++s) {
                const uint32_t e = idx[t * k + s];
                if (mv(L.w1[e], x + t * H, gate.data(), scratch, threads) ||
                    mv(L.w3[e], x + t * H, up.data(), scratch, threads))
                    return -1;
                for (size_t c = 0; c < I; ++c)
                    act[c] = (gate[c] / (1.0F + std::exp(-gate[c]))) * up[c];
                if (mv(L.w2[e], act.data(), eo.data(), scratch, threads)) return -1;
                const float w = weights[t * k + s];
                for (size_t c = 0; c < H; ++c) out[t * H + c] += w * eo[c];
            }
        return 0;
    }
    if (L.score != 0) return -2;  // the reference has no sigmoid router
    {
        vastloom::Result<vi::DeepseekV4RouteResult> route =
            L.hash_routing
                ? vi::deepseek_v4_route_hash_logits(logits, {token_ids, T},
                                                    {L.tid2eid, L.vocab * k}, T, L.vocab, E, k,
                                                    L.route_scale)
                : vi::deepseek_v4_route_learned_logits(logits, {L.bias, E}, T, E, k,
                                                       L.route_scale);
        if (copy_route(route, idx, weights)) return -1;
    }
    // execute_expert, deepseek_v4_graph.cpp:1826-1895
    const auto expert = [&](const vlr_matrix& w1, const vlr_matrix& w3, const vlr_matrix& w2,
                            const float* xt, const float* rw, float limit, float* o) {
        if (mv(w1, xt, gate.data(), scratch, threads) || mv(w3, xt, up.data(), scratch, threads))
            return -1;
        for (size_t c = 0; c < I; ++c) {
            double g = static_cast<double>(gate[c]);
            double u = static_cast<double>(up[c]);
            if (limit > 0.0F) {
                g = std::min(g, static_cast<double>(limit));
                u = std::clamp(u, -static_cast<double>(limit), static_cast<double>(limit));
            }
            double v = g / (1.0 + std::exp(-g)) * u;
            if (rw) v *= static_cast<double>(*rw);
            act[c] = static_cast<float>(v);
        }
        return mv(w2, act.data(), o, scratch, threads);
    };
    std::vector<float> shared;
    if (L.shared_w1) {
        shared.resize(T * H);
        for (size_t t = 0; t < T; ++t)
            if (expert(*L.shared_w1, *L.shared_w3, *L.shared_w2, x + t * H, nullptr,
                       L.shared_swiglu_limit, shared.data() + t * H))
                return -1;
    }
    std::memset(out, 0, T * H * sizeof(float));
    for (size_t e = 0; e < E; ++e)
        for (size_t t = 0; t < T; ++t)
            for (size_t s = 0; s < k; ++s) {
                if (idx[t * k + s] != e) continue;
                if (expert(L.w1[e], L.w3[e], L.w2[e], x + t * H, &weights[t * k + s],
                           L.routed_swiglu_limit, eo.data()))
                    return -1;
                for (size_t c = 0; c < H; ++c) out[t * H + c] += eo[c];
            }
    if (!shared.empty())
        for (size_t i = 0; i < T * H; ++i) out[i] += shared[i];
    return 0;
}

// One tensor of a reduced DeepSeek V4 graph handed over from a fixture: kind 0 is f32 (n values),
// kind 1 is u32 (n values), kind 2 a packed ggml matrix (n bytes; type, rows, logical and storage
// columns, cache identity).
struct vlr_graph_tensor {
    const char* name;
    int kind;
    const void* data;
    size_t n;
    uint32_t ggml_type;
    size_t rows, logical_columns, storage_columns;
    uint64_t identity;
};

// The graph's numeric configuration by field name (deepseek_v4_reference.hpp:61-102).
struct vlr_graph_config_entry {
    const char* key;
    double value;
};

namespace {

// A matvec accelerator that declines every row (so the graph computes it on its own CPU path) and
// records what it was offered: the matrix's cache identity and the row's padded input, in call
// order. Through it a test sees the graph's file-static moe_forward from outside: the MoE input
// (the shared expert's gate rows) and every expert's down-projection input.
class OfferRecorder final : public vi::DeepseekV4MatvecAccelerator {
public:
    OfferRecorder(uint64_t* ids, float* rows, size_t cols, size_t cap)
        : ids_(ids), rows_(rows), cols_(cols), cap_(cap) {}
    vastloom::Result<bool> matvec(const vi::DeepseekV4PackedMatrix& matrix, std::span<const float> input,
                                  std::span<float>) override {
        if (count_ < cap_) {
            ids_[count_] = matrix.cache_identity;
            float* row = rows_ + count_ * cols_;
            std::fill(row, row + cols_, 0.0F);
            std::copy_n(input.begin(), std::min(cols_, input.size()), row);
        }
        ++count_;
        return false;
    }
    size_t count() const { return count_; }

private:
    uint64_t* ids_;
    float* rows_;
    size_t cols_, cap_, count_ = 0;
};

bool set_config(vi::DeepseekV4ReferenceConfig& c, const std::string& key, double v) {
    const auto z = static_cast<size_t>(v);
    const auto f = static_cast<float>(v);
    if (key == "vocabulary_size") c.vocabulary_size = z;
    else if (key == "width") c.width = z;
    else if (key == "intermediate_width") c.intermediate_width = z;
    else if (key == "layers") c.layer_count = z;
    else if (key == "hash_layers") c.hash_layer_count = z;
    else if (key == "mtp_layers") c.mtp_layer_count = z;
    else if (key == "heads") c.head_count = z;
    else if (key == "experts") c.expert_count = z;
    else if (key == "experts_per_token") c.experts_per_token = z;
    else if (key == "query_lora_rank") c.query_lora_rank = z;
    else if (key == "head_width") c.head_width = z;
    else if (key == "rope_width") c.rope_width = z;
    else if (key == "output_groups") c.output_groups = z;
    else if (key == "output_lora_rank") c.output_lora_rank = z;
    else if (key == "window_size") c.window_size = z;
    else if (key == "compression_ratios") c.compression_ratios.push_back(z);
    else if (key == "mtp_compression_ratios") c.mtp_compression_ratios.push_back(z);
    else if (key == "compression_rope_theta") c.compression_rope_theta = f;
    else if (key == "original_context") c.original_context = z;
    else if (key == "rope_theta") c.rope_theta = f;
    else if (key == "rope_factor") c.rope_factor = f;
    else if (key == "beta_fast") c.beta_fast = f;
    else if (key == "beta_slow") c.beta_slow = f;
    else if (key == "index_heads") c.index_head_count = z;
    else if (key == "index_head_width") c.index_head_width = z;
    else if (key == "index_top_k") c.index_top_k = z;
    else if (key == "hyper_multiplier") c.hyper_multiplier = z;
    else if (key == "sinkhorn_iterations") c.sinkhorn_iterations = z;
    else if (key == "norm_epsilon") c.norm_epsilon = f;
    else if (key == "hyper_epsilon") c.hyper_epsilon = f;
    else if (key == "route_scale") c.route_scale = f;
    else if (key == "swiglu_limit") c.swiglu_limit = f;
    else return false;
    return true;
}

}  // namespace

// deepseek_v4_reference_prefill (deepseek_v4_graph.cpp:4651) over a reduced graph built from the
// given configuration entries (list-valued fields repeat their key, in order) and tensors.
// Outputs: logits [V]; route indices / weights [(layers + mtp_layers) x T x k], main layers first;
// every matvec row offered to the accelerator (only packed matrices are offered) as
// (identity, first rec_cols inputs), up to rec_cap rows, with the total count in *rec_n.
// Returns 0, or -1 with the reference's error message in err.
int vlr_graph_prefill(const vlr_graph_config_entry* cfg, size_t n_cfg, const vlr_graph_tensor* tensors,
                      size_t n_tensors, const uint32_t* token_ids, size_t T, float* logits, size_t V,
                      uint32_t* route_idx, float* route_w, size_t n_route_layers, uint64_t* rec_ids,
                      float* rec_rows, size_t rec_cols, size_t rec_cap, size_t* rec_n, char* err,
                      size_t err_cap) {
    const auto fail = [&](const std::string& m) {
        if (err && err_cap) {
            std::strncpy(err, m.c_str(), err_cap - 1);
            err[err_cap - 1] = '\0';
        }
        return -1;
    };
    try {
        vi::DeepseekV4ReferenceGraph graph;
        for (size_t i = 0; i < n_cfg; ++i)
            if (!set_config(graph.config, cfg[i].key, cfg[i].value))
                return fail(std::string("unknown configuration key ") + cfg[i].key);
        for (size_t i = 0; i < n_tensors; ++i) {
            const auto& t = tensors[i];
            if (t.kind == 0) {
                const auto* p = static_cast<const float*>(t.data);
                graph.float_tensors.emplace(t.name, std::vector<float>(p, p + t.n));
            } else if (t.kind == 1) {
                const auto* p = static_cast<const uint32_t*>(t.data);
                graph.integer_tensors.emplace(t.name, std::vector<uint32_t>(p, p + t.n));
            } else {
                const auto* p = static_cast<const std::byte*>(t.data);
                vi::DeepseekV4PackedMatrix m(t.ggml_type, t.rows, t.logical_columns, t.storage_columns,
                                             std::vector<std::byte>(p, p + t.n));
                m.cache_identity = t.identity;
                graph.packed_matrices.emplace(t.name, std::move(m));
            }
        }
        OfferRecorder recorder(rec_ids, rec_rows, rec_cols, rec_cap);
        graph.accelerator = &recorder;
        auto r = vi::deepseek_v4_reference_prefill(graph, {token_ids, T});
        if (!r) return fail(r.error().message + ": " + r.error().context);
        const auto& res = r.value();
        if (res.logits.size() != V) return fail("logit count differs from the vocabulary");
        std::memcpy(logits, res.logits.data(), V * sizeof(float));
        const size_t k = graph.config.experts_per_token;
        size_t layer = 0;
        for (const auto* traces : {&res.layers, &res.mtp_layers})
            for (const auto& tr : *traces) {
                if (layer >= n_route_layers) return fail("more routed layers than route buffers");
                if (tr.route.indices.size() != T * k || tr.route.weights.size() != T * k)
                    return fail("route shape differs from tokens x top_k");
                std::memcpy(route_idx + layer * T * k, tr.route.indices.data(), T * k * sizeof(uint32_t));
                std::memcpy(route_w + layer * T * k, tr.route.weights.data(), T * k * sizeof(float));
                ++layer;
            }
        if (layer != n_route_layers) return fail("fewer routed layers than route buffers");
        *rec_n = recorder.count();
        return 0;
    } catch (const std::exception& e) {
        return fail(e.what());
    }
}

}  // extern "C"
