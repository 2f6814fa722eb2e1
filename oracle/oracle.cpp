// TEST INFRASTRUCTURE ONLY -- the parity checker, never the product.
//
// CPU restatement of the arithmetic of ezzy0654/aps2026's GPU kernels for the
// non-GEMM prefill path (src/tensor.cu), written from the reference's
// semantics. Only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline / reference arm load this library; the aps2026_b200 package never
// does, and it has no CPU fallback.
//
// Each function follows the reference GPU KERNEL (not its CPU twin where the
// two differ) in operation order, including the places where nvcc contracts
// a multiply feeding an add into one fused multiply-add: those are written as
// explicit std::fma here and the file is built with -ffp-contract=off so the
// host compiler adds no others. Reductions are serial in ascending index, as
// the reference keeps them. The result is meant to equal the reference
// kernels bit for bit; tests pin that on the GPU against the reference's own
// kernels (oracle/_ref) and on the CPU against the reference's host ops.
//
// Built by oracle/Makefile into oracle/liboracle.so (g++ -O3 -fopenmp).

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <limits>
#include <unordered_map>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// k_layer_norm's moments (src/tensor.cu:2063-2128): mean = serial ascending
// sum / h; var = serial ascending sum of (x - mean)^2 where nvcc fuses
// `var += t * t` into fma(t, t, var); inv = 1 / sqrtf(var / h + eps).
inline void ln_moments(const float* s, std::size_t h, float eps, float& mean,
                       float& inv) {
    float sum = 0.0f;
    for (std::size_t j = 0; j < h; ++j) sum += s[j];
    const float m = sum / static_cast<float>(h);
    float var = 0.0f;
    for (std::size_t j = 0; j < h; ++j) {
        const float t = s[j] - m;
        var = std::fma(t, t, var);
    }
    mean = m;
    inv = 1.0f / std::sqrt(var / static_cast<float>(h) + eps);
}

// ln_write (src/tensor.cu:2031-2056): y = fma((s - mean) * inv, w, b).
inline void ln_write(const float* s, const float* w, const float* b, float* y,
                     std::size_t h, float mean, float inv) {
    for (std::size_t j = 0; j < h; ++j)
        y[j] = std::fma((s[j] - mean) * inv, w[j], b[j]);
}

// k_moe_combine's accumulation (src/tensor.cu:1979-1986): value starts at
// 0, then value += 0.5 * row for the lower expert id first; nvcc fuses each
// `+=` into fma(0.5, row, value).
inline float combine_one(float lo, float hi) {
    float v = 0.0f;
    v = std::fma(0.5f, lo, v);
    v = std::fma(0.5f, hi, v);
    return v;
}

}  // namespace

extern "C" {

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

// k_gather_rows (src/tensor.cu:2635-2642): out[i,:] = x[rows[i],:].
void orc_gather_rows(const float* x, std::size_t h, const std::uint32_t* rows,
                     std::size_t count, float* out) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < static_cast<long long>(count); ++i)
        std::memcpy(out + static_cast<std::size_t>(i) * h,
                    x + static_cast<std::size_t>(rows[i]) * h,
                    h * sizeof(float));
}

// k_layer_norm (src/tensor.cu:2130-2142).
void orc_layer_norm(const float* x, const float* w, const float* b, float* y,
                    std::size_t rows, std::size_t h, float eps) {
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < static_cast<long long>(rows); ++r) {
        const std::size_t base = static_cast<std::size_t>(r) * h;
        float mean, inv;
        ln_moments(x + base, h, eps, mean, inv);
        ln_write(x + base, w, b, y + base, h, mean, inv);
    }
}

// k_add_layer_norm (src/tensor.cu:2144-2178): x += residual (written back),
// then LayerNorm of the sum.
void orc_add_layer_norm(float* x, const float* res, const float* w,
                        const float* b, float* y, std::size_t rows,
                        std::size_t h, float eps) {
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < static_cast<long long>(rows); ++r) {
        const std::size_t base = static_cast<std::size_t>(r) * h;
        for (std::size_t j = 0; j < h; ++j) x[base + j] += res[base + j];
        float mean, inv;
        ln_moments(x + base, h, eps, mean, inv);
        ln_write(x + base, w, b, y + base, h, mean, inv);
    }
}

// rope_table (src/tensor.cu:2716-2724): float powf / cosf / sinf on host.
void orc_rope_table(std::size_t max_seq, std::size_t head_dim, float theta,
                    float* cosine, float* sine) {
    const std::size_t half = head_dim / 2;
    for (std::size_t p = 0; p < max_seq; ++p)
        for (std::size_t j = 0; j < half; ++j) {
            const float inv = std::pow(theta, -2.0f * static_cast<float>(j) /
                                                  static_cast<float>(head_dim));
            cosine[p * half + j] = std::cos(static_cast<float>(p) * inv);
            sine[p * half + j] = std::sin(static_cast<float>(p) * inv);
        }
}

// k_rope (src/tensor.cu:2180-2197), applied to q then k. nvcc fuses
// `x0 * c - x1 * s` into fma(x0, c, -(x1 * s)) and `x1 * c + x0 * s` into
// fma(x0, s, x1 * c) -- the second product is the fused one there (pinned
// against the reference kernel's own output, tests/golden/ref_kernels.npz).
static void rope_one(float* x, const std::uint32_t* row_pos,
                     const float* cosine, const float* sine, std::size_t rows,
                     std::size_t heads, std::size_t head_dim) {
    const std::size_t half = head_dim / 2;
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < static_cast<long long>(rows); ++r) {
        const std::size_t t = static_cast<std::size_t>(row_pos[r]) * half;
        for (std::size_t hd = 0; hd < heads; ++hd) {
            float* base = x + (static_cast<std::size_t>(r) * heads + hd) * head_dim;
            for (std::size_t j = 0; j < half; ++j) {
                const float c = cosine[t + j], s = sine[t + j];
                const float x0 = base[j], x1 = base[j + half];
                base[j] = std::fma(x0, c, -(x1 * s));
                base[j + half] = std::fma(x0, s, x1 * c);
            }
        }
    }
}

void orc_rope(float* q, float* k, const std::uint32_t* row_pos,
              std::size_t rows, std::size_t q_heads, std::size_t kv_heads,
              std::size_t head_dim, const float* cosine, const float* sine) {
    rope_one(q, row_pos, cosine, sine, rows, q_heads, head_dim);
    rope_one(k, row_pos, cosine, sine, rows, kv_heads, head_dim);
}

// Softmax section of k_attention_tree_gqa4 on a standalone score matrix.
// Scores are scaled (src/tensor.cu:2526, stored before the softmax reads
// them, so no fusion with the subtraction), window rule :2435-2439, max via
// fmaxf, e = (float)exp((double)(s - max)) (:2563-2564), denominator summed
// serially in ascending key order (:2572-2573), p = e / denom (:2584).
void orc_causal_softmax(const float* scores, float* probs, std::size_t heads,
                        std::size_t T, std::size_t ld, float scale,
                        std::size_t window) {
#pragma omp parallel
    {
        std::vector<float> e(T);
#pragma omp for schedule(dynamic, 16)
        for (long long hr = 0; hr < static_cast<long long>(heads * T); ++hr) {
            const std::size_t i = static_cast<std::size_t>(hr) % T;
            const float* s = scores + static_cast<std::size_t>(hr) * ld;
            float* p = probs + static_cast<std::size_t>(hr) * ld;
            const std::size_t begin = i + 1 > window ? i + 1 - window : 0;
            float maxv = -3.402823466e+38F;
            for (std::size_t j = begin; j <= i; ++j) {
                e[j] = s[j] * scale;
                maxv = std::fmax(maxv, e[j]);
            }
            float denom = 0.0f;
            for (std::size_t j = begin; j <= i; ++j) {
                e[j] = static_cast<float>(std::exp(static_cast<double>(e[j] - maxv)));
                denom += e[j];
            }
            for (std::size_t j = 0; j < T; ++j)
                p[j] = (j >= begin && j <= i) ? e[j] / denom : 0.0f;
        }
    }
}

// k_moe_top2 + k_moe_offsets_work + k_moe_fill_stable
// (src/tensor.cu:1293-1418), sequentially. Queues (may be null) are filled
// with 0xFFFFFFFF first, as the memsets at :2804-2809 do.
void orc_moe_route(const float* logits, std::size_t T, std::size_t E,
                   float quantum, float tie_eps, std::uint8_t* routes,
                   std::uint32_t* counts, std::uint32_t* offsets,
                   std::uint32_t* assignment_rows,
                   std::uint32_t* route_positions, std::uint32_t* we64,
                   std::uint32_t* ws64, std::uint32_t* we128,
                   std::uint32_t* ws128) {
    std::vector<float> scores(E);
    for (std::size_t e = 0; e < E; ++e) counts[e] = 0;
    for (std::size_t t = 0; t < T; ++t) {
        for (std::size_t e = 0; e < E; ++e) {
            const float score = logits[t * E + e];
            const float rounded =
                std::floor(std::fabs(score) / quantum + 0.5f) * quantum;
            scores[e] = score < 0.0f ? -rounded : rounded;
        }
        int first = -1;
        float first_value = -3.402823466e+38F;
        for (int e = 0; e < static_cast<int>(E); ++e)
            if (first < 0 || scores[e] > first_value + tie_eps) {
                first = e;
                first_value = scores[e];
            }
        int second = -1;
        float second_value = -3.402823466e+38F;
        for (int e = 0; e < static_cast<int>(E); ++e) {
            if (e == first) continue;
            if (second < 0 || scores[e] > second_value + tie_eps) {
                second = e;
                second_value = scores[e];
            }
        }
        routes[2 * t] = static_cast<std::uint8_t>(first);
        routes[2 * t + 1] = static_cast<std::uint8_t>(second);
        counts[first] += 1;
        counts[second] += 1;
    }
    offsets[0] = 0;
    for (std::size_t e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
    const std::size_t n64 = (2 * T + 63) / 64 + E, n128 = (2 * T + 127) / 128 + E;
    // Unused entries: 0xFFFFFFFF in the expert queues (the reference's
    // memsets); the start queues get the same marker (the reference leaves
    // them as they were, so tests compare only used start entries with it).
    for (std::size_t i = 0; i < n64; ++i) {
        if (we64) we64[i] = 0xFFFFFFFFu;
        if (ws64) ws64[i] = 0xFFFFFFFFu;
    }
    for (std::size_t i = 0; i < n128; ++i) {
        if (we128) we128[i] = 0xFFFFFFFFu;
        if (ws128) ws128[i] = 0xFFFFFFFFu;
    }
    std::size_t w64 = 0, w128 = 0;
    for (std::size_t e = 0; e < E; ++e) {
        for (std::uint32_t c = 0; c < (counts[e] + 63) / 64; ++c, ++w64) {
            if (we64) we64[w64] = static_cast<std::uint32_t>(e);
            if (ws64) ws64[w64] = offsets[e] + c * 64;
        }
        for (std::uint32_t c = 0; c < (counts[e] + 127) / 128; ++c, ++w128) {
            if (we128) we128[w128] = static_cast<std::uint32_t>(e);
            if (ws128) ws128[w128] = offsets[e] + c * 128;
        }
    }
    std::vector<std::uint32_t> cursor(offsets, offsets + E);
    for (std::size_t t = 0; t < T; ++t)
        for (std::size_t slot = 0; slot < 2; ++slot) {
            const std::uint32_t e = routes[2 * t + slot];
            const std::uint32_t pos = cursor[e]++;
            assignment_rows[pos] = static_cast<std::uint32_t>(t);
            route_positions[2 * t + slot] = pos;
        }
}

// k_attention_tree_gqa4 (src/tensor.cu:2425-2633): per (row, kv head), the
// keys are the row's ancestor chain [begin, pos] (begin = pos + 1 - window
// when positive, :2435-2439); for each of the `group` query heads the score
// of key w is the 128-wide dot product in four accumulators over d mod 4,
// each a fused multiply-add chain in ascending d (:2517-2524), combined as
// (acc0 + acc1) + (acc2 + acc3), times 1/sqrtf(head_dim) (:2448, :2526);
// then the softmax of orc_causal_softmax (max, (float)exp((double)(s-max)),
// serial ascending denominator, division, :2549-2585); then
// out[d] = fma chain of p[w] * v[chain[w]][d] in ascending w (:2596-2631).
void orc_attention_tree(const float* q, const float* k, const float* v, float* out,
                        const std::uint32_t* row_pos, const std::uint32_t* anc,
                        std::size_t anc_stride, std::size_t rows, std::size_t q_heads,
                        std::size_t kv_heads, std::size_t head_dim, std::size_t window) {
    const std::size_t group = q_heads / kv_heads;
    const float scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
#pragma omp parallel
    {
        std::vector<float> sc;
#pragma omp for schedule(dynamic, 8)
        for (long long task = 0; task < static_cast<long long>(rows * kv_heads); ++task) {
            const std::size_t row = static_cast<std::size_t>(task) / kv_heads;
            const std::size_t kh = static_cast<std::size_t>(task) % kv_heads;
            const std::size_t pos = row_pos[row];
            const std::size_t begin = pos + 1 > window ? pos + 1 - window : 0;
            const std::size_t W = pos - begin + 1;
            const std::uint32_t* chain = anc + row * anc_stride + begin;
            sc.resize(W);
            for (std::size_t g = 0; g < group; ++g) {
                const float* qv = q + (row * q_heads + kh * group + g) * head_dim;
                for (std::size_t w = 0; w < W; ++w) {
                    const float* kv = k + (static_cast<std::size_t>(chain[w]) * kv_heads + kh) * head_dim;
                    float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
                    std::size_t d = 0;
                    for (; d + 4 <= head_dim; d += 4) {
                        acc0 = std::fma(qv[d + 0], kv[d + 0], acc0);
                        acc1 = std::fma(qv[d + 1], kv[d + 1], acc1);
                        acc2 = std::fma(qv[d + 2], kv[d + 2], acc2);
                        acc3 = std::fma(qv[d + 3], kv[d + 3], acc3);
                    }
                    float score = (acc0 + acc1) + (acc2 + acc3);
                    for (; d < head_dim; ++d) score = std::fma(qv[d], kv[d], score);
                    sc[w] = score * scale;
                }
                float maxv = -3.402823466e+38F;
                for (std::size_t w = 0; w < W; ++w) maxv = std::fmax(maxv, sc[w]);
                float denom = 0.0f;
                for (std::size_t w = 0; w < W; ++w) {
                    sc[w] = static_cast<float>(std::exp(static_cast<double>(sc[w] - maxv)));
                    denom += sc[w];
                }
                for (std::size_t w = 0; w < W; ++w) sc[w] = sc[w] / denom;
                float* o = out + (row * q_heads + kh * group + g) * head_dim;
                for (std::size_t dd = 0; dd < head_dim; ++dd) {
                    float value = 0.0f;
                    for (std::size_t w = 0; w < W; ++w)
                        value = std::fma(sc[w], v[(static_cast<std::size_t>(chain[w]) * kv_heads + kh) * head_dim + dd],
                                         value);
                    o[dd] = value;
                }
            }
        }
    }
}

// k_silu_mul (src/tensor.cu:2001-2010) on strided rows.
void orc_silu_mul(const float* gate, std::size_t ldg, const float* up,
                  std::size_t ldu, float* out, std::size_t ldo,
                  std::size_t rows, std::size_t cols) {
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < static_cast<long long>(rows); ++r)
        for (std::size_t c = 0; c < cols; ++c) {
            const float x = gate[static_cast<std::size_t>(r) * ldg + c];
            const float act =
                x / (1.0f + static_cast<float>(std::exp(static_cast<double>(-x))));
            out[static_cast<std::size_t>(r) * ldo + c] =
                act * up[static_cast<std::size_t>(r) * ldu + c];
        }
}

// k_moe_combine (src/tensor.cu:1968-1988).
void orc_moe_combine(const float* expert_out, const std::uint8_t* routes,
                     const std::uint32_t* route_positions, float* out,
                     std::size_t T, std::size_t h) {
#pragma omp parallel for schedule(static)
    for (long long t = 0; t < static_cast<long long>(T); ++t) {
        const std::uint8_t e0 = routes[2 * t], e1 = routes[2 * t + 1];
        const std::size_t p0 = route_positions[2 * t], p1 = route_positions[2 * t + 1];
        const std::size_t lo = e0 < e1 ? p0 : p1, hi = e0 < e1 ? p1 : p0;
        for (std::size_t d = 0; d < h; ++d)
            out[static_cast<std::size_t>(t) * h + d] =
                combine_one(expert_out[lo * h + d], expert_out[hi * h + d]);
    }
}

// Fused combine -> carried residual add -> LayerNorm: k_moe_combine
// (src/tensor.cu:1968-1988) then k_add_layer_norm (:2144-2178) with
// x = combine output and residual = carry (src/layer.cu:283-287).
void orc_moe_combine_add_layer_norm(const float* expert_out,
                                    const std::uint8_t* routes,
                                    const std::uint32_t* route_positions,
                                    const float* carry, const float* w,
                                    const float* b, float* x_out, float* y,
                                    std::size_t T, std::size_t h, float eps) {
    orc_moe_combine(expert_out, routes, route_positions, x_out, T, h);
    orc_add_layer_norm(x_out, carry, w, b, y, T, h, eps);
}

// k_add (src/tensor.cu:1990-1993).
void orc_add(float* a, const float* b, std::size_t n) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < static_cast<long long>(n); ++i) a[i] += b[i];
}

// Prefix trie of PhiTinyMoEModel::generate (src/model.cu:64-117): nodes are
// numbered in creation order walking prompts in order; key = (parent+1)<<32
// | token with parent 0xFFFFFFFF as the virtual root; a new node's ancestor
// chain is the running chain of the prompt being walked. Returns the node
// count, or -1 on an invalid token.
long long orc_prefix_trie(const std::int32_t* ids, const std::uint32_t* lens,
                          std::size_t batch, std::size_t vocab,
                          std::uint32_t* token_node, std::uint32_t* node_token,
                          std::uint32_t* node_depth, std::uint32_t* node_anc,
                          std::size_t anc_stride) {
    std::unordered_map<std::uint64_t, std::uint32_t> children;
    std::vector<std::uint32_t> chain(anc_stride);
    std::size_t row = 0, nodes = 0;
    for (std::size_t b = 0; b < batch; ++b) {
        std::uint32_t parent = 0xFFFFFFFFu;
        for (std::size_t si = 0; si < lens[b]; ++si, ++row) {
            const std::int32_t token = ids[row];
            if (token < 0 || static_cast<std::size_t>(token) >= vocab) return -1;
            const std::uint64_t key =
                (static_cast<std::uint64_t>(parent + 1u) << 32) |
                static_cast<std::uint32_t>(token);
            auto it = children.find(key);
            std::uint32_t node;
            if (it == children.end()) {
                node = static_cast<std::uint32_t>(nodes++);
                node_token[node] = static_cast<std::uint32_t>(token);
                node_depth[node] = static_cast<std::uint32_t>(si);
                chain[si] = node;
                if (node_anc) {
                    std::uint32_t* a = node_anc + static_cast<std::size_t>(node) * anc_stride;
                    std::memset(a, 0, anc_stride * sizeof(std::uint32_t));
                    std::memcpy(a, chain.data(), (si + 1) * sizeof(std::uint32_t));
                }
                children.emplace(key, node);
            } else {
                node = it->second;
                chain[si] = node;
            }
            token_node[row] = node;
            parent = node;
        }
    }
    return static_cast<long long>(nodes);
}

}  // extern "C"
