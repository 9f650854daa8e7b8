// q38_oracle.cpp -- CPU restatement of the reference's gated full attention
// and Gated DeltaNet cores. TEST INFRASTRUCTURE ONLY (parity checker and timed
// CPU baseline); the product library never links it. See q38_oracle.h for the
// arithmetic contract and the reference lines each function follows.
//
// Build: g++ -O3 -ffp-contract=off -fopenmp -fPIC -shared (oracle/Makefile).
#include "q38_oracle.h"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <omp.h>

namespace {

constexpr float kRmsEps = 1e-6f;  // Q38_RMS_EPS, src/model/mod.rs:26
constexpr size_t kParallelMinWork = size_t(1) << 18;  // src/kernel/mod.rs:12

int g_threads = 0;  // 0: OpenMP default (all cores)

int threads() { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

// q38_parallel_over, src/kernel/mod.rs:19-21: split only when there are at
// least two items and the total work clears 2^18 element-operations.
bool parallel_over(size_t items, size_t per_item) {
    if (items < 2) return false;
    if (per_item != 0 && items > SIZE_MAX / per_item) return true;
    return items * per_item >= kParallelMinWork;
}

// rms_scale, ops.rs:476-483: f64 sum of squares, mean cast to f32.
float rms_scale(const float *v, size_t n) {
    double sum = 0.0;
    for (size_t i = 0; i < n; ++i) sum += double(v[i]) * double(v[i]);
    const float mean = float(sum / double(n));
    return 1.0f / std::sqrt(mean + kRmsEps);
}

// rmsnorm_inplace, ops.rs:493-498: x = x * scale * w (left to right).
void rmsnorm_inplace(float *v, const float *w, size_t n) {
    const float scale = rms_scale(v, n);
    for (size_t i = 0; i < n; ++i) v[i] = v[i] * scale * w[i];
}

// ops.rs:500-516.
inline float sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }
inline float silu(float x) { return x / (1.0f + std::exp(-x)); }
inline float softplus(float x) {
    if (x > 20.0f) return x;
    return std::log(1.0f + std::exp(x));
}

// l2norm, ops.rs:562-571: 1 / max(sqrt((f32) sum_f64), eps).
void l2norm(float *v, size_t n) {
    double sum = 0.0;
    for (size_t i = 0; i < n; ++i) sum += double(v[i]) * double(v[i]);
    const float norm = std::sqrt(float(sum));
    const float scale = 1.0f / (norm > kRmsEps ? norm : kRmsEps);
    for (size_t i = 0; i < n; ++i) v[i] *= scale;
}

// dot_128, ops.rs:573-579: sequential fma chain from 0.
inline float dot_128(const float *a, const float *b) {
    float t = 0.0f;
    for (int i = 0; i < Q38O_LINEAR_HEAD_DIM; ++i) t = std::fma(a[i], b[i], t);
    return t;
}

// mad_dot_128, ops.rs:584-591: out = fma(in, s, out), then fma-chain against r.
inline float mad_dot_128(float *out, const float *in, float s, const float *r) {
    float t = 0.0f;
    for (int i = 0; i < Q38O_LINEAR_HEAD_DIM; ++i) {
        out[i] = std::fma(in[i], s, out[i]);
        t = std::fma(out[i], r[i], t);
    }
    return t;
}

// rope, ops.rs:595-610: NEOX half rotation of lanes [0,64) of every head,
// pair (i, i+32) at angle theta_i, theta_0 = pos, theta_{i+1} = theta_i*scale.
void rope(float *v, size_t heads, uint32_t position) {
    const float theta_scale = std::pow(10000000.0f, -2.0f / 64.0f);
    for (size_t h = 0; h < heads; ++h) {
        float *x = v + h * Q38O_ATTN_HEAD_DIM;
        float theta = float(position);
        for (int p = 0; p < 32; ++p) {
            const float c = std::cos(theta);
            const float s = std::sin(theta);
            const float x0 = x[p];
            const float x1 = x[p + 32];
            x[p] = x0 * c - x1 * s;
            x[p + 32] = x0 * s + x1 * c;
            theta *= theta_scale;
        }
    }
}

// Round-to-nearest-even to bf16, returned as the f32 it represents.
float round_bf16(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
        u |= 0x00400000u;  // quiet NaN
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);
    }
    u &= 0xffff0000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// Per-head attention of full_core, ops.rs:877-914.
void full_core_head(size_t head, const float *q, const float *gate, float *head_scores,
                    float *head_out, const float *key_cache, const float *value_cache,
                    size_t full_index, size_t context_length, size_t positions) {
    const size_t groups = Q38O_ATTN_HEADS / Q38O_ATTN_KV_HEADS;
    const float score_scale = 1.0f / std::sqrt(float(Q38O_ATTN_HEAD_DIM));
    const size_t kv_head = head / groups;
    const float *qh = q + head * Q38O_ATTN_HEAD_DIM;
    float maximum = -INFINITY;
    for (size_t p = 0; p < positions; ++p) {
        const size_t row = (full_index * context_length + p) * Q38O_ATTN_KV_DIM +
                           kv_head * Q38O_ATTN_HEAD_DIM;
        const float *k = key_cache + row;
        float score = 0.0f;
        for (int i = 0; i < Q38O_ATTN_HEAD_DIM; ++i) score = std::fma(qh[i], k[i], score);
        score *= score_scale;
        head_scores[p] = score;
        if (score > maximum) maximum = score;
    }
    float denominator = 0.0f;
    for (size_t p = 0; p < positions; ++p) {
        head_scores[p] = std::exp(head_scores[p] - maximum);
        denominator += head_scores[p];
    }
    for (int i = 0; i < Q38O_ATTN_HEAD_DIM; ++i) head_out[i] = 0.0f;
    for (size_t p = 0; p < positions; ++p) {
        const size_t row = (full_index * context_length + p) * Q38O_ATTN_KV_DIM +
                           kv_head * Q38O_ATTN_HEAD_DIM;
        const float *v = value_cache + row;
        const float probability = head_scores[p] / denominator;
        for (int i = 0; i < Q38O_ATTN_HEAD_DIM; ++i)
            head_out[i] = std::fma(probability, v[i], head_out[i]);
    }
    const float *g = gate + head * Q38O_ATTN_HEAD_DIM;
    for (int i = 0; i < Q38O_ATTN_HEAD_DIM; ++i) head_out[i] *= sigmoid(g[i]);
}

// Steps (1)-(4) of full_core (ops.rs:832-866): split q/gate, q/k RMSNorm,
// RoPE, cache append. Returns -1 when the cache row is out of range.
int full_core_prepare(const float *q_norm, const float *k_norm, const float *q_and_gate,
                      float *key, const float *value, float *q, float *gate, float *key_cache,
                      float *value_cache, size_t cache_rows, size_t context_length,
                      uint32_t position, size_t layer, int kv_round_bf16) {
    for (size_t h = 0; h < Q38O_ATTN_HEADS; ++h) {
        const float *src = q_and_gate + h * 2 * Q38O_ATTN_HEAD_DIM;
        std::memcpy(q + h * Q38O_ATTN_HEAD_DIM, src, Q38O_ATTN_HEAD_DIM * sizeof(float));
        std::memcpy(gate + h * Q38O_ATTN_HEAD_DIM, src + Q38O_ATTN_HEAD_DIM,
                    Q38O_ATTN_HEAD_DIM * sizeof(float));
        rmsnorm_inplace(q + h * Q38O_ATTN_HEAD_DIM, q_norm, Q38O_ATTN_HEAD_DIM);
    }
    for (size_t h = 0; h < Q38O_ATTN_KV_HEADS; ++h)
        rmsnorm_inplace(key + h * Q38O_ATTN_HEAD_DIM, k_norm, Q38O_ATTN_HEAD_DIM);
    rope(q, Q38O_ATTN_HEADS, position);
    rope(key, Q38O_ATTN_KV_HEADS, position);
    if (kv_round_bf16 & 2)
        for (int i = 0; i < Q38O_ATTN_Q_DIM; ++i) q[i] = round_bf16(q[i]);

    const size_t full_index = layer / 4;
    const size_t row = full_index * context_length + size_t(position);
    if (row + 1 > cache_rows) return -1;
    float *kc = key_cache + row * Q38O_ATTN_KV_DIM;
    float *vc = value_cache + row * Q38O_ATTN_KV_DIM;
    for (int i = 0; i < Q38O_ATTN_KV_DIM; ++i) {
        kc[i] = (kv_round_bf16 & 1) ? round_bf16(key[i]) : key[i];
        vc[i] = (kv_round_bf16 & 1) ? round_bf16(value[i]) : value[i];
    }
    return 0;
}

}  // namespace

extern "C" {

void q38o_set_threads(int n) { g_threads = n; }
int q38o_get_threads(void) { return threads(); }

float q38o_rms_scale(const float *v, size_t n) { return rms_scale(v, n); }
void q38o_l2norm(float *v, size_t n) { l2norm(v, n); }
void q38o_rope(float *v, size_t heads, uint32_t position) { rope(v, heads, position); }
float q38o_sigmoid(float x) { return sigmoid(x); }
float q38o_silu(float x) { return silu(x); }
float q38o_softplus(float x) { return softplus(x); }
float q38o_round_bf16(float x) { return round_bf16(x); }

int q38o_linear_core(const float *conv_w, const float *dt_bias, const float *ssm_a,
                     const float *ssm_norm, float *conv_state, float *delta_state, float *qkv,
                     const float *z, float *beta, float *alpha, float *attention) {
    // (1) depthwise causal conv, kernel 4, multiply then add (ops.rs:665-676).
    for (size_t c = 0; c < Q38O_LINEAR_QKV_DIM; ++c) {
        float *s = conv_state + c * 3;
        const float *w = conv_w + c * 4;
        float v = s[0] * w[0];
        v += s[1] * w[1];
        v += s[2] * w[2];
        v += qkv[c] * w[3];
        s[0] = s[1];
        s[1] = s[2];
        s[2] = qkv[c];
        qkv[c] = v;
    }
    // (2) SiLU (ops.rs:677).
    for (size_t c = 0; c < Q38O_LINEAR_QKV_DIM; ++c) qkv[c] = silu(qkv[c]);
    // (3) L2-norm of q and k heads (ops.rs:679-684).
    float *query = qkv;
    float *key = qkv + Q38O_LINEAR_QK_DIM;
    const float *value = qkv + 2 * Q38O_LINEAR_QK_DIM;
    for (size_t h = 0; h < Q38O_LINEAR_QK_HEADS; ++h) {
        l2norm(query + h * Q38O_LINEAR_HEAD_DIM, Q38O_LINEAR_HEAD_DIM);
        l2norm(key + h * Q38O_LINEAR_HEAD_DIM, Q38O_LINEAR_HEAD_DIM);
    }
    // (4) gates (ops.rs:685-688).
    for (size_t h = 0; h < Q38O_LINEAR_V_HEADS; ++h) {
        beta[h] = sigmoid(beta[h]);
        alpha[h] = ssm_a[h] * softplus(alpha[h] + dt_bias[h]);
    }
    // (5) delta rule per value head (ops.rs:690-733).
    const float query_scale = 1.0f / std::sqrt(float(Q38O_LINEAR_HEAD_DIM));
    const size_t head_elems = size_t(Q38O_LINEAR_HEAD_DIM) * Q38O_LINEAR_HEAD_DIM;
    const bool par = parallel_over(Q38O_LINEAR_V_HEADS, head_elems);
#pragma omp parallel for schedule(static) num_threads(threads()) if (par)
    for (int vh = 0; vh < Q38O_LINEAR_V_HEADS; ++vh) {
        float *state = delta_state + size_t(vh) * head_elems;
        float *out = attention + size_t(vh) * Q38O_LINEAR_HEAD_DIM;
        const int kh = vh % Q38O_LINEAR_QK_HEADS;
        const float *qh = query + kh * Q38O_LINEAR_HEAD_DIM;
        const float *kv = key + kh * Q38O_LINEAR_HEAD_DIM;
        const float *vv = value + size_t(vh) * Q38O_LINEAR_HEAD_DIM;
        const float decay = std::exp(alpha[vh]);
        for (size_t i = 0; i < head_elems; ++i) state[i] *= decay;
        for (int col = 0; col < Q38O_LINEAR_HEAD_DIM; ++col) {
            float *row = state + size_t(col) * Q38O_LINEAR_HEAD_DIM;
            const float prediction = dot_128(row, kv);
            const float delta = (vv[col] - prediction) * beta[vh];
            const float result = mad_dot_128(row, kv, delta, qh);
            out[col] = result * query_scale;
        }
    }
    // (6) per-head RMSNorm, then *= silu(z) (ops.rs:735-740).
    for (size_t h = 0; h < Q38O_LINEAR_V_HEADS; ++h) {
        float *out = attention + h * Q38O_LINEAR_HEAD_DIM;
        rmsnorm_inplace(out, ssm_norm, Q38O_LINEAR_HEAD_DIM);
        const float *g = z + h * Q38O_LINEAR_HEAD_DIM;
        for (int i = 0; i < Q38O_LINEAR_HEAD_DIM; ++i) out[i] *= silu(g[i]);
    }
    return 0;
}

int q38o_full_core(const float *q_norm, const float *k_norm, const float *q_and_gate,
                   float *key, const float *value, float *q, float *gate, float *scores,
                   float *attention, float *key_cache, float *value_cache, size_t cache_rows,
                   size_t context_length, uint32_t current_position, size_t layer,
                   int kv_round_bf16) {
    if (full_core_prepare(q_norm, k_norm, q_and_gate, key, value, q, gate, key_cache,
                          value_cache, cache_rows, context_length, current_position, layer,
                          kv_round_bf16) != 0)
        return -1;
    const size_t full_index = layer / 4;
    const size_t positions = size_t(current_position) + 1;
    const bool par = parallel_over(Q38O_ATTN_HEADS, positions * Q38O_ATTN_HEAD_DIM);
#pragma omp parallel for schedule(static) num_threads(threads()) if (par)
    for (int h = 0; h < Q38O_ATTN_HEADS; ++h) {
        full_core_head(size_t(h), q, gate, scores + size_t(h) * context_length,
                       attention + size_t(h) * Q38O_ATTN_HEAD_DIM, key_cache, value_cache,
                       full_index, context_length, positions);
    }
    return 0;
}

int q38o_linear_prefill(const float *conv_w, const float *dt_bias, const float *ssm_a,
                        const float *ssm_norm, float *conv_state, float *delta_state,
                        float *qkv, const float *z, float *beta, float *alpha,
                        float *attention, size_t count) {
    for (size_t t = 0; t < count; ++t) {
        const int rc = q38o_linear_core(
            conv_w, dt_bias, ssm_a, ssm_norm, conv_state, delta_state,
            qkv + t * Q38O_LINEAR_QKV_DIM, z + t * Q38O_LINEAR_V_DIM,
            beta + t * Q38O_LINEAR_V_HEADS, alpha + t * Q38O_LINEAR_V_HEADS,
            attention + t * Q38O_LINEAR_V_DIM);
        if (rc != 0) return rc;
    }
    return 0;
}

int q38o_full_prefill_rows(const float *q_norm, const float *k_norm, const float *q_and_gate,
                           float *key, const float *value, float *attention,
                           float *key_cache, float *value_cache, size_t cache_rows,
                           size_t context_length, uint32_t base_position, size_t layer,
                           size_t count, const int64_t *rows, size_t row_count,
                           int kv_round_bf16) {
    std::vector<float> q(Q38O_ATTN_Q_DIM), gate(Q38O_ATTN_Q_DIM);
    std::vector<float> scores(size_t(Q38O_ATTN_HEADS) * context_length);
    size_t next_row = 0;
    for (size_t t = 0; t < count; ++t) {
        const uint32_t position = base_position + uint32_t(t);
        const bool wanted =
            rows == nullptr || (next_row < row_count && rows[next_row] == int64_t(t));
        if (rows != nullptr && wanted) ++next_row;
        int rc;
        if (wanted) {
            rc = q38o_full_core(q_norm, k_norm, q_and_gate + t * Q38O_ATTN_QG_DIM,
                                key + t * Q38O_ATTN_KV_DIM, value + t * Q38O_ATTN_KV_DIM,
                                q.data(), gate.data(), scores.data(),
                                attention + t * Q38O_ATTN_Q_DIM, key_cache, value_cache,
                                cache_rows, context_length, position, layer, kv_round_bf16);
        } else {
            rc = full_core_prepare(q_norm, k_norm, q_and_gate + t * Q38O_ATTN_QG_DIM,
                                   key + t * Q38O_ATTN_KV_DIM, value + t * Q38O_ATTN_KV_DIM,
                                   q.data(), gate.data(), key_cache, value_cache, cache_rows,
                                   context_length, position, layer, kv_round_bf16);
        }
        if (rc != 0) return rc;
    }
    return 0;
}

int q38o_full_prefill(const float *q_norm, const float *k_norm, const float *q_and_gate,
                      float *key, const float *value, float *attention, float *key_cache,
                      float *value_cache, size_t cache_rows, size_t context_length,
                      uint32_t base_position, size_t layer, size_t count, int kv_round_bf16) {
    return q38o_full_prefill_rows(q_norm, k_norm, q_and_gate, key, value, attention, key_cache,
                                  value_cache, cache_rows, context_length, base_position,
                                  layer, count, nullptr, 0, kv_round_bf16);
}

}  // extern "C"
