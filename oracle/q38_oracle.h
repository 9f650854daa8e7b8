/*
 * q38_oracle.h -- CPU restatement of the reference's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker and the timed
 * CPU baseline. Only tests/, __graft_entry__.smoke() and bench.py's CPU legs
 * may load it; the product path (libq38attn.so) never links or calls it.
 *
 * It restates, in C++, the scalar Rust of StepfenShawn/qwen3.8_27b_in_rust:
 *   src/model/ops.rs:454-610   elementwise primitives
 *   src/model/ops.rs:648-742   linear_core  (Gated DeltaNet step)
 *   src/model/ops.rs:813-940   full_core    (gated full attention step)
 *   src/model/ops.rs:1088-1099 per-token loop of batch_linear_attention
 *   src/model/ops.rs:1156-1172 per-token loop of batch_full_attention
 *   src/kernel/mod.rs:19-21    q38_parallel_over (the rayon gate)
 * with the geometry of src/model/mod.rs:6-26.
 *
 * Parity status: the reference is Rust and no Rust toolchain exists here, and
 * the reference has no golden vectors or known-answer tests for this path, so
 * the restatement is "parity unpinned" by the reference itself. It is pinned
 * instead by known-answer tests derived from the algorithm and by an
 * independent numpy restatement (tests/test_oracle.py).
 *
 * Arithmetic contract (so a faithful build is bit-identical to the Rust on the
 * same libm): compile with -ffp-contract=off (Rust never contracts a*b+c),
 * use fmaf exactly where the Rust uses mul_add, accumulate the RMS / L2 sums in
 * double, compute the RoPE angle by repeated f32 multiplication, and call the
 * platform expf/logf/cosf/sinf/powf as Rust's f32 methods do on Linux.
 */
#ifndef Q38_ORACLE_H
#define Q38_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Geometry constants, src/model/mod.rs:13-26. */
#define Q38O_LINEAR_QK_HEADS 16
#define Q38O_LINEAR_V_HEADS 48
#define Q38O_LINEAR_HEAD_DIM 128
#define Q38O_LINEAR_QK_DIM 2048
#define Q38O_LINEAR_V_DIM 6144
#define Q38O_LINEAR_QKV_DIM 10240
#define Q38O_ATTN_HEADS 24
#define Q38O_ATTN_KV_HEADS 4
#define Q38O_ATTN_HEAD_DIM 256
#define Q38O_ATTN_Q_DIM 6144
#define Q38O_ATTN_QG_DIM 12288
#define Q38O_ATTN_KV_DIM 1024

/* Number of OpenMP threads the rayon-style parallel regions use (<=0: all). */
void q38o_set_threads(int threads);
int q38o_get_threads(void);

/*
 * linear_core, src/model/ops.rs:647-742. Every pointer is a host f32 array:
 *   conv_w      [10240][4]   ssm_conv1d weight
 *   dt_bias     [48]         ssm_dt.bias
 *   ssm_a       [48]         ssm_a (= -exp(A_log))
 *   ssm_norm    [128]        ssm_norm weight (shared by every head)
 *   conv_state  [10240][3]   carried conv inputs, updated in place
 *   delta_state [48][128][128] recurrent state, updated in place
 *   qkv         [10240]      in: projections; out: conv+SiLU+L2 values
 *   z           [6144]       output gate logits
 *   beta        [48]         in: logits; out: sigmoid(beta)
 *   alpha       [48]         in: logits; out: ssm_a*softplus(alpha+dt_bias)
 *   attention   [6144]       output
 * Returns 0 (the reference's Ok(())).
 */
int q38o_linear_core(const float *conv_w, const float *dt_bias, const float *ssm_a,
                     const float *ssm_norm, float *conv_state, float *delta_state, float *qkv,
                     const float *z, float *beta, float *alpha, float *attention);

/*
 * full_core, src/model/ops.rs:812-940.
 *   q_norm, k_norm  [256]      attn_q_norm / attn_k_norm weights
 *   q_and_gate      [12288]    per head: 256 query lanes then 256 gate lanes
 *   key             [1024]     in: projection; out: RMSNorm + RoPE'd key
 *   value           [1024]
 *   q, gate         [6144]     scratch outputs (as in the reference)
 *   scores          [24][context_length] scratch
 *   attention       [6144]     output
 *   key_cache, value_cache     [cache_rows][1024], row = full_index*context+pos
 *   cache_rows                 rows in each cache array
 *   kv_round_bf16              bit 0 clear: f32 cache exactly as the reference
 *                              stores it. bit 0 set: the new row is rounded to
 *                              bf16 (RNE) before it is stored, modelling a bf16
 *                              KV cache; earlier rows are whatever the caller
 *                              stored. bit 1 set: the prepared query (after
 *                              RMSNorm and RoPE) is rounded to bf16 too, the
 *                              input precision of the tensor-core prefill.
 * Returns 0, or -1 when the cache row is out of range (ops.rs:860-864).
 */
int q38o_full_core(const float *q_norm, const float *k_norm, const float *q_and_gate,
                   float *key, const float *value, float *q, float *gate, float *scores,
                   float *attention, float *key_cache, float *value_cache, size_t cache_rows,
                   size_t context_length, uint32_t current_position, size_t layer,
                   int kv_round_bf16);

/*
 * The per-token prefill loop of batch_linear_attention (ops.rs:1088-1099):
 * count tokens, token-major arrays (qkv [count][10240], z [count][6144],
 * beta/alpha [count][48], attention [count][6144]).
 */
int q38o_linear_prefill(const float *conv_w, const float *dt_bias, const float *ssm_a,
                        const float *ssm_norm, float *conv_state, float *delta_state,
                        float *qkv, const float *z, float *beta, float *alpha,
                        float *attention, size_t count);

/*
 * The per-token prefill loop of batch_full_attention (ops.rs:1156-1172):
 * q_and_gate [count][12288], key/value [count][1024], attention [count][6144],
 * positions base_position .. base_position+count-1. Scratch q/gate/scores is
 * allocated internally.
 */
int q38o_full_prefill(const float *q_norm, const float *k_norm, const float *q_and_gate,
                      float *key, const float *value, float *attention, float *key_cache,
                      float *value_cache, size_t cache_rows, size_t context_length,
                      uint32_t base_position, size_t layer, size_t count, int kv_round_bf16);

/*
 * Same per-token loop, but only the attention rows listed in `rows` (indices
 * into 0..count-1, ascending) are computed in full; for every other token
 * only the cache append of full_core is performed (norm + RoPE + store).
 * The rows that are computed are bit-identical to q38o_full_prefill's: the
 * cache contents they read are the same. Used to check sampled query rows of
 * long prefills in bounded time.
 */
int q38o_full_prefill_rows(const float *q_norm, const float *k_norm, const float *q_and_gate,
                           float *key, const float *value, float *attention,
                           float *key_cache, float *value_cache, size_t cache_rows,
                           size_t context_length, uint32_t base_position, size_t layer,
                           size_t count, const int64_t *rows, size_t row_count,
                           int kv_round_bf16);

/*
 * Projections on either side of the cores (q38_oracle_proj.cpp): the Q8_K
 * activation quantizer (src/kernel/quant.rs:56-124), the integer dots of the
 * K-quant types against it (src/kernel/tensor.rs:301-460) and of IQ4_NL /
 * IQ4_XS (src/kernel/iq.rs:355-405; their f32 path iq.rs:311-335), the f32-input dots
 * (tensor.rs:79-117), the row loops with token-major output
 * (tensor.rs:954-1027) and project / batch_project (src/model/ops.rs:617-640,
 * 1016-1031). Weights are raw GGUF tensor bytes, rows of row_bytes(type,
 * width) each; outputs are [batch][rows].
 */
#define Q38O_GGML_F32 0
#define Q38O_GGML_F16 1
#define Q38O_GGML_Q8_0 8
#define Q38O_GGML_Q2_K 10
#define Q38O_GGML_Q3_K 11
#define Q38O_GGML_Q4_K 12
#define Q38O_GGML_Q5_K 13
#define Q38O_GGML_Q6_K 14
#define Q38O_GGML_BF16 30
#define Q38O_GGML_IQ4_NL 20
#define Q38O_GGML_IQ4_XS 23

/* Q38Q8KBlock, src/kernel/mod.rs:20-27: 292 bytes. */
typedef struct {
    float scale;
    int8_t quants[256];
    int16_t sums[16];
} q38o_q8k_block;

float q38o_f16_to_f32(uint16_t h);
int q38o_is_q8k_type(int type);
int q38o_row_bytes(int type, size_t width, size_t *out);
int q38o_quantize_q8_k(const float *input, size_t length, q38o_q8k_block *out);
float q38o_dot_row_f32(int type, const uint8_t *row, const float *x, size_t width);
float q38o_dot_row_q8_k(int type, const uint8_t *row, const q38o_q8k_block *q, size_t blocks);
int q38o_gemm_f32(int type, const uint8_t *w, size_t rows, size_t width, const float *input,
                  size_t batch, float *out);
int q38o_gemm_q8_k(int type, const uint8_t *w, size_t rows, size_t width,
                   const q38o_q8k_block *act, size_t batch, float *out);
int q38o_project(int type, const uint8_t *w, size_t rows, size_t width, const float *input,
                 size_t batch, float *out);

/* Primitives exposed for unit tests (ops.rs:476-610). */
float q38o_rms_scale(const float *values, size_t length);
void q38o_l2norm(float *values, size_t length);
void q38o_rope(float *values, size_t heads, uint32_t position);
float q38o_sigmoid(float value);
float q38o_silu(float value);
float q38o_softplus(float value);
float q38o_round_bf16(float value);

#ifdef __cplusplus
}
#endif

#endif /* Q38_ORACLE_H */
