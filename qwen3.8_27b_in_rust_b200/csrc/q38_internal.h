// q38_internal.h -- host-side structures shared by the C-ABI layer and the
// kernel launchers. Not part of the public ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/q38attn.h"

namespace q38 {

constexpr int kAttnHeadDim = 256;
constexpr int kRopeDims = 64;
constexpr int kGroup = 6;  // query heads per KV head (Q38_ATTN_HEADS / Q38_ATTN_KV_HEADS)
constexpr int kLinHeadDim = 128;
constexpr int kConvKernel = 4;

struct FullWeights {
    float *q_norm = nullptr;  // [256]
    float *k_norm = nullptr;  // [256]
};

struct LinearWeights {
    float *conv_w = nullptr;    // [qkv_dim][4]
    float *dt_bias = nullptr;   // [v_heads]
    float *ssm_a = nullptr;     // [v_heads]
    float *ssm_norm = nullptr;  // [128]
};

// Split-KV decode launch configuration.
struct DecodeSplitPlan {
    int chunk = 0;   // positions per split CTA (multiple of the tile)
    int nsplit = 0;  // split CTAs per (sequence, kv head)
};

}  // namespace q38

struct q38_ctx {
    int device = 0;
    q38_geom geom{};
    int sm_count = 0;
    float theta_scale = 0.f;  // rope_theta^(-2/rope_dims), computed with powf
    int qg_dim = 0, q_dim = 0, kv_dim = 0;
    int qk_dim = 0, v_dim = 0, qkv_dim = 0;
    std::map<int, q38::FullWeights> full;
    std::map<int, q38::LinearWeights> linear;
    void *proj_scratch = nullptr;   // quantized activations of the tensor-core projections
    size_t proj_scratch_bytes = 0;
    float *proj_part = nullptr;     // partial sums of the chunked f32-input projections
    size_t proj_part_bytes = 0;
};

struct q38_state {
    q38_ctx *ctx = nullptr;
    int batch = 0, context_length = 0, full_slots = 0, linear_slots = 0, kv_dtype = 0;
    size_t kv_elem = 0;             // bytes per cache element
    size_t kv_slot_elems = 0;       // batch*kv_heads*context_length*256
    void *kcache = nullptr, *vcache = nullptr;
    float *conv_state = nullptr;    // [linear_slots][batch][qkv_dim][3]
    float *delta_state = nullptr;   // [linear_slots][batch][v_heads][128][128]
    int *lin_group_count = nullptr; // [linear_slots][batch][qk_heads] (decode sweep)
    float *qprep = nullptr;         // [batch][heads][256]
    float *part_o = nullptr;        // [batch][heads][max_splits][256]
    float *part_ml = nullptr;       // [batch][heads][max_splits][2]
    int max_splits = 0;
    int *d_err = nullptr;           // device error bits
    float *prefill_rope = nullptr;       // RoPE table of the prompt's positions
    __half *prefill_v16 = nullptr;       // [v16_seqs][kv_heads][context][256] V as f16
    int prefill_v16_seqs = 0;
    size_t prefill_tokens = 0;
    float *prefill_lin = nullptr;        // chunked DeltaNet scratch
    size_t prefill_chunks = 0;           // chunk capacity of prefill_lin
    float *ckpt_conv = nullptr;          // checkpoint copies of conv_state / delta_state
    float *ckpt_delta = nullptr;
    std::vector<char> ckpt_valid;        // per sequence: has a checkpoint
    float *prefill_stage = nullptr;      // device staging of the *_prefill_host forms
    size_t prefill_stage_tokens = 0;     // tokens (all sequences) one staged piece holds
    // staging for the host-pointer calls (device, sized for `batch`)
    float *stage = nullptr;
    size_t stage_floats = 0;
    // projection outputs / core inputs of the layer-level decode calls
    float *proj_stage = nullptr;    // stage_floats
    // the same for the layer-level prefill calls (q38_state_reserve_attention_prefill)
    float *layer_prefill = nullptr;
    size_t layer_prefill_tokens = 0;
    int32_t *stage_pos = nullptr;
    // Host-pointer decode: a stream for the write-back copies that overlap the
    // state kernel, and its events (created on first use).
    cudaStream_t host_out = nullptr;
    cudaEvent_t host_ev_prep = nullptr, host_ev_back = nullptr;
    // Pinned word the host-pointer calls read the device error bits into.
    int *host_err = nullptr;
    // Error-path testing (q38_state_set_debug).
    int debug_flags = 0;
    uint64_t debug_wait_ns = 0;
    // Split-sequence decode over NCCL (q38_state_reserve_split).
    float *split_local = nullptr;     // [batch][heads][258]
    float *split_gathered = nullptr;  // [split_ranks][batch][heads][258]
    int split_ranks = 0;
    // Split-sequence exchange over peer memory (q38_state_split_p2p_*).
    void *p2p_buf = nullptr;          // this rank's exchange buffer (IPC-exported)
    int p2p_nranks = 0, p2p_rank = -1;
    std::vector<void *> p2p_opened;   // peers' buffers opened with cudaIpcOpenMemHandle
    // Device array [64] of the buffers' addresses, then the exchange's epoch
    // counter (a uint32: calls made so far, incremented on the device by each
    // call's prep kernel, so the launches carry no per-call value and can be
    // captured in a CUDA graph).
    float **p2p_peers_dev = nullptr;
    // Side streams and their fork / join events (created with the state):
    // the DeltaNet prefill's per-group state passes and the layer-level
    // decode call's concurrent projections fork onto them and join back into
    // the caller's stream.
    static constexpr int kSides = 4;
    cudaStream_t side[kSides] = {};
    cudaEvent_t side_fork = nullptr, side_join[kSides] = {};
    // f32-cache prefill: the K rows as f16 for the tensor cores.
    __half *prefill_k16 = nullptr;  // [v16_seqs][kv_heads][context][256]
};

namespace q38 {

// Layer-kind helpers (src/model/ops.rs:39-47).
inline bool is_full_attention(int layer) { return (layer + 1) % 4 == 0 || layer == 64; }
inline int full_index(int layer) { return layer / 4; }
inline int recurrent_index(int layer) { return layer - (layer + 1) / 4; }

// Sets the calling thread's q38_last_error() message (q38attn.cu).
void record_error(const char *msg);

// The layer-level DeltaNet decode (q38proj.cu): the core on projection
// outputs whose conv + SiLU and gates were applied by the projections'
// epilogues; and the layer's conv state / weights those epilogues need.
int linear_decode_prepped(q38_ctx *ctx, q38_state *st, int layer, int batch, float *qkv,
                          const float *z, float *beta, float *alpha, float *attention,
                          cudaStream_t stream);
int linear_layer_prologue_args(q38_ctx *ctx, q38_state *st, int layer, float **conv_state,
                               const float **conv_w, const float **dt_bias, const float **ssm_a);

// NCCL, resolved at run time (q38_nccl.cu). Both return a Q38 status and
// record the reason.
int nccl_comm_ranks(void *comm, int *nranks);
int nccl_all_gather_f32(void *comm, const float *send, float *recv, size_t count,
                        cudaStream_t stream);

// Kernel launchers (attn_decode.cu, deltanet_decode.cu).
struct AttnDecodeLaunch {
    const float *q_and_gate;
    float *key;
    const float *value;
    const int32_t *positions;
    float *attention;
    void *kcache;  // this slot: [batch][kv_heads][context_length][256]
    void *vcache;
    float *qprep, *part_o, *part_ml;
    int *err;
    const float *q_norm, *k_norm;
    int batch, context_length, heads, kv_heads, kv_dtype, max_position, max_splits;
    float theta_scale, eps;
    int pos_offset = 0;            // first global position held by this cache (sharding)
    float *partial_out = nullptr;  // non-null: packed (o, m, l) partials instead of output
    uint64_t wait_ns = 0;          // bounded-wait limit of the split kernel (0: the default)
    int skip_kv_loads = 0;         // error-path testing (Q38_DEBUG_SKIP_KV_LOADS)
    // Split-sequence exchange over peer memory (p2p_nranks > 0): the merge
    // kernel exchanges the shards' partials itself and writes `attention`.
    float *const *p2p_peers = nullptr;  // device array: every rank's exchange buffer
    int p2p_rank = 0, p2p_nranks = 0, p2p_batch = 0;
    uint32_t *p2p_epoch = nullptr;  // device counter of the exchange calls
};
cudaError_t launch_attn_decode(const AttnDecodeLaunch &a, int sm_count, cudaStream_t stream);
cudaError_t launch_attn_merge_shards(const float *partials, int nparts, int batch, int heads,
                                     const float *q_and_gate, float *attention,
                                     cudaStream_t stream);
DecodeSplitPlan plan_attn_decode(int batch, int kv_heads, int max_position, int kv_dtype,
                                 int sm_count);
int attn_decode_max_splits(int context_length, int kv_dtype);
// Bytes of one rank's split-sequence exchange buffer (partials and flags).
size_t attn_p2p_exchange_bytes(int nranks, int batch, int heads);

struct AttnPrefillLaunch {
    const float *q_and_gate;  // [nseq][count][heads*512]
    float *key;               // [nseq][count][kv_heads*256]
    const float *value;
    float *attention;         // [nseq][count][heads*256]
    float *rope;              // scratch: RoPE table (attn_prefill_rope_floats)
    void *kcache, *vcache;    // slot base [batch][kv_heads][ctx][256], bf16 or f32
    __half *v16;              // scratch [nseq][kv_heads][ctx][256]: V as f16
    __half *k16;              // f32 cache only: scratch [nseq][kv_heads][ctx][256], K as f16
    const float *q_norm, *k_norm;
    int *err;
    int batch, seq0, nseq, count, base, context_length, heads, kv_heads;
    int kv_head0, kv_head_count;  // the KV heads this call covers
    int kv_f32;                   // the cache holds f32 rows
    float theta_scale, eps;
};
cudaError_t launch_attn_prefill(const AttnPrefillLaunch &a, cudaStream_t stream);
// Floats of the RoPE table a prefill of up to max_tokens positions uses.
size_t attn_prefill_rope_floats(int max_tokens);

struct LinearPrefillLaunch {
    float *qkv;                 // [nseq][count][qkv_dim] in/out
    const float *z;             // [nseq][count][v_heads*128]
    float *beta, *alpha;        // [nseq][count][v_heads] in/out
    float *attention;           // [nseq][count][v_heads*128]
    float *conv_state;          // slot base [batch][qkv_dim][3]
    float *delta_state;         // slot base [batch][v_heads][128][128]
    const float *conv_w, *dt_bias, *ssm_a, *ssm_norm;
    float *scratch;             // linear_prefill_scratch_floats(nseq*nchunk, v_heads)
    int *err;                   // device error bits
    int seq0, nseq, count, qk_heads, v_heads;
    int v_head0, v_head_count;  // the value heads this call covers
    float eps;
    // Optional side streams (the state's): the state and output passes run
    // per group of sequences, forked from and joined back into the caller's
    // stream, so a group's output pass runs while the state pass of later
    // groups still occupies some SMs.
    const cudaStream_t *side = nullptr;
    cudaEvent_t fork = nullptr;
    const cudaEvent_t *join = nullptr;
    int nside = 0;
};
cudaError_t launch_linear_prefill(const LinearPrefillLaunch &a, cudaStream_t stream);
size_t linear_prefill_scratch_floats(int nchunk_total, int v_heads);

struct LinearDecodeLaunch {
    float *qkv;
    const float *z;
    float *beta, *alpha, *attention;
    float *conv_state;   // this slot: [batch][qkv_dim][3]
    float *delta_state;  // this slot: [batch][v_heads][128][128]
    const float *conv_w, *dt_bias, *ssm_a, *ssm_norm;
    int batch, qk_heads, v_heads;
    float eps;
    int prepped = 0;  // conv + SiLU and gates already applied (layer-level call)
    int *group_count = nullptr;  // this slot: [batch][qk_heads], zero between calls
    int *err = nullptr;
    uint64_t wait_ns = 0;        // bounded-wait limit (0: the library's)
    int sm_count = 0;
};
// prep_done (optional) is recorded once the prep kernel is done; the call then
// runs as two kernels (prep, state pass) instead of the fused sweep.
cudaError_t launch_linear_decode(const LinearDecodeLaunch &a, cudaStream_t stream,
                                 cudaEvent_t prep_done = nullptr);

}  // namespace q38
