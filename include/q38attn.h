/*
 * q38attn.h -- C ABI of the B200 (sm_100a) attention hot path of
 * StepfenShawn/qwen3.8_27b_in_rust: gated full attention and Gated DeltaNet,
 * decode and prefill.
 *
 * This is the boundary the reference's Rust host binds with a thin
 * `extern "C"` FFI crate. It replaces the two crate-private cores and the
 * per-token loops that call them:
 *
 *   linear_core   src/model/ops.rs:647-742   -> q38_linear_decode / q38_linear_core
 *   full_core     src/model/ops.rs:812-940   -> q38_full_decode   / q38_full_core
 *   batch_linear_attention loop  ops.rs:1088-1099 -> q38_linear_prefill
 *   batch_full_attention loop    ops.rs:1156-1172 -> q38_full_prefill
 *   Q38Model state fields  src/model/mod.rs:155-158, allocated at
 *   src/model/ops.rs:1461-1490  -> q38_state_create
 *
 * Conventions
 *  - Every function returns an int status: Q38_OK (0), Q38_ERR_ARG (-1, the
 *    reference's Err(-1): bad shape, bad layer kind, cache row out of range),
 *    Q38_ERR_CUDA (-2), Q38_ERR_TIMEOUT (-3, a bounded device wait gave up).
 *    q38_last_error() returns a message for the calling thread's last failure.
 *  - Functions named *_decode / *_prefill take DEVICE pointers and are
 *    stream-ordered on `stream` (a cudaStream_t passed as void*; NULL is the
 *    legacy default stream). They never allocate and never synchronise.
 *    Device-side argument errors (a position outside the cache) are recorded
 *    in the state and reported by q38_state_errors().
 *  - Functions named *_core and *_host take HOST pointers, copy through the
 *    state's staging buffers, and return after the stream has synchronised.
 *  - `layer` is the reference's layer index (0..64). Full-attention layers are
 *    those with (layer+1)%4==0 or layer==64 (ops.rs:39-41) and use KV slot
 *    layer/4; the others are DeltaNet layers with state slot
 *    layer-(layer+1)/4 (ops.rs:45-47). Calling a function of the wrong layer
 *    kind returns Q38_ERR_ARG, as the reference's let-else does.
 *  - Arrays are row-major f32 in the reference's layouts unless noted.
 *  - Not re-entrant on one state: calls on one state must be ordered (same
 *    stream, or externally synchronised), like the reference's &mut borrows.
 */
#ifndef Q38ATTN_H
#define Q38ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q38_OK 0
#define Q38_ERR_ARG (-1)
#define Q38_ERR_CUDA (-2)
#define Q38_ERR_TIMEOUT (-3)

/* KV cache element type. F32 matches the reference's Vec<f32> cache
 * (src/model/ops.rs:1465); BF16 halves the decode traffic. */
#define Q38_KV_F32 0
#define Q38_KV_BF16 1

/* Device error bits returned by q38_state_errors. */
#define Q38_DEVERR_POSITION 1
#define Q38_DEVERR_TIMEOUT 2
#define Q38_DEVERR_SHAPE 4
#define Q38_DEVERR_RANGE 8 /* a prefill V value beyond the f16 range (|v| > 65504) */

typedef struct q38_ctx q38_ctx;
typedef struct q38_state q38_state;

/* Model geometry, src/model/mod.rs:13-26. q38_geom_default fills the
 * reference's constants; the kernels are specialised for head_dim 256 with
 * RoPE on 64 dims and a GQA group of 6, and DeltaNet head_dim 128 with a
 * kernel-4 conv; other values are rejected with Q38_ERR_ARG. Head counts may
 * vary (attn_heads = 6*attn_kv_heads, linear_v_heads a multiple of
 * linear_qk_heads). */
typedef struct q38_geom {
    int32_t attn_heads;      /* Q38_ATTN_HEADS      24 */
    int32_t attn_kv_heads;   /* Q38_ATTN_KV_HEADS    4 */
    int32_t attn_head_dim;   /* Q38_ATTN_HEAD_DIM  256 */
    int32_t rope_dims;       /* rope(): lanes [0,64)    ops.rs:595-610 */
    float rope_theta;        /* 1e7                     ops.rs:596 */
    int32_t linear_qk_heads; /* Q38_LINEAR_QK_HEADS 16 */
    int32_t linear_v_heads;  /* Q38_LINEAR_V_HEADS  48 */
    int32_t linear_head_dim; /* Q38_LINEAR_HEAD_DIM 128 */
    int32_t conv_kernel;     /* ssm_conv1d width 4      ops.rs:665-676 */
    float rms_eps;           /* Q38_RMS_EPS 1e-6 */
} q38_geom;

void q38_geom_default(q38_geom *geom);

/* Last error message of the calling thread ("" if none). */
const char *q38_last_error(void);

/* Library version string. */
const char *q38_version(void);

/* ---------------------------------------------------------------- context */

/* Creates a context on CUDA device `device`. geom==NULL: the reference's
 * geometry. Replaces the weight/geometry half of Q38Model::bind
 * (src/model/ops.rs:1450-1459). */
int q38_ctx_create(const q38_geom *geom, int device, q38_ctx **out);
int q38_ctx_destroy(q38_ctx *ctx);

/* Copies a full-attention layer's F32 norm weights (HOST pointers, 256 each)
 * to the device: attn_q_norm / attn_k_norm, read via scalar() at
 * src/model/ops.rs:838-850. */
int q38_bind_full_layer(q38_ctx *ctx, int layer, const float *q_norm, const float *k_norm);

/* Copies a DeltaNet layer's F32 weights (HOST pointers) to the device:
 * ssm_conv1d [qkv_dim][4], ssm_dt.bias [v_heads], ssm_a [v_heads],
 * ssm_norm [head_dim] (src/model/ops.rs:658-663, 665-740). */
int q38_bind_linear_layer(q38_ctx *ctx, int layer, const float *conv1d, const float *dt_bias,
                          const float *ssm_a, const float *ssm_norm);

/* ------------------------------------------------------------ GGUF weights */

/* Reads the F32 tensor `name` of a GGUF checkpoint into HOST memory; n must
 * equal its element count. The container is checked as the reference's
 * Gguf::open checks it (src/gguf/mod.rs:459-533: magic, version 2..3,
 * metadata types, tensor shapes and types, power-of-two general.alignment,
 * tensor bytes inside the file). Returns Q38_ERR_ARG with the reason in
 * q38_last_error() when the file is malformed or the tensor is missing, not
 * F32, or of another size. Host only: needs no GPU. */
int q38_gguf_read_f32(const char *path, const char *name, float *dst, int64_t n);

/* Binds the F32 attention-core weights of layers first_layer..last_layer
 * (inclusive; layer 64 is the MTP block, KV slot 16) from a GGUF checkpoint,
 * by the reference's tensor names (bind_layer, ops.rs:53-100):
 *   full layers:     blk.L.attn_q_norm.weight, blk.L.attn_k_norm.weight
 *   DeltaNet layers: blk.L.ssm_conv1d.weight, blk.L.ssm_dt.bias, blk.L.ssm_a,
 *                    blk.L.ssm_norm.weight
 * Every layer of the range must be present; the result equals calling
 * q38_bind_full_layer / q38_bind_linear_layer with the same values. */
int q38_bind_gguf(q38_ctx *ctx, const char *path, int first_layer, int last_layer);

/* ------------------------------------------------------------------ state */

/* Allocates device-resident per-sequence state for `batch` sequences:
 * full_slots KV caches of context_length positions each (the reference has
 * 17: 16 layers + the MTP slot) and linear_slots conv/delta states (the
 * reference has 48), plus the decode scratch. Zero-initialised.
 * Replaces src/model/ops.rs:1461-1490. Device layouts:
 *   key/value cache [full_slot][batch][kv_heads][context_length][256] (kv_dtype)
 *   conv state      [linear_slot][batch][qkv_dim][3] f32 (reference layout)
 *   delta state     [linear_slot][batch][v_heads][128][128] f32 (reference layout) */
int q38_state_create(q38_ctx *ctx, int batch, int context_length, int full_slots,
                     int linear_slots, int kv_dtype, q38_state **out);
int q38_state_destroy(q38_state *st);

/* Zeroes all caches and recurrent state (Q38ModelOps::reset). */
int q38_state_reset(q38_state *st, void *stream);

/* Speculative-decoding rollback (checkpoint_state / restore_target_state,
 * src/model/ops.rs:1627-1647): q38_state_checkpoint copies the recurrent state
 * (conv and delta state of every DeltaNet slot) of sequences
 * [seq0, seq0 + nseq) into the state's checkpoint area on the device, and
 * q38_state_restore copies it back. The KV cache is not copied: as in the
 * reference, cache rows past the restored position are overwritten when the
 * committed tokens are re-run. The first checkpoint allocates the checkpoint
 * area (the size of the recurrent state); restoring sequences that were never
 * checkpointed is Q38_ERR_ARG. Device-to-device copies ordered on `stream`. */
int q38_state_checkpoint(q38_state *st, int seq0, int nseq, void *stream);
int q38_state_restore(q38_state *st, int seq0, int nseq, void *stream);

/* Reads and clears the device error bits (synchronises the device). */
int q38_state_errors(q38_state *st, int *bits);

/* Error-path testing only. flags = Q38_DEBUG_SKIP_KV_LOADS makes the split-KV
 * kernel of this state's decode calls issue none of its KV tile loads, so
 * its bounded waits run out: the kernel records Q38_DEVERR_TIMEOUT, returns
 * without touching memory beyond its own partials, and the host-pointer
 * decode call returns Q38_ERR_TIMEOUT (the step's outputs are then
 * undefined). wait_ns is the limit of those waits (0: the library's 1 s).
 * flags = 0, wait_ns = 0 restores normal operation. Nothing is in flight when
 * such a wait gives up, and the context stays usable. Not thread-safe with
 * calls in flight on the state. */
#define Q38_DEBUG_SKIP_KV_LOADS 1
int q38_state_set_debug(q38_state *st, int flags, uint64_t wait_ns);

/* Device pointers of one slot's buffers, for callers that manage their own
 * copies. Any output pointer may be NULL. */
int q38_state_full_slot(q38_state *st, int layer, void **key_cache, void **value_cache,
                        size_t *bytes_each);
int q38_state_linear_slot(q38_state *st, int layer, float **conv_state, float **delta_state);

/* Host <-> device copies in the reference's host layouts (synchronous).
 * KV rows: key_rows/value_rows [count][kv_heads*256] f32 for positions
 * first..first+count-1 of sequence `seq` (bf16 caches round on upload).
 * Linear: conv_state [qkv_dim][3], delta_state [v_heads][128][128]. */
int q38_state_upload_kv(q38_state *st, int layer, int seq, int first, int count,
                        const float *key_rows, const float *value_rows);
int q38_state_download_kv(q38_state *st, int layer, int seq, int first, int count,
                          float *key_rows, float *value_rows);
int q38_state_upload_linear(q38_state *st, int layer, int seq, const float *conv_state,
                            const float *delta_state);
int q38_state_download_linear(q38_state *st, int layer, int seq, float *conv_state,
                              float *delta_state);

/* ------------------------------------------------------------ decode (device) */

/* One full-attention decode step for `batch` sequences (full_core,
 * src/model/ops.rs:812-940, batched). DEVICE pointers:
 *   q_and_gate [batch][heads*512]   per head 256 query then 256 gate lanes
 *   key        [batch][kv_heads*256] in: projection; out: RMSNorm+RoPE'd key
 *   value      [batch][kv_heads*256]
 *   positions  [batch] int32         current_position of each sequence
 *   attention  [batch][heads*256]    output
 * max_position: host upper bound on every positions[b] (sizes the split grid;
 * <0 means context_length-1). A position outside [0, context_length) or above
 * max_position is flagged Q38_DEVERR_POSITION and that sequence is skipped. */
int q38_full_decode(q38_ctx *ctx, q38_state *st, int layer, int batch, const float *q_and_gate,
                    float *key, const float *value, const int32_t *positions, int max_position,
                    float *attention, void *stream);

/* Split-sequence decode, shard side: this state holds global positions
 * pos_offset .. pos_offset+context_length-1 of each sequence (one contiguous
 * range per GPU). Runs the same prep and split-KV attention over the rows this
 * shard holds that are <= positions[b] (RoPE at the global position; the new
 * K/V row is appended only by the shard whose range contains it) and writes,
 * instead of the output, the shard's softmax partial per (sequence, head):
 *   partials [batch][heads][258] f32 = o[256] (sum of exp(s-m) v), m, l
 * (m = -inf, l = 0 for a shard with no visible row). Replaces the position
 * loop of full_core (ops.rs:884-913) for one range of positions. */
int q38_full_decode_shard(q38_ctx *ctx, q38_state *st, int layer, int batch,
                          const float *q_and_gate, float *key, const float *value,
                          const int32_t *positions, int max_position, int pos_offset,
                          float *partials, void *stream);

/* Split-sequence decode in one call, with the exchange over NCCL: this rank
 * holds positions pos_offset .. pos_offset+context_length-1 of every
 * sequence (as for q38_full_decode_shard); the call runs the shard kernels,
 * an ncclAllGather of every rank's (o, m, l) partials into this state's
 * local gather buffer (24 x 258 floats per sequence and rank; no kernel
 * reads another GPU's memory), and the merge, all on `stream`. Every rank of
 * nccl_comm (an ncclComm_t of the caller's NCCL, or one from
 * q38_nccl_comm_create) makes the same call with the same q_and_gate / key /
 * value / positions and receives the full attention [batch][heads*256].
 * Needs q38_state_reserve_split(st, ranks of nccl_comm). The split-sequence
 * form of full_core's position loop (src/model/ops.rs:884-913), with the
 * positions spread over the ranks. */
int q38_full_decode_split(q38_ctx *ctx, q38_state *st, int layer, int batch,
                          const float *q_and_gate, float *key, const float *value,
                          const int32_t *positions, int max_position, int pos_offset,
                          void *nccl_comm, float *attention, void *stream);

/* Sizes the split-sequence buffers of q38_full_decode_split for `nranks`
 * ranks and the state's batch (allocates; call it once at set-up). */
int q38_state_reserve_split(q38_state *st, int nranks);

/* NCCL communicator helpers for hosts without their own NCCL plumbing. The
 * library resolves NCCL (libnccl.so.2) at run time, on first use, and uses
 * the copy the process has already loaded if there is one. Rank 0 makes an
 * id (Q38_NCCL_ID_BYTES bytes) with q38_nccl_unique_id, the host sends it to
 * every rank by its own means, and each rank creates its communicator on its
 * device with q38_nccl_comm_create (collective over the ranks: every rank
 * must call it). comm receives an ncclComm_t. */
#define Q38_NCCL_ID_BYTES 128
int q38_nccl_unique_id(void *id);
int q38_nccl_comm_create(const void *id, int nranks, int rank, int device, void **comm);
int q38_nccl_comm_destroy(void *comm);

/* Split-sequence decode with the exchange fused into the merge kernel, over
 * peer memory instead of NCCL. Set-up, once per state and group of ranks
 * (one process per GPU, every GPU able to reach every other by NVLink P2P):
 * each rank calls q38_state_split_p2p_handle(st, nranks, handle), which
 * allocates the state's exchange buffer (every rank's (o, m, l) partials per
 * sequence and head, twice, each value stored with its call's epoch in one
 * 8-byte word) and returns its CUDA IPC
 * handle (Q38_IPC_HANDLE_BYTES bytes); the host gathers the nranks handles,
 * rank-major, on every rank by its own means; each rank then calls
 * q38_state_split_p2p_open(st, rank, handles), which maps every peer's
 * buffer into this process (cudaIpcOpenMemHandle).
 *
 * Then every rank makes the same sequence of q38_full_decode_split_p2p calls
 * (same arguments as q38_full_decode_split, no communicator). The merge
 * kernel of each (sequence, head) stores this rank's partial straight into
 * every peer's buffer over NVLink, every value tagged with the call's epoch,
 * waits until its own buffer holds every rank's values of this epoch, and
 * merges: the exchange overlaps the other heads' merging, and no library
 * collective or second kernel runs. No kernel reads another GPU's memory.
 * The epoch is a counter in the state's device memory that each call
 * advances on the device, so the call's launches depend on no host-side
 * per-call value: a run of calls may be captured in a CUDA graph and
 * replayed, every replay being further calls (every rank replaying the same
 * number). A rank whose peers do not make the matching call gives up after
 * the bounded wait (1 s) and records Q38_DEVERR_TIMEOUT. Destroy the states
 * only after every rank has finished its last call. */
#define Q38_IPC_HANDLE_BYTES 64
int q38_state_split_p2p_handle(q38_state *st, int nranks, void *handle);
int q38_state_split_p2p_open(q38_state *st, int rank, const void *handles);
int q38_full_decode_split_p2p(q38_ctx *ctx, q38_state *st, int layer, int batch,
                              const float *q_and_gate, float *key, const float *value,
                              const int32_t *positions, int max_position, int pos_offset,
                              float *attention, void *stream);

/* Split-sequence decode, merge side: combines nparts shard partials
 * [nparts][batch][heads][258] (gathered from every shard, e.g. by an NCCL
 * all-gather) by log-sum-exp, normalises and applies the sigmoid output gate
 * of q_and_gate [batch][heads*512] (ops.rs:898-919) into attention
 * [batch][heads*256]. DEVICE pointers, stream-ordered. */
int q38_attn_merge_shards(q38_ctx *ctx, int nparts, int batch, const float *partials,
                          const float *q_and_gate, float *attention, void *stream);

/* One Gated DeltaNet decode step for `batch` sequences (linear_core,
 * src/model/ops.rs:647-742, batched). DEVICE pointers:
 *   qkv   [batch][qkv_dim]  in: projections; out: conv+SiLU+L2 values (as the
 *                           reference leaves them)
 *   z     [batch][v_heads*128]
 *   beta  [batch][v_heads]  in: logits; out: sigmoid(beta)
 *   alpha [batch][v_heads]  in: logits; out: ssm_a*softplus(alpha+dt_bias)
 *   attention [batch][v_heads*128] output */
int q38_linear_decode(q38_ctx *ctx, q38_state *st, int layer, int batch, float *qkv,
                      const float *z, float *beta, float *alpha, float *attention,
                      void *stream);

/* One full-attention decode step that allocates no device memory at all.
 * No counterpart in the reference: the reference runs on the CPU and owns
 * its buffers; this entry point exists for GPU callers that cannot call
 * cudaMalloc -- hosts that reserve all of HBM for their own memory pool or
 * KV-block arena (a library cudaMalloc would fail there, or synchronise the
 * device and stall their other streams, or create memory they cannot account
 * for).
 *
 * Same computation as q38_full_decode for the reference geometry (24 query
 * heads, 4 KV heads, head_dim 256), but without a q38_ctx or q38_state: the
 * caller passes every input and output as DEVICE pointers, including the
 * norm weights (q_norm/k_norm, 256 f32 each) and its own KV cache
 * (key_cache/value_cache laid out [batch][4][context_length][256] in kv_dtype).
 * error_bits is an optional device int that receives Q38_DEVERR_* bits (it is
 * OR-ed into, never cleared; NULL to skip).
 *
 * key_cache and value_cache must be 16-byte aligned and every other pointer
 * 4-byte aligned; a misaligned pointer is rejected with Q38_ERR_ARG before
 * any work.
 *
 * The kernels' scratch (prepared queries and split-KV partials) lives in a
 * fixed 16 MiB device array inside the library, held on every GPU where the
 * library's device code has been loaded, until the process exits. A call
 * whose batch and max_position would need more than 16 MiB is rejected with
 * Q38_ERR_ARG before any work. The first call on each device looks the
 * array's address up (cudaGetSymbolAddress) and caches it; under CUDA's
 * default lazy module loading this is also when the 16 MiB are taken from
 * the device. So make that first call (a warm-up step) before reserving the
 * device's free memory for a pool, and before any stream capture. The cached
 * address does not survive a cudaDeviceReset of that device. All calls on a
 * device share the array, which keeps the last call's contents (no call
 * relies on it starting at zero): calls whose executions overlap on the GPU
 * race on it, so order them on one stream. */
int q38_full_decode_noalloc(const float *q_norm, const float *k_norm, void *key_cache,
                            void *value_cache, int batch, int context_length, int kv_dtype,
                            const float *q_and_gate, float *key, const float *value,
                            const int32_t *positions, int max_position, float *attention,
                            int *error_bits, void *stream);

/* ------------------------------------------------------------ prefill */

/* Reserves the state's prefill scratch for up to max_tokens prompt tokens
 * per call (summed over the sequences of the call): the RoPE table of the
 * attention prefill (256 B per token) and an f16 copy of the V cache for the
 * sequences of one call (when the state has full slots), the chunk-local WY
 * quantities of the DeltaNet prefill (about 62 KB per token, when it has
 * linear slots), and the staging of the host-pointer forms. Allocates; call
 * it once at set-up. */
int q38_state_reserve_prefill(q38_state *st, int max_tokens);

/* Causal prefill of `count` prompt tokens for each of the nseq sequences
 * seq0..seq0+nseq-1, all starting at cache position base_position: token t
 * attends to positions 0..base_position+t, exactly as the reference's
 * per-token loop over full_core (batch_full_attention, ops.rs:1156-1172).
 * Runs on the tcgen05 tensor cores: S = Q K^T from bf16 Q and K, O = P V in
 * f16, f32 accumulation (tolerance 2e-3 against the f32 reference).
 * Needs q38_state_reserve_prefill(nseq*count). Either cache type: a
 * Q38_KV_F32 state keeps the reference's f32 rows in its cache (decode then
 * reads exactly what the reference's Vec<f32> cache holds) and the
 * tensor-core operands are bf16 / f16 copies in the prefill scratch; a
 * Q38_KV_BF16 state stores the rows in bf16.
 * DEVICE pointers (16-byte aligned, else Q38_ERR_ARG), token-major per
 * sequence:
 *   q_and_gate [nseq][count][heads*512]
 *   key        [nseq][count][kv_heads*256] in: projections; out: RMSNorm+RoPE'd
 *   value      [nseq][count][kv_heads*256]
 *   attention  [nseq][count][heads*256]  output
 * The K/V rows of positions base_position..base_position+count-1 are
 * appended to the cache. A V value beyond the f16 range (|v| > 65504) sets
 * Q38_DEVERR_RANGE (its rows' outputs are then not finite). */
int q38_full_prefill(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                     int base_position, const float *q_and_gate, float *key, const float *value,
                     float *attention, void *stream);

/* The same for the KV heads kv_head0 .. kv_head0+kv_head_count-1 only (their
 * 6 query heads each): the tensors keep their full row widths, and only the
 * range's columns of q_and_gate, key, value and attention are read or
 * written, and only the range's K/V cache rows appended. The reference runs
 * one task per query head with kv_head = head / 6 (ops.rs:922-938, :877);
 * a (sequence, KV-head group) is the unit that prefill shards across GPUs. */
int q38_full_prefill_heads(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq,
                           int count, int base_position, int kv_head0, int kv_head_count,
                           const float *q_and_gate, float *key, const float *value,
                           float *attention, void *stream);

/* Chunked Gated DeltaNet prefill of `count` prompt tokens for each of the
 * nseq sequences seq0..seq0+nseq-1, continuing each sequence's conv and
 * delta state: the same result as the reference's per-token loop over
 * linear_core (batch_linear_attention, ops.rs:1088-1099), computed in chunks
 * of 64 tokens in WY form: the chunk products run on the tcgen05 tensor cores
 * with every operand split into a bf16 (hi, lo) pair and f32 accumulation
 * (about 16 mantissa bits per operand; within ~1e-5 of the per-token
 * recurrence). Needs q38_state_reserve_prefill(nseq*count).
 * DEVICE pointers (qkv, z, attention 16-byte aligned, else Q38_ERR_ARG),
 * token-major per sequence:
 *   qkv   [nseq][count][qkv_dim]  in: projections; out: conv+SiLU+L2 values
 *   z     [nseq][count][v_heads*128]
 *   beta  [nseq][count][v_heads]  in: logits; out: sigmoid(beta)
 *   alpha [nseq][count][v_heads]  in: logits; out: ssm_a*softplus(alpha+dt_bias)
 *   attention [nseq][count][v_heads*128] output */
int q38_linear_prefill(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                       float *qkv, const float *z, float *beta, float *alpha, float *attention,
                       void *stream);

/* The same for the value heads v_head0 .. v_head0+v_head_count-1 only. The q
 * and k channels (all key heads) are convolved and normalised by every call,
 * since value head h reads key head h % qk_heads (ops.rs:699); of the v
 * channels, gates, z and output only the range's are read or written, and
 * only the range's conv-state channels and delta-state heads advance. The
 * reference runs one task per value head (ops.rs:717-733); value heads are
 * the unit that DeltaNet prefill shards across GPUs. */
int q38_linear_prefill_heads(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq,
                             int count, int v_head0, int v_head_count, float *qkv, const float *z,
                             float *beta, float *alpha, float *attention, void *stream);

/* Host-pointer forms of the two prefill calls, for the reference's host
 * slices (batch_full_attention / batch_linear_attention, ops.rs:1156-1172,
 * :1088-1099, which hold [count][dim] rows per sequence): the same
 * [nseq][count][dim] layouts as above in HOST memory (pinned for best speed).
 * The prompt is streamed through a device staging buffer that
 * q38_state_reserve_prefill sizes, piece by piece; each piece continues from
 * the cache rows / recurrent state the previous piece left, so the result is
 * that of one call. The in-place inputs (key; qkv, beta, alpha) are written
 * back, and the call synchronises `stream` before returning. */
int q38_full_prefill_host(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                          int base_position, const float *q_and_gate, float *key,
                          const float *value, float *attention, void *stream);
int q38_linear_prefill_host(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq,
                            int count, float *qkv, const float *z, float *beta, float *alpha,
                            float *attention, void *stream);

/* ---------------------------------------------------------- decode (host) */

/* Host-pointer forms of the two decode calls: copy the step's inputs from
 * host memory (pinned for best speed), run the step on the device-resident
 * state, copy the outputs (and the in-place-modified inputs) back, and
 * synchronise. positions is a HOST array here; an out-of-range position
 * returns Q38_ERR_ARG before any work, as full_core does (ops.rs:860-864). */
int q38_full_decode_host(q38_ctx *ctx, q38_state *st, int layer, int batch,
                         const float *q_and_gate, float *key, const float *value,
                         const int32_t *positions, float *attention, void *stream);
int q38_linear_decode_host(q38_ctx *ctx, q38_state *st, int layer, int batch, float *qkv,
                           const float *z, float *beta, float *alpha, float *attention,
                           void *stream);

/* ------------------------------------------------- reference-signature mirrors */

/* Exactly the argument meaning of the reference's linear_core
 * (src/model/ops.rs:647-657) with host slices: conv_state [qkv_dim][3] and
 * delta_state [v_heads][128][128] are uploaded into sequence 0 of `layer`'s
 * slot of `st`, the step runs on the GPU, and every &mut slice is written
 * back. For parity checks; resident-state callers use q38_linear_decode. */
int q38_linear_core(q38_ctx *ctx, q38_state *st, int layer, float *conv_state,
                    float *delta_state, float *qkv, const float *z, float *beta, float *alpha,
                    float *attention);

/* Exactly the argument meaning of the reference's full_core
 * (src/model/ops.rs:812-827) with host slices. key_cache/value_cache hold
 * cache_rows rows of kv_heads*256 floats, row = (layer/4)*context_length+pos;
 * positions 0..current_position-1 of this layer are uploaded into sequence 0
 * of `st`, the step runs on the GPU, and row current_position, key, q, gate,
 * scores (the softmax numerators exp(s-max) per head, as the reference leaves
 * them) and attention are written back. q/gate/scores may be NULL. */
int q38_full_core(q38_ctx *ctx, q38_state *st, int layer, const float *q_and_gate, float *key,
                  const float *value, float *q, float *gate, float *scores, float *attention,
                  float *key_cache, float *value_cache, size_t cache_rows,
                  size_t context_length, uint32_t current_position);

/* ------------------------------------------- projections around the cores */

/* ggml tensor types the projections accept (src/gguf/mod.rs:83-103). The
 * K-quants and IQ4_NL / IQ4_XS take the integer path of the reference's
 * `project` (matrix_type_q8_k, src/model/ops.rs:105-120): the f32 activation
 * is quantized to Q8_K blocks and dotted in integers (src/kernel/tensor.rs:
 * 301-460, src/kernel/iq.rs:355-405); the others take the f32 activation
 * directly. The reference's other IQ types (IQ1_S, IQ1_M, IQ2_XXS, IQ2_XS,
 * IQ2_S, IQ3_XXS, IQ3_S), which decode through ggml's lookup grids, are not
 * accepted here (Q38_ERR_ARG). */
#define Q38_GGML_F32 0
#define Q38_GGML_F16 1
#define Q38_GGML_Q8_0 8
#define Q38_GGML_Q2_K 10
#define Q38_GGML_Q3_K 11
#define Q38_GGML_Q4_K 12
#define Q38_GGML_Q5_K 13
#define Q38_GGML_Q6_K 14
#define Q38_GGML_IQ4_NL 20
#define Q38_GGML_IQ4_XS 23
#define Q38_GGML_BF16 30

/* Bytes of one Q8_K activation block in the reference's layout
 * (Q38Q8KBlock, src/kernel/mod.rs:20-27): f32 scale, int8 quants[256],
 * int16 sums[16]. */
#define Q38_Q8K_BLOCK_BYTES 292

typedef struct q38_weight q38_weight;

/* Copies a projection matrix to the device: `rows` rows of `width` inputs
 * each, the GGUF tensor of shape [width, rows] (TensorEntry, whose rows are
 * row_bytes(type, width) bytes, src/kernel/tensor.rs:46-53). data is a HOST
 * pointer to exactly rows * row_bytes bytes (nbytes). width must be a
 * multiple of 4 (of 256 for the integer-path types) and at most 32768; the model's
 * projections are 5120 and 6144 wide. */
int q38_weight_create(q38_ctx *ctx, int ggml_type, int64_t width, int64_t rows, const void *data,
                      size_t nbytes, q38_weight **out);
int q38_weight_destroy(q38_weight *w);
int q38_weight_info(const q38_weight *w, int *ggml_type, int64_t *width, int64_t *rows);

/* The same from a GGUF checkpoint: tensor `name` must be 2-D (as
 * tensor_gemv_* require, tensor.rs:1095-1110) of an accepted type. */
int q38_weight_from_gguf(q38_ctx *ctx, const char *path, const char *name, q38_weight **out);

/* Builds, once, the weight's integer planes for projections of 9 or more
 * tokens (Q4_K, Q5_K and Q6_K only; Q38_ERR_ARG for other types). Per weight
 * value the reference's integer product scale * quant is kept as two bytes,
 * and per (row, 256-block) a 16-byte record of d, dmin and the sub-block
 * mins: 2 bytes per weight + 1/16 byte, i.e. 3.7x a Q4_K matrix's bytes and
 * 2.5x a Q6_K one's, in device memory next to the GGUF copy. Every later
 * projection of 9+ tokens through this weight (q38_project, the layer calls)
 * then streams the planes into tcgen05 kind::i8 products instead of building
 * its tensor-core operands from the packed blocks; results stay
 * bit-identical to the reference's scalar integer dot. Synchronous;
 * q38_weight_destroy frees the planes. */
int q38_weight_build_planes(q38_weight *w);

/* quantize_q8_k (src/kernel/quant.rs:98-124) of `batch` rows of `width`
 * DEVICE floats (width a multiple of 256, input 16-byte aligned) into
 * batch * width / 256 DEVICE blocks of Q38_Q8K_BLOCK_BYTES in the reference's
 * layout. Bit-identical to the reference. */
int q38_quantize_q8_k(q38_ctx *ctx, int batch, int64_t width, const float *input, void *blocks,
                      void *stream);

/* project / batch_project (src/model/ops.rs:623-640, 1016-1031): output
 * [batch][rows] = W input[batch][width], DEVICE pointers, token-major as
 * gemm_rows writes it (tensor.rs:978-1000). K-quant weights: the input is
 * quantized to Q8_K on the device and each output is bit-identical to the
 * reference's scalar integer dot. F32/F16/BF16/Q8_0: f32 dot, equal to the
 * reference's within rounding. Up to 8 tokens the Q8_K quantization runs
 * inside the GEMV; 9 or more tokens over Q4_K / Q5_K / Q6_K weights run on
 * the tensor cores (from the weight's integer planes when
 * q38_weight_build_planes made them), with the quantized input in a context
 * scratch buffer that
 * grows on first use (q38_ctx_reserve_projection sizes it ahead, so that
 * later calls allocate nothing). Input must be 16-byte aligned. Launched as
 * a programmatic dependent of the previous kernel on the stream: the first
 * weight tiles are fetched while that kernel finishes. */
int q38_project(q38_ctx *ctx, const q38_weight *w, int batch, const float *input, float *output,
                void *stream);
/* Host-pointer form (synchronous). */
int q38_project_host(q38_ctx *ctx, const q38_weight *w, int batch, const float *input,
                     float *output);
/* Sizes the context's projection scratch (the quantized input of the
 * tensor-core path, and the partial sums of the chunked f32-input form that
 * 9+ tokens over F32/F16/BF16/Q8_0 weights of up to 128 rows take) for
 * `batch` tokens of `width` inputs (a multiple of 256), so that later
 * q38_project / *_attention_decode calls allocate nothing. Call it before
 * any stream capture. */
int q38_ctx_reserve_projection(q38_ctx *ctx, int batch, int64_t width);

/* The projections of one Gated DeltaNet layer (Q38Attention::Linear,
 * src/model/mod.rs:28-48): attn_qkv [hidden -> qkv_dim], attn_gate [hidden ->
 * v_dim], ssm_beta / ssm_alpha [hidden -> v_heads], ssm_out [v_dim -> hidden]. */
typedef struct q38_linear_projections {
    const q38_weight *qkv, *z, *beta, *alpha, *out;
} q38_linear_projections;

/* The projections of one full-attention layer (Q38Attention::Full):
 * attn_q [hidden -> 2*q_dim, query and gate per head], attn_k / attn_v
 * [hidden -> kv_dim], attn_output [q_dim -> hidden]. */
typedef struct q38_full_projections {
    const q38_weight *q, *k, *v, *out;
} q38_full_projections;

/* linear_attention (src/model/ops.rs:744-803) for `batch` sequences: norm
 * [batch][hidden] DEVICE (the attn_norm output), branch [batch][hidden]
 * DEVICE out. Quantizes norm once, runs the four input projections, the
 * DeltaNet step on the resident state (as q38_linear_decode), quantizes the
 * core's output and runs ssm_out. */
int q38_linear_attention_decode(q38_ctx *ctx, q38_state *st, int layer, int batch,
                                const q38_linear_projections *w, const float *norm, float *branch,
                                void *stream);

/* full_attention (src/model/ops.rs:941-981) for `batch` sequences at DEVICE
 * positions[batch] (max_position as for q38_full_decode). */
int q38_full_attention_decode(q38_ctx *ctx, q38_state *st, int layer, int batch,
                              const q38_full_projections *w, const float *norm,
                              const int32_t *positions, int max_position, float *branch,
                              void *stream);

/* Sizes, for up to max_tokens prompt tokens per call (summed over its
 * sequences), everything the two calls below use: the core prefill scratch
 * (as q38_state_reserve_prefill), the projections' outputs and the context's
 * projection scratch (~90 KB per token). Allocates; call it once at set-up. */
int q38_state_reserve_attention_prefill(q38_state *st, int max_tokens);

/* batch_linear_attention (src/model/ops.rs:1032-1114) for sequences
 * [seq0, seq0 + nseq) of `count` tokens each: norm [nseq][count][hidden]
 * DEVICE (the attn_norm output), branch [nseq][count][hidden] DEVICE out. The
 * four input projections over all nseq*count tokens (tensor cores from 9
 * tokens on), the chunked core on the resident state (as q38_linear_prefill),
 * the output projection. */
int q38_linear_attention_prefill(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                                 const q38_linear_projections *w, const float *norm, float *branch,
                                 void *stream);

/* batch_full_attention (src/model/ops.rs:1116-1185): positions base_position
 * .. base_position+count-1 of each sequence, as q38_full_prefill (bf16 KV
 * state). */
int q38_full_attention_prefill(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                               int base_position, const q38_full_projections *w, const float *norm,
                               float *branch, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* Q38ATTN_H */
