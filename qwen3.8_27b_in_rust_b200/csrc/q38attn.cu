// q38attn.cu -- the C ABI (include/q38attn.h): context, weights, device state,
// argument validation and the host-pointer mirrors of the reference's
// linear_core / full_core. Kernels live in attn_decode.cu and
// deltanet_decode.cu; nothing here computes on the CPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "q38_internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    cudaGetLastError();  // clear the sticky-free error so later calls start clean
    return fail(Q38_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define Q38_CUDA(call)                                             \
    do {                                                           \
        cudaError_t e_ = (call);                                   \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);        \
    } while (0)

// Makes `device` current for the duration of a call and restores the
// caller's device afterwards.
struct DeviceGuard {
    int prev = -1, dev;
    explicit DeviceGuard(int d) : dev(d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    }
};

uint16_t f32_to_bf16_bits(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return uint16_t((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return uint16_t(u >> 16);
}

float bf16_bits_to_f32(uint16_t h) {
    const uint32_t u = uint32_t(h) << 16;
    float x;
    std::memcpy(&x, &u, 4);
    return x;
}

int check_geom(const q38_geom &g) {
    if (g.attn_head_dim != q38::kAttnHeadDim || g.rope_dims != q38::kRopeDims)
        return fail(Q38_ERR_ARG, "attention head_dim must be 256 with 64 RoPE dims");
    if (g.attn_kv_heads <= 0 || g.attn_heads != q38::kGroup * g.attn_kv_heads)
        return fail(Q38_ERR_ARG, "attn_heads must be 6 * attn_kv_heads (got %d, %d)",
                    g.attn_heads, g.attn_kv_heads);
    if (g.linear_head_dim != q38::kLinHeadDim || g.conv_kernel != q38::kConvKernel)
        return fail(Q38_ERR_ARG, "DeltaNet head_dim must be 128 with a kernel-4 conv");
    if (g.linear_qk_heads <= 0 || g.linear_v_heads <= 0 ||
        g.linear_v_heads % g.linear_qk_heads != 0)
        return fail(Q38_ERR_ARG, "linear_v_heads must be a positive multiple of linear_qk_heads");
    if (!(g.rope_theta > 0.f) || !(g.rms_eps > 0.f))
        return fail(Q38_ERR_ARG, "rope_theta and rms_eps must be positive");
    return Q38_OK;
}

int check_ctx(const q38_ctx *ctx) {
    if (!ctx) return fail(Q38_ERR_ARG, "null context");
    return Q38_OK;
}

int check_state(const q38_ctx *ctx, const q38_state *st) {
    if (int rc = check_ctx(ctx)) return rc;
    if (!st) return fail(Q38_ERR_ARG, "null state");
    if (st->ctx != ctx) return fail(Q38_ERR_ARG, "state belongs to another context");
    return Q38_OK;
}

int full_slot_of(const q38_state *st, int layer, int *slot) {
    if (layer < 0 || layer > 64 || !q38::is_full_attention(layer))
        return fail(Q38_ERR_ARG, "layer %d is not a full-attention layer", layer);
    const int s = q38::full_index(layer);
    if (s >= st->full_slots)
        return fail(Q38_ERR_ARG, "layer %d needs KV slot %d but the state has %d", layer, s,
                    st->full_slots);
    *slot = s;
    return Q38_OK;
}

int linear_slot_of(const q38_state *st, int layer, int *slot) {
    if (layer < 0 || layer >= 64 || q38::is_full_attention(layer))
        return fail(Q38_ERR_ARG, "layer %d is not a Gated DeltaNet layer", layer);
    const int s = q38::recurrent_index(layer);
    if (s >= st->linear_slots)
        return fail(Q38_ERR_ARG, "layer %d needs recurrent slot %d but the state has %d", layer,
                    s, st->linear_slots);
    *slot = s;
    return Q38_OK;
}

size_t kv_seq_elems(const q38_state *st) {
    return size_t(st->ctx->geom.attn_kv_heads) * st->context_length * q38::kAttnHeadDim;
}

unsigned char *kv_seq_base(const q38_state *st, void *cache, int slot, int seq) {
    return static_cast<unsigned char *>(cache) +
           (size_t(slot) * st->kv_slot_elems + size_t(seq) * kv_seq_elems(st)) * st->kv_elem;
}

size_t conv_seq_floats(const q38_ctx *ctx) { return size_t(ctx->qkv_dim) * 3; }
size_t delta_seq_floats(const q38_ctx *ctx) {
    return size_t(ctx->geom.linear_v_heads) * q38::kLinHeadDim * q38::kLinHeadDim;
}

template <typename T>
int device_copy_of(const float *host, size_t n, T **dev) {
    Q38_CUDA(cudaMalloc(dev, n * sizeof(float)));
    Q38_CUDA(cudaMemcpy(*dev, host, n * sizeof(float), cudaMemcpyHostToDevice));
    return Q38_OK;
}

void free_full(q38::FullWeights &w) {
    cudaFree(w.q_norm);
    cudaFree(w.k_norm);
    w = {};
}

void free_linear(q38::LinearWeights &w) {
    cudaFree(w.conv_w);
    cudaFree(w.dt_bias);
    cudaFree(w.ssm_a);
    cudaFree(w.ssm_norm);
    w = {};
}

void free_state(q38_state *st) {
    cudaFree(st->kcache);
    cudaFree(st->vcache);
    cudaFree(st->conv_state);
    cudaFree(st->delta_state);
    cudaFree(st->lin_group_count);
    cudaFree(st->qprep);
    cudaFree(st->part_o);
    cudaFree(st->part_ml);
    cudaFree(st->d_err);
    cudaFree(st->stage);
    cudaFree(st->proj_stage);
    cudaFree(st->layer_prefill);
    cudaFree(st->stage_pos);
    cudaFree(st->prefill_rope);
    cudaFree(st->prefill_v16);
    cudaFree(st->prefill_lin);
    cudaFree(st->prefill_stage);
    cudaFree(st->ckpt_conv);
    cudaFree(st->ckpt_delta);
    cudaFree(st->split_local);
    cudaFree(st->split_gathered);
    for (void *q : st->p2p_opened) cudaIpcCloseMemHandle(q);
    st->p2p_opened.clear();
    cudaFree(st->p2p_buf);
    cudaFree(st->p2p_peers_dev);
    cudaFree(st->prefill_k16);
    if (st->host_err) cudaFreeHost(st->host_err);
    for (int i = 0; i < q38_state::kSides; ++i) {
        if (st->side[i]) cudaStreamDestroy(st->side[i]);
        if (st->side_join[i]) cudaEventDestroy(st->side_join[i]);
    }
    if (st->side_fork) cudaEventDestroy(st->side_fork);
    if (st->host_ev_prep) cudaEventDestroy(st->host_ev_prep);
    if (st->host_ev_back) cudaEventDestroy(st->host_ev_back);
    if (st->host_out) cudaStreamDestroy(st->host_out);
}

// The write-back stream and events of the host-pointer decode, created once
// per state.
cudaError_t ensure_host_out(q38_state *st) {
    if (st->host_out) return cudaSuccess;
    cudaError_t e = cudaEventCreateWithFlags(&st->host_ev_prep, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st->host_ev_back, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st->host_out, cudaStreamNonBlocking);
    return e;
}

// Host-pointer calls: enqueues on `s` a copy of the state's device error bits
// into a pinned host word (read after the call's final synchronisation by
// host_call_status).
cudaError_t enqueue_error_read(q38_state *st, cudaStream_t s) {
    if (!st->host_err) {
        cudaError_t e = cudaHostAlloc(reinterpret_cast<void **>(&st->host_err), sizeof(int),
                                      cudaHostAllocDefault);
        if (e != cudaSuccess) return e;
        *st->host_err = 0;
    }
    return cudaMemcpyAsync(st->host_err, st->d_err, sizeof(int), cudaMemcpyDeviceToHost, s);
}

// Status of a host-pointer call once its stream has synchronised: a bounded
// device wait that gave up (the bits stay set until q38_state_errors reads
// and clears them) is Q38_ERR_TIMEOUT.
int host_call_status(const q38_state *st) {
    if (st->host_err && (*st->host_err & Q38_DEVERR_TIMEOUT))
        return fail(Q38_ERR_TIMEOUT, "a bounded device wait gave up (device error bits 0x%x)",
                    *st->host_err);
    return Q38_OK;
}

// True when p lies in pinned host memory mapped into `device`'s address
// space (cudaHostAlloc, or registered with cudaHostRegisterMapped, against
// that device); *dev is then the device's address of p. Pageable memory, and
// pinned memory registered against another device, give false.
bool mapped_host(const void *p, int device, void **dev) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();  // the error is not sticky; clear it
        return false;
    }
    if (at.type != cudaMemoryTypeHost || !at.devicePointer || at.device != device) return false;
    *dev = at.devicePointer;
    return true;
}

// Validates a decode call and fills the launch arguments (device pointers).
// Sharded calls (split-sequence decode) write partials instead of `attention`
// and may see positions past this shard's capacity.
int prepare_full_decode(q38_ctx *ctx, q38_state *st, int layer, int batch,
                        const float *q_and_gate, float *key, const float *value,
                        const int32_t *positions, int max_position, float *attention,
                        q38::AttnDecodeLaunch *a, bool sharded = false) {
    if (int rc = check_state(ctx, st)) return rc;
    int slot;
    if (int rc = full_slot_of(st, layer, &slot)) return rc;
    if (batch <= 0 || batch > st->batch)
        return fail(Q38_ERR_ARG, "batch %d outside 1..%d", batch, st->batch);
    if (!q_and_gate || !key || !value || !positions || (!attention && !sharded))
        return fail(Q38_ERR_ARG, "null tensor argument");
    auto it = ctx->full.find(layer);
    if (it == ctx->full.end())
        return fail(Q38_ERR_ARG, "full-attention layer %d has no bound weights", layer);
    if (max_position < 0) max_position = st->context_length - 1;
    if (!sharded && max_position >= st->context_length)
        return fail(Q38_ERR_ARG, "max_position %d >= context_length %d", max_position,
                    st->context_length);
    const q38_geom &g = ctx->geom;
    *a = q38::AttnDecodeLaunch{};
    a->q_and_gate = q_and_gate;
    a->key = key;
    a->value = value;
    a->positions = positions;
    a->attention = attention;
    a->kcache = kv_seq_base(st, st->kcache, slot, 0);
    a->vcache = kv_seq_base(st, st->vcache, slot, 0);
    a->qprep = st->qprep;
    a->part_o = st->part_o;
    a->part_ml = st->part_ml;
    a->err = st->d_err;
    a->q_norm = it->second.q_norm;
    a->k_norm = it->second.k_norm;
    a->batch = batch;
    a->context_length = st->context_length;
    a->heads = g.attn_heads;
    a->kv_heads = g.attn_kv_heads;
    a->kv_dtype = st->kv_dtype;
    a->max_position = max_position;
    a->max_splits = st->max_splits;
    a->theta_scale = ctx->theta_scale;
    a->eps = g.rms_eps;
    a->wait_ns = st->debug_wait_ns;
    a->skip_kv_loads = (st->debug_flags & Q38_DEBUG_SKIP_KV_LOADS) ? 1 : 0;
    return Q38_OK;
}

int prepare_linear_decode(q38_ctx *ctx, q38_state *st, int layer, int batch, float *qkv,
                          const float *z, float *beta, float *alpha, float *attention,
                          q38::LinearDecodeLaunch *a) {
    if (int rc = check_state(ctx, st)) return rc;
    int slot;
    if (int rc = linear_slot_of(st, layer, &slot)) return rc;
    if (batch <= 0 || batch > st->batch)
        return fail(Q38_ERR_ARG, "batch %d outside 1..%d", batch, st->batch);
    if (!qkv || !z || !beta || !alpha || !attention)
        return fail(Q38_ERR_ARG, "null tensor argument");
    auto it = ctx->linear.find(layer);
    if (it == ctx->linear.end())
        return fail(Q38_ERR_ARG, "DeltaNet layer %d has no bound weights", layer);
    const q38_geom &g = ctx->geom;
    *a = q38::LinearDecodeLaunch{};
    a->qkv = qkv;
    a->z = z;
    a->beta = beta;
    a->alpha = alpha;
    a->attention = attention;
    a->conv_state = st->conv_state + size_t(slot) * st->batch * conv_seq_floats(ctx);
    a->delta_state = st->delta_state + size_t(slot) * st->batch * delta_seq_floats(ctx);
    a->conv_w = it->second.conv_w;
    a->dt_bias = it->second.dt_bias;
    a->ssm_a = it->second.ssm_a;
    a->ssm_norm = it->second.ssm_norm;
    a->batch = batch;
    a->qk_heads = g.linear_qk_heads;
    a->v_heads = g.linear_v_heads;
    a->eps = g.rms_eps;
    a->group_count = st->lin_group_count + size_t(slot) * st->batch * g.linear_qk_heads;
    a->err = st->d_err;
    a->wait_ns = st->debug_wait_ns;
    a->sm_count = ctx->sm_count;
    return Q38_OK;
}

}  // namespace

void q38::record_error(const char *msg) { g_last_error = msg ? msg : ""; }

int q38::linear_decode_prepped(q38_ctx *ctx, q38_state *st, int layer, int batch, float *qkv,
                               const float *z, float *beta, float *alpha, float *attention,
                               cudaStream_t stream) {
    q38::LinearDecodeLaunch a;
    if (int rc = prepare_linear_decode(ctx, st, layer, batch, qkv, z, beta, alpha, attention, &a))
        return rc;
    a.prepped = 1;
    DeviceGuard guard(ctx->device);
    cudaError_t e = q38::launch_linear_decode(a, stream);
    if (e != cudaSuccess) return cuda_fail(e, "DeltaNet decode launch");
    return Q38_OK;
}

int q38::linear_layer_prologue_args(q38_ctx *ctx, q38_state *st, int layer, float **conv_state,
                                    const float **conv_w, const float **dt_bias,
                                    const float **ssm_a) {
    if (int rc = check_state(ctx, st)) return rc;
    int slot;
    if (int rc = linear_slot_of(st, layer, &slot)) return rc;
    auto it = ctx->linear.find(layer);
    if (it == ctx->linear.end())
        return fail(Q38_ERR_ARG, "DeltaNet layer %d has no bound weights", layer);
    *conv_state = st->conv_state + size_t(slot) * st->batch * conv_seq_floats(ctx);
    *conv_w = it->second.conv_w;
    *dt_bias = it->second.dt_bias;
    *ssm_a = it->second.ssm_a;
    return Q38_OK;
}

extern "C" {

void q38_geom_default(q38_geom *g) {
    if (!g) return;
    g->attn_heads = 24;
    g->attn_kv_heads = 4;
    g->attn_head_dim = 256;
    g->rope_dims = 64;
    g->rope_theta = 10000000.0f;
    g->linear_qk_heads = 16;
    g->linear_v_heads = 48;
    g->linear_head_dim = 128;
    g->conv_kernel = 4;
    g->rms_eps = 1e-6f;
}

const char *q38_last_error(void) { return g_last_error.c_str(); }

const char *q38_version(void) { return "q38attn 0.1.0 (sm_100a)"; }

int q38_ctx_create(const q38_geom *geom, int device, q38_ctx **out) {
    if (!out) return fail(Q38_ERR_ARG, "null output pointer");
    *out = nullptr;
    q38_geom g;
    q38_geom_default(&g);
    if (geom) g = *geom;
    if (int rc = check_geom(g)) return rc;
    int count = 0;
    Q38_CUDA(cudaGetDeviceCount(&count));
    if (device < 0 || device >= count)
        return fail(Q38_ERR_ARG, "device %d outside 0..%d", device, count - 1);
    DeviceGuard guard(device);
    cudaDeviceProp prop;
    Q38_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(Q38_ERR_ARG, "device %d is sm_%d%d; this library is built for sm_100a",
                    device, prop.major, prop.minor);
    q38_ctx *ctx = new q38_ctx();
    ctx->device = device;
    ctx->geom = g;
    ctx->sm_count = prop.multiProcessorCount;
    // rope(): theta_scale = theta^(-2/64) (ops.rs:596), evaluated with powf.
    ctx->theta_scale = std::pow(g.rope_theta, -2.0f / float(g.rope_dims));
    ctx->q_dim = g.attn_heads * g.attn_head_dim;
    ctx->qg_dim = 2 * ctx->q_dim;
    ctx->kv_dim = g.attn_kv_heads * g.attn_head_dim;
    ctx->qk_dim = g.linear_qk_heads * g.linear_head_dim;
    ctx->v_dim = g.linear_v_heads * g.linear_head_dim;
    ctx->qkv_dim = 2 * ctx->qk_dim + ctx->v_dim;
    *out = ctx;
    return Q38_OK;
}

int q38_ctx_destroy(q38_ctx *ctx) {
    if (!ctx) return Q38_OK;
    {
        DeviceGuard guard(ctx->device);
        for (auto &kv : ctx->full) free_full(kv.second);
        for (auto &kv : ctx->linear) free_linear(kv.second);
        cudaFree(ctx->proj_scratch);
        cudaFree(ctx->proj_part);
    }
    delete ctx;
    return Q38_OK;
}

int q38_bind_full_layer(q38_ctx *ctx, int layer, const float *q_norm, const float *k_norm) {
    if (int rc = check_ctx(ctx)) return rc;
    if (layer < 0 || layer > 64 || !q38::is_full_attention(layer))
        return fail(Q38_ERR_ARG, "layer %d is not a full-attention layer", layer);
    if (!q_norm || !k_norm) return fail(Q38_ERR_ARG, "null weight");
    DeviceGuard guard(ctx->device);
    q38::FullWeights w;
    int rc = device_copy_of(q_norm, q38::kAttnHeadDim, &w.q_norm);
    if (!rc) rc = device_copy_of(k_norm, q38::kAttnHeadDim, &w.k_norm);
    if (rc) {
        free_full(w);
        return rc;
    }
    auto it = ctx->full.find(layer);
    if (it != ctx->full.end()) free_full(it->second);
    ctx->full[layer] = w;
    return Q38_OK;
}

int q38_bind_linear_layer(q38_ctx *ctx, int layer, const float *conv1d, const float *dt_bias,
                          const float *ssm_a, const float *ssm_norm) {
    if (int rc = check_ctx(ctx)) return rc;
    if (layer < 0 || layer >= 64 || q38::is_full_attention(layer))
        return fail(Q38_ERR_ARG, "layer %d is not a Gated DeltaNet layer", layer);
    if (!conv1d || !dt_bias || !ssm_a || !ssm_norm) return fail(Q38_ERR_ARG, "null weight");
    DeviceGuard guard(ctx->device);
    q38::LinearWeights w;
    const size_t vh = size_t(ctx->geom.linear_v_heads);
    int rc = device_copy_of(conv1d, size_t(ctx->qkv_dim) * q38::kConvKernel, &w.conv_w);
    if (!rc) rc = device_copy_of(dt_bias, vh, &w.dt_bias);
    if (!rc) rc = device_copy_of(ssm_a, vh, &w.ssm_a);
    if (!rc) rc = device_copy_of(ssm_norm, q38::kLinHeadDim, &w.ssm_norm);
    if (rc) {
        free_linear(w);
        return rc;
    }
    auto it = ctx->linear.find(layer);
    if (it != ctx->linear.end()) free_linear(it->second);
    ctx->linear[layer] = w;
    return Q38_OK;
}

int q38_state_create(q38_ctx *ctx, int batch, int context_length, int full_slots,
                     int linear_slots, int kv_dtype, q38_state **out) {
    if (!out) return fail(Q38_ERR_ARG, "null output pointer");
    *out = nullptr;
    if (int rc = check_ctx(ctx)) return rc;
    if (batch <= 0 || context_length <= 0 || full_slots < 0 || linear_slots < 0 ||
        full_slots > 17 || linear_slots > 48)
        return fail(Q38_ERR_ARG,
                    "bad state shape (batch %d, context %d, full slots %d, linear slots %d)",
                    batch, context_length, full_slots, linear_slots);
    if (kv_dtype != Q38_KV_F32 && kv_dtype != Q38_KV_BF16)
        return fail(Q38_ERR_ARG, "unknown kv_dtype %d", kv_dtype);
    DeviceGuard guard(ctx->device);
    q38_state *st = new q38_state();
    st->ctx = ctx;
    st->batch = batch;
    st->context_length = context_length;
    st->full_slots = full_slots;
    st->linear_slots = linear_slots;
    st->kv_dtype = kv_dtype;
    st->kv_elem = kv_dtype == Q38_KV_BF16 ? 2 : 4;
    st->kv_slot_elems = size_t(batch) * kv_seq_elems(st);
    st->max_splits = q38::attn_decode_max_splits(context_length, kv_dtype);
    const q38_geom &g = ctx->geom;
    const size_t kv_bytes = size_t(full_slots) * st->kv_slot_elems * st->kv_elem;
    const size_t conv_floats = size_t(linear_slots) * batch * conv_seq_floats(ctx);
    const size_t delta_floats = size_t(linear_slots) * batch * delta_seq_floats(ctx);
    const size_t parts = size_t(batch) * g.attn_heads * st->max_splits;
    const size_t full_stage = size_t(ctx->qg_dim) + 2 * ctx->kv_dim + ctx->q_dim;
    const size_t lin_stage = size_t(ctx->qkv_dim) + ctx->v_dim + 2 * g.linear_v_heads + ctx->v_dim;
    st->stage_floats = size_t(batch) * (full_stage > lin_stage ? full_stage : lin_stage);
    auto alloc = [&](void **p, size_t bytes) -> cudaError_t {
        if (bytes == 0) return cudaSuccess;
        cudaError_t e = cudaMalloc(p, bytes);
        if (e == cudaSuccess) e = cudaMemset(*p, 0, bytes);
        return e;
    };
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = alloc(&st->kcache, kv_bytes);
    if (e == cudaSuccess) e = alloc(&st->vcache, kv_bytes);
    if (e == cudaSuccess) e = alloc((void **)&st->conv_state, conv_floats * 4);
    if (e == cudaSuccess) e = alloc((void **)&st->delta_state, delta_floats * 4);
    if (e == cudaSuccess)
        e = alloc((void **)&st->lin_group_count,
                  size_t(linear_slots) * batch * g.linear_qk_heads * sizeof(int));
    if (e == cudaSuccess) e = alloc((void **)&st->qprep, size_t(batch) * ctx->q_dim * 4);
    if (e == cudaSuccess) e = alloc((void **)&st->part_o, parts * q38::kAttnHeadDim * 4);
    if (e == cudaSuccess) e = alloc((void **)&st->part_ml, parts * 2 * 4);
    if (e == cudaSuccess) e = alloc((void **)&st->d_err, sizeof(int));
    if (e == cudaSuccess) e = alloc((void **)&st->stage, st->stage_floats * 4);
    if (e == cudaSuccess) e = alloc((void **)&st->proj_stage, st->stage_floats * 4);
    if (e == cudaSuccess) e = alloc((void **)&st->stage_pos, size_t(batch) * 4);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st->side_fork, cudaEventDisableTiming);
    for (int i = 0; i < q38_state::kSides && e == cudaSuccess; ++i) {
        e = cudaStreamCreateWithFlags(&st->side[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st->side_join[i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) {
        free_state(st);
        delete st;
        return cuda_fail(e, "q38_state_create allocation");
    }
    *out = st;
    return Q38_OK;
}

int q38_state_destroy(q38_state *st) {
    if (!st) return Q38_OK;
    {
        DeviceGuard guard(st->ctx->device);
        free_state(st);
    }
    delete st;
    return Q38_OK;
}

int q38_state_reset(q38_state *st, void *stream) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    DeviceGuard guard(st->ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t kv_bytes = size_t(st->full_slots) * st->kv_slot_elems * st->kv_elem;
    if (kv_bytes) {
        Q38_CUDA(cudaMemsetAsync(st->kcache, 0, kv_bytes, s));
        Q38_CUDA(cudaMemsetAsync(st->vcache, 0, kv_bytes, s));
    }
    const size_t n = size_t(st->linear_slots) * st->batch;
    if (n) {
        Q38_CUDA(cudaMemsetAsync(st->conv_state, 0, n * conv_seq_floats(st->ctx) * 4, s));
        Q38_CUDA(cudaMemsetAsync(st->delta_state, 0, n * delta_seq_floats(st->ctx) * 4, s));
        Q38_CUDA(cudaMemsetAsync(st->lin_group_count, 0,
                                 n * st->ctx->geom.linear_qk_heads * sizeof(int), s));
    }
    return Q38_OK;
}

namespace {

// Copies sequences [seq0, seq0+nseq) of every DeltaNet slot between the state
// arrays and the checkpoint arrays: one strided copy per array (rows = slots).
int copy_recurrent(q38_state *st, int seq0, int nseq, bool to_checkpoint, cudaStream_t s) {
    const q38_ctx *ctx = st->ctx;
    const size_t rows = size_t(st->linear_slots);
    const size_t cs = conv_seq_floats(ctx) * 4, ds = delta_seq_floats(ctx) * 4;
    float *c_src = to_checkpoint ? st->conv_state : st->ckpt_conv;
    float *c_dst = to_checkpoint ? st->ckpt_conv : st->conv_state;
    float *d_src = to_checkpoint ? st->delta_state : st->ckpt_delta;
    float *d_dst = to_checkpoint ? st->ckpt_delta : st->delta_state;
    const size_t c_off = size_t(seq0) * cs, d_off = size_t(seq0) * ds;
    Q38_CUDA(cudaMemcpy2DAsync(reinterpret_cast<char *>(c_dst) + c_off, st->batch * cs,
                               reinterpret_cast<const char *>(c_src) + c_off, st->batch * cs,
                               size_t(nseq) * cs, rows, cudaMemcpyDeviceToDevice, s));
    Q38_CUDA(cudaMemcpy2DAsync(reinterpret_cast<char *>(d_dst) + d_off, st->batch * ds,
                               reinterpret_cast<const char *>(d_src) + d_off, st->batch * ds,
                               size_t(nseq) * ds, rows, cudaMemcpyDeviceToDevice, s));
    return Q38_OK;
}

int check_seq_range(const q38_state *st, int seq0, int nseq) {
    if (nseq <= 0 || seq0 < 0 || seq0 + nseq > st->batch)
        return fail(Q38_ERR_ARG, "sequences [%d, %d) outside the state's %d", seq0, seq0 + nseq,
                    st->batch);
    return Q38_OK;
}

}  // namespace

int q38_state_checkpoint(q38_state *st, int seq0, int nseq, void *stream) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    if (int rc = check_seq_range(st, seq0, nseq)) return rc;
    if (st->linear_slots == 0) return Q38_OK;  // no recurrent state to keep
    DeviceGuard guard(st->ctx->device);
    if (!st->ckpt_conv) {
        const size_t n = size_t(st->linear_slots) * st->batch;
        Q38_CUDA(cudaMalloc(&st->ckpt_conv, n * conv_seq_floats(st->ctx) * 4));
        Q38_CUDA(cudaMalloc(&st->ckpt_delta, n * delta_seq_floats(st->ctx) * 4));
        st->ckpt_valid.assign(size_t(st->batch), 0);
    }
    if (int rc = copy_recurrent(st, seq0, nseq, true, static_cast<cudaStream_t>(stream))) return rc;
    for (int b = seq0; b < seq0 + nseq; ++b) st->ckpt_valid[size_t(b)] = 1;
    return Q38_OK;
}

int q38_state_restore(q38_state *st, int seq0, int nseq, void *stream) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    if (int rc = check_seq_range(st, seq0, nseq)) return rc;
    if (st->linear_slots == 0) return Q38_OK;
    for (int b = seq0; b < seq0 + nseq; ++b)
        if (st->ckpt_conv == nullptr || !st->ckpt_valid[size_t(b)])
            return fail(Q38_ERR_ARG, "sequence %d has no checkpoint to restore", b);
    DeviceGuard guard(st->ctx->device);
    return copy_recurrent(st, seq0, nseq, false, static_cast<cudaStream_t>(stream));
}

int q38_state_errors(q38_state *st, int *bits) {
    if (!st || !bits) return fail(Q38_ERR_ARG, "null argument");
    DeviceGuard guard(st->ctx->device);
    Q38_CUDA(cudaDeviceSynchronize());
    Q38_CUDA(cudaMemcpy(bits, st->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    Q38_CUDA(cudaMemset(st->d_err, 0, sizeof(int)));
    // A decode sweep that gave up may leave key-head reader counts behind.
    if (*bits && st->lin_group_count)
        Q38_CUDA(cudaMemset(st->lin_group_count, 0,
                            size_t(st->linear_slots) * st->batch * st->ctx->geom.linear_qk_heads *
                                sizeof(int)));
    return Q38_OK;
}

int q38_state_set_debug(q38_state *st, int flags, uint64_t wait_ns) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    if (flags & ~Q38_DEBUG_SKIP_KV_LOADS) return fail(Q38_ERR_ARG, "unknown debug flags 0x%x", flags);
    st->debug_flags = flags;
    st->debug_wait_ns = wait_ns;
    return Q38_OK;
}

int q38_state_full_slot(q38_state *st, int layer, void **key_cache, void **value_cache,
                        size_t *bytes_each) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    int slot;
    if (int rc = full_slot_of(st, layer, &slot)) return rc;
    if (key_cache) *key_cache = kv_seq_base(st, st->kcache, slot, 0);
    if (value_cache) *value_cache = kv_seq_base(st, st->vcache, slot, 0);
    if (bytes_each) *bytes_each = st->kv_slot_elems * st->kv_elem;
    return Q38_OK;
}

int q38_state_linear_slot(q38_state *st, int layer, float **conv_state, float **delta_state) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    int slot;
    if (int rc = linear_slot_of(st, layer, &slot)) return rc;
    if (conv_state) *conv_state = st->conv_state + size_t(slot) * st->batch * conv_seq_floats(st->ctx);
    if (delta_state)
        *delta_state = st->delta_state + size_t(slot) * st->batch * delta_seq_floats(st->ctx);
    return Q38_OK;
}

int q38_state_upload_kv(q38_state *st, int layer, int seq, int first, int count,
                        const float *key_rows, const float *value_rows) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    int slot;
    if (int rc = full_slot_of(st, layer, &slot)) return rc;
    if (seq < 0 || seq >= st->batch || first < 0 || count < 0 ||
        size_t(first) + size_t(count) > size_t(st->context_length))
        return fail(Q38_ERR_ARG, "KV rows [%d, %d) of sequence %d out of range", first,
                    first + count, seq);
    if (count == 0) return Q38_OK;
    if (!key_rows || !value_rows) return fail(Q38_ERR_ARG, "null rows");
    DeviceGuard guard(st->ctx->device);
    const int kvh = st->ctx->geom.attn_kv_heads, D = q38::kAttnHeadDim;
    const size_t row = size_t(kvh) * D;
    for (int which = 0; which < 2; ++which) {
        const float *src = which ? value_rows : key_rows;
        unsigned char *base = kv_seq_base(st, which ? st->vcache : st->kcache, slot, seq);
        if (st->kv_dtype == Q38_KV_F32) {
            for (int h = 0; h < kvh; ++h)
                Q38_CUDA(cudaMemcpy2D(base + (size_t(h) * st->context_length + first) * D * 4,
                                      D * 4, src + size_t(h) * D, row * 4, D * 4, count,
                                      cudaMemcpyHostToDevice));
        } else {
            std::vector<uint16_t> tmp(size_t(count) * row);
            for (size_t i = 0; i < tmp.size(); ++i) tmp[i] = f32_to_bf16_bits(src[i]);
            for (int h = 0; h < kvh; ++h)
                Q38_CUDA(cudaMemcpy2D(base + (size_t(h) * st->context_length + first) * D * 2,
                                      D * 2, tmp.data() + size_t(h) * D, row * 2, D * 2, count,
                                      cudaMemcpyHostToDevice));
        }
    }
    return Q38_OK;
}

int q38_state_download_kv(q38_state *st, int layer, int seq, int first, int count,
                          float *key_rows, float *value_rows) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    int slot;
    if (int rc = full_slot_of(st, layer, &slot)) return rc;
    if (seq < 0 || seq >= st->batch || first < 0 || count < 0 ||
        size_t(first) + size_t(count) > size_t(st->context_length))
        return fail(Q38_ERR_ARG, "KV rows [%d, %d) of sequence %d out of range", first,
                    first + count, seq);
    if (count == 0) return Q38_OK;
    if (!key_rows || !value_rows) return fail(Q38_ERR_ARG, "null rows");
    DeviceGuard guard(st->ctx->device);
    const int kvh = st->ctx->geom.attn_kv_heads, D = q38::kAttnHeadDim;
    const size_t row = size_t(kvh) * D;
    for (int which = 0; which < 2; ++which) {
        float *dst = which ? value_rows : key_rows;
        const unsigned char *base = kv_seq_base(st, which ? st->vcache : st->kcache, slot, seq);
        if (st->kv_dtype == Q38_KV_F32) {
            for (int h = 0; h < kvh; ++h)
                Q38_CUDA(cudaMemcpy2D(dst + size_t(h) * D, row * 4,
                                      base + (size_t(h) * st->context_length + first) * D * 4,
                                      D * 4, D * 4, count, cudaMemcpyDeviceToHost));
        } else {
            std::vector<uint16_t> tmp(size_t(count) * row);
            for (int h = 0; h < kvh; ++h)
                Q38_CUDA(cudaMemcpy2D(tmp.data() + size_t(h) * D, row * 2,
                                      base + (size_t(h) * st->context_length + first) * D * 2,
                                      D * 2, D * 2, count, cudaMemcpyDeviceToHost));
            for (size_t i = 0; i < tmp.size(); ++i) dst[i] = bf16_bits_to_f32(tmp[i]);
        }
    }
    return Q38_OK;
}

int q38_state_upload_linear(q38_state *st, int layer, int seq, const float *conv_state,
                            const float *delta_state) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    float *conv, *delta;
    if (int rc = q38_state_linear_slot(st, layer, &conv, &delta)) return rc;
    if (seq < 0 || seq >= st->batch) return fail(Q38_ERR_ARG, "sequence %d out of range", seq);
    DeviceGuard guard(st->ctx->device);
    const size_t cn = conv_seq_floats(st->ctx), dn = delta_seq_floats(st->ctx);
    if (conv_state)
        Q38_CUDA(cudaMemcpy(conv + size_t(seq) * cn, conv_state, cn * 4, cudaMemcpyHostToDevice));
    if (delta_state)
        Q38_CUDA(cudaMemcpy(delta + size_t(seq) * dn, delta_state, dn * 4, cudaMemcpyHostToDevice));
    return Q38_OK;
}

int q38_state_download_linear(q38_state *st, int layer, int seq, float *conv_state,
                              float *delta_state) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    float *conv, *delta;
    if (int rc = q38_state_linear_slot(st, layer, &conv, &delta)) return rc;
    if (seq < 0 || seq >= st->batch) return fail(Q38_ERR_ARG, "sequence %d out of range", seq);
    DeviceGuard guard(st->ctx->device);
    const size_t cn = conv_seq_floats(st->ctx), dn = delta_seq_floats(st->ctx);
    if (conv_state)
        Q38_CUDA(cudaMemcpy(conv_state, conv + size_t(seq) * cn, cn * 4, cudaMemcpyDeviceToHost));
    if (delta_state)
        Q38_CUDA(cudaMemcpy(delta_state, delta + size_t(seq) * dn, dn * 4, cudaMemcpyDeviceToHost));
    return Q38_OK;
}

int q38_full_decode(q38_ctx *ctx, q38_state *st, int layer, int batch, const float *q_and_gate,
                    float *key, const float *value, const int32_t *positions, int max_position,
                    float *attention, void *stream) {
    q38::AttnDecodeLaunch a;
    if (int rc = prepare_full_decode(ctx, st, layer, batch, q_and_gate, key, value, positions,
                                     max_position, attention, &a))
        return rc;
    DeviceGuard guard(ctx->device);
    cudaError_t e = q38::launch_attn_decode(a, ctx->sm_count, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "full-attention decode launch");
    return Q38_OK;
}

int q38_full_decode_shard(q38_ctx *ctx, q38_state *st, int layer, int batch,
                          const float *q_and_gate, float *key, const float *value,
                          const int32_t *positions, int max_position, int pos_offset,
                          float *partials, void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    if (pos_offset < 0) return fail(Q38_ERR_ARG, "pos_offset must be >= 0");
    if (!partials) return fail(Q38_ERR_ARG, "null partials");
    if (max_position < 0) return fail(Q38_ERR_ARG, "max_position is required when sharding");
    q38::AttnDecodeLaunch a;
    if (int rc = prepare_full_decode(ctx, st, layer, batch, q_and_gate, key, value, positions,
                                     max_position, nullptr, &a, true))
        return rc;
    a.pos_offset = pos_offset;
    a.partial_out = partials;
    DeviceGuard guard(ctx->device);
    cudaError_t e = q38::launch_attn_decode(a, ctx->sm_count, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "sharded full-attention decode launch");
    return Q38_OK;
}

int q38_attn_merge_shards(q38_ctx *ctx, int nparts, int batch, const float *partials,
                          const float *q_and_gate, float *attention, void *stream) {
    if (int rc = check_ctx(ctx)) return rc;
    if (nparts <= 0 || batch <= 0) return fail(Q38_ERR_ARG, "nparts and batch must be positive");
    if (!partials || !q_and_gate || !attention) return fail(Q38_ERR_ARG, "null tensor argument");
    DeviceGuard guard(ctx->device);
    cudaError_t e = q38::launch_attn_merge_shards(partials, nparts, batch, ctx->geom.attn_heads,
                                                  q_and_gate, attention,
                                                  static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "shard merge launch");
    return Q38_OK;
}

int q38_state_reserve_split(q38_state *st, int nranks) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    if (nranks <= 0) return fail(Q38_ERR_ARG, "nranks must be positive");
    if (st->split_ranks == nranks) return Q38_OK;
    DeviceGuard guard(st->ctx->device);
    cudaFree(st->split_local);
    cudaFree(st->split_gathered);
    for (void *q : st->p2p_opened) cudaIpcCloseMemHandle(q);
    st->p2p_opened.clear();
    cudaFree(st->p2p_buf);
    cudaFree(st->p2p_peers_dev);
    st->split_local = st->split_gathered = nullptr;
    st->split_ranks = 0;
    const size_t per = size_t(st->batch) * st->ctx->geom.attn_heads * (q38::kAttnHeadDim + 2);
    Q38_CUDA(cudaMalloc(&st->split_local, per * sizeof(float)));
    Q38_CUDA(cudaMalloc(&st->split_gathered, size_t(nranks) * per * sizeof(float)));
    st->split_ranks = nranks;
    return Q38_OK;
}

int q38_full_decode_split(q38_ctx *ctx, q38_state *st, int layer, int batch,
                          const float *q_and_gate, float *key, const float *value,
                          const int32_t *positions, int max_position, int pos_offset,
                          void *nccl_comm, float *attention, void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    if (!nccl_comm || !attention) return fail(Q38_ERR_ARG, "null communicator or attention");
    if (!st->split_local) return fail(Q38_ERR_ARG, "q38_state_reserve_split was not called");
    if (batch <= 0 || batch > st->batch)
        return fail(Q38_ERR_ARG, "batch %d outside 1..%d", batch, st->batch);
    int nranks = 0;
    if (int rc = q38::nccl_comm_ranks(nccl_comm, &nranks)) return rc;
    if (nranks != st->split_ranks)
        return fail(Q38_ERR_ARG, "the communicator has %d ranks, the split buffers %d", nranks,
                    st->split_ranks);
    if (int rc = q38_full_decode_shard(ctx, st, layer, batch, q_and_gate, key, value, positions,
                                       max_position, pos_offset, st->split_local, stream))
        return rc;
    DeviceGuard guard(ctx->device);
    // Every rank's [batch][heads][258] partials, rank-major, in this GPU's memory.
    const size_t count = size_t(batch) * ctx->geom.attn_heads * (q38::kAttnHeadDim + 2);
    if (int rc = q38::nccl_all_gather_f32(nccl_comm, st->split_local, st->split_gathered, count,
                                          static_cast<cudaStream_t>(stream)))
        return rc;
    return q38_attn_merge_shards(ctx, nranks, batch, st->split_gathered, q_and_gate, attention,
                                 stream);
}

int q38_state_split_p2p_handle(q38_state *st, int nranks, void *handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == Q38_IPC_HANDLE_BYTES, "IPC handle size");
    if (!st || !handle) return fail(Q38_ERR_ARG, "null argument");
    if (nranks <= 0 || nranks > 64) return fail(Q38_ERR_ARG, "nranks %d outside 1..64", nranks);
    DeviceGuard guard(st->ctx->device);
    if (st->p2p_buf && st->p2p_nranks != nranks) {
        for (void *q : st->p2p_opened) cudaIpcCloseMemHandle(q);
        st->p2p_opened.clear();
        cudaFree(st->p2p_buf);
        st->p2p_buf = nullptr;
        st->p2p_rank = -1;
    }
    if (!st->p2p_buf) {
        const size_t bytes =
            q38::attn_p2p_exchange_bytes(nranks, st->batch, st->ctx->geom.attn_heads);
        Q38_CUDA(cudaMalloc(&st->p2p_buf, bytes));
        Q38_CUDA(cudaMemset(st->p2p_buf, 0, bytes));  // flags start below every epoch
        st->p2p_nranks = nranks;
        st->p2p_rank = -1;
    }
    Q38_CUDA(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(handle), st->p2p_buf));
    return Q38_OK;
}

int q38_state_split_p2p_open(q38_state *st, int rank, const void *handles) {
    if (!st || !handles) return fail(Q38_ERR_ARG, "null argument");
    if (!st->p2p_buf) return fail(Q38_ERR_ARG, "q38_state_split_p2p_handle was not called");
    const int nranks = st->p2p_nranks;
    if (rank < 0 || rank >= nranks) return fail(Q38_ERR_ARG, "rank %d outside 0..%d", rank, nranks - 1);
    DeviceGuard guard(st->ctx->device);
    for (void *q : st->p2p_opened) cudaIpcCloseMemHandle(q);
    st->p2p_opened.clear();
    st->p2p_rank = -1;
    std::vector<float *> ptrs(size_t(nranks), nullptr);
    for (int r = 0; r < nranks; ++r) {
        if (r == rank) {
            ptrs[size_t(r)] = static_cast<float *>(st->p2p_buf);
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const unsigned char *>(handles) + size_t(r) * sizeof h, sizeof h);
        void *q = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&q, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (void *o : st->p2p_opened) cudaIpcCloseMemHandle(o);
            st->p2p_opened.clear();
            return cuda_fail(e, "cudaIpcOpenMemHandle of a peer's exchange buffer");
        }
        st->p2p_opened.push_back(q);
        ptrs[size_t(r)] = static_cast<float *>(q);
    }
    // 64 addresses, then the epoch counter (zero: the first call's epoch is 1,
    // above the zeroed exchange words).
    if (!st->p2p_peers_dev) Q38_CUDA(cudaMalloc(&st->p2p_peers_dev, 64 * sizeof(float *) + 16));
    Q38_CUDA(cudaMemset(st->p2p_peers_dev + 64, 0, sizeof(uint32_t)));
    Q38_CUDA(cudaMemcpy(st->p2p_peers_dev, ptrs.data(), size_t(nranks) * sizeof(float *),
                        cudaMemcpyHostToDevice));
    st->p2p_rank = rank;
    return Q38_OK;
}

int q38_full_decode_split_p2p(q38_ctx *ctx, q38_state *st, int layer, int batch,
                              const float *q_and_gate, float *key, const float *value,
                              const int32_t *positions, int max_position, int pos_offset,
                              float *attention, void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    if (st->p2p_rank < 0) return fail(Q38_ERR_ARG, "q38_state_split_p2p_open was not called");
    if (pos_offset < 0) return fail(Q38_ERR_ARG, "pos_offset must be >= 0");
    if (max_position < 0) return fail(Q38_ERR_ARG, "max_position is required when sharding");
    if (!attention) return fail(Q38_ERR_ARG, "null attention");
    q38::AttnDecodeLaunch a;
    if (int rc = prepare_full_decode(ctx, st, layer, batch, q_and_gate, key, value, positions,
                                     max_position, attention, &a, true))
        return rc;
    a.pos_offset = pos_offset;
    a.p2p_peers = st->p2p_peers_dev;
    a.p2p_rank = st->p2p_rank;
    a.p2p_nranks = st->p2p_nranks;
    a.p2p_batch = st->batch;
    a.p2p_epoch = reinterpret_cast<uint32_t *>(st->p2p_peers_dev + 64);
    DeviceGuard guard(ctx->device);
    cudaError_t e = q38::launch_attn_decode(a, ctx->sm_count, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "split-sequence decode launch (peer exchange)");
    return Q38_OK;
}

int q38_linear_decode(q38_ctx *ctx, q38_state *st, int layer, int batch, float *qkv,
                      const float *z, float *beta, float *alpha, float *attention,
                      void *stream) {
    q38::LinearDecodeLaunch a;
    if (int rc = prepare_linear_decode(ctx, st, layer, batch, qkv, z, beta, alpha, attention, &a))
        return rc;
    DeviceGuard guard(ctx->device);
    cudaError_t e = q38::launch_linear_decode(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "DeltaNet decode launch");
    return Q38_OK;
}

namespace {

constexpr size_t kHostPieceTokens = 4096;

// Floats one token needs in the host-prefill staging buffer: the larger of
// the full-attention inputs+output and the DeltaNet inputs+output.
size_t host_prefill_token_floats(const q38_ctx *ctx) {
    const size_t full = size_t(ctx->qg_dim) + 2 * ctx->kv_dim + ctx->q_dim;
    const size_t lin = size_t(ctx->qkv_dim) + 2 * ctx->v_dim + 2 * ctx->geom.linear_v_heads;
    return std::max(full, lin);
}

// Tokens per sequence in one staged piece of a host prefill.
int host_piece(const q38_state *st, int nseq, int count, int align) {
    int piece = int(st->prefill_stage_tokens / size_t(nseq));
    if (piece >= align) piece -= piece % align;
    return std::max(1, std::min(piece, count));
}

// Copies rows [t0, t0+n) of each of nseq sequences of a [nseq][count][dim]
// tensor to or from a [nseq][n][dim] staging block.
cudaError_t copy_piece(float *dst, const float *src, int nseq, int count, int t0, int n, int dim,
                       cudaMemcpyKind kind, cudaStream_t s) {
    const size_t row = size_t(n) * dim * sizeof(float);
    if (kind == cudaMemcpyHostToDevice)
        return cudaMemcpy2DAsync(dst, row, src + size_t(t0) * dim, size_t(count) * dim * 4, row,
                                 nseq, kind, s);
    return cudaMemcpy2DAsync(dst + size_t(t0) * dim, size_t(count) * dim * 4, src, row, row, nseq,
                             kind, s);
}

}  // namespace

int q38_state_reserve_prefill(q38_state *st, int max_tokens) {
    if (!st) return fail(Q38_ERR_ARG, "null state");
    if (max_tokens <= 0) return fail(Q38_ERR_ARG, "max_tokens must be positive");
    if (size_t(max_tokens) <= st->prefill_tokens) return Q38_OK;
    DeviceGuard guard(st->ctx->device);
    cudaFree(st->prefill_rope);
    cudaFree(st->prefill_v16);
    cudaFree(st->prefill_k16);
    cudaFree(st->prefill_lin);
    cudaFree(st->prefill_stage);
    st->prefill_rope = nullptr;
    st->prefill_v16 = nullptr;
    st->prefill_k16 = nullptr;
    st->prefill_v16_seqs = 0;
    st->prefill_lin = nullptr;
    st->prefill_stage = nullptr;
    st->prefill_tokens = 0;
    st->prefill_chunks = 0;
    st->prefill_stage_tokens = 0;
    if (st->full_slots > 0) {
        // RoPE table of the prompt's positions (cos | sin of 32 angles each).
        Q38_CUDA(cudaMalloc(&st->prefill_rope,
                            q38::attn_prefill_rope_floats(max_tokens) * sizeof(float)));
        // f16 copy of the V rows a prefill reads (prefix and prompt), one
        // cache-sized plane per sequence that one call can cover.
        const int seqs = std::min(st->batch, max_tokens);
        const size_t v16_bytes = size_t(seqs) * st->ctx->kv_dim * st->context_length * 2;
        Q38_CUDA(cudaMalloc(&st->prefill_v16, v16_bytes));
        // Rows past a prompt's last position sit in its last key tile with
        // P = 0; they must hold finite values (0 * NaN would be NaN).
        Q38_CUDA(cudaMemset(st->prefill_v16, 0, v16_bytes));
        if (st->kv_dtype == Q38_KV_F32) {
            // An f32 cache keeps the reference's rows; Q K^T reads an f16 copy.
            Q38_CUDA(cudaMalloc(&st->prefill_k16, v16_bytes));
            Q38_CUDA(cudaMemset(st->prefill_k16, 0, v16_bytes));
        }
        st->prefill_v16_seqs = seqs;
    }
    if (st->linear_slots > 0) {
        // One partial chunk per sequence on top of the full chunks.
        const size_t chunks = (size_t(max_tokens) + 63) / 64 + size_t(st->batch);
        const size_t floats =
            q38::linear_prefill_scratch_floats(int(chunks), st->ctx->geom.linear_v_heads);
        Q38_CUDA(cudaMalloc(&st->prefill_lin, floats * sizeof(float)));
        st->prefill_chunks = chunks;
    }
    // Host-pointer prefill streams the prompt through a staging buffer of at
    // most kHostPieceTokens tokens (but never fewer than one per sequence).
    const size_t stage_tokens =
        std::min(size_t(max_tokens), std::max(kHostPieceTokens, size_t(st->batch)));
    Q38_CUDA(cudaMalloc(&st->prefill_stage,
                        stage_tokens * host_prefill_token_floats(st->ctx) * sizeof(float)));
    st->prefill_stage_tokens = stage_tokens;
    st->prefill_tokens = size_t(max_tokens);
    return Q38_OK;
}

namespace {

int full_prefill_impl(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                      int base_position, int kv_head0, int kv_head_count,
                      const float *q_and_gate, float *key, const float *value, float *attention,
                      void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    int slot;
    if (int rc = full_slot_of(st, layer, &slot)) return rc;
    if (kv_head_count <= 0 || kv_head0 < 0 || kv_head0 + kv_head_count > ctx->geom.attn_kv_heads)
        return fail(Q38_ERR_ARG, "KV heads [%d, %d) outside 0..%d", kv_head0,
                    kv_head0 + kv_head_count, ctx->geom.attn_kv_heads);
    if (kv_head_count > 8)
        return fail(Q38_ERR_ARG, "a prefill call covers at most 8 KV heads (got %d)", kv_head_count);
    if (nseq <= 0 || seq0 < 0 || seq0 + nseq > st->batch)
        return fail(Q38_ERR_ARG, "sequences [%d, %d) outside the state's %d", seq0, seq0 + nseq,
                    st->batch);
    if (count <= 0 || base_position < 0 ||
        int64_t(base_position) + count > int64_t(st->context_length))
        return fail(Q38_ERR_ARG, "positions [%d, %d) outside the %d-position cache",
                    base_position, base_position + count, st->context_length);
    if (size_t(nseq) * size_t(count) > st->prefill_tokens || nseq > st->prefill_v16_seqs)
        return fail(Q38_ERR_ARG, "%d tokens exceed the reserved prefill scratch (%zu)",
                    nseq * count, st->prefill_tokens);
    if (!q_and_gate || !key || !value || !attention)
        return fail(Q38_ERR_ARG, "null tensor argument");
    // The kernels move rows as 16-byte vectors and by TMA.
    if ((reinterpret_cast<uintptr_t>(q_and_gate) | reinterpret_cast<uintptr_t>(key) |
         reinterpret_cast<uintptr_t>(value) | reinterpret_cast<uintptr_t>(attention)) & 15u)
        return fail(Q38_ERR_ARG, "prefill tensors must be 16-byte aligned");
    auto it = ctx->full.find(layer);
    if (it == ctx->full.end())
        return fail(Q38_ERR_ARG, "full-attention layer %d has no bound weights", layer);
    q38::AttnPrefillLaunch a{};
    a.q_and_gate = q_and_gate;
    a.key = key;
    a.value = value;
    a.attention = attention;
    a.rope = st->prefill_rope;
    a.v16 = st->prefill_v16;
    a.k16 = st->prefill_k16;
    a.kv_f32 = st->kv_dtype == Q38_KV_F32 ? 1 : 0;
    a.kv_head0 = kv_head0;
    a.kv_head_count = kv_head_count;
    a.kcache = kv_seq_base(st, st->kcache, slot, 0);
    a.vcache = kv_seq_base(st, st->vcache, slot, 0);
    a.q_norm = it->second.q_norm;
    a.k_norm = it->second.k_norm;
    a.err = st->d_err;
    a.batch = st->batch;
    a.seq0 = seq0;
    a.nseq = nseq;
    a.count = count;
    a.base = base_position;
    a.context_length = st->context_length;
    a.heads = ctx->geom.attn_heads;
    a.kv_heads = ctx->geom.attn_kv_heads;
    a.theta_scale = ctx->theta_scale;
    a.eps = ctx->geom.rms_eps;
    DeviceGuard guard(ctx->device);
    cudaError_t e = q38::launch_attn_prefill(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "full-attention prefill launch");
    return Q38_OK;
}

int linear_prefill_impl(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                        int v_head0, int v_head_count, float *qkv, const float *z, float *beta,
                        float *alpha, float *attention, void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    int slot;
    if (int rc = linear_slot_of(st, layer, &slot)) return rc;
    if (v_head_count <= 0 || v_head0 < 0 || v_head0 + v_head_count > ctx->geom.linear_v_heads)
        return fail(Q38_ERR_ARG, "value heads [%d, %d) outside 0..%d", v_head0,
                    v_head0 + v_head_count, ctx->geom.linear_v_heads);
    if (nseq <= 0 || seq0 < 0 || seq0 + nseq > st->batch)
        return fail(Q38_ERR_ARG, "sequences [%d, %d) outside the state's %d", seq0, seq0 + nseq,
                    st->batch);
    if (count <= 0) return fail(Q38_ERR_ARG, "count must be positive");
    const size_t chunks = size_t(nseq) * ((size_t(count) + 63) / 64);
    if (size_t(nseq) * size_t(count) > st->prefill_tokens || chunks > st->prefill_chunks)
        return fail(Q38_ERR_ARG, "%d tokens exceed the reserved prefill scratch (%zu)",
                    nseq * count, st->prefill_tokens);
    if (!qkv || !z || !beta || !alpha || !attention)
        return fail(Q38_ERR_ARG, "null tensor argument");
    // The kernels read and write the per-token rows as 16-byte vectors.
    if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(z) |
         reinterpret_cast<uintptr_t>(attention)) & 15u)
        return fail(Q38_ERR_ARG, "prefill tensors must be 16-byte aligned");
    auto it = ctx->linear.find(layer);
    if (it == ctx->linear.end())
        return fail(Q38_ERR_ARG, "DeltaNet layer %d has no bound weights", layer);
    q38::LinearPrefillLaunch a{};
    a.qkv = qkv;
    a.z = z;
    a.beta = beta;
    a.alpha = alpha;
    a.attention = attention;
    a.conv_state = st->conv_state + size_t(slot) * st->batch * conv_seq_floats(ctx);
    a.delta_state = st->delta_state + size_t(slot) * st->batch * delta_seq_floats(ctx);
    a.conv_w = it->second.conv_w;
    a.dt_bias = it->second.dt_bias;
    a.ssm_a = it->second.ssm_a;
    a.ssm_norm = it->second.ssm_norm;
    a.scratch = st->prefill_lin;
    a.err = st->d_err;
    a.seq0 = seq0;
    a.nseq = nseq;
    a.count = count;
    a.qk_heads = ctx->geom.linear_qk_heads;
    a.v_heads = ctx->geom.linear_v_heads;
    a.v_head0 = v_head0;
    a.v_head_count = v_head_count;
    a.eps = ctx->geom.rms_eps;
    a.side = st->side;
    a.fork = st->side_fork;
    a.join = st->side_join;
    a.nside = q38_state::kSides;
    DeviceGuard guard(ctx->device);
    cudaError_t e = q38::launch_linear_prefill(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "DeltaNet prefill launch");
    return Q38_OK;
}

}  // namespace

int q38_full_prefill(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                     int base_position, const float *q_and_gate, float *key, const float *value,
                     float *attention, void *stream) {
    if (int rc = check_ctx(ctx)) return rc;
    return full_prefill_impl(ctx, st, layer, seq0, nseq, count, base_position, 0,
                             ctx->geom.attn_kv_heads, q_and_gate, key, value, attention, stream);
}

int q38_full_prefill_heads(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq,
                           int count, int base_position, int kv_head0, int kv_head_count,
                           const float *q_and_gate, float *key, const float *value,
                           float *attention, void *stream) {
    return full_prefill_impl(ctx, st, layer, seq0, nseq, count, base_position, kv_head0,
                             kv_head_count, q_and_gate, key, value, attention, stream);
}

int q38_linear_prefill(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                       float *qkv, const float *z, float *beta, float *alpha, float *attention,
                       void *stream) {
    if (int rc = check_ctx(ctx)) return rc;
    return linear_prefill_impl(ctx, st, layer, seq0, nseq, count, 0, ctx->geom.linear_v_heads, qkv,
                               z, beta, alpha, attention, stream);
}

int q38_linear_prefill_heads(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq,
                             int count, int v_head0, int v_head_count, float *qkv, const float *z,
                             float *beta, float *alpha, float *attention, void *stream) {
    return linear_prefill_impl(ctx, st, layer, seq0, nseq, count, v_head0, v_head_count, qkv, z,
                               beta, alpha, attention, stream);
}

int q38_full_prefill_host(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                          int base_position, const float *q_and_gate, float *key,
                          const float *value, float *attention, void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    if (!q_and_gate || !key || !value || !attention)
        return fail(Q38_ERR_ARG, "null tensor argument");
    if (nseq <= 0 || count <= 0 || seq0 < 0 || seq0 + nseq > st->batch)
        return fail(Q38_ERR_ARG, "sequences [%d, %d) x %d tokens outside the state's %d",
                    seq0, seq0 + nseq, count, st->batch);
    if (!st->prefill_stage || size_t(nseq) * size_t(count) > st->prefill_tokens)
        return fail(Q38_ERR_ARG, "%d tokens exceed the reserved prefill scratch (%zu)",
                    nseq * count, st->prefill_tokens);
    if (base_position < 0 || int64_t(base_position) + count > int64_t(st->context_length))
        return fail(Q38_ERR_ARG, "positions [%d, %d) outside the %d-position cache",
                    base_position, base_position + count, st->context_length);
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int piece = host_piece(st, nseq, count, 128);
    const size_t n_max = size_t(nseq) * piece;
    float *d_qg = st->prefill_stage, *d_k = d_qg + n_max * ctx->qg_dim,
          *d_v = d_k + n_max * ctx->kv_dim, *d_out = d_v + n_max * ctx->kv_dim;
    // Token t of a piece starting at t0 is prompt token t0+t at position
    // base_position+t0+t; earlier pieces are already in the cache, so the
    // pieces give the per-token loop's result.
    for (int t0 = 0; t0 < count; t0 += piece) {
        const int n = std::min(piece, count - t0);
        Q38_CUDA(copy_piece(d_qg, q_and_gate, nseq, count, t0, n, ctx->qg_dim,
                            cudaMemcpyHostToDevice, s));
        Q38_CUDA(copy_piece(d_k, key, nseq, count, t0, n, ctx->kv_dim, cudaMemcpyHostToDevice, s));
        Q38_CUDA(copy_piece(d_v, value, nseq, count, t0, n, ctx->kv_dim, cudaMemcpyHostToDevice, s));
        if (int rc = q38_full_prefill(ctx, st, layer, seq0, nseq, n, base_position + t0, d_qg, d_k,
                                      d_v, d_out, stream)) {
            cudaStreamSynchronize(s);  // the caller's buffers may go once we return
            return rc;
        }
        Q38_CUDA(copy_piece(attention, d_out, nseq, count, t0, n, ctx->q_dim,
                            cudaMemcpyDeviceToHost, s));
        Q38_CUDA(copy_piece(key, d_k, nseq, count, t0, n, ctx->kv_dim, cudaMemcpyDeviceToHost, s));
    }
    Q38_CUDA(enqueue_error_read(st, s));
    Q38_CUDA(cudaStreamSynchronize(s));
    return host_call_status(st);
}

int q38_linear_prefill_host(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq,
                            int count, float *qkv, const float *z, float *beta, float *alpha,
                            float *attention, void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    if (!qkv || !z || !beta || !alpha || !attention)
        return fail(Q38_ERR_ARG, "null tensor argument");
    if (nseq <= 0 || count <= 0 || seq0 < 0 || seq0 + nseq > st->batch)
        return fail(Q38_ERR_ARG, "sequences [%d, %d) x %d tokens outside the state's %d",
                    seq0, seq0 + nseq, count, st->batch);
    if (!st->prefill_stage || size_t(nseq) * size_t(count) > st->prefill_tokens)
        return fail(Q38_ERR_ARG, "%d tokens exceed the reserved prefill scratch (%zu)",
                    nseq * count, st->prefill_tokens);
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int piece = host_piece(st, nseq, count, 64);
    const size_t n_max = size_t(nseq) * piece;
    const int vh = ctx->geom.linear_v_heads;
    float *d_qkv = st->prefill_stage, *d_z = d_qkv + n_max * ctx->qkv_dim,
          *d_b = d_z + n_max * ctx->v_dim, *d_a = d_b + n_max * vh, *d_out = d_a + n_max * vh;
    // The conv and delta states carry from one piece to the next exactly as
    // from one token to the next.
    for (int t0 = 0; t0 < count; t0 += piece) {
        const int n = std::min(piece, count - t0);
        Q38_CUDA(copy_piece(d_qkv, qkv, nseq, count, t0, n, ctx->qkv_dim, cudaMemcpyHostToDevice,
                            s));
        Q38_CUDA(copy_piece(d_z, z, nseq, count, t0, n, ctx->v_dim, cudaMemcpyHostToDevice, s));
        Q38_CUDA(copy_piece(d_b, beta, nseq, count, t0, n, vh, cudaMemcpyHostToDevice, s));
        Q38_CUDA(copy_piece(d_a, alpha, nseq, count, t0, n, vh, cudaMemcpyHostToDevice, s));
        if (int rc = q38_linear_prefill(ctx, st, layer, seq0, nseq, n, d_qkv, d_z, d_b, d_a, d_out,
                                        stream)) {
            cudaStreamSynchronize(s);
            return rc;
        }
        Q38_CUDA(copy_piece(attention, d_out, nseq, count, t0, n, ctx->v_dim,
                            cudaMemcpyDeviceToHost, s));
        Q38_CUDA(copy_piece(qkv, d_qkv, nseq, count, t0, n, ctx->qkv_dim, cudaMemcpyDeviceToHost,
                            s));
        Q38_CUDA(copy_piece(beta, d_b, nseq, count, t0, n, vh, cudaMemcpyDeviceToHost, s));
        Q38_CUDA(copy_piece(alpha, d_a, nseq, count, t0, n, vh, cudaMemcpyDeviceToHost, s));
    }
    Q38_CUDA(enqueue_error_read(st, s));
    Q38_CUDA(cudaStreamSynchronize(s));
    return host_call_status(st);
}

int q38_full_decode_host(q38_ctx *ctx, q38_state *st, int layer, int batch,
                         const float *q_and_gate, float *key, const float *value,
                         const int32_t *positions, float *attention, void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    if (batch <= 0 || batch > st->batch)
        return fail(Q38_ERR_ARG, "batch %d outside 1..%d", batch, st->batch);
    if (!q_and_gate || !key || !value || !positions || !attention)
        return fail(Q38_ERR_ARG, "null tensor argument");
    int max_pos = 0;
    for (int b = 0; b < batch; ++b) {
        if (positions[b] < 0 || positions[b] >= st->context_length)
            return fail(Q38_ERR_ARG, "position %d of sequence %d outside the %d-position cache",
                        positions[b], b, st->context_length);
        max_pos = positions[b] > max_pos ? positions[b] : max_pos;
    }
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t nqg = size_t(batch) * ctx->qg_dim, nkv = size_t(batch) * ctx->kv_dim,
                 nq = size_t(batch) * ctx->q_dim;
    float *d_qg = st->stage, *d_k = d_qg + nqg, *d_v = d_k + nkv, *d_out = d_v + nkv;
    Q38_CUDA(cudaMemcpyAsync(d_qg, q_and_gate, nqg * 4, cudaMemcpyHostToDevice, s));
    Q38_CUDA(cudaMemcpyAsync(d_k, key, nkv * 4, cudaMemcpyHostToDevice, s));
    Q38_CUDA(cudaMemcpyAsync(d_v, value, nkv * 4, cudaMemcpyHostToDevice, s));
    Q38_CUDA(cudaMemcpyAsync(st->stage_pos, positions, size_t(batch) * 4, cudaMemcpyHostToDevice, s));
    // A pinned, mapped `attention` buffer is written by the merge kernel directly.
    void *att_dev = nullptr;
    const bool att_mapped = mapped_host(attention, ctx->device, &att_dev);
    if (int rc = q38_full_decode(ctx, st, layer, batch, d_qg, d_k, d_v, st->stage_pos, max_pos,
                                 att_mapped ? static_cast<float *>(att_dev) : d_out, stream))
        return rc;
    if (!att_mapped) Q38_CUDA(cudaMemcpyAsync(attention, d_out, nq * 4, cudaMemcpyDeviceToHost, s));
    Q38_CUDA(cudaMemcpyAsync(key, d_k, nkv * 4, cudaMemcpyDeviceToHost, s));
    Q38_CUDA(enqueue_error_read(st, s));
    Q38_CUDA(cudaStreamSynchronize(s));
    return host_call_status(st);
}

int q38_linear_decode_host(q38_ctx *ctx, q38_state *st, int layer, int batch, float *qkv,
                           const float *z, float *beta, float *alpha, float *attention,
                           void *stream) {
    if (int rc = check_state(ctx, st)) return rc;
    if (batch <= 0 || batch > st->batch)
        return fail(Q38_ERR_ARG, "batch %d outside 1..%d", batch, st->batch);
    if (!qkv || !z || !beta || !alpha || !attention)
        return fail(Q38_ERR_ARG, "null tensor argument");
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t nqkv = size_t(batch) * ctx->qkv_dim, nv = size_t(batch) * ctx->v_dim,
                 nh = size_t(batch) * ctx->geom.linear_v_heads;
    float *d_qkv = st->stage, *d_z = d_qkv + nqkv, *d_b = d_z + nv, *d_a = d_b + nh,
          *d_out = d_a + nh;
    // A pinned, mapped `attention` buffer is written by the state kernel
    // directly (posted writes over PCIe, overlapping its state sweep).
    void *att_dev = nullptr;
    const bool att_mapped = mapped_host(attention, ctx->device, &att_dev);
    q38::LinearDecodeLaunch a;
    if (int rc = prepare_linear_decode(ctx, st, layer, batch, d_qkv, d_z, d_b, d_a,
                                       att_mapped ? static_cast<float *>(att_dev) : d_out, &a))
        return rc;
    Q38_CUDA(ensure_host_out(st));
    Q38_CUDA(cudaMemcpyAsync(d_qkv, qkv, nqkv * 4, cudaMemcpyHostToDevice, s));
    Q38_CUDA(cudaMemcpyAsync(d_z, z, nv * 4, cudaMemcpyHostToDevice, s));
    Q38_CUDA(cudaMemcpyAsync(d_b, beta, nh * 4, cudaMemcpyHostToDevice, s));
    Q38_CUDA(cudaMemcpyAsync(d_a, alpha, nh * 4, cudaMemcpyHostToDevice, s));
    cudaError_t e = q38::launch_linear_decode(a, s, st->host_ev_prep);
    if (e != cudaSuccess) return cuda_fail(e, "DeltaNet decode launch");
    // The prep kernel's in-place results (qkv, beta, alpha) go back while the
    // state kernel, which only reads them, runs.
    Q38_CUDA(cudaStreamWaitEvent(st->host_out, st->host_ev_prep, 0));
    Q38_CUDA(cudaMemcpyAsync(qkv, d_qkv, nqkv * 4, cudaMemcpyDeviceToHost, st->host_out));
    Q38_CUDA(cudaMemcpyAsync(beta, d_b, nh * 4, cudaMemcpyDeviceToHost, st->host_out));
    Q38_CUDA(cudaMemcpyAsync(alpha, d_a, nh * 4, cudaMemcpyDeviceToHost, st->host_out));
    Q38_CUDA(cudaEventRecord(st->host_ev_back, st->host_out));
    if (!att_mapped)
        Q38_CUDA(cudaMemcpyAsync(attention, d_out, nv * 4, cudaMemcpyDeviceToHost, s));
    Q38_CUDA(cudaStreamWaitEvent(s, st->host_ev_back, 0));  // later work on s follows them
    Q38_CUDA(enqueue_error_read(st, s));
    Q38_CUDA(cudaStreamSynchronize(s));
    return host_call_status(st);
}

int q38_linear_core(q38_ctx *ctx, q38_state *st, int layer, float *conv_state,
                    float *delta_state, float *qkv, const float *z, float *beta, float *alpha,
                    float *attention) {
    if (int rc = check_state(ctx, st)) return rc;
    if (!conv_state || !delta_state) return fail(Q38_ERR_ARG, "null state slice");
    if (int rc = q38_state_upload_linear(st, layer, 0, conv_state, delta_state)) return rc;
    if (int rc = q38_linear_decode_host(ctx, st, layer, 1, qkv, z, beta, alpha, attention, nullptr))
        return rc;
    return q38_state_download_linear(st, layer, 0, conv_state, delta_state);
}

int q38_full_core(q38_ctx *ctx, q38_state *st, int layer, const float *q_and_gate, float *key,
                  const float *value, float *q, float *gate, float *scores, float *attention,
                  float *key_cache, float *value_cache, size_t cache_rows,
                  size_t context_length, uint32_t current_position) {
    (void)scores;  // scratch in the reference; its callers never read it
    if (int rc = check_state(ctx, st)) return rc;
    int slot;
    if (int rc = full_slot_of(st, layer, &slot)) return rc;
    if (!key_cache || !value_cache) return fail(Q38_ERR_ARG, "null cache");
    // ops.rs:858-864: the cache row must lie inside the caller's cache.
    const size_t row = size_t(q38::full_index(layer)) * context_length + current_position;
    if (row + 1 > cache_rows)
        return fail(Q38_ERR_ARG, "cache row %zu outside a %zu-row cache", row, cache_rows);
    if (current_position >= uint32_t(st->context_length))
        return fail(Q38_ERR_ARG, "position %u outside the state's %d-position cache",
                    current_position, st->context_length);
    const size_t kv = size_t(ctx->kv_dim);
    const float *layer_k = key_cache + size_t(q38::full_index(layer)) * context_length * kv;
    const float *layer_v = value_cache + size_t(q38::full_index(layer)) * context_length * kv;
    if (int rc = q38_state_upload_kv(st, layer, 0, 0, int(current_position), layer_k, layer_v))
        return rc;
    const int32_t pos = int32_t(current_position);
    if (int rc = q38_full_decode_host(ctx, st, layer, 1, q_and_gate, key, value, &pos, attention,
                                      nullptr))
        return rc;
    if (int rc = q38_state_download_kv(st, layer, 0, pos, 1, key_cache + row * kv,
                                       value_cache + row * kv))
        return rc;
    DeviceGuard guard(ctx->device);
    if (q) Q38_CUDA(cudaMemcpy(q, st->qprep, size_t(ctx->q_dim) * 4, cudaMemcpyDeviceToHost));
    if (gate) {
        const int D = q38::kAttnHeadDim;
        for (int h = 0; h < ctx->geom.attn_heads; ++h)
            std::memcpy(gate + size_t(h) * D, q_and_gate + size_t(h) * 2 * D + D, D * 4);
    }
    return Q38_OK;
}

}  // extern "C"
