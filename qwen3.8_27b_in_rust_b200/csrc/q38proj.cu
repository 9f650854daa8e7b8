// q38proj.cu -- C ABI of the projections on either side of the attention
// cores: weight upload, Q8_K quantization, project / batch_project and the
// layer-level decode calls linear_attention / full_attention
// (src/model/ops.rs:617-640, 744-803, 941-981, 1016-1031).
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "q38_proj.h"

namespace {

int proj_fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    q38::record_error(buf);
    return code;
}

int proj_cuda_fail(cudaError_t e, const char *what) {
    cudaGetLastError();
    return proj_fail(Q38_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct Guard {
    int prev = -1, dev;
    explicit Guard(int d) : dev(d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~Guard() {
        if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    }
};

int check_weight(const q38_ctx *ctx, const q38_weight *w, const char *what) {
    if (!w) return proj_fail(Q38_ERR_ARG, "null %s weight", what);
    if (w->ctx != ctx) return proj_fail(Q38_ERR_ARG, "%s weight belongs to another context", what);
    return Q38_OK;
}

// Grows the context's scratch for the tensor-core path's quantized input.
int reserve_scratch(q38_ctx *ctx, int batch, int64_t width) {
    const size_t need = q38::proj_mma_scratch_bytes(batch, width);
    if (need <= ctx->proj_scratch_bytes) return Q38_OK;
    if (ctx->proj_scratch) {
        // Earlier launches on any stream may still read the old buffer.
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return proj_cuda_fail(e, "projection scratch resize");
        cudaFree(ctx->proj_scratch);
        ctx->proj_scratch = nullptr;
        ctx->proj_scratch_bytes = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->proj_scratch, need);
    if (e != cudaSuccess) return proj_cuda_fail(e, "projection scratch allocation");
    ctx->proj_scratch_bytes = need;
    return Q38_OK;
}

// Grows the context's workspace for the chunked f32-input projections' partial
// sums (the same rules as the scratch above).
int reserve_part(q38_ctx *ctx, size_t need) {
    if (need <= ctx->proj_part_bytes) return Q38_OK;
    if (ctx->proj_part) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return proj_cuda_fail(e, "projection workspace resize");
        cudaFree(ctx->proj_part);
        ctx->proj_part = nullptr;
        ctx->proj_part_bytes = 0;
    }
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, need);
    if (e != cudaSuccess) return proj_cuda_fail(e, "projection workspace allocation");
    ctx->proj_part = static_cast<float *>(p);
    ctx->proj_part_bytes = need;
    return Q38_OK;
}

// One projection. K-quant weights: a batch of kProjMmaMinBatch or more tokens
// over Q4_K / Q5_K runs on the tensor cores (the input quantized into the
// context's scratch first); otherwise the integer GEMV quantizes the input
// inside its prologue.
bool takes_mma(const q38_weight *w, int batch) {
    return batch >= q38::kProjMmaMinBatch && q38::proj_mma_supported(w->w.type) &&
           w->w.row_bytes % 16 == 0;
}

// prequantized: the context's scratch already holds `input` quantized (MMA
// path only; see the layer call below). sm_budget: the SMs the launch may
// take (0: all; fewer while other projections run beside it).
int project_device(q38_ctx *ctx, const q38_weight *w, int batch, const float *input, float *out,
                   int *err, cudaStream_t s, const q38::ProjEpilogue &epi = {},
                   bool prequantized = false, int sm_budget = 0) {
    if (reinterpret_cast<uintptr_t>(input) % 16)
        return proj_fail(Q38_ERR_ARG, "projection input must be 16-byte aligned");
    cudaError_t e;
    if (takes_mma(w, batch)) {
        if (int rc = reserve_scratch(ctx, batch, w->w.width)) return rc;
        e = w->w.planes
                ? q38::launch_proj_planes(w->w, input, batch, out, long(w->w.rows), err, ctx->proj_scratch,
                                          s, epi, prequantized, sm_budget > 0 ? sm_budget : ctx->sm_count)
                : q38::launch_proj_mma(w->w, input, batch, out, long(w->w.rows), err, ctx->proj_scratch, s,
                                       epi, prequantized);
    } else if (q38::proj_is_q8k_type(w->w.type))
        e = q38::launch_proj_q8k(w->w, input, batch, out, long(w->w.rows), err, ctx->sm_count, s, epi);
    else {
        float *part = nullptr;
        if (q38::proj_f32_takes_tile(w->w.type, w->w.rows, w->w.width, batch)) {
            if (int rc = reserve_part(ctx, q38::proj_f32_tile_part_bytes(w->w.rows, w->w.width, batch))) return rc;
            part = ctx->proj_part;
        }
        e = q38::launch_proj_f32(w->w, input, batch, out, long(w->w.rows), s, epi, part);
    }
    if (e != cudaSuccess) return proj_cuda_fail(e, "projection launch");
    return Q38_OK;
}

}  // namespace

extern "C" {

int q38_weight_create(q38_ctx *ctx, int ggml_type, int64_t width, int64_t rows, const void *data,
                      size_t nbytes, q38_weight **out) {
    if (!out) return proj_fail(Q38_ERR_ARG, "null output pointer");
    *out = nullptr;
    if (!ctx || !data) return proj_fail(Q38_ERR_ARG, "null argument");
    if (!q38::proj_type_supported(ggml_type))
        return proj_fail(Q38_ERR_ARG, "unsupported projection type %d", ggml_type);
    const int64_t rb = q38::proj_row_bytes(ggml_type, width);
    if (rb < 0 || rows <= 0 || rows > (int64_t(1) << 30))
        return proj_fail(Q38_ERR_ARG, "type %d cannot hold %lld x %lld", ggml_type,
                         static_cast<long long>(rows), static_cast<long long>(width));
    if (q38::proj_is_q8k_type(ggml_type) && width % 256)
        return proj_fail(Q38_ERR_ARG, "K-quant rows must be whole 256-blocks");
    if (width % 4 || width > 32768)
        return proj_fail(Q38_ERR_ARG, "projection width %lld must be a multiple of 4 up to 32768",
                         static_cast<long long>(width));
    if (nbytes != size_t(rows * rb))
        return proj_fail(Q38_ERR_ARG, "weight holds %zu bytes, expected %lld", nbytes,
                         static_cast<long long>(rows * rb));
    Guard guard(ctx->device);
    const size_t padded = q38::proj_padded_bytes(ggml_type, rows, width);
    const int64_t drb = q38::proj_device_row_bytes(ggml_type, width);
    void *dev = nullptr;
    cudaError_t e = cudaMalloc(&dev, padded);
    if (e == cudaSuccess) e = cudaMemset(dev, 0, padded);
    if (e == cudaSuccess && drb == rb) {
        e = cudaMemcpy(dev, data, nbytes, cudaMemcpyHostToDevice);
    } else if (e == cudaSuccess) {
        // Q6_K: each 210-byte block into a 224-byte slot (the padding stays zero).
        const size_t nblocks = size_t(rows) * size_t(width / 256);
        std::vector<unsigned char> staged(nblocks * q38::kQ6KDeviceBlock, 0);
        const unsigned char *src = static_cast<const unsigned char *>(data);
        for (size_t i = 0; i < nblocks; ++i)
            std::memcpy(staged.data() + i * q38::kQ6KDeviceBlock, src + i * 210, 210);
        e = cudaMemcpy(dev, staged.data(), staged.size(), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        cudaFree(dev);
        return proj_cuda_fail(e, "weight upload");
    }
    q38_weight *w = new (std::nothrow) q38_weight();
    if (!w) {
        cudaFree(dev);
        return proj_fail(Q38_ERR_ARG, "out of host memory");
    }
    w->ctx = ctx;
    w->w.type = ggml_type;
    w->w.rows = rows;
    w->w.width = width;
    w->w.row_bytes = drb;
    w->w.data = dev;
    *out = w;
    return Q38_OK;
}

int q38_weight_destroy(q38_weight *w) {
    if (!w) return Q38_OK;
    {
        Guard guard(w->ctx->device);
        q38::free_proj_planes(w->w);
        cudaFree(w->w.data);
    }
    delete w;
    return Q38_OK;
}

int q38_weight_build_planes(q38_weight *w) {
    if (!w) return proj_fail(Q38_ERR_ARG, "null weight");
    if (!q38::proj_planes_type(w->w.type))
        return proj_fail(Q38_ERR_ARG, "integer planes are built for Q4_K, Q5_K and Q6_K weights, not type %d",
                         w->w.type);
    Guard guard(w->ctx->device);
    cudaError_t e = q38::build_proj_planes(w->w, nullptr);
    if (e != cudaSuccess) return proj_cuda_fail(e, "integer plane build");
    return Q38_OK;
}

int q38_weight_info(const q38_weight *w, int *ggml_type, int64_t *width, int64_t *rows) {
    if (!w) return proj_fail(Q38_ERR_ARG, "null weight");
    if (ggml_type) *ggml_type = w->w.type;
    if (width) *width = w->w.width;
    if (rows) *rows = w->w.rows;
    return Q38_OK;
}

int q38_ctx_reserve_projection(q38_ctx *ctx, int batch, int64_t width) {
    if (!ctx) return proj_fail(Q38_ERR_ARG, "null context");
    if (batch <= 0 || width <= 0 || width % 256)
        return proj_fail(Q38_ERR_ARG, "bad projection reservation (%d x %lld)", batch,
                         static_cast<long long>(width));
    Guard guard(ctx->device);
    if (int rc = reserve_scratch(ctx, batch, width)) return rc;
    // The chunked f32-input form's workspace, for weights of up to
    // kProjTileMaxRows rows at this width.
    return reserve_part(ctx, q38::proj_f32_tile_part_bytes(q38::kProjTileMaxRows, width, batch));
}

int q38_quantize_q8_k(q38_ctx *ctx, int batch, int64_t width, const float *input, void *blocks,
                      void *stream) {
    if (!ctx || !input || !blocks) return proj_fail(Q38_ERR_ARG, "null argument");
    if (batch <= 0 || width <= 0 || width % 256)
        return proj_fail(Q38_ERR_ARG, "input length %lld is not a multiple of 256",
                         static_cast<long long>(width));
    if (reinterpret_cast<uintptr_t>(input) % 16 || reinterpret_cast<uintptr_t>(blocks) % 4)
        return proj_fail(Q38_ERR_ARG, "input must be 16-byte and blocks 4-byte aligned");
    Guard guard(ctx->device);
    cudaError_t e = q38::launch_q8k_quantize(input, batch, int(width), q38::Q8KActivations{}, blocks,
                                             static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return proj_cuda_fail(e, "Q8_K quantize launch");
    return Q38_OK;
}

int q38_project(q38_ctx *ctx, const q38_weight *w, int batch, const float *input, float *output,
                void *stream) {
    if (!ctx) return proj_fail(Q38_ERR_ARG, "null context");
    if (int rc = check_weight(ctx, w, "projection")) return rc;
    if (batch <= 0 || !input || !output) return proj_fail(Q38_ERR_ARG, "bad batch or null tensor");
    Guard guard(ctx->device);
    return project_device(ctx, w, batch, input, output, nullptr, static_cast<cudaStream_t>(stream));
}

int q38_project_host(q38_ctx *ctx, const q38_weight *w, int batch, const float *input,
                     float *output) {
    if (!ctx) return proj_fail(Q38_ERR_ARG, "null context");
    if (int rc = check_weight(ctx, w, "projection")) return rc;
    if (batch <= 0 || !input || !output) return proj_fail(Q38_ERR_ARG, "bad batch or null tensor");
    Guard guard(ctx->device);
    const size_t in_bytes = size_t(batch) * w->w.width * 4, out_bytes = size_t(batch) * w->w.rows * 4;
    float *din = nullptr, *dout = nullptr;
    cudaError_t e = cudaMalloc(&din, in_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&dout, out_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(din, input, in_bytes, cudaMemcpyHostToDevice);
    int rc = Q38_OK;
    if (e == cudaSuccess) rc = project_device(ctx, w, batch, din, dout, nullptr, nullptr);
    if (e == cudaSuccess && rc == Q38_OK) e = cudaMemcpy(output, dout, out_bytes, cudaMemcpyDeviceToHost);
    cudaFree(din);
    cudaFree(dout);
    if (e != cudaSuccess) return proj_cuda_fail(e, "q38_project_host");
    return rc;
}

int q38_linear_attention_decode(q38_ctx *ctx, q38_state *st, int layer, int batch,
                                const q38_linear_projections *w, const float *norm, float *branch,
                                void *stream) {
    if (!ctx || !st || !w || !norm || !branch) return proj_fail(Q38_ERR_ARG, "null argument");
    if (st->ctx != ctx) return proj_fail(Q38_ERR_ARG, "state belongs to another context");
    if (batch <= 0 || batch > st->batch) return proj_fail(Q38_ERR_ARG, "batch %d outside 1..%d", batch, st->batch);
    for (auto [p, name] : {std::pair<const q38_weight *, const char *>{w->qkv, "qkv"}, {w->z, "z"},
                           {w->beta, "beta"}, {w->alpha, "alpha"}, {w->out, "out"}})
        if (int rc = check_weight(ctx, p, name)) return rc;
    const int64_t hidden = w->qkv->w.width;
    const int vh = ctx->geom.linear_v_heads;
    if (w->z->w.width != hidden || w->beta->w.width != hidden || w->alpha->w.width != hidden ||
        w->out->w.rows != hidden || w->qkv->w.rows != ctx->qkv_dim || w->z->w.rows != ctx->v_dim ||
        w->beta->w.rows != vh || w->alpha->w.rows != vh || w->out->w.width != ctx->v_dim)
        return proj_fail(Q38_ERR_ARG, "DeltaNet projection shapes do not match the geometry");
    Guard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float *qkv = st->proj_stage, *z = qkv + size_t(batch) * ctx->qkv_dim;
    float *beta = z + size_t(batch) * ctx->v_dim, *alpha = beta + size_t(batch) * vh;
    float *att = alpha + size_t(batch) * vh;
    // linear_attention, ops.rs:761-801: the four input projections (each
    // quantizes the normalised input itself), the core, the output projection.
    // The core's prologue is fused onto the projections' epilogues: the qkv
    // projection applies the conv (with the layer's carried state) and SiLU
    // to each channel it produces, the beta / alpha projections the gates,
    // and the state kernel L2-normalises q and k itself -- no separate prep
    // kernel. The results equal q38_linear_decode's (the same operations on
    // the same values; only the f64 sum of the L2 norm is added in another
    // order).
    q38::ProjEpilogue conv, gbeta, galpha;
    const float *conv_w = nullptr, *dt_bias = nullptr, *ssm_a = nullptr;
    if (int rc = q38::linear_layer_prologue_args(ctx, st, layer, &conv.conv_state, &conv_w, &dt_bias,
                                                 &ssm_a))
        return rc;
    conv.kind = q38::kEpiConvSilu;
    conv.conv_w = conv_w;
    gbeta.kind = q38::kEpiSigmoid;
    galpha.kind = q38::kEpiGateAlpha;
    galpha.dt_bias = dt_bias;
    galpha.ssm_a = ssm_a;
    const q38_weight *ins[4] = {w->qkv, w->z, w->beta, w->alpha};
    float *outs[4] = {qkv, z, beta, alpha};
    const q38::ProjEpilogue *epis[4] = {&conv, nullptr, &gbeta, &galpha};
    if (takes_mma(w->qkv, batch) && takes_mma(w->z, batch) && !takes_mma(w->beta, batch) &&
        !takes_mma(w->alpha, batch) && st->side_fork) {
        // Tensor-core qkv and z over the same quantized input, and the two
        // small gate projections, run concurrently: each alone leaves most
        // SMs idle (qkv 80, z 48 and each gate 48 CTAs, every CTA walking all
        // the row's blocks). The input is quantized once, then qkv runs on
        // the caller's stream, z on a side stream and the gates on another.
        if (int rc = reserve_scratch(ctx, batch, hidden)) return rc;
        cudaError_t e = q38::launch_proj_mma_quantize(norm, batch, hidden, ctx->proj_scratch, s);
        if (e == cudaSuccess) e = cudaEventRecord(st->side_fork, s);
        for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(st->side[i], st->side_fork, 0);
        if (e != cudaSuccess) return proj_cuda_fail(e, "layer projections fork");
        // Each of qkv and z may take the SMs the other leaves.
        const int tiles_qkv = int((w->qkv->w.rows + 127) / 128), tiles_z = int((w->z->w.rows + 127) / 128);
        const int budget_qkv = std::max(1, ctx->sm_count - tiles_z), budget_z = std::max(1, ctx->sm_count - tiles_qkv);
        if (int rc = project_device(ctx, w->qkv, batch, norm, qkv, st->d_err, s, conv, true, budget_qkv))
            return rc;
        if (int rc = project_device(ctx, w->z, batch, norm, z, st->d_err, st->side[0], {}, true, budget_z))
            return rc;
        if (int rc = project_device(ctx, w->beta, batch, norm, beta, st->d_err, st->side[1], gbeta))
            return rc;
        if (int rc = project_device(ctx, w->alpha, batch, norm, alpha, st->d_err, st->side[1], galpha))
            return rc;
        for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaEventRecord(st->side_join[i], st->side[i]);
        for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(s, st->side_join[i], 0);
        if (e != cudaSuccess) return proj_cuda_fail(e, "layer projections join");
    } else {
        for (int i = 0; i < 4; ++i)
            if (int rc = project_device(ctx, ins[i], batch, norm, outs[i], st->d_err, s,
                                        epis[i] ? *epis[i] : q38::ProjEpilogue{}))
                return rc;
    }
    if (int rc = q38::linear_decode_prepped(ctx, st, layer, batch, qkv, z, beta, alpha, att, s))
        return rc;
    return project_device(ctx, w->out, batch, att, branch, st->d_err, s);
}

int q38_full_attention_decode(q38_ctx *ctx, q38_state *st, int layer, int batch,
                              const q38_full_projections *w, const float *norm,
                              const int32_t *positions, int max_position, float *branch,
                              void *stream) {
    if (!ctx || !st || !w || !norm || !branch || !positions)
        return proj_fail(Q38_ERR_ARG, "null argument");
    if (st->ctx != ctx) return proj_fail(Q38_ERR_ARG, "state belongs to another context");
    if (batch <= 0 || batch > st->batch) return proj_fail(Q38_ERR_ARG, "batch %d outside 1..%d", batch, st->batch);
    for (auto [p, name] : {std::pair<const q38_weight *, const char *>{w->q, "q"}, {w->k, "k"},
                           {w->v, "v"}, {w->out, "out"}})
        if (int rc = check_weight(ctx, p, name)) return rc;
    const int64_t hidden = w->q->w.width;
    if (w->k->w.width != hidden || w->v->w.width != hidden || w->out->w.rows != hidden ||
        w->q->w.rows != ctx->qg_dim || w->k->w.rows != ctx->kv_dim || w->v->w.rows != ctx->kv_dim ||
        w->out->w.width != ctx->q_dim)
        return proj_fail(Q38_ERR_ARG, "full-attention projection shapes do not match the geometry");
    Guard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float *qg = st->proj_stage, *key = qg + size_t(batch) * ctx->qg_dim;
    float *value = key + size_t(batch) * ctx->kv_dim, *att = value + size_t(batch) * ctx->kv_dim;
    // full_attention, ops.rs:954-980.
    const q38_weight *ins[3] = {w->q, w->k, w->v};
    float *outs[3] = {qg, key, value};
    for (int i = 0; i < 3; ++i)
        if (int rc = project_device(ctx, ins[i], batch, norm, outs[i], st->d_err, s)) return rc;
    if (int rc = q38_full_decode(ctx, st, layer, batch, qg, key, value, positions, max_position, att,
                                 stream))
        return rc;
    return project_device(ctx, w->out, batch, att, branch, st->d_err, s);
}

// ---------------------------------------------------------------- prefill layer bodies

namespace {
size_t layer_prefill_floats_per_token(const q38_ctx *ctx) {
    const size_t lin = size_t(ctx->qkv_dim) + ctx->v_dim + 2 * ctx->geom.linear_v_heads + ctx->v_dim;
    const size_t full = size_t(ctx->qg_dim) + 2 * ctx->kv_dim + ctx->q_dim;
    return lin > full ? lin : full;
}

int check_prefill_layer(q38_ctx *ctx, q38_state *st, int seq0, int nseq, int count, const void *w,
                        const float *norm, float *branch) {
    if (!ctx || !st || !w || !norm || !branch) return proj_fail(Q38_ERR_ARG, "null argument");
    if (st->ctx != ctx) return proj_fail(Q38_ERR_ARG, "state belongs to another context");
    if (nseq <= 0 || count <= 0 || seq0 < 0 || seq0 + nseq > st->batch)
        return proj_fail(Q38_ERR_ARG, "sequences [%d, %d) outside the state's %d", seq0, seq0 + nseq, st->batch);
    if (size_t(nseq) * size_t(count) > st->layer_prefill_tokens)
        return proj_fail(Q38_ERR_ARG, "%d prompt tokens exceed q38_state_reserve_attention_prefill's %zu",
                         nseq * count, st->layer_prefill_tokens);
    return Q38_OK;
}
}  // namespace

int q38_state_reserve_attention_prefill(q38_state *st, int max_tokens) {
    if (!st) return proj_fail(Q38_ERR_ARG, "null state");
    if (max_tokens <= 0) return proj_fail(Q38_ERR_ARG, "max_tokens must be positive");
    if (int rc = q38_state_reserve_prefill(st, max_tokens)) return rc;
    q38_ctx *ctx = st->ctx;
    Guard guard(ctx->device);
    const int64_t widest = ctx->v_dim > ctx->q_dim ? ctx->v_dim : ctx->q_dim;
    if (int rc = reserve_scratch(ctx, max_tokens, widest > 5120 ? widest : 5120)) return rc;
    if (size_t(max_tokens) <= st->layer_prefill_tokens) return Q38_OK;
    cudaFree(st->layer_prefill);
    st->layer_prefill = nullptr;
    st->layer_prefill_tokens = 0;
    cudaError_t e = cudaMalloc(&st->layer_prefill,
                               size_t(max_tokens) * layer_prefill_floats_per_token(ctx) * sizeof(float));
    if (e != cudaSuccess) return proj_cuda_fail(e, "attention prefill buffers");
    st->layer_prefill_tokens = size_t(max_tokens);
    return Q38_OK;
}

int q38_linear_attention_prefill(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                                 const q38_linear_projections *w, const float *norm, float *branch,
                                 void *stream) {
    if (int rc = check_prefill_layer(ctx, st, seq0, nseq, count, w, norm, branch)) return rc;
    for (auto [p, name] : {std::pair<const q38_weight *, const char *>{w->qkv, "qkv"}, {w->z, "z"},
                           {w->beta, "beta"}, {w->alpha, "alpha"}, {w->out, "out"}})
        if (int rc = check_weight(ctx, p, name)) return rc;
    const int64_t hidden = w->qkv->w.width;
    const int vh = ctx->geom.linear_v_heads;
    if (w->z->w.width != hidden || w->beta->w.width != hidden || w->alpha->w.width != hidden ||
        w->out->w.rows != hidden || w->qkv->w.rows != ctx->qkv_dim || w->z->w.rows != ctx->v_dim ||
        w->beta->w.rows != vh || w->alpha->w.rows != vh || w->out->w.width != ctx->v_dim)
        return proj_fail(Q38_ERR_ARG, "DeltaNet projection shapes do not match the geometry");
    Guard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int tokens = nseq * count;
    float *qkv = st->layer_prefill, *z = qkv + size_t(tokens) * ctx->qkv_dim;
    float *beta = z + size_t(tokens) * ctx->v_dim, *alpha = beta + size_t(tokens) * vh;
    float *att = alpha + size_t(tokens) * vh;
    // batch_linear_attention, ops.rs:1032-1114: the projections of every
    // prompt token, the chunked core, the output projection.
    const q38_weight *ins[4] = {w->qkv, w->z, w->beta, w->alpha};
    float *outs[4] = {qkv, z, beta, alpha};
    for (int i = 0; i < 4; ++i)
        if (int rc = project_device(ctx, ins[i], tokens, norm, outs[i], st->d_err, s)) return rc;
    if (int rc = q38_linear_prefill(ctx, st, layer, seq0, nseq, count, qkv, z, beta, alpha, att, stream))
        return rc;
    return project_device(ctx, w->out, tokens, att, branch, st->d_err, s);
}

int q38_full_attention_prefill(q38_ctx *ctx, q38_state *st, int layer, int seq0, int nseq, int count,
                               int base_position, const q38_full_projections *w, const float *norm,
                               float *branch, void *stream) {
    if (int rc = check_prefill_layer(ctx, st, seq0, nseq, count, w, norm, branch)) return rc;
    for (auto [p, name] : {std::pair<const q38_weight *, const char *>{w->q, "q"}, {w->k, "k"},
                           {w->v, "v"}, {w->out, "out"}})
        if (int rc = check_weight(ctx, p, name)) return rc;
    const int64_t hidden = w->q->w.width;
    if (w->k->w.width != hidden || w->v->w.width != hidden || w->out->w.rows != hidden ||
        w->q->w.rows != ctx->qg_dim || w->k->w.rows != ctx->kv_dim || w->v->w.rows != ctx->kv_dim ||
        w->out->w.width != ctx->q_dim)
        return proj_fail(Q38_ERR_ARG, "full-attention projection shapes do not match the geometry");
    Guard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int tokens = nseq * count;
    float *qg = st->layer_prefill, *key = qg + size_t(tokens) * ctx->qg_dim;
    float *value = key + size_t(tokens) * ctx->kv_dim, *att = value + size_t(tokens) * ctx->kv_dim;
    // batch_full_attention, ops.rs:1116-1185.
    const q38_weight *ins[3] = {w->q, w->k, w->v};
    float *outs[3] = {qg, key, value};
    for (int i = 0; i < 3; ++i)
        if (int rc = project_device(ctx, ins[i], tokens, norm, outs[i], st->d_err, s)) return rc;
    if (int rc = q38_full_prefill(ctx, st, layer, seq0, nseq, count, base_position, qg, key, value, att, stream))
        return rc;
    return project_device(ctx, w->out, tokens, att, branch, st->d_err, s);
}

}  // extern "C"
