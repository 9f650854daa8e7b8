// q38_proj.h -- projection weights and launchers (proj.cu). Internal, not
// part of the public ABI.
#pragma once

#include "q38_common.cuh"

namespace q38 {

// What a projection does to each output before storing it: nothing, or the
// prologue of the DeltaNet core fused onto the projection's epilogue (the
// layer-level decode call, where the projection outputs are internal):
//   kEpiConvSilu   the qkv projection: kernel-4 causal conv of channel `row`
//                  with the sequence's carried state, multiply then add
//                  (ops.rs:665-676), state shifted in place, then SiLU
//                  (ops.rs:677);
//   kEpiSigmoid    the beta projection: sigmoid (ops.rs:685-686);
//   kEpiGateAlpha  the alpha projection: ssm_a * softplus(x + dt_bias)
//                  (ops.rs:687-688).
// Token t of a decode batch is sequence t.
constexpr int kEpiNone = 0, kEpiConvSilu = 1, kEpiSigmoid = 2, kEpiGateAlpha = 3;
struct ProjEpilogue {
    int kind = kEpiNone;
    float *conv_state = nullptr;    // kEpiConvSilu: [batch][rows][3]
    const float *conv_w = nullptr;  // kEpiConvSilu: [rows][4]
    const float *dt_bias = nullptr, *ssm_a = nullptr;  // kEpiGateAlpha: [rows]
    int tok0 = 0;                   // the launch's first token in the batch
};

// The values an epilogue reads for output (t, row), loaded ahead of the
// output itself so that their latency overlaps the row's dot products.
struct EpilogueIn {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;  // kEpiConvSilu: the carried conv state
    float4 w = {0.f, 0.f, 0.f, 0.f};     // kEpiConvSilu: the channel's conv weights
    float a = 0.f, bias = 0.f;           // kEpiGateAlpha: ssm_a, dt_bias
};

__device__ __forceinline__ EpilogueIn proj_epilogue_load(const ProjEpilogue &e, int rows, int t,
                                                         int row) {
    EpilogueIn in;
    if (e.kind == kEpiConvSilu) {
        const float *s = e.conv_state + (size_t(e.tok0 + t) * rows + row) * 3;
        in.s0 = s[0];
        in.s1 = s[1];
        in.s2 = s[2];
        in.w = reinterpret_cast<const float4 *>(e.conv_w)[row];
    } else if (e.kind == kEpiGateAlpha) {
        in.a = e.ssm_a[row];
        in.bias = e.dt_bias[row];
    }
    return in;
}

__device__ __forceinline__ float proj_epilogue_apply(const ProjEpilogue &e, const EpilogueIn &in,
                                                     int rows, int t, int row, float x) {
    switch (e.kind) {
        case kEpiConvSilu: {
            float v = in.s0 * in.w.x;
            v += in.s1 * in.w.y;
            v += in.s2 * in.w.z;
            v += x * in.w.w;
            float *s = e.conv_state + (size_t(e.tok0 + t) * rows + row) * 3;
            s[0] = in.s1;
            s[1] = in.s2;
            s[2] = x;
            return siluf_ref(v);
        }
        case kEpiSigmoid: return sigmoidf_ref(x);
        case kEpiGateAlpha: return in.a * softplusf_ref(x + in.bias);
        default: return x;
    }
}

__device__ __forceinline__ float proj_epilogue(const ProjEpilogue &e, int rows, int t, int row,
                                               float x) {
    return proj_epilogue_apply(e, proj_epilogue_load(e, rows, t, row), rows, t, row, x);
}

constexpr int kProjMaxTok = 8;          // tokens per integer-path launch (more: repeated launches)
constexpr int kProjMaxTileRows = 16;    // rows per weight tile at most
constexpr uint32_t kProjSmemBudget = 224 * 1024;

// Q8_K activations on the device, structure-of-arrays (token-major blocks):
// quants [tokens][nblk][256], scale [tokens][nblk], sums [tokens][nblk][16].
struct Q8KActivations {
    int8_t *quants = nullptr;
    float *scale = nullptr;
    int16_t *sums = nullptr;
};

// A projection matrix as the GGUF stores it: `rows` rows of row_bytes bytes,
// each row one output over `width` inputs (shape [width, rows]).
struct ProjWeight {
    int type = -1;
    int64_t rows = 0, width = 0, row_bytes = 0;  // row_bytes: device layout
    void *data = nullptr;  // device, proj_padded_bytes long
    // Integer planes for batched projections (proj_planes.cu), or null: the
    // tile-major atoms (planes) and the tile-major 16-byte side records
    // (plane_side), one allocation.
    void *planes = nullptr, *plane_side = nullptr;
    int64_t plane_rows = 0;
};

bool proj_is_q8k_type(int type);
bool proj_type_supported(int type);
// Q6_K blocks are 210 bytes in the checkpoint; on the device each is padded
// to 224 (14 x 16) so that every block starts 16-byte aligned and a tile of
// blocks is a valid TMA box. The other types keep their checkpoint layout.
constexpr int kQ6KDeviceBlock = 224;
int64_t proj_row_bytes(int type, int64_t width);         // checkpoint row bytes; -1: type cannot hold such rows
int64_t proj_device_row_bytes(int type, int64_t width);  // device row bytes
size_t proj_padded_bytes(int type, int64_t rows, int64_t width);

cudaError_t launch_q8k_quantize(const float *x, int batch, int width, Q8KActivations act, void *aos,
                                cudaStream_t stream);
// Quantizes x [batch][width] to Q8_K inside the kernel (no separate pass).
cudaError_t launch_proj_q8k(const ProjWeight &w, const float *x, int batch, float *out,
                            long out_ld, int *err, int sm_count, cudaStream_t stream,
                            const ProjEpilogue &epi = {});
// Tensor-core path for Q4_K / Q5_K weights and kProjMmaMinBatch+ tokens
// (proj_mma.cu): quantizes x into `scratch` (proj_mma_scratch_bytes), then
// one tcgen05 kind::i8 GEMM, bit-identical to the integer GEMV.
constexpr int kProjMmaMinBatch = 9;
bool proj_mma_supported(int type);
size_t proj_mma_scratch_bytes(int batch, int64_t width);
// prequantized: `scratch` already holds x's quantization (an earlier
// launch_proj_mma or launch_proj_mma_quantize of the same x and width).
cudaError_t launch_proj_mma(const ProjWeight &w, const float *x, int batch, float *out, long out_ld,
                            int *err, void *scratch, cudaStream_t stream,
                            const ProjEpilogue &epi = {}, bool prequantized = false);
cudaError_t launch_proj_mma_quantize(const float *x, int batch, int64_t width, void *scratch,
                                     cudaStream_t stream);

// Integer planes of a Q4_K / Q5_K / Q6_K weight (proj_planes.cu): built once
// (synchronously on `stream`), then every 9+ token projection of the weight
// streams them on the tensor cores, bit-identical to the integer GEMV.
bool proj_planes_type(int type);
size_t proj_plane_bytes(int type, int64_t rows, int64_t width);
cudaError_t build_proj_planes(ProjWeight &w, cudaStream_t stream);
void free_proj_planes(ProjWeight &w);
// sm_budget: the SMs this launch may assume free (fewer when projections run
// concurrently); it picks 16- or 32-token tiles.
cudaError_t launch_proj_planes(const ProjWeight &w, const float *x, int batch, float *out, long out_ld,
                               int *err, void *scratch, cudaStream_t stream, const ProjEpilogue &epi = {},
                               bool prequantized = false, int sm_budget = 148);

// f32-input projections (F32 / F16 / BF16 / Q8_0). part: a workspace of
// proj_f32_tile_part_bytes for the chunked form that batches of 9+ tokens
// over up to kProjTileMaxRows rows take (proj_f32_takes_tile), or null for
// the warp form.
constexpr int kProjTileMaxRows = 128;
bool proj_f32_takes_tile(int type, int64_t rows, int64_t width, int batch);
size_t proj_f32_tile_part_bytes(int64_t rows, int64_t width, int batch);
cudaError_t launch_proj_f32(const ProjWeight &w, const float *x, int batch, float *out, long out_ld,
                            cudaStream_t stream, const ProjEpilogue &epi = {}, float *part = nullptr);

}  // namespace q38

struct q38_weight {
    q38_ctx *ctx = nullptr;
    q38::ProjWeight w;
};
