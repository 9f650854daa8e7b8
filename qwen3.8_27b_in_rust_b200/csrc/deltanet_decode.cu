// deltanet_decode.cu -- Gated DeltaNet decode (linear_core, src/model/ops.rs:647-742)
// as two stream-ordered kernels chained with programmatic dependent launch:
//
//   D1 linear_decode_prep   one CTA per (128-channel block, sequence): the
//                           kernel-4 causal conv with carried state
//                           (ops.rs:665-676, multiply then add), SiLU
//                           (ops.rs:677), L2-norm of the q and k heads
//                           (ops.rs:679-684, f64 sum) and the beta/alpha gates
//                           (ops.rs:685-688). Writes qkv/beta/alpha in place,
//                           as the reference does.
//   D2 linear_decode_state  one CTA per (value head, sequence): streams the
//                           head's 128x128 f32 state once (64 KB in, 64 KB out),
//                           decay, delta rule per column (ops.rs:707-713), and
//                           the per-head RMSNorm + SiLU(z) epilogue
//                           (ops.rs:735-740). Its state loads are issued before
//                           it waits on D1, so they overlap D1's tail.
//
// In the layer-level decode call the projections' epilogues apply the conv,
// SiLU and gates (proj_epilogue), so D1 is not launched and D2 L2-normalises
// q and k in its prologue.
//
// HBM layout (reference layouts): conv state [batch][qkv_dim][3], delta state
// [batch][v_heads][128 columns][128], f32.
#include "q38_common.cuh"

namespace q38 {
namespace {

constexpr int kPrepThreads = kLinHeadDim;  // one channel per thread, one head per CTA
constexpr int kStateThreads = 256;          // 8 warps x 16 columns
constexpr int kColsPerWarp = kLinHeadDim / (kStateThreads / 32);

struct PrepParams {
    float *qkv;
    float *beta, *alpha;
    float *conv_state;
    const float *conv_w, *dt_bias, *ssm_a;
    int qk_heads, v_heads, qkv_dim;
    float eps;
};

__global__ void __launch_bounds__(kPrepThreads) linear_decode_prep_kernel(PrepParams p) {
    pdl_launch_dependents();
    __shared__ double red[32];
    const int blk = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    const int ch = blk * kLinHeadDim + t;
    float *s = p.conv_state + (size_t(b) * p.qkv_dim + ch) * 3;
    const float4 w = reinterpret_cast<const float4 *>(p.conv_w)[ch];
    float *x_ptr = p.qkv + size_t(b) * p.qkv_dim + ch;
    const float x = *x_ptr;
    const float s0 = s[0], s1 = s[1], s2 = s[2];
    // value = s0*w0; value += s1*w1; value += s2*w2; value += x*w3 (no fma).
    float v = s0 * w.x;
    v += s1 * w.y;
    v += s2 * w.z;
    v += x * w.w;
    s[0] = s1;
    s[1] = s2;
    s[2] = x;
    float y = siluf_ref(v);
    if (blk < 2 * p.qk_heads) {
        // l2norm (ops.rs:562-571): 1 / max(sqrt((f32) sum_f64), eps).
        const double sum = block_sum_f64(double(y) * double(y), red);
        const float scale = 1.0f / fmaxf(sqrtf(float(sum)), p.eps);
        y *= scale;
    } else if (t == 0) {
        const int hv = blk - 2 * p.qk_heads;
        float *bp = p.beta + size_t(b) * p.v_heads + hv;
        float *ap = p.alpha + size_t(b) * p.v_heads + hv;
        *bp = sigmoidf_ref(*bp);
        *ap = p.ssm_a[hv] * softplusf_ref(*ap + p.dt_bias[hv]);
    }
    *x_ptr = y;
}

struct StateParams {
    const float *qkv;
    const float *z;
    const float *beta, *alpha;
    float *delta_state;
    const float *ssm_norm;
    float *attention;
    int qk_heads, v_heads, qkv_dim;
    int l2_prologue;  // q and k arrive convolved but not yet L2-normalised
    float eps;
};

__global__ void __launch_bounds__(kStateThreads) linear_decode_state_kernel(StateParams p) {
    __shared__ float outs[kLinHeadDim];
    __shared__ double red[32];
    const int hv = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float4 *S = reinterpret_cast<float4 *>(
        p.delta_state + (size_t(b) * p.v_heads + hv) * kLinHeadDim * kLinHeadDim);
    const int col0 = warp * kColsPerWarp;

    // The state does not depend on D1: load this warp's 16 rows now.
    float4 s[kColsPerWarp];
#pragma unroll
    for (int i = 0; i < kColsPerWarp; ++i) s[i] = S[(col0 + i) * (kLinHeadDim / 4) + lane];

    pdl_wait_primary();  // D1's qkv / beta / alpha

    const int kh = hv % p.qk_heads;  // ops.rs:699
    const int qk_dim = p.qk_heads * kLinHeadDim;
    const float *row = p.qkv + size_t(b) * p.qkv_dim;
    float4 q = reinterpret_cast<const float4 *>(row + kh * kLinHeadDim)[lane];
    float4 k = reinterpret_cast<const float4 *>(row + qk_dim + kh * kLinHeadDim)[lane];
    if (p.l2_prologue) {
        // l2norm (ops.rs:562-571) of the key head's q and k, here rather than
        // in D1 (the layer-level call's projections already applied the conv,
        // SiLU and gates): every warp holds both heads whole, four values per
        // lane, and sums their squares in f64.
        const double sq = warp_sum_f64(double(q.x) * q.x + double(q.y) * q.y + double(q.z) * q.z +
                                       double(q.w) * q.w);
        const double sk = warp_sum_f64(double(k.x) * k.x + double(k.y) * k.y + double(k.z) * k.z +
                                       double(k.w) * k.w);
        const float cq = 1.0f / fmaxf(sqrtf(float(sq)), p.eps);
        const float ck = 1.0f / fmaxf(sqrtf(float(sk)), p.eps);
        q.x *= cq, q.y *= cq, q.z *= cq, q.w *= cq;
        k.x *= ck, k.y *= ck, k.z *= ck, k.w *= ck;
    }
    const float vmine = lane < kColsPerWarp ? row[2 * qk_dim + hv * kLinHeadDim + col0 + lane] : 0.f;
    const float beta = p.beta[size_t(b) * p.v_heads + hv];
    const float decay = expf(p.alpha[size_t(b) * p.v_heads + hv]);
    const float query_scale = 1.0f / sqrtf(float(kLinHeadDim));

#pragma unroll
    for (int i = 0; i < kColsPerWarp; ++i) {
        float4 r = s[i];
        r.x *= decay;
        r.y *= decay;
        r.z *= decay;
        r.w *= decay;
        // dot_128 (ops.rs:573-579): lane-local fma chain, then the warp tree.
        float pred = fmaf(r.w, k.w, fmaf(r.z, k.z, fmaf(r.y, k.y, r.x * k.x)));
        pred = warp_sum(pred);
        const float vj = __shfl_sync(0xffffffffu, vmine, i);
        const float delta = (vj - pred) * beta;
        // mad_dot_128 (ops.rs:584-591): state += k*delta (fma), then dot with q.
        r.x = fmaf(k.x, delta, r.x);
        r.y = fmaf(k.y, delta, r.y);
        r.z = fmaf(k.z, delta, r.z);
        r.w = fmaf(k.w, delta, r.w);
        float o = fmaf(r.w, q.w, fmaf(r.z, q.z, fmaf(r.y, q.y, r.x * q.x)));
        o = warp_sum(o);
        S[(col0 + i) * (kLinHeadDim / 4) + lane] = r;
        if (lane == 0) outs[col0 + i] = o * query_scale;
    }
    __syncthreads();
    // rmsnorm_inplace(ssm_norm) then *= silu(z) (ops.rs:735-740).
    const int t = threadIdx.x;
    const float o = t < kLinHeadDim ? outs[t] : 0.f;
    const double sum = block_sum_f64(t < kLinHeadDim ? double(o) * double(o) : 0.0, red);
    if (t < kLinHeadDim) {
        const float scale = rms_scale_from_sum(sum, kLinHeadDim, p.eps);
        float y = o * scale * p.ssm_norm[t];
        const size_t off = size_t(b) * p.v_heads * kLinHeadDim + size_t(hv) * kLinHeadDim + t;
        y *= siluf_ref(p.z[off]);
        p.attention[off] = y;
    }
}

}  // namespace

cudaError_t launch_linear_decode(const LinearDecodeLaunch &a, cudaStream_t stream, cudaEvent_t prep_done) {
    const int qkv_dim = (2 * a.qk_heads + a.v_heads) * kLinHeadDim;
    cudaError_t e = cudaSuccess;
    if (!a.prepped) {
        PrepParams pp{a.qkv,    a.beta,    a.alpha,     a.conv_state, a.conv_w, a.dt_bias,
                      a.ssm_a,  a.qk_heads, a.v_heads,  qkv_dim,      a.eps};
        linear_decode_prep_kernel<<<dim3(2 * a.qk_heads + a.v_heads, a.batch), kPrepThreads, 0,
                                    stream>>>(pp);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    // With prep_done recorded between the two kernels, D2 is an ordinary
    // launch (no programmatic overlap across the record).
    if (prep_done && (e = cudaEventRecord(prep_done, stream)) != cudaSuccess) return e;

    // Prepped inputs (conv, SiLU and gates applied by the projections): the
    // state kernel normalises q and k itself and follows the last projection
    // as its programmatic dependent.
    StateParams sp{a.qkv,      a.z,        a.beta,    a.alpha,   a.delta_state,
                   a.ssm_norm, a.attention, a.qk_heads, a.v_heads, qkv_dim,
                   a.prepped ? 1 : 0,       a.eps};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.v_heads, a.batch);
    cfg.blockDim = dim3(kStateThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = prep_done ? 0 : 1;
    return cudaLaunchKernelEx(&cfg, linear_decode_state_kernel, sp);
}

}  // namespace q38
