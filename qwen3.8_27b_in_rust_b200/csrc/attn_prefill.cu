// attn_prefill.cu -- causal gated full-attention prefill on tcgen05 tensor
// cores. Replaces the per-token full_core loop of batch_full_attention
// (src/model/ops.rs:1156-1172): token t of the prompt attends to cache
// positions 0..base+t, exactly as full_core at current_position = base+t.
//
//   P1 attn_prefill_prep  one CTA per (token, sequence), a warp per head: q/k RMSNorm
//                         (f64 sum), partial RoPE (iterative f32 angle), K/V
//                         append to the bf16 cache, key written back, and the
//                         prepared query rounded to bf16 into the Q scratch
//                         [seq][head][token][256].
//   P1b attn_prefill_prefix  only when base > 0: the cached prefix's V rows
//                         (bf16) copied as f16 into the V scratch.
//   P2 attn_prefill_pair  a cluster of two CTAs per (256-query pair of tiles,
//                         head, sequence), heaviest pairs first; every MMA is a
//                         cta_group::2 MMA that the leader CTA issues for both
//                         SMs (see the kernel's comment). Warp roles per CTA:
//                           warp 0   TMA: this CTA's Q rows once, then its half
//                                    (32 keys) of every K tile, 4-deep ring;
//                           warp 7   TMA: its half (128 dims) of every f16 V
//                                    tile, 4-deep ring;
//                           warps 1, 8  (leader) S = Q K^T of even / odd key
//                                    tiles, M=256 N=64 K=256, Q from shared
//                                    memory, into four TMEM S buffers;
//                           warp 6   (leader) O += P V, M=256 N=256 K=64, P
//                                    from TMEM (f16 over the S buffer), V
//                                    MN-major;
//                           warps 2-5 softmax, one query row per thread: S
//                                    from TMEM, causal mask, online max with
//                                    lazy O rescale (only when the max grows by
//                                    more than 2^8), P = exp2 in f16 into TMEM;
//                                    then the epilogue O / l * sigmoid(gate).
//                         TMEM per CTA: S0..S3 (64 columns each) | O (256).
//
// Precision: S = Q K^T from bf16 Q and K (the bf16 cache) or from f16 Q and K
// (an f32 cache: the f32 rows stay in the cache and f16 copies, 8x finer than
// bf16, feed the tensor cores); O = P V in f16 (P rounded to f16 has 4x less
// error than bf16, which matters for the first rows of a prompt that see only
// a few keys; bf16 V values are exact in f16 for 2^-14 <= |v| <= 65504). A
// value beyond the f16 range (|x| > 65504) in an f16 operand sets
// kDevErrRange. f32 accumulation throughout. Tolerance 2e-3.
#include "q38_sm100.cuh"

#include <cudaTypedefs.h>

namespace q38 {
namespace {

using namespace sm100;

constexpr int kBlockQ = 128;  // query rows per CTA (MMA M)
constexpr int kRopeHalf = kRopeDims / 2;  // RoPE angles per position
// RoPE table of a prefill call: per block of 128 positions, [64][128] f32
// (cos of angles 0-31, then their sin, each over the block's positions), so
// that one bulk copy brings a CTA's block and thread r reads column r.
constexpr int kRopeBlockFloats = kRopeDims * kBlockQ;
constexpr uint32_t kRopeBlockBytes = kRopeBlockFloats * 4;  // 32 KB
constexpr int kBlockK = 64;   // keys per tile (QK N, PV K)
constexpr int kThreadsPF = 288;
constexpr uint32_t kQBytes = kBlockQ * kAttnHeadDim * 2;      // 64 KB
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// --------------------------------------------------------------------------
// P1: prep
// --------------------------------------------------------------------------
struct PrefillPrepParams {
    float *key;               // [nseq][count][kv_heads*256]
    const float *value;
    void *kcache, *vcache;    // slot base: [batch][kv_heads][ctx][256], bf16 or f32 (kv_f32)
    __half *v16;              // [nseq][kv_heads][ctx][256]: V as f16 for P V
    __half *k16;              // kv_f32 only: [nseq][kv_heads][ctx][256], K as f16 for Q K^T
    float *rope;              // RoPE table, blocks of [64][128] (see kRopeBlockFloats)
    const float *k_norm;
    int *err;
    int seq0, count, base, context_length, kv_heads, kv_head0, kv_head_count, kv_f32;
    float theta_scale, eps;
};

// True when a bf16 pair (one 32-bit word) holds a value that f16 cannot
// represent (|v| > 65504, infinities included): the P V operand would
// overflow, so the call flags kDevErrRange.
__device__ __forceinline__ bool f16_overflow(uint32_t w) {
    const float2 f = bf16x2_to_float2(w);
    return fabsf(f.x) > 65504.f || fabsf(f.y) > 65504.f;
}

// One warp per (token, kv head of the call's range), 8 / kv_head_count tokens
// per CTA. Lane l holds dims [8l, 8l+8) of a head, so the RoPE partner of dim
// i < 32 (dim i + 32) sits in lane l ^ 4 at the same slot. The CTAs of the
// first sequence also write the RoPE table that the attention kernel applies
// to the queries.
constexpr int kPrepWarps = 8;

__global__ void __launch_bounds__(kPrepWarps * 32) attn_prefill_prep_kernel(PrefillPrepParams p) {
    pdl_launch_dependents();
    __shared__ float cs[kPrepWarps][32], sn[kPrepWarps][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tokens = kPrepWarps / p.kv_head_count;  // per CTA
    const int s = blockIdx.y;
    // rope (ops.rs:595-610): theta_i = pos * scale^i by repeated f32 products.
    if (warp < tokens) {
        const int t = blockIdx.x * tokens + warp;
        if (t < p.count) {
            float theta = float(p.base + t);
            for (int j = 0; j < lane; ++j) theta *= p.theta_scale;
            const float c = cosf(theta), sv = sinf(theta);
            cs[warp][lane] = c;
            sn[warp][lane] = sv;
            if (s == 0) {
                float *blk = p.rope + size_t(t / kBlockQ) * kRopeBlockFloats + t % kBlockQ;
                blk[lane * kBlockQ] = c;
                blk[(kRopeHalf + lane) * kBlockQ] = sv;
            }
        }
    }
    __syncthreads();
    const int slot = warp / p.kv_head_count, kvh = p.kv_head0 + warp % p.kv_head_count;
    const int t = blockIdx.x * tokens + slot;
    if (slot >= tokens || t >= p.count) return;
    const int pos = p.base + t;
    const size_t tok = size_t(s) * p.count + t;
    const int d0 = 8 * lane;
    const size_t off = (tok * p.kv_heads + kvh) * kAttnHeadDim + d0;
    const float4 a = reinterpret_cast<const float4 *>(p.key + off)[0];
    const float4 b = reinterpret_cast<const float4 *>(p.key + off)[1];
    const float4 va = reinterpret_cast<const float4 *>(p.value + off)[0];
    const float4 vb = reinterpret_cast<const float4 *>(p.value + off)[1];
    float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    // rmsnorm_inplace (ops.rs:493-498) with rms_scale's f64 accumulation.
    double sum = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += double(x[j]) * double(x[j]);
    sum = warp_sum_f64(sum);
    const float scale = rms_scale_from_sum(sum, kAttnHeadDim, p.eps);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = x[j] * scale * p.k_norm[d0 + j];
    // RoPE on dims [0, 64): lanes 0-3 hold dims i < 32, lanes 4-7 dims i+32.
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, x[j], 4);
        if (lane < 4) {
            const int i = d0 + j;
            x[j] = x[j] * cs[slot][i] - other * sn[slot][i];
        } else if (lane < 8) {
            const int i = d0 + j - 32;
            x[j] = other * sn[slot][i] + x[j] * cs[slot][i];
        }
    }
    reinterpret_cast<float4 *>(p.key + off)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4 *>(p.key + off)[1] = make_float4(x[4], x[5], x[6], x[7]);
    const size_t row =
        ((size_t(p.seq0 + s) * p.kv_heads + kvh) * p.context_length + pos) * kAttnHeadDim + d0;
    const size_t srow = ((size_t(s) * p.kv_heads + kvh) * p.context_length + pos) * kAttnHeadDim + d0;
    uint4 kk, vv, vh;
    kk.x = pack_bf16x2_rn(x[0], x[1]);
    kk.y = pack_bf16x2_rn(x[2], x[3]);
    kk.z = pack_bf16x2_rn(x[4], x[5]);
    kk.w = pack_bf16x2_rn(x[6], x[7]);
    if (p.kv_f32) {
        // The reference's f32 rows go to the cache; the tensor-core operands
        // are K and V as f16 (each rounded once from f32, 8x finer than bf16)
        // in the scratch, and the attention kernel rounds Q to f16 as well.
        float4 *kc = reinterpret_cast<float4 *>(static_cast<float *>(p.kcache) + row);
        float4 *vc = reinterpret_cast<float4 *>(static_cast<float *>(p.vcache) + row);
        kc[0] = make_float4(x[0], x[1], x[2], x[3]);
        kc[1] = make_float4(x[4], x[5], x[6], x[7]);
        vc[0] = va;
        vc[1] = vb;
        float kmax = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) kmax = fmaxf(kmax, fabsf(x[j]));
        *reinterpret_cast<uint4 *>(p.k16 + srow) =
            make_uint4(pack_f16x2(x[0], x[1]), pack_f16x2(x[2], x[3]), pack_f16x2(x[4], x[5]),
                       pack_f16x2(x[6], x[7]));
        const float vmax = fmaxf(fmaxf(fmaxf(fabsf(va.x), fabsf(va.y)), fmaxf(fabsf(va.z), fabsf(va.w))),
                                 fmaxf(fmaxf(fabsf(vb.x), fabsf(vb.y)), fmaxf(fabsf(vb.z), fabsf(vb.w))));
        if (fmaxf(vmax, kmax) > 65504.f) set_error(p.err, kDevErrRange);
        vh.x = pack_f16x2(va.x, va.y);
        vh.y = pack_f16x2(va.z, va.w);
        vh.z = pack_f16x2(vb.x, vb.y);
        vh.w = pack_f16x2(vb.z, vb.w);
    } else {
        vv.x = pack_bf16x2_rn(va.x, va.y);
        vv.y = pack_bf16x2_rn(va.z, va.w);
        vv.z = pack_bf16x2_rn(vb.x, vb.y);
        vv.w = pack_bf16x2_rn(vb.z, vb.w);
        *reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.kcache) + row) = kk;
        *reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.vcache) + row) = vv;
        // The same bf16 values as f16 (exact for 2^-14 <= |v| <= 65504).
        if (f16_overflow(vv.x) || f16_overflow(vv.y) || f16_overflow(vv.z) || f16_overflow(vv.w))
            set_error(p.err, kDevErrRange);
        float2 f;
        f = bf16x2_to_float2(vv.x); vh.x = pack_f16x2(f.x, f.y);
        f = bf16x2_to_float2(vv.y); vh.y = pack_f16x2(f.x, f.y);
        f = bf16x2_to_float2(vv.z); vh.z = pack_f16x2(f.x, f.y);
        f = bf16x2_to_float2(vv.w); vh.w = pack_f16x2(f.x, f.y);
    }
    *reinterpret_cast<uint4 *>(p.v16 + srow) = vh;
}

// --------------------------------------------------------------------------
// P1b: f16 copy of the cached prefix's V rows
// --------------------------------------------------------------------------
struct PrefixParams {
    const void *kcache, *vcache;  // slot base [batch][kv_heads][ctx][256], bf16 or f32 (kv_f32)
    __half *v16;                  // [nseq][kv_heads][ctx][256]
    __half *k16;                  // kv_f32 only: [nseq][kv_heads][ctx][256]
    int *err;
    int seq0, base, context_length, kv_heads, kv_head0, kv_f32;
};

// One thread per 8 values of the rows [0, base) of each (sequence, kv head of
// the call's range): V as f16 into the V scratch; for an f32 cache also K as
// f16 into the K scratch.
__global__ void __launch_bounds__(256) attn_prefill_prefix_kernel(PrefixParams p) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i >= p.base * (kAttnHeadDim / 8)) return;
    const int kvh = p.kv_head0 + blockIdx.y, s = blockIdx.z;
    const size_t row = size_t(i) / (kAttnHeadDim / 8), c8 = size_t(i) % (kAttnHeadDim / 8);
    const size_t src =
        ((size_t(p.seq0 + s) * p.kv_heads + kvh) * p.context_length + row) * kAttnHeadDim + c8 * 8;
    const size_t dst = ((size_t(s) * p.kv_heads + kvh) * p.context_length + row) * kAttnHeadDim + c8 * 8;
    uint4 w;
    if (p.kv_f32) {
        const float4 *kr = reinterpret_cast<const float4 *>(static_cast<const float *>(p.kcache) + src);
        const float4 *vr = reinterpret_cast<const float4 *>(static_cast<const float *>(p.vcache) + src);
        const float4 ka = kr[0], kb = kr[1], va = vr[0], vb = vr[1];
        *reinterpret_cast<uint4 *>(p.k16 + dst) =
            make_uint4(pack_f16x2(ka.x, ka.y), pack_f16x2(ka.z, ka.w), pack_f16x2(kb.x, kb.y),
                       pack_f16x2(kb.z, kb.w));
        const float vmax = fmaxf(fmaxf(fmaxf(fabsf(va.x), fabsf(va.y)), fmaxf(fabsf(va.z), fabsf(va.w))),
                                 fmaxf(fmaxf(fabsf(vb.x), fabsf(vb.y)), fmaxf(fabsf(vb.z), fabsf(vb.w))));
        const float kmax = fmaxf(fmaxf(fmaxf(fabsf(ka.x), fabsf(ka.y)), fmaxf(fabsf(ka.z), fabsf(ka.w))),
                                 fmaxf(fmaxf(fabsf(kb.x), fabsf(kb.y)), fmaxf(fabsf(kb.z), fabsf(kb.w))));
        if (fmaxf(vmax, kmax) > 65504.f) set_error(p.err, kDevErrRange);
        w = make_uint4(pack_f16x2(va.x, va.y), pack_f16x2(va.z, va.w), pack_f16x2(vb.x, vb.y),
                       pack_f16x2(vb.z, vb.w));
    } else {
        w = *reinterpret_cast<const uint4 *>(static_cast<const __nv_bfloat16 *>(p.vcache) + src);
        if (f16_overflow(w.x) || f16_overflow(w.y) || f16_overflow(w.z) || f16_overflow(w.w))
            set_error(p.err, kDevErrRange);
        float2 f;
        f = bf16x2_to_float2(w.x); w.x = pack_f16x2(f.x, f.y);
        f = bf16x2_to_float2(w.y); w.y = pack_f16x2(f.x, f.y);
        f = bf16x2_to_float2(w.z); w.z = pack_f16x2(f.x, f.y);
        f = bf16x2_to_float2(w.w); w.w = pack_f16x2(f.x, f.y);
    }
    *reinterpret_cast<uint4 *>(p.v16 + dst) = w;
}

// --------------------------------------------------------------------------
// P2: attention
// --------------------------------------------------------------------------
struct PrefillParams {
    const float *q_norm;  // [256]
    const float *rope;    // RoPE table, blocks of [64][128] (see kRopeBlockFloats)
    int *err;
    int kseq0;            // sequence index of the call's first sequence in the K map's planes
    int count, base, head0, kv_heads, n_qtiles;
    int op_f16;           // Q and K operands in f16 (f32 cache) instead of bf16
    float eps;
};

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(*reinterpret_cast<uint64_t *>(&a)), "l"(*reinterpret_cast<uint64_t *>(&b)));
    return *reinterpret_cast<float2 *>(&r);
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 1/(1+exp(-x)) from the approximate exp2 and reciprocal (relative error
// ~1e-7, far inside the prefill path's 2e-3 tolerance).
__device__ __forceinline__ float sigmoid_fast(float x) {
    float r;
    const float d = 1.0f + ex2(-1.4426950408889634f * x);
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
    return r;
}

// --------------------------------------------------------------------------
// P2 (pair form): two CTAs of a cluster share every MMA (cta_group::2).
// --------------------------------------------------------------------------
// The pair covers 256 query rows of one (head, sequence): the leader (rank 0)
// rows q0..q0+127, the peer rows q0+128..q0+255, each in its own TMEM lanes.
// One S = Q K^T instruction (M=256, N=64, Q from shared memory) and one
// O += P V instruction (M=256, N=256, P from TMEM) serve both SMs, so each
// SM pays half the per-instruction issue cost and stages only half of every
// K tile (32 keys) and half of every V tile (128 dims). With Q in shared
// memory, TMEM holds four S buffers next to O, so four QK tiles can be in
// flight; P(j) is written over the first 32 columns of S buffer j % 4, which
// is free again once PV(j) has completed. The leader's warps 1, 8 (QK) and 6
// (PV) issue all MMAs; both CTAs load, run the softmax and write their rows.
constexpr int kPairRows = 2 * kBlockQ;
constexpr int kPairSBuf = 4;
constexpr uint32_t kKHalf = (kBlockK / 2) * kAttnHeadDim * 2;  // 16 KB: 32 keys x 256 dims
constexpr uint32_t kVHalf = kBlockK * (kAttnHeadDim / 2) * 2;  // 16 KB: 64 keys x 128 dims
constexpr int kPairStagesK = 4;
constexpr int kPairStagesV = 4;
constexpr uint32_t kSmemPair =
    kQBytes + kPairStagesK * kKHalf + kPairStagesV * kVHalf + kRopeBlockBytes + 1024;
constexpr uint32_t kPairColO = kPairSBuf * kBlockK;  // 256: O after the four S buffers

struct __align__(8) PairBarriers {
    uint64_t q_full, q_conv, q_pair;
    uint64_t k_full[kPairStagesK], k_empty[kPairStagesK], v_full[kPairStagesV], v_empty[kPairStagesV];
    uint64_t s_full[kPairSBuf], p_full[kPairSBuf], s_free[kPairSBuf], o_final;
    uint64_t gate_full, epi_l, epi_box[8];
};

// Epilogue staging: the gate block of the CTA's 128 rows (f32) lands by TMA
// over the Q and K-ring region, free once the last S = Q K^T has completed,
// as eight 32-column boxes of 128 rows x 128 B (128-byte swizzle); the output
// O / l * sigmoid(gate) is written over it in place and stored by TMA.
constexpr int kEpiBoxCols = 32;
constexpr uint32_t kEpiBoxBytes = kBlockQ * kEpiBoxCols * 4;  // 16 KB
constexpr int kEpiBoxes = kAttnHeadDim / kEpiBoxCols;          // 8
static_assert(kEpiBoxes * kEpiBoxBytes == kQBytes + kPairStagesK * kKHalf,
              "the gate block fills the Q and K-ring region exactly");
constexpr int kGatePrefetchTiles = 8;  // L2 prefetch of the gate this many key tiles early
constexpr int kQueryWarps = 8;         // warps 1-8 prepare the query rows (two threads per row)

// Arrival on a barrier of the leader CTA (cluster address), ordered like the
// local tcgen05 handshakes (tcgen05.wait + fence::before_thread_sync first).
__device__ __forceinline__ void mbar_arrive_leader(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsPF, 1)
    attn_prefill_pair_kernel(const __grid_constant__ CUtensorMap map_k,
                             const __grid_constant__ CUtensorMap map_v,
                             const __grid_constant__ CUtensorMap map_g,
                             const __grid_constant__ CUtensorMap map_o, PrefillParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *sQ = smem;                          // this CTA's 128 query rows (bf16)
    unsigned char *sK = sQ + kQBytes;                  // kPairStagesK half tiles
    unsigned char *sV = sK + kPairStagesK * kKHalf;    // kPairStagesV half tiles (f16)
    unsigned char *sT = sV + kPairStagesV * kVHalf;    // RoPE rows of the CTA's positions
    __shared__ PairBarriers bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ volatile int abort_flag;
    __shared__ float inv_l_s[kBlockQ];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int n_pairs = (p.n_qtiles + 1) / 2;
    const int pair = n_pairs - 1 - int(blockIdx.x >> 1);  // latest (heaviest) pairs first
    const int h = p.head0 + int(blockIdx.y), s = blockIdx.z;
    const int kvh = h / kGroup;
    const int q0 = pair * kPairRows + int(rank) * kBlockQ;
    const int q_rows = min(kBlockQ, p.count - q0);        // may be <= 0 for the peer
    const int kend = p.base + min(pair * kPairRows + kPairRows, p.count);
    const int nkt = (kend + kBlockK - 1) / kBlockK;
    const bool has_rows = q_rows > 0;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(&bar.q_full, 1);
        mbar_init(&bar.q_conv, kQueryWarps);
        mbar_init(&bar.q_pair, 2 * kQueryWarps);  // used in the leader only
        for (int b = 0; b < kPairStagesK; ++b) {
            mbar_init(&bar.k_full[b], 1);
            mbar_init(&bar.k_empty[b], 1);
        }
        for (int b = 0; b < kPairStagesV; ++b) {
            mbar_init(&bar.v_full[b], 1);
            mbar_init(&bar.v_empty[b], 1);
        }
        for (int b = 0; b < kPairSBuf; ++b) {
            mbar_init(&bar.s_full[b], 1);
            mbar_init(&bar.p_full[b], 2 * 4);  // one arrival per softmax warp of each CTA
            mbar_init(&bar.s_free[b], 1);
        }
        mbar_init(&bar.o_final, 1);
        mbar_init(&bar.gate_full, 1);
        mbar_init(&bar.epi_l, 4);     // the four softmax warps
        for (int b = 0; b < kEpiBoxes; ++b)
            mbar_init(&bar.epi_box[b], 4);  // the four warps (lane quarters) that fill a box
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(&tmem_base_s, kTmemCols);
        tmem_relinquish_pair();
    }
    fence_before_sync();
    cluster_sync();  // barriers of both CTAs initialised before any remote use
    fence_after_sync();
    const uint32_t tmem = tmem_base_s;

    auto fail = [&]() {
        abort_flag = 1;
        set_error(p.err, kDevErrTimeout);
    };

    // ---------------------------------------------------------------- queries
    // The CTA's 128 query rows (f32, q half of q_and_gate) land by TMA as
    // eight 32-column boxes (128-byte swizzle): boxes 0, 1, 4, 5 over sQ and
    // 2, 3, 6, 7 in the V ring, and the RoPE angles of its positions by bulk
    // copy ([64][128]: cos of angles 0-31, then sin, each over the 128 rows).
    // Warps 1-8 prepare them, two threads per row (warps 1-4 dims 0-127,
    // warps 5-8 dims 128-255): q RMSNorm with an f32 sum of squares (the
    // reference sums in f64; these rows are rounded to bf16 for the tensor
    // cores, whose 4e-3 dwarfs the ~1e-7 difference), RoPE, and bf16 Q into
    // sQ in the SW128 K-major layout the QK MMA reads. A thread's bf16 output
    // only overwrites f32 rows that it has already read itself, so the
    // conversion needs no shared-memory hand-off beyond the two halves'
    // partial sums. The K ring is free throughout, so warp 0 streams K tiles
    // meanwhile; the V ring goes to its producer (q_conv) and the pair's Q to
    // the leader's QK issuers (q_pair) once every warp has finished.
    auto stage_box = [&](int cb) {
        return (((cb >> 1) & 1) ? sV : sQ) + ((cb & 1) + 2 * (cb >> 2)) * kEpiBoxBytes;
    };
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&map_g);
        mbar_arrive_expect_tx(&bar.q_full, kEpiBoxes * kEpiBoxBytes + (has_rows ? kRopeBlockBytes : 0u));
        for (int cb = 0; cb < kEpiBoxes; ++cb)
            tma_load_4d(stage_box(cb), &map_g, cb * kEpiBoxCols, h, q0, s, &bar.q_full);
        pdl_wait_primary();  // P1 wrote the RoPE table and the K/V rows loaded below
        if (has_rows)
            bulk_load(sT, p.rope + size_t(q0 / kBlockQ) * kRopeBlockFloats, kRopeBlockBytes, &bar.q_full);
    }
    if (warp >= 1) {
        const int quarter = warp & 3, half = warp >= 5 ? 1 : 0;
        const uint32_t r = uint32_t(quarter * 32 + lane);
        const bool ready = __all_sync(0xffffffffu, mbar_wait(&bar.q_full, 0));
        float part = 0.f;
        if (ready) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const unsigned char *row = stage_box(4 * half + k) + r * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float4 v = *reinterpret_cast<const float4 *>(row + ((c ^ (r & 7)) << 4));
                    acc[c] = fmaf(v.x, v.x, acc[c]);
                    acc[c] = fmaf(v.y, v.y, acc[c]);
                    acc[c] = fmaf(v.z, v.z, acc[c]);
                    acc[c] = fmaf(v.w, v.w, acc[c]);
                }
            }
            part = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
        }
        // Row total: half 1 hands its part to half 0, which returns the sum.
        // Both warps of a quarter reach both barriers unconditionally.
        if (half) inv_l_s[r] = part;
        named_barrier_sync(1 + quarter, 64);
        if (!half) inv_l_s[r] = part + inv_l_s[r];
        named_barrier_sync(1 + quarter, 64);
        const float sq = inv_l_s[r];
        if (ready) {
            // rmsnorm_inplace (ops.rs:493-498)
            const float scale = 1.0f / sqrtf(sq * (1.0f / kAttnHeadDim) + p.eps);
            // Rows past the prompt's end (zeros from the TMA) take the last
            // position's angles; a CTA without rows takes angle 0.
            const float *tab = reinterpret_cast<const float *>(sT) + (has_rows ? min(int(r), q_rows - 1) : 0);
#pragma unroll 1
            for (int qb = 2 * half; qb < 2 * half + 2; ++qb) {  // 64 dims: one 16 KB box of sQ
                float x[64];
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const unsigned char *row = stage_box(2 * qb + k) + r * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const float4 v = *reinterpret_cast<const float4 *>(row + ((c ^ (r & 7)) << 4));
                        x[k * 32 + 4 * c + 0] = v.x;
                        x[k * 32 + 4 * c + 1] = v.y;
                        x[k * 32 + 4 * c + 2] = v.z;
                        x[k * 32 + 4 * c + 3] = v.w;
                    }
                }
                const float4 *w4 = reinterpret_cast<const float4 *>(p.q_norm + qb * 64);
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const float4 w = __ldg(w4 + k);
                    x[4 * k + 0] = x[4 * k + 0] * scale * w.x;
                    x[4 * k + 1] = x[4 * k + 1] * scale * w.y;
                    x[4 * k + 2] = x[4 * k + 2] * scale * w.z;
                    x[4 * k + 3] = x[4 * k + 3] * scale * w.w;
                }
                if (qb == 0) {
                    // rope (ops.rs:595-610): the pair (i, i + 32) for i < 32.
#pragma unroll
                    for (int i = 0; i < kRopeHalf; ++i) {
                        const float c = has_rows ? tab[i * kBlockQ] : 1.f;
                        const float sn = has_rows ? tab[(kRopeHalf + i) * kBlockQ] : 0.f;
                        const float lo = x[i], hi = x[i + kRopeHalf];
                        x[i] = lo * c - hi * sn;
                        x[i + kRopeHalf] = lo * sn + hi * c;
                    }
                }
                unsigned char *dst = sQ + qb * (kQBytes / 4) + r * 128;
                if (p.op_f16) {
                    // f16 operands (f32 cache): the same type as the f16 K copy.
                    float qmax = 0.f;
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch) {
                        uint4 o;
                        o.x = pack_f16x2(x[8 * ch + 0], x[8 * ch + 1]);
                        o.y = pack_f16x2(x[8 * ch + 2], x[8 * ch + 3]);
                        o.z = pack_f16x2(x[8 * ch + 4], x[8 * ch + 5]);
                        o.w = pack_f16x2(x[8 * ch + 6], x[8 * ch + 7]);
                        *reinterpret_cast<uint4 *>(dst + ((ch ^ (r & 7)) << 4)) = o;
#pragma unroll
                        for (int e = 0; e < 8; ++e) qmax = fmaxf(qmax, fabsf(x[8 * ch + e]));
                    }
                    if (qmax > 65504.f) set_error(p.err, kDevErrRange);
                } else {
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch) {
                        uint4 o;
                        o.x = pack_bf16x2_rn(x[8 * ch + 0], x[8 * ch + 1]);
                        o.y = pack_bf16x2_rn(x[8 * ch + 2], x[8 * ch + 3]);
                        o.z = pack_bf16x2_rn(x[8 * ch + 4], x[8 * ch + 5]);
                        o.w = pack_bf16x2_rn(x[8 * ch + 6], x[8 * ch + 7]);
                        *reinterpret_cast<uint4 *>(dst + ((ch ^ (r & 7)) << 4)) = o;
                    }
                }
            }
            fence_proxy_async_smem();  // the QK MMA reads sQ through the async proxy
        }
        __syncwarp();
        if (lane == 0) {
            if (!ready) fail();
            mbar_arrive(&bar.q_conv);
            mbar_arrive_remote(cluster_addr(&bar.q_pair, 0));
        }
    }

    if (warp == 0) {
        // ------------------------------------------------------------ K-half producer
        if (lane == 0) {
            tma_prefetch_desc(&map_k);
            const int kplane = (p.kseq0 + s) * p.kv_heads + kvh;
            bool ok = true;
            const int gate_x = kAttnHeadDim;  // the gate half of each head's 512 values
            for (int j = 0; ok && j < nkt; ++j) {
                const int b = j % kPairStagesK;
                if (j >= kPairStagesK &&
                    !mbar_wait(&bar.k_empty[b], uint32_t(j / kPairStagesK - 1) & 1u)) {
                    ok = false;
                    break;
                }
                if (leader) mbar_arrive_expect_tx(&bar.k_full[b], 2 * kKHalf);
                const uint32_t full = cluster_addr(&bar.k_full[b], 0);
                for (int cb = 0; cb < 4; ++cb)
                    tma_load_3d_pair(sK + b * kKHalf + cb * (kKHalf / 4), &map_k, cb * 64,
                                     j * kBlockK + int(rank) * (kBlockK / 2), kplane, full);
                if (has_rows && j == max(nkt - kGatePrefetchTiles, 0))
                    for (int cb = 0; cb < kEpiBoxes; ++cb)
                        tma_prefetch_4d(&map_g, gate_x + cb * kEpiBoxCols, h, q0, s);
                if (abort_flag) { ok = false; break; }
            }
            // The gate block replaces Q and the K ring once the last two S = Q K^T
            // (one per issuing warp) have completed. Tile j's completion is phase
            // j / 4 of k_empty[j % 4], whose earlier phases this thread waited for
            // before loading tile j, so the parity waits are exact.
            for (int j = max(nkt - 2, 0); ok && j < nkt; ++j)
                if (!mbar_wait(&bar.k_empty[j % kPairStagesK], uint32_t(j / kPairStagesK) & 1u))
                    ok = false;
            if (!ok) {
                fail();
            } else if (has_rows) {
                mbar_arrive_expect_tx(&bar.gate_full, kEpiBoxes * kEpiBoxBytes);
                for (int cb = 0; cb < kEpiBoxes; ++cb)
                    tma_load_4d(smem + cb * kEpiBoxBytes, &map_g, gate_x + cb * kEpiBoxCols, h, q0, s,
                                &bar.gate_full);
            }
        }
    } else if (warp == 7) {
        // ------------------------------------------------------------ V-half producer (f16)
        if (lane == 0) {
            tma_prefetch_desc(&map_v);
            pdl_wait_primary();  // P1 wrote the V rows
            const int vplane = s * p.kv_heads + kvh;
            if (!mbar_wait(&bar.q_conv, 0)) fail();  // the V ring held query rows until now
            for (int j = 0; j < nkt && !abort_flag; ++j) {
                const int b = j % kPairStagesV;
                if (j >= kPairStagesV &&
                    !mbar_wait(&bar.v_empty[b], uint32_t(j / kPairStagesV - 1) & 1u)) {
                    fail();
                    break;
                }
                if (leader) mbar_arrive_expect_tx(&bar.v_full[b], 2 * kVHalf);
                const uint32_t full = cluster_addr(&bar.v_full[b], 0);
                for (int cb = 0; cb < 2; ++cb)
                    tma_load_3d_pair(sV + b * kVHalf + cb * (kVHalf / 2), &map_v,
                                     int(rank) * (kAttnHeadDim / 2) + cb * 64, j * kBlockK, vplane,
                                     full);
            }
        }
    } else if (warp == 1 || warp == 8) {
        // ------------------------------------------------------------ S = Q K^T issuers (leader)
        // A thread issuing tcgen05.mma waits ~100 cycles per instruction, so
        // even and odd tiles are issued from two warps.
        if (leader && lane == 0) {
            // Q and K: both bf16 (bf16 cache) or both f16 (f32 cache).
            const uint32_t id_qk = idesc_f16_f32(kPairRows, kBlockK, 0, 0, p.op_f16 == 0);
            const uint32_t sq = smem_addr(sQ), sk = smem_addr(sK);
            bool ok = mbar_wait_cluster(&bar.q_pair, 0);  // Q of both CTAs in shared memory
            for (int j = warp == 1 ? 0 : 1; ok && j < nkt; j += 2) {
                const int b = j % kPairSBuf, kb = j % kPairStagesK;
                if (!mbar_wait(&bar.k_full[kb], uint32_t(j / kPairStagesK) & 1u)) { ok = false; break; }
                // S buffer b held S and P of tile j-4 until PV(j-4) completed.
                if (j >= kPairSBuf && !mbar_wait(&bar.s_free[b], uint32_t(j / kPairSBuf - 1) & 1u)) {
                    ok = false;
                    break;
                }
                fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < kAttnHeadDim / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * (kQBytes / 4) + (kk & 3) * 32;
                    const uint64_t ad = smem_desc_sw128(sq + off, 16, 1024);
                    const uint64_t bd = smem_desc_sw128(
                        sk + kb * kKHalf + (kk >> 2) * (kKHalf / 4) + (kk & 3) * 32, 16, 1024);
                    mma_pair_ss(tmem + b * kBlockK, ad, bd, id_qk, kk > 0 ? 1u : 0u);
                }
                mma_commit_pair(&bar.s_full[b]);
                mma_commit_pair(&bar.k_empty[kb]);
                if (abort_flag) { ok = false; break; }
            }
            if (!ok) fail();
        }
    } else if (warp == 6) {
        // ------------------------------------------------------------ O += P V issuer (leader)
        if (leader && lane == 0) {
            const uint32_t id_pv = idesc_f16_f32(kPairRows, kAttnHeadDim, 0, 1, false);
            const uint32_t sv = smem_addr(sV);
            bool ok = true;
            for (int j = 0; j < nkt; ++j) {
                const int b = j % kPairSBuf, vb = j % kPairStagesV;
                if (!mbar_wait(&bar.p_full[b], uint32_t(j / kPairSBuf) & 1u)) { ok = false; break; }
                if (!mbar_wait(&bar.v_full[vb], uint32_t(j / kPairStagesV) & 1u)) { ok = false; break; }
                fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < kBlockK / 16; ++kk) {
                    const uint64_t bd =
                        smem_desc_sw128(sv + vb * kVHalf + kk * 2048, kVHalf / 2, 1024);
                    // P(j): f16 pairs in the first 32 columns of S buffer b.
                    mma_pair_ta(tmem + kPairColO, tmem + b * kBlockK + kk * 8, bd, id_pv,
                                (j > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit_pair(&bar.v_empty[vb]);
                mma_commit_pair(&bar.s_free[b]);
                if (abort_flag) { ok = false; break; }
            }
            // One completion for the epilogue, after the last PV.
            if (ok) mma_commit_pair(&bar.o_final);
            if (!ok) fail();
        }
    } else {
        // ------------------------------------------------------------ softmax (both CTAs)
        // tcgen05.ld/st are warp-collective: every decision that guards one is
        // made uniform across the warp.
        const int sub = warp & 3;
        const int r = sub * 32 + lane;
        const uint32_t lane_addr = uint32_t(sub * 32) << 16;
        const int t = q0 + r;
        const int qpos = p.base + min(t, p.count - 1);  // rows past the end mirror the last
        const int qpos_first = p.base + min(q0, p.count - 1);
        const float sl2 = 1.4426950408889634f / 16.0f;  // log2(e) * score_scale
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        auto wait_all = [&](uint64_t *b, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(b, parity));
        };
        for (int j = 0; ok && j < nkt; ++j) {
            const int b = j % kPairSBuf;
            if (!wait_all(&bar.s_full[b], uint32_t(j / kPairSBuf) & 1u)) { ok = false; break; }
            fence_after_sync();
            uint32_t sr[2][32];
            tmem_ld32(tmem + lane_addr + b * kBlockK, sr[0]);
            tmem_ld32(tmem + lane_addr + b * kBlockK + 32, sr[1]);
            tmem_wait_ld();
            float sv[kBlockK];
            const int key0 = j * kBlockK;
            float mx8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
            if (key0 + kBlockK - 1 <= qpos_first) {
#pragma unroll
                for (int c = 0; c < kBlockK; ++c) {
                    sv[c] = __uint_as_float(sr[c >> 5][c & 31]);
                    mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < kBlockK; ++c) {
                    const float v = __uint_as_float(sr[c >> 5][c & 31]);
                    sv[c] = (key0 + c <= qpos) ? v : -INFINITY;
                    mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
                }
            }
            const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            const float m_new = fmaxf(m, mx * sl2);
            if (__any_sync(0xffffffffu, m_new > m + kRescaleThreshold)) {
                const float corr = ex2(m - m_new);  // 0 on the first tile
                if (j > 0) {
                    // O holds PV(0..j-1). PV(j-1) completing is phase (j-1)/4 of
                    // s_free[(j-1)%4]; that barrier is at most one phase behind
                    // (QK(j-1) needed PV(j-5)) and cannot be ahead (PV(j+3) needs
                    // P(j+3)), so the parity wait is exact. PVs complete in order.
                    const int jp = j - 1;
                    if (!wait_all(&bar.s_free[jp % kPairSBuf], uint32_t(jp / kPairSBuf) & 1u)) {
                        ok = false;
                        break;
                    }
                    fence_after_sync();
#pragma unroll 1
                    for (int c = 0; c < kAttnHeadDim; c += 32) {
                        uint32_t o[32];
                        tmem_ld32(tmem + lane_addr + kPairColO + c, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
                        tmem_st32(tmem + lane_addr + kPairColO + c, o);
                    }
                }
                l *= corr;
                m = m_new;
            }
            // P = 2^(s*sl2 - m) as f16 pairs over the first 32 columns of S
            // buffer b (S is in registers now). Masked scores give exactly 0.
            uint32_t pw[32];
            float2 ps2[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) ps2[i] = make_float2(0.f, 0.f);
            const float2 scale2 = make_float2(sl2, sl2), negm2 = make_float2(-m, -m);
#pragma unroll
            for (int c = 0; c < kBlockK / 2; ++c) {
                const float2 x = ffma2(make_float2(sv[2 * c], sv[2 * c + 1]), scale2, negm2);
                const float2 pr = make_float2(ex2(x.x), ex2(x.y));
                ps2[c & 3] = fadd2(ps2[c & 3], pr);
                pw[c] = pack_f16x2(pr.x, pr.y);
            }
            tmem_st32(tmem + lane_addr + b * kBlockK, pw);
            l += ((ps2[0].x + ps2[0].y) + (ps2[1].x + ps2[1].y)) +
                 ((ps2[2].x + ps2[2].y) + (ps2[3].x + ps2[3].y));
            tmem_wait_st();
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive_leader(cluster_addr(&bar.p_full[b], 0));
            if (__any_sync(0xffffffffu, abort_flag != 0)) { ok = false; break; }
        }
        // Publish 1/l for the epilogue warps that do not hold it.
        if (ok) {
            inv_l_s[r] = 1.0f / l;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar.epi_l);
        } else if (lane == 0) {
            fail();
        }
    }
    __syncwarp();

    // ---------------------------------------------------------------- epilogue
    // Warps 0-7 (TMEM lane quarter warp % 4; warps 2-5 columns 0-127, the
    // others 128-255): out = O / l * sigmoid(gate) in place over the staged
    // gate block, one 32-column box at a time; warp 8 stores each box by TMA
    // as soon as its four warps have filled it.
    if (warp < 8 && has_rows) {
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const int cb0 = (warp >= 2 && warp <= 5) ? 0 : kEpiBoxes / 2;
        auto wait_all = [&](uint64_t *b, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(b, parity));
        };
        const bool ready =
            wait_all(&bar.o_final, 0) && wait_all(&bar.epi_l, 0) && wait_all(&bar.gate_full, 0);
        if (ready) fence_after_sync();
        else if (lane == 0) fail();
        const float inv_l = inv_l_s[r];
        const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
#pragma unroll 1
        for (int cb = cb0; cb < cb0 + kEpiBoxes / 2; ++cb) {
            if (ready) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_addr + kPairColO + cb * kEpiBoxCols, o);
                tmem_wait_ld();
                unsigned char *row = smem + cb * kEpiBoxBytes + r * 128;
#pragma unroll
                for (int c = 0; c < kEpiBoxCols / 4; ++c) {
                    float4 *pg = reinterpret_cast<float4 *>(row + ((c ^ (r & 7)) << 4));
                    const float4 g = *pg;
                    float4 y;
                    y.x = __uint_as_float(o[4 * c + 0]) * inv_l * sigmoid_fast(g.x);
                    y.y = __uint_as_float(o[4 * c + 1]) * inv_l * sigmoid_fast(g.y);
                    y.z = __uint_as_float(o[4 * c + 2]) * inv_l * sigmoid_fast(g.z);
                    y.w = __uint_as_float(o[4 * c + 3]) * inv_l * sigmoid_fast(g.w);
                    *pg = y;
                }
                fence_proxy_async_smem();  // the TMA store reads these writes
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar.epi_box[cb]);
        }
    } else if (warp == 8 && has_rows && lane == 0) {
        // Boxes complete in the order 0, 4, 1, 5, ... (two warps per quarter).
        bool ok = true;
        for (int k = 0; k < kEpiBoxes; ++k) {
            const int cb = (k & 1) * (kEpiBoxes / 2) + (k >> 1);
            if (!mbar_wait(&bar.epi_box[cb], 0)) {
                ok = false;
                break;
            }
            if (abort_flag) break;
            tma_store_4d(&map_o, cb * kEpiBoxCols, h, q0, s, smem + cb * kEpiBoxBytes);
            bulk_commit_group();
        }
        if (!ok) fail();
        bulk_wait_group_read0();  // shared memory stays valid until the stores have read it
    }

    fence_before_sync();
    cluster_sync();  // no CTA leaves while the pair's MMAs may use its memory
    fence_after_sync();
    if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// 3-D map of 16-bit elements over [planes][rows][256] with a box of
// 64 x box_rows x 1 and 128-byte swizzle.
bool make_map_16(CUtensorMap *m, const void *base, CUtensorMapDataType type, uint64_t rows,
                 uint64_t planes, uint32_t box_rows) {
    auto enc = encode_tiled();
    if (!enc) return false;
    cuuint64_t dims[3] = {uint64_t(kAttnHeadDim), rows, planes};
    cuuint64_t strides[2] = {uint64_t(kAttnHeadDim) * 2, uint64_t(kAttnHeadDim) * 2 * rows};
    cuuint32_t box[3] = {64, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, type, 3, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D map of f32 over [nseq][count][heads][width] (row stride `width`) with a
// box of 32 x 1 x 128 x 1 and 128-byte swizzle: the gate half of q_and_gate
// (width 512) for loads, the attention output (width 256) for stores. Rows
// past `count` fall outside the map, so loads read zeros and stores skip them.
bool make_map_rows_f32(CUtensorMap *m, const void *base, uint64_t width, uint64_t heads,
                       uint64_t count, uint64_t nseq) {
    auto enc = encode_tiled();
    if (!enc) return false;
    cuuint64_t dims[4] = {width, heads, count, nseq};
    cuuint64_t strides[3] = {width * 4, width * 4 * heads, width * 4 * heads * count};
    cuuint32_t box[4] = {uint32_t(kEpiBoxCols), 1, uint32_t(kBlockQ), 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void *>(base), dims, strides, box,
               es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t attn_prefill_rope_floats(int max_tokens) {
    return size_t((max_tokens + kBlockQ - 1) / kBlockQ) * kRopeBlockFloats;
}

cudaError_t launch_attn_prefill(const AttnPrefillLaunch &a, cudaStream_t stream) {
    cudaError_t e;
    const int nkvh = a.kv_head_count;
    if (nkvh <= 0 || nkvh > kPrepWarps || a.kv_head0 < 0 || a.kv_head0 + nkvh > a.kv_heads ||
        (a.kv_f32 && !a.k16))
        return cudaErrorInvalidValue;
    if (a.base > 0) {
        PrefixParams xp{a.kcache, a.vcache, a.v16, a.k16, a.err, a.seq0, a.base, a.context_length,
                        a.kv_heads, a.kv_head0, a.kv_f32};
        const int n8 = a.base * (kAttnHeadDim / 8);
        attn_prefill_prefix_kernel<<<dim3((n8 + 255) / 256, nkvh, a.nseq), 256, 0, stream>>>(xp);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    PrefillPrepParams pp{a.key,  a.value, a.kcache, a.vcache, a.v16, a.k16,
                         a.rope, a.k_norm, a.err,   a.seq0,   a.count, a.base,
                         a.context_length, a.kv_heads, a.kv_head0, nkvh, a.kv_f32,
                         a.theta_scale, a.eps};
    const int prep_tokens = kPrepWarps / nkvh;
    attn_prefill_prep_kernel<<<dim3((a.count + prep_tokens - 1) / prep_tokens, a.nseq),
                               kPrepWarps * 32, 0, stream>>>(pp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    CUtensorMap mk, mv, mg, mo;
    if (!make_map_rows_f32(&mg, a.q_and_gate, 2 * kAttnHeadDim, uint64_t(a.heads), uint64_t(a.count),
                           uint64_t(a.nseq)) ||
        !make_map_rows_f32(&mo, a.attention, kAttnHeadDim, uint64_t(a.heads), uint64_t(a.count),
                           uint64_t(a.nseq)) ||
        // Q K^T reads the bf16 cache itself, or (f32 cache) the f16 K scratch.
        !make_map_16(&mk, a.kv_f32 ? static_cast<void *>(a.k16) : a.kcache,
                     a.kv_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                     uint64_t(a.context_length),
                     uint64_t(a.kv_f32 ? a.nseq : a.batch) * a.kv_heads, kBlockK / 2) ||
        !make_map_16(&mv, a.v16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, uint64_t(a.context_length),
                     uint64_t(a.nseq) * a.kv_heads, kBlockK))
        return cudaErrorInvalidValue;

    const int n_qtiles = (a.count + kBlockQ - 1) / kBlockQ;
    const int n_pairs = (n_qtiles + 1) / 2;
    PrefillParams p{a.q_norm, a.rope, a.err, a.kv_f32 ? 0 : a.seq0, a.count, a.base,
                    kGroup * a.kv_head0, a.kv_heads, n_qtiles, a.kv_f32, a.eps};
    e = cudaFuncSetAttribute(attn_prefill_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(kSmemPair));
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * n_pairs, kGroup * nkvh, a.nseq);
    cfg.blockDim = dim3(kThreadsPF);
    cfg.dynamicSmemBytes = kSmemPair;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_prefill_pair_kernel, mk, mv, mg, mo, p);
}

}  // namespace q38
