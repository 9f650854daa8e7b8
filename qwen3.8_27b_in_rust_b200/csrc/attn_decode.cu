// attn_decode.cu -- gated full-attention decode (full_core, src/model/ops.rs:812-940)
// as three stream-ordered kernels chained with programmatic dependent launch:
//
//   K1 attn_decode_prep   one CTA per (head, sequence): split q/gate, q/k RMSNorm
//                         (f64 sum, ops.rs:476-498), partial RoPE with the
//                         iterative f32 angle (ops.rs:595-610), KV append at
//                         the sequence's position (ops.rs:858-866).
//   K2 attn_decode_split  one CTA per (split, kv head, sequence): flash-decoding
//                         over a contiguous range of cached positions. KV tiles
//                         of 32 KB are staged global->shared by the bulk-copy
//                         engine (cp.async.bulk + mbarrier, 3-deep ring). The 6
//                         query heads of the GQA group share every tile. Pass 1
//                         computes scores for the split (q in registers, FFMA2,
//                         warp-shuffle transpose-reduce); per-head max and
//                         exp-sum follow; pass 2 accumulates exp(s-m)*V.
//                         Writes the partial (m, l, o) triple per head.
//   K3 attn_decode_merge  one CTA per (head, sequence): LSE merge of the split
//                         partials, normalisation and the sigmoid output gate
//                         (ops.rs:915-919).
//
// HBM layout of one KV slot: [batch][kv_heads][context_length][256] in f32 or
// bf16, so a split's range of one kv head is one contiguous byte range.
#include "q38_common.cuh"
#include "q38_sm100.cuh"

#include <cudaTypedefs.h>

#include <algorithm>

namespace q38 {
namespace {

constexpr int kThreads = 256;      // 8 warps
constexpr int kWarps = kThreads / 32;
constexpr int kTileBytes = 32768;  // one staged KV tile
constexpr int kMaxChunk = 4096;    // positions per split (scores smem: chunk*32 B)
constexpr int kMaxChunkTc = 2048;  // bf16 (tensor-core) splits also stage P: chunk*64 B
constexpr int kFastChunk = 512;    // largest chunk that keeps 2 CTAs per SM (112 KB smem)
constexpr int kMinSplitsCap = 128;

template <typename KV>
struct Tile {
    static constexpr int kPositions = kTileBytes / (kAttnHeadDim * int(sizeof(KV)));  // 64 | 32
    static constexpr int kPerWarp = kPositions / kWarps;                             // 8 | 4
    // Ring depth: the bf16 kernel also holds its tensor-core query operand, so
    // two stages keep it at two CTAs per SM.
    static constexpr int kStages = sizeof(KV) == 2 ? 2 : 3;
};

// bf16 scores on tcgen05: per 64-key tile S^T = K Q^T as an M=64, N=16, K=256
// MMA (6 query heads in B rows 0-5), with the f32 queries split into bf16
// (hi, lo) pairs (two products into separate TMEM columns). Shared memory:
// the query operand after the scores, 4 SW128 boxes of 8 rows (rows 6-7 zero;
// the MMA also reads rows 8-15, the next kilobyte, whose columns are unused)
// for hi and for lo, then 1 KB of padding.
constexpr uint32_t kQOperandBytes = 4 * 1024;
constexpr uint32_t kQRegionBytes = 2 * kQOperandBytes + 1024;
constexpr uint32_t kDecodeTmemCols = 256;  // 32 columns (hi | lo) per tile, 8 tiles in turn

__host__ __device__ inline int tile_positions(int kv_dtype) {
    return kv_dtype == Q38_KV_BF16 ? 64 : 32;
}

// ----------------------------------------------------------------------------
// K1: prep
// ----------------------------------------------------------------------------
struct PrepParams {
    const float *q_and_gate;
    float *key;
    const float *value;
    const int32_t *positions;
    void *kcache, *vcache;
    float *qprep;
    int *err;
    const float *q_norm, *k_norm;
    int context_length, heads, kv_heads, max_position, pos_offset, sharded;
    float theta_scale, eps;
    uint32_t *p2p_epoch;  // peer-memory exchange: the call counter this kernel advances, or null
};

// A sequence at global position pos appends its K/V row at local cache row
// pos - pos_offset (pos_offset is 0 unless the sequence's positions are
// sharded across GPUs); RoPE always uses the global position. Unsharded, a
// position outside the cache is an error; sharded, a position past this
// shard's range only means the shard contributes all its rows and appends
// nothing.
__device__ __forceinline__ bool position_ok(int pos, int pos_offset, int context_length,
                                            int max_position, int sharded) {
    if (pos < 0 || pos > max_position) return false;
    return sharded || pos - pos_offset < context_length;
}

template <typename KV>
__global__ void __launch_bounds__(kAttnHeadDim) attn_decode_prep_kernel(PrepParams p) {
    // Launched as a programmatic dependent so that it is resident when the
    // previous kernel ends; nothing is read or written before that kernel has
    // completed.
    pdl_wait_primary();
    pdl_launch_dependents();
    // This call's exchange epoch: the previous call's merge, the last reader
    // of the counter, has finished; this call's merge reads it after waiting
    // for the split kernel, which waited for this kernel.
    if (p.p2p_epoch && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *p.p2p_epoch += 1u;
    __shared__ double red[32];
    __shared__ float cs[32], sn[32];
    __shared__ float xs[kAttnHeadDim];
    const int h = blockIdx.x, b = blockIdx.y, i = threadIdx.x;
    const int pos = p.positions[b];
    if (!position_ok(pos, p.pos_offset, p.context_length, p.max_position, p.sharded)) {
        if (h == 0 && i == 0) set_error(p.err, kDevErrPosition);
        return;
    }
    // Local row of the new K/V; outside [0, context_length) another shard owns it.
    const int row_local = pos - p.pos_offset;
    const bool is_q = h < p.heads;
    const int kvh = h - p.heads;
    float x = is_q ? p.q_and_gate[(size_t(b) * p.heads + h) * 2 * kAttnHeadDim + i]
                   : p.key[(size_t(b) * p.kv_heads + kvh) * kAttnHeadDim + i];
    // rmsnorm_inplace (ops.rs:493-498) with rms_scale's f64 accumulation.
    const double sum = block_sum_f64(double(x) * double(x), red);
    const float scale = rms_scale_from_sum(sum, kAttnHeadDim, p.eps);
    x = x * scale * (is_q ? p.q_norm[i] : p.k_norm[i]);
    // rope (ops.rs:595-610): theta_j = pos * scale^j by repeated f32 products.
    if (i < kRopeDims / 2) {
        float theta = float(pos);
        for (int j = 0; j < i; ++j) theta *= p.theta_scale;
        cs[i] = cosf(theta);
        sn[i] = sinf(theta);
    }
    xs[i] = x;
    __syncthreads();
    if (i < kRopeDims / 2) {
        x = xs[i] * cs[i] - xs[i + kRopeDims / 2] * sn[i];
    } else if (i < kRopeDims) {
        const int j = i - kRopeDims / 2;
        x = xs[j] * sn[j] + xs[i] * cs[j];
    }
    if (is_q) {
        p.qprep[(size_t(b) * p.heads + h) * kAttnHeadDim + i] = x;
    } else {
        const size_t kv_off = (size_t(b) * p.kv_heads + kvh) * kAttnHeadDim + i;
        p.key[kv_off] = x;
        if (row_local >= 0 && row_local < p.context_length) {
            const size_t row =
                ((size_t(b) * p.kv_heads + kvh) * p.context_length + row_local) * kAttnHeadDim + i;
            static_cast<KV *>(p.kcache)[row] = KvTraits<KV>::store(x);
            static_cast<KV *>(p.vcache)[row] = KvTraits<KV>::store(p.value[kv_off]);
        }
    }
}

// ----------------------------------------------------------------------------
// K2: split-KV attention
// ----------------------------------------------------------------------------
struct SplitParams {
    const void *kcache, *vcache;
    const float *qprep;
    const int32_t *positions;
    float *part_o, *part_ml;
    int *err;
    int context_length, heads, kv_heads, chunk, max_splits, max_position, pos_offset, sharded;
    uint64_t wait_ns;  // limit of every bounded wait
    int skip_loads;    // error-path testing: issue no KV loads (every wait runs out)
};

// Rows of the local cache a sequence at global position pos attends to.
__device__ __forceinline__ int local_rows(int pos, int pos_offset, int context_length) {
    return min(pos - pos_offset + 1, context_length);
}

// Dimension of the head that slot j (0..7) of lane `lane` owns. bf16 rows are
// 512 B: lane l owns dims [8l, 8l+8), one 16-byte load. f32 rows are 1 KB:
// lane l owns [4l, 4l+4) and [128+4l, 128+4l+4), two conflict-free 16-byte loads.
template <typename KV>
__device__ __forceinline__ int lane_dim(int lane, int j) {
    if constexpr (sizeof(KV) == 2) {
        return 8 * lane + j;
    } else {
        return j < 4 ? 4 * lane + j : 128 + 4 * lane + (j - 4);
    }
}

// Loads the 8 elements of row `row` (a smem pointer to 256 elements) that
// this lane owns, as 4 float pairs.
template <typename KV>
__device__ __forceinline__ void load_row8(const unsigned char *row, int lane, float2 (&v)[4]) {
    if constexpr (sizeof(KV) == 2) {
        const uint4 w = *reinterpret_cast<const uint4 *>(row + lane * 16);
        v[0] = bf16x2_to_float2(w.x);
        v[1] = bf16x2_to_float2(w.y);
        v[2] = bf16x2_to_float2(w.z);
        v[3] = bf16x2_to_float2(w.w);
    } else {
        const float4 a = *reinterpret_cast<const float4 *>(row + lane * 16);
        const float4 c = *reinterpret_cast<const float4 *>(row + 512 + lane * 16);
        v[0] = make_float2(a.x, a.y);
        v[1] = make_float2(a.z, a.w);
        v[2] = make_float2(c.x, c.y);
        v[3] = make_float2(c.z, c.w);
    }
}

// One halving step of the transpose-reduce: lanes whose `mask` bit is set keep
// the upper half of the array, the others the lower half; each adds its
// partner's copy of the half it keeps.
template <int N>
__device__ __forceinline__ void halve(const float (&in)[N], float (&out)[N / 2], int lane,
                                      int mask) {
    const bool up = (lane & mask) != 0;
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
        const float keep = up ? in[N / 2 + i] : in[i];
        const float send = up ? in[i] : in[N / 2 + i];
        out[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
    }
}

// Reduces part[P][6] over the 32 lanes. On return the lane holds the totals
// of position *pp and heads *h0..*h0+2, and *writer says whether it is the
// lane that stores them.
template <int P>
__device__ __forceinline__ void transpose_reduce(const float (&part)[P * kGroup], int lane,
                                                 float (&tot)[3], int *pp, int *h0,
                                                 bool *writer) {
    static_assert(P == 8 || P == 4, "positions per warp");
    if constexpr (P == 8) {
        float a[24], b[12], c[6];
        halve<48>(part, a, lane, 16);
        halve<24>(a, b, lane, 8);
        halve<12>(b, c, lane, 4);
        halve<6>(c, tot, lane, 2);
#pragma unroll
        for (int i = 0; i < 3; ++i) tot[i] += __shfl_xor_sync(0xffffffffu, tot[i], 1);
        *pp = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
        *h0 = ((lane >> 1) & 1) * 3;
        *writer = (lane & 1) == 0;
    } else {
        float a[12], c[6];
        halve<24>(part, a, lane, 16);
        halve<12>(a, c, lane, 8);
        halve<6>(c, tot, lane, 4);
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            tot[i] += __shfl_xor_sync(0xffffffffu, tot[i], 2);
            tot[i] += __shfl_xor_sync(0xffffffffu, tot[i], 1);
        }
        *pp = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
        *h0 = ((lane >> 2) & 1) * 3;
        *writer = (lane & 3) == 0;
    }
}

// Scores of this warp's kPerWarp positions (rows [pl0, pl0+kPerWarp) of the
// tile) for the 6 heads, reduced over the warp; written to scores[][8].
template <typename KV, bool kFull>
__device__ __forceinline__ void score_rows(const unsigned char *tile, int rows, int pl0, int lane,
                                           const float2 (&q2)[kGroup][4], float *score_rows_out,
                                           float score_scale) {
    using T = Tile<KV>;
    constexpr int kRowBytes = kAttnHeadDim * int(sizeof(KV));
    float part[T::kPerWarp * kGroup];
#pragma unroll
    for (int pp = 0; pp < T::kPerWarp; ++pp) {
        float2 k2[4];
        if (kFull || pl0 + pp < rows) {
            load_row8<KV>(tile + (pl0 + pp) * kRowBytes, lane, k2);
        } else {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) k2[jj] = make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            float2 d = make_float2(0.f, 0.f);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) d = ffma2(q2[h][jj], k2[jj], d);
            part[pp * kGroup + h] = d.x + d.y;
        }
    }
    float tot[3];
    int pp, h0;
    bool writer;
    transpose_reduce<T::kPerWarp>(part, lane, tot, &pp, &h0, &writer);
    if (writer && (kFull || pl0 + pp < rows)) {
        float *dst = score_rows_out + (pl0 + pp) * 8 + h0;
#pragma unroll
        for (int i = 0; i < 3; ++i) dst[i] = tot[i] * score_scale;
    }
}

// acc[h] += e[pos][h] * V[pos] over this warp's kPerWarp rows of the tile.
template <typename KV, bool kFull>
__device__ __forceinline__ void accumulate_rows(const unsigned char *tile, int rows, int pl0,
                                                int lane, const float *e_rows,
                                                float2 (&acc)[kGroup][4]) {
    using T = Tile<KV>;
    constexpr int kRowBytes = kAttnHeadDim * int(sizeof(KV));
#pragma unroll
    for (int pp = 0; pp < T::kPerWarp; ++pp) {
        if (kFull || pl0 + pp < rows) {
            float2 v2[4];
            load_row8<KV>(tile + (pl0 + pp) * kRowBytes, lane, v2);
            const float4 *e4 = reinterpret_cast<const float4 *>(e_rows + (pl0 + pp) * 8);
            const float4 ea = e4[0], eb = e4[1];
            const float e[kGroup] = {ea.x, ea.y, ea.z, ea.w, eb.x, eb.y};
#pragma unroll
            for (int h = 0; h < kGroup; ++h) {
                const float2 ee = make_float2(e[h], e[h]);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) acc[h][jj] = ffma2(ee, v2[jj], acc[h][jj]);
            }
        }
    }
}

template <typename KV>
__global__ void __launch_bounds__(kThreads, 2)
    attn_decode_split_kernel(const __grid_constant__ CUtensorMap map_k,
                             const __grid_constant__ CUtensorMap map_v, SplitParams p) {
    using T = Tile<KV>;
    constexpr int kStages = T::kStages;
    constexpr bool kTc = sizeof(KV) == 2;  // scores on the tensor cores
    constexpr int kRowBytes = kAttnHeadDim * int(sizeof(KV));
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *stage = smem;                                             // kStages * 32 KB
    float *scores = reinterpret_cast<float *>(smem + kStages * kTileBytes);  // [chunk][8]
    unsigned char *qsm = smem + kStages * kTileBytes + size_t(p.chunk) * 8 * sizeof(float);
    unsigned char *psm = qsm + kQRegionBytes;  // bf16: P (hi, lo) operand of the PV MMAs
    __shared__ uint64_t bars[kStages];
    __shared__ uint64_t mma_done[kStages], read_done[kStages], pv_final;
    __shared__ int issued_s;  // tiles issued so far (thread 0 issues them all)
    __shared__ uint32_t tmem_base_s;
    __shared__ float ml_s[kGroup][2];
    __shared__ volatile int abort_flag;

    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = p.positions[b];
    if (!position_ok(pos, p.pos_offset, p.context_length, p.max_position, p.sharded)) return;
    const int n = local_rows(pos, p.pos_offset, p.context_length);
    const int start = split * p.chunk;
    if (start >= n) return;
    const int cnt = min(n, start + p.chunk) - start;
    const int ntiles = (cnt + T::kPositions - 1) / T::kPositions;
    const int total_tiles = 2 * ntiles;

    const size_t head_base = (size_t(b) * p.kv_heads + kvh) * p.context_length + start;
    const unsigned char *kbase =
        static_cast<const unsigned char *>(p.kcache) + head_base * kRowBytes;
    const unsigned char *vbase =
        static_cast<const unsigned char *>(p.vcache) + head_base * kRowBytes;

    // Tile j < ntiles is K tile j, tile j >= ntiles is V tile j - ntiles.
    auto tile_rows = [&](int j) {
        const int t = j < ntiles ? j : j - ntiles;
        return min(T::kPositions, cnt - t * T::kPositions);
    };
    auto issue = [&](int j) {
        const int t = j < ntiles ? j : j - ntiles;
        if (p.skip_loads) return;  // nothing in flight: every wait on this tile runs out
        issued_s = j + 1;
        if (kTc) {
            // K or V tile as an SW128 MMA operand (K-major A of the scores, MN-major
            // A of P V): 4 boxes of 64 dims; rows past the cache's end read as zeros.
            mbar_arrive_expect_tx(&bars[j % kStages], kTileBytes);
            for (int bx = 0; bx < 4; ++bx)
                sm100::tma_load_3d(stage + (j % kStages) * kTileBytes + bx * (kTileBytes / 4),
                                   j < ntiles ? &map_k : &map_v, bx * 64, start + t * T::kPositions,
                                   b * p.kv_heads + kvh, &bars[j % kStages]);
            return;
        }
        const unsigned char *src = (j < ntiles ? kbase : vbase) + size_t(t) * kTileBytes;
        const uint32_t bytes = uint32_t(tile_rows(j)) * kRowBytes;
        mbar_arrive_expect_tx(&bars[j % kStages], bytes);
        bulk_load(stage + (j % kStages) * kTileBytes, src, bytes, &bars[j % kStages]);
    };
    // Waits for tile j; false (and the CTA-wide abort flag set) on timeout.
    auto wait_tile = [&](int j) {
        if (!mbar_wait_ns(&bars[j % kStages], uint32_t(j / kStages) & 1u, p.wait_ns)) {
            abort_flag = 1;
            set_error(p.err, kDevErrTimeout);
        }
    };
    // After every thread is done with tile j's stage: refill it with tile j+kStages.
    auto release = [&](int j) {
        __syncthreads();
        if (threadIdx.x == 0 && !abort_flag && j + kStages < total_tiles) issue(j + kStages);
    };

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars[s], 1);
            mbar_init(&mma_done[s], 2);  // one commit per issuing warp
            mbar_init(&read_done[s], 4);  // the four reader warps
        }
        mbar_init(&pv_final, 2);  // the two P V chains
        issued_s = 0;
        fence_barrier_init();
    }
    if (kTc && warp == 0) {
        sm100::tmem_alloc(&tmem_base_s, kDecodeTmemCols);
        sm100::tmem_relinquish();
    }
    sm100::fence_before_sync();
    __syncthreads();
    sm100::fence_after_sync();
    // K1 triggers this launch only after its own wait on the kernel before it,
    // so everything before K1 has completed, and K1 writes only the
    // sequence's new KV row, local row pos - pos_offset, and the prepared
    // queries. A split whose rows end before that row fetches its first tiles
    // now, while K1 runs; the split holding it waits first.
    const int new_row = pos - p.pos_offset;
    const bool early = new_row >= p.context_length || start + cnt <= new_row;
    if (early && threadIdx.x == 0) {
        for (int j = 0; j < kStages && j < total_tiles; ++j) issue(j);
    }
    pdl_wait_primary();
    if (!early && threadIdx.x == 0) {
        for (int j = 0; j < kStages && j < total_tiles; ++j) issue(j);
    }
    const float score_scale = 1.0f / sqrtf(float(kAttnHeadDim));  // ops.rs:873
    const int pl0 = warp * T::kPerWarp;
    int next = 0;  // first tile not yet waited for

    // Pass 1: scores of the split's positions for the 6 heads of the group.
    if constexpr (kTc) {
        using namespace sm100;
        const uint32_t tmem = tmem_base_s;
        // Queries as bf16 (hi, lo) pairs, B operand rows 0-5; thread = (row
        // tid / 32, 8 dims); rows 6-7 and the padding are zero.
        {
            const int h = threadIdx.x >> 5, c8 = threadIdx.x & 31;
            uint4 hq = make_uint4(0u, 0u, 0u, 0u), lq = hq;
            if (h < kGroup) {
                const float4 *q4 = reinterpret_cast<const float4 *>(
                    p.qprep + ((size_t(b) * p.heads + size_t(kvh) * kGroup + h) * kAttnHeadDim + 8 * c8));
                const float4 a = q4[0], c = q4[1];
                const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    hw[i] = pack_bf16x2_rn(v[2 * i], v[2 * i + 1]);
                    const float2 hf = bf16x2_to_float2(hw[i]);
                    lw[i] = pack_bf16x2_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
                }
                hq = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                lq = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
            const uint32_t off = (c8 >> 3) * 1024 + h * 128 + (((c8 & 7) ^ h) << 4);
            *reinterpret_cast<uint4 *>(qsm + off) = hq;
            *reinterpret_cast<uint4 *>(qsm + kQOperandBytes + off) = lq;
            if (threadIdx.x < 64)
                reinterpret_cast<uint4 *>(qsm + 2 * kQOperandBytes)[threadIdx.x] = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (warp == 5 || warp == 6) {
            // MMA issuers (a thread issuing tcgen05.mma waits ~100 cycles per
            // instruction, so the hi and lo products come from two warps):
            // S^T of tile j into TMEM columns 32 (j % 8) (hi, warp 5) and
            // 32 (j % 8) + 16 (lo, warp 6). Tile j's load follows the readout
            // of tile j - kStages by every reader, so columns are never
            // overwritten unread.
            if (lane == 0) {
                const uint32_t idesc = idesc_bf16_f32(64, 16, 0, 0);
                const int part = warp - 5;  // 0: hi, 1: lo
                const uint32_t qx = smem_addr(qsm) + part * kQOperandBytes;
                for (int j = 0; j < ntiles; ++j) {
                    if (!mbar_wait_ns(&bars[j % kStages], uint32_t(j / kStages) & 1u, p.wait_ns)) {
                        abort_flag = 1;
                        set_error(p.err, kDevErrTimeout);
                        break;
                    }
                    fence_after_sync();
                    const uint32_t ks = smem_addr(stage + (j % kStages) * kTileBytes);
#pragma unroll
                    for (int kk = 0; kk < kAttnHeadDim / 16; ++kk) {
                        const uint64_t ad =
                            smem_desc_sw128(ks + (kk >> 2) * (kTileBytes / 4) + (kk & 3) * 32, 16, 1024);
                        const uint32_t boff = (kk >> 2) * 1024 + (kk & 3) * 32;
                        mma_bf16(tmem + 32 * (j & 7) + 16 * part, ad, smem_desc_sw128(qx + boff, 16, 1024),
                                 idesc, kk > 0 ? 1u : 0u);
                    }
                    mma_commit(&mma_done[j % kStages]);
                    if (abort_flag) break;
                }
            }
        } else if (warp < 4) {
            // Readers: an M=64 result has row m in TMEM lane 32 (m / 16) + m % 16,
            // so lanes 0-15 of warp w hold keys 16 w .. 16 w + 15 of the tile.
            const uint32_t lane_addr = uint32_t(32 * warp) << 16;
            for (int j = 0; j < ntiles; ++j) {
                if (!__all_sync(0xffffffffu, mbar_wait_ns(&mma_done[j % kStages], uint32_t(j / kStages) & 1u, p.wait_ns))) {
                    if (lane == 0) {
                        abort_flag = 1;
                        set_error(p.err, kDevErrTimeout);
                    }
                    break;
                }
                fence_after_sync();
                uint32_t hi[16], lo[16];
                tmem_ld16(tmem + lane_addr + 32 * (j & 7), hi);
                tmem_ld16(tmem + lane_addr + 32 * (j & 7) + 16, lo);
                tmem_wait_ld();
                const int key = 16 * warp + lane;
                if (lane < 16 && key < tile_rows(j)) {
                    float *dst = scores + (size_t(j) * T::kPositions + key) * 8;
#pragma unroll
                    for (int h = 0; h < kGroup; ++h)
                        dst[h] = (__uint_as_float(hi[h]) + __uint_as_float(lo[h])) * score_scale;
                }
                // Once every reader is done with tile j (and its MMAs, which
                // completed before, with the stage), refill the stage.
                fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&read_done[j % kStages]);
                if (threadIdx.x == 0 && !abort_flag && j + kStages < total_tiles) {
                    if (mbar_wait_ns(&read_done[j % kStages], uint32_t(j / kStages) & 1u, p.wait_ns)) {
                        issue(j + kStages);
                    } else {
                        abort_flag = 1;
                        set_error(p.err, kDevErrTimeout);
                    }
                }
                if (__any_sync(0xffffffffu, abort_flag != 0)) break;
            }
        }
        fence_before_sync();
        __syncthreads();
        fence_after_sync();
        next = ntiles;
    } else {
        float2 q2[kGroup][4];
        const float *qg = p.qprep + (size_t(b) * p.heads + size_t(kvh) * kGroup) * kAttnHeadDim;
#pragma unroll
        for (int h = 0; h < kGroup; ++h)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                q2[h][j] = make_float2(qg[h * kAttnHeadDim + lane_dim<KV>(lane, 2 * j)],
                                       qg[h * kAttnHeadDim + lane_dim<KV>(lane, 2 * j + 1)]);
        for (int j = 0; j < ntiles; ++j) {
            wait_tile(j);
            next = j + 1;
            if (!abort_flag) {
                const unsigned char *tile = stage + (j % kStages) * kTileBytes;
                float *out = scores + size_t(j) * T::kPositions * 8;
                const int rows = tile_rows(j);
                if (rows == T::kPositions)
                    score_rows<KV, true>(tile, rows, pl0, lane, q2, out, score_scale);
                else
                    score_rows<KV, false>(tile, rows, pl0, lane, q2, out, score_scale);
            }
            release(j);
            if (abort_flag) break;
        }
    }

    // Softmax statistics of the split: max and sum of exp(s - max); scores
    // are replaced by exp(s - max).
    if (!abort_flag && warp < kGroup) {
        float m = -INFINITY;
        for (int q = lane; q < cnt; q += 32) m = fmaxf(m, scores[q * 8 + warp]);
        m = warp_max(m);
        float l = 0.f;
        for (int q = lane; q < cnt; q += 32) {
            const float e = expf(scores[q * 8 + warp] - m);
            scores[q * 8 + warp] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml_s[warp][0] = m;
            ml_s[warp][1] = l;
        }
    }
    __syncthreads();

    if constexpr (kTc) {
        // Pass 2 on tcgen05: O^T [256 dims][heads] += V^T P^T per tile, as two
        // M=128 (dims), N=16, K=16 MMA chains (warp 5 dims 0-127, warp 6 dims
        // 128-255), each with P as a bf16 (hi, lo) pair into separate TMEM
        // columns (O^T reuses the score columns, all read by now).
        using namespace sm100;
        const uint32_t tmem = tmem_base_s;
        // P^T operand: K-major rows = heads (6-7 zero; the MMA also reads rows
        // 8-15, the next kilobyte), one SW128 box per 64 keys; keys past the
        // split's end are zero. Thread = (head row, 8 keys).
        const int nbox = p.chunk / 64;
        const uint32_t p_half = uint32_t(nbox) * 1024;
        for (int idx = threadIdx.x; idx < 8 * nbox * 8; idx += kThreads) {
            const int h = idx & 7, c8 = idx >> 3;  // c8: 8-key group
            uint32_t hw[4] = {0u, 0u, 0u, 0u}, lw[4] = {0u, 0u, 0u, 0u};
            if (h < kGroup && !abort_flag) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int q0 = 8 * c8 + 2 * i;
                    const float e0 = q0 < cnt ? scores[q0 * 8 + h] : 0.f;
                    const float e1 = q0 + 1 < cnt ? scores[(q0 + 1) * 8 + h] : 0.f;
                    hw[i] = pack_bf16x2_rn(e0, e1);
                    const float2 hf = bf16x2_to_float2(hw[i]);
                    lw[i] = pack_bf16x2_rn(e0 - hf.x, e1 - hf.y);
                }
            }
            const uint32_t off = (c8 >> 3) * 1024 + h * 128 + (((c8 & 7) ^ h) << 4);
            *reinterpret_cast<uint4 *>(psm + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(psm + p_half + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        if (threadIdx.x < 64)
            reinterpret_cast<uint4 *>(psm + 2 * p_half)[threadIdx.x] = make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_smem();
        fence_before_sync();
        __syncthreads();
        fence_after_sync();
        if ((warp == 5 || warp == 6) && lane == 0 && !abort_flag) {
            const int mt = warp - 5;
            const uint32_t idesc = idesc_bf16_f32(128, 16, 1, 0);  // A (V^T) MN-major
            const uint32_t pb = smem_addr(psm);
            for (int j = ntiles; j < total_tiles; ++j) {
                const int t = j - ntiles;
                if (!mbar_wait_ns(&bars[j % kStages], uint32_t(j / kStages) & 1u, p.wait_ns)) {
                    abort_flag = 1;
                    set_error(p.err, kDevErrTimeout);
                    break;
                }
                fence_after_sync();
                const uint32_t vs = smem_addr(stage + (j % kStages) * kTileBytes) + 2 * mt * (kTileBytes / 4);
#pragma unroll
                for (int kk = 0; kk < T::kPositions / 16; ++kk) {
                    const uint64_t ad = smem_desc_sw128(vs + kk * 2048, kTileBytes / 4, 1024);
                    const uint32_t boff = t * 1024 + kk * 32;
                    const uint32_t acc = (t | kk) ? 1u : 0u;
                    mma_bf16(tmem + 32 * mt, ad, smem_desc_sw128(pb + boff, 16, 1024), idesc, acc);
                    mma_bf16(tmem + 32 * mt + 16, ad, smem_desc_sw128(pb + p_half + boff, 16, 1024),
                             idesc, acc);
                }
                mma_commit(&mma_done[j % kStages]);
                if (abort_flag) break;
            }
            mma_commit(&pv_final);  // every MMA of this chain, whatever happened
        } else if (threadIdx.x == 0) {
            // Refill each stage once both chains have read it.
            for (int j = ntiles; j + kStages < total_tiles && !abort_flag; ++j) {
                if (!mbar_wait_ns(&mma_done[j % kStages], uint32_t(j / kStages) & 1u, p.wait_ns)) {
                    abort_flag = 1;
                    set_error(p.err, kDevErrTimeout);
                    break;
                }
                issue(j + kStages);
            }
        }
        // Epilogue: warps 0-3 read O^T (lane = dim) once the last tile's MMAs
        // (and so all earlier ones) have completed.
        if (warp < 4) {
            const bool ok = !abort_flag && __all_sync(0xffffffffu, mbar_wait_ns(&pv_final, 0, p.wait_ns));
            if (ok) {
                fence_after_sync();
#pragma unroll 1
                for (int mt = 0; mt < 2; ++mt) {
                    uint32_t hi[16], lo[16];
                    tmem_ld16(tmem + (uint32_t(32 * warp) << 16) + 32 * mt, hi);
                    tmem_ld16(tmem + (uint32_t(32 * warp) << 16) + 32 * mt + 16, lo);
                    tmem_wait_ld();
                    const int d = 128 * mt + 32 * warp + lane;
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) {
                        const size_t slot = (size_t(b) * p.heads + size_t(kvh) * kGroup + h) * p.max_splits + split;
                        p.part_o[slot * kAttnHeadDim + d] = __uint_as_float(hi[h]) + __uint_as_float(lo[h]);
                        if (d == 0) {
                            p.part_ml[slot * 2 + 0] = ml_s[h][0];
                            p.part_ml[slot * 2 + 1] = ml_s[h][1];
                        }
                    }
                }
            } else if (lane == 0) {
                abort_flag = 1;
                set_error(p.err, kDevErrTimeout);
            }
        }
        fence_before_sync();
        __syncthreads();
        if (abort_flag && threadIdx.x == 0) {
            // Copies still in flight are among the last kStages issued (each
            // refill waited for the tile kStages before it): let them land.
            for (int j = max(0, issued_s - kStages); j < issued_s; ++j)
                (void)mbar_wait_ns(&bars[j % kStages], uint32_t(j / kStages) & 1u, p.wait_ns);
        }
        if (warp == 0) {
            __syncwarp();
            tmem_dealloc(tmem, kDecodeTmemCols);
        }
    } else {
    // Pass 2 on the CUDA cores (f32 cache): acc[h] += exp(s-m)[h] * V.
    float2 acc[kGroup][4];
#pragma unroll
    for (int h = 0; h < kGroup; ++h)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[h][j] = make_float2(0.f, 0.f);
    if (!abort_flag) {
        for (int j = ntiles; j < total_tiles; ++j) {
            wait_tile(j);
            next = j + 1;
            if (!abort_flag) {
                const int t = j - ntiles;
                const unsigned char *tile = stage + (j % kStages) * kTileBytes;
                const float *e_rows = scores + size_t(t) * T::kPositions * 8;
                const int rows = tile_rows(j);
                if (rows == T::kPositions)
                    accumulate_rows<KV, true>(tile, rows, pl0, lane, e_rows, acc);
                else
                    accumulate_rows<KV, false>(tile, rows, pl0, lane, e_rows, acc);
            }
            release(j);
            if (abort_flag) break;
        }
    }

    if (abort_flag) {
        // Let copies still in flight land before the CTA's shared memory is
        // released (bounded as well).
        if (threadIdx.x == 0) {
            const int issued = min(total_tiles, next + kStages - 1);
            for (int j = max(0, next - 1); j < issued; ++j)
                (void)mbar_wait_ns(&bars[j % kStages], uint32_t(j / kStages) & 1u, p.wait_ns);
        }
        return;
    }

    // Cross-warp reduction of acc through the (now idle) stage buffers.
    float *red = reinterpret_cast<float *>(stage);  // [warps][6][256]
#pragma unroll
    for (int h = 0; h < kGroup; ++h)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            red[(warp * kGroup + h) * kAttnHeadDim + lane_dim<KV>(lane, 2 * jj)] = acc[h][jj].x;
            red[(warp * kGroup + h) * kAttnHeadDim + lane_dim<KV>(lane, 2 * jj + 1)] = acc[h][jj].y;
        }
    __syncthreads();
    const int d = threadIdx.x;
#pragma unroll 1
    for (int h = 0; h < kGroup; ++h) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) o += red[(w * kGroup + h) * kAttnHeadDim + d];
        const size_t slot = (size_t(b) * p.heads + size_t(kvh) * kGroup + h) * p.max_splits + split;
        p.part_o[slot * kAttnHeadDim + d] = o;
        if (d == 0) {
            p.part_ml[slot * 2 + 0] = ml_s[h][0];
            p.part_ml[slot * 2 + 1] = ml_s[h][1];
        }
    }
    }  // f32 pass 2
}

// ----------------------------------------------------------------------------
// K3: merge + gate
// ----------------------------------------------------------------------------
struct MergeParams {
    const float *part_o, *part_ml;
    const float *q_and_gate;
    const int32_t *positions;
    float *attention;
    float *partial_out;  // non-null: write (o, m, l) [batch][heads][258] instead
    int context_length, heads, chunk, max_splits, max_position, pos_offset, sharded;
    int merge_ctas;      // CTAs (one cluster) per (head, sequence)
    // Split-sequence exchange over peer memory (p2p_nranks > 0; see
    // p2p_exchange_merge): every rank's exchange buffer, this rank's index,
    // the buffers' batch (the state's), the epoch counter, the wait limit and
    // the error word.
    float *const *p2p_peers;
    int p2p_rank, p2p_nranks, p2p_batch;
    const uint32_t *p2p_epoch;  // device counter, advanced by this call's prep kernel
    uint64_t wait_ns;
    int *err;
};

// One exchanged value with the epoch of its call: (epoch << 32) | bits. An
// aligned 8-byte store is seen whole or not at all, so a reader that finds
// the current epoch in a word also has its value: no fence and no separate
// flag are needed.
__device__ __forceinline__ void st_word_sys(unsigned long long *p, float v, uint32_t epoch) {
    const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// Waits (at most limit_ns of %globaltimer) for the word to carry `epoch`;
// returns its value, or NaN if the wait gave up (*ok cleared).
__device__ __forceinline__ float wait_word_sys(const unsigned long long *p, uint32_t epoch,
                                               uint64_t limit_ns, bool *ok) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    if (uint32_t(w >> 32) == epoch) return __uint_as_float(uint32_t(w));
    const uint64_t t0 = global_timer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 64; ++i) {
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
            if (uint32_t(w >> 32) == epoch) return __uint_as_float(uint32_t(w));
        }
        if (global_timer_ns() - t0 > limit_ns) {
            *ok = false;
            return __uint_as_float(0x7fc00000u);
        }
    }
}

// Exchange buffer of one rank (allocated by q38_state_split_p2p_handle):
//   [2][nranks][batch][heads][258] 8-byte words (o[256], m, l, each with its
//   call's epoch).
// The leading 2 is the epoch's parity: a rank writes epoch e + 2 into a
// peer's slot only after it has read that peer's words of e + 1, which the
// peer writes only after it has finished reading epoch e, so no slot is
// overwritten before it is read.
__host__ __device__ inline size_t p2p_words(int nranks, int batch, int heads) {
    return size_t(2) * nranks * batch * heads * (kAttnHeadDim + 2);
}

// The split-sequence exchange of one (head, sequence), by CTA 0 of its merge
// cluster after the local merge: thread d stores this rank's o[d] (threads 0
// and 1 also m and l) as epoch-tagged words into slot p2p_rank of every
// rank's exchange buffer over NVLink (plain stores; the buffers are CUDA IPC
// mappings), then waits (bounded) until its own words of every rank carry
// the epoch, and the CTA merges the nranks partials by log-sum-exp and writes
// the gated output. No kernel reads another GPU's memory and nothing is
// exchanged by TMA.
__device__ void p2p_exchange_merge(const MergeParams &p, int h, int b, float ot, float m, float lt,
                                   bool has_rows) {
    const int d = threadIdx.x;
    const int R = p.p2p_nranks, H = p.heads, B = p.p2p_batch;
    const uint32_t epoch = *reinterpret_cast<const volatile uint32_t *>(p.p2p_epoch);
    const int par = int(epoch & 1u);
    auto slot = [&](int r) { return (((size_t(par) * R + r) * B + b) * H + h) * (kAttnHeadDim + 2); };
    const float o_send = has_rows ? ot : 0.f;
    for (int r = 0; r < R; ++r) {
        unsigned long long *dst =
            reinterpret_cast<unsigned long long *>(p.p2p_peers[r]) + slot(p.p2p_rank);
        st_word_sys(dst + d, o_send, epoch);
        if (d < 2) st_word_sys(dst + kAttnHeadDim + d, d == 0 ? m : lt, epoch);
    }
    const unsigned long long *mine = reinterpret_cast<const unsigned long long *>(p.p2p_peers[p.p2p_rank]);
    bool ok = true;
    float mm = -INFINITY;
    for (int r = 0; r < R; ++r)
        mm = fmaxf(mm, wait_word_sys(mine + slot(r) + kAttnHeadDim, epoch, p.wait_ns, &ok));
    float lsum = 0.f, osum = 0.f;
    for (int r = 0; r < R && ok; ++r) {
        const float mr = wait_word_sys(mine + slot(r) + kAttnHeadDim, epoch, p.wait_ns, &ok);
        const float lr = wait_word_sys(mine + slot(r) + kAttnHeadDim + 1, epoch, p.wait_ns, &ok);
        const float orr = wait_word_sys(mine + slot(r) + d, epoch, p.wait_ns, &ok);
        if (mr == -INFINITY) continue;  // a shard without visible rows
        const float w = expf(mr - mm);
        lsum += w * lr;
        osum += w * orr;
    }
    if (!ok) set_error(p.err, kDevErrTimeout);  // the output is then undefined
    const float gate = p.q_and_gate[(size_t(b) * H + h) * 2 * kAttnHeadDim + kAttnHeadDim + d];
    p.attention[(size_t(b) * H + h) * kAttnHeadDim + d] = (osum / lsum) * sigmoidf_ref(gate);
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// A cluster of merge_ctas CTAs (256 threads each) per (head, sequence); CTA g
// of the cluster merges splits [g * per, (g + 1) * per). Inside a CTA all 8
// warps read at once: warp w takes splits w, w + 8, ..., lane l dims
// [8l, 8l + 8) of each (two 16-byte loads), and the 8 per-warp sums are added
// in shared memory in warp order. Each CTA then stores its (o, m, l) into CTA
// 0's shared memory (distributed shared memory, remote stores), and after one
// cluster barrier CTA 0 combines them by log-sum-exp, so a single long
// sequence's hundreds of splits are read by many SMs at once.
__global__ void __launch_bounds__(kAttnHeadDim) attn_decode_merge_kernel(MergeParams p) {
    __shared__ float red[kWarps][kAttnHeadDim];
    __shared__ float lred[kWarps], mred[kWarps];
    // CTA 0 of a cluster: every CTA's (o, m, l), pushed here by remote stores.
    __shared__ float gath_o[8][kAttnHeadDim], gath_ml[8][2];
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int G = p.merge_ctas;
    const uint32_t g = G > 1 ? sm100::cluster_ctarank() : 0u;
    const int pos = p.positions[b];
    pdl_wait_primary();
    pdl_launch_dependents();  // the next call's prep may become resident
    // Uniform over the cluster (one sequence), so every CTA of it returns here or none.
    if (!position_ok(pos, p.pos_offset, p.context_length, p.max_position, p.sharded)) return;
    const int n = local_rows(pos, p.pos_offset, p.context_length);
    const int nsplit = n > 0 ? (n + p.chunk - 1) / p.chunk : 0;
    const int per = (nsplit + G - 1) / G;
    const int s0 = min(nsplit, int(g) * per), s1 = min(nsplit, s0 + per);
    const size_t base = (size_t(b) * p.heads + h) * p.max_splits;
    const float2 *ml = reinterpret_cast<const float2 *>(p.part_ml) + base;
    // This warp's first two splits are loaded before the CTA-wide max, so
    // that their loads overlap it; they are added first, in the same order.
    float2 vpre[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    float4 apre[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    float4 cpre[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int s = s0 + warp + u * kWarps;
        if (s < s1) {
            vpre[u] = ml[s];
            const float4 *src = reinterpret_cast<const float4 *>(p.part_o + (base + s) * kAttnHeadDim) + 2 * lane;
            apre[u] = src[0];
            cpre[u] = src[1];
        }
    }
    float m = -INFINITY;
    for (int s = s0 + tid; s < s1; s += kAttnHeadDim) m = fmaxf(m, ml[s].x);
    m = warp_max(m);
    if (lane == 0) mred[warp] = m;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, mred[w]);
    float l = 0.f;
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    auto add_split = [&](const float2 v, const float4 a, const float4 c) {
        const float w = expf(v.x - m);
        l += w * v.y;
        o[0] += w * a.x; o[1] += w * a.y; o[2] += w * a.z; o[3] += w * a.w;
        o[4] += w * c.x; o[5] += w * c.y; o[6] += w * c.z; o[7] += w * c.w;
    };
#pragma unroll
    for (int u = 0; u < 2; ++u)
        if (s0 + warp + u * kWarps < s1) add_split(vpre[u], apre[u], cpre[u]);
#pragma unroll 4
    for (int s = s0 + warp + 2 * kWarps; s < s1; s += kWarps) {
        const float4 *src = reinterpret_cast<const float4 *>(p.part_o + (base + s) * kAttnHeadDim) + 2 * lane;
        add_split(ml[s], src[0], src[1]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp][8 * lane + i] = o[i];
    if (lane == 0) lred[warp] = l;
    __syncthreads();
    float ot = 0.f, lt = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        ot += red[w][tid];
        lt += lred[w];
    }
    if (G > 1) {
        // This CTA's (o, m, l) (m = -inf, l = o = 0 for a CTA without splits)
        // stored straight into CTA 0's shared memory; one cluster barrier
        // (release / acquire) orders the stores before CTA 0 reads them, and
        // the other CTAs are done.
        st_cluster_f32(sm100::cluster_addr(&gath_o[g][tid], 0u), s1 > s0 ? ot : 0.f);
        if (tid == 0) {
            st_cluster_f32(sm100::cluster_addr(&gath_ml[g][0], 0u), m);
            st_cluster_f32(sm100::cluster_addr(&gath_ml[g][1], 0u), lt);
        }
        sm100::cluster_sync();
        if (g != 0) return;
        float mm = -INFINITY;
        for (int r = 0; r < G; ++r) mm = fmaxf(mm, gath_ml[r][0]);
        float lsum = 0.f, osum = 0.f;
        for (int r = 0; r < G; ++r) {
            const float mr = gath_ml[r][0];
            if (mr == -INFINITY) continue;
            const float w = expf(mr - mm);
            lsum += w * gath_ml[r][1];
            osum += w * gath_o[r][tid];
        }
        m = mm;
        lt = lsum;
        ot = osum;
    }
    const int d = tid;
    if (p.p2p_nranks > 0) {
        p2p_exchange_merge(p, h, b, ot, m, lt, nsplit > 0);
        return;
    }
    if (p.partial_out) {
        // This shard's (o, m, l) relative to its own max m (m = -inf, l = 0,
        // o = 0 when the shard holds no visible row).
        float *dst = p.partial_out + (size_t(b) * p.heads + h) * (kAttnHeadDim + 2);
        dst[d] = nsplit > 0 ? ot : 0.f;
        if (d == 0) {
            dst[kAttnHeadDim] = m;
            dst[kAttnHeadDim + 1] = lt;
        }
        return;
    }
    const float gate = p.q_and_gate[(size_t(b) * p.heads + h) * 2 * kAttnHeadDim + kAttnHeadDim + d];
    p.attention[(size_t(b) * p.heads + h) * kAttnHeadDim + d] = (ot / lt) * sigmoidf_ref(gate);
}

// Cross-shard merge: nparts packed (o, m, l) partials per (sequence, head),
// [nparts][batch][heads][258], combined by log-sum-exp, normalised and gated.
struct ShardMergeParams {
    const float *partials;
    const float *q_and_gate;
    float *attention;
    int nparts, batch, heads;
};

__global__ void __launch_bounds__(kAttnHeadDim) attn_merge_shards_kernel(ShardMergeParams p) {
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const size_t stride = size_t(p.batch) * p.heads * (kAttnHeadDim + 2);
    const float *base = p.partials + (size_t(b) * p.heads + h) * (kAttnHeadDim + 2);
    float m = -INFINITY;
    for (int r = 0; r < p.nparts; ++r) m = fmaxf(m, base[r * stride + kAttnHeadDim]);
    float l = 0.f, o = 0.f;
    for (int r = 0; r < p.nparts; ++r) {
        const float *part = base + r * stride;
        const float mr = part[kAttnHeadDim];
        if (mr == -INFINITY) continue;  // an empty shard
        const float w = expf(mr - m);
        l += w * part[kAttnHeadDim + 1];
        o += w * part[d];
    }
    const float gate = p.q_and_gate[(size_t(b) * p.heads + h) * 2 * kAttnHeadDim + kAttnHeadDim + d];
    p.attention[(size_t(b) * p.heads + h) * kAttnHeadDim + d] = (o / l) * sigmoidf_ref(gate);
}

// 3-D map of the bf16 key cache [planes][rows][256] with a box of 64 dims x
// 64 rows and 128-byte swizzle: one quarter of a K tile as the MMA operand.
bool make_map_kcache(CUtensorMap *m, const void *base, uint64_t rows, uint64_t planes) {
    static PFN_cuTensorMapEncodeTiled_v12000 enc = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    if (!enc) return false;
    cuuint64_t dims[3] = {uint64_t(kAttnHeadDim), rows, planes};
    cuuint64_t strides[2] = {uint64_t(kAttnHeadDim) * 2, uint64_t(kAttnHeadDim) * 2 * rows};
    cuuint32_t box[3] = {64, 64, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box,
               es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Encoded tensor maps of recent calls, per host thread: a decode call's maps
// depend only on the cache's base address and shape, which stay the same
// from one step to the next, so each is encoded once (keeps the host side of
// a launch-bound decode step short).
bool cached_map_kcache(CUtensorMap *m, const void *base, uint64_t rows, uint64_t planes) {
    struct Entry {
        const void *base = nullptr;
        uint64_t rows = 0, planes = 0;
        CUtensorMap map;
    };
    constexpr int kEntries = 8;
    thread_local Entry cache[kEntries];
    thread_local int next = 0;
    for (const Entry &e : cache)
        if (e.base == base && e.rows == rows && e.planes == planes) {
            *m = e.map;
            return true;
        }
    if (!make_map_kcache(m, base, rows, planes)) return false;
    cache[next] = Entry{base, rows, planes, *m};
    next = (next + 1) % kEntries;
    return true;
}

// Largest dynamic shared memory a split launch can ask for (the largest
// chunk the planner can choose), set as the kernel's limit once per device.
template <typename KV>
cudaError_t ensure_split_smem_limit() {
    constexpr bool kTc = sizeof(KV) == 2;
    constexpr int kMaxC = kTc ? kMaxChunkTc : kMaxChunk;
    constexpr size_t kSmemMax = size_t(Tile<KV>::kStages) * kTileBytes + size_t(kMaxC) * 8 * sizeof(float) +
                                (kTc ? kQRegionBytes + size_t(kMaxC / 64) * 2048 + 1024 : 0) + 1024;
    static_assert(kSmemMax <= 227 * 1024, "split kernel shared memory");
    static bool set[128] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 128 && set[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(attn_decode_split_kernel<KV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(kSmemMax));
    if (e == cudaSuccess && dev < 128) set[dev] = true;
    return e;
}

template <typename KV>
cudaError_t launch_typed(const AttnDecodeLaunch &a, int sm_count, cudaStream_t stream) {
    // Rows any sequence of this call attends to in the local cache.
    const int max_rows = std::min(a.max_position - a.pos_offset + 1, a.context_length);
    const DecodeSplitPlan plan =
        plan_attn_decode(a.batch, a.kv_heads, std::max(max_rows, 1) - 1, a.kv_dtype, sm_count);
    if (plan.nsplit > a.max_splits) return cudaErrorInvalidValue;

    const int sharded = (a.partial_out != nullptr || a.p2p_nranks > 0) ? 1 : 0;
    PrepParams pp{a.q_and_gate, a.key,      a.value,        a.positions,  a.kcache,
                  a.vcache,     a.qprep,    a.err,          a.q_norm,     a.k_norm,
                  a.context_length, a.heads, a.kv_heads,    a.max_position, a.pos_offset,
                  sharded,      a.theta_scale, a.eps, a.p2p_nranks > 0 ? a.p2p_epoch : nullptr};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t pcfg{};
    pcfg.gridDim = dim3(a.heads + a.kv_heads, a.batch);
    pcfg.blockDim = dim3(kAttnHeadDim);
    pcfg.stream = stream;
    pcfg.attrs = attr;
    pcfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&pcfg, attn_decode_prep_kernel<KV>, pp);
    if (e != cudaSuccess) return e;

    SplitParams sp{a.kcache,   a.vcache,  a.qprep,  a.positions,       a.part_o,
                   a.part_ml,  a.err,     a.context_length, a.heads, a.kv_heads,
                   plan.chunk, a.max_splits, a.max_position, a.pos_offset,
                   sharded, a.wait_ns ? a.wait_ns : kWaitTimeoutNs,
                   a.skip_kv_loads};
    constexpr bool kTc = sizeof(KV) == 2;
    CUtensorMap map_k{}, map_v{};
    if (kTc && (!cached_map_kcache(&map_k, a.kcache, uint64_t(a.context_length),
                                   uint64_t(a.batch) * a.kv_heads) ||
                !cached_map_kcache(&map_v, a.vcache, uint64_t(a.context_length),
                                   uint64_t(a.batch) * a.kv_heads)))
        return cudaErrorInvalidValue;
    // bf16: query operand, P operand (2 x 1 KB per 64 keys + 1 KB); all: alignment.
    auto extra_for = [&](int chunk) {
        return (kTc ? kQRegionBytes + size_t(chunk / 64) * 2048 + 1024 : 0) + 1024;
    };
    const size_t smem = size_t(Tile<KV>::kStages) * kTileBytes + size_t(plan.chunk) * 8 * sizeof(float) +
                        extra_for(plan.chunk);
    if ((e = ensure_split_smem_limit<KV>()) != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(plan.nsplit, a.kv_heads, a.batch);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, attn_decode_split_kernel<KV>, map_k, map_v, sp);
    if (e != cudaSuccess) return e;

    // Merge CTAs per (head, sequence): one while the (head, sequence) grid
    // alone fills the SMs twice over; otherwise a cluster of up to 8 (a
    // portable size), about 32 splits each, so that a small batch's many
    // splits are read by many SMs.
    const int fill = std::max(1, (2 * sm_count) / std::max(1, a.heads * a.batch));
    const int merge_ctas = std::min({8, fill, std::max(1, (plan.nsplit + 31) / 32)});
    MergeParams mp{a.part_o,   a.part_ml,  a.q_and_gate, a.positions,  a.attention,
                   a.partial_out, a.context_length, a.heads, plan.chunk, a.max_splits,
                   a.max_position, a.pos_offset, sharded, merge_ctas,
                   a.p2p_peers, a.p2p_rank, a.p2p_nranks, a.p2p_batch, a.p2p_epoch,
                   a.wait_ns ? a.wait_ns : kWaitTimeoutNs, a.err};
    cudaLaunchAttribute mattr[2];
    mattr[0] = attr[0];
    mattr[1].id = cudaLaunchAttributeClusterDimension;
    mattr[1].val.clusterDim.x = 1;
    mattr[1].val.clusterDim.y = 1;
    mattr[1].val.clusterDim.z = unsigned(merge_ctas);
    cfg.gridDim = dim3(a.heads, a.batch, merge_ctas);
    cfg.blockDim = dim3(kAttnHeadDim);
    cfg.dynamicSmemBytes = 0;
    cfg.attrs = mattr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, attn_decode_merge_kernel, mp);
}

}  // namespace

// Splits per (sequence, kv head) that the partial buffers hold for a cache of
// context_length positions: enough for splits of a quarter of kFastChunk at
// any length (the partials then stay near 2% of the KV bytes), at least
// kMinSplitsCap, never more than one per tile.
int attn_decode_max_splits(int context_length, int kv_dtype) {
    const int tile = tile_positions(kv_dtype);
    const int max_chunk = kv_dtype == Q38_KV_BF16 ? kMaxChunkTc : kMaxChunk;
    const int by_tile = (context_length + tile - 1) / tile;
    const int by_chunk = (context_length + max_chunk - 1) / max_chunk;
    const int by_quarter = (context_length + kFastChunk / 4 - 1) / (kFastChunk / 4);
    return std::min(by_tile, std::max({kMinSplitsCap, by_chunk, by_quarter}));
}

// Split plan: the chunk (a whole number of tiles, at most kFastChunk so that
// two CTAs fit on an SM) that minimises the estimated makespan
//   ceil(CTAs / (2 * SMs)) * (chunk + per-CTA overhead),
// i.e. whole waves of equal CTAs; a smaller chunk replaces a larger one only
// when it is at least 3% cheaper (fewer partials to write and merge).
// Batched long-context decode keeps 512-position splits; a single long
// sequence gets enough splits to fill every SM in near-whole waves.
DecodeSplitPlan plan_attn_decode(int batch, int kv_heads, int max_position, int kv_dtype,
                                 int sm_count) {
    constexpr int kOverheadPositions = 128;  // setup, softmax and partial write of a CTA
    const int tile = tile_positions(kv_dtype);
    const int max_chunk = kv_dtype == Q38_KV_BF16 ? kMaxChunkTc : kMaxChunk;
    const int n = std::max(max_position + 1, 1);
    const int tiles = (n + tile - 1) / tile;
    const int64_t units = std::max(1, batch * kv_heads);
    const int64_t slots = 2 * int64_t(std::max(sm_count, 1));
    // Never more splits than attn_decode_max_splits allows for this n (the
    // state's partial buffers hold that many for its whole context).
    const int cap = attn_decode_max_splits(n, kv_dtype);
    int best_ct = 0;
    int64_t best = 0;
    for (int ct = std::min(kFastChunk / tile, tiles); ct >= 1; --ct) {
        const int nsplit = (tiles + ct - 1) / ct;
        if (nsplit > cap) break;  // smaller chunks only need more splits
        const int64_t waves = (units * nsplit + slots - 1) / slots;
        const int64_t cost = waves * (int64_t(ct) * tile + kOverheadPositions);
        if (best_ct == 0 || cost * 100 < best * 97) {
            best = cost;
            best_ct = ct;
        }
    }
    int chunk = best_ct * tile;
    if (best_ct == 0) {
        // Longer than cap fast splits: the smallest chunk that respects the cap.
        chunk = ((n + cap - 1) / cap + tile - 1) / tile * tile;
        chunk = std::min(chunk, max_chunk);
    }
    DecodeSplitPlan plan;
    plan.chunk = chunk;
    plan.nsplit = (n + chunk - 1) / chunk;
    return plan;
}

size_t attn_p2p_exchange_bytes(int nranks, int batch, int heads) {
    return p2p_words(nranks, batch, heads) * sizeof(unsigned long long);
}

cudaError_t launch_attn_merge_shards(const float *partials, int nparts, int batch, int heads,
                                     const float *q_and_gate, float *attention,
                                     cudaStream_t stream) {
    ShardMergeParams p{partials, q_and_gate, attention, nparts, batch, heads};
    attn_merge_shards_kernel<<<dim3(heads, batch), kAttnHeadDim, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_attn_decode(const AttnDecodeLaunch &a, int sm_count, cudaStream_t stream) {
    if (a.kv_dtype == Q38_KV_BF16) return launch_typed<__nv_bfloat16>(a, sm_count, stream);
    return launch_typed<float>(a, sm_count, stream);
}

}  // namespace q38
