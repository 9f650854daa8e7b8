// proj_mma.cu -- K-quant projections of many tokens on the tensor cores
// (tcgen05.mma kind::i8), bit-identical to the reference's integer path.
//
// The reference's dot of a Q4_K / Q5_K row with Q8_K activations
// (dot_q4_k_q8_k_scalar / dot_q5_k_q8_k_scalar, src/kernel/tensor.rs:365-428)
// is, per 256-block, weighted = sum_j sc_j * dot_j over its eight 32-value
// sub-blocks (sc_j 6-bit), minimum = sum_j mn_j * (activation sum of j), and
// the f32 term d*weighted - dmin*minimum added to a running total in block
// order. Split each scale into 3-bit halves, sc = lo + 8 hi: a packed word of
// four values (each <= 31) times a 3-bit factor keeps every byte below 256,
// so one integer multiply per word forms four scaled weights, and
//   weighted = A_lo . a + 8 * (A_hi . a),  A_lo = q * lo(sc), A_hi = q * hi(sc)
// are two exact u8 x s8 -> s32 products over the whole block, one tcgen05
// accumulator each. The epilogue adds the minimum term (8 integer products
// per row and token) and the f32 term exactly as the reference does, so the
// result is bit-identical.
//
// CTA: 128 weight rows x 32 tokens, 10 warps.
//   warp 0      TMA: the raw weight blocks [128 rows][block bytes] (issued
//               before the programmatic-dependent wait: weights are constant)
//               and the activation quants [32 tokens][256] (SW128).
//   warp 1      TMEM allocation and the MMA issue: per block 2 x 8 kind::i8
//               MMAs (M=128, N=32, K=32) into the block's (lo, hi) pair of
//               32-column accumulators, double-buffered.
//   warps 2-9   thread = weight row (TMEM lane): warps 2-5 unpack sub-blocks
//               0-3 and finish tokens 0-15, warps 6-9 sub-blocks 4-7 and
//               tokens 16-31; the unpacked, scaled operands go to shared
//               memory in the SW128 K-major layout (two buffers).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "q38_proj.h"
#include "q38_sm100.cuh"

namespace q38 {
namespace {

constexpr int kMmaRows = 128;
constexpr int kMmaTok = 32;
constexpr int kMmaWarps = 10;
constexpr int kMmaThreads = 32 * kMmaWarps;
constexpr int kUnpackWarps = 8;
constexpr uint32_t kAtomA = kMmaRows * 128;     // one SW128 atom of A: 128 rows x 128 B
constexpr uint32_t kOperandA = 2 * kAtomA;      // 256 K of one A operand
constexpr uint32_t kBufA = 2 * kOperandA;       // lo | hi
constexpr uint32_t kAtomB = kMmaTok * 128;      // 32 tokens x 128 B
constexpr uint32_t kStageB = 2 * kAtomB;
constexpr int kMaxMmaStages = 3;
constexpr uint32_t kMmaTmemCols = 128;          // 2 buffers x (lo 32 | hi 32)

// kind::i8: D s32, A u8 (the scaled weights are 0..217), B s8 (Q8_K quants),
// both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (0u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ float half_bits(uint32_t h) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xffffu)));
}

struct MmaParams {
    const float *scale;    // [batch][nblk] activation block scales
    const int16_t *sums;   // [batch][nblk][16] activation group sums
    float *out;            // out[t * out_ld + row]
    int *err;
    long out_ld;
    int rows, nblk, batch, stages;
    uint32_t raw_bytes;    // kMmaRows * block bytes
};

struct MmaSmem {
    uint32_t a, raw, b, scl, ps, total;
};

__host__ __device__ inline MmaSmem mma_smem_plan(int stages, uint32_t raw_bytes, int nblk) {
    MmaSmem s{};
    s.a = 0;
    s.raw = 2 * kBufA;
    s.b = s.raw + stages * raw_bytes;  // raw_bytes is a multiple of 1024
    s.scl = s.b + stages * kStageB;
    s.ps = s.scl + uint32_t(kMmaTok * nblk * 4);
    s.total = s.ps + uint32_t(kMmaTok * nblk * 16);
    return s;
}

template <int T> constexpr uint32_t kMmaBlockBytes = T == Q38_GGML_Q4_K ? 144 : 176;

// SW128 K-major position of 16-byte chunk u (0..7) of row r in an atom.
__device__ __forceinline__ uint32_t sw128_chunk(uint32_t r, uint32_t u) {
    return r * 128u + ((u ^ (r & 7u)) << 4);
}

template <int T>
__global__ void __launch_bounds__(kMmaThreads, 1)
    proj_mma_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
                    MmaParams p) {
    using namespace sm100;
    constexpr uint32_t bb = kMmaBlockBytes<T>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t raw_full[kMaxMmaStages], raw_empty[kMaxMmaStages];
    __shared__ __align__(8) uint64_t b_full[kMaxMmaStages], b_empty[kMaxMmaStages];
    __shared__ __align__(8) uint64_t a_full[2], mma_done[2];
    __shared__ uint32_t tmem_base_s;
    __shared__ volatile int abort_flag;
    const MmaSmem lay = mma_smem_plan(p.stages, p.raw_bytes, p.nblk);
    float *scl = reinterpret_cast<float *>(smem + lay.scl);
    int16_t *ps = reinterpret_cast<int16_t *>(smem + lay.ps);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * kMmaRows, tok0 = blockIdx.y * kMmaTok;
    const int S = p.stages;

    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kUnpackWarps);
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&a_full[i], kUnpackWarps);
            mbar_init(&mma_done[i], 1);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_s, kMmaTmemCols);
        tmem_relinquish();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_base_s;
    const int first = min(S, p.nblk);
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&map_w);
        tma_prefetch_desc(&map_a);
        // The weights are constant: their first blocks are requested before
        // the wait for the kernel that quantized the activations.
        for (int b = 0; b < first; ++b) {
            mbar_arrive_expect_tx(&raw_full[b], p.raw_bytes);
            tma_load_3d(smem + lay.raw + b * p.raw_bytes, &map_w, b * int(bb), row0, 0, &raw_full[b]);
        }
    }
    pdl_wait_primary();
    pdl_launch_dependents();
    // This CTA's tokens: block scales and the eight 32-value sums per block.
    for (int i = tid; i < kMmaTok * p.nblk; i += kMmaThreads) {
        const int t = i / p.nblk, b = i - t * p.nblk;
        const bool in = tok0 + t < p.batch;
        scl[i] = in ? p.scale[size_t(tok0 + t) * p.nblk + b] : 0.f;
        const int16_t *g = p.sums + (size_t(tok0 + t) * p.nblk + b) * 16;
#pragma unroll
        for (int j = 0; j < 8; ++j) ps[i * 8 + j] = in ? int16_t(g[2 * j] + g[2 * j + 1]) : int16_t(0);
    }
    __syncthreads();

    if (warp == 0) {
        // ---------------------------------------------------------- TMA
        if (lane == 0) {
            bool ok = true;
            for (int b = 0; b < first; ++b) {
                mbar_arrive_expect_tx(&b_full[b], kStageB);
                for (int h = 0; h < 2; ++h)
                    tma_load_3d(smem + lay.b + b * kStageB + h * kAtomB, &map_a, b * 256 + h * 128, tok0, 0,
                                &b_full[b]);
            }
            for (int b = first; b < p.nblk && ok; ++b) {
                const int s = b % S;
                const uint32_t ph = uint32_t(b / S - 1) & 1u;
                ok = mbar_wait(&raw_empty[s], ph) && mbar_wait(&b_empty[s], ph) && !abort_flag;
                if (!ok) break;
                mbar_arrive_expect_tx(&raw_full[s], p.raw_bytes);
                tma_load_3d(smem + lay.raw + s * p.raw_bytes, &map_w, b * int(bb), row0, 0, &raw_full[s]);
                mbar_arrive_expect_tx(&b_full[s], kStageB);
                for (int h = 0; h < 2; ++h)
                    tma_load_3d(smem + lay.b + s * kStageB + h * kAtomB, &map_a, b * 256 + h * 128, tok0, 0,
                                &b_full[s]);
            }
            if (!ok) {
                abort_flag = 1;
                set_error(p.err, kDevErrTimeout);
            }
            // Every copy this CTA issued lands before it exits.
            for (int b = max(0, p.nblk - S); b < p.nblk; ++b) {
                mbar_wait(&raw_full[b % S], uint32_t(b / S) & 1u);
                mbar_wait(&b_full[b % S], uint32_t(b / S) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(kMmaRows, kMmaTok);
            for (int b = 0; b < p.nblk; ++b) {
                const int s = b % S, buf = b & 1;
                if (!mbar_wait(&a_full[buf], uint32_t(b >> 1) & 1u) ||
                    !mbar_wait(&b_full[s], uint32_t(b / S) & 1u) || abort_flag) {
                    abort_flag = 1;
                    set_error(p.err, kDevErrTimeout);
                    break;
                }
                fence_after_sync();
                const uint32_t a_lo = smem_addr(smem + lay.a + buf * kBufA), a_hi = a_lo + kOperandA;
                const uint32_t bs = smem_addr(smem + lay.b + s * kStageB);
#pragma unroll
                for (int k = 0; k < 8; ++k) {  // K-steps of 32 bytes
                    const uint32_t off = (k >> 2) * kAtomA + (k & 3) * 32;
                    const uint64_t bd = smem_desc_sw128(bs + (k >> 2) * kAtomB + (k & 3) * 32, 16, 1024);
                    mma_i8(tmem + buf * 64, smem_desc_sw128(a_lo + off, 16, 1024), bd, idesc, k > 0 ? 1u : 0u);
                    mma_i8(tmem + buf * 64 + 32, smem_desc_sw128(a_hi + off, 16, 1024), bd, idesc,
                           k > 0 ? 1u : 0u);
                }
                mma_commit(&mma_done[buf]);
                mma_commit(&b_empty[s]);
            }
        }
    } else {
        // ---------------------------------------------------------- unpack + epilogue
        const int g = (warp - 2) >> 2;      // sub-blocks 4g..4g+3, tokens 16g..16g+15
        const int q = warp & 3;             // TMEM lane quarter
        const int r = 32 * q + lane;        // weight row within the tile
        const uint32_t lane_addr = uint32_t(32 * q) << 16;
        float total[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) total[t] = 0.f;
        int mn_prev[8];
        uint32_t dm_prev = 0;
        bool ok = true;
        auto epilogue = [&](int b, const int (&mn)[8], uint32_t dm) {
            const int buf = b & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&mma_done[buf], uint32_t(b >> 1) & 1u))) {
                ok = false;
                return;
            }
            fence_after_sync();
            uint32_t lo[16], hi[16];
            tmem_ld16(tmem + lane_addr + buf * 64 + 16 * g, lo);
            tmem_ld16(tmem + lane_addr + buf * 64 + 32 + 16 * g, hi);
            tmem_wait_ld();
            const float d16 = half_bits(dm), dmin16 = half_bits(dm >> 16);
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                const int i = (16 * g + t) * p.nblk + b;
                const uint4 pw = *reinterpret_cast<const uint4 *>(ps + i * 8);
                const uint32_t pv[4] = {pw.x, pw.y, pw.z, pw.w};
                int minimum = 0;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    minimum += mn[2 * j] * int(int16_t(pv[j] & 0xffffu));
                    minimum += mn[2 * j + 1] * int(int16_t(pv[j] >> 16));
                }
                const int weighted = int(lo[t]) + 8 * int(hi[t]);
                const float as = scl[i];
                const float d = d16 * as;
                const float dmin = dmin16 * as;
                total[t] = total[t] + (d * float(weighted) - dmin * float(minimum));
            }
        };
        for (int b = 0; b < p.nblk && ok; ++b) {
            const int s = b % S, buf = b & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[s], uint32_t(b / S) & 1u))) {
                ok = false;
                break;
            }
            const unsigned char *w = smem + lay.raw + s * p.raw_bytes + r * bb;
            const uint32_t dm = *reinterpret_cast<const uint32_t *>(w);
            const uint32_t sw[3] = {*reinterpret_cast<const uint32_t *>(w + 4),
                                    *reinterpret_cast<const uint32_t *>(w + 8),
                                    *reinterpret_cast<const uint32_t *>(w + 12)};
            auto sb = [&](int k) { return int((sw[k >> 2] >> (8 * (k & 3))) & 0xffu); };
            int sc[8], mn[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {  // scale_min_k4, tensor.rs:23-32
                if (j < 4) {
                    sc[j] = sb(j) & 63;
                    mn[j] = sb(j + 4) & 63;
                } else {
                    sc[j] = (sb(j + 4) & 15) | ((sb(j - 4) >> 6) << 4);
                    mn[j] = (sb(j + 4) >> 4) | ((sb(j) >> 6) << 4);
                }
            }
            uint32_t hb[8] = {};
            if constexpr (T == Q38_GGML_Q5_K) {
                const uint4 h0 = *reinterpret_cast<const uint4 *>(w + 16), h1 = *reinterpret_cast<const uint4 *>(w + 32);
                hb[0] = h0.x, hb[1] = h0.y, hb[2] = h0.z, hb[3] = h0.w;
                hb[4] = h1.x, hb[5] = h1.y, hb[6] = h1.z, hb[7] = h1.w;
            }
            constexpr uint32_t qs_off = T == Q38_GGML_Q4_K ? 16 : 48;
            unsigned char *alo = smem + lay.a + buf * kBufA + g * kAtomA, *ahi = alo + kOperandA;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {  // byte chunk c = 2g + cc holds sub-blocks 2c, 2c+1
                const int c = 2 * g + cc;
                const uint4 v0 = *reinterpret_cast<const uint4 *>(w + qs_off + 32 * c);
                const uint4 v1 = *reinterpret_cast<const uint4 *>(w + qs_off + 32 * c + 16);
                const uint32_t qw[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                for (int half = 0; half < 2; ++half) {  // low nibbles: sub-block 2c, high: 2c+1
                    const int j = 2 * c + half;
                    const uint32_t slo = uint32_t(sc[j] & 7), shi = uint32_t(sc[j] >> 3);
                    uint32_t lw[8], hw[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        uint32_t v = (qw[k] >> (4 * half)) & 0x0f0f0f0fu;
                        if constexpr (T == Q38_GGML_Q5_K) v |= ((hb[k] >> j) & 0x01010101u) << 4;
                        lw[k] = v * slo;  // bytes <= 31 * 7: no carry between bytes
                        hw[k] = v * shi;
                    }
                    const uint32_t u0 = 2 * (j - 4 * g);  // 16-byte chunk within the atom
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t o = sw128_chunk(uint32_t(r), u0 + h);
                        *reinterpret_cast<uint4 *>(alo + o) = make_uint4(lw[4 * h], lw[4 * h + 1], lw[4 * h + 2], lw[4 * h + 3]);
                        *reinterpret_cast<uint4 *>(ahi + o) = make_uint4(hw[4 * h], hw[4 * h + 1], hw[4 * h + 2], hw[4 * h + 3]);
                    }
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&raw_empty[s]);
                mbar_arrive(&a_full[buf]);
            }
            if (b > 0) {
                epilogue(b - 1, mn_prev, dm_prev);
                if (!ok) break;
                fence_before_sync();  // TMEM reads done before the next a_full arrive reuses the buffer
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) mn_prev[j] = mn[j];
            dm_prev = dm;
        }
        if (ok) epilogue(p.nblk - 1, mn_prev, dm_prev);
        if (!ok) {
            if (lane == 0) {
                abort_flag = 1;
                set_error(p.err, kDevErrTimeout);
            }
        } else if (row0 + r < p.rows) {
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                const int tok = tok0 + 16 * g + t;
                if (tok < p.batch) p.out[size_t(tok) * p.out_ld + row0 + r] = total[t];
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 1) tmem_dealloc(tmem, kMmaTmemCols);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_proj() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// 3-D uint8 map over [1][rows][cols] bytes with a box of box_cols x box_rows.
bool make_map_u8(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                 uint32_t box_rows, bool swizzle) {
    auto enc = encode_tiled_proj();
    if (!enc) return false;
    cuuint64_t dims[3] = {cols, rows, 1};
    cuuint64_t strides[2] = {cols, cols * rows};
    cuuint32_t box[3] = {box_cols, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int T>
cudaError_t launch_mma(const CUtensorMap &mw, const CUtensorMap &ma, const MmaParams &p, cudaStream_t stream) {
    const MmaSmem lay = mma_smem_plan(p.stages, p.raw_bytes, p.nblk);
    const size_t smem = lay.total + 1024;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(proj_mma_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kProjSmemBudget));
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((p.rows + kMmaRows - 1) / kMmaRows, (p.batch + kMmaTok - 1) / kMmaTok);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, proj_mma_kernel<T>, mw, ma, p);
}

}  // namespace

bool proj_mma_supported(int type) { return type == Q38_GGML_Q4_K || type == Q38_GGML_Q5_K; }

size_t proj_mma_scratch_bytes(int batch, int64_t width) {
    const size_t nb = size_t(batch) * size_t(width / 256);
    return nb * 256 + nb * 4 + nb * 32;
}

cudaError_t launch_proj_mma(const ProjWeight &w, const float *x, int batch, float *out, long out_ld,
                            int *err, void *scratch, cudaStream_t stream) {
    if (!proj_mma_supported(w.type) || w.width % 256 || w.row_bytes % 16) return cudaErrorInvalidValue;
    const int nblk = int(w.width / 256);
    const size_t nb = size_t(batch) * nblk;
    unsigned char *sp = static_cast<unsigned char *>(scratch);
    Q8KActivations act;
    act.quants = reinterpret_cast<int8_t *>(sp);
    act.scale = reinterpret_cast<float *>(sp + nb * 256);
    act.sums = reinterpret_cast<int16_t *>(sp + nb * 256 + nb * 4);
    cudaError_t e = launch_q8k_quantize(x, batch, int(w.width), act, nullptr, stream);
    if (e != cudaSuccess) return e;
    const uint32_t bb = w.type == Q38_GGML_Q4_K ? 144 : 176;
    CUtensorMap mw, ma;
    if (!make_map_u8(&mw, w.data, uint64_t(w.row_bytes), uint64_t(w.rows), bb, kMmaRows, false) ||
        !make_map_u8(&ma, act.quants, uint64_t(w.width), uint64_t(batch), 128, kMmaTok, true))
        return cudaErrorInvalidValue;
    MmaParams p{};
    p.scale = act.scale;
    p.sums = act.sums;
    p.out = out;
    p.err = err;
    p.out_ld = out_ld;
    p.rows = int(w.rows);
    p.nblk = nblk;
    p.batch = batch;
    p.raw_bytes = kMmaRows * bb;
    const uint32_t fixed = mma_smem_plan(0, p.raw_bytes, nblk).total + 1024;
    p.stages = std::min<int>(kMaxMmaStages, int((kProjSmemBudget - fixed) / (p.raw_bytes + kStageB)));
    if (p.stages < 2) return cudaErrorInvalidValue;
    return w.type == Q38_GGML_Q4_K ? launch_mma<Q38_GGML_Q4_K>(mw, ma, p, stream)
                                   : launch_mma<Q38_GGML_Q5_K>(mw, ma, p, stream);
}

}  // namespace q38
