// proj_planes.cu -- K-quant projections of many tokens from integer planes
// built once at upload, on the tensor cores (tcgen05.mma kind::i8),
// bit-identical to the reference's integer path.
//
// The reference's K-quant dot (dot_q4_k_q8_k_scalar, dot_q5_k_q8_k_scalar,
// dot_q6_k_q8_k_scalar, src/kernel/tensor.rs:365-460) forms per 256-block
//   weighted = sum over the block's values of scale(value) * quant(value) * a
//   minimum  = sum over 32-value sub-blocks of min(sub) * (activation sum of
//              the sub-block)                      (Q4_K / Q5_K only)
// and adds d*weighted - dmin*minimum (f32, d and dmin times the activation
// block scale) to a running total in block order. Both are integers, so any
// exact way of forming them gives the reference's bits.
//
// Two plane forms, both exact, no operand building at run time:
//   Q4_K / Q5_K  quant planes: one byte q (0..31) per weight value. A K-step
//                of a kind::i8 MMA covers 32 values, exactly one sub-block,
//                so each sub-block's integer dot D_j lands in its own
//                accumulator and the epilogue forms weighted = sum_j sc_j D_j
//                in integers. The 16-byte side record per (row, block) is the
//                block's own header: d, dmin and the 12 packed 6-bit scales
//                and mins; `minimum` comes from the mins and the
//                activations' group sums (dp2a).
//   Q6_K         product planes: its scales cover 16 values, half a K-step,
//                so the product p = sc * (q - 32) (-4064..4096) is stored as
//                lo = p & 255 (u8) and hi = p >> 8 (s8): weighted = D_lo +
//                256 D_hi from two accumulators; the 4-byte side record holds
//                d.
// HBM cost per weight: 1 byte (quant planes: 1.8x the Q4_K bytes) or 2 bytes
// (product planes: 2.4x Q6_K), plus the side records, in exchange for a
// projection that streams them. Built on request (q38_weight_build_planes);
// without planes, projections keep the operand-building kernel of
// proj_mma.cu.
//
// Plane layout: the kernel's K loop runs in steps of 32 KB of planes per
// 128-row tile -- a whole block of quant planes (two atoms of 128 values), or
// half a block of product planes (its lo and hi atoms). An atom is 128 rows x
// 128 B already in the SW128 K-major layout of a tcgen05 operand (16-byte
// chunk u of row r at chunk u ^ (r % 8)). Steps are stored step-major,
// [step][row tile][32 KB]: one bulk copy fills a stage, and at each step the
// CTAs together read one contiguous slab. (Bulk copies cost a roughly fixed
// ~0.3 us each on an SM: 16 KB copies capped a CTA near 58 GB/s, 32 KB ones
// reached ~120 GB/s.) The side records are tile-major, [row tile][block][128
// rows], so a CTA copies all of its own into shared memory once.
//
// CTA: 128 weight rows x 32 (or 16) tokens, 19 warps.
//   warp 0      copies: a step's 32 KB of planes (one bulk copy; the first
//               stages before the programmatic-dependent wait, weights are
//               constant) and its activation quants [32 tokens][128 B] per
//               atom (TMA, SW128).
//   warps 1, 2  MMA issue, kind::i8 (M=128, N=32, K=32): quant planes, warp
//               1 + c the 4 sub-blocks of atom c, each K-step into its own 32
//               columns (256 columns a block, two buffers); product planes,
//               warp 1 chain lo and warp 2 chain hi, each accumulating over
//               the block (64 columns a block, four buffers).
//   warps 3-18  epilogue (warps 3-10 for 16 tokens): thread = weight row
//               (TMEM lane quarter = warp % 4), 8 tokens per warp; per block
//               the f32 term per (row, token), added in block order.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "q38_proj.h"
#include "q38_sm100.cuh"

namespace q38 {
namespace {

constexpr int kPlRows = 128;
constexpr int kPlEpiWarp0 = 3;
constexpr int kPlThreads = 32 * (kPlEpiWarp0 + 16);
constexpr uint32_t kPlAtomA = kPlRows * 128;               // a plane atom: 128 rows x 128 B
constexpr uint32_t kPlStepPlanes = 2 * kPlAtomA;           // 32 KB of planes per step
constexpr int kPlMaxStages = 8;
constexpr int kPlLargeBatch = 128;  // tokens from which 64-token tiles are used

// The two plane forms (see the file comment), for token tiles of kTok = 16,
// 32 or 64: 32 for decode batches; 16 when a matrix of few row tiles splits
// its tokens over two CTAs so that more SMs stream it (the second CTA's
// plane reads mostly hit L2); 64 for prompt-sized batches, where each CTA's
// planes serve twice the tokens (quant planes then fill TMEM with one
// block's 8 x 64 accumulators, so MMA and epilogue alternate).
template <int T, int kTok>
struct PlForm {
    static constexpr bool kQuant = T != Q38_GGML_Q6_K;         // quant planes
    static constexpr int kStepValues = kQuant ? 256 : 128;      // K values per step
    static constexpr int kStepAct = kQuant ? 2 : 1;             // activation atoms per step
    static constexpr uint32_t kAtomB = kTok * 128;              // an activation atom: kTok tokens x 128 B
    static constexpr uint32_t kStage = kPlStepPlanes + kStepAct * kAtomB;
    static constexpr uint32_t kAccCols = kQuant ? 8 * kTok : 2 * kTok;
    static constexpr int kAcc = int(512 / kAccCols) > 4 ? 4 : int(512 / kAccCols);  // accumulator buffers
    static constexpr uint32_t kTmemCols = kAcc * kAccCols;      // <= 512
    static constexpr uint32_t kSide = kQuant ? 16 : 4;          // side record bytes
    static constexpr int kEpiWarps = kTok >= 32 ? 16 : 8;       // 4 lane quarters x token groups
    static constexpr int kTokPerWarp = kTok * 4 / kEpiWarps;    // 8 or 16
    static_assert(kTmemCols == 128 || kTmemCols == 256 || kTmemCols == 512, "TMEM allocation");
};
constexpr bool plane_quant(int type) { return type != Q38_GGML_Q6_K; }
constexpr uint32_t plane_side_bytes(int type) { return plane_quant(type) ? 16 : 4; }
constexpr int plane_bytes_per_value(int type) { return plane_quant(type) ? 1 : 2; }

__host__ __device__ constexpr uint32_t pl_idesc_i8(int M, int N, bool a_signed) {
    return (2u << 4) | (uint32_t(a_signed ? 1 : 0) << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void pl_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void pl_tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ float pl_half(uint32_t h) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xffffu)));
}

// ---- plane building (once per weight) --------------------------------------
// Grid (rows, blocks), 256 threads: thread v = value v of the block, the
// reference's value order (the Q8_K quant it multiplies).
template <int T>
__global__ void __launch_bounds__(256) planes_build_kernel(const unsigned char *raw, int64_t row_bytes,
                                                           unsigned char *planes, unsigned char *side,
                                                           int64_t width) {
    using F = PlForm<T, 32>;
    const int b = blockIdx.y, v = threadIdx.x;
    const int64_t row = blockIdx.x;
    const int nblk = int(width / 256);
    const size_t tiles = size_t(gridDim.x + kPlRows - 1) / kPlRows;
    const uint32_t r = uint32_t(row & (kPlRows - 1));
    const int k = v & 127;  // value within its 128-value half
    const size_t in_atom = r * 128u + (((uint32_t(k) >> 4) ^ (r & 7u)) << 4) + (k & 15);
    // Step s of row tile rt at [s][rt][32 KB]; atom a of the step at a * 16 KB.
    auto at = [&](int s, int a) {
        return planes + (size_t(s) * tiles + size_t(row / kPlRows)) * kPlStepPlanes + size_t(a) * kPlAtomA + in_atom;
    };
    unsigned char *rec_at = side + ((size_t(row / kPlRows) * nblk + b) * kPlRows + r) * F::kSide;
    if constexpr (T == Q38_GGML_Q6_K) {
        // Q6_K (tensor.rs:430-460; device block padded to 224 bytes): value
        // 128h + 32k + i takes the low (k < 2) or high nibble of
        // ql[64h + 32(k&1) + i], bits 2k..2k+1 of qh[32h + i], scale
        // sc[8h + 2k + i/16].
        const unsigned char *blk = raw + row * row_bytes + size_t(b) * kQ6KDeviceBlock;
        const int h = v >> 7, kk = (v >> 5) & 3, i = v & 31;
        const unsigned char l = blk[64 * h + 32 * (kk & 1) + i];
        const int lo4 = kk >= 2 ? (l >> 4) : (l & 15);
        const int hb = (blk[128 + 32 * h + i] >> (2 * kk)) & 3;
        const int q = lo4 | (hb << 4);
        const int sc = int(int8_t(blk[192 + 8 * h + 2 * kk + i / 16]));
        const int p = sc * (q - 32);
        *at(2 * b + h, 0) = static_cast<unsigned char>(p & 255);
        *at(2 * b + h, 1) = static_cast<unsigned char>((p >> 8) & 255);  // s8
        if (v == 0) *reinterpret_cast<uint32_t *>(rec_at) = uint32_t(blk[208]) | (uint32_t(blk[209]) << 8);
    } else {
        // Q4_K / Q5_K (tensor.rs:365-428): value 32j + i of sub-block j takes
        // the low (j even) or high nibble of qs[32(j/2) + i] (Q5_K: plus 16 if
        // bit j of qh[i] is set). The side record is the block's first 16
        // bytes: d, dmin, the packed scales and mins.
        constexpr bool kQ5 = T == Q38_GGML_Q5_K;
        constexpr int kBytes = kQ5 ? 176 : 144;
        const unsigned char *blk = raw + row * row_bytes + size_t(b) * kBytes;
        const int j = v >> 5, i = v & 31;
        const unsigned char *qs = blk + (kQ5 ? 48 : 16);
        int q = (qs[32 * (j >> 1) + i] >> (4 * (j & 1))) & 15;
        if constexpr (kQ5) q += (blk[16 + i] >> j) & 1 ? 16 : 0;
        *at(b, v >> 7) = static_cast<unsigned char>(q);
        if (v < 16) rec_at[v] = blk[v];
    }
}

// ---- the projection ---------------------------------------------------------
struct PlParams {
    const unsigned char *planes;  // step-major (see the file comment)
    const float *scale;           // [batch][nblk] activation block scales
    const int16_t *sums;          // [batch][nblk][16] activation group sums
    const unsigned char *side;    // [row tiles][nblk][128] side records
    float *out;                   // out[t * out_ld + row]
    int *err;
    long out_ld;
    ProjEpilogue epi;
    int rows, nblk, batch, stages;
};

struct PlSmem {
    uint32_t stage, side, psum, scl, total;
};

// side_bytes: the form's record size; psum: whether the group-sum table is
// needed (quant planes).
__host__ __device__ inline PlSmem pl_smem_plan(int stages, int nblk, uint32_t stage_bytes,
                                               uint32_t side_bytes, bool psum, int tok) {
    PlSmem s{};
    s.stage = 0;
    s.side = uint32_t(stages) * stage_bytes;                           // [nblk][128 rows] records
    s.psum = s.side + (uint32_t(nblk) * kPlRows * side_bytes + 15) / 16 * 16;
    s.scl = s.psum + (psum ? uint32_t(nblk) * tok * 16 : 0);          // psum: [nblk][tok] x 4 words
    s.total = s.scl + uint32_t(nblk) * tok * 4;                       // scl: [nblk][tok] f32
    return s;
}

// Byte k of the 12 packed scale bytes held in words y, z, w of a side record.
__device__ __forceinline__ int pl_sbyte(const uint4 &rec, int k) {
    const uint32_t w = k < 4 ? rec.y : k < 8 ? rec.z : rec.w;
    return int((w >> (8 * (k & 3))) & 0xffu);
}

template <int T, int kTok>
__global__ void __launch_bounds__(kPlThreads, 1)
    proj_planes_kernel(const __grid_constant__ CUtensorMap map_a, PlParams p) {
    using namespace sm100;
    using F = PlForm<T, kTok>;
    constexpr bool kQ = F::kQuant;
    constexpr uint32_t kStage = F::kStage;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[kPlMaxStages], empty[kPlMaxStages];
    __shared__ __align__(8) uint64_t acc_full[F::kAcc], acc_empty[F::kAcc], side_full;
    __shared__ uint32_t tmem_base_s;
    __shared__ volatile int abort_flag;
    const int S = p.stages;
    const PlSmem lay = pl_smem_plan(S, p.nblk, kStage, F::kSide, kQ, kTok);
    uint4 *psum = reinterpret_cast<uint4 *>(smem + lay.psum);
    const unsigned char *side_s = smem + lay.side;
    float *scl = reinterpret_cast<float *>(smem + lay.scl);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * kPlRows, tok0 = blockIdx.y * kTok;
    const int steps = p.nblk * 256 / F::kStepValues;
    // This CTA's planes: step s at stripe + s * step_stride.
    const unsigned char *stripe = p.planes + size_t(blockIdx.x) * kPlStepPlanes;
    const size_t step_stride = size_t(gridDim.x) * kPlStepPlanes;

    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2);  // one commit per issuing warp
        }
        for (int a = 0; a < F::kAcc; ++a) {
            mbar_init(&acc_full[a], 2);
            mbar_init(&acc_empty[a], F::kEpiWarps);
        }
        mbar_init(&side_full, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_s, F::kTmemCols);
        tmem_relinquish();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_base_s;
    const int first = min(S, steps);
    // Step s's activation atoms: values [s * kStepValues + 128 c, +128).
    auto load_act = [&](int s, int st) {
#pragma unroll
        for (int c = 0; c < F::kStepAct; ++c)
            tma_load_3d(smem + st * kStage + kPlStepPlanes + c * F::kAtomB, &map_a, s * F::kStepValues + 128 * c,
                        tok0, 0, &full[st]);
    };
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&map_a);
        // The planes are constant: this CTA's side records and the first
        // stages' planes are requested before the wait for the kernel that
        // quantized the activations.
        const uint32_t side_bytes = uint32_t(p.nblk) * kPlRows * F::kSide;
        mbar_arrive_expect_tx(&side_full, side_bytes);
        const unsigned char *side_g = p.side + size_t(blockIdx.x) * side_bytes;
        for (uint32_t off = 0; off < side_bytes; off += 16384)
            bulk_load(smem + lay.side + off, side_g + off, min(16384u, side_bytes - off), &side_full);
        for (int s = 0; s < first; ++s) {
            mbar_arrive_expect_tx(&full[s], kStage);
            bulk_load(smem + s * kStage, stripe + size_t(s) * step_stride, kPlStepPlanes, &full[s]);
        }
    }
    pdl_wait_primary();
    pdl_launch_dependents();
    // Per (block, token): the activation scale and, for quant planes, the
    // four packed pairs of sub-block sums (sub-block j = Q8_K groups 2j, 2j+1).
    for (int i = tid; i < kTok * p.nblk; i += kPlThreads) {
        const int b = i / kTok, t = i - b * kTok;
        const bool in = tok0 + t < p.batch;
        scl[i] = in ? p.scale[size_t(tok0 + t) * p.nblk + b] : 0.f;
        if constexpr (kQ) {
            uint4 w = make_uint4(0u, 0u, 0u, 0u);
            if (in) {
                // 16 int16 group sums as 8 words (lo half: group 2i, hi: 2i+1).
                const uint32_t *g = reinterpret_cast<const uint32_t *>(p.sums + (size_t(tok0 + t) * p.nblk + b) * 16);
                uint32_t gw[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) gw[k] = __ldg(g + k);
                uint32_t pw[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int s0 = int(int16_t(gw[2 * k] & 0xffffu)) + int(int16_t(gw[2 * k] >> 16));
                    const int s1 = int(int16_t(gw[2 * k + 1] & 0xffffu)) + int(int16_t(gw[2 * k + 1] >> 16));
                    pw[k] = (uint32_t(s0) & 0xffffu) | (uint32_t(s1) << 16);
                }
                w = make_uint4(pw[0], pw[1], pw[2], pw[3]);
            }
            psum[i] = w;
        }
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------------------ copies
        if (lane == 0) {
            bool ok = true;
            for (int s = 0; s < first; ++s) load_act(s, s);
            for (int s = first; s < steps && ok; ++s) {
                const int st = s % S;
                ok = mbar_wait(&empty[st], uint32_t(s / S - 1) & 1u) && !abort_flag;
                if (!ok) break;
                mbar_arrive_expect_tx(&full[st], kStage);
                bulk_load(smem + st * kStage, stripe + size_t(s) * step_stride, kPlStepPlanes, &full[st]);
                load_act(s, st);
            }
            if (!ok) {
                abort_flag = 1;
                set_error(p.err, kDevErrTimeout);
            }
            // Every copy this CTA issued lands before it exits.
            for (int s = max(0, steps - S); s < steps; ++s) mbar_wait(&full[s % S], uint32_t(s / S) & 1u);
            mbar_wait(&side_full, 0);
        }
    } else if (warp < kPlEpiWarp0) {
        // ------------------------------------------------------------ MMA
        // Quant planes: warp 1 + c takes atom c (sub-blocks 4c..4c+3) of each
        // block. Product planes: warp 1 + c runs chain c (lo, hi) over both
        // half-blocks of each block.
        const int c = warp - 1;
        if (lane == 0) {
            const uint32_t idesc = pl_idesc_i8(kPlRows, kTok, !kQ && c == 1);
            constexpr int kStepsPerBlock = 256 / F::kStepValues;
            for (int b = 0; b < p.nblk; ++b) {
                const int a = b % F::kAcc;
                if (b >= F::kAcc && !mbar_wait(&acc_empty[a], uint32_t(b / F::kAcc - 1) & 1u)) {
                    abort_flag = 1;
                    set_error(p.err, kDevErrTimeout);
                    break;
                }
                fence_after_sync();
                const uint32_t dacc = tmem + uint32_t(a) * F::kAccCols;
                bool ok = true;
#pragma unroll 1
                for (int h = 0; h < kStepsPerBlock; ++h) {
                    const int s = kStepsPerBlock * b + h, st = s % S;
                    if (!mbar_wait(&full[st], uint32_t(s / S) & 1u) || abort_flag) {
                        ok = false;
                        break;
                    }
                    fence_after_sync();
                    const uint32_t abase = smem_addr(smem + st * kStage + c * kPlAtomA);
                    const uint32_t bbase = smem_addr(smem + st * kStage + kPlStepPlanes + (kQ ? c * F::kAtomB : 0));
#pragma unroll
                    for (int k = 0; k < 4; ++k) {  // K-steps of 32 values within the atom
                        const uint64_t ad = smem_desc_sw128(abase + k * 32, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(bbase + k * 32, 16, 1024);
                        if constexpr (kQ)
                            // sub-block 4c + k into its own 32 columns
                            pl_mma_i8(dacc + uint32_t(4 * c + k) * kTok, ad, bd, idesc, 0u);
                        else
                            pl_mma_i8(dacc + uint32_t(c) * kTok, ad, bd, idesc, (h | k) ? 1u : 0u);
                    }
                    mma_commit(&empty[st]);
                }
                if (!ok) {
                    abort_flag = 1;
                    set_error(p.err, kDevErrTimeout);
                    break;
                }
                mma_commit(&acc_full[a]);
            }
        }
    } else if (warp < kPlEpiWarp0 + F::kEpiWarps) {
        // ------------------------------------------------------------ epilogue
        constexpr int kTPW = F::kTokPerWarp;
        const int e = warp - kPlEpiWarp0;
        const int quarter = warp & 3;  // the TMEM lanes this warp may read
        const int tg0 = (e >> 2) * kTPW;  // this warp's first token in the tile
        const uint32_t r = uint32_t(32 * quarter + lane);
        const uint32_t lane_addr = uint32_t(32 * quarter) << 16;
        float total[kTPW];
#pragma unroll
        for (int t = 0; t < kTPW; ++t) total[t] = 0.f;
        bool ok = __all_sync(0xffffffffu, mbar_wait(&side_full, 0));
        for (int b = 0; b < p.nblk && ok; ++b) {
            const int a = b % F::kAcc;
            uint4 cur;
            if constexpr (kQ)
                cur = reinterpret_cast<const uint4 *>(side_s)[b * kPlRows + r];
            else
                cur = make_uint4(reinterpret_cast<const uint32_t *>(side_s)[b * kPlRows + r], 0u, 0u, 0u);
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[a], uint32_t(b / F::kAcc) & 1u))) {
                ok = false;
                break;
            }
            fence_after_sync();
            const uint32_t dacc = tmem + lane_addr + uint32_t(a) * F::kAccCols;
            int sc[8];
            uint32_t mins0 = 0, mins1 = 0;
            if constexpr (kQ) {
                // scale_min_k4 (tensor.rs:23-32): the sub-blocks' scales and mins.
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    int mn;
                    if (j < 4) {
                        sc[j] = pl_sbyte(cur, j) & 63;
                        mn = pl_sbyte(cur, j + 4) & 63;
                    } else {
                        sc[j] = (pl_sbyte(cur, j + 4) & 15) | ((pl_sbyte(cur, j - 4) >> 6) << 4);
                        mn = (pl_sbyte(cur, j + 4) >> 4) | ((pl_sbyte(cur, j) >> 6) << 4);
                    }
                    if (j < 4)
                        mins0 |= uint32_t(mn) << (8 * j);
                    else
                        mins1 |= uint32_t(mn) << (8 * (j - 4));
                }
            }
            // This warp's tokens in chunks of 8: the block's integer sums
            // weighted (and minimum) per token, then the f32 term.
            int weighted[kTPW];
#pragma unroll
            for (int tc = 0; tc < kTPW; tc += 8) {
                const uint32_t col = uint32_t(tg0 + tc);
                if constexpr (kQ) {
                    // weighted = sum_j sc_j D_j
#pragma unroll
                    for (int t = 0; t < 8; ++t) weighted[tc + t] = 0;
#pragma unroll
                    for (int jh = 0; jh < 2; ++jh) {
                        uint32_t D[4][8];
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) pl_tmem_ld8(dacc + uint32_t(4 * jh + jj) * kTok + col, D[jj]);
                        tmem_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                            for (int t = 0; t < 8; ++t) weighted[tc + t] += sc[4 * jh + jj] * int(D[jj][t]);
                    }
                } else {
                    uint32_t dlo[8], dhi[8];
                    pl_tmem_ld8(dacc + col, dlo);
                    pl_tmem_ld8(dacc + kTok + col, dhi);
                    tmem_wait_ld();
#pragma unroll
                    for (int t = 0; t < 8; ++t) weighted[tc + t] = int(dlo[t]) + 256 * int(dhi[t]);
                }
            }
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
#pragma unroll
            for (int tc = 0; tc < kTPW; tc += 8) {
                const float4 s0 = *reinterpret_cast<const float4 *>(scl + b * kTok + tg0 + tc);
                const float4 s1 = *reinterpret_cast<const float4 *>(scl + b * kTok + tg0 + tc + 4);
                const float as[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const float d = pl_half(cur.x) * as[t];
                    float term;
                    if constexpr (kQ) {
                        const uint4 ps = psum[b * kTok + tg0 + tc + t];
                        int minimum = __dp2a_lo(int(ps.x), int(mins0), 0);
                        minimum = __dp2a_hi(int(ps.y), int(mins0), minimum);
                        minimum = __dp2a_lo(int(ps.z), int(mins1), minimum);
                        minimum = __dp2a_hi(int(ps.w), int(mins1), minimum);
                        const float dmin = pl_half(cur.x >> 16) * as[t];
                        term = d * float(weighted[tc + t]) - dmin * float(minimum);
                    } else {
                        term = d * float(weighted[tc + t]);
                    }
                    total[tc + t] = total[tc + t] + term;
                }
            }
        }
        if (!ok) {
            if (lane == 0) {
                abort_flag = 1;
                set_error(p.err, kDevErrTimeout);
            }
        } else if (row0 + int(r) < p.rows) {
            // In chunks of 8 tokens: all the chunk's epilogue inputs first, then
            // its outputs.
#pragma unroll
            for (int tc = 0; tc < kTPW; tc += 8) {
                EpilogueIn ein[8];
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const int tok = tok0 + tg0 + tc + t;
                    if (tok < p.batch) ein[t] = proj_epilogue_load(p.epi, p.rows, tok, int(row0 + r));
                }
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const int tok = tok0 + tg0 + tc + t;
                    if (tok < p.batch)
                        p.out[size_t(tok) * p.out_ld + row0 + r] =
                            proj_epilogue_apply(p.epi, ein[t], p.rows, tok, int(row0 + r), total[tc + t]);
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 1) tmem_dealloc(tmem, F::kTmemCols);
}

PFN_cuTensorMapEncodeTiled_v12000 pl_encode_tiled() {
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

// 3-D uint8 map over [1][rows][cols] bytes, box 128 B x box_rows, SW128.
bool pl_map_u8(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
    auto enc = pl_encode_tiled();
    if (!enc) return false;
    cuuint64_t dims[3] = {cols, rows, 1};
    cuuint64_t strides[2] = {cols, cols * rows};
    cuuint32_t box[3] = {128, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// As many stages as the shared-memory budget holds (at least 2); 0: none fit.
int pl_stages_for(int type, int nblk, int tok) {
    const bool quant = plane_quant(type);
    const uint32_t stage = kPlStepPlanes + (quant ? 2 : 1) * uint32_t(tok) * 128;
    for (int s = kPlMaxStages; s >= 2; --s)
        if (pl_smem_plan(s, nblk, stage, plane_side_bytes(type), quant, tok).total + 1024 <= kProjSmemBudget)
            return s;
    return 0;
}

template <int T, int kTok>
cudaError_t launch_planes_typed(const CUtensorMap &ma, const PlParams &p, cudaStream_t stream) {
    using F = PlForm<T, kTok>;
    const size_t smem = pl_smem_plan(p.stages, p.nblk, F::kStage, F::kSide, F::kQuant, kTok).total + 1024;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(proj_planes_kernel<T, kTok>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kProjSmemBudget));
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((p.rows + kPlRows - 1) / kPlRows, (p.batch + kTok - 1) / kTok);
    cfg.blockDim = dim3(kPlThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, proj_planes_kernel<T, kTok>, ma, p);
}

}  // namespace

bool proj_planes_type(int type) {
    return type == Q38_GGML_Q4_K || type == Q38_GGML_Q5_K || type == Q38_GGML_Q6_K;
}

int64_t proj_plane_rows(int64_t rows) { return (rows + kPlRows - 1) / kPlRows * kPlRows; }

size_t proj_plane_bytes(int type, int64_t rows, int64_t width) {
    const size_t rp = size_t(proj_plane_rows(rows));
    return size_t(plane_bytes_per_value(type)) * rp * size_t(width) +
           size_t(width / 256) * rp * plane_side_bytes(type);
}

cudaError_t build_proj_planes(ProjWeight &w, cudaStream_t stream) {
    if (!proj_planes_type(w.type) || w.width % 256 || pl_stages_for(w.type, int(w.width / 256), 32) == 0)
        return cudaErrorInvalidValue;
    if (w.planes) return cudaSuccess;
    const int64_t rp = proj_plane_rows(w.rows);
    const size_t atoms_bytes = size_t(plane_bytes_per_value(w.type)) * size_t(rp) * size_t(w.width);
    const size_t bytes = proj_plane_bytes(w.type, w.rows, w.width);
    unsigned char *buf = nullptr;
    cudaError_t e = cudaMalloc(&buf, bytes);
    if (e != cudaSuccess) return e;
    // Rows past the matrix stay zero (their outputs are never stored).
    if ((e = cudaMemsetAsync(buf, 0, bytes, stream)) != cudaSuccess) {
        cudaFree(buf);
        return e;
    }
    const dim3 grid(unsigned(w.rows), unsigned(w.width / 256));
    const unsigned char *raw = static_cast<const unsigned char *>(w.data);
    unsigned char *planes = buf, *side = buf + atoms_bytes;
    switch (w.type) {
        case Q38_GGML_Q4_K:
            planes_build_kernel<Q38_GGML_Q4_K><<<grid, 256, 0, stream>>>(raw, w.row_bytes, planes, side, w.width);
            break;
        case Q38_GGML_Q5_K:
            planes_build_kernel<Q38_GGML_Q5_K><<<grid, 256, 0, stream>>>(raw, w.row_bytes, planes, side, w.width);
            break;
        default:
            planes_build_kernel<Q38_GGML_Q6_K><<<grid, 256, 0, stream>>>(raw, w.row_bytes, planes, side, w.width);
            break;
    }
    if ((e = cudaGetLastError()) == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        cudaFree(buf);
        return e;
    }
    w.planes = planes;
    w.plane_side = side;
    w.plane_rows = rp;
    return cudaSuccess;
}

void free_proj_planes(ProjWeight &w) {
    cudaFree(w.planes);  // one allocation: planes | side records
    w.planes = w.plane_side = nullptr;
    w.plane_rows = 0;
}

cudaError_t launch_proj_planes(const ProjWeight &w, const float *x, int batch, float *out, long out_ld,
                               int *err, void *scratch, cudaStream_t stream, const ProjEpilogue &epi,
                               bool prequantized, int sm_budget) {
    if (!w.planes || w.width % 256) return cudaErrorInvalidValue;
    const int nblk = int(w.width / 256);
    // 16-token tiles when the batch fits one, or when twice the 32-token grid
    // still fits the SMs this launch may take; 64-token tiles for prompt-sized
    // batches (when their stages fit); else 32.
    const int tiles = int((w.rows + kPlRows - 1) / kPlRows);
    int tok = batch <= 16 || 2 * tiles * ((batch + 31) / 32) <= sm_budget ? 16 : 32;
    if (batch >= kPlLargeBatch && pl_stages_for(w.type, nblk, 64) > 0) tok = 64;
    const int stages = pl_stages_for(w.type, nblk, tok);
    if (stages == 0) return cudaErrorInvalidValue;
    cudaError_t e = cudaSuccess;
    if (!prequantized && (e = launch_proj_mma_quantize(x, batch, w.width, scratch, stream)) != cudaSuccess)
        return e;
    // The scratch's layout (launch_proj_mma_quantize): quants [batch][nblk][256],
    // scales [batch][nblk], group sums [batch][nblk][16].
    const size_t nb = size_t(batch) * size_t(nblk);
    unsigned char *sp = static_cast<unsigned char *>(scratch);
    CUtensorMap ma;
    if (!pl_map_u8(&ma, sp, uint64_t(w.width), uint64_t(batch), uint32_t(tok))) return cudaErrorInvalidValue;
    PlParams p{};
    p.planes = static_cast<const unsigned char *>(w.planes);
    p.scale = reinterpret_cast<const float *>(sp + nb * 256);
    p.sums = reinterpret_cast<const int16_t *>(sp + nb * 256 + nb * 4);
    p.side = static_cast<const unsigned char *>(w.plane_side);
    p.out = out;
    p.err = err;
    p.out_ld = out_ld;
    p.epi = epi;
    p.rows = int(w.rows);
    p.nblk = nblk;
    p.batch = batch;
    p.stages = stages;
    if (tok == 16) {
        switch (w.type) {
            case Q38_GGML_Q4_K: return launch_planes_typed<Q38_GGML_Q4_K, 16>(ma, p, stream);
            case Q38_GGML_Q5_K: return launch_planes_typed<Q38_GGML_Q5_K, 16>(ma, p, stream);
            default: return launch_planes_typed<Q38_GGML_Q6_K, 16>(ma, p, stream);
        }
    }
    if (tok == 64) {
        switch (w.type) {
            case Q38_GGML_Q4_K: return launch_planes_typed<Q38_GGML_Q4_K, 64>(ma, p, stream);
            case Q38_GGML_Q5_K: return launch_planes_typed<Q38_GGML_Q5_K, 64>(ma, p, stream);
            default: return launch_planes_typed<Q38_GGML_Q6_K, 64>(ma, p, stream);
        }
    }
    switch (w.type) {
        case Q38_GGML_Q4_K: return launch_planes_typed<Q38_GGML_Q4_K, 32>(ma, p, stream);
        case Q38_GGML_Q5_K: return launch_planes_typed<Q38_GGML_Q5_K, 32>(ma, p, stream);
        default: return launch_planes_typed<Q38_GGML_Q6_K, 32>(ma, p, stream);
    }
}

}  // namespace q38
