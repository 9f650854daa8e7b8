// proj_mma.cu -- K-quant projections of many tokens on the tensor cores
// (tcgen05.mma kind::i8), bit-identical to the reference's integer path.
//
// The reference's dot of a K-quant row with Q8_K activations
// (dot_q4_k_q8_k_scalar, dot_q5_k_q8_k_scalar, dot_q6_k_q8_k_scalar,
// src/kernel/tensor.rs:365-460) forms per 256-block an integer `weighted`
// (and, for Q4_K / Q5_K, `minimum`) and adds the f32 term
// d*weighted - dmin*minimum to a running total in block order. Both integers
// are sums over the block's 256 values of (small integer per value) x
// (activation quant), with a per-sub-block scale inside. Writing the scale as
// a few small non-negative digits makes every factor a byte, so each integer
// is an exact combination of u8 x s8 -> s32 products over the whole block --
// one tcgen05 accumulator ("chain") each:
//   Q4_K, Q5_K (q 0..31, 6-bit sc, 6-bit mn per 32 values):
//     chains q*(sc&7), q*(sc>>3), mn        weighted = D0 + 8 D1, minimum = D2
//   Q6_K (value q-32 with q 0..63, signed 8-bit sc per 16 values), sc in
//     two's-complement 2-bit digits d0..d3:
//     chains (q-32)*d_k (s8) for k<4       weighted = D0 + 4 D1 + 16 D2 + 64 D3
// A packed word of four values times a 2- or 3-bit digit keeps every byte
// below 256, so one integer multiply forms four operand bytes. The epilogue
// combines the chains and adds the f32 term exactly as the reference does.
//
// CTA: 128 weight rows x 32 tokens, 21 warps; the K loop runs in blocks (two
// SW128 atoms of 128 values per chain).
//   warp 0      TMA: raw weight blocks [128 rows][block bytes] (the first ones
//               before the programmatic-dependent wait: weights are constant;
//               up to 6 stages, and L2 prefetches a further 4 blocks ahead)
//               and the activation quants [32 tokens][256] (SW128).
//   warps 1-4   warp 1 + c issues chain c: per block 8 K-steps of
//               kind::i8 MMAs (M=128, N=32, K=32) into the chain's
//               accumulator (two blocks' worth of columns, alternating); a
//               thread waits on each issue, so the chains issue in parallel.
//               Warp 1 also allocates TMEM.
//   warps 5-20  thread = weight row (TMEM lane); four groups of four warps:
//               group g builds values 32g..32g+31 of each half-block and
//               finishes tokens 8g..8g+7; a block's MMAs overlap the
//               previous block's epilogue. (Separate build and epilogue warps
//               measured slower: the operand build is the binding cost.)
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "q38_proj.h"
#include "q38_sm100.cuh"

namespace q38 {
namespace {

constexpr int kMmaRows = 128;
constexpr int kMmaTok = 32;
constexpr int kIssueWarps = 4;   // one MMA-issuing warp per chain (a thread waits on each issue)
constexpr int kUnpackWarps = 16;
constexpr int kBuildWarp0 = 1 + kIssueWarps;
constexpr int kMmaWarps = kBuildWarp0 + kUnpackWarps;
constexpr int kMmaThreads = 32 * kMmaWarps;
constexpr int kGroupTok = kMmaTok / 4;  // tokens finished by one builder group
constexpr uint32_t kAtomA = kMmaRows * 128;     // one chain's half-block: 128 rows x 128 B
constexpr uint32_t kAtomB = kMmaTok * 128;      // 32 tokens x 128 B
constexpr uint32_t kStageB = 2 * kAtomB;        // a block's activations
constexpr int kMaxMmaStages = 6;
constexpr int kMaxABufs = 3;       // operand buffers: the builders run two half-blocks ahead
constexpr int kPrefetchAhead = 4;  // raw weight blocks requested into L2 beyond the stages

// kind::i8: D s32, A u8 or s8, B s8 (Q8_K quants), both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, bool a_signed) {
    return (2u << 4) | (uint32_t(a_signed ? 1 : 0) << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

// L2 prefetch of a 3-D tile (no shared-memory destination).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap *map, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
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
__device__ __forceinline__ uint32_t lds32(const unsigned char *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ int byte_at(const uint32_t (&w)[3], int k) { return int((w[k >> 2] >> (8 * (k & 3))) & 0xffu); }

// 8 consecutive 32-bit TMEM columns per lane (warp-collective).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7])
                 : "r"(taddr));
}

// SW128 K-major position of 16-byte chunk u (0..7) of row r in an atom.
__device__ __forceinline__ uint32_t sw128_chunk(uint32_t r, uint32_t u) {
    return r * 128u + ((u ^ (r & 7u)) << 4);
}
__device__ __forceinline__ void st_chunk(unsigned char *atom, uint32_t r, uint32_t u, uint32_t a, uint32_t b,
                                         uint32_t c, uint32_t d) {
    *reinterpret_cast<uint4 *>(atom + sw128_chunk(r, u)) = make_uint4(a, b, c, d);
}

// ---- per-type chain builders --------------------------------------------
// build(w, h, g, row, atoms): the 32 values [128h + 32g, +32) of this row's
// block (raw bytes at w) as the chains' operand bytes, written to 16-byte
// chunks 2g, 2g+1 of each chain's atom. dscale(w): the f16 d (and dmin) bits.
// term(D, dbits, as): the block's f32 term from the chain accumulators.

// Q4_K / Q5_K (dot_q4_k_q8_k_scalar / dot_q5_k_q8_k_scalar, tensor.rs:365-428):
// 144 / 176 bytes: d, dmin | 12 packed 6-bit scales and mins | (Q5_K: 32
// high-bit bytes) | 128 nibble bytes, sub-block 2c in the low nibbles of
// bytes 32c..32c+31 and 2c+1 in their high nibbles.
template <bool kQ5>
struct ChainsQ45 {
    static constexpr int kChains = 3;
    static constexpr uint32_t kBytes = kQ5 ? 176 : 144;
    __device__ static bool is_signed(int) { return false; }
    __device__ static uint32_t dscale(const unsigned char *w) { return lds32(w); }
    __device__ static void build(const unsigned char *w, int h, int g, uint32_t r, unsigned char *const *atoms) {
        const uint32_t sw[3] = {lds32(w + 4), lds32(w + 8), lds32(w + 12)};
        const int j = 4 * h + g;  // this group's sub-block: byte chunk j/2, low nibbles if j is even
        const int c = j >> 1, half = j & 1;
        constexpr uint32_t qs = kQ5 ? 48 : 16;
        const uint4 v0 = *reinterpret_cast<const uint4 *>(w + qs + 32 * c);
        const uint4 v1 = *reinterpret_cast<const uint4 *>(w + qs + 32 * c + 16);
        const uint32_t qw[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint32_t hb[8] = {};
        if constexpr (kQ5) {
            const uint4 h0 = *reinterpret_cast<const uint4 *>(w + 16), h1 = *reinterpret_cast<const uint4 *>(w + 32);
            hb[0] = h0.x, hb[1] = h0.y, hb[2] = h0.z, hb[3] = h0.w, hb[4] = h1.x, hb[5] = h1.y, hb[6] = h1.z, hb[7] = h1.w;
        }
        {
            // scale_min_k4, tensor.rs:23-32.
            int sc, mn;
            if (j < 4) {
                sc = byte_at(sw, j) & 63;
                mn = byte_at(sw, j + 4) & 63;
            } else {
                sc = (byte_at(sw, j + 4) & 15) | ((byte_at(sw, j - 4) >> 6) << 4);
                mn = (byte_at(sw, j + 4) >> 4) | ((byte_at(sw, j) >> 6) << 4);
            }
            const uint32_t slo = uint32_t(sc & 7), shi = uint32_t(sc >> 3), mw = uint32_t(mn) * 0x01010101u;
            uint32_t lo[8], hi[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                uint32_t v = (qw[k] >> (4 * half)) & 0x0f0f0f0fu;
                if constexpr (kQ5) v |= ((hb[k] >> j) & 0x01010101u) << 4;
                lo[k] = v * slo;  // bytes <= 31 * 7: no carry between bytes
                hi[k] = v * shi;
            }
            const uint32_t u = 2 * g;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                st_chunk(atoms[0], r, u + e, lo[4 * e], lo[4 * e + 1], lo[4 * e + 2], lo[4 * e + 3]);
                st_chunk(atoms[1], r, u + e, hi[4 * e], hi[4 * e + 1], hi[4 * e + 2], hi[4 * e + 3]);
                st_chunk(atoms[2], r, u + e, mw, mw, mw, mw);
            }
        }
    }
    __device__ static float term(const uint32_t (&D)[kChains], uint32_t dm, float as) {
        const int weighted = int(D[0]) + 8 * int(D[1]);
        const int minimum = int(D[2]);
        const float d = half_bits(dm) * as;
        const float dmin = half_bits(dm >> 16) * as;
        return d * float(weighted) - dmin * float(minimum);
    }
};

// Q6_K (dot_q6_k_q8_k_scalar, tensor.rs:430-460), padded to 224 bytes on the
// device: 128 low-nibble bytes | 64 high-bit bytes | 16 signed scales | d.
// Half h of the block is the reference's `half`; its values 32k + i (k < 4)
// take the low (k < 2) or high nibble of ql[64h + 32(k&1) + i] and bits
// 2k..2k+1 of qh[32h + i], and the scale sc[8h + 2k + i/16]. The signed
// scale in two's-complement 2-bit digits, sc = d0 + 4 d1 + 16 d2 + 64 d3
// (d0..d2 in 0..3, d3 = sc >> 6 in -2..1), gives four s8 chains
// (q - 32) * d_k (|value| <= 96), and weighted = D0 + 4 D1 + 16 D2 + 64 D3.
struct ChainsQ6 {
    static constexpr int kChains = 4;
    static constexpr uint32_t kBytes = kQ6KDeviceBlock;
    __device__ static bool is_signed(int) { return true; }
    __device__ static uint32_t dscale(const unsigned char *w) { return *reinterpret_cast<const uint16_t *>(w + 208); }
    __device__ static void build(const unsigned char *w, int h, int g, uint32_t r, unsigned char *const *atoms) {
        const uint4 s4 = *reinterpret_cast<const uint4 *>(w + 192);
        const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
        {  // quarter k = g: values 32k .. 32k+31 of the half
            const int k = g;
            const unsigned char *ql = w + 64 * h + 32 * (k & 1);
            const unsigned char *qh = w + 128 + 32 * h;
            uint32_t q[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const uint32_t l = lds32(ql + 4 * m), hh = lds32(qh + 4 * m);
                const uint32_t lo4 = (k >= 2 ? (l >> 4) : l) & 0x0f0f0f0fu;
                q[m] = lo4 | (((hh >> (2 * k)) & 0x03030303u) << 4);  // 0..63
            }
#pragma unroll
            for (int half16 = 0; half16 < 2; ++half16) {  // two 16-value scale groups
                const int si = 8 * h + 2 * k + half16;
                const int sc = int(int8_t(uint8_t(sw[si >> 2] >> (8 * (si & 3)))));
                const uint32_t ch = 2 * g + half16;  // 16-byte chunk of the atom
                const uint32_t *qq = q + 4 * half16;
#pragma unroll
                for (int d = 0; d < 4; ++d) {
                    const int dig = d < 3 ? (sc >> (2 * d)) & 3 : sc >> 6;
                    const uint32_t mag = uint32_t(dig < 0 ? -dig : dig);
                    const uint32_t off = 0x20202020u * mag;  // 32 * |digit| per byte
                    uint32_t v[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        // q * |digit| <= 189 (no carry), minus 32 |digit| per byte:
                        // (q - 32) * |digit| in two's-complement bytes.
                        const uint32_t t = __vsub4(qq[e] * mag, off);
                        v[e] = dig < 0 ? __vsub4(0u, t) : t;
                    }
                    st_chunk(atoms[d], r, ch, v[0], v[1], v[2], v[3]);
                }
            }
        }
    }
    __device__ static float term(const uint32_t (&D)[kChains], uint32_t dbits, float as) {
        const int weighted = int(D[0]) + 4 * int(D[1]) + 16 * int(D[2]) + 64 * int(D[3]);
        const float d = half_bits(dbits) * as;
        return d * float(weighted);
    }
};

template <int T> struct ChainsOf;
template <> struct ChainsOf<Q38_GGML_Q4_K> { using type = ChainsQ45<false>; };
template <> struct ChainsOf<Q38_GGML_Q5_K> { using type = ChainsQ45<true>; };
template <> struct ChainsOf<Q38_GGML_Q6_K> { using type = ChainsQ6; };

struct MmaParams {
    const float *scale;    // [batch][nblk] activation block scales
    float *out;            // out[t * out_ld + row]
    int *err;
    long out_ld;
    ProjEpilogue epi;      // applied to every output before it is stored
    int rows, nblk, batch, stages, abufs;
    uint32_t raw_bytes;    // kMmaRows * block bytes
};

struct MmaSmem {
    uint32_t a, raw, b, scl, total;
};

__host__ __device__ inline MmaSmem mma_smem_plan(int chains, int abufs, int stages, uint32_t raw_bytes, int nblk) {
    MmaSmem s{};
    s.a = 0;
    s.raw = uint32_t(abufs * chains) * 2 * kAtomA;  // a buffer: every chain's two half-block atoms
    s.b = s.raw + stages * ((raw_bytes + 1023) / 1024 * 1024);
    s.scl = s.b + stages * kStageB;
    s.total = s.scl + uint32_t(kMmaTok * nblk * 4);
    return s;
}

__host__ __device__ constexpr uint32_t tmem_cols_for(int chains) {
    return 2 * chains * 32 <= 128 ? 128 : 2 * chains * 32 <= 256 ? 256 : 512;
}

template <int T>
__global__ void __launch_bounds__(kMmaThreads, 1)
    proj_mma_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
                    MmaParams p) {
    using namespace sm100;
    using C = typename ChainsOf<T>::type;
    constexpr int NC = C::kChains;
    constexpr uint32_t kCols = tmem_cols_for(NC);
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t raw_full[kMaxMmaStages], raw_empty[kMaxMmaStages];
    __shared__ __align__(8) uint64_t b_full[kMaxMmaStages], b_empty[kMaxMmaStages];
    __shared__ __align__(8) uint64_t a_full[kMaxABufs], a_free[kMaxABufs], mma_done[2];
    __shared__ uint32_t tmem_base_s;
    __shared__ volatile int abort_flag;
    const int S = p.stages, NA = p.abufs;
    const MmaSmem lay = mma_smem_plan(NC, NA, S, p.raw_bytes, p.nblk);
    const uint32_t raw_stride = (p.raw_bytes + 1023) / 1024 * 1024;
    float *scl = reinterpret_cast<float *>(smem + lay.scl);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * kMmaRows, tok0 = blockIdx.y * kMmaTok;
    const int steps = p.nblk;  // one block (two half-block atoms per chain) per step

    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kUnpackWarps);
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], NC);  // one commit per chain's issuer
        }
        for (int i = 0; i < NA; ++i) {
            mbar_init(&a_full[i], kUnpackWarps);
            mbar_init(&a_free[i], NC);
        }
        for (int i = 0; i < 2; ++i) mbar_init(&mma_done[i], NC);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_s, kCols);
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
            tma_load_3d(smem + lay.raw + b * raw_stride, &map_w, b * int(C::kBytes), row0, 0, &raw_full[b]);
        }
        for (int b = first; b < min(p.nblk, first + kPrefetchAhead); ++b)
            tma_prefetch_3d(&map_w, b * int(C::kBytes), row0, 0);
    }
    pdl_wait_primary();
    pdl_launch_dependents();
    for (int i = tid; i < kMmaTok * p.nblk; i += kMmaThreads) {  // scl[b][t]
        const int b = i / kMmaTok, t = i - b * kMmaTok;
        scl[i] = tok0 + t < p.batch ? p.scale[size_t(tok0 + t) * p.nblk + b] : 0.f;
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
                tma_load_3d(smem + lay.raw + s * raw_stride, &map_w, b * int(C::kBytes), row0, 0, &raw_full[s]);
                if (b + kPrefetchAhead < p.nblk)
                    tma_prefetch_3d(&map_w, (b + kPrefetchAhead) * int(C::kBytes), row0, 0);
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
    } else if (warp < kBuildWarp0) {
        // ---------------------------------------------------------- MMA: warp 1 + c issues chain c
        const int c = warp - 1;
        if (lane == 0 && c < NC) {
            const uint32_t idesc = idesc_i8(kMmaRows, kMmaTok, C::is_signed(c));
            for (int b = 0; b < steps; ++b) {
                const int s = b % S, ab = b % NA;
                if (!mbar_wait(&a_full[ab], uint32_t(b / NA) & 1u) ||
                    !mbar_wait(&b_full[s], uint32_t(b / S) & 1u) || abort_flag) {
                    abort_flag = 1;
                    set_error(p.err, kDevErrTimeout);
                    break;
                }
                fence_after_sync();
                const uint32_t abase = smem_addr(smem + lay.a + (ab * NC + c) * 2 * kAtomA);
                const uint32_t bbase = smem_addr(smem + lay.b + s * kStageB);
                const uint32_t dcol = uint32_t((b & 1) * NC * 32);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int k = 0; k < 4; ++k)  // K-steps of 32 bytes within each half-block atom
                        mma_i8(tmem + dcol + c * 32, smem_desc_sw128(abase + h * kAtomA + k * 32, 16, 1024),
                               smem_desc_sw128(bbase + h * kAtomB + k * 32, 16, 1024), idesc,
                               (h | k) ? 1u : 0u);
                mma_commit(&a_free[ab]);
                mma_commit(&mma_done[b & 1]);
                mma_commit(&b_empty[s]);
            }
        }
    } else {
        // ---------------------------------------------------------- build + epilogue
        const int g = (warp - kBuildWarp0) >> 2;  // values 32g..32g+31 of a half-block; tokens 8g..8g+7
        const int q = warp & 3;             // TMEM lane quarter
        const uint32_t r = uint32_t(32 * q + lane);
        const uint32_t lane_addr = uint32_t(32 * q) << 16;
        float total[kGroupTok];
#pragma unroll
        for (int t = 0; t < kGroupTok; ++t) total[t] = 0.f;
        uint32_t dprev = 0, dcur = 0;
        bool ok = true;
        auto epilogue = [&](int b, uint32_t dbits) {
            if (!__all_sync(0xffffffffu, mbar_wait(&mma_done[b & 1], uint32_t(b >> 1) & 1u))) {
                ok = false;
                return;
            }
            fence_after_sync();
            uint32_t D[NC][kGroupTok];
#pragma unroll
            for (int c = 0; c < NC; ++c) tmem_ld8(tmem + lane_addr + (b & 1) * NC * 32 + c * 32 + kGroupTok * g, D[c]);
            const float4 s0 = *reinterpret_cast<const float4 *>(scl + b * kMmaTok + kGroupTok * g);
            const float4 s1 = *reinterpret_cast<const float4 *>(scl + b * kMmaTok + kGroupTok * g + 4);
            const float as[kGroupTok] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
            tmem_wait_ld();
#pragma unroll
            for (int t = 0; t < kGroupTok; ++t) {
                uint32_t d[NC];
#pragma unroll
                for (int c = 0; c < NC; ++c) d[c] = D[c][t];
                total[t] = total[t] + C::term(d, dbits, as[t]);
            }
        };
        for (int b = 0; b < steps && ok; ++b) {
            const int s = b % S, ab = b % NA;
            if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[s], uint32_t(b / S) & 1u))) {
                ok = false;
                break;
            }
            if (b >= NA && !__all_sync(0xffffffffu, mbar_wait(&a_free[ab], uint32_t(b / NA - 1) & 1u))) {
                ok = false;
                break;
            }
            const unsigned char *w = smem + lay.raw + s * raw_stride + r * C::kBytes;
            dcur = C::dscale(w);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                unsigned char *atoms[NC];
#pragma unroll
                for (int c = 0; c < NC; ++c) atoms[c] = smem + lay.a + ((ab * NC + c) * 2 + h) * kAtomA;
                C::build(w, h, g, r, atoms);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[ab]);
                mbar_arrive(&raw_empty[s]);
            }
            if (b > 0) {
                epilogue(b - 1, dprev);
                if (!ok) break;
                fence_before_sync();  // TMEM reads done before the next a_full arrive
            }
            dprev = dcur;
        }
        if (ok) epilogue(p.nblk - 1, dprev);
        if (!ok) {
            if (lane == 0) {
                abort_flag = 1;
                set_error(p.err, kDevErrTimeout);
            }
        } else if (row0 + int(r) < p.rows) {
            // All tokens' epilogue inputs first, then the outputs.
            EpilogueIn ein[kGroupTok];
#pragma unroll
            for (int t = 0; t < kGroupTok; ++t) {
                const int tok = tok0 + kGroupTok * g + t;
                if (tok < p.batch) ein[t] = proj_epilogue_load(p.epi, p.rows, tok, int(row0 + r));
            }
#pragma unroll
            for (int t = 0; t < kGroupTok; ++t) {
                const int tok = tok0 + kGroupTok * g + t;
                if (tok < p.batch)
                    p.out[size_t(tok) * p.out_ld + row0 + r] =
                        proj_epilogue_apply(p.epi, ein[t], p.rows, tok, int(row0 + r), total[t]);
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 1) tmem_dealloc(tmem, kCols);
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
    using C = typename ChainsOf<T>::type;
    const MmaSmem lay = mma_smem_plan(C::kChains, p.abufs, p.stages, p.raw_bytes, p.nblk);
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

template <int T>
bool plan_mma(MmaParams &p) {
    using C = typename ChainsOf<T>::type;
    p.raw_bytes = kMmaRows * C::kBytes;
    // Three operand buffers if they fit (the MMA round trip is long next to
    // a build step), then as many raw/activation stages (up to 6) as the
    // budget allows; L2 prefetches keep the weight copies short.
    for (int abufs = kMaxABufs; abufs >= 1; --abufs)
        for (int stages = kMaxMmaStages; stages >= 2; --stages)
            if (mma_smem_plan(C::kChains, abufs, stages, p.raw_bytes, p.nblk).total + 1024 <= kProjSmemBudget) {
                p.abufs = abufs;
                p.stages = stages;
                return true;
            }
    return false;
}

}  // namespace

bool proj_mma_supported(int type) {
    return type == Q38_GGML_Q4_K || type == Q38_GGML_Q5_K || type == Q38_GGML_Q6_K;
}

size_t proj_mma_scratch_bytes(int batch, int64_t width) {
    const size_t nb = size_t(batch) * size_t(width / 256);
    return nb * 256 + nb * 4 + nb * 32;
}

namespace {
// The scratch's layout: quants [batch][nblk][256], scales, group sums.
Q8KActivations mma_activations(void *scratch, int batch, int64_t width) {
    const size_t nb = size_t(batch) * size_t(width / 256);
    unsigned char *sp = static_cast<unsigned char *>(scratch);
    Q8KActivations act;
    act.quants = reinterpret_cast<int8_t *>(sp);
    act.scale = reinterpret_cast<float *>(sp + nb * 256);
    act.sums = reinterpret_cast<int16_t *>(sp + nb * 256 + nb * 4);
    return act;
}
}  // namespace

cudaError_t launch_proj_mma_quantize(const float *x, int batch, int64_t width, void *scratch,
                                     cudaStream_t stream) {
    if (width % 256) return cudaErrorInvalidValue;
    return launch_q8k_quantize(x, batch, int(width), mma_activations(scratch, batch, width), nullptr,
                               stream);
}

cudaError_t launch_proj_mma(const ProjWeight &w, const float *x, int batch, float *out, long out_ld,
                            int *err, void *scratch, cudaStream_t stream, const ProjEpilogue &epi,
                            bool prequantized) {
    if (!proj_mma_supported(w.type) || w.width % 256 || w.row_bytes % 16) return cudaErrorInvalidValue;
    const int nblk = int(w.width / 256);
    const Q8KActivations act = mma_activations(scratch, batch, w.width);
    cudaError_t e = cudaSuccess;
    if (!prequantized && (e = launch_q8k_quantize(x, batch, int(w.width), act, nullptr, stream)) != cudaSuccess)
        return e;
    const uint32_t bb = w.type == Q38_GGML_Q6_K ? kQ6KDeviceBlock : w.type == Q38_GGML_Q4_K ? 144 : 176;
    CUtensorMap mw, ma;
    if (!make_map_u8(&mw, w.data, uint64_t(w.row_bytes), uint64_t(w.rows), bb, kMmaRows, false) ||
        !make_map_u8(&ma, act.quants, uint64_t(w.width), uint64_t(batch), 128, kMmaTok, true))
        return cudaErrorInvalidValue;
    MmaParams p{};
    p.scale = act.scale;
    p.out = out;
    p.err = err;
    p.out_ld = out_ld;
    p.epi = epi;
    p.rows = int(w.rows);
    p.nblk = nblk;
    p.batch = batch;
    switch (w.type) {
        case Q38_GGML_Q4_K:
            if (!plan_mma<Q38_GGML_Q4_K>(p)) return cudaErrorInvalidValue;
            return launch_mma<Q38_GGML_Q4_K>(mw, ma, p, stream);
        case Q38_GGML_Q5_K:
            if (!plan_mma<Q38_GGML_Q5_K>(p)) return cudaErrorInvalidValue;
            return launch_mma<Q38_GGML_Q5_K>(mw, ma, p, stream);
        default:
            if (!plan_mma<Q38_GGML_Q6_K>(p)) return cudaErrorInvalidValue;
            return launch_mma<Q38_GGML_Q6_K>(mw, ma, p, stream);
    }
}

}  // namespace q38
