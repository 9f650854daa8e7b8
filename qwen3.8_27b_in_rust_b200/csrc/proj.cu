// proj.cu -- the projections on either side of the attention cores (sm_100a).
//
// The reference feeds every attention core from `project` (src/model/ops.rs:
// 623-640; batch_project, :1016-1031): the f32 activation is quantized once to
// Q8_K blocks (quantize_q8_k, src/kernel/quant.rs:56-124) and each K-quant
// weight row (Q2_K..Q6_K) is dotted with it in integers
// (dot_q*_k_q8_k_scalar, src/kernel/tensor.rs:301-460); F32 / F16 / BF16 /
// Q8_0 weights take the f32 activation directly (tensor.rs:79-117). Outputs
// are token-major, output[token * rows + row] (gemm_rows, tensor.rs:978-1000).
//
// Kernels:
//   q8k_quantize_kernel   one warp per 256-value block. Bit-exact with
//                         quantize_block: first largest magnitude (strict >),
//                         -127/max and 1/inverse as IEEE divisions, the
//                         round-half-even trick of nearest_int, clamp at 127.
//   proj_q8k_kernel<T>    persistent, one CTA per SM. Weight tiles (tile_rows
//                         consecutive rows = one contiguous byte range) stream
//                         through a ring of shared-memory stages by bulk copy
//                         (cp.async.bulk + mbarrier); the Q8_K activations of
//                         up to kMaxTok tokens sit in shared memory. A thread
//                         owns one (row, 256-block) pair and computes its
//                         integer sums with dp4a -- exact, so their order is
//                         free -- then the block's f32 term
//                         d*weighted - dmin*minimum. Each (row, token) output
//                         adds its block terms in block order, so the result
//                         is bit-identical to the reference's scalar dot.
//   proj_f32_kernel<T>    warp per row, lanes over the row, f32 fma partial
//                         sums and a warp tree: agrees with the reference's
//                         sequential fma chain to rounding (the reference's
//                         own AVX2 form also sums in lanes, x86/tensor.rs).
//
// Weight rows are the GGUF tensor bytes unchanged; the device copy is padded
// so that every tile copy (a whole number of 16-byte units) stays inside it.
#include <cuda_fp16.h>

#include <algorithm>

#include "q38_proj.h"
#include "q38_sm100.cuh"

namespace q38 {
namespace {

constexpr int kProjThreads = 256;
constexpr int kActStride = 272;  // shared bytes per activation block: 256 quants + 16 (bank spread)
constexpr int kMaxStages = 4;
constexpr uint32_t kNibbles = 0x0f0f0f0fu;

__device__ __forceinline__ float half_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}
__device__ __forceinline__ uint32_t ld32(const uint8_t *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}
// 32-bit word at a 2-byte-aligned shared address (Q3_K / Q6_K blocks are 110
// and 210 bytes).
__device__ __forceinline__ uint32_t ld32_a2(const uint8_t *p) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
    return uint32_t(h[0]) | (uint32_t(h[1]) << 16);
}
__device__ __forceinline__ uint4 ld128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ int byte_of(uint32_t w, int k) { return int((w >> (8 * k)) & 0xffu); }

// scale_min_k4 (src/kernel/tensor.rs:23-32) over the 12 packed bytes held in
// three words.
__device__ __forceinline__ void scale_min_k4(int j, const uint32_t (&s)[3], int &sc, int &mn) {
    auto b = [&](int k) { return byte_of(s[k >> 2], k & 3); };
    if (j < 4) {
        sc = b(j) & 63;
        mn = b(j + 4) & 63;
    } else {
        sc = (b(j + 4) & 15) | ((b(j - 4) >> 6) << 4);
        mn = (b(j + 4) >> 4) | ((b(j) >> 6) << 4);
    }
}

// Sum of two adjacent 16-value activation sums (the 32-value sub-block of
// Q4_K / Q5_K).
__device__ __forceinline__ int pair_sum(const int16_t *sums, int g) { return int(sums[g]) + int(sums[g + 1]); }

// ---- per-block terms, one per K-quant type ----------------------------------
// w: the weight block in shared memory; a: its 256 activation quants; sums:
// the 16 activation group sums; as: the activation block scale. Returns the
// block's term of the reference's running total.

// dot_q4_k_q8_k_scalar, tensor.rs:365-391. 144 bytes: d, dmin | 12 scale bytes | 128 nibble bytes.
__device__ __forceinline__ float block_q4_k(const uint8_t *w, const int8_t *a8, const int16_t *sums, float as) {
    const uint8_t *a = reinterpret_cast<const uint8_t *>(a8);
    const uint32_t dm = ld32(w);
    const uint32_t sc[3] = {ld32(w + 4), ld32(w + 8), ld32(w + 12)};
    int weighted = 0, minimum = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        int sc0, mn0, sc1, mn1;
        scale_min_k4(2 * c, sc, sc0, mn0);
        scale_min_k4(2 * c + 1, sc, sc1, mn1);
        const uint4 q[2] = {ld128(w + 16 + 32 * c), ld128(w + 32 + 32 * c)};
        const uint4 lo[2] = {ld128(a + 64 * c), ld128(a + 64 * c + 16)};
        const uint4 hi[2] = {ld128(a + 64 * c + 32), ld128(a + 64 * c + 48)};
        int dot0 = 0, dot1 = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t qw[4] = {q[h].x, q[h].y, q[h].z, q[h].w};
            const uint32_t lw[4] = {lo[h].x, lo[h].y, lo[h].z, lo[h].w};
            const uint32_t hw[4] = {hi[h].x, hi[h].y, hi[h].z, hi[h].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                dot0 = __dp4a(int(qw[k] & kNibbles), int(lw[k]), dot0);
                dot1 = __dp4a(int((qw[k] >> 4) & kNibbles), int(hw[k]), dot1);
            }
        }
        weighted += sc0 * dot0 + sc1 * dot1;
        minimum += mn0 * pair_sum(sums, 4 * c) + mn1 * pair_sum(sums, 4 * c + 2);
    }
    const float d = half_to_float(dm) * as;
    const float dmin = half_to_float(dm >> 16) * as;
    return d * float(weighted) - dmin * float(minimum);
}

// dot_q5_k_q8_k_scalar, tensor.rs:393-428. 176 bytes: d, dmin | 12 scales | 32 high-bit bytes | 128 nibble bytes.
__device__ __forceinline__ float block_q5_k(const uint8_t *w, const int8_t *a8, const int16_t *sums, float as) {
    const uint8_t *a = reinterpret_cast<const uint8_t *>(a8);
    const uint32_t dm = ld32(w);
    const uint32_t sc[3] = {ld32(w + 4), ld32(w + 8), ld32(w + 12)};
    const uint4 hb4[2] = {ld128(w + 16), ld128(w + 32)};
    const uint32_t hb[8] = {hb4[0].x, hb4[0].y, hb4[0].z, hb4[0].w, hb4[1].x, hb4[1].y, hb4[1].z, hb4[1].w};
    int weighted = 0, minimum = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        int sc0, mn0, sc1, mn1;
        scale_min_k4(2 * c, sc, sc0, mn0);
        scale_min_k4(2 * c + 1, sc, sc1, mn1);
        const uint4 q[2] = {ld128(w + 48 + 32 * c), ld128(w + 64 + 32 * c)};
        const uint4 lo[2] = {ld128(a + 64 * c), ld128(a + 64 * c + 16)};
        const uint4 hi[2] = {ld128(a + 64 * c + 32), ld128(a + 64 * c + 48)};
        int dot0 = 0, dot1 = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t qw[4] = {q[h].x, q[h].y, q[h].z, q[h].w};
            const uint32_t lw[4] = {lo[h].x, lo[h].y, lo[h].z, lo[h].w};
            const uint32_t hw[4] = {hi[h].x, hi[h].y, hi[h].z, hi[h].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t hbits = hb[4 * h + k];
                const uint32_t q0 = (qw[k] & kNibbles) | (((hbits >> (2 * c)) & 0x01010101u) << 4);
                const uint32_t q1 = ((qw[k] >> 4) & kNibbles) | (((hbits >> (2 * c + 1)) & 0x01010101u) << 4);
                dot0 = __dp4a(int(q0), int(lw[k]), dot0);
                dot1 = __dp4a(int(q1), int(hw[k]), dot1);
            }
        }
        weighted += sc0 * dot0 + sc1 * dot1;
        minimum += mn0 * pair_sum(sums, 4 * c) + mn1 * pair_sum(sums, 4 * c + 2);
    }
    const float d = half_to_float(dm) * as;
    const float dmin = half_to_float(dm >> 16) * as;
    return d * float(weighted) - dmin * float(minimum);
}

// dot_q6_k_q8_k_scalar, tensor.rs:430-460. 210 bytes: 128 low-nibble bytes |
// 64 high-bit bytes | 16 signed scales | d. Values are 6-bit minus 32.
__device__ __forceinline__ float block_q6_k(const uint8_t *w, const int8_t *a8, const int16_t *, float as) {
    const uint8_t *a = reinterpret_cast<const uint8_t *>(a8);
    int weighted = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const uint32_t s4 = ld32_a2(w + 192 + 8 * half), s4b = ld32_a2(w + 196 + 8 * half);
        const int8_t sc[8] = {int8_t(byte_of(s4, 0)), int8_t(byte_of(s4, 1)), int8_t(byte_of(s4, 2)),
                              int8_t(byte_of(s4, 3)), int8_t(byte_of(s4b, 0)), int8_t(byte_of(s4b, 1)),
                              int8_t(byte_of(s4b, 2)), int8_t(byte_of(s4b, 3))};
#pragma unroll
        for (int g = 0; g < 2; ++g) {  // 16 of the 32 positions i per group
            int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = 16 * g + 4 * k;
                const uint32_t l0 = ld32_a2(w + 64 * half + i), l1 = ld32_a2(w + 64 * half + 32 + i);
                const uint32_t hh = ld32_a2(w + 128 + 32 * half + i);
                const uint32_t q0 = __vsub4((l0 & kNibbles) | ((hh & 0x03030303u) << 4), 0x20202020u);
                const uint32_t q1 = __vsub4((l1 & kNibbles) | (((hh >> 2) & 0x03030303u) << 4), 0x20202020u);
                const uint32_t q2 = __vsub4(((l0 >> 4) & kNibbles) | (((hh >> 4) & 0x03030303u) << 4), 0x20202020u);
                const uint32_t q3 = __vsub4(((l1 >> 4) & kNibbles) | (((hh >> 6) & 0x03030303u) << 4), 0x20202020u);
                const uint8_t *ab = a + 128 * half + i;
                d0 = __dp4a(int(q0), int(ld32(ab)), d0);
                d1 = __dp4a(int(q1), int(ld32(ab + 32)), d1);
                d2 = __dp4a(int(q2), int(ld32(ab + 64)), d2);
                d3 = __dp4a(int(q3), int(ld32(ab + 96)), d3);
            }
            weighted += sc[g] * d0 + sc[g + 2] * d1 + sc[g + 4] * d2 + sc[g + 6] * d3;
        }
    }
    const float d = half_to_float(ld32_a2(w + 208)) * as;
    return d * float(weighted);
}

// dot_q3_k_q8_k_scalar, tensor.rs:335-363. 110 bytes: 32 high-bit-mask bytes |
// 64 two-bit bytes | 12 packed scales | d. Values are 3-bit minus 4.
__device__ __forceinline__ float block_q3_k(const uint8_t *w, const int8_t *a8, const int16_t *, float as) {
    const uint8_t *a = reinterpret_cast<const uint8_t *>(a8);
    // unpack_q3_scales, tensor.rs:34-44.
    uint8_t p[12];
#pragma unroll
    for (int k = 0; k < 6; ++k) {
        const uint32_t h = *reinterpret_cast<const uint16_t *>(w + 96 + 2 * k);
        p[2 * k] = uint8_t(h);
        p[2 * k + 1] = uint8_t(h >> 8);
    }
    int sc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int low = i < 8 ? (p[i] & 15) : (p[i - 8] >> 4);
        const int high = (p[8 + i % 4] >> (2 * (i / 4))) & 3;
        sc[i] = (low | (high << 4)) - 32;
    }
    int weighted = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int field = 0; field < 4; ++field) {
            const int group = 4 * half + field;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                int dsum = 0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int l = 16 * g + 4 * k;
                    const uint32_t lw = ld32_a2(w + 32 + 32 * half + l), hw = ld32_a2(w + l);
                    const uint32_t q2 = (lw >> (2 * field)) & 0x03030303u;
                    const uint32_t hbit = (hw >> group) & 0x01010101u;
                    const uint32_t q = __vsub4(q2 | (hbit << 2), 0x04040404u);
                    dsum = __dp4a(int(q), int(ld32(a + 128 * half + 32 * field + l)), dsum);
                }
                weighted += sc[2 * group + g] * dsum;
            }
        }
    }
    const float d = half_to_float(ld32_a2(w + 108)) * as;
    return d * float(weighted);
}

// dot_q2_k_q8_k_scalar, tensor.rs:301-333. 84 bytes: 16 (scale | min << 4)
// bytes | 64 two-bit bytes | d | dmin.
__device__ __forceinline__ float block_q2_k(const uint8_t *w, const int8_t *a8, const int16_t *sums, float as) {
    const uint8_t *a = reinterpret_cast<const uint8_t *>(a8);
    int weighted = 0, minimum = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const uint32_t s0 = ld32(w + 8 * half), s1 = ld32(w + 8 * half + 4);
#pragma unroll
        for (int field = 0; field < 4; ++field) {
            const int si = 2 * field;  // within this half's 8 scale bytes
            const int b0 = byte_of(si < 4 ? s0 : s1, si & 3), b1 = byte_of(si < 4 ? s0 : s1, (si & 3) + 1);
            int dot0 = 0, dot1 = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t q0 = (ld32(w + 16 + 32 * half + 4 * k) >> (2 * field)) & 0x03030303u;
                const uint32_t q1 = (ld32(w + 16 + 32 * half + 16 + 4 * k) >> (2 * field)) & 0x03030303u;
                dot0 = __dp4a(int(q0), int(ld32(a + 128 * half + 32 * field + 4 * k)), dot0);
                dot1 = __dp4a(int(q1), int(ld32(a + 128 * half + 32 * field + 16 + 4 * k)), dot1);
            }
            weighted += (b0 & 15) * dot0 + (b1 & 15) * dot1;
            minimum += (b0 >> 4) * int(sums[8 * half + si]) + (b1 >> 4) * int(sums[8 * half + si + 1]);
        }
    }
    const uint32_t dm = ld32(w + 80);
    const float d = half_to_float(dm) * as;
    const float dmin = half_to_float(dm >> 16) * as;
    return d * float(weighted) - dmin * float(minimum);
}

template <int T>
__device__ __forceinline__ float block_term(const uint8_t *w, const int8_t *a, const int16_t *sums, float as) {
    if constexpr (T == Q38_GGML_Q4_K) return block_q4_k(w, a, sums, as);
    else if constexpr (T == Q38_GGML_Q5_K) return block_q5_k(w, a, sums, as);
    else if constexpr (T == Q38_GGML_Q6_K) return block_q6_k(w, a, sums, as);
    else if constexpr (T == Q38_GGML_Q3_K) return block_q3_k(w, a, sums, as);
    else return block_q2_k(w, a, sums, as);
}

template <int T> constexpr int kBlockBytes = 0;
template <> constexpr int kBlockBytes<Q38_GGML_Q2_K> = 84;
template <> constexpr int kBlockBytes<Q38_GGML_Q3_K> = 110;
template <> constexpr int kBlockBytes<Q38_GGML_Q4_K> = 144;
template <> constexpr int kBlockBytes<Q38_GGML_Q5_K> = 176;
template <> constexpr int kBlockBytes<Q38_GGML_Q6_K> = 210;

// ---------------------------------------------------------------------------
// Q8_K quantization, one warp per 256-value block (quant.rs:56-96).
// ---------------------------------------------------------------------------
struct QuantizeParams {
    const float *x;     // [batch][width]
    Q8KActivations act; // SoA output (aos == nullptr)
    unsigned char *aos; // reference block layout, 292 bytes per block (or nullptr)
    int nblk, batch;
};

__device__ __forceinline__ int32_t nearest_int(float v) {
    const float shifted = __fadd_rn(v, 12582912.0f);
    return int32_t(__float_as_uint(shifted) & 0x007fffffu) - 0x00400000;
}

__global__ void __launch_bounds__(128) q8k_quantize_kernel(QuantizeParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * 4 + warp, t = blockIdx.y;
    if (blk >= p.nblk) return;
    const float *src = p.x + (size_t(t) * p.nblk + blk) * 256 + lane * 8;
    const float4 v0 = reinterpret_cast<const float4 *>(src)[0], v1 = reinterpret_cast<const float4 *>(src)[1];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    // First largest magnitude: the lane's own scan, then (magnitude, index)
    // pairs where a tie keeps the smaller index. NaN never compares greater,
    // as in the reference's scan.
    float amax = 0.f, mx = 0.f;
    int idx = 1 << 30;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = fabsf(v[i]);
        if (a > amax) {
            amax = a;
            mx = v[i];
            idx = lane * 8 + i;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const float om = __shfl_xor_sync(0xffffffffu, mx, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            mx = om;
            idx = oi;
        }
    }
    int8_t q[8];
    float scale = 0.f;
    if (amax == 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float inverse = __fdiv_rn(-127.0f, mx);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int32_t r = nearest_int(__fmul_rn(inverse, v[i]));
            if (r > 127) r = 127;
            q[i] = int8_t(r);
        }
        scale = __fdiv_rn(1.0f, inverse);
    }
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += q[i];
    s += __shfl_down_sync(0xffffffffu, s, 1);  // lanes 2g and 2g+1 hold group g
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w0 |= uint32_t(uint8_t(q[i])) << (8 * i);
        w1 |= uint32_t(uint8_t(q[i + 4])) << (8 * i);
    }
    if (p.aos) {
        unsigned char *b = p.aos + (size_t(t) * p.nblk + blk) * 292;
        if (lane == 0) *reinterpret_cast<float *>(b) = scale;
        // 292-byte blocks: the quants are only 4-byte aligned.
        reinterpret_cast<uint32_t *>(b + 4 + lane * 8)[0] = w0;
        reinterpret_cast<uint32_t *>(b + 4 + lane * 8)[1] = w1;
        if ((lane & 1) == 0) *reinterpret_cast<int16_t *>(b + 260 + lane) = int16_t(s);
    } else {
        const size_t bi = size_t(t) * p.nblk + blk;
        if (lane == 0) p.act.scale[bi] = scale;
        *reinterpret_cast<uint2 *>(p.act.quants + bi * 256 + lane * 8) = make_uint2(w0, w1);
        if ((lane & 1) == 0) p.act.sums[bi * 16 + (lane >> 1)] = int16_t(s);
    }
}

// ---------------------------------------------------------------------------
// Integer-path GEMV over K-quant weights.
// ---------------------------------------------------------------------------
struct ProjQ8KParams {
    const uint8_t *w;      // [rows][rb], padded to whole tiles
    Q8KActivations act;    // tokens tok0 .. tok0+batch-1
    float *out;            // out[t * out_ld + row]
    int *err;
    long out_ld;
    int rows, nblk, rb, batch, tile_rows, ntiles, stages;
    uint32_t tile_bytes;
};

struct ProjSmem {
    uint32_t ring, act_q, act_d, act_s, vbuf, total;
};

__host__ __device__ ProjSmem proj_smem_plan(int stages, uint32_t tile_bytes, int batch, int nblk, int tile_rows) {
    ProjSmem s{};
    s.ring = 0;
    s.act_q = stages * tile_bytes;
    s.act_d = s.act_q + uint32_t(batch * nblk * kActStride);
    s.act_s = s.act_d + uint32_t(batch * nblk * 4);
    s.vbuf = s.act_s + uint32_t(batch * nblk * 32);
    s.total = s.vbuf + uint32_t(tile_rows * batch * nblk * 4);
    return s;
}

template <int T>
__global__ void __launch_bounds__(kProjThreads, 1) proj_q8k_kernel(ProjQ8KParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full[kMaxStages];
    const ProjSmem lay = proj_smem_plan(p.stages, p.tile_bytes, p.batch, p.nblk, p.tile_rows);
    int8_t *aq = reinterpret_cast<int8_t *>(smem + lay.act_q);
    float *ad = reinterpret_cast<float *>(smem + lay.act_d);
    int16_t *asums = reinterpret_cast<int16_t *>(smem + lay.act_s);
    float *vbuf = reinterpret_cast<float *>(smem + lay.vbuf);
    const int tid = threadIdx.x;

    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            const int tile = blockIdx.x + s * gridDim.x;
            if (tile >= p.ntiles) break;
            mbar_arrive_expect_tx(&full[s], p.tile_bytes);
            bulk_load(smem + s * p.tile_bytes, p.w + size_t(tile) * p.tile_rows * p.rb, p.tile_bytes, &full[s]);
        }
    }
    // Activations: quants (16-byte pieces into 272-byte rows), scales, sums.
    const int nb = p.batch * p.nblk;
    for (int i = tid; i < nb * 16; i += kProjThreads) {
        const int blk = i >> 4, c = i & 15;
        *reinterpret_cast<uint4 *>(aq + blk * kActStride + 16 * c) =
            reinterpret_cast<const uint4 *>(p.act.quants + size_t(blk) * 256)[c];
    }
    for (int i = tid; i < nb; i += kProjThreads) ad[i] = p.act.scale[i];
    for (int i = tid; i < nb * 8; i += kProjThreads)
        reinterpret_cast<uint32_t *>(asums)[i] = reinterpret_cast<const uint32_t *>(p.act.sums)[i];
    __syncthreads();

    const int pairs = p.tile_rows * p.nblk;
    int k = 0;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++k) {
        const int s = k % p.stages;
        const bool ok = mbar_wait(&full[s], uint32_t(k / p.stages) & 1u);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) set_error(p.err, kDevErrTimeout);
            break;
        }
        const uint8_t *tw = smem + s * p.tile_bytes;
        const int row0 = tile * p.tile_rows;
        for (int pr = tid; pr < pairs; pr += kProjThreads) {
            const int r = pr / p.nblk, b = pr - r * p.nblk;
            if (row0 + r >= p.rows) continue;
            const uint8_t *wb = tw + size_t(r) * p.rb + size_t(b) * kBlockBytes<T>;
            for (int t = 0; t < p.batch; ++t) {
                const int ab = t * p.nblk + b;
                vbuf[(r * p.batch + t) * p.nblk + b] = block_term<T>(wb, aq + ab * kActStride, asums + ab * 16, ad[ab]);
            }
        }
        __syncthreads();
        if (tid == 0) {
            const int next = tile + p.stages * gridDim.x;
            if (next < p.ntiles) {
                sm100::fence_proxy_async_smem();  // generic reads of this stage before the async overwrite
                mbar_arrive_expect_tx(&full[s], p.tile_bytes);
                bulk_load(smem + s * p.tile_bytes, p.w + size_t(next) * p.tile_rows * p.rb, p.tile_bytes, &full[s]);
            }
        }
        for (int q = tid; q < p.tile_rows * p.batch; q += kProjThreads) {
            const int r = q / p.batch, t = q - r * p.batch;
            if (row0 + r >= p.rows) continue;
            const float *v = vbuf + q * p.nblk;
            float total = 0.f;
            for (int b = 0; b < p.nblk; ++b) total = __fadd_rn(total, v[b]);
            p.out[size_t(t) * p.out_ld + row0 + r] = total;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// f32-input GEMV (F32, F16, BF16, Q8_0 weights), warp per row.
// ---------------------------------------------------------------------------
struct ProjF32Params {
    const uint8_t *w;
    const float *x;  // [batch][width]
    float *out;
    long out_ld;
    int rows, width, rb, batch;
};

template <int T>
__device__ __forceinline__ float weight_at(const uint8_t *row, int i) {
    if constexpr (T == Q38_GGML_F32) return reinterpret_cast<const float *>(row)[i];
    else if constexpr (T == Q38_GGML_F16) return half_to_float(reinterpret_cast<const uint16_t *>(row)[i]);
    else return __uint_as_float(uint32_t(reinterpret_cast<const uint16_t *>(row)[i]) << 16);  // BF16
}

template <int T>
__global__ void __launch_bounds__(256) proj_f32_kernel(ProjF32Params p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= p.rows) return;
    const uint8_t *w = p.w + size_t(row) * p.rb;
    float acc[kProjMaxTok];
#pragma unroll
    for (int t = 0; t < kProjMaxTok; ++t) acc[t] = 0.f;
    if constexpr (T == Q38_GGML_Q8_0) {
        // dot_q8_0_scalar, tensor.rs:103-117: (d * q) * x accumulated by fma.
        const int nb = p.width / 32;
        for (int b = lane; b < nb; b += 32) {
            const uint8_t *blk = w + size_t(b) * 34;
            const float d = half_to_float(*reinterpret_cast<const uint16_t *>(blk));
            for (int i = 0; i < 32; i += 2) {
                const uint32_t qq = *reinterpret_cast<const uint16_t *>(blk + 2 + i);
                const float w0 = d * float(int8_t(qq & 0xffu)), w1 = d * float(int8_t(qq >> 8));
#pragma unroll
                for (int t = 0; t < kProjMaxTok; ++t)
                    if (t < p.batch) {
                        const float *x = p.x + size_t(t) * p.width + b * 32 + i;
                        acc[t] = fmaf(w1, x[1], fmaf(w0, x[0], acc[t]));
                    }
            }
        }
    } else {
        for (int i = lane; i < p.width; i += 32) {
            const float wv = weight_at<T>(w, i);
#pragma unroll
            for (int t = 0; t < kProjMaxTok; ++t)
                if (t < p.batch) acc[t] = fmaf(wv, p.x[size_t(t) * p.width + i], acc[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < kProjMaxTok; ++t) {
        float v = acc[t];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0 && t < p.batch) p.out[size_t(t) * p.out_ld + row] = v;
    }
}

template <int T>
cudaError_t launch_q8k(const ProjQ8KParams &base, int sm_count, cudaStream_t stream) {
    ProjQ8KParams p = base;
    const ProjSmem lay = proj_smem_plan(p.stages, p.tile_bytes, p.batch, p.nblk, p.tile_rows);
    cudaError_t e = cudaFuncSetAttribute(proj_q8k_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(lay.total));
    if (e != cudaSuccess) return e;
    const int grid = std::min(p.ntiles, sm_count);
    proj_q8k_kernel<T><<<grid, kProjThreads, lay.total, stream>>>(p);
    return cudaGetLastError();
}

template <int T>
cudaError_t launch_f32(const ProjF32Params &p, cudaStream_t stream) {
    proj_f32_kernel<T><<<(p.rows + 7) / 8, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

bool proj_is_q8k_type(int type) {
    return type == Q38_GGML_Q2_K || type == Q38_GGML_Q3_K || type == Q38_GGML_Q4_K ||
           type == Q38_GGML_Q5_K || type == Q38_GGML_Q6_K;
}

bool proj_type_supported(int type) {
    return proj_is_q8k_type(type) || type == Q38_GGML_F32 || type == Q38_GGML_F16 ||
           type == Q38_GGML_BF16 || type == Q38_GGML_Q8_0;
}

int64_t proj_row_bytes(int type, int64_t width) {
    int64_t el, by;
    switch (type) {
        case Q38_GGML_F32: el = 1; by = 4; break;
        case Q38_GGML_F16:
        case Q38_GGML_BF16: el = 1; by = 2; break;
        case Q38_GGML_Q8_0: el = 32; by = 34; break;
        case Q38_GGML_Q2_K: el = 256; by = 84; break;
        case Q38_GGML_Q3_K: el = 256; by = 110; break;
        case Q38_GGML_Q4_K: el = 256; by = 144; break;
        case Q38_GGML_Q5_K: el = 256; by = 176; break;
        case Q38_GGML_Q6_K: el = 256; by = 210; break;
        default: return -1;
    }
    if (width <= 0 || width % el) return -1;
    return width / el * by;
}

size_t proj_padded_bytes(int type, int64_t rows, int64_t width) {
    const int64_t rb = proj_row_bytes(type, width);
    return size_t((rows + kProjMaxTileRows) * rb) + 16;
}

cudaError_t launch_q8k_quantize(const float *x, int batch, int width, Q8KActivations act,
                                void *aos, cudaStream_t stream) {
    QuantizeParams p{x, act, static_cast<unsigned char *>(aos), width / 256, batch};
    const dim3 grid((p.nblk + 3) / 4, batch);
    q8k_quantize_kernel<<<grid, 128, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_proj_q8k(const ProjWeight &w, const Q8KActivations &act, int batch, float *out,
                            long out_ld, int *err, int sm_count, cudaStream_t stream) {
    const int nblk = int(w.width / 256);
    const int rb = int(w.row_bytes);
    // Rows per tile: even enough that every tile starts 16-byte aligned, and
    // small enough that the tiles cover the SMs about twice.
    int step = 1;
    while ((int64_t(step) * rb) % 16) ++step;
    int tile_rows = std::max(1, kProjThreads / nblk);
    tile_rows = std::min(tile_rows, kProjMaxTileRows);
    const int64_t want = std::max<int64_t>(1, w.rows / (2 * int64_t(sm_count)));
    if (want < tile_rows) tile_rows = int(want);
    tile_rows = std::max(step, tile_rows / step * step);
    const uint32_t tile_bytes = uint32_t((int64_t(tile_rows) * rb + 15) / 16 * 16);
    ProjQ8KParams p{};
    p.w = static_cast<const uint8_t *>(w.data);
    p.out_ld = out_ld;
    p.err = err;
    p.rows = int(w.rows);
    p.nblk = nblk;
    p.rb = rb;
    p.tile_rows = tile_rows;
    p.ntiles = int((w.rows + tile_rows - 1) / tile_rows);
    p.tile_bytes = tile_bytes;
    for (int t0 = 0; t0 < batch; t0 += kProjMaxTok) {
        p.batch = std::min(kProjMaxTok, batch - t0);
        p.act.quants = act.quants + size_t(t0) * nblk * 256;
        p.act.scale = act.scale + size_t(t0) * nblk;
        p.act.sums = act.sums + size_t(t0) * nblk * 16;
        p.out = out + size_t(t0) * out_ld;
        const uint32_t fixed = proj_smem_plan(0, tile_bytes, p.batch, nblk, tile_rows).total;
        int stages = int((kProjSmemBudget - fixed) / tile_bytes);
        stages = std::min(stages, kMaxStages);
        if (stages < 2) return cudaErrorInvalidValue;
        p.stages = stages;
        cudaError_t e;
        switch (w.type) {
            case Q38_GGML_Q2_K: e = launch_q8k<Q38_GGML_Q2_K>(p, sm_count, stream); break;
            case Q38_GGML_Q3_K: e = launch_q8k<Q38_GGML_Q3_K>(p, sm_count, stream); break;
            case Q38_GGML_Q4_K: e = launch_q8k<Q38_GGML_Q4_K>(p, sm_count, stream); break;
            case Q38_GGML_Q5_K: e = launch_q8k<Q38_GGML_Q5_K>(p, sm_count, stream); break;
            case Q38_GGML_Q6_K: e = launch_q8k<Q38_GGML_Q6_K>(p, sm_count, stream); break;
            default: return cudaErrorInvalidValue;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_proj_f32(const ProjWeight &w, const float *x, int batch, float *out,
                            long out_ld, cudaStream_t stream) {
    ProjF32Params p{};
    p.w = static_cast<const uint8_t *>(w.data);
    p.out_ld = out_ld;
    p.rows = int(w.rows);
    p.width = int(w.width);
    p.rb = int(w.row_bytes);
    for (int t0 = 0; t0 < batch; t0 += kProjMaxTok) {
        p.batch = std::min(kProjMaxTok, batch - t0);
        p.x = x + size_t(t0) * w.width;
        p.out = out + size_t(t0) * out_ld;
        cudaError_t e;
        switch (w.type) {
            case Q38_GGML_F32: e = launch_f32<Q38_GGML_F32>(p, stream); break;
            case Q38_GGML_F16: e = launch_f32<Q38_GGML_F16>(p, stream); break;
            case Q38_GGML_BF16: e = launch_f32<Q38_GGML_BF16>(p, stream); break;
            case Q38_GGML_Q8_0: e = launch_f32<Q38_GGML_Q8_0>(p, stream); break;
            default: return cudaErrorInvalidValue;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace q38
