// proj.cu -- the projections on either side of the attention cores (sm_100a).
//
// The reference feeds every attention core from `project` (src/model/ops.rs:
// 623-640; batch_project, :1016-1031): the f32 activation is quantized once to
// Q8_K blocks (quantize_q8_k, src/kernel/quant.rs:56-124) and each K-quant
// weight row (Q2_K..Q6_K, IQ4_NL, IQ4_XS) is dotted with it in integers
// (dot_q*_k_q8_k_scalar, src/kernel/tensor.rs:301-460; dot_iq4_*_q8_k,
// src/kernel/iq.rs:355-405); F32 / F16 / BF16 /
// Q8_0 weights take the f32 activation directly (tensor.rs:79-117). Outputs
// are token-major, output[token * rows + row] (gemm_rows, tensor.rs:978-1000).
//
// Kernels:
//   q8k_quantize_kernel   one warp per 256-value block. Bit-exact with
//                         quantize_block: first largest magnitude (strict >),
//                         -127/max and 1/inverse as IEEE divisions, the
//                         round-half-even trick of nearest_int, clamp at 127.
//   proj_q8k_kernel<T,W>  persistent, one CTA per SM, W consumer warps (16
//                         for one token, else 8). Weight tiles (tile_rows
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

constexpr int kProjConsumerWarps = 8;    // the general kernel
constexpr int kProjOneTokenWarps = 16;  // one token, rows of up to 32 blocks
constexpr int kProjTileRows = kProjMaxTileRows;
constexpr int kActStride = 272;  // shared bytes per activation block: 256 quants + 16 (bank spread)
constexpr int kMaxStages = 4;
constexpr int kMaxDevices = 64;
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
__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
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

// The eight 32-value sums of a block from its 16 group sums, read as two
// 16-byte loads (the 2-byte reads of lanes 32 bytes apart hit 4-8-way bank
// conflicts).
__device__ __forceinline__ void pair_sums8(const int16_t *sums, int (&ps)[8]) {
    const uint4 a = reinterpret_cast<const uint4 *>(sums)[0], b = reinterpret_cast<const uint4 *>(sums)[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) ps[j] = int(int16_t(w[j] & 0xffffu)) + int(int16_t(w[j] >> 16));
}

// ---- per-block terms, one per K-quant type ----------------------------------
// Each type is a register image of one weight block: load() reads the block
// from shared memory once (unpacking its scales), term() is the block's term
// of the reference's running total for one token: `a` its 256 activation
// quants, `sums` the 16 activation group sums, `as` the activation scale. A
// thread reuses the image for every token of the launch.

// dot_q4_k_q8_k_scalar, tensor.rs:365-391. 144 bytes: d, dmin | 12 scale
// bytes | 128 nibble bytes (sub-block 2c in the low nibbles of bytes
// 32c..32c+31, sub-block 2c+1 in their high nibbles).
struct BlockQ4K {
    uint32_t q[32];
    int sc[8], mn[8];
    uint32_t dm;
    __device__ __forceinline__ void load(const uint8_t *w) {
        dm = ld32(w);
        const uint32_t s[3] = {ld32(w + 4), ld32(w + 8), ld32(w + 12)};
#pragma unroll
        for (int j = 0; j < 8; ++j) scale_min_k4(j, s, sc[j], mn[j]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint4 v = ld128(w + 16 + 16 * k);
            q[4 * k] = v.x, q[4 * k + 1] = v.y, q[4 * k + 2] = v.z, q[4 * k + 3] = v.w;
        }
    }
    __device__ __forceinline__ float term(const uint8_t *a, const int16_t *sums, float as) const {
        int weighted = 0, minimum = 0;
        int ps[8];
        pair_sums8(sums, ps);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            int dot0 = 0, dot1 = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint4 lo = ld128(a + 64 * c + 16 * h), hi = ld128(a + 64 * c + 32 + 16 * h);
                const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w}, hw[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t qw = q[8 * c + 4 * h + k];
                    dot0 = __dp4a(int(qw & kNibbles), int(lw[k]), dot0);
                    dot1 = __dp4a(int((qw >> 4) & kNibbles), int(hw[k]), dot1);
                }
            }
            weighted += sc[2 * c] * dot0 + sc[2 * c + 1] * dot1;
            minimum += mn[2 * c] * ps[2 * c] + mn[2 * c + 1] * ps[2 * c + 1];
        }
        const float d = half_to_float(dm) * as;
        const float dmin = half_to_float(dm >> 16) * as;
        return d * float(weighted) - dmin * float(minimum);
    }
};

// dot_q5_k_q8_k_scalar, tensor.rs:393-428. 176 bytes: d, dmin | 12 scales |
// 32 high-bit bytes | 128 nibble bytes. The fifth bit of sub-block j's value
// i is bit j of high byte i.
struct BlockQ5K {
    uint32_t q[32], hb[8];
    int sc[8], mn[8];
    uint32_t dm;
    __device__ __forceinline__ void load(const uint8_t *w) {
        dm = ld32(w);
        const uint32_t s[3] = {ld32(w + 4), ld32(w + 8), ld32(w + 12)};
#pragma unroll
        for (int j = 0; j < 8; ++j) scale_min_k4(j, s, sc[j], mn[j]);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint4 v = ld128(w + 16 + 16 * k);
            hb[4 * k] = v.x, hb[4 * k + 1] = v.y, hb[4 * k + 2] = v.z, hb[4 * k + 3] = v.w;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint4 v = ld128(w + 48 + 16 * k);
            q[4 * k] = v.x, q[4 * k + 1] = v.y, q[4 * k + 2] = v.z, q[4 * k + 3] = v.w;
        }
    }
    __device__ __forceinline__ float term(const uint8_t *a, const int16_t *sums, float as) const {
        int weighted = 0, minimum = 0;
        int ps[8];
        pair_sums8(sums, ps);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            int dot0 = 0, dot1 = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint4 lo = ld128(a + 64 * c + 16 * h), hi = ld128(a + 64 * c + 32 + 16 * h);
                const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w}, hw[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t qw = q[8 * c + 4 * h + k], hbits = hb[4 * h + k];
                    const uint32_t q0 = (qw & kNibbles) | (((hbits >> (2 * c)) & 0x01010101u) << 4);
                    const uint32_t q1 = ((qw >> 4) & kNibbles) | (((hbits >> (2 * c + 1)) & 0x01010101u) << 4);
                    dot0 = __dp4a(int(q0), int(lw[k]), dot0);
                    dot1 = __dp4a(int(q1), int(hw[k]), dot1);
                }
            }
            weighted += sc[2 * c] * dot0 + sc[2 * c + 1] * dot1;
            minimum += mn[2 * c] * ps[2 * c] + mn[2 * c + 1] * ps[2 * c + 1];
        }
        const float d = half_to_float(dm) * as;
        const float dmin = half_to_float(dm >> 16) * as;
        return d * float(weighted) - dmin * float(minimum);
    }
};

// dot_q6_k_q8_k_scalar, tensor.rs:430-460. 210 bytes, padded to 224 on the
// device: 128 low-nibble bytes | 64 high-bit bytes | 16 signed scales | d.
// The 6-bit values minus 32 are formed per byte with __vsub4.
struct BlockQ6K {
    uint32_t ql[32], qh[16], sc[4];
    uint32_t d16;
    __device__ __forceinline__ void load(const uint8_t *w) {  // 224-byte device blocks: 16-byte aligned
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint4 v = ld128(w + 16 * k);
            ql[4 * k] = v.x, ql[4 * k + 1] = v.y, ql[4 * k + 2] = v.z, ql[4 * k + 3] = v.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 v = ld128(w + 128 + 16 * k);
            qh[4 * k] = v.x, qh[4 * k + 1] = v.y, qh[4 * k + 2] = v.z, qh[4 * k + 3] = v.w;
        }
        const uint4 v = ld128(w + 192);
        sc[0] = v.x, sc[1] = v.y, sc[2] = v.z, sc[3] = v.w;
        d16 = *reinterpret_cast<const uint16_t *>(w + 208);
    }
    __device__ __forceinline__ int scale(int i) const { return int(int8_t(byte_of(sc[i >> 2], i & 3))); }
    __device__ __forceinline__ float term(const uint8_t *a, const int16_t *, float as) const {
        int weighted = 0;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int g = 0; g < 2; ++g) {  // positions i = 16g .. 16g+15 of this half
                int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int wi = 4 * g + k;  // word index within the 32 positions
                    const uint32_t l0 = ql[16 * half + wi], l1 = ql[16 * half + 8 + wi];
                    const uint32_t hh = qh[8 * half + wi];
                    const uint32_t q0 = __vsub4((l0 & kNibbles) | ((hh & 0x03030303u) << 4), 0x20202020u);
                    const uint32_t q1 = __vsub4((l1 & kNibbles) | (((hh >> 2) & 0x03030303u) << 4), 0x20202020u);
                    const uint32_t q2 = __vsub4(((l0 >> 4) & kNibbles) | (((hh >> 4) & 0x03030303u) << 4), 0x20202020u);
                    const uint32_t q3 = __vsub4(((l1 >> 4) & kNibbles) | (((hh >> 6) & 0x03030303u) << 4), 0x20202020u);
                    const uint8_t *ab = a + 128 * half + 4 * wi;
                    d0 = __dp4a(int(q0), int(ld32(ab)), d0);
                    d1 = __dp4a(int(q1), int(ld32(ab + 32)), d1);
                    d2 = __dp4a(int(q2), int(ld32(ab + 64)), d2);
                    d3 = __dp4a(int(q3), int(ld32(ab + 96)), d3);
                }
                const int si = 8 * half + g;
                weighted += scale(si) * d0 + scale(si + 2) * d1 + scale(si + 4) * d2 + scale(si + 6) * d3;
            }
        }
        const float d = half_to_float(d16) * as;
        return d * float(weighted);
    }
};

// dot_q3_k_q8_k_scalar, tensor.rs:335-363. 110 bytes (2-byte aligned): 32
// high-bit-mask bytes | 64 two-bit bytes | 12 packed scales | d. Values are
// the two bits minus 4 unless the mask bit is set.
struct BlockQ3K {
    uint32_t hm[8], qs[16];
    int sc[16];
    uint32_t d16;
    __device__ __forceinline__ void load(const uint8_t *w) {
#pragma unroll
        for (int k = 0; k < 8; ++k) hm[k] = ld32_a2(w + 4 * k);
#pragma unroll
        for (int k = 0; k < 16; ++k) qs[k] = ld32_a2(w + 32 + 4 * k);
        // unpack_q3_scales, tensor.rs:34-44.
        uint32_t pw[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) pw[k] = ld32_a2(w + 96 + 4 * k);
        auto pb = [&](int i) { return byte_of(pw[i >> 2], i & 3); };
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int low = i < 8 ? (pb(i) & 15) : (pb(i - 8) >> 4);
            const int high = (pb(8 + i % 4) >> (2 * (i / 4))) & 3;
            sc[i] = (low | (high << 4)) - 32;
        }
        d16 = *reinterpret_cast<const uint16_t *>(w + 108);
    }
    __device__ __forceinline__ float term(const uint8_t *a, const int16_t *, float as) const {
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
                        const int wi = 4 * g + k;  // lanes 4wi .. 4wi+3
                        const uint32_t q2 = (qs[8 * half + wi] >> (2 * field)) & 0x03030303u;
                        const uint32_t hbit = (hm[wi] >> group) & 0x01010101u;
                        const uint32_t qv = __vsub4(q2 | (hbit << 2), 0x04040404u);
                        dsum = __dp4a(int(qv), int(ld32(a + 128 * half + 32 * field + 4 * wi)), dsum);
                    }
                    weighted += sc[2 * group + g] * dsum;
                }
            }
        }
        const float d = half_to_float(d16) * as;
        return d * float(weighted);
    }
};

// dot_q2_k_q8_k_scalar, tensor.rs:301-333. 84 bytes: 16 (scale | min << 4)
// bytes | 64 two-bit bytes | d | dmin.
struct BlockQ2K {
    uint32_t s[4], qs[16];
    uint32_t dm;
    __device__ __forceinline__ void load(const uint8_t *w) {
#pragma unroll
        for (int k = 0; k < 4; ++k) s[k] = ld32(w + 4 * k);
#pragma unroll
        for (int k = 0; k < 16; ++k) qs[k] = ld32(w + 16 + 4 * k);
        dm = ld32(w + 80);
    }
    __device__ __forceinline__ float term(const uint8_t *a, const int16_t *sums, float as) const {
        int weighted = 0, minimum = 0;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int field = 0; field < 4; ++field) {
                const int si = 8 * half + 2 * field;
                const int b0 = byte_of(s[si >> 2], si & 3), b1 = byte_of(s[(si + 1) >> 2], (si + 1) & 3);
                int dot0 = 0, dot1 = 0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t q0 = (qs[8 * half + k] >> (2 * field)) & 0x03030303u;
                    const uint32_t q1 = (qs[8 * half + 4 + k] >> (2 * field)) & 0x03030303u;
                    dot0 = __dp4a(int(q0), int(ld32(a + 128 * half + 32 * field + 4 * k)), dot0);
                    dot1 = __dp4a(int(q1), int(ld32(a + 128 * half + 32 * field + 16 + 4 * k)), dot1);
                }
                weighted += (b0 & 15) * dot0 + (b1 & 15) * dot1;
                minimum += (b0 >> 4) * int(sums[si]) + (b1 >> 4) * int(sums[si + 1]);
            }
        }
        const float d = half_to_float(dm) * as;
        const float dmin = half_to_float(dm >> 16) * as;
        return d * float(weighted) - dmin * float(minimum);
    }
};

// ---- IQ4_NL / IQ4_XS (src/kernel/iq.rs:355-405) ----------------------------
// A 4-bit index selects one of 16 signed values (kvalues_iq4nl,
// src/kernel/iq_tables.rs:52-56: the format's own table). Within a 32-value
// group, byte i holds value i in its low nibble and value i + 16 in its high
// nibble.
constexpr int8_t kIq4Values[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
__host__ __device__ constexpr uint32_t iq4_word(int k) {
    return uint32_t(uint8_t(kIq4Values[4 * k])) | (uint32_t(uint8_t(kIq4Values[4 * k + 1])) << 8) |
           (uint32_t(uint8_t(kIq4Values[4 * k + 2])) << 16) | (uint32_t(uint8_t(kIq4Values[4 * k + 3])) << 24);
}

// The table values of four indices (bits 0-3 of each byte of idx), packed as
// four signed bytes: two byte permutes over the table's halves pick by the low
// three bits, bit 3 chooses between them.
__device__ __forceinline__ uint32_t iq4_values4(uint32_t idx) {
    uint32_t x = idx & 0x07070707u;
    x = (x | (x >> 4)) & 0x00ff00ffu;
    const uint32_t sel = (x | (x >> 8)) & 0xffffu;  // one 3-bit selector per nibble
    const uint32_t lo = __byte_perm(iq4_word(0), iq4_word(1), sel);
    const uint32_t hi = __byte_perm(iq4_word(2), iq4_word(3), sel);
    const uint32_t m = ((idx >> 3) & 0x01010101u) * 0xffu;
    return (hi & m) | (lo & ~m);
}

// The integer sum of one 32-value group: 4 nibble words against its 32
// activation quants (low nibbles with a[0..15], high with a[16..31]).
__device__ __forceinline__ int iq4_group_sum(const uint32_t *q, const uint8_t *a) {
    const uint4 lo = ld128(a), hi = ld128(a + 16);
    const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w}, hw[4] = {hi.x, hi.y, hi.z, hi.w};
    int s = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        s = __dp4a(int(iq4_values4(q[k] & kNibbles)), int(lw[k]), s);
        s = __dp4a(int(iq4_values4((q[k] >> 4) & kNibbles)), int(hw[k]), s);
    }
    return s;
}

// dot_iq4_xs_q8_k, iq.rs:379-405. 136 bytes (8-byte aligned): d | scales_h |
// scales_l[4] | 128 nibble bytes; group g's scale is 4 bits of scales_l and 2
// of scales_h, minus 32; one term per block.
struct BlockIQ4XS {
    uint32_t q[32];
    uint32_t dsh, sl;  // d | scales_h << 16, scales_l
    __device__ __forceinline__ void load(const uint8_t *w) {
        const uint2 h = *reinterpret_cast<const uint2 *>(w);
        dsh = h.x, sl = h.y;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const uint2 v = *reinterpret_cast<const uint2 *>(w + 8 + 8 * k);
            q[2 * k] = v.x, q[2 * k + 1] = v.y;
        }
    }
    __device__ __forceinline__ float term(const uint8_t *a, const int16_t *, float as) const {
        int weighted = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const int scale = int((sl >> (4 * g)) & 15u) | int(((dsh >> (16 + 2 * g)) & 3u) << 4);
            weighted += (scale - 32) * iq4_group_sum(q + 4 * g, a + 32 * g);
        }
        const float d = half_to_float(dsh) * as;
        return d * float(weighted);
    }
};

// dot_iq4_nl_q8_k, iq.rs:355-377. Eight 18-byte blocks per 256 values (a
// 144-byte unit; groups 2-byte aligned): an f16 scale and 16 nibble bytes per
// 32-value group, and one term per GROUP added to the running total, so a
// 256-value unit yields eight terms in order (terms()).
struct BlockIQ4NL {
    uint32_t q[32];
    uint32_t d16[8];
    __device__ __forceinline__ void load(const uint8_t *w) {
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            d16[g] = *reinterpret_cast<const uint16_t *>(w + 18 * g);
#pragma unroll
            for (int k = 0; k < 4; ++k) q[4 * g + k] = ld32_a2(w + 18 * g + 2 + 4 * k);
        }
    }
    __device__ __forceinline__ void terms(const uint8_t *a, const int16_t *, float as, float *dst) const {
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const float d = half_to_float(d16[g]) * as;
            dst[g] = d * float(iq4_group_sum(q + 4 * g, a + 32 * g));
        }
    }
};

template <int T> struct BlockOf;
template <> struct BlockOf<Q38_GGML_Q2_K> { using type = BlockQ2K; };
template <> struct BlockOf<Q38_GGML_Q3_K> { using type = BlockQ3K; };
template <> struct BlockOf<Q38_GGML_Q4_K> { using type = BlockQ4K; };
template <> struct BlockOf<Q38_GGML_Q5_K> { using type = BlockQ5K; };
template <> struct BlockOf<Q38_GGML_Q6_K> { using type = BlockQ6K; };
template <> struct BlockOf<Q38_GGML_IQ4_NL> { using type = BlockIQ4NL; };
template <> struct BlockOf<Q38_GGML_IQ4_XS> { using type = BlockIQ4XS; };

// f32 terms a 256-value unit adds to a row's running total: one, or eight for
// IQ4_NL (a term per 32-value group).
template <int T> constexpr int kTermsPerBlock = T == Q38_GGML_IQ4_NL ? 8 : 1;
__host__ __device__ inline int proj_terms_per_block(int type) { return type == Q38_GGML_IQ4_NL ? 8 : 1; }

// A unit's terms into dst[0 .. kTermsPerBlock<T>).
template <int T, class B>
__device__ __forceinline__ void block_terms(const B &blk, const uint8_t *a, const int16_t *sums, float as,
                                            float *dst) {
    if constexpr (kTermsPerBlock<T> == 1)
        dst[0] = blk.term(a, sums, as);
    else
        blk.terms(a, sums, as, dst);
}

template <int T> constexpr int kBlockBytes = 0;
template <> constexpr int kBlockBytes<Q38_GGML_Q2_K> = 84;
template <> constexpr int kBlockBytes<Q38_GGML_Q3_K> = 110;
template <> constexpr int kBlockBytes<Q38_GGML_Q4_K> = 144;
template <> constexpr int kBlockBytes<Q38_GGML_Q5_K> = 176;
template <> constexpr int kBlockBytes<Q38_GGML_Q6_K> = kQ6KDeviceBlock;  // padded on upload
template <> constexpr int kBlockBytes<Q38_GGML_IQ4_NL> = 144;            // eight 18-byte blocks
template <> constexpr int kBlockBytes<Q38_GGML_IQ4_XS> = 136;

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

// quantize_block (quant.rs:56-96) of the 256 values at src by one warp: lane
// l owns values 8l..8l+7. Returns the lane's eight quants packed in two
// words, the block scale, and (in even lanes) the sum of group l/2.
struct WarpQ8K {
    uint32_t w0, w1;
    float scale;
    int group_sum;
};

__device__ __forceinline__ WarpQ8K quantize_values_warp(const float4 v0, const float4 v1, int lane) {
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
    WarpQ8K r;
    r.scale = 0.f;
    if (amax == 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float inverse = __fdiv_rn(-127.0f, mx);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int32_t n = nearest_int(__fmul_rn(inverse, v[i]));
            if (n > 127) n = 127;
            q[i] = int8_t(n);
        }
        r.scale = __fdiv_rn(1.0f, inverse);
    }
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += q[i];
    r.group_sum = sum + __shfl_down_sync(0xffffffffu, sum, 1);  // lanes 2g, 2g+1 hold group g
    r.w0 = r.w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        r.w0 |= uint32_t(uint8_t(q[i])) << (8 * i);
        r.w1 |= uint32_t(uint8_t(q[i + 4])) << (8 * i);
    }
    return r;
}

__device__ __forceinline__ WarpQ8K quantize_block_warp(const float *src, int lane) {
    return quantize_values_warp(reinterpret_cast<const float4 *>(src)[2 * lane],
                                reinterpret_cast<const float4 *>(src)[2 * lane + 1], lane);
}

__global__ void __launch_bounds__(128) q8k_quantize_kernel(QuantizeParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * 4 + warp, t = blockIdx.y;
    if (blk >= p.nblk) return;
    const WarpQ8K r = quantize_block_warp(p.x + (size_t(t) * p.nblk + blk) * 256, lane);
    if (p.aos) {
        unsigned char *b = p.aos + (size_t(t) * p.nblk + blk) * 292;
        if (lane == 0) *reinterpret_cast<float *>(b) = r.scale;
        // 292-byte blocks: the quants are only 4-byte aligned.
        reinterpret_cast<uint32_t *>(b + 4 + lane * 8)[0] = r.w0;
        reinterpret_cast<uint32_t *>(b + 4 + lane * 8)[1] = r.w1;
        if ((lane & 1) == 0) *reinterpret_cast<int16_t *>(b + 260 + lane) = int16_t(r.group_sum);
    } else {
        const size_t bi = size_t(t) * p.nblk + blk;
        if (lane == 0) p.act.scale[bi] = r.scale;
        *reinterpret_cast<uint2 *>(p.act.quants + bi * 256 + lane * 8) = make_uint2(r.w0, r.w1);
        if ((lane & 1) == 0) p.act.sums[bi * 16 + (lane >> 1)] = int16_t(r.group_sum);
    }
}

// ---------------------------------------------------------------------------
// Integer-path GEMV over K-quant weights.
// ---------------------------------------------------------------------------
struct ProjQ8KParams {
    const uint8_t *w;      // [rows][rb], padded to whole tiles
    const float *x;        // f32 input [batch][nblk * 256], quantized in the prologue
    float *out;            // out[t * out_ld + row]
    int *err;
    long out_ld;
    ProjEpilogue epi;      // applied to every output before it is stored
    int rows, nblk, rb, batch, ntiles, stages;
    int tile_rows;         // 16, or 8 for wide rows (a tile is one contiguous byte range)
    uint32_t tile_bytes;   // tile_rows * rb (a multiple of 16: rb is even)
};

// Shared-memory plan: the weight ring, the activations, and one combine
// buffer per consumer warp ([batch][nblk + 1] block terms).
struct ProjSmem {
    uint32_t ring, act_q, act_d, act_s, vt, total;
};

// Floats per consumer warp's combine buffer: [batch][nblk + 1] block terms,
// at least 32 (the one-token path stages one term per lane) and a multiple of
// four so that every warp's buffer starts on a 16-byte boundary.
__host__ __device__ inline int proj_vt_stride(int batch, int nblk) {
    const int n = batch * (nblk + 1);
    return n < 32 ? 32 : (n + 3) & ~3;
}

// The first n (<= 32) floats of a 16-byte-aligned buffer added in order:
// all loads first, then the serial adds.
__device__ __forceinline__ float ordered_sum32(const float *v, int n) {
    float4 t4[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) t4[i] = reinterpret_cast<const float4 *>(v)[i];
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float e[4] = {t4[i].x, t4[i].y, t4[i].z, t4[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (4 * i + j < n) total = __fadd_rn(total, e[j]);
    }
    return total;
}

__host__ __device__ inline ProjSmem proj_smem_plan(int stages, uint32_t tile_bytes, int batch, int nblk,
                                                   int warps, int terms) {
    ProjSmem s{};
    s.ring = 0;
    s.act_q = stages * tile_bytes;
    s.act_d = s.act_q + uint32_t(batch * nblk * kActStride);
    s.act_s = (s.act_d + uint32_t(batch * nblk * 4) + 15u) & ~15u;  // 16-byte loads of the sums
    s.vt = s.act_s + uint32_t(batch * nblk * 32);
    s.total = s.vt + uint32_t(warps * proj_vt_stride(batch, nblk * terms) * 4);
    return s;
}

// Warp roles: warps 0..W-1 compute (warp w owns rows w, w + W, ... of each
// tile; lane j owns blocks j, j+32, ...),
// the last warp streams the tiles. Each row's block terms go through the
// warp's combine buffer, where lane t adds token t's terms in block order.
// W = kProjOneTokenWarps is the one-token form (the host sends it only one
// token and rows of up to 32 blocks): twice the warps, each with at most 120
// registers, to hide the latency of the per-row work.
template <int T, int W>
__global__ void __launch_bounds__(32 * (W + 1), 1) proj_q8k_kernel(ProjQ8KParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
    __shared__ volatile int abort_flag;
    constexpr int kT = kTermsPerBlock<T>;
    const int nterms = p.nblk * kT;  // f32 terms per (row, token)
    const ProjSmem lay = proj_smem_plan(p.stages, p.tile_bytes, p.batch, p.nblk, W, kT);
    const uint8_t *aq = smem + lay.act_q;
    float *ad = reinterpret_cast<float *>(smem + lay.act_d);
    int16_t *asums = reinterpret_cast<int16_t *>(smem + lay.act_s);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        fence_barrier_init();
    }
    __syncthreads();
    // The weights are constant: the first tiles are requested before waiting
    // for the previous kernel in the stream (programmatic dependent launch).
    const int first = min(p.stages, (p.ntiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x));
    if (warp == W && lane == 0)
        for (int k = 0; k < first; ++k) {
            mbar_arrive_expect_tx(&full[k], p.tile_bytes);
            bulk_load(smem + k * p.tile_bytes,
                      p.w + size_t(blockIdx.x + k * gridDim.x) * p.tile_rows * p.rb, p.tile_bytes, &full[k]);
        }
    pdl_wait_primary();
    pdl_launch_dependents();
    // quantize_q8_k of the launch's tokens into shared memory, one warp per
    // 256-block (the same steps as q8k_quantize_kernel).
    // Each warp's blocks are loaded before any is quantized, so the global
    // loads overlap instead of running one round-trip per block.
    constexpr int kQWarps = W + 1, kQAhead = 4;
    for (int base = warp; base < p.batch * p.nblk; base += kQWarps * kQAhead) {
        float4 v[kQAhead][2];
#pragma unroll
        for (int u = 0; u < kQAhead; ++u) {
            const int blk = base + u * kQWarps;
            if (blk < p.batch * p.nblk) {
                const float4 *src = reinterpret_cast<const float4 *>(p.x + size_t(blk) * 256);
                v[u][0] = src[2 * lane];
                v[u][1] = src[2 * lane + 1];
            }
        }
#pragma unroll
        for (int u = 0; u < kQAhead; ++u) {
            const int blk = base + u * kQWarps;
            if (blk >= p.batch * p.nblk) break;
            const WarpQ8K r = quantize_values_warp(v[u][0], v[u][1], lane);
            *reinterpret_cast<uint2 *>(smem + lay.act_q + blk * kActStride + lane * 8) = make_uint2(r.w0, r.w1);
            if (lane == 0) ad[blk] = r.scale;
            if ((lane & 1) == 0) asums[blk * 16 + (lane >> 1)] = int16_t(r.group_sum);
        }
    }
    __syncthreads();

    if (warp == W) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            int k = first;
            for (int tile = blockIdx.x + first * gridDim.x; tile < p.ntiles; tile += gridDim.x, ++k) {
                const int s = k % p.stages;
                if (!mbar_wait(&empty[s], uint32_t(k / p.stages - 1) & 1u)) {
                    abort_flag = 1;
                    set_error(p.err, kDevErrTimeout);
                    break;
                }
                if (abort_flag) break;
                mbar_arrive_expect_tx(&full[s], p.tile_bytes);
                bulk_load(smem + s * p.tile_bytes, p.w + size_t(tile) * p.tile_rows * p.rb, p.tile_bytes,
                          &full[s]);
            }
            // Every issued copy lands before the CTA exits: the last use of
            // each stage completes its barrier phase once.
            const int issued = k;
            for (int j = issued - p.stages; j < issued; ++j)
                if (j >= 0) mbar_wait(&full[j % p.stages], uint32_t(j / p.stages) & 1u);
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    float *vt = reinterpret_cast<float *>(smem + lay.vt) + warp * proj_vt_stride(p.batch, nterms);
    int k = 0;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++k) {
        const int s = k % p.stages;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], uint32_t(k / p.stages) & 1u))) {
            if (lane == 0) {
                abort_flag = 1;
                set_error(p.err, kDevErrTimeout);
            }
            break;
        }
        const uint8_t *tw = smem + s * p.tile_bytes;
#pragma unroll 1
        for (int r = warp; r < p.tile_rows; r += W) {
            const int row = tile * p.tile_rows + r;
            if (row >= p.rows) break;  // rows ascend with r
            // The epilogue's inputs for this row, requested now: lane t
            // finishes token t (lane 0 the single token of the one-token form).
            const EpilogueIn ein = (p.epi.kind != kEpiNone && lane < p.batch)
                                       ? proj_epilogue_load(p.epi, p.rows, lane, row)
                                       : EpilogueIn{};
            if constexpr (W == kProjOneTokenWarps) {
                // One token, one block per lane: the block terms staged in
                // the warp's buffer, where lane 0 reads them with vector
                // loads and adds them in block order (only the adds are
                // serial).
                if constexpr (kT == 1) {
                    float v = 0.f;
                    if (lane < p.nblk) {
                        typename BlockOf<T>::type blk;
                        blk.load(tw + size_t(r) * p.rb + size_t(lane) * kBlockBytes<T>);
                        v = blk.term(aq + lane * kActStride, asums + lane * 16, ad[lane]);
                    }
                    vt[lane] = v;
                    __syncwarp();
                    if (lane == 0)
                        p.out[row] = proj_epilogue_apply(p.epi, ein, p.rows, 0, row, ordered_sum32(vt, p.nblk));
                } else {
                    if (lane < p.nblk) {
                        typename BlockOf<T>::type blk;
                        blk.load(tw + size_t(r) * p.rb + size_t(lane) * kBlockBytes<T>);
                        blk.terms(aq + lane * kActStride, asums + lane * 16, ad[lane], vt + lane * kT);
                    }
                    __syncwarp();
                    if (lane == 0) {
                        float total = 0.f;
#pragma unroll 8
                        for (int i = 0; i < nterms; ++i) total = __fadd_rn(total, vt[i]);
                        p.out[row] = proj_epilogue_apply(p.epi, ein, p.rows, 0, row, total);
                    }
                }
                __syncwarp();
            } else {
                for (int b = lane; b < p.nblk; b += 32) {
                    typename BlockOf<T>::type blk;
                    blk.load(tw + size_t(r) * p.rb + size_t(b) * kBlockBytes<T>);
                    for (int t = 0; t < p.batch; ++t) {
                        const int ab = t * p.nblk + b;
                        block_terms<T>(blk, aq + ab * kActStride, asums + ab * 16, ad[ab],
                                       vt + t * (nterms + 1) + b * kT);
                    }
                }
                __syncwarp();
                if (lane < p.batch) {
                    const float *v = vt + lane * (nterms + 1);
                    float total = 0.f;
#pragma unroll 8
                    for (int i = 0; i < nterms; ++i) total = __fadd_rn(total, v[i]);
                    p.out[size_t(lane) * p.out_ld + row] = proj_epilogue_apply(p.epi, ein, p.rows, lane, row, total);
                }
                __syncwarp();
            }
        }
        if (lane == 0) mbar_arrive(&empty[s]);
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
    ProjEpilogue epi;  // applied to every output before it is stored
    int rows, width, rb, batch;
    int per;         // tokens per CTA (grid.y covers the batch)
    int split;       // warps per row: 1 (eight rows per CTA) or 8 (one row per CTA)
};

// Weight element i of a row, four at a time (i a multiple of 4).
template <int T>
__device__ __forceinline__ void weights4(const uint8_t *row, int i, float (&wv)[4]) {
    if constexpr (T == Q38_GGML_F32) {
        const float4 v = *reinterpret_cast<const float4 *>(row + 4 * size_t(i));
        wv[0] = v.x, wv[1] = v.y, wv[2] = v.z, wv[3] = v.w;
    } else if constexpr (T == Q38_GGML_Q8_0) {
        // dot_q8_0_scalar, tensor.rs:103-117: the weight is d * q (one f32
        // product), then fma'd with x.
        const uint8_t *blk = row + size_t(i >> 5) * 34;
        const uint16_t *qs = reinterpret_cast<const uint16_t *>(blk + 2 + (i & 31));
        const uint32_t q01 = qs[0], q23 = qs[1];
        const float d = half_to_float(*reinterpret_cast<const uint16_t *>(blk));
        wv[0] = d * float(int8_t(q01 & 0xffu));
        wv[1] = d * float(int8_t(q01 >> 8));
        wv[2] = d * float(int8_t(q23 & 0xffu));
        wv[3] = d * float(int8_t(q23 >> 8));
    } else {
        const uint2 v = *reinterpret_cast<const uint2 *>(row + 2 * size_t(i));
        const uint32_t h[4] = {v.x & 0xffffu, v.x >> 16, v.y & 0xffffu, v.y >> 16};
#pragma unroll
        for (int e = 0; e < 4; ++e)
            wv[e] = T == Q38_GGML_F16 ? half_to_float(h[e]) : __uint_as_float(h[e] << 16);
    }
}

// The launch's tokens sit in shared memory ([batch][width] f32). Each warp
// covers a row (split 1) or an eighth of one (split 8); lanes take four
// consecutive elements per 128-element stride, four strides' loads issued
// before their fmas; the partial sums of a split row are added in warp order.
template <int T>
__global__ void __launch_bounds__(256) proj_f32_kernel(ProjF32Params p) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float part[8][kProjMaxTok];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // blockIdx.y: this CTA's group of up to p.per tokens.
    const int t0 = blockIdx.y * p.per, nt = min(p.per, p.batch - t0);
    const float *xg = p.x + size_t(t0) * p.width;
    float *outg = p.out + size_t(t0) * p.out_ld;
    if (blockIdx.y == 0) {
        // The weights are constant: this CTA's rows are requested into L2
        // before the wait for the previous kernel, so the loads below find
        // them there (once per row: the first token group asks).
        const int r0 = p.split == 1 ? blockIdx.x * 8 : blockIdx.x;
        const int nr = p.split == 1 ? min(8, p.rows - r0) : 1;
        const uint8_t *base = p.w + size_t(r0) * p.rb;
        const size_t bytes = size_t(nr) * p.rb;
        for (size_t off = size_t(threadIdx.x) * 128; off < bytes; off += 256 * 128) prefetch_l2(base + off);
    }
    pdl_wait_primary();  // x comes from an earlier kernel in the stream
    pdl_launch_dependents();
    for (int i = threadIdx.x; i < nt * p.width / 4; i += 256)
        reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(xg)[i];
    __syncthreads();
    const int row = p.split == 1 ? blockIdx.x * 8 + warp : blockIdx.x;
    const int len = p.width / p.split;
    const int i0 = p.split == 1 ? 0 : warp * len;
    float acc[kProjMaxTok];
#pragma unroll
    for (int t = 0; t < kProjMaxTok; ++t) acc[t] = 0.f;
    if (row < p.rows) {
        const uint8_t *w = p.w + size_t(row) * p.rb;
#pragma unroll 4
        for (int i = i0 + 4 * lane; i < i0 + len; i += 128) {
            float wv[4];
            weights4<T>(w, i, wv);
#pragma unroll
            for (int t = 0; t < kProjMaxTok; ++t)
                if (t < nt) {
                    const float4 x = *reinterpret_cast<const float4 *>(xs + t * p.width + i);
                    acc[t] = fmaf(wv[3], x.w, fmaf(wv[2], x.z, fmaf(wv[1], x.y, fmaf(wv[0], x.x, acc[t]))));
                }
        }
    }
#pragma unroll
    for (int t = 0; t < kProjMaxTok; ++t) {
        float v = acc[t];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        acc[t] = v;
    }
    if (p.split == 1) {
        if (lane == 0 && row < p.rows)
            for (int t = 0; t < nt; ++t)
                outg[size_t(t) * p.out_ld + row] = proj_epilogue(p.epi, p.rows, t0 + t, row, acc[t]);
        return;
    }
    if (lane == 0)
#pragma unroll
        for (int t = 0; t < kProjMaxTok; ++t) part[warp][t] = acc[t];
    __syncthreads();
    if (threadIdx.x < nt && row < p.rows) {
        float v = 0.f;
        for (int k = 0; k < 8; ++k) v += part[k][threadIdx.x];
        outg[size_t(threadIdx.x) * p.out_ld + row] = proj_epilogue(p.epi, p.rows, t0 + int(threadIdx.x), row, v);
    }
}

template <int T, int W>
cudaError_t launch_q8k(const ProjQ8KParams &p, int sm_count, cudaStream_t stream) {
    const ProjSmem lay = proj_smem_plan(p.stages, p.tile_bytes, p.batch, p.nblk, W, kTermsPerBlock<T>);
    // The attribute is set once per device to the budget, so later launches
    // make no extra driver calls (and can be captured in a graph).
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= kMaxDevices || !attr_set[dev]) {
        e = cudaFuncSetAttribute(proj_q8k_kernel<T, W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kProjSmemBudget));
        if (e != cudaSuccess) return e;
        if (dev < kMaxDevices) attr_set[dev] = true;
    }
    // One CTA per SM (the general form's block images take ~150 registers
    // a thread),
    // launched as a programmatic dependent of the previous kernel.
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(std::min(p.ntiles, sm_count));
    cfg.blockDim = dim3(32 * (W + 1));
    cfg.dynamicSmemBytes = lay.total;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, proj_q8k_kernel<T, W>, p);
}

template <int T>
cudaError_t launch_f32(const ProjF32Params &p, cudaStream_t stream) {
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= kMaxDevices || !attr_set[dev]) {
        e = cudaFuncSetAttribute(proj_f32_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kProjSmemBudget));
        if (e != cudaSuccess) return e;
        if (dev < kMaxDevices) attr_set[dev] = true;
    }
    const size_t smem = size_t(p.per) * p.width * sizeof(float);
    if (smem > kProjSmemBudget) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(p.split == 1 ? (p.rows + 7) / 8 : p.rows, (p.batch + p.per - 1) / p.per);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, proj_f32_kernel<T>, p);
}

// ---- f32-input projection of many tokens over few rows ---------------------
// Batches of 9+ tokens over up to 128 rows (the 48-row DeltaNet gates): the
// warp form above would stage each CTA's eight tokens whole (160 KB for a
// 5120-wide row) for one row, re-reading the batch from L2 once per row. Here
// a CTA takes one 128-value chunk of the width for 64 rows x 32 tokens: the
// tokens' values transposed ([k][t]) and the rows' weights decoded to f32
// ([k][row]) in shared memory, each thread a 4-row x 4-token register tile of
// fma chains over the chunk. The chunks' partial sums go to a workspace and a
// second kernel adds them in chunk order, then applies the epilogue.
// (Agrees with the reference's sequential fma chain to rounding, as the warp
// form does.)
constexpr int kTileK = 128, kTileRows = 64, kTileTok = 32, kTileThreads = 128;
constexpr int kTileXStride = kTileTok + 4;   // floats per k of the token tile (16-byte rows)
constexpr int kTileWStride = kTileRows + 4;  // floats per k of the weight tile
constexpr uint32_t kTileSmem = uint32_t(kTileK) * (kTileXStride + kTileWStride) * sizeof(float);
constexpr int kTileOut = kTileRows * kTileTok;  // partial sums per CTA

struct ProjTileParams {
    const uint8_t *w;
    const float *x;  // [batch][width]
    float *part;     // [chunk][row block][token block][kTileTok][kTileRows]
    float *out;
    long out_ld;
    ProjEpilogue epi;
    int rows, width, rb, batch, chunks;
};

template <int T>
__global__ void __launch_bounds__(kTileThreads) proj_f32_tile_kernel(ProjTileParams p) {
    extern __shared__ __align__(16) float tile_smem[];
    float *xs = tile_smem;                          // [kTileK][kTileXStride]
    float *ws = tile_smem + kTileK * kTileXStride;  // [kTileK][kTileWStride]
    const int chunk = blockIdx.x, r0 = blockIdx.y * kTileRows, t0 = blockIdx.z * kTileTok;
    const int k0 = chunk * kTileK, tid = threadIdx.x;
    // The weights are constant: decoded before the wait for the kernel that
    // wrote x. Lanes run over rows, so the transposed stores hit distinct banks;
    // the loops are unrolled so that every load is in flight before the first
    // is used.
    constexpr int kWIters = kTileRows * (kTileK / 4) / kTileThreads;
    constexpr int kXIters = kTileTok * (kTileK / 4) / kTileThreads;
    {
        float wv[kWIters][4];
#pragma unroll
        for (int it = 0; it < kWIters; ++it) {
            const int i = tid + it * kTileThreads, r = i % kTileRows, kq = (i / kTileRows) * 4;
#pragma unroll
            for (int e = 0; e < 4; ++e) wv[it][e] = 0.f;
            if (r0 + r < p.rows) weights4<T>(p.w + size_t(r0 + r) * p.rb, k0 + kq, wv[it]);
        }
#pragma unroll
        for (int it = 0; it < kWIters; ++it) {
            const int i = tid + it * kTileThreads, r = i % kTileRows, kq = (i / kTileRows) * 4;
#pragma unroll
            for (int e = 0; e < 4; ++e) ws[(kq + e) * kTileWStride + r] = wv[it][e];
        }
    }
    pdl_wait_primary();
    pdl_launch_dependents();
    {
        float4 xv[kXIters];
#pragma unroll
        for (int it = 0; it < kXIters; ++it) {
            const int i = tid + it * kTileThreads, t = i % kTileTok, kq = (i / kTileTok) * 4;
            xv[it] = t0 + t < p.batch ? *reinterpret_cast<const float4 *>(p.x + size_t(t0 + t) * p.width + k0 + kq)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int it = 0; it < kXIters; ++it) {
            const int i = tid + it * kTileThreads, t = i % kTileTok, kq = (i / kTileTok) * 4;
            xs[(kq + 0) * kTileXStride + t] = xv[it].x;
            xs[(kq + 1) * kTileXStride + t] = xv[it].y;
            xs[(kq + 2) * kTileXStride + t] = xv[it].z;
            xs[(kq + 3) * kTileXStride + t] = xv[it].w;
        }
    }
    __syncthreads();
    // Thread: rows 4 rq .. +3, tokens 4 tq .. +3.
    const int rq = tid & 15, tq = tid >> 4;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 4
    for (int k = 0; k < kTileK; ++k) {
        const float4 w4 = *reinterpret_cast<const float4 *>(ws + k * kTileWStride + 4 * rq);
        const float4 x4 = *reinterpret_cast<const float4 *>(xs + k * kTileXStride + 4 * tq);
        const float wr[4] = {w4.x, w4.y, w4.z, w4.w}, xt[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(wr[i], xt[j], acc[i][j]);
    }
    float *part = p.part + ((size_t(chunk) * gridDim.y + blockIdx.y) * gridDim.z + blockIdx.z) * kTileOut;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float4 *>(part + (4 * tq + j) * kTileRows + 4 * rq) =
            make_float4(acc[0][j], acc[1][j], acc[2][j], acc[3][j]);
}

// Output (t, row) = the chunks' partial sums added in chunk order, then the
// epilogue. Grid: (kTileOut / 256, row blocks, token blocks).
__global__ void __launch_bounds__(256) proj_f32_tile_reduce_kernel(ProjTileParams p) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    const int tl = i / kTileRows, rl = i % kTileRows;
    const int row = blockIdx.y * kTileRows + rl, t = blockIdx.z * kTileTok + tl;
    pdl_wait_primary();
    pdl_launch_dependents();
    if (row >= p.rows || t >= p.batch) return;
    const size_t stride = size_t(gridDim.y) * gridDim.z * kTileOut;
    const float *part = p.part + (size_t(blockIdx.y) * gridDim.z + blockIdx.z) * kTileOut + i;
    // Eight chunks' partials loaded at a time, added in chunk order.
    float v = part[0];
    int c = 1;
    for (; c + 8 <= p.chunks; c += 8) {
        float pv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) pv[u] = part[size_t(c + u) * stride];
#pragma unroll
        for (int u = 0; u < 8; ++u) v += pv[u];
    }
    for (; c < p.chunks; ++c) v += part[size_t(c) * stride];
    p.out[size_t(t) * p.out_ld + row] = proj_epilogue(p.epi, p.rows, t, row, v);
}

template <int T>
cudaError_t launch_f32_tile(const ProjTileParams &p, cudaStream_t stream) {
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= kMaxDevices || !attr_set[dev]) {
        e = cudaFuncSetAttribute(proj_f32_tile_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kTileSmem));
        if (e != cudaSuccess) return e;
        if (dev < kMaxDevices) attr_set[dev] = true;
    }
    const dim3 blocks((p.rows + kTileRows - 1) / kTileRows, (p.batch + kTileTok - 1) / kTileTok);
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(p.chunks, blocks.x, blocks.y);
    cfg.blockDim = dim3(kTileThreads);
    cfg.dynamicSmemBytes = kTileSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if ((e = cudaLaunchKernelEx(&cfg, proj_f32_tile_kernel<T>, p)) != cudaSuccess) return e;
    cfg.gridDim = dim3(kTileOut / 256, blocks.x, blocks.y);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&cfg, proj_f32_tile_reduce_kernel, p);
}

}  // namespace

size_t proj_f32_tile_part_bytes(int64_t rows, int64_t width, int batch) {
    return size_t((rows + kTileRows - 1) / kTileRows) * size_t((batch + kTileTok - 1) / kTileTok) *
           size_t(width / kTileK) * kTileOut * sizeof(float);
}

bool proj_f32_takes_tile(int type, int64_t rows, int64_t width, int batch) {
    return !proj_is_q8k_type(type) && batch >= 9 && rows <= kProjTileMaxRows && width % kTileK == 0 &&
           width >= kTileK;
}

bool proj_is_q8k_type(int type) {
    return type == Q38_GGML_Q2_K || type == Q38_GGML_Q3_K || type == Q38_GGML_Q4_K ||
           type == Q38_GGML_Q5_K || type == Q38_GGML_Q6_K || type == Q38_GGML_IQ4_NL ||
           type == Q38_GGML_IQ4_XS;
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
        case Q38_GGML_IQ4_NL: el = 32; by = 18; break;
        case Q38_GGML_IQ4_XS: el = 256; by = 136; break;
        default: return -1;
    }
    if (width <= 0 || width % el) return -1;
    return width / el * by;
}

int64_t proj_device_row_bytes(int type, int64_t width) {
    if (type == Q38_GGML_Q6_K && width > 0 && width % 256 == 0) return width / 256 * kQ6KDeviceBlock;
    return proj_row_bytes(type, width);
}

size_t proj_padded_bytes(int type, int64_t rows, int64_t width) {
    const int64_t rb = proj_device_row_bytes(type, width);
    return size_t((rows + kProjMaxTileRows) * rb) + 16;
}

cudaError_t launch_q8k_quantize(const float *x, int batch, int width, Q8KActivations act,
                                void *aos, cudaStream_t stream) {
    QuantizeParams p{x, act, static_cast<unsigned char *>(aos), width / 256, batch};
    const dim3 grid((p.nblk + 3) / 4, batch);
    q8k_quantize_kernel<<<grid, 128, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_proj_q8k(const ProjWeight &w, const float *x, int batch, float *out,
                            long out_ld, int *err, int sm_count, cudaStream_t stream,
                            const ProjEpilogue &epi) {
    const int nblk = int(w.width / 256);
    const int rb = int(w.row_bytes);
    ProjQ8KParams p{};
    p.w = static_cast<const uint8_t *>(w.data);
    p.out_ld = out_ld;
    p.err = err;
    p.rows = int(w.rows);
    p.nblk = nblk;
    p.rb = rb;
    // 16-row tiles, or 8 when three stages of 16 rows would not fit beside
    // one token's activations (so the copies stay ahead of the compute).
    // The one-token form (16 warps, a row each) keeps 16-row tiles while two
    // stages fit.
    const bool one_token = batch == 1 && nblk <= 32;
    p.tile_rows = kProjTileRows;
    const int terms = proj_terms_per_block(w.type);
    if (proj_smem_plan(0, 16u * rb, 1, nblk, kProjConsumerWarps, terms).total + (one_token ? 2u : 3u) * 16u * rb >
        kProjSmemBudget)
        p.tile_rows = 8;
    p.ntiles = int((w.rows + p.tile_rows - 1) / p.tile_rows);
    p.tile_bytes = uint32_t(p.tile_rows * rb);
    // Tokens per launch: up to kProjMaxTok, fewer when the activations would
    // leave room for less than two weight stages (wide Q6_K rows).
    int per = kProjMaxTok;
    while (per > 1 &&
           proj_smem_plan(0, p.tile_bytes, per, nblk, kProjConsumerWarps, terms).total + 2 * p.tile_bytes >
               kProjSmemBudget)
        --per;
    for (int t0 = 0; t0 < batch; t0 += per) {
        p.batch = std::min(per, batch - t0);
        p.x = x + size_t(t0) * nblk * 256;
        p.out = out + size_t(t0) * out_ld;
        p.epi = epi;
        p.epi.tok0 = epi.tok0 + t0;
        // Stages: as many as the budget allows, up to 4.
        // One token over rows of up to 32 blocks: the 16-warp form.
        const bool one = p.batch == 1 && nblk <= 32;
        const uint32_t fixed =
            proj_smem_plan(0, p.tile_bytes, p.batch, nblk, one ? kProjOneTokenWarps : kProjConsumerWarps, terms)
                .total;
        int stages = int((kProjSmemBudget - fixed) / p.tile_bytes);
        stages = std::min(stages, kMaxStages);
        if (stages < 2) return cudaErrorInvalidValue;
        p.stages = stages;
        cudaError_t e;
        switch (w.type) {
            case Q38_GGML_Q2_K:
                e = one ? launch_q8k<Q38_GGML_Q2_K, kProjOneTokenWarps>(p, sm_count, stream)
                        : launch_q8k<Q38_GGML_Q2_K, kProjConsumerWarps>(p, sm_count, stream);
                break;
            case Q38_GGML_Q3_K:
                e = one ? launch_q8k<Q38_GGML_Q3_K, kProjOneTokenWarps>(p, sm_count, stream)
                        : launch_q8k<Q38_GGML_Q3_K, kProjConsumerWarps>(p, sm_count, stream);
                break;
            case Q38_GGML_Q4_K:
                e = one ? launch_q8k<Q38_GGML_Q4_K, kProjOneTokenWarps>(p, sm_count, stream)
                        : launch_q8k<Q38_GGML_Q4_K, kProjConsumerWarps>(p, sm_count, stream);
                break;
            case Q38_GGML_Q5_K:
                e = one ? launch_q8k<Q38_GGML_Q5_K, kProjOneTokenWarps>(p, sm_count, stream)
                        : launch_q8k<Q38_GGML_Q5_K, kProjConsumerWarps>(p, sm_count, stream);
                break;
            case Q38_GGML_Q6_K:
                e = one ? launch_q8k<Q38_GGML_Q6_K, kProjOneTokenWarps>(p, sm_count, stream)
                        : launch_q8k<Q38_GGML_Q6_K, kProjConsumerWarps>(p, sm_count, stream);
                break;
            case Q38_GGML_IQ4_NL:
                e = one ? launch_q8k<Q38_GGML_IQ4_NL, kProjOneTokenWarps>(p, sm_count, stream)
                        : launch_q8k<Q38_GGML_IQ4_NL, kProjConsumerWarps>(p, sm_count, stream);
                break;
            case Q38_GGML_IQ4_XS:
                e = one ? launch_q8k<Q38_GGML_IQ4_XS, kProjOneTokenWarps>(p, sm_count, stream)
                        : launch_q8k<Q38_GGML_IQ4_XS, kProjConsumerWarps>(p, sm_count, stream);
                break;
            default: return cudaErrorInvalidValue;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_proj_f32(const ProjWeight &w, const float *x, int batch, float *out,
                            long out_ld, cudaStream_t stream, const ProjEpilogue &epi, float *part) {
    if (part && proj_f32_takes_tile(w.type, w.rows, w.width, batch)) {
        if (reinterpret_cast<uintptr_t>(x) % 16) return cudaErrorInvalidValue;
        ProjTileParams t{};
        t.w = static_cast<const uint8_t *>(w.data);
        t.x = x;
        t.part = part;
        t.out = out;
        t.out_ld = out_ld;
        t.epi = epi;
        t.rows = int(w.rows);
        t.width = int(w.width);
        t.rb = int(w.row_bytes);
        t.batch = batch;
        t.chunks = int(w.width / kTileK);
        switch (w.type) {
            case Q38_GGML_F32: return launch_f32_tile<Q38_GGML_F32>(t, stream);
            case Q38_GGML_F16: return launch_f32_tile<Q38_GGML_F16>(t, stream);
            case Q38_GGML_BF16: return launch_f32_tile<Q38_GGML_BF16>(t, stream);
            case Q38_GGML_Q8_0: return launch_f32_tile<Q38_GGML_Q8_0>(t, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    ProjF32Params p{};
    p.epi = epi;
    p.w = static_cast<const uint8_t *>(w.data);
    p.out_ld = out_ld;
    p.rows = int(w.rows);
    p.width = int(w.width);
    p.rb = int(w.row_bytes);
    // Few rows: eight warps per row (each an eighth of it, whole Q8_0 blocks).
    p.split = (w.rows < 2 * 148 && w.width % 256 == 0) ? 8 : 1;
    // Tokens per launch: as many as fit the shared-memory budget, up to 8.
    const int per = std::min<int64_t>(kProjMaxTok, kProjSmemBudget / (w.width * sizeof(float)));
    if (per < 1 || w.width % 4) return cudaErrorInvalidValue;
    p.batch = batch;
    p.per = per;
    p.x = x;
    p.out = out;
    switch (w.type) {
        case Q38_GGML_F32: return launch_f32<Q38_GGML_F32>(p, stream);
        case Q38_GGML_F16: return launch_f32<Q38_GGML_F16>(p, stream);
        case Q38_GGML_BF16: return launch_f32<Q38_GGML_BF16>(p, stream);
        case Q38_GGML_Q8_0: return launch_f32<Q38_GGML_Q8_0>(p, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace q38
