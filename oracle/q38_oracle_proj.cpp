// q38_oracle_proj.cpp -- CPU restatement of the reference's projections on
// either side of the attention cores. TEST INFRASTRUCTURE ONLY (parity checker
// and timed CPU baseline); the product library never links it.
//
// Follows, in the reference (StepfenShawn/qwen3.8_27b_in_rust):
//   src/kernel/quant.rs:16-45     f16_to_f32 (ggml half -> f32, subnormals included)
//   src/kernel/quant.rs:56-124    quantize_block / quantize_q8_k (Q8_K activations)
//   src/kernel/tensor.rs:23-44    scale_min_k4, unpack_q3_scales
//   src/kernel/tensor.rs:46-53    row_bytes
//   src/kernel/tensor.rs:79-117   dot_{f32,f16,bf16,q8_0}_scalar (the f32-input path)
//   src/kernel/tensor.rs:301-460  dot_q{2,3,4,5,6}_k_q8_k_scalar (the integer path)
//   src/kernel/iq.rs:96-135, 311-335, 355-405  IQ4_NL / IQ4_XS: group layout,
//                                 f32 decode + fma dot, integer dots
//   src/kernel/iq_tables.rs:52-56 kvalues_iq4nl
//   src/kernel/tensor.rs:954-1027 gemv_rows / gemm_rows (token-major output)
//   src/model/ops.rs:105-120      matrix_type_q8_k (which weights take the integer path)
//   src/model/ops.rs:617-640      quantize_input / project
//   src/model/ops.rs:1016-1031    batch_project
// The scalar forms are the definition: the reference's AVX2 forms of the same
// dots (src/kernel/x86/tensor.rs) sum in 8 lanes and agree with them to
// rounding, which the reference's own tests accept (tensor.rs:604-700).
//
// Built with -ffp-contract=off, so a*b - c*d is two rounded products and a
// rounded difference, as in Rust.
#include "q38_oracle.h"

#include <cmath>
#include <cstdint>
#include <cstring>

#include <omp.h>

namespace {

constexpr size_t kBlock = 256;  // Q38_Q8_K_BLOCK_SIZE, src/kernel/mod.rs:2

inline uint16_t rd16(const uint8_t *p) { return uint16_t(p[0] | (uint16_t(p[1]) << 8)); }
inline float rdf32(const uint8_t *p) {
    float f;
    std::memcpy(&f, p, 4);
    return f;
}

// f16_to_f32, quant.rs:21-45: IEEE half to single, subnormals normalised by
// shifting the mantissa up.
float f16_to_f32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    const uint32_t exponent = (h >> 10) & 0x1fu;
    uint32_t mantissa = h & 0x3ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            uint32_t shift = 0;
            while ((mantissa & 0x400u) == 0) {
                mantissa <<= 1;
                ++shift;
            }
            mantissa &= 0x3ffu;
            bits = sign | ((127u - 14u - shift) << 23) | (mantissa << 13);
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

float bf16_to_f32(const uint8_t *p) {
    const uint32_t bits = uint32_t(rd16(p)) << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// nearest_int, quant.rs:16-20: round to nearest even through the f32 adder
// (1.5 * 2^23 pins the integer into the low mantissa bits).
int32_t nearest_int(float v) {
    const float shifted = v + 12582912.0f;
    uint32_t bits;
    std::memcpy(&bits, &shifted, 4);
    return int32_t(bits & 0x007fffffu) - 0x00400000;
}

// quantize_block, quant.rs:56-96. The block maximum is the first value of the
// largest magnitude (strict >), and keeps its sign.
void quantize_block(q38o_q8k_block *out, const float *v) {
    float maximum = 0.0f, amax = 0.0f;
    for (size_t i = 0; i < kBlock; ++i) {
        const float a = std::fabs(v[i]);
        if (a > amax) {
            amax = a;
            maximum = v[i];
        }
    }
    if (amax == 0.0f) {
        out->scale = 0.0f;
        std::memset(out->quants, 0, sizeof(out->quants));
        std::memset(out->sums, 0, sizeof(out->sums));
        return;
    }
    const float inverse = -127.0f / maximum;
    for (size_t i = 0; i < kBlock; ++i) {
        int32_t q = nearest_int(inverse * v[i]);
        if (q > 127) q = 127;
        out->quants[i] = int8_t(q);
    }
    for (size_t g = 0; g < kBlock / 16; ++g) {
        int32_t s = 0;
        for (size_t i = 0; i < 16; ++i) s += out->quants[g * 16 + i];
        out->sums[g] = int16_t(s);
    }
    out->scale = 1.0f / inverse;
}

// scale_min_k4, tensor.rs:23-32: the 6-bit (scale, min) pair j of a K-quant
// super-block from its 12 packed bytes.
inline void scale_min_k4(int j, const uint8_t *q, int &sc, int &mn) {
    if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// unpack_q3_scales, tensor.rs:34-44: sixteen signed 6-bit scales.
inline void unpack_q3_scales(const uint8_t *p, int8_t (&s)[16]) {
    for (int i = 0; i < 16; ++i) {
        const int low = i < 8 ? (p[i] & 15) : (p[i - 8] >> 4);
        const int high = (p[8 + i % 4] >> (2 * (i / 4))) & 3;
        s[i] = int8_t((low | (high << 4)) - 32);
    }
}

// ---- f32-input dots, tensor.rs:79-117 -------------------------------------

float dot_f32(const uint8_t *d, const float *x, size_t n) {
    float t = 0.0f;
    for (size_t i = 0; i < n; ++i) t = std::fmaf(rdf32(d + 4 * i), x[i], t);
    return t;
}

float dot_f16(const uint8_t *d, const float *x, size_t n) {
    float t = 0.0f;
    for (size_t i = 0; i < n; ++i) t = std::fmaf(f16_to_f32(rd16(d + 2 * i)), x[i], t);
    return t;
}

float dot_bf16(const uint8_t *d, const float *x, size_t n) {
    float t = 0.0f;
    for (size_t i = 0; i < n; ++i) t = std::fmaf(bf16_to_f32(d + 2 * i), x[i], t);
    return t;
}

float dot_q8_0(const uint8_t *d, const float *x, size_t n) {
    float t = 0.0f;
    for (size_t base = 0, b = 0; base < n; base += 32, ++b) {
        const uint8_t *blk = d + b * 34;
        const float scale = f16_to_f32(rd16(blk));
        for (int i = 0; i < 32; ++i) t = std::fmaf(scale * float(int8_t(blk[2 + i])), x[base + i], t);
    }
    return t;
}

// ---- integer dots against Q8_K activations, tensor.rs:301-460 -------------

float dot_q2_k(const uint8_t *data, const q38o_q8k_block *q, size_t blocks) {
    float total = 0.0f;
    for (size_t b = 0; b < blocks; ++b) {
        const uint8_t *blk = data + b * 84;
        const uint8_t *scales = blk, *quants = blk + 16;
        const float d = f16_to_f32(rd16(blk + 80)) * q[b].scale;
        const float dmin = f16_to_f32(rd16(blk + 82)) * q[b].scale;
        int32_t weighted = 0, minimum = 0;
        for (int half = 0; half < 2; ++half) {
            for (int field = 0; field < 4; ++field) {
                const int si = half * 8 + field * 2, shift = field * 2;
                int32_t dot0 = 0, dot1 = 0;
                for (int l = 0; l < 16; ++l) {
                    dot0 += ((quants[half * 32 + l] >> shift) & 3) * q[b].quants[half * 128 + field * 32 + l];
                    dot1 += ((quants[half * 32 + 16 + l] >> shift) & 3) *
                            q[b].quants[half * 128 + field * 32 + 16 + l];
                }
                weighted += (scales[si] & 15) * dot0 + (scales[si + 1] & 15) * dot1;
                minimum += (scales[si] >> 4) * q[b].sums[si];
                minimum += (scales[si + 1] >> 4) * q[b].sums[si + 1];
            }
        }
        total += d * float(weighted) - dmin * float(minimum);
    }
    return total;
}

float dot_q3_k(const uint8_t *data, const q38o_q8k_block *q, size_t blocks) {
    float total = 0.0f;
    for (size_t b = 0; b < blocks; ++b) {
        const uint8_t *blk = data + b * 110;
        const uint8_t *high = blk, *low = blk + 32;
        int8_t scales[16];
        unpack_q3_scales(blk + 96, scales);
        const float d = f16_to_f32(rd16(blk + 108)) * q[b].scale;
        int32_t weighted = 0;
        int group = 0;
        for (int half = 0; half < 2; ++half) {
            for (int field = 0; field < 4; ++field, ++group) {
                const uint8_t bit = uint8_t(1u << group);
                for (int l = 0; l < 32; ++l) {
                    const int qv = ((low[half * 32 + l] >> (field * 2)) & 3) - ((high[l] & bit) ? 0 : 4);
                    const int sc = l < 16 ? scales[group * 2] : scales[group * 2 + 1];
                    weighted += sc * qv * q[b].quants[half * 128 + field * 32 + l];
                }
            }
        }
        total += d * float(weighted);
    }
    return total;
}

float dot_q4_k(const uint8_t *data, const q38o_q8k_block *q, size_t blocks) {
    float total = 0.0f;
    for (size_t b = 0; b < blocks; ++b) {
        const uint8_t *blk = data + b * 144;
        const float d = f16_to_f32(rd16(blk)) * q[b].scale;
        const float dmin = f16_to_f32(rd16(blk + 2)) * q[b].scale;
        const uint8_t *scales = blk + 4, *quants = blk + 16;
        int32_t weighted = 0, minimum = 0;
        for (int c = 0; c < 4; ++c) {
            int sc0, mn0, sc1, mn1;
            scale_min_k4(2 * c, scales, sc0, mn0);
            scale_min_k4(2 * c + 1, scales, sc1, mn1);
            int32_t dot0 = 0, dot1 = 0;
            for (int i = 0; i < 32; ++i) {
                dot0 += (quants[c * 32 + i] & 15) * q[b].quants[c * 64 + i];
                dot1 += (quants[c * 32 + i] >> 4) * q[b].quants[c * 64 + 32 + i];
            }
            weighted += sc0 * dot0 + sc1 * dot1;
            minimum += mn0 * (q[b].sums[c * 4] + q[b].sums[c * 4 + 1]);
            minimum += mn1 * (q[b].sums[c * 4 + 2] + q[b].sums[c * 4 + 3]);
        }
        total += d * float(weighted) - dmin * float(minimum);
    }
    return total;
}

float dot_q5_k(const uint8_t *data, const q38o_q8k_block *q, size_t blocks) {
    float total = 0.0f;
    for (size_t b = 0; b < blocks; ++b) {
        const uint8_t *blk = data + b * 176;
        const float d = f16_to_f32(rd16(blk)) * q[b].scale;
        const float dmin = f16_to_f32(rd16(blk + 2)) * q[b].scale;
        const uint8_t *scales = blk + 4, *high = blk + 16, *low = blk + 48;
        int32_t weighted = 0, minimum = 0;
        for (int c = 0; c < 4; ++c) {
            int sc0, mn0, sc1, mn1;
            scale_min_k4(2 * c, scales, sc0, mn0);
            scale_min_k4(2 * c + 1, scales, sc1, mn1);
            const uint8_t h0 = uint8_t(1u << (2 * c)), h1 = uint8_t(2u << (2 * c));
            int32_t dot0 = 0, dot1 = 0;
            for (int i = 0; i < 32; ++i) {
                const int q0 = (low[c * 32 + i] & 15) + ((high[i] & h0) ? 16 : 0);
                const int q1 = (low[c * 32 + i] >> 4) + ((high[i] & h1) ? 16 : 0);
                dot0 += q0 * q[b].quants[c * 64 + i];
                dot1 += q1 * q[b].quants[c * 64 + 32 + i];
            }
            weighted += sc0 * dot0 + sc1 * dot1;
            minimum += mn0 * (q[b].sums[c * 4] + q[b].sums[c * 4 + 1]);
            minimum += mn1 * (q[b].sums[c * 4 + 2] + q[b].sums[c * 4 + 3]);
        }
        total += d * float(weighted) - dmin * float(minimum);
    }
    return total;
}

float dot_q6_k(const uint8_t *data, const q38o_q8k_block *q, size_t blocks) {
    float total = 0.0f;
    for (size_t b = 0; b < blocks; ++b) {
        const uint8_t *blk = data + b * 210;
        const float d = f16_to_f32(rd16(blk + 208)) * q[b].scale;
        const int8_t *scales = reinterpret_cast<const int8_t *>(blk + 192);
        int32_t weighted = 0;
        for (int half = 0; half < 2; ++half) {
            const int base = half * 128;
            for (int i = 0; i < 32; ++i) {
                const int si = half * 8 + i / 16;
                const uint8_t l0 = blk[half * 64 + i], l1 = blk[half * 64 + i + 32];
                const uint8_t h = blk[128 + half * 32 + i];
                const int q0 = ((l0 & 15) | ((h & 3) << 4)) - 32;
                const int q1 = ((l1 & 15) | (((h >> 2) & 3) << 4)) - 32;
                const int q2 = ((l0 >> 4) | (((h >> 4) & 3) << 4)) - 32;
                const int q3 = ((l1 >> 4) | (((h >> 6) & 3) << 4)) - 32;
                weighted += scales[si] * q0 * q[b].quants[base + i];
                weighted += scales[si + 2] * q1 * q[b].quants[base + 32 + i];
                weighted += scales[si + 4] * q2 * q[b].quants[base + 64 + i];
                weighted += scales[si + 6] * q3 * q[b].quants[base + 96 + i];
            }
        }
        total += d * float(weighted);
    }
    return total;
}

// ---- IQ4_NL / IQ4_XS, src/kernel/iq.rs -------------------------------------
// Both map a 4-bit index to one of 16 signed values (kvalues_iq4nl,
// iq_tables.rs:52-56: the format's own table, kept as it is). Within a
// 32-value group, byte i holds value i in its low nibble and value i + 16 in
// its high nibble.
constexpr int8_t kIq4Values[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                   1,    13,   25,  38,  53,  69,  89,  113};
constexpr size_t kIq4NlSuper = 144;  // eight 18-byte IQ4_NL blocks per 256 values
constexpr size_t kIq4XsBlock = 136;

// IQ4_XS group scale (iq.rs:392-393): 4 bits from scales_l, 2 from scales_h.
inline int iq4_xs_scale(const uint8_t *blk, int g) {
    const uint16_t high = rd16(blk + 2);
    return ((blk[4 + g / 2] >> (4 * (g % 2))) & 15) | (((high >> (2 * g)) & 3) << 4);
}

// dot_iq4_nl_q8_k, iq.rs:355-377: per 32-value group an f16 scale and 16
// nibble bytes; every group adds its own term d * weighted to the total.
float dot_iq4_nl(const uint8_t *data, const q38o_q8k_block *q, size_t blocks) {
    float total = 0.0f;
    for (size_t b = 0; b < blocks; ++b)
        for (int g = 0; g < 8; ++g) {
            const uint8_t *grp = data + b * kIq4NlSuper + g * 18;
            const float d = f16_to_f32(rd16(grp)) * q[b].scale;
            int32_t weighted = 0;
            for (int i = 0; i < 16; ++i) {
                weighted += q[b].quants[g * 32 + i] * kIq4Values[grp[2 + i] & 15];
                weighted += q[b].quants[g * 32 + i + 16] * kIq4Values[grp[2 + i] >> 4];
            }
            total += d * float(weighted);
        }
    return total;
}

// dot_iq4_xs_q8_k, iq.rs:379-405: 136 bytes (d | scales_h | scales_l[4] |
// 128 nibble bytes); the group sums weighted by (scale - 32), one term per
// block.
float dot_iq4_xs(const uint8_t *data, const q38o_q8k_block *q, size_t blocks) {
    float total = 0.0f;
    for (size_t b = 0; b < blocks; ++b) {
        const uint8_t *blk = data + b * kIq4XsBlock;
        const float d = f16_to_f32(rd16(blk)) * q[b].scale;
        int32_t weighted = 0;
        for (int g = 0; g < 8; ++g) {
            int32_t sub = 0;
            for (int i = 0; i < 16; ++i) {
                const uint8_t packed = blk[8 + 16 * g + i];
                sub += q[b].quants[g * 32 + i] * kIq4Values[packed & 15];
                sub += q[b].quants[g * 32 + i + 16] * kIq4Values[packed >> 4];
            }
            weighted += (iq4_xs_scale(blk, g) - 32) * sub;
        }
        total += d * float(weighted);
    }
    return total;
}

// dequant_block (iq.rs:109-135) of one 256-value unit, then dot_row_f32
// (iq.rs:311-335): an fma chain over the decoded values in element order.
float dot_iq4_f32(int type, const uint8_t *data, const float *x, size_t n) {
    float total = 0.0f;
    float v[256];
    for (size_t base = 0, b = 0; base < n; base += 256, ++b) {
        if (type == Q38O_GGML_IQ4_NL) {
            for (int g = 0; g < 8; ++g) {
                const uint8_t *grp = data + b * kIq4NlSuper + g * 18;
                const float d = f16_to_f32(rd16(grp));
                for (int i = 0; i < 16; ++i) {
                    v[g * 32 + i] = d * float(kIq4Values[grp[2 + i] & 15]);
                    v[g * 32 + i + 16] = d * float(kIq4Values[grp[2 + i] >> 4]);
                }
            }
        } else {
            const uint8_t *blk = data + b * kIq4XsBlock;
            const float d = f16_to_f32(rd16(blk));
            for (int g = 0; g < 8; ++g) {
                const float ds = d * float(iq4_xs_scale(blk, g) - 32);
                for (int i = 0; i < 16; ++i) {
                    const uint8_t packed = blk[8 + 16 * g + i];
                    v[g * 32 + i] = ds * float(kIq4Values[packed & 15]);
                    v[g * 32 + i + 16] = ds * float(kIq4Values[packed >> 4]);
                }
            }
        }
        for (int i = 0; i < 256; ++i) total = std::fmaf(v[i], x[base + i], total);
    }
    return total;
}

bool parallel_rows(size_t rows, size_t per_row) {
    // q38_parallel_over, src/kernel/mod.rs:15-17 (the result does not depend
    // on it: every output is the same dot on the same bytes).
    return rows >= 2 && rows * per_row >= (size_t(1) << 18);
}

}  // namespace

extern "C" {

float q38o_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

int q38o_is_q8k_type(int type) {
    return type == Q38O_GGML_Q2_K || type == Q38O_GGML_Q3_K || type == Q38O_GGML_Q4_K ||
           type == Q38O_GGML_Q5_K || type == Q38O_GGML_Q6_K || type == Q38O_GGML_IQ4_NL ||
           type == Q38O_GGML_IQ4_XS;
}

int q38o_row_bytes(int type, size_t width, size_t *out) {
    size_t elems, bytes;
    switch (type) {
        case Q38O_GGML_F32: elems = 1; bytes = 4; break;
        case Q38O_GGML_F16:
        case Q38O_GGML_BF16: elems = 1; bytes = 2; break;
        case Q38O_GGML_Q8_0: elems = 32; bytes = 34; break;
        case Q38O_GGML_Q2_K: elems = 256; bytes = 84; break;
        case Q38O_GGML_Q3_K: elems = 256; bytes = 110; break;
        case Q38O_GGML_Q4_K: elems = 256; bytes = 144; break;
        case Q38O_GGML_Q5_K: elems = 256; bytes = 176; break;
        case Q38O_GGML_Q6_K: elems = 256; bytes = 210; break;
        case Q38O_GGML_IQ4_NL: elems = 32; bytes = 18; break;
        case Q38O_GGML_IQ4_XS: elems = 256; bytes = 136; break;
        default: return -1;
    }
    if (width % elems) return -1;
    *out = width / elems * bytes;
    return 0;
}

int q38o_quantize_q8_k(const float *input, size_t length, q38o_q8k_block *out) {
    if (length % kBlock) return -1;
    const size_t blocks = length / kBlock;
#pragma omp parallel for schedule(static) if (parallel_rows(blocks, kBlock)) num_threads(q38o_get_threads())
    for (size_t b = 0; b < blocks; ++b) quantize_block(out + b, input + b * kBlock);
    return 0;
}

float q38o_dot_row_f32(int type, const uint8_t *row, const float *x, size_t width) {
    switch (type) {
        case Q38O_GGML_F32: return dot_f32(row, x, width);
        case Q38O_GGML_F16: return dot_f16(row, x, width);
        case Q38O_GGML_BF16: return dot_bf16(row, x, width);
        case Q38O_GGML_Q8_0: return dot_q8_0(row, x, width);
        // The IQ kernels step over 256-value units (iq.rs:43-61).
        case Q38O_GGML_IQ4_NL:
        case Q38O_GGML_IQ4_XS: return width % kBlock ? NAN : dot_iq4_f32(type, row, x, width);
        default: return NAN;
    }
}

float q38o_dot_row_q8_k(int type, const uint8_t *row, const q38o_q8k_block *q, size_t blocks) {
    switch (type) {
        case Q38O_GGML_Q2_K: return dot_q2_k(row, q, blocks);
        case Q38O_GGML_Q3_K: return dot_q3_k(row, q, blocks);
        case Q38O_GGML_Q4_K: return dot_q4_k(row, q, blocks);
        case Q38O_GGML_Q5_K: return dot_q5_k(row, q, blocks);
        case Q38O_GGML_Q6_K: return dot_q6_k(row, q, blocks);
        case Q38O_GGML_IQ4_NL: return dot_iq4_nl(row, q, blocks);
        case Q38O_GGML_IQ4_XS: return dot_iq4_xs(row, q, blocks);
        default: return NAN;
    }
}

int q38o_gemm_f32(int type, const uint8_t *w, size_t rows, size_t width, const float *input,
                  size_t batch, float *out) {
    size_t rb;
    if (q38o_row_bytes(type, width, &rb) || q38o_is_q8k_type(type) || batch == 0) return -1;
#pragma omp parallel for schedule(static) if (parallel_rows(rows, width * batch)) num_threads(q38o_get_threads())
    for (size_t r = 0; r < rows; ++r)
        for (size_t t = 0; t < batch; ++t)
            out[t * rows + r] = q38o_dot_row_f32(type, w + r * rb, input + t * width, width);
    return 0;
}

int q38o_gemm_q8_k(int type, const uint8_t *w, size_t rows, size_t width,
                   const q38o_q8k_block *act, size_t batch, float *out) {
    size_t rb;
    if (q38o_row_bytes(type, width, &rb) || !q38o_is_q8k_type(type) || width % kBlock || batch == 0)
        return -1;
    const size_t blocks = width / kBlock;
#pragma omp parallel for schedule(static) if (parallel_rows(rows, width * batch)) num_threads(q38o_get_threads())
    for (size_t r = 0; r < rows; ++r)
        for (size_t t = 0; t < batch; ++t)
            out[t * rows + r] = q38o_dot_row_q8_k(type, w + r * rb, act + t * blocks, blocks);
    return 0;
}

int q38o_project(int type, const uint8_t *w, size_t rows, size_t width, const float *input,
                 size_t batch, float *out) {
    if (!q38o_is_q8k_type(type)) return q38o_gemm_f32(type, w, rows, width, input, batch, out);
    if (width % kBlock) return -1;
    const size_t blocks = width / kBlock;
    q38o_q8k_block *act = new q38o_q8k_block[batch * blocks];
    int rc = 0;
    for (size_t t = 0; t < batch && rc == 0; ++t)
        rc = q38o_quantize_q8_k(input + t * width, width, act + t * blocks);
    if (rc == 0) rc = q38o_gemm_q8_k(type, w, rows, width, act, batch, out);
    delete[] act;
    return rc;
}

}  // extern "C"
