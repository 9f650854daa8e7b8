// deltanet_prefill.cu -- chunked Gated DeltaNet prefill. Replaces the per-token
// linear_core loop of batch_linear_attention (src/model/ops.rs:1088-1099).
//
// The reference's step for value head h (ops.rs:690-713), per token r:
//   S <- e^{g_r} S;  u_r = beta_r (v_r - S k_r);  S <- S + u_r k_r^T;
//   o_r = (S q_r) / sqrt(128)
// where S is [128 value rows][128 key dims]. Over a chunk of C = 64 tokens
// with in-chunk cumulative log-decay gamma_r = g_1 + ... + g_r and the state
// S0 before the chunk, the same recurrence in closed form (WY/UT form) is
//   A[r][s] = beta_r e^{gamma_r - gamma_s} (k_r . k_s)   (s < r),  T = (I + A)^-1
//   W  = T diag(beta e^gamma) K,      Ut = T diag(beta) V        (chunk-local)
//   U  = Ut - W S0^T                                             (needs S0)
//   O  = diag(e^gamma) Q S0^T + P U,  P[r][s] = e^{gamma_r-gamma_s} (q_r . k_s) (s <= r)
//   S' = e^{gamma_C} S0 + U^T diag(e^{gamma_C - gamma}) K
// Rows of S evolve independently (row j only sees v[j] and u[j]), so the
// state pass splits each head's 128 rows into 4 slices of 32.
//
//   L1 linear_prefill_conv   one thread per (channel, 64-token segment,
//                            sequence): the kernel-4 causal conv with the
//                            carried state (multiply then add, ops.rs:665-676)
//                            and SiLU, in place; a pre-pass saves the three
//                            original inputs before each segment so segments
//                            run in parallel; the last three inputs become the
//                            new conv state.
//   L2 linear_prefill_norm   one CTA per (token, sequence): L2-norm of the q and
//                            k heads (f64 sums) and the beta/alpha gates, in place.
//   L3 linear_prefill_local  one CTA per (chunk, value head, sequence): the
//                            chunk-local W, Ut, P and gamma (all chunks in
//                            parallel).
//   L4 linear_prefill_state  one CTA per (32-row slice, value head, sequence):
//                            walks the chunks in order, carrying its state
//                            slice in shared memory; writes O (scaled by
//                            1/sqrt(128)) and the final state.
//   L5 linear_prefill_out    one CTA per (token, sequence): per-head RMSNorm
//                            with ssm_norm and the SiLU(z) gate (ops.rs:735-740).
//
// Everything is f32 on the CUDA cores (register-tiled products from shared
// memory), so the chunked result stays within f32 rounding of the per-token
// recurrence.
#include "q38_common.cuh"

namespace q38 {
namespace {

constexpr int kC = 64;       // chunk length
constexpr int kD = kLinHeadDim;  // 128
constexpr int kSlice = 32;   // state rows per CTA in the state pass

// ----------------------------------------------------------------------------
// L1: conv + SiLU, 64-token segments in parallel
// ----------------------------------------------------------------------------
struct ConvParams {
    float *qkv;          // [nseq][count][qkv_dim]
    float *conv_state;   // slot base [batch][qkv_dim][3]
    const float *conv_w; // [qkv_dim][4]
    float *bounds;       // [nseq][nseg][3][qkv_dim]: inputs preceding each segment
    int seq0, count, qkv_dim, nseg;
};

constexpr int kSeg = 64;  // tokens per conv segment

// The three inputs that precede segment g: the carried conv state for g = 0,
// otherwise the (not yet convolved) inputs g*kSeg-3 .. g*kSeg-1.
__global__ void __launch_bounds__(128) linear_prefill_conv_bounds_kernel(ConvParams p) {
    const int c = blockIdx.x * 128 + threadIdx.x;
    const int g = blockIdx.y, s = blockIdx.z;
    if (c >= p.qkv_dim) return;
    float *dst = p.bounds + (size_t(s) * p.nseg + g) * 3 * p.qkv_dim + c;
    if (g == 0) {
        const float *st = p.conv_state + (size_t(p.seq0 + s) * p.qkv_dim + c) * 3;
        for (int k = 0; k < 3; ++k) dst[size_t(k) * p.qkv_dim] = st[k];
    } else {
        const float *x = p.qkv + (size_t(s) * p.count + g * kSeg - 3) * p.qkv_dim + c;
        for (int k = 0; k < 3; ++k) dst[size_t(k) * p.qkv_dim] = x[size_t(k) * p.qkv_dim];
    }
}

// One thread per (channel, segment, sequence): the kernel-4 causal conv over
// the segment (multiply then add, ops.rs:665-676) and SiLU, in place. The
// last segment leaves the last three inputs as the new conv state.
__global__ void __launch_bounds__(128) linear_prefill_conv_kernel(ConvParams p) {
    const int c = blockIdx.x * 128 + threadIdx.x;
    const int g = blockIdx.y, s = blockIdx.z;
    if (c >= p.qkv_dim) return;
    const float *bnd = p.bounds + (size_t(s) * p.nseg + g) * 3 * p.qkv_dim + c;
    float s0 = bnd[0], s1 = bnd[p.qkv_dim], s2 = bnd[2 * size_t(p.qkv_dim)];
    const float4 w = reinterpret_cast<const float4 *>(p.conv_w)[c];
    const int t0 = g * kSeg, t1 = min(p.count, t0 + kSeg);
    float *x = p.qkv + size_t(s) * p.count * p.qkv_dim + c;
#pragma unroll 8
    for (int t = t0; t < t1; ++t) {
        const float xt = x[size_t(t) * p.qkv_dim];
        float v = s0 * w.x;
        v += s1 * w.y;
        v += s2 * w.z;
        v += xt * w.w;
        s0 = s1;
        s1 = s2;
        s2 = xt;
        x[size_t(t) * p.qkv_dim] = siluf_ref(v);
    }
    if (g == p.nseg - 1) {
        float *st = p.conv_state + (size_t(p.seq0 + s) * p.qkv_dim + c) * 3;
        st[0] = s0;
        st[1] = s1;
        st[2] = s2;
    }
}

// ----------------------------------------------------------------------------
// L2: q/k L2-norm and gates
// ----------------------------------------------------------------------------
struct NormParams {
    float *qkv;
    float *beta, *alpha;  // [nseq][count][v_heads]
    const float *dt_bias, *ssm_a;
    int count, qk_heads, v_heads, qkv_dim;
    float eps;
};

__global__ void __launch_bounds__(256) linear_prefill_norm_kernel(NormParams p) {
    const int t = blockIdx.x, s = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t tok = size_t(s) * p.count + t;
    float *row = p.qkv + tok * p.qkv_dim;
    // 2*qk_heads heads of 128 channels (q heads then k heads), one warp each.
    for (int hh = warp; hh < 2 * p.qk_heads; hh += 8) {
        float4 *v4 = reinterpret_cast<float4 *>(row + hh * kD) + lane;
        float4 v = *v4;
        double sum = double(v.x) * v.x + double(v.y) * v.y + double(v.z) * v.z + double(v.w) * v.w;
        sum = warp_sum_f64(sum);
        const float scale = 1.0f / fmaxf(sqrtf(float(sum)), p.eps);
        v.x *= scale;
        v.y *= scale;
        v.z *= scale;
        v.w *= scale;
        *v4 = v;
    }
    for (int h = threadIdx.x; h < p.v_heads; h += blockDim.x) {
        float *bp = p.beta + tok * p.v_heads + h;
        float *ap = p.alpha + tok * p.v_heads + h;
        *bp = sigmoidf_ref(*bp);
        *ap = p.ssm_a[h] * softplusf_ref(*ap + p.dt_bias[h]);
    }
}

// ----------------------------------------------------------------------------
// L3: chunk-local quantities
// ----------------------------------------------------------------------------
struct LocalParams {
    const float *qkv;            // normalised [nseq][count][qkv_dim]
    const float *beta, *alpha;   // sigmoid(beta), g
    float *w_out, *ut_out;       // [nseq][nchunk][v_heads][64][128]
    float *p_out;                // [nseq][nchunk][v_heads][64][64]
    float *gam_out;              // [nseq][nchunk][v_heads][64]  gamma_r (log space)
    int count, nchunk, qk_heads, v_heads, qkv_dim;
};

constexpr int kPad = kD + 1;  // padded smem rows (bank-conflict-free column walks)

__global__ void __launch_bounds__(256, 2) linear_prefill_local_kernel(LocalParams p) {
    extern __shared__ float sm[];
    float *Ks = sm;                  // [64][129]
    float *Xs = Ks + kC * kPad;      // [64][129]  Q, then V
    float *As = Xs + kC * kPad;      // [64][65]
    float *Ts = As + kC * (kC + 1);  // [64][65]
    __shared__ float gam[kC], bet[kC], egs[kC];

    const int chunk = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x;
    const int kh = h % p.qk_heads;  // ops.rs:699
    const int t0 = chunk * kC;
    const int qk_dim = p.qk_heads * kD;

    // Load K and Q rows of the chunk (zero rows past the prompt's end).
    for (int idx = tid; idx < kC * (kD / 4); idx += 256) {
        const int r = idx / (kD / 4), c4 = idx % (kD / 4);
        float4 k = make_float4(0.f, 0.f, 0.f, 0.f), q = k;
        if (t0 + r < p.count) {
            const float *row = p.qkv + (size_t(s) * p.count + t0 + r) * p.qkv_dim;
            k = reinterpret_cast<const float4 *>(row + qk_dim + kh * kD)[c4];
            q = reinterpret_cast<const float4 *>(row + kh * kD)[c4];
        }
        float *kd = Ks + r * kPad + c4 * 4;
        float *qd = Xs + r * kPad + c4 * 4;
        kd[0] = k.x; kd[1] = k.y; kd[2] = k.z; kd[3] = k.w;
        qd[0] = q.x; qd[1] = q.y; qd[2] = q.z; qd[3] = q.w;
    }
    if (tid < kC) {
        const bool in = t0 + tid < p.count;
        const size_t gi = (size_t(s) * p.count + t0 + tid) * p.v_heads + h;
        bet[tid] = in ? p.beta[gi] : 0.f;
        gam[tid] = in ? p.alpha[gi] : 0.f;
    }
    __syncthreads();
    if (tid < 32) {
        // Inclusive prefix sum of g over the 64 tokens (two per lane).
        float a = gam[2 * tid], b = gam[2 * tid + 1];
        b += a;
        float run = b;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const float n = __shfl_up_sync(0xffffffffu, run, off);
            if (tid >= off) run += n;
        }
        const float prev = run - b;
        gam[2 * tid] = prev + a;
        gam[2 * tid + 1] = run;
    }
    __syncthreads();
    if (tid < kC) egs[tid] = expf(gam[tid]);

    // K K^T -> A (scaled, strictly lower) and Q K^T -> P (decayed, lower).
    // Thread (ty, tx) of a 16x16 grid owns rows 4ty.., columns 4tx...
    {
        const int ty = tid / 16, tx = tid % 16;
        float akk[4][4] = {}, aqk[4][4] = {};
#pragma unroll 4
        for (int i = 0; i < kD; ++i) {
            float kr[4], qr[4], kc[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                kr[a] = Ks[(4 * ty + a) * kPad + i];
                qr[a] = Xs[(4 * ty + a) * kPad + i];
                kc[a] = Ks[(4 * tx + a) * kPad + i];
            }
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    akk[a][b] = fmaf(kr[a], kc[b], akk[a][b]);
                    aqk[a][b] = fmaf(qr[a], kc[b], aqk[a][b]);
                }
        }
        float *pout = p.p_out + ((size_t(s) * p.nchunk + chunk) * p.v_heads + h) * kC * kC;
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int r = 4 * ty + a, c = 4 * tx + b;
                const float dec = expf(gam[r] - gam[c]);
                As[r * (kC + 1) + c] = c < r ? bet[r] * dec * akk[a][b] : 0.f;
                pout[r * kC + c] = c <= r ? dec * aqk[a][b] : 0.f;
            }
    }
    __syncthreads();

    // T = (I + A)^-1 by forward substitution, one row per step:
    // T[r][c] = delta_rc - sum_{c <= m < r} A[r][m] T[m][c]; four threads per column.
    {
        const int c = tid >> 2, part = tid & 3;
        if (part == 0) Ts[0 * (kC + 1) + c] = (c == 0) ? 1.f : 0.f;
        __syncthreads();
        for (int r = 1; r < kC; ++r) {
            float acc = 0.f;
            if (c < r) {
                for (int m = c + part; m < r; m += 4) acc = fmaf(As[r * (kC + 1) + m], Ts[m * (kC + 1) + c], acc);
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (part == 0) Ts[r * (kC + 1) + c] = (c < r) ? -acc : (c == r ? 1.f : 0.f);
            __syncthreads();
        }
    }

    // W = T diag(beta e^gamma) K and Ut = T diag(beta) V. Thread: 8 rows x 4 columns.
    const size_t wbase = ((size_t(s) * p.nchunk + chunk) * p.v_heads + h) * kC * kD;
    const int rb = tid / 32, cg = tid % 32;
    auto tri_times = [&](const float *X, const float *scale_a, const float *scale_b,
                         float *out) {
        float acc[8][4] = {};
#pragma unroll 4
        for (int m = 0; m < kC; ++m) {
            const float f = scale_a[m] * (scale_b ? scale_b[m] : 1.f);
            float x[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) x[b] = X[m * kPad + cg * 4 + b] * f;
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                const float tv = Ts[(rb * 8 + a) * (kC + 1) + m];
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(tv, x[b], acc[a][b]);
            }
        }
#pragma unroll
        for (int a = 0; a < 8; ++a)
            reinterpret_cast<float4 *>(out + (rb * 8 + a) * kD)[cg] =
                make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    };
    tri_times(Ks, bet, egs, p.w_out + wbase);
    __syncthreads();  // Xs (Q) is no longer needed: load V
    for (int idx = tid; idx < kC * (kD / 4); idx += 256) {
        const int r = idx / (kD / 4), c4 = idx % (kD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + r < p.count) {
            const float *row = p.qkv + (size_t(s) * p.count + t0 + r) * p.qkv_dim;
            v = reinterpret_cast<const float4 *>(row + 2 * qk_dim + h * kD)[c4];
        }
        float *vd = Xs + r * kPad + c4 * 4;
        vd[0] = v.x; vd[1] = v.y; vd[2] = v.z; vd[3] = v.w;
    }
    __syncthreads();
    tri_times(Xs, bet, nullptr, p.ut_out + wbase);
    if (tid < kC)
        p.gam_out[((size_t(s) * p.nchunk + chunk) * p.v_heads + h) * kC + tid] = gam[tid];
}

// ----------------------------------------------------------------------------
// L4: sequential state pass over the chunks
// ----------------------------------------------------------------------------
struct StateParams {
    const float *qkv;
    const float *w, *ut, *pm, *gam;  // from L3
    float *delta_state;             // slot base [batch][v_heads][128][128]
    float *o_out;                   // [nseq][count][v_heads*128]
    int seq0, count, nchunk, qk_heads, v_heads, qkv_dim;
};

__global__ void __launch_bounds__(256) linear_prefill_state_kernel(StateParams p) {
    extern __shared__ float sm[];
    float *Ss = sm;                    // [32][129]   state slice (rows j, dims i)
    float *Bs = Ss + kSlice * kPad;    // [64][129]   W, then K
    float *Qs = Bs + kC * kPad;        // [64][129]   Q
    float *Ps = Qs + kC * kPad;        // [64][65]    P
    float *Us = Ps + kC * (kC + 1);    // [64][33]    U slice
    __shared__ float gs[kC];

    const int slice = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x;
    const int kh = h % p.qk_heads;
    const int j0 = slice * kSlice;
    const int qk_dim = p.qk_heads * kD;
    float *S = p.delta_state + ((size_t(p.seq0 + s) * p.v_heads + h) * kD + j0) * kD;
    const float query_scale = 1.0f / sqrtf(float(kD));

    for (int idx = tid; idx < kSlice * kD; idx += 256)
        Ss[(idx / kD) * kPad + idx % kD] = S[idx];

    // Thread tiles: for U and O (64 rows x 32 cols): 2 rows... use rows ru..ru+7, col cu.
    const int ru = (tid / 32) * 8, cu = tid % 32;
    // For the state update (32 rows x 128 dims): row js, dims 4*id..4*id+3 (8 rows per thread).
    const int jsb = (tid / 32) * 4, idb = tid % 32;

    for (int chunk = 0; chunk < p.nchunk; ++chunk) {
        const int t0 = chunk * kC;
        const size_t lb = ((size_t(s) * p.nchunk + chunk) * p.v_heads + h);
        __syncthreads();
        // Stage W, Q, P and e^gamma for this chunk.
        for (int idx = tid; idx < kC * (kD / 4); idx += 256) {
            const int r = idx / (kD / 4), c4 = idx % (kD / 4);
            const float4 w4 = reinterpret_cast<const float4 *>(p.w + lb * kC * kD)[idx];
            float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + r < p.count)
                q4 = reinterpret_cast<const float4 *>(
                    p.qkv + (size_t(s) * p.count + t0 + r) * p.qkv_dim + kh * kD)[c4];
            float *wd = Bs + r * kPad + c4 * 4;
            float *qd = Qs + r * kPad + c4 * 4;
            wd[0] = w4.x; wd[1] = w4.y; wd[2] = w4.z; wd[3] = w4.w;
            qd[0] = q4.x; qd[1] = q4.y; qd[2] = q4.z; qd[3] = q4.w;
        }
        for (int idx = tid; idx < kC * kC; idx += 256)
            Ps[(idx / kC) * (kC + 1) + idx % kC] = p.pm[lb * kC * kC + idx];
        if (tid < kC) gs[tid] = p.gam[lb * kC + tid];
        __syncthreads();

        // U = Ut - W S^T  (rows r: ru..ru+7, column j = cu) and Q S^T for O.
        float u[8], qs[8];
        {
            const float *ut = p.ut + lb * kC * kD;
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                u[a] = ut[(ru + a) * kD + j0 + cu];
                qs[a] = 0.f;
            }
            float wsum[8] = {}, qsum[8] = {};
#pragma unroll 4
            for (int i = 0; i < kD; ++i) {
                const float sv = Ss[cu * kPad + i];
#pragma unroll
                for (int a = 0; a < 8; ++a) {
                    wsum[a] = fmaf(Bs[(ru + a) * kPad + i], sv, wsum[a]);
                    qsum[a] = fmaf(Qs[(ru + a) * kPad + i], sv, qsum[a]);
                }
            }
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                u[a] -= wsum[a];
                qs[a] = qsum[a];
                Us[(ru + a) * (kSlice + 1) + cu] = u[a];
            }
        }
        __syncthreads();
        // O = diag(e^gamma) Q S^T + P U, scaled by 1/sqrt(128).
        {
            float o[8];
#pragma unroll
            for (int a = 0; a < 8; ++a) o[a] = expf(gs[ru + a]) * qs[a];
#pragma unroll 4
            for (int m = 0; m < kC; ++m) {
                const float um = Us[m * (kSlice + 1) + cu];
#pragma unroll
                for (int a = 0; a < 8; ++a) o[a] = fmaf(Ps[(ru + a) * (kC + 1) + m], um, o[a]);
            }
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                const int t = t0 + ru + a;
                if (t < p.count)
                    p.o_out[(size_t(s) * p.count + t) * (size_t(p.v_heads) * kD) + h * kD + j0 + cu] =
                        o[a] * query_scale;
            }
        }
        // Stage K (over W) for the state update.
        __syncthreads();
        for (int idx = tid; idx < kC * (kD / 4); idx += 256) {
            const int r = idx / (kD / 4), c4 = idx % (kD / 4);
            float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + r < p.count)
                k4 = reinterpret_cast<const float4 *>(
                    p.qkv + (size_t(s) * p.count + t0 + r) * p.qkv_dim + qk_dim + kh * kD)[c4];
            float *kd = Bs + r * kPad + c4 * 4;
            kd[0] = k4.x; kd[1] = k4.y; kd[2] = k4.z; kd[3] = k4.w;
        }
        __syncthreads();
        // S' = e^{gamma_C} S + U^T diag(e^{gamma_C - gamma}) K.
        {
            const float gC = gs[kC - 1];
            float acc[4][4];
            const float egC = expf(gC);
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = egC * Ss[(jsb + a) * kPad + idb * 4 + b];
#pragma unroll 2
            for (int m = 0; m < kC; ++m) {
                const float dec = expf(gC - gs[m]);
                float kv[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) kv[b] = Bs[m * kPad + idb * 4 + b] * dec;
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float um = Us[m * (kSlice + 1) + jsb + a];
#pragma unroll
                    for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(um, kv[b], acc[a][b]);
                }
            }
            __syncthreads();
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) Ss[(jsb + a) * kPad + idb * 4 + b] = acc[a][b];
        }
    }
    __syncthreads();
    for (int idx = tid; idx < kSlice * kD; idx += 256) S[idx] = Ss[(idx / kD) * kPad + idx % kD];
}

// ----------------------------------------------------------------------------
// L5: per-head RMSNorm + SiLU(z)
// ----------------------------------------------------------------------------
struct OutParams {
    const float *z;
    const float *ssm_norm;
    float *attention;  // in: O; out: normalised, gated
    int count, v_heads;
    float eps;
};

__global__ void __launch_bounds__(256) linear_prefill_out_kernel(OutParams p) {
    const int t = blockIdx.x, s = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t base = (size_t(s) * p.count + t) * size_t(p.v_heads) * kD;
    for (int h = warp; h < p.v_heads; h += 8) {
        float4 *o4 = reinterpret_cast<float4 *>(p.attention + base + h * kD) + lane;
        const float4 z4 = reinterpret_cast<const float4 *>(p.z + base + h * kD)[lane];
        const float4 w4 = reinterpret_cast<const float4 *>(p.ssm_norm)[lane];
        float4 o = *o4;
        double sum = double(o.x) * o.x + double(o.y) * o.y + double(o.z) * o.z + double(o.w) * o.w;
        sum = warp_sum_f64(sum);
        const float scale = rms_scale_from_sum(sum, kD, p.eps);
        o.x = o.x * scale * w4.x * siluf_ref(z4.x);
        o.y = o.y * scale * w4.y * siluf_ref(z4.y);
        o.z = o.z * scale * w4.z * siluf_ref(z4.z);
        o.w = o.w * scale * w4.w * siluf_ref(z4.w);
        *o4 = o;
    }
}

}  // namespace

size_t linear_prefill_scratch_floats(int nchunk_total, int v_heads) {
    // W and Ut: [chunks][v_heads][64][128] each; P: [chunks][v_heads][64][64]; gamma.
    return size_t(nchunk_total) * v_heads * kC * (2 * kD + kC + 1);
}

cudaError_t launch_linear_prefill(const LinearPrefillLaunch &a, cudaStream_t stream) {
    const int qkv_dim = (2 * a.qk_heads + a.v_heads) * kD;
    const int nchunk = (a.count + kC - 1) / kC;
    // The segment boundaries live at the start of the W scratch, which L3
    // only writes after the conv has finished.
    const int nseg = (a.count + kSeg - 1) / kSeg;
    ConvParams cp{a.qkv, a.conv_state, a.conv_w, a.scratch, a.seq0, a.count, qkv_dim, nseg};
    const dim3 conv_grid((qkv_dim + 127) / 128, nseg, a.nseq);
    linear_prefill_conv_bounds_kernel<<<conv_grid, 128, 0, stream>>>(cp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    linear_prefill_conv_kernel<<<conv_grid, 128, 0, stream>>>(cp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    NormParams np{a.qkv, a.beta, a.alpha, a.dt_bias, a.ssm_a, a.count, a.qk_heads, a.v_heads,
                  qkv_dim, a.eps};
    linear_prefill_norm_kernel<<<dim3(a.count, a.nseq), 256, 0, stream>>>(np);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    const size_t per = size_t(a.nseq) * nchunk * a.v_heads;
    float *w = a.scratch;
    float *ut = w + per * kC * kD;
    float *pm = ut + per * kC * kD;
    float *gm = pm + per * kC * kC;
    LocalParams lp{a.qkv, a.beta, a.alpha, w, ut, pm, gm, a.count, nchunk, a.qk_heads,
                   a.v_heads, qkv_dim};
    const size_t smem_l = size_t(2 * kC * kPad + 2 * kC * (kC + 1)) * sizeof(float);
    if ((e = cudaFuncSetAttribute(linear_prefill_local_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_l))) !=
        cudaSuccess)
        return e;
    linear_prefill_local_kernel<<<dim3(nchunk, a.v_heads, a.nseq), 256, smem_l, stream>>>(lp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    StateParams sp{a.qkv, w, ut, pm, gm, a.delta_state, a.attention, a.seq0, a.count, nchunk,
                   a.qk_heads, a.v_heads, qkv_dim};
    const size_t smem_s = size_t(kSlice * kPad + 2 * kC * kPad + kC * (kC + 1) +
                                 kC * (kSlice + 1)) * sizeof(float);
    if ((e = cudaFuncSetAttribute(linear_prefill_state_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_s))) !=
        cudaSuccess)
        return e;
    linear_prefill_state_kernel<<<dim3(kD / kSlice, a.v_heads, a.nseq), 256, smem_s, stream>>>(sp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    OutParams op{a.z, a.ssm_norm, a.attention, a.count, a.v_heads, a.eps};
    linear_prefill_out_kernel<<<dim3(a.count, a.nseq), 256, 0, stream>>>(op);
    return cudaGetLastError();
}

}  // namespace q38
