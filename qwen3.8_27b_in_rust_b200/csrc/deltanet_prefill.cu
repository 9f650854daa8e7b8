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
//                            and SiLU, in place, then the L2-norm of the q and
//                            k heads (f64 sums; a CTA's 128 channels are one
//                            head); a pre-pass saves the three original inputs
//                            before each segment so segments run in parallel;
//                            the last three inputs become the new conv state.
//   L2 linear_prefill_norm   one CTA per (token, sequence): the beta/alpha
//                            gates, in place.
//   L3 linear_prefill_local  one CTA per (chunk, key head, sequence): K K^T and
//                            Q K^T once, then per value head of that key head
//                            the chunk-local W, Ut, P, K~ and e^gamma (all
//                            chunks in parallel).
//   L4 linear_prefill_state  one CTA per (value head, sequence): walks the
//                            chunks in order with the head's state resident
//                            in TMEM; all products on tcgen05 (kind::f16 with
//                            bf16 hi/lo operand pairs); writes O (scaled by
//                            1/sqrt(128)) and the final state.
//   L5 linear_prefill_out    one CTA per (token, sequence): per-head RMSNorm
//                            with ssm_norm and the SiLU(z) gate (ops.rs:735-740).
//
// L1-L3 and L5 are f32 CUDA-core kernels; L4's split-bf16 products keep the
// chunked result within ~1e-5 of the per-token recurrence.
#include "q38_sm100.cuh"

#include <cudaTypedefs.h>

#include <algorithm>

namespace q38 {
namespace {

constexpr int kC = 64;       // chunk length
constexpr int kD = kLinHeadDim;  // 128


// ----------------------------------------------------------------------------
// L1: conv + SiLU, 64-token segments in parallel
// ----------------------------------------------------------------------------
struct ConvParams {
    float *qkv;          // [nseq][count][qkv_dim]
    float *conv_state;   // slot base [batch][qkv_dim][3]
    const float *conv_w; // [qkv_dim][4]
    float *bounds;       // [nseq][nseg][3][qkv_dim]: inputs preceding each segment
    int seq0, count, qkv_dim, nseg;
    int qk_channels;     // 2 * qk_heads * 128: the q and k channels, L2-normalised per head
    int v_head0;         // the call's first value head: grid block qk_channels/128 + i is
                         // the channel block of value head v_head0 + i
    float eps;
    int *err;
};

// Channel block (128 channels) of grid block bx: every q and k block, then the
// blocks of the call's value heads.
__device__ __forceinline__ int conv_channel_block(const ConvParams &p, int bx) {
    const int qk_blocks = p.qk_channels / 128;
    return bx < qk_blocks ? bx : qk_blocks + p.v_head0 + (bx - qk_blocks);
}

constexpr int kSeg = 64;  // tokens per conv segment

// The three inputs that precede segment g: the carried conv state for g = 0,
// otherwise the (not yet convolved) inputs g*kSeg-3 .. g*kSeg-1.
__global__ void __launch_bounds__(128) linear_prefill_conv_bounds_kernel(ConvParams p) {
    const int c = conv_channel_block(p, blockIdx.x) * 128 + threadIdx.x;
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

// One CTA per (128 channels, 64-token segment, sequence); the segment's
// [64 tokens][128 channels] f32 tile comes in by one TMA load and goes back by
// one TMA store (rows past the prompt's end read as zeros and are not
// written). Thread = channel: the kernel-4 causal conv (multiply then add,
// ops.rs:665-676) and SiLU, in place in shared memory; the last segment
// leaves the last three inputs as the new conv state. The first qk_channels
// channels are the q and k heads (a CTA's 128 channels are one head): those
// rows are then L2-normalised per token (l2norm, ops.rs:562-571: f64 sum of
// squares, 1 / max(sqrt, eps)), a warp per token, so L2 only handles the
// gates.
constexpr uint32_t kConvTileBytes = kSeg * 128 * 4;  // 32 KB

__global__ void __launch_bounds__(128) linear_prefill_conv_kernel(const __grid_constant__ CUtensorMap map_x,
                                                                   ConvParams p) {
    using namespace sm100;
    extern __shared__ __align__(128) float tile[];  // [kSeg][128]
    __shared__ __align__(8) uint64_t bar;
    const int cb = conv_channel_block(p, blockIdx.x), g = blockIdx.y, s = blockIdx.z;
    const int c = cb * 128 + threadIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool live = c < p.qkv_dim;
    const int t0 = g * kSeg, n = min(p.count - t0, kSeg);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, kConvTileBytes);
        tma_load_3d(tile, &map_x, cb * 128, t0, s, &bar);
    }
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
    float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) {
        const float *bnd = p.bounds + (size_t(s) * p.nseg + g) * 3 * p.qkv_dim + c;
        s0 = bnd[0];
        s1 = bnd[p.qkv_dim];
        s2 = bnd[2 * size_t(p.qkv_dim)];
        w = reinterpret_cast<const float4 *>(p.conv_w)[c];
    }
    __syncthreads();  // barrier initialised before anyone waits on it
    if (!__syncthreads_and(mbar_wait(&bar, 0))) {
        if (threadIdx.x == 0) set_error(p.err, kDevErrTimeout);
        return;  // (uniform) a TMA that never completed: nothing of this tile is written
    }
    float *col = tile + threadIdx.x;
#pragma unroll 8
    for (int t = 0; t < n; ++t) {
        const float xt = col[t * 128];
        float v = s0 * w.x;
        v += s1 * w.y;
        v += s2 * w.z;
        v += xt * w.w;
        s0 = s1;
        s1 = s2;
        s2 = xt;
        // SiLU with the hardware exp2 and a fast divide (a few ulp from
        // x / (1 + exp(-x)); the prefill path's tolerance is 1e-3).
        col[t * 128] = __fdividef(v, 1.0f + __expf(-v));
    }
    if (live && g == p.nseg - 1) {
        float *st = p.conv_state + (size_t(p.seq0 + s) * p.qkv_dim + c) * 3;
        st[0] = s0;
        st[1] = s1;
        st[2] = s2;
    }
    if (cb * 128 < p.qk_channels) {
        __syncthreads();
        for (int t = warp; t < n; t += 4) {
            float4 *v4 = reinterpret_cast<float4 *>(tile + t * 128) + lane;
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
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
        tma_store_3d(&map_x, cb * 128, t0, s, tile);
        bulk_commit_group();
        bulk_wait_group_read0();
    }
}

// ----------------------------------------------------------------------------
// L2: gates
// ----------------------------------------------------------------------------
struct NormParams {
    float *qkv;
    float *beta, *alpha;  // [nseq][count][v_heads]
    const float *dt_bias, *ssm_a;
    int count, qk_heads, v_heads, qkv_dim, v_head0, v_head_count;
    float eps;
};

__global__ void __launch_bounds__(256) linear_prefill_norm_kernel(NormParams p) {
    const int t = blockIdx.x, s = blockIdx.y;
    const size_t tok = size_t(s) * p.count + t;
    for (int h = p.v_head0 + threadIdx.x; h < p.v_head0 + p.v_head_count; h += blockDim.x) {
        float *bp = p.beta + tok * p.v_heads + h;
        float *ap = p.alpha + tok * p.v_heads + h;
        *bp = sigmoidf_ref(*bp);
        *ap = p.ssm_a[h] * softplusf_ref(*ap + p.dt_bias[h]);
    }
}

// ----------------------------------------------------------------------------
// L3: chunk-local quantities
// ----------------------------------------------------------------------------
// Operands of the state pass are stored as bf16 (hi, lo) pairs: plane
// [2][rows][cols] with hi = bf16(x) and lo = bf16(x - hi), per (sequence,
// chunk, value head) = "plane".
struct LocalParams {
    const float *qkv;            // normalised [nseq][count][qkv_dim]
    const float *beta, *alpha;   // sigmoid(beta), g
    __nv_bfloat16 *w2;           // [planes][2][64 r][128 i]   W
    __nv_bfloat16 *q2;           // [planes][2][64 r][128 i]   Q~ = diag(e^gamma) Q
    __nv_bfloat16 *p2;           // [planes][2][64 r][64 s]    P
    __nv_bfloat16 *k2;           // [planes][2][64 r][128 i]   K~ = diag(e^{gamma_C-gamma}) K
    float *ut_out;               // [planes][64][128]          Ut (f32)
    float *eg_out;               // [planes][64]               e^{gamma_r}
    int *err;
    int count, nchunk, qk_heads, v_heads, qkv_dim, v_head0, v_head_count;
};

// (a, b) -> bf16x2 pairs hi = bf16(a, b), lo = bf16(a - hi.a, b - hi.b): hi + lo
// keeps ~16 bits of each value's mantissa.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t &hi, uint32_t &lo) {
    hi = pack_bf16x2_rn(a, b);
    const float2 hf = bf16x2_to_float2(hi);
    lo = pack_bf16x2_rn(a - hf.x, b - hf.y);
}

constexpr int kPadA = kC + 1;  // padded f32 rows of A and T (conflict-free column walks)

// Shared-memory plan of L3 (bytes). Region R is reused phase by phase:
//   G phase:       [K; Q] hi | [K; Q] lo, each two SW128 boxes of 128 rows x 64 dims
//   A/P phase:     A f32 [64][65] | decay factors [64][65] | ... | P staging (hi | lo) at 40 KB
//   inverse phase: A f32 [64][65] | T f32 [64][65] | ... | block products [32][65] at 40 KB
//   MMA phase:     B_W hi | B_W lo | B_U hi | B_U lo, each two SW128 boxes of 64 rows x 64 cols
//   epilogue:      W hi | W lo | Ut staging for coalesced stores
// Staging tiles hold 16-byte chunk c of row r at chunk c ^ (r % chunks per
// row), so that one-row-per-thread writes and one-chunk-per-lane reads are
// both free of bank conflicts.
// then Tu = T diag(beta) hi | lo (SW128, 64 rows x 64 columns; an M=128 MMA
// also reads 64 further rows, so 8 KB of padding follow), then the barriers.
constexpr uint32_t kLocR = 64 * 1024;
constexpr uint32_t kLocKQBox = 128 * 128;          // 128 rows x 128 B
constexpr uint32_t kLocBBox = 64 * 128;            // 64 rows x 128 B
constexpr uint32_t kLocTs = kC * kPadA * 4;        // offset of T within R
constexpr uint32_t kLocXs = 40 * 1024;             // the inverse's block products (P staging, stored by then)
constexpr uint32_t kLocPst = 40 * 1024;            // P (hi | lo) staging during the A/P phase
constexpr uint32_t kLocTu = kLocR;                 // Tu hi at +0, lo at +8 KB, padding +16 KB
constexpr uint32_t kLocSmem = kLocR + 3 * 8192 + 1024;
static_assert(2 * kC * kPadA * 4 <= kLocXs && kLocXs + 32 * kPadA * 4 <= kLocR &&
                  kLocPst + 2 * kC * kC * 2 <= kLocR,
              "inverse workspace and P staging fit R");
constexpr uint32_t kLocTmemCols = 256;  // G (64) while it is read out, then W (128) | Ut (128)

// e^x for the in-chunk decay factors e^{gamma_r - gamma_s} (x <= 0): the
// hardware exp2 of x log2(e). Relative error ~1e-6 for |x| < 20 (smaller
// factors vanish against the others), below the ~1e-5 of the bf16-pair
// products these factors feed.
__device__ __forceinline__ float decay_exp(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
    return y;
}

// Byte offset of 16-byte chunk c of row r in a staging tile of `chunks`
// chunks per row (a power of two).
__device__ __forceinline__ uint32_t stage_at(uint32_t r, uint32_t c, uint32_t chunks) {
    return (r * chunks + (c ^ (r & (chunks - 1)))) * 16u;
}

// Element (row, col) of a SW128 tile of 64-column (128-byte) rows.
__device__ __forceinline__ uint32_t sw128_bf16_at(uint32_t row, uint32_t col) {
    return row * 128u + ((((col & 63u) >> 3) ^ (row & 7u)) << 4) + (col & 7u) * 2u;
}

// One CTA per (chunk, key head, sequence); 8 warps, two CTAs per SM. The
// value heads h with h % qk_heads == kh (ops.rs:699) share the chunk's K and
// Q, so G = [K; Q] K^T (K K^T in TMEM lanes 0-63, Q K^T in lanes 64-127) is
// one M=128, N=64, K=128 tcgen05 product, read out once into registers
// (thread = row, 32 columns). Per value head: A and P from G on the CUDA
// cores, the blocked inverse T = (I + A)^-1 in f32, then W = Tu (e^gamma K)
// and Ut = Tu V with Tu = T diag(beta) as two M=128 (64 real rows), N=128,
// K=64 products. Every product is hi.hi + lo.hi + hi.lo of bf16 pairs
// (kind::f16, f32 accumulation), the same ~16-bit operands as the state pass.
__global__ void __launch_bounds__(256, 2) linear_prefill_local_kernel(LocalParams p) {
    using namespace sm100;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *R = smem;
    unsigned char *tu_hi = smem + kLocTu, *tu_lo = tu_hi + 8192;
    float *As = reinterpret_cast<float *>(R);
    float *Ts = reinterpret_cast<float *>(R + kLocTs);
    float *Xs = reinterpret_cast<float *>(R + kLocXs);
    __shared__ float gam[kC], bet[kC], egs[kC], dec[kC];
    __shared__ __align__(8) uint64_t g_done, mma_done;
    __shared__ uint32_t tmem_base_s;

    const int chunk = blockIdx.x, kh = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = chunk * kC;
    // The call's value heads that read key head kh; none: nothing to do.
    auto in_call = [&](int h) { return h >= p.v_head0 && h < p.v_head0 + p.v_head_count; };
    {
        bool any = false;
        for (int h = kh; h < p.v_heads; h += p.qk_heads) any = any || in_call(h);
        if (!any) return;
    }
    const int qk_dim = p.qk_heads * kD;
    const float *rows = p.qkv + (size_t(s) * p.count + t0) * p.qkv_dim;  // the chunk's first row
    auto row_ok = [&](int r) { return t0 + r < p.count; };

    if (tid == 0) {
        mbar_init(&g_done, 1);
        mbar_init(&mma_done, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base_s, kLocTmemCols);
        tmem_relinquish();
    }
    // [K; Q] as bf16 (hi, lo) in SW128 K-major boxes; rows past the prompt's
    // end are zero. Thread: row = tid / 2, 64 dims.
    {
        const int row = tid >> 1, half = tid & 1;  // row < 128: 0-63 K, 64-127 Q
        const int r = row & 63;
        const float *src = rows + size_t(r) * p.qkv_dim + (row < kC ? qk_dim : 0) + kh * kD + half * 64;
        unsigned char *hi = R + half * kLocKQBox, *lo = R + 2 * kLocKQBox + half * kLocKQBox;
        float4 v[16];  // all loads in flight before any shared-memory store
#pragma unroll
        for (int i = 0; i < 16; ++i)
            v[i] = row_ok(r) ? __ldg(reinterpret_cast<const float4 *>(src) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
            const float4 a = v[2 * c8], b = v[2 * c8 + 1];
            uint4 h, l;
            split_bf16x2(a.x, a.y, h.x, l.x);
            split_bf16x2(a.z, a.w, h.y, l.y);
            split_bf16x2(b.x, b.y, h.z, l.z);
            split_bf16x2(b.z, b.w, h.w, l.w);
            const uint32_t off = sw128_bf16_at(uint32_t(row), uint32_t(8 * c8));
            *reinterpret_cast<uint4 *>(hi + off) = h;
            *reinterpret_cast<uint4 *>(lo + off) = l;
        }
        // Tu's padding rows (read by the M=128 MMAs, results unused): zeros.
        for (int i = tid; i < 8192 / 16; i += 256)
            reinterpret_cast<uint4 *>(tu_hi + 2 * 8192)[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_base_s;
    bool ok = true;

    if (tid == 0) {
        const uint32_t idesc = idesc_bf16_f32(128, kC, 0, 0);
        const uint32_t kq_hi = smem_addr(R), kq_lo = kq_hi + 2 * kLocKQBox;
#pragma unroll 1
        for (int prod = 0; prod < 3; ++prod) {  // hi.hi, lo.hi, hi.lo
            const uint32_t a_base = prod == 1 ? kq_lo : kq_hi;
            const uint32_t b_base = prod == 2 ? kq_lo : kq_hi;
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
                const uint32_t off = (kk >> 2) * kLocKQBox + (kk & 3) * 32;
                mma_bf16(tmem, smem_desc_sw128(a_base + off, 16, 1024),
                         smem_desc_sw128(b_base + off, 16, 1024), idesc, (prod | kk) ? 1u : 0u);
            }
        }
        mma_commit(&g_done);
    }
    // G -> registers: warps 0, 1, 4, 5 hold K K^T rows, warps 2, 3, 6, 7 Q K^T
    // rows (TMEM lane quarter = warp % 4); warps 0-3 columns 0-31, 4-7 32-63.
    const bool is_kk = (warp & 3) < 2;
    const int gr = 32 * (warp & 1) + lane;  // row of K K^T or Q K^T
    const int gc0 = warp < 4 ? 0 : 32;
    float gv[32];
    {
        ok = __all_sync(0xffffffffu, mbar_wait(&g_done, 0));
        fence_after_sync();
        uint32_t raw[32];
        tmem_ld32(tmem + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(gc0), raw);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) gv[i] = __uint_as_float(raw[i]);
    }
    if (!ok && lane == 0) set_error(p.err, kDevErrTimeout);

    const uint32_t idesc_x = idesc_bf16_f32(128, kD, 0, 1);
    const uint32_t d_w = tmem, d_u = tmem + kD;  // W columns 0-127, Ut columns 128-255
    // The call's value heads of key head kh, in order; each head's gates
    // (beta, g of the chunk's tokens) are loaded one head ahead.
    auto next_head = [&](int h) {
        for (h += p.qk_heads; h < p.v_heads; h += p.qk_heads)
            if (in_call(h)) return h;
        return -1;
    };
    auto load_gates = [&](int h, float &bv, float &gv_) {
        bv = gv_ = 0.f;
        if (h >= 0 && tid < kC && row_ok(tid)) {
            const size_t gi = (size_t(s) * p.count + t0 + tid) * p.v_heads + h;
            bv = p.beta[gi];
            gv_ = p.alpha[gi];
        }
    };
    int h = in_call(kh) ? kh : next_head(kh);
    float nb, ng;  // the gates of head h
    load_gates(h, nb, ng);
    int head_i = -1;  // value heads of this CTA processed so far, minus one
    for (; h >= 0; h = next_head(h)) {
        ++head_i;
        const size_t plane = (size_t(s) * p.nchunk + chunk) * p.v_heads + h;
        fence_before_sync();
        __syncthreads();  // previous head done with R, gam/bet and TMEM
        fence_after_sync();
        if (tid < kC) {
            bet[tid] = nb;
            gam[tid] = ng;
        }
        load_gates(next_head(h), nb, ng);
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
        if (tid < kC) {
            egs[tid] = expf(gam[tid]);
            dec[tid] = expf(gam[kC - 1] - gam[tid]);
        }
        // A = beta_r e^{gamma_r - gamma_s} K K^T (strictly lower) into smem;
        // P = e^{gamma_r - gamma_s} Q K^T (lower) as bf16 pairs to global.
        // Every warp forms the decay factors of its own (rows, columns) block.
        {
            const int r = gr;
            const float gr_ = gam[r];
            if (is_kk) {
                const float br = bet[r];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int c = gc0 + i;
                    const float d = (c <= r) ? decay_exp(gr_ - gam[c]) : 0.f;
                    As[r * kPadA + c] = c < r ? br * d * gv[i] : 0.f;
                }
            } else {
                unsigned char *pst = R + kLocPst;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float pv[8];
#pragma unroll
                    for (int b = 0; b < 8; ++b) {
                        const int c = gc0 + 8 * q + b;
                        pv[b] = c <= r ? decay_exp(gr_ - gam[c]) * gv[8 * q + b] : 0.f;
                    }
                    uint4 hq, lq;
                    split_bf16x2(pv[0], pv[1], hq.x, lq.x);
                    split_bf16x2(pv[2], pv[3], hq.y, lq.y);
                    split_bf16x2(pv[4], pv[5], hq.z, lq.z);
                    split_bf16x2(pv[6], pv[7], hq.w, lq.w);
                    const uint32_t off = stage_at(uint32_t(r), uint32_t(gc0 / 8 + q), 8);
                    *reinterpret_cast<uint4 *>(pst + off) = hq;
                    *reinterpret_cast<uint4 *>(pst + kC * kC * 2 + off) = lq;
                }
            }
        }
        __syncthreads();
        {
            // P (hi | lo) to global, one 16-byte chunk per lane.
            const unsigned char *pst = R + kLocPst;
            uint4 *dst = reinterpret_cast<uint4 *>(p.p2 + plane * 2 * kC * kC);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int idx = tid + 256 * k, pl = idx >> 9, r = (idx >> 3) & 63, c = idx & 7;
                dst[idx] = *reinterpret_cast<const uint4 *>(pst + pl * kC * kC * 2 + stage_at(r, c, 8));
            }
        }

        // T = (I + A)^-1 (A strictly lower) by block doubling: for a lower
        // block matrix L = [L11 0; L21 L22], L^-1 = [T11 0; -T22 L21 T11 T22],
        // and the off-diagonal block of L = I + A is A's. The four 16x16
        // diagonal blocks by forward substitution, one warp each; then the two
        // 16x16 pairs (T10 = -T11 A10 T00, T32 = -T33 A32 T22); then the
        // 32x32 halves (T[32:64][0:32] = -T_BB A_BA T_AA). The products run
        // on 2x2 register tiles (four shared-memory loads per four FMAs).
        for (int idx = tid; idx < kC * kPadA; idx += 256) Ts[idx] = 0.f;
        __syncthreads();
        if (warp < 4 && lane < 16) {
            // Column c of (I + A_ii)^-1 by right-looking forward substitution:
            // once t[m] is final it updates every later row, so the dependent
            // chain is 16 steps long instead of 120.
            const int b0 = warp * 16, c = lane;
            float t[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) t[r] = (r == c) ? 1.f : 0.f;
#pragma unroll
            for (int m = 0; m < 15; ++m) {
#pragma unroll
                for (int r = m + 1; r < 16; ++r) t[r] = fmaf(-As[(b0 + r) * kPadA + b0 + m], t[m], t[r]);
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) Ts[(b0 + r) * kPadA + b0 + c] = t[r];
        }
        __syncthreads();
        // X [n x n] (row stride kPadA, in Xs) = L (rows lr0, cols lc0) x R
        // (rows rr0, cols rc0), k over [k0, k1); thread tiles (2 rows, 2 cols).
        // sign: +1 or -1 applied to the result.
        auto prod2x2 = [&](const float *L, int lr0, int lc0, const float *R, int rr0, int rc0, float *X,
                           int xr0, int xc0, int ti, int tj, int kbeg, int kend, float sign) {
            const int r = 2 * ti, c = 2 * tj;
            float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
            for (int k = kbeg; k < kend; ++k) {
                const float l0 = L[(lr0 + r) * kPadA + lc0 + k], l1 = L[(lr0 + r + 1) * kPadA + lc0 + k];
                const float r0 = R[(rr0 + k) * kPadA + rc0 + c], r1 = R[(rr0 + k) * kPadA + rc0 + c + 1];
                a00 = fmaf(l0, r0, a00);
                a01 = fmaf(l0, r1, a01);
                a10 = fmaf(l1, r0, a10);
                a11 = fmaf(l1, r1, a11);
            }
            X[(xr0 + r) * kPadA + xc0 + c] = sign * a00;
            X[(xr0 + r) * kPadA + xc0 + c + 1] = sign * a01;
            X[(xr0 + r + 1) * kPadA + xc0 + c] = sign * a10;
            X[(xr0 + r + 1) * kPadA + xc0 + c + 1] = sign * a11;
        };
        {
            // Level 1: X0 = A10 T00 and X1 = A32 T22 (64 tiles of 2x2 each,
            // threads 0-127), into Xs rows 0-15 / 16-31, columns 0-15.
            // T00 is lower triangular: row k of T00 is zero left of k, so
            // column c needs k >= c only -- the full range is kept (zeros).
            if (tid < 128) {
                const int pr = tid >> 6, e = tid & 63, ti = e >> 3, tj = e & 7;
                const int bi = 16 + 32 * pr, bj = 32 * pr;  // A block (i, j), T block (j, j)
                prod2x2(As, bi, bj, Ts, bj, bj, Xs, 16 * pr, 0, ti, tj, 0, 16, 1.f);
            }
            __syncthreads();
            // T10 = -T11 X0, T32 = -T33 X1 (T11 lower triangular: k <= row).
            if (tid < 128) {
                const int pr = tid >> 6, e = tid & 63, ti = e >> 3, tj = e & 7;
                const int bi = 16 + 32 * pr;
                prod2x2(Ts, bi, bi, Xs, 16 * pr, 0, Ts, bi, 32 * pr, ti, tj, 0, 2 * ti + 2, -1.f);
            }
            __syncthreads();
            // Level 2: X = A[32:64][0:32] T[0:32][0:32] (256 tiles of 2x2).
            {
                const int ti = tid >> 4, tj = tid & 15;
                prod2x2(As, 32, 0, Ts, 0, 0, Xs, 0, 0, ti, tj, 0, 32, 1.f);
            }
            __syncthreads();
            // T[32:64][0:32] = -T[32:64][32:64] X (lower triangular: k <= row).
            {
                const int ti = tid >> 4, tj = tid & 15;
                prod2x2(Ts, 32, 32, Xs, 0, 0, Ts, 32, 0, ti, tj, 0, 2 * ti + 2, -1.f);
            }
            __syncthreads();
        }
        // Tu = T diag(beta) as bf16 pairs (K-major A operand): thread = (row
        // tid / 4, 16 columns).
        {
            const int r = tid >> 2, m0 = 16 * (tid & 3);
#pragma unroll
            for (int c8 = 0; c8 < 2; ++c8) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = Ts[r * kPadA + m0 + 8 * c8 + e] * bet[m0 + 8 * c8 + e];
                uint4 hq, lq;
                split_bf16x2(v[0], v[1], hq.x, lq.x);
                split_bf16x2(v[2], v[3], hq.y, lq.y);
                split_bf16x2(v[4], v[5], hq.z, lq.z);
                split_bf16x2(v[6], v[7], hq.w, lq.w);
                const uint32_t off = sw128_bf16_at(uint32_t(r), uint32_t(m0 + 8 * c8));
                *reinterpret_cast<uint4 *>(tu_hi + off) = hq;
                *reinterpret_cast<uint4 *>(tu_lo + off) = lq;
            }
        }
        __syncthreads();  // T and A are consumed: R takes the B operands
        // B_W = diag(e^gamma) K and B_U = V (MN-major: rows m, 128 columns in
        // two SW128 boxes), and K~ = diag(e^{gamma_C - gamma}) K (bf16 pairs,
        // row-major, the state update's MN-major B operand) from the same K
        // registers. Thread: 8 columns (chunk tid % 16) of rows tid / 16 + 16 k.
        {
            const int c = tid & 15;
            unsigned char *bw_hi = R, *bw_lo = R + 2 * kLocBBox, *bu_hi = R + 4 * kLocBBox,
                          *bu_lo = R + 6 * kLocBBox;
            const uint32_t box = (c >> 3) * kLocBBox;
            __nv_bfloat16 *kth = p.k2 + plane * 2 * kC * kD + 8 * c, *ktl = kth + kC * kD;
            float4 x[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int m = (tid >> 4) + 16 * k;
                const float *krow = rows + size_t(m) * p.qkv_dim + qk_dim + kh * kD + 8 * c;
                x[2 * k] = row_ok(m) ? __ldg(reinterpret_cast<const float4 *>(krow)) : make_float4(0.f, 0.f, 0.f, 0.f);
                x[2 * k + 1] = row_ok(m) ? __ldg(reinterpret_cast<const float4 *>(krow) + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int m = (tid >> 4) + 16 * k;
                const float e = egs[m], dk = dec[m];
                const float4 ka = x[2 * k], kb = x[2 * k + 1];
                const uint32_t off = box + sw128_bf16_at(uint32_t(m), uint32_t(8 * c));
                uint4 hq, lq;
                split_bf16x2(ka.x * e, ka.y * e, hq.x, lq.x);
                split_bf16x2(ka.z * e, ka.w * e, hq.y, lq.y);
                split_bf16x2(kb.x * e, kb.y * e, hq.z, lq.z);
                split_bf16x2(kb.z * e, kb.w * e, hq.w, lq.w);
                *reinterpret_cast<uint4 *>(bw_hi + off) = hq;
                *reinterpret_cast<uint4 *>(bw_lo + off) = lq;
                split_bf16x2(dk * ka.x, dk * ka.y, hq.x, lq.x);
                split_bf16x2(dk * ka.z, dk * ka.w, hq.y, lq.y);
                split_bf16x2(dk * kb.x, dk * kb.y, hq.z, lq.z);
                split_bf16x2(dk * kb.z, dk * kb.w, hq.w, lq.w);
                *reinterpret_cast<uint4 *>(kth + m * kD) = hq;
                *reinterpret_cast<uint4 *>(ktl + m * kD) = lq;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int m = (tid >> 4) + 16 * k;
                const float *vrow = rows + size_t(m) * p.qkv_dim + 2 * qk_dim + h * kD + 8 * c;
                x[2 * k] = row_ok(m) ? __ldg(reinterpret_cast<const float4 *>(vrow)) : make_float4(0.f, 0.f, 0.f, 0.f);
                x[2 * k + 1] = row_ok(m) ? __ldg(reinterpret_cast<const float4 *>(vrow) + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int m = (tid >> 4) + 16 * k;
                const float4 va = x[2 * k], vb = x[2 * k + 1];
                const uint32_t off = box + sw128_bf16_at(uint32_t(m), uint32_t(8 * c));
                uint4 hq, lq;
                split_bf16x2(va.x, va.y, hq.x, lq.x);
                split_bf16x2(va.z, va.w, hq.y, lq.y);
                split_bf16x2(vb.x, vb.y, hq.z, lq.z);
                split_bf16x2(vb.z, vb.w, hq.w, lq.w);
                *reinterpret_cast<uint4 *>(bu_hi + off) = hq;
                *reinterpret_cast<uint4 *>(bu_lo + off) = lq;
            }
        }
        fence_proxy_async_smem();
        fence_before_sync();
        __syncthreads();
        if (tid == 0) {
            fence_after_sync();
            const uint32_t a_hi = smem_addr(tu_hi), a_lo = smem_addr(tu_lo);
            const uint32_t bw_hi = smem_addr(R), bw_lo = bw_hi + 2 * kLocBBox;
            const uint32_t bu_hi = bw_hi + 4 * kLocBBox, bu_lo = bw_hi + 6 * kLocBBox;
#pragma unroll 1
            for (int prod = 0; prod < 3; ++prod) {
                const uint32_t a = prod == 1 ? a_lo : a_hi;
#pragma unroll
                for (int kk = 0; kk < kC / 16; ++kk) {
                    const uint64_t ad = smem_desc_sw128(a + kk * 32, 16, 1024);
                    const uint32_t acc = (prod | kk) ? 1u : 0u;
                    mma_bf16(d_w, ad, smem_desc_sw128((prod == 2 ? bw_lo : bw_hi) + kk * 2048, kLocBBox, 1024),
                             idesc_x, acc);
                    mma_bf16(d_u, ad, smem_desc_sw128((prod == 2 ? bu_lo : bu_hi) + kk * 2048, kLocBBox, 1024),
                             idesc_x, acc);
                }
            }
            mma_commit(&mma_done);
        }
        if (!is_kk) {
            // Warps 2, 3, 6, 7 (128 threads), while the MMAs run: Q~ =
            // diag(e^gamma) Q from the normalised rows. Thread: 8 columns
            // (chunk t % 16) of rows t / 16 + 8 k, one 16-byte chunk per lane
            // in each store.
            const int t = 32 * ((warp & 1) + 2 * (warp >> 2)) + lane;  // 0..127
            const int c = t & 15;
            __nv_bfloat16 *qh = p.q2 + plane * 2 * kC * kD + 8 * c, *ql = qh + kC * kD;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float4 x[8];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int r = (t >> 4) + 8 * (4 * half + k);
                    const float4 *q4 = reinterpret_cast<const float4 *>(rows + size_t(r) * p.qkv_dim + kh * kD + 8 * c);
                    x[2 * k] = row_ok(r) ? __ldg(q4) : make_float4(0.f, 0.f, 0.f, 0.f);
                    x[2 * k + 1] = row_ok(r) ? __ldg(q4 + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int r = (t >> 4) + 8 * (4 * half + k);
                    const float e = egs[r];
                    const float4 a = x[2 * k], b = x[2 * k + 1];
                    uint4 hq, lq;
                    split_bf16x2(a.x * e, a.y * e, hq.x, lq.x);
                    split_bf16x2(a.z * e, a.w * e, hq.y, lq.y);
                    split_bf16x2(b.x * e, b.y * e, hq.z, lq.z);
                    split_bf16x2(b.z * e, b.w * e, hq.w, lq.w);
                    *reinterpret_cast<uint4 *>(qh + r * kD) = hq;
                    *reinterpret_cast<uint4 *>(ql + r * kD) = lq;
                }
            }
            if (t < kC) p.eg_out[plane * kC + t] = egs[t];
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&mma_done, uint32_t(head_i & 1)))) {
            if (lane == 0) set_error(p.err, kDevErrTimeout);
        }
        fence_after_sync();
        if (is_kk) {
            // W (bf16 pairs) and Ut (f32) rows 0-63 from TMEM lanes 0-63
            // (warps 0, 1 columns 0-63, warps 4, 5 columns 64-127), staged in R
            // (free once the MMAs have completed) and stored one 16-byte chunk
            // per lane by these four warps.
            const int r = gr, cbase = warp < 4 ? 0 : 64;
            const uint32_t lane_addr = uint32_t(32 * (warp & 3)) << 16;
            unsigned char *wst = R, *ust = R + 2 * kC * kD * 2;  // W hi | W lo | Ut
#pragma unroll 1
            for (int c32 = 0; c32 < 2; ++c32) {
                const int c = cbase + 32 * c32;
                uint32_t w[32], u[32];
                tmem_ld32(d_w + lane_addr + uint32_t(c), w);
                tmem_ld32(d_u + lane_addr + uint32_t(c), u);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint4 hq, lq;
                    split_bf16x2(__uint_as_float(w[8 * q + 0]), __uint_as_float(w[8 * q + 1]), hq.x, lq.x);
                    split_bf16x2(__uint_as_float(w[8 * q + 2]), __uint_as_float(w[8 * q + 3]), hq.y, lq.y);
                    split_bf16x2(__uint_as_float(w[8 * q + 4]), __uint_as_float(w[8 * q + 5]), hq.z, lq.z);
                    split_bf16x2(__uint_as_float(w[8 * q + 6]), __uint_as_float(w[8 * q + 7]), hq.w, lq.w);
                    const uint32_t off = stage_at(uint32_t(r), uint32_t(c / 8 + q), 16);
                    *reinterpret_cast<uint4 *>(wst + off) = hq;
                    *reinterpret_cast<uint4 *>(wst + kC * kD * 2 + off) = lq;
                }
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    *reinterpret_cast<uint4 *>(ust + stage_at(uint32_t(r), uint32_t(c / 4 + q), 32)) =
                        make_uint4(u[4 * q], u[4 * q + 1], u[4 * q + 2], u[4 * q + 3]);
            }
            named_barrier_sync(1, 128);  // the four K K^T warps
            const int t = 32 * ((warp & 1) + 2 * (warp >> 2)) + lane;  // 0..127
            uint4 *wdst = reinterpret_cast<uint4 *>(p.w2 + plane * 2 * kC * kD);
#pragma unroll 4
            for (int k = 0; k < 16; ++k) {  // W hi | lo: 2 x 64 rows x 16 chunks
                const int idx = t + 128 * k, pl = idx >> 10, rr = (idx >> 4) & 63, cc = idx & 15;
                wdst[idx] = *reinterpret_cast<const uint4 *>(wst + pl * kC * kD * 2 + stage_at(rr, cc, 16));
            }
            uint4 *udst = reinterpret_cast<uint4 *>(p.ut_out + plane * kC * kD);
#pragma unroll 4
            for (int k = 0; k < 16; ++k) {  // Ut: 64 rows x 32 chunks
                const int idx = t + 128 * k, rr = idx >> 5, cc = idx & 31;
                udst[idx] = *reinterpret_cast<const uint4 *>(ust + stage_at(rr, cc, 32));
            }
        }
        tmem_wait_ld();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 0) tmem_dealloc(tmem, kLocTmemCols);
}

// ----------------------------------------------------------------------------
// L4: sequential state pass over the chunks, on tcgen05 (bf16 hi/lo split)
// ----------------------------------------------------------------------------
// One CTA per (value head, sequence). The head's state S [128 j][128 i] lives
// in TMEM (lane j) for the whole prompt; per chunk, with U^T [j][r] = U[r][j]:
//   D_U | D_O = S [W ; Q~]^T      (M=128, N=128, K=128; A = S from TMEM)
//   U^T       = Ut^T - D_U         (epilogue warps)
//   D_PU      = U^T P^T            (M=128, N=64,  K=64;  A = U^T from TMEM)
//   S         = e^{gamma_C} S + U^T K~   (M=128, N=128, K=64, into the f32 state)
//   O[r][j]   = (D_O[j][r] + D_PU[j][r]) / sqrt(128),   Q~ = diag(e^gamma) Q
// Every operand X is a bf16 pair hi = bf16(X), lo = bf16(X - hi), and each
// product is hi.hi + lo.hi + hi.lo (three kind::f16 MMAs, f32 accumulation):
// ~16 bits of each operand, so the chunked result stays within ~1e-5 of the
// per-token recurrence, at K = 16 per instruction. The f32 state is the MMA
// accumulator; after each update the epilogue writes its (hi, lo) copy for
// the next chunk's products and pre-multiplies it by the next chunk's decay.
constexpr int kThreadsLS = 352;  // w0 TMA, w1 MMA (S products), w2-5 + w7-10 epilogue, w6 MMA (P U^T)
constexpr uint32_t kB1Half = 128 * 128 * 2;   // [W ; Q~] hi or lo: 2 column blocks of 128 rows x 128 B
constexpr uint32_t kPmHalf = 64 * 64 * 2;     // P hi or lo: 64 rows x 128 B
constexpr uint32_t kKtHalf = 64 * 128 * 2;    // K~ hi or lo: 2 column blocks of 64 rows x 128 B
constexpr uint32_t kStageLS = 2 * (kB1Half + kPmHalf + kKtHalf);  // 112 KB
constexpr uint32_t kSmemLS = 2 * kStageLS + 1024;
// TMEM columns: f32 state | S hi | S lo (bf16 pairs) | D_U | D_O | U^T hi | U^T lo | D_PU.
constexpr uint32_t kColS = 0, kColSh = 128, kColSl = 192, kColU = 256, kColOq = 320,
                   kColUh = 384, kColUl = 416, kColPU = 448, kTmemColsLS = 512;

struct StateTcParams {
    const float *ut;      // [planes][64][128]
    const float *eg;      // [planes][64]  e^{gamma_r}
    float *delta_state;   // slot base [batch][v_heads][128][128]
    float *o_out;         // [nseq][count][v_heads*128]
    int *err;
    int seq0, count, nchunk, qk_heads, v_heads, v_head0;
    int s_off;  // the launch's first sequence within the call
};

struct __align__(8) StateTcBarriers {
    uint64_t b1_full[2], b1_free[2], p_full[2], p_free[2], k_full[2], k_free[2];
    uint64_t s_ready, uo_full, u_ready, pu_full, s_done;
};

// (hi, lo) bf16 pairs of 32 f32 values, 2 per 32-bit word, into TMEM:
// hi = bf16x2(a, b), lo = bf16x2(a - hi.a, b - hi.b) with packed conversions.
__device__ __forceinline__ void st_split_bf16(uint32_t t_hi, uint32_t t_lo, const uint32_t (&w)[32]) {
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float a = __uint_as_float(w[2 * i]), b = __uint_as_float(w[2 * i + 1]);
        hi[i] = pack_bf16x2_rn(a, b);
        const float2 hf = bf16x2_to_float2(hi[i]);
        lo[i] = pack_bf16x2_rn(a - hf.x, b - hf.y);
    }
    sm100::tmem_st16(t_hi, hi);
    sm100::tmem_st16(t_lo, lo);
}

__global__ void __launch_bounds__(kThreadsLS, 1)
    linear_prefill_state_kernel(const __grid_constant__ CUtensorMap map_w,
                                const __grid_constant__ CUtensorMap map_q,
                                const __grid_constant__ CUtensorMap map_p,
                                const __grid_constant__ CUtensorMap map_kt, StateTcParams p) {
    using namespace sm100;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // Stage layout: B1 hi | B1 lo | P hi | P lo | K~ hi | K~ lo.
    auto b1h = [&](int st) { return smem + st * kStageLS; };
    auto b1l = [&](int st) { return smem + st * kStageLS + kB1Half; };
    auto pmh = [&](int st) { return smem + st * kStageLS + 2 * kB1Half; };
    auto pml = [&](int st) { return smem + st * kStageLS + 2 * kB1Half + kPmHalf; };
    auto kth = [&](int st) { return smem + st * kStageLS + 2 * kB1Half + 2 * kPmHalf; };
    auto ktl = [&](int st) { return smem + st * kStageLS + 2 * kB1Half + 2 * kPmHalf + kKtHalf; };
    __shared__ StateTcBarriers bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = p.v_head0 + int(blockIdx.x), s = p.s_off + int(blockIdx.y);
    auto plane = [&](int c) { return (s * p.nchunk + c) * p.v_heads + h; };

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bar.b1_full[b], 1);
            mbar_init(&bar.b1_free[b], 1);
            mbar_init(&bar.p_full[b], 1);
            mbar_init(&bar.p_free[b], 1);
            mbar_init(&bar.k_full[b], 1);
            mbar_init(&bar.k_free[b], 1);
        }
        mbar_init(&bar.s_ready, 256);
        mbar_init(&bar.uo_full, 1);
        mbar_init(&bar.u_ready, 256);
        mbar_init(&bar.pu_full, 1);
        mbar_init(&bar.s_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_s, kTmemColsLS);
        tmem_relinquish();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_base_s;
    auto fail = [&]() {
        abort_flag = 1;
        set_error(p.err, kDevErrTimeout);
    };

    if (warp == 0) {
        // ---------------------------------------------------------- TMA: [W ; Q~], P, K~
        if (lane == 0) {
            tma_prefetch_desc(&map_w);
            tma_prefetch_desc(&map_q);
            tma_prefetch_desc(&map_p);
            tma_prefetch_desc(&map_kt);
            for (int c = 0; c < p.nchunk && !abort_flag; ++c) {
                const int st = c & 1;
                const uint32_t ph = uint32_t((c - 2) >> 1) & 1u;
                const int pl2 = 2 * plane(c);  // hi plane; lo = hi + 1
                if (c >= 2 && !mbar_wait(&bar.b1_free[st], ph)) { fail(); break; }
                mbar_arrive_expect_tx(&bar.b1_full[st], 2 * kB1Half);
                for (int hl = 0; hl < 2; ++hl) {
                    unsigned char *dst = hl ? b1l(st) : b1h(st);
                    for (int blk = 0; blk < 2; ++blk) {
                        tma_load_3d(dst + blk * 16384, &map_w, blk * 64, 0, pl2 + hl, &bar.b1_full[st]);
                        tma_load_3d(dst + blk * 16384 + 8192, &map_q, blk * 64, 0, pl2 + hl,
                                    &bar.b1_full[st]);
                    }
                }
                if (c >= 2 && !mbar_wait(&bar.p_free[st], ph)) { fail(); break; }
                mbar_arrive_expect_tx(&bar.p_full[st], 2 * kPmHalf);
                tma_load_3d(pmh(st), &map_p, 0, 0, pl2, &bar.p_full[st]);
                tma_load_3d(pml(st), &map_p, 0, 0, pl2 + 1, &bar.p_full[st]);
                if (c >= 2 && !mbar_wait(&bar.k_free[st], ph)) { fail(); break; }
                mbar_arrive_expect_tx(&bar.k_full[st], 2 * kKtHalf);
                for (int blk = 0; blk < 2; ++blk) {
                    tma_load_3d(kth(st) + blk * (kKtHalf / 2), &map_kt, blk * 64, 0, pl2, &bar.k_full[st]);
                    tma_load_3d(ktl(st) + blk * (kKtHalf / 2), &map_kt, blk * 64, 0, pl2 + 1,
                                &bar.k_full[st]);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA: S [W ; Q~]^T and the update
        if (lane == 0) {
            const uint32_t id_n128 = idesc_bf16_f32(128, 128, 0, 0);
            bool ok = true;
            for (int c = 0; ok && c < p.nchunk; ++c) {
                const int st = c & 1;
                const uint32_t ph1 = uint32_t(c) & 1u, ph2 = uint32_t(c >> 1) & 1u;
                // s_ready(c): S of this chunk split into (hi, lo), the f32 state
                // pre-multiplied by e^{gamma_C}, and the epilogue done with the
                // previous chunk's D_U, D_O and D_PU.
                if (!mbar_wait(&bar.s_ready, ph1) || !mbar_wait(&bar.b1_full[st], ph2)) {
                    ok = false;
                    break;
                }
                fence_after_sync();
                const uint32_t bh = smem_addr(b1h(st)), bl = smem_addr(b1l(st));
#pragma unroll 1
                for (int kk = 0; kk < kD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    const uint64_t dh = smem_desc_sw128(bh + off, 16, 1024);
                    const uint64_t dl = smem_desc_sw128(bl + off, 16, 1024);
                    mma_f16_ta(tmem + kColU, tmem + kColSh + kk * 8, dh, id_n128, kk > 0 ? 1u : 0u);
                    mma_f16_ta(tmem + kColU, tmem + kColSl + kk * 8, dh, id_n128, 1u);
                    mma_f16_ta(tmem + kColU, tmem + kColSh + kk * 8, dl, id_n128, 1u);
                }
                mma_commit(&bar.uo_full);
                mma_commit(&bar.b1_free[st]);
                if (!mbar_wait(&bar.u_ready, ph1) || !mbar_wait(&bar.k_full[st], ph2)) {
                    ok = false;
                    break;
                }
                fence_after_sync();
                // K~ [64 r][128 i] is the MN-major B operand (K = r, N = i):
                // K-step kk is 16 rows (2048 B) in, the two 64-column blocks
                // are kKtHalf / 2 apart.
                const uint32_t kh_ = smem_addr(kth(st)), kl_ = smem_addr(ktl(st));
                const uint32_t id_n128_mn = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll 1
                for (int kk = 0; kk < kC / 16; ++kk) {
                    const uint64_t dh = smem_desc_sw128(kh_ + kk * 2048, kKtHalf / 2, 1024);
                    const uint64_t dl = smem_desc_sw128(kl_ + kk * 2048, kKtHalf / 2, 1024);
                    mma_f16_ta(tmem + kColS, tmem + kColUh + kk * 8, dh, id_n128_mn, 1u);
                    mma_f16_ta(tmem + kColS, tmem + kColUl + kk * 8, dh, id_n128_mn, 1u);
                    mma_f16_ta(tmem + kColS, tmem + kColUh + kk * 8, dl, id_n128_mn, 1u);
                }
                mma_commit(&bar.s_done);
                mma_commit(&bar.k_free[st]);
                if (abort_flag) { ok = false; break; }
            }
            if (!ok) fail();
        }
    } else if (warp == 6) {
        // ---------------------------------------------------------- MMA: D_PU = U^T P^T
        if (lane == 0) {
            const uint32_t id_n64 = idesc_bf16_f32(128, 64, 0, 0);
            bool ok = true;
            for (int c = 0; ok && c < p.nchunk; ++c) {
                const int st = c & 1;
                if (!mbar_wait(&bar.u_ready, uint32_t(c) & 1u) ||
                    !mbar_wait(&bar.p_full[st], uint32_t(c >> 1) & 1u)) {
                    ok = false;
                    break;
                }
                fence_after_sync();
                const uint32_t ph_ = smem_addr(pmh(st)), pl_ = smem_addr(pml(st));
#pragma unroll 1
                for (int kk = 0; kk < kC / 16; ++kk) {
                    const uint64_t dh = smem_desc_sw128(ph_ + kk * 32, 16, 1024);
                    const uint64_t dl = smem_desc_sw128(pl_ + kk * 32, 16, 1024);
                    mma_f16_ta(tmem + kColPU, tmem + kColUh + kk * 8, dh, id_n64, kk > 0 ? 1u : 0u);
                    mma_f16_ta(tmem + kColPU, tmem + kColUl + kk * 8, dh, id_n64, 1u);
                    mma_f16_ta(tmem + kColPU, tmem + kColUh + kk * 8, dl, id_n64, 1u);
                }
                mma_commit(&bar.pu_full);
                mma_commit(&bar.p_free[st]);
                if (abort_flag) ok = false;
            }
            if (!ok) fail();
        }
    } else {
        // ---------------------------------------------------------- epilogue
        // Warps 2-5 and 7-10: two threads per state row j, each handling half
        // of the row's columns (r in [32*half, 32*half+32) for U and O, state
        // columns [64*half, 64*half+64)).
        const int sub = warp & 3;
        const int half = warp >= 7 ? 1 : 0;
        const int j = sub * 32 + lane;
        const uint32_t lane_addr = uint32_t(sub * 32) << 16;
        const float query_scale = 1.0f / sqrtf(float(kD));
        float *S = p.delta_state + ((size_t(p.seq0 + s) * p.v_heads + h) * kD + j) * kD;
        auto wait_all = [&](uint64_t *b, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(b, parity));
        };
        const int r0 = 32 * half;
        // Initial state: (hi, lo) for chunk 0's products, e^{gamma_C(0)} S0 as the accumulator.
        bool ok = true;
        {
            const float eg0 = p.eg[size_t(plane(0)) * kC + kC - 1];
#pragma unroll 1
            for (int cb = 2 * half; cb < 2 * half + 2; ++cb) {
                uint32_t w[32];
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 v = *reinterpret_cast<const float4 *>(S + cb * 32 + i);
                    w[i] = __float_as_uint(v.x);
                    w[i + 1] = __float_as_uint(v.y);
                    w[i + 2] = __float_as_uint(v.z);
                    w[i + 3] = __float_as_uint(v.w);
                }
                st_split_bf16(tmem + lane_addr + kColSh + cb * 16, tmem + lane_addr + kColSl + cb * 16, w);
#pragma unroll
                for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(__uint_as_float(w[i]) * eg0);
                tmem_st32(tmem + lane_addr + kColS + cb * 32, w);
            }
            tmem_wait_st();
            fence_before_sync();
            mbar_arrive(&bar.s_ready);
        }
        for (int c = 0; ok && c < p.nchunk; ++c) {
            const uint32_t ph = uint32_t(c) & 1u;
            const size_t lb = size_t(plane(c));
            const float *utp = p.ut + (lb * kC + r0) * kD + j;
            float ut[32];
#pragma unroll
            for (int r = 0; r < 32; ++r) ut[r] = utp[r * kD];
            if (!wait_all(&bar.uo_full, ph)) { ok = false; break; }
            fence_after_sync();
            // U^T row j (this half's r) = Ut^T - D_U as bf16 (hi, lo).
            {
                uint32_t d[32];
                tmem_ld32(tmem + lane_addr + kColU + r0, d);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) d[i] = __float_as_uint(ut[i] - __uint_as_float(d[i]));
                st_split_bf16(tmem + lane_addr + kColUh + half * 16, tmem + lane_addr + kColUl + half * 16, d);
            }
            // e^{gamma_r} (S0 q_r) (Q~ carries the decay), kept until D_PU is ready.
            float os[32];
            {
                uint32_t d[32];
                tmem_ld32(tmem + lane_addr + kColOq + r0, d);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) os[i] = __uint_as_float(d[i]);
            }
            tmem_wait_st();
            fence_before_sync();
            mbar_arrive(&bar.u_ready);
            if (!wait_all(&bar.pu_full, ph)) { ok = false; break; }
            fence_after_sync();
            const int t0 = c * kC + r0;
            float *orow = p.o_out + (size_t(s) * p.count + t0) * (size_t(p.v_heads) * kD) + h * kD + j;
            {
                uint32_t d[32];
                tmem_ld32(tmem + lane_addr + kColPU + r0, d);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (t0 + i < p.count)
                        orow[size_t(i) * p.v_heads * kD] = (os[i] + __uint_as_float(d[i])) * query_scale;
            }
            // The updated state: (hi, lo) for the next chunk's products and the
            // f32 accumulator pre-multiplied by the next chunk's e^{gamma_C};
            // after the last chunk, the final state.
            if (!wait_all(&bar.s_done, ph)) { ok = false; break; }
            fence_after_sync();
            const bool last = c == p.nchunk - 1;
            const float egn = last ? 1.f : p.eg[size_t(plane(c + 1)) * kC + kC - 1];
            const float2 egn2 = make_float2(egn, egn);
#pragma unroll 1
            for (int cb = 2 * half; cb < 2 * half + 2; ++cb) {
                uint32_t w[32];
                tmem_ld32(tmem + lane_addr + kColS + cb * 32, w);
                tmem_wait_ld();
                if (last) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(S + cb * 32 + i) =
                            make_float4(__uint_as_float(w[i]), __uint_as_float(w[i + 1]),
                                        __uint_as_float(w[i + 2]), __uint_as_float(w[i + 3]));
                } else {
                    st_split_bf16(tmem + lane_addr + kColSh + cb * 16,
                                  tmem + lane_addr + kColSl + cb * 16, w);
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float2 v = fmul2(make_float2(__uint_as_float(w[i]), __uint_as_float(w[i + 1])), egn2);
                        w[i] = __float_as_uint(v.x);
                        w[i + 1] = __float_as_uint(v.y);
                    }
                    tmem_st32(tmem + lane_addr + kColS + cb * 32, w);
                }
            }
            if (!last) {
                tmem_wait_st();
                fence_before_sync();
                mbar_arrive(&bar.s_ready);
            }
            if (__any_sync(0xffffffffu, abort_flag != 0)) { ok = false; break; }
        }
        if (!ok && lane == 0) fail();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 1) tmem_dealloc(tmem, kTmemColsLS);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_ls() {
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

// 3-D bf16 map over [planes][rows][cols] with a box of 64 x box_rows x 1 and
// 128-byte swizzle (K-major operand tiles of 64 bf16 per row).
bool make_map_bf16_ls(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows,
                      uint64_t planes, uint32_t box_rows) {
    auto enc = encode_tiled_ls();
    if (!enc) return false;
    cuuint64_t dims[3] = {cols, rows, planes};
    cuuint64_t strides[2] = {cols * 2, cols * 2 * rows};
    cuuint32_t box[3] = {64, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides,
               box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D map of f32 over [planes][rows][cols] with a box of 128 x kSeg x 1, no
// swizzle: a conv segment's channel block.
bool make_map_f32_rows(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows,
                       uint64_t planes) {
    auto enc = encode_tiled_ls();
    if (!enc) return false;
    cuuint64_t dims[3] = {cols, rows, planes};
    cuuint64_t strides[2] = {cols * 4, cols * 4 * rows};
    cuuint32_t box[3] = {128, uint32_t(kSeg), 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(base), dims, strides, box,
               es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ----------------------------------------------------------------------------
// L5: per-head RMSNorm + SiLU(z)
// ----------------------------------------------------------------------------
struct OutParams {
    const float *z;
    const float *ssm_norm;
    float *attention;  // in: O; out: normalised, gated
    int count, v_heads, v_head0, v_head_count;
    float eps;
    int s_off;         // the launch's first sequence within the call
};

__global__ void __launch_bounds__(256) linear_prefill_out_kernel(OutParams p) {
    const int t = blockIdx.x, s = p.s_off + int(blockIdx.y);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t base = (size_t(s) * p.count + t) * size_t(p.v_heads) * kD;
    for (int h = p.v_head0 + warp; h < p.v_head0 + p.v_head_count; h += 8) {
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
    // Per (chunk, value head), in f32 units: W, Q~ as bf16 (hi, lo) [2][64][128]
    // (one f32 each per element pair), P [2][64][64] bf16, K~ [2][64][128]
    // bf16, Ut [64][128] f32, e^gamma [64] f32.
    return size_t(nchunk_total) * v_heads * kC * (4 * kD + kC + 1);
}

cudaError_t launch_linear_prefill(const LinearPrefillLaunch &a, cudaStream_t stream) {
    const int qkv_dim = (2 * a.qk_heads + a.v_heads) * kD;
    const int nchunk = (a.count + kC - 1) / kC;
    // The segment boundaries live at the start of the W scratch, which L3
    // only writes after the conv has finished.
    const int nseg = (a.count + kSeg - 1) / kSeg;
    if (a.v_head_count <= 0 || a.v_head0 < 0 || a.v_head0 + a.v_head_count > a.v_heads)
        return cudaErrorInvalidValue;
    ConvParams cp{a.qkv, a.conv_state, a.conv_w, a.scratch, a.seq0, a.count, qkv_dim, nseg,
                  2 * a.qk_heads * kD, a.v_head0, a.eps, a.err};
    // Every q and k channel block, and the blocks of the call's value heads.
    const dim3 conv_grid(2 * a.qk_heads + a.v_head_count, nseg, a.nseq);
    linear_prefill_conv_bounds_kernel<<<conv_grid, 128, 0, stream>>>(cp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap mx;
    if (!make_map_f32_rows(&mx, a.qkv, uint64_t(qkv_dim), uint64_t(a.count), uint64_t(a.nseq)))
        return cudaErrorInvalidValue;
    if ((e = cudaFuncSetAttribute(linear_prefill_conv_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, int(kConvTileBytes))) !=
        cudaSuccess)
        return e;
    linear_prefill_conv_kernel<<<conv_grid, 128, kConvTileBytes, stream>>>(mx, cp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    NormParams np{a.qkv, a.beta, a.alpha, a.dt_bias, a.ssm_a, a.count, a.qk_heads, a.v_heads,
                  qkv_dim, a.v_head0, a.v_head_count, a.eps};
    linear_prefill_norm_kernel<<<dim3(a.count, a.nseq), 256, 0, stream>>>(np);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    const size_t per = size_t(a.nseq) * nchunk * a.v_heads;
    __nv_bfloat16 *w2 = reinterpret_cast<__nv_bfloat16 *>(a.scratch);
    __nv_bfloat16 *q2 = w2 + per * 2 * kC * kD;
    __nv_bfloat16 *p2 = q2 + per * 2 * kC * kD;
    __nv_bfloat16 *k2 = p2 + per * 2 * kC * kC;
    float *ut = reinterpret_cast<float *>(k2 + per * 2 * kD * kC);
    float *eg = ut + per * kC * kD;
    LocalParams lp{a.qkv, a.beta, a.alpha, w2, q2, p2, k2, ut, eg, a.err, a.count, nchunk,
                   a.qk_heads, a.v_heads, qkv_dim, a.v_head0, a.v_head_count};
    if ((e = cudaFuncSetAttribute(linear_prefill_local_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, int(kLocSmem))) !=
        cudaSuccess)
        return e;
    linear_prefill_local_kernel<<<dim3(nchunk, a.qk_heads, a.nseq), 256, kLocSmem, stream>>>(lp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;

    CUtensorMap mw, mq, mp, mk;
    if (!make_map_bf16_ls(&mw, w2, kD, kC, 2 * per, kC) ||
        !make_map_bf16_ls(&mq, q2, kD, kC, 2 * per, kC) ||
        !make_map_bf16_ls(&mp, p2, kC, kC, 2 * per, kC) ||
        !make_map_bf16_ls(&mk, k2, kD, kC, 2 * per, kC))
        return cudaErrorInvalidValue;
    StateTcParams sp{ut, eg, a.delta_state, a.attention, a.err, a.seq0, a.count, nchunk,
                     a.qk_heads, a.v_heads, a.v_head0, 0};
    if ((e = cudaFuncSetAttribute(linear_prefill_state_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemLS))) !=
        cudaSuccess)
        return e;
    OutParams op{a.z, a.ssm_norm, a.attention, a.count, a.v_heads, a.v_head0, a.v_head_count,
                 a.eps, 0};
    // The state pass has one CTA per (value head, sequence) and needs a whole
    // SM each, so a large call runs in more than one wave; the output pass of
    // a sequence only needs that sequence's state pass. With side streams,
    // groups of sequences get their own state + output passes (launched in
    // sequence order, so the first groups fill the first wave), and a
    // group's output pass runs on the SMs the last wave leaves idle.
    const int groups = (a.nside > 1 && a.side && a.join && a.fork) ? std::min(a.nside, a.nseq) : 1;
    if (groups <= 1) {
        linear_prefill_state_kernel<<<dim3(a.v_head_count, a.nseq), kThreadsLS, kSmemLS, stream>>>(
            mw, mq, mp, mk, sp);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        linear_prefill_out_kernel<<<dim3(a.count, a.nseq), 256, 0, stream>>>(op);
        return cudaGetLastError();
    }
    if ((e = cudaEventRecord(a.fork, stream)) != cudaSuccess) return e;
    for (int g = 0; g < groups; ++g) {
        const int s0 = a.nseq * g / groups, s1 = a.nseq * (g + 1) / groups;
        cudaStream_t side = a.side[g];
        if ((e = cudaStreamWaitEvent(side, a.fork, 0)) != cudaSuccess) return e;
        sp.s_off = s0;
        op.s_off = s0;
        linear_prefill_state_kernel<<<dim3(a.v_head_count, s1 - s0), kThreadsLS, kSmemLS, side>>>(
            mw, mq, mp, mk, sp);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        linear_prefill_out_kernel<<<dim3(a.count, s1 - s0), 256, 0, side>>>(op);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        if ((e = cudaEventRecord(a.join[g], side)) != cudaSuccess) return e;
    }
    for (int g = 0; g < groups; ++g)
        if ((e = cudaStreamWaitEvent(stream, a.join[g], 0)) != cudaSuccess) return e;
    return cudaSuccess;
}

}  // namespace q38
