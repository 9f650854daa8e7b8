// deltanet_decode.cu -- Gated DeltaNet decode (linear_core, src/model/ops.rs:647-742).
//
//   D3 linear_decode_sweep  the device entry points' kernel: one persistent
//                           CTA per SM streams (sequence, value head) units,
//                           each a 64 KB f32 state read and written once by
//                           bulk copies through shared memory, and does per
//                           unit the conv with carried state (ops.rs:665-676,
//                           multiply then add), SiLU (ops.rs:677), the q / k
//                           L2 norms (ops.rs:679-684, f64 sum), the gates
//                           (ops.rs:685-688), the decay and delta rule per
//                           state row (ops.rs:707-713) and the per-head RMSNorm
//                           + SiLU(z) epilogue (ops.rs:735-740). qkv, beta and
//                           alpha are rewritten in place, as the reference does.
//
// The host-pointer entry point splits the same work in two stream-ordered
// kernels, so that the in-place qkv / beta / alpha can be copied back while
// the state pass runs:
//
//   D1 linear_decode_prep   one CTA per (128-channel block, sequence): conv,
//                           SiLU, L2 norms and gates, in place.
//   D2 linear_decode_state  one CTA per (value head, sequence): the state pass
//                           and the epilogue; its state loads are issued
//                           before it waits on D1, so they overlap D1's tail.
//
// In the layer-level decode call the projections' epilogues apply the conv,
// SiLU and gates (proj_epilogue), and the sweep only L2-normalises q and k.
//
// HBM layout (reference layouts): conv state [batch][qkv_dim][3], delta state
// [batch][v_heads][128 columns][128], f32.
#include <algorithm>

#include "q38_sm100.cuh"

namespace q38 {
namespace {

constexpr int kPrepThreads = kLinHeadDim;  // one channel per thread, one head per CTA
constexpr int kStateThreads = 256;          // 8 warps x 16 columns
constexpr int kColsPerWarp = kLinHeadDim / (kStateThreads / 32);

struct PrepParams {
    float *qkv;
    float *beta, *alpha;
    float *conv_state;
    const float *conv_w, *dt_bias, *ssm_a;
    int qk_heads, v_heads, qkv_dim;
    float eps;
};

__global__ void __launch_bounds__(kPrepThreads) linear_decode_prep_kernel(PrepParams p) {
    pdl_launch_dependents();
    __shared__ double red[32];
    const int blk = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    const int ch = blk * kLinHeadDim + t;
    float *s = p.conv_state + (size_t(b) * p.qkv_dim + ch) * 3;
    const float4 w = reinterpret_cast<const float4 *>(p.conv_w)[ch];
    float *x_ptr = p.qkv + size_t(b) * p.qkv_dim + ch;
    const float x = *x_ptr;
    const float s0 = s[0], s1 = s[1], s2 = s[2];
    // value = s0*w0; value += s1*w1; value += s2*w2; value += x*w3 (no fma).
    float v = s0 * w.x;
    v += s1 * w.y;
    v += s2 * w.z;
    v += x * w.w;
    s[0] = s1;
    s[1] = s2;
    s[2] = x;
    float y = siluf_ref(v);
    if (blk < 2 * p.qk_heads) {
        // l2norm (ops.rs:562-571): 1 / max(sqrt((f32) sum_f64), eps).
        const double sum = block_sum_f64(double(y) * double(y), red);
        const float scale = 1.0f / fmaxf(sqrtf(float(sum)), p.eps);
        y *= scale;
    } else if (t == 0) {
        const int hv = blk - 2 * p.qk_heads;
        float *bp = p.beta + size_t(b) * p.v_heads + hv;
        float *ap = p.alpha + size_t(b) * p.v_heads + hv;
        *bp = sigmoidf_ref(*bp);
        *ap = p.ssm_a[hv] * softplusf_ref(*ap + p.dt_bias[hv]);
    }
    *x_ptr = y;
}

struct StateParams {
    const float *qkv;
    const float *z;
    const float *beta, *alpha;
    float *delta_state;
    const float *ssm_norm;
    float *attention;
    int qk_heads, v_heads, qkv_dim;
    int l2_prologue;  // q and k arrive convolved but not yet L2-normalised
    float eps;
};

__global__ void __launch_bounds__(kStateThreads) linear_decode_state_kernel(StateParams p) {
    __shared__ float outs[kLinHeadDim];
    __shared__ double red[32];
    const int hv = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float4 *S = reinterpret_cast<float4 *>(
        p.delta_state + (size_t(b) * p.v_heads + hv) * kLinHeadDim * kLinHeadDim);
    const int col0 = warp * kColsPerWarp;

    // The state does not depend on D1: load this warp's 16 rows now.
    float4 s[kColsPerWarp];
#pragma unroll
    for (int i = 0; i < kColsPerWarp; ++i) s[i] = S[(col0 + i) * (kLinHeadDim / 4) + lane];

    pdl_wait_primary();  // D1's qkv / beta / alpha

    const int kh = hv % p.qk_heads;  // ops.rs:699
    const int qk_dim = p.qk_heads * kLinHeadDim;
    const float *row = p.qkv + size_t(b) * p.qkv_dim;
    float4 q = reinterpret_cast<const float4 *>(row + kh * kLinHeadDim)[lane];
    float4 k = reinterpret_cast<const float4 *>(row + qk_dim + kh * kLinHeadDim)[lane];
    if (p.l2_prologue) {
        // l2norm (ops.rs:562-571) of the key head's q and k, here rather than
        // in D1 (the layer-level call's projections already applied the conv,
        // SiLU and gates): every warp holds both heads whole, four values per
        // lane, and sums their squares in f64.
        const double sq = warp_sum_f64(double(q.x) * q.x + double(q.y) * q.y + double(q.z) * q.z +
                                       double(q.w) * q.w);
        const double sk = warp_sum_f64(double(k.x) * k.x + double(k.y) * k.y + double(k.z) * k.z +
                                       double(k.w) * k.w);
        const float cq = 1.0f / fmaxf(sqrtf(float(sq)), p.eps);
        const float ck = 1.0f / fmaxf(sqrtf(float(sk)), p.eps);
        q.x *= cq, q.y *= cq, q.z *= cq, q.w *= cq;
        k.x *= ck, k.y *= ck, k.z *= ck, k.w *= ck;
    }
    const float vmine = lane < kColsPerWarp ? row[2 * qk_dim + hv * kLinHeadDim + col0 + lane] : 0.f;
    const float beta = p.beta[size_t(b) * p.v_heads + hv];
    const float decay = expf(p.alpha[size_t(b) * p.v_heads + hv]);
    const float query_scale = 1.0f / sqrtf(float(kLinHeadDim));

#pragma unroll
    for (int i = 0; i < kColsPerWarp; ++i) {
        float4 r = s[i];
        r.x *= decay;
        r.y *= decay;
        r.z *= decay;
        r.w *= decay;
        // dot_128 (ops.rs:573-579): lane-local fma chain, then the warp tree.
        float pred = fmaf(r.w, k.w, fmaf(r.z, k.z, fmaf(r.y, k.y, r.x * k.x)));
        pred = warp_sum(pred);
        const float vj = __shfl_sync(0xffffffffu, vmine, i);
        const float delta = (vj - pred) * beta;
        // mad_dot_128 (ops.rs:584-591): state += k*delta (fma), then dot with q.
        r.x = fmaf(k.x, delta, r.x);
        r.y = fmaf(k.y, delta, r.y);
        r.z = fmaf(k.z, delta, r.z);
        r.w = fmaf(k.w, delta, r.w);
        float o = fmaf(r.w, q.w, fmaf(r.z, q.z, fmaf(r.y, q.y, r.x * q.x)));
        o = warp_sum(o);
        S[(col0 + i) * (kLinHeadDim / 4) + lane] = r;
        if (lane == 0) outs[col0 + i] = o * query_scale;
    }
    __syncthreads();
    // rmsnorm_inplace(ssm_norm) then *= silu(z) (ops.rs:735-740).
    const int t = threadIdx.x;
    const float o = t < kLinHeadDim ? outs[t] : 0.f;
    const double sum = block_sum_f64(t < kLinHeadDim ? double(o) * double(o) : 0.0, red);
    if (t < kLinHeadDim) {
        const float scale = rms_scale_from_sum(sum, kLinHeadDim, p.eps);
        float y = o * scale * p.ssm_norm[t];
        const size_t off = size_t(b) * p.v_heads * kLinHeadDim + size_t(hv) * kLinHeadDim + t;
        y *= siluf_ref(p.z[off]);
        p.attention[off] = y;
    }
}

// ---------------------------------------------------------------------------
// D3 linear_decode_sweep: D1 and D2 as one persistent kernel, one CTA per SM.
// A unit is one (sequence, value head): its 64 KB state is one contiguous
// range, so a producer warp streams units through a ring of kSweepStages
// shared-memory stages with bulk copies (load, then the updated state stored
// back from the same stage) while 16 compute warps run each unit's prep
// (conv, SiLU, gates), its delta-rule sweep over the staged state and its
// output epilogue, with the next unit's inputs loaded during the sweep.
//
// The q and k channels of key head kh are read by every value head with
// hv % qk_heads == kh (ops.rs:699), in different units; each unit convolves
// them itself from the carried conv state. The conv state and the in-place
// q / k outputs of that key head are written once, by the last of its
// readers: a per-(sequence, key head) counter in the state counts the units
// that have read them, and the unit that brings it to the reader count writes
// them and resets the counter, so no reader can see an advanced conv state.
// ---------------------------------------------------------------------------
constexpr int kSweepStages = 3;
constexpr int kSweepWarps = 16;                            // compute warps
constexpr int kSweepThreads = (kSweepWarps + 1) * 32;      // + the producer warp
constexpr int kSweepCols = kLinHeadDim / kSweepWarps;      // state rows per warp
constexpr uint32_t kStateBytes = kLinHeadDim * kLinHeadDim * 4;
constexpr int kSweepComputeThreads = kSweepWarps * 32;
constexpr int kBarCompute = 1, kBarEpilogue = 2;           // named barriers (0: __syncthreads)

struct SweepParams {
    float *qkv;
    const float *z;
    float *beta, *alpha;
    float *conv_state;
    float *delta_state;
    const float *conv_w, *dt_bias, *ssm_a, *ssm_norm;
    float *attention;
    int *group_count;  // [batch][qk_heads] readers of a key head so far (0 between calls)
    int *err;
    int batch, qk_heads, v_heads, qkv_dim;
    int prepped;       // conv, SiLU and gates already applied by the projections
    float eps;
    uint64_t wait_ns;
};

struct SweepSmem {
    float4 state[kSweepStages][kLinHeadDim * kLinHeadDim / 4];
    float q[kLinHeadDim], k[kLinHeadDim], v[kLinHeadDim];
    float outs[kLinHeadDim];
    float gate[2];  // beta, decay
    double red_qk[8];  // per-warp sums of squares: q (warps 0-3), k (4-7)
    double red_o[4];   // the epilogue's per-warp sums of squares
    int last;          // this unit is the last reader of its key head
    uint64_t full[kSweepStages], done[kSweepStages];
};

__device__ __forceinline__ void bulk_store(void *dst_gmem, const void *src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_gmem),
                 "r"(smem_addr(src_smem)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_wait_group0() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// True on every participating thread if `pred` holds on any of them.
__device__ __forceinline__ bool named_barrier_any(int id, int threads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(pred ? 1u : 0u), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

// One channel's raw prep inputs (threads 0-383: q, k, v channels), or the
// unit's gate inputs (thread 384).
struct SweepIn {
    float x = 0.f, s0 = 0.f, s1 = 0.f, s2 = 0.f;
    float4 w = {0.f, 0.f, 0.f, 0.f};
};

__device__ __forceinline__ int sweep_channel(const SweepParams &p, int tid, int hv) {
    const int kh = hv % p.qk_heads, qk_dim = p.qk_heads * kLinHeadDim;
    const int c = tid & (kLinHeadDim - 1);
    if (tid < kLinHeadDim) return kh * kLinHeadDim + c;
    if (tid < 2 * kLinHeadDim) return qk_dim + kh * kLinHeadDim + c;
    return 2 * qk_dim + hv * kLinHeadDim + c;
}

__device__ __forceinline__ SweepIn sweep_load(const SweepParams &p, int tid, int b, int hv) {
    SweepIn in;
    if (tid < 3 * kLinHeadDim) {
        const int ch = sweep_channel(p, tid, hv);
        in.x = p.qkv[size_t(b) * p.qkv_dim + ch];
        if (!p.prepped) {
            const float *s = p.conv_state + (size_t(b) * p.qkv_dim + ch) * 3;
            in.s0 = s[0];
            in.s1 = s[1];
            in.s2 = s[2];
            in.w = reinterpret_cast<const float4 *>(p.conv_w)[ch];
        }
    } else if (tid == 3 * kLinHeadDim) {
        in.x = p.beta[size_t(b) * p.v_heads + hv];
        in.s0 = p.alpha[size_t(b) * p.v_heads + hv];
        if (!p.prepped) {
            in.s1 = p.ssm_a[hv];
            in.s2 = p.dt_bias[hv];
        }
    }
    return in;
}

// Sums eight per-lane values over the warp: the total of value j lands in
// the four lanes with (lane >> 2) & 7 == j, bitwise equal. Three exchange
// steps halve the values each lane carries, two more finish the sums (9
// shuffles for 8 sums instead of 40).
__device__ __forceinline__ float warp_sum8(const float (&v)[8], int lane) {
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
    float a[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const float keep = h16 ? v[t + 4] : v[t];
        const float send = h16 ? v[t] : v[t + 4];
        a[t] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float c2[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float keep = h8 ? a[t + 2] : a[t];
        const float send = h8 ? a[t] : a[t + 2];
        c2[t] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float c = (h4 ? c2[1] : c2[0]) + __shfl_xor_sync(0xffffffffu, h4 ? c2[0] : c2[1], 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

// rmsnorm_inplace(ssm_norm) then *= silu(z) (ops.rs:735-740) of a unit's 128
// outputs, by warps 12-15 (t = output index).
__device__ __forceinline__ void sweep_epilogue(const SweepParams &p, SweepSmem &sm, int t, int unit,
                                               float zv) {
    const int lane = t & 31, w = t >> 5;
    const float o = sm.outs[t];
    const double part = warp_sum_f64(double(o) * double(o));
    if (lane == 0) sm.red_o[w] = part;
    sm100::named_barrier_sync(kBarEpilogue, kLinHeadDim);
    const double sum = sm.red_o[0] + sm.red_o[1] + sm.red_o[2] + sm.red_o[3];
    const float scale = rms_scale_from_sum(sum, kLinHeadDim, p.eps);
    float y = o * scale * p.ssm_norm[t];
    y *= siluf_ref(zv);
    p.attention[size_t(unit) * kLinHeadDim + t] = y;
}

__global__ void __launch_bounds__(kSweepThreads, 1) linear_decode_sweep_kernel(SweepParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    SweepSmem &sm = *reinterpret_cast<SweepSmem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int units = p.batch * p.v_heads;
    const int n = (units - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);
    auto unit_of = [&](int i) { return int(blockIdx.x) + i * int(gridDim.x); };
    auto state_of = [&](int i) {
        return reinterpret_cast<float4 *>(p.delta_state) + size_t(unit_of(i)) * (kLinHeadDim * kLinHeadDim / 4);
    };

    if (tid == 0) {
        for (int s = 0; s < kSweepStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.done[s], kSweepWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    // Inputs and state may be written by the preceding kernel in the stream.
    pdl_wait_primary();

    if (warp == kSweepWarps) {
        // Producer: unit i's load goes into stage i % S once unit i - S's
        // updated state has been stored from it.
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            for (int i = 0; i < n && ok; ++i) {
                const int s = i % kSweepStages;
                if (i >= kSweepStages) {
                    if (!mbar_wait_ns(&sm.done[s], ((i - kSweepStages) / kSweepStages) & 1, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    bulk_store(state_of(i - kSweepStages), sm.state[s], kStateBytes);
                    sm100::bulk_commit_group();
                    sm100::bulk_wait_group_read0();
                }
                mbar_arrive_expect_tx(&sm.full[s], kStateBytes);
                bulk_load(sm.state[s], state_of(i), kStateBytes, &sm.full[s]);
                issued = i + 1;
            }
            for (int i = issued > kSweepStages ? issued - kSweepStages : 0; i < issued && ok; ++i) {
                const int s = i % kSweepStages;
                if (!mbar_wait_ns(&sm.done[s], (i / kSweepStages) & 1, p.wait_ns)) {
                    ok = false;
                    break;
                }
                bulk_store(state_of(i), sm.state[s], kStateBytes);
                sm100::bulk_commit_group();
            }
            if (!ok) {
                set_error(p.err, kDevErrTimeout);
                // Loads still in flight land before the CTA may exit: wait
                // (bounded) for the last load issued into every stage.
                for (int i = issued > kSweepStages ? issued - kSweepStages : 0; i < issued; ++i)
                    mbar_wait_ns(&sm.full[i % kSweepStages], (i / kSweepStages) & 1, p.wait_ns);
            }
            bulk_wait_group0();
        }
        return;
    }

    // Compute warps. Per unit i: warps 0-11 convolve the unit's q, k and v
    // channels (and warps 0-7 sum the squares of q and k) while warps 12-15
    // finish unit i-1's output epilogue and warp 12 computes the gates; then
    // all 16 sweep the staged state, 8 rows per warp.
    const int qk_dim = p.qk_heads * kLinHeadDim;
    const int readers = p.v_heads / p.qk_heads;
    const float query_scale = 1.0f / sqrtf(float(kLinHeadDim));
    const int col0 = warp * kSweepCols;
    const int my_col = (lane >> 2) & 7;  // the row whose sums this lane receives (warp_sum8)
    SweepIn in = n > 0 ? sweep_load(p, tid, unit_of(0) / p.v_heads, unit_of(0) % p.v_heads)
                       : SweepIn{};
    float zv = 0.f;      // warps 12-15: z of the unit whose epilogue comes next
    int prev_unit = -1;  // that unit
    bool aborted = false;
    for (int i = 0; i < n; ++i) {
        const int u = unit_of(i), b = u / p.v_heads, hv = u % p.v_heads, kh = hv % p.qk_heads;
        const int s = i % kSweepStages;
        float4 *S = sm.state[s];

        if (warp < 12) {
            // D1's per-channel work for this unit's channels.
            float y = in.x;
            if (!p.prepped) {
                // value = s0*w0; value += s1*w1; value += s2*w2; value += x*w3 (ops.rs:665-676)
                float c = in.s0 * in.w.x;
                c += in.s1 * in.w.y;
                c += in.s2 * in.w.z;
                c += in.x * in.w.w;
                y = siluf_ref(c);  // ops.rs:677
                if (warp >= 8) {
                    // The value channels belong to this unit alone.
                    const int ch = sweep_channel(p, tid, hv);
                    float *cs = p.conv_state + (size_t(b) * p.qkv_dim + ch) * 3;
                    cs[0] = in.s1;
                    cs[1] = in.s2;
                    cs[2] = in.x;
                    p.qkv[size_t(b) * p.qkv_dim + ch] = y;
                }
            }
            float *dst = warp < 4 ? sm.q : warp < 8 ? sm.k : sm.v;
            dst[tid & (kLinHeadDim - 1)] = y;
            // l2norm (ops.rs:562-571): f64 sum of squares, per warp here and
            // over the head's four warps below.
            if (warp < 8) {
                const double part = warp_sum_f64(double(y) * double(y));
                if (lane == 0) sm.red_qk[warp] = part;
            }
        } else {
            if (prev_unit >= 0) sweep_epilogue(p, sm, tid - 12 * 32, prev_unit, zv);
            if (tid == 12 * 32) {
                float bt = in.x, al = in.s0;
                if (!p.prepped) {
                    bt = sigmoidf_ref(bt);                   // ops.rs:685-686
                    al = in.s1 * softplusf_ref(al + in.s2);  // ops.rs:687-688
                    p.beta[size_t(b) * p.v_heads + hv] = bt;
                    p.alpha[size_t(b) * p.v_heads + hv] = al;
                }
                sm.gate[0] = bt;
                sm.gate[1] = expf(al);
            }
        }
        sm100::named_barrier_sync(kBarCompute, kSweepComputeThreads);

        // Every thread's raw q / k reads have returned (their values were
        // used above, before the barrier): count this unit as a reader of its
        // key head. The add is relaxed so that warp 0 does not wait for it;
        // its result is first used after the sweep. A unit that sees every
        // other reader counted writes only after that result, so its writes
        // follow the other readers' completed reads.
        int old = 0;
        if (!p.prepped && tid == 0) old = atomicAdd(p.group_count + size_t(b) * p.qk_heads + kh, 1);
        // The q / k channels' new conv state, in case this unit writes it.
        const float ns0 = in.s1, ns1 = in.s2, ns2 = in.x;
        // The next unit's inputs and this unit's z, loaded during the sweep.
        if (i + 1 < n) in = sweep_load(p, tid, unit_of(i + 1) / p.v_heads, unit_of(i + 1) % p.v_heads);
        if (warp >= 12) zv = p.z[size_t(u) * kLinHeadDim + (tid - 12 * 32)];
        prev_unit = u;

        float4 q = reinterpret_cast<const float4 *>(sm.q)[lane];
        float4 k = reinterpret_cast<const float4 *>(sm.k)[lane];
        {
            const double sq = sm.red_qk[0] + sm.red_qk[1] + sm.red_qk[2] + sm.red_qk[3];
            const double sk = sm.red_qk[4] + sm.red_qk[5] + sm.red_qk[6] + sm.red_qk[7];
            const float cq = 1.0f / fmaxf(sqrtf(float(sq)), p.eps);
            const float ck = 1.0f / fmaxf(sqrtf(float(sk)), p.eps);
            q.x *= cq, q.y *= cq, q.z *= cq, q.w *= cq;
            k.x *= ck, k.y *= ck, k.z *= ck, k.w *= ck;
        }
        const float vmine = sm.v[col0 + my_col];
        const float beta = sm.gate[0], decay = sm.gate[1];

        const bool ok = mbar_wait_ns(&sm.full[s], (i / kSweepStages) & 1, p.wait_ns);
        if (named_barrier_any(kBarCompute, kSweepComputeThreads, !ok)) {
            if (tid == 0) set_error(p.err, kDevErrTimeout);
            aborted = true;
            break;
        }
        // Per state row (ops.rs:707-713): decay; pred = dot_128(row, k);
        // delta = (v - pred) * beta; row += k * delta (fma, mad_dot_128,
        // ops.rs:584-591); o = dot(row, q). Each lane holds four elements of
        // the warp's 8 rows; the dot products are lane-local fma chains, then
        // one reduction of all 8 rows at once.
        float4 r[kSweepCols];
        float part[kSweepCols];
#pragma unroll
        for (int j = 0; j < kSweepCols; ++j) {
            r[j] = S[(col0 + j) * (kLinHeadDim / 4) + lane];
            r[j].x *= decay;
            r[j].y *= decay;
            r[j].z *= decay;
            r[j].w *= decay;
            part[j] = fmaf(r[j].w, k.w, fmaf(r[j].z, k.z, fmaf(r[j].y, k.y, r[j].x * k.x)));
        }
        const float pred = warp_sum8(part, lane);
        const float delta_mine = (vmine - pred) * beta;
#pragma unroll
        for (int j = 0; j < kSweepCols; ++j) {
            const float delta = __shfl_sync(0xffffffffu, delta_mine, 4 * j);
            r[j].x = fmaf(k.x, delta, r[j].x);
            r[j].y = fmaf(k.y, delta, r[j].y);
            r[j].z = fmaf(k.z, delta, r[j].z);
            r[j].w = fmaf(k.w, delta, r[j].w);
            part[j] = fmaf(r[j].w, q.w, fmaf(r[j].z, q.z, fmaf(r[j].y, q.y, r[j].x * q.x)));
            S[(col0 + j) * (kLinHeadDim / 4) + lane] = r[j];
        }
        const float o = warp_sum8(part, lane);
        if ((lane & 3) == 0) sm.outs[col0 + my_col] = o * query_scale;
        // The producer's bulk store reads the stage through the async proxy.
        sm100::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.done[s]);
        if (!p.prepped && tid == 0) sm.last = old == readers - 1;
        sm100::named_barrier_sync(kBarCompute, kSweepComputeThreads);

        if (!p.prepped && sm.last) {
            // The last reader of key head kh: its conv state and in-place
            // normalised q / k.
            if (warp < 8) {
                const int ch = sweep_channel(p, tid, hv);
                float *cs = p.conv_state + (size_t(b) * p.qkv_dim + ch) * 3;
                cs[0] = ns0;
                cs[1] = ns1;
                cs[2] = ns2;
            }
            if (warp == 0) {
                float4 *row = reinterpret_cast<float4 *>(p.qkv + size_t(b) * p.qkv_dim);
                row[(kh * kLinHeadDim) / 4 + lane] = q;
                row[(qk_dim + kh * kLinHeadDim) / 4 + lane] = k;
                if (lane == 0) p.group_count[size_t(b) * p.qk_heads + kh] = 0;
            }
        }
    }
    if (!aborted && warp >= 12 && prev_unit >= 0) sweep_epilogue(p, sm, tid - 12 * 32, prev_unit, zv);
}

}  // namespace

static_assert(sizeof(SweepSmem) <= 227 * 1024, "sweep kernel shared memory");

cudaError_t ensure_sweep_smem_limit() {
    static bool set[128] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 128 && set[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(linear_decode_sweep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(sizeof(SweepSmem)));
    if (e == cudaSuccess && dev < 128) set[dev] = true;
    return e;
}

cudaError_t launch_linear_decode(const LinearDecodeLaunch &a, cudaStream_t stream, cudaEvent_t prep_done) {
    const int qkv_dim = (2 * a.qk_heads + a.v_heads) * kLinHeadDim;
    cudaError_t e = cudaSuccess;
    // The fused sweep, unless the caller needs the prep's results before the
    // state pass (prep_done) or the geometry has key heads that no value head
    // reads an equal number of times.
    const bool sweep = !prep_done && a.sm_count > 0 && a.qk_heads > 0 &&
                       a.v_heads % a.qk_heads == 0 && (a.prepped || a.group_count);
    if (sweep) {
        if ((e = ensure_sweep_smem_limit()) != cudaSuccess) return e;
        SweepParams sp{a.qkv,      a.z,          a.beta,     a.alpha,     a.conv_state,
                       a.delta_state, a.conv_w,  a.dt_bias,  a.ssm_a,     a.ssm_norm,
                       a.attention, a.group_count, a.err,    a.batch,     a.qk_heads,
                       a.v_heads,  qkv_dim,      a.prepped ? 1 : 0,       a.eps,
                       a.wait_ns ? a.wait_ns : kWaitTimeoutNs};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(std::min(a.batch * a.v_heads, a.sm_count));
        cfg.blockDim = dim3(kSweepThreads);
        cfg.dynamicSmemBytes = sizeof(SweepSmem);
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, linear_decode_sweep_kernel, sp);
    }
    if (!a.prepped) {
        PrepParams pp{a.qkv,    a.beta,    a.alpha,     a.conv_state, a.conv_w, a.dt_bias,
                      a.ssm_a,  a.qk_heads, a.v_heads,  qkv_dim,      a.eps};
        linear_decode_prep_kernel<<<dim3(2 * a.qk_heads + a.v_heads, a.batch), kPrepThreads, 0,
                                    stream>>>(pp);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    // With prep_done recorded between the two kernels, D2 is an ordinary
    // launch (no programmatic overlap across the record).
    if (prep_done && (e = cudaEventRecord(prep_done, stream)) != cudaSuccess) return e;

    // Prepped inputs (conv, SiLU and gates applied by the projections): the
    // state kernel normalises q and k itself and follows the last projection
    // as its programmatic dependent.
    StateParams sp{a.qkv,      a.z,        a.beta,    a.alpha,   a.delta_state,
                   a.ssm_norm, a.attention, a.qk_heads, a.v_heads, qkv_dim,
                   a.prepped ? 1 : 0,       a.eps};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.v_heads, a.batch);
    cfg.blockDim = dim3(kStateThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = prep_done ? 0 : 1;
    return cudaLaunchKernelEx(&cfg, linear_decode_state_kernel, sp);
}

}  // namespace q38
