// attn_decode_noalloc.cu -- q38_full_decode_noalloc: the full-attention decode
// step for callers that cannot allocate device memory.
//
// Who needs it: a host that owns all of the GPU's memory itself -- a serving
// engine that reserves HBM up front for its own KV-block pool and hands out
// every byte through its own arena, or an FFI caller whose allocator must see
// every device buffer -- cannot let a library call cudaMalloc: the call may
// fail once the pool holds the memory, it may synchronise the device and stall
// the caller's other streams, and it creates memory the caller cannot account
// for. Such a caller already owns the step's inputs, outputs and KV cache;
// the only memory the decode kernels need beyond those is their split-KV
// scratch (prepared queries and the per-split (m, l, o) partials). Here that
// scratch is a fixed, file-scope device array, so the entry point allocates
// nothing.
//
// The array holds kNoAllocScratchBytes (16 MiB) on every GPU whose context
// loads this library's device code, until the process exits. Under CUDA's
// default lazy module loading that happens at the first call on the device
// (the address lookup below loads the module), so a caller that reserves all
// free HBM for its own pool must make one call before reserving it. Every
// call on a device shares the array and it keeps the last call's contents;
// nothing in it needs to start at zero, because each word a call reads was
// written earlier in the same call. Calls whose executions overlap on the GPU
// (different streams, or different host threads without ordering) race on
// the array and corrupt each other's results: order them. The looked-up
// address is kept per device for the life of the process; a cudaDeviceReset
// invalidates it, so a caller that resets a device must not call this entry
// point on that device afterwards.
#include "q38_common.cuh"

#include <cmath>
#include <cstdio>
#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

// The scratch itself. Host code must not pass this name to a kernel: on the
// host it is only a stand-in symbol, not a device address. The device address
// comes from cudaGetSymbolAddress, once per device (scratch_on_device).
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 128;
std::mutex g_setup_mu;
void *g_scratch_addr[kMaxDevices] = {};

// Device address of g_decode_scratch on `device` (the current device),
// looked up on the first call per device and cached.
cudaError_t scratch_on_device(int device, void **addr) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[device] = p;
    }
    *addr = g_scratch_addr[device];
    return cudaSuccess;
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

struct ScratchLayout {
    size_t qprep = 0, part_o = 0, part_ml = 0, total = 0;
};

ScratchLayout layout_for(int batch, int heads, int nsplit) {
    ScratchLayout l;
    l.qprep = 0;
    l.part_o = align256(size_t(batch) * heads * q38::kAttnHeadDim * 4);
    l.part_ml = l.part_o + align256(size_t(batch) * heads * nsplit * q38::kAttnHeadDim * 4);
    l.total = l.part_ml + align256(size_t(batch) * heads * nsplit * 2 * 4);
    return l;
}

}  // namespace

extern "C" int q38_full_decode_noalloc(const float *q_norm, const float *k_norm, void *key_cache,
                                       void *value_cache, int batch, int context_length,
                                       int kv_dtype, const float *q_and_gate, float *key,
                                       const float *value, const int32_t *positions,
                                       int max_position, float *attention, int *error_bits,
                                       void *stream) {
    auto reject = [](int code, const char *msg) {
        q38::record_error(msg);
        return code;
    };
    if (!q_norm || !k_norm || !key_cache || !value_cache || !q_and_gate || !key || !value ||
        !positions || !attention)
        return reject(Q38_ERR_ARG, "null pointer argument");
    if (batch <= 0 || context_length <= 0)
        return reject(Q38_ERR_ARG, "batch and context_length must be positive");
    if (kv_dtype != Q38_KV_F32 && kv_dtype != Q38_KV_BF16)
        return reject(Q38_ERR_ARG, "kv_dtype must be Q38_KV_F32 or Q38_KV_BF16");
    if (max_position < 0) max_position = context_length - 1;
    if (max_position >= context_length)
        return reject(Q38_ERR_ARG, "max_position must be below context_length");
    // The split kernel streams the caller's KV cache with the bulk-copy engine
    // (f32) or by TMA (bf16); both need 16-byte aligned rows. Every other
    // buffer is read and written as 4-byte words.
    auto addr = [](const void *p) { return reinterpret_cast<uintptr_t>(p); };
    if ((addr(key_cache) | addr(value_cache)) & 15u)
        return reject(Q38_ERR_ARG, "key_cache and value_cache must be 16-byte aligned");
    if ((addr(q_norm) | addr(k_norm) | addr(q_and_gate) | addr(key) | addr(value) |
         addr(positions) | addr(attention) | addr(error_bits)) & 3u)
        return reject(Q38_ERR_ARG, "tensor arguments must be 4-byte aligned");

    int device = 0, sms = 0, major = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) {
        cudaGetLastError();
        return reject(Q38_ERR_CUDA, "cannot query the current CUDA device");
    }
    if (major != 10) return reject(Q38_ERR_ARG, "the current device is not an sm_100 GPU");

    // Reference geometry (src/model/mod.rs:20-24): 24 query heads, 4 KV heads.
    const int heads = 24, kv_heads = 4;
    // Pick the split plan of the regular entry point; if its partials do not
    // fit the fixed scratch, ask the planner for fewer splits (larger chunks).
    int plan_sms = sms;
    q38::DecodeSplitPlan plan{};
    ScratchLayout lay{};
    for (;;) {
        plan = q38::plan_attn_decode(batch, kv_heads, max_position, kv_dtype, plan_sms);
        lay = layout_for(batch, heads, plan.nsplit);
        if (lay.total <= kNoAllocScratchBytes || plan_sms == 1) break;
        plan_sms = plan_sms > 1 ? plan_sms / 2 : 1;
    }
    if (lay.total > kNoAllocScratchBytes) {
        char msg[256];
        std::snprintf(msg, sizeof msg,
                      "batch %d at %d positions needs %zu bytes of decode scratch; the "
                      "no-allocation entry point holds at most %zu",
                      batch, max_position + 1, lay.total, kNoAllocScratchBytes);
        return reject(Q38_ERR_ARG, msg);
    }

    void *base = nullptr;
    if (const cudaError_t e = scratch_on_device(device, &base); e != cudaSuccess) {
        cudaGetLastError();
        char msg[256];
        std::snprintf(msg, sizeof msg, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        return reject(Q38_ERR_CUDA, msg);
    }
    unsigned char *s = static_cast<unsigned char *>(base);

    q38::AttnDecodeLaunch a{};
    a.q_and_gate = q_and_gate;
    a.key = key;
    a.value = value;
    a.positions = positions;
    a.attention = attention;
    a.kcache = key_cache;
    a.vcache = value_cache;
    a.qprep = reinterpret_cast<float *>(s + lay.qprep);
    a.part_o = reinterpret_cast<float *>(s + lay.part_o);
    a.part_ml = reinterpret_cast<float *>(s + lay.part_ml);
    a.err = error_bits;
    a.q_norm = q_norm;
    a.k_norm = k_norm;
    a.batch = batch;
    a.context_length = context_length;
    a.heads = heads;
    a.kv_heads = kv_heads;
    a.kv_dtype = kv_dtype;
    a.max_position = max_position;
    a.max_splits = plan.nsplit;
    a.theta_scale = std::pow(10000000.0f, -2.0f / 64.0f);  // rope(), ops.rs:596
    a.eps = 1e-6f;
    const cudaError_t e = q38::launch_attn_decode(a, plan_sms, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        cudaGetLastError();
        char msg[256];
        std::snprintf(msg, sizeof msg, "no-allocation decode launch: %s", cudaGetErrorString(e));
        return reject(Q38_ERR_CUDA, msg);
    }
    return Q38_OK;
}
