// Decode attention for callers that cannot allocate device memory.
//
// krk_k_rope_kv_attn_decode needs a caller-provided scratch buffer (`work`) for
// the per-split softmax partials whenever a sequence's cache spans more than one
// split.  Some callers have no way to provide one: a host that binds only this C
// header and links no CUDA allocator of its own (for example a Rust or C program
// that owns no device-memory API), or a process whose device memory is entirely
// owned by another allocator or a fixed budget that forbids extra cudaMalloc
// calls.  krk_k_rope_kv_attn_decode_noalloc serves them with a fixed scratch
// array that is part of this library's device image instead of a buffer.
//
// The array below holds KRK_ATTN_NOALLOC_MAX_FLOATS floats (4 MiB).  Every GPU
// that loads this library's device code keeps it until the process exits.  All
// calls on a GPU share it, so calls that overlap on that GPU (concurrent
// streams, or several host threads) race on it; the caller must serialise them.
// Nothing in it has to start at zero: every partial that the combine step reads
// is written earlier in the same call, and the array keeps whatever the last
// call left in it.
//
// The call runs on the device that owns `stream` (the current device for the
// default stream) and leaves the caller's current device as it was.  The
// array's device address is looked up on the first call on each device (that
// first call should come before any stream capture) and kept for later calls
// in the same CUDA context of that device; after a device reset the next call
// looks it up again in the new context.
#include <cuda.h>  // driver types only (CUcontext, CUresult); the entry points come from the runtime
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/krikil_cuda.h"
#include "kernels.h"

namespace krk {
int report_error(int status, const std::string& msg);  // capi.cu: sets krk_last_error()
}

namespace {

static __device__ __align__(256) float g_attn_scratch[KRK_ATTN_NOALLOC_MAX_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct Cached {
    unsigned long long ctx_id = 0;  // 0: not looked up yet
    float* ptr = nullptr;
};
Cached g_scratch[kMaxDevices];

// Unique id of the calling thread's current CUDA context (the device's primary
// context once the runtime has used it); 0 if it cannot be read.  Context ids
// are never reused within a process, so a reset device shows a new id.
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(f);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// Device address of g_attn_scratch on the current device `dev`.  The array's
// name in host code is only a host-side handle, so the address is looked up
// with that device current, and cached per device and context.
int scratch_for_device(int dev, float** out) {
    if (dev < 0 || dev >= kMaxDevices) return krk::report_error(KRK_INVALID, "device ordinal out of range");
    // binds the device's primary context to this thread (initialising it if
    // needed), so that its id can be read; allocates nothing
    cudaError_t e = cudaSetDevice(dev);
    if (e != cudaSuccess) return krk::report_error(KRK_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    const unsigned long long id = current_context_id();
    std::lock_guard<std::mutex> lock(g_mu);
    Cached& c = g_scratch[dev];
    if (id == 0 || c.ctx_id != id || !c.ptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p)
            return krk::report_error(KRK_CUDA,
                                     std::string("cudaGetSymbolAddress(attention scratch): ") + cudaGetErrorString(e));
        c.ptr = static_cast<float*>(p);
        c.ctx_id = id;  // id 0 (unreadable): looked up again on every call
    }
    *out = c.ptr;
    return KRK_OK;
}

// Makes `dev` current for the scope and restores the caller's device after.
struct OnDevice {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit OnDevice(int dev) {
        err = cudaGetDevice(&prev);
        if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
    }
    ~OnDevice() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" int krk_k_rope_kv_attn_decode_noalloc(const float* q, const float* k, const float* v, float* kc,
                                                 float* vc, const int32_t* pos, float* out, int B, int H, int dh,
                                                 int ctx, int split, float theta, void* stream) {
    if (split <= 0) split = 256;
    if (B <= 0 || H <= 0 || dh <= 0 || ctx <= 0)
        return krk::report_error(KRK_INVALID, "B, H, dh and ctx must be positive");
    const size_t need = krk::attn_decode_work_floats(B, H, dh, ctx, split);
    const bool multi_split = ctx > split;
    if (multi_split && need > (size_t)KRK_ATTN_NOALLOC_MAX_FLOATS)
        return krk::report_error(
            KRK_INVALID, "attention needs " + std::to_string(need) + " floats of scratch but the fixed scratch holds " +
                             std::to_string((size_t)KRK_ATTN_NOALLOC_MAX_FLOATS) +
                             "; use a larger split, fewer sequences per call, or krk_k_rope_kv_attn_decode with a "
                             "caller-provided buffer");
    int dev = -1;
    cudaError_t se = cudaStreamGetDevice((cudaStream_t)stream, &dev);
    if (se != cudaSuccess)
        return krk::report_error(KRK_INVALID, std::string("stream's device: ") + cudaGetErrorString(se));
    OnDevice on(dev);
    if (on.err != cudaSuccess)
        return krk::report_error(KRK_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(on.err));
    float* scratch = nullptr;
    int rc = scratch_for_device(dev, &scratch);
    if (rc != KRK_OK) return rc;
    krk::AttnDecodeArgs a{};
    a.q = q; a.k = k; a.v = v; a.in_sb = (int64_t)H * dh; a.in_sh = dh;
    a.kc = kc; a.vc = vc; a.c_sb = (int64_t)H * ctx * dh; a.c_sh = (int64_t)ctx * dh; a.c_st = dh;
    a.pos = pos; a.active = nullptr;
    a.out = out; a.o_sb = (int64_t)H * dh; a.o_sh = dh; a.o_sd = 1;
    a.work = scratch;
    a.B = B; a.H = H; a.dh = dh; a.ctx = ctx; a.split = split; a.theta = theta;
    cudaError_t e = krk::attn_decode(a, (cudaStream_t)stream);
    if (e == cudaSuccess) return KRK_OK;
    return krk::report_error(e == cudaErrorInvalidValue ? KRK_INVALID : KRK_CUDA,
                             std::string("rope_kv_attn_decode_noalloc: ") + cudaGetErrorString(e));
}
