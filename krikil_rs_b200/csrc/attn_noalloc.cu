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
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_attn_scratch on the current device.  The array's name in
// host code is only a host-side handle, so the address is looked up once per
// device with that device current, and cached.
int scratch_for_current_device(float** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return krk::report_error(KRK_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return krk::report_error(KRK_INVALID, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p)
            return krk::report_error(KRK_CUDA,
                                     std::string("cudaGetSymbolAddress(attention scratch): ") + cudaGetErrorString(e));
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_ptr[dev];
    return KRK_OK;
}

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
    float* scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
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
