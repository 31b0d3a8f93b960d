// Shared device helpers for the krikil B200 kernels (fp32 throughout).
//
// Every kernel in this library is compiled with --fmad=false, so a*b+c is a
// rounded multiply followed by a rounded add, exactly as the reference's Rust
// code evaluates it; fused multiply-adds appear only where written as fmaf().
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define KRK_DEV __device__ __forceinline__

namespace krk {

// src/math.rs:3-6
KRK_DEV float silu(float x) { return x / (1.0f + expf(-x)); }

// src/math.rs:8-15
KRK_DEV float softplus(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

// src/math.rs:23-39: erf by Abramowitz & Stegun formula 7.1.26 (the published
// five-term polynomial in t = 1/(1+p|x|) times exp(-x^2)).
KRK_DEV float as_erf(float x) {
    const float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f;
    const float a4 = -1.453152027f, a5 = 1.061405429f, p = 0.3275911f;
    float sign = x < 0.0f ? -1.0f : 1.0f;
    float ax = fabsf(x);
    float t = 1.0f / (1.0f + p * ax);
    float poly = ((((a5 * t + a4) * t) + a3) * t + a2) * t + a1;
    return sign * (1.0f - poly * t * expf(-ax * ax));
}

// src/math.rs:17-21 (FRAC_1_SQRT_2 as an f32 constant)
KRK_DEV float gelu(float x) { return 0.5f * x * (1.0f + as_erf(x * 0.70710678118654752f)); }

// Programmatic dependent launch (sm_90+): a kernel launched with programmatic
// stream serialization may be scheduled once every block of the kernel before
// it has called pdl_trigger() (or exited); pdl_wait() then blocks until that
// kernel has completed and its writes are visible.  Both are no-ops for
// kernels launched without the attribute.
KRK_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
KRK_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

bool pdl_enabled();     // a PdlScope(true) is alive on this thread (kernels.h)
int launch_priority();  // a PriorityScope's priority, or 0 (kernels.h)

// kern<<<grid, block, smem, s>>>(args...), with programmatic stream
// serialization while pdl_enabled() and the launch priority of a live
// PriorityScope.  Only for kernels that call pdl_wait() in every block before
// they touch memory other than weights.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    unsigned na = 0;
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (const int prio = launch_priority()) {
        attr[na].id = cudaLaunchAttributePriority;
        attr[na].val.priority = prio;
        ++na;
    }
    cfg.attrs = na ? attr : nullptr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

KRK_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

KRK_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 16-byte global->shared asynchronous copy (bypasses L1).
KRK_DEV void cp_async16(void* smem, const void* gmem) {
    unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
KRK_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
KRK_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---- bulk (TMA engine) copies completing on a shared-memory mbarrier -------
KRK_DEV uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
KRK_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the bulk-copy engine.
KRK_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
// One arrival that also announces `bytes` of bulk-copy data for the phase.
KRK_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte
// aligned) that completes on `bar`.  No multicast.
KRK_DEV void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
KRK_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for phase `parity` of `bar` for at most `limit` polls (each poll may
// suspend the thread for a short hardware-defined time); false on timeout.
KRK_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int limit) {
    for (int i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// ---- checked builds ---------------------------------------------------------
// Compiled with -DKRIKIL_CHECKED (make CHECKED=1), kernels test the
// preconditions on device data that the host cannot see before a launch --
// token ids, sequence positions, table entries read on the device -- and where
// one fails they set a bit of their translation unit's device status word and
// skip the access instead of making it; krk_check_status() reads the words,
// and the model API's calls turn a set bit into KRK_CHECK_FAILED.  No trap and
// no assert: the kernel carries on or returns, and the context stays usable.
// In other builds the checks compile to nothing (the guards every build has
// stay as they are).
enum CheckBits : unsigned {
    CHK_TOKEN = 1u,     // a token id >= vocab reached a kernel
    CHK_POSITION = 2u,  // a sequence position outside [0, ctx), or past the launch's key bound
    CHK_TABLE = 4u,     // a prefill table entry outside its sequence or its key bound
    CHK_COLUMN = 8u,    // a gather column outside its matrix
};
#ifdef KRIKIL_CHECKED
constexpr bool kChecked = true;
#else
constexpr bool kChecked = false;
#endif
// Registers a translation unit's reader of its status word (defined in capi.cu).
void register_check_word(unsigned (*read)(bool clear));

namespace {
#ifdef KRIKIL_CHECKED
__device__ unsigned g_check_word;  // one per translation unit (each is its own device module)
KRK_DEV void check_fail(unsigned bit) { atomicOr(&g_check_word, bit); }
unsigned read_check_word(bool clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_check_word, sizeof v) != cudaSuccess) {
        cudaGetLastError();  // leave no error behind for an unrelated later check
        return 0;
    }
    if (clear && v) {
        const unsigned z = 0;
        if (cudaMemcpyToSymbol(g_check_word, &z, sizeof z) != cudaSuccess) cudaGetLastError();
    }
    return v;
}
const bool g_check_word_registered = (register_check_word(&read_check_word), true);
#else
KRK_DEV void check_fail(unsigned) {}
#endif
}  // namespace

}  // namespace krk
