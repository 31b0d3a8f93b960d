// RMSNorm family, embedding gather and pointwise ops (fp32).
#include "common.cuh"
#include "kernels.h"

namespace krk {

// ---------------------------------------------------------------------------
// Launch bookkeeping shared by every launcher of the library.
// ---------------------------------------------------------------------------
static unsigned long long g_launches = 0;
uint64_t launch_count() { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }
void add_launches(uint64_t n) { __atomic_fetch_add(&g_launches, (unsigned long long)n, __ATOMIC_RELAXED); }

static thread_local bool t_pdl = false;
bool pdl_enabled() { return t_pdl; }
PdlScope::PdlScope(bool on) : prev_(t_pdl) { t_pdl = on; }
PdlScope::~PdlScope() { t_pdl = prev_; }

static thread_local int t_priority = 0;
int launch_priority() { return t_priority; }
PriorityScope::PriorityScope(int priority) : prev_(t_priority) { t_priority = priority; }
PriorityScope::~PriorityScope() { t_priority = prev_; }

cudaError_t DeviceOnce::set_smem(const void* func, size_t bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    unsigned long long bit = 1ull << (dev & 63);
    if (__atomic_load_n(&mask, __ATOMIC_ACQUIRE) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) __atomic_fetch_or(&mask, bit, __ATOMIC_RELEASE);
    else cudaGetLastError();  // reported here: not again by a later launch's error check
    return e;
}

namespace {

// ---------------------------------------------------------------------------
// Feature-major RMSNorm: out[k][m] = x[k][m] * scale(m) * w[k].
//
// One CTA owns 8 columns (sequences).  The [K][8] column block is staged into
// shared memory with cp.async; then each column's sum of squares
// (src/math.rs:45-48) is formed as 32 partials -- partial p adds x[k][c]^2 for
// k = p, p + 32, ... in order -- folded by warp shuffles and then across the
// eight warps in warp order, and all threads write the normalised block
// (x * scale) * w (src/math.rs:51-53).  The sum is
// the reference's up to the order of its additions (the reference adds the
// squares one after the other), so results agree within rounding; the order
// is fixed, so they do not depend on the batch, the part or the CTA.  K <= 1216.
// ---------------------------------------------------------------------------
constexpr int NORM_COLS = 8;
constexpr int NORM_MAXK = 1216;
constexpr int NORM_WS_MAX_COLS = 128;  // up to this many columns the weights are staged

// WS (few columns, where the kernel's latency is the whole cost): the weights
// are staged in shared memory while the column block is in flight, instead of
// one global read per written element.
template <bool WS>
__global__ void __launch_bounds__(256) rmsnorm_fm_kernel(const float* __restrict__ x, int ldx,
                                                         const float* __restrict__ w, float eps, int K, int M,
                                                         float* __restrict__ out, int ldo) {
    extern __shared__ __align__(16) float blk[];  // [K][NORM_COLS], then (WS) w [K]
    __shared__ __align__(16) float scale_s[NORM_COLS];
    __shared__ float part_s[8 * NORM_COLS];  // [warp][column] partial sums of squares
    float* ws = blk + (size_t)K * NORM_COLS;
    const int tid = threadIdx.x;
    const int m0 = blockIdx.x * NORM_COLS;
    const int ncols = min(NORM_COLS, M - m0);
    // The whole 8-column block is copied whenever it lies inside the rows (a
    // padded batch: columns past M are read, their sums unused, and never
    // written), so a partial block takes the copy path too.
    const bool full = (m0 + NORM_COLS <= ldx) && ((ldx & 3) == 0) && ((((uintptr_t)x) & 15) == 0);
    // the weights travel with the block when both are 16-byte pieces
    const bool wasync = WS && (K & 3) == 0 && (((uintptr_t)w) & 15) == 0;
    if (wasync) {  // the weights first: x comes from the kernels before this one
        for (int i = tid; i < K / 4; i += 256) cp_async16(ws + 4 * i, w + 4 * i);
    } else if (WS) {
        for (int k = tid; k < K; k += 256) ws[k] = w[k];
    }
    pdl_wait();
    pdl_trigger();
    if (full) {
        for (int i = tid; i < K * (NORM_COLS / 4); i += 256) {
            const int k = i / (NORM_COLS / 4), c4 = i % (NORM_COLS / 4);
            cp_async16(blk + k * NORM_COLS + c4 * 4, x + (size_t)k * ldx + m0 + c4 * 4);
        }
    } else {
        for (int i = tid; i < K * NORM_COLS; i += 256) {
            int k = i / NORM_COLS, c = i % NORM_COLS;
            blk[i] = c < ncols ? x[(size_t)k * ldx + m0 + c] : 0.0f;
        }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();  // the block is visible to every warp
    {
        // thread t sums column t % 8 over rows k = t / 8 (mod 32): each warp
        // load is 4 whole rows (32 consecutive words, no bank conflict)
        static_assert(NORM_COLS == 8, "8 columns per CTA");
        const int col = tid & 7, lane = tid & 31, warp = tid >> 5;
        float ss = 0.0f;
        for (int k = tid >> 3; k < K; k += 32) {
            const float v = blk[k * NORM_COLS + col];
            ss += v * v;
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 8);  // the warp's 4 lanes of this column
        ss += __shfl_xor_sync(0xffffffffu, ss, 16);
        if (lane < NORM_COLS) part_s[warp * NORM_COLS + lane] = ss;
        __syncthreads();
        if (tid < NORM_COLS) {
            float t = part_s[tid];
            for (int w8 = 1; w8 < 8; ++w8) t += part_s[w8 * NORM_COLS + tid];
            scale_s[tid] = 1.0f / sqrtf(t / (float)K + eps);
        }
    }
    __syncthreads();
    const bool vec = ncols == NORM_COLS && (ldo & 3) == 0 && (((uintptr_t)out) & 15) == 0;
    if (vec) {  // thread t writes columns 4(t%2) .. 4(t%2)+3 of rows t/2, t/2 + 128, ...
        const int c4 = (tid & 1) * 4;
        const float4 sc = *reinterpret_cast<const float4*>(scale_s + c4);
        for (int k = tid >> 1; k < K; k += 128) {
            const float4 v = *reinterpret_cast<const float4*>(blk + k * NORM_COLS + c4);
            const float wk = WS ? ws[k] : w[k];
            *reinterpret_cast<float4*>(out + (size_t)k * ldo + m0 + c4) =
                make_float4(v.x * sc.x * wk, v.y * sc.y * wk, v.z * sc.z * wk, v.w * sc.w * wk);
        }
    } else {
        const int c = tid % NORM_COLS;
        if (c < ncols) {
            const float sc = scale_s[c];
            for (int k = tid / NORM_COLS; k < K; k += 256 / NORM_COLS)
                out[(size_t)k * ldo + m0 + c] = blk[k * NORM_COLS + c] * sc * (WS ? ws[k] : w[k]);
        }
    }
}

// ---------------------------------------------------------------------------
// Row-major RMSNorm and the fused gated RMSNorm + residual: one warp per row,
// the row held in registers as float4s (VPL float4 per lane, dim = 128*VPL).
// The sum of squares is per-lane sequential then a warp tree.
// ---------------------------------------------------------------------------
template <int VPL, bool GATED>
__global__ void __launch_bounds__(256, VPL <= 4 ? 4 : 1) rownorm_kernel(const float* __restrict__ x, const float* __restrict__ z,
                                                      const float* __restrict__ res, const float* __restrict__ w,
                                                      float eps, int64_t rows, float* __restrict__ y) {
    constexpr int DIM = 128 * VPL;
    const int lane = threadIdx.x & 31;
    const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp_global; r < rows; r += nwarps) {
        const float4* xr = reinterpret_cast<const float4*>(x + r * DIM);
        float4 g[VPL], rr[VPL];
#pragma unroll
        for (int i = 0; i < VPL; ++i) g[i] = __ldcs(xr + lane + 32 * i);
        if (GATED) {
            const float4* zr = reinterpret_cast<const float4*>(z + r * DIM);
            float4 zz[VPL];
#pragma unroll
            for (int i = 0; i < VPL; ++i) zz[i] = __ldcs(zr + lane + 32 * i);
            // y *= silu(z) (src/model.rs:688-690)
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                g[i].x = g[i].x * silu(zz[i].x);
                g[i].y = g[i].y * silu(zz[i].y);
                g[i].z = g[i].z * silu(zz[i].z);
                g[i].w = g[i].w * silu(zz[i].w);
            }
        }
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            ss += g[i].x * g[i].x;
            ss += g[i].y * g[i].y;
            ss += g[i].z * g[i].z;
            ss += g[i].w * g[i].w;
        }
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / (float)DIM + eps);
        if (GATED) {  // the residual row, read once the squares are summed
            const float4* rs = reinterpret_cast<const float4*>(res + r * DIM);
#pragma unroll
            for (int i = 0; i < VPL; ++i) rr[i] = __ldcs(rs + lane + 32 * i);
        }
        float4* yr = reinterpret_cast<float4*>(y + r * DIM);
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + lane + 32 * i);  // L1-resident
            float4 o;
            o.x = g[i].x * scale * wv.x;
            o.y = g[i].y * scale * wv.y;
            o.z = g[i].z * scale * wv.z;
            o.w = g[i].w * scale * wv.w;
            if (GATED) {
                o.x = o.x + rr[i].x;
                o.y = o.y + rr[i].y;
                o.z = o.z + rr[i].z;
                o.w = o.w + rr[i].w;
            }
            __stcs(yr + lane + 32 * i, o);
        }
    }
}

template <bool GATED>
cudaError_t launch_rownorm(const float* x, const float* z, const float* res, const float* w, float eps,
                           int64_t rows, int dim, float* y, cudaStream_t s) {
    if (rows <= 0 || dim % 128 || dim > 1024 || ((uintptr_t)x | (uintptr_t)y | (uintptr_t)w) % 16 ||
        (GATED && ((uintptr_t)z | (uintptr_t)res) % 16))
        return cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // At most one wave of resident CTAs whose warps stride over the rows, as
    // few as give every warp the same number of rows (no partly idle last pass).
    auto grid_for = [&](const void* fn) {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 256, 0) != cudaSuccess || per_sm < 1) per_sm = 1;
        const int64_t cap = (int64_t)sms * per_sm;           // CTAs of 8 warps
        const int64_t per_warp = (rows + cap * 8 - 1) / (cap * 8);
        const int64_t ctas = (rows + per_warp * 8 - 1) / (per_warp * 8);
        return (int)(ctas < cap ? ctas : cap);
    };
    switch (dim / 128) {
#define KRK_CASE(V)                                                                                 \
    case V:                                                                                         \
        rownorm_kernel<V, GATED><<<grid_for((const void*)rownorm_kernel<V, GATED>), 256, 0, s>>>( \
            x, z, res, w, eps, rows, y);                                                            \
        break;
        KRK_CASE(1) KRK_CASE(2) KRK_CASE(3) KRK_CASE(4) KRK_CASE(5) KRK_CASE(6) KRK_CASE(7) KRK_CASE(8)
#undef KRK_CASE
        default: return cudaErrorInvalidValue;
    }
    add_launches(1);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Embedding gather (src/model.rs:336-337, :598) into feature-major layout,
// transposed through a 32x32 shared tile.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) embed_fm_kernel(const uint32_t* __restrict__ tok,
                                                       const float* __restrict__ wte, int vocab, int K, int M,
                                                       float* __restrict__ out, int ldo) {
    __shared__ float tile[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int m0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    pdl_wait();  // the tokens come from the kernels before this one
    pdl_trigger();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int m = m0 + ty + 8 * i, k = k0 + tx;
        uint32_t t = m < M ? tok[m] : 0u;
        if (kChecked && m < M && k == 0 && t >= (uint32_t)vocab) check_fail(CHK_TOKEN);
        tile[ty + 8 * i][tx] = (m < M && k < K && t < (uint32_t)vocab) ? wte[(size_t)t * K + k] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int k = k0 + ty + 8 * i, m = m0 + tx;
        if (m < M && k < K) out[(size_t)k * ldo + m] = tile[tx][ty + 8 * i];
    }
}

__global__ void pointwise_kernel(int op, const float* __restrict__ x, float* __restrict__ y, int64_t n) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = x[i];
    y[i] = op == 0 ? silu(v) : (op == 1 ? softplus(v) : gelu(v));
}

}  // namespace

cudaError_t rmsnorm_fm(const float* x, int ldx, const float* w, float eps, int K, int M, float* out, int ldo,
                       cudaStream_t s) {
    if (K <= 0 || M <= 0 || K > NORM_MAXK || ldx < M || ldo < M) return cudaErrorInvalidValue;
    const bool ws = M <= NORM_WS_MAX_COLS;
    static DeviceOnce once[2];
    const size_t smem = (size_t)K * (NORM_COLS + (ws ? 1 : 0)) * sizeof(float);
    const void* fn = ws ? (const void*)rmsnorm_fm_kernel<true> : (const void*)rmsnorm_fm_kernel<false>;
    cudaError_t e = once[ws ? 1 : 0].set_smem(fn, (size_t)NORM_MAXK * (NORM_COLS + 1) * sizeof(float));
    if (e != cudaSuccess) return e;
    e = launch_pdl(ws ? rmsnorm_fm_kernel<true> : rmsnorm_fm_kernel<false>, dim3((M + NORM_COLS - 1) / NORM_COLS),
                   dim3(256), smem, s, x, ldx, w, eps, K, M, out, ldo);
    if (e != cudaSuccess) return e;
    add_launches(1);
    return cudaGetLastError();
}

cudaError_t rmsnorm_rows(const float* x, const float* w, float eps, int64_t rows, int dim, float* y, cudaStream_t s) {
    return launch_rownorm<false>(x, nullptr, nullptr, w, eps, rows, dim, y, s);
}

cudaError_t gated_rmsnorm_residual(const float* x, const float* z, const float* res, const float* w, float eps,
                                   int64_t rows, int dim, float* y, cudaStream_t s) {
    return launch_rownorm<true>(x, z, res, w, eps, rows, dim, y, s);
}

cudaError_t embed_fm(const uint32_t* tok, const float* wte, int vocab, int K, int M, float* out, int ldo,
                     cudaStream_t s) {
    if (K <= 0 || M <= 0 || ldo < M) return cudaErrorInvalidValue;
    dim3 grid((M + 31) / 32, (K + 31) / 32);
    const cudaError_t e = launch_pdl(embed_fm_kernel, grid, dim3(256), 0, s, tok, wte, vocab, K, M, out, ldo);
    if (e != cudaSuccess) return e;
    add_launches(1);
    return cudaGetLastError();
}

cudaError_t pointwise(int op, const float* x, float* y, int64_t n, cudaStream_t s) {
    if (n <= 0 || op < 0 || op > 2) return cudaErrorInvalidValue;
    pointwise_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(op, x, y, n);
    add_launches(1);
    return cudaGetLastError();
}

}  // namespace krk
