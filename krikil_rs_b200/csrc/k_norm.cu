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

cudaError_t DeviceOnce::set_smem(const void* func, size_t bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    unsigned long long bit = 1ull << (dev & 63);
    if (__atomic_load_n(&mask, __ATOMIC_ACQUIRE) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) __atomic_fetch_or(&mask, bit, __ATOMIC_RELEASE);
    return e;
}

namespace {

// ---------------------------------------------------------------------------
// Feature-major RMSNorm: out[k][m] = x[k][m] * scale(m) * w[k].
//
// One CTA owns 8 columns (sequences).  The [K][8] column block is staged into
// shared memory with cp.async in NORM_CHUNKS row chunks (each its own commit
// group), and thread m forms column m's sum of squares in exactly the
// reference's order -- x[k][m]^2 added for k = 0..K-1 one after the other
// (src/math.rs:45-48), a latency-bound chain, hence few columns per CTA and
// many CTAs -- chunk by chunk as the chunks land, so the chain overlaps the
// loads.  Then all threads write the normalised block (x * scale) * w
// (src/math.rs:51-53).  K <= 1216.
// ---------------------------------------------------------------------------
constexpr int NORM_COLS = 8;
constexpr int NORM_MAXK = 1216;
constexpr int NORM_CHUNKS = 8;
constexpr int NORM_WS_MAX_COLS = 128;  // up to this many columns the weights are staged

// cp.async.wait_group with a run-time count n in [0, NORM_CHUNKS).
KRK_DEV void cp_async_wait_upto(int n) {
    switch (n) {
        case 0: cp_async_wait<0>(); break;
        case 1: cp_async_wait<1>(); break;
        case 2: cp_async_wait<2>(); break;
        case 3: cp_async_wait<3>(); break;
        case 4: cp_async_wait<4>(); break;
        case 5: cp_async_wait<5>(); break;
        case 6: cp_async_wait<6>(); break;
        default: cp_async_wait<7>(); break;
    }
}

// WS (few columns, where the kernel's latency is the whole cost): the weights
// are staged in shared memory while the column block is in flight, instead of
// one global read per written element.
template <bool WS>
__global__ void __launch_bounds__(256) rmsnorm_fm_kernel(const float* __restrict__ x, int ldx,
                                                         const float* __restrict__ w, float eps, int K, int M,
                                                         float* __restrict__ out, int ldo) {
    extern __shared__ __align__(16) float blk[];  // [K][NORM_COLS], then (WS) w [K]
    __shared__ float scale_s[NORM_COLS];
    float* ws = blk + (size_t)K * NORM_COLS;
    const int tid = threadIdx.x;
    const int m0 = blockIdx.x * NORM_COLS;
    const int ncols = min(NORM_COLS, M - m0);
    const bool full = (ncols == NORM_COLS) && ((ldx & 3) == 0) && ((((uintptr_t)x) & 15) == 0);
    const int kc = (K + NORM_CHUNKS - 1) / NORM_CHUNKS;  // rows per chunk
    if (full) {
        for (int c = 0; c < NORM_CHUNKS; ++c) {
            const int k0 = c * kc, nk = max(0, min(K, k0 + kc) - k0);
            for (int i = tid; i < nk * (NORM_COLS / 4); i += 256) {
                const int k = k0 + i / (NORM_COLS / 4), c4 = i % (NORM_COLS / 4);
                cp_async16(blk + k * NORM_COLS + c4 * 4, x + (size_t)k * ldx + m0 + c4 * 4);
            }
            cp_async_commit();
        }
    } else {
        for (int i = tid; i < K * NORM_COLS; i += 256) {
            int k = i / NORM_COLS, c = i % NORM_COLS;
            blk[i] = c < ncols ? x[(size_t)k * ldx + m0 + c] : 0.0f;
        }
    }
    if (WS)
        for (int k = tid; k < K; k += 256) ws[k] = w[k];
    float ss = 0.0f;
    for (int c = 0; c < NORM_CHUNKS; ++c) {
        if (full) cp_async_wait_upto(NORM_CHUNKS - 1 - c);
        __syncthreads();  // chunk c visible to the summing threads
        if (tid < NORM_COLS) {
            const int k1 = min(K, (c + 1) * kc);
#pragma unroll 8
            for (int k = c * kc; k < k1; ++k) {
                const float v = blk[k * NORM_COLS + tid];
                ss += v * v;
            }
        }
    }
    if (tid < NORM_COLS) {
        float mean = ss / (float)K;
        scale_s[tid] = 1.0f / sqrtf(mean + eps);
    }
    __syncthreads();
    const int c = tid % NORM_COLS;
    if (c < ncols) {
        const float sc = scale_s[c];
        if (WS) {
#pragma unroll 4
            for (int k = tid / NORM_COLS; k < K; k += 256 / NORM_COLS)
                out[(size_t)k * ldo + m0 + c] = blk[k * NORM_COLS + c] * sc * ws[k];
        } else {
            for (int k = tid / NORM_COLS; k < K; k += 256 / NORM_COLS)
                out[(size_t)k * ldo + m0 + c] = blk[k * NORM_COLS + c] * sc * w[k];
        }
    }
}

// ---------------------------------------------------------------------------
// Row-major RMSNorm and the fused gated RMSNorm + residual: one warp per row,
// the row held in registers as float4s (VPL float4 per lane, dim = 128*VPL).
// The sum of squares is per-lane sequential then a warp tree.
// ---------------------------------------------------------------------------
template <int VPL, bool GATED>
__global__ void __launch_bounds__(256, VPL <= 4 ? 3 : 1) rownorm_kernel(const float* __restrict__ x, const float* __restrict__ z,
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
            const float4* rs = reinterpret_cast<const float4*>(res + r * DIM);
            float4 zz[VPL];
#pragma unroll
            for (int i = 0; i < VPL; ++i) {
                zz[i] = __ldcs(zr + lane + 32 * i);
                rr[i] = __ldcs(rs + lane + 32 * i);
            }
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
    // one wave of resident CTAs whose warps stride over the rows
    const int64_t want = (rows + 7) / 8;
    auto grid_for = [&](const void* fn) {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 256, 0) != cudaSuccess || per_sm < 1) per_sm = 1;
        const int64_t cap = (int64_t)sms * per_sm;
        return (int)(want < cap ? want : cap);
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
    if (ws) rmsnorm_fm_kernel<true><<<(M + NORM_COLS - 1) / NORM_COLS, 256, smem, s>>>(x, ldx, w, eps, K, M, out, ldo);
    else rmsnorm_fm_kernel<false><<<(M + NORM_COLS - 1) / NORM_COLS, 256, smem, s>>>(x, ldx, w, eps, K, M, out, ldo);
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
    embed_fm_kernel<<<grid, 256, 0, s>>>(tok, wte, vocab, K, M, out, ldo);
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
