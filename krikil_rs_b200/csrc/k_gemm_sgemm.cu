// fp32 C = A . W^T summed in the order of matrixmultiply 0.3.11's sgemm, the
// crate behind the reference's prefill projections (gemm_transb,
// src/math.rs:188-211; Cargo.toml:11 pins 0.3.11).  In that order every output
// element is one fused multiply-add chain over k, starting from zero, within
// each 256-long block of K (the f32 kc of its blocked algorithm and the 8x8
// AVX/FMA micro-kernel's one accumulator per element), and the blocks' sums
// reach the output in order: the first is stored, each later one added to it
// (alpha = beta = 1: one rounded add).
//
// A plain register-tiled GEMM computes exactly that: a thread owns a block of
// outputs and walks k in increasing order, so no dot-lane partials need
// folding (unlike gemm_lane8_kernel, which reproduces the gemv dot order of
// the decode projections).  Operands as in k_gemm.cu: A feature-major
// (At[k][m]) and W K-major (Wt[k][n]), staged through a two-slot cp.async
// ring of 32-row K-blocks (eight K-blocks make one 256-long sgemm block).
#include "common.cuh"
#include "kernels.h"

namespace krk {
namespace {

constexpr int SG_BM = 64, SG_BN = 32, SG_BK = 32, SG_NT = 128, SG_KC = 256;
static_assert(SG_KC % SG_BK == 0, "sgemm blocks must end on K-block boundaries");

__global__ void __launch_bounds__(SG_NT) gemm_sgemm_order_kernel(const float* __restrict__ At, int lda,
                                                                 const float* __restrict__ Wt, int ldw,
                                                                 float* __restrict__ C, int ldc, int K) {
    __shared__ __align__(16) float As[2][SG_BK * SG_BM];
    __shared__ __align__(16) float Ws[2][SG_BK * SG_BN];
    const int tid = threadIdx.x, tm = tid >> 3, tn = tid & 7;  // rows tm*4.., columns tn*4..
    const int m0 = blockIdx.x * SG_BM, n0 = blockIdx.y * SG_BN;
    const int nkb = K / SG_BK;

    auto load = [&](int slot, int kb) {
        const size_t k0 = (size_t)kb * SG_BK;
#pragma unroll
        for (int i = 0; i < SG_BK * SG_BM / 4 / SG_NT; ++i) {
            const int idx = tid + i * SG_NT, kk = idx / (SG_BM / 4), c4 = idx % (SG_BM / 4);
            cp_async16(&As[slot][kk * SG_BM + c4 * 4], At + (k0 + kk) * lda + m0 + c4 * 4);
        }
#pragma unroll
        for (int i = 0; i < SG_BK * SG_BN / 4 / SG_NT; ++i) {
            const int idx = tid + i * SG_NT, kk = idx / (SG_BN / 4), c4 = idx % (SG_BN / 4);
            cp_async16(&Ws[slot][kk * SG_BN + c4 * 4], Wt + (k0 + kk) * ldw + n0 + c4 * 4);
        }
        cp_async_commit();
    };

    // acc: this 256-long block's chains; tot: the sum of the finished blocks.
    // Pairs of columns (c, c+1) share one __ffma2_rn, each rounded as fmaf.
    float2 acc[4][2], tot[4][2];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < 2; ++j) acc[r][j] = tot[r][j] = make_float2(0.0f, 0.0f);

    load(0, 0);
    for (int kb = 0; kb < nkb; ++kb) {
        if (kb + 1 < nkb) {
            load((kb + 1) & 1, kb + 1);  // the slot read in iteration kb - 1, released by its closing barrier
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float* as = As[kb & 1];
        const float* ws = Ws[kb & 1];
#pragma unroll 8
        for (int kk = 0; kk < SG_BK; ++kk) {  // k in increasing order
            const float4 a = *reinterpret_cast<const float4*>(as + kk * SG_BM + tm * 4);
            const float4 w = *reinterpret_cast<const float4*>(ws + kk * SG_BN + tn * 4);
            const float ar[4] = {a.x, a.y, a.z, a.w};
            const float2 w01 = make_float2(w.x, w.y), w23 = make_float2(w.z, w.w);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float2 aa = make_float2(ar[r], ar[r]);
                acc[r][0] = __ffma2_rn(aa, w01, acc[r][0]);
                acc[r][1] = __ffma2_rn(aa, w23, acc[r][1]);
            }
        }
        __syncthreads();
        const int k_end = (kb + 1) * SG_BK;
        if (k_end % SG_KC == 0 || kb + 1 == nkb) {  // a 256-long block of K (or the last, shorter one) ends
            const bool first = k_end <= SG_KC;
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    tot[r][j] = first ? acc[r][j] : make_float2(acc[r][j].x + tot[r][j].x, acc[r][j].y + tot[r][j].y);
                    acc[r][j] = make_float2(0.0f, 0.0f);
                }
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
        *reinterpret_cast<float4*>(C + (size_t)(m0 + tm * 4 + r) * ldc + n0 + tn * 4) =
            make_float4(tot[r][0].x, tot[r][0].y, tot[r][1].x, tot[r][1].y);
}

// The wide form for M % 256 == 0: 256x32 CTA tiles, an 8x8 output block per
// thread (four 16-byte shared loads per 32 packed FMAs).  To keep the 64
// chains in registers, a finished 256-long block's sums go to C directly --
// stored by the first block, added to C by each later one -- and only the
// thread that owns an element ever reads or writes it.
constexpr int SW_BM = 256, SW_BN = 32, SW_BK = 32, SW_NT = 128;
constexpr size_t SW_SMEM = 2 * (size_t)SW_BK * (SW_BM + SW_BN) * sizeof(float);

__global__ void __launch_bounds__(SW_NT) gemm_sgemm_order_wide_kernel(const float* __restrict__ At, int lda,
                                                                      const float* __restrict__ Wt, int ldw,
                                                                      float* __restrict__ C, int ldc, int K) {
    extern __shared__ __align__(16) float sw[];
    float* As = sw;                          // [2][SW_BK][SW_BM]
    float* Ws = sw + 2 * SW_BK * SW_BM;      // [2][SW_BK][SW_BN]
    const int tid = threadIdx.x, tm = tid >> 2, tn = tid & 3;  // rows tm*8.., columns tn*8..
    const int m0 = blockIdx.x * SW_BM, n0 = blockIdx.y * SW_BN;
    const int nkb = K / SW_BK;

    auto load = [&](int slot, int kb) {
        const size_t k0 = (size_t)kb * SW_BK;
        float* as = As + slot * SW_BK * SW_BM;
        float* ws = Ws + slot * SW_BK * SW_BN;
#pragma unroll
        for (int i = 0; i < SW_BK * SW_BM / 4 / SW_NT; ++i) {
            const int idx = tid + i * SW_NT, kk = idx / (SW_BM / 4), c4 = idx % (SW_BM / 4);
            cp_async16(as + kk * SW_BM + c4 * 4, At + (k0 + kk) * lda + m0 + c4 * 4);
        }
#pragma unroll
        for (int i = 0; i < SW_BK * SW_BN / 4 / SW_NT; ++i) {
            const int idx = tid + i * SW_NT, kk = idx / (SW_BN / 4), c4 = idx % (SW_BN / 4);
            cp_async16(ws + kk * SW_BN + c4 * 4, Wt + (k0 + kk) * ldw + n0 + c4 * 4);
        }
        cp_async_commit();
    };

    float2 acc[8][4];  // rows r, column pairs (2j, 2j+1)
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[r][j] = make_float2(0.0f, 0.0f);

    load(0, 0);
    for (int kb = 0; kb < nkb; ++kb) {
        if (kb + 1 < nkb) {
            load((kb + 1) & 1, kb + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float* as = As + (kb & 1) * SW_BK * SW_BM;
        const float* ws = Ws + (kb & 1) * SW_BK * SW_BN;
#pragma unroll 4
        for (int kk = 0; kk < SW_BK; ++kk) {  // k in increasing order
            const float4 a0 = *reinterpret_cast<const float4*>(as + kk * SW_BM + tm * 8);
            const float4 a1 = *reinterpret_cast<const float4*>(as + kk * SW_BM + tm * 8 + 4);
            const float4 w0 = *reinterpret_cast<const float4*>(ws + kk * SW_BN + tn * 8);
            const float4 w1 = *reinterpret_cast<const float4*>(ws + kk * SW_BN + tn * 8 + 4);
            const float ar[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float2 wp[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                                  make_float2(w1.z, w1.w)};
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float2 aa = make_float2(ar[r], ar[r]);
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[r][j] = __ffma2_rn(aa, wp[j], acc[r][j]);
            }
        }
        __syncthreads();
        const int k_end = (kb + 1) * SW_BK;
        if (k_end % SG_KC == 0 || kb + 1 == nkb) {  // a 256-long block of K (or the last, shorter one) ends
            const bool first = k_end <= SG_KC;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                float4* c = reinterpret_cast<float4*>(C + (size_t)(m0 + tm * 8 + r) * ldc + n0 + tn * 8);
                float4 lo = make_float4(acc[r][0].x, acc[r][0].y, acc[r][1].x, acc[r][1].y);
                float4 hi = make_float4(acc[r][2].x, acc[r][2].y, acc[r][3].x, acc[r][3].y);
                if (!first) {
                    const float4 p0 = c[0], p1 = c[1];
                    lo = make_float4(lo.x + p0.x, lo.y + p0.y, lo.z + p0.z, lo.w + p0.w);
                    hi = make_float4(hi.x + p1.x, hi.y + p1.y, hi.z + p1.z, hi.w + p1.w);
                }
                c[0] = lo;
                c[1] = hi;
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[r][j] = make_float2(0.0f, 0.0f);
            }
        }
    }
}

}  // namespace

cudaError_t gemm_sgemm_order(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N,
                             int K, cudaStream_t s) {
    if (M <= 0 || N <= 0 || K <= 0 || M % SG_BM || N % SG_BN || K % SG_BK || N / SG_BN > 65535 || lda % 4 ||
        ldw % 4 || ldc % 4 || lda < M || ldw < N || ldc < N || ((uintptr_t)At | (uintptr_t)Wt | (uintptr_t)C) % 16)
        return cudaErrorInvalidValue;
    if (M % SW_BM == 0) {
        static DeviceOnce once;
        cudaError_t e;
        if ((e = once.set_smem((const void*)gemm_sgemm_order_wide_kernel, (int)SW_SMEM)) != cudaSuccess) return e;
        gemm_sgemm_order_wide_kernel<<<dim3(M / SW_BM, N / SW_BN), SW_NT, SW_SMEM, s>>>(At, lda, Wt, ldw, C, ldc, K);
    } else {
        gemm_sgemm_order_kernel<<<dim3(M / SG_BM, N / SG_BN), SG_NT, 0, s>>>(At, lda, Wt, ldw, C, ldc, K);
    }
    add_launches(1);
    return cudaGetLastError();
}

}  // namespace krk
