// Greedy token selection and generation bookkeeping.
#include "common.cuh"
#include "kernels.h"

namespace krk {
namespace {

// One CTA per sequence.  src/sampler.rs:50-80: the penalty divides positive
// and multiplies non-positive logits of every token seen so far; the greedy
// pick is the first index holding the maximum (strict '>' scan from -inf, so
// NaN never wins and an all-NaN/-inf row yields token 0).
__global__ void __launch_bounds__(256) greedy_kernel(GreedyArgs a) {
    const int b = blockIdx.x, tid = threadIdx.x;
    __shared__ float bv_s[8];
    __shared__ int bi_s[8];
    __shared__ int step_s;
    if (tid == 0) step_s = a.step ? *a.step : 0;
    const bool was_active = a.active ? a.active[b] != 0 : true;
    const float* lg = a.logits + (size_t)b * a.ld;
    const uint32_t* seen = a.seen ? a.seen + (size_t)b * (a.vocab / 32) : nullptr;
    const bool pen = seen && fabsf(a.penalty - 1.0f) > 1e-4f;
    float best = -INFINITY;
    int bi = a.vocab;
    for (int i = tid; i < a.vocab; i += 256) {
        float v = lg[i];
        if (pen && ((seen[i >> 5] >> (i & 31)) & 1u)) v = v > 0.0f ? v / a.penalty : v * a.penalty;
        if (v > best) { best = v; bi = i; }
    }
    // (value, index) reduction: larger value wins, ties go to the lower index.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if ((tid & 31) == 0) { bv_s[tid >> 5] = best; bi_s[tid >> 5] = bi; }
    __syncthreads();
    if (tid == 0) {
        best = bv_s[0]; bi = bi_s[0];
        for (int w = 1; w < 8; ++w)
            if (bv_s[w] > best || (bv_s[w] == best && bi_s[w] < bi)) { best = bv_s[w]; bi = bi_s[w]; }
        const uint32_t t = bi >= a.vocab ? 0u : (uint32_t)bi;
        if (was_active) {
            if (a.pos) a.pos[b] += 1;
            const int step = step_s;
            if (a.tlimit && step >= a.tlimit[b]) {
                if (a.active) a.active[b] = 0;  // sampled after the last counted token: unused
            } else {
                a.tok[b] = t;
                if (a.seen) atomicOr(a.seen + (size_t)b * (a.vocab / 32) + (t >> 5), 1u << (t & 31));
                if (a.hist) a.hist[(size_t)step * a.B + b] = t;
                const bool stop = (a.stop_eos && t == a.eos) || (a.slimit && step + 1 > a.slimit[b]);
                if (stop && a.active) a.active[b] = 0;
            }
        }
    }
}

__global__ void bump_step_kernel(int32_t* step) { *step += 1; }

__global__ void mark_seen_kernel(const uint32_t* __restrict__ tok, const int32_t* __restrict__ row_seq, int rows,
                                 uint32_t* __restrict__ seen, int words) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const uint32_t t = tok[r];
    if (t >= (uint32_t)words * 32u) return;
    atomicOr(seen + (size_t)row_seq[r] * words + (t >> 5), 1u << (t & 31));
}

__global__ void advance_pos_kernel(int32_t* pos, const uint8_t* active, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B && (!active || active[b])) pos[b] += 1;
}

__global__ void gather_cols_kernel(const float* __restrict__ src, int lds, const int32_t* __restrict__ scol,
                                   float* __restrict__ dst, int ldd, const int32_t* __restrict__ dcol, int K, int n) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int k = blockIdx.y;
    if (j >= n || k >= K) return;
    dst[(size_t)k * ldd + dcol[j]] = src[(size_t)k * lds + scol[j]];
}

}  // namespace

cudaError_t greedy(const GreedyArgs& a, cudaStream_t s) {
    if (a.B <= 0 || a.vocab <= 0 || a.vocab % 32 || !a.tok) return cudaErrorInvalidValue;
    greedy_kernel<<<a.B, 256, 0, s>>>(a);
    add_launches(1);
    if (a.step) {
        bump_step_kernel<<<1, 1, 0, s>>>(a.step);
        add_launches(1);
    }
    return cudaGetLastError();
}

cudaError_t mark_seen(const uint32_t* tok, const int32_t* row_seq, int rows, uint32_t* seen, int words,
                      cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    mark_seen_kernel<<<(rows + 255) / 256, 256, 0, s>>>(tok, row_seq, rows, seen, words);
    add_launches(1);
    return cudaGetLastError();
}

cudaError_t advance_pos(int32_t* pos, const uint8_t* active, int B, cudaStream_t s) {
    advance_pos_kernel<<<(B + 255) / 256, 256, 0, s>>>(pos, active, B);
    add_launches(1);
    return cudaGetLastError();
}

cudaError_t gather_cols(const float* src, int lds, const int32_t* scol, float* dst, int ldd, const int32_t* dcol,
                        int K, int n, cudaStream_t s) {
    if (n <= 0 || K <= 0) return cudaSuccess;
    dim3 grid((n + 127) / 128, K);
    gather_cols_kernel<<<grid, 128, 0, s>>>(src, lds, scol, dst, ldd, dcol, K, n);
    add_launches(1);
    return cudaGetLastError();
}

}  // namespace krk
