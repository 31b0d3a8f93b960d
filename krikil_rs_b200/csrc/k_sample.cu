// Greedy token selection and generation bookkeeping.
#include "common.cuh"
#include "kernels.h"

namespace krk {
namespace {

// Records pick t of sequence b at generation step `step` (src/generate.rs:86-114):
// advances the position, pushes the token unless the sequence's pick limit is
// reached, marks it seen, and deactivates the sequence on EOS or its step limit.
KRK_DEV void commit_pick(const GreedyArgs& a, int b, uint32_t t, int step) {
    if (a.pos) a.pos[b] += 1;
    if (a.tlimit && step >= a.tlimit[b]) {
        if (a.active) a.active[b] = 0;  // sampled after the last counted token: unused
        return;
    }
    a.tok[b] = t;
    if (a.seen) atomicOr(a.seen + (size_t)b * (a.vocab / 32) + (t >> 5), 1u << (t & 31));
    if (a.hist) a.hist[(size_t)step * a.B + b] = t;
    const bool stop = (a.stop_eos && t == a.eos) || (a.slimit && step + 1 > a.slimit[b]);
    if (stop && a.active) a.active[b] = 0;
}

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
        if (was_active) commit_pick(a, b, t, step_s);
    }
}

// ---- stochastic pick --------------------------------------------------------
KRK_DEV uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }
KRK_DEV void chacha_qr(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
    a += b; d ^= a; d = rotl32(d, 16);
    c += d; b ^= c; b = rotl32(b, 12);
    a += b; d ^= a; d = rotl32(d, 8);
    c += d; b ^= c; b = rotl32(b, 7);
}
// Next 32-bit word of the ChaCha12 keystream of state st (key st[0..7], word
// index st[8..9]; 64-bit block counter in words 12-13, zero stream id), as
// rand_chacha's ChaCha12Rng::next_u32; advances the index.
KRK_DEV uint32_t rng_next_u32(uint32_t* st) {
    const uint64_t n = (uint64_t)st[8] | ((uint64_t)st[9] << 32);
    const uint64_t blk = n >> 4;
    uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, st[0], st[1], st[2], st[3],
                       st[4], st[5], st[6], st[7], (uint32_t)blk, (uint32_t)(blk >> 32), 0u, 0u};
    uint32_t x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = in[i];
#pragma unroll
    for (int r = 0; r < 12; r += 2) {
        chacha_qr(x[0], x[4], x[8], x[12]);
        chacha_qr(x[1], x[5], x[9], x[13]);
        chacha_qr(x[2], x[6], x[10], x[14]);
        chacha_qr(x[3], x[7], x[11], x[15]);
        chacha_qr(x[0], x[5], x[10], x[15]);
        chacha_qr(x[1], x[6], x[11], x[12]);
        chacha_qr(x[2], x[7], x[8], x[13]);
        chacha_qr(x[3], x[4], x[9], x[14]);
    }
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (i == (int)(n & 15)) w = x[i] + in[i];
    const uint64_t n1 = n + 1;
    st[8] = (uint32_t)n1;
    st[9] = (uint32_t)(n1 >> 32);
    return w;
}

// Candidate order: larger value first; equal values (left in an unspecified
// order by the reference's unstable sort) by ascending id; NaN last.
KRK_DEV bool precedes(float va, uint32_t ia, float vb, uint32_t ib) {
    const bool na = isnan(va), nb = isnan(vb);
    if (na != nb) return nb;
    if (!na && va != vb) return va > vb;
    return ia < ib;
}

// One CTA per sequence.  src/sampler.rs:43-152: penalty, logits * (1/T), sort
// descending (bitonic, in shared memory), top-k, softmax with the sequential
// sum of the reference, top-p cut and renormalisation, then the first
// candidate whose running sum reaches r = (next_u32 >> 8) * 2^-24.
__global__ void __launch_bounds__(256) sample_kernel(GreedyArgs a, int npow2) {
    extern __shared__ __align__(16) float sv[];
    uint32_t* si = reinterpret_cast<uint32_t*>(sv + npow2);
    __shared__ int step_s;
    const int b = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) step_s = a.step ? *a.step : 0;
    const bool was_active = a.active ? a.active[b] != 0 : true;
    const float* lg = a.logits + (size_t)b * a.ld;
    const uint32_t* seen = a.seen ? a.seen + (size_t)b * (a.vocab / 32) : nullptr;
    const bool pen = seen && fabsf(a.penalty - 1.0f) > 1e-4f;
    const float inv_temp = 1.0f / a.temperature;
    for (int i = tid; i < npow2; i += 256) {
        float v = __int_as_float(0x7fc00000);  // padding: NaN, sorted last
        if (i < a.vocab) {
            v = lg[i];
            if (pen && ((seen[i >> 5] >> (i & 31)) & 1u)) v = v > 0.0f ? v / a.penalty : v * a.penalty;
            v = v * inv_temp;
        }
        sv[i] = v;
        si[i] = (uint32_t)i;
    }
    __syncthreads();
    for (int k = 2; k <= npow2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < npow2; i += 256) {
                const int l = i ^ j;
                if (l > i) {
                    const bool up = (i & k) == 0;  // this run in candidate order
                    const float vi = sv[i], vl = sv[l];
                    const uint32_t ii = si[i], il = si[l];
                    if (up ? precedes(vl, il, vi, ii) : precedes(vi, ii, vl, il)) {
                        sv[i] = vl; sv[l] = vi;
                        si[i] = il; si[l] = ii;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (tid == 0 && was_active) {
        int n = (a.top_k > 0 && a.top_k < a.vocab) ? a.top_k : a.vocab;
        const float mx = sv[0];
        float sum = 0.0f;
        for (int i = 0; i < n; ++i) {
            const float p = expf(sv[i] - mx);
            sv[i] = p;
            sum += p;
        }
        const float inv_sum = 1.0f / sum;
        for (int i = 0; i < n; ++i) sv[i] = sv[i] * inv_sum;
        if (a.top_p < 1.0f) {
            float cum = 0.0f;
            int cut = n;
            for (int i = 0; i < n; ++i) {
                cum += sv[i];
                if (cum >= a.top_p) {
                    cut = min(i + 1, n);
                    break;
                }
            }
            n = cut;
            float ns = 0.0f;
            for (int i = 0; i < n; ++i) ns += sv[i];
            const float inv_ns = 1.0f / ns;
            for (int i = 0; i < n; ++i) sv[i] = sv[i] * inv_ns;
        }
        const float r = (float)(rng_next_u32(a.rng + (size_t)b * 10) >> 8) * (1.0f / 16777216.0f);
        float acc = 0.0f;
        uint32_t t = si[0];
        for (int i = 0; i < n; ++i) {
            acc += sv[i];
            if (r <= acc) {
                t = si[i];
                break;
            }
        }
        commit_pick(a, b, t < (uint32_t)a.vocab ? t : 0u, step_s);
    }
}

__global__ void bump_step_kernel(int32_t* step) { *step += 1; }

__global__ void mark_seen_kernel(const uint32_t* __restrict__ tok, const int32_t* __restrict__ row_seq, int rows,
                                 uint32_t* __restrict__ seen, int words) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const uint32_t t = tok[r];
    if (t >= (uint32_t)words * 32u) {
        check_fail(CHK_TOKEN);
        return;
    }
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
    const int dc = dcol[j], sc = scol[j];
    if (kChecked && (dc < 0 || dc >= ldd || sc < 0 || sc >= lds)) {
        check_fail(CHK_COLUMN);
        return;
    }
    dst[(size_t)k * ldd + dc] = src[(size_t)k * lds + sc];
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

cudaError_t sample(const GreedyArgs& a, cudaStream_t s) {
    if (a.temperature <= 1e-6f) return greedy(a, s);
    if (a.B <= 0 || a.vocab <= 0 || a.vocab % 32 || a.vocab > 4096 || !a.tok || !a.rng) return cudaErrorInvalidValue;
    int np2 = 32;
    while (np2 < a.vocab) np2 <<= 1;
    const size_t smem = (size_t)np2 * (sizeof(float) + sizeof(uint32_t));
    sample_kernel<<<a.B, 256, smem, s>>>(a, np2);
    add_launches(1);
    if (a.step) {
        bump_step_kernel<<<1, 1, 0, s>>>(a.step);
        add_launches(1);
    }
    return cudaGetLastError();
}

// rand_core 0.6 SeedableRng::seed_from_u64: the 32-byte seed from a PCG32
// (XSH-RR) sequence whose state is advanced before each 4-byte output.
void rng_seed_state(uint64_t seed, uint32_t st[10]) {
    uint64_t x = seed;
    for (int i = 0; i < 8; ++i) {
        x = x * 6364136223846793005ULL + 11634580027462260723ULL;
        const uint32_t xs = (uint32_t)(((x >> 18) ^ x) >> 27);
        const uint32_t rot = (uint32_t)(x >> 59);
        st[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
    }
    st[8] = 0;
    st[9] = 0;
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
