// fp32 projections C = A . W^T on the SIMT FP32 pipes, reproducing the
// reference's dot-product rounding exactly.
//
// The reference computes every projection output as dot(W[r], x) with the AVX2
// kernel of src/math.rs:89-124: eight lanes, lane j accumulating
// a[j+8i]*b[j+8i] with a fused multiply-add in increasing i, folded as
// ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)).  (All K here are multiples of 8, so
// its scalar tail is empty.)  This kernel maps those eight lanes onto the eight
// warps of a CTA: warp w owns the k = w (mod 8) slice of every K-block and keeps
// a full 64x32 (or 32x32, 16x32) output tile of partial sums in registers; the
// eight warp tiles are folded in the reference's order through shared memory in
// the epilogue.  The result is bit-identical to the reference gemv for any M.
// For up to 8 rows (a small decode batch) gemm_skinny_kernel keeps the same
// lane-per-warp order with one thread per (output column, lane), optionally
// normalising A (the RMSNorm that feeds the projection) in the same launch.
// The multiply-adds are issued as packed pairs (__ffma2_rn, sm_100): each
// component is rounded exactly as fmaf, and one instruction does two, which
// halves the issue slots the FP32 pipes need.
//
// Operands: A feature-major (At[k][m], contiguous along m) and W K-major
// (Wt[k][n], contiguous along n), so that the rows of both are dense runs that
// cp.async moves straight into shared memory, and the inner loop reads 8 m and
// 8 n values with four 16-byte shared loads.  Since warp w only ever reads the
// rows k = w (mod 8), each warp stages its own four rows of every K-block in a
// private 4-deep ring: the main loop synchronises the warp, never the CTA.
#include "common.cuh"
#include "kernels.h"

namespace krk {
namespace {

constexpr int BN = 32, BK = 32, NT = 256, WSTAGE = 4;
constexpr int WROWS = BK / 8;  // K-block rows owned by one warp
constexpr int RLD_BM = BN + 4;  // partials red[w][m][n] for batch-major output
constexpr int SKINNY_MAX_K = 2432;  // the widest projection input (fc2 over the MLP width)

template <int BM>
struct Tile {
    static constexpr int TM = BM / 8;                 // rows per thread (8 lanes of rows per warp)
    static constexpr int WST = WROWS * (BM + BN);     // one warp's stage: 4 rows of A, then 4 of W
    static constexpr int PIPE = 8 * WSTAGE * WST;
    static constexpr int RLD_FM = BM + 4;             // partials red[w][n][m] for feature-major output
    static constexpr int RED = 8 * BM * RLD_BM > 8 * BN * RLD_FM ? 8 * BM * RLD_BM : 8 * BN * RLD_FM;
    static constexpr int SMEM_FLOATS = RED > PIPE ? RED : PIPE;
    static constexpr size_t SMEM_BYTES = SMEM_FLOATS * sizeof(float);
    static constexpr int A_F4 = BM / 32;              // float4 copies of A per lane per K-block (BM = 16: half the lanes copy one)
    static constexpr int OUT_F4 = (BM * BN / 4 + NT - 1) / NT;  // output float4s per thread (BM = 16: half the threads)
    static constexpr int MIN_CTAS = BM == 64 ? 2 : BM == 32 ? 3 : 4;
};

KRK_DEV float4 f4add(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }

// ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)): the fold of src/math.rs:110-117.
KRK_DEV float4 fold8(const float4* l) {
    float4 s04 = f4add(l[0], l[4]), s15 = f4add(l[1], l[5]), s26 = f4add(l[2], l[6]), s37 = f4add(l[3], l[7]);
    return f4add(f4add(s04, s26), f4add(s15, s37));
}

// Thread (lm, ln) of a warp owns rows m(r) and columns n(c), r < TM, c < 8:
//   BM = 64: m in {lm*4 + i, 32 + lm*4 + i};  BM = 32: m = lm*4 + i;  BM = 16: m = lm*2 + i
//   n in {ln*4 + j, 16 + ln*4 + j}
// so each 16-byte shared load of a warp hits distinct banks.
template <int BM>
KRK_DEV int row_of(int lm, int r) {
    if (BM == 16) return lm * 2 + r;
    return (r < 4) ? lm * 4 + r : 32 + lm * 4 + (r - 4);
}
KRK_DEV int col_of(int ln, int c) { return (c < 4) ? ln * 4 + c : 16 + ln * 4 + (c - 4); }

template <int BM, int EPI, bool OUT_FM>
__global__ void __launch_bounds__(NT, Tile<BM>::MIN_CTAS)
    gemm_lane8_kernel(const float* __restrict__ At, int lda, const float* __restrict__ Wt, int ldw,
                      float* __restrict__ C, int ldc, int K, const GemmConv cv) {
    using T = Tile<BM>;
    constexpr int TM = T::TM;
    extern __shared__ __align__(16) float sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lm = lane >> 2, ln = lane & 3;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int nkb = K / BK;

    float* ring = sm + warp * (WSTAGE * T::WST);
    // Element offsets of this lane's copy sources (rows k = warp + 8r of the
    // next K-block), advanced by BK rows per stage: one integer add per operand
    // instead of a wide multiply per copy.  The host keeps A^T and W^T below
    // 2^31 elements, so the 32-bit offsets cannot wrap.
    constexpr int AR = 32 / (BM / 4);  // A rows covered by one pass of the 32 lanes
    unsigned a_off = (unsigned)(warp + 8 * (lane / (BM / 4))) * lda + m0 + (lane % (BM / 4)) * 4;
    unsigned w_off = (unsigned)(warp + 8 * (lane >> 3)) * ldw + n0 + (lane & 7) * 4;
    // This warp's four rows of the next K-block into the ring slot at As.
    auto load_a = [&](float* As) {
#pragma unroll
        for (int j = 0; j < T::A_F4; ++j)
            cp_async16(As + (lane / (BM / 4) + j * AR) * BM + (lane % (BM / 4)) * 4, At + a_off + j * (8 * AR) * lda);
        if (BM == 16 && lane < 16) cp_async16(As + (lane >> 2) * BM + (lane & 3) * 4, At + a_off);
        a_off += BK * lda;
    };
    auto load_w = [&](float* As) {
        cp_async16(As + WROWS * BM + (lane >> 3) * BN + (lane & 7) * 4, Wt + w_off);
        w_off += BK * ldw;
    };
    auto load_stage = [&](float* As) {
        load_a(As);
        load_w(As);
    };

    // Partial sums in pairs, one __ffma2_rn per pair.  Batch-major output pairs
    // rows: acc2[i*8 + c] = rows (2i, 2i+1) of column c; feature-major output
    // pairs columns: acc2[r*4 + j] = columns (2j, 2j+1) of row r (indices of
    // row_of / col_of).  The two forms differ only in register allocation;
    // with two rows per thread (BM = 16) columns are paired in both.
    constexpr bool PAIR_ROWS = !OUT_FM && TM >= 4;
    float2 acc2[TM * 4];
#pragma unroll
    for (int i = 0; i < TM * 4; ++i) acc2[i] = make_float2(0.0f, 0.0f);

    int wr = (WSTAGE - 1) * T::WST, rd = 0;  // ring offsets of the slot filled next and the slot read next
    // The first slots' weights are copied before A, which the kernels before
    // this one write: they join the first slot's copy group.
#pragma unroll
    for (int s = 0; s < WSTAGE - 1; ++s)
        if (s < nkb) load_w(ring + s * T::WST);
    pdl_wait();
    pdl_trigger();
#pragma unroll
    for (int s = 0; s < WSTAGE - 1; ++s) {
        if (s < nkb) load_a(ring + s * T::WST);
        cp_async_commit();
    }
    for (int kb = 0; kb < nkb; ++kb) {
        cp_async_wait<WSTAGE - 2>();
        // All lanes' copies of slot kb are visible, and every lane is done
        // reading the slot refilled next (consumed in iteration kb - 1).
        __syncwarp();
        if (kb + WSTAGE - 1 < nkb) load_stage(ring + wr);
        cp_async_commit();
        wr = wr == (WSTAGE - 1) * T::WST ? 0 : wr + T::WST;
        const float* As = ring + rd;
        const float* Ws = As + WROWS * BM;
        rd = rd == (WSTAGE - 1) * T::WST ? 0 : rd + T::WST;
#pragma unroll
        for (int i = 0; i < WROWS; ++i) {  // k = kb*32 + warp + 8i: this warp's lane of the reference dot
            float a[TM];
            if (TM == 2) {
                const float2 a0 = *reinterpret_cast<const float2*>(As + i * BM + lm * 2);
                a[0] = a0.x; a[TM == 2 ? 1 : 0] = a0.y;
            } else {
                const float4 a0 = *reinterpret_cast<const float4*>(As + i * BM + lm * 4);
                a[0] = a0.x; a[TM > 2 ? 1 : 0] = a0.y; a[TM > 2 ? 2 : 0] = a0.z; a[TM > 2 ? 3 : 0] = a0.w;
                if (TM == 8) {
                    const float4 a1 = *reinterpret_cast<const float4*>(As + i * BM + 32 + lm * 4);
                    a[TM == 8 ? 4 : 0] = a1.x; a[TM == 8 ? 5 : 1] = a1.y;
                    a[TM == 8 ? 6 : 2] = a1.z; a[TM == 8 ? 7 : 3] = a1.w;
                }
            }
            const float4 w0 = *reinterpret_cast<const float4*>(Ws + i * BN + ln * 4);
            const float4 w1 = *reinterpret_cast<const float4*>(Ws + i * BN + 16 + ln * 4);
            const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            // two fused multiply-adds per instruction, each rounded as fmaf
            if (PAIR_ROWS) {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float2 wc = make_float2(w[c], w[c]);
#pragma unroll
                    for (int r = 0; r < TM / 2; ++r)
                        acc2[r * 8 + c] = __ffma2_rn(make_float2(a[2 * r], a[2 * r + 1]), wc, acc2[r * 8 + c]);
                }
            } else {
#pragma unroll
                for (int r = 0; r < TM; ++r) {
                    const float2 ar = make_float2(a[r], a[r]);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        acc2[r * 4 + j] = __ffma2_rn(ar, make_float2(w[2 * j], w[2 * j + 1]), acc2[r * 4 + j]);
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    // Spill the eight lane-partial tiles, laid out along the output's
    // contiguous dimension.
    auto acc = [&](int r, int c) -> float {
        if (PAIR_ROWS) return (r & 1) ? acc2[(r >> 1) * 8 + c].y : acc2[(r >> 1) * 8 + c].x;
        return (c & 1) ? acc2[r * 4 + (c >> 1)].y : acc2[r * 4 + (c >> 1)].x;
    };
    float* red = sm;
    if (!OUT_FM) {
        float* base = red + warp * (BM * RLD_BM);
#pragma unroll
        for (int r = 0; r < TM; ++r) {
            float* d = base + row_of<BM>(lm, r) * RLD_BM;
            *reinterpret_cast<float4*>(d + ln * 4) = make_float4(acc(r, 0), acc(r, 1), acc(r, 2), acc(r, 3));
            *reinterpret_cast<float4*>(d + 16 + ln * 4) = make_float4(acc(r, 4), acc(r, 5), acc(r, 6), acc(r, 7));
        }
    } else {
        float* base = red + warp * (BN * T::RLD_FM);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float* d = base + col_of(ln, c) * T::RLD_FM;
            if (TM == 2) {
                *reinterpret_cast<float2*>(d + lm * 2) = make_float2(acc(0, c), acc(1, c));
                continue;
            }
            *reinterpret_cast<float4*>(d + lm * 4) =
                make_float4(acc(0, c), acc(TM > 2 ? 1 : 0, c), acc(TM > 2 ? 2 : 0, c), acc(TM > 2 ? 3 : 0, c));
            if (TM == 8)
                *reinterpret_cast<float4*>(d + 32 + lm * 4) = make_float4(
                    acc(TM == 8 ? 4 : 0, c), acc(TM == 8 ? 5 : 1, c), acc(TM == 8 ? 6 : 2, c), acc(TM == 8 ? 7 : 3, c));
        }
    }
    __syncthreads();

#pragma unroll
    for (int j = 0; j < T::OUT_F4; ++j) {
        const int idx = tid + j * NT;
        if (BM * BN / 4 < NT && idx >= BM * BN / 4) break;
        const float* part;
        int wstride;
        float* out;
        if (!OUT_FM) {
            const int m = idx >> 3, n4 = idx & 7;
            part = red + m * RLD_BM + n4 * 4;
            wstride = BM * RLD_BM;
            out = C + (size_t)(m0 + m) * ldc + n0 + n4 * 4;
        } else {
            const int n = idx / (BM / 4), m4 = idx % (BM / 4);
            part = red + n * T::RLD_FM + m4 * 4;
            wstride = BN * T::RLD_FM;
            out = C + (size_t)(n0 + n) * ldc + m0 + m4 * 4;
        }
        float4 l[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) l[w] = *reinterpret_cast<const float4*>(part + w * wstride);
        float4 v = fold8(l);
        if (EPI == EPI_CONV) {  // src/model.rs:643-654 on the channels this tile holds
            const int m = m0 + (idx >> 3), n = n0 + (idx & 7) * 4;
            if (n >= cv.lo && n < cv.hi && m < cv.rows && (!cv.active || cv.active[m])) {
                const int c = n - cv.lo;
                float4* sp = reinterpret_cast<float4*>(cv.state + ((size_t)m * (cv.hi - cv.lo) + c) * 4);
                const float4* wp = reinterpret_cast<const float4*>(cv.w) + c;
                float xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 st = sp[e], wv = wp[e];
                    // after the shift the window is [st.y, st.z, st.w, x]
                    const float val = st.y * wv.x + st.z * wv.y + st.w * wv.z + xv[e] * wv.w + cv.bias[c + e];
                    sp[e] = make_float4(st.y, st.z, st.w, xv[e]);
                    xv[e] = silu(val);
                }
                v = make_float4(xv[0], xv[1], xv[2], xv[3]);
            }
        } else if (EPI == EPI_RESIDUAL) {
            float4 o = *reinterpret_cast<const float4*>(out);  // x += out (src/model.rs:699-701)
            v = f4add(o, v);
        } else if (EPI == EPI_GELU) {
            v = make_float4(gelu(v.x), gelu(v.y), gelu(v.z), gelu(v.w));
        }
        *reinterpret_cast<float4*>(out) = v;
    }
}

// Projection of a few rows (the decode step of up to SKINNY_MAX_ROWS
// sequences): thread (j, c) of a CTA -- warp j, lane c -- is lane j of the
// reference dot for output column n0 + c, accumulating one FMA chain per row
// over k = j, j + 8, ... in order; the eight lane partials are folded in the
// reference's order through shared memory.  The same arithmetic as
// gemm_lane8_kernel, so the results are bitwise those of any tile height, but
// a launch reads W^T once and its longest chain is K/8 FMAs instead of a
// 16- to 64-row tile's K loop.  Warp j streams its rows of W^T (the CTA's 32
// columns) through a private SK_STAGES-deep cp.async ring of 4-row stages, so
// ~32 rows are in flight per warp.  Only the M rows given are computed.
constexpr int SKINNY_MAX_ROWS = 8;
constexpr int SK_STAGES = 8, SK_ROWS = 4, SK_ST = SK_ROWS * BN;  // one stage of one warp: 4 rows x 32 columns

// MT: M rounded up to 1, 2, 4 or 8 (the extra columns of A are read from the
// operand's padding and their outputs never written).  A is staged permuted,
// sa[(j * K/8 + i) * MT + m] = A(m, j + 8i), so a thread's four chain rows of a
// stage are 4 * MT consecutive floats.
// NORM: A is rms_norm(A) (src/math.rs:41-54) -- the staged copy is
// normalised in place first, its scales formed as rmsnorm_fm_kernel forms
// them (32 partials p: A(m, k)^2 for k = p, p + 32, ... in order; per group of
// four ((p0+p1)+(p2+p3)); the eight groups in order; 1 / sqrt(sum / K + eps))
// and each element as (x * scale) * w[k]: bitwise rmsnorm_fm and then the
// projection, in one launch.
// LPW: dot lanes per warp (1: 8 warps, 32 columns per CTA; 2: 4 warps, 16
// columns per CTA, half-warp h taking lane w + 4h) -- twice the CTAs for
// projections whose 32-column grid leaves most SMs idle.
template <int MT, int EPI, bool OUT_FM, bool NORM, int LPW>
__global__ void __launch_bounds__(256 / LPW) gemm_skinny_kernel(const float* __restrict__ At, int lda,
                                                                const float* __restrict__ Wt, int ldw,
                                                                float* __restrict__ C, int ldc, int M, int K,
                                                                const GemmConv cv, const GemmNorm nm) {
    constexpr int NWARPS = 8 / LPW, NTH = 32 * NWARPS, CW = BN / LPW;
    extern __shared__ __align__(16) float smk[];  // rings [warps][SK_STAGES][4 * LPW][CW], then A [8][K/8][MT]
    __shared__ float red[8][SKINNY_MAX_ROWS][CW + 1];
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
    const int h = l / CW, c = l % CW, j = w + NWARPS * h;  // this thread's dot lane and column
    const int n0 = blockIdx.x * CW;
    const int kj = K / 8;  // rows of one dot lane
    float* ring = smk + w * (SK_STAGES * SK_ST);
    float* sa = smk + NWARPS * SK_STAGES * SK_ST;
    const int nst = K / (8 * SK_ROWS);  // stages of a lane's rows k = j + 8i
    // lane l copies 16 bytes of stage row rho = l / (CW / 4) (the warp's lane
    // w + NWARPS * (rho / 4), chain row 4 st + rho % 4): columns n0 + 4 (l % (CW / 4)) ..
    const int rho = l / (CW / 4), col4 = l % (CW / 4);
    const float* wsrc =
        Wt + (size_t)(w + NWARPS * (rho / SK_ROWS) + 8 * (rho % SK_ROWS)) * ldw + n0 + col4 * 4;
    const size_t wstage = (size_t)8 * SK_ROWS * ldw;
    const int wdst = rho * CW + col4 * 4;
#pragma unroll
    for (int st = 0; st < SK_STAGES - 1; ++st) {
        if (st < nst) cp_async16(ring + st * SK_ST + wdst, wsrc + st * wstage);
        cp_async_commit();
    }
    // the weights are in flight; A (and the output, the conv state) belong to
    // the kernels before this one
    pdl_wait();
    pdl_trigger();
    for (int i = tid; i < K * MT; i += NTH) {
        const int k = i / MT, m = i % MT;
        sa[((k & 7) * kj + (k >> 3)) * MT + m] = At[(size_t)k * lda + m];
    }
    __syncthreads();
    if (NORM) {
        __shared__ float ps[32][MT];
        __shared__ float scl[MT];
        for (int pi = tid; pi < 32 * MT; pi += NTH) {
            const int m = pi % MT, q = pi / MT;
            float ss = 0.0f;
            for (int k = q; k < K; k += 32) {
                const float v = sa[((k & 7) * kj + (k >> 3)) * MT + m];
                ss += v * v;
            }
            ps[q][m] = ss;
        }
        __syncthreads();
        if (tid < MT) {
            float t = 0.0f;
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                const float s4 = (ps[4 * g][tid] + ps[4 * g + 1][tid]) + (ps[4 * g + 2][tid] + ps[4 * g + 3][tid]);
                t = g == 0 ? s4 : t + s4;
            }
            scl[tid] = 1.0f / sqrtf(t / (float)K + nm.eps);
        }
        __syncthreads();
        for (int i = tid; i < K * MT; i += NTH) {
            const int pos = i / MT, m = i % MT;
            sa[i] = sa[i] * scl[m] * __ldg(nm.w + (pos / kj) + 8 * (pos % kj));
        }
        __syncthreads();
    }
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
    const float* aj = sa + (size_t)j * kj * MT;
    for (int st = 0; st < nst; ++st) {
        cp_async_wait<SK_STAGES - 2>();
        __syncwarp();  // every lane's copy of stage st is visible; stage st - 1 is read
        const int nx = st + SK_STAGES - 1;
        if (nx < nst) cp_async16(ring + (nx % SK_STAGES) * SK_ST + wdst, wsrc + nx * wstage);
        cp_async_commit();
        const float* ws = ring + (st % SK_STAGES) * SK_ST + h * SK_ROWS * CW;
        float av[SK_ROWS * MT];  // rows 4st .. 4st+3 of this lane's chain, MT values each
#pragma unroll
        for (int q = 0; q < SK_ROWS * MT / 4; ++q) {
            const float4 v = *reinterpret_cast<const float4*>(aj + (SK_ROWS * st) * MT + 4 * q);
            av[4 * q] = v.x; av[4 * q + 1] = v.y; av[4 * q + 2] = v.z; av[4 * q + 3] = v.w;
        }
#pragma unroll
        for (int r = 0; r < SK_ROWS; ++r) {  // k = j + 8(4 st + r): this lane's chain in order
            const float wv = ws[r * CW + c];
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[m] = fmaf(av[r * MT + m], wv, acc[m]);
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int m = 0; m < MT; ++m) red[j][m][c] = acc[m];
    __syncthreads();
    if (tid >= M * CW) return;
    const int m = tid / CW, cc = tid % CW, n = n0 + cc;
    float lp[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) lp[q] = red[q][m][cc];
    float v = ((lp[0] + lp[4]) + (lp[2] + lp[6])) + ((lp[1] + lp[5]) + (lp[3] + lp[7]));  // src/math.rs:110-117
    float* out = OUT_FM ? C + (size_t)n * ldc + m : C + (size_t)m * ldc + n;
    if (EPI == EPI_CONV) {  // src/model.rs:643-654 for this (row, channel)
        if (n >= cv.lo && n < cv.hi && m < cv.rows && (!cv.active || cv.active[m])) {
            const int ch = n - cv.lo;
            float4* sp = reinterpret_cast<float4*>(cv.state + ((size_t)m * (cv.hi - cv.lo) + ch) * 4);
            const float4 sv = *sp, wv = reinterpret_cast<const float4*>(cv.w)[ch];
            // after the shift the window is [sv.y, sv.z, sv.w, x]
            const float val = sv.y * wv.x + sv.z * wv.y + sv.w * wv.z + v * wv.w + cv.bias[ch];
            *sp = make_float4(sv.y, sv.z, sv.w, v);
            v = silu(val);
        }
    } else if (EPI == EPI_RESIDUAL) {
        v = *out + v;  // x += out (src/model.rs:699-701)
    } else if (EPI == EPI_GELU) {
        v = gelu(v);
    }
    *out = v;
}

template <int MT, int EPI, bool OUT_FM, bool NORM, int LPW>
cudaError_t launch_skinny_mt(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                             cudaStream_t s, const GemmConv& cv, const GemmNorm& nm) {
    static DeviceOnce once;
    constexpr size_t ring_bytes = (size_t)(8 / LPW) * SK_STAGES * SK_ST * sizeof(float);
    const size_t smem = ring_bytes + (size_t)K * MT * sizeof(float);
    cudaError_t e = once.set_smem((const void*)gemm_skinny_kernel<MT, EPI, OUT_FM, NORM, LPW>,
                                  ring_bytes + (size_t)SKINNY_MAX_K * MT * sizeof(float));
    if (e != cudaSuccess) return e;
    e = launch_pdl(gemm_skinny_kernel<MT, EPI, OUT_FM, NORM, LPW>, dim3(N / (BN / LPW)), dim3(256 / LPW), smem, s, At,
                   lda, Wt, ldw, C, ldc, M, K, cv, nm);
    if (e != cudaSuccess) return e;
    add_launches(1);
    return cudaGetLastError();
}

template <int MT, int EPI, bool OUT_FM, bool NORM>
cudaError_t launch_skinny_mt(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                             cudaStream_t s, const GemmConv& cv, const GemmNorm& nm) {
    // 16 columns per CTA where that measured faster (CUDA graphs of the decode
    // projections): one or two rows, at most 2048 columns and no norm inside --
    // fc2 8.7 -> 7.8 us, wo 4.0 -> 3.6 us at one row; wider projections, more
    // rows and the norm's pass over the staged rows lose the warps it takes.
    if (!NORM && M <= 2 && N <= 2048)
        return launch_skinny_mt<MT, EPI, OUT_FM, NORM, 2>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv, nm);
    return launch_skinny_mt<MT, EPI, OUT_FM, NORM, 1>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv, nm);
}

// M <= 8 rows; lda >= 4 * ceil(M / 4) (lda % 4 == 0 and lda >= M guarantee it)
template <int EPI, bool OUT_FM, bool NORM = false>
cudaError_t launch_skinny(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                          cudaStream_t s, const GemmConv& cv = GemmConv{}, const GemmNorm& nm = GemmNorm{}) {
    if (M == 1) return launch_skinny_mt<1, EPI, OUT_FM, NORM>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv, nm);
    if (M == 2) return launch_skinny_mt<2, EPI, OUT_FM, NORM>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv, nm);
    if (M <= 4) return launch_skinny_mt<4, EPI, OUT_FM, NORM>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv, nm);
    return launch_skinny_mt<8, EPI, OUT_FM, NORM>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv, nm);
}

template <int BM, int EPI, bool OUT_FM>
cudaError_t launch(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                   cudaStream_t s, const GemmConv& cv = GemmConv{}) {
    static DeviceOnce once;
    cudaError_t e = once.set_smem((const void*)gemm_lane8_kernel<BM, EPI, OUT_FM>, Tile<BM>::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    e = launch_pdl(gemm_lane8_kernel<BM, EPI, OUT_FM>, dim3(M / BM, N / BN), dim3(NT), Tile<BM>::SMEM_BYTES, s, At,
                   lda, Wt, ldw, C, ldc, K, cv);
    if (e != cudaSuccess) return e;
    add_launches(1);
    return cudaGetLastError();
}

template <int BM>
cudaError_t dispatch(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                     int epilogue, bool out_fm, cudaStream_t s) {
    switch (epilogue * 2 + (out_fm ? 1 : 0)) {
        case EPI_STORE * 2 + 0: return launch<BM, EPI_STORE, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
        case EPI_STORE * 2 + 1: return launch<BM, EPI_STORE, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
        case EPI_RESIDUAL * 2 + 0: return launch<BM, EPI_RESIDUAL, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
        case EPI_RESIDUAL * 2 + 1: return launch<BM, EPI_RESIDUAL, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
        case EPI_GELU * 2 + 0: return launch<BM, EPI_GELU, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
        case EPI_GELU * 2 + 1: return launch<BM, EPI_GELU, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
        default: return cudaErrorInvalidValue;
    }
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0, v = 148;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) v = 148;
        n = v;
    }
    return n;
}

// 32x32 tiles through shared memory (padded rows: no bank conflicts).
__global__ void transpose_pad_kernel(const float* __restrict__ in, int rows, int cols, float* __restrict__ out,
                                     int ld) {
    __shared__ float t[32][33];
    const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        t[i][threadIdx.x] = (r < rows && c < cols) ? in[(size_t)r * cols + c] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (c < cols && r < ld) out[(size_t)c * ld + r] = t[threadIdx.x][i];
    }
}

}  // namespace

cudaError_t transpose_pad(const float* in, int rows, int cols, float* out, int ld, cudaStream_t s) {
    if (rows <= 0 || cols <= 0 || ld < rows) return cudaErrorInvalidValue;
    dim3 grid((cols + 31) / 32, (ld + 31) / 32);
    transpose_pad_kernel<<<grid, dim3(32, 8), 0, s>>>(in, rows, cols, out, ld);
    add_launches(1);
    return cudaGetLastError();
}

// Tile choice (gemm_tile_rows, below).  When a tile height of 16, 32 or 64
// rows puts the whole projection in one wave (no more CTAs than SMs: the
// decode step of a small batch, where a launch lasts one tile's K loop), the
// smallest such height, whose warps have the shortest loop (at 64 rows:
// 16-row tiles for the 608-column projections, 32 for wqkv and the LM head, 64
// for in_proj and fc1, measured as the fastest of the three each).  Otherwise
// 32-row tiles (3 CTAs per SM) below 256 rows -- at 128 rows they beat 64-row
// tiles by 4-27% on in_proj, out_proj, wo, fc1 and fc2 -- and 64-row tiles
// from 256 rows on, where they match or beat 32-row ones on every projection
// (at 320, 384 and 1024 rows, 8 back-to-back launches per timing: fc2 at 1024
// rows 0.497 vs 0.483 of nominal FP32).  Every choice gives bit-identical
// results.
cudaError_t gemm_few_norm(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                          int epilogue, bool out_fm, const GemmNorm& nm, const GemmConv* cv, cudaStream_t s) {
    if (M <= 0 || M > GEMM_FEW_ROWS || N <= 0 || K <= 0 || K > SKINNY_MAX_K || N % BN || K % BK || lda % 4 ||
        ldw % 4 || ldc % 4 || lda < M || ldw < N || ldc < (out_fm ? M : N) || !nm.w ||
        (int64_t)K * lda >= (1ll << 31) || (int64_t)K * ldw >= (1ll << 31) ||
        ((uintptr_t)At | (uintptr_t)Wt | (uintptr_t)C) % 16)
        return cudaErrorInvalidValue;
    if (cv) {
        if (epilogue != EPI_CONV || out_fm || !cv->state || !cv->w || !cv->bias || cv->lo < 0 || cv->lo % BN ||
            cv->hi % BN || cv->hi <= cv->lo || cv->hi > N || cv->rows < 0 || cv->rows > M ||
            ((uintptr_t)cv->state | (uintptr_t)cv->w) % 16)
            return cudaErrorInvalidValue;
        return launch_skinny<EPI_CONV, false, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s, *cv, nm);
    }
    switch (epilogue * 2 + (out_fm ? 1 : 0)) {  // the forms the model uses
        case EPI_STORE * 2 + 0: return launch_skinny<EPI_STORE, false, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s, {}, nm);
        case EPI_RESIDUAL * 2 + 1:
            return launch_skinny<EPI_RESIDUAL, true, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s, {}, nm);
        case EPI_GELU * 2 + 1: return launch_skinny<EPI_GELU, true, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s, {}, nm);
        default: return cudaErrorInvalidValue;
    }
}

// The few-rows form beats every tile height (CUDA graphs of the decode
// projections) at up to 4 rows for every shape, and at 5-8 rows for the
// projections of 1024+ columns; 16-row tiles win for the 608-column ones there.
bool gemm_few_rows(int M, int N) { return M > 0 && M <= GEMM_FEW_ROWS && (M <= 4 || N >= 1024); }

int gemm_tile_rows(int M, int N) {
    const int64_t cols = N / BN, sms = sm_count();
    for (int t = 16; t <= 64; t *= 2)
        if (M % t == 0 && (int64_t)(M / t) * cols <= sms) return t;
    if (M % 32) return 16;
    if (M % 64) return 32;
    return M < 256 ? 32 : 64;
}

cudaError_t gemm_tiled(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                       int epilogue, bool out_fm, int tile_rows, cudaStream_t s) {
    if (tile_rows == 0) tile_rows = gemm_tile_rows(M, N);
    const bool skinny = tile_rows == 1;  // the few-rows form
    if (M <= 0 || N <= 0 || K <= 0 || (tile_rows != 1 && tile_rows != 16 && tile_rows != 32 && tile_rows != 64) ||
        M % tile_rows || (skinny && (M > SKINNY_MAX_ROWS || K > SKINNY_MAX_K)) ||
        N % BN || K % BK || lda % 4 || ldw % 4 || ldc % 4 || lda < M || ldw < N || ldc < (out_fm ? M : N) ||
        (int64_t)K * lda >= (1ll << 31) || (int64_t)K * ldw >= (1ll << 31) ||
        ((uintptr_t)At | (uintptr_t)Wt | (uintptr_t)C) % 16)
        return cudaErrorInvalidValue;
    if (tile_rows == 1) {
        switch (epilogue * 2 + (out_fm ? 1 : 0)) {
            case EPI_STORE * 2 + 0: return launch_skinny<EPI_STORE, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
            case EPI_STORE * 2 + 1: return launch_skinny<EPI_STORE, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
            case EPI_RESIDUAL * 2 + 0: return launch_skinny<EPI_RESIDUAL, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
            case EPI_RESIDUAL * 2 + 1: return launch_skinny<EPI_RESIDUAL, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
            case EPI_GELU * 2 + 0: return launch_skinny<EPI_GELU, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
            case EPI_GELU * 2 + 1: return launch_skinny<EPI_GELU, true>(At, lda, Wt, ldw, C, ldc, M, N, K, s);
            default: return cudaErrorInvalidValue;
        }
    }
    if (tile_rows == 16) return dispatch<16>(At, lda, Wt, ldw, C, ldc, M, N, K, epilogue, out_fm, s);
    if (tile_rows == 32) return dispatch<32>(At, lda, Wt, ldw, C, ldc, M, N, K, epilogue, out_fm, s);
    return dispatch<64>(At, lda, Wt, ldw, C, ldc, M, N, K, epilogue, out_fm, s);
}

cudaError_t gemm_conv(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                      int tile_rows, const GemmConv& cv, cudaStream_t s) {
    if (tile_rows == 0) tile_rows = gemm_tile_rows(M, N);
    const bool skinny = tile_rows == 1;  // the few-rows form
    if (M <= 0 || N <= 0 || K <= 0 || (tile_rows != 1 && tile_rows != 16 && tile_rows != 32 && tile_rows != 64) ||
        M % tile_rows || (skinny && (M > SKINNY_MAX_ROWS || K > SKINNY_MAX_K)) ||
        N % BN || K % BK || lda % 4 || ldw % 4 || ldc % 4 || lda < M || ldw < N || ldc < N || !cv.state || !cv.w ||
        !cv.bias ||
        (int64_t)K * lda >= (1ll << 31) || (int64_t)K * ldw >= (1ll << 31) ||
        cv.lo < 0 || cv.lo % BN || cv.hi % BN || cv.hi <= cv.lo || cv.hi > N || cv.rows < 0 || cv.rows > M ||
        ((uintptr_t)At | (uintptr_t)Wt | (uintptr_t)C | (uintptr_t)cv.state | (uintptr_t)cv.w) % 16)
        return cudaErrorInvalidValue;
    if (skinny) return launch_skinny<EPI_CONV, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv);
    if (tile_rows == 16) return launch<16, EPI_CONV, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv);
    if (tile_rows == 32) return launch<32, EPI_CONV, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv);
    return launch<64, EPI_CONV, false>(At, lda, Wt, ldw, C, ldc, M, N, K, s, cv);
}

cudaError_t gemm(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                 int epilogue, bool out_fm, cudaStream_t s) {
    return gemm_tiled(At, lda, Wt, ldw, C, ldc, M, N, K, epilogue, out_fm, 0, s);
}

}  // namespace krk
