// Mamba2 kernels: causal depthwise conv1d + SiLU, and the SSD state update as a
// single decode step and as a prefill scan over packed sequences (fp32).
//
// SSD recurrence (src/model.rs:661-685, per token, head h, row p, state n):
//   dt  = softplus(dt_raw[h] + dt_bias[h]);  dA = exp(dt * A[h])
//   s[p][n] = s[p][n]*dA + B[n]*(x[p]*dt);  y[p] = sum_n s[p][n]*C[n] + D[h]*x[p]
// followed by the gate y *= silu(z) (src/model.rs:688-690).
#include "common.cuh"
#include "kernels.h"

namespace krk {
namespace {

constexpr int SSD_P = 64;   // Mamba head dim (src/model.rs:25)
constexpr int SSD_N = 128;  // d_state (src/model.rs:22)

// ---------------------------------------------------------------------------
// Decode: one CTA per (sequence b, head h), 4 warps.  The head's 64x128 state
// block (32 KB) is streamed once: each warp walks 16 rows p, a row being 32
// lanes x float4 (one coalesced 512-byte load and store).  The state update
// uses the reference's unfused rounding, so the new state is bit-identical to
// the reference given the same x, B, dt; y[p] is a per-lane sequential sum of
// four products followed by a warp tree.  CONV: the head's 64 x channels go
// through the 4-tap causal conv + SiLU first, on a 3-slot state [B][H*P][3].
// ---------------------------------------------------------------------------
// RPW: state rows per warp.  16: one CTA per (sequence, head); 4 (small
// batches, no conv): the head's 64 rows over four CTAs of four warps
// (gridDim.z = 4), each warp's rows requested in one round trip -- the same
// arithmetic per row, so bitwise the same state and y.
template <bool CONV, int RPW>
__global__ void __launch_bounds__(128) ssd_step_kernel(SsdStepArgs a) {
    static_assert(RPW == 16 || (RPW == 4 && !CONV), "rows per warp");
    constexpr int G0 = RPW < 8 ? RPW : 8;  // rows requested up front
    const int b = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // The first 8 of this warp's 16 state rows are requested before anything
    // else (the active flag and the x, B, C, dt reads would otherwise put two
    // dependent round trips in front of the state stream); the other 8 after
    // the first are consumed (16 up front would cost occupancy: 122 registers).
    float* st = a.ssm + ((size_t)b * a.H + h) * (SSD_P * SSD_N) + lane * 4;
    const int pb = (blockIdx.z * 4 + warp) * RPW;
    float4 s0[G0], s1[G0];
#pragma unroll
    for (int i = 0; i < G0; ++i) s0[i] = __ldcs(reinterpret_cast<const float4*>(st + (pb + i) * SSD_N));
    // Launched behind the projection that writes x, B, C, dt and z: the state
    // (last written by this layer's update a step earlier, several launches
    // back) is already in flight.
    pdl_wait();
    pdl_trigger();
    if (a.active && !a.active[b]) return;
    __shared__ float xs[SSD_P], gs[SSD_P];
    const int c0 = h * SSD_P;
    if (tid < SSD_P) {
        const int c = c0 + tid;
        float xv;
        if (CONV) {
            float* cs = a.conv_state + ((size_t)b * a.H * SSD_P + c) * 3;
            const float s0 = cs[0], s1 = cs[1], s2 = cs[2];
            const float xr = a.x[(size_t)b * a.x_sb + c];
            const float* w = a.conv_w + (size_t)c * 4;
            const float val = s0 * w[0] + s1 * w[1] + s2 * w[2] + xr * w[3] + a.conv_b[c];
            cs[0] = s1;
            cs[1] = s2;
            cs[2] = xr;
            xv = silu(val);
        } else {
            xv = a.x[(size_t)b * a.x_sb + c];
        }
        xs[tid] = xv;
        gs[tid] = a.z ? silu(a.z[(size_t)b * a.z_sb + c]) : 1.0f;
    }
    const float dtv = softplus(a.dt[(size_t)b * a.dt_sb + h] + a.dt_bias[h]);
    const float dA = expf(dtv * a.a_neg[h]);
    const float dsk = a.dsk[h];
    const float4 B4 = *reinterpret_cast<const float4*>(a.bm + (size_t)b * a.bc_sb + lane * 4);
    const float4 C4 = *reinterpret_cast<const float4*>(a.cm + (size_t)b * a.bc_sb + lane * 4);
    __syncthreads();

    const bool gate = a.z != nullptr;
#pragma unroll
    for (int r0 = 0; r0 < RPW; r0 += G0) {
        const int pbase = pb + r0;
        if (r0 == 8) {
#pragma unroll
            for (int i = 0; i < G0; ++i) s1[i] = __ldcs(reinterpret_cast<const float4*>(st + (pb + 8 + i) * SSD_N));
        }
        float4* s = r0 == 0 ? s0 : s1;
#pragma unroll
        for (int i = 0; i < G0; ++i) {
            const int p = pbase + i;
            const float xp = xs[p];
            const float xdt = xp * dtv;
            float4 ns;
            ns.x = s[i].x * dA + B4.x * xdt;
            ns.y = s[i].y * dA + B4.y * xdt;
            ns.z = s[i].z * dA + B4.z * xdt;
            ns.w = s[i].w * dA + B4.w * xdt;
            __stcs(reinterpret_cast<float4*>(st + p * SSD_N), ns);
            float part = ns.x * C4.x;
            part = part + ns.y * C4.y;
            part = part + ns.z * C4.z;
            part = part + ns.w * C4.w;
            part = warp_sum(part);
            if (lane == 0) {
                float yv = part + dsk * xp;
                if (gate) yv = yv * gs[p];
                a.y[(size_t)b * a.y_sb + (size_t)(c0 + p) * a.y_sc] = yv;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Decode conv on the model's shift-register state [B][C][4] (src/model.rs:643-654).
// ---------------------------------------------------------------------------
__global__ void conv_step4_kernel(float* __restrict__ xbc, int64_t x_sb, float* __restrict__ state,
                                  const float* __restrict__ w, const float* __restrict__ bias, int B, int C,
                                  const uint8_t* __restrict__ active) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
    if (c >= C || (active && !active[b])) return;
    float4* sp = reinterpret_cast<float4*>(state + ((size_t)b * C + c) * 4);
    const float4 s = *sp;
    float* xp = xbc + (size_t)b * x_sb + c;
    const float x = *xp;
    const float4 wv = *reinterpret_cast<const float4*>(w + (size_t)c * 4);
    // after the shift the window is [s.y, s.z, s.w, x]
    const float val = s.y * wv.x + s.z * wv.y + s.w * wv.z + x * wv.w + bias[c];
    *sp = make_float4(s.y, s.z, s.w, x);
    *xp = silu(val);
}

// ---------------------------------------------------------------------------
// Prefill conv: one thread per (sequence, channel) walks the sequence's rows in
// order with the 4-slot window in registers (src/model.rs:399-410).
// ---------------------------------------------------------------------------
__global__ void conv_prefill4_kernel(const float* __restrict__ xin, int64_t x_rs, float* __restrict__ xout,
                                     int64_t o_rs, float* __restrict__ state, const float* __restrict__ w,
                                     const float* __restrict__ bias, const int32_t* __restrict__ cu, int C) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, sq = blockIdx.y;
    if (c >= C) return;
    const int r0 = cu[sq], r1 = cu[sq + 1];
    float4* sp = reinterpret_cast<float4*>(state + ((size_t)sq * C + c) * 4);
    float4 s = *sp;
    const float4 wv = *reinterpret_cast<const float4*>(w + (size_t)c * 4);
    const float bb = bias[c];
    int r = r0;
    for (; r + 4 <= r1; r += 4) {
        float xv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[i] = xin[(size_t)(r + i) * x_rs + c];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            s = make_float4(s.y, s.z, s.w, xv[i]);
            const float val = s.x * wv.x + s.y * wv.y + s.z * wv.z + s.w * wv.w + bb;
            xout[(size_t)(r + i) * o_rs + c] = silu(val);
        }
    }
    for (; r < r1; ++r) {
        s = make_float4(s.y, s.z, s.w, xin[(size_t)r * x_rs + c]);
        const float val = s.x * wv.x + s.y * wv.y + s.z * wv.z + s.w * wv.w + bb;
        xout[(size_t)r * o_rs + c] = silu(val);
    }
    *sp = s;
}

// ---------------------------------------------------------------------------
// Prefill scan: one CTA per (sequence, head), 256 threads.  Warp w owns state
// columns n = 16w .. 16w+15; lane l keeps rows p = 4(l/2) .. +3 of the column
// half 8(l%2) .. +7 (32 elements) in registers for the whole sequence.  Per
// token a lane reads its 8 B and 8 C values (16-byte loads at two addresses
// per warp), its 4 x values (one 16-byte load) and the token's (dt, dA); the y
// partial of a row over the lane's 8 columns is an FMA chain, the two halves
// of the warp's 16 columns meet by one shuffle, and the eight warps' partials
// meet in shared memory once per chunk and are added in warp order.  Tokens
// are staged SCAN_CH at a time (x, silu(z), B, C, dt, dA); y of the chunk is
// buffered and written coalesced.  The state update uses one FMA per element
// (s = fma(s, dA, B*xdt)), issued as packed pairs (__fmul2_rn / __ffma2_rn
// round each component like the scalar forms), so results agree with the
// sequential reference within rounding.
// CONV: conv + SiLU of the head's 64 x channels (src/model.rs:399-410) from
// the chunk's raw x and the 3 raw rows before it (the conv state, then the
// previous chunk's last rows): each output needs only its own window, so all
// threads compute the chunk's outputs at once, each with the reference's
// expression.
// ---------------------------------------------------------------------------
constexpr int SCAN_CH = 16;
constexpr int SCAN_YLD = SCAN_CH + 1;
constexpr int SCAN_WARPS = 8;
constexpr size_t SCAN_SMEM = sizeof(float) * (SCAN_CH * SSD_N * 2 + SCAN_CH * SSD_P * 3 + 3 * SSD_P +
                                              SCAN_CH * 2 + SSD_P * SCAN_YLD + SCAN_CH * SCAN_WARPS * SSD_P);

template <bool CONV, bool GATE>
__global__ void __launch_bounds__(256, 3) ssd_scan_kernel(SsdScanArgs a) {
    extern __shared__ __align__(16) float sm[];
    float* sB = sm;                       // [CH][N]
    float* sC = sB + SCAN_CH * SSD_N;     // [CH][N]
    float* sxr = sC + SCAN_CH * SSD_N;    // [CH][P] x as staged
    float* sxc = sxr + SCAN_CH * SSD_P;   // [CH][P] CONV: conv + SiLU of x
    float* sg = sxc + SCAN_CH * SSD_P;    // [CH][P] silu(z)
    float* xh = sg + SCAN_CH * SSD_P;     // [3][P] CONV: the raw x rows before the chunk, oldest first
    float* sdd = xh + 3 * SSD_P;          // [CH][2] (dt, dA)
    float* sy = sdd + 2 * SCAN_CH;        // [P][CH+1]
    float* syp = sy + SSD_P * SCAN_YLD;   // [CH][warps][P]: y partials over each warp's columns
    const float* xs = CONV ? sxc : sxr;   // x as the scan reads it

    const int h = blockIdx.x, sq = blockIdx.y;  // heads of a sequence adjacent: B, C shared in L2
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
    const int r0 = a.cu_seqlens ? a.cu_seqlens[sq] : sq * a.uniform_len;
    const int r1 = a.cu_seqlens ? a.cu_seqlens[sq + 1] : (sq + 1) * a.uniform_len;
    const float dtb = a.dt_bias[h], an = a.a_neg[h], dsk = a.dsk[h];
    const int c0 = h * SSD_P;
    const int row0 = 4 * (l >> 1), col0 = 16 * w + 8 * (l & 1);

    // s[r][j]: row row0 + r, columns col0 + 2j, +1
    float* st = a.ssm + (((size_t)sq * a.H + h) * SSD_P + row0) * SSD_N + col0;
    float2 s[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const float4 v0 = *reinterpret_cast<const float4*>(st + r * SSD_N);
        const float4 v1 = *reinterpret_cast<const float4*>(st + r * SSD_N + 4);
        s[r][0] = make_float2(v0.x, v0.y); s[r][1] = make_float2(v0.z, v0.w);
        s[r][2] = make_float2(v1.x, v1.y); s[r][3] = make_float2(v1.z, v1.w);
    }
    // CONV: this thread's channel (tid % 64: the same for all its outputs)
    float cw0 = 0.f, cw1 = 0.f, cw2 = 0.f, cw3 = 0.f, cb = 0.f;
    float* cst = nullptr;
    if (CONV) {
        const int c = c0 + (tid & (SSD_P - 1));
        cst = a.conv_state + ((size_t)sq * a.H * SSD_P + c) * 3;
        cw0 = a.conv_w[c * 4]; cw1 = a.conv_w[c * 4 + 1]; cw2 = a.conv_w[c * 4 + 2]; cw3 = a.conv_w[c * 4 + 3];
        cb = a.conv_b[c];
        if (tid < SSD_P) {
            xh[tid] = cst[0]; xh[SSD_P + tid] = cst[1]; xh[2 * SSD_P + tid] = cst[2];
        }
    }

    for (int base = r0; base < r1; base += SCAN_CH) {
        const int nt = min(SCAN_CH, r1 - base);
        __syncthreads();  // the previous chunk is done with every buffer
        for (int i = tid; i < nt * (SSD_N / 4); i += 256) {
            const int t = i / (SSD_N / 4), c4 = i % (SSD_N / 4);
            const size_t row = (size_t)(base + t);
            *reinterpret_cast<float4*>(sB + t * SSD_N + c4 * 4) =
                __ldg(reinterpret_cast<const float4*>(a.bm + row * a.bc_rs + c4 * 4));
            *reinterpret_cast<float4*>(sC + t * SSD_N + c4 * 4) =
                __ldg(reinterpret_cast<const float4*>(a.cm + row * a.bc_rs + c4 * 4));
        }
        for (int i = tid; i < nt * (SSD_P / 4); i += 256) {
            const int t = i / (SSD_P / 4), c4 = i % (SSD_P / 4);
            const size_t row = (size_t)(base + t);
            *reinterpret_cast<float4*>(sxr + t * SSD_P + c4 * 4) =
                __ldg(reinterpret_cast<const float4*>(a.x + row * a.x_rs + c0 + c4 * 4));
            if (GATE) {
                float4 zv = __ldg(reinterpret_cast<const float4*>(a.z + row * a.z_rs + c0 + c4 * 4));
                *reinterpret_cast<float4*>(sg + t * SSD_P + c4 * 4) =
                    make_float4(silu(zv.x), silu(zv.y), silu(zv.z), silu(zv.w));
            }
        }
        if (tid < nt) {
            const float dtv = softplus(a.dt[(size_t)(base + tid) * a.dt_rs + h] + dtb);
            sdd[2 * tid] = dtv;
            sdd[2 * tid + 1] = expf(dtv * an);
        }
        __syncthreads();
        if (CONV) {
            const int p = tid & (SSD_P - 1);
            auto raw = [&](int j) { return j >= 0 ? sxr[j * SSD_P + p] : xh[(j + 3) * SSD_P + p]; };
            for (int t = tid / SSD_P; t < nt; t += 256 / SSD_P) {
                // the window [x(t-3), x(t-2), x(t-1), x(t)] of src/model.rs:399-410
                const float val = raw(t - 3) * cw0 + raw(t - 2) * cw1 + raw(t - 1) * cw2 + raw(t) * cw3 + cb;
                sxc[t * SSD_P + p] = silu(val);
            }
            __syncthreads();  // every window read the old halo
            if (tid < SSD_P) {  // the raw rows before the next chunk
                const float n0 = raw(nt - 3), n1 = raw(nt - 2), n2 = raw(nt - 1);
                xh[p] = n0; xh[SSD_P + p] = n1; xh[2 * SSD_P + p] = n2;
            }
        }
        for (int t = 0; t < nt; ++t) {
            const float2 dd = *reinterpret_cast<const float2*>(sdd + 2 * t);
            const float2 dA2 = make_float2(dd.y, dd.y);
            const float4 xv = *reinterpret_cast<const float4*>(xs + t * SSD_P + row0);
            const float xr[4] = {xv.x, xv.y, xv.z, xv.w};
            const float4 b0 = *reinterpret_cast<const float4*>(sB + t * SSD_N + col0);
            const float4 b1 = *reinterpret_cast<const float4*>(sB + t * SSD_N + col0 + 4);
            const float4 q0 = *reinterpret_cast<const float4*>(sC + t * SSD_N + col0);
            const float4 q1 = *reinterpret_cast<const float4*>(sC + t * SSD_N + col0 + 4);
            const float2 bp[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                                  make_float2(b1.z, b1.w)};
            const float2 cp[4] = {make_float2(q0.x, q0.y), make_float2(q0.z, q0.w), make_float2(q1.x, q1.y),
                                  make_float2(q1.z, q1.w)};
            float part[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float xd = xr[r] * dd.x;
                const float2 xdt = make_float2(xd, xd);
                float2 ya = make_float2(0.f, 0.f);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    s[r][j] = __ffma2_rn(s[r][j], dA2, __fmul2_rn(bp[j], xdt));
                    ya = __ffma2_rn(s[r][j], cp[j], ya);
                }
                part[r] = ya.x + ya.y;
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) part[r] += __shfl_xor_sync(0xffffffffu, part[r], 1);
            if ((l & 1) == 0)
                *reinterpret_cast<float4*>(syp + (t * SCAN_WARPS + w) * SSD_P + row0) =
                    make_float4(part[0], part[1], part[2], part[3]);
        }
        __syncthreads();
        for (int i = tid; i < nt * SSD_P; i += 256) {  // y of the chunk: the warps' partials in order
            const int t = i / SSD_P, p = i % SSD_P;
            const float* yp = syp + t * SCAN_WARPS * SSD_P + p;
            float y = yp[0];
#pragma unroll
            for (int ww = 1; ww < SCAN_WARPS; ++ww) y = y + yp[ww * SSD_P];
            float yv = y + dsk * xs[t * SSD_P + p];
            if (GATE) yv = yv * sg[t * SSD_P + p];
            sy[p * SCAN_YLD + t] = yv;
        }
        __syncthreads();
        if (a.y_rs == 1) {  // feature-major output: each channel's rows are contiguous
            for (int i = tid; i < SSD_P * nt; i += 256) {
                const int pp = i / nt, t = i % nt;
                a.y[(size_t)(base + t) + (size_t)(c0 + pp) * a.y_cs] = sy[pp * SCAN_YLD + t];
            }
        } else {
            for (int i = tid; i < nt * SSD_P; i += 256) {
                const int t = i / SSD_P, pp = i % SSD_P;
                a.y[(size_t)(base + t) * a.y_rs + (size_t)(c0 + pp) * a.y_cs] = sy[pp * SCAN_YLD + t];
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        *reinterpret_cast<float4*>(st + r * SSD_N) = make_float4(s[r][0].x, s[r][0].y, s[r][1].x, s[r][1].y);
        *reinterpret_cast<float4*>(st + r * SSD_N + 4) = make_float4(s[r][2].x, s[r][2].y, s[r][3].x, s[r][3].y);
    }
    if (CONV) {
        __syncthreads();  // the last halo is written
        if (tid < SSD_P) {
            cst[0] = xh[tid]; cst[1] = xh[SSD_P + tid]; cst[2] = xh[2 * SSD_P + tid];
        }
    }
}

}  // namespace

cudaError_t ssd_step(const SsdStepArgs& a, bool conv, cudaStream_t s) {
    if (a.P != SSD_P || a.N != SSD_N || a.B <= 0 || a.H <= 0 || (a.bc_sb & 3) ||
        (((uintptr_t)a.bm | (uintptr_t)a.cm | (uintptr_t)a.ssm) & 15))
        return cudaErrorInvalidValue;
    cudaError_t e;
    if (conv) {
        e = launch_pdl(ssd_step_kernel<true, 16>, dim3(a.B, a.H), dim3(128), 0, s, a);
    } else if ((int64_t)a.B * a.H <= 148) {  // at most one CTA per SM: four CTAs per head, one round trip each
        e = launch_pdl(ssd_step_kernel<false, 4>, dim3(a.B, a.H, 4), dim3(128), 0, s, a);
    } else {
        e = launch_pdl(ssd_step_kernel<false, 16>, dim3(a.B, a.H), dim3(128), 0, s, a);
    }
    if (e != cudaSuccess) return e;
    add_launches(1);
    return cudaGetLastError();
}

cudaError_t conv_step4(float* xbc, int64_t x_sb, float* state, const float* w, const float* bias, int B, int C,
                       const uint8_t* active, cudaStream_t s) {
    if (B <= 0 || C <= 0 || (((uintptr_t)state | (uintptr_t)w) & 15)) return cudaErrorInvalidValue;
    dim3 grid((C + 127) / 128, B);
    conv_step4_kernel<<<grid, 128, 0, s>>>(xbc, x_sb, state, w, bias, B, C, active);
    add_launches(1);
    return cudaGetLastError();
}

cudaError_t conv_prefill4(const float* xin, int64_t x_rs, float* xout, int64_t o_rs, float* state, const float* w,
                          const float* bias, const int32_t* cu_seqlens, int S, int C, cudaStream_t s) {
    if (S <= 0 || C <= 0 || (((uintptr_t)state | (uintptr_t)w) & 15)) return cudaErrorInvalidValue;
    dim3 grid((C + 127) / 128, S);
    conv_prefill4_kernel<<<grid, 128, 0, s>>>(xin, x_rs, xout, o_rs, state, w, bias, cu_seqlens, C);
    add_launches(1);
    return cudaGetLastError();
}

cudaError_t ssd_scan(const SsdScanArgs& a, bool conv, cudaStream_t s) {
    if (a.P != SSD_P || a.N != SSD_N || a.S <= 0 || a.H <= 0 || (a.bc_rs & 3) || (a.x_rs & 3) ||
        (a.z && (a.z_rs & 3)) || (!a.cu_seqlens && a.uniform_len <= 0) ||
        (((uintptr_t)a.bm | (uintptr_t)a.cm | (uintptr_t)a.ssm | (uintptr_t)a.x | (uintptr_t)a.z) & 15))
        return cudaErrorInvalidValue;
    if (a.S > 65535) return cudaErrorInvalidValue;
    dim3 grid(a.H, a.S);
    cudaError_t e;
#define KRK_SCAN(CV, GT)                                                                              \
    {                                                                                                 \
        static DeviceOnce once;                                                                       \
        e = once.set_smem((const void*)ssd_scan_kernel<CV, GT>, SCAN_SMEM);                           \
        if (e != cudaSuccess) return e;                                                               \
        ssd_scan_kernel<CV, GT><<<grid, 256, SCAN_SMEM, s>>>(a);                                      \
    }
    if (conv) {
        if (a.z) KRK_SCAN(true, true) else KRK_SCAN(true, false)
    } else {
        if (a.z) KRK_SCAN(false, true) else KRK_SCAN(false, false)
    }
#undef KRK_SCAN
    add_launches(1);
    return cudaGetLastError();
}

}  // namespace krk
