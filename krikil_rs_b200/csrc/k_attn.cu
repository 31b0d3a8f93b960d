// Attention kernels: RoPE + KV-cache append + single-query softmax attention
// for decode (split over the cache like flash-decoding), and RoPE/append plus
// causal attention for prefill (fp32).
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace krk {
namespace {

// src/math.rs:70-124: the reference dot product (8 FMA lanes, fixed fold,
// unfused scalar tail).  a and b are 16-byte aligned shared or global rows.
KRK_DEV float dot_ref(const float* a, const float* b, int len) {
    float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f, l4 = 0.f, l5 = 0.f, l6 = 0.f, l7 = 0.f;
    const int chunks = len >> 3;
    for (int c = 0; c < chunks; ++c) {
        const float4 a0 = *reinterpret_cast<const float4*>(a + 8 * c);
        const float4 a1 = *reinterpret_cast<const float4*>(a + 8 * c + 4);
        const float4 b0 = *reinterpret_cast<const float4*>(b + 8 * c);
        const float4 b1 = *reinterpret_cast<const float4*>(b + 8 * c + 4);
        l0 = fmaf(a0.x, b0.x, l0); l1 = fmaf(a0.y, b0.y, l1);
        l2 = fmaf(a0.z, b0.z, l2); l3 = fmaf(a0.w, b0.w, l3);
        l4 = fmaf(a1.x, b1.x, l4); l5 = fmaf(a1.y, b1.y, l5);
        l6 = fmaf(a1.z, b1.z, l6); l7 = fmaf(a1.w, b1.w, l7);
    }
    float r = ((l0 + l4) + (l2 + l6)) + ((l1 + l5) + (l3 + l7));
    for (int i = chunks * 8; i < len; ++i) r = r + a[i] * b[i];
    return r;
}

// src/math.rs:243-257: rotate-half on the pair (i, i + dh/2) at position pos.
KRK_DEV void rope_pair(float& x0, float& x1, float c, float s) {
    const float a = x0, b = x1;
    x0 = a * c - b * s;
    x1 = a * s + b * c;
}
// (cos, sin) of pair i at position pos (src/math.rs:243-247): the angle is the
// reference's f32 product pos * inv_freq[i], with inv_freq[i] = 1/powf(theta,
// 2i/dh) computed on the host by the same libm powf the reference calls (the
// angle reaches ~2047 rad, so inv_freq must be exact: one ulp of it moves the
// angle by ~1e-4), and cos/sin from CUDA's sincosf (within 2 ulp).
KRK_DEV void rope_cs(const RopeFreqs& fr, int i, int pos, float& c, float& s) {
    const float ang = (float)pos * fr.f[i];
    sincosf(ang, &s, &c);
}

constexpr int AD_THREADS = 128;
constexpr int AD_TILE = 64;
constexpr int AD_RED = 512;

template <int DH>
struct AdLayout {
    static constexpr int DH4 = DH / 4;
    static constexpr int KLD = (DH4 & 1) ? DH : DH + 4;  // odd float4 stride: conflict-free row reads
    static constexpr int G = AD_THREADS / DH4;           // key groups in the PV phase
};

template <int DH>
size_t ad_smem_bytes(int split) {
    return sizeof(float) * (3 * DH + AD_RED + split + AD_TILE * AdLayout<DH>::KLD + 64);
}

KRK_DEV float block_reduce(float v, float* scratch, bool is_max) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = is_max ? warp_max(v) : warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = scratch[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = is_max ? fmaxf(r, scratch[w]) : r + scratch[w];
    return r;
}

template <int DH>
__global__ void __launch_bounds__(AD_THREADS) attn_decode_kernel(AttnDecodeArgs a, int max_splits) {
    using L = AdLayout<DH>;
    constexpr int HALF = DH / 2;
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;
    float* kn = qs + DH;
    float* vn = kn + DH;
    float* red = vn + DH;
    float* sc = red + AD_RED;
    float* tile = sc + a.split;
    float* scratch = tile + AD_TILE * L::KLD;
    // behind the projection that writes q, k and v: wait for it, then let the
    // merge (or the next projection) be scheduled behind this kernel's blocks
    pdl_wait();
    pdl_trigger();

    const int b = blockIdx.x, h = blockIdx.y, sp = blockIdx.z, tid = threadIdx.x;
    if (a.active && !a.active[b]) return;
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.ctx) {  // the host rejects these before launch
        if (tid == 0) check_fail(CHK_POSITION);
        return;
    }
    const int nkeys = pos + 1;
    const int j0 = sp * a.split;
    if (j0 >= nkeys) return;
    const int j1 = min(nkeys, j0 + a.split);
    const int nsplit = (nkeys + a.split - 1) / a.split;

    const size_t in_off = (size_t)b * a.in_sb + (size_t)h * a.in_sh;
    if (tid < DH) {
        qs[tid] = a.q[in_off + tid];
        kn[tid] = a.k[in_off + tid];
        vn[tid] = a.v[in_off + tid];
    }
    __syncthreads();
    if (tid < HALF) {  // src/model.rs:721-728
        float c, s;
        if (a.rope) {
            const float2 cs = a.rope[(size_t)pos * HALF + tid];
            c = cs.x;
            s = cs.y;
        } else {
            rope_cs(a.freq, tid, pos, c, s);
        }
        rope_pair(qs[tid], qs[tid + HALF], c, s);
        rope_pair(kn[tid], kn[tid + HALF], c, s);
    }
    __syncthreads();
    const size_t cbase = (size_t)b * a.c_sb + (size_t)h * a.c_sh;
    if (j1 == nkeys && tid < DH) {  // KV append (src/model.rs:730-733), done by the split holding slot pos
        a.kc[cbase + (size_t)pos * a.c_st + tid] = kn[tid];
        a.vc[cbase + (size_t)pos * a.c_st + tid] = vn[tid];
    }

    // scores (src/model.rs:742-748): dot(q_h, k_j) * (1/sqrt(dh))
    const float scale = 1.0f / sqrtf((float)DH);
    float mx = -INFINITY;
    for (int t0 = j0; t0 < j1; t0 += AD_TILE) {
        const int nk = min(AD_TILE, j1 - t0);
        for (int i = tid; i < nk * L::DH4; i += AD_THREADS) {
            const int r = i / L::DH4, c4 = i % L::DH4;
            float* dst = tile + r * L::KLD + c4 * 4;
            const int j = t0 + r;
            if (j == pos) *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(kn + c4 * 4);
            else cp_async16(dst, a.kc + cbase + (size_t)j * a.c_st + c4 * 4);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        if (tid < nk) {
            const float sv = dot_ref(qs, tile + tid * L::KLD, DH) * scale;
            sc[t0 - j0 + tid] = sv;
            mx = fmaxf(mx, sv);
        }
        __syncthreads();
    }
    // softmax over this split (src/math.rs:213-232)
    const float m = block_reduce(mx, scratch, true);
    const int n = j1 - j0;
    float lsum = 0.0f;
    for (int j = tid; j < n; j += AD_THREADS) {
        const float e = expf(sc[j] - m);
        sc[j] = e;
        lsum += e;
    }
    const float l = block_reduce(lsum, scratch, false);
    if (nsplit == 1) {
        const float inv = 1.0f / l;
        for (int j = tid; j < n; j += AD_THREADS) sc[j] = sc[j] * inv;
    }
    __syncthreads();

    // out += w_j * v_j (src/model.rs:752-759)
    const int g = tid / L::DH4, d4 = tid % L::DH4;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t0 = j0; t0 < j1; t0 += AD_TILE) {
        const int nk = min(AD_TILE, j1 - t0);
        for (int i = tid; i < nk * L::DH4; i += AD_THREADS) {
            const int r = i / L::DH4, c4 = i % L::DH4;
            float* dst = tile + r * L::KLD + c4 * 4;
            const int j = t0 + r;
            if (j == pos) *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(vn + c4 * 4);
            else cp_async16(dst, a.vc + cbase + (size_t)j * a.c_st + c4 * 4);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        if (g < L::G) {
            for (int r = g; r < nk; r += L::G) {
                const float w = sc[t0 - j0 + r];
                const float4 vv = *reinterpret_cast<const float4*>(tile + r * L::KLD + d4 * 4);
                o.x = o.x + w * vv.x;
                o.y = o.y + w * vv.y;
                o.z = o.z + w * vv.z;
                o.w = o.w + w * vv.w;
            }
        }
        __syncthreads();
    }
    if (g < L::G) *reinterpret_cast<float4*>(red + g * DH + d4 * 4) = o;
    __syncthreads();
    if (tid < DH) {
        float acc = red[tid];
        for (int gg = 1; gg < L::G; ++gg) acc = acc + red[gg * DH + tid];
        if (nsplit == 1) {
            a.out[(size_t)b * a.o_sb + (size_t)h * a.o_sh + (size_t)tid * a.o_sd] = acc;
        } else {
            float* wp = a.work + (((size_t)b * a.H + h) * max_splits + sp) * (DH + 2);
            wp[tid] = acc;
            if (tid == 0) {
                wp[DH] = m;
                wp[DH + 1] = l;
            }
        }
    }
}

// Split of 16*NW keys per CTA, 16 keys per warp, everything warp-private
// until the CTA's final merge: each warp requests its K and V rows at entry as
// bulk copies (one per lane and row, completing on two mbarriers; V stays in
// flight while the scores run), ropes its own copy of q, computes
// its scores with two lanes per key, its softmax partial (max, sum) with
// shuffles and its PV partial; the NW partials are merged after the CTA's only
// barrier.
//
// The score of key j is the reference dot (src/math.rs:89-124) split across a
// lane pair: the even lane accumulates FMA lanes 0-3 (first float4 of every
// 8-float chunk), the odd lane lanes 4-7, and the even lane folds
// ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)) and adds the unfused tail -- the same
// rounding as the single-thread dot.
constexpr int AW_KEYS = 16;  // keys per warp
constexpr int AW_WAIT_POLLS = 1 << 20;  // mbarrier polls before a copy wait gives up

template <int DH>
struct AwLayout {
    // K row stride in float4s = 2 (mod 4): the 8 lanes of one shared-memory
    // phase (4 keys x 2 halves) hit 8 distinct 16-byte bank groups.
    static constexpr int KLD = DH == 64 ? 72 : 88;
    static constexpr int ND = (DH + 31) / 32;
    // two mbarriers (16 B), K rows, V rows, q, partial; rounded to whole
    // float4s so every warp's region starts 16-byte aligned
    static constexpr int WARP_FLOATS = (4 + AW_KEYS * KLD + AW_KEYS * DH + DH + (DH + 2) + 3) / 4 * 4;
};
static_assert(AwLayout<64>::WARP_FLOATS % 4 == 0 && AwLayout<76>::WARP_FLOATS % 4 == 0, "alignment");
static_assert(AwLayout<64>::KLD % 8 == 0 && (AwLayout<64>::KLD / 4) % 4 == 2, "K stride");
static_assert((AwLayout<76>::KLD / 4) % 4 == 2 && AwLayout<76>::KLD >= 76, "K stride");

template <int DH>
size_t aw_smem_bytes(int nw) {
    return sizeof(float) * (size_t)nw * AwLayout<DH>::WARP_FLOATS;
}

template <int DH, int NW, bool BULK>
__global__ void __launch_bounds__(NW * 32) attn_decode_warp_kernel(AttnDecodeArgs a, int max_splits) {
    using L = AwLayout<DH>;
    constexpr int HALF = DH / 2, DH4 = DH / 4, SPLIT = NW * AW_KEYS, CHUNKS = DH / 8;
    extern __shared__ __align__(16) float sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + warp * L::WARP_FLOATS);  // [2]: K rows, V rows
    float* kt = sm + warp * L::WARP_FLOATS + 4;  // [16][KLD]
    float* vt = kt + AW_KEYS * L::KLD;           // [16][DH]
    float* qw = vt + AW_KEYS * DH;           // [DH]
    float* part = qw + DH;                   // [DH + 2]: o, max, sum
    pdl_trigger();  // the combine kernel may be scheduled behind the last blocks

    const int b = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
    const int j0 = sp * SPLIT;
    const int jw = j0 + warp * AW_KEYS;  // this warp's first key
    const size_t cbase = (size_t)b * a.c_sb + (size_t)h * a.c_sh;
    constexpr uint32_t ROW_BYTES = DH * sizeof(float);

    // BULK (cache rows apart, as the model's [ctx][heads*dh] rows): the copies
    // go out before the sequence's position is known -- learning it takes a
    // dependent global load -- one bulk copy per row and lane (lanes 0-15 K,
    // 16-31 V, each set completing on its own mbarrier) for every row of the
    // warp's block below the batch's key bound; rows past pos are masked in
    // the scores and the new row pos is overwritten once the copies landed.
    int nrows = 0;
    if (BULK) {
        const int rows_max = a.max_keys > 0 && a.max_keys < a.ctx ? a.max_keys : a.ctx;  // no pos + 1 exceeds it
        nrows = max(0, min(AW_KEYS, rows_max - jw));
        if (nrows > 0) {
            if (lane == 0) {
                mbar_init(&bar[0], 1);
                mbar_init(&bar[1], 1);
                fence_mbar_init();
                mbar_arrive_expect_tx(&bar[0], (uint32_t)nrows * ROW_BYTES);
                mbar_arrive_expect_tx(&bar[1], (uint32_t)nrows * ROW_BYTES);
            }
            __syncwarp();
            const int r = lane & 15;
            if (r < nrows) {
                if (lane < 16)
                    bulk_copy_g2s(kt + r * L::KLD, a.kc + cbase + (size_t)(jw + r) * a.c_st, ROW_BYTES, &bar[0]);
                else
                    bulk_copy_g2s(vt + r * DH, a.vc + cbase + (size_t)(jw + r) * a.c_st, ROW_BYTES, &bar[1]);
            }
        }
    }
    // Before leaving early, the copies of this warp land (bounded waits).
    auto drain = [&]() {
        if (BULK && nrows > 0) {
            mbar_wait_bounded(&bar[0], 0, AW_WAIT_POLLS);
            mbar_wait_bounded(&bar[1], 0, AW_WAIT_POLLS);
        }
    };
    const bool live = !a.active || a.active[b];
    const int pos = a.pos[b];
    if (!live || pos < 0 || pos >= a.ctx) {  // the host rejects bad positions before launch
        if (live && threadIdx.x == 0) check_fail(CHK_POSITION);
        drain();
        return;
    }
    // the copies above covered the rows below the batch's key bound only
    if (kChecked && BULK && a.max_keys > 0 && pos + 1 > a.max_keys) {
        if (threadIdx.x == 0) check_fail(CHK_POSITION);
        drain();
        return;
    }
    const int nkeys = pos + 1;
    if (j0 >= nkeys) {  // uniform over the CTA
        drain();
        return;
    }
    const int nsplit = (nkeys + SPLIT - 1) / SPLIT;
    const int nkw = max(0, min(AW_KEYS, nkeys - jw));  // this warp's key count
    const bool owner = nkw > 0 && pos < jw + nkw;
    const int rn = pos - jw;

    // Otherwise (rows back to back): 16-byte cp.async pieces, which the load
    // units merge into whole lines, in two commit groups; the row pos is
    // written from registers instead.
    if (!BULK) {
        for (int i = lane; i < nkw * DH4; i += 32) {
            const int r = i / DH4, c4 = i % DH4;
            if (jw + r != pos)
                cp_async16(kt + r * L::KLD + c4 * 4, a.kc + cbase + (size_t)(jw + r) * a.c_st + c4 * 4);
        }
        cp_async_commit();
        for (int i = lane; i < nkw * DH4; i += 32) {
            const int r = i / DH4, c4 = i % DH4;
            if (jw + r != pos) cp_async16(vt + r * DH + c4 * 4, a.vc + cbase + (size_t)(jw + r) * a.c_st + c4 * 4);
        }
        cp_async_commit();
    }

    // RoPE on q (every warp its own copy) and, in the warp holding slot pos,
    // on the new k, which is appended with v (src/model.rs:721-733).
    const size_t in_off = (size_t)b * a.in_sb + (size_t)h * a.in_sh;
    float kn[2][2], vn[2][2];  // the new row's pairs (i = lane, lane + 32)
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int i = lane + 32 * t;
        if (i >= HALF) break;
        float c, s;
        if (a.rope) {
            const float2 cs = a.rope[(size_t)pos * HALF + i];
            c = cs.x;
            s = cs.y;
        } else {
            rope_cs(a.freq, i, pos, c, s);
        }
        float q0 = a.q[in_off + i], q1 = a.q[in_off + i + HALF];
        rope_pair(q0, q1, c, s);
        qw[i] = q0;
        qw[i + HALF] = q1;
        if (owner) {
            float k0 = a.k[in_off + i], k1 = a.k[in_off + i + HALF];
            rope_pair(k0, k1, c, s);
            const float v0 = a.v[in_off + i], v1 = a.v[in_off + i + HALF];
            kn[t][0] = k0; kn[t][1] = k1;
            vn[t][0] = v0; vn[t][1] = v1;
            if (!BULK) {
                kt[rn * L::KLD + i] = k0;
                kt[rn * L::KLD + i + HALF] = k1;
                vt[rn * DH + i] = v0;
                vt[rn * DH + i + HALF] = v1;
            }
            float* kd = a.kc + cbase + (size_t)pos * a.c_st;
            float* vd = a.vc + cbase + (size_t)pos * a.c_st;
            kd[i] = k0;
            kd[i + HALF] = k1;
            vd[i] = v0;
            vd[i + HALF] = v1;
        }
    }
    // A bounded wait: a copy that never lands flags an error instead of hanging.
    bool ok = true;
    if (!BULK) {
        cp_async_wait<1>();
    } else {
        ok = nrows == 0 || mbar_wait_bounded(&bar[0], 0, AW_WAIT_POLLS);
        if (owner) {  // the copied row pos is the cache's old content
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int i = lane + 32 * t;
                if (i < HALF) {
                    kt[rn * L::KLD + i] = kn[t][0];
                    kt[rn * L::KLD + i + HALF] = kn[t][1];
                }
            }
        }
    }
    __syncwarp();

    // scores (src/model.rs:742-748): dot(q_h, k_j) * (1/sqrt(dh)), keys lane/2
    const float scale = 1.0f / sqrtf((float)DH);
    const int r = lane >> 1, hf = lane & 1;
    const bool valid = r < nkw;
    float sv = -INFINITY;
    {
        const float* kr = kt + (valid ? r : 0) * L::KLD + 4 * hf;
        const float* qr = qw + 4 * hf;
        float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            const float4 x = *reinterpret_cast<const float4*>(qr + 8 * c);
            const float4 y = *reinterpret_cast<const float4*>(kr + 8 * c);
            l0 = fmaf(x.x, y.x, l0); l1 = fmaf(x.y, y.y, l1);
            l2 = fmaf(x.z, y.z, l2); l3 = fmaf(x.w, y.w, l3);
        }
        const float l4 = __shfl_xor_sync(0xffffffffu, l0, 1), l5 = __shfl_xor_sync(0xffffffffu, l1, 1);
        const float l6 = __shfl_xor_sync(0xffffffffu, l2, 1), l7 = __shfl_xor_sync(0xffffffffu, l3, 1);
        float d = ((l0 + l4) + (l2 + l6)) + ((l1 + l5) + (l3 + l7));
        for (int i = CHUNKS * 8; i < DH; ++i) d = d + qw[i] * kt[(valid ? r : 0) * L::KLD + i];
        d = __shfl_sync(0xffffffffu, d, lane & ~1);  // the even lane's fold
        if (valid) sv = d * scale;
    }
    // softmax partial over the warp's keys (src/math.rs:213-232)
    const float mw = warp_max(sv);
    const float e = valid ? expf(sv - mw) : 0.0f;
    const float lw = warp_sum(hf == 0 ? e : 0.0f);
    if (!BULK) {
        cp_async_wait<0>();
    } else {
        ok = (nrows == 0 || mbar_wait_bounded(&bar[1], 0, AW_WAIT_POLLS)) && ok;
        if (owner) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int i = lane + 32 * t;
                if (i < HALF) {
                    vt[rn * DH + i] = vn[t][0];
                    vt[rn * DH + i + HALF] = vn[t][1];
                }
            }
        }
    }
    __syncwarp();

    // out += w_j * v_j (src/model.rs:752-759) over the warp's keys, in order
    float o[L::ND];
#pragma unroll
    for (int i = 0; i < L::ND; ++i) o[i] = 0.0f;
    for (int k = 0; k < nkw; ++k) {
        const float w = __shfl_sync(0xffffffffu, e, 2 * k);
#pragma unroll
        for (int i = 0; i < L::ND; ++i) {
            const int d = lane + 32 * i;
            if (d < DH) o[i] = o[i] + w * vt[k * DH + d];
        }
    }
#pragma unroll
    for (int i = 0; i < L::ND; ++i) {
        const int d = lane + 32 * i;
        if (d < DH) part[d] = o[i];
    }
    if (lane == 0) {
        part[DH] = nkw > 0 && ok ? mw : -INFINITY;  // a timed-out warp contributes nothing
        part[DH + 1] = ok ? lw : 0.0f;
        if (!ok && a.err) atomicOr(a.err, 1);
    }
    __syncthreads();

    // merge the warps' partials
    for (int d = threadIdx.x; d < DH; d += NW * 32) {
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) m = fmaxf(m, sm[w * L::WARP_FLOATS + 4 + AW_KEYS * (L::KLD + DH) + DH + DH]);
        float acc = 0.0f, l = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float* pw = sm + w * L::WARP_FLOATS + 4 + AW_KEYS * (L::KLD + DH) + DH;
            if (pw[DH] == -INFINITY) continue;  // a warp past the last key
            const float f = expf(pw[DH] - m);
            acc = acc + pw[d] * f;
            l = l + pw[DH + 1] * f;
        }
        if (nsplit == 1) {
            a.out[(size_t)b * a.o_sb + (size_t)h * a.o_sh + (size_t)d * a.o_sd] = acc * (1.0f / l);
        } else {
            float* wp = a.work + (((size_t)b * a.H + h) * max_splits + sp) * (DH + 2);
            wp[d] = acc;
            if (d == 0) {
                wp[DH] = m;
                wp[DH + 1] = l;
            }
        }
    }
    if (!ok) drain();  // give copies still in flight a last bounded chance before the CTA exits
}

// The failure path of the bounded copy waits, runnable on purpose: one warp
// arms an mbarrier for a 16-byte bulk copy as attn_decode_warp_kernel arms its
// K/V barriers and waits with the same bounded wait.  Without the copy nothing
// ever completes the phase, the wait gives up after `polls` polls, and the
// kernel flags it in *err as the attention kernel does, then returns (no copy
// is in flight when the block exits).
__global__ void wait_probe_kernel(const float* src, int polls, int copy, int* err) {
    __shared__ __align__(16) float buf[4];
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar, (uint32_t)sizeof(buf));
        if (copy) bulk_copy_g2s(buf, src, (uint32_t)sizeof(buf), &bar);
    }
    __syncwarp();
    const bool ok = mbar_wait_bounded(&bar, 0, polls);
    if (threadIdx.x == 0 && !ok && err) atomicOr(err, 1);
}

// Decode attention without split scratch: the AC_CTAS CTAs of one (sequence,
// head) form a thread-block cluster.  CTA r of the cluster takes the r-th of
// AC_CTAS equal ranges of the keys 0..pos (whole 16-key groups), so the
// cluster's CTAs finish together whatever the position.  A CTA works as
// attn_decode_kernel does on one split -- 64-key K tiles staged with cp.async
// for the scores, the softmax partial of its range, then 64-key V tiles for
// the weighted sum -- and keeps its partial (max, sum, unnormalised output) in
// shared memory.  After a cluster barrier CTA 0 merges the AC_CTAS partials
// through distributed shared memory and writes the output; a second cluster
// barrier keeps every CTA's shared memory alive until then.  No thread leaves
// early: every thread of every CTA reaches both cluster barriers, and the CTA
// barriers inside a range's work are taken by the whole CTA or skipped by the
// whole CTA (an empty range is CTA-uniform).
constexpr int AC_CTAS = 8;

// keys per CTA at most for a cache of ctx slots (a multiple of 16)
inline int ac_per_max(int ctx) { return ((ctx + AC_CTAS - 1) / AC_CTAS + 15) / 16 * 16; }

template <int DH>
size_t ac_smem_bytes(int ctx) {
    return sizeof(float) * (3 * DH + AD_RED + ac_per_max(ctx) + AD_TILE * AdLayout<DH>::KLD + 64 + DH + 4);
}

template <int DH>
__global__ void __cluster_dims__(1, 1, AC_CTAS) __launch_bounds__(AD_THREADS)
    attn_decode_cluster_kernel(AttnDecodeArgs a, int per_max) {
    using L = AdLayout<DH>;
    namespace cg = cooperative_groups;
    constexpr int HALF = DH / 2;
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;
    float* kn = qs + DH;
    float* vn = kn + DH;
    float* red = vn + DH;
    float* sc = red + AD_RED;
    float* tile = sc + per_max;
    float* scratch = tile + AD_TILE * L::KLD;
    float* cpart = scratch + 64;  // [DH + 2]: the CTA's unnormalised output, max, sum
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int b = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;

    const bool live = !a.active || a.active[b];
    const int pos = live ? a.pos[b] : -1;
    const bool ok = live && pos >= 0 && pos < a.ctx;  // the host rejects bad positions before launch
    if (live && !ok && rank == 0 && tid == 0) check_fail(CHK_POSITION);
    const int nkeys = ok ? pos + 1 : 0;
    const int per = ((nkeys + AC_CTAS - 1) / AC_CTAS + 15) / 16 * 16;  // <= per_max
    const int j0 = min(nkeys, rank * per), j1 = min(nkeys, j0 + per);

    if (j1 > j0) {  // uniform over the CTA
        const size_t in_off = (size_t)b * a.in_sb + (size_t)h * a.in_sh;
        if (tid < DH) {
            qs[tid] = a.q[in_off + tid];
            kn[tid] = a.k[in_off + tid];
            vn[tid] = a.v[in_off + tid];
        }
        __syncthreads();
        if (tid < HALF) {  // src/model.rs:721-728
            float c, s;
            if (a.rope) {
                const float2 cs = a.rope[(size_t)pos * HALF + tid];
                c = cs.x;
                s = cs.y;
            } else {
                rope_cs(a.freq, tid, pos, c, s);
            }
            rope_pair(qs[tid], qs[tid + HALF], c, s);
            rope_pair(kn[tid], kn[tid + HALF], c, s);
        }
        __syncthreads();
        const size_t cbase = (size_t)b * a.c_sb + (size_t)h * a.c_sh;
        if (j1 == nkeys && tid < DH) {  // KV append (src/model.rs:730-733), by the CTA holding slot pos
            a.kc[cbase + (size_t)pos * a.c_st + tid] = kn[tid];
            a.vc[cbase + (size_t)pos * a.c_st + tid] = vn[tid];
        }
        // scores (src/model.rs:742-748): dot(q_h, k_j) * (1/sqrt(dh))
        const float scale = 1.0f / sqrtf((float)DH);
        float mx = -INFINITY;
        for (int t0 = j0; t0 < j1; t0 += AD_TILE) {
            const int nk = min(AD_TILE, j1 - t0);
            for (int i = tid; i < nk * L::DH4; i += AD_THREADS) {
                const int r = i / L::DH4, c4 = i % L::DH4;
                float* dst = tile + r * L::KLD + c4 * 4;
                const int j = t0 + r;
                if (j == pos) *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(kn + c4 * 4);
                else cp_async16(dst, a.kc + cbase + (size_t)j * a.c_st + c4 * 4);
            }
            cp_async_commit();
            cp_async_wait<0>();
            __syncthreads();
            if (tid < nk) {
                const float sv = dot_ref(qs, tile + tid * L::KLD, DH) * scale;
                sc[t0 - j0 + tid] = sv;
                mx = fmaxf(mx, sv);
            }
            __syncthreads();
        }
        // softmax partial over this range (src/math.rs:213-232)
        const float m = block_reduce(mx, scratch, true);
        const int n = j1 - j0;
        float lsum = 0.0f;
        for (int j = tid; j < n; j += AD_THREADS) {
            const float e = expf(sc[j] - m);
            sc[j] = e;
            lsum += e;
        }
        const float l = block_reduce(lsum, scratch, false);
        __syncthreads();
        // out += w_j * v_j (src/model.rs:752-759)
        const int g = tid / L::DH4, d4 = tid % L::DH4;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int t0 = j0; t0 < j1; t0 += AD_TILE) {
            const int nk = min(AD_TILE, j1 - t0);
            for (int i = tid; i < nk * L::DH4; i += AD_THREADS) {
                const int r = i / L::DH4, c4 = i % L::DH4;
                float* dst = tile + r * L::KLD + c4 * 4;
                const int j = t0 + r;
                if (j == pos) *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(vn + c4 * 4);
                else cp_async16(dst, a.vc + cbase + (size_t)j * a.c_st + c4 * 4);
            }
            cp_async_commit();
            cp_async_wait<0>();
            __syncthreads();
            if (g < L::G) {
                for (int r = g; r < nk; r += L::G) {
                    const float w = sc[t0 - j0 + r];
                    const float4 vv = *reinterpret_cast<const float4*>(tile + r * L::KLD + d4 * 4);
                    o.x = o.x + w * vv.x;
                    o.y = o.y + w * vv.y;
                    o.z = o.z + w * vv.z;
                    o.w = o.w + w * vv.w;
                }
            }
            __syncthreads();
        }
        if (g < L::G) *reinterpret_cast<float4*>(red + g * DH + d4 * 4) = o;
        __syncthreads();
        if (tid < DH) {
            float acc = red[tid];
            for (int gg = 1; gg < L::G; ++gg) acc = acc + red[gg * DH + tid];
            cpart[tid] = acc;
        }
        if (tid == 0) {
            cpart[DH] = m;
            cpart[DH + 1] = l;
        }
    } else {
        if (tid < DH) cpart[tid] = 0.0f;
        if (tid == 0) {
            cpart[DH] = -INFINITY;
            cpart[DH + 1] = 0.0f;
        }
    }
    cluster.sync();  // every CTA partial written and visible across the cluster
    if (rank == 0 && ok && tid < DH) {
        float mp[AC_CTAS];
        float m = -INFINITY;
#pragma unroll
        for (int c = 0; c < AC_CTAS; ++c) {
            mp[c] = cluster.map_shared_rank(cpart, c)[DH];
            m = fmaxf(m, mp[c]);
        }
        float acc = 0.0f, l = 0.0f;
#pragma unroll
        for (int c = 0; c < AC_CTAS; ++c) {
            if (mp[c] == -INFINITY) continue;  // an empty range
            const float* pc = cluster.map_shared_rank(cpart, c);
            const float f = expf(mp[c] - m);
            acc = acc + pc[tid] * f;
            l = l + pc[DH + 1] * f;
        }
        a.out[(size_t)b * a.o_sb + (size_t)h * a.o_sh + (size_t)tid * a.o_sd] = acc * (1.0f / l);
    }
    cluster.sync();  // CTA 0 has read every partial: shared memory may go
}

constexpr int ACW_MIN_SPLITS = 9;  // the wide merge from this many splits per sequence on

// Merges the per-split (max, sum, unnormalised out) partials of one (b, h).
// Launched as a programmatic dependent of the split kernel: it reads the
// positions while that kernel drains, then waits for its partials.
__global__ void attn_combine_kernel(AttnDecodeArgs a, int max_splits) {
    const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    // Every block waits, also those with nothing to merge: this kernel's
    // completion then implies the split kernel's, which the next kernel (a
    // programmatic launch too) relies on for the outputs written unmerged.
    pdl_wait();
    pdl_trigger();
    if (a.active && !a.active[b]) return;
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.ctx) {
        if (threadIdx.x == 0) check_fail(CHK_POSITION);
        return;
    }
    const int nsplit = (pos + a.split) / a.split;
    if (nsplit <= 1 || d >= a.dh) return;
    // Fewer than ACW_MIN_SPLITS splits here: every partial this thread needs
    // is requested at once (one round trip), then merged in split order.
    const float* wp = a.work + ((size_t)b * a.H + h) * max_splits * (a.dh + 2);
    float mc[ACW_MIN_SPLITS - 1], lc[ACW_MIN_SPLITS - 1], oc[ACW_MIN_SPLITS - 1];
#pragma unroll
    for (int c = 0; c < ACW_MIN_SPLITS - 1; ++c) {
        const float* p = wp + c * (a.dh + 2);
        mc[c] = c < nsplit ? p[a.dh] : -INFINITY;
        lc[c] = c < nsplit ? p[a.dh + 1] : 0.0f;
        oc[c] = c < nsplit ? p[d] : 0.0f;
    }
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < ACW_MIN_SPLITS - 1; ++c) m = fmaxf(m, mc[c]);
    float l = 0.0f, o = 0.0f;
#pragma unroll
    for (int c = 0; c < ACW_MIN_SPLITS - 1; ++c) {
        if (c < nsplit) {
            const float e = expf(mc[c] - m);
            l = l + lc[c] * e;
            o = o + oc[c] * e;
        }
    }
    a.out[(size_t)b * a.o_sb + (size_t)h * a.o_sh + (size_t)d * a.o_sd] = o * (1.0f / l);
}

// The same merge for long caches (many splits per sequence): every load of a
// pass is independent of the others -- thread c reads split c's max and sum,
// and the weighted output sums run in groups of consecutive splits, one
// thread per dim and group -- so it costs a few memory latencies however many
// splits there are.  Also a programmatic dependent of the split kernel.
constexpr int ACW_THREADS = 256;

size_t acw_smem_bytes(int max_splits, int dh) {
    return sizeof(float) * (2 * (size_t)max_splits + (size_t)(ACW_THREADS / dh) * dh);
}

__global__ void __launch_bounds__(ACW_THREADS) attn_combine_wide_kernel(AttnDecodeArgs a, int max_splits) {
    extern __shared__ __align__(16) float cm[];
    __shared__ float mred[ACW_THREADS / 32];
    const int b = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    pdl_wait();  // in every block (see attn_combine_kernel)
    pdl_trigger();
    if (a.active && !a.active[b]) return;
    const int pos = a.pos[b];
    if (pos < 0 || pos >= a.ctx) {
        if (threadIdx.x == 0) check_fail(CHK_POSITION);
        return;
    }
    const int nsplit = (pos + a.split) / a.split;
    if (nsplit <= 1) return;
    const int dh = a.dh, st = dh + 2, groups = ACW_THREADS / dh;
    float* wt = cm;               // [max_splits]: split max, then its weight
    float* ls = cm + max_splits;  // [max_splits]: split sum
    float* po = ls + max_splits;  // [groups][dh]: weighted output sums
    const float* wp = a.work + ((size_t)b * a.H + h) * max_splits * st;
    float m = -INFINITY;
    for (int c = tid; c < nsplit; c += ACW_THREADS) {
        const float mc = wp[(size_t)c * st + dh];
        wt[c] = mc;
        ls[c] = wp[(size_t)c * st + dh + 1];
        m = fmaxf(m, mc);
    }
    m = warp_max(m);
    if ((tid & 31) == 0) mred[tid >> 5] = m;
    __syncthreads();
    m = mred[0];
#pragma unroll
    for (int w = 1; w < ACW_THREADS / 32; ++w) m = fmaxf(m, mred[w]);
    for (int c = tid; c < nsplit; c += ACW_THREADS) wt[c] = expf(wt[c] - m);
    __syncthreads();
    const int g = tid / dh, d = tid % dh;
    if (g < groups) {
        const int per = (nsplit + groups - 1) / groups;
        const int c0 = g * per, c1 = min(nsplit, c0 + per);
        float o = 0.0f;
#pragma unroll 8
        for (int c = c0; c < c1; ++c) o = o + wp[(size_t)c * st + d] * wt[c];
        po[g * dh + d] = o;
    }
    __syncthreads();
    if (tid < dh) {
        float o = 0.0f, l = 0.0f;
        for (int gg = 0; gg < groups; ++gg) o = o + po[gg * dh + tid];
        for (int c = 0; c < nsplit; ++c) l = l + ls[c] * wt[c];
        a.out[(size_t)b * a.o_sb + (size_t)h * a.o_sh + (size_t)tid * a.o_sd] = o * (1.0f / l);
    }
}

// ---------------------------------------------------------------------------
// Prefill: RoPE on q (in place) and k, append k and v to the cache
// (src/model.rs:489-511).  One thread per (row, head, pair i < dh/2).
// ---------------------------------------------------------------------------
__global__ void rope_kv_prefill_kernel(float* __restrict__ qkv, int64_t q_rs, float* __restrict__ kc,
                                       float* __restrict__ vc, int64_t c_sb, int64_t c_sh, int64_t c_st,
                                       const int32_t* __restrict__ cu, const int32_t* __restrict__ start, int S,
                                       int H, int dh, int total_rows, const RopeFreqs freq,
                                       const float2* __restrict__ rope) {
    const int half = dh / 2;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)total_rows * H * half) return;
    const int i = (int)(gid % half);
    const int h = (int)((gid / half) % H);
    const int row = (int)(gid / ((int64_t)half * H));
    int lo = 0, hi = S;  // sequence of this row: cu[s] <= row < cu[s+1]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (cu[mid] <= row) lo = mid; else hi = mid;
    }
    const int sq = lo;
    const int pos = start[sq] + (row - cu[sq]);
    float c, s;
    if (rope) {
        const float2 cs = rope[(size_t)pos * half + i];
        c = cs.x;
        s = cs.y;
    } else {
        rope_cs(freq, i, pos, c, s);
    }
    float* qr = qkv + (size_t)row * q_rs + (size_t)h * dh;
    float* kr = qkv + (size_t)row * q_rs + (size_t)H * dh + (size_t)h * dh;
    const float* vr = qkv + (size_t)row * q_rs + (size_t)2 * H * dh + (size_t)h * dh;
    rope_pair(qr[i], qr[i + half], c, s);
    float k0 = kr[i], k1 = kr[i + half];
    rope_pair(k0, k1, c, s);
    const size_t cb = (size_t)sq * c_sb + (size_t)h * c_sh + (size_t)pos * c_st;
    kc[cb + i] = k0;
    kc[cb + i + half] = k1;
    vc[cb + i] = vr[i];
    vc[cb + i + half] = vr[i + half];
}

// Causal attention for packed prefill rows (src/model.rs:519-548), a CTA per
// block of ROWS consecutive query rows of one sequence and one head, a warp per
// row.  The rows of a block share their sequence's K and V rows, so the CTA
// stages them in shared memory a tile of PF_KT keys at a time (cp.async, K
// tiles for the scores, then V tiles for the output) and every warp reads
// them from there.  Per row the arithmetic is the reference's: full reference
// dots (lane per key), the max and the sum of exponentials over all keys,
// then out[d] = sum_j (e_j / l) * v_j[d] in key order, lane d owning dims
// d + 32i.  Scores are kept per row in shared memory ([ROWS][kmax]).
constexpr int PF_KT = 64;
constexpr int PF_MAX_SMEM = 227 * 1024;

template <int DH>
struct PfLayout {
    static constexpr int KLD = ((DH / 4) & 1) ? DH : DH + 4;  // odd float4 row stride: conflict-free
};

template <int DH, int ROWS>
size_t pf_smem_bytes(int kmax) {
    return sizeof(float) * ((size_t)PF_KT * PfLayout<DH>::KLD + (size_t)ROWS * DH + (size_t)ROWS * kmax);
}

template <int DH, int ROWS>
__global__ void __launch_bounds__(ROWS * 32) attn_prefill_kernel(
    const float* __restrict__ qkv, int64_t q_rs, const float* __restrict__ kc, const float* __restrict__ vc,
    int64_t c_sb, int64_t c_sh, int64_t c_st, const int32_t* __restrict__ cu, const int32_t* __restrict__ start,
    const int2* __restrict__ blocks, int kmax, float* __restrict__ out, int64_t o_rs, int64_t o_cs) {
    constexpr int ND = (DH + 31) / 32, KLD = PfLayout<DH>::KLD, DH4 = DH / 4, NT = ROWS * 32;
    extern __shared__ __align__(16) float sm[];
    float* kt = sm;                   // [PF_KT][KLD]: the staged K or V tile
    float* qsh = kt + PF_KT * KLD;    // [ROWS][DH]
    float* sc = qsh + ROWS * DH;      // [ROWS][kmax]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, h = blockIdx.y;
    const int2 blk = blocks[blockIdx.x];
    const int sq = blk.x, r0 = blk.y;
    const int len = cu[sq + 1] - cu[sq];
    const int r = r0 + warp;  // this warp's row within its sequence
    const bool valid = r < len;
    const int nk = valid ? start[sq] + r + 1 : 0;
    const int nk_blk = start[sq] + min(r0 + ROWS, len);  // keys some row of the block needs
    if (kChecked && (r0 < 0 || r0 >= len || start[sq] < 0 || nk_blk > kmax)) {  // uniform over the CTA
        if (threadIdx.x == 0) check_fail(CHK_TABLE);
        return;
    }
    const size_t row = (size_t)(cu[sq] + (valid ? r : 0));
    float* qw = qsh + warp * DH;
    float* scw = sc + (size_t)warp * kmax;
    if (valid)
        for (int d = lane; d < DH; d += 32) qw[d] = qkv[row * q_rs + (size_t)h * DH + d];
    __syncwarp();
    const float scale = 1.0f / sqrtf((float)DH);
    const size_t cb = (size_t)sq * c_sb + (size_t)h * c_sh;

    auto stage = [&](const float* src, int t0, int nt) {
        __syncthreads();  // every warp is done with the previous tile
        for (int i = threadIdx.x; i < nt * DH4; i += NT) {
            const int rr = i / DH4, c4 = i % DH4;
            cp_async16(kt + rr * KLD + c4 * 4, src + cb + (size_t)(t0 + rr) * c_st + c4 * 4);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
    };

    // scores, lane j % 32 for key j as in the row-per-warp form
    float mx = -INFINITY;
    for (int t0 = 0; t0 < nk_blk; t0 += PF_KT) {
        const int nt = min(PF_KT, nk_blk - t0);
        stage(kc, t0, nt);
        const int jend = min(t0 + nt, nk);
        for (int j = t0 + lane; j < jend; j += 32) {
            const float sv = dot_ref(qw, kt + (j - t0) * KLD, DH) * scale;
            scw[j] = sv;
            mx = fmaxf(mx, sv);
        }
    }
    mx = warp_max(mx);
    float ls = 0.0f;
    for (int j = lane; j < nk; j += 32) {
        const float e = expf(scw[j] - mx);
        scw[j] = e;
        ls += e;
    }
    ls = warp_sum(ls);
    const float inv = 1.0f / ls;
    __syncwarp();
    float o[ND];
#pragma unroll
    for (int i = 0; i < ND; ++i) o[i] = 0.0f;
    for (int t0 = 0; t0 < nk_blk; t0 += PF_KT) {
        const int nt = min(PF_KT, nk_blk - t0);
        stage(vc, t0, nt);
        const int jend = min(t0 + nt, nk);
        for (int j = t0; j < jend; ++j) {
            const float w = scw[j] * inv;
            const float* vr = kt + (j - t0) * KLD;
#pragma unroll
            for (int i = 0; i < ND; ++i) {
                const int d = lane + 32 * i;
                if (d < DH) o[i] = o[i] + w * vr[d];
            }
        }
    }
    if (!valid) return;
#pragma unroll
    for (int i = 0; i < ND; ++i) {
        const int d = lane + 32 * i;
        if (d < DH) out[row * o_rs + (size_t)(h * DH + d) * o_cs] = o[i];
    }
}

}  // namespace

RopeFreqs rope_freqs(int dh, float theta) {
    RopeFreqs r{};
    for (int i = 0; i < dh / 2 && i < ROPE_MAX_PAIRS; ++i)
        r.f[i] = 1.0f / powf(theta, ((float)i * 2.0f) / (float)dh);  // src/math.rs:243-245, host libm
    return r;
}

size_t attn_decode_work_floats(int B, int H, int dh, int ctx, int split) {
    const int ms = (ctx + split - 1) / split;
    return (size_t)B * H * ms * (dh + 2);
}

cudaError_t attn_decode(const AttnDecodeArgs& args, cudaStream_t s) {
    AttnDecodeArgs a = args;
    if (!a.rope) a.freq = rope_freqs(a.dh, a.theta);
    if (a.split == 0) {  // clusters of AC_CTAS CTAs per (sequence, head), merged in distributed shared memory
        if (a.B <= 0 || a.H <= 0 || a.H > 65535 || a.ctx <= 0 || (a.dh != 64 && a.dh != 76) || (a.c_sb & 3) ||
            (a.c_sh & 3) || (a.c_st & 3) || (((uintptr_t)a.kc | (uintptr_t)a.vc) & 15))
            return cudaErrorInvalidValue;
        const dim3 grid(a.B, a.H, AC_CTAS);
        const int per_max = ac_per_max(a.ctx);
        cudaError_t e;
        if (a.dh == 76) {
            static DeviceOnce once;
            const size_t smem = ac_smem_bytes<76>(a.ctx);
            if (smem > 227 * 1024) return cudaErrorInvalidValue;
            if ((e = once.set_smem((const void*)attn_decode_cluster_kernel<76>, 227 * 1024)) != cudaSuccess) return e;
            attn_decode_cluster_kernel<76><<<grid, AD_THREADS, smem, s>>>(a, per_max);
        } else {
            static DeviceOnce once;
            const size_t smem = ac_smem_bytes<64>(a.ctx);
            if (smem > 227 * 1024) return cudaErrorInvalidValue;
            if ((e = once.set_smem((const void*)attn_decode_cluster_kernel<64>, 227 * 1024)) != cudaSuccess) return e;
            attn_decode_cluster_kernel<64><<<grid, AD_THREADS, smem, s>>>(a, per_max);
        }
        add_launches(1);
        return cudaGetLastError();
    }
    if (a.B <= 0 || a.H <= 0 || a.ctx <= 0 || a.split <= 0 || a.split % 64 || (a.dh != 64 && a.dh != 76) ||
        (a.c_sb & 3) || (a.c_sh & 3) || (a.c_st & 3) || (((uintptr_t)a.kc | (uintptr_t)a.vc) & 15))
        return cudaErrorInvalidValue;
    const int max_splits = (a.ctx + a.split - 1) / a.split;
    if (max_splits > 1 && !a.work) return cudaErrorInvalidValue;
    // blocks past the longest sequence would exit at once: leave them out
    const int keys = a.max_keys > 0 && a.max_keys < a.ctx ? a.max_keys : a.ctx;
    dim3 grid(a.B, a.H, (keys + a.split - 1) / a.split);
    cudaError_t e;
    if (a.split == 16 * 4 || a.split == 16 * 8) {
        const int nw = a.split / 16;
        const bool bulk = a.c_st != a.dh;
        const void* fns[8] = {(const void*)attn_decode_warp_kernel<64, 4, false>,
                              (const void*)attn_decode_warp_kernel<64, 4, true>,
                              (const void*)attn_decode_warp_kernel<64, 8, false>,
                              (const void*)attn_decode_warp_kernel<64, 8, true>,
                              (const void*)attn_decode_warp_kernel<76, 4, false>,
                              (const void*)attn_decode_warp_kernel<76, 4, true>,
                              (const void*)attn_decode_warp_kernel<76, 8, false>,
                              (const void*)attn_decode_warp_kernel<76, 8, true>};
        const int v = (a.dh == 76 ? 4 : 0) + (nw == 8 ? 2 : 0) + (bulk ? 1 : 0);
        const size_t smem = a.dh == 76 ? aw_smem_bytes<76>(nw) : aw_smem_bytes<64>(nw);
        static DeviceOnce once[8];
        if ((e = once[v].set_smem(fns[v], smem)) != cudaSuccess) return e;
        void* params[] = {&a, (void*)&max_splits};
        if ((e = cudaLaunchKernel(fns[v], grid, dim3(nw * 32), params, smem, s)) != cudaSuccess) return e;
    } else if (a.dh == 76) {
        static DeviceOnce once;
        const size_t smem = ad_smem_bytes<76>(a.split);
        if (smem > 227 * 1024) return cudaErrorInvalidValue;
        if ((e = once.set_smem((const void*)attn_decode_kernel<76>, 227 * 1024)) != cudaSuccess) return e;
        if ((e = launch_pdl(attn_decode_kernel<76>, grid, dim3(AD_THREADS), smem, s, a, max_splits)) != cudaSuccess)
            return e;
    } else {
        static DeviceOnce once;
        const size_t smem = ad_smem_bytes<64>(a.split);
        if (smem > 227 * 1024) return cudaErrorInvalidValue;
        if ((e = once.set_smem((const void*)attn_decode_kernel<64>, 227 * 1024)) != cudaSuccess) return e;
        if ((e = launch_pdl(attn_decode_kernel<64>, grid, dim3(AD_THREADS), smem, s, a, max_splits)) != cudaSuccess)
            return e;
    }
    add_launches(1);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // With one split in the grid (max_keys bounds every position), every
    // sequence has one split, which the split kernel already wrote as the
    // output, and the merge would find nothing to do: it is not launched.
    if (max_splits > 1 && grid.z > 1) {
        // splits of the longest sequence: many take the wide merge
        const bool wide = (keys + a.split - 1) / a.split >= ACW_MIN_SPLITS;
        const size_t cs = wide ? acw_smem_bytes(max_splits, a.dh) : 0;
        if (cs > 48 * 1024) {
            if (cs > 226 * 1024) return cudaErrorInvalidValue;
            static DeviceOnce once;
            if ((e = once.set_smem((const void*)attn_combine_wide_kernel, 226 * 1024)) != cudaSuccess) return e;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(a.B, a.H);
        cfg.blockDim = dim3(wide ? ACW_THREADS : 128);
        cfg.dynamicSmemBytes = cs;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = wide ? cudaLaunchKernelEx(&cfg, attn_combine_wide_kernel, a, max_splits)
                 : cudaLaunchKernelEx(&cfg, attn_combine_kernel, a, max_splits);
        if (e != cudaSuccess) return e;
        add_launches(1);
        e = cudaGetLastError();
    }
    return e;
}

cudaError_t wait_probe(const float* src, int polls, bool copy, int* err, cudaStream_t s) {
    if (polls < 1 || polls > AW_WAIT_POLLS || (copy && (!src || ((uintptr_t)src & 15)))) return cudaErrorInvalidValue;
    wait_probe_kernel<<<1, 32, 0, s>>>(src, polls, copy ? 1 : 0, err);
    add_launches(1);
    return cudaGetLastError();
}

cudaError_t rope_kv_prefill(float* qkv, int64_t q_rs, float* kc, float* vc, int64_t c_sb, int64_t c_sh,
                            int64_t c_st, const int32_t* cu_seqlens, const int32_t* start, int S, int H, int dh,
                            int total_rows, float theta, const float2* rope, cudaStream_t s) {
    if (S <= 0 || H <= 0 || dh <= 0 || (dh & 1) || dh > 2 * ROPE_MAX_PAIRS || total_rows <= 0)
        return cudaErrorInvalidValue;
    const int64_t n = (int64_t)total_rows * H * (dh / 2);
    rope_kv_prefill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(qkv, q_rs, kc, vc, c_sb, c_sh, c_st,
                                                                       cu_seqlens, start, S, H, dh, total_rows,
                                                                       rope_freqs(dh, theta), rope);
    add_launches(1);
    return cudaGetLastError();
}

int attn_prefill_rows(int kmax, int dh) {
    const size_t need = dh == 76 ? pf_smem_bytes<76, PF_ROWS>(kmax) : pf_smem_bytes<64, PF_ROWS>(kmax);
    return need <= PF_MAX_SMEM ? PF_ROWS : 1;
}

cudaError_t attn_prefill_check(const float* qkv, int64_t q_rs, const float* kc, const float* vc, int64_t c_sb,
                               int64_t c_sh, int64_t c_st, int nblocks, int rows_per_block, int H, int dh,
                               int kmax) {
    if (H <= 0 || nblocks <= 0 || kmax <= 0 || (dh != 64 && dh != 76) || (q_rs & 3) || (c_st & 3) ||
        (c_sh & 3) || (c_sb & 3) || (((uintptr_t)qkv | (uintptr_t)kc | (uintptr_t)vc) & 15) ||
        (rows_per_block != PF_ROWS && rows_per_block != 1))
        return cudaErrorInvalidValue;
    const bool wide = rows_per_block == PF_ROWS;
    const size_t smem = dh == 76 ? (wide ? pf_smem_bytes<76, PF_ROWS>(kmax) : pf_smem_bytes<76, 1>(kmax))
                                 : (wide ? pf_smem_bytes<64, PF_ROWS>(kmax) : pf_smem_bytes<64, 1>(kmax));
    return smem > PF_MAX_SMEM ? cudaErrorInvalidValue : cudaSuccess;
}

cudaError_t attn_prefill(const float* qkv, int64_t q_rs, const float* kc, const float* vc, int64_t c_sb,
                         int64_t c_sh, int64_t c_st, const int32_t* cu_seqlens, const int32_t* start,
                         const int2* blocks, int nblocks, int rows_per_block, int H, int dh, int kmax, float* out,
                         int64_t o_rs, int64_t o_cs, cudaStream_t s) {
    cudaError_t e = attn_prefill_check(qkv, q_rs, kc, vc, c_sb, c_sh, c_st, nblocks, rows_per_block, H, dh, kmax);
    if (e != cudaSuccess) return e;
    const bool wide = rows_per_block == PF_ROWS;
    const size_t smem = dh == 76 ? (wide ? pf_smem_bytes<76, PF_ROWS>(kmax) : pf_smem_bytes<76, 1>(kmax))
                                 : (wide ? pf_smem_bytes<64, PF_ROWS>(kmax) : pf_smem_bytes<64, 1>(kmax));
    const void* fns[4] = {(const void*)attn_prefill_kernel<64, 1>, (const void*)attn_prefill_kernel<64, PF_ROWS>,
                          (const void*)attn_prefill_kernel<76, 1>, (const void*)attn_prefill_kernel<76, PF_ROWS>};
    const int v = (dh == 76 ? 2 : 0) + (wide ? 1 : 0);
    static DeviceOnce once[4];
    if ((e = once[v].set_smem(fns[v], PF_MAX_SMEM)) != cudaSuccess) return e;
    dim3 grid(nblocks, H);
    void* params[] = {(void*)&qkv, (void*)&q_rs, (void*)&kc, (void*)&vc, (void*)&c_sb, (void*)&c_sh,
                      (void*)&c_st, (void*)&cu_seqlens, (void*)&start, (void*)&blocks, (void*)&kmax,
                      (void*)&out, (void*)&o_rs, (void*)&o_cs};
    if ((e = cudaLaunchKernel(fns[v], grid, dim3(rows_per_block * 32), params, smem, s)) != cudaSuccess) return e;
    add_launches(1);
    return cudaGetLastError();
}

}  // namespace krk
