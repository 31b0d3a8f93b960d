/*
 * krikil_oracle.c -- CPU ORACLE (test infrastructure only).
 *
 * A plain-C restatement of the krikil-rs fp32 inference path (Pebble-25M hybrid
 * Mamba2 + attention), used ONLY as the checker for the CUDA implementation:
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.  The
 * product (krikil_rs_b200/) never links, calls or falls back to this file.
 *
 * Parity pinning: the reference's full-model golden vectors
 * (test_reference_logits.json / test_reference_step_logits.json) need the real
 * Pebble-25M weights, which are not available, so full-model parity against the
 * reference is UNPINNED; what is pinned are the reference's own known-answer unit
 * tests (src/math.rs:266-297, src/sampler.rs:160-182), restated in
 * tests/test_oracle_cpu.py.  Everything else follows the reference line by line:
 *
 *   - arithmetic is evaluated in the reference's order with no FMA contraction
 *     (this file is compiled with -ffp-contract=off), except where the reference
 *     itself uses FMA (the AVX2 dot product, src/math.rs:89-124);
 *   - transcendental calls go to the same glibc libm entry points Rust's f32
 *     methods lower to (expf, logf, powf, sinf, cosf), and sqrtf is IEEE;
 *   - the one third-party piece, matrixmultiply 0.3.11's sgemm used by
 *     gemm_transb (src/math.rs:188-211), is restated from its published blocked
 *     algorithm in a second, selectable order (orc_set_prefill_gemm_order): the
 *     default prefill projections use the gemv dot order (the order the CUDA
 *     projections reproduce), and the restated sgemm order measures how far the
 *     reference's own prefill sits from it.  That restatement is unpinned
 *     against the crate itself (no Rust toolchain to run it).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#define EXPORT __attribute__((visibility("default")))

/* ---- model constants: src/model.rs:12-30 ---- */
enum {
    HIDDEN = 608, VOCAB = 2048, INTER = 2432, NLAYERS = 8, NHEADS = 8, HDIM = 76,
    DSTATE = 128, DCONV = 4, DINNER = 1216, MHDIM = 64, MHEADS = 19,
    DINPROJ = 2707, DXBC = 1472
};
static const float ROPE_THETA = 10000.0f;
static const float RMS_EPS = 1e-6f;
static const float MNORM_EPS = 1e-5f;

/* ------------------------------------------------------------------------- */
/* src/math.rs                                                                */
/* ------------------------------------------------------------------------- */

/* src/math.rs:3-6 */
EXPORT float orc_silu(float x) { return x / (1.0f + expf(-x)); }

/* src/math.rs:8-15 */
EXPORT float orc_softplus(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

/* src/math.rs:23-39: Abramowitz & Stegun formula 7.1.26 (published constants). */
static float as_erf(float x) {
    const float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f;
    const float a4 = -1.453152027f, a5 = 1.061405429f, p = 0.3275911f;
    float sign = x < 0.0f ? -1.0f : 1.0f;
    float ax = fabsf(x);
    float t = 1.0f / (1.0f + p * ax);
    float poly = ((((a5 * t + a4) * t) + a3) * t + a2) * t + a1;
    float y = 1.0f - poly * t * expf(-ax * ax);
    return sign * y;
}

/* src/math.rs:17-21; the f32 constant FRAC_1_SQRT_2 rounds to 0.70710677f */
EXPORT float orc_gelu(float x) { return 0.5f * x * (1.0f + as_erf(x * 0.70710678118654752f)); }

/* src/math.rs:41-54 */
EXPORT void orc_rms_norm(const float *x, const float *w, float eps, float *out, int dim) {
    float ss = 0.0f;
    for (int i = 0; i < dim; i++) ss += x[i] * x[i];
    float mean = ss / (float)dim;
    float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < dim; i++) out[i] = x[i] * scale * w[i];
}

/* src/math.rs:56-68 */
EXPORT void orc_rms_norm_inplace(float *x, const float *w, float eps, int dim) {
    float ss = 0.0f;
    for (int i = 0; i < dim; i++) ss += x[i] * x[i];
    float mean = ss / (float)dim;
    float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < dim; i++) x[i] = x[i] * scale * w[i];
}

/*
 * src/math.rs:70-124: dot product as the AVX2/FMA path computes it.  Lane j
 * (j = 0..7) accumulates a[j+8i]*b[j+8i] with a fused multiply-add; the lanes are
 * folded as ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)) (extract-high + add,
 * movehl + add, shuffle + add_ss), then the len%8 tail is added with separate
 * multiply and add.
 */
EXPORT float orc_dot(const float *a, const float *b, int len) {
    float l[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int chunks = len / 8;
    for (int c = 0; c < chunks; c++)
        for (int j = 0; j < 8; j++) l[j] = fmaf(a[8 * c + j], b[8 * c + j], l[j]);
    float s04 = l[0] + l[4], s15 = l[1] + l[5], s26 = l[2] + l[6], s37 = l[3] + l[7];
    float res = (s04 + s26) + (s15 + s37);
    for (int i = chunks * 8; i < len; i++) {
        float p = a[i] * b[i];
        res += p;
    }
    return res;
}

/* src/math.rs:130-153: rows >= 256 split into 64-row chunks across threads
 * (rayon there, OpenMP here); each row is one dot, so threading never changes
 * the result. */
EXPORT void orc_gemv(const float *w, const float *x, float *out, int rows, int cols) {
    if (rows >= 256) {
        int nchunks = (rows + 63) / 64;
#pragma omp parallel for schedule(dynamic, 1)
        for (int c = 0; c < nchunks; c++) {
            int r1 = (c + 1) * 64 < rows ? (c + 1) * 64 : rows;
            for (int r = c * 64; r < r1; r++) out[r] = orc_dot(w + (size_t)r * cols, x, cols);
        }
    } else {
        for (int r = 0; r < rows; r++) out[r] = orc_dot(w + (size_t)r * cols, x, cols);
    }
}

/*
 * src/math.rs:188-211 gemm_transb (C[m,n] = A[m,:] . B[n,:]) in the summation
 * order of matrixmultiply 0.3.11's sgemm, restated from its published
 * BLIS-style algorithm (the crate is a dependency the reference does not
 * vendor; Cargo.toml:11 pins 0.3.11 with default features, so no threading):
 * the K dimension is cut into blocks of KC = 256 (its f32 default); within a
 * block the 8x8 AVX/FMA micro-kernel keeps one accumulator per C element,
 * starting at zero and updated k by k with a fused multiply-add; the first
 * block stores C = 1.0 * ab (beta 0), every later block C = 1.0 * ab + 1.0 * C
 * (beta 1), which with alpha = beta = 1 is one rounded add whether or not the
 * store fuses it.  Packing, the M/N blocking and the masked edge tiles move
 * data only, so they do not change any element's order.
 */
static float sgemm_order_dot(const float *a, const float *b, int k) {
    enum { KC = 256 };
    float c = 0.0f;
    for (int k0 = 0; k0 < k; k0 += KC) {
        int k1 = k0 + KC < k ? k0 + KC : k;
        float ab = 0.0f;
        for (int kk = k0; kk < k1; kk++) ab = fmaf(a[kk], b[kk], ab);
        c = k0 == 0 ? ab : ab + c;
    }
    return c;
}

/* 0: each element is the gemv dot of src/math.rs:70-124 (the default, and the
 * order the CUDA projections reproduce bit for bit); 1: the restated
 * matrixmultiply sgemm order above.  Test infrastructure: set it only while
 * no prefill runs. */
static int g_prefill_gemm_order = 0;
EXPORT void orc_set_prefill_gemm_order(int order) { g_prefill_gemm_order = order; }
EXPORT int orc_prefill_gemm_order(void) { return g_prefill_gemm_order; }

EXPORT void orc_gemm_transb(const float *a, const float *b, float *c, int m, int k, int n) {
    const int mm = g_prefill_gemm_order == 1;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < m; i++)
        for (int r = 0; r < n; r++)
            c[(size_t)i * n + r] = mm ? sgemm_order_dot(a + (size_t)i * k, b + (size_t)r * k, k)
                                      : orc_dot(a + (size_t)i * k, b + (size_t)r * k, k);
}

/* src/math.rs:213-232 */
EXPORT void orc_softmax_inplace(float *x, int n) {
    if (n <= 0) return;
    float mx = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* src/math.rs:234-260: rotate-half RoPE, frequencies recomputed per pair */
EXPORT void orc_apply_rope(float *q, float *k, int pos, int nh, int hd, float theta) {
    int half = hd / 2;
    for (int h = 0; h < nh; h++) {
        float *qh = q + h * hd, *kh = k + h * hd;
        for (int i = 0; i < half; i++) {
            float invf = 1.0f / powf(theta, ((float)i * 2.0f) / (float)hd);
            float ang = (float)pos * invf;
            float c = cosf(ang), s = sinf(ang);
            float q0 = qh[i], q1 = qh[i + half];
            qh[i] = q0 * c - q1 * s;
            qh[i + half] = q0 * s + q1 * c;
            float k0 = kh[i], k1 = kh[i + half];
            kh[i] = k0 * c - k1 * s;
            kh[i + half] = k0 * s + k1 * c;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* src/model.rs                                                               */
/* ------------------------------------------------------------------------- */

/* Weight pointers (src/model.rs:86-117).  a_neg_exp = -exp(A_log) is computed
 * by orc_precompute_a (src/model.rs:273-274). */
typedef struct {
    const float *ln_w, *in_proj_w, *conv1d_w, *conv1d_b, *dt_bias, *a_neg_exp, *d, *norm_w, *out_proj_w;
    const float *ln1_w, *wqkv_w, *wo_w, *ln2_w, *fc1_w, *fc2_w;
} OrcLayer;

typedef struct {
    const float *wte, *lnf_w;
    OrcLayer layers[NLAYERS];
} OrcModel;

/* Per-sequence state (src/model.rs:119-159, 196-201): Mamba layers own
 * conv[1472*4] and ssm[19*64*128]; attention layers own k/v caches [ctx*608]. */
typedef struct {
    float *conv[NLAYERS], *ssm[NLAYERS], *kc[NLAYERS], *vc[NLAYERS];
    int64_t cur_len[NLAYERS];
    int64_t context_limit, current_pos;
} OrcState;

static int is_mamba(int i) { return i % 4 < 3; } /* src/model.rs:207, :261 */

EXPORT void orc_precompute_a(const float *a_log, float *a_neg_exp, int n) {
    for (int i = 0; i < n; i++) a_neg_exp[i] = -expf(a_log[i]);
}

/* One conv + SSD + gate + gated-norm token update: src/model.rs:643-693
 * (identical to the per-token body of prefill at :398-451). `row` is the
 * in_proj output [2707] = z | xBC | dt; writes y[1216] (normed). */
static void mamba_token(const OrcLayer *m, float *conv, float *ssm, const float *row, float *y) {
    const float *z = row, *xbc = row + DINNER, *dt = row + DINNER + DXBC;
    float conv_out[DXBC];
    for (int c = 0; c < DXBC; c++) {
        float *cs = conv + c * DCONV;
        cs[0] = cs[1];
        cs[1] = cs[2];
        cs[2] = cs[3];
        cs[3] = xbc[c];
        const float *cw = m->conv1d_w + c * DCONV;
        float val = cs[0] * cw[0] + cs[1] * cw[1] + cs[2] * cw[2] + cs[3] * cw[3] + m->conv1d_b[c];
        conv_out[c] = orc_silu(val);
    }
    const float *xs = conv_out, *bs = conv_out + DINNER, *cs_ = conv_out + DINNER + DSTATE;
    for (int h = 0; h < MHEADS; h++) {
        float dtv = orc_softplus(dt[h] + m->dt_bias[h]);
        float da = expf(dtv * m->a_neg_exp[h]);
        float dv = m->d[h];
        float *st = ssm + (size_t)h * MHDIM * DSTATE;
        for (int p = 0; p < MHDIM; p++) {
            float xp = xs[h * MHDIM + p];
            float xdt = xp * dtv;
            float *row_s = st + p * DSTATE;
            float sy = 0.0f;
            for (int n = 0; n < DSTATE; n++) {
                float ns = row_s[n] * da + bs[n] * xdt;
                row_s[n] = ns;
                sy += ns * cs_[n];
            }
            y[h * MHDIM + p] = sy + dv * xp;
        }
    }
    for (int i = 0; i < DINNER; i++) y[i] *= orc_silu(z[i]);
    orc_rms_norm_inplace(y, m->norm_w, MNORM_EPS, DINNER);
}

/* Single-query attention over cache rows 0..nkeys-1 for all heads:
 * src/model.rs:736-760 (and the per-query body of :519-548). out must be zeroed. */
static void attend(const float *q, const float *kc, const float *vc, int64_t nkeys, float *out, float *scores) {
    float scale = 1.0f / sqrtf((float)HDIM);
    for (int h = 0; h < NHEADS; h++) {
        const float *qh = q + h * HDIM;
        for (int64_t j = 0; j < nkeys; j++) scores[j] = orc_dot(qh, kc + j * HIDDEN + h * HDIM, HDIM) * scale;
        orc_softmax_inplace(scores, (int)nkeys);
        float *oh = out + h * HDIM;
        for (int64_t j = 0; j < nkeys; j++) {
            const float *vj = vc + j * HIDDEN + h * HDIM;
            float w = scores[j];
            for (int d = 0; d < HDIM; d++) oh[d] += w * vj[d];
        }
    }
}

/* src/model.rs:370-464 */
static void prefill_mamba(const OrcLayer *m, float *conv, float *ssm, float *x, int t) {
    float *h = malloc(sizeof(float) * (size_t)t * HIDDEN);
    float *zx = malloc(sizeof(float) * (size_t)t * DINPROJ);
    float *ys = malloc(sizeof(float) * (size_t)t * DINNER);
    float *out = malloc(sizeof(float) * (size_t)t * HIDDEN);
    for (int i = 0; i < t; i++) orc_rms_norm(x + (size_t)i * HIDDEN, m->ln_w, RMS_EPS, h + (size_t)i * HIDDEN, HIDDEN);
    orc_gemm_transb(h, m->in_proj_w, zx, t, HIDDEN, DINPROJ);
    for (int s = 0; s < t; s++) mamba_token(m, conv, ssm, zx + (size_t)s * DINPROJ, ys + (size_t)s * DINNER);
    orc_gemm_transb(ys, m->out_proj_w, out, t, DINNER, HIDDEN);
    for (size_t i = 0; i < (size_t)t * HIDDEN; i++) x[i] += out[i];
    free(h); free(zx); free(ys); free(out);
}

/* src/model.rs:466-583 */
static void prefill_attention(const OrcLayer *a, float *kc, float *vc, int64_t *cur_len, float *x, int t,
                              int64_t start_pos) {
    size_t tt = (size_t)t;
    float *h = malloc(sizeof(float) * tt * HIDDEN);
    float *qkv = malloc(sizeof(float) * tt * 3 * HIDDEN);
    float *qs = malloc(sizeof(float) * tt * HIDDEN);
    float *ao = calloc(tt * HIDDEN, sizeof(float));
    float *tmp = malloc(sizeof(float) * tt * INTER);
    float *tmp2 = malloc(sizeof(float) * tt * HIDDEN);
    for (int i = 0; i < t; i++) orc_rms_norm(x + i * HIDDEN, a->ln1_w, RMS_EPS, h + i * HIDDEN, HIDDEN);
    orc_gemm_transb(h, a->wqkv_w, qkv, t, HIDDEN, 3 * HIDDEN);
    for (int s = 0; s < t; s++) {
        float *row = qkv + (size_t)s * 3 * HIDDEN;
        float kcur[HIDDEN];
        memcpy(qs + (size_t)s * HIDDEN, row, sizeof(float) * HIDDEN);
        memcpy(kcur, row + HIDDEN, sizeof(float) * HIDDEN);
        orc_apply_rope(qs + (size_t)s * HIDDEN, kcur, (int)(start_pos + s), NHEADS, HDIM, ROPE_THETA);
        int64_t off = (*cur_len + s) * HIDDEN;
        memcpy(kc + off, kcur, sizeof(float) * HIDDEN);
        memcpy(vc + off, row + 2 * HIDDEN, sizeof(float) * HIDDEN);
    }
    int64_t total = *cur_len + t;
    float *scores = malloc(sizeof(float) * (size_t)total);
    for (int s = 0; s < t; s++) attend(qs + (size_t)s * HIDDEN, kc, vc, *cur_len + s + 1, ao + (size_t)s * HIDDEN, scores);
    free(scores);
    *cur_len = total;
    orc_gemm_transb(ao, a->wo_w, tmp2, t, HIDDEN, HIDDEN);
    for (size_t i = 0; i < tt * HIDDEN; i++) x[i] += tmp2[i];
    for (int i = 0; i < t; i++) orc_rms_norm(x + i * HIDDEN, a->ln2_w, RMS_EPS, h + i * HIDDEN, HIDDEN);
    orc_gemm_transb(h, a->fc1_w, tmp, t, HIDDEN, INTER);
    for (size_t i = 0; i < tt * INTER; i++) tmp[i] = orc_gelu(tmp[i]);
    orc_gemm_transb(tmp, a->fc2_w, tmp2, t, INTER, HIDDEN);
    for (size_t i = 0; i < tt * HIDDEN; i++) x[i] += tmp2[i];
    free(h); free(qkv); free(qs); free(ao); free(tmp); free(tmp2);
}

/* Status codes shared with the CUDA library's C ABI. */
enum { ORC_OK = 0, ORC_BAD_TOKEN = 1, ORC_CONTEXT_OVERFLOW = 2, ORC_EMPTY = 3 };

/* src/model.rs:316-368.  logits may be NULL. */
EXPORT int orc_forward_prefill(const OrcModel *md, OrcState *st, const uint32_t *tokens, int t, float *logits) {
    if (t <= 0) return ORC_EMPTY;                                     /* :317-319 */
    if (st->current_pos + t > st->context_limit) return ORC_CONTEXT_OVERFLOW; /* :321-327 */
    for (int i = 0; i < t; i++)
        if (tokens[i] >= VOCAB) return ORC_BAD_TOKEN;                 /* :333-335 */
    float *x = malloc(sizeof(float) * (size_t)t * HIDDEN);
    for (int i = 0; i < t; i++) memcpy(x + (size_t)i * HIDDEN, md->wte + (size_t)tokens[i] * HIDDEN, sizeof(float) * HIDDEN);
    for (int l = 0; l < NLAYERS; l++) {
        if (is_mamba(l)) prefill_mamba(&md->layers[l], st->conv[l], st->ssm[l], x, t);
        else prefill_attention(&md->layers[l], st->kc[l], st->vc[l], &st->cur_len[l], x, t, st->current_pos);
    }
    st->current_pos += t;
    if (logits) {
        float normed[HIDDEN];
        orc_rms_norm(x + (size_t)(t - 1) * HIDDEN, md->lnf_w, RMS_EPS, normed, HIDDEN);
        orc_gemv(md->wte, normed, logits, VOCAB, HIDDEN);
    }
    free(x);
    return ORC_OK;
}

/* src/model.rs:586-783.  logits may be NULL. */
EXPORT int orc_forward_step(const OrcModel *md, OrcState *st, uint32_t tok, float *logits) {
    if (tok >= VOCAB) return ORC_BAD_TOKEN;                           /* :588-590 */
    if (st->current_pos >= st->context_limit) return ORC_CONTEXT_OVERFLOW; /* :591-593 */
    int64_t pos = st->current_pos;
    float h[HIDDEN], nb[HIDDEN], zx[DINPROJ], y[DINNER], mo[HIDDEN], qkv[3 * HIDDEN];
    float ao[HIDDEN], mh[INTER];
    memcpy(h, md->wte + (size_t)tok * HIDDEN, sizeof h);
    for (int l = 0; l < NLAYERS; l++) {
        const OrcLayer *L = &md->layers[l];
        if (is_mamba(l)) {                                            /* :626-702 */
            orc_rms_norm(h, L->ln_w, RMS_EPS, nb, HIDDEN);
            orc_gemv(L->in_proj_w, nb, zx, DINPROJ, HIDDEN);
            mamba_token(L, st->conv[l], st->ssm[l], zx, y);
            orc_gemv(L->out_proj_w, y, mo, HIDDEN, DINNER);
            for (int i = 0; i < HIDDEN; i++) h[i] += mo[i];
        } else {                                                      /* :704-783 */
            orc_rms_norm(h, L->ln1_w, RMS_EPS, nb, HIDDEN);
            orc_gemv(L->wqkv_w, nb, qkv, 3 * HIDDEN, HIDDEN);
            float q[HIDDEN], k[HIDDEN];
            memcpy(q, qkv, sizeof q);
            memcpy(k, qkv + HIDDEN, sizeof k);
            orc_apply_rope(q, k, (int)pos, NHEADS, HDIM, ROPE_THETA);
            int64_t off = st->cur_len[l] * HIDDEN;
            memcpy(st->kc[l] + off, k, sizeof k);
            memcpy(st->vc[l] + off, qkv + 2 * HIDDEN, sizeof(float) * HIDDEN);
            st->cur_len[l] += 1;
            memset(ao, 0, sizeof ao);
            float *scores = malloc(sizeof(float) * (size_t)st->cur_len[l]);
            attend(q, st->kc[l], st->vc[l], st->cur_len[l], ao, scores);
            free(scores);
            orc_gemv(L->wo_w, ao, mo, HIDDEN, HIDDEN);
            for (int i = 0; i < HIDDEN; i++) h[i] += mo[i];
            orc_rms_norm(h, L->ln2_w, RMS_EPS, nb, HIDDEN);
            orc_gemv(L->fc1_w, nb, mh, INTER, HIDDEN);
            for (int i = 0; i < INTER; i++) mh[i] = orc_gelu(mh[i]);
            orc_gemv(L->fc2_w, mh, mo, HIDDEN, INTER);
            for (int i = 0; i < HIDDEN; i++) h[i] += mo[i];
        }
    }
    st->current_pos += 1;
    if (logits) {
        orc_rms_norm(h, md->lnf_w, RMS_EPS, nb, HIDDEN);
        orc_gemv(md->wte, nb, logits, VOCAB, HIDDEN);
    }
    return ORC_OK;
}

/* src/model.rs:221-229 (attention reset only rewinds current_len) */
EXPORT void orc_state_reset(OrcState *st) {
    st->current_pos = 0;
    for (int l = 0; l < NLAYERS; l++) {
        if (is_mamba(l)) {
            memset(st->conv[l], 0, sizeof(float) * DXBC * DCONV);
            memset(st->ssm[l], 0, sizeof(float) * MHEADS * MHDIM * DSTATE);
        } else {
            st->cur_len[l] = 0;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* src/sampler.rs:43-80 (repetition penalty over the SET of context tokens,   */
/* then first-maximum greedy argmax; the lowest index wins ties)              */
/* ------------------------------------------------------------------------- */
EXPORT uint32_t orc_sample_greedy(const float *logits, int vocab, const uint32_t *ctx, int nctx, float penalty,
                                  float *scratch) {
    memcpy(scratch, logits, sizeof(float) * (size_t)vocab);
    if (fabsf(penalty - 1.0f) > 1e-4f) {
        unsigned char *seen = calloc((size_t)vocab, 1);
        for (int i = 0; i < nctx; i++)
            if (ctx[i] < (uint32_t)vocab) seen[ctx[i]] = 1;
        for (int tkn = 0; tkn < vocab; tkn++) {
            if (!seen[tkn]) continue;
            float l = scratch[tkn];
            scratch[tkn] = l > 0.0f ? l / penalty : l * penalty;
        }
        free(seen);
    }
    int best = 0;
    float bv = -INFINITY;
    for (int i = 0; i < vocab; i++)
        if (scratch[i] > bv) { bv = scratch[i]; best = i; }
    return (uint32_t)best;
}

/* ------------------------------------------------------------------------- */
/* Stochastic sampling (src/sampler.rs:83-152) and its random stream.          */
/*                                                                             */
/* The reference draws from rand 0.8's StdRng, which is rand_chacha 0.3's      */
/* ChaCha12Rng, seeded by rand_core 0.6's SeedableRng::seed_from_u64; neither  */
/* crate's source is in the reference tree.  Restated from the published       */
/* algorithms:                                                                 */
/*   - seed_from_u64: 8 key words from a PCG32 (XSH-RR) sequence: the 64-bit   */
/*     state advances first (state = state*6364136223846793005 +               */
/*     11634580027462260723), the output is ((state>>18)^state)>>27 rotated    */
/*     right by state>>59, stored little-endian;                               */
/*   - ChaCha with 12 rounds (6 column + diagonal double rounds), the          */
/*     "expand 32-byte k" constants, a 64-bit block counter in words 12-13     */
/*     and a zero 64-bit stream id in words 14-15; next_u32 returns the        */
/*     keystream's 32-bit words in order (block n/16, word n%16);              */
/*   - Rng::gen::<f32>() (Standard): (next_u32 >> 8) * 2^-24, in [0, 1).       */
/* The ChaCha block function is checked against the published ChaCha20 test   */
/* vectors (same code with 20 rounds), and the keyed generator (key layout,    */
/* counter and stream words, 12 rounds, word order) against the value-         */
/* stability known answers of rand 0.8's StdRng and rand_chacha 0.3's          */
/* ChaCha20Rng; the PCG expansion and the f32 conversion have no vectors, so   */
/* the seeded stream as a whole stays unpinned against the reference.          */
/* ------------------------------------------------------------------------- */
static uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

#define QR(a, b, c, d)                                                                                   \
    do {                                                                                                 \
        a += b; d ^= a; d = rotl32(d, 16);                                                               \
        c += d; b ^= c; b = rotl32(b, 12);                                                               \
        a += b; d ^= a; d = rotl32(d, 8);                                                                \
        c += d; b ^= c; b = rotl32(b, 7);                                                                \
    } while (0)

/* One ChaCha block: 16 input words (constants, key, counter, stream) -> out. */
EXPORT void orc_chacha_block(const uint32_t in[16], int rounds, uint32_t out[16]) {
    uint32_t x[16];
    memcpy(x, in, sizeof(x));
    for (int r = 0; r < rounds; r += 2) {
        QR(x[0], x[4], x[8], x[12]);
        QR(x[1], x[5], x[9], x[13]);
        QR(x[2], x[6], x[10], x[14]);
        QR(x[3], x[7], x[11], x[15]);
        QR(x[0], x[5], x[10], x[15]);
        QR(x[1], x[6], x[11], x[12]);
        QR(x[2], x[7], x[8], x[13]);
        QR(x[3], x[4], x[9], x[14]);
    }
    for (int i = 0; i < 16; i++) out[i] = x[i] + in[i];
}

/* Sampler random state: key[8], then the index of the next keystream word
 * (lo, hi). */
EXPORT void orc_rng_seed(uint64_t seed, uint32_t st[10]) {
    uint64_t s = seed;
    for (int i = 0; i < 8; i++) {
        s = s * 6364136223846793005ULL + 11634580027462260723ULL;
        const uint32_t xs = (uint32_t)(((s >> 18) ^ s) >> 27);
        const uint32_t rot = (uint32_t)(s >> 59);
        st[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
    }
    st[8] = 0;
    st[9] = 0;
}

EXPORT uint32_t orc_rng_next_u32(uint32_t st[10]) {
    const uint64_t n = (uint64_t)st[8] | ((uint64_t)st[9] << 32);
    const uint64_t blk = n >> 4;
    uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
    for (int i = 0; i < 8; i++) in[4 + i] = st[i];
    in[12] = (uint32_t)blk;
    in[13] = (uint32_t)(blk >> 32);
    in[14] = 0;
    in[15] = 0;
    uint32_t out[16];
    orc_chacha_block(in, 12, out);
    const uint64_t n1 = n + 1;
    st[8] = (uint32_t)n1;
    st[9] = (uint32_t)(n1 >> 32);
    return out[n & 15];
}

EXPORT float orc_rng_f32(uint32_t st[10]) { return (float)(orc_rng_next_u32(st) >> 8) * (1.0f / 16777216.0f); }

typedef struct {
    float v;
    uint32_t id;
} OrcCand;

/* Descending by value; equal values (which the reference's unstable sort
 * leaves in an unspecified order) by ascending id; NaN after everything. */
static int cand_cmp(const void *pa, const void *pb) {
    const OrcCand *a = pa, *b = pb;
    const int na = isnan(a->v), nb = isnan(b->v);
    if (na || nb) return na == nb ? (a->id < b->id ? -1 : (a->id > b->id)) : (na ? 1 : -1);
    if (a->v > b->v) return -1;
    if (a->v < b->v) return 1;
    return a->id < b->id ? -1 : (a->id > b->id);
}

/* src/sampler.rs:43-152 with temperature > 1e-6 (the greedy branch is
 * orc_sample_greedy).  rng: the state above, advanced by one word. */
EXPORT uint32_t orc_sample(const float *logits, int vocab, const uint32_t *ctx, int nctx, float temperature, float top_p,
                           int top_k, float penalty, uint32_t rng[10]) {
    float *m = malloc(sizeof(float) * (size_t)vocab);
    memcpy(m, logits, sizeof(float) * (size_t)vocab);
    if (fabsf(penalty - 1.0f) > 1e-4f) { /* :50-66 */
        unsigned char *seen = calloc((size_t)vocab, 1);
        for (int i = 0; i < nctx; i++)
            if (ctx[i] < (uint32_t)vocab) seen[ctx[i]] = 1;
        for (int t = 0; t < vocab; t++)
            if (seen[t]) m[t] = m[t] > 0.0f ? m[t] / penalty : m[t] * penalty;
        free(seen);
    }
    const float inv_temp = 1.0f / temperature; /* :82-86 */
    OrcCand *c = malloc(sizeof(OrcCand) * (size_t)vocab);
    for (int i = 0; i < vocab; i++) {
        c[i].v = m[i] * inv_temp;
        c[i].id = (uint32_t)i;
    }
    qsort(c, (size_t)vocab, sizeof(OrcCand), cand_cmp); /* :88-96 */
    int n = (top_k > 0 && top_k < vocab) ? top_k : vocab; /* :98-101 */
    const float mx = c[0].v;                                /* :103-118 */
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        c[i].v = expf(c[i].v - mx);
        sum += c[i].v;
    }
    const float inv_sum = 1.0f / sum;
    for (int i = 0; i < n; i++) c[i].v *= inv_sum;
    if (top_p < 1.0f) { /* :120-139 */
        float cum = 0.0f;
        int cut = n;
        for (int i = 0; i < n; i++) {
            cum += c[i].v;
            if (cum >= top_p) {
                cut = i + 1 < n ? i + 1 : n;
                break;
            }
        }
        n = cut;
        float ns = 0.0f;
        for (int i = 0; i < n; i++) ns += c[i].v;
        const float inv_ns = 1.0f / ns;
        for (int i = 0; i < n; i++) c[i].v *= inv_ns;
    }
    const float r = orc_rng_f32(rng); /* :141-151 */
    float acc = 0.0f;
    uint32_t pick = c[0].id;
    for (int i = 0; i < n; i++) {
        acc += c[i].v;
        if (r <= acc) {
            pick = c[i].id;
            break;
        }
    }
    free(c);
    free(m);
    return pick;
}

/* ------------------------------------------------------------------------- */
/* Stand-alone forms of the fused layer ops, on the synthetic benchmark       */
/* layouts.  Each is the reference's arithmetic for that op, generalised to   */
/* the benchmark's sizes.                                                     */
/* ------------------------------------------------------------------------- */

/* y = rmsnorm(x*silu(z))*w + res per row: the gate of src/model.rs:688-690,
 * rms_norm_inplace (src/math.rs:56-68), then a residual add (:699-701). */
EXPORT void orc_gated_rmsnorm_residual(const float *x, const float *z, const float *res, const float *w, float eps,
                                       float *y, int64_t rows, int dim) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * dim, *zr = z + r * dim, *rr = res + r * dim;
        float *yr = y + r * dim;
        for (int i = 0; i < dim; i++) yr[i] = xr[i] * orc_silu(zr[i]);
        orc_rms_norm_inplace(yr, w, eps, dim);
        for (int i = 0; i < dim; i++) yr[i] += rr[i];
    }
}

/* Plain RMSNorm over rows (src/math.rs:41-54). */
EXPORT void orc_rms_norm_rows(const float *x, const float *w, float eps, float *y, int64_t rows, int dim) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) orc_rms_norm(x + r * dim, w, eps, y + r * dim, dim);
}

/*
 * Decode RoPE + KV append + single-query attention on a [B,H,T,Dh] cache:
 * src/model.rs:717-760 per sequence, with head dim `dh` and per-sequence
 * positions.  q,k,v: [B,H,Dh]; kc,vc: [B,H,ctx,Dh]; out: [B,H,Dh].
 */
EXPORT void orc_rope_kv_attn_decode(const float *q, const float *k, const float *v, float *kc, float *vc,
                                    const int32_t *pos, float *out, int bsz, int nh, int dh, int ctx, float theta) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < bsz; b++) {
        float *qb = malloc(sizeof(float) * nh * dh), *kb = malloc(sizeof(float) * nh * dh);
        memcpy(qb, q + (size_t)b * nh * dh, sizeof(float) * nh * dh);
        memcpy(kb, k + (size_t)b * nh * dh, sizeof(float) * nh * dh);
        orc_apply_rope(qb, kb, pos[b], nh, dh, theta);
        int64_t nk = (int64_t)pos[b] + 1;
        float *scores = malloc(sizeof(float) * (size_t)nk);
        float scale = 1.0f / sqrtf((float)dh);
        for (int h = 0; h < nh; h++) {
            size_t base = ((size_t)b * nh + h) * (size_t)ctx * dh;
            memcpy(kc + base + (size_t)pos[b] * dh, kb + h * dh, sizeof(float) * dh);
            memcpy(vc + base + (size_t)pos[b] * dh, v + ((size_t)b * nh + h) * dh, sizeof(float) * dh);
            for (int64_t j = 0; j < nk; j++) scores[j] = orc_dot(qb + h * dh, kc + base + j * dh, dh) * scale;
            orc_softmax_inplace(scores, (int)nk);
            float *o = out + ((size_t)b * nh + h) * dh;
            for (int d = 0; d < dh; d++) o[d] = 0.0f;
            for (int64_t j = 0; j < nk; j++) {
                const float *vj = vc + base + j * dh;
                for (int d = 0; d < dh; d++) o[d] += scores[j] * vj[d];
            }
        }
        free(scores); free(qb); free(kb);
    }
}

/*
 * One token of causal depthwise conv (kernel 4) + SiLU on `nch` channels whose
 * state holds the previous 3 inputs [t-3,t-2,t-1] (the reference's 4-slot
 * shift register of src/model.rs:643-654 minus its dead oldest slot), followed
 * by the Mamba2 SSD update of src/model.rs:661-685 for `nh` heads of `p` x
 * channels with B, C [n] given directly.  Used for both the one-step benchmark
 * and (looped over t) the prefill scan.
 *   x: [nch] raw conv input; conv_state [nch*3]; conv_w [nch*4]; conv_b [nch]
 *   dt_raw [nh]; ssm [nh*p*n]; y [nh*p] (nch == nh*p)
 */
static void conv_ssd_token(const float *x, const float *bm, const float *cm, const float *dt_raw, float *conv_state,
                           const float *conv_w, const float *conv_b, const float *dt_bias, const float *a_neg,
                           const float *dsk, float *ssm, float *y, int nh, int p, int n, float *xact) {
    int nch = nh * p;
    for (int c = 0; c < nch; c++) {
        float *cs = conv_state + c * 3;
        const float *cw = conv_w + c * 4;
        float s0 = cs[0], s1 = cs[1], s2 = cs[2], xc = x[c];
        float val = s0 * cw[0] + s1 * cw[1] + s2 * cw[2] + xc * cw[3] + conv_b[c];
        cs[0] = s1; cs[1] = s2; cs[2] = xc;
        xact[c] = orc_silu(val);
    }
    for (int h = 0; h < nh; h++) {
        float dtv = orc_softplus(dt_raw[h] + dt_bias[h]);
        float da = expf(dtv * a_neg[h]);
        for (int pp = 0; pp < p; pp++) {
            float xp = xact[h * p + pp];
            float xdt = xp * dtv;
            float *rs = ssm + ((size_t)h * p + pp) * n;
            float sy = 0.0f;
            for (int i = 0; i < n; i++) {
                float ns = rs[i] * da + bm[i] * xdt;
                rs[i] = ns;
                sy += ns * cm[i];
            }
            y[h * p + pp] = sy + dsk[h] * xp;
        }
    }
}

/* Batched one-step form: x [B,nh*p], B/C [B,n], dt [B,nh], conv_state [B,nh*p,3],
 * ssm [B,nh,p,n], y [B,nh*p]. */
EXPORT void orc_conv_ssd_step(const float *x, const float *bm, const float *cm, const float *dt_raw, float *conv_state,
                              const float *conv_w, const float *conv_b, const float *dt_bias, const float *a_neg,
                              const float *dsk, float *ssm, float *y, int bsz, int nh, int p, int n) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < bsz; b++) {
        int nch = nh * p;
        float *xact = malloc(sizeof(float) * nch);
        conv_ssd_token(x + (size_t)b * nch, bm + (size_t)b * n, cm + (size_t)b * n, dt_raw + (size_t)b * nh,
                       conv_state + (size_t)b * nch * 3, conv_w, conv_b, dt_bias, a_neg, dsk,
                       ssm + (size_t)b * nh * p * n, y + (size_t)b * nch, nh, p, n, xact);
        free(xact);
    }
}

/* Prefill form over T tokens: x [B,T,nh*p], B/C [B,T,n], dt [B,T,nh], y [B,T,nh*p];
 * the same token recurrence applied in order (src/model.rs:392-454). */
EXPORT void orc_conv_ssd_scan(const float *x, const float *bm, const float *cm, const float *dt_raw, float *conv_state,
                              const float *conv_w, const float *conv_b, const float *dt_bias, const float *a_neg,
                              const float *dsk, float *ssm, float *y, int bsz, int t, int nh, int p, int n) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < bsz; b++) {
        int nch = nh * p;
        float *xact = malloc(sizeof(float) * nch);
        for (int s = 0; s < t; s++) {
            size_t bt = (size_t)b * t + s;
            conv_ssd_token(x + bt * nch, bm + bt * n, cm + bt * n, dt_raw + bt * nh, conv_state + (size_t)b * nch * 3,
                           conv_w, conv_b, dt_bias, a_neg, dsk, ssm + (size_t)b * nh * p * n, y + bt * nch, nh, p, n,
                           xact);
        }
        free(xact);
    }
}

EXPORT int orc_num_threads(void) { return omp_get_max_threads(); }
EXPORT void orc_set_num_threads(int n) { omp_set_num_threads(n); }
