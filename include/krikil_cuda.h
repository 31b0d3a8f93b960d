/*
 * krikil_cuda.h -- C ABI of the B200 (sm_100a) implementation of krikil-rs's
 * per-layer inference path for the Pebble-25M hybrid Mamba2 + attention model.
 *
 * The reference is a Rust library whose public surface is src/lib.rs:1-6; its
 * model API (src/model.rs) is what a Rust `build.rs` + `extern "C"` binding of
 * this header replaces.  Each entry point below names the reference interface
 * it stands in for.  All computation is fp32, on the GPU; there is no CPU
 * fallback -- if the device or the kernels are unusable, calls fail with
 * KRK_CUDA and krk_last_error() says why.
 *
 * Conventions
 *  - Every function returns a krk_status; 0 is success.  On failure the
 *    calling thread's krk_last_error() holds a message (the reference's
 *    anyhow error text where one exists).  Nothing throws across the ABI.
 *  - Handles are opaque.  A model is immutable after load and may be shared by
 *    states on the same device; a state is owned by one thread at a time
 *    ("thread-compatible": calls on one state must not overlap).
 *  - Host buffers belong to the caller and are only read/written during the
 *    call.  Per-kernel entry points (krk_k_*) take DEVICE pointers and a CUDA
 *    stream (cudaStream_t passed as void*, NULL = legacy default stream) and
 *    are asynchronous.
 *  - A state holds `batch` independent sequences (the reference has exactly
 *    one, i.e. batch = 1).
 */
#ifndef KRIKIL_CUDA_H
#define KRIKIL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KRK_ABI_VERSION 1

#if defined(__GNUC__)
#define KRK_API __attribute__((visibility("default")))
#else
#define KRK_API
#endif

/* Model dimensions (src/model.rs:12-30). */
#define KRK_HIDDEN 608
#define KRK_VOCAB 2048
#define KRK_INTERMEDIATE 2432
#define KRK_LAYERS 8
#define KRK_ATTN_HEADS 8
#define KRK_ATTN_HEAD_DIM 76
#define KRK_MAMBA_D_STATE 128
#define KRK_MAMBA_D_CONV 4
#define KRK_MAMBA_D_INNER 1216
#define KRK_MAMBA_HEAD_DIM 64
#define KRK_MAMBA_HEADS 19
#define KRK_MAMBA_D_IN_PROJ 2707
#define KRK_MAMBA_D_XBC 1472
#define KRK_EOS_TOKEN 0

typedef enum krk_status {
    KRK_OK = 0,
    KRK_BAD_TOKEN = 1,        /* token id >= vocab (src/model.rs:333-335, :588-590) */
    KRK_CONTEXT_OVERFLOW = 2, /* position would exceed the context limit (src/model.rs:321-327, :591-593) */
    KRK_EMPTY = 3,            /* empty prompt (src/model.rs:317-319) */
    KRK_IO = 4,               /* file missing / unreadable / malformed safetensors (src/model.rs:235-239) */
    KRK_NOT_FOUND = 5,        /* tensor missing from the checkpoint (src/model.rs:243-244) */
    KRK_INVALID = 6,          /* bad argument (null handle, size or alignment) */
    KRK_CUDA = 7,             /* CUDA runtime error or no usable device */
    KRK_CHECK_FAILED = 8      /* internal consistency check failed */
} krk_status;

typedef struct krk_model krk_model;
typedef struct krk_state krk_state;

/* Message of the last failure on this thread ("" if none). */
KRK_API const char* krk_last_error(void);
KRK_API const char* krk_status_string(int status);
KRK_API int krk_abi_version(void);

/* ------------------------------------------------------------------ model */

/* PebbleModel::load_safetensors (src/model.rs:233-313).  Reads the tensors the
 * reference reads, by the same names (wte.weight, lnf.weight,
 * blocks.{i}.ln.weight, blocks.{i}.mixer.{in_proj.weight, conv1d.weight,
 * conv1d.bias, dt_bias, A_log, D, norm.weight, out_proj.weight} for Mamba
 * layers i%4<3, blocks.{i}.{ln1,wqkv,wo,ln2,fc1,fc2}.weight otherwise),
 * precomputes A = -exp(A_log) (src/model.rs:273-274) and uploads everything to
 * `device`.  Like the reference it does not check shapes, only that each
 * tensor is little-endian F32 with exactly the element count the model uses.
 * File and format errors are reported before the device is touched. */
KRK_API int krk_model_load(const char* path, int device, krk_model** out);
KRK_API int krk_model_free(krk_model* model);
KRK_API int krk_model_device(const krk_model* model, int* device);
/* The CUDA stream (cudaStream_t) the model's states run on. */
KRK_API int krk_model_stream(const krk_model* model, void** stream);

/* ------------------------------------------------------------------ state */

/* PebbleState::new(&config, max_ctx) (src/model.rs:204-219), for `batch`
 * independent sequences: per sequence 6 Mamba layers of conv [1472][4] and SSD
 * [19][64][128] state, 2 attention layers of K/V caches [max_ctx][608], all in
 * device memory and zeroed.  batch and max_ctx are at most 883,008 (a full-context
 * prefill is one projection over that many rows, indexed with 32-bit offsets). */
KRK_API int krk_state_create(const krk_model* model, int batch, int max_ctx, krk_state** out);
KRK_API int krk_state_free(krk_state* state);
/* PebbleState::reset (src/model.rs:221-229) for the sequences whose mask byte
 * is non-zero (mask NULL = all): position 0, Mamba state zeroed, attention
 * length 0. */
KRK_API int krk_state_reset(krk_state* state, const uint8_t* mask);
KRK_API int krk_state_batch(const krk_state* state, int* batch);
KRK_API int krk_state_context_limit(const krk_state* state, int* max_ctx);
/* current_pos of each sequence (src/model.rs:200), pos_out[batch]. */
KRK_API int krk_state_positions(const krk_state* state, int64_t* pos_out);

/* PebbleModel::forward_prefill (src/model.rs:316-368), batched: sequence b
 * consumes tokens[off_b .. off_b + lens[b]) (prompts packed back to back,
 * off_b = lens[0] + ... + lens[b-1]) starting at its current position.
 * logits_out (host, [batch][2048], may be NULL) receives each sequence's
 * last-token logits.  Checks, in the reference's order, before any state is
 * touched: every lens[b] >= 1 (KRK_EMPTY), pos_b + lens[b] <= max_ctx
 * (KRK_CONTEXT_OVERFLOW), every token < 2048 (KRK_BAD_TOKEN). */
KRK_API int krk_prefill(const krk_model* model, krk_state* state, const uint32_t* tokens, const int32_t* lens,
                        float* logits_out);

/* PebbleModel::forward_step (src/model.rs:586-624), batched: sequence b
 * consumes tokens[b] at its current position.  logits_out (host,
 * [batch][2048], may be NULL).  Checks before any state change: every token <
 * 2048 (KRK_BAD_TOKEN), then every position < max_ctx (KRK_CONTEXT_OVERFLOW). */
KRK_API int krk_step(const krk_model* model, krk_state* state, const uint32_t* tokens, float* logits_out);

/* The greedy path of GenerationEngine::generate_with_callback
 * (src/generate.rs:55-133) with Sampler::sample at temperature 0
 * (src/sampler.rs:43-80), run for all sequences at once with the sampling on
 * the device: reset, prefill the packed prompts, then per step choose each
 * sequence's token (repetition penalty over prompt + generated tokens when
 * repetition_penalty != 1, first maximum wins) and feed it back.  A sequence
 * stops after max_new_tokens tokens, when its position reaches max_ctx, or --
 * if stop_at_eos -- when it picks KRK_EOS_TOKEN (not emitted).  With
 * stop_at_eos = 0 every sequence emits min(max_new_tokens, max_ctx - len + 1)
 * tokens.  tokens_out (host, [batch][max_new_tokens]) and n_out (host,
 * [batch]) receive the generated ids and their counts.  Each decode step
 * replays a CUDA graph held by the state (see krk_state_set_step_graphs)
 * unless per-kernel profiling is on; krk_generate_sample does the same.  The
 * call synchronises with the device once, at its end. */
KRK_API int krk_generate_greedy(const krk_model* model, krk_state* state, const uint32_t* prompts,
                                const int32_t* lens, int max_new_tokens, float repetition_penalty, int stop_at_eos,
                                uint32_t* tokens_out, int32_t* n_out);

/* The same loop with Sampler::sample at any temperature (src/sampler.rs:43-152):
 * repetition penalty, logits * (1/temperature), candidates sorted by logit
 * (equal logits by ascending id), top_k (0 = all), softmax, top_p (1 = all)
 * with renormalisation, then the first candidate whose running probability
 * reaches r = Rng::gen::<f32>().  Sequence b draws from its own
 * StdRng::seed_from_u64(seeds[b]) stream (rand 0.8's ChaCha12), as a reference
 * Sampler built with config.seed = Some(seeds[b]); one word per pick.
 * temperature <= 1e-6 is krk_generate_greedy (seeds may then be NULL). */
KRK_API int krk_generate_sample(const krk_model* model, krk_state* state, const uint32_t* prompts,
                                const int32_t* lens, int max_new_tokens, float temperature, float top_p, int top_k,
                                float repetition_penalty, const uint64_t* seeds, int stop_at_eos,
                                uint32_t* tokens_out, int32_t* n_out);

/* Test hook: copies one sequence's layer state to host memory.
 *   what 0: conv state [1472][4] (Mamba layers)   what 1: SSD state [19][64][128]
 *   what 2: K cache [max_ctx][608] (attention)     what 3: V cache [max_ctx][608]
 * n = number of floats available at out (must be >= the size above). */
KRK_API int krk_state_export(const krk_state* state, int seq, int layer, int what, float* out, int64_t n);

/* Kernels this library launched in this process (graph replays count each
 * kernel node). */
KRK_API int krk_launch_count(uint64_t* count);

/* Checked builds (no reference counterpart; the reference's bounds checks are
 * Rust's own).  `make CHECKED=1` builds lib/libkrikil_cuda_checked.so, whose
 * kernels test the preconditions on device data the host cannot see before a
 * launch (token ids, positions, table entries read on the device); a kernel
 * that finds one violated sets a KRK_CHECK_* bit of a device status word and
 * skips the access (no trap, no assert), and krk_prefill / krk_step /
 * krk_generate_* then fail with KRK_CHECK_FAILED naming the checks.
 * krk_checked_build: 1 for a checked build, else 0.  krk_check_status: the
 * bits set on the current device since they were last cleared (always 0 in
 * other builds); call it after the checked work has finished (the model calls
 * synchronise before they return; for a per-kernel entry point synchronise its
 * stream first); clear != 0 resets them. */
#define KRK_CHECK_TOKEN 1u    /* a token id >= vocab reached a kernel */
#define KRK_CHECK_POSITION 2u /* a position outside [0, ctx) or past the launch's key bound */
#define KRK_CHECK_TABLE 4u    /* a prefill table entry outside its sequence or key bound */
#define KRK_CHECK_COLUMN 8u   /* a gather column outside its matrix */
KRK_API int krk_checked_build(void);
KRK_API int krk_check_status(uint32_t* bits, int clear);

/* Measurement hook (no reference counterpart; the reference only times whole
 * calls, src/generate.rs:76-78, :116-122): with profiling on, every later
 * prefill / step / generate call on this state brackets each kernel launch
 * with CUDA events on its stream and accumulates the device time per
 * kernel class; KRK_PROF_DEVICE_TOTAL is the device time of whole calls, from
 * after the inputs reach the device to before the outputs leave it.
 * krk_state_profile resets the totals. */
enum {
    KRK_PROF_DEVICE_TOTAL = 0,
    KRK_PROF_GEMM = 1,         /* projections */
    KRK_PROF_SSD_STEP = 2,     /* decode SSD update + gate */
    KRK_PROF_ATTN_DECODE = 3,  /* RoPE + KV append + decode attention (+ split combine) */
    KRK_PROF_NORM = 4,         /* RMSNorm / gated RMSNorm */
    KRK_PROF_CONV = 5,         /* causal conv1d + SiLU */
    KRK_PROF_SSD_SCAN = 6,     /* prefill SSD scan */
    KRK_PROF_ATTN_PREFILL = 7, /* prefill causal attention */
    KRK_PROF_OTHER = 8,        /* embedding, RoPE prefill, sampling, bookkeeping */
    KRK_PROF_CLASSES = 9
};
/* Decode scheduling (no reference counterpart): a decode batch of 256+
 * sequences runs as up to n parts of whole 64-row tiles (at least two tiles
 * each, sizes within one tile) on their own streams, so that one part's
 * projections overlap the others' HBM-bound kernels; n = 3 is the default,
 * n <= 4.  Prefills of more than 16,384 prompt tokens run up to three groups
 * of whole sequences at once on the same streams.  n = 1 runs decode and
 * prefill on the model stream alone.  Results are identical for every n. */
KRK_API int krk_state_set_decode_streams(krk_state* state, int n);

/* Decode scheduling (no reference counterpart): with enable != 0 (the
 * default) the generation loops replay each decode step as a CUDA graph held
 * by the state -- one per count of 64-key attention blocks, captured on the
 * model's streams the first time the count comes up -- instead of launching
 * its kernels one by one; 0 launches them one by one and drops the graphs.
 * Results are identical either way.  Per-kernel profiling also launches them
 * one by one.  Generation calls of states that share a model must not run
 * concurrently (the capture runs on the model's streams). */
KRK_API int krk_state_set_step_graphs(krk_state* state, int enable);

/* enable: 0 off, 1 every kernel class and the whole-call total, 2 the
 * whole-call total only (two events per call: no per-kernel event records and
 * no per-kernel readback after the call). */
KRK_API int krk_state_profile(krk_state* state, int enable);
KRK_API int krk_state_profile_read(const krk_state* state, int cls, double* total_ms, int64_t* launches);
/* Decode sequences processed by the timed launches of a class (the sum over
 * its decode launches of the sequences each covered; prefill launches add 0).
 * A decode batch of 256+ sequences runs in parts on up to three streams, and
 * a large prefill in groups on up to three streams, each launch timed on its
 * own stream, so per-class times are kernel times that may overlap and can add
 * up to more than KRK_PROF_DEVICE_TOTAL. */
KRK_API int krk_state_profile_units(const krk_state* state, int cls, int64_t* units);

/* ------------------------------------------------------ per-kernel entry points
 * Device pointers, fp32, asynchronous on `stream`.  Each names the reference
 * code it computes. */

/* src/math.rs:41-54 on rows: y[r] = rms_norm(x[r], w, eps), [rows][dim],
 * dim % 128 == 0, dim <= 1024. */
KRK_API int krk_k_rmsnorm_rows(const float* x, const float* w, float eps, int64_t rows, int dim, float* y,
                               void* stream);

/* src/math.rs:41-54 on feature-major activations (column m of x[k*ldx + m],
 * k < K <= 1216, m < M): out[k*ldo+m] = x*scale(m)*w[k].  The sum of squares
 * is formed as 32 partials (partial p over k = p, p + 32, ... in order) added
 * in a fixed tree: within a few ulps of the reference's sequential sum, and
 * the same for a column whatever M or its place in the batch.  x holds K full
 * rows of ldx floats: columns M .. ldx-1 may be read (never written). */
KRK_API int krk_k_rmsnorm_fm(const float* x, int ldx, const float* w, float eps, int K, int M, float* out, int ldo,
                             void* stream);

/* Gate + gated RMSNorm + residual (src/model.rs:688-693, src/math.rs:56-68,
 * residual add src/model.rs:699-701): y = rms_norm(x * silu(z), w, eps) + res
 * over [rows][dim], dim % 128 == 0, dim <= 1024. */
KRK_API int krk_k_gated_rmsnorm_residual(const float* x, const float* z, const float* res, const float* w, float eps,
                                         int64_t rows, int dim, float* y, void* stream);

/* Projection C = A . W^T (src/math.rs:130-153 gemv and :188-211 gemm_transb)
 * with the reference dot's exact rounding.  At: A feature-major [K][lda];
 * Wt: W K-major [K][ldw]; C batch-major [M][ldc] (out_fm = 0) or
 * feature-major [N][ldc] (out_fm = 1).  epilogue 0: store, 1: C += result
 * (residual), 2: store gelu(result) (src/math.rs:17-39).  M % 16 == 0,
 * N % 32 == 0, K % 32 == 0, leading dims % 4 == 0, pointers 16-byte aligned,
 * K * lda and K * ldw below 2^31 (KRK_INVALID otherwise). */
KRK_API int krk_k_gemm(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                       int epilogue, int out_fm, void* stream);

/* krk_k_gemm with an explicit CTA tile height: 64, 32 or 16 output rows per
 * CTA (M must be a multiple of it), 0 = the automatic choice krk_k_gemm makes,
 * 1 = the few-rows form for M <= 8 and K <= 2432 (one thread per output
 * column and dot lane; only the M rows are read and written, so lda, ldc may
 * be a padded batch).  Every choice gives bit-identical results. */
KRK_API int krk_k_gemm_tiled(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N,
                             int K, int epilogue, int out_fm, int tile_rows, void* stream);

/* C = A . W^T with the operand layouts of krk_k_gemm (batch-major C, store
 * only), every element summed in the order of matrixmultiply 0.3.11's sgemm,
 * which the reference's gemm_transb (src/math.rs:188-211) calls for its prefill
 * projections (src/model.rs:387, 458, 484, 554, 570, 577): a fused
 * multiply-add chain over k from zero within each 256-long block of K, the
 * blocks' sums added to the output in order.  That order is restated from the
 * crate's published algorithm (the crate is not part of the reference tree);
 * the model's prefill keeps krk_k_gemm's gemv dot order.  M % 64 == 0,
 * N % 32 == 0, K % 32 == 0, leading dims % 4 == 0, pointers 16-byte aligned. */
KRK_API int krk_k_gemm_sgemm_order(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M,
                                   int N, int K, void* stream);

/* The tile height krk_k_gemm chooses for an M x N output on the current
 * device (148 SMs assumed when no device answers): the smallest of 16 / 32 /
 * 64 rows whose grid fits in one wave of one CTA per SM, else 32 below 256
 * rows and 64 from there on.  Host only; launches nothing. */
KRK_API int krk_k_gemm_tile_rows(int M, int N);

/* Embedding gather (src/model.rs:330-338, :598) into feature-major
 * out[k*ldo + m] = wte[tok[m]*K + k]. */
KRK_API int krk_k_embed(const uint32_t* tok, const float* wte, int vocab, int K, int M, float* out, int ldo,
                        void* stream);

/* Pointwise silu (op 0, src/math.rs:3-6), softplus (op 1, :8-15),
 * gelu (op 2, :17-39). */
KRK_API int krk_k_pointwise(int op, const float* x, float* y, int64_t n, void* stream);

/* Causal depthwise conv1d (kernel 4) + SiLU on x, then the Mamba2 SSD single-
 * step update (src/model.rs:643-685) for batch B, H heads of P = 64 channels,
 * N = 128 states, B/C given directly:
 *   x [B][H*P] raw conv input, bm/cm [B][N], dt [B][H] (raw; softplus(dt +
 *   dt_bias) inside), conv_state [B][H*P][3] (previous 3 inputs, updated),
 *   conv_w [H*P][4], conv_b [H*P], ssm [B][H][P][N] (updated), dt_bias/a_neg/
 *   dsk [H] (a_neg = A = -exp(A_log)), y [B][H*P] = sum_n s*C + D*x. */
KRK_API int krk_k_conv_ssd_step(const float* x, const float* bm, const float* cm, const float* dt,
                                float* conv_state, const float* conv_w, const float* conv_b, float* ssm,
                                const float* dt_bias, const float* a_neg, const float* dsk, float* y, int B, int H,
                                int P, int N, void* stream);

/* The same conv + SSD recurrence over T tokens per sequence (the prefill form,
 * src/model.rs:392-454): x [B][T][H*P], bm/cm [B][T][N], dt [B][T][H],
 * y [B][T][H*P]; the SSD state is carried in registers across the sequence
 * and the inputs are staged through shared memory chunk by chunk. */
KRK_API int krk_k_conv_ssd_scan(const float* x, const float* bm, const float* cm, const float* dt,
                                float* conv_state, const float* conv_w, const float* conv_b, float* ssm,
                                const float* dt_bias, const float* a_neg, const float* dsk, float* y, int B, int T,
                                int H, int P, int N, void* stream);

/* Decode RoPE (src/math.rs:234-260) + KV-cache append (src/model.rs:730-733)
 * + single-query softmax attention (src/model.rs:736-760) on a [B][H][ctx][dh]
 * cache: q,k,v [B][H][dh] (dh = 64 or 76), pos [B] (int32, < ctx), kc/vc
 * updated at slot pos[b], out [B][H][dh].
 *   split = 0: eight CTAs per (sequence, head) form a thread-block cluster and
 *     share the keys 0..pos evenly; CTA 0 merges their softmax partials through
 *     distributed shared memory.  One launch, no scratch: `work` may be NULL and
 *     krk_attn_work_floats() is 0.
 *   split > 0 (multiple of 64): keys in splits of `split` keys, one CTA each,
 *     and a second launch merging the splits; when a sequence needs more than
 *     one split, `work` must hold krk_attn_work_floats() floats of device
 *     scratch. */
KRK_API size_t krk_attn_work_floats(int B, int H, int dh, int ctx, int split);
KRK_API int krk_k_rope_kv_attn_decode(const float* q, const float* k, const float* v, float* kc, float* vc,
                                      const int32_t* pos, float* out, float* work, int B, int H, int dh, int ctx,
                                      int split, float theta, void* stream);

/* Prefill RoPE (src/math.rs:234-260) + KV-cache append + causal softmax
 * attention (src/model.rs:486-548) of packed query rows for S sequences.
 * Sequence s owns rows cu_seqlens[s] .. cu_seqlens[s+1]-1 of qkv (q | k | v of
 * H*dh floats each, row stride q_rs; total_rows rows in all) and its first row
 * sits at position start[s], keys 0..start[s]-1 being in its cache already.  q
 * is rotated in place; the rotated k and v of row r go to
 * kc/vc[s*c_sb + h*c_sh + pos*c_st + d]; out[r*o_rs + (h*dh + d)*o_cs] gets row
 * r's attention over keys 0..its position (dh = 64 or 76).  The rows run in
 * blocks of rows_per_block = krk_k_attn_prefill_rows(kmax, dh) consecutive rows
 * of one sequence: blocks holds nblocks int32 pairs (sequence, first row
 * within it) on the device, covering every row once; kmax >= start[s] + rows of
 * s for every s.  RoPE angles use the host-libm inverse frequencies and
 * sincosf.  The model calls the same two kernels with its host-libm angle
 * table. */
KRK_API int krk_k_attn_prefill_rows(int kmax, int dh);
KRK_API int krk_k_rope_kv_attn_prefill(float* qkv, int64_t q_rs, float* kc, float* vc, int64_t c_sb, int64_t c_sh,
                                       int64_t c_st, const int32_t* cu_seqlens, const int32_t* start, int S,
                                       int total_rows, int H, int dh, float theta, const int32_t* blocks,
                                       int nblocks, int rows_per_block, int kmax, float* out, int64_t o_rs,
                                       int64_t o_cs, void* stream);

/* Allocation-free variant of krk_k_rope_kv_attn_decode (no counterpart in the
 * reference, which has no device memory).  For callers that cannot allocate or
 * pass device scratch -- a host that binds only this header and has no CUDA
 * allocator of its own, or a process whose device memory belongs to another
 * allocator or a fixed budget: the split partials go to a fixed array inside
 * the library's device image, KRK_ATTN_NOALLOC_MAX_FLOATS floats (4 MiB) held by
 * every GPU that loads the library until the process exits.  Same arguments and
 * results as krk_k_rope_kv_attn_decode without `work`, with `split` > 0 (0 picks
 * 256 here); when the cache needs more than one split and
 * krk_attn_work_floats() for that split exceeds the maximum, the call
 * fails with KRK_INVALID before launching anything.  It calls no allocator.  The
 * call runs on the device that owns `stream` (the current device for the
 * default stream) and restores the caller's current device.  The first call on
 * a device looks up the array's device address (once per device and CUDA
 * context, with that device current; after a device reset the next call looks
 * it up again), so make it before any stream capture.  All calls on a GPU share
 * the array: calls that overlap on the GPU race and must be serialised by the
 * caller.  No part of the array needs clearing between calls (each call writes
 * every partial it reads). */
#define KRK_ATTN_NOALLOC_MAX_FLOATS (1 << 20)
KRK_API int krk_k_rope_kv_attn_decode_noalloc(const float* q, const float* k, const float* v, float* kc, float* vc,
                                              const int32_t* pos, float* out, int B, int H, int dh, int ctx,
                                              int split, float theta, void* stream);

/* Test hook of the copy-wait failure path (no counterpart in the reference).
 * One warp arms a shared-memory mbarrier for a 16-byte bulk copy exactly as the
 * decode attention arms it for its K/V rows, then waits with the same bounded
 * wait, `polls` polls at most (1 .. 2^20).  copy != 0: the copy of src16
 * (16-byte aligned device memory) is issued and lands, and *status (device)
 * is left alone; copy == 0: no copy is issued, the wait runs out, and bit 0 of
 * *status is set -- the status word krk_step / krk_generate_* read back after
 * the attention kernels.  The kernel returns either way and the context stays
 * usable. */
KRK_API int krk_k_wait_probe(const float* src16, int polls, int copy, int32_t* status, void* stream);

/* Greedy pick (src/sampler.rs:50-80) per row of logits [B][ld]: repetition
 * penalty on tokens whose bit is set in seen [B][vocab/32] (seen may be NULL;
 * penalty 1 disables it), then the first maximum; tok [B]. */
KRK_API int krk_k_greedy(const float* logits, int64_t ld, int vocab, int B, uint32_t* seen, float penalty,
                         uint32_t* tok, void* stream);

/* One pick per row as krk_generate_sample does it (src/sampler.rs:43-152,
 * vocab <= 4096): rng_state [B][10] (device) is each row's sampler state, from
 * krk_rng_seed_state, advanced by one word per row; the pick's bit is set in
 * seen when seen is not NULL.  temperature <= 1e-6 is krk_k_greedy. */
KRK_API int krk_k_sample(const float* logits, int64_t ld, int vocab, int B, uint32_t* seen, float temperature,
                         float top_p, int top_k, float penalty, uint32_t* rng_state, uint32_t* tok, void* stream);

/* StdRng::seed_from_u64(seed) as sampler state: 8 ChaCha12 key words from
 * rand_core's PCG32 expansion, then the next keystream word's index (0, 0);
 * host memory, 10 words. */
KRK_API int krk_rng_seed_state(uint64_t seed, uint32_t* state10);

#ifdef __cplusplus
}
#endif
#endif /* KRIKIL_CUDA_H */
