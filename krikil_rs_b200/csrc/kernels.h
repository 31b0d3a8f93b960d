// Host-side launchers of the krikil B200 kernels (internal C++ interface; the
// public boundary is the C ABI in include/krikil_cuda.h).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace krk {

// Number of kernels this library has launched in this process (graph replays
// count every kernel node of the graph).
uint64_t launch_count();
void add_launches(uint64_t n);

// Raises a kernel's dynamic shared-memory limit once per device.
struct DeviceOnce {
    unsigned long long mask = 0;
    cudaError_t set_smem(const void* func, size_t bytes);
};

// Programmatic dependent launch of a decode step's chain of kernels.  While a
// PdlScope(true) lives on the calling thread, the launchers of the
// projections (both forms), feature-major RMSNorm, embedding gather, SSD
// update and decode attention launch their kernels with programmatic stream
// serialization: a kernel is scheduled while the one before it in the stream
// is finishing, issues only reads of weights, and waits (pdl_wait) for that
// kernel's completion before it reads or writes any other memory -- so the
// launch latency and the weight prefetch overlap the previous kernel.  Other
// launchers, and these outside a scope, launch as usual.
bool pdl_enabled();
class PdlScope {
  public:
    explicit PdlScope(bool on);
    ~PdlScope();
    PdlScope(const PdlScope&) = delete;
    PdlScope& operator=(const PdlScope&) = delete;

  private:
    bool prev_;
};

// Launch priority of the same launchers while a PriorityScope lives on the
// calling thread (0: the stream's own; lower is more urgent, down to the
// device's greatest priority).  Kernel nodes of a captured graph keep it.
int launch_priority();
class PriorityScope {
  public:
    explicit PriorityScope(int priority);
    ~PriorityScope();
    PriorityScope(const PriorityScope&) = delete;
    PriorityScope& operator=(const PriorityScope&) = delete;

  private:
    int prev_;
};

// ---------------------------------------------------------------- projections
// C = A . W^T in fp32 with the reference's dot-product order (see k_gemm.cu).
//   At: A stored feature-major, At[k*lda + m]  (M columns, K rows)
//   Wt: W stored K-major,       Wt[k*ldw + n]
//   out_fm=false: C[m*ldc + n];  out_fm=true: C[n*ldc + m]
// M % 16 == 0, N % 32 == 0, K % 32 == 0; leading dims % 4 == 0; 16-B aligned.
enum GemmEpilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_GELU = 2, EPI_CONV = 3 };
// EPI_CONV (batch-major output only): output columns [lo, hi) are the decode
// conv channels; for rows m < rows whose active flag is set (or all, when
// active is null), the epilogue shifts the channel's 4-slot state
// state[(m*(hi-lo) + c)*4] and stores silu(conv) instead of the raw value --
// conv_step4 fused into the projection that produces its input.
struct GemmConv {
    float* state;
    const float* w;     // [hi-lo][4]
    const float* bias;  // [hi-lo]
    const uint8_t* active;
    int rows, lo, hi;
};
cudaError_t gemm(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                 int epilogue, bool out_fm, cudaStream_t s);
// gemm_tiled() with the EPI_CONV epilogue (batch-major output; lo and hi
// multiples of 32).
cudaError_t gemm_conv(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                      int tile_rows, const GemmConv& cv, cudaStream_t s);
// out[c*ld + r] = in[r*cols + c] for r < rows, 0 for rows <= r < ld (c < cols):
// a row-major weight [rows][cols] into the K-major layout the projections read.
cudaError_t transpose_pad(const float* in, int rows, int cols, float* out, int ld, cudaStream_t s);
// tile_rows 1 in gemm_tiled / gemm_conv: the few-rows form for M <= 8 rows
// (K <= 2432): one thread per (output column, dot lane), bitwise the same.
constexpr int GEMM_FEW_ROWS = 8;
// Whether the decode step uses the few-rows form for M real rows and N columns.
bool gemm_few_rows(int M, int N);
// The few-rows projection of rms_norm(A) (w [K], eps): each CTA normalises
// its staged copy of A's M rows with rmsnorm_fm's partial sums, tree and
// expression, so the result is bitwise rmsnorm_fm and then the projection, in
// one launch.  Forms: store (batch-major), residual / gelu (feature-major),
// and the in_proj conv epilogue (cv non-null, batch-major).
struct GemmNorm {
    const float* w;
    float eps;
};
cudaError_t gemm_few_norm(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                          int epilogue, bool out_fm, const GemmNorm& nm, const GemmConv* cv, cudaStream_t s);
// C = A . W^T (batch-major C[M][ldc]) summed in matrixmultiply 0.3.11 sgemm's
// order (k_gemm_sgemm.cu).  M % 64 == 0, N % 32 == 0, K % 32 == 0.
cudaError_t gemm_sgemm_order(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N,
                             int K, cudaStream_t s);
// Rows per CTA tile (64, 32 or 16) gemm() uses for an M x N output.
int gemm_tile_rows(int M, int N);
// gemm() with an explicit CTA tile height (16, 32 or 64; 1 = the few-rows form; 0 = gemm_tile_rows).
cudaError_t gemm_tiled(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                       int epilogue, bool out_fm, int tile_rows, cudaStream_t s);

// ---------------------------------------------------------------- norms
// out[k*ldo+m] = x[k*ldx+m] * scale(m) * w[k] (src/math.rs:41-54) -- feature-major
// activations; the sum of squares over k in a fixed order of 32 partials, the
// same for a column whatever its batch (the reference's sequential sum up to
// rounding).
cudaError_t rmsnorm_fm(const float* x, int ldx, const float* w, float eps, int K, int M, float* out, int ldo,
                       cudaStream_t s);
// Row-major RMSNorm over [rows, dim].
cudaError_t rmsnorm_rows(const float* x, const float* w, float eps, int64_t rows, int dim, float* y, cudaStream_t s);
// y = rmsnorm(x * silu(z)) * w + res over [rows, dim] (dim % 128 == 0, dim <= 1024).
cudaError_t gated_rmsnorm_residual(const float* x, const float* z, const float* res, const float* w, float eps,
                                   int64_t rows, int dim, float* y, cudaStream_t s);
// Embedding gather into feature-major out[k*ldo + m] = wte[tok[m]*K + k]
// (ids >= vocab, which the host rejects beforehand, gather zeros).
cudaError_t embed_fm(const uint32_t* tok, const float* wte, int vocab, int K, int M, float* out, int ldo,
                     cudaStream_t s);
// Elementwise silu / softplus / gelu (op 0/1/2) for unit tests.
cudaError_t pointwise(int op, const float* x, float* y, int64_t n, cudaStream_t s);

// ---------------------------------------------------------------- Mamba2
struct SsdStepArgs {
    const float* x; int64_t x_sb;            // x(b,c) = x[b*x_sb + c], c < H*P (raw if conv, else activated)
    const float* bm; const float* cm; int64_t bc_sb;  // B(b,n), C(b,n)
    const float* dt; int64_t dt_sb;          // dt_raw(b,h)
    const float* z; int64_t z_sb;            // gate input z(b,c) or nullptr
    float* conv_state;                       // conv on x channels only: [B][H*P][3]
    const float* conv_w; const float* conv_b;  // [H*P][4], [H*P]
    float* ssm;                              // [B][H][P][N]
    const float* dt_bias; const float* a_neg; const float* dsk;  // [H]
    float* y; int64_t y_sb; int64_t y_sc;    // y(b,c) = y[b*y_sb + c*y_sc]
    const uint8_t* active;                   // [B] or nullptr: inactive sequences are left untouched
    int B, H, P, N;
};
cudaError_t ssd_step(const SsdStepArgs& a, bool conv, cudaStream_t s);

// Decode conv on the model's 4-slot shift-register state (src/model.rs:643-654):
// xbc(b,c) (in place, raw -> silu(conv)), state [B][C][4].
cudaError_t conv_step4(float* xbc, int64_t x_sb, float* state, const float* w, const float* bias, int B, int C,
                       const uint8_t* active, cudaStream_t s);

// Prefill conv over packed sequences (rows cu[s]..cu[s+1]), 4-slot state [S][C][4].
cudaError_t conv_prefill4(const float* xin, int64_t x_rs, float* xout, int64_t o_rs, float* state, const float* w,
                          const float* bias, const int32_t* cu_seqlens, int S, int C, cudaStream_t s);

struct SsdScanArgs {
    const float* x; int64_t x_rs;            // x(row,c)
    const float* bm; const float* cm; int64_t bc_rs;
    const float* dt; int64_t dt_rs;
    const float* z; int64_t z_rs;            // nullable
    float* conv_state; const float* conv_w; const float* conv_b;  // conv on x channels: [S][H*P][3]
    float* ssm;                              // [S][H][P][N]
    const float* dt_bias; const float* a_neg; const float* dsk;
    float* y; int64_t y_rs; int64_t y_cs;    // y(row,c) = y[row*y_rs + c*y_cs]
    const int32_t* cu_seqlens;               // [S+1]; nullptr: sequence s is rows [s*uniform_len, (s+1)*uniform_len)
    int uniform_len;
    int S, H, P, N;
};
cudaError_t ssd_scan(const SsdScanArgs& a, bool conv, cudaStream_t s);

// ---------------------------------------------------------------- attention
// Decode: per sequence b and head h, RoPE on q and the new k at position pos[b],
// append k,v at slot pos[b], softmax(q.K^T/sqrt(dh)).V over slots 0..pos[b].
// Cache element (b,h,t,d) at cache[b*c_sb + h*c_sh + t*c_st + d].
// RoPE inverse frequencies 1/theta^(2i/dh) from the host libm (i < dh/2 <= 64).
constexpr int ROPE_MAX_PAIRS = 64;
struct RopeFreqs {
    float f[ROPE_MAX_PAIRS];
};
RopeFreqs rope_freqs(int dh, float theta);

struct AttnDecodeArgs {
    const float* q; const float* k; const float* v; int64_t in_sb; int64_t in_sh;  // (b,h,d) at b*in_sb + h*in_sh + d
    float* kc; float* vc; int64_t c_sb; int64_t c_sh; int64_t c_st;
    const int32_t* pos;                      // [B]
    const uint8_t* active;                   // [B] or nullptr
    float* out; int64_t o_sb; int64_t o_sh; int64_t o_sd;  // out(b,h,d)
    float* work;                             // split partials: [B*H*max_splits*(dh+2)] floats
    int B, H, dh, ctx, split;                // keys per split (multiple of 64)
    float theta;
    const float2* rope;                      // optional (cos, sin) table [ctx][dh/2]; null: computed in-kernel
    int max_keys;                            // > 0: no sequence has pos + 1 above this; 0: unknown (ctx)
    RopeFreqs freq;                          // filled by attn_decode() when rope is null
    int* err;                                // nullable: bit 0 set if a K/V copy wait timed out
};
size_t attn_decode_work_floats(int B, int H, int dh, int ctx, int split);
cudaError_t attn_decode(const AttnDecodeArgs& a, cudaStream_t s);
// The bounded copy wait of the decode attention on one armed mbarrier: with
// copy a 16-byte bulk copy of src lands; without, the wait runs out after
// `polls` polls and bit 0 of *err is set.
cudaError_t wait_probe(const float* src, int polls, bool copy, int* err, cudaStream_t s);

// Prefill: RoPE q in place and k into the cache, v into the cache, for packed rows.
// qkv(row) = qkv[row*q_rs + ...] with q | k | v of H*dh each; cache layout as above
// with c_sb the per-sequence stride; start[s] = first position of sequence s.
cudaError_t rope_kv_prefill(float* qkv, int64_t q_rs, float* kc, float* vc, int64_t c_sb, int64_t c_sh,
                            int64_t c_st, const int32_t* cu_seqlens, const int32_t* start, int S, int H, int dh,
                            int total_rows, float theta, const float2* rope, cudaStream_t s);
// Causal attention of packed query rows over their sequence's cache, by
// blocks of rows_per_block consecutive rows of one sequence: blocks[i] =
// (sequence, first row within it); kmax >= start[s] + rows of s for every s.
// rows_per_block = attn_prefill_rows(kmax, dh): PF_ROWS, or 1 when the
// scores of PF_ROWS rows over kmax keys do not fit in shared memory.
constexpr int PF_ROWS = 8;
int attn_prefill_rows(int kmax, int dh);
// The argument checks attn_prefill makes (dh, stride and pointer alignment,
// rows_per_block, shared memory for kmax), for a caller to make before the
// RoPE/KV launch that precedes it.
cudaError_t attn_prefill_check(const float* qkv, int64_t q_rs, const float* kc, const float* vc, int64_t c_sb,
                               int64_t c_sh, int64_t c_st, int nblocks, int rows_per_block, int H, int dh,
                               int kmax);
cudaError_t attn_prefill(const float* qkv, int64_t q_rs, const float* kc, const float* vc, int64_t c_sb,
                         int64_t c_sh, int64_t c_st, const int32_t* cu_seqlens, const int32_t* start,
                         const int2* blocks, int nblocks, int rows_per_block, int H, int dh, int kmax, float* out,
                         int64_t o_rs, int64_t o_cs, cudaStream_t s);

// ---------------------------------------------------------------- sampling
// Greedy choice per sequence (src/sampler.rs:50-80): repetition penalty on the
// tokens whose bit is set in seen[b][vocab/32] (when penalty != 1), then the
// first maximum.  Writes tok[b] and sets its seen bit.  Bookkeeping of batched
// generation, mirroring src/generate.rs:86-114 (any pointer may be null):
//   pos[b] += 1          the logits came from a decode step of sequence b
//   step                 index of this pick (the caller's counter, bumped after)
//   tlimit[b]            picks at step >= tlimit[b] are discarded
//   hist[step*B + b]     the recorded pick
//   active[b] = 0        after an EOS pick (stop_eos), a discarded pick, or a
//                        pick with step + 1 > slimit[b] (no further decode step)
struct GreedyArgs {
    const float* logits; int64_t ld; int vocab; int B;
    uint32_t* seen; float penalty;
    uint32_t* tok;
    uint8_t* active;
    uint32_t* hist; int32_t* step; int32_t* pos; const int32_t* tlimit; const int32_t* slimit;
    int stop_eos; uint32_t eos;
    // stochastic sampling (src/sampler.rs:83-152) when temperature > 1e-6
    float temperature; float top_p; int top_k;
    uint32_t* rng;  // [B][10]: ChaCha12 key (8 words), index of the next keystream word (lo, hi)
};
cudaError_t greedy(const GreedyArgs& a, cudaStream_t s);
// greedy() when temperature <= 1e-6, else the stochastic pick with the same
// bookkeeping (vocab <= 4096).
cudaError_t sample(const GreedyArgs& a, cudaStream_t s);
// StdRng::seed_from_u64 (rand_core 0.6 over rand_chacha 0.3's ChaCha12):
// the sampler state [10] for `seed`, on the host.
void rng_seed_state(uint64_t seed, uint32_t st[10]);
// Sets the seen bit of each packed row's token for its sequence.
cudaError_t mark_seen(const uint32_t* tok, const int32_t* row_seq, int rows, uint32_t* seen, int words,
                      cudaStream_t s);
// pos[b] += 1 for active sequences.
cudaError_t advance_pos(int32_t* pos, const uint8_t* active, int B, cudaStream_t s);
// dst[k*ldd + dcol[j]] = src[k*lds + scol[j]] for j < n, k < K (feature-major column gather).
cudaError_t gather_cols(const float* src, int lds, const int32_t* scol, float* dst, int ldd, const int32_t* dcol,
                        int K, int n, cudaStream_t s);

}  // namespace krk
