// Host runtime behind include/krikil_cuda.h: weights, per-sequence state in
// HBM, batched prefill / decode orchestration, and the C ABI.
//
// Layouts in device memory (fp32):
//  weights   projections stored K-major (W^T, [in][out], out padded to 32):
//            in_proj [608][2720], out_proj [1216][608], wqkv [608][1824],
//            wo [608][608], fc1 [608][2432], fc2 [2432][608], LM head = wte^T
//            [608][2048]; wte [2048][608] row-major for the embedding gather.
//  state     per Mamba layer conv [B][1472][4] and SSD [B][19][64][128]; per
//            attention layer K and V caches [B][ctx][608] (row t = the 8 heads'
//            76-dim vectors, as src/model.rs:141-142).
//  decode    activations between projections are feature-major ([features]
//            [Mp], Mp = B rounded up to 64) so each projection's A operand is a
//            dense K-major tile; projection outputs that feed per-sequence
//            kernels (in_proj, wqkv, logits) are batch-major.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <memory>
#include <string>
#include <vector>

#include "../../include/krikil_cuda.h"
#include "kernels.h"
#include "safetensors.h"

namespace {

constexpr int HID = KRK_HIDDEN, VOC = KRK_VOCAB, INTER = KRK_INTERMEDIATE, NL = KRK_LAYERS;
constexpr int NH = KRK_ATTN_HEADS, HD = KRK_ATTN_HEAD_DIM;
constexpr int DS = KRK_MAMBA_D_STATE, DI = KRK_MAMBA_D_INNER, MP = KRK_MAMBA_HEAD_DIM, MH = KRK_MAMBA_HEADS;
constexpr int DIP = KRK_MAMBA_D_IN_PROJ, DXBC = KRK_MAMBA_D_XBC;
constexpr int DIP_PAD = 2720;  // in_proj output width padded to the 32-column tile
constexpr int QKV = 3 * HID;
constexpr float RMS_EPS = 1e-6f, MNORM_EPS = 1e-5f, THETA = 10000.0f;
constexpr int SEEN_WORDS = VOC / 32;
constexpr int64_t PREFILL_GROUP_TOKENS = 16384;
// Largest multiple of 64 rows whose widest projection operand ([INTER][rows])
// stays below 2^31 elements.
constexpr int64_t MAX_ROWS = ((int64_t(1) << 31) - 1) / INTER / 64 * 64;
constexpr int PREFILL_STREAMS = 3;  // prefill groups in flight at once, each on its own stream

// Column offsets inside one in_proj output row: z | x | B | C | dt (src/model.rs:638-640, :656-658).
constexpr int OFF_Z = 0, OFF_X = DI, OFF_B = DI + DI, OFF_C = DI + DI + DS, OFF_DT = DI + DXBC;

inline bool is_mamba(int l) { return l % 4 < 3; }  // src/model.rs:207, :261
inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

thread_local std::string g_err;

int fail(int status, const std::string& msg) {
    g_err = msg;
    return status;
}

struct KrkError {
    int status;
    std::string msg;
};

inline void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw KrkError{KRK_CUDA, std::string(what) + ": " + cudaGetErrorString(e)};
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) ck(cudaSetDevice(dev), "cudaSetDevice");
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// A device arena: one cudaMalloc, bump-allocated 256-byte aligned slices.
struct Arena {
    char* base = nullptr;
    size_t cap = 0, used = 0;
    void reserve(size_t bytes) {
        release();
        if (bytes == 0) return;
        ck(cudaMalloc(&base, bytes), "cudaMalloc");
        cap = bytes;
        used = 0;
    }
    template <typename T>
    T* take(size_t count) {
        size_t off = round_up((int64_t)used, 256);
        size_t bytes = count * sizeof(T);
        if (off + bytes > cap) throw KrkError{KRK_CHECK_FAILED, "internal arena overflow"};
        used = off + bytes;
        return reinterpret_cast<T*>(base + off);
    }
    void release() {
        if (base) cudaFree(base);
        base = nullptr;
        cap = used = 0;
    }
    ~Arena() { release(); }
};

// Byte budget of a list of slices (mirrors Arena::take's alignment).
struct Budget {
    size_t bytes = 0;
    template <typename T>
    void add(size_t count) { bytes = round_up((int64_t)bytes, 256) + count * sizeof(T); }
};

// Pinned host memory for a call's small host<->device traffic (prefill group
// tables, generation limits, seeds, positions, the generated tokens): copies
// from and to it are truly asynchronous, so a call issues all its work and
// synchronises once at its end.  Every API call of a state ends with a
// stream synchronisation, so the next call may reuse the buffer; ensure() is
// only called at the start of a call, when no copy from it is pending.
struct HostStage {
    char* base = nullptr;
    size_t cap = 0, used = 0;
    void ensure(size_t bytes) {
        used = 0;
        if (bytes <= cap) return;
        release();
        ck(cudaHostAlloc((void**)&base, bytes, cudaHostAllocDefault), "cudaHostAlloc");
        cap = bytes;
    }
    template <typename T>
    T* take(size_t count) {
        size_t off = round_up((int64_t)used, 256);
        size_t bytes = count * sizeof(T);
        if (off + bytes > cap) throw KrkError{KRK_CHECK_FAILED, "internal host staging overflow"};
        used = off + bytes;
        return reinterpret_cast<T*>(base + off);
    }
    void release() {
        if (base) cudaFreeHost(base);
        base = nullptr;
        cap = used = 0;
    }
    ~HostStage() { release(); }
};

struct LayerW {
    // Mamba (src/model.rs:86-96)
    float *ln = nullptr, *in_t = nullptr, *conv_w = nullptr, *conv_b = nullptr, *dt_bias = nullptr,
          *a_neg = nullptr, *dsk = nullptr, *norm_w = nullptr, *out_t = nullptr;
    // Attention (src/model.rs:98-105)
    float *ln1 = nullptr, *qkv_t = nullptr, *wo_t = nullptr, *ln2 = nullptr, *fc1_t = nullptr, *fc2_t = nullptr;
};

}  // namespace

struct krk_model {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t stream2 = nullptr;  // second part of a split decode batch
    cudaStream_t stream3 = nullptr, stream4 = nullptr;  // third and fourth parts
    Arena arena;
    float *wte = nullptr, *wte_t = nullptr, *lnf = nullptr;
    LayerW L[NL];
};

namespace {

// Per-kernel-class CUDA-event timing of a state's calls (krk_state_profile).
struct Prof {
    bool on = false;
    bool per_kernel = false;  // false: only the KRK_PROF_DEVICE_TOTAL bracket
    bool total_open = false;
    cudaEvent_t total_start = nullptr;
    std::vector<cudaEvent_t> pool;
    struct Pending {
        int cls;
        cudaEvent_t a, b;
        int64_t units;
    };
    std::vector<Pending> pending;
    double ms[KRK_PROF_CLASSES] = {};
    int64_t n[KRK_PROF_CLASSES] = {};
    int64_t units[KRK_PROF_CLASSES] = {};
    cudaEvent_t get() {
        if (pool.empty()) {
            cudaEvent_t e;
            ck(cudaEventCreate(&e), "event create");
            return e;
        }
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    void clear_events() {
        for (auto& p : pending) {
            pool.push_back(p.a);
            pool.push_back(p.b);
        }
        pending.clear();
        if (total_start) pool.push_back(total_start);
        total_start = nullptr;
        total_open = false;
    }
    ~Prof() {
        clear_events();
        for (auto e : pool) cudaEventDestroy(e);
    }
};

struct PrefillWs {
    int64_t cap_tokens = 0;
    int cap_seqs = 0;
    Arena arena;
    float *x_t, *hn_t, *zx, *xbc, *y_t, *yn_t, *qkv, *ao_t, *mlp_t;
};

}  // namespace

struct krk_state {
    const krk_model* m = nullptr;
    int B = 0, ctx = 0;
    int64_t Mp = 0;
    Arena arena;
    float *conv[NL] = {}, *ssm[NL] = {}, *kc[NL] = {}, *vc[NL] = {};
    int32_t* pos_d = nullptr;
    uint8_t* active_d = nullptr;
    uint32_t* seen_d = nullptr;
    uint32_t* tok_d = nullptr;
    int32_t* step_d = nullptr;
    int32_t* err_d = nullptr;  // set by a decode attention kernel whose K/V copy wait timed out
    uint32_t* rng_d = nullptr;  // [B][10] sampler random state (stochastic generation)
    float *h_t, *hn_t, *zx, *y_t, *yn_t, *qkv, *ao_t, *mlp_t, *logits, *attn_work;
    float2* rope = nullptr;  // (cos, sin) per [position][pair], from the host libm as src/math.rs:243-247
    int attn_split = 2048;
    int decode_streams = 3;  // decode batches of 256+ in up to this many parts on their own streams
    std::vector<int64_t> pos_h;
    PrefillWs pre[PREFILL_STREAMS];  // one workspace per prefill stream
    HostStage stage;                 // pinned per-call host tables (see HostStage)
    Arena meta_arena;                // their device copy: one H2D copy per call, same layout
    Arena prompt_arena;              // the call's packed prompt tokens on the device
    size_t prompt_cap = 0;
    Prof prof;
    Arena hist_arena;
    int64_t hist_cap = 0;
    uint32_t* hist_d = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;  // ordering of the decode streams
    cudaEvent_t ev_join3 = nullptr, ev_join4 = nullptr;
    // CUDA graphs of one decode step for batches of one 64-row tile, one per
    // count of attention key blocks (index: blocks - 1); captured on first use.
    std::vector<cudaGraphExec_t> step_graphs;
    std::vector<uint64_t> step_graph_kernels;
    bool step_graphs_on = true;
};

namespace {

// ------------------------------------------------------------------ loading
struct HostTensor {
    const float* p;
    size_t n;
};

HostTensor get_tensor(const krk::SafeTensorsFile& f, const std::string& name, size_t expect) {
    const krk::TensorInfo* t = f.info(name);
    if (!t) throw KrkError{KRK_NOT_FOUND, "Tensor '" + name + "' not found in model"};
    if (t->dtype != "F32") throw KrkError{KRK_IO, "Tensor '" + name + "' has dtype " + t->dtype + ", expected F32"};
    size_t n = (size_t)((t->end - t->begin) / 4);
    if (n != expect)
        throw KrkError{KRK_IO, "Tensor '" + name + "' holds " + std::to_string(n) + " floats, expected " +
                                   std::to_string(expect)};
    return {reinterpret_cast<const float*>(f.data(*t)), n};  // x86 host: little-endian, unaligned loads are fine
}

std::vector<float> copy_vec(const HostTensor& t) {
    std::vector<float> v(t.n);
    memcpy(v.data(), t.p, t.n * 4);
    return v;
}

// What upload_weights copies: a tensor straight from the mapped file (plain),
// a [rows][cols] tensor to be transposed on the device into [cols][ld] (the
// K-major layout of the projections), or a host-computed vector.
struct HostWeights {
    struct Upload {
        float** dst;
        const float* src = nullptr;  // in the mapped file
        size_t n = 0;                // floats at src (plain / transposed) or in data
        int rows = 0, cols = 0, ld = 0;  // ld > 0: transposed
        std::vector<float> data;         // host-computed
        size_t dst_floats() const { return ld > 0 ? (size_t)cols * ld : (data.empty() ? n : data.size()); }
    };
    krk::SafeTensorsFile file;  // mapped until the upload is done
    std::vector<Upload> ups;
};

// Reads and checks every tensor (src/model.rs:256-294); touches no device.
void read_weights(krk_model* m, const std::string& path, HostWeights& hw) {
    krk::SafeTensorsFile& f = hw.file;
    std::string err;
    if (!f.open(path, err)) throw KrkError{KRK_IO, err};
    auto plain = [&](float** dst, const HostTensor& t) {
        HostWeights::Upload u;
        u.dst = dst; u.src = t.p; u.n = t.n;
        hw.ups.push_back(std::move(u));
    };
    auto transposed = [&](float** dst, const HostTensor& t, int rows, int cols, int ld) {
        HostWeights::Upload u;
        u.dst = dst; u.src = t.p; u.n = t.n; u.rows = rows; u.cols = cols; u.ld = ld;
        hw.ups.push_back(std::move(u));
    };

    HostTensor wte = get_tensor(f, "wte.weight", (size_t)VOC * HID);
    plain(&m->wte, wte);
    transposed(&m->wte_t, wte, VOC, HID, VOC);
    plain(&m->lnf, get_tensor(f, "lnf.weight", HID));
    for (int i = 0; i < NL; ++i) {
        const std::string p = "blocks." + std::to_string(i) + ".";
        LayerW& L = m->L[i];
        if (is_mamba(i)) {
            plain(&L.ln, get_tensor(f, p + "ln.weight", HID));
            transposed(&L.in_t, get_tensor(f, p + "mixer.in_proj.weight", (size_t)DIP * HID), DIP, HID, DIP_PAD);
            plain(&L.conv_w, get_tensor(f, p + "mixer.conv1d.weight", (size_t)DXBC * 4));
            plain(&L.conv_b, get_tensor(f, p + "mixer.conv1d.bias", DXBC));
            plain(&L.dt_bias, get_tensor(f, p + "mixer.dt_bias", MH));
            HostWeights::Upload a;
            a.dst = &L.a_neg;
            a.data = copy_vec(get_tensor(f, p + "mixer.A_log", MH));
            for (float& v : a.data) v = -expf(v);  // A = -exp(A_log) (src/model.rs:273-274), host libm
            hw.ups.push_back(std::move(a));
            plain(&L.dsk, get_tensor(f, p + "mixer.D", MH));
            plain(&L.norm_w, get_tensor(f, p + "mixer.norm.weight", DI));
            transposed(&L.out_t, get_tensor(f, p + "mixer.out_proj.weight", (size_t)HID * DI), HID, DI, HID);
        } else {
            plain(&L.ln1, get_tensor(f, p + "ln1.weight", HID));
            transposed(&L.qkv_t, get_tensor(f, p + "wqkv.weight", (size_t)QKV * HID), QKV, HID, QKV);
            transposed(&L.wo_t, get_tensor(f, p + "wo.weight", (size_t)HID * HID), HID, HID, HID);
            plain(&L.ln2, get_tensor(f, p + "ln2.weight", HID));
            transposed(&L.fc1_t, get_tensor(f, p + "fc1.weight", (size_t)INTER * HID), INTER, HID, INTER);
            transposed(&L.fc2_t, get_tensor(f, p + "fc2.weight", (size_t)HID * INTER), HID, INTER, HID);
        }
    }
}

// Copies every tensor from the mapped file to the device; the projections go
// through a staging buffer and are transposed by a kernel.
void upload_weights(krk_model* m, HostWeights& hw) {
    Budget bud;
    size_t stage = 0;
    for (auto& u : hw.ups) {
        bud.add<float>(u.dst_floats());
        if (u.ld > 0) stage = std::max(stage, u.n);
    }
    m->arena.reserve(bud.bytes);
    float* staging = nullptr;
    if (stage) ck(cudaMalloc(&staging, stage * 4), "staging alloc");
    try {
        for (auto& u : hw.ups) {
            *u.dst = m->arena.take<float>(u.dst_floats());
            // all on the model stream: the copy into the staging buffer, the
            // transpose that reads it, and the next copy that refills it
            if (u.ld > 0) {
                ck(cudaMemcpyAsync(staging, u.src, u.n * 4, cudaMemcpyHostToDevice, m->stream), "weight upload");
                ck(krk::transpose_pad(staging, u.rows, u.cols, *u.dst, u.ld, m->stream), "weight transpose");
            } else if (!u.data.empty()) {
                ck(cudaMemcpyAsync(*u.dst, u.data.data(), u.data.size() * 4, cudaMemcpyHostToDevice, m->stream),
                   "weight upload");
            } else {
                ck(cudaMemcpyAsync(*u.dst, u.src, u.n * 4, cudaMemcpyHostToDevice, m->stream), "weight upload");
            }
        }
        ck(cudaStreamSynchronize(m->stream), "weight upload");
    } catch (...) {
        if (staging) cudaFree(staging);
        throw;
    }
    if (staging) ck(cudaFree(staging), "staging free");
}

// ------------------------------------------------------------------ state
void create_state(krk_state* s, const krk_model* m, int B, int ctx) {
    s->m = m;
    s->B = B;
    s->ctx = ctx;
    s->Mp = round_up(B, 64);
    const int64_t Mp = s->Mp;
    // 512 keys per split (attn_decode_kernel): one CTA per (sequence, head)
    // up to 512 positions, and a one-round-trip merge beyond; +1.6% tokens/s at
    // 1024 and 128 sequences over 64-key blocks with their merge.
    s->attn_split = 512;
    const size_t work = krk::attn_decode_work_floats(B, NH, HD, ctx, s->attn_split);
    Budget b;
    for (int l = 0; l < NL; ++l) {
        if (is_mamba(l)) {
            b.add<float>((size_t)B * DXBC * 4);
            b.add<float>((size_t)B * MH * MP * DS);
        } else {
            b.add<float>((size_t)B * ctx * HID);
            b.add<float>((size_t)B * ctx * HID);
        }
    }
    b.add<int32_t>(B); b.add<uint8_t>(B); b.add<uint32_t>((size_t)B * SEEN_WORDS); b.add<uint32_t>(Mp);
    b.add<int32_t>(1); b.add<int32_t>(1); b.add<uint32_t>((size_t)B * 10);
    b.add<float>(HID * Mp); b.add<float>(HID * Mp); b.add<float>(Mp * DIP_PAD); b.add<float>(DI * Mp);
    b.add<float>(DI * Mp); b.add<float>(Mp * QKV); b.add<float>(HID * Mp); b.add<float>(INTER * Mp);
    b.add<float>(Mp * VOC); b.add<float>(work); b.add<float2>((size_t)ctx * (HD / 2));
    s->arena.reserve(b.bytes);
    for (int l = 0; l < NL; ++l) {
        if (is_mamba(l)) {
            s->conv[l] = s->arena.take<float>((size_t)B * DXBC * 4);
            s->ssm[l] = s->arena.take<float>((size_t)B * MH * MP * DS);
        } else {
            s->kc[l] = s->arena.take<float>((size_t)B * ctx * HID);
            s->vc[l] = s->arena.take<float>((size_t)B * ctx * HID);
        }
    }
    s->pos_d = s->arena.take<int32_t>(B);
    s->active_d = s->arena.take<uint8_t>(B);
    s->seen_d = s->arena.take<uint32_t>((size_t)B * SEEN_WORDS);
    s->tok_d = s->arena.take<uint32_t>(Mp);
    s->step_d = s->arena.take<int32_t>(1);
    s->err_d = s->arena.take<int32_t>(1);
    s->rng_d = s->arena.take<uint32_t>((size_t)B * 10);
    s->h_t = s->arena.take<float>(HID * Mp);
    s->hn_t = s->arena.take<float>(HID * Mp);
    s->zx = s->arena.take<float>(Mp * DIP_PAD);
    s->y_t = s->arena.take<float>(DI * Mp);
    s->yn_t = s->arena.take<float>(DI * Mp);
    s->qkv = s->arena.take<float>(Mp * QKV);
    s->ao_t = s->arena.take<float>(HID * Mp);
    s->mlp_t = s->arena.take<float>(INTER * Mp);
    s->logits = s->arena.take<float>(Mp * VOC);
    s->attn_work = s->arena.take<float>(work);
    s->rope = s->arena.take<float2>((size_t)ctx * (HD / 2));
    ck(cudaMemsetAsync(s->arena.base, 0, s->arena.cap, m->stream), "state memset");
    // RoPE coefficients exactly as src/math.rs:243-247 computes them, with the
    // host's f32 powf / cosf / sinf (the functions the reference calls).
    std::vector<float2> rope((size_t)ctx * (HD / 2));
    for (int p = 0; p < ctx; ++p)
        for (int i = 0; i < HD / 2; ++i) {
            const float invf = 1.0f / powf(THETA, ((float)i * 2.0f) / (float)HD);
            const float ang = (float)p * invf;
            rope[(size_t)p * (HD / 2) + i] = make_float2(cosf(ang), sinf(ang));
        }
    ck(cudaMemcpyAsync(s->rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice, m->stream),
       "rope table");
    ck(cudaStreamSynchronize(m->stream), "state init");
    s->pos_h.assign(B, 0);
    ck(cudaEventCreateWithFlags(&s->ev_fork, cudaEventDisableTiming), "event create");
    ck(cudaEventCreateWithFlags(&s->ev_join, cudaEventDisableTiming), "event create");
    ck(cudaEventCreateWithFlags(&s->ev_join3, cudaEventDisableTiming), "event create");
    ck(cudaEventCreateWithFlags(&s->ev_join4, cudaEventDisableTiming), "event create");
}

void sync_model_streams(const krk_model* m) {
    for (cudaStream_t x : {m->stream, m->stream2, m->stream3, m->stream4})
        if (x) ck(cudaStreamSynchronize(x), "stream sync");
}

void ensure_prefill_ws(krk_state* s, int k, int64_t tokens, int seqs) {
    PrefillWs& w = s->pre[k];
    if (tokens <= w.cap_tokens && seqs <= w.cap_seqs) return;
    const int64_t T = round_up(std::max<int64_t>(tokens, w.cap_tokens), 64);
    const int S = std::max(seqs, w.cap_seqs);
    Budget b;
    b.add<float>(HID * T); b.add<float>(HID * T); b.add<float>(T * DIP_PAD); b.add<float>(T * DXBC);
    b.add<float>(DI * T); b.add<float>(DI * T); b.add<float>(T * QKV); b.add<float>(HID * T);
    b.add<float>(INTER * T);
    sync_model_streams(s->m);  // the old workspace may still be in use on any stream
    w.arena.reserve(b.bytes);
    w.x_t = w.arena.take<float>(HID * T);
    w.hn_t = w.arena.take<float>(HID * T);
    w.zx = w.arena.take<float>(T * DIP_PAD);
    w.xbc = w.arena.take<float>(T * DXBC);
    w.y_t = w.arena.take<float>(DI * T);
    w.yn_t = w.arena.take<float>(DI * T);
    w.qkv = w.arena.take<float>(T * QKV);
    w.ao_t = w.arena.take<float>(HID * T);
    w.mlp_t = w.arena.take<float>(INTER * T);
    ck(cudaMemsetAsync(w.arena.base, 0, w.arena.cap, s->m->stream), "prefill ws memset");
    w.cap_tokens = T;
    w.cap_seqs = S;
}

inline void kk(cudaError_t e, const char* what) { ck(e, what); }

// Zeroes the padding columns [valid, ld) of a feature-major [rows][ld] buffer.
void zero_pad_cols(float* buf, int64_t ld, int64_t valid, int rows, cudaStream_t st) {
    if (valid >= ld) return;
    kk(cudaMemset2DAsync(buf + valid, ld * 4, 0, (ld - valid) * 4, rows, st), "memset2d");
}

// Records CUDA events around f() on stream st when profiling is on; units is
// the number of decode sequences the launch processes (0 elsewhere).
template <typename F>
void timed_on(krk_state* s, cudaStream_t st, int cls, int64_t units, F&& f) {
    if (!s->prof.on || !s->prof.per_kernel) {
        f();
        return;
    }
    cudaEvent_t a = s->prof.get(), b = s->prof.get();
    kk(cudaEventRecord(a, st), "event");
    f();
    kk(cudaEventRecord(b, st), "event");
    s->prof.pending.push_back({cls, a, b, units});
}
template <typename F>
void timed(krk_state* s, int cls, F&& f) {
    timed_on(s, s->m->stream, cls, 0, f);
}

// Device-time bracket of a whole call: opened after the call's inputs reached
// the device, closed before its outputs leave it.
void total_begin(krk_state* s) {
    if (!s->prof.on || s->prof.total_open) return;
    s->prof.total_start = s->prof.get();
    kk(cudaEventRecord(s->prof.total_start, s->m->stream), "event");
    s->prof.total_open = true;
}
void total_end(krk_state* s) {
    if (!s->prof.on || !s->prof.total_open) return;
    cudaEvent_t b = s->prof.get();
    kk(cudaEventRecord(b, s->m->stream), "event");
    s->prof.pending.push_back({KRK_PROF_DEVICE_TOTAL, s->prof.total_start, b, 0});
    s->prof.total_start = nullptr;
    s->prof.total_open = false;
}
// Called after the stream is synchronised: folds pending event pairs into totals.
void prof_collect(krk_state* s) {
    if (!s->prof.on) return;
    for (auto& p : s->prof.pending) {
        float ms = 0.0f;
        kk(cudaEventElapsedTime(&ms, p.a, p.b), "event elapsed");
        s->prof.ms[p.cls] += ms;
        s->prof.n[p.cls] += 1;
        s->prof.units[p.cls] += p.units;
    }
    s->prof.clear_events();
}

// Event pairs are read back lazily (reading each pair costs host time between
// calls that the device would spend idle): at krk_state_profile_read, or once
// many are pending.
void prof_collect_if_large(krk_state* s) {
    if (s->prof.pending.size() > 400000) prof_collect(s);
}

// ------------------------------------------------------------------ forward
// A slice of the decode batch: sequences [b0, b0 + nb), which are columns
// [b0, b0 + M) of the feature-major activations (M = nb rounded up to 64, or
// the padded remainder), run on stream st.
struct Part {
    int b0, nb, M;
    cudaStream_t st;
    int tile_rows;  // GEMM CTA tile height (0: chosen for the kernel running alone)
    // Launch priority of the part's projections (0: the stream's).  With parts
    // on several streams the projections, the FP32-bound critical path, take
    // the device's most urgent priority, and the HBM-bound SSD updates and
    // attention of the other parts fill the SMs they leave: +1.0% tokens/s at
    // 1024 sequences (the opposite, urgent SSD update and attention, -0.6%).
    int gemm_priority = 0;
};

// The device's most urgent stream priority (queried once per process).
int urgent_priority() {
    static int p = 1;
    if (p == 1) {
        int least = 0, greatest = 0;
        p = cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess ? greatest : 0;
        if (p == 1) p = 0;
    }
    return p;
}

template <typename F>
void timed(krk_state* s, const Part& p, int cls, F&& f) {
    timed_on(s, p.st, cls, p.nb, f);
}

// A single-part decode of a few sequences computes a projection of N columns
// in the few-rows form, over the real rows only (every consumer reads only
// those), where that form is the faster one.
bool few_rows(const Part& p, int N) { return p.tile_rows == 0 && krk::gemm_few_rows(p.nb, N); }

// Final norm + tied LM head (src/model.rs:620-621).
void lm_head(krk_state* s, const Part& p) {
    const krk_model* m = s->m;
    const int Mp = (int)s->Mp;
    const bool few = few_rows(p, VOC);
    if (few) {  // lnf inside the few-rows projection
        timed(s, p, KRK_PROF_GEMM, [&] {
            kk(krk::gemm_few_norm(s->h_t + p.b0, Mp, m->wte_t, VOC, s->logits + (size_t)p.b0 * VOC, VOC, p.nb, VOC,
                                  HID, krk::EPI_STORE, false, krk::GemmNorm{m->lnf, RMS_EPS}, nullptr, p.st),
               "lnf + lm head");
        });
        return;
    }
    timed(s, p, KRK_PROF_NORM, [&] {
        kk(krk::rmsnorm_fm(s->h_t + p.b0, Mp, m->lnf, RMS_EPS, HID, p.nb, s->hn_t + p.b0, Mp, p.st), "lnf");
    });
    timed(s, p, KRK_PROF_GEMM, [&] {
        kk(krk::gemm_tiled(s->hn_t + p.b0, Mp, m->wte_t, VOC, s->logits + (size_t)p.b0 * VOC, VOC, p.M, VOC, HID,
                           krk::EPI_STORE, false, p.tile_rows, p.st),
           "lm head");
    });
}

void lm_head(krk_state* s) { lm_head(s, Part{0, s->B, (int)s->Mp, s->m->stream, 0}); }

void decode_embed(krk_state* s, const Part& p) {
    const int Mp = (int)s->Mp;
    timed(s, p, KRK_PROF_OTHER, [&] {
        kk(krk::embed_fm(s->tok_d + p.b0, s->m->wte, VOC, HID, p.nb, s->h_t + p.b0, Mp, p.st), "embed");
    });
}

// Layer l of one decode step for a slice of the batch (src/model.rs:626-783).
void decode_layer(krk_state* s, int l, const uint8_t* active, int max_keys, const Part& p) {
    const krk_model* m = s->m;
    const LayerW& L = m->L[l];
    const int Mp = (int)s->Mp, b0 = p.b0, nb = p.nb;
    // rows and tile height of a projection of N columns
    auto rows = [&](int N) { return few_rows(p, N) ? nb : p.M; };
    auto tile = [&](int N) { return few_rows(p, N) ? 1 : p.tile_rows; };
    cudaStream_t st = p.st;
    const uint8_t* act = active ? active + b0 : nullptr;
    float* h = s->h_t + b0;
    float* hn = s->hn_t + b0;
    auto gemm = [&](const float* A, const float* W, int N, int K, float* C, int ldc, int epi, bool fm, const char* w) {
        timed(s, p, KRK_PROF_GEMM,
              [&] {
                  krk::PriorityScope pr(p.gemm_priority);
                  kk(krk::gemm_tiled(A, Mp, W, N, C, ldc, rows(N), N, K, epi, fm, tile(N), st), w);
              });
    };
    auto norm = [&](const float* x, const float* w, float eps, int K, float* out, const char* what) {
        timed(s, p, KRK_PROF_NORM, [&] { kk(krk::rmsnorm_fm(x, Mp, w, eps, K, nb, out, Mp, st), what); });
    };
    // rms_norm(x) into xn and the projection of xn, or both in one few-rows launch
    auto norm_gemm = [&](const float* x, const float* nw, float eps, float* xn, const float* W, int N, int K, float* C,
                         int ldc, int epi, bool fm, const char* what) {
        if (few_rows(p, N)) {
            timed(s, p, KRK_PROF_GEMM, [&] {
                kk(krk::gemm_few_norm(x, Mp, W, N, C, ldc, nb, N, K, epi, fm, krk::GemmNorm{nw, eps}, nullptr, st), what);
            });
        } else {
            norm(x, nw, eps, K, xn, what);
            gemm(xn, W, N, K, C, ldc, epi, fm, what);
        }
    };
    if (is_mamba(l)) {  // src/model.rs:626-702
        float* zx = s->zx + (size_t)b0 * DIP_PAD;
        // in_proj with the decode conv + SiLU of its x, B, C columns in the epilogue
        krk::GemmConv cv{s->conv[l] + (size_t)b0 * DXBC * 4, L.conv_w, L.conv_b, act, nb, OFF_X, OFF_X + DXBC};
        if (few_rows(p, DIP_PAD)) {  // ln inside the few-rows projection
            timed(s, p, KRK_PROF_GEMM, [&] {
                kk(krk::gemm_few_norm(h, Mp, L.in_t, DIP_PAD, zx, DIP_PAD, nb, DIP_PAD, HID, krk::EPI_CONV, false,
                                      krk::GemmNorm{L.ln, RMS_EPS}, &cv, st),
                   "ln + in_proj + conv");
            });
        } else {
            norm(h, L.ln, RMS_EPS, HID, hn, "ln");
            timed(s, p, KRK_PROF_GEMM, [&] {
                krk::PriorityScope pr(p.gemm_priority);
                kk(krk::gemm_conv(hn, Mp, L.in_t, DIP_PAD, zx, DIP_PAD, p.M, DIP_PAD, HID, p.tile_rows, cv, st),
                   "in_proj + conv");
            });
        }
        krk::SsdStepArgs a{};
        a.x = zx + OFF_X; a.x_sb = DIP_PAD;
        a.bm = zx + OFF_B; a.cm = zx + OFF_C; a.bc_sb = DIP_PAD;
        a.dt = zx + OFF_DT; a.dt_sb = DIP_PAD;
        a.z = zx + OFF_Z; a.z_sb = DIP_PAD;
        a.ssm = s->ssm[l] + (size_t)b0 * MH * MP * DS;
        a.dt_bias = L.dt_bias; a.a_neg = L.a_neg; a.dsk = L.dsk;
        a.y = s->y_t + b0; a.y_sb = 1; a.y_sc = Mp;
        a.active = act;
        a.B = nb; a.H = MH; a.P = MP; a.N = DS;
        timed(s, p, KRK_PROF_SSD_STEP, [&] {
            kk(krk::ssd_step(a, false, st), "ssd step");
        });
        norm_gemm(s->y_t + b0, L.norm_w, MNORM_EPS, s->yn_t + b0, L.out_t, HID, DI, h, Mp, krk::EPI_RESIDUAL, true,
                  "gated norm + out_proj");
    } else {  // src/model.rs:704-783
        float* qkv = s->qkv + (size_t)b0 * QKV;
        norm_gemm(h, L.ln1, RMS_EPS, hn, L.qkv_t, QKV, HID, qkv, QKV, krk::EPI_STORE, false, "ln1 + wqkv");
        krk::AttnDecodeArgs a{};
        a.q = qkv; a.k = qkv + HID; a.v = qkv + 2 * HID; a.in_sb = QKV; a.in_sh = HD;
        a.c_sb = (int64_t)s->ctx * HID; a.c_sh = HD; a.c_st = HID;
        a.kc = s->kc[l] + (size_t)b0 * a.c_sb; a.vc = s->vc[l] + (size_t)b0 * a.c_sb;
        a.pos = s->pos_d + b0; a.active = act;
        a.out = s->ao_t + b0; a.o_sb = 1; a.o_sh = (int64_t)HD * Mp; a.o_sd = Mp;
        const size_t max_splits = (size_t)(s->ctx + s->attn_split - 1) / s->attn_split;
        a.work = s->attn_work + (size_t)b0 * NH * max_splits * (HD + 2);
        a.B = nb; a.H = NH; a.dh = HD; a.ctx = s->ctx; a.split = s->attn_split; a.theta = THETA;
        a.rope = s->rope;
        a.max_keys = max_keys;
        a.err = s->err_d;
        timed(s, p, KRK_PROF_ATTN_DECODE, [&] {
            kk(krk::attn_decode(a, st), "attention");
        });
        gemm(s->ao_t + b0, L.wo_t, HID, HID, h, Mp, krk::EPI_RESIDUAL, true, "wo");
        norm_gemm(h, L.ln2, RMS_EPS, hn, L.fc1_t, INTER, HID, s->mlp_t + b0, Mp, krk::EPI_GELU, true, "ln2 + fc1");
        gemm(s->mlp_t + b0, L.fc2_t, HID, INTER, h, Mp, krk::EPI_RESIDUAL, true, "fc2");
    }
}

// One decode step for all sequences: tokens in tok_d, positions in pos_d
// (src/model.rs:586-624).  Does not advance positions.  max_keys is an upper
// bound on pos + 1 over the batch (the attention grid covers no key block
// beyond it).
//
// A batch of 256 or more sequences runs as two halves on two streams, layer by
// layer.  The halves are independent, so while one half's projections keep the
// FP32 pipes busy the other half's SSD update or attention streams its state
// through HBM, and each kernel's last partial wave is filled by the other half.
// The decode batch as one part, or split into up to decode_streams parts of
// whole 64-row tiles (two tiles at least, sizes differing by one tile at most)
// on the model's streams.
int decode_parts(const krk_state* s, Part parts[4]) {
    const krk_model* m = s->m;
    const int B = s->B, Mp = (int)s->Mp;
    const int n = std::min(s->decode_streams, Mp / 128);  // parts of at least two tiles
    cudaStream_t st[4] = {m->stream, m->stream2, m->stream3, m->stream4};
    if (n >= 2 && s->ev_fork) {
        const int tiles = Mp / 64;  // parts of tiles / n or tiles / n + 1 whole tiles, larger first
        int np = 0, b0 = 0;
        for (int i = 0; i < n && b0 < B; ++i) {
            const int M = 64 * (tiles / n + (i < tiles % n ? 1 : 0));
            parts[np++] = Part{b0, std::min(M, B - b0), M, st[i], 64, urgent_priority()};
            b0 += M;
        }
        if (np >= 2) return np;
    }
    parts[0] = Part{0, B, Mp, m->stream, 0};
    return 1;
}

void decode_forward(krk_state* s, const uint8_t* active, int max_keys) {
    const krk_model* m = s->m;
    Part parts[4];
    const int np = decode_parts(s, parts);
    // The step of a few sequences is a chain of ~30 kernels of a few
    // microseconds each, whose launch gaps and first memory round trips are a
    // large share of the step: each kernel is scheduled behind the one before
    // it and prefetches its weights meanwhile (programmatic dependent launch;
    // step graphs: +7% tokens/s at 1 sequence, +2% at 8).  From 32 sequences
    // on it measured slower (-9% at 32, -6% at 128), and parts on several
    // streams fill each other's gaps anyway.  Per-kernel event timing wants
    // the kernels apart.
    krk::PdlScope pdl(np == 1 && s->B <= krk::GEMM_FEW_ROWS && !(s->prof.on && s->prof.per_kernel));
    cudaEvent_t joins[4] = {nullptr, s->ev_join, s->ev_join3, s->ev_join4};
    if (np >= 2) {
        kk(cudaEventRecord(s->ev_fork, m->stream), "fork");
        for (int i = 1; i < np; ++i) kk(cudaStreamWaitEvent(parts[i].st, s->ev_fork, 0), "fork");
    }
    for (int i = 0; i < np; ++i) decode_embed(s, parts[i]);
    for (int l = 0; l < NL; ++l)
        for (int i = 0; i < np; ++i) decode_layer(s, l, active, max_keys, parts[i]);
    for (int i = 0; i < np; ++i) lm_head(s, parts[i]);
    for (int i = 1; i < np; ++i) {
        kk(cudaEventRecord(joins[i], parts[i].st), "join");
        kk(cudaStreamWaitEvent(m->stream, joins[i], 0), "join");
    }
}

// A decode step is ~90 launches per part (~260 for one 64-row tile with the
// sampling, ~800 for three parts); for small batches their launch gaps, not
// their work, set the time per token, and for large ones the host's launch
// time approaches the device's.  The generation loop therefore replays a CUDA
// graph of decode_forward -- the parts' streams, forks and joins included --
// one graph per count of 64-key attention blocks (the attention grid's depth),
// captured the first time that count comes up.  The graph's attention reads up
// to blocks * 64 rows (fewer than ctx): rows past a sequence's position are
// masked as always.  Not used while per-kernel profiling records events around
// each launch, nor when the state's step graphs are switched off.
void decode_step(krk_state* s, int max_keys) {
    if ((s->prof.on && s->prof.per_kernel) || !s->step_graphs_on) {
        decode_forward(s, s->active_d, max_keys);
        return;
    }
    const int keys_cap = std::min(std::max(max_keys, 1), s->ctx);
    const int z = (keys_cap + s->attn_split - 1) / s->attn_split;
    const int keys = std::min(z * s->attn_split, s->ctx);
    if ((int)s->step_graphs.size() < z) {
        s->step_graphs.resize(z, nullptr);
        s->step_graph_kernels.resize(z, 0);
    }
    cudaStream_t st = s->m->stream;
    cudaGraphExec_t& ex = s->step_graphs[z - 1];
    if (!ex) {
        // capture: the launchers count their launches as they are recorded,
        // which stands for this first replay
        const uint64_t n0 = krk::launch_count();
        cudaGraph_t g = nullptr;
        kk(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "graph capture");
        try {
            decode_forward(s, s->active_d, keys);
        } catch (...) {
            cudaStreamEndCapture(st, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        kk(cudaStreamEndCapture(st, &g), "graph capture");
        const cudaError_t e = cudaGraphInstantiate(&ex, g, cudaGraphInstantiateFlagUseNodePriority);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) ex = nullptr;
        kk(e, "graph instantiate");
        s->step_graph_kernels[z - 1] = krk::launch_count() - n0;
    } else {
        krk::add_launches(s->step_graph_kernels[z - 1]);
    }
    kk(cudaGraphLaunch(ex, st), "graph launch");
}

// Device pointers to one prefill group's tables (in the call's metadata copy).
struct GroupDev {
    const uint32_t* tok;  // the group's packed prompt tokens
    const int32_t *cu, *start, *last, *dst, *row_seq;
    const int2* blk;
};

// Prefill of sequences [g0, g0+S) whose packed tokens and tables are on the device.
void prefill_group(krk_state* s, int g0, int S, int64_t rows, int nblk, int blk_rows, int kmax, PrefillWs& w,
                   const GroupDev& gd, cudaStream_t st) {
    const krk_model* m = s->m;
    auto timed = [&](krk_state* sp, int cls, auto&& f) { timed_on(sp, st, cls, 0, f); };
    const int T = (int)round_up(rows, 64);
    const int R = (int)rows;
    zero_pad_cols(w.x_t, T, R, HID, st);
    zero_pad_cols(w.hn_t, T, R, HID, st);
    zero_pad_cols(w.y_t, T, R, DI, st);
    zero_pad_cols(w.yn_t, T, R, DI, st);
    zero_pad_cols(w.ao_t, T, R, HID, st);
    timed(s, KRK_PROF_OTHER, [&] { kk(krk::embed_fm(gd.tok, m->wte, VOC, HID, R, w.x_t, T, st), "embed"); });
    for (int l = 0; l < NL; ++l) {
        const LayerW& L = m->L[l];
        if (is_mamba(l)) {  // src/model.rs:370-464
            timed(s, KRK_PROF_NORM, [&] { kk(krk::rmsnorm_fm(w.x_t, T, L.ln, RMS_EPS, HID, R, w.hn_t, T, st), "ln"); });
            timed(s, KRK_PROF_GEMM, [&] { kk(krk::gemm(w.hn_t, T, L.in_t, DIP_PAD, w.zx, DIP_PAD, T, DIP_PAD, HID, krk::EPI_STORE, false, st),
               "in_proj"); });
            timed(s, KRK_PROF_CONV, [&] { kk(krk::conv_prefill4(w.zx + OFF_X, DIP_PAD, w.xbc, DXBC, s->conv[l] + (size_t)g0 * DXBC * 4, L.conv_w,
                                  L.conv_b, gd.cu, S, DXBC, st),
               "conv"); });
            krk::SsdScanArgs a{};
            a.x = w.xbc; a.x_rs = DXBC;
            a.bm = w.xbc + DI; a.cm = w.xbc + DI + DS; a.bc_rs = DXBC;
            a.dt = w.zx + OFF_DT; a.dt_rs = DIP_PAD;
            a.z = w.zx + OFF_Z; a.z_rs = DIP_PAD;
            a.ssm = s->ssm[l] + (size_t)g0 * MH * MP * DS;
            a.dt_bias = L.dt_bias; a.a_neg = L.a_neg; a.dsk = L.dsk;
            a.y = w.y_t; a.y_rs = 1; a.y_cs = T;
            a.cu_seqlens = gd.cu;
            a.S = S; a.H = MH; a.P = MP; a.N = DS;
            timed(s, KRK_PROF_SSD_SCAN, [&] { kk(krk::ssd_scan(a, false, st), "ssd scan"); });
            timed(s, KRK_PROF_NORM, [&] { kk(krk::rmsnorm_fm(w.y_t, T, L.norm_w, MNORM_EPS, DI, R, w.yn_t, T, st), "gated norm"); });
            timed(s, KRK_PROF_GEMM, [&] { kk(krk::gemm(w.yn_t, T, L.out_t, HID, w.x_t, T, T, HID, DI, krk::EPI_RESIDUAL, true, st), "out_proj"); });
        } else {  // src/model.rs:466-583
            timed(s, KRK_PROF_NORM, [&] { kk(krk::rmsnorm_fm(w.x_t, T, L.ln1, RMS_EPS, HID, R, w.hn_t, T, st), "ln1"); });
            timed(s, KRK_PROF_GEMM, [&] { kk(krk::gemm(w.hn_t, T, L.qkv_t, QKV, w.qkv, QKV, T, QKV, HID, krk::EPI_STORE, false, st), "wqkv"); });
            float* kc = s->kc[l] + (size_t)g0 * s->ctx * HID;
            float* vc = s->vc[l] + (size_t)g0 * s->ctx * HID;
            const int64_t c_sb = (int64_t)s->ctx * HID;
            timed(s, KRK_PROF_OTHER, [&] { kk(krk::rope_kv_prefill(w.qkv, QKV, kc, vc, c_sb, HD, HID, gd.cu, gd.start, S, NH, HD, R, THETA, s->rope, st),
               "rope/kv"); });
            timed(s, KRK_PROF_ATTN_PREFILL, [&] { kk(krk::attn_prefill(w.qkv, QKV, kc, vc, c_sb, HD, HID, gd.cu, gd.start, gd.blk, nblk, blk_rows, NH, HD,
                                 kmax, w.ao_t, 1, T, st),
               "attention"); });
            timed(s, KRK_PROF_GEMM, [&] { kk(krk::gemm(w.ao_t, T, L.wo_t, HID, w.x_t, T, T, HID, HID, krk::EPI_RESIDUAL, true, st), "wo"); });
            timed(s, KRK_PROF_NORM, [&] { kk(krk::rmsnorm_fm(w.x_t, T, L.ln2, RMS_EPS, HID, R, w.hn_t, T, st), "ln2"); });
            timed(s, KRK_PROF_GEMM, [&] { kk(krk::gemm(w.hn_t, T, L.fc1_t, INTER, w.mlp_t, T, T, INTER, HID, krk::EPI_GELU, true, st), "fc1"); });
            timed(s, KRK_PROF_GEMM, [&] { kk(krk::gemm(w.mlp_t, T, L.fc2_t, HID, w.x_t, T, T, HID, INTER, krk::EPI_RESIDUAL, true, st), "fc2"); });
        }
    }
    // last token of each sequence -> decode residual buffer column g0 + s
    timed(s, KRK_PROF_OTHER, [&] { kk(krk::gather_cols(w.x_t, T, gd.last, s->h_t, (int)s->Mp, gd.dst, HID, S, st), "gather last"); });
}

// A validated batched prefill split into groups of whole sequences of up to
// PREFILL_GROUP_TOKENS tokens.  The groups are independent (disjoint
// sequences, states and cache rows), so up to PREFILL_STREAMS of them run at
// once, group i on stream i % PREFILL_STREAMS with that stream's workspace:
// one group's projections overlap another's scan, attention and norms.
// Stream order makes a workspace's reuse safe.  The group tables are built in
// the state's pinned stage and reach the device with the call's one metadata
// copy.
struct PrefillPlan {
    struct Group {
        int g0 = 0, S = 0;
        int64_t rows = 0, off = 0;  // packed rows and their offset in the prompt array
        int blk_rows = 1, kmax = 1, nblk = 0;
        int32_t *cu = nullptr, *start = nullptr, *last = nullptr, *dst = nullptr, *row_seq = nullptr;
        int2* blk = nullptr;  // prefill attention blocks: (sequence, first row)
    };
    std::vector<Group> groups;
    int64_t total = 0;
    int32_t* pos_after = nullptr;  // [B] positions after the prefill (stage)
};

inline int64_t start_pos(const krk_state* s, int b, bool from_zero) { return from_zero ? 0 : s->pos_h[b]; }

// The reference's checks in its order (src/model.rs:317-335): empty, context,
// token.  from_zero: against positions 0 (the prefill follows a reset).
int check_prefill(const krk_state* s, const uint32_t* tokens, const int32_t* lens, bool from_zero,
                  int64_t* total_out) {
    const int B = s->B;
    if (!lens) return fail(KRK_INVALID, "null lens");
    int64_t total = 0;
    for (int b = 0; b < B; ++b) {
        if (lens[b] <= 0) return fail(KRK_EMPTY, "Cannot prefill empty sequence");
        total += lens[b];
    }
    if (!tokens) return fail(KRK_INVALID, "null tokens");
    for (int b = 0; b < B; ++b) {
        const int64_t end = start_pos(s, b, from_zero) + lens[b];
        if (end > s->ctx)
            return fail(KRK_CONTEXT_OVERFLOW, "Sequence length " + std::to_string(end) + " exceeds context limit " +
                                                  std::to_string(s->ctx));
    }
    for (int64_t i = 0; i < total; ++i)
        if (tokens[i] >= (uint32_t)VOC)
            return fail(KRK_BAD_TOKEN,
                        "Token ID " + std::to_string(tokens[i]) + " exceeds vocab size " + std::to_string(VOC));
    *total_out = total;
    return KRK_OK;
}

// Forms the groups and adds their host tables to the call's stage budget.
void plan_prefill(const krk_state* s, const int32_t* lens, bool from_zero, PrefillPlan& p, Budget& bud) {
    const int B = s->B;
    int64_t off = 0;
    int g0 = 0;
    while (g0 < B) {
        int g1 = g0;
        int64_t rows = 0;
        while (g1 < B && (g1 == g0 || rows + lens[g1] <= PREFILL_GROUP_TOKENS)) rows += lens[g1++];
        PrefillPlan::Group g;
        g.g0 = g0; g.S = g1 - g0; g.rows = rows; g.off = off;
        for (int i = g0; i < g1; ++i) g.kmax = std::max<int>(g.kmax, (int)(start_pos(s, i, from_zero) + lens[i]));
        g.blk_rows = krk::attn_prefill_rows(g.kmax, HD);
        for (int i = g0; i < g1; ++i) g.nblk += (lens[i] + g.blk_rows - 1) / g.blk_rows;
        bud.add<int32_t>(g.S + 1); bud.add<int32_t>(g.S); bud.add<int32_t>(g.S); bud.add<int32_t>(g.S);
        bud.add<int32_t>(rows); bud.add<int2>(g.nblk);
        p.groups.push_back(g);
        p.total += rows;
        off += rows;
        g0 = g1;
    }
    bud.add<int32_t>(B);
}

// Writes the group tables into the stage (after stage.ensure of the budget).
void fill_prefill(krk_state* s, const int32_t* lens, bool from_zero, PrefillPlan& p) {
    HostStage& hs = s->stage;
    for (auto& g : p.groups) {
        g.cu = hs.take<int32_t>(g.S + 1); g.start = hs.take<int32_t>(g.S); g.last = hs.take<int32_t>(g.S);
        g.dst = hs.take<int32_t>(g.S); g.row_seq = hs.take<int32_t>(g.rows); g.blk = hs.take<int2>(g.nblk);
        g.cu[0] = 0;
        int nb = 0;
        for (int i = 0; i < g.S; ++i) {
            const int b = g.g0 + i;
            g.cu[i + 1] = g.cu[i] + lens[b];
            g.start[i] = (int32_t)start_pos(s, b, from_zero);
            g.last[i] = g.cu[i + 1] - 1;
            g.dst[i] = b;
            for (int r = g.cu[i]; r < g.cu[i + 1]; ++r) g.row_seq[r] = i;
            for (int r = 0; r < lens[b]; r += g.blk_rows) g.blk[nb++] = make_int2(i, r);
        }
    }
    p.pos_after = hs.take<int32_t>(s->B);
    for (int b = 0; b < s->B; ++b) p.pos_after[b] = (int32_t)(start_pos(s, b, from_zero) + lens[b]);
}

// Device address of a pointer into the stage's first `meta_bytes` (the part
// upload_call copied to the device).
template <typename T>
T* meta_dev(const krk_state* s, const T* host) {
    return reinterpret_cast<T*>(s->meta_arena.base + (reinterpret_cast<const char*>(host) - s->stage.base));
}

// Copies the stage's first meta_bytes and the packed prompt tokens to the
// device on the model stream (two asynchronous copies).  Grows the device
// buffers when needed (after the model's streams are idle).
void upload_call(krk_state* s, const uint32_t* tokens, int64_t ntok, size_t meta_bytes) {
    cudaStream_t st = s->m->stream;
    if (meta_bytes > s->meta_arena.cap || (size_t)ntok * 4 > s->prompt_cap) {
        sync_model_streams(s->m);
        if (meta_bytes > s->meta_arena.cap) s->meta_arena.reserve(std::max(meta_bytes, s->stage.cap));
        if ((size_t)ntok * 4 > s->prompt_cap) {
            s->prompt_arena.reserve((size_t)ntok * 4);
            s->prompt_cap = (size_t)ntok * 4;
        }
    }
    if (meta_bytes) kk(cudaMemcpyAsync(s->meta_arena.base, s->stage.base, meta_bytes, cudaMemcpyHostToDevice, st),
                       "h2d tables");
    if (ntok) kk(cudaMemcpyAsync(s->prompt_arena.base, tokens, (size_t)ntok * 4, cudaMemcpyHostToDevice, st),
                 "h2d tokens");
}

// Launches a planned, uploaded prefill; afterwards (in stream order) the decode
// buffers hold the logits of each sequence's last token.  mark: record prompt
// tokens in the repetition-penalty bitmaps.  No host synchronisation.
void launch_prefill(krk_state* s, const PrefillPlan& p, bool mark) {
    const krk_model* m = s->m;
    cudaStream_t st = m->stream;
    const auto& groups = p.groups;
    // decode_streams == 1 keeps the prefill on the model stream too
    const int ns = s->decode_streams == 1 ? 1 : std::min<int>(PREFILL_STREAMS, (int)groups.size());
    cudaStream_t streams[PREFILL_STREAMS] = {m->stream, m->stream2, m->stream3};
    for (int k = 0; k < ns; ++k) {
        int64_t rows = 0;
        int seqs = 0;
        for (size_t i = k; i < groups.size(); i += ns) {
            rows = std::max(rows, groups[i].rows);
            seqs = std::max(seqs, groups[i].S);
        }
        ensure_prefill_ws(s, k, rows, seqs);
    }
    if (ns > 1) {
        kk(cudaEventRecord(s->ev_fork, st), "fork");
        for (int k = 1; k < ns; ++k) kk(cudaStreamWaitEvent(streams[k], s->ev_fork, 0), "fork");
    }
    const uint32_t* tok_d = reinterpret_cast<const uint32_t*>(s->prompt_arena.base);
    for (size_t i = 0; i < groups.size(); ++i) {
        const PrefillPlan::Group& g = groups[i];
        const int k = (int)(i % ns);
        cudaStream_t gs = streams[k];
        GroupDev gd{tok_d + g.off, meta_dev(s, g.cu), meta_dev(s, g.start), meta_dev(s, g.last), meta_dev(s, g.dst),
                    meta_dev(s, g.row_seq), meta_dev(s, g.blk)};
        prefill_group(s, g.g0, g.S, g.rows, g.nblk, g.blk_rows, g.kmax, s->pre[k], gd, gs);
        if (mark)
            timed_on(s, gs, KRK_PROF_OTHER, 0, [&] {
                kk(krk::mark_seen(gd.tok, gd.row_seq, (int)g.rows, s->seen_d + (size_t)g.g0 * SEEN_WORDS, SEEN_WORDS,
                                  gs),
                   "mark seen");
            });
    }
    cudaEvent_t joins[PREFILL_STREAMS] = {nullptr, s->ev_join, s->ev_join3};
    for (int k = 1; k < ns; ++k) {
        kk(cudaEventRecord(joins[k], streams[k]), "join");
        kk(cudaStreamWaitEvent(st, joins[k], 0), "join");
    }
    lm_head(s);
    for (int b = 0; b < s->B; ++b) s->pos_h[b] = p.pos_after[b];
    kk(cudaMemcpyAsync(s->pos_d, meta_dev(s, p.pos_after), (size_t)s->B * 4, cudaMemcpyDeviceToDevice, st), "pos");
}

int copy_logits(krk_state* s, float* logits_out) {
    if (!logits_out) return KRK_OK;
    kk(cudaMemcpy2DAsync(logits_out, VOC * 4, s->logits, VOC * 4, VOC * 4, s->B, cudaMemcpyDeviceToHost,
                         s->m->stream),
       "d2h logits");
    kk(cudaStreamSynchronize(s->m->stream), "d2h logits");
    return KRK_OK;
}

template <typename F>
int guarded(F&& f) {  // runs f, turning exceptions into a status + message
    try {
        g_err.clear();
        return f();
    } catch (const KrkError& e) {
        return fail(e.status, e.msg);
    } catch (const std::bad_alloc&) {
        return fail(KRK_CHECK_FAILED, "host out of memory");
    } catch (const std::exception& e) {
        return fail(KRK_CHECK_FAILED, e.what());
    }
}

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return KRK_OK;
    return fail(e == cudaErrorInvalidValue ? KRK_INVALID : KRK_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// state.reset() for every sequence (mask null) or the masked ones
// (src/model.rs:220-229).  Stream-ordered; sync: wait for it on the host.
void reset_state(krk_state* s, const uint8_t* mask, bool sync) {
    cudaStream_t st = s->m->stream;
    if (!mask) {  // every sequence: one memset per array
        for (int l = 0; l < NL; ++l) {
            if (!is_mamba(l)) continue;
            kk(cudaMemsetAsync(s->conv[l], 0, (size_t)s->B * DXBC * 4 * 4, st), "reset conv");
            kk(cudaMemsetAsync(s->ssm[l], 0, (size_t)s->B * MH * MP * DS * 4, st), "reset ssm");
        }
        kk(cudaMemsetAsync(s->seen_d, 0, (size_t)s->B * SEEN_WORDS * 4, st), "reset seen");
        kk(cudaMemsetAsync(s->pos_d, 0, (size_t)s->B * 4, st), "reset pos");
        std::fill(s->pos_h.begin(), s->pos_h.end(), 0);
    } else {
        for (int b = 0; b < s->B; ++b) {
            if (!mask[b]) continue;
            s->pos_h[b] = 0;
            for (int l = 0; l < NL; ++l) {
                if (!is_mamba(l)) continue;  // attention reset only rewinds the length
                kk(cudaMemsetAsync(s->conv[l] + (size_t)b * DXBC * 4, 0, (size_t)DXBC * 4 * 4, st), "reset conv");
                kk(cudaMemsetAsync(s->ssm[l] + (size_t)b * MH * MP * DS, 0, (size_t)MH * MP * DS * 4, st),
                   "reset ssm");
            }
            kk(cudaMemsetAsync(s->seen_d + (size_t)b * SEEN_WORDS, 0, SEEN_WORDS * 4, st), "reset seen");
        }
        s->stage.ensure(round_up((int64_t)s->B * 4, 256));
        int32_t* p32 = s->stage.take<int32_t>(s->B);
        for (int b = 0; b < s->B; ++b) p32[b] = (int32_t)s->pos_h[b];
        kk(cudaMemcpyAsync(s->pos_d, p32, s->B * 4, cudaMemcpyHostToDevice, st), "h2d pos");
    }
    if (sync || mask) kk(cudaStreamSynchronize(st), "reset");  // a masked reset's table is in the stage
}

}  // namespace

namespace krk {
// Sets the calling thread's krk_last_error() message (for other translation units).
int report_error(int status, const std::string& msg) { return fail(status, msg); }

// The device check words of a checked build, one reader per translation unit
// with kernels (registered while the library loads).
static std::vector<unsigned (*)(bool)>& check_readers() {
    static std::vector<unsigned (*)(bool)> v;
    return v;
}
void register_check_word(unsigned (*read)(bool clear)) { check_readers().push_back(read); }
static unsigned read_checks(bool clear) {
    unsigned bits = 0;
    for (auto f : check_readers()) bits |= f(clear);
    return bits;
}
}  // namespace krk

namespace {
// In a checked build, a call that launched kernels ends by reading (and
// clearing) the device check words of its device: a set bit means a kernel
// found a precondition on device data violated and skipped the access.
int checked_result(int rc) {
#ifdef KRIKIL_CHECKED
    const unsigned bits = krk::read_checks(true);
    if (bits) {
        std::string what;
        const char* names[] = {"token id >= vocab", "position outside the cache or the key bound",
                               "prefill table entry out of range", "gather column out of range"};
        for (int i = 0; i < 4; ++i)
            if (bits & (1u << i)) what += std::string(what.empty() ? "" : "; ") + names[i];
        return fail(KRK_CHECK_FAILED, "device check failed: " + what + "; outputs of this call are not valid");
    }
#endif
    return rc;
}
}  // namespace

// =================================================================== C ABI
extern "C" {

const char* krk_last_error(void) { return g_err.c_str(); }

const char* krk_status_string(int status) {
    switch (status) {
        case KRK_OK: return "ok";
        case KRK_BAD_TOKEN: return "token id exceeds vocab size";
        case KRK_CONTEXT_OVERFLOW: return "context limit exceeded";
        case KRK_EMPTY: return "empty sequence";
        case KRK_IO: return "i/o or format error";
        case KRK_NOT_FOUND: return "tensor not found";
        case KRK_INVALID: return "invalid argument";
        case KRK_CUDA: return "cuda error";
        case KRK_CHECK_FAILED: return "internal check failed";
        default: return "unknown status";
    }
}

int krk_abi_version(void) { return KRK_ABI_VERSION; }

int krk_model_load(const char* path, int device, krk_model** out) {
    return guarded([&]() -> int {
        if (!path || !out) return fail(KRK_INVALID, "null path or output handle");
        *out = nullptr;
        std::unique_ptr<krk_model> m(new krk_model());
        HostWeights hw;
        read_weights(m.get(), path, hw);  // file and format errors come first, as in the reference
        int ndev = 0;
        cudaError_t e = cudaGetDeviceCount(&ndev);
        if (e != cudaSuccess || ndev == 0)
            return fail(KRK_CUDA, std::string("no CUDA device: ") + cudaGetErrorString(e));
        if (device < 0 || device >= ndev) return fail(KRK_INVALID, "device index out of range");
        DeviceGuard g(device);
        m->device = device;
        ck(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "stream create");
        try {
            ck(cudaStreamCreateWithFlags(&m->stream2, cudaStreamNonBlocking), "stream create");
            ck(cudaStreamCreateWithFlags(&m->stream3, cudaStreamNonBlocking), "stream create");
            ck(cudaStreamCreateWithFlags(&m->stream4, cudaStreamNonBlocking), "stream create");
            upload_weights(m.get(), hw);
        } catch (...) {
            m->arena.release();
            if (m->stream2) cudaStreamDestroy(m->stream2);
            if (m->stream3) cudaStreamDestroy(m->stream3);
            if (m->stream4) cudaStreamDestroy(m->stream4);
            cudaStreamDestroy(m->stream);
            throw;
        }
        *out = m.release();
        return KRK_OK;
    });
}

int krk_model_free(krk_model* m) {
    if (!m) return KRK_OK;
    return guarded([&]() -> int {
        DeviceGuard g(m->device);
        cudaStreamSynchronize(m->stream);
        cudaStreamSynchronize(m->stream2);
        cudaStreamSynchronize(m->stream3);
        cudaStreamSynchronize(m->stream4);
        m->arena.release();
        cudaStreamDestroy(m->stream2);
        cudaStreamDestroy(m->stream3);
        cudaStreamDestroy(m->stream4);
        cudaStreamDestroy(m->stream);
        delete m;
        return KRK_OK;
    });
}

int krk_model_device(const krk_model* m, int* device) {
    if (!m || !device) return fail(KRK_INVALID, "null argument");
    *device = m->device;
    return KRK_OK;
}

int krk_model_stream(const krk_model* m, void** stream) {
    if (!m || !stream) return fail(KRK_INVALID, "null argument");
    *stream = (void*)m->stream;
    return KRK_OK;
}

int krk_state_create(const krk_model* m, int batch, int max_ctx, krk_state** out) {
    return guarded([&]() -> int {
        if (!m || !out) return fail(KRK_INVALID, "null model or output handle");
        if (batch <= 0 || max_ctx <= 0) return fail(KRK_INVALID, "batch and max_ctx must be positive");
        // A prefill of one full context is one projection over round_up(max_ctx, 64)
        // rows, whose operands the GEMM indexes with 32-bit offsets.
        if (round_up(max_ctx, 64) * INTER >= (int64_t(1) << 31) || round_up(batch, 64) * INTER >= (int64_t(1) << 31))
            return fail(KRK_INVALID, "max_ctx and batch must be at most " + std::to_string(MAX_ROWS));
        *out = nullptr;
        DeviceGuard g(m->device);
        std::unique_ptr<krk_state> s(new krk_state());
        create_state(s.get(), m, batch, max_ctx);
        *out = s.release();
        return KRK_OK;
    });
}

int krk_state_free(krk_state* s) {
    if (!s) return KRK_OK;
    return guarded([&]() -> int {
        DeviceGuard g(s->m->device);
        cudaStreamSynchronize(s->m->stream);
        cudaStreamSynchronize(s->m->stream2);
        cudaStreamSynchronize(s->m->stream3);
        cudaStreamSynchronize(s->m->stream4);
        if (s->ev_fork) cudaEventDestroy(s->ev_fork);
        if (s->ev_join) cudaEventDestroy(s->ev_join);
        if (s->ev_join3) cudaEventDestroy(s->ev_join3);
        if (s->ev_join4) cudaEventDestroy(s->ev_join4);
        for (cudaGraphExec_t g : s->step_graphs)
            if (g) cudaGraphExecDestroy(g);
        for (auto& w : s->pre) w.arena.release();
        s->hist_arena.release();
        s->arena.release();
        delete s;
        return KRK_OK;
    });
}

int krk_state_reset(krk_state* s, const uint8_t* mask) {
    return guarded([&]() -> int {
        if (!s) return fail(KRK_INVALID, "null state");
        DeviceGuard g(s->m->device);
        reset_state(s, mask, true);
        return KRK_OK;
    });
}

int krk_state_batch(const krk_state* s, int* batch) {
    if (!s || !batch) return fail(KRK_INVALID, "null argument");
    *batch = s->B;
    return KRK_OK;
}

int krk_state_context_limit(const krk_state* s, int* max_ctx) {
    if (!s || !max_ctx) return fail(KRK_INVALID, "null argument");
    *max_ctx = s->ctx;
    return KRK_OK;
}

int krk_state_positions(const krk_state* s, int64_t* pos_out) {
    if (!s || !pos_out) return fail(KRK_INVALID, "null argument");
    for (int b = 0; b < s->B; ++b) pos_out[b] = s->pos_h[b];
    return KRK_OK;
}

int krk_prefill(const krk_model* m, krk_state* s, const uint32_t* tokens, const int32_t* lens, float* logits_out) {
    return guarded([&]() -> int {
        if (!m || !s || s->m != m) return fail(KRK_INVALID, "null handle or state of another model");
        int64_t total = 0;
        int rc = check_prefill(s, tokens, lens, false, &total);
        if (rc) return rc;
        DeviceGuard g(m->device);
        PrefillPlan plan;
        Budget bud;
        plan_prefill(s, lens, false, plan, bud);
        s->stage.ensure(bud.bytes);
        fill_prefill(s, lens, false, plan);
        upload_call(s, tokens, total, s->stage.used);
        total_begin(s);
        launch_prefill(s, plan, false);
        total_end(s);
        rc = copy_logits(s, logits_out);
        kk(cudaStreamSynchronize(m->stream), "prefill");
        prof_collect_if_large(s);
        return checked_result(rc);
    });
}

// A decode attention kernel gave up waiting for its K/V copies (bounded
// waits; the outputs of that step are not valid).  Clears the flag.
static int device_wait_error(krk_state* s) {
    kk(cudaMemsetAsync(s->err_d, 0, 4, s->m->stream), "status reset");
    kk(cudaStreamSynchronize(s->m->stream), "status reset");
    return fail(KRK_CUDA, "decode attention: a K/V copy wait timed out; outputs of this call are not valid");
}

int krk_step(const krk_model* m, krk_state* s, const uint32_t* tokens, float* logits_out) {
    return guarded([&]() -> int {
        if (!m || !s || s->m != m) return fail(KRK_INVALID, "null handle or state of another model");
        if (!tokens) return fail(KRK_INVALID, "null tokens");
        for (int b = 0; b < s->B; ++b)
            if (tokens[b] >= (uint32_t)VOC)
                return fail(KRK_BAD_TOKEN,
                            "Token ID " + std::to_string(tokens[b]) + " exceeds vocab size " + std::to_string(VOC));
        for (int b = 0; b < s->B; ++b)
            if (s->pos_h[b] >= s->ctx)
                return fail(KRK_CONTEXT_OVERFLOW, "Context limit " + std::to_string(s->ctx) + " reached");
        DeviceGuard g(m->device);
        cudaStream_t st = m->stream;
        kk(cudaMemcpyAsync(s->tok_d, tokens, s->B * 4, cudaMemcpyHostToDevice, st), "h2d tokens");
        total_begin(s);
        decode_forward(s, nullptr, (int)*std::max_element(s->pos_h.begin(), s->pos_h.end()) + 1);
        timed(s, KRK_PROF_OTHER, [&] { kk(krk::advance_pos(s->pos_d, nullptr, s->B, st), "advance"); });
        for (int b = 0; b < s->B; ++b) s->pos_h[b] += 1;
        total_end(s);
        int rc = KRK_OK;
        if (logits_out) rc = copy_logits(s, logits_out);
        int32_t err_h = 0;
        kk(cudaMemcpyAsync(&err_h, s->err_d, 4, cudaMemcpyDeviceToHost, st), "d2h status");
        kk(cudaStreamSynchronize(st), "step");
        prof_collect_if_large(s);
        if (err_h) return device_wait_error(s);
        return checked_result(rc);
    });
}

// Sampler settings of a generation call (src/sampler.rs:5-13); temperature
// <= 1e-6 is the greedy branch and needs no seeds.
struct SampleCfg {
    float temperature = 0.0f, top_p = 1.0f;
    int top_k = 0;
    const uint64_t* seeds = nullptr;  // [B]
};

static int generate_impl(const krk_model* m, krk_state* s, const uint32_t* prompts, const int32_t* lens,
                         int max_new_tokens, float repetition_penalty, const SampleCfg& cfg, int stop_at_eos,
                         uint32_t* tokens_out, int32_t* n_out);

int krk_generate_greedy(const krk_model* m, krk_state* s, const uint32_t* prompts, const int32_t* lens,
                        int max_new_tokens, float repetition_penalty, int stop_at_eos, uint32_t* tokens_out,
                        int32_t* n_out) {
    return generate_impl(m, s, prompts, lens, max_new_tokens, repetition_penalty, SampleCfg{}, stop_at_eos,
                         tokens_out, n_out);
}

int krk_generate_sample(const krk_model* m, krk_state* s, const uint32_t* prompts, const int32_t* lens,
                        int max_new_tokens, float temperature, float top_p, int top_k, float repetition_penalty,
                        const uint64_t* seeds, int stop_at_eos, uint32_t* tokens_out, int32_t* n_out) {
    SampleCfg cfg;
    cfg.temperature = temperature;
    cfg.top_p = top_p;
    cfg.top_k = top_k;
    cfg.seeds = seeds;
    return generate_impl(m, s, prompts, lens, max_new_tokens, repetition_penalty, cfg, stop_at_eos, tokens_out,
                         n_out);
}

static int generate_impl(const krk_model* m, krk_state* s, const uint32_t* prompts, const int32_t* lens,
                         int max_new_tokens, float repetition_penalty, const SampleCfg& cfg, int stop_at_eos,
                         uint32_t* tokens_out, int32_t* n_out) {
    return guarded([&]() -> int {
        if (!m || !s || s->m != m) return fail(KRK_INVALID, "null handle or state of another model");
        if (max_new_tokens <= 0 || !tokens_out || !n_out) return fail(KRK_INVALID, "bad output arguments");
        const bool stochastic = cfg.temperature > 1e-6f;
        if (stochastic && !cfg.seeds) return fail(KRK_INVALID, "sampling with temperature > 0 needs seeds");
        if (stochastic && !(cfg.temperature == cfg.temperature)) return fail(KRK_INVALID, "bad temperature");
        DeviceGuard g(m->device);
        cudaStream_t st = m->stream;
        const int B = s->B;
        // state.reset() (src/generate.rs:65), then forward_prefill's checks
        // against the reset positions; a failing prefill leaves the state reset.
        int64_t total = 0;
        int rc = check_prefill(s, prompts, lens, true, &total);
        if (rc) {
            reset_state(s, nullptr, true);
            return rc;
        }
        // src/generate.rs:86-114 per sequence: a pick is pushed unless it is EOS;
        // after a push the loop stops if current_pos >= context_limit, else it
        // runs forward_step -- also after the max_new_tokens-th push.  So a
        // sequence pushes at most tlimit = min(max_new, ctx - len + 1) tokens
        // and runs at most slimit = min(max_new, ctx - len) decode steps.
        int max_picks = 0, max_steps = 0;
        for (int b = 0; b < B; ++b) {
            max_picks = std::max<int>(max_picks, (int)std::min<int64_t>(max_new_tokens, (int64_t)s->ctx - lens[b] + 1));
            max_steps = std::max<int>(max_steps, (int)std::min<int64_t>(max_new_tokens, (int64_t)s->ctx - lens[b]));
        }
        if ((int64_t)max_picks * B > s->hist_cap) {
            s->hist_arena.reserve((size_t)max_picks * B * 4 + 256);
            s->hist_d = s->hist_arena.take<uint32_t>((size_t)max_picks * B);
            s->hist_cap = (int64_t)max_picks * B;
        }
        // Host tables of the call in the pinned stage: the prefill groups, the
        // limits and seeds (copied to the device together), then room for the
        // results read back at the end.
        PrefillPlan plan;
        Budget bud;
        plan_prefill(s, lens, true, plan, bud);
        bud.add<int32_t>(B); bud.add<int32_t>(B);
        if (stochastic) bud.add<uint32_t>((size_t)B * 10);
        bud.add<uint32_t>((size_t)max_picks * B); bud.add<int32_t>(B); bud.add<int32_t>(1);
        s->stage.ensure(bud.bytes);
        fill_prefill(s, lens, true, plan);
        int32_t* tlimit = s->stage.take<int32_t>(B);
        int32_t* slimit = s->stage.take<int32_t>(B);
        for (int b = 0; b < B; ++b) {
            tlimit[b] = (int32_t)std::min<int64_t>(max_new_tokens, (int64_t)s->ctx - lens[b] + 1);
            slimit[b] = (int32_t)std::min<int64_t>(max_new_tokens, (int64_t)s->ctx - lens[b]);
        }
        uint32_t* rng = nullptr;
        if (stochastic) {  // Sampler::new with config.seed (src/sampler.rs:34-40), one per sequence
            rng = s->stage.take<uint32_t>((size_t)B * 10);
            for (int b = 0; b < B; ++b) krk::rng_seed_state(cfg.seeds[b], rng + (size_t)b * 10);
        }
        const size_t meta_bytes = s->stage.used;
        uint32_t* hist = s->stage.take<uint32_t>((size_t)max_picks * B);
        int32_t* pos = s->stage.take<int32_t>(B);
        int32_t* err_h = s->stage.take<int32_t>(1);
        upload_call(s, prompts, total, meta_bytes);
        // device time from here on: the inputs are on the device
        total_begin(s);
        reset_state(s, nullptr, false);
        launch_prefill(s, plan, true);
        kk(cudaMemsetAsync(s->active_d, 1, B, st), "active");
        kk(cudaMemsetAsync(s->step_d, 0, 4, st), "step");
        kk(cudaMemsetAsync(s->hist_d, 0xff, (size_t)max_picks * B * 4, st), "hist");
        if (stochastic)
            kk(cudaMemcpyAsync(s->rng_d, meta_dev(s, rng), (size_t)B * 40, cudaMemcpyDeviceToDevice, st), "rng");
        krk::GreedyArgs ga{};
        ga.temperature = cfg.temperature; ga.top_p = cfg.top_p; ga.top_k = cfg.top_k; ga.rng = s->rng_d;
        ga.logits = s->logits; ga.ld = VOC; ga.vocab = VOC; ga.B = B;
        ga.seen = s->seen_d; ga.penalty = repetition_penalty;
        ga.tok = s->tok_d; ga.active = s->active_d; ga.hist = s->hist_d; ga.step = s->step_d;
        ga.tlimit = meta_dev(s, tlimit); ga.slimit = meta_dev(s, slimit);
        ga.stop_eos = stop_at_eos; ga.eos = KRK_EOS_TOKEN;
        ga.pos = nullptr;
        // first pick from the prefill logits (src/generate.rs:81-82)
        timed(s, KRK_PROF_OTHER, [&] { kk(krk::sample(ga, st), "sample"); });
        ga.pos = s->pos_d;
        // step i runs every active sequence at position pos_h[b] + i at most
        const int64_t pos0 = *std::max_element(s->pos_h.begin(), s->pos_h.end());
        for (int i = 0; i < max_steps; ++i) {
            decode_step(s, (int)(pos0 + i + 1));
            timed(s, KRK_PROF_OTHER, [&] { kk(krk::sample(ga, st), "sample"); });
        }
        total_end(s);
        kk(cudaMemcpyAsync(hist, s->hist_d, (size_t)max_picks * B * 4, cudaMemcpyDeviceToHost, st), "d2h tokens");
        kk(cudaMemcpyAsync(pos, s->pos_d, B * 4, cudaMemcpyDeviceToHost, st), "d2h pos");
        kk(cudaMemcpyAsync(err_h, s->err_d, 4, cudaMemcpyDeviceToHost, st), "d2h status");
        kk(cudaStreamSynchronize(st), "generate");  // the call's one host synchronisation
        prof_collect_if_large(s);
        if (*err_h) return device_wait_error(s);
        for (int b = 0; b < B; ++b) {
            int n = 0;
            for (int i = 0; i < tlimit[b]; ++i) {
                uint32_t t = hist[(size_t)i * B + b];
                if (t == 0xffffffffu || (stop_at_eos && t == (uint32_t)KRK_EOS_TOKEN)) break;
                tokens_out[(size_t)b * max_new_tokens + n++] = t;
            }
            n_out[b] = n;
            s->pos_h[b] = pos[b];
        }
        return checked_result(KRK_OK);
    });
}

int krk_state_export(const krk_state* s, int seq, int layer, int what, float* out, int64_t n) {
    return guarded([&]() -> int {
        if (!s || !out || seq < 0 || seq >= s->B || layer < 0 || layer >= NL)
            return fail(KRK_INVALID, "bad export arguments");
        const float* src = nullptr;
        int64_t cnt = 0;
        if (is_mamba(layer) && what == 0) {
            src = s->conv[layer] + (size_t)seq * DXBC * 4;
            cnt = (int64_t)DXBC * 4;
        } else if (is_mamba(layer) && what == 1) {
            src = s->ssm[layer] + (size_t)seq * MH * MP * DS;
            cnt = (int64_t)MH * MP * DS;
        } else if (!is_mamba(layer) && what == 2) {
            src = s->kc[layer] + (size_t)seq * s->ctx * HID;
            cnt = (int64_t)s->ctx * HID;
        } else if (!is_mamba(layer) && what == 3) {
            src = s->vc[layer] + (size_t)seq * s->ctx * HID;
            cnt = (int64_t)s->ctx * HID;
        } else {
            return fail(KRK_INVALID, "layer has no such state");
        }
        if (n < cnt) return fail(KRK_INVALID, "output buffer too small");
        DeviceGuard g(s->m->device);
        kk(cudaMemcpyAsync(out, src, cnt * 4, cudaMemcpyDeviceToHost, s->m->stream), "d2h state");
        kk(cudaStreamSynchronize(s->m->stream), "export");
        return KRK_OK;
    });
}

// Drops the state's step graphs (they hold the old part layout).
static void drop_step_graphs(krk_state* s) {
    if (s->step_graphs.empty()) return;
    DeviceGuard g(s->m->device);
    sync_model_streams(s->m);
    for (cudaGraphExec_t& ex : s->step_graphs)
        if (ex) cudaGraphExecDestroy(ex);
    s->step_graphs.clear();
    s->step_graph_kernels.clear();
}

int krk_state_set_decode_streams(krk_state* s, int n) {
    if (!s || n < 1 || n > 4) return fail(KRK_INVALID, "decode streams must be 1 to 4");
    return guarded([&]() -> int {
        if (n != s->decode_streams) drop_step_graphs(s);
        s->decode_streams = n;
        return KRK_OK;
    });
}

int krk_state_set_step_graphs(krk_state* s, int enable) {
    if (!s) return fail(KRK_INVALID, "null state");
    return guarded([&]() -> int {
        if (!enable) drop_step_graphs(s);
        s->step_graphs_on = enable != 0;
        return KRK_OK;
    });
}

int krk_state_profile(krk_state* s, int enable) {
    return guarded([&]() -> int {
        if (!s) return fail(KRK_INVALID, "null state");
        DeviceGuard g(s->m->device);
        kk(cudaStreamSynchronize(s->m->stream), "profile");
        s->prof.clear_events();
        s->prof.on = enable != 0;
        s->prof.per_kernel = enable == 1;
        for (int i = 0; i < KRK_PROF_CLASSES; ++i) {
            s->prof.ms[i] = 0.0;
            s->prof.n[i] = 0;
            s->prof.units[i] = 0;
        }
        return KRK_OK;
    });
}

// Folds the event pairs still pending (the state's calls have all returned, so
// their streams are idle once synchronised).
static void prof_settle(const krk_state* cs) {
    krk_state* s = const_cast<krk_state*>(cs);  // the totals are a cache of the recorded events
    if (s->prof.pending.empty()) return;
    DeviceGuard g(s->m->device);
    kk(cudaStreamSynchronize(s->m->stream), "profile");
    kk(cudaStreamSynchronize(s->m->stream2), "profile");
    kk(cudaStreamSynchronize(s->m->stream3), "profile");
    kk(cudaStreamSynchronize(s->m->stream4), "profile");
    prof_collect(s);
}

int krk_state_profile_read(const krk_state* s, int cls, double* total_ms, int64_t* launches) {
    if (!s || cls < 0 || cls >= KRK_PROF_CLASSES || !total_ms || !launches)
        return fail(KRK_INVALID, "bad profile arguments");
    return guarded([&]() -> int {
        prof_settle(s);
        *total_ms = s->prof.ms[cls];
        *launches = s->prof.n[cls];
        return KRK_OK;
    });
}

int krk_state_profile_units(const krk_state* s, int cls, int64_t* units) {
    if (!s || cls < 0 || cls >= KRK_PROF_CLASSES || !units) return fail(KRK_INVALID, "bad profile arguments");
    return guarded([&]() -> int {
        prof_settle(s);
        *units = s->prof.units[cls];
        return KRK_OK;
    });
}

int krk_checked_build(void) {
#ifdef KRIKIL_CHECKED
    return 1;
#else
    return 0;
#endif
}

int krk_check_status(uint32_t* bits, int clear) {
    if (!bits) return fail(KRK_INVALID, "null argument");
    *bits = krk::read_checks(clear != 0);
    return KRK_OK;
}

int krk_launch_count(uint64_t* count) {
    if (!count) return fail(KRK_INVALID, "null argument");
    *count = krk::launch_count();
    return KRK_OK;
}

// ------------------------------------------------------ per-kernel entry points
int krk_k_rmsnorm_rows(const float* x, const float* w, float eps, int64_t rows, int dim, float* y, void* stream) {
    return cuda_status(krk::rmsnorm_rows(x, w, eps, rows, dim, y, (cudaStream_t)stream), "rmsnorm_rows");
}

int krk_k_rmsnorm_fm(const float* x, int ldx, const float* w, float eps, int K, int M, float* out, int ldo,
                     void* stream) {
    return cuda_status(krk::rmsnorm_fm(x, ldx, w, eps, K, M, out, ldo, (cudaStream_t)stream), "rmsnorm_fm");
}

int krk_k_gated_rmsnorm_residual(const float* x, const float* z, const float* res, const float* w, float eps,
                                 int64_t rows, int dim, float* y, void* stream) {
    return cuda_status(krk::gated_rmsnorm_residual(x, z, res, w, eps, rows, dim, y, (cudaStream_t)stream),
                       "gated_rmsnorm_residual");
}

int krk_k_gemm(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
               int epilogue, int out_fm, void* stream) {
    if (epilogue < 0 || epilogue > 2) return fail(KRK_INVALID, "epilogue must be 0, 1 or 2");
    return cuda_status(krk::gemm(At, lda, Wt, ldw, C, ldc, M, N, K, epilogue, out_fm != 0, (cudaStream_t)stream),
                       "gemm");
}

int krk_k_gemm_tiled(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N, int K,
                     int epilogue, int out_fm, int tile_rows, void* stream) {
    if (epilogue < 0 || epilogue > 2) return fail(KRK_INVALID, "epilogue must be 0, 1 or 2");
    return cuda_status(
        krk::gemm_tiled(At, lda, Wt, ldw, C, ldc, M, N, K, epilogue, out_fm != 0, tile_rows, (cudaStream_t)stream),
        "gemm");
}

int krk_k_gemm_tile_rows(int M, int N) { return M > 0 && N > 0 ? krk::gemm_tile_rows(M, N) : 0; }

int krk_k_embed(const uint32_t* tok, const float* wte, int vocab, int K, int M, float* out, int ldo, void* stream) {
    return cuda_status(krk::embed_fm(tok, wte, vocab, K, M, out, ldo, (cudaStream_t)stream), "embed");
}

int krk_k_pointwise(int op, const float* x, float* y, int64_t n, void* stream) {
    return cuda_status(krk::pointwise(op, x, y, n, (cudaStream_t)stream), "pointwise");
}

int krk_k_conv_ssd_step(const float* x, const float* bm, const float* cm, const float* dt, float* conv_state,
                        const float* conv_w, const float* conv_b, float* ssm, const float* dt_bias,
                        const float* a_neg, const float* dsk, float* y, int B, int H, int P, int N, void* stream) {
    if (P != 64 || N != 128) return fail(KRK_INVALID, "conv_ssd_step supports head dim 64 and d_state 128");
    krk::SsdStepArgs a{};
    a.x = x; a.x_sb = (int64_t)H * P;
    a.bm = bm; a.cm = cm; a.bc_sb = N;
    a.dt = dt; a.dt_sb = H;
    a.conv_state = conv_state; a.conv_w = conv_w; a.conv_b = conv_b;
    a.ssm = ssm; a.dt_bias = dt_bias; a.a_neg = a_neg; a.dsk = dsk;
    a.y = y; a.y_sb = (int64_t)H * P; a.y_sc = 1;
    a.B = B; a.H = H; a.P = P; a.N = N;
    return cuda_status(krk::ssd_step(a, true, (cudaStream_t)stream), "conv_ssd_step");
}

int krk_k_conv_ssd_scan(const float* x, const float* bm, const float* cm, const float* dt, float* conv_state,
                        const float* conv_w, const float* conv_b, float* ssm, const float* dt_bias,
                        const float* a_neg, const float* dsk, float* y, int B, int T, int H, int P, int N,
                        void* stream) {
    if (P != 64 || N != 128) return fail(KRK_INVALID, "conv_ssd_scan supports head dim 64 and d_state 128");
    if (T <= 0) return fail(KRK_INVALID, "T must be positive");
    krk::SsdScanArgs a{};
    a.x = x; a.x_rs = (int64_t)H * P;
    a.bm = bm; a.cm = cm; a.bc_rs = N;
    a.dt = dt; a.dt_rs = H;
    a.conv_state = conv_state; a.conv_w = conv_w; a.conv_b = conv_b;
    a.ssm = ssm; a.dt_bias = dt_bias; a.a_neg = a_neg; a.dsk = dsk;
    a.y = y; a.y_rs = (int64_t)H * P; a.y_cs = 1;
    a.cu_seqlens = nullptr; a.uniform_len = T;
    a.S = B; a.H = H; a.P = P; a.N = N;
    return cuda_status(krk::ssd_scan(a, true, (cudaStream_t)stream), "conv_ssd_scan");
}

size_t krk_attn_work_floats(int B, int H, int dh, int ctx, int split) {
    if (split <= 0) return 0;  // 0: the cluster kernel, which needs no scratch
    if (B <= 0 || H <= 0 || dh <= 0 || ctx <= 0) return 0;
    return krk::attn_decode_work_floats(B, H, dh, ctx, split);
}

int krk_k_rope_kv_attn_decode(const float* q, const float* k, const float* v, float* kc, float* vc,
                              const int32_t* pos, float* out, float* work, int B, int H, int dh, int ctx,
                              int split, float theta, void* stream) {
    krk::AttnDecodeArgs a{};
    a.q = q; a.k = k; a.v = v; a.in_sb = (int64_t)H * dh; a.in_sh = dh;
    a.kc = kc; a.vc = vc; a.c_sb = (int64_t)H * ctx * dh; a.c_sh = (int64_t)ctx * dh; a.c_st = dh;
    a.pos = pos; a.active = nullptr;
    a.out = out; a.o_sb = (int64_t)H * dh; a.o_sh = dh; a.o_sd = 1;
    a.work = work;
    if (split < 0) return fail(KRK_INVALID, "split must be 0 (cluster kernel) or a positive multiple of 64");
    a.B = B; a.H = H; a.dh = dh; a.ctx = ctx; a.split = split; a.theta = theta;
    a.rope = nullptr;
    return cuda_status(krk::attn_decode(a, (cudaStream_t)stream), "rope_kv_attn_decode");
}

int krk_k_gemm_sgemm_order(const float* At, int lda, const float* Wt, int ldw, float* C, int ldc, int M, int N,
                           int K, void* stream) {
    return cuda_status(krk::gemm_sgemm_order(At, lda, Wt, ldw, C, ldc, M, N, K, (cudaStream_t)stream),
                       "gemm_sgemm_order");
}

int krk_k_attn_prefill_rows(int kmax, int dh) {
    if (kmax <= 0 || (dh != 64 && dh != 76)) return 0;
    return krk::attn_prefill_rows(kmax, dh);
}

int krk_k_rope_kv_attn_prefill(float* qkv, int64_t q_rs, float* kc, float* vc, int64_t c_sb, int64_t c_sh,
                               int64_t c_st, const int32_t* cu_seqlens, const int32_t* start, int S, int total_rows,
                               int H, int dh, float theta, const int32_t* blocks, int nblocks, int rows_per_block,
                               int kmax, float* out, int64_t o_rs, int64_t o_cs, void* stream) {
    if (S <= 0 || total_rows <= 0 || H <= 0 || nblocks <= 0)
        return fail(KRK_INVALID, "prefill attention needs S, total_rows, H and nblocks > 0");
    if (q_rs < (int64_t)3 * H * dh) return fail(KRK_INVALID, "q_rs shorter than a q | k | v row");
    if (kmax <= 0 || rows_per_block != krk_k_attn_prefill_rows(kmax, dh))
        return fail(KRK_INVALID, "rows_per_block must be krk_k_attn_prefill_rows(kmax, dh)");
    if (krk::attn_prefill_check(qkv, q_rs, kc, vc, c_sb, c_sh, c_st, nblocks, rows_per_block, H, dh, kmax) !=
        cudaSuccess)
        return fail(KRK_INVALID, "prefill attention: dh must be 64 or 76, strides multiples of 4 floats, "
                                 "qkv/kc/vc 16-byte aligned, and the scores of kmax keys must fit in shared memory");
    const cudaStream_t s = (cudaStream_t)stream;
    int st = cuda_status(krk::rope_kv_prefill(qkv, q_rs, kc, vc, c_sb, c_sh, c_st, cu_seqlens, start, S, H, dh,
                                              total_rows, theta, nullptr, s),
                         "rope_kv_prefill");
    if (st != KRK_OK) return st;
    return cuda_status(krk::attn_prefill(qkv, q_rs, kc, vc, c_sb, c_sh, c_st, cu_seqlens, start,
                                         reinterpret_cast<const int2*>(blocks), nblocks, rows_per_block, H, dh, kmax,
                                         out, o_rs, o_cs, s),
                       "attn_prefill");
}

int krk_k_wait_probe(const float* src16, int polls, int copy, int32_t* status, void* stream) {
    return cuda_status(krk::wait_probe(src16, polls, copy != 0, status, (cudaStream_t)stream), "wait_probe");
}

int krk_k_greedy(const float* logits, int64_t ld, int vocab, int B, uint32_t* seen, float penalty, uint32_t* tok,
                 void* stream) {
    krk::GreedyArgs a{};
    a.logits = logits; a.ld = ld; a.vocab = vocab; a.B = B; a.seen = seen; a.penalty = penalty; a.tok = tok;
    return cuda_status(krk::greedy(a, (cudaStream_t)stream), "greedy");
}

int krk_k_sample(const float* logits, int64_t ld, int vocab, int B, uint32_t* seen, float temperature,
                 float top_p, int top_k, float penalty, uint32_t* rng_state, uint32_t* tok, void* stream) {
    if (temperature > 1e-6f && !rng_state) return fail(KRK_INVALID, "sampling needs a random state");
    krk::GreedyArgs a{};
    a.logits = logits; a.ld = ld; a.vocab = vocab; a.B = B; a.seen = seen;
    a.penalty = penalty; a.tok = tok;
    a.temperature = temperature; a.top_p = top_p; a.top_k = top_k; a.rng = rng_state;
    return cuda_status(krk::sample(a, (cudaStream_t)stream), "sample");
}

int krk_rng_seed_state(uint64_t seed, uint32_t* state10) {
    if (!state10) return fail(KRK_INVALID, "null state");
    krk::rng_seed_state(seed, state10);
    return KRK_OK;
}

}  // extern "C"
