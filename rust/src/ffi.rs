//! Raw declarations of the C ABI in `include/krikil_cuda.h`, one for one (same
//! names, argument order and C types).  Handles are opaque; every function
//! returns a `krk_status` (`KRK_OK` = 0) unless noted, with the message of the
//! last failure on the calling thread in `krk_last_error()`.  Device pointers
//! are passed as raw pointers; `stream` is a `cudaStream_t` (null = the
//! default stream).
#![allow(non_camel_case_types, dead_code)]

use std::ffi::{c_char, c_double, c_float, c_int, c_void};

pub const KRK_ABI_VERSION: c_int = 1;

pub const KRK_HIDDEN: usize = 608;
pub const KRK_VOCAB: usize = 2048;
pub const KRK_INTERMEDIATE: usize = 2432;
pub const KRK_LAYERS: usize = 8;
pub const KRK_ATTN_HEADS: usize = 8;
pub const KRK_ATTN_HEAD_DIM: usize = 76;
pub const KRK_MAMBA_D_STATE: usize = 128;
pub const KRK_MAMBA_D_CONV: usize = 4;
pub const KRK_MAMBA_D_INNER: usize = 1216;
pub const KRK_MAMBA_HEAD_DIM: usize = 64;
pub const KRK_MAMBA_HEADS: usize = 19;
pub const KRK_MAMBA_D_IN_PROJ: usize = 2707;
pub const KRK_MAMBA_D_XBC: usize = 1472;
pub const KRK_EOS_TOKEN: u32 = 0;

// enum krk_status
pub const KRK_OK: c_int = 0;
pub const KRK_BAD_TOKEN: c_int = 1;
pub const KRK_CONTEXT_OVERFLOW: c_int = 2;
pub const KRK_EMPTY: c_int = 3;
pub const KRK_IO: c_int = 4;
pub const KRK_NOT_FOUND: c_int = 5;
pub const KRK_INVALID: c_int = 6;
pub const KRK_CUDA: c_int = 7;
pub const KRK_CHECK_FAILED: c_int = 8;

// krk_state_profile classes
pub const KRK_PROF_DEVICE_TOTAL: c_int = 0;
pub const KRK_PROF_GEMM: c_int = 1;
pub const KRK_PROF_SSD_STEP: c_int = 2;
pub const KRK_PROF_ATTN_DECODE: c_int = 3;
pub const KRK_PROF_NORM: c_int = 4;
pub const KRK_PROF_CONV: c_int = 5;
pub const KRK_PROF_SSD_SCAN: c_int = 6;
pub const KRK_PROF_ATTN_PREFILL: c_int = 7;
pub const KRK_PROF_OTHER: c_int = 8;
pub const KRK_PROF_CLASSES: c_int = 9;

pub const KRK_ATTN_NOALLOC_MAX_FLOATS: usize = 1 << 20;

// krk_check_status bits (checked builds)
pub const KRK_CHECK_TOKEN: u32 = 1;
pub const KRK_CHECK_POSITION: u32 = 2;
pub const KRK_CHECK_TABLE: u32 = 4;
pub const KRK_CHECK_COLUMN: u32 = 8;

#[repr(C)]
pub struct krk_model {
    _private: [u8; 0],
}
#[repr(C)]
pub struct krk_state {
    _private: [u8; 0],
}

extern "C" {
    pub fn krk_last_error() -> *const c_char;
    pub fn krk_status_string(status: c_int) -> *const c_char;
    pub fn krk_abi_version() -> c_int;

    pub fn krk_model_load(path: *const c_char, device: c_int, out: *mut *mut krk_model) -> c_int;
    pub fn krk_model_free(model: *mut krk_model) -> c_int;
    pub fn krk_model_device(model: *const krk_model, device: *mut c_int) -> c_int;
    pub fn krk_model_stream(model: *const krk_model, stream: *mut *mut c_void) -> c_int;

    pub fn krk_state_create(model: *const krk_model, batch: c_int, max_ctx: c_int, out: *mut *mut krk_state) -> c_int;
    pub fn krk_state_free(state: *mut krk_state) -> c_int;
    pub fn krk_state_reset(state: *mut krk_state, mask: *const u8) -> c_int;
    pub fn krk_state_batch(state: *const krk_state, batch: *mut c_int) -> c_int;
    pub fn krk_state_context_limit(state: *const krk_state, max_ctx: *mut c_int) -> c_int;
    pub fn krk_state_positions(state: *const krk_state, pos_out: *mut i64) -> c_int;

    pub fn krk_prefill(model: *const krk_model, state: *mut krk_state, tokens: *const u32, lens: *const i32,
                       logits_out: *mut c_float) -> c_int;
    pub fn krk_step(model: *const krk_model, state: *mut krk_state, tokens: *const u32, logits_out: *mut c_float)
                    -> c_int;
    pub fn krk_generate_greedy(model: *const krk_model, state: *mut krk_state, prompts: *const u32,
                               lens: *const i32, max_new_tokens: c_int, repetition_penalty: c_float,
                               stop_at_eos: c_int, tokens_out: *mut u32, n_out: *mut i32) -> c_int;
    pub fn krk_generate_sample(model: *const krk_model, state: *mut krk_state, prompts: *const u32,
                               lens: *const i32, max_new_tokens: c_int, temperature: c_float, top_p: c_float,
                               top_k: c_int, repetition_penalty: c_float, seeds: *const u64, stop_at_eos: c_int,
                               tokens_out: *mut u32, n_out: *mut i32) -> c_int;
    pub fn krk_state_export(state: *const krk_state, seq: c_int, layer: c_int, what: c_int, out: *mut c_float,
                            n: i64) -> c_int;
    pub fn krk_launch_count(count: *mut u64) -> c_int;
    pub fn krk_checked_build() -> c_int;
    pub fn krk_check_status(bits: *mut u32, clear: c_int) -> c_int;
    pub fn krk_state_set_decode_streams(state: *mut krk_state, n: c_int) -> c_int;
    pub fn krk_state_set_step_graphs(state: *mut krk_state, enable: c_int) -> c_int;
    pub fn krk_state_profile(state: *mut krk_state, enable: c_int) -> c_int;
    pub fn krk_state_profile_read(state: *const krk_state, cls: c_int, total_ms: *mut c_double,
                                  launches: *mut i64) -> c_int;
    pub fn krk_state_profile_units(state: *const krk_state, cls: c_int, units: *mut i64) -> c_int;

    // per-kernel entry points (device pointers, asynchronous on `stream`)
    pub fn krk_k_rmsnorm_rows(x: *const c_float, w: *const c_float, eps: c_float, rows: i64, dim: c_int,
                              y: *mut c_float, stream: *mut c_void) -> c_int;
    pub fn krk_k_rmsnorm_fm(x: *const c_float, ldx: c_int, w: *const c_float, eps: c_float, k: c_int, m: c_int,
                            out: *mut c_float, ldo: c_int, stream: *mut c_void) -> c_int;
    pub fn krk_k_gated_rmsnorm_residual(x: *const c_float, z: *const c_float, res: *const c_float,
                                        w: *const c_float, eps: c_float, rows: i64, dim: c_int, y: *mut c_float,
                                        stream: *mut c_void) -> c_int;
    pub fn krk_k_gemm(at: *const c_float, lda: c_int, wt: *const c_float, ldw: c_int, c: *mut c_float, ldc: c_int,
                      m: c_int, n: c_int, k: c_int, epilogue: c_int, out_fm: c_int, stream: *mut c_void) -> c_int;
    pub fn krk_k_gemm_tiled(at: *const c_float, lda: c_int, wt: *const c_float, ldw: c_int, c: *mut c_float,
                            ldc: c_int, m: c_int, n: c_int, k: c_int, epilogue: c_int, out_fm: c_int,
                            tile_rows: c_int, stream: *mut c_void) -> c_int;
    pub fn krk_k_gemm_tile_rows(m: c_int, n: c_int) -> c_int;
    pub fn krk_k_embed(tok: *const u32, wte: *const c_float, vocab: c_int, k: c_int, m: c_int, out: *mut c_float,
                       ldo: c_int, stream: *mut c_void) -> c_int;
    pub fn krk_k_pointwise(op: c_int, x: *const c_float, y: *mut c_float, n: i64, stream: *mut c_void) -> c_int;
    pub fn krk_k_conv_ssd_step(x: *const c_float, bm: *const c_float, cm: *const c_float, dt: *const c_float,
                               conv_state: *mut c_float, conv_w: *const c_float, conv_b: *const c_float,
                               ssm: *mut c_float, dt_bias: *const c_float, a_neg: *const c_float,
                               dsk: *const c_float, y: *mut c_float, b: c_int, h: c_int, p: c_int, n: c_int,
                               stream: *mut c_void) -> c_int;
    pub fn krk_k_conv_ssd_scan(x: *const c_float, bm: *const c_float, cm: *const c_float, dt: *const c_float,
                               conv_state: *mut c_float, conv_w: *const c_float, conv_b: *const c_float,
                               ssm: *mut c_float, dt_bias: *const c_float, a_neg: *const c_float,
                               dsk: *const c_float, y: *mut c_float, b: c_int, t: c_int, h: c_int, p: c_int,
                               n: c_int, stream: *mut c_void) -> c_int;
    /// Returns a size, not a status.
    pub fn krk_attn_work_floats(b: c_int, h: c_int, dh: c_int, ctx: c_int, split: c_int) -> usize;
    pub fn krk_k_rope_kv_attn_decode(q: *const c_float, k: *const c_float, v: *const c_float, kc: *mut c_float,
                                     vc: *mut c_float, pos: *const i32, out: *mut c_float, work: *mut c_float,
                                     b: c_int, h: c_int, dh: c_int, ctx: c_int, split: c_int, theta: c_float,
                                     stream: *mut c_void) -> c_int;
    pub fn krk_k_gemm_sgemm_order(at: *const c_float, lda: c_int, wt: *const c_float, ldw: c_int, c: *mut c_float,
                                  ldc: c_int, m: c_int, n: c_int, k: c_int, stream: *mut c_void) -> c_int;
    pub fn krk_k_attn_prefill_rows(kmax: c_int, dh: c_int) -> c_int;
    pub fn krk_k_rope_kv_attn_prefill(qkv: *mut c_float, q_rs: i64, kc: *mut c_float, vc: *mut c_float, c_sb: i64,
                                      c_sh: i64, c_st: i64, cu_seqlens: *const i32, start: *const i32, s: c_int,
                                      total_rows: c_int, h: c_int, dh: c_int, theta: c_float, blocks: *const i32,
                                      nblocks: c_int, rows_per_block: c_int, kmax: c_int, out: *mut c_float,
                                      o_rs: i64, o_cs: i64, stream: *mut c_void) -> c_int;
    pub fn krk_k_rope_kv_attn_decode_noalloc(q: *const c_float, k: *const c_float, v: *const c_float,
                                             kc: *mut c_float, vc: *mut c_float, pos: *const i32,
                                             out: *mut c_float, b: c_int, h: c_int, dh: c_int, ctx: c_int,
                                             split: c_int, theta: c_float, stream: *mut c_void) -> c_int;
    pub fn krk_k_wait_probe(src16: *const c_float, polls: c_int, copy: c_int, status: *mut i32,
                            stream: *mut c_void) -> c_int;
    pub fn krk_k_greedy(logits: *const c_float, ld: i64, vocab: c_int, b: c_int, seen: *mut u32, penalty: c_float,
                        tok: *mut u32, stream: *mut c_void) -> c_int;
    pub fn krk_k_sample(logits: *const c_float, ld: i64, vocab: c_int, b: c_int, seen: *mut u32,
                        temperature: c_float, top_p: c_float, top_k: c_int, penalty: c_float, rng_state: *mut u32,
                        tok: *mut u32, stream: *mut c_void) -> c_int;
    pub fn krk_rng_seed_state(seed: u64, state10: *mut u32) -> c_int;
}
