//! Drop-in for krikil-rs's `model` module (src/model.rs) on a B200: the same
//! public names, signatures, error messages and state bookkeeping, with the
//! weights and the per-sequence state resident on the GPU and the forward
//! pass in the CUDA library of `include/krikil_cuda.h`.
//!
//! * `PebbleModel::load_safetensors` (src/model.rs:233-313) maps the file and
//!   copies every tensor to the device (`krk_model_load`, device 0 or
//!   `KRIKIL_DEVICE`).  Besides the reference's errors it refuses non-F32
//!   tensors and wrong element counts, which the reference would read as
//!   garbage.
//! * `PebbleState::new(&config, max_ctx)` (src/model.rs:204-219) takes no model,
//!   as in the reference, so the device state is created on the first forward
//!   call with the model that makes it; `current_pos` and `context_limit` stay
//!   public fields that src/generate.rs reads unchanged.
//! * `forward_prefill` / `forward_step` (src/model.rs:316, :586) return the
//!   last-token logits as an owned `Vec<f32>` of 2048 and advance
//!   `current_pos`, with the reference's checks in its order before anything
//!   changes.
//!
//! Threading: a `PebbleModel` owns one CUDA stream; calls on states of the same
//! model must not run concurrently from several threads (the type is `Send`,
//! not `Sync`).  Drop every state before its model.
use crate::ffi;
use anyhow::{bail, Result};
use std::ffi::{CStr, CString};
use std::path::Path;

pub const HIDDEN_SIZE: usize = 608;
pub const VOCAB_SIZE: usize = 2048;
pub const INTERMEDIATE_SIZE: usize = 2432;
pub const NUM_LAYERS: usize = 8;
pub const NUM_ATTN_HEADS: usize = 8;
pub const ATTN_HEAD_DIM: usize = 76;
pub const ROPE_THETA: f32 = 10000.0;
pub const RMS_NORM_EPS: f32 = 1e-6;
pub const MAMBA_D_STATE: usize = 128;
pub const MAMBA_D_CONV: usize = 4;
pub const MAMBA_EXPAND: usize = 2;
pub const MAMBA_HEAD_DIM: usize = 64;
pub const MAMBA_D_INNER: usize = HIDDEN_SIZE * MAMBA_EXPAND;
pub const MAMBA_NUM_HEADS: usize = MAMBA_D_INNER / MAMBA_HEAD_DIM;
pub const MAMBA_D_IN_PROJ: usize = 2 * MAMBA_D_INNER + 2 * MAMBA_D_STATE + MAMBA_NUM_HEADS;
pub const MAMBA_D_XBC: usize = MAMBA_D_INNER + 2 * MAMBA_D_STATE;
pub const MAMBA_NORM_EPS: f32 = 1e-5;

/// The model dimensions (src/model.rs:32-84).  The library is built for these
/// dimensions; other values are refused when a state is created.
#[derive(Debug, Clone)]
pub struct PebbleConfig {
    pub vocab_size: usize,
    pub hidden_size: usize,
    pub num_hidden_layers: usize,
    pub num_attention_heads: usize,
    pub intermediate_size: usize,
    pub max_position_embeddings: usize,
    pub block_pattern: String,
}

impl Default for PebbleConfig {
    fn default() -> Self {
        Self {
            vocab_size: VOCAB_SIZE,
            hidden_size: HIDDEN_SIZE,
            num_hidden_layers: NUM_LAYERS,
            num_attention_heads: NUM_ATTN_HEADS,
            intermediate_size: INTERMEDIATE_SIZE,
            max_position_embeddings: 2048,
            block_pattern: "mmma|mmma".to_string(),
        }
    }
}

fn last_error() -> String {
    unsafe {
        let p = ffi::krk_last_error();
        if p.is_null() {
            return String::new();
        }
        CStr::from_ptr(p).to_string_lossy().into_owned()
    }
}

/// A non-zero status as an `anyhow` error carrying the library's message (the
/// reference's own wording for the errors it raises itself).
fn check(rc: std::ffi::c_int) -> Result<()> {
    if rc == ffi::KRK_OK {
        Ok(())
    } else {
        bail!("{}", last_error())
    }
}

pub struct PebbleModel {
    pub config: PebbleConfig,
    h: *mut ffi::krk_model,
}

// One CUDA stream per model: movable between threads, not shared by them.
unsafe impl Send for PebbleModel {}

pub struct PebbleState {
    pub context_limit: usize,
    pub current_pos: usize,
    config: PebbleConfig,
    h: *mut ffi::krk_state,
    model: *const ffi::krk_model,
}

unsafe impl Send for PebbleState {}

impl PebbleState {
    /// src/model.rs:204-219.  The device state is made on first use.
    pub fn new(config: &PebbleConfig, max_ctx: usize) -> Self {
        Self { context_limit: max_ctx, current_pos: 0, config: config.clone(), h: std::ptr::null_mut(),
               model: std::ptr::null() }
    }

    /// src/model.rs:221-229: position 0, Mamba conv/SSD state zeroed, attention
    /// caches rewound.
    pub fn reset(&mut self) {
        self.current_pos = 0;
        if !self.h.is_null() {
            let rc = unsafe { ffi::krk_state_reset(self.h, std::ptr::null()) };
            assert_eq!(rc, ffi::KRK_OK, "state reset: {}", last_error());
        }
    }

    /// The device state of `model` for this sequence, created on first use.
    fn bind(&mut self, model: &PebbleModel) -> Result<*mut ffi::krk_state> {
        if self.h.is_null() {
            let c = &self.config;
            let d = PebbleConfig::default();
            if c.vocab_size != d.vocab_size || c.hidden_size != d.hidden_size
                || c.num_hidden_layers != d.num_hidden_layers || c.num_attention_heads != d.num_attention_heads
                || c.intermediate_size != d.intermediate_size || c.block_pattern != d.block_pattern {
                bail!("the B200 library is built for the Pebble-25M dimensions; got {:?}", c);
            }
            let mut h = std::ptr::null_mut();
            check(unsafe { ffi::krk_state_create(model.h, 1, self.context_limit as i32, &mut h) })?;
            self.h = h;
            self.model = model.h;
            if self.current_pos != 0 {
                bail!("internal: a new device state at position {}", self.current_pos);
            }
        } else if self.model != model.h as *const _ {
            bail!("this state belongs to another model");
        }
        Ok(self.h)
    }

    fn device_pos(&self) -> Result<usize> {
        let mut p = 0i64;
        check(unsafe { ffi::krk_state_positions(self.h, &mut p) })?;
        Ok(p as usize)
    }
}

impl Drop for PebbleState {
    fn drop(&mut self) {
        if !self.h.is_null() {
            unsafe { ffi::krk_state_free(self.h) };
        }
    }
}

impl PebbleModel {
    /// src/model.rs:233-313.
    pub fn load_safetensors(model_path: impl AsRef<Path>) -> Result<Self> {
        let path = CString::new(model_path.as_ref().to_string_lossy().as_bytes())?;
        let device = std::env::var("KRIKIL_DEVICE").ok().and_then(|v| v.parse::<i32>().ok()).unwrap_or(0);
        let mut h = std::ptr::null_mut();
        check(unsafe { ffi::krk_model_load(path.as_ptr(), device, &mut h) })?;
        Ok(Self { config: PebbleConfig::default(), h })
    }

    /// src/model.rs:316-368: prefill `tokens` at the state's position and
    /// return the last token's logits.  Errors (before any change): empty
    /// input, context overflow, token id >= vocab.
    pub fn forward_prefill(&self, tokens: &[u32], state: &mut PebbleState) -> Result<Vec<f32>> {
        if tokens.is_empty() {
            bail!("Cannot prefill empty sequence");
        }
        let end = state.current_pos + tokens.len();
        if end > state.context_limit {
            bail!("Sequence length {} exceeds context limit {}", end, state.context_limit);
        }
        let h = state.bind(self)?;
        let lens = [tokens.len() as i32];
        let mut logits = vec![0.0f32; VOCAB_SIZE];
        check(unsafe { ffi::krk_prefill(self.h, h, tokens.as_ptr(), lens.as_ptr(), logits.as_mut_ptr()) })?;
        state.current_pos = state.device_pos()?;
        Ok(logits)
    }

    /// src/model.rs:586-624: one token at the state's position.  Errors
    /// (before any change): token id >= vocab, then the context limit.
    pub fn forward_step(&self, token: u32, state: &mut PebbleState) -> Result<Vec<f32>> {
        if token as usize >= VOCAB_SIZE {
            bail!("Token ID {} exceeds vocab size {}", token, VOCAB_SIZE);
        }
        if state.current_pos >= state.context_limit {
            bail!("Context limit {} reached", state.context_limit);
        }
        let h = state.bind(self)?;
        let mut logits = vec![0.0f32; VOCAB_SIZE];
        check(unsafe { ffi::krk_step(self.h, h, &token, logits.as_mut_ptr()) })?;
        state.current_pos = state.device_pos()?;
        Ok(logits)
    }

    /// The whole greedy or sampled generation of one sequence on the device
    /// (reset, prefill, then per token the pick and the step), the loop of
    /// src/generate.rs:65-114 with Sampler::sample (src/sampler.rs:43-152) at
    /// `temperature` (<= 1e-6: greedy) and `seed` for rand's StdRng.  Returns
    /// the generated tokens (EOS not included).
    #[allow(clippy::too_many_arguments)]
    pub fn generate_on_device(&self, prompt: &[u32], state: &mut PebbleState, max_new_tokens: usize,
                              temperature: f32, top_p: f32, top_k: usize, repetition_penalty: f32, seed: u64,
                              stop_at_eos: bool) -> Result<Vec<u32>> {
        state.current_pos = 0;
        let h = state.bind(self)?;
        let lens = [prompt.len() as i32];
        let mut out = vec![0u32; max_new_tokens.max(1)];
        let mut n = 0i32;
        check(unsafe {
            ffi::krk_generate_sample(self.h, h, prompt.as_ptr(), lens.as_ptr(), max_new_tokens as i32, temperature,
                                     top_p, top_k as i32, repetition_penalty, &seed, stop_at_eos as i32,
                                     out.as_mut_ptr(), &mut n)
        })?;
        state.current_pos = state.device_pos()?;
        out.truncate(n as usize);
        Ok(out)
    }
}

impl Drop for PebbleModel {
    fn drop(&mut self) {
        unsafe { ffi::krk_model_free(self.h) };
    }
}
