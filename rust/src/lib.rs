//! B200 forward path for krikil-rs.  `model` is a drop-in for the reference's
//! `src/model.rs` public API (src/lib.rs:3 `pub mod model;`): point that module
//! at this crate (`pub use krikil_b200::model;` or copy the module path) and
//! src/generate.rs, src/main.rs and the reference's tests compile unchanged,
//! running the forward pass on the GPU.  `ffi` is the raw C ABI of
//! include/krikil_cuda.h.
pub mod ffi;
pub mod model;

pub use model::{PebbleConfig, PebbleModel, PebbleState};

/// The library's ABI version (include/krikil_cuda.h KRK_ABI_VERSION).
pub fn abi_version() -> i32 {
    unsafe { ffi::krk_abi_version() }
}
