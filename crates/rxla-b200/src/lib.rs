//! Safe Rust layer over librxla_b200: the B200 (sm_100a) W8A16 linear, the
//! paged GQA decode attention and the W8 decoder runner of rxla's
//! quantized-inference path, behind the plain C ABI of `include/rxla_b200.h`
//! (raw declarations in [`ffi`]).
//!
//! Device memory stays the caller's: the wrappers take raw device pointers
//! ([`DevicePtr`]) and a CUDA stream ([`Stream`]) and are `unsafe` where the
//! library cannot check that the pointers name live device buffers of the
//! stated sizes.  Failures carry the library's status class, which maps one to
//! one onto rxla's `PjrtErrorCode` (crates/rxla-pjrt/src/runtime.rs:46-107),
//! and the library's message.
//!
//! With the `rxla-pjrt` feature, [`register_custom_calls`] registers the XLA
//! custom-call handlers with an rxla PJRT plugin
//! (`Plugin::register_gpu_custom_call`, GpuCustomCallApi::Legacy).

pub mod ffi;

use std::ffi::{c_void, CStr, CString};
use std::fmt;

/// Status classes the library returns (negated absl codes), named as rxla's
/// `PjrtErrorCode` names them.
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum ErrorCode {
    InvalidArgument,
    DeadlineExceeded,
    NotFound,
    ResourceExhausted,
    FailedPrecondition,
    OutOfRange,
    Unimplemented,
    Internal,
    Unavailable,
    /// A status this crate does not know (a newer library).
    Unrecognized(i32),
}

impl ErrorCode {
    /// The class of a nonzero library status.
    pub fn from_status(status: i32) -> Self {
        match status {
            ffi::RXLA_B200_INVALID_ARGUMENT => Self::InvalidArgument,
            ffi::RXLA_B200_DEADLINE_EXCEEDED => Self::DeadlineExceeded,
            ffi::RXLA_B200_NOT_FOUND => Self::NotFound,
            ffi::RXLA_B200_RESOURCE_EXHAUSTED => Self::ResourceExhausted,
            ffi::RXLA_B200_FAILED_PRECONDITION => Self::FailedPrecondition,
            ffi::RXLA_B200_OUT_OF_RANGE => Self::OutOfRange,
            ffi::RXLA_B200_UNIMPLEMENTED => Self::Unimplemented,
            ffi::RXLA_B200_INTERNAL => Self::Internal,
            ffi::RXLA_B200_UNAVAILABLE => Self::Unavailable,
            other => Self::Unrecognized(other),
        }
    }

    /// The same retry rule as `PjrtErrorCode::is_retryable`
    /// (crates/rxla-pjrt/src/runtime.rs:94-107).
    pub fn is_retryable(self) -> bool {
        matches!(self, Self::DeadlineExceeded | Self::ResourceExhausted | Self::Unavailable)
    }
}

#[cfg(feature = "rxla-pjrt")]
impl From<ErrorCode> for rxla_pjrt::PjrtErrorCode {
    fn from(code: ErrorCode) -> Self {
        use rxla_pjrt::PjrtErrorCode as P;
        match code {
            ErrorCode::InvalidArgument => P::InvalidArgument,
            ErrorCode::DeadlineExceeded => P::DeadlineExceeded,
            ErrorCode::NotFound => P::NotFound,
            ErrorCode::ResourceExhausted => P::ResourceExhausted,
            ErrorCode::FailedPrecondition => P::FailedPrecondition,
            ErrorCode::OutOfRange => P::OutOfRange,
            ErrorCode::Unimplemented => P::Unimplemented,
            ErrorCode::Internal => P::Internal,
            ErrorCode::Unavailable => P::Unavailable,
            ErrorCode::Unrecognized(c) => P::Unrecognized((-c) as u32),
        }
    }
}

/// A failing library call: its status class and the library's message.
#[derive(Clone, Debug, PartialEq, Eq)]
pub struct Error {
    pub code: ErrorCode,
    pub message: String,
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "{:?}: {}", self.code, self.message)
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

/// Turn a library status into a `Result`, reading the calling thread's
/// message on failure.
pub fn check(status: i32) -> Result<()> {
    if status == ffi::RXLA_B200_OK {
        return Ok(());
    }
    let message = unsafe {
        let p = ffi::rxla_b200_last_error_message();
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    };
    Err(Error { code: ErrorCode::from_status(status), message })
}

/// A CUDA stream (`cudaStream_t`), null for the legacy default stream.
pub type Stream = *mut c_void;
/// A device pointer the caller owns.
pub type DevicePtr = *mut c_void;

fn cstring(s: &str) -> Result<CString> {
    CString::new(s).map_err(|_| Error {
        code: ErrorCode::InvalidArgument,
        message: format!("string with an interior NUL: {s:?}"),
    })
}

/// Library ABI version (`RXLA_B200_ABI_VERSION` of the header it was built from).
pub fn abi_version() -> i32 {
    unsafe { ffi::rxla_b200_abi_version() }
}

/// SM count and compute capability of `device`.
pub fn device_info(device: i32) -> Result<(i32, i32, i32)> {
    let (mut sm, mut major, mut minor) = (0, 0, 0);
    check(unsafe { ffi::rxla_b200_device_info(device, &mut sm, &mut major, &mut minor) })?;
    Ok((sm, major, minor))
}

/// The current device's status word: `Ok` or the error a bounded device-side
/// wait recorded (`DeadlineExceeded`); `reset` clears it.
pub fn device_status(reset: bool) -> Result<()> {
    check(unsafe { ffi::rxla_b200_device_status(reset as i32) })
}

/// Budget of every bounded device-side wait on the current device.
pub fn set_wait_timeout(ns: i64) -> Result<()> {
    check(unsafe { ffi::rxla_b200_set_wait_timeout(ns) })
}

/// `QuantizedLinear::apply` at BF16 layer compute
/// (crates/rxla-nn/src/layers.rs:257-298): `y = bf16(x) · W_deqᵀ` with the
/// epilogue `epilogue` (`ffi::RXLA_B200_EPI_*`).
///
/// # Safety
/// `x` [m, k] (`x_dtype`), `weight` u8 [n or 2n, k], `scale` f32
/// [rows, k / group_size] and `y` [m, n] (`y_dtype`) must be live device
/// buffers of those sizes, not overlapping `y` except as the epilogue allows,
/// and stay valid until the work queued on `stream` has run.
#[allow(clippy::too_many_arguments)]
pub unsafe fn w8a16_linear(
    x: DevicePtr, x_dtype: i32, weight: DevicePtr, scale: DevicePtr, group_size: i64, m: i64,
    n: i64, k: i64, y: DevicePtr, y_dtype: i32, epilogue: i32, stream: Stream,
) -> Result<()> {
    check(ffi::rxla_b200_w8a16_linear(
        x, x_dtype, weight as *const u8, scale as *const f32, group_size, m, n, k, y, y_dtype,
        epilogue, stream,
    ))
}

/// The same linear with the input RMSNorm of the f32 residual `h` fused into
/// the kernel (crates/rxla-core/src/ops.rs:929-945, then the bf16 cast).
///
/// # Safety
/// As [`w8a16_linear`], with `h` f32 [m, k] and `norm_weight` f32 [k]; `y`
/// must not overlap `h`.
#[allow(clippy::too_many_arguments)]
pub unsafe fn w8a16_norm_linear(
    h: DevicePtr, norm_weight: DevicePtr, eps: f32, weight: DevicePtr, scale: DevicePtr,
    group_size: i64, m: i64, n: i64, k: i64, y: DevicePtr, y_dtype: i32, epilogue: i32,
    stream: Stream,
) -> Result<()> {
    check(ffi::rxla_b200_w8a16_norm_linear(
        h as *const f32, norm_weight as *const f32, eps, weight as *const u8,
        scale as *const f32, group_size, m, n, k, y, y_dtype, epilogue, stream,
    ))
}

/// Bytes of split-K workspace [`paged_decode_attention`] needs for a shape.
pub fn paged_decode_workspace_size(
    batch: i32, q_heads: i32, kv_heads: i32, head_dim: i32, max_context: i32,
) -> Result<usize> {
    let mut bytes = 0usize;
    check(unsafe {
        ffi::rxla_b200_paged_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_context, &mut bytes)
    })?;
    Ok(bytes)
}

/// An empty argument block for the decode attention (sizes and pointers to
/// be filled in), with `struct_size` set.
pub fn paged_decode_args() -> ffi::rxla_b200_paged_decode_args {
    let mut a: ffi::rxla_b200_paged_decode_args = unsafe { std::mem::zeroed() };
    a.struct_size = std::mem::size_of::<ffi::rxla_b200_paged_decode_args>() as u32;
    a.page_size = 16;
    a
}

/// One decode step of GQA over the paged bf16 cache: q/k RMSNorm, RoPE, the
/// KV append (`KvCache::update_at(_checked)`, crates/rxla-core/src/kv_cache.rs:53-112)
/// and `softmax(q·Kᵀ·scale + causal mask)·V` (crates/rxla-core/src/attention.rs:83-252).
///
/// # Safety
/// Every pointer in `args` must name a live device buffer of the size the
/// header documents for it, until the work queued on `stream` has run.
pub unsafe fn paged_decode_attention(args: &ffi::rxla_b200_paged_decode_args, stream: Stream) -> Result<()> {
    check(ffi::rxla_b200_paged_decode_attention(args, stream))
}

/// [`paged_decode_attention`] with the split-K scratch taken from the
/// library's fixed array instead of `args.workspace`: for callers that may
/// not allocate device memory.
///
/// # Safety
/// As [`paged_decode_attention`]; calls that can overlap on the GPU share
/// the one array and race.
pub unsafe fn paged_decode_attention_noalloc(
    args: &ffi::rxla_b200_paged_decode_args, stream: Stream,
) -> Result<()> {
    check(ffi::rxla_b200_paged_decode_attention_noalloc(args, stream))
}

/// A tensor-parallel communicator (NCCL over NVLink; replaces rxla's PJRT
/// distributed client + key-value rendezvous, crates/rxla-pjrt/src/distributed.rs:40-120).
pub struct Comm {
    raw: *mut ffi::rxla_b200_comm,
}

impl Comm {
    /// The rendezvous id rank 0 creates and sends to every rank.
    pub fn unique_id() -> Result<[u8; ffi::RXLA_B200_COMM_ID_BYTES]> {
        let mut id = [0u8; ffi::RXLA_B200_COMM_ID_BYTES];
        check(unsafe { ffi::rxla_b200_comm_unique_id(id.as_mut_ptr()) })?;
        Ok(id)
    }

    /// Collective: every rank calls this with the same id.
    pub fn init(id: &[u8; ffi::RXLA_B200_COMM_ID_BYTES], rank: i32, world: i32, device: i32) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { ffi::rxla_b200_comm_init(id.as_ptr(), rank, world, device, &mut raw) })?;
        Ok(Self { raw })
    }

    pub fn as_raw(&self) -> *mut ffi::rxla_b200_comm {
        self.raw
    }
}

impl Drop for Comm {
    fn drop(&mut self) {
        unsafe { ffi::rxla_b200_comm_destroy(self.raw) };
    }
}

/// The W8 decoder runner: a Qwen3-style decoder with paged bf16 KV state,
/// one CUDA-graph replay per step (`BoundModel::run` / `Session::run`,
/// crates/rxla-nn/src/applied.rs:222-237, crates/rxla-core/src/state.rs:1200-1228).
pub struct Decoder {
    raw: *mut ffi::rxla_b200_decoder,
}

impl Decoder {
    /// A decoder on `device` (tensor-parallel over `comm` when
    /// `config.tp_size > 1`; the comm must outlive the decoder).
    pub fn new(mut config: ffi::rxla_b200_decoder_config, device: i32, comm: Option<&Comm>) -> Result<Self> {
        config.struct_size = std::mem::size_of::<ffi::rxla_b200_decoder_config>() as u32;
        let mut raw = std::ptr::null_mut();
        let c = comm.map_or(std::ptr::null_mut(), |c| c.raw);
        check(unsafe { ffi::rxla_b200_decoder_create(&config, device, c, &mut raw) })?;
        Ok(Self { raw })
    }

    /// Copy a named checkpoint tensor (host bytes) into the decoder.
    pub fn set_parameter(&mut self, name: &str, host: &[u8]) -> Result<()> {
        let n = cstring(name)?;
        check(unsafe {
            ffi::rxla_b200_decoder_set_parameter(self.raw, n.as_ptr(), host.as_ptr().cast(), host.len() as i64)
        })
    }

    /// Load every parameter from an `rxla-qwen3.5-w8-v1` safetensors file;
    /// returns (loaded, skipped) tensor counts.
    pub fn load_safetensors(&mut self, path: &str, prefix: &str) -> Result<(i32, i32)> {
        let (p, x) = (cstring(path)?, cstring(prefix)?);
        let (mut loaded, mut skipped) = (0, 0);
        check(unsafe {
            ffi::rxla_b200_decoder_load_safetensors(self.raw, p.as_ptr(), x.as_ptr(), &mut loaded, &mut skipped)
        })?;
        Ok((loaded, skipped))
    }

    /// One decode step from host tokens to host next tokens (copies and a
    /// stream synchronisation inside).
    pub fn step_host(&mut self, tokens: &[i32], next: &mut [i32], stream: Stream) -> Result<()> {
        if next.len() < tokens.len() {
            return Err(Error { code: ErrorCode::InvalidArgument, message: "next shorter than tokens".into() });
        }
        check(unsafe {
            ffi::rxla_b200_decoder_step_host(self.raw, tokens.as_ptr(), tokens.len() as i32, next.as_mut_ptr(), stream)
        })
    }

    /// One decode step on device buffers (graph replay; no synchronisation).
    ///
    /// # Safety
    /// `tokens` and `next_tokens` are device int32 [batch]; `logits` null or
    /// device f32 [batch, vocab / tp].
    pub unsafe fn step(&mut self, tokens: *const i32, batch: i32, next_tokens: *mut i32, logits: *mut f32,
                       stream: Stream) -> Result<()> {
        check(ffi::rxla_b200_decoder_step(self.raw, tokens, batch, next_tokens, logits, stream))
    }

    /// Run a prompt through the layers for sequence `seq`.
    ///
    /// # Safety
    /// `tokens` is device, managed or pinned int32 [count]; `next_token` null
    /// or device int32 [1]; `logits` null or device f32 [vocab / tp].
    pub unsafe fn prefill(&mut self, seq: i32, tokens: *const i32, count: i32, next_token: *mut i32,
                          logits: *mut f32, stream: Stream) -> Result<()> {
        check(ffi::rxla_b200_decoder_prefill(self.raw, seq, tokens, count, next_token, logits, stream))
    }

    pub fn reset(&mut self, stream: Stream) -> Result<()> {
        check(unsafe { ffi::rxla_b200_decoder_reset(self.raw, stream) })
    }

    pub fn as_raw(&self) -> *mut ffi::rxla_b200_decoder {
        self.raw
    }
}

impl Drop for Decoder {
    fn drop(&mut self) {
        unsafe { ffi::rxla_b200_decoder_destroy(self.raw) };
    }
}

/// backend_config bytes of `rxla_b200_xla_w8a16_linear(_status)`.
pub fn xla_linear_config(
    m: i64, n: i64, k: i64, group_size: i64, x_dtype: i32, y_dtype: i32, epilogue: i32,
    fused_norm: bool, eps: f32,
) -> ffi::rxla_b200_xla_linear_config {
    ffi::rxla_b200_xla_linear_config {
        magic: ffi::RXLA_B200_XLA_LINEAR_MAGIC,
        version: 1,
        m,
        n,
        k,
        group_size,
        x_dtype,
        y_dtype,
        epilogue,
        fused_norm: fused_norm as i32,
        eps,
        reserved: 0,
    }
}

/// The little-endian bytes XLA passes to the handler as `opaque` (the
/// custom call's backend_config), after the library's own validation.
pub fn config_bytes<T: Copy>(target: &str, config: &T) -> Result<Vec<u8>> {
    let bytes = unsafe {
        std::slice::from_raw_parts((config as *const T).cast::<u8>(), std::mem::size_of::<T>())
    }
    .to_vec();
    let t = cstring(target)?;
    check(unsafe { ffi::rxla_b200_xla_check_config(t.as_ptr(), bytes.as_ptr().cast(), bytes.len()) })?;
    Ok(bytes)
}

/// The custom-call targets and their handlers (XLA's status-returning
/// legacy signature, custom-call api_version 2).  Handlers live in
/// librxla_b200.so, which stays loaded for the process lifetime.
pub fn custom_call_handlers() -> [(&'static str, *mut c_void); 2] {
    [
        ("rxla_b200_xla_w8a16_linear_status", ffi::rxla_b200_xla_w8a16_linear_status as *mut c_void),
        (
            "rxla_b200_xla_paged_decode_attention_status",
            ffi::rxla_b200_xla_paged_decode_attention_status as *mut c_void,
        ),
    ]
}

/// Register the handlers with an rxla PJRT plugin through its GPU custom-call
/// extension (crates/rxla-pjrt/src/runtime.rs:395-436), legacy ABI.
///
/// # Safety
/// The plugin must be a CUDA plugin whose XLA calls legacy handlers with the
/// signature above; the library must stay loaded for the process lifetime.
#[cfg(feature = "rxla-pjrt")]
pub unsafe fn register_custom_calls(plugin: &rxla_pjrt::Plugin) -> std::result::Result<(), rxla_pjrt::Error> {
    use std::ptr::NonNull;
    for (name, handler) in custom_call_handlers() {
        let execute = NonNull::new(handler).expect("handler address");
        plugin.register_gpu_custom_call(
            name,
            rxla_pjrt::GpuCustomCallApi::Legacy,
            rxla_pjrt::GpuCustomCallHandlers::execute_only(execute),
        )?;
    }
    Ok(())
}

#[cfg(test)]
mod tests {
    use super::*;

    #[test]
    fn config_layouts_are_the_wire_format() {
        assert_eq!(std::mem::size_of::<ffi::rxla_b200_xla_linear_config>(), 64);
        assert_eq!(std::mem::size_of::<ffi::rxla_b200_xla_attention_config>(), 64);
        assert_eq!(std::mem::offset_of!(ffi::rxla_b200_xla_linear_config, eps), 56);
        assert_eq!(std::mem::offset_of!(ffi::rxla_b200_xla_attention_config, num_pages), 32);
        assert_eq!(std::mem::offset_of!(ffi::rxla_b200_xla_attention_config, scale), 60);
    }

    #[test]
    fn status_classes_map_to_codes() {
        assert_eq!(ErrorCode::from_status(-3), ErrorCode::InvalidArgument);
        assert_eq!(ErrorCode::from_status(-4), ErrorCode::DeadlineExceeded);
        assert!(ErrorCode::from_status(-14).is_retryable());
        assert_eq!(ErrorCode::from_status(-99), ErrorCode::Unrecognized(-99));
    }

    #[test]
    fn linear_config_is_checked_by_the_library() {
        assert_eq!(abi_version(), ffi::RXLA_B200_ABI_VERSION);
        let c = xla_linear_config(4, 64, 128, 128, ffi::RXLA_B200_BF16, ffi::RXLA_B200_BF16, 0, false, 1e-6);
        assert_eq!(config_bytes("rxla_b200_xla_w8a16_linear_status", &c).unwrap().len(), 64);
        let bad = xla_linear_config(4, 64, 128, 48, ffi::RXLA_B200_BF16, ffi::RXLA_B200_BF16, 0, false, 1e-6);
        let e = config_bytes("rxla_b200_xla_w8a16_linear_status", &bad).unwrap_err();
        assert_eq!(e.code, ErrorCode::InvalidArgument);
    }
}
