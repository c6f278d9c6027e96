//! Rust binding of `libqwqmm.so`, the sm_100a affine group-quantized matmul
//! library, for the CUDA build of mlxcel-core.
//!
//! The `extern "C"` block below declares every entry point of
//! `include/qw_qmm.h` with the same argument order and meaning; each one
//! stands in for one function of mlxcel-core's cxx bridge
//! (`crates/mlxcel-core/src/lib.rs`), e.g. `qw_quantized_matmul` for
//! `quantized_matmul` (lib.rs:1134-1143) and `qw_quantized_linear_forward`
//! for `quantized_linear_forward` (lib.rs:591-601).  Arrays are described by
//! [`QwArray`] (device pointer, dtype, shape, strides) instead of
//! `MlxArray`; outputs are preallocated by the caller; every call is
//! asynchronous on the caller's CUDA stream; errors come back as status
//! codes with a message from [`last_error`] instead of a C++ exception (which
//! the bridge turns into `std::terminate`, layers.rs:1255-1285).
//!
//! [`linear`] holds the CUDA arm of `UnifiedLinear::forward`
//! (layers.rs:2023-2093) written over this binding.
//!
//! Built and tested where cargo is available; a Python test of this
//! repository checks that the block below and the C header agree name by
//! name and argument by argument.

use std::ffi::{c_char, c_int, c_void, CStr};
use std::fmt;

pub mod linear;

/// `QW_ABI_VERSION` of the header this crate was written against.
pub const QW_ABI_VERSION: c_int = 1;

pub const QW_OK: c_int = 0;
pub const QW_EINVAL: c_int = 1;
pub const QW_EUNSUPPORTED: c_int = 2;
pub const QW_ECUDA: c_int = 3;
pub const QW_ETIMEOUT: c_int = 4;
pub const QW_ENOMEM: c_int = 5;

pub const QW_U32: i32 = 1;
pub const QW_F16: i32 = 2;
pub const QW_BF16: i32 = 3;
pub const QW_F32: i32 = 4;

pub const QW_IPC_HANDLE_BYTES: usize = 64;

/// A device array (the role `MlxArray` plays at the bridge).  `strides` are
/// in elements; all-zero strides mean row-contiguous.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct QwArray {
    pub data: *mut c_void,
    pub dtype: i32,
    pub ndim: i32,
    pub shape: [i64; 4],
    pub strides: [i64; 4],
}

impl QwArray {
    /// A row-contiguous array of `shape` (1 to 4 dimensions) at `data`.
    pub fn contiguous(data: *mut c_void, dtype: i32, shape: &[i64]) -> Self {
        assert!((1..=4).contains(&shape.len()), "1 to 4 dimensions");
        let mut a = QwArray { data, dtype, ndim: shape.len() as i32, shape: [0; 4], strides: [0; 4] };
        let mut stride = 1i64;
        for i in (0..shape.len()).rev() {
            a.shape[i] = shape[i];
            a.strides[i] = stride;
            stride *= shape[i];
        }
        a
    }

    /// Rows of `cols` halves placed `ld` elements apart (a column slice of
    /// a wider fp16 matrix, which the matmuls accept as x without a copy).
    pub fn f16_rows(data: *mut c_void, rows: i64, cols: i64, ld: i64) -> Self {
        let mut a = Self::contiguous(data, QW_F16, &[rows, cols]);
        a.strides[0] = ld;
        a
    }
}

/// One matmul of a chained launch (`qw_quantized_matmul_chain`).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct QwQmmOp {
    pub x: *const QwArray,
    pub w: *const QwArray,
    pub scales: *const QwArray,
    pub biases: *const QwArray,
    pub y: *mut QwArray,
}

/// Opaque peer-allreduce communicator.
#[repr(C)]
pub struct QwAllreduce {
    _private: [u8; 0],
}

#[link(name = "qwqmm")]
unsafe extern "C" {
    pub fn qw_quantized_matmul(x: *const QwArray, w: *const QwArray, scales: *const QwArray,
        biases: *const QwArray, transpose: c_int, group_size: c_int, bits: c_int,
        mode: *const c_char, y: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_quantized_matmul_chain(ops: *const QwQmmOp, n_ops: c_int, group_size: c_int,
        bits: c_int, mode: *const c_char, stream: *mut c_void) -> c_int;
    pub fn qw_quantized_matmul_argmax(x: *const QwArray, w: *const QwArray, scales: *const QwArray,
        biases: *const QwArray, group_size: c_int, bits: c_int, mode: *const c_char,
        logits: *mut QwArray, idx: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_topk(logits: *const QwArray, k: c_int, idx: *mut QwArray, values: *mut QwArray,
        stream: *mut c_void) -> c_int;
    pub fn qw_quantized_matmul_topk(x: *const QwArray, w: *const QwArray, scales: *const QwArray,
        biases: *const QwArray, group_size: c_int, bits: c_int, mode: *const c_char, k: c_int,
        logits: *mut QwArray, idx: *mut QwArray, values: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_quantized_matmul_swiglu(x: *const QwArray, w_gate: *const QwArray,
        scales_gate: *const QwArray, biases_gate: *const QwArray, w_up: *const QwArray,
        scales_up: *const QwArray, biases_up: *const QwArray, transpose: c_int, group_size: c_int,
        bits: c_int, mode: *const c_char, y: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_swiglu_activation(gate: *const QwArray, up: *const QwArray, y: *mut QwArray,
        stream: *mut c_void) -> c_int;
    pub fn qw_swiglu_mlp(x: *const QwArray, w_gate: *const QwArray, scales_gate: *const QwArray,
        biases_gate: *const QwArray, w_up: *const QwArray, scales_up: *const QwArray,
        biases_up: *const QwArray, w_down: *const QwArray, scales_down: *const QwArray,
        biases_down: *const QwArray, group_size: c_int, bits: c_int, mode: *const c_char,
        y: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_quantized_matmul_static_scratch(x: *const QwArray, w: *const QwArray,
        scales: *const QwArray, biases: *const QwArray, transpose: c_int, group_size: c_int,
        bits: c_int, mode: *const c_char, y: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_allreduce_init(world: c_int, rank: c_int, max_elems: i64, comm: *mut *mut QwAllreduce,
        handle: *mut u8) -> c_int;
    pub fn qw_allreduce_connect(comm: *mut QwAllreduce, handles: *const u8) -> c_int;
    pub fn qw_allreduce_sum(comm: *mut QwAllreduce, partial: *const QwArray, y: *mut QwArray,
        stream: *mut c_void) -> c_int;
    pub fn qw_allreduce_destroy(comm: *mut QwAllreduce) -> c_int;
    pub fn qw_decode_schedule(m: i64, n: i64, k: i64, bits: c_int, group_size: c_int, swiglu: c_int,
        sm_count: c_int, out: *mut i64) -> c_int;
    pub fn qw_allreduce_matmul(comm: *mut QwAllreduce, x: *const QwArray, w: *const QwArray,
        scales: *const QwArray, biases: *const QwArray, group_size: c_int, bits: c_int,
        mode: *const c_char, y: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_allreduce_argmax(comm: *mut QwAllreduce, x: *const QwArray, w: *const QwArray,
        scales: *const QwArray, biases: *const QwArray, group_size: c_int, bits: c_int,
        mode: *const c_char, index_base: i64, logits: *mut QwArray, idx: *mut QwArray,
        stream: *mut c_void) -> c_int;
    pub fn qw_quantized_linear_forward(x: *const QwArray, w: *const QwArray, scales: *const QwArray,
        biases: *const QwArray, linear_bias: *const QwArray, group_size: c_int, bits: c_int,
        mode: *const c_char, y: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_quantized_linear_forward_global_scale(x: *const QwArray, w: *const QwArray,
        scales: *const QwArray, biases: *const QwArray, global_scale: *const QwArray,
        linear_bias: *const QwArray, group_size: c_int, bits: c_int, mode: *const c_char,
        y: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_dequantize(w: *const QwArray, scales: *const QwArray, biases: *const QwArray,
        group_size: c_int, bits: c_int, mode: *const c_char, out: *mut QwArray,
        stream: *mut c_void) -> c_int;
    pub fn qw_dequantize_rounding(w: *const QwArray, scales: *const QwArray, biases: *const QwArray,
        group_size: c_int, bits: c_int, mode: *const c_char, rounding: c_int, out: *mut QwArray,
        stream: *mut c_void) -> c_int;
    pub fn qw_quantize(w: *const QwArray, group_size: c_int, bits: c_int, mode: *const c_char,
        wq: *mut QwArray, scales: *mut QwArray, biases: *mut QwArray, stream: *mut c_void) -> c_int;
    pub fn qw_last_error() -> *const c_char;
    pub fn qw_device_status(device: c_int, status: *mut u32, clear: c_int) -> c_int;
    pub fn qw_abi_version() -> c_int;
}

/// A failed call: its status code and the library's message.
#[derive(Clone, Debug, PartialEq, Eq)]
pub struct QwError {
    pub code: c_int,
    pub message: String,
}

impl fmt::Display for QwError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        let kind = match self.code {
            QW_EINVAL => "invalid arguments",
            QW_EUNSUPPORTED => "unsupported quantization",
            QW_ECUDA => "CUDA error",
            QW_ETIMEOUT => "device wait timed out",
            QW_ENOMEM => "out of device memory",
            _ => "error",
        };
        write!(f, "{kind} ({}): {}", self.code, self.message)
    }
}

impl std::error::Error for QwError {}

/// Message of this thread's last failing call.
pub fn last_error() -> String {
    // SAFETY: the library returns a thread-local NUL-terminated string.
    unsafe { CStr::from_ptr(qw_last_error()) }.to_string_lossy().into_owned()
}

/// `Ok(())` for `QW_OK`, the code and message otherwise.
pub fn check(rc: c_int) -> Result<(), QwError> {
    if rc == QW_OK { Ok(()) } else { Err(QwError { code: rc, message: last_error() }) }
}

/// The library's ABI version must be the one this crate declares.
pub fn check_abi() -> Result<(), QwError> {
    // SAFETY: no arguments, no device work.
    let v = unsafe { qw_abi_version() };
    if v == QW_ABI_VERSION {
        Ok(())
    } else {
        Err(QwError { code: QW_EINVAL, message: format!("libqwqmm ABI {v}, crate expects {QW_ABI_VERSION}") })
    }
}

/// The device status word: `Ok(())` when every bounded wait of the work
/// issued so far completed (synchronises the device).
pub fn device_status(device: i32, clear: bool) -> Result<(), QwError> {
    let mut word = 0u32;
    // SAFETY: `word` outlives the call.
    check(unsafe { qw_device_status(device, &mut word, clear as c_int) })
}

#[cfg(test)]
mod tests {
    //! Argument checks that run before any device work, in the manner of
    //! mlxcel-core's ffi_tests: the shapes the reference's validators reject
    //! come back as status codes here.
    use super::*;
    use std::ptr::null_mut;

    fn affine() -> std::ffi::CString {
        std::ffi::CString::new("affine").unwrap()
    }

    #[test]
    fn abi_version_matches() {
        check_abi().unwrap();
    }

    #[test]
    fn transpose_false_is_unsupported() {
        let x = QwArray::contiguous(8 as *mut c_void, QW_F16, &[1, 128]);
        let w = QwArray::contiguous(8 as *mut c_void, QW_U32, &[4, 16]);
        let s = QwArray::contiguous(8 as *mut c_void, QW_F16, &[4, 2]);
        let mut y = QwArray::contiguous(8 as *mut c_void, QW_F16, &[1, 4]);
        let m = affine();
        let rc = unsafe { qw_quantized_matmul(&x, &w, &s, &s, 0, 64, 4, m.as_ptr(), &mut y, null_mut()) };
        assert_eq!(rc, QW_EUNSUPPORTED);
    }

    #[test]
    fn packing_invariant_is_checked() {
        // packed_in * 32 == bits * groups * group_size (layers.rs:1568-1570)
        let x = QwArray::contiguous(8 as *mut c_void, QW_F16, &[1, 128]);
        let w = QwArray::contiguous(8 as *mut c_void, QW_U32, &[4, 15]);
        let s = QwArray::contiguous(8 as *mut c_void, QW_F16, &[4, 2]);
        let mut y = QwArray::contiguous(8 as *mut c_void, QW_F16, &[1, 4]);
        let m = affine();
        let rc = unsafe { qw_quantized_matmul(&x, &w, &s, &s, 1, 64, 4, m.as_ptr(), &mut y, null_mut()) };
        assert_eq!(rc, QW_EINVAL);
        assert!(!last_error().is_empty());
    }
}
