//! The CUDA arm of mlxcel-core's `UnifiedLinear::forward`
//! (crates/mlxcel-core/src/layers.rs:2023-2093) over device arrays.
//!
//! In the reference the quantized arm has three branches, all one FFI call
//! into MLX: a global-scale weight (NVFP4 sidecar) with the fused helper, the
//! same with the fused helper disabled (plain matmul, then the scalar, then
//! the dense bias), and the plain affine case.  Here the first two are one
//! call of `qw_quantized_linear_forward_global_scale` (it evaluates
//! fp16(fp16(x W^T) * s) + b, the unfused branch's op order, which the fused
//! branch also follows) and the third is `qw_quantized_linear_forward`.
//! The library implements affine codes only: an NVFP4 weight reaches the
//! library and comes back as `QW_EUNSUPPORTED`, never a process abort.
//!
//! mlxcel-core's CUDA build adds this module's call behind a `cuda` cargo
//! feature at the head of `UnifiedLinear::forward`'s `Quantized` arm, taking
//! the weight's device arrays in place of its `MlxArray`s; the `Regular`
//! (dense) arm is not on this path.

use std::ffi::{c_void, CString};

use crate::{QwArray, QwError, check};

/// Anything that can describe itself as a device array: the CUDA build's
/// tensor type implements this.
pub trait DeviceArray {
    fn desc(&self) -> QwArray;
}

impl DeviceArray for QwArray {
    fn desc(&self) -> QwArray {
        *self
    }
}

/// The device-resident counterpart of mlxcel-core's `QuantizedWeight`
/// (layers.rs:35-174): packed u32 codes, fp16 scales and biases, the
/// quantization parameters and the optional per-tensor global scale.
pub struct QuantizedDeviceWeight<A: DeviceArray> {
    pub weight: A,
    pub scales: A,
    pub biases: Option<A>,
    pub group_size: i32,
    pub bits: i32,
    pub mode: String,
    pub global_scale: Option<A>,
}

impl<A: DeviceArray> QuantizedDeviceWeight<A> {
    /// Affine weight; checks the packing invariant the reference's loader
    /// enforces (`packed_in * 32 == bits * groups * group_size`,
    /// layers.rs:1568-1570, 1846-1852) and biases shaped like scales
    /// (layers.rs:1855-1866) before any launch.
    pub fn affine(weight: A, scales: A, biases: A, group_size: i32, bits: i32) -> Result<Self, QwError> {
        let (w, s, b) = (weight.desc(), scales.desc(), biases.desc());
        let packed_in = w.shape[(w.ndim - 1) as usize];
        let groups = s.shape[(s.ndim - 1) as usize];
        if packed_in * 32 != bits as i64 * groups * group_size as i64 {
            return Err(QwError {
                code: crate::QW_EINVAL,
                message: format!("packed width {packed_in} does not match {groups} groups of {group_size} at {bits} bits"),
            });
        }
        if s.ndim != b.ndim || s.shape != b.shape {
            return Err(QwError { code: crate::QW_EINVAL, message: "biases must have the shape of scales".into() });
        }
        Ok(Self { weight, scales, biases: Some(biases), group_size, bits, mode: "affine".into(), global_scale: None })
    }

    /// Output features (rows of the packed weight).
    pub fn out_features(&self) -> i64 {
        self.weight.desc().shape[0]
    }
}

/// y = x @ dequantize(weight)^T (* global scale) (+ bias), into the caller's
/// y, asynchronously on `stream` (a `cudaStream_t`).
pub fn quantized_linear_forward<A: DeviceArray>(
    x: &A,
    weight: &QuantizedDeviceWeight<A>,
    bias: Option<&A>,
    y: &mut QwArray,
    stream: *mut c_void,
) -> Result<(), QwError> {
    let mode = CString::new(weight.mode.as_str()).map_err(|_| QwError {
        code: crate::QW_EINVAL,
        message: "mode contains a NUL byte".into(),
    })?;
    let xd = x.desc();
    let wd = weight.weight.desc();
    let sd = weight.scales.desc();
    let bd = weight.biases.as_ref().map(|b| b.desc());
    let lb = bias.map(|b| b.desc());
    let bptr = bd.as_ref().map_or(std::ptr::null(), |b| b as *const QwArray);
    let lbptr = lb.as_ref().map_or(std::ptr::null(), |b| b as *const QwArray);
    // SAFETY: every descriptor lives until the call returns; the library
    // reads them during the call only and launches on `stream`.
    let rc = match weight.global_scale.as_ref() {
        Some(gs) => {
            let g = gs.desc();
            unsafe {
                crate::qw_quantized_linear_forward_global_scale(&xd, &wd, &sd, bptr, &g, lbptr, weight.group_size,
                    weight.bits, mode.as_ptr(), y, stream)
            }
        }
        None => unsafe {
            crate::qw_quantized_linear_forward(&xd, &wd, &sd, bptr, lbptr, weight.group_size, weight.bits,
                mode.as_ptr(), y, stream)
        },
    };
    check(rc)
}
