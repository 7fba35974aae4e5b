//! Raw bindings to libtrs_b200, the C ABI of `include/trs.h`: the B200
//! (sm_100a) broadcast-elementwise / axis-reduction path of tensorrs.
//!
//! tensorrs itself is `#![forbid(unsafe_code)]` (src/lib.rs:50), so the
//! foreign calls live here, in a separate crate; [`safe`] turns every status
//! back into the reference's own behaviour (its panic with its panic text, or
//! `None`).  Every item mirrors a declaration of trs.h one to one (checked
//! against the header by tests/test_rust_binding_cpu.py).
#![allow(non_camel_case_types)]
#![allow(clippy::missing_safety_doc)]

use std::os::raw::{c_char, c_void};

pub const TRS_MAX_DIMS: usize = 8;
pub const TRS_ABI_VERSION: i32 = 1;

/// A cudaStream_t (null: the legacy default stream).
pub type trs_stream = *mut c_void;
/// A trs_status value (a C enum: int).
pub type trs_status = i32;

// trs_dtype
pub const TRS_F32: i32 = 0;
pub const TRS_F64: i32 = 1;
pub const TRS_I32: i32 = 2;
pub const TRS_I64: i32 = 3;

// trs_status
pub const TRS_OK: trs_status = 0;
pub const TRS_NONE: trs_status = 1;
pub const TRS_ERR_SHAPE: trs_status = 2;
pub const TRS_ERR_AXIS: trs_status = 3;
pub const TRS_ERR_EMPTY_AXIS: trs_status = 4;
pub const TRS_ERR_VIEW: trs_status = 5;
pub const TRS_ERR_DTYPE: trs_status = 6;
pub const TRS_ERR_ALIAS: trs_status = 7;
pub const TRS_ERR_OOM: trs_status = 8;
pub const TRS_ERR_CUDA: trs_status = 9;
pub const TRS_ERR_NCCL: trs_status = 10;
pub const TRS_ERR_TIMEOUT: trs_status = 11;
pub const TRS_ERR_ARG: trs_status = 12;
pub const TRS_ERR_DIV_ZERO: trs_status = 13;
pub const TRS_ERR_UNAVAILABLE: trs_status = 14;

// trs_binop
pub const TRS_ADD: i32 = 0;
pub const TRS_SUB: i32 = 1;
pub const TRS_MUL: i32 = 2;
pub const TRS_DIV: i32 = 3;
pub const TRS_POW: i32 = 4;

// trs_unop
pub const TRS_UN_NONE: i32 = 0;
pub const TRS_UN_NEG: i32 = 1;
pub const TRS_UN_RELU: i32 = 2;
pub const TRS_UN_SIGMOID: i32 = 3;
pub const TRS_UN_TANH: i32 = 4;
pub const TRS_UN_ELU: i32 = 5;
pub const TRS_UN_LEAKY_RELU: i32 = 6;
pub const TRS_UN_SELU: i32 = 7;
pub const TRS_UN_EXP: i32 = 8;
pub const TRS_UN_LN: i32 = 9;
pub const TRS_UN_ABS: i32 = 10;
pub const TRS_UN_SIGN: i32 = 11;
pub const TRS_UN_CLAMP: i32 = 12;
pub const TRS_UN_ADD_SCALAR: i32 = 13;
pub const TRS_UN_SUB_SCALAR: i32 = 14;
pub const TRS_UN_RSUB_SCALAR: i32 = 15;
pub const TRS_UN_MUL_SCALAR: i32 = 16;
pub const TRS_UN_DIV_SCALAR: i32 = 17;
pub const TRS_UN_POW_SCALAR: i32 = 18;
pub const TRS_UN_RPOW_SCALAR: i32 = 19;

/// A strided view of a device buffer: the reference's `Tensor` metadata
/// (linalg/tensor/base.rs:159-164) plus the length of its storage.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct trs_view {
    pub data: *mut c_void,
    pub storage_len: i64,
    pub dtype: i32,
    pub ndim: i32,
    pub shape: [i64; TRS_MAX_DIMS],
    pub strides: [i64; TRS_MAX_DIMS],
    pub offset: i64,
}

/// A scalar operand: `f` for f32/f64 tensors, `i` for i32/i64 tensors.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct trs_scalar {
    pub f: f64,
    pub i: i64,
}

/// A fused element-wise program over up to three inputs.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct trs_ew_program {
    pub n_in: i32,
    pub op1: i32,
    pub op2: i32,
    pub epilogue: i32,
    pub p0: trs_scalar,
    pub p1: trs_scalar,
}

/// A communicator of the several-GPU entry points (opaque).
#[repr(C)]
pub struct trs_comm {
    _private: [u8; 0],
}

extern "C" {
    pub fn trs_abi_version() -> i32;
    pub fn trs_last_error(buf: *mut c_char, len: usize) -> usize;
    pub fn trs_status_string(status: i32) -> *const c_char;
    pub fn trs_launch_count() -> u64;
    pub fn trs_scratch_alloc_count() -> u64;
    pub fn trs_async_error(code: *mut i32) -> trs_status;
    pub fn trs_broadcast_shape(a: *const i64, a_ndim: i32, b: *const i64, b_ndim: i32, out_shape: *mut i64, out_ndim: *mut i32) -> trs_status;
    pub fn trs_plan_elementwise(prog: *const trs_ew_program, in_: *const trs_view, out_: *const trs_view, variant: *mut i32, folded_ndim: *mut i32, folded_shape: *mut i64, strides_out: *mut i64, vector_width: *mut i32) -> trs_status;
    pub fn trs_binary(op: i32, a: *const trs_view, b: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_unary(op: i32, x: *const trs_view, params: *const trs_scalar, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_elementwise(prog: *const trs_ew_program, in_: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_elementwise_sum(prog: *const trs_ew_program, in_: *const trs_view, out_: *mut trs_view, sum_out: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_elementwise_row_sums(prog: *const trs_ew_program, in_: *const trs_view, out_: *mut trs_view, row_sums: *mut trs_view, total: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_pack(x: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sum(x: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sum_noalloc(x: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sum_axis(x: *const trs_view, axis: i32, keepdim: i32, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_mean_axis(x: *const trs_view, axis: i32, keepdim: i32, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_max_axis(x: *const trs_view, axis: i32, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_argmax_axis(x: *const trs_view, axis: i32, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_reduce_broadcast_grad(g: *const trs_view, target: *const i64, target_ndim: i32, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sum_to_shape_fused(g: *const trs_view, gate: *const trs_view, mul: *const trs_view, target: *const i64, target_ndim: i32, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_affine_relu_backward(g: *const trs_view, x: *const trs_view, scale: *const trs_view, bias: *const trs_view, grad_scale: *mut trs_view, grad_bias: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_softmax_lastdim(x: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_layer_norm_lastdim(x: *const trs_view, gamma: *const trs_view, beta: *const trs_view, eps: f64, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sgd_step(param: *mut trs_view, grad: *const trs_view, lr: f64, stream: trs_stream) -> trs_status;
    pub fn trs_rmsprop_step(param: *mut trs_view, grad: *const trs_view, v: *mut trs_view, lr: f64, alpha: f64, eps: f64, stream: trs_stream) -> trs_status;
    pub fn trs_adam_step(param: *mut trs_view, grad: *const trs_view, m: *mut trs_view, v: *mut trs_view, lr: f64, beta1: f64, beta2: f64, eps: f64, t: i64, stream: trs_stream) -> trs_status;
    pub fn trs_max_pool2d(x: *const trs_view, kh: i64, kw: i64, sh: i64, sw: i64, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_avg_pool2d(x: *const trs_view, kh: i64, kw: i64, sh: i64, sw: i64, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_max_pool2d_backward(x: *const trs_view, grad_out: *const trs_view, kh: i64, kw: i64, sh: i64, sw: i64, accumulate: i32, grad_x: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_matmul(a: *const trs_view, b: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_matmul_tf32x3(a: *const trs_view, b: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_unfold_2d(x: *const trs_view, kh: i64, kw: i64, sh: i64, sw: i64, ph: i64, pw: i64, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_fold_2d(cols: *const trs_view, kh: i64, kw: i64, sh: i64, sw: i64, ph: i64, pw: i64, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_fill_uniform(out_: *mut trs_view, seed: u64, first: u64, lo: f64, hi: f64, stream: trs_stream) -> trs_status;
    pub fn trs_fill_normal(out_: *mut trs_view, seed: u64, first: u64, stream: trs_stream) -> trs_status;
    pub fn trs_set_device(device: i32) -> trs_status;
    pub fn trs_malloc(ptr: *mut *mut c_void, bytes: usize) -> trs_status;
    pub fn trs_free(ptr: *mut c_void) -> trs_status;
    pub fn trs_memcpy_htod(dst: *mut c_void, src: *const c_void, bytes: usize, stream: trs_stream) -> trs_status;
    pub fn trs_memcpy_dtoh(dst: *mut c_void, src: *const c_void, bytes: usize, stream: trs_stream) -> trs_status;
    pub fn trs_stream_synchronize(stream: trs_stream) -> trs_status;
    pub fn trs_comm_unique_id(id: *mut u8) -> trs_status;
    pub fn trs_comm_init_rank(id: *const u8, nranks: i32, rank: i32, timeout_ms: i32, comm: *mut *mut trs_comm) -> trs_status;
    pub fn trs_comm_destroy(comm: *mut trs_comm) -> trs_status;
    pub fn trs_comm_abort(comm: *mut trs_comm) -> trs_status;
    pub fn trs_comm_peer_exchange(comm: *const trs_comm, active: *mut i32) -> trs_status;
    pub fn trs_sharded_sum(comm: *mut trs_comm, shard: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sharded_elementwise_sum(comm: *mut trs_comm, prog: *const trs_ew_program, in_: *const trs_view, out_: *mut trs_view, sum_out: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sharded_sum_axis0(comm: *mut trs_comm, shard: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sharded_max_axis0(comm: *mut trs_comm, shard: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
    pub fn trs_sharded_argmax_axis0(comm: *mut trs_comm, shard: *const trs_view, out_: *mut trs_view, stream: trs_stream) -> trs_status;
}

/// Safe helpers over the raw calls: the status of a call mapped back onto
/// what the reference does in that case.
pub mod safe {
    use super::*;
    use std::ffi::CStr;

    /// The text of the calling thread's last failure (the reference's panic
    /// message where it has one).
    pub fn last_error() -> String {
        let mut buf = vec![0 as c_char; 4096];
        unsafe {
            trs_last_error(buf.as_mut_ptr(), buf.len());
            CStr::from_ptr(buf.as_ptr()).to_string_lossy().into_owned()
        }
    }

    /// TRS_OK -> Some(()), TRS_NONE -> None (the reference's Option::None);
    /// any other status panics with the library's message, which for the
    /// reference's own panics is the reference's text.
    pub fn check(status: trs_status) -> Option<()> {
        match status {
            TRS_OK => Some(()),
            TRS_NONE => None,
            _ => panic!("{}", last_error()),
        }
    }

    impl trs_view {
        /// A view of `ndim` dimensions; strides default to row-major.
        pub fn new(data: *mut c_void, storage_len: i64, dtype: i32, shape: &[i64], strides: Option<&[i64]>,
                   offset: i64) -> trs_view {
            assert!(shape.len() <= TRS_MAX_DIMS, "rank above TRS_MAX_DIMS");
            let mut v = trs_view { data, storage_len, dtype, ndim: shape.len() as i32, shape: [0; TRS_MAX_DIMS],
                                   strides: [0; TRS_MAX_DIMS], offset };
            let mut step = 1i64;
            for d in (0..shape.len()).rev() {
                v.shape[d] = shape[d];
                v.strides[d] = match strides { Some(s) => s[d], None => step };
                step *= shape[d];
            }
            v
        }
    }
}
