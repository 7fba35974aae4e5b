/*
 * trs.h -- C ABI of the B200 (sm_100a) broadcast-elementwise / axis-reduction
 * path of tensorrs (GooseKIller/Tensors, crate `tensorrs` 0.4.1).
 *
 * Every entry point below replaces one function of the reference's strided
 * `Tensor<T>` (src/linalg/tensor/base.rs, src/linalg/tensor/ops.rs) or one
 * composition its callers build out of those functions (src/activation,
 * src/autodiff, src/nn).  The citation on each declaration names the
 * reference code whose result it reproduces.
 *
 * Conventions
 *   - Plain pointers and sizes only.  `trs_view.data` is a DEVICE address of
 *     element 0 of a storage buffer; shape/strides/offset are in elements and
 *     describe a (possibly broadcast, transposed, reversed, offset) view into
 *     it exactly like the reference's `shape`, `strides: Vec<isize>` and
 *     `offset: isize` fields (base.rs:159-164).
 *   - The caller owns every buffer.  Outputs are written through an output
 *     view; the output of an element-wise op must have the broadcast shape.
 *   - Calls are ordered on the given CUDA stream (`trs_stream`, a
 *     cudaStream_t; NULL is the legacy default stream) and return before the
 *     GPU work finishes, except where a comment says the call synchronises.
 *   - No call aborts the process.  Where the reference panics, the call
 *     returns a status and leaves a message (the reference's own panic text)
 *     for trs_last_error(); where the reference returns `None`, the call
 *     returns TRS_NONE.
 *   - Scratch memory that a call needs beyond its inputs and outputs comes
 *     from the device's stream-ordered memory pool (cudaMallocAsync /
 *     cudaFreeAsync on the call's stream).
 */
#ifndef TRS_H
#define TRS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TRS_MAX_DIMS 8
#define TRS_ABI_VERSION 1

typedef void* trs_stream;

/* Element types.  The reference's `Num` covers i16/i32/i64/i128/f32/f64
 * (src/lib.rs:69-94); this path serves f32 and f64 (the `Float` types,
 * src/lib.rs:110-141) and the i32/i64 tensors its own unit tests use. */
typedef enum trs_dtype {
  TRS_F32 = 0,
  TRS_F64 = 1,
  TRS_I32 = 2,
  TRS_I64 = 3
} trs_dtype;

typedef enum trs_status {
  TRS_OK = 0,
  TRS_NONE = 1,             /* the reference returns None (Option::None)          */
  TRS_ERR_SHAPE = 2,        /* shapes do not broadcast ("!!!Add: incompatible shapes!!!") */
  TRS_ERR_AXIS = 3,         /* "!!!Axis index out of range!!!" (base.rs:1052)     */
  TRS_ERR_EMPTY_AXIS = 4,   /* "!!!Cannot reduce an empty axis!!!" (base.rs:1513) */
  TRS_ERR_VIEW = 5,         /* a view reaches outside its storage, or bad rank    */
  TRS_ERR_DTYPE = 6,        /* dtype not served by this op, or dtypes disagree    */
  TRS_ERR_ALIAS = 7,        /* output overlaps an input through another layout    */
  TRS_ERR_OOM = 8,          /* scratch allocation failed                          */
  TRS_ERR_CUDA = 9,         /* a CUDA runtime call failed                         */
  TRS_ERR_NCCL = 10,        /* an NCCL call failed                                */
  TRS_ERR_TIMEOUT = 11,     /* a communicator did not come up / finish in time    */
  TRS_ERR_ARG = 12,         /* null pointer, unknown op code, bad count           */
  TRS_ERR_DIV_ZERO = 13,    /* integer division by zero (the reference panics)    */
  TRS_ERR_UNAVAILABLE = 14  /* NCCL could not be loaded                           */
} trs_status;

/* A strided view of a device buffer: the reference's Tensor metadata
 * (base.rs:159-164) plus the length of the storage it points into, which the
 * library uses to reject views that would read or write outside it. */
typedef struct trs_view {
  void* data;              /* device address of storage element 0              */
  int64_t storage_len;     /* number of elements in that storage               */
  int32_t dtype;           /* trs_dtype                                         */
  int32_t ndim;            /* 0..TRS_MAX_DIMS (0 = one element)                 */
  int64_t shape[TRS_MAX_DIMS];
  int64_t strides[TRS_MAX_DIMS]; /* elements; 0 = broadcast; may be negative    */
  int64_t offset;          /* elements                                          */
} trs_view;

/* A scalar operand or parameter.  `f` is read for f32/f64 tensors, `i` for
 * i32/i64 tensors. */
typedef struct trs_scalar {
  double f;
  int64_t i;
} trs_scalar;

/* Binary element-wise operators of binary_op (ops.rs:240-300). */
typedef enum trs_binop {
  TRS_ADD = 0,  /* add       ops.rs:303  (operator +) */
  TRS_SUB = 1,  /* sub       ops.rs:362  (operator -) */
  TRS_MUL = 2,  /* mul_elem  ops.rs:423  (operator &) */
  TRS_DIV = 3,  /* div       ops.rs:498  (operator /) */
  TRS_POW = 4   /* powf      ops.rs:487  (operator ^), f32/f64 only */
} trs_binop;

/* Unary maps.  Each one computes exactly what the cited reference code
 * computes, including the order of its roundings. */
typedef enum trs_unop {
  TRS_UN_NONE = 0,        /* identity (a strided copy: packed_data, base.rs:430) */
  TRS_UN_NEG = 1,         /* Neg, ops.rs:152-175 */
  TRS_UN_RELU = 2,        /* ReLU::forward: x & map(x > 0 ? 1 : 0), activation/relu.rs:32-42 */
  TRS_UN_SIGMOID = 3,     /* sigmoid_op two-branch form, autodiff/ops.rs:585-594 */
  TRS_UN_TANH = 4,        /* tanh_op: map(tanh), autodiff/ops.rs:547-548 */
  TRS_UN_ELU = 5,         /* ELU::forward, activation/elu.rs:43-64; p0 = alpha */
  TRS_UN_LEAKY_RELU = 6,  /* LeakyReLU::forward, activation/leaky_relu.rs:35-53; p0 = alpha */
  TRS_UN_SELU = 7,        /* SELU::forward, activation/selu.rs:48-71; p0 = alpha, p1 = lambda */
  TRS_UN_EXP = 8,         /* Tensor::scalar(E) ^ x = powf(E, x), activation/elu.rs:58-60 */
  TRS_UN_LN = 9,          /* log_op: map(ln), autodiff/ops.rs:162-164 */
  TRS_UN_ABS = 10,        /* abs_op: map(abs), autodiff/ops.rs:199-201 */
  TRS_UN_SIGN = 11,       /* Float::sign, src/lib.rs:151-159 */
  TRS_UN_CLAMP = 12,      /* clamp_op, autodiff/ops.rs:245-247; p0 = min, p1 = max */
  TRS_UN_ADD_SCALAR = 13, /* &t + s,  ops.rs:52-58 */
  TRS_UN_SUB_SCALAR = 14, /* &t - s,  ops.rs:87-93 */
  TRS_UN_RSUB_SCALAR = 15,/* s - &t,  ops.rs:124-131 */
  TRS_UN_MUL_SCALAR = 16, /* &t * s,  ops.rs:179-185 */
  TRS_UN_DIV_SCALAR = 17, /* &t / s,  ops.rs:214-220 */
  TRS_UN_POW_SCALAR = 18, /* x ^ s: powf(x, s), autodiff/impl_ops.rs:95-99 */
  TRS_UN_RPOW_SCALAR = 19 /* s ^ x: powf(s, x), activation/softmax.rs:59-61 with s = E */
} trs_unop;

/* A fused element-wise program over up to three inputs:
 *   v = in[0]
 *   v = op1(v, in[1])        when n_in >= 2
 *   v = op2(v, in[2])        when n_in == 3
 *   out = epilogue(v; p0, p1)
 * Every stage rounds to the element type, as the chain of separate reference
 * calls does (e.g. `&(&a & &b) + &c`, or ReLU::forward over `&(&x & &s) + &b`),
 * so a fused program gives the same bits as the unfused chain. */
typedef struct trs_ew_program {
  int32_t n_in;       /* 1..3 */
  int32_t op1;        /* trs_binop, used when n_in >= 2 */
  int32_t op2;        /* trs_binop, used when n_in == 3 */
  int32_t epilogue;   /* trs_unop */
  trs_scalar p0;      /* epilogue parameter 0 */
  trs_scalar p1;      /* epilogue parameter 1 */
} trs_ew_program;

/* ------------------------------------------------------------------ */
/* Library                                                             */
/* ------------------------------------------------------------------ */

/* ABI version (TRS_ABI_VERSION). */
int32_t trs_abi_version(void);

/* Text of the last failure on the calling thread (the reference's panic
 * message where there is one).  Returns the full length; copies at most
 * len-1 bytes and a NUL. */
size_t trs_last_error(char* buf, size_t len);

/* Static description of a status code. */
const char* trs_status_string(int32_t status);

/* Number of kernels this library has launched in this process (all devices).
 * Used by benchmarks to report how many GPU launches a timed region made. */
uint64_t trs_launch_count(void);

/* Number of scratch allocations (per-block partials, flags, per-rank
 * buffers) this library has made from its stream-ordered pool in this
 * process (all devices).  Used by tests to show that a call allocated
 * nothing. */
uint64_t trs_scratch_alloc_count(void);

/* Reads and clears the current device's async-error word.  A kernel that
 * waits gives up after a bounded number of polls, sets a bit of this word and
 * returns instead of hanging: bit 0 (1) when it waited on its own bulk
 * copies, bit 1 (2) when a sharded sum waited on a peer rank's partial;
 * *code receives the word (0 = none).  Synchronises the device.  Returns
 * TRS_ERR_TIMEOUT when the word was set. */
trs_status trs_async_error(int32_t* code);

/* ------------------------------------------------------------------ */
/* Host planning (no GPU needed)                                        */
/* ------------------------------------------------------------------ */

/* Broadcast two shapes the way broadcast_shape does (ops.rs:27-45).
 * Writes the result rank to *out_ndim and the shape to out_shape
 * (TRS_MAX_DIMS entries).  Returns TRS_ERR_SHAPE if they do not broadcast. */
trs_status trs_broadcast_shape(const int64_t* a, int32_t a_ndim,
                               const int64_t* b, int32_t b_ndim,
                               int64_t* out_shape, int32_t* out_ndim);

/* Describe the launch plan of trs_elementwise for the given views without
 * running it: the folded rank, folded shape, folded strides of the output
 * (slot 0) and of each input (slots 1..n_in), and the kernel variant chosen
 * (0 = contiguous-inner vector kernel, 1 = tiled transpose kernel,
 * 2 = generic strided kernel).  `strides_out` holds 4 x TRS_MAX_DIMS
 * entries.  Used by host-side tests of the view folding. */
trs_status trs_plan_elementwise(const trs_ew_program* prog, const trs_view* in,
                                const trs_view* out, int32_t* variant,
                                int32_t* folded_ndim, int64_t* folded_shape,
                                int64_t* strides_out, int32_t* vector_width);

/* ------------------------------------------------------------------ */
/* Element-wise (K-EW)                                                  */
/* ------------------------------------------------------------------ */

/* binary_op (ops.rs:240-300) for add/sub/mul_elem/div/powf: out = a op b
 * with numpy-style right-aligned broadcasting (broadcast_to, base.rs:556-599).
 * `out` must have the broadcast shape. */
trs_status trs_binary(int32_t op, const trs_view* a, const trs_view* b,
                      trs_view* out, trs_stream stream);

/* One unary map (Tensor::map, base.rs:1708-1716, with the closures the
 * reference's activations and scalar operators use). `params` may be NULL
 * when the op takes none; otherwise it points at two entries (p0, p1). */
trs_status trs_unary(int32_t op, const trs_view* x, const trs_scalar* params,
                     trs_view* out, trs_stream stream);

/* A fused program (see trs_ew_program) over n_in = prog->n_in inputs. */
trs_status trs_elementwise(const trs_ew_program* prog, const trs_view* in,
                           trs_view* out, trs_stream stream);

/* A fused program whose output is also summed: `out` receives the element-wise
 * result and `sum_out` (a one-element f32/f64 view of the same dtype) receives
 * sum() of it (base.rs:1024-1030), accumulated in f64 and rounded once.
 * `out` may be NULL to skip writing the element-wise result. */
trs_status trs_elementwise_sum(const trs_ew_program* prog, const trs_view* in,
                               trs_view* out, trs_view* sum_out,
                               trs_stream stream);

/* The chain `y = prog(in); y.sum_axis(last); y.sum()` (binary_op,
 * ops.rs:240-300; sum_axis, base.rs:1051-1107; sum, base.rs:1024-1030) in
 * one pass: `out` receives y (shape: the inputs' broadcast shape, rank >= 1),
 * `row_sums` its sums along the last axis (the reduced shape, with or without
 * the axis kept as size 1) and `total` (one element) the sum of all of y.
 * Either sum may be NULL, not both.  Sums accumulate in f64 (wrapping
 * integers) and round once, as trs_sum_axis and trs_sum do.  A contiguous
 * `out` of at least 256 rows whose inputs run along the last axis with unit
 * stride (or are constant along it) takes one kernel plus a one-CTA fold;
 * other layouts run the three passes.  The sums may overlap no other
 * operand (TRS_ERR_ALIAS). */
trs_status trs_elementwise_row_sums(const trs_ew_program* prog, const trs_view* in,
                                    trs_view* out, trs_view* row_sums, trs_view* total,
                                    trs_stream stream);

/* packed_data / get_data / Clone (base.rs:430-434, 252, 1934-1945):
 * copy any view into the layout of `out` (normally contiguous). */
trs_status trs_pack(const trs_view* x, trs_view* out, trs_stream stream);

/* ------------------------------------------------------------------ */
/* Reductions (K-RED)                                                   */
/* ------------------------------------------------------------------ */

/* sum (base.rs:1024-1030): every element into a one-element view.
 * Floats accumulate in f64 and round once; integers wrap like the
 * reference's release build. */
trs_status trs_sum(const trs_view* x, trs_view* out, trs_stream stream);

/* sum() of x, like trs_sum, for callers that cannot allocate device memory
 * while they run (a host that owns all device memory through its own arena,
 * or a code path that must not enter the CUDA allocator).  No counterpart in
 * the reference: it exists for those callers only.
 *
 * It calls no cudaMalloc, cudaFree or stream-ordered allocation: the
 * per-block partial sums live in a static device array of 64 KiB (8192
 * partials) that every GPU loading the library holds until the process exits.
 * A sum that would need more partials than that is rejected with TRS_ERR_ARG.
 * The first call on a device looks the array's address up (with that device
 * current), which also loads the library's device code on that device if
 * nothing has yet (CUDA loads modules lazily) and so commits the array's
 * memory then: make that first call at start-up, before the host's arena
 * reserves the device's memory and before any stream capture.  All calls
 * share the array and every call rewrites the partials it reads, but calls
 * that overlap on the GPU (on different streams) race on it. */
trs_status trs_sum_noalloc(const trs_view* x, trs_view* out, trs_stream stream);

/* sum_axis (base.rs:1051-1107) with keepdim = 0, sum_axis_keepdim
 * (base.rs:1534-1594) with keepdim = 1. */
trs_status trs_sum_axis(const trs_view* x, int32_t axis, int32_t keepdim,
                        trs_view* out, trs_stream stream);

/* The mean its callers build: sum_axis(_keepdim) divided by the axis length
 * with an IEEE division in the element type (nn/layer_norm.rs:26).
 * f32/f64 only. */
trs_status trs_mean_axis(const trs_view* x, int32_t axis, int32_t keepdim,
                         trs_view* out, trs_stream stream);

/* max_axis (base.rs:1396-1436): strict `>` running maximum seeded with the
 * first element, so ties keep the first value and a NaN only wins at index 0. */
trs_status trs_max_axis(const trs_view* x, int32_t axis, trs_view* out,
                        trs_stream stream);

/* argmax_axis (base.rs:1458-1505): the index that max_axis takes its value
 * from; `out` is an i64 view (the reference returns Vec<usize>). */
trs_status trs_argmax_axis(const trs_view* x, int32_t axis, trs_view* out,
                           trs_stream stream);

/* reduce_broadcast_grad / reduce_to_shape (base.rs:1617-1686): sum `g` down
 * to `target` (leading axes summed away, axes the target holds as 1 summed
 * with keepdim).  Returns TRS_NONE when the reference returns None.  `out`
 * has the target shape. */
trs_status trs_reduce_broadcast_grad(const trs_view* g, const int64_t* target,
                                     int32_t target_ndim, trs_view* out,
                                     trs_stream stream);

/* The un-broadcast of a Mul backward (autodiff/core.rs:206-227) in one pass:
 *   out = reduce_broadcast_grad(g & gate_mask & mul, target)
 * where gate_mask = map(v > 0 ? 1 : 0) of `gate` (the mask ReLU builds,
 * activation/relu.rs:36-39) and either of `gate` / `mul` may be NULL.  Each
 * product is rounded like the separate `&` calls; the sum accumulates in f64. */
trs_status trs_sum_to_shape_fused(const trs_view* g, const trs_view* gate,
                                  const trs_view* mul, const int64_t* target,
                                  int32_t target_ndim, trs_view* out,
                                  trs_stream stream);

/* The backward of ReLU(x & scale + bias) for the scale and bias gradients
 * (NCHW activations with [1,C,1,1] scale and bias): with z = (x & s) + b and
 * m = map(z > 0 ? 1 : 0),
 *   grad_bias  = reduce_broadcast_grad(g & m, [1,C,1,1])
 *   grad_scale = reduce_broadcast_grad((g & m) & x, [1,C,1,1])
 * (autodiff/core.rs:173-227 applied to activation/relu.rs:32-42).  The mask
 * is recomputed from x, scale and bias instead of being read.  Either output
 * may be NULL. */
trs_status trs_affine_relu_backward(const trs_view* g, const trs_view* x,
                                    const trs_view* scale, const trs_view* bias,
                                    trs_view* grad_scale, trs_view* grad_bias,
                                    trs_stream stream);

/* SoftMax::forward over the last axis (activation/softmax.rs:42-68):
 * e = powf(E, x - max_axis(x)), out = e / sum_axis_keepdim(e).  f32/f64. */
trs_status trs_softmax_lastdim(const trs_view* x, trs_view* out,
                               trs_stream stream);

/* ------------------------------------------------------------------ */
/* Callers of the path: LayerNorm and the optimiser steps               */
/* ------------------------------------------------------------------ */

/* LayerNorm::forward over the last axis (nn/layer_norm.rs:20-33) in one
 * kernel: mean = sum_axis_keepdim(x) / F, sq = (x - mean) ^ 2,
 * var = sum_axis_keepdim(sq) / F, denom = (var + eps) ^ 0.5,
 * out = ((x - mean) / denom) & gamma + beta, with F the last dimension and
 * gamma / beta of F elements each ([1, F] in the reference).  The sums
 * accumulate in f64 and round once; every other step rounds as the separate
 * reference calls do.  f32/f64. */
trs_status trs_layer_norm_lastdim(const trs_view* x, const trs_view* gamma,
                                  const trs_view* beta, double eps,
                                  trs_view* out, trs_stream stream);

/* One SGD step in place (optim/sgd.rs:29-37): param = param - grad * lr.
 * `param` and `grad` contiguous, of one shape and dtype (f32/f64). */
trs_status trs_sgd_step(trs_view* param, const trs_view* grad, double lr,
                        trs_stream stream);

/* One RMSprop step in place (optim/rmsprop.rs:30-46):
 * v = v * alpha + (grad & grad) * (1 - alpha);
 * param = param - (grad * lr) / map(v, sqrt(x) + eps).
 * The reference's defaults are alpha = 0.99, eps = 1e-8.  Contiguous views
 * of one shape. */
trs_status trs_rmsprop_step(trs_view* param, const trs_view* grad, trs_view* v,
                            double lr, double alpha, double eps,
                            trs_stream stream);

/* One Adam step in place (optim/adam.rs:119-144) for step number t >= 1:
 * m = m * beta1 + grad * (1 - beta1); v = v * beta2 + (grad & grad) * (1 - beta2);
 * m_hat = m / (1 - beta1^t); v_hat = v / (1 - beta2^t);
 * param = param - (m_hat * lr) / map(v_hat, sqrt(x) + eps).
 * beta^t is powf in the element type, computed on the host as the reference
 * does; the reference's defaults are beta1 = 0.9, beta2 = 0.999, eps = 1e-8.
 * Contiguous views of one shape. */
trs_status trs_adam_step(trs_view* param, const trs_view* grad, trs_view* m,
                         trs_view* v, double lr, double beta1, double beta2,
                         double eps, int64_t t, trs_stream stream);

/* MaxPool2d::forward (nn/pool.rs:137-144), replacing its chain
 * reshape -> unfold_2d (linalg/tensor/conv.rs:360-418) -> max_axis(1): x is
 * [N, C, H, W] (any strides), windows kh x kw at strides sh x sw, no padding;
 * `out` is [N, C, (H - kh) / sh + 1, (W - kw) / sw + 1].  Each output is the
 * window's first element replaced only by a strictly greater one, in row-major
 * window order (so a NaN first element stays).  f32/f64.
 * Errors: x not 4-D, out of another shape, or H < kh / W < kw: TRS_ERR_SHAPE;
 * a stride of 0: TRS_ERR_ARG; kh * kw == 0: TRS_ERR_EMPTY_AXIS; out
 * overlapping x: TRS_ERR_ALIAS. */
trs_status trs_max_pool2d(const trs_view* x, int64_t kh, int64_t kw,
                          int64_t sh, int64_t sw, trs_view* out,
                          trs_stream stream);

/* AvgPool2d::forward (nn/pool.rs:223-233): unfold_2d -> sum_axis(1) ->
 * divided by kh * kw.  Each window is summed in the element type in
 * row-major order from 0, as sum_axis does (base.rs:1051-1107), then divided
 * once, so the result is the reference's bit for bit.  Shapes and errors as
 * trs_max_pool2d, except that an empty window (kh * kw == 0) gives 0 / 0. */
trs_status trs_avg_pool2d(const trs_view* x, int64_t kh, int64_t kw,
                          int64_t sh, int64_t sw, trs_view* out,
                          trs_stream stream);

/* The gradient MaxPool2d passes back to its input: max_axis's backward
 * (autodiff/core.rs:352-375: each window's gradient to the first of its
 * largest elements, argmax_axis base.rs:1458-1505), then unfold's backward
 * fold_2d (conv.rs:434-488: a pixel sums, from 0 and in window order, the
 * gradients of the windows that read it).  grad_out is [N, C, OH, OW] and
 * grad_x [N, C, H, W]; with accumulate != 0, grad_x = grad_x + that sum (the
 * accumulation `current + grad` of autodiff/traits.rs:141-150), else
 * grad_x = the sum.  grad_x may not overlap x or grad_out (TRS_ERR_ALIAS). */
trs_status trs_max_pool2d_backward(const trs_view* x, const trs_view* grad_out,
                                   int64_t kh, int64_t kw, int64_t sh,
                                   int64_t sw, int32_t accumulate,
                                   trs_view* grad_x, trs_stream stream);

/* ------------------------------------------------------------------ */
/* Contraction and the im2col pair (callers of the path: Linear,       */
/* Conv2d, MultiHeadAttention)                                          */
/* ------------------------------------------------------------------ */

/* Tensor::matmul (linalg/tensor/base.rs:896-1013): a [..., M, K] times
 * b [..., K, N] into out [batch..., M, N], where the batch dimensions of a
 * and b broadcast against each other (a dimension of 1 is reused).  Both
 * operands are read through their strides.  Every output is the reference's
 * chain acc = acc + a[i, k] * b[k, j] over k = 0 .. K-1 from acc = 0, each
 * step rounded once in the element type (integers wrap), so results are
 * bit-identical to the reference's.  Panics of the reference map to
 * TRS_ERR_SHAPE with its text ("matmul: both tensors must be at least 2D",
 * "matmul: inner dimensions must match (A.shape[-1] == B.shape[-2])",
 * "matmul: batch shapes not broadcastable"); out may not overlap a or b
 * (TRS_ERR_ALIAS). */
trs_status trs_matmul(const trs_view* a, const trs_view* b, trs_view* out,
                      trs_stream stream);

/* Tensor::matmul (linalg/tensor/base.rs:896-1013) for f32 on the tensor cores
 * (tcgen05, TF32 inputs): shapes, broadcasting, views and panics as
 * trs_matmul, but not bit-identical.  Each operand is split into two TF32
 * parts (hi = x with its 13 low mantissa bits cleared, lo = x - hi) and every
 * product taken as hi*hi + hi*lo + lo*hi, accumulated in f32 by the tensor
 * cores in their own order: finite results are within about the rounding
 * error of an f32 sum of the products (the tests hold them to
 * 1e-5 * sum_k |a_ik b_kj| of the reference's).  Infinities and NaNs
 * propagate, without the reference's exact special-value rules.  Scratch for
 * the split operands comes from the stream-ordered pool. */
trs_status trs_matmul_tf32x3(const trs_view* a, const trs_view* b, trs_view* out,
                             trs_stream stream);

/* Tensor::unfold_2d (linalg/tensor/conv.rs:360-418): every (kh, kw) window of
 * x [B, C, H, W] (stride (sh, sw), zero padding (ph, pw) on each side) as one
 * row of out [B * OH * OW, C * kh * kw], rows in (b, oh, ow) order, each row
 * in (c, i, j) order; OH = (H + 2 ph - kh) / sh + 1, likewise OW.  Panics of
 * unfold_dims (conv.rs:490-510) map to TRS_ERR_SHAPE / TRS_ERR_ARG. */
trs_status trs_unfold_2d(const trs_view* x, int64_t kh, int64_t kw, int64_t sh,
                         int64_t sw, int64_t ph, int64_t pw, trs_view* out,
                         trs_stream stream);

/* Tensor::fold_2d (linalg/tensor/conv.rs:434-488): the rows of an unfold,
 * cols [B * OH * OW, C * kh * kw], added back into out [B, C, H, W] (its
 * shape is the reference's output_shape) wherever windows overlap; each
 * pixel adds its windows' values in increasing (oh, ow) order from +0, as the
 * reference's loop does, so results are bit-identical.  A cols shape that is
 * not an unfold of out is TRS_ERR_SHAPE with the reference's text. */
trs_status trs_fold_2d(const trs_view* cols, int64_t kh, int64_t kw, int64_t sh,
                       int64_t sw, int64_t ph, int64_t pw, trs_view* out,
                       trs_stream stream);

/* ------------------------------------------------------------------ */
/* Seeded synthetic inputs                                              */
/* ------------------------------------------------------------------ */

/* Fill a view with lo + (hi - lo) * u, u = (splitmix64(seed, first + i) >> 40)
 * * 2^-24 for the i-th element in row-major order of the view, computed in
 * f64 and rounded once.  `first` lets a shard generate exactly its rows of a
 * larger tensor.  With (lo, hi) = (-1, 1) every value is exact in f32. */
trs_status trs_fill_uniform(trs_view* out, uint64_t seed, uint64_t first, double lo,
                            double hi, trs_stream stream);

/* Fill a view with N(0,1) samples (Box-Muller over the splitmix64 uniforms
 * 2(first+i) and 2(first+i)+1, evaluated in f64 and rounded once).  Not
 * bit-identical to a host generator; meant for device-resident benchmark
 * inputs. */
trs_status trs_fill_normal(trs_view* out, uint64_t seed, uint64_t first, trs_stream stream);

/* ------------------------------------------------------------------ */
/* Memory and streams, for hosts that do not link the CUDA runtime       */
/* ------------------------------------------------------------------ */

trs_status trs_set_device(int32_t device);
trs_status trs_malloc(void** ptr, size_t bytes);
trs_status trs_free(void* ptr);
trs_status trs_memcpy_htod(void* dst, const void* src, size_t bytes, trs_stream stream);
trs_status trs_memcpy_dtoh(void* dst, const void* src, size_t bytes, trs_stream stream);
trs_status trs_stream_synchronize(trs_stream stream);

/* ------------------------------------------------------------------ */
/* Several GPUs: leading-dimension shards, NCCL over NVLink              */
/* ------------------------------------------------------------------ */

typedef struct trs_comm trs_comm;

/* 128-byte NCCL unique id, created on one rank and passed to all. */
trs_status trs_comm_unique_id(uint8_t id[128]);

/* Join a communicator of nranks ranks as `rank` on the current device.  The
 * communicator is created non-blocking and polled; if it is not up within
 * timeout_ms the attempt is aborted and TRS_ERR_TIMEOUT returned. */
trs_status trs_comm_init_rank(const uint8_t id[128], int32_t nranks,
                              int32_t rank, int32_t timeout_ms,
                              trs_comm** comm);
trs_status trs_comm_destroy(trs_comm* comm);
trs_status trs_comm_abort(trs_comm* comm);

/* *active = 1 when this communicator's sharded sums combine over NVLink peer
 * memory (every rank mapped every peer's slot buffer at creation), 0 when
 * they combine with ncclAllReduce. */
trs_status trs_comm_peer_exchange(const trs_comm* comm, int32_t* active);

/* sum() of a tensor whose leading dimension is split across the ranks:
 * every rank passes its shard; every rank receives the global sum (f64
 * partials combined in rank order, rounded once).  The combine is done by the
 * kernel that folds this rank's partials: it writes its accumulator into
 * every peer's slot buffer over NVLink and reads theirs (mapped at
 * communicator creation with CUDA IPC), so no collective is launched; where
 * that mapping could not be made on every rank, an ncclAllReduce combines
 * instead.  Calls on one communicator must be made by every rank in the same
 * order and, per rank, on one stream (their slots are reused call after
 * call).  A peer that does not make the call leaves this rank's kernel
 * waiting about 2 s, after which it gives up: the sum is NaN (0 for
 * integers) and trs_async_error() reports bit 1. */
trs_status trs_sharded_sum(trs_comm* comm, const trs_view* shard,
                           trs_view* out, trs_stream stream);

/* trs_elementwise_sum over leading-dimension shards: each rank writes its
 * shard of the element-wise result and every rank receives the global sum,
 * combined as in trs_sharded_sum. */
trs_status trs_sharded_elementwise_sum(trs_comm* comm,
                                       const trs_ew_program* prog,
                                       const trs_view* in, trs_view* out,
                                       trs_view* sum_out, trs_stream stream);

/* sum_axis(0) / max_axis(0) / argmax_axis(0) of a tensor split on axis 0:
 * each rank reduces its rows into partials (sum: f64 / wrapping accumulators;
 * max: value-and-index records), and every rank combines all ranks' partials
 * in rank order (sums rounded once; ties keep the lowest global index, as the
 * reference's scan does).  Where every rank mapped every peer's exchange
 * buffer (trs_comm_peer_exchange) and the partials fit 8 MiB, the combine
 * reads the peers' partials over NVLink in one kernel after each rank has
 * published its own (no collective for the sum; max/argmax exchange their row
 * counts first, for the global indices and the empty-axis check); otherwise
 * through an NCCL all-reduce / all-gather.  A peer that does not make the call
 * leaves the combine waiting about 2 s: the results are then NaN (0 for
 * integers, -1 for argmax) and trs_async_error() reports bit 1.  `out` is the
 * full [rest...] result on every rank; argmax writes global indices as i64. */
trs_status trs_sharded_sum_axis0(trs_comm* comm, const trs_view* shard,
                                 trs_view* out, trs_stream stream);
trs_status trs_sharded_max_axis0(trs_comm* comm, const trs_view* shard,
                                 trs_view* out, trs_stream stream);
trs_status trs_sharded_argmax_axis0(trs_comm* comm, const trs_view* shard,
                                    trs_view* out, trs_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* TRS_H */
