/*
 * nnrcu.h - C ABI of the B200 (sm_100a) backend for nnr's conv/GEMM hot path.
 *
 * The entry points are what nnr's backend_t::CUDA operators (a new
 * src/backend/cuda/ beside src/backend/cpu/) call from operator_t::reshape()
 * and operator_t::exec(). Plain pointers and sizes only; every function
 * returns NNRCU_OK (0) or a negative NNRCU_ERR_* code, mirroring nnr's
 * bool-return convention (reference: src/nnr.h:331-461, operator_t), and
 * nnrcu_last_error() returns the message of the last failure on the calling
 * thread.
 *
 * Object lifecycle, matching operator_t:
 *   nnrcu_*_create   <-> operator_t::reshape()  (shape checks, weight packing
 *                        and upload, requant constants; once per shape)
 *   nnrcu_*_run      <-> operator_t::exec()     (enqueue on a stream; no
 *                        allocation, no host synchronisation)
 *   nnrcu_op_destroy <-> operator_t::~operator_t() (frees device buffers)
 *   nnrcu_op_workspace_size <-> operator_t::workspace_size(), but for a
 *                        device workspace that the caller's device arena
 *                        provides to *_run.
 *   nnrcu_op_num_ops <-> operator_t::num_ops() (2 * MACs).
 *
 * Tensor pointers passed to *_run are device pointers. Activations may be
 * NCHW (nnr's default) or NHWC (nnr's memory_layout_t::NHWC, the layout the
 * device prefers); see nnrcu_conv_desc.
 */
#ifndef NNRCU_H
#define NNRCU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NNRCU_OK 0
#define NNRCU_ERR_INVALID (-1)     /* bad argument or shape */
#define NNRCU_ERR_UNSUPPORTED (-2) /* valid ONNX, not handled on the device (caller's registry may decline) */
#define NNRCU_ERR_CUDA (-3)        /* CUDA runtime / driver error */
#define NNRCU_ERR_DEVICE (-4)      /* a kernel reported a failure through the device status word */
#define NNRCU_ERR_NOMEM (-5)       /* device allocation failed */

#define NNRCU_LAYOUT_NCHW 0
#define NNRCU_LAYOUT_NHWC 1

/* Requantisation formula of QLinearConv. nnr's x64 CPU path uses a different
 * fp32 operation order per kernel; bit-exact parity needs the same one.
 *   AUTO: the one nnr's dispatch would pick for this shape on an AVX-512
 *         VNNI host (reference: src/backend/cpu/QLinearConv.cpp:1337-1351):
 *         R3 for the small-IC stem with NCHW input, R1 when the output is
 *         NCHW with oH*oW <= 256, R2 otherwise.
 *   R1: exec_direct_int8 (QLinearConv.cpp:616-646)
 *   R2: packed NR48 JIT epilogue (backend/x64/jit_conv_int8_ukernel.cpp:950-965)
 *   R3: first-layer kernel (backend/x64/conv_first_layer_int8_avx512.h:262-270) */
#define NNRCU_RQ_AUTO 0
#define NNRCU_RQ_R1 1
#define NNRCU_RQ_R2 2
#define NNRCU_RQ_R3 3

/* Fused post-op of Conv/Gemm/MatMul: nnr sets operator_t::post_fn to the
 * consumer's fusable_apply (graph_optimizer/fuse_post_ops.cpp:69-71); the
 * device equivalent is this enum plus two parameters. */
#define NNRCU_POST_NONE 0
#define NNRCU_POST_RELU 1
#define NNRCU_POST_CLIP 2      /* a = min, b = max   (backend/cpu/Clip.cpp:20-40) */
#define NNRCU_POST_HARDSWISH 3 /* x*clamp(x/6+0.5,0,1) (backend/cpu/HardSwish.cpp:18-35) */
#define NNRCU_POST_SIGMOID 4
#define NNRCU_POST_LEAKYRELU 5 /* a = alpha */
#define NNRCU_POST_TANH 6

typedef struct nnrcu_op nnrcu_op; /* opaque: one prepared operator instance */

/* Shape and attributes of a 2-D convolution (ONNX Conv / QLinearConv).
 * Weights are ONNX OIHW [oc, c/group, kh, kw]. */
typedef struct nnrcu_conv_desc {
  int n, c, h, w;        /* input dims (logical NCHW) */
  int oc, kh, kw;        /* output channels, kernel size */
  int group;             /* 1, or c == oc == group for depthwise */
  int stride_h, stride_w;
  int pad_top, pad_left, pad_bottom, pad_right; /* ONNX pads after auto_pad resolution */
  int dil_h, dil_w;
  int in_layout, out_layout; /* NNRCU_LAYOUT_* */
  int post_op;               /* NNRCU_POST_*; for QLinearConv any non-zero value means a fused
                                activation exists (qmin = max(lo, y_zp), QLinearConv.cpp:419) */
  float post_a, post_b;
  int requant;               /* NNRCU_RQ_* (QLinearConv only) */
} nnrcu_conv_desc;

/* ---------------------------------------------------------------- runtime */
int nnrcu_init(int device);             /* select + initialise a device on this thread */
int nnrcu_last_error(char* buf, size_t len);
/* Reads and clears the device status word that kernels set instead of
 * trapping (e.g. a pipeline wait that ran out of time). 0 = clean. */
int nnrcu_device_status(int* status_out);
int nnrcu_stream_create(void** stream);
int nnrcu_stream_destroy(void* stream);
int nnrcu_stream_sync(void* stream);
int nnrcu_malloc(void** ptr, size_t bytes);
int nnrcu_free(void* ptr);
int nnrcu_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int nnrcu_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int nnrcu_memset(void* dst, int value, size_t bytes, void* stream);
/* Page-lock an existing host buffer (a graph input or output that nnr owns)
 * so that copies from and to it run at the link's rate and asynchronously;
 * a buffer already registered is accepted. nnrcu_host_unregister undoes it. */
int nnrcu_host_register(void* ptr, size_t bytes);
int nnrcu_host_unregister(void* ptr);
/* Stream capture of a run loop into one CUDA graph (replaces nnr's
 * exec_steps loop, src/nnr.cpp:908-1051, for a fixed batch). */
int nnrcu_graph_begin(void* stream);
int nnrcu_graph_end(void* stream, void** graph_exec);
int nnrcu_graph_launch(void* graph_exec, void* stream);
int nnrcu_graph_destroy(void* graph_exec);

/* ---------------------------------------------------------------- operators (common) */
int nnrcu_op_workspace_size(const nnrcu_op* op, size_t* bytes);
int nnrcu_op_num_ops(const nnrcu_op* op, int64_t* ops);
int nnrcu_op_destroy(nnrcu_op* op);

/* ---------------------------------------------------------------- QLinearConv (u8 x, s8 w, u8 y)
 * Replaces QLinearConv_operator::reshape/exec (backend/cpu/QLinearConv_reshape.h:18-340,
 * backend/cpu/QLinearConv.cpp:1354-1368). w_scale has 1 or oc entries; w_zp has 0, 1 or
 * oc entries and must be all zero (nnr's VNNI paths require symmetric weights);
 * bias may be NULL. */
int nnrcu_qlinearconv_create(const nnrcu_conv_desc* desc, const int8_t* w_host, const float* w_scale,
                             int n_w_scale, const int8_t* w_zp, int n_w_zp, const int32_t* bias_host,
                             float x_scale, uint8_t x_zp, float y_scale, uint8_t y_zp, nnrcu_op** op);
int nnrcu_qlinearconv_run(nnrcu_op* op, const uint8_t* x, uint8_t* y, void* workspace, void* stream);
/* QuantizeLinear(x, x_scale, x_zp) followed by QLinearConv in one call: x is
 * fp32 in the op's input layout, quantised per tensor with QuantizeLinear's
 * float sequence (backend/cpu/QuantizeLinear.cpp:128-160: the 16-wide body
 * rne(x * (1/scale)) + zp, the scalar tail nearbyint(x / scale) + zp) inside
 * the op's input reorder, so the u8 image never reaches HBM. Results equal
 * nnrcu_quantize_linear_u8 then nnrcu_qlinearconv_run. Space-to-depth ops only
 * (stride 2 over at most 4 channels: the stem); others return
 * NNRCU_ERR_UNSUPPORTED. */
int nnrcu_qlinearconv_run_quantize(nnrcu_op* op, const float* x, float x_scale, uint8_t x_zp, uint8_t* y,
                                   void* workspace, void* stream);

/* QLinearConv followed by QLinearAdd(conv_out, residual) in one kernel: the
 * conv output is requantised to u8 exactly as above, then combined with the
 * u8 residual (same NHWC shape, scale res_scale, zero point res_zp) into y
 * (out_scale, out_zp) with QLinearAdd's float sequence
 * (backend/cpu/QLinearAdd.cpp:46-104). Results equal the two unfused
 * operators; the conv output never reaches HBM. NHWC output only. (The
 * reference's binary post-op fusion is unused, fuse_post_ops.cpp:67; this
 * is its device form.) */
int nnrcu_qlinearconv_run_add(nnrcu_op* op, const uint8_t* x, const uint8_t* residual, float res_scale,
                              uint8_t res_zp, float out_scale, uint8_t out_zp, uint8_t* y, void* workspace,
                              void* stream);
/* Padded activations between two QLinearConvs (a device-executor layout
 * choice with no counterpart in nnr, whose convs pad inside their own
 * kernels). Some convs (stride-1 spatial kernels over 64/128-byte channel
 * strides) read an x_zp-bordered copy of their NHWC input, made in their
 * workspace on every run; _input_padding reports that border (top, left,
 * bottom, right; zeros when the op reads its input as is). _set_padded_io
 * then lets a producer write straight into such a buffer and the consumer
 * skip the copy:
 *   in_padded = 1: x passed to nnrcu_qlinearconv_run is already
 *     [n][h+top+bottom][w+left+right][c] with every border byte = x_zp
 *     (no workspace is used);
 *   out_* > 0: nnrcu_qlinearconv_run writes y into the interior of
 *     [n][oh+top+bottom][ow+left+right][oc] (NHWC, oc % 16 == 0) and leaves
 *     the border alone (the caller fills it once with the consumer's x_zp).
 * Results are unchanged. */
int nnrcu_qlinearconv_input_padding(const nnrcu_op* op, int* pads);
int nnrcu_qlinearconv_set_padded_io(nnrcu_op* op, int in_padded, int out_top, int out_left, int out_bottom,
                                    int out_right);

/* ---------------------------------------------------------------- QLinearMatMul (u8 a, s8 b, u8 y)
 * Replaces QLinearMatMul_operator (backend/cpu/QLinearMatMul.cpp:33-232) for a 2-D B
 * initializer [k, n] (prepacked once, as nnr does when B is constant, :73-92); a is
 * [m, k] row-major (leading batch dims folded into m). Requant R4 (:188-198). */
int nnrcu_qlinearmatmul_create(int m, int k, int n, float a_scale, uint8_t a_zp, const int8_t* b_host,
                               float b_scale, int8_t b_zp, float y_scale, uint8_t y_zp, nnrcu_op** op);
int nnrcu_qlinearmatmul_run(nnrcu_op* op, const uint8_t* a, uint8_t* y, void* workspace, void* stream);

/* QLinearMatMul that allocates no device memory. No counterpart in the
 * reference: nnr runs on the CPU and has no device allocations to avoid.
 * For callers that cannot call cudaMalloc when they run an operator (device
 * memory reserved up front by another allocator, a policy of no allocation
 * after start-up). a u8 [m,k], b s8 [k,n] (raw ONNX layout) and y u8 [m,n]
 * are device pointers the caller owns; k must be a multiple of 16 and a
 * 16-byte aligned. Everything derived from b (transposed tiles, zero-point
 * sums) goes to one static device array of NNRCU_NOALLOC_SCRATCH_BYTES per
 * device, held until the process exits; calls needing more
 * (round_up(n,256)*round_up(k,128) + 4n (+ 4m when b_zp != 0) bytes, each
 * rounded to 256) fail with NNRCU_ERR_INVALID. The first call on a device
 * looks up the array's device address, so make that first call before any
 * stream capture. Calls share the array: calls that overlap on the GPU race
 * and must be serialised by the caller. A non-NULL stream must belong to the
 * current device (checked). Every error is returned before anything is
 * queued on the stream. Same requant (R4) and results as
 * nnrcu_qlinearmatmul_create/_run. */
#define NNRCU_NOALLOC_SCRATCH_BYTES (8u << 20)
int nnrcu_qlinearmatmul_noalloc(const uint8_t* a, const int8_t* b, uint8_t* y, int m, int k, int n, float a_scale,
                                uint8_t a_zp, float b_scale, int8_t b_zp, float y_scale, uint8_t y_zp,
                                void* stream);

/* ---------------------------------------------------------------- fp32 Conv (Conv+BN folded + post-op)
 * Replaces Conv_operator::reshape/exec<float> (backend/cpu/Conv_reshape.h:17-380,
 * backend/cpu/Conv_exec.h:1163-1192). Dense convs run on the tensor cores as
 * split-bf16 (3 products, fp32 accumulation); depthwise (group == c == oc) on
 * CUDA cores. bias may be NULL. */
int nnrcu_conv_f32_create(const nnrcu_conv_desc* desc, const float* w_host, const float* bias_host,
                          nnrcu_op** op);
/* residual (may be NULL) has y's shape and layout and is added after the post-op
 * (an unfused Conv -> Add, binary_math.cpp:57-77). */
int nnrcu_conv_f32_run(nnrcu_op* op, const float* x, float* y, const float* residual, void* workspace,
                       void* stream);

/* Depthwise -> 1x1 chains without the fp32 round trip. A dense fp32 Conv runs
 * on the tensor cores from two bf16 planes of its input (hi = bf16(x),
 * lo = bf16(x - hi), NHWC with a padded channel stride cs), which
 * nnrcu_conv_f32_run makes with a split pass over x. When x is the output of
 * an fp32 depthwise Conv with no other consumer (MobileNet's depthwise ->
 * projection pairs, Conv_depthwise.h:11 feeding Conv_exec.h:760-829), the
 * depthwise conv can write those planes itself:
 *   nnrcu_conv_f32_plane_stride  the channel stride cs of a 1x1 stride-1 NHWC
 *                                fp32 Conv's planes (NNRCU_ERR_UNSUPPORTED for
 *                                any other Conv: it splits its input itself);
 *   nnrcu_conv_f32_run_to_planes a depthwise fp32 Conv (NHWC in and out) whose
 *                                result goes to y_hi / y_lo ([n*oh*ow][cs]
 *                                uint16 each, channels oc .. cs-1 zero);
 *   nnrcu_conv_f32_run_planes    the 1x1 Conv on such planes (no workspace).
 * The consumer's result is bit-identical to running both convs with
 * nnrcu_conv_f32_run. */
int nnrcu_conv_f32_plane_stride(const nnrcu_op* op, int* cs);
int nnrcu_conv_f32_run_to_planes(nnrcu_op* op, const float* x, uint16_t* y_hi, uint16_t* y_lo, int cs,
                                 void* stream);
int nnrcu_conv_f32_run_planes(nnrcu_op* op, const uint16_t* x_hi, const uint16_t* x_lo, float* y,
                              const float* residual, void* stream);

/* ---------------------------------------------------------------- fp32 Gemm / MatMul
 * Y[m,n] = alpha * op(A)[m,k] * op(B)[k,n] + beta * C, B a constant initializer
 * (prepacked, Gemm.cpp:72-103), C NULL or a [n] row vector or a full [m,n] matrix
 * (c_rows = 1 or m), plus a post-op. MatMul is alpha = 1, beta = 0, trans = 0 with
 * leading batch dims of A folded into m (MatMul.cpp:156-172). */
int nnrcu_gemm_f32_create(int m, int n, int k, int trans_a, int trans_b, float alpha, float beta,
                          const float* b_host, const float* c_host, int c_rows, int post_op, float post_a,
                          float post_b, nnrcu_op** op);
int nnrcu_gemm_f32_run(nnrcu_op* op, const float* a, float* y, void* workspace, void* stream);

/* Precision of an fp32 Gemm / MatMul:
 *   SPLIT_BF16: fp32 emulated as split bf16 (three products, ~2e-5 relative);
 *   BF16: both operands rounded to bf16 (nearest even), one product each,
 *         fp32 accumulation: nnr's own fp32 MatMul with a constant B on hosts
 *         with AVX-512 BF16 (MatMul.cpp:128-152, :382-428 exec_f32_via_bf16),
 *         so results follow that reference path. */
#define NNRCU_PREC_SPLIT_BF16 0
#define NNRCU_PREC_BF16 1
int nnrcu_gemm_f32_create_ex(int m, int n, int k, int trans_a, int trans_b, float alpha, float beta,
                             const float* b_host, const float* c_host, int c_rows, int post_op, float post_a,
                             float post_b, int precision, nnrcu_op** op);

/* MatMul with both operands computed at run time (nnr's MatMul_operator with
 * a non-initializer B, MatMul.cpp:32-94 shapes and broadcast strides,
 * :194-228 exec): for b in [0, batch),
 *   Y[b] = A[a_batch_stride * b] (m x k) x B[b_batch_stride * b] (k x n)
 * row-major, strides in elements (0 broadcasts), Y batches contiguous, plus a
 * post-op. Each batch is split into bf16 hi/lo planes in the workspace
 * (nnrcu_matmul_f32_workspace bytes) and runs on the split-bf16 engine. */
int nnrcu_matmul_f32_workspace(int m, int n, int k, size_t* bytes);
/* The same for bf16 / fp16 tensors (dtype NNRCU_DT_*; nnr's 16-bit MatMul
 * converts to fp32, multiplies and rounds back): one kind::f16 product per
 * multiply-add, fp32 sums, the result rounded to the type (nearest even). */
int nnrcu_matmul_half_workspace(int m, int n, int k, size_t* bytes);
int nnrcu_matmul_half_run(const uint16_t* a, const uint16_t* b, uint16_t* y, int batch, int m, int n, int k,
                          long long a_batch_stride, long long b_batch_stride, int dtype, int post_op, float post_a,
                          float post_b, void* workspace, size_t workspace_bytes, void* stream);
int nnrcu_matmul_f32_run(const float* a, const float* b, float* y, int batch, int m, int n, int k,
                         long long a_batch_stride, long long b_batch_stride, int post_op, float post_a, float post_b,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- 16-bit Conv / Gemm (bf16 or fp16 I/O)
 * Replace nnr's 16-bit I/O paths, which convert to fp32, compute in fp32,
 * apply the post-op and round back (Conv_exec_entry.h:188-381, Gemm.cpp:
 * 297-513): one kind::f16 product per multiply-add (exact in fp32), fp32
 * accumulation and epilogue, the result rounded to the 16-bit type (nearest
 * even). Tensors hold the raw 16-bit values; weights and bias too. */
#define NNRCU_DT_BF16 1
#define NNRCU_DT_F16 2
int nnrcu_conv_half_create(const nnrcu_conv_desc* desc, int dtype, const uint16_t* w_host, const uint16_t* bias_host,
                           nnrcu_op** op);
int nnrcu_conv_half_run(nnrcu_op* op, const uint16_t* x, uint16_t* y, void* workspace, void* stream);
/* alpha must be 1; C is a [n] row or a full [m, n] matrix (c_rows = 1 or m) of the 16-bit type */
int nnrcu_gemm_half_create(int m, int n, int k, int trans_a, int trans_b, float alpha, float beta, int dtype,
                           const uint16_t* b_host, const uint16_t* c_host, int c_rows, int post_op, float post_a,
                           float post_b, nnrcu_op** op);
int nnrcu_gemm_half_run(nnrcu_op* op, const uint16_t* a, uint16_t* y, void* workspace, void* stream);

/* ---------------------------------------------------------------- QDQ glue of int8 networks
 * Device versions of the ops around QLinearConv/QLinearMatMul in a QDQ graph,
 * so that a whole int8 network stays on the device. Same float operation
 * order as nnr's x64 paths (bit-exact u8 results). */
/* QuantizeLinear fp32 NCHW -> u8, per-tensor (backend/cpu/QuantizeLinear.cpp:128-160);
 * out_layout NCHW, or NHWC with channel stride out_cs >= c (extra channels = zp). */
int nnrcu_quantize_linear_u8(const float* x, uint8_t* y, int n, int c, int h, int w, float scale, uint8_t zp,
                             int out_layout, int out_cs, void* stream);
/* MaxPool on u8 NHWC (backend/cpu/MaxPool.cpp:279, dilation 1). */
int nnrcu_maxpool_u8_nhwc(const uint8_t* x, uint8_t* y, int n, int h, int w, int c, int kh, int kw, int sh, int sw,
                          int pt, int pl, int pb, int pr, void* stream);
/* QLinearAdd of two same-shape u8 tensors (backend/cpu/QLinearAdd.cpp:46-104). */
int nnrcu_qlinearadd_u8(const uint8_t* a, float a_scale, uint8_t a_zp, const uint8_t* b, float b_scale, uint8_t b_zp,
                        float y_scale, uint8_t y_zp, uint8_t* y, size_t n, void* stream);
/* DequantizeLinear -> GlobalAveragePool -> QuantizeLinear on u8 NHWC [n, hw, c] -> u8 [n, c]
 * (DequantizeLinear.cpp:135-160, kernel/pool.h:109-125, QuantizeLinear.cpp:128-160). */
int nnrcu_dq_gap_q_u8_nhwc(const uint8_t* x, int n, int hw, int c, float x_scale, uint8_t x_zp, float y_scale,
                           uint8_t y_zp, uint8_t* y, void* stream);
/* DequantizeLinear of u8 [rows, cols] followed by an fp32 Add of bias[cols] (bias may be NULL)
 * (DequantizeLinear.cpp:135-160, binary_math.cpp:57-77). */
int nnrcu_dequantize_linear_u8(const uint8_t* x, float scale, uint8_t zp, const float* bias, int rows, int cols,
                               float* y, void* stream);

/* fp32 Add y = a + b with b repeating every `period` elements (period = total
 * for a same-shape Add, the row length for a broadcast bias row); y may
 * alias a (backend/cpu/binary_math.cpp:57-77, Add). */
int nnrcu_add_f32(const float* a, const float* b, float* y, size_t total, size_t period, void* stream);

/* GlobalAveragePool on fp32 NHWC [n, hw, c] -> [n, c] (kernel/pool.h:109-125). */
int nnrcu_gap_f32_nhwc(const float* x, int n, int hw, int c, float* y, void* stream);

/* ---------------------------------------------------------------- layout helpers
 * Device versions of nnr's boundary reorders (src/nnr.cpp:953-1031, kernel/layout.h). */
int nnrcu_nchw_to_nhwc(const void* src, void* dst, int n, int c, int h, int w, int elem_size, void* stream);
int nnrcu_nhwc_to_nchw(const void* src, void* dst, int n, int c, int h, int w, int elem_size, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* NNRCU_H */
