// QLinearConv and QLinearMatMul on the tcgen05 int8 engine.
//
// Weight packing and the requantisation constants are computed once here
// (the device counterpart of QLinearConv_reshape.h:18-340 and
// QLinearMatMul.cpp:33-94); *_run only enqueues kernels.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "internal.h"
#include "tc_gemm.cuh"

namespace nnrcu {

template <typename T>
static int upload(T** dst, const std::vector<T>& src) {
  NNRCU_CUDA(cudaMalloc(reinterpret_cast<void**>(dst), std::max<size_t>(1, src.size() * sizeof(T))));
  NNRCU_CUDA(cudaMemcpy(*dst, src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice));
  return NNRCU_OK;
}
#define NNRCU_TRY(x)          \
  do {                        \
    int _r = (x);             \
    if (_r != NNRCU_OK) {     \
      nnrcu_op_destroy(op);   \
      return _r;              \
    }                         \
  } while (0)

static inline int round_up(int v, int a) { return (v + a - 1) / a * a; }

int conv_out_dims(const nnrcu_conv_desc& d, int* oh, int* ow) {
  if (d.n <= 0 || d.c <= 0 || d.h <= 0 || d.w <= 0 || d.oc <= 0 || d.kh <= 0 || d.kw <= 0 || d.stride_h <= 0 ||
      d.stride_w <= 0 || d.dil_h <= 0 || d.dil_w <= 0 || d.pad_top < 0 || d.pad_left < 0 || d.pad_bottom < 0 ||
      d.pad_right < 0 || d.group <= 0)
    return set_error(NNRCU_ERR_INVALID, "conv descriptor has a non-positive dimension or negative pad");
  if (d.in_layout != NNRCU_LAYOUT_NCHW && d.in_layout != NNRCU_LAYOUT_NHWC)
    return set_error(NNRCU_ERR_INVALID, "bad input layout %d", d.in_layout);
  if (d.out_layout != NNRCU_LAYOUT_NCHW && d.out_layout != NNRCU_LAYOUT_NHWC)
    return set_error(NNRCU_ERR_INVALID, "bad output layout %d", d.out_layout);
  // ONNX / compute_conv_output_shape (backend/cpu/conv_shape.h:21-79) with explicit pads.
  const int eh = d.dil_h * (d.kh - 1) + 1, ew = d.dil_w * (d.kw - 1) + 1;
  const int ph = d.h + d.pad_top + d.pad_bottom - eh, pw = d.w + d.pad_left + d.pad_right - ew;
  if (ph < 0 || pw < 0) return set_error(NNRCU_ERR_INVALID, "kernel larger than padded input");
  *oh = ph / d.stride_h + 1;
  *ow = pw / d.stride_w + 1;
  return NNRCU_OK;
}

}  // namespace nnrcu

using namespace nnrcu;

namespace nnrcu {
// The int8 weights as shared-memory images per (N tile, K slab), read by the
// engine with one contiguous bulk copy per slab (a tensor-map load moves a
// 128-byte box row per few cycles; a 256-row B slab cost as much as the A
// slab it multiplies).
static int make_b_images(Op* op, int kslab) {
  const int n_tiles = (op->N + op->bn - 1) / op->bn;
  const size_t bytes = (size_t)n_tiles * op->num_kb * op->bn * kslab;
  NNRCU_CUDA(cudaMalloc(&op->wBimg, bytes));
  return pack_b_images(&op->tmB, op->bn, kslab, n_tiles, op->num_kb, op->wBimg);
}
}  // namespace nnrcu

extern "C" {

int nnrcu_qlinearconv_create(const nnrcu_conv_desc* desc, const int8_t* w_host, const float* w_scale, int n_w_scale,
                             const int8_t* w_zp, int n_w_zp, const int32_t* bias_host, float x_scale, uint8_t x_zp,
                             float y_scale, uint8_t y_zp, nnrcu_op** out) {
  if (!desc || !w_host || !w_scale || !out) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  *out = nullptr;
  const nnrcu_conv_desc& d = *desc;
  int oh = 0, ow = 0;
  int rc = conv_out_dims(d, &oh, &ow);
  if (rc != NNRCU_OK) return rc;
  if (n_w_scale != 1 && n_w_scale != d.oc)
    return set_error(NNRCU_ERR_INVALID, "w_scale has %d entries (expected 1 or %d)", n_w_scale, d.oc);
  if (d.group == d.c && d.oc == d.c && d.group > 1)  // depthwise: nnr's exec_dw_int8_nhwc (qdw.cu)
    return qdw_create(d, oh, ow, w_host, w_scale, n_w_scale, w_zp, n_w_zp, bias_host, x_scale, x_zp, y_scale, y_zp,
                      out);
  if (d.group != 1) {
    if (d.c % d.group || d.oc % d.group)
      return set_error(NNRCU_ERR_INVALID, "group %d does not divide channels %d / %d", d.group, d.c, d.oc);
    const std::vector<int8_t> dense = grouped_to_dense(w_host, d.oc, d.c, d.group, d.kh, d.kw);
    nnrcu_conv_desc d1 = d;
    d1.group = 1;
    // nnr runs grouped int8 convs on its VNNI im2col path (the direct and
    // packed paths take group 1 only), whose requant is R1
    // (QLinearConv.cpp:1171-1185, QLinearConv_reshape.h:212-222)
    if (d1.requant == NNRCU_RQ_AUTO) d1.requant = NNRCU_RQ_R1;
    rc = nnrcu_qlinearconv_create(&d1, dense.data(), w_scale, n_w_scale, w_zp, n_w_zp, bias_host, x_scale, x_zp,
                                  y_scale, y_zp, out);
    if (rc == NNRCU_OK) (*out)->num_ops /= d.group;
    return rc;
  }
  for (int i = 0; i < n_w_zp; ++i)
    if (w_zp && w_zp[i] != 0)
      return set_error(NNRCU_ERR_UNSUPPORTED, "non-zero weight zero point (nnr's VNNI paths require symmetric weights)");
  if (!(y_scale > 0.0f) || !(x_scale > 0.0f)) return set_error(NNRCU_ERR_INVALID, "scales must be positive");

  nnrcu_op* op = new nnrcu_op();
  NNRCU_TRY(cuda_check(cudaGetDevice(&op->device), "cudaGetDevice"));
  op->kind = OP_QCONV;
  op->d = d;
  op->oh = oh;
  op->ow = ow;
  op->cs = round_up(d.c, 16);
  op->M = d.n * oh * ow;
  op->N = d.oc;
  op->K = d.kh * d.kw * d.c;
  op->kbytes = d.kh * d.kw * op->cs;
  op->kpad_bytes = round_up(op->kbytes, BKB);
  op->num_kb = op->kpad_bytes / BKB;
  op->npad = round_up(d.oc, 256);
  op->nplane = 1;
  op->bn = pick_bn(op->M, op->N, 1, num_sms());
  op->num_ops = 2LL * op->M * d.oc * (long long)op->K;
  op->x_zp = x_zp;

  // Requant formula: what nnr's x64 VNNI dispatch picks for this layer
  // (QLinearConv.cpp:1337-1351; stem predicate QLinearConv_reshape.h:245-246
  // and QLinearConv.cpp:668-675; direct predicate :579-583).
  int rq = d.requant;
  if (rq == NNRCU_RQ_AUTO) {
    const bool stem = d.c <= 4 && d.kh >= 3 && d.oc >= 16 && d.dil_h == 1 && d.dil_w == 1 &&
                      d.pad_top == d.pad_bottom && d.pad_left == d.pad_right && d.in_layout == NNRCU_LAYOUT_NCHW;
    const bool direct = d.dil_h == 1 && d.dil_w == 1 && oh * ow <= 256 && d.out_layout == NNRCU_LAYOUT_NCHW;
    rq = stem ? NNRCU_RQ_R3 : (direct ? NNRCU_RQ_R1 : NNRCU_RQ_R2);
  }
  if (rq < NNRCU_RQ_R1 || rq > NNRCU_RQ_R3) {
    nnrcu_op_destroy(op);
    return set_error(NNRCU_ERR_INVALID, "unknown requant formula %d", rq);
  }
  op->epi = rq == NNRCU_RQ_R1 ? EPI_R1 : (rq == NNRCU_RQ_R2 ? EPI_R2 : EPI_R3);

  // A operand: plain TMA tiles for a 1x1/s1/p0 conv over an NHWC input that
  // needs no channel padding; the implicit-im2col gather otherwise.
  const bool one_by_one = d.kh == 1 && d.kw == 1 && d.stride_h == 1 && d.stride_w == 1 && d.pad_top == 0 &&
                          d.pad_left == 0 && d.pad_bottom == 0 && d.pad_right == 0;
  op->need_in_copy = d.in_layout == NNRCU_LAYOUT_NCHW || d.c != op->cs;
  // K-slab width for TMA-fed A: 128 bytes, or 64 for 64-byte channel strides
  const int kslab = op->cs % 128 == 0 ? 128 : (op->cs % 64 == 0 ? 64 : 0);
  op->amode = (one_by_one && kslab && op->kbytes >= kslab && op->epi != EPI_R3) ? A_TMA : A_GATHER;
  // Hardware im2col (TMA) when the channel stride is whole 128-byte slabs.
  // Its out-of-bounds fill is zero, which equals the padding value when
  // x_zp = 0 or there is no padding; an NCHW input with x_zp != 0 is instead
  // reordered into a spatially padded copy whose border holds x_zp. Tensors
  // under 128 KB keep the gather path.
  const bool has_pad = d.pad_top || d.pad_left || d.pad_bottom || d.pad_right;
  const bool im2col_shape = op->amode == A_GATHER && op->epi != EPI_R3 && kslab != 0 &&
                            (size_t)d.n * d.h * d.w * op->cs >= 128 * 1024;
  if (im2col_shape && (x_zp == 0 || !has_pad)) {
    op->amode = A_IM2COL;
  } else if (im2col_shape && d.in_layout == NNRCU_LAYOUT_NCHW && (d.h * d.w) % 4 == 0) {
    op->amode = A_IM2COL;
    op->pad_in = true;
  }
  op->kslab = op->amode == A_GATHER ? BKB : kslab;
  op->num_kb = (op->kbytes + op->kslab - 1) / op->kslab;
  // Small-channel convs with a spatial kernel (the 3-channel stem): padding
  // every pixel to a 16-byte channel stride would waste most of K and the
  // gather would touch many taps per slab; materialise a dense im2col matrix
  // [M][round_up(KH*KW*C, 64)] instead and feed it to the engine by TMA.
  if (d.c < 16 && d.kh * d.kw > 1) {
    op->explicit_im2col = true;
    op->amode = A_TMA;
    op->need_in_copy = false;
    op->pad_in = false;
    op->kslab = 64;
    op->kbytes = round_up(d.kh * d.kw * d.c, 64);
    op->kpad_bytes = round_up(op->kbytes, BKB);
    op->num_kb = op->kbytes / 64;
  }
  // Stride-2 convs over at most 4 channels (the stem): space-to-depth. Input
  // row 2*oh - pt + kh lands in s2d row oh + floor((kh - pt) / 2) at parity
  // dy, so the conv becomes a stride-1 conv over 16-byte s2d pixels with an
  // s2d kernel of s2d_kh x s2d_kw taps; weights of kernel positions outside
  // the original kernel are zero, so the integer accumulators are unchanged.
  if (d.c * 4 <= 16 && d.stride_h == 2 && d.stride_w == 2 && d.dil_h == 1 && d.dil_w == 1 && d.kh * d.kw > 1) {
    auto fdiv2 = [](int a) { return a >= 0 ? a / 2 : -((1 - a) / 2); };  // floor(a / 2)
    op->s2d = true;
    op->explicit_im2col = false;
    op->s2d_pt = -fdiv2(-d.pad_top);
    op->s2d_pl = -fdiv2(-d.pad_left);
    op->s2d_kh = fdiv2(d.kh - 1 - d.pad_top) - fdiv2(-d.pad_top) + 1;
    op->s2d_kw = fdiv2(d.kw - 1 - d.pad_left) - fdiv2(-d.pad_left) + 1;
    op->s2d_hp = oh + op->s2d_kh - 1;  // exactly the rows the stride-1 conv reads
    op->s2d_wp = ow + op->s2d_kw - 1;
    op->amode = A_IM2COL;
    op->need_in_copy = false;
    op->pad_in = false;
    op->cs = 16;
    op->kslab = 16;
    // kernel rows of at most 8 taps: one contiguous copy per kernel row
    // (A_ROWS), taps padded to 2 / 4 / 8 per row; else hardware im2col
    if (op->s2d_kw <= 8) {
      op->s2d_tpr = op->s2d_kw <= 2 ? 2 : (op->s2d_kw <= 4 ? 4 : 8);
      op->amode = A_ROWS;
    }
    const int taps = op->s2d_tpr ? op->s2d_kh * op->s2d_tpr : op->s2d_kh * op->s2d_kw;
    op->num_kb = (taps + 7) / 8;
    op->kbytes = taps * 16;
    op->kpad_bytes = op->num_kb * 128;
    op->bn = std::min(op->bn, 128);
    // four taps per kernel row: 64-byte kernel rows through an overlapping-row
    // tensor map (A_XROWS), if the driver accepts that map
    if (op->s2d_tpr == 4 && xrows_enabled() && xrows_map_ok()) {
      op->amode = A_XROWS;
      op->kslab = 64;
      op->num_kb = op->s2d_kh;
      op->kbytes = op->s2d_kh * 64;
      op->kpad_bytes = round_up(op->kbytes, BKB);
    }
  }
  // Shifted-patch mode (A_SHIFT in tc_gemm.cuh): stride-1 spatial convs over
  // whole 64/128-byte channel slabs whose K slabs (at most 9) fit a resident
  // B, the input copied once into a spatially padded NHWC buffer with an
  // x_zp border.
  if (shift_enabled() && !op->s2d && !op->explicit_im2col && d.stride_h == 1 && d.stride_w == 1 &&
      d.kh * d.kw > 1 && kslab != 0 && op->epi != EPI_R3 &&
      ((d.in_layout == NNRCU_LAYOUT_NCHW && (d.h * d.w) % 4 == 0) || (d.in_layout == NNRCU_LAYOUT_NHWC && d.c == op->cs))) {
    const int hp = d.h + d.pad_top + d.pad_bottom, wp = d.w + d.pad_left + d.pad_right;
    // (slabs start on 1024-byte boundaries: the swizzle pattern repeats there)
    const int prows = round_up(BM + (d.kh - 1) * d.dil_h * wp + (d.kw - 1) * d.dil_w, 1024 / kslab);
    const int nslab = op->cs / kslab;
    const int nkb = d.kh * d.kw * nslab;
    // N tile 128 (16 epilogue warps) when the output channels are whole
    // 128-column tiles and the patch still fits beside the larger B
    const int patch_bytes = nslab * prows * kslab;
    const bool bn128 = kslab == 128 && d.oc % 128 == 0 && (d.oc / 128 == 1 || d.oc / 128 == 2 || d.oc / 128 == 4) &&
                       patch_bytes <= KernelCfg<128, 1, A_SHIFT, EPI_R2, 128, 9>::PATCH_BYTES;
    const int nt = (d.oc + 63) / 64;
    const int patch_cap = kslab == 128 ? KernelCfg<64, 1, A_SHIFT, EPI_R2, 128, 9>::PATCH_BYTES
                                       : KernelCfg<64, 1, A_SHIFT, EPI_R2, 64, 9>::PATCH_BYTES;
    if (prows <= 256 && nkb <= 9 && (bn128 || ((nt == 1 || nt == 2 || nt == 4) && patch_bytes <= patch_cap))) {
      op->amode = A_SHIFT;
      op->bn = bn128 ? 128 : 64;
      op->kslab = kslab;
      op->num_kb = nkb;
      op->pad_in = true;
      op->need_in_copy = true;
      op->shift_prows = prows;
    }
  }
  const size_t hp = d.h + (op->pad_in ? d.pad_top + d.pad_bottom : 0);
  const size_t wp = d.w + (op->pad_in ? d.pad_left + d.pad_right : 0);
  op->ws_bytes = op->need_in_copy ? (size_t)d.n * hp * wp * op->cs : 0;
  if (op->explicit_im2col) op->ws_bytes = (size_t)op->M * op->kbytes;
  // (A_ROWS copies read up to BM + 8 pixels from a row start: slack at the end)
  if (op->s2d) op->ws_bytes = (size_t)d.n * op->s2d_hp * op->s2d_wp * 16 + (op->s2d_tpr ? ROWS_BYTES : 0);
  // Pack B = W as [npad][kpad] K-major with k = (kh, kw, ic); padded channels,
  // taps and rows are zero. wsum feeds the x_zp compensation.
  std::vector<int8_t> B((size_t)op->npad * op->kpad_bytes, 0);
  std::vector<int32_t> colcorr(d.oc), bias_i(d.oc, 0);
  std::vector<float> csv(d.oc), bias_f(d.oc, 0.0f), osv(d.oc);
  const float inv_y = 1.0f / y_scale;  // QLinearConv.cpp:420 / QLinearConv_reshape.h:291
  for (int o = 0; o < d.oc; ++o) {
    int32_t wsum = 0;
    for (int ic = 0; ic < d.c; ++ic)
      for (int y = 0; y < d.kh; ++y)
        for (int x = 0; x < d.kw; ++x) {
          const int8_t v = w_host[(((size_t)o * d.c + ic) * d.kh + y) * d.kw + x];
          if (op->s2d && op->amode == A_XROWS) {
            // K-major [npad][kpad]: s2d tap (ky, kx) at (ky * 4 + kx) * 16
            const int ry = y + 2 * op->s2d_pt - d.pad_top, rx = x + 2 * op->s2d_pl - d.pad_left;
            B[(size_t)o * op->kpad_bytes + (size_t)((ry >> 1) * 4 + (rx >> 1)) * 16 + ((ry & 1) * 2 + (rx & 1)) * d.c + ic] = v;
          } else if (op->s2d) {
            // per (N tile, K slab) the stage's smem image [8 taps][bn rows][16 B]:
            // s2d tap (ky, kx), byte (dy * 2 + dx) * C + ic
            const int ry = y + 2 * op->s2d_pt - d.pad_top, rx = x + 2 * op->s2d_pl - d.pad_left;
            const int tap = (ry >> 1) * (op->s2d_tpr ? op->s2d_tpr : op->s2d_kw) + (rx >> 1);
            const int nt = o / op->bn, r = o - nt * op->bn;
            B[((((size_t)nt * op->num_kb + tap / 8) * 8 + tap % 8) * op->bn + r) * 16 + ((ry & 1) * 2 + (rx & 1)) * d.c + ic] = v;
          } else {
            const int tap_stride = op->explicit_im2col ? d.c : op->cs;  // dense K for explicit im2col
            B[(size_t)o * op->kpad_bytes + (size_t)(y * d.kw + x) * tap_stride + ic] = v;
          }
          wsum += v;
        }
    colcorr[o] = (int32_t)(0u - (uint32_t)x_zp * (uint32_t)wsum);
    const float ws = n_w_scale > 1 ? w_scale[o] : w_scale[0];
    csv[o] = x_scale * ws;                                   // combined scale
    if (bias_host) {
      bias_i[o] = bias_host[o];
      bias_f[o] = (float)bias_host[o] * csv[o];
    }
    osv[o] = csv[o] * inv_y;                                 // QLinearConv_reshape.h:310
  }
  const int lo = 0, hi = 255;
  const int qmin = d.post_op != NNRCU_POST_NONE ? std::max(lo, (int)y_zp) : lo;
  op->inv_y = inv_y;
  op->yzp_f = (float)y_zp;
  op->qmin_f = (float)qmin;
  op->qmax_f = (float)hi;
  op->rq_lo = (float)lo - (float)y_zp;                       // QLinearConv_reshape.h:326-327
  op->rq_hi = (float)hi - (float)y_zp;
  op->yzp = y_zp;
  op->y_scale = y_scale;

  void* wB = nullptr;
  NNRCU_TRY(cuda_check(cudaMalloc(&wB, B.size()), "cudaMalloc(weights)"));
  op->wB = wB;
  NNRCU_TRY(cuda_check(cudaMemcpy(wB, B.data(), B.size(), cudaMemcpyHostToDevice), "upload weights"));
  NNRCU_TRY(upload(&op->colcorr, colcorr));
  NNRCU_TRY(upload(&op->bias_i, bias_i));
  NNRCU_TRY(upload(&op->cs_arr, csv));
  NNRCU_TRY(upload(&op->bias_f, bias_f));
  NNRCU_TRY(upload(&op->os, osv));
  if (!op->s2d || op->amode == A_XROWS) {  // (A_ROWS s2d weights are read by plain bulk copies)
    NNRCU_TRY(encode_tmap_2d(&op->tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, wB, op->kpad_bytes, op->npad, op->kpad_bytes,
                             op->kslab, op->bn,
                             op->kslab == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B));
    NNRCU_TRY(make_b_images(op, op->kslab));
  }
  *out = op;
  return NNRCU_OK;
}

// xf != NULL: the input is fp32 and QuantizeLinear(xf, q_scale, q_zp) is
// fused into the input reorder (space-to-depth ops only); x is then unused.
static int qconv_run(nnrcu_op* op, const uint8_t* x, uint8_t* y, void* workspace, void* stream, const uint8_t* res,
                     float res_scale, uint8_t res_zp, float out_scale, uint8_t out_zp, const float* xf = nullptr,
                     float q_scale = 0.0f, uint8_t q_zp = 0) {
  if (op && op->kind == OP_QDW) {
    if (!x || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
    if (res || xf) return set_error(NNRCU_ERR_UNSUPPORTED, "depthwise QLinearConv: no fused add or quantisation");
    return qdw_run(op, x, y, workspace, static_cast<cudaStream_t>(stream));
  }
  if (!op || op->kind != OP_QCONV) return set_error(NNRCU_ERR_INVALID, "not a QLinearConv operator");
  if ((!x && !xf) || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if (xf && !op->s2d)
    return set_error(NNRCU_ERR_UNSUPPORTED, "QuantizeLinear fusion needs a space-to-depth QLinearConv (stride 2, <= 4 channels)");
  if (xf && !(q_scale > 0.0f)) return set_error(NNRCU_ERR_INVALID, "QuantizeLinear scale must be positive");
  if (op->ws_bytes && !workspace && !op->in_padded)
    return set_error(NNRCU_ERR_INVALID, "workspace of %zu bytes required", op->ws_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const nnrcu_conv_desc& d = op->d;
  const uint8_t* xin = x;
  if (op->s2d) {
    int rc = xf ? launch_quantize_s2d(xf, d.in_layout == NNRCU_LAYOUT_NCHW, static_cast<uint8_t*>(workspace), d.n, d.c,
                                      d.h, d.w, op->s2d_hp, op->s2d_wp, op->s2d_pt, op->s2d_pl, (uint8_t)op->x_zp,
                                      q_scale, q_zp, st)
                : launch_s2d_u8(x, d.in_layout == NNRCU_LAYOUT_NCHW, static_cast<uint8_t*>(workspace), d.n, d.c, d.h,
                                d.w, op->s2d_hp, op->s2d_wp, op->s2d_pt, op->s2d_pl, (uint8_t)op->x_zp, st);
    if (rc != NNRCU_OK) return rc;
    xin = static_cast<const uint8_t*>(workspace);
  } else if (op->explicit_im2col) {
    int rc = launch_im2col_u8(x, static_cast<uint8_t*>(workspace), d.in_layout == NNRCU_LAYOUT_NCHW, d.n, d.c, d.h,
                              d.w, op->oh, op->ow, d.kh, d.kw, d.stride_h, d.stride_w, d.pad_top, d.pad_left, d.dil_h,
                              d.dil_w, op->kbytes, (uint8_t)op->x_zp, st);
    if (rc != NNRCU_OK) return rc;
    xin = static_cast<const uint8_t*>(workspace);
  } else if (op->in_padded) {
    xin = x;  // the caller's buffer already is the padded copy
  } else if (op->need_in_copy) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int rc = op->pad_in && d.in_layout == NNRCU_LAYOUT_NHWC
                 ? launch_pad_spatial_nhwc_u8(x, ws, d.n, d.h, d.w, op->cs, d.pad_top, d.pad_left, d.pad_bottom,
                                              d.pad_right, (uint8_t)op->x_zp, st)
             : op->pad_in ? launch_nchw_to_nhwc_u8_padded(x, ws, d.n, d.c, d.h, d.w, d.pad_top, d.pad_left,
                                                         d.pad_bottom, d.pad_right, op->cs, (uint8_t)op->x_zp, st)
             : d.in_layout == NNRCU_LAYOUT_NCHW
                 ? launch_nchw_to_nhwc_u8(x, ws, d.n, d.c, d.h, d.w, op->cs, (uint8_t)op->x_zp, st)
                 : launch_pad_nhwc_u8(x, ws, d.n * d.h * d.w, d.c, op->cs, (uint8_t)op->x_zp, st);
    if (rc != NNRCU_OK) return rc;
    xin = ws;
  }
  CUtensorMap tmA{};
  if (op->amode == A_TMA) {
    const int arow = op->explicit_im2col ? op->kbytes : op->cs;  // bytes per A row
    int rc = encode_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, xin, arow, (uint64_t)op->M, arow, op->kslab, BM,
                            op->kslab == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc != NNRCU_OK) return rc;
  }
  GatherGeom g{};
  g.wb = bimg_enabled() ? static_cast<const uint8_t*>(op->wBimg) : nullptr;
  g.x = xin;
  g.x2 = nullptr;
  // a spatially pre-padded input is convolved with zero pads
  const int pt = op->pad_in ? 0 : d.pad_top, pl = op->pad_in ? 0 : d.pad_left;
  const int pb = op->pad_in ? 0 : d.pad_bottom, pr = op->pad_in ? 0 : d.pad_right;
  g.N = d.n;
  g.H = d.h + (op->pad_in ? d.pad_top + d.pad_bottom : 0);
  g.W = d.w + (op->pad_in ? d.pad_left + d.pad_right : 0);
  g.cbytes = op->cs;
  g.OH = op->oh; g.OW = op->ow; g.KH = d.kh; g.KW = d.kw;
  g.sh = d.stride_h; g.sw = d.stride_w; g.ph = pt; g.pw = pl; g.dh = d.dil_h; g.dw = d.dil_w;
  if (op->s2d) {
    g.H = op->s2d_hp; g.W = op->s2d_wp; g.KH = op->s2d_kh; g.KW = op->s2d_kw;
    g.sh = g.sw = 1; g.ph = g.pw = 0; g.dh = g.dw = 1;
    g.tpr = op->s2d_tpr;
    g.wb = static_cast<const uint8_t*>(op->wB);
    if (op->amode == A_XROWS) {
      // rows 16 bytes apart, 64 bytes wide: row p = s2d pixels p .. p + 3.
      // Every pixel starts a row; the last rows reach up to 48 bytes past the
      // image into the workspace's slack (taps past the kernel width have
      // zero weights, and real taps never leave the image)
      g.wb = bimg_enabled() ? static_cast<const uint8_t*>(op->wBimg) : nullptr;
      int rc = encode_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, xin, 64, (uint64_t)g.N * g.H * g.W, 16, 64, BM,
                              CU_TENSOR_MAP_SWIZZLE_64B);
      if (rc != NNRCU_OK) return rc;
    } else if (!op->s2d_tpr) {
      int rc = encode_tmap_im2col(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, xin, g.N, g.H, g.W, 16, 0, 0, 0, 0, g.KH,
                                  g.KW, 1, 1, 1, 1, 16);
      if (rc != NNRCU_OK) return rc;
    }
  } else if (op->amode == A_SHIFT) {
    g.prows = op->shift_prows;
    int rc = encode_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, xin, op->cs, (uint64_t)g.N * g.H * g.W, op->cs,
                            op->kslab, op->shift_prows,
                            op->kslab == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc != NNRCU_OK) return rc;
  } else if (op->amode == A_IM2COL) {
    int rc = encode_tmap_im2col(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, xin, g.N, g.H, g.W, op->cs, pt, pl, pb, pr,
                                d.kh, d.kw, d.dil_h, d.dil_w, d.stride_h, d.stride_w, op->kslab);
    if (rc != NNRCU_OK) return rc;
  }
  g.kbytes = op->kbytes;
  g.pad_word = 0x01010101u * (uint32_t)op->x_zp;

  EpiParams e{};
  e.M = op->M; e.N = op->N;
  e.colcorr = op->colcorr; e.bias_i = op->bias_i; e.cs = op->cs_arr; e.bias_f = op->bias_f; e.os = op->os;
  e.inv_y = op->inv_y; e.yzp_f = op->yzp_f; e.qmin_f = op->qmin_f; e.qmax_f = op->qmax_f;
  e.rq_lo = op->rq_lo; e.rq_hi = op->rq_hi; e.yzp = op->yzp;
  e.r2_sat = r2_sat_enabled() && op->yzp == 0 && op->rq_lo == 0.0f && op->rq_hi == 255.0f;
  e.y = y;
  e.y_layout = d.out_layout == NNRCU_LAYOUT_NCHW ? 1 : 0;
  e.ldy = d.oc;
  e.ohw = op->oh * op->ow;
  e.status = status_ptr();
  if (op->out_pad[0] | op->out_pad[1] | op->out_pad[2] | op->out_pad[3]) {
    if (res || xf) return set_error(NNRCU_ERR_UNSUPPORTED, "a padded output is available through nnrcu_qlinearconv_run only");
    e.opad = 1;
    e.o_w = op->ow;
    e.o_hw = op->oh * op->ow;
    e.o_wp = op->ow + op->out_pad[1] + op->out_pad[3];
    e.o_hwp = (op->oh + op->out_pad[0] + op->out_pad[2]) * e.o_wp;
    e.o_off = op->out_pad[0] * e.o_wp + op->out_pad[1];
  }
  if (res) {
    if (d.out_layout != NNRCU_LAYOUT_NHWC)
      return set_error(NNRCU_ERR_UNSUPPORTED, "a fused residual add needs an NHWC output");
    if (!(out_scale > 0.0f)) return set_error(NNRCU_ERR_INVALID, "add output scale must be positive");
    // QLinearAdd constants in nnr's order (QLinearAdd.cpp:46-66); GCC
    // contracts sa*a_zp + sb*b_zp into fma(sa, a_zp, sb*b_zp)
    e.qres = res;
    e.qa_sa = op->y_scale / out_scale;
    e.qa_sb = res_scale / out_scale;
    e.qa_fixed = (float)out_zp - std::fma(e.qa_sa, (float)op->yzp, e.qa_sb * (float)res_zp);
    e.qa_azp = op->yzp;
    e.qa_bzp = res_zp;
    e.qa_yzp = out_zp;
    const long long n = (long long)op->M * op->N;
    e.qa_vec_end = n / 16 * 16;
    e.qa_ovf = 255.0 * (std::fabs((double)e.qa_sa) + std::fabs((double)e.qa_sb)) + std::fabs((double)e.qa_fixed) >=
               1073741824.0;
  }

  TcLaunch L{};
  L.bn = op->bn; L.nplane = 1; L.amode = op->amode; L.epi = op->epi;
  L.m_tiles = (op->amode == A_ROWS || op->amode == A_XROWS) ? d.n * op->oh * ((op->ow + BM - 1) / BM)
                                                            : (op->M + BM - 1) / BM;
  if (op->amode == A_SHIFT) {
    // GEMM rows = padded-grid positions up to the last output pixel
    e.M = ((d.n - 1) * g.H + op->oh - 1) * g.W + op->ow;
    L.m_tiles = (e.M + BM - 1) / BM;
  }
  L.n_tiles = (op->N + op->bn - 1) / op->bn;
  L.tmA0 = &tmA; L.tmA1 = &tmA; L.tmB = &op->tmB;
  L.b_plane_rows = op->npad;
  L.num_kb = op->num_kb;
  L.kb_bytes = op->kslab;
  return tc_launch(L, g, e, st);
}

int nnrcu_qlinearconv_input_padding(const nnrcu_op* op, int* pads) {
  if (!op || (op->kind != OP_QCONV && op->kind != OP_QDW) || !pads)
    return set_error(NNRCU_ERR_INVALID, "not a QLinearConv operator");
  const bool padded = op->amode == A_SHIFT && op->d.in_layout == NNRCU_LAYOUT_NHWC;
  pads[0] = padded ? op->d.pad_top : 0;
  pads[1] = padded ? op->d.pad_left : 0;
  pads[2] = padded ? op->d.pad_bottom : 0;
  pads[3] = padded ? op->d.pad_right : 0;
  return NNRCU_OK;
}

int nnrcu_qlinearconv_set_padded_io(nnrcu_op* op, int in_padded, int out_top, int out_left, int out_bottom,
                                    int out_right) {
  if (!op || op->kind != OP_QCONV) return set_error(NNRCU_ERR_INVALID, "not a QLinearConv operator");
  if (in_padded && !(op->amode == A_SHIFT && op->d.in_layout == NNRCU_LAYOUT_NHWC))
    return set_error(NNRCU_ERR_INVALID, "this QLinearConv does not read a padded input copy");
  if (out_top < 0 || out_left < 0 || out_bottom < 0 || out_right < 0)
    return set_error(NNRCU_ERR_INVALID, "negative output padding");
  if ((out_top | out_left | out_bottom | out_right) &&
      (op->d.out_layout != NNRCU_LAYOUT_NHWC || op->s2d || op->d.oc % 16 != 0))
    return set_error(NNRCU_ERR_UNSUPPORTED, "a padded output needs an NHWC output with a multiple of 16 channels");
  op->in_padded = in_padded != 0;
  op->out_pad[0] = out_top; op->out_pad[1] = out_left; op->out_pad[2] = out_bottom; op->out_pad[3] = out_right;
  return NNRCU_OK;
}

int nnrcu_qlinearconv_run(nnrcu_op* op, const uint8_t* x, uint8_t* y, void* workspace, void* stream) {
  return qconv_run(op, x, y, workspace, stream, nullptr, 0.0f, 0, 0.0f, 0);
}

int nnrcu_qlinearconv_run_quantize(nnrcu_op* op, const float* x, float x_scale, uint8_t x_zp, uint8_t* y,
                                   void* workspace, void* stream) {
  return qconv_run(op, nullptr, y, workspace, stream, nullptr, 0.0f, 0, 0.0f, 0, x, x_scale, x_zp);
}

int nnrcu_qlinearconv_run_add(nnrcu_op* op, const uint8_t* x, const uint8_t* residual, float res_scale,
                              uint8_t res_zp, float out_scale, uint8_t out_zp, uint8_t* y, void* workspace,
                              void* stream) {
  if (!residual) return set_error(NNRCU_ERR_INVALID, "NULL residual");
  return qconv_run(op, x, y, workspace, stream, residual, res_scale, res_zp, out_scale, out_zp);
}

int nnrcu_qlinearmatmul_create(int m, int k, int n, float a_scale, uint8_t a_zp, const int8_t* b_host, float b_scale,
                               int8_t b_zp, float y_scale, uint8_t y_zp, nnrcu_op** out) {
  if (!b_host || !out) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  *out = nullptr;
  if (m <= 0 || k <= 0 || n <= 0) return set_error(NNRCU_ERR_INVALID, "QLinearMatMul dims must be positive");
  nnrcu_op* op = new nnrcu_op();
  NNRCU_TRY(cuda_check(cudaGetDevice(&op->device), "cudaGetDevice"));
  op->kind = OP_QMATMUL;
  op->M = m; op->N = n; op->K = k;
  op->cs = round_up(k, 16);            // A row stride on the device
  op->kbytes = op->cs;
  op->kpad_bytes = round_up(op->kbytes, BKB);
  op->num_kb = op->kpad_bytes / BKB;
  op->npad = round_up(n, 256);
  op->nplane = 1;
  op->epi = EPI_R4;
  op->bn = pick_bn(m, n, 1, num_sms());
  op->num_ops = 2LL * m * n * (long long)k;
  op->a_zp = a_zp;
  op->b_zp = b_zp;
  op->need_in_copy = op->cs != k;
  op->amode = op->kbytes >= BKB ? A_TMA : A_GATHER;
  op->ws_bytes = (op->need_in_copy ? round_up(m * op->cs, 256) : 0) + (b_zp != 0 ? (size_t)m * 4 : 0);

  // Combined scale a*b/y in that order (QLinearMatMul.cpp:134).
  op->combined = a_scale * b_scale / y_scale;
  op->yzp_f = (float)y_zp;

  std::vector<int8_t> B((size_t)op->npad * op->kpad_bytes, 0);
  std::vector<int32_t> colcorr(n);
  for (int j = 0; j < n; ++j) {
    int32_t s = 0;
    for (int kk = 0; kk < k; ++kk) {
      const int8_t v = b_host[(size_t)kk * n + j];
      B[(size_t)j * op->kpad_bytes + kk] = v;
      s += v;
    }
    // sum (a - a_zp)(b - b_zp) = sum ab - a_zp*colsum - b_zp*rowsum + k*a_zp*b_zp
    // (zero-point algebra of backend/x64/gemm_int8_avx512.h:1-11)
    colcorr[j] = (int32_t)(0u - (uint32_t)a_zp * (uint32_t)s + (uint32_t)k * (uint32_t)a_zp * (uint32_t)(int32_t)b_zp);
  }
  void* wB = nullptr;
  NNRCU_TRY(cuda_check(cudaMalloc(&wB, B.size()), "cudaMalloc(weights)"));
  op->wB = wB;
  NNRCU_TRY(cuda_check(cudaMemcpy(wB, B.data(), B.size(), cudaMemcpyHostToDevice), "upload weights"));
  NNRCU_TRY(upload(&op->colcorr, colcorr));
  NNRCU_TRY(encode_tmap_2d(&op->tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, wB, op->kpad_bytes, op->npad, op->kpad_bytes,
                           BKB, op->bn));
  NNRCU_TRY(make_b_images(op, BKB));
  *out = op;
  return NNRCU_OK;
}

int nnrcu_qlinearmatmul_run(nnrcu_op* op, const uint8_t* a, uint8_t* y, void* workspace, void* stream) {
  if (!op || op->kind != OP_QMATMUL) return set_error(NNRCU_ERR_INVALID, "not a QLinearMatMul operator");
  if (!a || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if (op->ws_bytes && !workspace)
    return set_error(NNRCU_ERR_INVALID, "workspace of %zu bytes required", op->ws_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* ain = a;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* rowcorr = nullptr;
  if (op->need_in_copy) {
    int rc = launch_pad_nhwc_u8(a, ws, op->M, op->K, op->cs, (uint8_t)op->a_zp, st);
    if (rc != NNRCU_OK) return rc;
    ain = ws;
    ws += round_up(op->M * op->cs, 256);
  }
  if (op->b_zp != 0) {
    rowcorr = reinterpret_cast<int32_t*>(ws);
    int rc = launch_rowcorr_u8(ain, op->M, op->K, op->cs, op->b_zp, rowcorr, st);
    if (rc != NNRCU_OK) return rc;
  }
  CUtensorMap tmA{};
  if (op->amode == A_TMA) {
    int rc = encode_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, ain, op->cs, (uint64_t)op->M, op->cs, BKB, BM);
    if (rc != NNRCU_OK) return rc;
  }
  GatherGeom g{};
  g.wb = bimg_enabled() ? static_cast<const uint8_t*>(op->wBimg) : nullptr;
  g.x = ain;
  g.N = 1; g.H = 1; g.W = op->M;
  g.cbytes = op->cs;
  g.OH = 1; g.OW = op->M; g.KH = 1; g.KW = 1; g.sh = 1; g.sw = 1; g.ph = 0; g.pw = 0; g.dh = 1; g.dw = 1;
  g.kbytes = op->kbytes;
  g.pad_word = 0;
  EpiParams e{};
  e.M = op->M; e.N = op->N;
  e.colcorr = op->colcorr;
  e.rowcorr = rowcorr;
  e.combined = op->combined;
  e.yzp_f = op->yzp_f;
  e.y = y;
  e.y_layout = 0;
  e.ldy = op->N;
  e.ohw = 1;
  e.status = status_ptr();
  TcLaunch L{};
  L.bn = op->bn; L.nplane = 1; L.amode = op->amode; L.epi = EPI_R4;
  L.m_tiles = (op->M + BM - 1) / BM;
  L.n_tiles = (op->N + op->bn - 1) / op->bn;
  L.tmA0 = &tmA; L.tmA1 = &tmA; L.tmB = &op->tmB;
  L.b_plane_rows = op->npad;
  L.num_kb = op->num_kb;
  return tc_launch(L, g, e, st);
}

}  // extern "C"
