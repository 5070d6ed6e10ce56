// fp32 Conv (dense: split-bf16 on tcgen05; depthwise: CUDA cores) and
// fp32 Gemm / MatMul (split-bf16 on tcgen05).
#include <algorithm>
#include <cstring>

#include "internal.h"
#include "tc_gemm.cuh"

namespace nnrcu {
int conv_out_dims(const nnrcu_conv_desc& d, int* oh, int* ow);
static inline int round_up(int v, int a) { return (v + a - 1) / a * a; }
static inline size_t round_up_sz(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <typename T>
static int upload_vec(T** dst, const std::vector<T>& src) {
  NNRCU_CUDA(cudaMalloc(reinterpret_cast<void**>(dst), std::max<size_t>(1, src.size() * sizeof(T))));
  NNRCU_CUDA(cudaMemcpy(*dst, src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice));
  return NNRCU_OK;
}

static int map_post(int post_op, float a, float b, Op* op) {
  switch (post_op) {
    case NNRCU_POST_NONE: op->act = ACT_NONE; break;
    case NNRCU_POST_RELU: op->act = ACT_RELU; break;
    case NNRCU_POST_CLIP: op->act = ACT_CLIP; break;
    case NNRCU_POST_HARDSWISH: op->act = ACT_HARDSWISH; break;
    case NNRCU_POST_SIGMOID: op->act = ACT_SIGMOID; break;
    case NNRCU_POST_LEAKYRELU: op->act = ACT_LEAKYRELU; break;
    case NNRCU_POST_TANH: op->act = ACT_TANH; break;
    default: return set_error(NNRCU_ERR_INVALID, "unknown post-op %d", post_op);
  }
  op->act_a = a;
  op->act_b = b;
  return NNRCU_OK;
}

// Packs a K-major fp32 matrix (rows x k, accessor get(r, kk)) into two bf16
// planes [2][npad][kpad_bytes/2] and uploads it.
template <typename F>
static int pack_split_planes(Op* op, int rows, int k, F get) {
  const size_t kpe = op->kpad_bytes / 2;
  std::vector<uint16_t> B((size_t)2 * op->npad * kpe, 0);
  for (int r = 0; r < rows; ++r)
    for (int kk = 0; kk < k; ++kk) {
      const float v = get(r, kk);
      if (v == 0.0f) continue;
      uint16_t h, l;
      host_split_bf16(v, &h, &l);
      B[(size_t)r * kpe + kk] = h;
      B[((size_t)op->npad + r) * kpe + kk] = l;
    }
  NNRCU_CUDA(cudaMalloc(&op->wB, B.size() * 2));
  NNRCU_CUDA(cudaMemcpy(op->wB, B.data(), B.size() * 2, cudaMemcpyHostToDevice));
  return encode_tmap_2d(&op->tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, op->wB, kpe, (uint64_t)2 * op->npad,
                        op->kpad_bytes, op->kslab / 2, op->bn,
                        op->kslab == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

}  // namespace nnrcu

using namespace nnrcu;

#define NNRCU_TRY(x)          \
  do {                        \
    int _r = (x);             \
    if (_r != NNRCU_OK) {     \
      nnrcu_op_destroy(op);   \
      return _r;              \
    }                         \
  } while (0)

extern "C" {

int nnrcu_conv_f32_create(const nnrcu_conv_desc* desc, const float* w_host, const float* bias_host, nnrcu_op** out) {
  if (!desc || !w_host || !out) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  *out = nullptr;
  const nnrcu_conv_desc& d = *desc;
  int oh = 0, ow = 0;
  int rc = conv_out_dims(d, &oh, &ow);
  if (rc != NNRCU_OK) return rc;
  const bool depthwise = d.group == d.c && d.group == d.oc && d.group > 1;
  if (d.group != 1 && !depthwise) {
    if (d.c % d.group || d.oc % d.group)
      return set_error(NNRCU_ERR_INVALID, "group %d does not divide channels %d / %d", d.group, d.c, d.oc);
    const std::vector<float> dense = grouped_to_dense(w_host, d.oc, d.c, d.group, d.kh, d.kw);
    nnrcu_conv_desc d1 = d;
    d1.group = 1;
    rc = nnrcu_conv_f32_create(&d1, dense.data(), bias_host, out);
    if (rc == NNRCU_OK) (*out)->num_ops /= d.group;
    return rc;
  }
  if (depthwise && (d.c % 4) != 0)
    return set_error(NNRCU_ERR_UNSUPPORTED, "depthwise Conv needs channels %% 4 == 0 (got %d)", d.c);

  nnrcu_op* op = new nnrcu_op();
  NNRCU_TRY(cuda_check(cudaGetDevice(&op->device), "cudaGetDevice"));
  op->d = d;
  op->oh = oh;
  op->ow = ow;
  op->M = d.n * oh * ow;
  op->N = d.oc;
  op->K = d.kh * d.kw * (d.c / d.group);
  op->num_ops = 2LL * op->M * d.oc * (long long)op->K;
  NNRCU_TRY(map_post(d.post_op, d.post_a, d.post_b, op));
  if (bias_host) NNRCU_TRY(upload_vec(&op->bias, std::vector<float>(bias_host, bias_host + d.oc)));

  if (depthwise) {
    op->kind = OP_DWCONV_F32;
    std::vector<float> w((size_t)d.kh * d.kw * d.c);
    for (int ch = 0; ch < d.c; ++ch)
      for (int y = 0; y < d.kh; ++y)
        for (int x = 0; x < d.kw; ++x) w[((size_t)y * d.kw + x) * d.c + ch] = w_host[((size_t)ch * d.kh + y) * d.kw + x];
    NNRCU_TRY(upload_vec(&op->w_dw, w));
    const size_t in_bytes = d.in_layout == NNRCU_LAYOUT_NCHW ? (size_t)d.n * d.h * d.w * d.c * 4 : 0;
    const size_t out_bytes = d.out_layout == NNRCU_LAYOUT_NCHW ? (size_t)op->M * d.oc * 4 : 0;
    op->ws_bytes = round_up_sz(in_bytes, 256) + out_bytes;
    *out = op;
    return NNRCU_OK;
  }

  op->kind = OP_CONV_F32;
  op->nplane = 2;
  op->epi = EPI_F32;
  op->kslab = BKB;
  op->cs = round_up(d.c, 8);  // bf16 elements: 16-byte pixel stride
  const bool one_by_one = d.kh == 1 && d.kw == 1 && d.stride_h == 1 && d.stride_w == 1 && d.pad_top == 0 &&
                          d.pad_left == 0 && d.pad_bottom == 0 && d.pad_right == 0;
  // 1x1 convs over fewer than 64 channels: channel stride padded to 32 or 64
  // bf16 so that A is one 64- or 128-byte slab per pixel, fed by 2-D TMA
  if (one_by_one && d.c < 64) {
    op->cs = d.c <= 32 ? 32 : 64;
    op->kslab = d.c <= 32 ? 64 : 128;
  }
  op->kbytes = d.kh * d.kw * op->cs * 2;
  op->kpad_bytes = round_up(op->kbytes, op->kslab);
  op->num_kb = op->kpad_bytes / op->kslab;
  op->npad = round_up(d.oc, 256);
  // N tile 64 for every split-bf16 conv: on MobileNetV2 (N 16-1280) the
  // batch-128 forward took 2.30 ms against 2.36 with pick_bn's choice and
  // 2.35 with 128 wherever N > 64 (the fp32 epilogue, not the A re-reads,
  // sets the tile cost)
  op->bn = 64;
  op->amode = (one_by_one && op->kbytes >= op->kslab) ? A_TMA : A_GATHER;
  // hardware im2col (TMA) when a pixel is whole 128-byte slabs of bf16 (C a
  // multiple of 64); its zero fill is the fp32 padding value
  if (op->amode == A_GATHER && (op->cs * 2) % BKB == 0 && (size_t)d.n * d.h * d.w * op->cs * 2 >= 128 * 1024)
    op->amode = A_IM2COL;
  // Small-channel convs with a spatial kernel (the 3-channel stem): A is
  // materialised as dense split-bf16 rows [M][kp] (k = (kh, kw, ic), kp = K
  // rounded to 32 or 64 elements) by one im2col pass, then fed by 2-D TMA
  if (d.c < 16 && d.kh * d.kw > 1) {
    op->explicit_im2col = true;
    const int kd = d.kh * d.kw * d.c;
    op->cs = kd <= 32 ? 32 : round_up(kd, 64);
    op->kslab = kd <= 32 ? 64 : 128;
    op->kbytes = op->cs * 2;
    op->kpad_bytes = op->kbytes;
    op->num_kb = op->kbytes / op->kslab;
    op->amode = A_TMA;
  }
  const size_t plane = op->explicit_im2col ? round_up_sz((size_t)op->M * op->cs * 2, 256)
                                           : round_up_sz((size_t)d.n * d.h * d.w * op->cs * 2, 256);
  op->ws_bytes = 2 * plane;
  const int cs = op->explicit_im2col ? d.c : op->cs;  // dense (kh, kw, ic) K for explicit im2col
  NNRCU_TRY(pack_split_planes(op, d.oc, op->kpad_bytes / 2, [&](int r, int kk) -> float {
    const int tap = kk / cs, ic = kk - tap * cs;
    if (tap >= d.kh * d.kw || ic >= d.c) return 0.0f;
    const int y = tap / d.kw, x = tap - y * d.kw;
    return w_host[(((size_t)r * d.c + ic) * d.kh + y) * d.kw + x];
  }));
  *out = op;
  return NNRCU_OK;
}

static int conv_f32_planes(nnrcu_op* op, const uint16_t* hi, const uint16_t* lo, float* y, const float* residual,
                           cudaStream_t st);

int nnrcu_conv_f32_run(nnrcu_op* op, const float* x, float* y, const float* residual, void* workspace, void* stream) {
  if (!op || (op->kind != OP_CONV_F32 && op->kind != OP_DWCONV_F32))
    return set_error(NNRCU_ERR_INVALID, "not an fp32 Conv operator");
  if (!x || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if (op->ws_bytes && !workspace)
    return set_error(NNRCU_ERR_INVALID, "workspace of %zu bytes required", op->ws_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const nnrcu_conv_desc& d = op->d;
  uint8_t* ws = static_cast<uint8_t*>(workspace);

  if (op->kind == OP_DWCONV_F32) {
    const float* xin = x;
    if (d.in_layout == NNRCU_LAYOUT_NCHW) {
      int rc = launch_transpose_generic(x, ws, d.n, d.c, d.h * d.w, 4, 1, st);
      if (rc != NNRCU_OK) return rc;
      xin = reinterpret_cast<const float*>(ws);
      ws += round_up_sz((size_t)d.n * d.h * d.w * d.c * 4, 256);
    }
    if (d.out_layout == NNRCU_LAYOUT_NHWC) return launch_depthwise_f32(*op, xin, y, residual, st);
    if (residual)
      return set_error(NNRCU_ERR_UNSUPPORTED, "depthwise Conv with NCHW output and a residual is not implemented");
    float* tmp = reinterpret_cast<float*>(ws);
    int rc = launch_depthwise_f32(*op, xin, tmp, nullptr, st);
    if (rc != NNRCU_OK) return rc;
    return launch_transpose_generic(tmp, y, d.n, d.oc, op->oh * op->ow, 4, 0, st);
  }

  const size_t plane = op->explicit_im2col ? round_up_sz((size_t)op->M * op->cs * 2, 256)
                                           : round_up_sz((size_t)d.n * d.h * d.w * op->cs * 2, 256);
  uint16_t* hi = reinterpret_cast<uint16_t*>(ws);
  uint16_t* lo = reinterpret_cast<uint16_t*>(ws + plane);
  int rc = op->explicit_im2col
               ? launch_im2col_split_bf16(x, d.in_layout == NNRCU_LAYOUT_NCHW, hi, lo, d.n, d.c, d.h, d.w, op->oh,
                                          op->ow, d.kh, d.kw, d.stride_h, d.stride_w, d.pad_top, d.pad_left, d.dil_h,
                                          d.dil_w, op->cs, st)
               : launch_split_bf16_nhwc(x, d.in_layout == NNRCU_LAYOUT_NCHW, hi, lo, d.n, d.c, d.h, d.w, op->cs, st);
  if (rc != NNRCU_OK) return rc;
  return conv_f32_planes(op, hi, lo, y, residual, st);
}

// The split-bf16 GEMM of a dense fp32 Conv over A planes already split
// (hi / lo, NHWC with channel stride op->cs, or the explicit im2col rows).
static int conv_f32_planes(nnrcu_op* op, const uint16_t* hi, const uint16_t* lo, float* y, const float* residual,
                           cudaStream_t st) {
  const nnrcu_conv_desc& d = op->d;
  int rc = NNRCU_OK;
  CUtensorMap tmA0{}, tmA1{};
  if (op->amode == A_TMA) {
    // rows: input pixels (1x1) or output pixels (explicit im2col)
    const uint64_t rows = op->explicit_im2col ? (uint64_t)op->M : (uint64_t)d.n * d.h * d.w;
    const CUtensorMapSwizzle sw = op->kslab == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    rc = encode_tmap_2d(&tmA0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, hi, op->cs, rows, op->cs * 2, op->kslab / 2, BM, sw);
    if (rc != NNRCU_OK) return rc;
    rc = encode_tmap_2d(&tmA1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lo, op->cs, rows, op->cs * 2, op->kslab / 2, BM, sw);
    if (rc != NNRCU_OK) return rc;
  } else if (op->amode == A_IM2COL) {
    rc = encode_tmap_im2col(&tmA0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hi, d.n, d.h, d.w, op->cs, d.pad_top,
                            d.pad_left, d.pad_bottom, d.pad_right, d.kh, d.kw, d.dil_h, d.dil_w, d.stride_h,
                            d.stride_w, BKB);
    if (rc != NNRCU_OK) return rc;
    rc = encode_tmap_im2col(&tmA1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, lo, d.n, d.h, d.w, op->cs, d.pad_top,
                            d.pad_left, d.pad_bottom, d.pad_right, d.kh, d.kw, d.dil_h, d.dil_w, d.stride_h,
                            d.stride_w, BKB);
    if (rc != NNRCU_OK) return rc;
  }
  GatherGeom g{};
  g.x = reinterpret_cast<const uint8_t*>(hi);
  g.x2 = reinterpret_cast<const uint8_t*>(lo);
  g.N = d.n; g.H = d.h; g.W = d.w;
  g.cbytes = op->cs * 2;
  g.OH = op->oh; g.OW = op->ow; g.KH = d.kh; g.KW = d.kw;
  g.sh = d.stride_h; g.sw = d.stride_w; g.ph = d.pad_top; g.pw = d.pad_left; g.dh = d.dil_h; g.dw = d.dil_w;
  g.kbytes = op->kbytes;
  g.pad_word = 0;
  EpiParams e{};
  e.M = op->M; e.N = op->N;
  e.bias = op->bias;
  e.residual = residual;
  e.res_mode = residual ? 2 : 0;
  e.res_scale = 1.0f;
  e.act = op->act; e.act_a = op->act_a; e.act_b = op->act_b;
  e.y = y;
  e.y_layout = d.out_layout == NNRCU_LAYOUT_NCHW ? 1 : 0;
  e.ldy = d.oc;
  e.ohw = op->oh * op->ow;
  e.status = status_ptr();
  TcLaunch L{};
  L.bn = op->bn; L.nplane = 2; L.amode = op->amode; L.epi = EPI_F32;
  L.m_tiles = (op->M + BM - 1) / BM;
  L.n_tiles = (op->N + op->bn - 1) / op->bn;
  L.tmA0 = &tmA0; L.tmA1 = &tmA1; L.tmB = &op->tmB;
  L.b_plane_rows = op->npad;
  L.num_kb = op->num_kb;
  L.kb_bytes = op->kslab;
  return tc_launch(L, g, e, st);
}

int nnrcu_conv_f32_plane_stride(const nnrcu_op* op, int* cs) {
  if (!op || !cs) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  if (op->kind != OP_CONV_F32 || op->explicit_im2col || op->amode != A_TMA || op->d.in_layout != NNRCU_LAYOUT_NHWC)
    return set_error(NNRCU_ERR_UNSUPPORTED, "only a 1x1 stride-1 NHWC fp32 Conv reads pre-split planes");
  *cs = op->cs;
  return NNRCU_OK;
}

int nnrcu_conv_f32_run_planes(nnrcu_op* op, const uint16_t* x_hi, const uint16_t* x_lo, float* y,
                              const float* residual, void* stream) {
  int cs = 0;
  int rc = nnrcu_conv_f32_plane_stride(op, &cs);
  if (rc != NNRCU_OK) return rc;
  if (!x_hi || !x_lo || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if ((reinterpret_cast<uintptr_t>(x_hi) | reinterpret_cast<uintptr_t>(x_lo)) & 15)
    return set_error(NNRCU_ERR_INVALID, "the planes must be 16-byte aligned");
  return conv_f32_planes(op, x_hi, x_lo, y, residual, static_cast<cudaStream_t>(stream));
}

int nnrcu_conv_f32_run_to_planes(nnrcu_op* op, const float* x, uint16_t* y_hi, uint16_t* y_lo, int cs,
                                 void* stream) {
  if (!op || op->kind != OP_DWCONV_F32) return set_error(NNRCU_ERR_INVALID, "not an fp32 depthwise Conv operator");
  if (!x || !y_hi || !y_lo) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if (op->d.in_layout != NNRCU_LAYOUT_NHWC || op->d.out_layout != NNRCU_LAYOUT_NHWC)
    return set_error(NNRCU_ERR_UNSUPPORTED, "planes output needs NHWC input and output");
  if (cs < op->d.oc || cs % 4 != 0)
    return set_error(NNRCU_ERR_INVALID, "plane channel stride %d must be a multiple of 4 and >= %d", cs, op->d.oc);
  if ((reinterpret_cast<uintptr_t>(y_hi) | reinterpret_cast<uintptr_t>(y_lo)) & 7)
    return set_error(NNRCU_ERR_INVALID, "the planes must be 8-byte aligned");
  return launch_depthwise_f32_planes(*op, x, y_hi, y_lo, cs, static_cast<cudaStream_t>(stream));
}

int nnrcu_gemm_f32_create(int m, int n, int k, int trans_a, int trans_b, float alpha, float beta, const float* b_host,
                          const float* c_host, int c_rows, int post_op, float post_a, float post_b, nnrcu_op** out) {
  if (!b_host || !out) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  *out = nullptr;
  if (m <= 0 || n <= 0 || k <= 0) return set_error(NNRCU_ERR_INVALID, "Gemm dims must be positive");
  if (c_host && c_rows != 1 && c_rows != m)
    return set_error(NNRCU_ERR_UNSUPPORTED, "Gemm C must be a [n] row or a full [m, n] matrix (c_rows=%d)", c_rows);
  nnrcu_op* op = new nnrcu_op();
  NNRCU_TRY(cuda_check(cudaGetDevice(&op->device), "cudaGetDevice"));
  op->kind = OP_GEMM_F32;
  op->M = m; op->N = n; op->K = k;
  op->nplane = 2;
  op->epi = EPI_F32;
  op->trans_a = trans_a;
  op->cs = round_up(k, 8);       // bf16 elements per A row on the device
  op->kbytes = op->cs * 2;
  op->kpad_bytes = round_up(op->kbytes, BKB);
  op->num_kb = op->kpad_bytes / BKB;
  op->npad = round_up(n, 256);
  op->bn = pick_bn(m, n, 2, num_sms());
  op->amode = op->kbytes >= BKB ? A_TMA : A_GATHER;
  op->num_ops = 2LL * m * n * (long long)k;
  op->beta = beta;
  op->c_rows = c_host ? c_rows : 0;
  op->ws_bytes = 2 * round_up_sz((size_t)m * op->cs * 2, 256);
  NNRCU_TRY(map_post(post_op, post_a, post_b, op));
  // alpha is folded into the packed B.
  NNRCU_TRY(pack_split_planes(op, n, k, [&](int r, int kk) -> float {
    const float v = trans_b ? b_host[(size_t)r * k + kk] : b_host[(size_t)kk * n + r];
    return alpha * v;
  }));
  if (c_host && c_rows == 1) {
    std::vector<float> b(n);
    for (int j = 0; j < n; ++j) b[j] = beta * c_host[j];
    NNRCU_TRY(upload_vec(&op->bias, b));
  } else if (c_host) {
    NNRCU_TRY(upload_vec(&op->cmat, std::vector<float>(c_host, c_host + (size_t)m * n)));
  }
  *out = op;
  return NNRCU_OK;
}

int nnrcu_gemm_f32_run(nnrcu_op* op, const float* a, float* y, void* workspace, void* stream) {
  if (op && op->kind == OP_GEMM_F32_BF16) {
    if (!a || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
    return gemm_f32_bf16_run(op, a, y, workspace, static_cast<cudaStream_t>(stream));
  }
  if (!op || op->kind != OP_GEMM_F32) return set_error(NNRCU_ERR_INVALID, "not a Gemm operator");
  if (!a || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if (!workspace) return set_error(NNRCU_ERR_INVALID, "workspace of %zu bytes required", op->ws_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t plane = round_up_sz((size_t)op->M * op->cs * 2, 256);
  uint16_t* hi = reinterpret_cast<uint16_t*>(ws);
  uint16_t* lo = reinterpret_cast<uint16_t*>(ws + plane);
  int rc = launch_split_bf16_rows(a, op->trans_a, hi, lo, op->M, op->K, op->cs, st);
  if (rc != NNRCU_OK) return rc;
  CUtensorMap tmA0{}, tmA1{};
  if (op->amode == A_TMA) {
    rc = encode_tmap_2d(&tmA0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, hi, op->cs, op->M, op->cs * 2, BKB / 2, BM);
    if (rc != NNRCU_OK) return rc;
    rc = encode_tmap_2d(&tmA1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lo, op->cs, op->M, op->cs * 2, BKB / 2, BM);
    if (rc != NNRCU_OK) return rc;
  }
  GatherGeom g{};
  g.x = reinterpret_cast<const uint8_t*>(hi);
  g.x2 = reinterpret_cast<const uint8_t*>(lo);
  g.N = 1; g.H = 1; g.W = op->M;
  g.cbytes = op->cs * 2;
  g.OH = 1; g.OW = op->M; g.KH = 1; g.KW = 1; g.sh = 1; g.sw = 1; g.ph = 0; g.pw = 0; g.dh = 1; g.dw = 1;
  g.kbytes = op->kbytes;
  EpiParams e{};
  e.M = op->M; e.N = op->N;
  e.bias = op->bias;
  e.residual = op->cmat;
  e.res_mode = op->cmat ? 1 : 0;
  e.res_scale = op->beta;
  e.act = op->act; e.act_a = op->act_a; e.act_b = op->act_b;
  e.y = y;
  e.y_layout = 0;
  e.ldy = op->N;
  e.ohw = 1;
  e.status = status_ptr();
  TcLaunch L{};
  L.bn = op->bn; L.nplane = 2; L.amode = op->amode; L.epi = EPI_F32;
  L.m_tiles = (op->M + BM - 1) / BM;
  L.n_tiles = (op->N + op->bn - 1) / op->bn;
  L.tmA0 = &tmA0; L.tmA1 = &tmA1; L.tmB = &op->tmB;
  L.b_plane_rows = op->npad;
  L.num_kb = op->num_kb;
  return tc_launch(L, g, e, st);
}

namespace {
struct MatmulGeom {
  int cs, kbytes, kpad_bytes, num_kb, npad;
  size_t a_plane, b_plane;
};
MatmulGeom matmul_geom(int m, int n, int k) {
  MatmulGeom g;
  g.cs = round_up(k, 8);  // bf16 elements per operand row
  g.kbytes = g.cs * 2;
  g.kpad_bytes = round_up(g.kbytes, BKB);
  g.num_kb = g.kpad_bytes / BKB;
  g.npad = round_up(n, 256);
  g.a_plane = round_up_sz((size_t)m * g.cs * 2, 256);
  g.b_plane = round_up_sz((size_t)g.npad * g.cs * 2, 256);
  return g;
}
}  // namespace

int nnrcu_matmul_f32_workspace(int m, int n, int k, size_t* bytes) {
  if (!bytes || m <= 0 || n <= 0 || k <= 0) return set_error(NNRCU_ERR_INVALID, "MatMul dims must be positive");
  const MatmulGeom g = matmul_geom(m, n, k);
  *bytes = 2 * g.a_plane + 2 * g.b_plane;
  return NNRCU_OK;
}

int nnrcu_matmul_f32_run(const float* a, const float* b, float* y, int batch, int m, int n, int k,
                         long long a_batch_stride, long long b_batch_stride, int post_op, float post_a, float post_b,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!a || !b || !y || !workspace) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  if (batch <= 0 || m <= 0 || n <= 0 || k <= 0 || a_batch_stride < 0 || b_batch_stride < 0)
    return set_error(NNRCU_ERR_INVALID, "MatMul: dims must be positive and strides non-negative");
  const MatmulGeom mg = matmul_geom(m, n, k);
  if (workspace_bytes < 2 * mg.a_plane + 2 * mg.b_plane)
    return set_error(NNRCU_ERR_INVALID, "MatMul workspace of %zu bytes required", 2 * mg.a_plane + 2 * mg.b_plane);
  nnrcu_op post{};  // carries the mapped post-op only
  int rc = map_post(post_op, post_a, post_b, &post);
  if (rc != NNRCU_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* ahi = reinterpret_cast<uint16_t*>(ws);
  uint16_t* alo = reinterpret_cast<uint16_t*>(ws + mg.a_plane);
  uint16_t* bhi = reinterpret_cast<uint16_t*>(ws + 2 * mg.a_plane);  // [2][npad][cs]: hi rows, then lo rows
  uint16_t* blo = bhi + (size_t)mg.npad * mg.cs;
  const int amode = mg.kbytes >= BKB ? A_TMA : A_GATHER;
  const int bn = pick_bn(m, n, 2, num_sms());
  CUtensorMap tmA0{}, tmA1{}, tmB{};
  if (amode == A_TMA) {
    rc = encode_tmap_2d(&tmA0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, ahi, mg.cs, m, mg.cs * 2, BKB / 2, BM);
    if (rc != NNRCU_OK) return rc;
    rc = encode_tmap_2d(&tmA1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, alo, mg.cs, m, mg.cs * 2, BKB / 2, BM);
    if (rc != NNRCU_OK) return rc;
  }
  // B planes: rows past n are never written; they only feed output columns
  // past n, which are not stored. K past cs is the map's zero fill.
  rc = encode_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, bhi, mg.cs, (uint64_t)2 * mg.npad, mg.cs * 2, BKB / 2, bn);
  if (rc != NNRCU_OK) return rc;
  GatherGeom g{};
  g.x = reinterpret_cast<const uint8_t*>(ahi);
  g.x2 = reinterpret_cast<const uint8_t*>(alo);
  g.N = 1; g.H = 1; g.W = m;
  g.cbytes = mg.cs * 2;
  g.OH = 1; g.OW = m; g.KH = 1; g.KW = 1; g.sh = 1; g.sw = 1; g.ph = 0; g.pw = 0; g.dh = 1; g.dw = 1;
  g.kbytes = mg.kbytes;
  EpiParams e{};
  e.M = m; e.N = n;
  e.act = post.act; e.act_a = post.act_a; e.act_b = post.act_b;
  e.y_layout = 0;
  e.ldy = n;
  e.ohw = 1;
  e.status = status_ptr();
  TcLaunch L{};
  L.bn = bn; L.nplane = 2; L.amode = amode; L.epi = EPI_F32;
  L.m_tiles = (m + BM - 1) / BM;
  L.n_tiles = (n + bn - 1) / bn;
  L.tmA0 = &tmA0; L.tmA1 = &tmA1; L.tmB = &tmB;
  L.b_plane_rows = mg.npad;
  L.num_kb = mg.num_kb;
  for (int bi = 0; bi < batch; ++bi) {
    // (a broadcast operand is split once)
    if (bi == 0 || a_batch_stride)
      if ((rc = launch_split_bf16_rows(a + a_batch_stride * bi, 0, ahi, alo, m, k, mg.cs, st)) != NNRCU_OK) return rc;
    if (bi == 0 || b_batch_stride)
      if ((rc = launch_split_bf16_rows(b + b_batch_stride * bi, 1, bhi, blo, n, k, mg.cs, st)) != NNRCU_OK) return rc;
    e.y = y + (size_t)bi * m * n;
    if ((rc = tc_launch(L, g, e, st)) != NNRCU_OK) return rc;
  }
  return NNRCU_OK;
}

}  // extern "C"
