// 16-bit Conv / Gemm / MatMul on one bf16 or fp16 plane (tcgen05 kind::f16,
// fp32 accumulation), the device form of nnr's 16-bit I/O paths:
//   Conv_exec_entry.h:188-381 (exec_f16_as_f32 / exec_bf16_as_f32) and
//   Gemm.cpp:297-513 convert the 16-bit inputs to fp32, compute in fp32,
//   apply the post-op and round the result back to the 16-bit type.
// A product of two 16-bit values is exact in fp32, so one kind::f16 MMA per
// multiply-add with fp32 accumulation computes the same fp32 sums (up to the
// summation order); the epilogue's fp32 result is rounded to the 16-bit type
// (round to nearest even) by a second pass.
//
// nnrcu_gemm_f32_create_ex(..., NNRCU_PREC_BF16) is nnr's fp32 MatMul as it
// runs on hosts with AVX-512 BF16 (MatMul.cpp:128-152 packs a constant B to
// bf16, :382-428 rounds A to bf16 and runs VDPBF16PS): both operands rounded
// to bf16 (nearest even), one product each, fp32 accumulation.
#include <algorithm>
#include <cstring>
#include <vector>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"
#include "tc_gemm.cuh"

namespace nnrcu {
int conv_out_dims(const nnrcu_conv_desc& d, int* oh, int* ow);

namespace {

inline int round_up(int v, int a) { return (v + a - 1) / a * a; }
inline size_t round_up_sz(size_t v, size_t a) { return (v + a - 1) / a * a; }
int blocks(long long total, int threads) {
  return (int)std::max<long long>(1, std::min<long long>((total + threads - 1) / threads, (long long)num_sms() * 32));
}

// 16-bit activations, NCHW or NHWC [n, c, h, w] -> NHWC with channel stride cs (zero padded)
__global__ void half_to_nhwc_kernel(const uint16_t* __restrict src, int src_nchw, uint16_t* __restrict dst, int n,
                                    int c, int hw, int cs) {
  const long long total = (long long)n * hw * cs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % cs);
    const long long p = i / cs;  // n * hw + pixel
    uint16_t v = 0;
    if (ch < c) {
      const long long img = p / hw, pix = p - img * hw;
      v = src_nchw ? src[((size_t)img * c + ch) * hw + pix] : src[(size_t)p * c + ch];
    }
    dst[i] = v;
  }
}

// rows of A [m, k] (or A^T stored [k, m]) -> [m][kp] 16-bit, zero padded;
// from 16-bit (f32src = 0) or from fp32 rounded to bf16 (f32src = 1)
__global__ void rows_to_half_kernel(const void* __restrict src, int f32src, int trans, uint16_t* __restrict dst, int m,
                                    int k, int kp) {
  const long long total = (long long)m * kp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / kp), kk = (int)(i - (long long)r * kp);
    uint16_t v = 0;
    if (kk < k) {
      const size_t at = trans ? (size_t)kk * m + r : (size_t)r * k + kk;
      if (f32src) {
        const __nv_bfloat16 b = __float2bfloat16_rn(static_cast<const float*>(src)[at]);
        v = *reinterpret_cast<const uint16_t*>(&b);
      } else {
        v = static_cast<const uint16_t*>(src)[at];
      }
    }
    dst[i] = v;
  }
}

// fp32 -> bf16 (dtype 0) or fp16 (dtype 1), round to nearest even
__global__ void f32_to_half_kernel(const float* __restrict src, uint16_t* __restrict dst, long long n, int dtype) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    if (dtype == 0) {
      const __nv_bfloat16 b = __float2bfloat16_rn(src[i]);
      dst[i] = *reinterpret_cast<const uint16_t*>(&b);
    } else {
      const __half h = __float2half_rn(src[i]);
      dst[i] = *reinterpret_cast<const uint16_t*>(&h);
    }
  }
}

float half_to_float_host(uint16_t v, int dtype) {
  if (dtype == NNRCU_DT_BF16) {
    const uint32_t u = (uint32_t)v << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  }
  // IEEE binary16 -> binary32 (exact)
  const uint32_t sign = (uint32_t)(v & 0x8000u) << 16;
  uint32_t exp = (v >> 10) & 0x1Fu, man = v & 0x3FFu, u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else {  // subnormal: normalise
      exp = 127 - 15 + 1;
      while (!(man & 0x400u)) { man <<= 1; --exp; }
      u = sign | (exp << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7F800000u | (man << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t float_to_bf16_host(float v) {  // round to nearest even (NaN kept quiet)
  uint32_t u;
  std::memcpy(&u, &v, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

int map_post_half(int post_op, float a, float b, Op* op) {
  static const int acts[] = {ACT_NONE, ACT_RELU, ACT_CLIP, ACT_HARDSWISH, ACT_SIGMOID, ACT_LEAKYRELU, ACT_TANH};
  if (post_op < 0 || post_op > NNRCU_POST_TANH) return set_error(NNRCU_ERR_INVALID, "unknown post-op %d", post_op);
  op->act = acts[post_op];
  op->act_a = a;
  op->act_b = b;
  return NNRCU_OK;
}

CUtensorMapDataType tmap_type(int nplane) {
  return nplane == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// B [npad][kpad_bytes / 2] 16-bit, K-major; get(r, kk) returns the 16-bit bits
template <typename F>
int pack_half_b(Op* op, int rows, int k, F get) {
  const size_t kpe = op->kpad_bytes / 2;
  std::vector<uint16_t> B((size_t)op->npad * kpe, 0);
  for (int r = 0; r < rows; ++r)
    for (int kk = 0; kk < k; ++kk) B[(size_t)r * kpe + kk] = get(r, kk);
  NNRCU_CUDA(cudaMalloc(&op->wB, B.size() * 2));
  NNRCU_CUDA(cudaMemcpy(op->wB, B.data(), B.size() * 2, cudaMemcpyHostToDevice));
  return encode_tmap_2d(&op->tmB, tmap_type(op->nplane), op->wB, kpe, (uint64_t)op->npad, op->kpad_bytes, BKB / 2,
                        op->bn, CU_TENSOR_MAP_SWIZZLE_128B);
}

int upload_f32(float** dst, const std::vector<float>& v) {
  NNRCU_CUDA(cudaMalloc(reinterpret_cast<void**>(dst), std::max<size_t>(4, v.size() * 4)));
  NNRCU_CUDA(cudaMemcpy(*dst, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  return NNRCU_OK;
}

// one engine launch over a prepared 16-bit A (rows of cs elements, or NHWC pixels)
int half_launch(Op* op, const uint16_t* a, int a_rows, const GatherGeom& g0, float* y32, int y_layout, int ldy,
                int ohw, cudaStream_t st) {
  CUtensorMap tmA{};
  if (op->amode == A_TMA) {
    int rc = encode_tmap_2d(&tmA, tmap_type(op->nplane), a, op->cs, (uint64_t)a_rows, (uint64_t)op->cs * 2, BKB / 2,
                            BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != NNRCU_OK) return rc;
  }
  GatherGeom g = g0;
  g.x = reinterpret_cast<const uint8_t*>(a);
  g.x2 = nullptr;
  g.cbytes = op->cs * 2;
  g.kbytes = op->kbytes;
  g.pad_word = 0;
  EpiParams e{};
  e.M = op->M;
  e.N = op->N;
  e.bias = op->bias;
  e.residual = op->cmat;
  e.res_mode = op->cmat ? 1 : 0;
  e.res_scale = op->beta;
  e.act = op->act;
  e.act_a = op->act_a;
  e.act_b = op->act_b;
  e.y = y32;
  e.y_layout = y_layout;
  e.ldy = ldy;
  e.ohw = ohw;
  e.status = status_ptr();
  TcLaunch L{};
  L.bn = op->bn;
  L.nplane = op->nplane;
  L.amode = op->amode;
  L.epi = EPI_F32;
  L.m_tiles = (op->M + BM - 1) / BM;
  L.n_tiles = (op->N + op->bn - 1) / op->bn;
  L.tmA0 = &tmA;
  L.tmA1 = &tmA;
  L.tmB = &op->tmB;
  L.b_plane_rows = op->npad;
  L.num_kb = op->num_kb;
  L.kb_bytes = BKB;
  return tc_launch(L, g, e, st);
}

int to_half(const float* y32, uint16_t* y, size_t n, int dtype, cudaStream_t st) {
  f32_to_half_kernel<<<blocks((long long)n, 256), 256, 0, st>>>(y32, y, (long long)n, dtype == NNRCU_DT_BF16 ? 0 : 1);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

}  // namespace
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

int nnrcu_conv_half_create(const nnrcu_conv_desc* desc, int dtype, const uint16_t* w_host, const uint16_t* bias_host,
                           nnrcu_op** out) {
  if (!desc || !w_host || !out) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  if (dtype != NNRCU_DT_BF16 && dtype != NNRCU_DT_F16) return set_error(NNRCU_ERR_INVALID, "dtype must be bf16 or fp16");
  *out = nullptr;
  const nnrcu_conv_desc& d = *desc;
  int oh = 0, ow = 0;
  int rc = conv_out_dims(d, &oh, &ow);
  if (rc != NNRCU_OK) return rc;
  // depthwise with whole 4-channel vectors: the fp32 depthwise kernels with
  // 16-bit loads and stores (nnr widens 16-bit tensors around its fp32
  // depthwise conv, Conv_exec_entry.h:188-381, Conv_depthwise.h:11)
  if (d.group == d.c && d.group == d.oc && d.group > 1 && d.c % 4 == 0) {
    nnrcu_op* op = new nnrcu_op();
    NNRCU_TRY(cuda_check(cudaGetDevice(&op->device), "cudaGetDevice"));
    op->kind = OP_CONV_HALF;
    op->d = d;
    op->oh = oh;
    op->ow = ow;
    op->M = d.n * oh * ow;
    op->N = d.oc;
    op->K = d.kh * d.kw;
    op->num_ops = 2LL * op->M * d.oc * (long long)op->K;
    op->nplane = dtype == NNRCU_DT_BF16 ? 3 : 4;
    NNRCU_TRY(map_post_half(d.post_op, d.post_a, d.post_b, op));
    std::vector<float> w((size_t)d.kh * d.kw * d.c);
    for (int ch = 0; ch < d.c; ++ch)
      for (int t = 0; t < d.kh * d.kw; ++t) w[(size_t)t * d.c + ch] = half_to_float_host(w_host[(size_t)ch * d.kh * d.kw + t], dtype);
    NNRCU_TRY(upload_f32(&op->w_dw, w));
    if (bias_host) {
      std::vector<float> b(d.oc);
      for (int i = 0; i < d.oc; ++i) b[i] = half_to_float_host(bias_host[i], dtype);
      NNRCU_TRY(upload_f32(&op->bias, b));
    }
    // workspace: the NHWC copy of an NCHW input, then the NHWC result of an NCHW output
    op->out_off = d.in_layout == NNRCU_LAYOUT_NCHW ? round_up_sz((size_t)d.n * d.h * d.w * d.c * 2, 256) : 0;
    op->ws_bytes = op->out_off + (d.out_layout == NNRCU_LAYOUT_NCHW ? (size_t)op->M * d.oc * 2 : 0);
    *out = op;
    return NNRCU_OK;
  }
  if (d.group != 1) {
    if (d.c % d.group || d.oc % d.group)
      return set_error(NNRCU_ERR_INVALID, "group %d does not divide channels %d / %d", d.group, d.c, d.oc);
    const std::vector<uint16_t> dense = grouped_to_dense(w_host, d.oc, d.c, d.group, d.kh, d.kw);
    nnrcu_conv_desc d1 = d;
    d1.group = 1;
    rc = nnrcu_conv_half_create(&d1, dtype, dense.data(), bias_host, out);
    if (rc == NNRCU_OK) (*out)->num_ops /= d.group;
    return rc;
  }
  nnrcu_op* op = new nnrcu_op();
  NNRCU_TRY(cuda_check(cudaGetDevice(&op->device), "cudaGetDevice"));
  op->kind = OP_CONV_HALF;
  op->d = d;
  op->oh = oh;
  op->ow = ow;
  op->M = d.n * oh * ow;
  op->N = d.oc;
  op->K = d.kh * d.kw * d.c;
  op->num_ops = 2LL * op->M * d.oc * (long long)op->K;
  op->nplane = dtype == NNRCU_DT_BF16 ? 3 : 4;
  op->epi = EPI_F32;
  op->kslab = BKB;
  op->cs = round_up(d.c, 8);  // 16-byte pixel stride
  const bool one_by_one = d.kh == 1 && d.kw == 1 && d.stride_h == 1 && d.stride_w == 1 && d.pad_top == 0 &&
                          d.pad_left == 0 && d.pad_bottom == 0 && d.pad_right == 0;
  op->kbytes = d.kh * d.kw * op->cs * 2;
  op->kpad_bytes = round_up(op->kbytes, BKB);
  op->num_kb = op->kpad_bytes / BKB;
  op->npad = round_up(d.oc, 256);
  op->bn = pick_bn(op->M, op->N, 1, num_sms());
  op->amode = (one_by_one && op->cs >= 64) ? A_TMA : A_GATHER;
  NNRCU_TRY(map_post_half(d.post_op, d.post_a, d.post_b, op));
  if (bias_host) {
    std::vector<float> b(d.oc);
    for (int i = 0; i < d.oc; ++i) b[i] = half_to_float_host(bias_host[i], dtype);
    NNRCU_TRY(upload_f32(&op->bias, b));
  }
  // workspace: the NHWC 16-bit input, then the fp32 result
  op->out_off = round_up_sz((size_t)d.n * d.h * d.w * op->cs * 2, 256);
  op->ws_bytes = op->out_off + (size_t)op->M * d.oc * 4;
  const int cs = op->cs;
  NNRCU_TRY(pack_half_b(op, d.oc, op->kpad_bytes / 2, [&](int r, int kk) -> uint16_t {
    const int tap = kk / cs, ic = kk - tap * cs;
    if (tap >= d.kh * d.kw || ic >= d.c) return 0;
    const int y = tap / d.kw, x = tap - y * d.kw;
    return w_host[(((size_t)r * d.c + ic) * d.kh + y) * d.kw + x];
  }));
  *out = op;
  return NNRCU_OK;
}

int nnrcu_conv_half_run(nnrcu_op* op, const uint16_t* x, uint16_t* y, void* workspace, void* stream) {
  if (!op || op->kind != OP_CONV_HALF) return set_error(NNRCU_ERR_INVALID, "not a 16-bit Conv operator");
  if (!x || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if (op->ws_bytes && !workspace) return set_error(NNRCU_ERR_INVALID, "workspace of %zu bytes required", op->ws_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const nnrcu_conv_desc& d = op->d;
  const int dtype = op->nplane == 3 ? NNRCU_DT_BF16 : NNRCU_DT_F16;
  if (op->w_dw) {  // depthwise
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const uint16_t* xin = x;
    if (d.in_layout == NNRCU_LAYOUT_NCHW) {
      int rc = launch_transpose_generic(x, ws, d.n, d.c, d.h * d.w, 2, 1, st);
      if (rc != NNRCU_OK) return rc;
      xin = reinterpret_cast<const uint16_t*>(ws);
    }
    if (d.out_layout == NNRCU_LAYOUT_NHWC) return launch_depthwise_half(*op, xin, y, dtype, st);
    uint16_t* tmp = reinterpret_cast<uint16_t*>(ws + op->out_off);
    int rc = launch_depthwise_half(*op, xin, tmp, dtype, st);
    if (rc != NNRCU_OK) return rc;
    return launch_transpose_generic(tmp, y, d.n, d.oc, op->oh * op->ow, 2, 0, st);
  }
  uint16_t* a = static_cast<uint16_t*>(workspace);
  float* y32 = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + op->out_off);
  const long long total = (long long)d.n * d.h * d.w * op->cs;
  half_to_nhwc_kernel<<<blocks(total, 256), 256, 0, st>>>(x, d.in_layout == NNRCU_LAYOUT_NCHW, a, d.n, d.c, d.h * d.w,
                                                         op->cs);
  NNRCU_CUDA(cudaGetLastError());
  GatherGeom g{};
  g.N = d.n; g.H = d.h; g.W = d.w;
  g.OH = op->oh; g.OW = op->ow; g.KH = d.kh; g.KW = d.kw;
  g.sh = d.stride_h; g.sw = d.stride_w; g.ph = d.pad_top; g.pw = d.pad_left; g.dh = d.dil_h; g.dw = d.dil_w;
  int rc = half_launch(op, a, d.n * d.h * d.w, g, y32, d.out_layout == NNRCU_LAYOUT_NCHW ? 1 : 0, d.oc,
                       op->oh * op->ow, st);
  if (rc != NNRCU_OK) return rc;
  return to_half(y32, y, (size_t)op->M * d.oc, dtype, st);
}

int nnrcu_gemm_half_create(int m, int n, int k, int trans_a, int trans_b, float alpha, float beta, int dtype,
                           const uint16_t* b_host, const uint16_t* c_host, int c_rows, int post_op, float post_a,
                           float post_b, nnrcu_op** out) {
  if (!b_host || !out) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  if (dtype != NNRCU_DT_BF16 && dtype != NNRCU_DT_F16) return set_error(NNRCU_ERR_INVALID, "dtype must be bf16 or fp16");
  *out = nullptr;
  if (m <= 0 || n <= 0 || k <= 0) return set_error(NNRCU_ERR_INVALID, "Gemm dims must be positive");
  if (alpha != 1.0f)
    return set_error(NNRCU_ERR_UNSUPPORTED, "16-bit Gemm with alpha != 1 is not implemented on the device");
  if (c_host && c_rows != 1 && c_rows != m)
    return set_error(NNRCU_ERR_UNSUPPORTED, "Gemm C must be a [n] row or a full [m, n] matrix (c_rows=%d)", c_rows);
  nnrcu_op* op = new nnrcu_op();
  NNRCU_TRY(cuda_check(cudaGetDevice(&op->device), "cudaGetDevice"));
  op->kind = OP_GEMM_HALF;
  op->M = m; op->N = n; op->K = k;
  op->nplane = dtype == NNRCU_DT_BF16 ? 3 : 4;
  op->epi = EPI_F32;
  op->trans_a = trans_a;
  op->cs = round_up(k, 8);
  op->kbytes = op->cs * 2;
  op->kpad_bytes = round_up(op->kbytes, BKB);
  op->num_kb = op->kpad_bytes / BKB;
  op->npad = round_up(n, 256);
  op->bn = pick_bn(m, n, 1, num_sms());
  op->amode = op->kbytes >= BKB ? A_TMA : A_GATHER;
  op->num_ops = 2LL * m * n * (long long)k;
  op->beta = beta;
  NNRCU_TRY(map_post_half(post_op, post_a, post_b, op));
  NNRCU_TRY(pack_half_b(op, n, k, [&](int r, int kk) -> uint16_t {
    return trans_b ? b_host[(size_t)r * k + kk] : b_host[(size_t)kk * n + r];
  }));
  if (c_host && c_rows == 1) {  // beta * C as an fp32 bias row (one rounding, as nnr's fp32 beta * c)
    std::vector<float> b(n);
    for (int j = 0; j < n; ++j) b[j] = beta * half_to_float_host(c_host[j], dtype);
    NNRCU_TRY(upload_f32(&op->bias, b));
  } else if (c_host) {
    std::vector<float> c((size_t)m * n);
    for (size_t i = 0; i < c.size(); ++i) c[i] = half_to_float_host(c_host[i], dtype);
    NNRCU_TRY(upload_f32(&op->cmat, c));
  }
  op->out_off = round_up_sz((size_t)m * op->cs * 2, 256);
  op->ws_bytes = op->out_off + (size_t)m * n * 4;
  *out = op;
  return NNRCU_OK;
}

int nnrcu_gemm_half_run(nnrcu_op* op, const uint16_t* a, uint16_t* y, void* workspace, void* stream) {
  if (!op || op->kind != OP_GEMM_HALF) return set_error(NNRCU_ERR_INVALID, "not a 16-bit Gemm operator");
  if (!a || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if (!workspace) return set_error(NNRCU_ERR_INVALID, "workspace of %zu bytes required", op->ws_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint16_t* ap = static_cast<uint16_t*>(workspace);
  float* y32 = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + op->out_off);
  rows_to_half_kernel<<<blocks((long long)op->M * op->cs, 256), 256, 0, st>>>(a, 0, op->trans_a, ap, op->M, op->K,
                                                                            op->cs);
  NNRCU_CUDA(cudaGetLastError());
  GatherGeom g{};
  g.N = 1; g.H = 1; g.W = op->M; g.OH = 1; g.OW = op->M; g.KH = 1; g.KW = 1;
  g.sh = 1; g.sw = 1; g.ph = 0; g.pw = 0; g.dh = 1; g.dw = 1;
  int rc = half_launch(op, ap, op->M, g, y32, 0, op->N, 1, st);
  if (rc != NNRCU_OK) return rc;
  return to_half(y32, y, (size_t)op->M * op->N, op->nplane == 3 ? NNRCU_DT_BF16 : NNRCU_DT_F16, st);
}

int nnrcu_gemm_f32_create_ex(int m, int n, int k, int trans_a, int trans_b, float alpha, float beta,
                             const float* b_host, const float* c_host, int c_rows, int post_op, float post_a,
                             float post_b, int precision, nnrcu_op** out) {
  if (precision == NNRCU_PREC_SPLIT_BF16)
    return nnrcu_gemm_f32_create(m, n, k, trans_a, trans_b, alpha, beta, b_host, c_host, c_rows, post_op, post_a,
                                 post_b, out);
  if (precision != NNRCU_PREC_BF16) return set_error(NNRCU_ERR_INVALID, "unknown precision %d", precision);
  if (!b_host || !out) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  *out = nullptr;
  if (m <= 0 || n <= 0 || k <= 0) return set_error(NNRCU_ERR_INVALID, "Gemm dims must be positive");
  if (c_host && c_rows != 1 && c_rows != m)
    return set_error(NNRCU_ERR_UNSUPPORTED, "Gemm C must be a [n] row or a full [m, n] matrix (c_rows=%d)", c_rows);
  nnrcu_op* op = new nnrcu_op();
  NNRCU_TRY(cuda_check(cudaGetDevice(&op->device), "cudaGetDevice"));
  op->kind = OP_GEMM_F32_BF16;
  op->M = m; op->N = n; op->K = k;
  op->nplane = 3;
  op->epi = EPI_F32;
  op->trans_a = trans_a;
  op->cs = round_up(k, 8);
  op->kbytes = op->cs * 2;
  op->kpad_bytes = round_up(op->kbytes, BKB);
  op->num_kb = op->kpad_bytes / BKB;
  op->npad = round_up(n, 256);
  op->bn = pick_bn(m, n, 1, num_sms());
  op->amode = op->kbytes >= BKB ? A_TMA : A_GATHER;
  op->num_ops = 2LL * m * n * (long long)k;
  op->beta = beta;
  NNRCU_TRY(map_post_half(post_op, post_a, post_b, op));
  NNRCU_TRY(pack_half_b(op, n, k, [&](int r, int kk) -> uint16_t {
    const float v = trans_b ? b_host[(size_t)r * k + kk] : b_host[(size_t)kk * n + r];
    return float_to_bf16_host(alpha * v);
  }));
  if (c_host && c_rows == 1) {
    std::vector<float> b(n);
    for (int j = 0; j < n; ++j) b[j] = beta * c_host[j];
    NNRCU_TRY(upload_f32(&op->bias, b));
  } else if (c_host) {
    NNRCU_TRY(upload_f32(&op->cmat, std::vector<float>(c_host, c_host + (size_t)m * n)));
  }
  op->ws_bytes = round_up_sz((size_t)m * op->cs * 2, 256);
  *out = op;
  return NNRCU_OK;
}

// MatMul of two 16-bit device tensors computed at run time (nnr's MatMul
// with a non-initializer B on bf16 / fp16 tensors: MatMul.cpp:32-94 shapes,
// exec_f16_as_f32 and its bf16 twin convert to fp32, multiply, round back).
// Per batch: A rows and B's columns (transposed) to K-major 16-bit planes,
// one kind::f16 engine launch into an fp32 buffer, rounding to the type.
namespace {
struct HalfMM {
  int cs, kbytes, kpad_bytes, num_kb, npad;
  size_t a_plane, b_plane, y32;
};
HalfMM half_mm_geom(int m, int n, int k) {
  HalfMM g;
  g.cs = round_up(k, 8);
  g.kbytes = g.cs * 2;
  g.kpad_bytes = round_up(g.kbytes, BKB);
  g.num_kb = g.kpad_bytes / BKB;
  g.npad = round_up(n, 256);
  g.a_plane = round_up_sz((size_t)m * g.cs * 2, 256);
  g.b_plane = round_up_sz((size_t)g.npad * g.cs * 2, 256);
  g.y32 = round_up_sz((size_t)m * n * 4, 256);
  return g;
}
}  // namespace

int nnrcu_matmul_half_workspace(int m, int n, int k, size_t* bytes) {
  if (!bytes || m <= 0 || n <= 0 || k <= 0) return set_error(NNRCU_ERR_INVALID, "MatMul dims must be positive");
  const HalfMM g = half_mm_geom(m, n, k);
  *bytes = g.a_plane + g.b_plane + g.y32;
  return NNRCU_OK;
}

int nnrcu_matmul_half_run(const uint16_t* a, const uint16_t* b, uint16_t* y, int batch, int m, int n, int k,
                          long long a_batch_stride, long long b_batch_stride, int dtype, int post_op, float post_a,
                          float post_b, void* workspace, size_t workspace_bytes, void* stream) {
  if (!a || !b || !y || !workspace) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  if (dtype != NNRCU_DT_BF16 && dtype != NNRCU_DT_F16) return set_error(NNRCU_ERR_INVALID, "dtype must be bf16 or fp16");
  if (batch <= 0 || m <= 0 || n <= 0 || k <= 0 || a_batch_stride < 0 || b_batch_stride < 0)
    return set_error(NNRCU_ERR_INVALID, "MatMul: dims must be positive and strides non-negative");
  const HalfMM hg = half_mm_geom(m, n, k);
  if (workspace_bytes < hg.a_plane + hg.b_plane + hg.y32)
    return set_error(NNRCU_ERR_INVALID, "MatMul workspace of %zu bytes required", hg.a_plane + hg.b_plane + hg.y32);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* ap = reinterpret_cast<uint16_t*>(ws);
  uint16_t* bp = reinterpret_cast<uint16_t*>(ws + hg.a_plane);
  float* y32 = reinterpret_cast<float*>(ws + hg.a_plane + hg.b_plane);
  nnrcu_op op{};  // the launch geometry only (no device buffers of its own)
  op.M = m; op.N = n; op.K = k;
  op.nplane = dtype == NNRCU_DT_BF16 ? 3 : 4;
  op.epi = EPI_F32;
  op.cs = hg.cs;
  op.kbytes = hg.kbytes;
  op.kpad_bytes = hg.kpad_bytes;
  op.num_kb = hg.num_kb;
  op.npad = hg.npad;
  op.bn = pick_bn(m, n, 1, num_sms());
  op.amode = op.kbytes >= BKB ? A_TMA : A_GATHER;
  int rc = map_post_half(post_op, post_a, post_b, &op);
  if (rc != NNRCU_OK) return rc;
  // B rows past n are never written; they only feed output columns past n
  rc = encode_tmap_2d(&op.tmB, tmap_type(op.nplane), bp, hg.cs, (uint64_t)hg.npad, (uint64_t)hg.cs * 2, BKB / 2,
                      op.bn, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != NNRCU_OK) return rc;
  GatherGeom g{};
  g.N = 1; g.H = 1; g.W = m; g.OH = 1; g.OW = m; g.KH = 1; g.KW = 1;
  g.sh = 1; g.sw = 1; g.ph = 0; g.pw = 0; g.dh = 1; g.dw = 1;
  for (int bi = 0; bi < batch; ++bi) {
    if (bi == 0 || a_batch_stride) {
      rows_to_half_kernel<<<blocks((long long)m * hg.cs, 256), 256, 0, st>>>(a + a_batch_stride * bi, 0, 0, ap, m, k,
                                                                            hg.cs);
      NNRCU_CUDA(cudaGetLastError());
    }
    if (bi == 0 || b_batch_stride) {
      // B [k][n] read as the transposed rows of [n][cs]
      rows_to_half_kernel<<<blocks((long long)n * hg.cs, 256), 256, 0, st>>>(b + b_batch_stride * bi, 0, 1, bp, n, k,
                                                                            hg.cs);
      NNRCU_CUDA(cudaGetLastError());
    }
    if ((rc = half_launch(&op, ap, m, g, y32, 0, n, 1, st)) != NNRCU_OK) return rc;
    if ((rc = to_half(y32, y + (size_t)bi * m * n, (size_t)m * n, dtype, st)) != NNRCU_OK) return rc;
  }
  return NNRCU_OK;
}

}  // extern "C"

namespace nnrcu {
// fp32 A rounded to bf16 rows, one bf16 product per multiply-add, fp32 out
int gemm_f32_bf16_run(nnrcu_op* op, const float* a, float* y, void* workspace, cudaStream_t st) {
  if (!workspace) return set_error(NNRCU_ERR_INVALID, "workspace of %zu bytes required", op->ws_bytes);
  uint16_t* ap = static_cast<uint16_t*>(workspace);
  rows_to_half_kernel<<<blocks((long long)op->M * op->cs, 256), 256, 0, st>>>(a, 1, op->trans_a, ap, op->M, op->K,
                                                                            op->cs);
  NNRCU_CUDA(cudaGetLastError());
  GatherGeom g{};
  g.N = 1; g.H = 1; g.W = op->M; g.OH = 1; g.OW = op->M; g.KH = 1; g.KW = 1;
  g.sh = 1; g.sw = 1; g.ph = 0; g.pw = 0; g.dh = 1; g.dw = 1;
  return half_launch(op, ap, op->M, g, y, 0, op->N, 1, st);
}
}  // namespace nnrcu
