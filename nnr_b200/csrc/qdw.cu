// Depthwise QLinearConv (group == C == OC) on u8 NHWC activations, the device
// form of nnr's exec_dw_int8_nhwc (backend/cpu/QLinearConv.cpp:425-531,
// kernels in backend/x64/depthwise_int8_avx512.h:70-351):
//   acc[c] = sum over taps of (x - x_zp) * (w[c] - w_zp)      (exact int32)
//   f = fma(float(acc), cs[c], bias_f[c]); q = rne(f * (1/y_scale)) + y_zp;
//   q = max(min(q, 255), 0)
// with cs = x_scale * w_scale[c] and bias_f = float(bias[c]) * cs in
// QLinearConv_reshape.h:306-317's order. nnr passes the plain u8 bounds to
// this kernel (QLinearConv.cpp:502-507: clamp_min, not the fused-Relu
// qmin), so a fused activation does not change the result here either.
// nnr takes this path for NHWC outputs only; other layouts are declined.
//
// CUDA cores, HBM bound: each thread computes 16 channels of one output
// pixel with 16-byte loads of the input and the [taps][C] weights (L1/L2
// resident), the accumulators in registers.
#include <algorithm>
#include <cmath>
#include <vector>

#include "internal.h"

namespace nnrcu {

namespace {

__device__ __forceinline__ int s8_at(uint32_t w, int j) { return (int)(int8_t)((w >> (8 * j)) & 0xFFu); }
__device__ __forceinline__ int u8_at(uint32_t w, int j) { return (int)((w >> (8 * j)) & 0xFFu); }

__device__ __forceinline__ uint32_t requant_dw(int32_t acc, float cs, float bf, float inv_y, float yzp) {
  float f = __fmaf_rn(__int2float_rn(acc), cs, bf);
  f = rintf(__fmul_rn(f, inv_y));
  f = __fadd_rn(f, yzp);
  f = fmaxf(fminf(f, 255.0f), 0.0f);
  return (uint32_t)__float2int_rn(f);
}

// One thread: output pixel p (n, oh, ow), channels [16 g, 16 g + 16).
// C % 16 == 0 (16-byte vectors); x, y NHWC dense; w [taps][C] s8.
__global__ void qdw_u8_nhwc_vec_kernel(const uint8_t* __restrict x, const int8_t* __restrict w,
                                       const float* __restrict cs, const float* __restrict bias_f,
                                       uint8_t* __restrict y, int N, int H, int W, int C, int OH, int OW, int KH, int KW,
                                       int sh, int sw, int pt, int pl, int dh, int dw, int x_zp, int w_zp,
                                       float inv_y, float yzp) {
  const int groups = C >> 4;
  const long long total = (long long)N * OH * OW * groups;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(t % groups);
    const long long p = t / groups;
    const int ow = (int)(p % OW);
    const int oh = (int)((p / OW) % OH);
    const int n = (int)(p / ((long long)OW * OH));
    int acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0;
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * sh - pt + kh * dh;
      if ((unsigned)ih >= (unsigned)H) continue;  // padding: (x_zp - x_zp) * w = 0
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * sw - pl + kw * dw;
        if ((unsigned)iw >= (unsigned)W) continue;
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (((size_t)n * H + ih) * W + iw) * C) + g);
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + (size_t)(kh * KW + kw) * C) + g);
        const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w}, ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[4 * q + j] += (u8_at(xs[q], j) - x_zp) * (s8_at(ws[q], j) - w_zp);
      }
    }
    const int c0 = g * 16;
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = c0 + 4 * q + j;
        word |= requant_dw(acc[4 * q + j], cs[c], bias_f[c], inv_y, yzp) << (8 * j);
      }
      o[q] = word;
    }
    reinterpret_cast<uint4*>(y + (size_t)p * C)[g] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Any C: one thread per output element.
__global__ void qdw_u8_nhwc_kernel(const uint8_t* __restrict x, const int8_t* __restrict w,
                                   const float* __restrict cs, const float* __restrict bias_f, uint8_t* __restrict y,
                                   int N, int H, int W, int C, int OH, int OW, int KH, int KW, int sh, int sw, int pt,
                                   int pl, int dh, int dw, int x_zp, int w_zp, float inv_y, float yzp) {
  const long long total = (long long)N * OH * OW * C;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(t % C);
    const long long p = t / C;
    const int ow = (int)(p % OW);
    const int oh = (int)((p / OW) % OH);
    const int n = (int)(p / ((long long)OW * OH));
    int acc = 0;
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * sh - pt + kh * dh;
      if ((unsigned)ih >= (unsigned)H) continue;
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * sw - pl + kw * dw;
        if ((unsigned)iw >= (unsigned)W) continue;
        acc += ((int)x[(((size_t)n * H + ih) * W + iw) * C + c] - x_zp) * ((int)w[(size_t)(kh * KW + kw) * C + c] - w_zp);
      }
    }
    y[t] = (uint8_t)requant_dw(acc, cs[c], bias_f[c], inv_y, yzp);
  }
}

int grid_for(long long total, int threads) {
  const long long b = (total + threads - 1) / threads;
  return (int)std::max<long long>(1, std::min<long long>(b, (long long)num_sms() * 16));
}

}  // namespace

int qdw_create(const nnrcu_conv_desc& d, int oh, int ow, const int8_t* w_host, const float* w_scale, int n_w_scale,
               const int8_t* w_zp, int n_w_zp, const int32_t* bias_host, float x_scale, uint8_t x_zp, float y_scale,
               uint8_t y_zp, nnrcu_op** out) {
  if (d.out_layout != NNRCU_LAYOUT_NHWC)
    return set_error(NNRCU_ERR_UNSUPPORTED,
                     "depthwise QLinearConv: nnr's int8 depthwise path writes NHWC outputs only (QLinearConv.cpp:468)");
  for (int i = 1; i < n_w_zp; ++i)
    if (w_zp[i] != w_zp[0])
      return set_error(NNRCU_ERR_UNSUPPORTED, "depthwise QLinearConv: per-channel weight zero points");
  if (!(y_scale > 0.0f) || !(x_scale > 0.0f)) return set_error(NNRCU_ERR_INVALID, "scales must be positive");
  nnrcu_op* op = new nnrcu_op();
  op->kind = OP_QDW;
  cudaGetDevice(&op->device);
  op->d = d;
  op->oh = oh;
  op->ow = ow;
  op->M = d.n * oh * ow;
  op->N = d.oc;
  op->K = d.kh * d.kw;
  op->num_ops = 2LL * op->M * d.oc * op->K;
  op->x_zp = x_zp;
  op->b_zp = n_w_zp > 0 && w_zp ? w_zp[0] : 0;  // (the weight zero point)
  op->inv_y = 1.0f / y_scale;                  // QLinearConv.cpp:420
  op->yzp_f = (float)y_zp;
  // weights [taps][C]; constants in nnr's order (QLinearConv_reshape.h:306-317)
  const int taps = d.kh * d.kw;
  std::vector<int8_t> wr((size_t)taps * d.c);
  std::vector<float> csv(d.c), bfv(d.c, 0.0f);
  for (int c = 0; c < d.c; ++c) {
    for (int k = 0; k < taps; ++k) wr[(size_t)k * d.c + c] = w_host[(size_t)c * taps + k];
    csv[c] = x_scale * (n_w_scale > 1 ? w_scale[c] : w_scale[0]);
    if (bias_host) bfv[c] = (float)bias_host[c] * csv[c];
  }
  auto up = [&](void** dst, const void* src, size_t bytes) {
    if (cudaMalloc(dst, std::max<size_t>(bytes, 16)) != cudaSuccess) return false;
    return cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
  };
  if (!up(&op->wB, wr.data(), wr.size()) || !up(reinterpret_cast<void**>(&op->cs_arr), csv.data(), csv.size() * 4) ||
      !up(reinterpret_cast<void**>(&op->bias_f), bfv.data(), bfv.size() * 4)) {
    nnrcu_op_destroy(op);
    return set_error(NNRCU_ERR_CUDA, "depthwise QLinearConv: weight upload failed");
  }
  // an NCHW input is reordered into the workspace first
  op->need_in_copy = d.in_layout == NNRCU_LAYOUT_NCHW;
  op->ws_bytes = op->need_in_copy ? (size_t)d.n * d.c * d.h * d.w : 0;
  *out = op;
  return NNRCU_OK;
}

int qdw_run(nnrcu_op* op, const uint8_t* x, uint8_t* y, void* workspace, cudaStream_t st) {
  const nnrcu_conv_desc& d = op->d;
  const uint8_t* xin = x;
  if (op->need_in_copy) {
    if (!workspace) return set_error(NNRCU_ERR_INVALID, "workspace of %zu bytes required", op->ws_bytes);
    int rc = launch_nchw_to_nhwc_u8(x, static_cast<uint8_t*>(workspace), d.n, d.c, d.h, d.w, d.c, (uint8_t)op->x_zp, st);
    if (rc != NNRCU_OK) return rc;
    xin = static_cast<const uint8_t*>(workspace);
  }
  const bool vec = d.c % 16 == 0 && (reinterpret_cast<uintptr_t>(xin) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  const long long total = (long long)d.n * op->oh * op->ow * (vec ? d.c / 16 : d.c);
  if (vec)
    qdw_u8_nhwc_vec_kernel<<<grid_for(total, 128), 128, 0, st>>>(
        xin, static_cast<const int8_t*>(op->wB), op->cs_arr, op->bias_f, y, d.n, d.h, d.w, d.c, op->oh, op->ow, d.kh,
        d.kw, d.stride_h, d.stride_w, d.pad_top, d.pad_left, d.dil_h, d.dil_w, op->x_zp, op->b_zp, op->inv_y,
        op->yzp_f);
  else
    qdw_u8_nhwc_kernel<<<grid_for(total, 256), 256, 0, st>>>(
        xin, static_cast<const int8_t*>(op->wB), op->cs_arr, op->bias_f, y, d.n, d.h, d.w, d.c, op->oh, op->ow, d.kh,
        d.kw, d.stride_h, d.stride_w, d.pad_top, d.pad_left, d.dil_h, d.dil_w, op->x_zp, op->b_zp, op->inv_y,
        op->yzp_f);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

}  // namespace nnrcu
