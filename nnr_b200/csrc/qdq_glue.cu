// Device versions of the QDQ glue around the conv/GEMM path of an int8
// network (nnr's QuantizeLinear, MaxPool on u8, QLinearAdd,
// DequantizeLinear -> GlobalAveragePool -> QuantizeLinear, DequantizeLinear
// + Add). All are HBM-bound elementwise / reduction kernels.
//
// Bit-exactness: each kernel performs the float operations of nnr's x64 path
// in nnr's order. Where nnr runs a 16-wide AVX-512 body and a scalar tail
// over the last n % 16 elements, the tail elements follow the scalar
// expression (as GCC compiles it with FMA contraction, -march=native).
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace nnrcu {
namespace {

__device__ __forceinline__ uint8_t sat_u8(int v) { return (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v)); }

// QuantizeLinear (QuantizeLinear.cpp:128-160): element i of the NCHW tensor
// uses the vector body  rne(x * inv_scale) + zp, clamped (min 255, max 0),
// unless it lies in the final partial 16-group, which uses
// nearbyint(x / scale) + zp, clamped as an integer.
__global__ void quantize_u8_kernel(const float* __restrict x, uint8_t* __restrict y, long long total, int c, int hw,
                                   float scale, float inv_scale, int zp, int out_nhwc, int cs, long long vec_end) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const float v = x[i];
    uint8_t q;
    if (i < vec_end) {
      float f = rintf(__fmul_rn(v, inv_scale));
      f = __fadd_rn(f, (float)zp);
      f = fmaxf(fminf(f, 255.0f), 0.0f);
      q = (uint8_t)__float2int_rn(f);
    } else {
      q = sat_u8(ptx::cvt_rne_x86(__fdiv_rn(v, scale)) + zp);
    }
    if (!out_nhwc) {
      y[i] = q;
    } else {
      const long long img = i / ((long long)c * hw);
      const long long r = i - img * c * hw;
      const int ch = (int)(r / hw);
      const long long p = r - (long long)ch * hw;
      y[(img * hw + p) * cs + ch] = q;
    }
  }
}

__global__ void fill_u8_kernel(uint8_t* __restrict y, long long pixels, int c, int cs, uint8_t v) {
  const long long total = pixels * (cs - c);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / (cs - c);
    y[p * cs + c + (i - p * (cs - c))] = v;
  }
}

// MaxPool over u8 NHWC (MaxPool.cpp:279): padding positions are skipped.
// One block per output row (image, oy); threads over (ox, 16-channel vector).
__global__ void maxpool_u8_nhwc_kernel(const uint8_t* __restrict x, uint8_t* __restrict y, int h, int w, int c,
                                       int oh, int ow, int kh, int kw, int sh, int sw, int pt, int pl) {
  const int cv = c / 16;
  const int row = blockIdx.x;  // img * oh + oy
  const int img = row / oh, oy = row - img * oh;
  const int y0 = oy * sh - pt;
  const int ya = max(y0, 0), yb = min(y0 + kh, h);
  const uint4* xin = reinterpret_cast<const uint4*>(x + (size_t)img * h * w * c);
  uint4* out = reinterpret_cast<uint4*>(y + (size_t)row * ow * c);
  for (int i = threadIdx.x; i < ow * cv; i += blockDim.x) {
    const int ox = i / cv, v = i - ox * cv;
    const int x0 = ox * sw - pl;
    const int xa = max(x0, 0), xb = min(x0 + kw, w);
    uint4 m = make_uint4(0, 0, 0, 0);
    for (int iy = ya; iy < yb; ++iy)
      for (int ix = xa; ix < xb; ++ix) {
        const uint4 t = xin[((size_t)iy * w + ix) * cv + v];
        m.x = __vmaxu4(m.x, t.x);
        m.y = __vmaxu4(m.y, t.y);
        m.z = __vmaxu4(m.z, t.z);
        m.w = __vmaxu4(m.w, t.w);
      }
    out[i] = m;
  }
}

// Separable form of the same max (max is associative, so the result is
// identical): the block first takes the column max over the window's input
// rows for every input column into shared memory (each input row read once
// per output row, coalesced), then the row max over kw columns from there.
// KMAX > 0: windows of at most KMAX x KMAX; the window's loads of a column
// are unrolled so that they are all in flight together.
template <int KMAX>
__global__ void maxpool_u8_nhwc_sep_kernel(const uint8_t* __restrict x, uint8_t* __restrict y, int h, int w, int c,
                                           int oh, int ow, int kh, int kw, int sh, int sw, int pt, int pl) {
  extern __shared__ uint4 colmax[];
  const int cv = c / 16;
  const int row = blockIdx.x;
  const int img = row / oh, oy = row - img * oh;
  const int y0 = oy * sh - pt;
  const int ya = max(y0, 0), yb = min(y0 + kh, h);
  const uint4* xin = reinterpret_cast<const uint4*>(x + (size_t)img * h * w * c) + (size_t)ya * w * cv;
  const int rowv = w * cv;
  const int nr = yb - ya;
  for (int i = threadIdx.x; i < rowv; i += blockDim.x) {
    uint4 m = make_uint4(0, 0, 0, 0);
    const uint4* p = xin + i;
    if constexpr (KMAX > 0) {
      uint4 t[KMAX];
#pragma unroll
      for (int r = 0; r < KMAX; ++r) t[r] = r < nr ? __ldg(p + (size_t)r * rowv) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int r = 0; r < KMAX; ++r) {
        m.x = __vmaxu4(m.x, t[r].x);
        m.y = __vmaxu4(m.y, t[r].y);
        m.z = __vmaxu4(m.z, t[r].z);
        m.w = __vmaxu4(m.w, t[r].w);
      }
    } else {
      for (int iy = ya; iy < yb; ++iy, p += rowv) {
        const uint4 t = __ldg(p);
        m.x = __vmaxu4(m.x, t.x);
        m.y = __vmaxu4(m.y, t.y);
        m.z = __vmaxu4(m.z, t.z);
        m.w = __vmaxu4(m.w, t.w);
      }
    }
    colmax[i] = m;
  }
  __syncthreads();
  uint4* out = reinterpret_cast<uint4*>(y + (size_t)row * ow * c);
  for (int i = threadIdx.x; i < ow * cv; i += blockDim.x) {
    const int ox = i / cv, v = i - ox * cv;
    const int x0 = ox * sw - pl;
    const int xa = max(x0, 0), xb = min(x0 + kw, w);
    uint4 m = make_uint4(0, 0, 0, 0);
    for (int ix = xa; ix < xb; ++ix) {
      const uint4 t = colmax[ix * cv + v];
      m.x = __vmaxu4(m.x, t.x);
      m.y = __vmaxu4(m.y, t.y);
      m.z = __vmaxu4(m.z, t.z);
      m.w = __vmaxu4(m.w, t.w);
    }
    out[i] = m;
  }
}

__global__ void maxpool_u8_nhwc_scalar_kernel(const uint8_t* __restrict x, uint8_t* __restrict y, int n, int h, int w,
                                              int c, int oh, int ow, int kh, int kw, int sh, int sw, int pt, int pl) {
  const long long total = (long long)n * oh * ow * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % c);
    long long p = i / c;
    const int ox = (int)(p % ow);
    p /= ow;
    const int oy = (int)(p % oh);
    const int img = (int)(p / oh);
    int m = 0;
    for (int a = 0; a < kh; ++a) {
      const int iy = oy * sh - pt + a;
      if ((unsigned)iy >= (unsigned)h) continue;
      for (int b = 0; b < kw; ++b) {
        const int ix = ox * sw - pl + b;
        if ((unsigned)ix >= (unsigned)w) continue;
        const int t = x[(((size_t)img * h + iy) * w + ix) * c + ch];
        m = t > m ? t : m;
      }
    }
    y[i] = (uint8_t)m;
  }
}

// QLinearAdd, same shape (QLinearAdd.cpp:46-104). Vector body:
//   v = fma(a, sa, fma(b, sb, fixed)); r = rne(v); max 0; unsigned saturate.
// Tail (final n % 16): val = fma(sa, a - a_zp, sb * (b - b_zp)) + y_zp; nearbyint; clamp.
__global__ void qlinearadd_u8_kernel(const uint8_t* __restrict a, const uint8_t* __restrict b, uint8_t* __restrict y,
                                     long long n, long long vec_end, float sa, float sb, float fixed, int a_zp,
                                     int b_zp, int y_zp) {
  const long long nv = vec_end / 16;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv; i += (long long)gridDim.x * blockDim.x) {
    const uint4 av = reinterpret_cast<const uint4*>(a)[i];
    const uint4 bv = reinterpret_cast<const uint4*>(b)[i];
    const uint32_t aw[4] = {av.x, av.y, av.z, av.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
    uint32_t ow[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t o = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float fa = (float)((aw[k] >> (8 * j)) & 0xffu);
        const float fb = (float)((bw[k] >> (8 * j)) & 0xffu);
        float v = __fmaf_rn(fb, sb, fixed);
        v = __fmaf_rn(fa, sa, v);
        int r = ptx::cvt_rne_x86(v);
        r = r < 0 ? 0 : (r > 255 ? 255 : r);
        o |= (uint32_t)r << (8 * j);
      }
      ow[k] = o;
    }
    reinterpret_cast<uint4*>(y)[i] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
  for (long long i = vec_end + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float da = (float)((int)a[i] - a_zp), db = (float)((int)b[i] - b_zp);
    const float val = __fadd_rn(__fmaf_rn(sa, da, __fmul_rn(sb, db)), (float)y_zp);
    y[i] = sat_u8(ptx::cvt_rne_x86(val));
  }
}

// DequantizeLinear -> GlobalAveragePool (NHWC) -> QuantizeLinear, fused.
// DQ: (float(x) - float(zp)) * scale (DequantizeLinear.cpp:135-160).
// GAP: per channel, sum from 0 over the spatial positions in order, then
// * (1/spatial) (kernel/pool.h:109-125, x64/ops_x64.h:197-214).
// Q: vector body rne(v * (1/y_scale)) + zp clamped, or the scalar tail for
// the final partial 16-group of the [n, c] output.
__global__ void dq_gap_q_kernel(const uint8_t* __restrict x, uint8_t* __restrict y, int n, int hw, int c, float xs,
                                float xzp, float inv_hw, float ys, float inv_ys, int yzp, long long vec_end) {
  const long long total = (long long)n * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int img = (int)(i / c), ch = (int)(i - (long long)img * c);
    const uint8_t* px = x + (size_t)img * hw * c + ch;
    float sum = 0.0f;
    for (int s = 0; s < hw; ++s) sum = __fadd_rn(sum, __fmul_rn(__fsub_rn((float)px[(size_t)s * c], xzp), xs));
    const float v = __fmul_rn(sum, inv_hw);
    uint8_t q;
    if (i < vec_end) {
      float f = __fadd_rn(rintf(__fmul_rn(v, inv_ys)), (float)yzp);
      f = fmaxf(fminf(f, 255.0f), 0.0f);
      q = (uint8_t)__float2int_rn(f);
    } else {
      q = sat_u8(ptx::cvt_rne_x86(__fdiv_rn(v, ys)) + yzp);
    }
    y[i] = q;
  }
}

// DequantizeLinear of u8 [rows, cols] (+ fp32 bias[cols], an Add).
__global__ void dequant_bias_kernel(const uint8_t* __restrict x, float scale, float zp, const float* __restrict bias,
                                    int cols, long long total, float* __restrict y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    float v = __fmul_rn(__fsub_rn((float)x[i], zp), scale);
    if (bias) v = __fadd_rn(v, bias[i % cols]);
    y[i] = v;
  }
}

// fp32 Add with the second operand repeating every `period` elements (a
// same-shape tensor, or a trailing row vector such as a bias): one IEEE
// addition per element, as binary_math.cpp:57-77 does on the host.
__global__ void add_f32_kernel(const float* __restrict a, const float* __restrict b, long long period,
                               long long total, float* __restrict y) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x)
    y[i] = __fadd_rn(a[i], b[period == total ? i : i % period]);
}

// GlobalAveragePool on fp32 NHWC [n, hw, c] (kernel/pool.h:109-125): per
// channel a sequential sum over the positions, times 1/spatial. One thread per
// (image, channel): consecutive threads read consecutive channels.
__global__ void gap_f32_kernel(const float* __restrict x, float* __restrict y, int n, int hw, int c, float inv_hw) {
  const long long total = (long long)n * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int img = (int)(i / c), ch = (int)(i - (long long)img * c);
    const float* px = x + (size_t)img * hw * c + ch;
    float sum = 0.0f;
    for (int s = 0; s < hw; ++s) sum = __fadd_rn(sum, px[(size_t)s * c]);
    y[i] = __fmul_rn(sum, inv_hw);
  }
}

int blocks_for(long long total, int threads) {
  long long b = (total + threads - 1) / threads;
  const long long cap = (long long)num_sms() * 32;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace
}  // namespace nnrcu

using namespace nnrcu;

extern "C" {

int nnrcu_quantize_linear_u8(const float* x, uint8_t* y, int n, int c, int h, int w, float scale, uint8_t zp,
                             int out_layout, int out_cs, void* stream) {
  if (!x || !y || n <= 0 || c <= 0 || h <= 0 || w <= 0 || !(scale > 0.0f))
    return set_error(NNRCU_ERR_INVALID, "nnrcu_quantize_linear_u8: bad arguments");
  const int nhwc = out_layout == NNRCU_LAYOUT_NHWC;
  const int cs = nhwc ? (out_cs > 0 ? out_cs : c) : c;
  if (cs < c) return set_error(NNRCU_ERR_INVALID, "channel stride %d < channels %d", cs, c);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long total = (long long)n * c * h * w;
  // nnr vectorises only when the tensor has >= 64 elements (QuantizeLinear.cpp:132)
  const long long vec_end = total >= 64 ? total / 16 * 16 : 0;
  const float inv = 1.0f / scale;
  quantize_u8_kernel<<<blocks_for(total, 256), 256, 0, st>>>(x, y, total, c, h * w, scale, inv, zp, nhwc, cs, vec_end);
  NNRCU_CUDA(cudaGetLastError());
  if (nhwc && cs > c) {
    fill_u8_kernel<<<blocks_for((long long)n * h * w * (cs - c), 256), 256, 0, st>>>(y, (long long)n * h * w, c, cs, zp);
    NNRCU_CUDA(cudaGetLastError());
  }
  return NNRCU_OK;
}

int nnrcu_maxpool_u8_nhwc(const uint8_t* x, uint8_t* y, int n, int h, int w, int c, int kh, int kw, int sh, int sw,
                          int pt, int pl, int pb, int pr, void* stream) {
  if (!x || !y || n <= 0 || h <= 0 || w <= 0 || c <= 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || pt < 0 ||
      pl < 0 || pb < 0 || pr < 0)
    return set_error(NNRCU_ERR_INVALID, "nnrcu_maxpool_u8_nhwc: bad arguments");
  const int oh = (h + pt + pb - kh) / sh + 1, ow = (w + pl + pr - kw) / sw + 1;
  if (oh <= 0 || ow <= 0) return set_error(NNRCU_ERR_INVALID, "MaxPool window larger than the padded input");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (c % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    const size_t row_bytes = (size_t)w * c;
    if (row_bytes <= 48 * 1024) {
      auto kern = kh <= 3 ? maxpool_u8_nhwc_sep_kernel<3> : maxpool_u8_nhwc_sep_kernel<0>;
      kern<<<n * oh, 256, row_bytes, st>>>(x, y, h, w, c, oh, ow, kh, kw, sh, sw, pt, pl);
    } else {
      maxpool_u8_nhwc_kernel<<<n * oh, 256, 0, st>>>(x, y, h, w, c, oh, ow, kh, kw, sh, sw, pt, pl);
    }
  } else {
    const long long total = (long long)n * oh * ow * c;
    maxpool_u8_nhwc_scalar_kernel<<<blocks_for(total, 256), 256, 0, st>>>(x, y, n, h, w, c, oh, ow, kh, kw, sh, sw,
                                                                          pt, pl);
  }
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int nnrcu_qlinearadd_u8(const uint8_t* a, float a_scale, uint8_t a_zp, const uint8_t* b, float b_scale, uint8_t b_zp,
                        float y_scale, uint8_t y_zp, uint8_t* y, size_t n, void* stream) {
  if (!a || !b || !y || !(y_scale > 0.0f)) return set_error(NNRCU_ERR_INVALID, "nnrcu_qlinearadd_u8: bad arguments");
  if (n == 0) return NNRCU_OK;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(y)) & 15)
    return set_error(NNRCU_ERR_INVALID, "nnrcu_qlinearadd_u8: tensors must be 16-byte aligned");
  // constants in nnr's order; GCC contracts sa*a_zp + sb*b_zp into fma(sa, a_zp, sb*b_zp)
  const float sa = a_scale / y_scale, sb = b_scale / y_scale;
  const float fixed = (float)y_zp - std::fma(sa, (float)a_zp, sb * (float)b_zp);
  const long long vec_end = (long long)(n / 16 * 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  qlinearadd_u8_kernel<<<blocks_for(vec_end / 16 + 1, 256), 256, 0, st>>>(a, b, y, (long long)n, vec_end, sa, sb, fixed,
                                                                          a_zp, b_zp, y_zp);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int nnrcu_dq_gap_q_u8_nhwc(const uint8_t* x, int n, int hw, int c, float x_scale, uint8_t x_zp, float y_scale,
                           uint8_t y_zp, uint8_t* y, void* stream) {
  if (!x || !y || n <= 0 || hw <= 0 || c <= 0 || !(y_scale > 0.0f))
    return set_error(NNRCU_ERR_INVALID, "nnrcu_dq_gap_q_u8_nhwc: bad arguments");
  const long long total = (long long)n * c;
  const long long vec_end = total >= 64 ? total / 16 * 16 : 0;
  const float inv_hw = 1.0f / (float)hw;
  const float inv_ys = 1.0f / y_scale;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dq_gap_q_kernel<<<blocks_for(total, 256), 256, 0, st>>>(x, y, n, hw, c, x_scale, (float)x_zp, inv_hw, y_scale, inv_ys,
                                                          y_zp, vec_end);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int nnrcu_gap_f32_nhwc(const float* x, int n, int hw, int c, float* y, void* stream) {
  if (!x || !y || n <= 0 || hw <= 0 || c <= 0) return set_error(NNRCU_ERR_INVALID, "nnrcu_gap_f32_nhwc: bad arguments");
  const long long total = (long long)n * c;
  gap_f32_kernel<<<blocks_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n, hw, c,
                                                                                     1.0f / (float)hw);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int nnrcu_dequantize_linear_u8(const uint8_t* x, float scale, uint8_t zp, const float* bias, int rows, int cols,
                               float* y, void* stream) {
  if (!x || !y || rows <= 0 || cols <= 0) return set_error(NNRCU_ERR_INVALID, "nnrcu_dequantize_linear_u8: bad arguments");
  const long long total = (long long)rows * cols;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dequant_bias_kernel<<<blocks_for(total, 256), 256, 0, st>>>(x, scale, (float)zp, bias, cols, total, y);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int nnrcu_add_f32(const float* a, const float* b, float* y, size_t total, size_t period, void* stream) {
  if (!a || !b || !y || total == 0 || period == 0 || total % period != 0)
    return set_error(NNRCU_ERR_INVALID, "nnrcu_add_f32: bad arguments");
  add_f32_kernel<<<blocks_for((long long)total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      a, b, (long long)period, (long long)total, y);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

}  // extern "C"
