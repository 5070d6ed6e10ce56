// Memory-bound helper kernels: layout reorders, the fp32 -> split-bf16
// operand preparation, row sums for QLinearMatMul zero points, and the
// depthwise fp32 convolution (CUDA cores, NHWC, 128-bit channel vectors).
#include <algorithm>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <type_traits>

#include "internal.h"
#include "tc_gemm.cuh"

namespace nnrcu {

namespace {

// NCHW u8 -> NHWC u8 with channel stride cs >= c (extra channels = fill).
// One block transposes a 32-channel x 32-pixel tile through shared memory.
__global__ void nchw_to_nhwc_u8_kernel(const uint8_t* __restrict src, uint8_t* __restrict dst, int c, int hw,
                                       int cs, uint8_t fill) {
  __shared__ uint8_t tile[32][33];
  const int img = blockIdx.z;
  const int p0 = blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  const uint8_t* s = src + (size_t)img * c * hw;
  uint8_t* d = dst + (size_t)img * hw * cs;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int ch = c0 + i, p = p0 + threadIdx.x;
    tile[i][threadIdx.x] = (ch < c && p < hw) ? s[(size_t)ch * hw + p] : fill;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int p = p0 + i, ch = c0 + threadIdx.x;
    if (p < hw && ch < cs) d[(size_t)p * cs + ch] = tile[threadIdx.x][i];
  }
}

// Vectorised variant for hw % 4 == 0 and cs % 4 == 0: a 64-channel x
// 128-pixel tile is read as 32-bit words along pixels and written as 32-bit
// words along channels. The destination may be spatially padded
// ([n][hp][wp][cs], pixel (y, x) stored at (y + pt, x + pl)); its border is
// filled by the caller.
// border != 0: the grid has one more block column (the last blockIdx.x),
// which writes the fill into the border pixels of its 64 channels.
__global__ void nchw_to_nhwc_u8_vec_kernel(const uint8_t* __restrict src, uint8_t* __restrict dst, int c, int w,
                                           int hw, int hp, int wp, int pt, int pl, int cs, uint8_t fill,
                                           int border = 0) {
  __shared__ uint8_t tile[64][128 + 4];
  const int img = blockIdx.z;
  const int p0 = blockIdx.x * 128;
  const int c0 = blockIdx.y * 64;
  const uint8_t* s = src + (size_t)img * c * hw;
  uint8_t* d = dst + (size_t)img * hp * wp * cs;
  const uint32_t fill4 = 0x01010101u * fill;
  if (border && blockIdx.x == gridDim.x - 1) {
    // border pixels: the top pt and bottom rows whole, then the left pl and
    // right wp - w - pl columns of the h interior rows
    const int h = hw / w, pb = hp - h - pt, pr = wp - w - pl;
    const int n_tb = (pt + pb) * wp, side = pl + pr;
    const int nb = n_tb + h * side;
    const int cw = min(64, cs - c0) / 4;  // words of this block's channels
    for (int idx = threadIdx.x; idx < nb * 16; idx += blockDim.x) {
      const int bp = idx >> 4, wd = idx & 15;
      if (wd >= cw) continue;
      int y, x;
      if (bp < n_tb) {
        const int r = bp / wp;
        y = r < pt ? r : h + r;  // rows pt .. pt + h - 1 are interior
        x = bp - r * wp;
      } else {
        const int q = bp - n_tb, r = q / side, j = q - r * side;
        y = pt + r;
        x = j < pl ? j : w + j;
      }
      *reinterpret_cast<uint32_t*>(d + ((size_t)y * wp + x) * cs + c0 + wd * 4) = fill4;
    }
    return;
  }
  for (int idx = threadIdx.x; idx < 64 * 32; idx += blockDim.x) {
    const int ch = idx >> 5, wd = idx & 31;
    const int p = p0 + wd * 4;
    uint32_t v = fill4;
    if (c0 + ch < c && p < hw) v = *reinterpret_cast<const uint32_t*>(s + (size_t)(c0 + ch) * hw + p);
    *reinterpret_cast<uint32_t*>(&tile[ch][wd * 4]) = v;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 128 * 16; idx += blockDim.x) {
    const int pp = idx >> 4, wd = idx & 15;
    const int p = p0 + pp, ch = c0 + wd * 4;
    if (p >= hw || ch >= cs) continue;
    const int y = p / w, x = p - y * w;
    const uint32_t v = (uint32_t)tile[wd * 4][pp] | ((uint32_t)tile[wd * 4 + 1][pp] << 8) |
                       ((uint32_t)tile[wd * 4 + 2][pp] << 16) | ((uint32_t)tile[wd * 4 + 3][pp] << 24);
    *reinterpret_cast<uint32_t*>(d + ((size_t)(y + pt) * wp + (x + pl)) * cs + ch) = v;
  }
}

// Explicit im2col for small-channel convs (the 3-channel stem): row m (output
// pixel) of A[M][kp] holds x[(kh, kw, ic)] densely, k = (kh*KW + kw)*C + ic;
// padding pixels hold x_zp, k >= KH*KW*C holds 0. Input NCHW or NHWC u8.
// One thread writes 16 bytes of one row.
__global__ void im2col_u8_kernel(const uint8_t* __restrict x, uint8_t* __restrict a, int nchw, int n, int c, int h,
                                 int w, int oh, int ow, int kh, int kw, int sh, int sw, int pt, int pl, int dh, int dw,
                                 int kp, uint8_t x_zp) {
  const int chunks = kp / 16;
  const long long total = (long long)n * oh * ow * chunks;
  const int kreal = kh * kw * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / chunks;
    const int ck = (int)(i - m * chunks);
    const int img = (int)(m / ((long long)oh * ow));
    const int p = (int)(m - (long long)img * oh * ow);
    const int oy = p / ow, ox = p - oy * ow;
    uint32_t wv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t word = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int k = ck * 16 + q * 4 + b;
        uint32_t v = 0;
        if (k < kreal) {
          const int tap = k / c, ic = k - tap * c;
          const int ky = tap / kw, kx = tap - ky * kw;
          const int iy = oy * sh - pt + ky * dh, ix = ox * sw - pl + kx * dw;
          if ((unsigned)iy < (unsigned)h && (unsigned)ix < (unsigned)w)
            v = nchw ? x[(((size_t)img * c + ic) * h + iy) * w + ix] : x[(((size_t)img * h + iy) * w + ix) * c + ic];
          else
            v = x_zp;
        }
        word |= v << (8 * b);
      }
      wv[q] = word;
    }
    reinterpret_cast<uint4*>(a + (size_t)m * kp)[ck] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// Space-to-depth reorder of a small-channel image into 16-byte s2d pixels
// inside a fill border (the s2d conv path). Block (Y, image), threads over X.
__global__ void s2d_u8_kernel(const uint8_t* __restrict x, int nchw, uint8_t* __restrict dst, int c, int h, int w,
                              int hp, int wp, int pt, int pl, uint8_t fill) {
  const int Y = blockIdx.x, b = blockIdx.y;
  const int ih0 = 2 * (Y - pt);
  const uint32_t f4 = 0x01010101u * fill;
  uint4* out = reinterpret_cast<uint4*>(dst) + ((size_t)b * hp + Y) * wp;
  for (int X = threadIdx.x; X < wp; X += blockDim.x) {
    uint32_t wv[4] = {f4, f4, f4, f4};
    const int iw0 = 2 * (X - pl);
#pragma unroll
    for (int dy = 0; dy < 2; ++dy) {
      const int ih = ih0 + dy;
      if (ih < 0 || ih >= h) continue;
#pragma unroll
      for (int dx = 0; dx < 2; ++dx) {
        const int iw = iw0 + dx;
        if (iw < 0 || iw >= w) continue;
#pragma unroll 4
        for (int ci = 0; ci < c; ++ci) {
          const uint8_t v = nchw ? x[(((size_t)b * c + ci) * h + ih) * w + iw] : x[(((size_t)b * h + ih) * w + iw) * c + ci];
          const int byte = (dy * 2 + dx) * c + ci;
          const int sh = 8 * (byte & 3);
          wv[byte >> 2] = (wv[byte >> 2] & ~(0xFFu << sh)) | ((uint32_t)v << sh);
        }
      }
    }
    out[X] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// QuantizeLinear of element i (flat index of the fp32 tensor), as nnr does
// it (QuantizeLinear.cpp:128-160): the 16-wide body rne(x * inv) + zp clamped
// in float for i < vec_end, the scalar tail nearbyint(x / scale) + zp
// saturated as an integer (x86 conversion: out of range -> INT_MIN).
__device__ __forceinline__ uint32_t quantize_elem(float v, long long i, float scale, float inv, int zp,
                                                  long long vec_end) {
  if (i < vec_end) {
    float f = __fadd_rn(rintf(__fmul_rn(v, inv)), (float)zp);
    f = fmaxf(fminf(f, 255.0f), 0.0f);
    return (uint32_t)__float2int_rn(f);
  }
  const float d = __fdiv_rn(v, scale);
  const int r = (fabsf(d) < 2147483648.0f ? __float2int_rn(d) : (int)0x80000000) + zp;
  return (uint32_t)(r < 0 ? 0 : (r > 255 ? 255 : r));
}

// QuantizeLinear fused into the space-to-depth reorder: fp32 NCHW / NHWC
// input straight to the padded 16-byte s2d pixels. Block (Y, image).
// pairs: NCHW input with an even width, so the two columns (dx = 0, 1) of a
// pixel are one aligned float2 (coalesced across the warp). CC > 0 fixes the
// channel count at compile time so that all loads of a pixel issue at once.
template <int CC>
__global__ void quantize_s2d_kernel(const float* __restrict x, int nchw, uint8_t* __restrict dst, int c_rt, int h,
                                    int w, int hp, int wp, int pt, int pl, uint8_t fill, float scale, float inv, int zp,
                                    long long vec_end, int pairs) {
  const int c = CC > 0 ? CC : c_rt;
  const int Y = blockIdx.x, b = blockIdx.y;
  const int ih0 = 2 * (Y - pt);
  const uint32_t f4 = 0x01010101u * fill;
  uint4* out = reinterpret_cast<uint4*>(dst) + ((size_t)b * hp + Y) * wp;
  for (int X = threadIdx.x; X < wp; X += blockDim.x) {
    uint32_t wv[4] = {f4, f4, f4, f4};
    const int iw0 = 2 * (X - pl);
#pragma unroll
    for (int dy = 0; dy < 2; ++dy) {
      const int ih = ih0 + dy;
      if (ih < 0 || ih >= h) continue;
      if (pairs && iw0 >= 0 && iw0 + 1 < w) {
        const long long i00 = (((long long)b * c) * h + ih) * w + iw0;
#pragma unroll 4
        for (int ci = 0; ci < c; ++ci) {
          const long long i = i00 + (long long)ci * h * w;
          const float2 v = __ldg(reinterpret_cast<const float2*>(x + i));
          const uint32_t q0 = quantize_elem(v.x, i, scale, inv, zp, vec_end);
          const uint32_t q1 = quantize_elem(v.y, i + 1, scale, inv, zp, vec_end);
          const int b0 = (dy * 2) * c + ci, b1 = (dy * 2 + 1) * c + ci;
          wv[b0 >> 2] = (wv[b0 >> 2] & ~(0xFFu << (8 * (b0 & 3)))) | (q0 << (8 * (b0 & 3)));
          wv[b1 >> 2] = (wv[b1 >> 2] & ~(0xFFu << (8 * (b1 & 3)))) | (q1 << (8 * (b1 & 3)));
        }
        continue;
      }
#pragma unroll
      for (int dx = 0; dx < 2; ++dx) {
        const int iw = iw0 + dx;
        if (iw < 0 || iw >= w) continue;
#pragma unroll 4
        for (int ci = 0; ci < c; ++ci) {
          const long long i = nchw ? (((long long)b * c + ci) * h + ih) * w + iw : (((long long)b * h + ih) * w + iw) * c + ci;
          const uint32_t v = quantize_elem(x[i], i, scale, inv, zp, vec_end);
          const int byte = (dy * 2 + dx) * c + ci;
          const int sh = 8 * (byte & 3);
          wv[byte >> 2] = (wv[byte >> 2] & ~(0xFFu << sh)) | (v << sh);
        }
      }
    }
    out[X] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// NHWC u8 [n][h][w][cs] -> spatially padded [n][hp][wp][cs] whose border
// pixels hold the fill byte (the input zero point). Block (padded row, image):
// threads over the row's wp * cv 16-byte vectors.
__global__ void pad_spatial_nhwc_u8_kernel(const uint4* __restrict src, uint4* __restrict dst, int h, int w, int hp,
                                           int wp, int pt, int pl, int cv, uint32_t fill4) {
  const int py = blockIdx.x, img = blockIdx.y;
  const int y = py - pt;
  const int rowv = wp * cv;
  uint4* out = dst + ((size_t)img * hp + py) * rowv;
  const bool yin = (unsigned)y < (unsigned)h;
  const uint4* in = src + ((size_t)img * h + (yin ? y : 0)) * w * cv;
  const uint4 fill = make_uint4(fill4, fill4, fill4, fill4);
  for (int i = threadIdx.x; i < rowv; i += blockDim.x) {
    const int px = i / cv, v = i - px * cv;
    const int x = px - pl;
    out[i] = (yin && (unsigned)x < (unsigned)w) ? __ldg(in + x * cv + v) : fill;
  }
}

__global__ void pad_nhwc_u8_kernel(const uint8_t* __restrict src, uint8_t* __restrict dst, long long pixels, int c,
                                   int cs, uint8_t fill) {
  const long long total = pixels * cs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / cs;
    const int ch = (int)(i - p * cs);
    dst[i] = ch < c ? src[p * c + ch] : fill;
  }
}

__device__ __forceinline__ void split_bf16(float v, uint16_t& hi, uint16_t& lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  const __nv_bfloat16 l = __float2bfloat16_rn(v - __bfloat162float(h));
  hi = __bfloat16_as_ushort(h);
  lo = __bfloat16_as_ushort(l);
}

// fp32 activations (NCHW or NHWC) -> two NHWC bf16 planes with channel stride cs.
__global__ void split_bf16_nhwc_kernel(const float* __restrict src, int src_nchw, uint16_t* __restrict hi,
                                       uint16_t* __restrict lo, long long pixels, int c, int hw, int cs) {
  const long long total = pixels * cs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / cs;
    const int ch = (int)(i - p * cs);
    float v = 0.0f;
    if (ch < c) {
      if (src_nchw) {
        const long long img = p / hw;
        const long long q = p - img * hw;
        v = src[(img * c + ch) * hw + q];
      } else {
        v = src[p * c + ch];
      }
    }
    uint16_t h, l;
    split_bf16(v, h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

// NHWC fp32 [pixels][c] -> planes [pixels][cs], c and cs multiples of 4:
// one 4-channel vector per thread (zeros past c).
__global__ void split_bf16_nhwc_vec_kernel(const float4* __restrict src, uint2* __restrict hi, uint2* __restrict lo,
                                           unsigned total4, unsigned c4, unsigned cs4) {
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += gridDim.x * blockDim.x) {
    const unsigned p = i / cs4, cv = i - p * cs4;
    const float4 v = cv < c4 ? src[(size_t)p * c4 + cv] : make_float4(0.f, 0.f, 0.f, 0.f);
    uint16_t h0, l0, h1, l1, h2, l2, h3, l3;
    split_bf16(v.x, h0, l0);
    split_bf16(v.y, h1, l1);
    split_bf16(v.z, h2, l2);
    split_bf16(v.w, h3, l3);
    hi[i] = make_uint2(h0 | ((uint32_t)h1 << 16), h2 | ((uint32_t)h3 << 16));
    lo[i] = make_uint2(l0 | ((uint32_t)l1 << 16), l2 | ((uint32_t)l3 << 16));
  }
}

// Tiled NCHW -> NHWC split for fp32 inputs: coalesced reads along pixels,
// coalesced writes along channels.
__global__ void split_bf16_nchw_tiled_kernel(const float* __restrict src, uint16_t* __restrict hi,
                                             uint16_t* __restrict lo, int c, int hw, int cs) {
  __shared__ float tile[32][33];
  const int img = blockIdx.z;
  const int p0 = blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  const float* s = src + (size_t)img * c * hw;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int ch = c0 + i, p = p0 + threadIdx.x;
    tile[i][threadIdx.x] = (ch < c && p < hw) ? s[(size_t)ch * hw + p] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int p = p0 + i, ch = c0 + threadIdx.x;
    if (p < hw && ch < cs) {
      uint16_t h, l;
      split_bf16(tile[threadIdx.x][i], h, l);
      const size_t o = ((size_t)img * hw + p) * cs + ch;
      hi[o] = h;
      lo[o] = l;
    }
  }
}

// Rows of A (or columns when trans) -> K-major bf16 planes [m, kp].
__global__ void split_bf16_rows_kernel(const float* __restrict src, int trans, uint16_t* __restrict hi,
                                       uint16_t* __restrict lo, int m, int k, int kp) {
  const long long total = (long long)m * kp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / kp);
    const int kk = (int)(i - (long long)r * kp);
    float v = 0.0f;
    if (kk < k) v = trans ? src[(size_t)kk * m + r] : src[(size_t)r * k + kk];
    uint16_t h, l;
    split_bf16(v, h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

__global__ void split_bf16_rows_vec_kernel(const float4* __restrict src, uint2* __restrict hi, uint2* __restrict lo,
                                           long long n4) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 v = src[i];
    uint16_t h0, l0, h1, l1, h2, l2, h3, l3;
    split_bf16(v.x, h0, l0);
    split_bf16(v.y, h1, l1);
    split_bf16(v.z, h2, l2);
    split_bf16(v.w, h3, l3);
    hi[i] = make_uint2(h0 | ((uint32_t)h1 << 16), h2 | ((uint32_t)h3 << 16));
    lo[i] = make_uint2(l0 | ((uint32_t)l1 << 16), l2 | ((uint32_t)l3 << 16));
  }
}

// out[r] = -b_zp * sum_k a[r, k]  (QLinearMatMul row correction for b_zp != 0).
__global__ void rowcorr_u8_kernel(const uint8_t* __restrict a, int m, int k, int lda, int b_zp,
                                  int32_t* __restrict out) {
  const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= m) return;
  int s = 0;
  for (int i = lane; i < k; i += 32) s += a[(size_t)r * lda + i];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[r] = (int32_t)((uint32_t)(-b_zp) * (uint32_t)s);
}

template <typename T>
__global__ void transpose_kernel(const T* __restrict src, T* __restrict dst, int c, int hw, int to_nhwc) {
  __shared__ T tile[32][33];
  const int img = blockIdx.z;
  // to_nhwc: src [c][hw] -> dst [hw][c]; else src [hw][c] -> dst [c][hw]
  const int rows = to_nhwc ? c : hw, cols = to_nhwc ? hw : c;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const T* s = src + (size_t)img * c * hw;
  T* d = dst + (size_t)img * c * hw;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, cc = c0 + threadIdx.x;
    if (r < rows && cc < cols) tile[i][threadIdx.x] = s[(size_t)r * cols + cc];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int cc = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && cc < cols) d[(size_t)cc * rows + r] = tile[threadIdx.x][i];
  }
}

// Depthwise I/O types: 0 = fp32, 1 = bf16, 2 = fp16. A 4-channel vector is a
// float4 or a uint2 of four 16-bit values; 16-bit tensors are widened to fp32
// on load and rounded to nearest even on store, the way nnr's 16-bit Conv
// converts around its fp32 kernels (Conv_exec_entry.h:188-381).
// IO 3: fp32 input, and the output written as two bf16 planes (PlaneOut).
template <int IO>
struct Vec4IO {
  using T = std::conditional_t<IO == 0 || IO == 3, float, uint16_t>;     // element
  using V = std::conditional_t<IO == 0 || IO == 3, float4, uint2>;       // 4-channel vector
  static __device__ __forceinline__ float h2f(uint32_t b) {
    if constexpr (IO == 1) return __uint_as_float(b << 16);
    else return __half2float(__ushort_as_half((unsigned short)b));
  }
  static __device__ __forceinline__ uint32_t f2h(float v) {
    if constexpr (IO == 1) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
    else return __half_as_ushort(__float2half_rn(v));
  }
  static __device__ __forceinline__ float4 cvt(const V& u) {
    if constexpr (IO == 0 || IO == 3) return u;
    else return make_float4(h2f(u.x & 0xFFFFu), h2f(u.x >> 16), h2f(u.y & 0xFFFFu), h2f(u.y >> 16));
  }
  static __device__ __forceinline__ V pack(float4 v) {
    if constexpr (IO == 0 || IO == 3) return v;
    else return make_uint2(f2h(v.x) | (f2h(v.y) << 16), f2h(v.z) | (f2h(v.w) << 16));
  }
};

// Output of a depthwise conv as the split-bf16 operand of the dense conv
// that consumes it: hi = bf16(v), lo = bf16(v - hi), NHWC with channel
// stride cs4 * 4 (channels c .. cs - 1 zero), the layout and values the
// consumer's own split (split_bf16_nhwc_kernel) would produce from the fp32
// tensor.
struct PlaneOut {
  uint2* hi;
  uint2* lo;
  int cs4;
};

__device__ __forceinline__ void store_planes(const PlaneOut& po, size_t pixel, int cv, const float (&r)[4]) {
  uint16_t h[4], l[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) split_bf16(r[u], h[u], l[u]);
  const size_t i = pixel * po.cs4 + cv;
  po.hi[i] = make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
  po.lo[i] = make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
}

// the padding channels [c4, cs4) of one output row's pixels
__device__ __forceinline__ void zero_plane_pad(const PlaneOut& po, size_t pixel0, int ow, int c4) {
  const int pad = po.cs4 - c4;
  if (pad <= 0) return;
  for (int t = threadIdx.x; t < ow * pad; t += blockDim.x) {
    const int ox = t / pad, cv = c4 + (t - ox * pad);
    const size_t i = (pixel0 + ox) * po.cs4 + cv;
    po.hi[i] = make_uint2(0u, 0u);
    po.lo[i] = make_uint2(0u, 0u);
  }
}

// Depthwise fp32 conv, NHWC in/out. Each thread produces 4 consecutive
// channels (one float4) of one output pixel; weights are [kh][kw][c].
// Depthwise fp32 conv on NHWC (Conv_depthwise.h:11). One block per output
// row (image, oy); threads over (ox, 4-channel vector), so consecutive threads
// read consecutive channels of one pixel. Bias, post-op and residual fused.
template <int ACT, int IO = 0>
__global__ void depthwise_f32_kernel(const typename Vec4IO<IO>::T* __restrict x, const float* __restrict w,
                                     const float* __restrict bias, typename Vec4IO<IO>::T* __restrict y,
                                     const typename Vec4IO<IO>::T* __restrict residual, int h, int wd, int c,
                                     int oh, int ow, int kh, int kw, int sh, int sw, int ph, int pw, int dh, int dw,
                                     int act, float act_a, float act_b, PlaneOut po) {
  const int c4 = c >> 2;
  const int row = blockIdx.x;  // img * oh + oy
  const int img = row / oh, oy = row - img * oh;
  using IOT = Vec4IO<IO>;
  using VT = typename IOT::V;
  const VT* xin = reinterpret_cast<const VT*>(x) + (size_t)img * h * wd * c4;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  VT* out = reinterpret_cast<VT*>(y) + (size_t)row * ow * c4;
  const VT* res = residual ? reinterpret_cast<const VT*>(residual) + (size_t)row * ow * c4 : nullptr;
  for (int t = threadIdx.x; t < ow * c4; t += blockDim.x) {
    const int ox = t / c4, cv = t - ox * c4;
    float4 acc = bias ? reinterpret_cast<const float4*>(bias)[cv] : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int ky = 0; ky < kh; ++ky) {
      const int iy = oy * sh - ph + ky * dh;
      if ((unsigned)iy >= (unsigned)h) continue;
      const VT* xr = xin + (size_t)iy * wd * c4 + cv;
      const float4* wr = w4 + (size_t)ky * kw * c4 + cv;
      for (int kx = 0; kx < kw; ++kx) {
        const int ix = ox * sw - pw + kx * dw;
        if ((unsigned)ix >= (unsigned)wd) continue;
        const float4 xv = IOT::cvt(xr[(size_t)ix * c4]);
        const float4 wv = wr[(size_t)kx * c4];
        acc.x = fmaf(xv.x, wv.x, acc.x);
        acc.y = fmaf(xv.y, wv.y, acc.y);
        acc.z = fmaf(xv.z, wv.z, acc.z);
        acc.w = fmaf(xv.w, wv.w, acc.w);
      }
    }
    float o[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if constexpr (ACT == ACT_CLIP) o[u] = fminf(fmaxf(o[u], act_a), act_b);
      else if constexpr (ACT == ACT_RELU) o[u] = fmaxf(o[u], 0.0f);
      else if constexpr (ACT != ACT_NONE) o[u] = apply_act(o[u], act, act_a, act_b);
    }
    if (res) {
      const float4 rr = IOT::cvt(res[t]);
      o[0] += rr.x; o[1] += rr.y; o[2] += rr.z; o[3] += rr.w;
    }
    if constexpr (IO == 3) store_planes(po, (size_t)row * ow + ox, cv, o);
    else out[t] = IOT::pack(make_float4(o[0], o[1], o[2], o[3]));
  }
  if constexpr (IO == 3) zero_plane_pad(po, (size_t)row * ow, ow, c4);
}

// 3x3 depthwise fp32 conv (stride SW, dilation 1) on NHWC: each thread makes
// two consecutive outputs along x for one 4-channel vector, with the input
// vectors they share loaded once, up front (all loads in flight together).
// One block per output row; three blocks per SM (85 registers a thread).
// Measured on the MobileNetV2 shapes: at stride 2, 1.3-1.4x faster than two
// blocks per SM; at stride 1, the batch-128 forward took 2.36 ms against 2.43
// with four outputs a thread at two blocks per SM and 2.55 with one output at
// four blocks per SM.
template <int ACT, int SW, int IO = 0>
__global__ void __launch_bounds__(256, 3)
    dw3x3_f32_kernel(const typename Vec4IO<IO>::T* __restrict x, const float* __restrict w,
                     const float* __restrict bias, typename Vec4IO<IO>::T* __restrict y,
                     const typename Vec4IO<IO>::T* __restrict residual, int h, int wd, int c, int oh,
                                 int ow, int ph, int pw, int act, float act_a, float act_b, PlaneOut po) {
  constexpr int OXT = 2, NC = (OXT - 1) * SW + 3;
  const int c4 = c >> 2;
  const int row = blockIdx.x;
  const int img = row / oh, oy = row - img * oh;
  using IOT = Vec4IO<IO>;
  using VT = typename IOT::V;
  const VT* xin = reinterpret_cast<const VT*>(x) + (size_t)img * h * wd * c4;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  VT* out = reinterpret_cast<VT*>(y) + (size_t)row * ow * c4;
  const VT* res = residual ? reinterpret_cast<const VT*>(residual) + (size_t)row * ow * c4 : nullptr;
  const int groups = (ow + OXT - 1) / OXT;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = threadIdx.x; t < groups * c4; t += blockDim.x) {
    const int g = t / c4, cv = t - g * c4;
    const int ox0 = g * OXT;
    float4 xv[3][NC];
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
      const int iy = oy * SW - ph + ky;
      const bool vy = (unsigned)iy < (unsigned)h;
      const VT* xr = xin + (size_t)(vy ? iy : 0) * wd * c4 + cv;
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        const int ix = ox0 * SW - pw + j;
        xv[ky][j] = (vy && (unsigned)ix < (unsigned)wd) ? IOT::cvt(xr[(size_t)ix * c4]) : z;
      }
    }
    const float4 b4 = bias ? reinterpret_cast<const float4*>(bias)[cv] : z;
    float4 accs[OXT];
#pragma unroll
    for (int o = 0; o < OXT; ++o) accs[o] = b4;
    // taps outer, outputs inner: a weight vector is live for one tap only
#pragma unroll
    for (int ky = 0; ky < 3; ++ky)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const float4 ww = w4[(size_t)(ky * 3 + kx) * c4 + cv];
#pragma unroll
        for (int o = 0; o < OXT; ++o) {
          const float4 xx = xv[ky][o * SW + kx];
          accs[o].x = fmaf(xx.x, ww.x, accs[o].x);
          accs[o].y = fmaf(xx.y, ww.y, accs[o].y);
          accs[o].z = fmaf(xx.z, ww.z, accs[o].z);
          accs[o].w = fmaf(xx.w, ww.w, accs[o].w);
        }
      }
#pragma unroll
    for (int o = 0; o < OXT; ++o) {
      if (ox0 + o >= ow) break;
      const float4 acc = accs[o];
      float r[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if constexpr (ACT == ACT_CLIP) r[u] = fminf(fmaxf(r[u], act_a), act_b);
        else if constexpr (ACT == ACT_RELU) r[u] = fmaxf(r[u], 0.0f);
        else if constexpr (ACT != ACT_NONE) r[u] = apply_act(r[u], act, act_a, act_b);
      }
      const size_t oi = (size_t)(ox0 + o) * c4 + cv;
      if (res) {
        const float4 rr = IOT::cvt(res[oi]);
        r[0] += rr.x; r[1] += rr.y; r[2] += rr.z; r[3] += rr.w;
      }
      if constexpr (IO == 3) store_planes(po, (size_t)row * ow + ox0 + o, cv, r);
      else out[oi] = IOT::pack(make_float4(r[0], r[1], r[2], r[3]));
    }
  }
  if constexpr (IO == 3) zero_plane_pad(po, (size_t)row * ow, ow, c4);
}

// Explicit im2col for fp32 small-channel convs, written as split bf16:
// row m (output pixel) holds k = (kh, kw, ic) for k < KH*KW*C, zeros up to kp;
// hi = bf16(x), lo = bf16(x - hi). One thread per output pixel, 8 elements
// (16 bytes) per store.
// (C, KH, KW, KP nonzero: a compile-time shape, e.g. MobileNet's 3-channel
// 3x3 stem, so the tap / channel index arithmetic folds away)
template <int C_, int KH_, int KW_, int KP_>
__global__ void im2col_split_bf16_kernel(const float* __restrict x, int nchw, uint16_t* __restrict hi,
                                         uint16_t* __restrict lo, long long m_total, int c_rt, int h, int w, int oh,
                                         int ow, int kh_rt, int kw_rt, int sh, int sw, int pt, int pl, int dh, int dw,
                                         int kp_rt) {
  const int c = C_ ? C_ : c_rt, kh = KH_ ? KH_ : kh_rt, kw = KW_ ? KW_ : kw_rt, kp = KP_ ? KP_ : kp_rt;
  for (long long m = blockIdx.x * (long long)blockDim.x + threadIdx.x; m < m_total;
       m += (long long)gridDim.x * blockDim.x) {
    const int ox = (int)(m % ow);
    const long long r = m / ow;
    const int oy = (int)(r % oh);
    const int img = (int)(r / oh);
    const int kd = kh * kw * c;
    uint4* hrow = reinterpret_cast<uint4*>(hi + m * kp);
    uint4* lrow = reinterpret_cast<uint4*>(lo + m * kp);
#pragma unroll
    for (int k0 = 0; k0 < kp; k0 += 8) {
      uint32_t hw_[4], lw_[4];
#pragma unroll
      for (int q = 0; q < 8; q += 2) {
        float v[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int k = k0 + q + u;
          float val = 0.0f;
          if (k < kd) {
            const int tap = k / c, ic = k - tap * c;
            const int ky = tap / kw, kx = tap - ky * kw;
            const int iy = oy * sh - pt + ky * dh, ix = ox * sw - pl + kx * dw;
            if ((unsigned)iy < (unsigned)h && (unsigned)ix < (unsigned)w)
              val = nchw ? x[(((size_t)img * c + ic) * h + iy) * w + ix] : x[(((size_t)img * h + iy) * w + ix) * c + ic];
          }
          v[u] = val;
        }
        const __nv_bfloat16 h0 = __float2bfloat16_rn(v[0]), h1 = __float2bfloat16_rn(v[1]);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(v[0] - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(v[1] - __bfloat162float(h1));
        hw_[q / 2] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
        lw_[q / 2] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
      }
      hrow[k0 / 8] = make_uint4(hw_[0], hw_[1], hw_[2], hw_[3]);
      lrow[k0 / 8] = make_uint4(lw_[0], lw_[1], lw_[2], lw_[3]);
    }
  }
}

// Explicit im2col of one output row (oy) of one image per block: the kh input
// rows it needs (all c channels, full width, x_zp outside the image) are first
// staged in shared memory with coalesced reads, then rows of A are written as
// 16-byte chunks. NCHW or NHWC input; smem = c * kh * w bytes.
__global__ void im2col_rows_u8_kernel(const uint8_t* __restrict x, uint8_t* __restrict a, int nchw, int c, int h,
                                      int w, int oh, int ow, int kh, int kw, int sh, int sw, int pt, int pl, int dh,
                                      int dw, int kp, uint8_t x_zp) {
  extern __shared__ uint8_t smem_dyn[];
  // per-k table: row offset (ic * kh + ky) * w into the staged rows (-1 for the
  // K padding) and the tap's column offset kx * dw
  int* koff = reinterpret_cast<int*>(smem_dyn);
  int* kcol = koff + kp;
  uint8_t* rows = reinterpret_cast<uint8_t*>(kcol + kp);  // [c][kh][w]
  const int oy = blockIdx.x, img = blockIdx.y;
  const int kreal = kh * kw * c;
  for (int k = threadIdx.x; k < kp; k += blockDim.x) {
    if (k < kreal) {
      const int tap = k / c, ic = k - tap * c;
      const int ky = tap / kw, kx = tap - ky * kw;
      koff[k] = (ic * kh + ky) * w;
      kcol[k] = kx * dw;
    } else {
      koff[k] = -1;
      kcol[k] = 0;
    }
  }
  const int nwarps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // stage the c * kh input rows (warp per row, lanes along the row)
  for (int rr = warp; rr < c * kh; rr += nwarps) {
    const int ic = rr / kh, r = rr - ic * kh;
    const int iy = oy * sh - pt + r * dh;
    uint8_t* dstrow = rows + rr * w;
    if ((unsigned)iy >= (unsigned)h) {
      for (int ix = lane; ix < w; ix += 32) dstrow[ix] = x_zp;
    } else if (nchw) {
      const uint8_t* src = x + (((size_t)img * c + ic) * h + iy) * w;
      if ((w & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 3) == 0) {
        for (int q = lane; q < (w >> 2); q += 32)
          reinterpret_cast<uint32_t*>(dstrow)[q] = reinterpret_cast<const uint32_t*>(src)[q];
      } else {
        for (int ix = lane; ix < w; ix += 32) dstrow[ix] = src[ix];
      }
    } else {
      const uint8_t* src = x + (((size_t)img * h + iy) * w) * c + ic;
      for (int ix = lane; ix < w; ix += 32) dstrow[ix] = src[(size_t)ix * c];
    }
  }
  __syncthreads();
  // Rows of A are assembled in shared memory (row pitch kp + 16 to spread
  // banks). Each warp owns fixed 16-byte K chunks and keeps their table
  // entries in registers while its lanes sweep the output pixels; the
  // block's contiguous output is then copied out coalesced.
  const int chunks = kp / 16;
  const int pitch = kp + 16;
  uint8_t* sout = rows + ((c * kh * w + 15) & ~15);
  for (int ck = warp; ck < chunks; ck += nwarps) {
    int toff[16], tcol[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      toff[b] = koff[ck * 16 + b];
      tcol[b] = kcol[ck * 16 + b];
    }
    for (int ox = lane; ox < ow; ox += 32) {
      const int ix0 = ox * sw - pl;
      uint32_t wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int off = toff[q * 4 + b];
          const int ix = ix0 + tcol[q * 4 + b];
          uint32_t v = 0;
          if (off >= 0) v = (unsigned)ix < (unsigned)w ? rows[off + ix] : x_zp;
          word |= v << (8 * b);
        }
        wv[q] = word;
      }
      *reinterpret_cast<uint4*>(sout + ox * pitch + ck * 16) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
  }
  __syncthreads();
  uint4* dst = reinterpret_cast<uint4*>(a + ((size_t)img * oh + oy) * ow * kp);
  for (int i = threadIdx.x; i < ow * chunks; i += blockDim.x) {
    const int ox = i / chunks, ck = i - ox * chunks;
    dst[i] = *reinterpret_cast<const uint4*>(sout + ox * pitch + ck * 16);
  }
}

int grid_for(long long total, int threads) {
  long long b = (total + threads - 1) / threads;
  const long long cap = (long long)num_sms() * 16;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

void host_split_bf16(float v, uint16_t* hi, uint16_t* lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  const __nv_bfloat16 l = __float2bfloat16_rn(v - __bfloat162float(h));
  *hi = __bfloat16_as_ushort(h);
  *lo = __bfloat16_as_ushort(l);
}

int launch_nchw_to_nhwc_u8(const uint8_t* src, uint8_t* dst, int n, int c, int h, int w, int cs, uint8_t fill,
                           cudaStream_t st) {
  const int hw = h * w;
  if ((hw & 3) == 0 && (cs & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(dst) & 3) == 0) {
    dim3 grid((hw + 127) / 128, (cs + 63) / 64, n);
    nchw_to_nhwc_u8_vec_kernel<<<grid, 256, 0, st>>>(src, dst, c, w, hw, h, w, 0, 0, cs, fill);
    NNRCU_CUDA(cudaGetLastError());
    return NNRCU_OK;
  }
  dim3 grid((hw + 31) / 32, (cs + 31) / 32, n), block(32, 8);
  nchw_to_nhwc_u8_kernel<<<grid, block, 0, st>>>(src, dst, c, hw, cs, fill);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_nchw_to_nhwc_u8_padded(const uint8_t* src, uint8_t* dst, int n, int c, int h, int w, int pt, int pl,
                                  int pb, int pr, int cs, uint8_t fill, cudaStream_t st) {
  const int hp = h + pt + pb, wp = w + pl + pr;
  if ((h * w) % 4 != 0 || cs % 4 != 0 || (reinterpret_cast<uintptr_t>(src) & 3) || (reinterpret_cast<uintptr_t>(dst) & 3))
    return set_error(NNRCU_ERR_INVALID, "padded reorder needs h*w %% 4 == 0 and 4-byte aligned buffers");
  // the interior by 128-pixel tiles, the border (x_zp) by one extra block column
  const int border = (hp * wp != h * w) ? 1 : 0;
  dim3 grid((h * w + 127) / 128 + border, (cs + 63) / 64, n);
  nchw_to_nhwc_u8_vec_kernel<<<grid, 256, 0, st>>>(src, dst, c, w, h * w, hp, wp, pt, pl, cs, fill, border);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_im2col_u8(const uint8_t* x, uint8_t* a, int nchw, int n, int c, int h, int w, int oh, int ow, int kh,
                     int kw, int sh, int sw, int pt, int pl, int dh, int dw, int kp, uint8_t x_zp, cudaStream_t st) {
  const size_t smem = (size_t)kp * 8 + (((size_t)c * kh * w + 15) & ~(size_t)15) + (size_t)ow * (kp + 16);
  if (smem <= 48 * 1024 && n <= 65535) {
    im2col_rows_u8_kernel<<<dim3(oh, n), 256, smem, st>>>(x, a, nchw, c, h, w, oh, ow, kh, kw, sh, sw, pt, pl, dh, dw,
                                                          kp, x_zp);
    NNRCU_CUDA(cudaGetLastError());
    return NNRCU_OK;
  }
  const long long total = (long long)n * oh * ow * (kp / 16);
  im2col_u8_kernel<<<grid_for(total, 256), 256, 0, st>>>(x, a, nchw, n, c, h, w, oh, ow, kh, kw, sh, sw, pt, pl, dh, dw,
                                                          kp, x_zp);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_s2d_u8(const uint8_t* x, int nchw, uint8_t* dst, int n, int c, int h, int w, int hp, int wp, int pt, int pl,
                  uint8_t fill, cudaStream_t st) {
  if (c * 4 > 16 || (reinterpret_cast<uintptr_t>(dst) & 15))
    return set_error(NNRCU_ERR_INVALID, "space-to-depth needs 4c <= 16 and a 16-byte aligned destination");
  if (n > 65535) return set_error(NNRCU_ERR_INVALID, "space-to-depth: batch above 65535");
  s2d_u8_kernel<<<dim3(hp, n), 128, 0, st>>>(x, nchw, dst, c, h, w, hp, wp, pt, pl, fill);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_quantize_s2d(const float* x, int nchw, uint8_t* dst, int n, int c, int h, int w, int hp, int wp, int pt,
                        int pl, uint8_t fill, float scale, uint8_t zp, cudaStream_t st) {
  if (c * 4 > 16 || (reinterpret_cast<uintptr_t>(dst) & 15) || n > 65535)
    return set_error(NNRCU_ERR_INVALID, "quantize + space-to-depth: needs 4c <= 16, an aligned destination, n <= 65535");
  const long long total = (long long)n * c * h * w;
  const long long vec_end = total >= 64 ? total / 16 * 16 : 0;  // QuantizeLinear.cpp:132
  const int pairs = nchw && (w % 2) == 0 && (reinterpret_cast<uintptr_t>(x) & 7) == 0;
  auto kern = c == 3 ? quantize_s2d_kernel<3> : quantize_s2d_kernel<0>;
  kern<<<dim3(hp, n), 128, 0, st>>>(x, nchw, dst, c, h, w, hp, wp, pt, pl, fill, scale, 1.0f / scale, zp, vec_end, pairs);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_pad_spatial_nhwc_u8(const uint8_t* src, uint8_t* dst, int n, int h, int w, int cs, int pt, int pl, int pb,
                               int pr, uint8_t fill, cudaStream_t st) {
  if ((cs & 15) || ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15))
    return set_error(NNRCU_ERR_INVALID, "spatial pad: needs 16-byte aligned tensors and channel stride");
  if (n > 65535) return set_error(NNRCU_ERR_INVALID, "spatial pad: batch over 65535");
  const int hp = h + pt + pb, wp = w + pl + pr, cv = cs / 16;
  pad_spatial_nhwc_u8_kernel<<<dim3(hp, n), 256, 0, st>>>(reinterpret_cast<const uint4*>(src),
                                                           reinterpret_cast<uint4*>(dst), h, w, hp, wp, pt, pl, cv,
                                                           0x01010101u * fill);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_pad_nhwc_u8(const uint8_t* src, uint8_t* dst, int pixels, int c, int cs, uint8_t fill, cudaStream_t st) {
  const long long total = (long long)pixels * cs;
  pad_nhwc_u8_kernel<<<grid_for(total, 256), 256, 0, st>>>(src, dst, pixels, c, cs, fill);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_split_bf16_nhwc(const float* src, int src_nchw, uint16_t* hi, uint16_t* lo, int n, int c, int h, int w,
                           int cs, cudaStream_t st) {
  const int hw = h * w;
  if (src_nchw) {
    dim3 grid((hw + 31) / 32, (cs + 31) / 32, n), block(32, 8);
    split_bf16_nchw_tiled_kernel<<<grid, block, 0, st>>>(src, hi, lo, c, hw, cs);
  } else if (c == cs && (c % 4) == 0) {
    const long long n4 = (long long)n * hw * c / 4;
    split_bf16_rows_vec_kernel<<<grid_for(n4, 256), 256, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                                   reinterpret_cast<uint2*>(hi),
                                                                   reinterpret_cast<uint2*>(lo), n4);
  } else if ((c % 4) == 0 && (cs % 4) == 0 && (long long)n * hw * (cs / 4) < (1LL << 31) &&
             (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const unsigned total4 = (unsigned)((long long)n * hw * (cs / 4));
    split_bf16_nhwc_vec_kernel<<<grid_for(total4, 256), 256, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                                       reinterpret_cast<uint2*>(hi),
                                                                       reinterpret_cast<uint2*>(lo), total4,
                                                                       (unsigned)(c / 4), (unsigned)(cs / 4));
  } else {
    const long long pixels = (long long)n * hw;
    split_bf16_nhwc_kernel<<<grid_for(pixels * cs, 256), 256, 0, st>>>(src, 0, hi, lo, pixels, c, hw, cs);
  }
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_im2col_split_bf16(const float* x, int nchw, uint16_t* hi, uint16_t* lo, int n, int c, int h, int w,
                             int oh, int ow, int kh, int kw, int sh, int sw, int pt, int pl, int dh, int dw, int kp,
                             cudaStream_t st) {
  if (kp % 8 != 0 || (reinterpret_cast<uintptr_t>(hi) & 15) || (reinterpret_cast<uintptr_t>(lo) & 15))
    return set_error(NNRCU_ERR_INVALID, "im2col split: kp %% 8 and 16-byte aligned planes required");
  const long long m = (long long)n * oh * ow;
  if (c == 3 && kh == 3 && kw == 3 && kp == 32)
    im2col_split_bf16_kernel<3, 3, 3, 32><<<grid_for(m, 256), 256, 0, st>>>(x, nchw, hi, lo, m, c, h, w, oh, ow, kh,
                                                                          kw, sh, sw, pt, pl, dh, dw, kp);
  else
    im2col_split_bf16_kernel<0, 0, 0, 0><<<grid_for(m, 256), 256, 0, st>>>(x, nchw, hi, lo, m, c, h, w, oh, ow, kh,
                                                                        kw, sh, sw, pt, pl, dh, dw, kp);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_split_bf16_rows(const float* src, int trans, uint16_t* hi, uint16_t* lo, int m, int k, int kp,
                           cudaStream_t st) {
  if (!trans && k == kp && (k % 4) == 0) {
    const long long n4 = (long long)m * k / 4;
    split_bf16_rows_vec_kernel<<<grid_for(n4, 256), 256, 0, st>>>(reinterpret_cast<const float4*>(src),
                                                                   reinterpret_cast<uint2*>(hi),
                                                                   reinterpret_cast<uint2*>(lo), n4);
  } else {
    split_bf16_rows_kernel<<<grid_for((long long)m * kp, 256), 256, 0, st>>>(src, trans, hi, lo, m, k, kp);
  }
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_rowcorr_u8(const uint8_t* a, int m, int k, int lda, int b_zp, int32_t* out, cudaStream_t st) {
  rowcorr_u8_kernel<<<(m + 7) / 8, 256, 0, st>>>(a, m, k, lda, b_zp, out);
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_transpose_generic(const void* src, void* dst, int n, int c, int hw, int elem, int to_nhwc,
                             cudaStream_t st) {
  const int rows = to_nhwc ? c : hw, cols = to_nhwc ? hw : c;
  dim3 grid((cols + 31) / 32, (rows + 31) / 32, n), block(32, 8);
  switch (elem) {
    case 1: transpose_kernel<uint8_t><<<grid, block, 0, st>>>((const uint8_t*)src, (uint8_t*)dst, c, hw, to_nhwc); break;
    case 2: transpose_kernel<uint16_t><<<grid, block, 0, st>>>((const uint16_t*)src, (uint16_t*)dst, c, hw, to_nhwc); break;
    case 4: transpose_kernel<uint32_t><<<grid, block, 0, st>>>((const uint32_t*)src, (uint32_t*)dst, c, hw, to_nhwc); break;
    default: return set_error(NNRCU_ERR_INVALID, "element size %d not supported", elem);
  }
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

template <int IO>
int launch_depthwise(const Op& op, const void* x_v, void* y_v, const void* residual_v, cudaStream_t st,
                     PlaneOut po = PlaneOut{}) {
  using T = typename Vec4IO<IO>::T;
  const T* x_nhwc = static_cast<const T*>(x_v);
  T* y = static_cast<T*>(y_v);
  const T* residual = static_cast<const T*>(residual_v);
  const nnrcu_conv_desc& d = op.d;
  const int rows = d.n * op.oh;
  const int threads = std::min(256, std::max(32, (op.ow * (d.c / 4) + 31) / 32 * 32));
#define NNRCU_DW(A)                                                                                                   \
  depthwise_f32_kernel<A, IO><<<rows, threads, 0, st>>>(x_nhwc, op.w_dw, op.bias, y, residual, d.h, d.w, d.c, op.oh,      \
                                                    op.ow, d.kh, d.kw, d.stride_h, d.stride_w, d.pad_top, d.pad_left,  \
                                                    d.dil_h, d.dil_w, op.act, op.act_a, op.act_b, po)
  if (d.kh == 3 && d.kw == 3 && d.dil_h == 1 && d.dil_w == 1 && d.stride_h == d.stride_w &&
      (d.stride_h == 1 || d.stride_h == 2)) {
    const int oxt = 2;  // outputs per thread (the kernel's OXT)
    const int groups = (op.ow + oxt - 1) / oxt;
    const int th = std::min(256, std::max(32, (groups * (d.c / 4) + 31) / 32 * 32));
#define NNRCU_DW3(A, S)                                                                                                 \
  dw3x3_f32_kernel<A, S, IO><<<rows, th, 0, st>>>(x_nhwc, op.w_dw, op.bias, y, residual, d.h, d.w, d.c, op.oh, op.ow,     \
                                              d.pad_top, d.pad_left, op.act, op.act_a, op.act_b, po)
#define NNRCU_DW3S(A) \
  if (d.stride_h == 1) NNRCU_DW3(A, 1); else NNRCU_DW3(A, 2)
    switch (op.act) {
      case ACT_NONE: NNRCU_DW3S(ACT_NONE); break;
      case ACT_RELU: NNRCU_DW3S(ACT_RELU); break;
      case ACT_CLIP: NNRCU_DW3S(ACT_CLIP); break;
      default: NNRCU_DW3S(ACT_HARDSWISH); break;
    }
#undef NNRCU_DW3S
#undef NNRCU_DW3
    NNRCU_CUDA(cudaGetLastError());
    return NNRCU_OK;
  }
  switch (op.act) {
    case ACT_NONE: NNRCU_DW(ACT_NONE); break;
    case ACT_RELU: NNRCU_DW(ACT_RELU); break;
    case ACT_CLIP: NNRCU_DW(ACT_CLIP); break;
    default: NNRCU_DW(ACT_HARDSWISH); break;  // generic post-op switch
  }
#undef NNRCU_DW
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

int launch_depthwise_f32(const Op& op, const float* x_nhwc, float* y, const float* residual, cudaStream_t st) {
  return launch_depthwise<0>(op, x_nhwc, y, residual, st);
}

int launch_depthwise_f32_planes(const Op& op, const float* x_nhwc, uint16_t* hi, uint16_t* lo, int cs,
                                cudaStream_t st) {
  PlaneOut po{reinterpret_cast<uint2*>(hi), reinterpret_cast<uint2*>(lo), cs / 4};
  return launch_depthwise<3>(op, x_nhwc, nullptr, nullptr, st, po);
}

int launch_depthwise_half(const Op& op, const uint16_t* x_nhwc, uint16_t* y, int dtype, cudaStream_t st) {
  return dtype == NNRCU_DT_BF16 ? launch_depthwise<1>(op, x_nhwc, y, nullptr, st)
                                : launch_depthwise<2>(op, x_nhwc, y, nullptr, st);
}

}  // namespace nnrcu

extern "C" {

int nnrcu_nchw_to_nhwc(const void* src, void* dst, int n, int c, int h, int w, int elem_size, void* stream) {
  if (!src || !dst || n <= 0 || c <= 0 || h <= 0 || w <= 0)
    return nnrcu::set_error(NNRCU_ERR_INVALID, "nnrcu_nchw_to_nhwc: bad arguments");
  return nnrcu::launch_transpose_generic(src, dst, n, c, h * w, elem_size, 1, static_cast<cudaStream_t>(stream));
}
int nnrcu_nhwc_to_nchw(const void* src, void* dst, int n, int c, int h, int w, int elem_size, void* stream) {
  if (!src || !dst || n <= 0 || c <= 0 || h <= 0 || w <= 0)
    return nnrcu::set_error(NNRCU_ERR_INVALID, "nnrcu_nhwc_to_nchw: bad arguments");
  return nnrcu::launch_transpose_generic(src, dst, n, c, h * w, elem_size, 0, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
