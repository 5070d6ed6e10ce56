// Harness around nnr's own Xbyak-free int8 direct convolution kernel
// (backend/x64/conv_int8_direct_avx512.h), compiled from the nnr source tree
// where it lies into oracle/_ref/libnnr_ref_int8.so by oracle/Makefile.
// TEST INFRASTRUCTURE ONLY: it pins the C restatement in nnr_oracle.c (tests)
// and is the "reference" CPU timing of the QLinearConv layer (bench.py).
//
// ref_qlinearconv_direct() follows exec_direct_int8 (backend/cpu/
// QLinearConv.cpp:536-655) step by step: pre-pad x with x_zp per image, run
// conv_int8_direct_avx512 for raw int32 dot products, subtract x_zp*sum(w),
// then the vectorised R1 requant for each 16-wide block and the scalar
// tail for the remainder. The requant lines restate :616-646 because the
// enclosing operator class cannot be compiled without Xbyak.
#include <immintrin.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "backend/x64/conv_int8_direct_avx512.h"
#include "backend/x64/depthwise_int8_avx512.h"
#include "backend/x64/conv_first_layer_int8_avx512.h"

extern "C" {

// Returns 1 when the host has AVX-512 VNNI (the kernel refuses to run without it).
int ref_has_vnni(void) { return (nnr::has_avx512() && nnr::cpu_features().avx512vnni) ? 1 : 0; }

// Sets nnr's worker thread count before the pool's first use (0 = nnr's
// default, all cores); thread_pool_t::configure, thread_pool.h:74.
void ref_set_threads(int n) {
  if (n > 0) nnr::thread_pool_t::configure(n);
}
int ref_get_threads(void) { return nnr::thread_pool_t::get().num_threads(); }

// NCHW u8 x [n, c, h, w], OIHW s8 w, NCHW u8 y. Returns 0 on success, -1 if
// the kernel declined (no VNNI) or the arguments are invalid.
int ref_qlinearconv_direct(const uint8_t* x, int n, int c, int h, int w, const int8_t* wt, int oc, int kh, int kw,
                           int sh, int sw, int pt, int pl, int pb, int pr, const float* w_scale, int n_w_scale,
                           const int32_t* bias, float x_scale, uint8_t x_zp, float y_scale, uint8_t y_zp,
                           int has_post, uint8_t* y, int32_t* raw_out) {
  if (!ref_has_vnni()) return -1;
  const int oh = (h + pt + pb - kh) / sh + 1, ow = (w + pl + pr - kw) / sw + 1;
  if (oh <= 0 || ow <= 0) return -1;
  std::vector<int8_t> wpk(nnr::pack_weights_int8_direct_size(oc, c, kh, kw));
  nnr::pack_weights_int8_direct(wpk.data(), wt, oc, c, kh, kw);
  std::vector<int32_t> wsum(oc);
  nnr::compute_weight_sums_int8_direct(wsum.data(), wt, oc, c, kh, kw);

  const int spatial = oh * ow;
  const int IC4 = (c + 3) / 4, IC_padded = IC4 * 4;
  const int padded_H = h + pt + pb, padded_W = w + pl + pr;
  const size_t pad_plane = (size_t)padded_H * padded_W;
  std::vector<uint8_t> x_pad((size_t)IC_padded * pad_plane + 64);
  std::vector<int32_t> y_i32((size_t)((oc + 15) / 16 * 16) * spatial + 64);
  const float inv_y_scale = 1.0f / y_scale;
  const int clamp_max = 255;
  const int qmin = has_post ? std::max(0, (int)y_zp) : 0;
  for (int img = 0; img < n; img++) {
    memset(x_pad.data(), x_zp, IC_padded * pad_plane);
    for (int ic = 0; ic < c; ic++) {
      const uint8_t* src = x + ((size_t)img * c + ic) * h * w;
      uint8_t* dst = x_pad.data() + (size_t)ic * pad_plane + pt * padded_W + pl;
      for (int r = 0; r < h; r++) memcpy(dst + r * padded_W, src + r * w, w);
    }
    if (!nnr::conv_int8_direct_avx512(y_i32.data(), x_pad.data(), wpk.data(), c, padded_H, padded_W, oc, oh, ow, kh,
                                      kw, sh, sw))
      return -1;
    if (raw_out) memcpy(raw_out + (size_t)img * oc * spatial, y_i32.data(), sizeof(int32_t) * (size_t)oc * spatial);
    uint8_t* out_n = y + (size_t)img * oc * spatial;
    const __m512 vis = _mm512_set1_ps(inv_y_scale);
    const __m512 vzp = _mm512_set1_ps((float)y_zp);
    const __m512 vqmin = _mm512_set1_ps((float)qmin);
    const __m512 vqmax = _mm512_set1_ps((float)clamp_max);
    for (int o = 0; o < oc; o++) {
      const float ws = n_w_scale > 1 ? w_scale[o] : w_scale[0];
      const float combined_scale = x_scale * ws;
      const float bias_val = bias ? (float)bias[o] * combined_scale : 0.0f;
      const int32_t zp_comp = (int32_t)x_zp * wsum[o];
      const __m512 vcs = _mm512_set1_ps(combined_scale);
      const __m512 vbias = _mm512_set1_ps(bias_val);
      const __m512i vzpc = _mm512_set1_epi32(zp_comp);
      const int32_t* irow = y_i32.data() + (size_t)o * spatial;
      uint8_t* out = out_n + (size_t)o * spatial;
      int s = 0;
      for (; s + 16 <= spatial; s += 16) {
        __m512i raw = _mm512_loadu_si512(irow + s);
        __m512 fv = _mm512_cvtepi32_ps(_mm512_sub_epi32(raw, vzpc));
        fv = _mm512_fmadd_ps(fv, vcs, vbias);
        fv = _mm512_add_ps(_mm512_roundscale_ps(_mm512_mul_ps(fv, vis), _MM_FROUND_TO_NEAREST_INT), vzp);
        fv = _mm512_max_ps(_mm512_min_ps(fv, vqmax), vqmin);
        _mm_storeu_si128((__m128i*)(out + s), _mm512_cvtepi32_epi8(_mm512_cvtps_epi32(fv)));
      }
      for (; s < spatial; s++) {
        const int32_t raw_val = irow[s] - zp_comp;
        const float val = std::fma((float)raw_val, combined_scale, bias_val);  // GCC contracts a*b+c here
        const int32_t q = (int32_t)std::nearbyint(val * inv_y_scale) + (int32_t)y_zp;
        out[s] = (uint8_t)std::clamp(q, qmin, clamp_max);
      }
    }
  }
  return 0;
}

// Depthwise QLinearConv through nnr's own Xbyak-free AVX-512 kernels, the
// way exec_dw_int8_nhwc (QLinearConv.cpp:425-531) calls them: weights
// repacked by repack_depthwise_weights, padding taps read from a buffer of
// x_zp bytes, depthwise_int8_nhwc_avx512_direct for dilation 1 and the
// indirection-buffer kernel otherwise (at most 5x5 taps there), with the
// plain u8 clamp bounds nnr passes (:502-507). The per-channel constants
// restate QLinearConv_reshape.h:306-317 (that class needs Xbyak). x [n,h,w,c]
// u8, w [c,1,kh,kw] s8, y [n,oh,ow,c] u8; channels past the last whole group
// of 16 are left as the caller filled them (nnr's kernels skip them).
int ref_qdwconv_nhwc(const uint8_t* x, int n, int c, int h, int w, const int8_t* wt, int kh, int kw, int sh, int sw,
                     int pt, int pl, int pb, int pr, int dh, int dw, const float* w_scale, int n_w_scale, int8_t w_zp,
                     const int32_t* bias, float x_scale, uint8_t x_zp, float y_scale, uint8_t y_zp, uint8_t* y) {
  if (!ref_has_vnni()) return -1;
  const int oh = (h + pt + pb - (dh * (kh - 1) + 1)) / sh + 1, ow = (w + pl + pr - (dw * (kw - 1) + 1)) / sw + 1;
  if (oh <= 0 || ow <= 0) return -1;
  if ((dh != 1 || dw != 1) && kh * kw > 25) return -1;
  std::vector<int8_t> wrep(nnr::int8::repack_depthwise_weights_size(c, kh, kw));
  nnr::int8::repack_depthwise_weights(wrep.data(), wt, c, kh, kw);
  std::vector<float> cs(c), bias_f(bias ? c : 0);
  for (int o = 0; o < c; ++o) {
    cs[o] = x_scale * (n_w_scale > 1 ? w_scale[o] : w_scale[0]);
    if (bias) bias_f[o] = (float)bias[o] * cs[o];
  }
  std::vector<uint8_t> zero_buf((c + 15) & ~15, x_zp);
  std::vector<const uint8_t*> ind((size_t)oh * ow * kh * kw);
  const float inv_y = 1.0f / y_scale;
  for (int img = 0; img < n; ++img) {
    const uint8_t* xn = x + (size_t)img * h * w * c;
    uint8_t* yn = y + (size_t)img * oh * ow * c;
    if (dh == 1 && dw == 1) {
      nnr::int8::depthwise_int8_nhwc_avx512_direct(yn, xn, wrep.data(), cs.data(), bias ? bias_f.data() : nullptr,
                                                   zero_buf.data(), c, oh, ow, h, w, kh, kw, sh, sw, pt, pl, (int)x_zp,
                                                   (int)w_zp, inv_y, (float)y_zp, 0.0f, 255.0f);
    } else {
      nnr::int8::build_depthwise_indirection(ind.data(), xn, zero_buf.data(), oh, ow, h, w, c, kh, kw, sh, sw, pt, pl,
                                             dh, dw);
      nnr::int8::depthwise_int8_nhwc_avx512_mt(yn, ind.data(), wrep.data(), cs.data(), bias ? bias_f.data() : nullptr,
                                               c, oh, ow, kh * kw, (int)x_zp, (int)w_zp, inv_y, (float)y_zp, 0.0f,
                                               255.0f);
    }
  }
  return 0;
}

// nnr's first-layer int8 conv (R3), as exec_first_layer_int8 calls it
// (backend/cpu/QLinearConv.cpp:661-698): NCHW u8 x [n, c <= 4, h, w], OIHW s8
// w, symmetric pads (ph, pw), NCHW or NHWC u8 y. The requant (vector body
// and, for NCHW outputs, the scalar tail of each row's last oW % 16 pixels)
// is nnr's own code in conv_first_layer_int8_avx512.h.
int ref_qconv_first_layer(const uint8_t* x, int n, int c, int h, int w, const int8_t* wt, int oc, int kh, int kw,
                          int sh, int sw, int ph, int pw, const float* w_scale, int n_w_scale, const int32_t* bias,
                          float x_scale, uint8_t x_zp, float y_scale, uint8_t y_zp, int has_post, int out_nhwc,
                          uint8_t* y) {
  if (!ref_has_vnni() || c < 1 || c > 4) return -1;
  const int oh = (h + 2 * ph - kh) / sh + 1, ow = (w + 2 * pw - kw) / sw + 1;
  if (oh <= 0 || ow <= 0) return -1;
  std::vector<int8_t> wpk(nnr::pack_weights_first_layer_int8_size(oc, c, kh, kw));
  nnr::pack_weights_first_layer_int8(wpk.data(), wt, oc, c, kh, kw);
  std::vector<int32_t> wsum(oc);
  nnr::compute_weight_sums_first_layer_int8(wsum.data(), wt, oc, c, kh, kw);
  // v.qmin / v.clamp_max of QLinearConv.cpp:419 for a u8 output
  const int32_t qmin = has_post ? std::max(0, (int)y_zp) : 0, qmax = 255;
  const float inv_y = 1.0f / y_scale;
  for (int img = 0; img < n; img++) {
    if (!nnr::conv_first_layer_int8_avx512(y + (size_t)img * oc * oh * ow, x + (size_t)img * c * h * w, wpk.data(),
                                           wsum.data(), bias, w_scale, n_w_scale, x_scale, inv_y, (int32_t)x_zp,
                                           (int32_t)y_zp, qmin, qmax, c, h, w, oc, oh, ow, kh, kw, sh, sw, ph, pw,
                                           out_nhwc != 0))
      return -1;
  }
  return 0;
}

}  // extern "C"
