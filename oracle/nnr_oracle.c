/*
 * nnr_oracle.c - CPU restatement of nnr's arithmetic for the conv/GEMM hot
 * path. TEST INFRASTRUCTURE ONLY: the parity tests, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference arm use it as the checker. The
 * product (libnnrcu.so) never calls it.
 *
 * What it restates (paths relative to the nnr source tree):
 *   - QLinearConv: exact int32 sum of (x - x_zp) * w with padding pixels equal
 *     to x_zp (backend/cpu/QLinearConv.cpp:593-620, backend/x64/
 *     conv_int8_direct_avx512.h:1-12), then one of nnr's four requantisation
 *     sequences, selected the way nnr's x64 VNNI dispatch selects them:
 *       R1 QLinearConv.cpp:616-646          (exec_direct_int8)
 *       R2 backend/x64/jit_conv_int8_ukernel.cpp:950-965 (packed NR48 / NR16)
 *       R3 backend/x64/conv_first_layer_int8_avx512.h:262-270 (stem; NCHW
 *          outputs use R1 for each row's last ow % 16 pixels, :301-309)
 *     with the constants of QLinearConv_reshape.h:287-337.
 *   - QLinearMatMul: exact int32 sum of (a - a_zp)(b - b_zp) and the R4
 *     requant of QLinearMatMul.cpp:134,188-198.
 *   - fp32 Conv / Gemm: the mathematical result (double accumulation) with
 *     bias, the fused post-op (Relu/Clip/HardSwish/Sigmoid/LeakyRelu/Tanh,
 *     backend/cpu/{Relu,Clip,HardSwish,Sigmoid,LeakyRelu,Tanh}.cpp) and an
 *     optional residual Add (backend/cpu/binary_math.cpp:57-77). nnr's own
 *     fp32 kernels (Winograd, packed GEMM) differ from it by float rounding
 *     only; parity for fp32 is a relative-error bound, not bit equality.
 *
 * Floating-point operation order: every multiply-add that nnr executes as a
 * fused AVX-512 instruction (_mm512_fmadd_ps) is an explicit fmaf() here;
 * everything else is a separately rounded operation. The file must be
 * compiled with -ffp-contract=off so the compiler adds no contractions.
 * nnr's scalar tail loops write `a*b + c` in C++; GCC contracts those to FMA
 * under its default -ffp-contract=fast on FMA-capable targets, which makes
 * them agree with the vector body, and this file follows that.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_OK 0
#define ORACLE_ERR (-1)

/* formulas */
#define RQ_R1 1
#define RQ_R2 2
#define RQ_R3 3

/* post-ops (same numbering as NNRCU_POST_*) */
#define POST_NONE 0
#define POST_RELU 1
#define POST_CLIP 2
#define POST_HARDSWISH 3
#define POST_SIGMOID 4
#define POST_LEAKYRELU 5
#define POST_TANH 6

static int out_dim(int in, int pb, int pe, int k, int s, int d) {
  const int e = d * (k - 1) + 1;
  const int p = in + pb + pe - e;
  return p < 0 ? -1 : p / s + 1;
}

static inline int32_t wrap_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
static inline int32_t wrap_mul(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }

/* R1: f = fma((float)acc, cs, bias_f); f = rne(f * inv_y); f += y_zp;
 * f = max(min(f, hi), qmin); y = (uint8)f. (QLinearConv.cpp:629-645) */
static inline uint8_t rq_r1(int32_t acc, float cs, float bias_f, float inv_y, float yzp_f, float qmin_f,
                            float qmax_f) {
  float f = fmaf((float)acc, cs, bias_f);
  f = nearbyintf(f * inv_y);
  f = f + yzp_f;
  f = fminf(f, qmax_f);
  f = fmaxf(f, qmin_f);
  return (uint8_t)(int32_t)f;
}

/* R2: v = acc + bias (int32); f = (float)v * os; f = max(f, lo - y_zp);
 * f = min(f, hi - y_zp); r = rne(f) + y_zp; unsigned saturate.
 * (jit_conv_int8_ukernel.cpp:950-965) */
static inline uint8_t rq_r2(int32_t acc, int32_t bias, float os, float rq_lo, float rq_hi, int32_t yzp) {
  const int32_t v = wrap_add(acc, bias);
  float f = (float)v * os;
  f = fmaxf(f, rq_lo);
  f = fminf(f, rq_hi);
  int32_t r = (int32_t)nearbyintf(f) + yzp;
  if (r < 0) r = 0;
  if (r > 255) r = 255;
  return (uint8_t)r;
}

/* R3: f = fma((float)acc, cs, bias_f); f = fma(f, inv_y, y_zp);
 * f = max(min(f, hi), qmin); r = rne(f). (conv_first_layer_int8_avx512.h:262-270) */
static inline uint8_t rq_r3(int32_t acc, float cs, float bias_f, float inv_y, float yzp_f, float qmin_f,
                            float qmax_f) {
  float f = fmaf((float)acc, cs, bias_f);
  f = fmaf(f, inv_y, yzp_f);
  f = fminf(f, qmax_f);
  f = fmaxf(f, qmin_f);
  return (uint8_t)(int32_t)nearbyintf(f);
}

/* R3's scalar tail: f = fma((float)acc, cs, bias_f); q = (int32)rne(f * inv_y)
 * + y_zp (x86 conversion: out-of-range values become INT_MIN); clamp to
 * [qmin, hi] in integers. (conv_first_layer_int8_avx512.h:301-309) */
static inline uint8_t rq_r3_tail(int32_t acc, float cs, float bias_f, float inv_y, int32_t yzp, int32_t qmin,
                                 int32_t qmax) {
  const float r = nearbyintf(fmaf((float)acc, cs, bias_f) * inv_y);
  int32_t q = (r >= -2147483648.0f && r < 2147483648.0f) ? (int32_t)r : INT32_MIN;
  q = wrap_add(q, yzp);
  if (q < qmin) q = qmin;
  if (q > qmax) q = qmax;
  return (uint8_t)q;
}

/*
 * QLinearConv, u8 x / s8 w / u8 y, group 1, w_zp = 0.
 * x: in_layout 0 = NCHW [n,c,h,w], 1 = NHWC [n,h,w,c]; y likewise per out_layout.
 * w: OIHW [oc, c, kh, kw]. w_scale: 1 or oc entries. bias: NULL or [oc].
 * formula: RQ_R1 / RQ_R2 / RQ_R3. has_post: a fused activation exists (qmin = max(0, y_zp)).
 * acc_out: optional int32 [n, oc, oh, ow] (NCHW) of the exact accumulators.
 */
int oracle_qlinearconv(const uint8_t* x, int in_layout, int n, int c, int h, int w, const int8_t* wt, int oc, int kh,
                       int kw, int sh, int sw, int pt, int pl, int pb, int pr, int dh, int dw, const float* w_scale,
                       int n_w_scale, const int32_t* bias, float x_scale, uint8_t x_zp, float y_scale, uint8_t y_zp,
                       int formula, int has_post, int out_layout, uint8_t* y, int32_t* acc_out) {
  const int oh = out_dim(h, pt, pb, kh, sh, dh), ow = out_dim(w, pl, pr, kw, sw, dw);
  if (oh <= 0 || ow <= 0 || formula < RQ_R1 || formula > RQ_R3) return ORACLE_ERR;
  const int K = c * kh * kw;
  /* Constants in nnr's order (QLinearConv_reshape.h:287-319, QLinearConv.cpp:418-420). */
  const float inv_y = 1.0f / y_scale;
  const int lo = 0, hi = 255;
  const int qmin = has_post ? (y_zp > lo ? y_zp : lo) : lo;
  const float rq_lo = (float)lo - (float)y_zp, rq_hi = (float)hi - (float)y_zp;
  float* cs = (float*)malloc(sizeof(float) * oc);
  float* bf = (float*)malloc(sizeof(float) * oc);
  float* os = (float*)malloc(sizeof(float) * oc);
  int16_t* w16 = (int16_t*)malloc(sizeof(int16_t) * (size_t)oc * K);
  if (!cs || !bf || !os || !w16) {
    free(cs); free(bf); free(os); free(w16);
    return ORACLE_ERR;
  }
  for (int o = 0; o < oc; ++o) {
    const float ws = n_w_scale > 1 ? w_scale[o] : w_scale[0];
    cs[o] = x_scale * ws;
    bf[o] = bias ? (float)bias[o] * cs[o] : 0.0f;
    os[o] = cs[o] * inv_y;
    /* weights reordered to (kh, kw, ic) so the gathered column is contiguous */
    for (int ic = 0; ic < c; ++ic)
      for (int a = 0; a < kh; ++a)
        for (int b = 0; b < kw; ++b)
          w16[(size_t)o * K + ((size_t)a * kw + b) * c + ic] = wt[(((size_t)o * c + ic) * kh + a) * kw + b];
  }
  const long long npix = (long long)n * oh * ow;
  int rc = ORACLE_OK;
#pragma omp parallel
  {
    int16_t* col = (int16_t*)malloc(sizeof(int16_t) * (size_t)K);
    if (!col) {
      rc = ORACLE_ERR;
    } else {
#pragma omp for schedule(static)
      for (long long p = 0; p < npix; ++p) {
        const int img = (int)(p / ((long long)oh * ow));
        const int rem = (int)(p - (long long)img * oh * ow);
        const int oy = rem / ow, ox = rem - oy * ow;
        /* column of (x - x_zp); padding pixels hold x_zp, i.e. contribute 0 */
        for (int a = 0; a < kh; ++a) {
          const int iy = oy * sh - pt + a * dh;
          for (int b = 0; b < kw; ++b) {
            const int ix = ox * sw - pl + b * dw;
            int16_t* dst = col + ((size_t)a * kw + b) * c;
            if (iy < 0 || iy >= h || ix < 0 || ix >= w) {
              memset(dst, 0, sizeof(int16_t) * c);
            } else if (in_layout == 1) {
              const uint8_t* src = x + (((size_t)img * h + iy) * w + ix) * c;
              for (int ic = 0; ic < c; ++ic) dst[ic] = (int16_t)((int)src[ic] - (int)x_zp);
            } else {
              for (int ic = 0; ic < c; ++ic)
                dst[ic] = (int16_t)((int)x[(((size_t)img * c + ic) * h + iy) * w + ix] - (int)x_zp);
            }
          }
        }
        for (int o = 0; o < oc; ++o) {
          const int16_t* wr = w16 + (size_t)o * K;
          int32_t acc = 0;
          for (int k = 0; k < K; ++k) acc += (int32_t)col[k] * (int32_t)wr[k];
          uint8_t q;
          if (formula == RQ_R1)
            q = rq_r1(acc, cs[o], bf[o], inv_y, (float)y_zp, (float)qmin, (float)hi);
          else if (formula == RQ_R2)
            q = rq_r2(acc, bias ? bias[o] : 0, os[o], rq_lo, rq_hi, y_zp);
          else if (out_layout == 0 && ox >= ow / 16 * 16)
            /* the first-layer kernel's NCHW scalar tail (the last ow % 16
             * pixels of a row): f*cs+bs contracted, rne(f * inv_y) + y_zp,
             * integer clamp (conv_first_layer_int8_avx512.h:301-309) */
            q = rq_r3_tail(acc, cs[o], bf[o], inv_y, y_zp, qmin, hi);
          else
            q = rq_r3(acc, cs[o], bf[o], inv_y, (float)y_zp, (float)qmin, (float)hi);
          const size_t oi = out_layout == 1 ? ((size_t)p * oc + o)
                                            : (((size_t)img * oc + o) * oh + oy) * ow + ox;
          y[oi] = q;
          if (acc_out) acc_out[(((size_t)img * oc + o) * oh + oy) * ow + ox] = acc;
        }
      }
      free(col);
    }
  }
  free(cs); free(bf); free(os); free(w16);
  return rc;
}

/*
 * QLinearMatMul, a u8 [m,k], b s8 [k,n] row-major, y u8 [m,n].
 * R4: val = fma((float)acc, a_s*b_s/y_s, (float)y_zp); nearbyint; clamp [0,255].
 */
/*
 * Depthwise QLinearConv on u8 NHWC (group = c = oc), nnr's
 * exec_dw_int8_nhwc (QLinearConv.cpp:425-531) with the kernel
 * depthwise_int8_nhwc_avx512_direct (depthwise_int8_avx512.h:207-351):
 * acc = sum (x - x_zp) * (w - w_zp) over the in-bounds taps (padding taps
 * contribute (x_zp - x_zp) * w = 0), then R1 with the plain u8 bounds: nnr
 * passes clamp_min, not the fused-Relu qmin, to this kernel (:502-507).
 * cs = x_scale * w_scale[c], bias_f = (float)bias[c] * cs
 * (QLinearConv_reshape.h:306-317). x [n,h,w,c], w [c,1,kh,kw], y [n,oh,ow,c].
 * Every channel is computed (nnr's kernel skips the channels past the last
 * whole group of 16).
 */
int oracle_qdwconv_u8_nhwc(const uint8_t* x, int n, int c, int h, int w, const int8_t* wt, int kh, int kw, int sh,
                           int sw, int pt, int pl, int pb, int pr, int dh, int dw, const float* w_scale,
                           int n_w_scale, int8_t w_zp, const int32_t* bias, float x_scale, uint8_t x_zp,
                           float y_scale, uint8_t y_zp, uint8_t* y) {
  const int oh = out_dim(h, pt, pb, kh, sh, dh), ow = out_dim(w, pl, pr, kw, sw, dw);
  if (oh <= 0 || ow <= 0) return ORACLE_ERR;
  const float inv_y = 1.0f / y_scale;
#pragma omp parallel for schedule(static)
  for (long long p = 0; p < (long long)n * oh * ow; ++p) {
    const int img = (int)(p / ((long long)oh * ow));
    const int r = (int)(p - (long long)img * oh * ow);
    const int oy = r / ow, ox = r - oy * ow;
    for (int ch = 0; ch < c; ++ch) {
      int32_t acc = 0;
      for (int ky = 0; ky < kh; ++ky) {
        const int iy = oy * sh - pt + ky * dh;
        if (iy < 0 || iy >= h) continue;
        for (int kx = 0; kx < kw; ++kx) {
          const int ix = ox * sw - pl + kx * dw;
          if (ix < 0 || ix >= w) continue;
          const int xv = (int)x[(((size_t)img * h + iy) * w + ix) * c + ch] - (int)x_zp;
          const int wv = (int)wt[((size_t)ch * kh + ky) * kw + kx] - (int)w_zp;
          acc = wrap_add(acc, wrap_mul(xv, wv));
        }
      }
      const float cs = x_scale * (n_w_scale > 1 ? w_scale[ch] : w_scale[0]);
      const float bf = bias ? (float)bias[ch] * cs : 0.0f;
      y[(size_t)p * c + ch] = rq_r1(acc, cs, bf, inv_y, (float)y_zp, 0.0f, 255.0f);
    }
  }
  return ORACLE_OK;
}

int oracle_qlinearmatmul(const uint8_t* a, const int8_t* b, int m, int k, int n, float a_scale, uint8_t a_zp,
                         float b_scale, int8_t b_zp, float y_scale, uint8_t y_zp, uint8_t* y) {
  if (m <= 0 || k <= 0 || n <= 0) return ORACLE_ERR;
  const float combined = a_scale * b_scale / y_scale; /* QLinearMatMul.cpp:134 */
  int16_t* bt = (int16_t*)malloc(sizeof(int16_t) * (size_t)n * k);
  if (!bt) return ORACLE_ERR;
  for (int kk = 0; kk < k; ++kk)
    for (int j = 0; j < n; ++j) bt[(size_t)j * k + kk] = (int16_t)((int)b[(size_t)kk * n + j] - (int)b_zp);
  int rc = ORACLE_OK;
#pragma omp parallel
  {
    int16_t* ar = (int16_t*)malloc(sizeof(int16_t) * (size_t)k);
    if (!ar) {
      rc = ORACLE_ERR;
    } else {
#pragma omp for schedule(static)
      for (int r = 0; r < m; ++r) {
        for (int kk = 0; kk < k; ++kk) ar[kk] = (int16_t)((int)a[(size_t)r * k + kk] - (int)a_zp);
        for (int j = 0; j < n; ++j) {
          const int16_t* br = bt + (size_t)j * k;
          int32_t acc = 0;
          for (int kk = 0; kk < k; ++kk) acc += (int32_t)ar[kk] * (int32_t)br[kk];
          const float val = fmaf((float)acc, combined, (float)y_zp);
          int32_t q = (int32_t)nearbyintf(val);
          if (q < 0) q = 0;
          if (q > 255) q = 255;
          y[(size_t)r * n + j] = (uint8_t)q;
        }
      }
      free(ar);
    }
  }
  free(bt);
  return rc;
}

static double post_op(double v, int post, double a, double b) {
  switch (post) {
    case POST_RELU: return v > 0 ? v : 0;
    case POST_CLIP: return v < a ? a : (v > b ? b : v);
    case POST_HARDSWISH: {
      double t = v / 6.0 + 0.5;
      t = t < 0 ? 0 : (t > 1 ? 1 : t);
      return v * t;
    }
    case POST_SIGMOID: return 1.0 / (1.0 + exp(-v));
    case POST_LEAKYRELU: return v >= 0 ? v : v * a;
    case POST_TANH: return tanh(v);
    default: return v;
  }
}

/*
 * fp32 Conv (group 1 or depthwise), NCHW or NHWC in/out. y = post(conv + bias) (+ residual).
 */
int oracle_conv_f32(const float* x, int in_layout, int n, int c, int h, int w, const float* wt, int oc, int kh, int kw,
                    int group, int sh, int sw, int pt, int pl, int pb, int pr, int dh, int dw, const float* bias,
                    int post, float pa, float pbv, const float* residual, int out_layout, float* y) {
  const int oh = out_dim(h, pt, pb, kh, sh, dh), ow = out_dim(w, pl, pr, kw, sw, dw);
  if (oh <= 0 || ow <= 0 || group <= 0 || c % group || oc % group) return ORACLE_ERR;
  const int cpg = c / group, opg = oc / group;
  const long long total = (long long)n * oc * oh * ow;
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < total; ++i) {
    long long t = i;
    const int ox = (int)(t % ow); t /= ow;
    const int oy = (int)(t % oh); t /= oh;
    const int o = (int)(t % oc);
    const int img = (int)(t / oc);
    const int g = o / opg;
    double acc = bias ? bias[o] : 0.0;
    for (int icg = 0; icg < cpg; ++icg) {
      const int ic = g * cpg + icg;
      for (int a = 0; a < kh; ++a) {
        const int iy = oy * sh - pt + a * dh;
        if (iy < 0 || iy >= h) continue;
        for (int b = 0; b < kw; ++b) {
          const int ix = ox * sw - pl + b * dw;
          if (ix < 0 || ix >= w) continue;
          const float xv = in_layout == 1 ? x[(((size_t)img * h + iy) * w + ix) * c + ic]
                                          : x[(((size_t)img * c + ic) * h + iy) * w + ix];
          acc += (double)xv * (double)wt[(((size_t)o * cpg + icg) * kh + a) * kw + b];
        }
      }
    }
    double v = post_op(acc, post, pa, pbv);
    const size_t oi = out_layout == 1 ? (((size_t)img * oh + oy) * ow + ox) * oc + o
                                      : (((size_t)img * oc + o) * oh + oy) * ow + ox;
    if (residual) v += residual[oi];
    y[oi] = (float)v;
  }
  return ORACLE_OK;
}

/*
 * fp32 Gemm: y[m,n] = post(alpha * op(A) op(B) + beta * C), C NULL, [n] (c_rows = 1) or [m,n].
 * Only rows [row0, row0 + rows) of y are computed (y points at row row0), so a
 * large problem can be spot-checked.
 */
int oracle_gemm_f32(const float* a, const float* b, const float* cm, int m, int n, int k, int trans_a, int trans_b,
                    float alpha, float beta, int c_rows, int post, float pa, float pbv, int row0, int rows, float* y) {
  if (row0 < 0 || rows < 0 || row0 + rows > m) return ORACLE_ERR;
#pragma omp parallel for schedule(static)
  for (int r = row0; r < row0 + rows; ++r) {
    for (int j = 0; j < n; ++j) {
      double acc = 0.0;
      for (int kk = 0; kk < k; ++kk) {
        const double av = trans_a ? a[(size_t)kk * m + r] : a[(size_t)r * k + kk];
        const double bv = trans_b ? b[(size_t)j * k + kk] : b[(size_t)kk * n + j];
        acc += av * bv;
      }
      double v = (double)alpha * acc;
      if (cm) v += (double)beta * (c_rows == 1 ? cm[j] : cm[(size_t)r * n + j]);
      y[(size_t)(r - row0) * n + j] = (float)post_op(v, post, pa, pbv);
    }
  }
  return ORACLE_OK;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Sets the OpenMP thread count explicitly (callers use it so that an
 * inherited OMP_NUM_THREADS, e.g. torchrun's 1, does not decide it). */
void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------------ QDQ glue (int8 networks) */

static inline uint8_t sat_u8(int v) { return (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v)); }

/* QuantizeLinear fp32 -> u8, per tensor (QuantizeLinear.cpp:128-160). Element
 * i in the 16-wide body: rne(x * (1/scale)) + zp, min 255 then max 0; the
 * final partial 16-group (and tensors under 64 elements): nearbyint(x/scale)
 * + zp, integer clamp. x and y share the element order. */
int oracle_quantize_u8(const float* x, uint8_t* y, long long total, float scale, uint8_t zp) {
  const float inv = 1.0f / scale;
  const long long vec_end = total >= 64 ? total / 16 * 16 : 0;
  for (long long i = 0; i < total; ++i) {
    if (i < vec_end) {
      float f = nearbyintf(x[i] * inv) + (float)zp;
      f = fmaxf(fminf(f, 255.0f), 0.0f);
      y[i] = (uint8_t)(int)f;
    } else {
      y[i] = sat_u8((int)nearbyintf(x[i] / scale) + zp);
    }
  }
  return ORACLE_OK;
}

/* MaxPool on u8 NHWC (MaxPool.cpp:279): padding skipped. */
int oracle_maxpool_u8_nhwc(const uint8_t* x, uint8_t* y, int n, int h, int w, int c, int kh, int kw, int sh, int sw,
                           int pt, int pl, int pb, int pr) {
  const int oh = out_dim(h, pt, pb, kh, sh, 1), ow = out_dim(w, pl, pr, kw, sw, 1);
  if (oh <= 0 || ow <= 0) return ORACLE_ERR;
  for (int img = 0; img < n; ++img)
    for (int oy = 0; oy < oh; ++oy)
      for (int ox = 0; ox < ow; ++ox)
        for (int ch = 0; ch < c; ++ch) {
          int m = 0;
          for (int a = 0; a < kh; ++a) {
            const int iy = oy * sh - pt + a;
            if (iy < 0 || iy >= h) continue;
            for (int b = 0; b < kw; ++b) {
              const int ix = ox * sw - pl + b;
              if (ix < 0 || ix >= w) continue;
              const int t = x[(((size_t)img * h + iy) * w + ix) * c + ch];
              if (t > m) m = t;
            }
          }
          y[(((size_t)img * oh + oy) * ow + ox) * c + ch] = (uint8_t)m;
        }
  return ORACLE_OK;
}

/* QLinearAdd, same shape (QLinearAdd.cpp:46-104). sa = a_s/y_s, sb = b_s/y_s,
 * fixed = y_zp - (sa*a_zp + sb*b_zp) as GCC contracts it with FMA
 * (fma(sa, a_zp, sb*b_zp)). Body: v = fma(a, sa, fma(b, sb, fixed)), rne,
 * max 0, unsigned saturate. Tail (final n % 16):
 * fma(sa, a - a_zp, sb*(b - b_zp)) + y_zp, nearbyint, clamp. */
int oracle_qlinearadd_u8(const uint8_t* a, float a_scale, uint8_t a_zp, const uint8_t* b, float b_scale, uint8_t b_zp,
                         float y_scale, uint8_t y_zp, uint8_t* y, long long n) {
  const float sa = a_scale / y_scale, sb = b_scale / y_scale;
  const float fixed = (float)y_zp - fmaf(sa, (float)a_zp, sb * (float)b_zp);
  const long long vec_end = n / 16 * 16;
  for (long long i = 0; i < n; ++i) {
    if (i < vec_end) {
      float v = fmaf((float)b[i], sb, fixed);
      v = fmaf((float)a[i], sa, v);
      y[i] = sat_u8((int)nearbyintf(v));
    } else {
      const float da = (float)((int)a[i] - a_zp), db = (float)((int)b[i] - b_zp);
      y[i] = sat_u8((int)nearbyintf(fmaf(sa, da, sb * db) + (float)y_zp));
    }
  }
  return ORACLE_OK;
}

/* DequantizeLinear -> GlobalAveragePool (NHWC, per-channel sum from 0 over
 * the spatial positions in order, times 1/spatial; kernel/pool.h:109-125)
 * -> QuantizeLinear, on u8 [n, hw, c] -> u8 [n, c]. */
int oracle_dq_gap_q_u8_nhwc(const uint8_t* x, int n, int hw, int c, float xs, uint8_t xzp, float ys, uint8_t yzp,
                            uint8_t* y) {
  const float inv_hw = 1.0f / (float)hw;
  float* v = (float*)malloc(sizeof(float) * (size_t)n * c);
  if (!v) return ORACLE_ERR;
  for (int img = 0; img < n; ++img)
    for (int ch = 0; ch < c; ++ch) {
      float sum = 0.0f;
      for (int s = 0; s < hw; ++s) sum += ((float)x[((size_t)img * hw + s) * c + ch] - (float)xzp) * xs;
      v[(size_t)img * c + ch] = sum * inv_hw;
    }
  const int rc = oracle_quantize_u8(v, y, (long long)n * c, ys, yzp);
  free(v);
  return rc;
}

/* GlobalAveragePool on fp32 NHWC [n, hw, c] -> [n, c]: per channel a sum
 * from 0 over the spatial positions in order, times 1/spatial
 * (kernel/pool.h:109-125). */
int oracle_gap_f32_nhwc(const float* x, int n, int hw, int c, float* y) {
  const float inv_hw = 1.0f / (float)hw;
  for (int img = 0; img < n; ++img)
    for (int ch = 0; ch < c; ++ch) {
      float sum = 0.0f;
      for (int s = 0; s < hw; ++s) sum += x[((size_t)img * hw + s) * c + ch];
      y[(size_t)img * c + ch] = sum * inv_hw;
    }
  return 0;
}

/* DequantizeLinear of u8 [rows, cols] then + bias[cols] (fp32 Add). */
int oracle_dequantize_u8(const uint8_t* x, float scale, uint8_t zp, const float* bias, int rows, int cols, float* y) {
  for (long long i = 0; i < (long long)rows * cols; ++i) {
    float v = ((float)x[i] - (float)zp) * scale;
    if (bias) v = v + bias[i % cols];
    y[i] = v;
  }
  return ORACLE_OK;
}
