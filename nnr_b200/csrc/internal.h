// Internal declarations shared by the translation units of libnnrcu.so.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <vector>

#include "nnrcu.h"

namespace nnrcu {

// Records a formatted message as this thread's last error and returns code.
int set_error(int code, const char* fmt, ...);
// Maps a CUDA error to NNRCU_ERR_CUDA with a message; NNRCU_OK on success.
int cuda_check(cudaError_t e, const char* what);
#define NNRCU_CUDA(call)                                  \
  do {                                                    \
    int _rc = ::nnrcu::cuda_check((call), #call);         \
    if (_rc != NNRCU_OK) return _rc;                      \
  } while (0)

// Whether engine kernels are launched with programmatic dependent launch
// (on unless the environment sets NNRCU_PDL=0).
bool pdl_enabled();

// Grouped conv weights [oc][c / g][kh][kw] as the block-diagonal dense
// weights [oc][c][kh][kw] of the same conv (zeros between the groups): a
// grouped Conv / QLinearConv runs as a group-1 conv whose extra products are
// exact zeros (nnr's grouped path computes each group's sums on their own).
template <typename T>
std::vector<T> grouped_to_dense(const T* w, int oc, int c, int g, int kh, int kw) {
  const int cg = c / g, og = oc / g, taps = kh * kw;
  std::vector<T> d((size_t)oc * c * taps, T(0));
  for (int o = 0; o < oc; ++o) {
    const int gi = o / og;
    for (int ic = 0; ic < cg; ++ic)
      for (int t = 0; t < taps; ++t)
        d[((size_t)o * c + gi * cg + ic) * taps + t] = w[((size_t)o * cg + ic) * taps + t];
  }
  return d;
}
bool shift_enabled();
bool r2_sat_enabled();

// Device address of this device's status word (set up once per device).
int* status_ptr();

// cuTensorMapEncodeTiled through the runtime's driver entry point.
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// cuTensorMapEncodeIm2col over an NHWC tensor [n][h][w][c] (c in elements,
// row of c*elem bytes): boxes of 128 pixels x (128 bytes of channels), with
// the bounding box of a conv with the given pads/kernel/dilation/stride.
int encode_tmap_im2col(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, int n, int h,
                       int w, int c, int pt, int pl, int pb, int pr, int kh, int kw, int dh, int dw, int sh, int sw,
                       int kslab = 128);

// cuTensorMapEncodeTiled of a rank 1..5 tensor (dims innermost first, rank - 1 strides).
int encode_tmap_nd(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);
// cuTensorMapEncodeTiled of a 3-d tensor (dims innermost first).
int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
                   const uint64_t strides_bytes[2], const uint32_t box[3],
                   CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

enum OpKind : int { OP_QCONV = 1, OP_QMATMUL = 2, OP_CONV_F32 = 3, OP_GEMM_F32 = 4, OP_DWCONV_F32 = 5, OP_QDW = 6, OP_CONV_HALF = 7,
                   OP_GEMM_HALF = 8, OP_GEMM_F32_BF16 = 9 };

// One prepared operator: packed weights on the device plus everything the
// launch needs. Created by nnrcu_*_create, consumed by nnrcu_*_run.
struct Op {
  int kind = 0;
  int device = 0;
  nnrcu_conv_desc d{};
  // GEMM view
  int M = 0, N = 0, K = 0;      // K in elements
  int kbytes = 0;               // real K per plane in bytes
  int kpad_bytes = 0;           // packed B row length in bytes (multiple of 128)
  int num_kb = 0;
  int npad = 0;                 // packed B rows per plane
  int bn = 128;
  int kslab = 128;              // K bytes per pipeline stage (128 or 64)
  int amode = 1;                // A_TMA / A_GATHER
  int epi = 0;
  int nplane = 1;
  int oh = 0, ow = 0;
  int cs = 0;                   // device channel stride (elements) of the NHWC operand
  bool need_in_copy = false;    // input must be re-laid-out into the workspace first
  bool pad_in = false;
  int shift_prows = 0;  // A_SHIFT: patch rows per K slab
  bool in_padded = false;        // x is already the x_zp-bordered padded copy (A_SHIFT, NHWC input)
  int out_pad[4] = {0, 0, 0, 0};  // output written into a padded NHWC buffer (top, left, bottom, right)
  bool explicit_im2col = false; // small-C conv: A materialised densely as [M][kpad] in the workspace
  // Space-to-depth form of a stride-2 small-channel conv (the stem): the
  // input is reordered into s2d pixels of 16 bytes ((dy, dx, c) for 4c <= 16)
  // inside an x_zp border, and convolved at stride 1 with an s2d kernel
  // s2d_kh x s2d_kw (taps of 16 bytes, 8 per 128-byte K slab).
  bool s2d = false;
  int s2d_kh = 0, s2d_kw = 0, s2d_pt = 0, s2d_pl = 0, s2d_hp = 0, s2d_wp = 0;
  int s2d_tpr = 0;              // A_ROWS: taps per s2d kernel row in K (0: hardware im2col instead)
  // device buffers (owned)
  void* wB = nullptr;
  void* wBimg = nullptr;       // int8 B as per-(N tile, K slab) shared-memory images (bulk-copied)
  int32_t* colcorr = nullptr;
  int32_t* bias_i = nullptr;
  float* cs_arr = nullptr;
  float* bias_f = nullptr;
  float* os = nullptr;
  float* bias = nullptr;
  float* cmat = nullptr;        // Gemm C when it is a full matrix
  float* w_dw = nullptr;        // depthwise weights [kh][kw][c]
  CUtensorMap tmB{};
  // requant scalars
  float inv_y = 0, yzp_f = 0, qmin_f = 0, qmax_f = 0, rq_lo = 0, rq_hi = 0, combined = 0;
  int yzp = 0;
  float y_scale = 0;
  int x_zp = 0;
  int a_zp = 0, b_zp = 0;
  // fp32 post-op
  int act = 0;
  float act_a = 0, act_b = 0;
  float beta = 0;
  int c_rows = 0;
  int trans_a = 0;
  size_t ws_bytes = 0;
  size_t out_off = 0;           // 16-bit ops: offset of the fp32 result in the workspace
  int64_t num_ops = 0;
};

// Launch of the tcgen05 engine (tc_launch.cu).
struct TcLaunch {
  int bn, nplane, amode, epi;
  int m_tiles, n_tiles;
  const CUtensorMap* tmA0;
  const CUtensorMap* tmA1;
  const CUtensorMap* tmB;
  int b_plane_rows;
  int num_kb;
  int kb_bytes = 128;  // K bytes per pipeline stage (128, or 64 for 64-byte channel strides);
                       // 16: 128-byte stages of eight 16-byte taps (the s2d path)
};
struct GatherGeom;
struct EpiParams;
int tc_launch(const TcLaunch& L, const GatherGeom& g, const EpiParams& e, cudaStream_t stream);
// Picks the N tile (64/128/256) that minimises the estimated waves x tile cost.
int pick_bn(int M, int N, int nplane, int num_sms);
// Lays B (through its tensor map: box kb_bytes x bn) out as the shared-memory
// image of every (N tile, K slab), in that order, into out
// (n_tiles * num_kb * bn * kb_bytes bytes). Synchronous.
int pack_b_images(const CUtensorMap* tmB, int bn, int kb_bytes, int n_tiles, int num_kb, void* out);
bool bimg_enabled();
bool xrows_enabled();
bool xrows_map_ok();
int num_sms();
// Depthwise QLinearConv (qdw.cu).
int qdw_create(const nnrcu_conv_desc& d, int oh, int ow, const int8_t* w_host, const float* w_scale, int n_w_scale,
               const int8_t* w_zp, int n_w_zp, const int32_t* bias_host, float x_scale, uint8_t x_zp, float y_scale,
               uint8_t y_zp, nnrcu_op** out);
int qdw_run(nnrcu_op* op, const uint8_t* x, uint8_t* y, void* workspace, cudaStream_t st);
// fp32 Gemm with bf16-rounded operands (half.cu, NNRCU_PREC_BF16).
int gemm_f32_bf16_run(nnrcu_op* op, const float* a, float* y, void* workspace, cudaStream_t st);


// Auxiliary kernels (aux_kernels.cu).
int launch_nchw_to_nhwc_u8(const uint8_t* src, uint8_t* dst, int n, int c, int h, int w, int cs, uint8_t fill,
                           cudaStream_t st);
int launch_nchw_to_nhwc_u8_padded(const uint8_t* src, uint8_t* dst, int n, int c, int h, int w, int pt, int pl,
                                  int pb, int pr, int cs, uint8_t fill, cudaStream_t st);
int launch_im2col_u8(const uint8_t* x, uint8_t* a, int nchw, int n, int c, int h, int w, int oh, int ow, int kh,
                     int kw, int sh, int sw, int pt, int pl, int dh, int dw, int kp, uint8_t x_zp, cudaStream_t st);
// Space-to-depth reorder into the padded layout of the s2d conv path:
// dst[n][hp][wp][16], pixel (Y, X) holds input (2(Y - pt) + dy, 2(X - pl) + dx)
// channels c at byte (dy * 2 + dx) * C + c; out-of-image bytes and the bytes
// past 4C hold fill.
int launch_s2d_u8(const uint8_t* x, int nchw, uint8_t* dst, int n, int c, int h, int w, int hp, int wp, int pt, int pl,
                  uint8_t fill, cudaStream_t st);
// QuantizeLinear (per tensor) fused into launch_s2d_u8's reorder, from fp32.
int launch_quantize_s2d(const float* x, int nchw, uint8_t* dst, int n, int c, int h, int w, int hp, int wp, int pt,
                        int pl, uint8_t fill, float scale, uint8_t zp, cudaStream_t st);
int launch_pad_nhwc_u8(const uint8_t* src, uint8_t* dst, int pixels, int c, int cs, uint8_t fill, cudaStream_t st);
// NHWC [n][h][w][cs] -> [n][h+pt+pb][w+pl+pr][cs] with a border of fill bytes.
int launch_pad_spatial_nhwc_u8(const uint8_t* src, uint8_t* dst, int n, int h, int w, int cs, int pt, int pl, int pb,
                               int pr, uint8_t fill, cudaStream_t st);
int launch_split_bf16_nhwc(const float* src, int src_nchw, uint16_t* hi, uint16_t* lo, int n, int c, int h, int w,
                           int cs, cudaStream_t st);
// Explicit im2col of an fp32 conv input into split-bf16 rows [M][kp].
int launch_im2col_split_bf16(const float* x, int nchw, uint16_t* hi, uint16_t* lo, int n, int c, int h, int w,
                             int oh, int ow, int kh, int kw, int sh, int sw, int pt, int pl, int dh, int dw, int kp,
                             cudaStream_t st);
int launch_split_bf16_rows(const float* src, int trans, uint16_t* hi, uint16_t* lo, int m, int k, int kp,
                           cudaStream_t st);
int launch_rowcorr_u8(const uint8_t* a, int m, int k, int lda, int b_zp, int32_t* out, cudaStream_t st);
int launch_transpose_generic(const void* src, void* dst, int n, int c, int hw, int elem, int to_nhwc,
                             cudaStream_t st);
int launch_depthwise_f32(const Op& op, const float* x_nhwc, float* y, const float* residual, cudaStream_t st);
int launch_depthwise_f32_planes(const Op& op, const float* x_nhwc, uint16_t* hi, uint16_t* lo, int cs,
                                cudaStream_t st);
// 16-bit NHWC depthwise (dtype NNRCU_DT_BF16 / NNRCU_DT_F16): fp32 sums, rounded once
int launch_depthwise_half(const Op& op, const uint16_t* x_nhwc, uint16_t* y, int dtype, cudaStream_t st);

void host_split_bf16(float v, uint16_t* hi, uint16_t* lo);

}  // namespace nnrcu

struct nnrcu_op : nnrcu::Op {};
