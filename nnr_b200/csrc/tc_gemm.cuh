// Implicit-GEMM engine on the 5th-generation tensor cores (tcgen05) for the
// Conv / QLinearConv / QLinearMatMul / Gemm / MatMul operators.
//
// GEMM view: D[M, N] = A[M, K] * B[N, K]^T, both operands K-major in bytes.
//   * conv:   M = output pixels (n, oh, ow), N = output channels,
//             K = (kh, kw, ic) with ic padded to a 16-byte channel stride.
//   * matmul: M = rows of A, N = columns of B, K = the reduction dim.
//
// One CTA computes a 128 x BN tile of D:
//   warps 0-3  epilogue (TMEM -> registers -> requant / bias / post-op -> HBM)
//   warps 4-7  A producers in gather mode (cp.async from NHWC activations,
//              padding pixels filled with the input zero point)
//   warp 8     TMA producer (B tiles always; A tiles in TMA mode, i.e. plain
//              2-D tiles, and in im2col mode, i.e. hardware implicit im2col
//              over an NHWC tensor whose channel stride is a multiple of 128 B)
//   warp 9     TMEM allocator and single-thread tcgen05.mma issuer
// The kernel is persistent: one CTA per SM loops over tiles, with the
// accumulator double-buffered in TMEM.
// Shared memory holds STAGES stages of {A planes, B planes}, each plane a
// 128-byte-wide K slab in the 128-byte swizzled K-major layout that both TMA
// (SWIZZLE_128B) and the UMMA descriptors understand.
//
// NPLANE = 1: int8 (kind::i8, u8 activations x s8 weights, s32 accumulate).
// NPLANE = 3 / 4: one bf16 / fp16 plane (kind::f16, f32 accumulate): the
//             16-bit I/O variants, one exact product per multiply-add.
// NPLANE = 2: fp32 emulated as split bf16 (kind::f16, f32 accumulate):
//             a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi with x_hi = bf16(x),
//             x_lo = bf16(x - x_hi); the dropped a_lo*b_lo term is < 2^-16
//             relative per product.
#pragma once
#include <cstdint>
#include <type_traits>
#include <cuda.h>
#include "ptx.cuh"

namespace nnrcu {

// A_ROWS: stride-1 convs over 16-byte pixels of a padded NHWC image (the
// space-to-depth path). A tile covers up to 128 pixels of ONE output row; for
// each kernel row one contiguous bulk copy brings BM + 8 input pixels, and the
// kernel's taps along that row are the same rows shifted by 16 bytes each.
// A_SHIFT: stride-1 convs over an NHWC input whose spatial border (the
// padding, x_zp bytes) is materialised. Output positions are enumerated on
// the padded grid [N][Hp][Wp] (positions with oh >= OH or ow >= OW are
// computed and discarded), so the input rows that tap (kh, kw) needs for a
// tile's 128 positions are the tile's own rows shifted by kh * Wp + kw: one
// TMA copy per K slab brings the tile's patch (BM + (KH-1) * Wp + KW - 1 rows)
// once, and every tap is a view of it starting at a shifted row. The 64/128-
// byte swizzle is a function of the shared-memory address, so a view may
// start at any row of the swizzled patch. B is resident.
// A_XROWS: the same space-to-depth convs with 4 taps per kernel row, read
// as 64-byte rows: a 2-D tensor map over the s2d image whose rows are 16
// bytes apart (row p = taps p .. p + 3 of one s2d row), so that one K slab is
// one kernel row of a tile in the 64-byte swizzled layout (a swizzled MMA
// operand instead of the 16-byte-interleaved one of A_ROWS).
enum : int { A_TMA = 0, A_GATHER = 1, A_IM2COL = 2, A_ROWS = 3, A_SHIFT = 4, A_XROWS = 5 };
constexpr int ROWS_BYTES = (128 + 8) * 16;  // one A_ROWS copy: BM + 8 pixels of 16 bytes
// EPI_R2A: the R2 requant followed by a fused QLinearAdd whose residual
// tiles are TMA-prefetched one tile ahead (u8 row-major output via TMA store).
// EPI_R3N: R3 with an NCHW output, whose last OW % 16 pixels of each output
// row take the first-layer kernel's scalar tail sequence (a separate
// instance, so that the NHWC stem keeps its register budget).
enum : int { EPI_R1 = 1, EPI_R2 = 2, EPI_R3 = 3, EPI_R4 = 4, EPI_R2A = 5, EPI_R3N = 6, EPI_F32 = 10 };
enum : int { ACT_NONE = 0, ACT_RELU = 1, ACT_CLIP = 2, ACT_HARDSWISH = 3, ACT_SIGMOID = 4, ACT_LEAKYRELU = 5,
             ACT_TANH = 6 };
enum : int { ST_OK = 0, ST_TIMEOUT_FULL = 1, ST_TIMEOUT_EMPTY = 2, ST_TIMEOUT_ACCUM = 3, ST_SMEM = 4 };

// Opt-in phase trace for performance analysis (built only with -DNNRCU_TRACE):
// clock64 stamps of CTAs 0-3, per warp, per local tile (first 16), 4 events.
#ifdef NNRCU_TRACE
__device__ unsigned long long g_trace[4 * 24 * 16 * 4];
#define NNRCU_TRACE_AT(w, t, ev)                                                       \
  do {                                                                                 \
    if (blockIdx.x < 4 && (t) < 16) g_trace[((blockIdx.x * 24 + (w)) * 16 + (t)) * 4 + (ev)] = clock64(); \
  } while (0)
// finer stamps inside a tile's epilogue: CTAs 0-1, first 4 tiles, 16 events
__device__ unsigned long long g_trace2[2 * 24 * 4 * 16];
#define NNRCU_TRACE2_AT(w, t, ev)                                                       \
  do {                                                                                  \
    if (blockIdx.x < 2 && (t) < 4 && (ev) < 16) g_trace2[((blockIdx.x * 24 + (w)) * 4 + (t)) * 16 + (ev)] = clock64(); \
  } while (0)
// per launch (trace_seq): earliest CTA start, latest CTA end, earliest CTA
// end, latest CTA start, in globaltimer ns
__device__ unsigned long long g_span[256 * 4];
#define NNRCU_SPAN_BEGIN() const unsigned long long span_t0 = ptx::globaltimer()
#define NNRCU_SPAN_END()                                                                       \
  do {                                                                                         \
    if (threadIdx.x == 0 && e.trace_seq >= 0 && e.trace_seq < 256) {                            \
      const unsigned long long t1 = ptx::globaltimer();                                        \
      atomicMin(&g_span[e.trace_seq * 4 + 0], span_t0);                                        \
      atomicMax(&g_span[e.trace_seq * 4 + 1], t1);                                             \
      atomicMin(&g_span[e.trace_seq * 4 + 2], t1);                                             \
      atomicMax(&g_span[e.trace_seq * 4 + 3], span_t0);                                        \
    }                                                                                          \
  } while (0)
#else
#define NNRCU_SPAN_BEGIN() \
  do {                     \
  } while (0)
#define NNRCU_SPAN_END() \
  do {                   \
  } while (0)
#define NNRCU_TRACE2_AT(w, t, ev) \
  do {                            \
  } while (0)
#define NNRCU_TRACE_AT(w, t, ev) \
  do {                           \
  } while (0)
#endif

constexpr int BM = 128;       // rows per tile (TMEM lanes)
constexpr int BKB = 128;      // K bytes per stage per plane (one swizzle row); 64 for the 64-byte-slab variant
// Warp roles per A-operand mode and N tile:
//   gather mode:    warps 0-3 epilogue, 4-7 gather producers, 8 TMA, 9 MMA
//   TMA / im2col:   warps 0 .. 4*SPLIT-1 epilogue, then 3 TMA producers, then MMA, with
//                   SPLIT epilogue warps per TMEM lane quarter, each draining
//                   BN / SPLIT columns (16 warps for BN >= 128: the epilogue,
//                   not the tensor core, bounds the small-K layers)
template <int AMODE, int BN, int EPI = 0>
struct Roles {
  static constexpr int SPLIT = AMODE == A_GATHER ? 1 : (BN >= 128 ? 4 : 2);
  // 64-wide N tiles of u8 epilogues (other than the residual-prefetching
  // EPI_R2A): two groups of 4 x SPLIT epilogue warps take alternate tiles,
  // one per TMEM accumulator, so that two tiles' requantisation is in flight
  static constexpr int EGROUPS =
      (BN == 64 && AMODE != A_GATHER && EPI != 0 && EPI != EPI_R2A && EPI != EPI_F32) ? 2 : 1;
  static constexpr int TMA_WARP = AMODE == A_GATHER ? 8 : 4 * SPLIT * EGROUPS;
  // TMA-fed modes issue their copies from three producer warps (stage it
  // goes to warp it % NPROD): one warp's copies complete at about one per
  // several hundred cycles, so more issuing warps raise the load rate (1.4x
  // with two, 1.8x with four). Three keeps the warp count a multiple of four,
  // so each SM sub-partition holds the same number of warps and the
  // register budget per thread stays at 96 with sixteen epilogue warps.
  // (A_SHIFT issues one patch copy per K slab per tile: one producer.)
  static constexpr int NPROD = (AMODE == A_GATHER || AMODE == A_SHIFT) ? 1 : 3;
  static constexpr int MMA_WARP = TMA_WARP + NPROD;
  static constexpr int THREADS = (MMA_WARP + 1) * 32;
  static constexpr int CW = 32;  // accumulator columns per TMEM load
};

// Geometry of the implicit im2col gather (A_GATHER). All sizes in bytes where noted.
struct GatherGeom {
  const uint8_t* x;      // NHWC activations, plane 0
  const uint8_t* x2;     // plane 1 (bf16 low halves) or null
  int N, H, W;
  int cbytes;            // bytes per pixel (channel stride), multiple of 16
  int OH, OW, KH, KW, sh, sw, ph, pw, dh, dw;
  int kbytes;            // real K in bytes = KH*KW*cbytes
  uint32_t pad_word;     // value written for padding pixels (x_zp replicated, or 0)
  int tpr;               // A_ROWS: taps per kernel row in K (2, 4 or 8; taps past KW have zero weights)
  int prows;             // A_SHIFT: patch rows per K slab (BM + (KH-1)*W + KW-1, rounded up to a 1 KB multiple)
  const uint8_t* wb;     // KB = 16: weights as per-(N tile, K slab) shared-memory images of BN x 128 bytes
};

struct EpiParams {
  int M, N;              // logical GEMM extent
  // int8 requantisation (per output channel arrays are indexed by n)
  const int32_t* colcorr;  // -x_zp * sum(w) (+ K*a_zp*b_zp), or null
  const int32_t* rowcorr;  // per-row correction (QLinearMatMul with b_zp != 0), or null
  const int32_t* bias_i;   // R2 int32 bias, or null
  const float* cs;         // R1/R3 combined scale x_scale*w_scale[n]
  const float* bias_f;     // R1/R3 float bias = bias*cs, or null
  const float* os;         // R2 output scale cs*inv_y
  float inv_y, yzp_f, qmin_f, qmax_f;  // R1/R3/R4
  float rq_lo, rq_hi;                  // R2 clamp bounds (lo - y_zp, hi - y_zp)
  float combined;                      // R4 scalar scale a_s*b_s/y_s
  int yzp;                             // R2 integer zero point
  int r2_sat;                          // R2 bounds are [0, 255] with y_zp = 0: one saturating conversion
  // Fused QLinearAdd after the requant (u8 epilogues): y = QLinearAdd(q, qres)
  // with qres laid out like y. Same float sequence as the standalone op.
  const uint8_t* qres;                 // residual operand b, or null
  float qa_sa, qa_sb, qa_fixed;        // a_s / y_s, b_s / y_s, y_zp - fma(sa, a_zp, sb * b_zp)
  int qa_azp, qa_bzp, qa_yzp;
  long long qa_vec_end;                // elements below use the 16-wide body, the rest the scalar tail
  int qa_ovf;                          // the add value may reach 2^31 (255 (|sa| + |sb|) + |fixed| >= 2^30)
  // fp32 epilogue
  const float* bias;       // per-n bias or null
  const float* residual;   // same layout as y, or null
  int res_mode;            // 1: v = act(acc + bias + res_scale*res); 2: v = act(acc + bias) + res
  float res_scale;
  int act; float act_a, act_b;
  // output
  void* y;
  int y_layout;            // 0: row-major [M, ldy]; 1: NCHW with M = img*ohw + p
  int ldy, ohw;
  // opad: u8 row-major output written into the interior of a spatially padded
  // NHWC buffer: output pixel m = (img, oy, ox) of an o_h x o_w image goes to
  // row img * o_hwp + oy * o_wp + ox + o_off (o_off = top * o_wp + left)
  int opad, o_w, o_hw, o_wp, o_hwp, o_off;
  int* status;             // device status word (first error wins)
  int trace_seq;           // trace builds: this launch's slot in g_span
};

// NKBR > 0: the whole B operand (num_kb <= NKBR slabs of one N tile) stays
// resident in shared memory, loaded once per CTA; the stage ring holds A only.
// PATCH (A_SHIFT): the stage ring is two patch buffers that share what the
// resident B leaves; outputs are stored directly (no staging).
template <int BN, int NPLANE, int EPI, int KB = BKB, int SPLIT = 1, int NKBR = 0, int PATCH = 0>
struct TileCfg {
  static constexpr int BUDGET = 212 * 1024;  // stages + staging + resident B
  // K bytes per stage: KB, except KB = 16 (eight 16-byte taps per 128-byte stage)
  static constexpr int SLAB = KB == 16 ? 128 : KB;
  static constexpr int B_BYTES = BN * SLAB;
  static constexpr int BRES_BYTES = NKBR * B_BYTES;
  static constexpr int PATCH_BYTES = PATCH ? ((BUDGET - BRES_BYTES) / 2) & ~1023 : 0;  // per patch buffer
  static constexpr int A_BYTES = PATCH ? PATCH_BYTES : BM * SLAB;  // 16 KB per plane (8 KB with 64-byte slabs)
  static constexpr int PL = NPLANE == 2 ? 2 : 1;  // shared-memory planes per operand
  static constexpr int STAGE_BYTES = PL * (A_BYTES + (NKBR ? 0 : B_BYTES));
  // Epilogues stage each warp's 32-row output block for a TMA store: u8
  // always; fp32 (4 bytes per element) when that still leaves three stages.
  static constexpr int ESZ = EPI == EPI_F32 ? 4 : 1;
  static constexpr int OUT_BLOCK_RAW = 4 * 32 * BN * ESZ;  // one 32 x HB block per epilogue warp
  static constexpr int OUT_BLOCK =
      PATCH ? 0 : ((EPI == EPI_F32 && (BUDGET - OUT_BLOCK_RAW - BRES_BYTES) / STAGE_BYTES < 3) ? 0 : OUT_BLOCK_RAW);
  // EPI_R2A: two residual blocks per epilogue warp (tile i in use, tile i+1 landing)
  // The residual block of EPI_R2A: TMA-prefetched one tile ahead into
  // shared memory, or (64-byte K slabs, i.e. the K = 64 layers whose
  // epilogue is the bottleneck) read by each lane with plain loads issued
  // before its requantisation: there the TMA issue of the prefetch stalled
  // the epilogue warps for ~500 cycles per tile behind the producers' copies.
  static constexpr bool RES_TMA = KB != 64;
  static constexpr int RES_BYTES = (EPI == EPI_R2A && RES_TMA) ? 2 * OUT_BLOCK : 0;
  // Output staging is double-buffered (the store of tile i drains while tile
  // i+1 is requantised) when that still leaves three pipeline stages.
  static constexpr int OUT_BUFS = (BUDGET - 2 * OUT_BLOCK - RES_BYTES - BRES_BYTES) / STAGE_BYTES >= 3 ? 2 : 1;
  static constexpr int OUT_BYTES = OUT_BUFS * OUT_BLOCK;
  // Epilogue warps: 4 x SPLIT, each covering 32 TMEM lanes x BN / SPLIT columns.
  static constexpr int HB = BN / SPLIT;
  static constexpr int ROW_BYTES = HB * ESZ;                       // bytes of one staged row
  static constexpr int OUT_SEG = ROW_BYTES >= 128 ? 128 : ROW_BYTES;  // bytes per staged row segment (= TMA box width)
  static constexpr int STAGES_RAW = (BUDGET - OUT_BYTES - RES_BYTES - BRES_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = PATCH ? 2 : (STAGES_RAW > 12 ? 12 : STAGES_RAW);
  // Gather producers publish a stage LAG iterations after issuing it: LAG
  // stages of copies in flight, STAGES - 1 - LAG stages of slack for the MMA.
  static constexpr int LAG = (STAGES - 1) / 2 > 1 ? (STAGES - 1) / 2 : 1;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators (power of two)
  static constexpr int PARAM_BYTES = (BN == 64 ? 2 : 1) * 4 * SPLIT /*epilogue warps*/ * 3 * HB * 4;
  static constexpr int BAR_BYTES = 1024;  // mbarriers, TMEM slot, abort flag
  static constexpr int SMEM_BYTES =
      1024 /*align slack*/ + STAGES * STAGE_BYTES + BRES_BYTES + OUT_BYTES + RES_BYTES + BAR_BYTES + PARAM_BYTES;
  static_assert(STAGES >= 2, "need at least two pipeline stages");
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

// The tile configuration of one engine instance; the kernel's shared-memory
// carve-up and the launcher's allocation both come from this one alias.
template <int BN, int NPLANE, int AMODE, int EPI, int KB, int NKBR>
using KernelCfg = TileCfg<BN, NPLANE, EPI, KB, Roles<AMODE, BN>::SPLIT, NKBR, AMODE == A_SHIFT ? 1 : 0>;

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ float apply_act(float v, int act, float a, float b) {
  switch (act) {
    case ACT_RELU: return fmaxf(v, 0.0f);
    case ACT_CLIP: return fminf(fmaxf(v, a), b);
    case ACT_HARDSWISH: {
      // HardSwish(x) = x * max(0, min(1, x/6 + 0.5))
      float t = fmaf(v, 1.0f / 6.0f, 0.5f);
      t = fminf(fmaxf(t, 0.0f), 1.0f);
      return v * t;
    }
    case ACT_SIGMOID: return 1.0f / (1.0f + expf(-v));
    case ACT_LEAKYRELU: return v >= 0.0f ? v : v * a;
    case ACT_TANH: return tanhf(v);
    default: return v;
  }
}

// Rounding through the float adder: for |x| <= 2^22, x + 1.5 * 2^23 is
// rounded to an integer (ulp 1 in [2^23, 2^24)) with ties to even, because
// 1.5 * 2^23 is even; the integer rne(x) then sits in the low mantissa bits
// (bits = 0x4B400000 + rne(x), two's complement offset). This is exact
// round-to-nearest-even, done on the FMA pipe instead of the conversion unit.
constexpr float RND_MAGIC = 12582912.0f;   // 1.5 * 2^23, bits 0x4B400000
constexpr float BYTE_MAGIC = 8388608.0f;   // 2^23, bits 0x4B000000: 0x4B0000bb = 2^23 + bb

// R2 requant up to the rounding: returns RND_MAGIC + rne(f) as a float,
// where f = clamp(float(acc + bias) * os, lo - y_zp, hi - y_zp) (|f| <= 255).
__device__ __forceinline__ float r2_magic(int32_t raw, int32_t ci, float os, float lo, float hi) {
  const int32_t v = (int32_t)((uint32_t)raw + (uint32_t)ci);
  float f = __fmul_rn(__int2float_rn(v), os);
  f = fminf(fmaxf(f, lo), hi);
  return __fadd_rn(f, RND_MAGIC);
}
__device__ __forceinline__ float r2_magic(int32_t raw, int32_t ci, float os, const EpiParams& e) {
  return r2_magic(raw, ci, os, e.rq_lo, e.rq_hi);
}

// Requantise one int32 accumulator to u8 with the formula EPI selects; the
// result is in the low byte of the returned word (upper bytes unspecified).
// ci is the per-column int32 correction (-x_zp*sum(w), plus the int32 bias
// for R2); f1/f2 are the per-column floats (R1/R3: cs, bias_f; R2: os).
template <int EPI>
__device__ __forceinline__ uint32_t requant_u8(int32_t raw, int32_t ci, int32_t rowc, float f1, float f2,
                                               const EpiParams& e) {
  if constexpr (EPI == EPI_R1) {
    // f = fma(float(acc), cs, bias_f); f = rne(f * inv_y) + y_zp; min(hi) then max(qmin)
    int32_t acc = (int32_t)((uint32_t)raw + (uint32_t)ci);
    float f = __fmaf_rn(__int2float_rn(acc), f1, f2);
    f = rintf(__fmul_rn(f, e.inv_y));
    f = __fadd_rn(f, e.yzp_f);
    f = fmaxf(fminf(f, e.qmax_f), e.qmin_f);
    return (uint32_t)__float2int_rn(f);
  } else if constexpr (EPI == EPI_R2 || EPI == EPI_R2A) {
    // f = float(acc + bias) * os; max(lo - y_zp) then min(hi - y_zp); rne; + y_zp.
    // f lies in [-y_zp, 255 - y_zp] (integral bounds), so rne(f) + y_zp is
    // already in [0, 255]: the unsigned saturation of the reference is a no-op
    return __float_as_uint(r2_magic(raw, ci, f1, e)) + (uint32_t)e.yzp;
  } else if constexpr (EPI == EPI_R3 || EPI == EPI_R3N) {
    // f = fma(float(acc), cs, bias_f); f = fma(f, inv_y, y_zp); min(hi) then max(qmin); rne
    // (the clamp bounds are integers in [0, 255], so rne commutes with the clamp)
    int32_t acc = (int32_t)((uint32_t)raw + (uint32_t)ci);
    float f = __fmaf_rn(__int2float_rn(acc), f1, f2);
    f = __fmaf_rn(f, e.inv_y, e.yzp_f);
    f = fmaxf(fminf(f, e.qmax_f), e.qmin_f);
    return __float_as_uint(__fadd_rn(f, RND_MAGIC));
  } else {  // EPI_R4
    // val = fma(float(acc), a_s*b_s/y_s, y_zp); nearbyint; clamp [0, 255]
    // == rne(clamp(val, 0, 255)), the clamp bounds being integers, except that
    // the x86 conversion turns values >= 2^31 into INT_MIN (clamped to 0)
    int32_t acc = (int32_t)((uint32_t)raw + (uint32_t)ci + (uint32_t)rowc);
    float f = __fmaf_rn(__int2float_rn(acc), e.combined, e.yzp_f);
    f = f >= 2147483648.0f ? 0.0f : fminf(fmaxf(f, 0.0f), 255.0f);
    return __float_as_uint(__fadd_rn(f, RND_MAGIC));
  }
}

// R3 for one output row: the vector body
//   f = fma(float(acc), cs, bias_f); q = rne(clamp(fma(f, inv_y, y_zp), qmin, 255))
// or, for the first-layer kernel's NCHW remainder pixels (tail), its scalar
//   q = clamp(int(rne(f * inv_y)) + y_zp, qmin, 255)
// with the x86 conversion (out-of-range values become INT_MIN). add_f / add_i
// place y_zp before or after the rounding; the clamp bounds are integers, so
// clamping after the rounding equals the body's clamp before it, and the
// saturating conversion keeps huge values at the upper bound there.
__device__ __forceinline__ uint32_t requant_r3_row(int32_t raw, int32_t ci, float f1, float f2, float add_f,
                                                   int32_t add_i, bool tail, const EpiParams& e) {
  const int32_t acc = (int32_t)((uint32_t)raw + (uint32_t)ci);
  const float g = __fmaf_rn(__fmaf_rn(__int2float_rn(acc), f1, f2), e.inv_y, add_f);
  int32_t q = tail ? ptx::cvt_rne_x86(g) : __float2int_rn(g);
  q = (int32_t)((uint32_t)q + (uint32_t)add_i);
  q = max(q, (int32_t)e.qmin_f);
  q = min(q, (int32_t)e.qmax_f);
  return (uint32_t)q;
}

// Low bytes of four words packed into one (byte j from word j).
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Byte j of w as an exact float: bits 0x4B0000bb = 2^23 + bb, minus 2^23.
__device__ __forceinline__ float byte_to_float(uint32_t w, int j) {
  return __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650 | j)), BYTE_MAGIC);
}

// Persistent warp-specialised kernel. One CTA per SM walks the tiles
// blockIdx.x, blockIdx.x + gridDim.x, ...; tile t covers rows
// [(t / n_tiles) * 128, +128) and columns [(t % n_tiles) * BN, +BN).
//   warps 0-3  epilogue: TMEM -> registers -> requant / bias / post-op -> HBM
//   warps 4-7  A producers in gather mode (implicit im2col with cp.async)
//   warp 8     TMA producer (B always, A in TMA mode)
//   warp 9     TMEM allocator + single-thread tcgen05.mma issuer
// The smem stage ring runs continuously across tiles, and the accumulator is
// double-buffered in TMEM (2 x BN columns), so the epilogue of tile i overlaps
// the loads and MMAs of tile i + 1.
template <int BN, int NPLANE, int AMODE, int EPI, int KB, int NKBR = 0>
__global__ void __launch_bounds__(Roles<AMODE, BN, EPI>::THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
               const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmY,
               const __grid_constant__ CUtensorMap tmR, int y_tma,
               int b_plane_rows, GatherGeom g, EpiParams e, int num_kb, int m_tiles, int n_tiles) {
  // In TMA / im2col modes the gather warps 4-7 are free and join the epilogue:
  // warps w and w + 4 drain the same 32 TMEM lanes, each half of the columns.
  using R = Roles<AMODE, BN, EPI>;
  constexpr int EG = R::EGROUPS;
  constexpr int SPLIT = R::SPLIT;
  constexpr int CW = R::CW;
  constexpr int HB = BN / SPLIT;
  using Cfg = KernelCfg<BN, NPLANE, AMODE, EPI, KB, NKBR>;
  static_assert(NKBR == 0 || (NPLANE == 1 && KB != 16 && AMODE != A_GATHER), "resident B: int8, TMA-fed A");
  static_assert(KB == BKB || AMODE != A_GATHER, "the gather producers fill 128-byte slabs");
  static_assert(AMODE != A_SHIFT || (NKBR > 0 && NPLANE == 1 && (KB == 64 || KB == 128)),
                "shifted-patch mode: int8, resident B, 64/128-byte slabs");
  constexpr int STAGES = Cfg::STAGES;
  constexpr int PL = Cfg::PL;             // planes per operand (split-bf16: hi and lo)
  constexpr bool HALF = NPLANE >= 2;      // 16-bit elements (kind::f16)
  constexpr int A_BYTES = Cfg::A_BYTES;
  constexpr int B_BYTES = Cfg::B_BYTES;

  NNRCU_SPAN_BEGIN();
  extern __shared__ uint8_t smem_raw[];
  {
    // the launch must provide this instance's whole layout (checked before any shared access)
    uint32_t dsmem;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dsmem));
    if (dsmem < (uint32_t)Cfg::SMEM_BYTES) {
      if (threadIdx.x == 0) record_status(e.status, ST_SMEM);
      return;
    }
  }
  // 1024-byte aligned base, derived by pointer arithmetic on the shared array
  // so that accesses through it stay shared-memory (not generic) accesses
  uint8_t* smem = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;                                        // [STAGES][PL][A_BYTES]
  uint8_t* sB = sA + STAGES * PL * A_BYTES;                  // [STAGES][PL][B_BYTES], or [NKBR][B_BYTES]
  uint8_t* sOut = sB + (NKBR ? Cfg::BRES_BYTES : STAGES * PL * B_BYTES);  // u8 epilogue staging
  uint8_t* sRes = sOut + Cfg::OUT_BYTES;                      // [2][8 warps][32 rows][HB] (EPI_R2A)
  // sOut: [OUT_BUFS][8 warps][32 rows][HB]
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sRes + Cfg::RES_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;                  // [2] accumulator ready
  uint64_t* tempty_bar = tfull_bar + 2;                      // [2] accumulator drained
  uint64_t* res_bar = tempty_bar + 2;                        // [2][16] residual block landed (buffer, warp)
  uint64_t* bres_bar = res_bar + 32;                         // resident B landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = m_tiles * n_tiles;
  if (threadIdx.x == 0) NNRCU_TRACE_AT(23, 15, 3);  // CTA start
  // per-column constants, one private copy per epilogue warp (no cross-warp sync)
  int32_t* s_ci = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(full_bar) + Cfg::BAR_BYTES +
                                             (warp % (4 * SPLIT * EG)) * (3 * HB * 4));
  float* s_f1 = reinterpret_cast<float*>(s_ci + HB);
  float* s_f2 = s_f1 + HB;

  if (threadIdx.x == 0) {
    const uint32_t full_count = (AMODE == A_GATHER) ? (4u + 1u) : 1u;  // 4 gather warps + TMA
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full_bar[s], full_count);
      ptx::mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 32; ++a) ptx::mbar_init(&res_bar[a], 1);
    ptx::mbar_init(bres_bar, 1);
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull_bar[a], 1);
      ptx::mbar_init(&tempty_bar[a], 4 * SPLIT);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == R::TMA_WARP && lane == 0) {
    ptx::tma_prefetch_desc(&tmB);
    if (AMODE != A_GATHER) {
      ptx::tma_prefetch_desc(&tmA0);
      if (NPLANE == 2) ptx::tma_prefetch_desc(&tmA1);
    }
    if (y_tma) ptx::tma_prefetch_desc(&tmY);
    if (EPI == EPI_R2A) ptx::tma_prefetch_desc(&tmR);
  }
  if (warp == R::MMA_WARP) ptx::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The prologue above touches no tensor data. With programmatic dependent
  // launch it overlaps the previous kernel's tail; every read of activations
  // and every write of outputs comes after this wait.
  ptx::pdl_launch_dependents();
  if (NKBR > 0 && warp == R::TMA_WARP && lane == 0) {
    // this CTA's N tile's B, all K slabs, once per CTA (the grid is a
    // multiple of n_tiles, so a CTA's tiles all have N tile blockIdx.x %
    // n_tiles). B is a constant operand (the weights), written by no
    // kernel, so its copy starts before the wait for the previous kernel.
    const int bn0 = (int)(blockIdx.x % n_tiles) * BN;
    ptx::mbar_arrive_expect_tx(bres_bar, (uint32_t)(num_kb * Cfg::B_BYTES));
    for (int kb = 0; kb < num_kb; ++kb) {
      if (g.wb)  // the slab's shared-memory image: one plain bulk copy
        ptx::bulk_load(sB + (size_t)kb * Cfg::B_BYTES, g.wb + ((size_t)(bn0 / BN) * num_kb + kb) * Cfg::B_BYTES,
                       Cfg::B_BYTES, bres_bar);
      else
        ptx::tma_load_2d(sB + (size_t)kb * Cfg::B_BYTES, &tmB, bres_bar, kb * KB, bn0);
    }
  }
  ptx::pdl_wait();

  // Output rows of an M tile: mb = first GEMM row, nvr = valid rows; A_ROWS
  // tiles also give the output row (image * OH + oh) and first column ow0.
  auto tile_rows = [&](const int mt, int& mb, int& nvr, int& orow, int& ow0) {
if constexpr (AMODE == A_ROWS || AMODE == A_XROWS) {
      const int owt = (g.OW + BM - 1) / BM;
      orow = mt / owt;
      ow0 = (mt - orow * owt) * BM;
      mb = orow * g.OW + ow0;
      nvr = min(BM, g.OW - ow0);
    } else {
      orow = 0;
      ow0 = 0;
      mb = mt * BM;
      nvr = min(BM, e.M - mb);
    }
  };

  auto fail = [&](int code) {
    record_status(e.status, code);
    *abort_flag = 1;
  };

  if (warp >= R::TMA_WARP && warp < R::TMA_WARP + R::NPROD) {
    // ------------------------------------------------------------ TMA producers
    const int pw = warp - R::TMA_WARP;  // this producer issues stages it with it % NPROD == pw
    if (lane == 0) {
      constexpr uint32_t tx =
          AMODE == A_ROWS ? 0u : (AMODE != A_GATHER ? PL * A_BYTES : 0) + (NKBR ? 0 : PL * B_BYTES);
      if constexpr (AMODE == A_SHIFT) {
        // one patch per tile: each K slab's rows [m0, m0 + prows) of the padded input
        const int nslab = g.cbytes / KB;
        const uint32_t ptx_bytes = (uint32_t)(nslab * g.prows * KB);
        int tlt = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tlt) {
          const int s = tlt & 1;
          const uint32_t ph = (uint32_t)(tlt >> 1) & 1u;
          if (!ptx::mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag)) { fail(ST_TIMEOUT_EMPTY); ptx::settle_ns(200000); break; }
          NNRCU_TRACE_AT(warp, tlt, 0);
          ptx::mbar_arrive_expect_tx(&full_bar[s], ptx_bytes);
          const int m0 = (tile / n_tiles) * BM;
          for (int sl = 0; sl < nslab; ++sl)
            ptx::tma_load_2d(sA + (size_t)s * A_BYTES + (size_t)sl * g.prows * KB, &tmA0, &full_bar[s], sl * KB, m0);
        }
      } else {
      const uint32_t tx_rows = (uint32_t)(8 / max(g.tpr, 1)) * ROWS_BYTES + B_BYTES;  // A_ROWS stage bytes
      bool aborted = false;
      int it = 0, tlt = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !aborted; tile += gridDim.x, ++tlt) {
        NNRCU_TRACE_AT(warp, tlt, 0);
        const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
        // im2col: input position of the tile's first output pixel
        int i_n = 0, i_h = 0, i_w = 0;
        if (AMODE == A_IM2COL) {
          const int ohw = g.OH * g.OW;
          i_n = m0 / ohw;
          const int p = m0 - i_n * ohw;
          const int oh = p / g.OW;
          i_h = oh * g.sh - g.ph;
          i_w = (p - oh * g.OW) * g.sw - g.pw;
        }
        int r_mb = 0, r_nvr = 0, r_orow = 0, r_ow0 = 0;
        if (AMODE == A_ROWS || AMODE == A_XROWS) tile_rows(tile / n_tiles, r_mb, r_nvr, r_orow, r_ow0);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          if (R::NPROD > 1 && it % R::NPROD != pw) continue;
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!ptx::mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag)) { fail(ST_TIMEOUT_EMPTY); aborted = true; break; }
          ptx::mbar_arrive_expect_tx(&full_bar[s], AMODE == A_ROWS ? tx_rows : tx);
          uint8_t* a_st = sA + (size_t)s * PL * A_BYTES;
          uint8_t* b_st = sB + (size_t)s * PL * B_BYTES;
          const int kx = kb * KB / (HALF ? 2 : 1);  // element coordinate along K
          if constexpr (KB == 16) {
            // B: [tap][row][16 B] -> eight taps x BN rows x 16 B; A: one
            // hardware im2col copy (128 pixels x 16 B) per tap. Taps past the
            // kernel (zero weights) re-read the last tap to keep the byte count.
            // B: the stage's exact smem image ([8 taps][BN rows][16 B]), one contiguous copy
            ptx::bulk_load(b_st, g.wb + ((size_t)(n0 / BN) * num_kb + kb) * B_BYTES, B_BYTES, &full_bar[s]);
            if constexpr (AMODE == A_ROWS) {
              // kernel rows kb * rps .. + rps - 1 (rows past KH re-read the last one: zero weights)
              const int rps = 8 / g.tpr;
              const int img = r_orow / g.OH, oh = r_orow - img * g.OH;
#pragma unroll 1
              for (int j = 0; j < rps; ++j) {
                const int kr = min(kb * rps + j, g.KH - 1);
                const uint8_t* src = g.x + (((size_t)img * g.H + oh + kr) * g.W + r_ow0) * 16;
                ptx::bulk_load(a_st + j * ROWS_BYTES, src, ROWS_BYTES, &full_bar[s]);
              }
            } else {
            const int taps = g.KH * g.KW;
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
              const int tap = min(kb * 8 + j, taps - 1);
              const int kh = tap / g.KW, kw = tap - kh * g.KW;
              ptx::tma_load_im2col_4d(a_st + j * (BM * 16), &tmA0, &full_bar[s], 0, i_w, i_h, i_n,
                                      (uint16_t)(kw * g.dw), (uint16_t)(kh * g.dh));
            }
            }
          } else {
          if (NKBR == 0) {
            if (NPLANE == 1 && g.wb) {
              // B's shared-memory image for (N tile, K slab): one contiguous
              // bulk copy instead of BN tensor-map rows
              ptx::bulk_load(b_st, g.wb + ((size_t)(n0 / BN) * num_kb + kb) * B_BYTES, B_BYTES, &full_bar[s]);
            } else {
              for (int p = 0; p < PL; ++p)
                ptx::tma_load_2d(b_st + p * B_BYTES, &tmB, &full_bar[s], kx, p * b_plane_rows + n0);
            }
          }
          if (AMODE == A_TMA) {
            ptx::tma_load_2d(a_st, &tmA0, &full_bar[s], kx, m0);
            if (NPLANE == 2) ptx::tma_load_2d(a_st + A_BYTES, &tmA1, &full_bar[s], kx, m0);
          } else if (AMODE == A_XROWS) {
            // kernel row kb of the tile's output row: 128 consecutive 64-byte rows
            const int img = r_orow / g.OH, oh = r_orow - img * g.OH;
            ptx::tma_load_2d(a_st, &tmA0, &full_bar[s], 0, ((img * g.H + oh + kb) * g.W + r_ow0));
          } else if (AMODE == A_IM2COL) {
            // one K slab = 128 bytes of channels of a single filter tap
            const int kbyte = kb * KB;
            const int tap = kbyte / g.cbytes;
            const int cc = (kbyte - tap * g.cbytes) / (HALF ? 2 : 1);
            const int kh = tap / g.KW, kw = tap - kh * g.KW;
            const uint16_t ow_off = (uint16_t)(kw * g.dw), oh_off = (uint16_t)(kh * g.dh);
            ptx::tma_load_im2col_4d(a_st, &tmA0, &full_bar[s], cc, i_w, i_h, i_n, ow_off, oh_off);
            if (NPLANE == 2) ptx::tma_load_im2col_4d(a_st + A_BYTES, &tmA1, &full_bar[s], cc, i_w, i_h, i_n, ow_off, oh_off);
          }
          }
        }
        NNRCU_TRACE_AT(warp, tlt, 1);
      }
      if (aborted) ptx::settle_ns(200000);  // let copies already in flight land before the CTA exits
      }
    }
  } else if (warp == R::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // s32 += u8 x s8; f32 += bf16 x bf16 (NPLANE 2, 3); f32 += f16 x f16 (NPLANE 4)
      constexpr uint32_t idesc = (NPLANE == 1)   ? ptx::umma_idesc(2, 0, 1, BM, BN)
                                 : (NPLANE == 4) ? ptx::umma_idesc(1, 0, 0, BM, BN)
                                                 : ptx::umma_idesc(1, 1, 1, BM, BN);
      bool aborted = false;
      int it = 0, lt = 0;
      // A_SHIFT: per K step, the A view's start offset within a patch buffer (16-byte units)
      uint32_t shift_off[AMODE == A_SHIFT ? NKBR : 1];
      uint64_t bdesc0 = 0;
      if constexpr (AMODE == A_SHIFT) {
        const int nslab = g.cbytes / KB;
#pragma unroll
        for (int kb = 0; kb < NKBR; ++kb) {
          const int tap = kb / nslab, sl = kb - tap * nslab;
          const int kh = tap / g.KW, kw = tap - kh * g.KW;
          shift_off[kb] = (uint32_t)(((sl * g.prows + kh * g.dh * g.W + kw * g.dw) * KB) >> 4);
        }
        bdesc0 = ptx::umma_desc_sw<KB>(ptx::smem_u32(sB));
      }
      if (NKBR > 0 && !ptx::mbar_wait(bres_bar, 0u, abort_flag)) {
        fail(ST_TIMEOUT_FULL);
        aborted = true;
      }
      for (int tile = blockIdx.x; tile < num_tiles && !aborted; tile += gridDim.x, ++lt) {
        const int acc = lt & 1;
        const uint32_t use_ph = (uint32_t)(lt >> 1) & 1u;
        if (!ptx::mbar_wait(&tempty_bar[acc], use_ph ^ 1u, abort_flag)) { fail(ST_TIMEOUT_ACCUM); aborted = true; break; }
        NNRCU_TRACE_AT(warp, lt, 0);
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        if constexpr (AMODE == A_SHIFT) {
          // K step kb = (tap, slab): the slab's patch viewed from row kh * W + kw.
          // Descriptors are the buffer's base descriptor plus precomputed
          // start-address offsets (16-byte units; addresses stay below 2^18,
          // so the 14-bit field never carries): a few instructions per MMA.
          const int s = lt & 1;
          if (!ptx::mbar_wait(&full_bar[s], (uint32_t)(lt >> 1) & 1u, abort_flag)) { fail(ST_TIMEOUT_FULL); aborted = true; break; }
          NNRCU_TRACE_AT(warp, lt, 1);
          ptx::tc_fence_after();
          const uint64_t adesc = ptx::umma_desc_sw<KB>(ptx::smem_u32(sA + (size_t)s * A_BYTES));
#pragma unroll
          for (int kb = 0; kb < NKBR; ++kb) {
            if (kb < num_kb) {
#pragma unroll
              for (int k = 0; k < KB / 32; ++k)
                ptx::mma_i8(d_tmem, adesc + (uint64_t)(shift_off[kb] + k * 2),
                            bdesc0 + (uint64_t)((kb * B_BYTES + k * 32) >> 4), idesc, (kb | k) != 0);
            }
          }
          ptx::mma_commit(&empty_bar[s]);
          ptx::mma_commit(&tfull_bar[acc]);
          NNRCU_TRACE_AT(warp, lt, 2);
          continue;
        }
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!ptx::mbar_wait(&full_bar[s], ph, abort_flag)) { fail(ST_TIMEOUT_FULL); aborted = true; break; }
          if (kb == 0) NNRCU_TRACE_AT(warp, lt, 1);
          if (kb < 8) NNRCU_TRACE2_AT(warp, lt, 2 * kb);
          ptx::tc_fence_after();
          // (stages filled by TMA are async-proxy writes already; the gather
          // producers fence their cp.async writes before arriving)
          const uint32_t a_addr = ptx::smem_u32(sA + (size_t)s * PL * A_BYTES);
          const uint32_t b_addr = ptx::smem_u32(NKBR ? sB + (size_t)kb * B_BYTES : sB + (size_t)s * PL * B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::SLAB / 32; ++k) {
            const uint32_t koff = k * 32;
            if constexpr (AMODE == A_ROWS) {
              // taps 2k, 2k + 1 lie in one kernel row's copy: the same pixel
              // rows shifted by 16 bytes per tap (K-adjacent columns 16 B apart)
              const int tap0 = 2 * k, j = tap0 / g.tpr, kw0 = tap0 - j * g.tpr;
              ptx::mma_i8(d_tmem, ptx::umma_desc_interleaved(a_addr + j * ROWS_BYTES + kw0 * 16, 16, 128),
                          ptx::umma_desc_interleaved(b_addr + k * 2 * (BN * 16), BN * 16, 128), idesc, (kb | k) != 0);
            } else if constexpr (KB == 16) {
              // two 16-byte tap columns per K step
              ptx::mma_i8(d_tmem, ptx::umma_desc_interleaved(a_addr + k * 2 * (BM * 16), BM * 16, 128),
                          ptx::umma_desc_interleaved(b_addr + k * 2 * (BN * 16), BN * 16, 128), idesc, (kb | k) != 0);
            } else if constexpr (NPLANE == 1) {
              // stage descriptors plus the K offset (16-byte units)
              ptx::mma_i8(d_tmem, ptx::umma_desc_sw<KB>(a_addr) + (uint64_t)(koff >> 4),
                          ptx::umma_desc_sw<KB>(b_addr) + (uint64_t)(koff >> 4), idesc, (kb | k) != 0);
            } else if constexpr (NPLANE >= 3) {
              // one 16-bit plane: one exact product per multiply-add
              ptx::mma_f16(d_tmem, ptx::umma_desc_sw<KB>(a_addr + koff), ptx::umma_desc_sw<KB>(b_addr + koff), idesc,
                           (kb | k) != 0);
            } else {
              // hi*hi, hi*lo, lo*hi
              ptx::mma_f16(d_tmem, ptx::umma_desc_sw<KB>(a_addr + koff), ptx::umma_desc_sw<KB>(b_addr + koff), idesc,
                           (kb | k) != 0);
              ptx::mma_f16(d_tmem, ptx::umma_desc_sw<KB>(a_addr + koff),
                           ptx::umma_desc_sw<KB>(b_addr + B_BYTES + koff), idesc, 1u);
              ptx::mma_f16(d_tmem, ptx::umma_desc_sw<KB>(a_addr + A_BYTES + koff),
                           ptx::umma_desc_sw<KB>(b_addr + koff), idesc, 1u);
            }
          }
          if (kb < 8) NNRCU_TRACE2_AT(warp, lt, 2 * kb + 1);
          ptx::mma_commit(&empty_bar[s]);
        }
        if (!aborted) ptx::mma_commit(&tfull_bar[acc]);  // fires when this tile's MMAs have completed
        NNRCU_TRACE_AT(warp, lt, 2);
      }
      if (aborted) ptx::settle_ns(200000);  // MMAs already issued finish before TMEM is freed
    }
  } else if (warp >= 4 && AMODE == A_GATHER) {
    // ------------------------------------------------------------ gather producers (warps 4-7)
    if constexpr (AMODE == A_GATHER) {
      // Thread t owns tile row t (one output pixel) and copies its whole
      // 128-byte K slab per stage: one address per filter tap touched, then
      // consecutive 16-byte cp.async chunks into the swizzled row.
      const int r = threadIdx.x - 128;
      uint8_t* const row_dst0 = sA + (r >> 3) * 1024 + (r & 7) * 128;
      const int rsw = r & 7;
      const int ohw = g.OH * g.OW;
      constexpr int LAG = Cfg::LAG;
      bool aborted = false;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !aborted; tile += gridDim.x) {
        const int m = (tile / n_tiles) * BM + r;
        const bool rvalid = m < e.M;
        int r_n = 0, r_ih = 0, r_iw = 0;
        if (rvalid) {
          const int img = m / ohw;
          const int p = m - img * ohw;
          const int oh = p / g.OW;
          const int ow = p - oh * g.OW;
          r_n = img;
          r_ih = oh * g.sh - g.ph;
          r_iw = ow * g.sw - g.pw;
        }
        const size_t img_base = (size_t)r_n * g.H;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag));
          if (!ok) { fail(ST_TIMEOUT_EMPTY); aborted = true; break; }
          uint8_t* const row_dst = row_dst0 + (size_t)s * PL * A_BYTES;
          int kbyte = kb * BKB;
          int tap = kbyte / g.cbytes;
          int cc = kbyte - tap * g.cbytes;
          int j = 0;
          while (j < 8) {
            // chunks [j, j + run) lie in one filter tap
            const int run = min(8 - j, (g.cbytes - cc) >> 4);
            const bool kvalid = kbyte < g.kbytes;
            const uint8_t* src = nullptr;
            bool inb = false;
            if (kvalid && rvalid) {
              const int kh = tap / g.KW;
              const int kw = tap - kh * g.KW;
              const int ih = r_ih + kh * g.dh;
              const int iw = r_iw + kw * g.dw;
              inb = (unsigned)ih < (unsigned)g.H && (unsigned)iw < (unsigned)g.W;
              if (inb) src = g.x + ((img_base + ih) * g.W + iw) * (size_t)g.cbytes + cc;
            }
            for (int u = 0; u < run; ++u) {
              uint8_t* dst = row_dst + (((j + u) ^ rsw) << 4);
              if (inb) {
                ptx::cp_async16(dst, src + u * 16, 16);
                if (NPLANE == 2) ptx::cp_async16(dst + A_BYTES, g.x2 + (src - g.x) + u * 16, 16);
              } else {
                // padding pixel (x_zp pattern), K tail or row beyond M (zeros)
                const uint32_t wv = (kvalid && rvalid) ? g.pad_word : 0u;
                ptx::st_shared_v4(dst, wv, wv, wv, wv);
                if (NPLANE == 2) ptx::st_shared_v4(dst + A_BYTES, 0u, 0u, 0u, 0u);
              }
            }
            j += run;
            kbyte += run * 16;
            cc += run * 16;
            if (cc >= g.cbytes) { cc = 0; ++tap; }
          }
          ptx::cp_async_commit();
          // Publish the stage issued LAG iterations ago: its copies are done
          // once at most LAG groups remain in flight. Refilling stage it needs
          // stage it - STAGES consumed, which was published at iteration
          // it - STAGES + LAG <= it - 1, leaving STAGES - 1 - LAG iterations of
          // slack for the MMA (LAG = STAGES - 1 would lock the two in step).
          // Each lane waits for its own copies and fences them for the async
          // proxy; one arrival per warp (after __syncwarp) then publishes the
          // warp's 32 rows, instead of 32 serialised arrivals.
          if (it >= LAG) {
            ptx::cp_async_wait<LAG>();
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&full_bar[(it - LAG) % STAGES]);
          }
        }
      }
      // Drain: publish the last LAG stages.
      ptx::cp_async_wait<0>();
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (!aborted && lane == 0) {
        const int first = it > LAG ? it - LAG : 0;
        for (int q = first; q < it; ++q) ptx::mbar_arrive(&full_bar[q % STAGES]);
      }
    }
  } else if (warp < 4 * SPLIT * EG) {
    // ------------------------------------------------------------ epilogue (warps 0-3, and 4-7 when SPLIT = 2)
    static_assert(EG == 1 || Cfg::OUT_BLOCK == 0 || Cfg::OUT_BUFS == 2, "epilogue groups need a staging buffer each");
    const int group = warp / (4 * SPLIT);  // EG = 2: tiles lt with lt % 2 == group
    const int wig = warp % (4 * SPLIT);    // warp within its group
    const int eq = wig & 3;            // TMEM lane quarter
    const int col0 = (wig >> 2) * HB;  // this warp's columns [col0, col0 + HB) of the tile
    const int row = eq * 32 + lane;    // TMEM lane == tile row
    int lt = group;
    int cached_n0 = -1;
    // epilogue scalars held in registers for the whole kernel
    const float kp_lo = e.rq_lo, kp_hi = e.rq_hi, kp_sa = e.qa_sa, kp_sb = e.qa_sb, kp_fx = e.qa_fixed;
    const float kp_ca = __fsub_rn(e.yzp_f, RND_MAGIC);
    const uint32_t kp_yzp = (uint32_t)e.yzp;
    const bool kp_ovf = e.qa_ovf != 0;
    const bool kp_sat = e.r2_sat != 0;
    const bool shift_direct = e.y_layout == 0 && (e.ldy & 15) == 0 && (reinterpret_cast<uintptr_t>(e.y) & 15) == 0;
    const bool direct = AMODE == A_SHIFT || e.opad != 0;  // lean path stores rows straight to HBM
    // EPI_R2A: TMA load of this warp's 32 x HB residual block of tile t into buffer buf
    auto issue_res = [&](const int t, const int buf) {
      constexpr int SEG = Cfg::OUT_SEG;
      const int rm0 = (t / n_tiles) * BM, rn0 = (t % n_tiles) * BN;
      uint64_t* bar = &res_bar[buf * 16 + warp];
      uint8_t* dst = sRes + buf * Cfg::OUT_BLOCK + warp * (32 * HB);
      ptx::mbar_arrive_expect_tx(bar, 32 * HB);
      for (int h = 0; h < HB / SEG; ++h) ptx::tma_load_2d(dst + h * (32 * SEG), &tmR, bar, rn0 + col0 + h * SEG, rm0 + eq * 32);
    };
    if (EPI == EPI_R2A && Cfg::RES_TMA && lane == 0 && (int)blockIdx.x < num_tiles) issue_res(blockIdx.x, 0);
    bool res_failed = false;
    for (int tile = blockIdx.x + group * gridDim.x; tile < num_tiles; tile += EG * gridDim.x, lt += EG) {
      int m0 = 0, nvr = 0, orow = 0, ow0 = 0;
      tile_rows(tile / n_tiles, m0, nvr, orow, ow0);
      const int n0 = (tile % n_tiles) * BN;
      const int acc = lt & 1;
      const uint32_t use_ph = (uint32_t)(lt >> 1) & 1u;
      if (n0 != cached_n0) {
        // per-column constants of this column block (this warp's copy)
        __syncwarp();
        for (int i = lane; i < HB; i += 32) {
          const int n = n0 + col0 + i;
          const bool ok = n < e.N;
          int32_t ci = (ok && e.colcorr) ? e.colcorr[n] : 0;
          float f1 = 0.0f, f2 = 0.0f;
          if (EPI == EPI_R2 || EPI == EPI_R2A) {
            if (ok && e.bias_i) ci = (int32_t)((uint32_t)ci + (uint32_t)e.bias_i[n]);
            f1 = (ok && e.os) ? e.os[n] : 0.0f;
          } else if (EPI == EPI_F32) {
            f2 = (ok && e.bias) ? e.bias[n] : 0.0f;
          } else {
            f1 = (ok && e.cs) ? e.cs[n] : 0.0f;
            f2 = (ok && e.bias_f) ? e.bias_f[n] : 0.0f;
          }
          s_ci[i] = ci;
          s_f1[i] = f1;
          s_f2[i] = f2;
        }
        __syncwarp();
        cached_n0 = n0;
      }
      // the staging block may be rewritten once the previous tile's stores have read it
      if (lane == 0) NNRCU_TRACE_AT(warp, lt, 0);
      // (EG = 2: each group has its own staging buffer)
      uint8_t* const stg = sOut + (Cfg::OUT_BUFS == 2 ? (EG == 2 ? group : (lt & 1)) * Cfg::OUT_BLOCK : 0) +
                           wig * (32 * Cfg::ROW_BYTES);
      constexpr int SEG = Cfg::OUT_SEG;
      // swizzle of a staged row (the store / residual maps' 128B, 64B or 32B
      // swizzle): row r, 16-byte chunk c of a segment lives at r*SEG + ((c ^ f(r)) << 4)
      const int swz = SEG == 128 ? (lane & 7) : (SEG == 64 ? ((lane >> 1) & 3) : ((lane >> 2) & 1));
      if (Cfg::OUT_BLOCK > 0 && y_tma) {
        if (lane == 0) {
          // the store that last used this buffer has read it
          ptx::bulk_wait_read<EG == 2 ? 0 : Cfg::OUT_BUFS - 1>();
          NNRCU_TRACE2_AT(warp, lt, 12);
          if constexpr (EPI == EPI_R2A && Cfg::RES_TMA) {
            // prefetch the residual block of this warp's next tile into the
            // other buffer (its previous contents were consumed by tile lt - 1)
            const int nxt = tile + gridDim.x;
            if (nxt < num_tiles) issue_res(nxt, (lt + 1) & 1);
          }
        }
        __syncwarp();
      }
      if (lane == 0) NNRCU_TRACE2_AT(warp, lt, 13);
      if (!__all_sync(0xffffffffu, ptx::mbar_wait(&tfull_bar[acc], use_ph, abort_flag))) {
        fail(ST_TIMEOUT_ACCUM);
        res_failed = true;
        break;
      }
      ptx::tc_fence_after();
      if (lane == 0) NNRCU_TRACE_AT(warp, lt, 1);
      const uint8_t* rstg = sRes + (lt & 1) * Cfg::OUT_BLOCK + warp * (32 * HB);
      if (EPI == EPI_R2A && Cfg::RES_TMA &&
          !__all_sync(0xffffffffu, ptx::mbar_wait(&res_bar[(lt & 1) * 16 + warp], (uint32_t)(lt >> 1) & 1u, abort_flag))) {
        fail(ST_TIMEOUT_ACCUM);
        res_failed = true;
        break;
      }
      if (lane == 0) NNRCU_TRACE_AT(warp, lt, 2);
      int m = m0 + row;  // output row (A_SHIFT: GEMM rows are padded-grid positions, mapped below)
      bool mvalid = row < nvr;
      if constexpr (AMODE == A_SHIFT) {
        const int pr = m / g.W, px = m - pr * g.W;
        const int im = pr / g.H, py = pr - im * g.H;
        mvalid = mvalid && px < g.OW && py < g.OH;
        m = (im * g.OH + py) * g.OW + px;
      }
      int32_t rowc = 0;
      if (EPI == EPI_R4 && e.rowcorr && mvalid) rowc = e.rowcorr[m];
      int img = 0, pix = 0;
      if (e.y_layout == 1 && mvalid) { img = m / e.ohw; pix = m - img * e.ohw; }
      // R3 with an NCHW output: the last OW % 16 pixels of each output row take
      // the first-layer kernel's scalar tail sequence
      const bool r3_tail = EPI == EPI_R3N && e.y_layout == 1 && mvalid && (pix % g.OW) >= (g.OW & ~15);
      const float r3_add_f = r3_tail ? 0.0f : e.yzp_f;  // y_zp added before the rounding (body) ...
      const int32_t r3_add_i = r3_tail ? e.yzp : 0;     // ... or after it (tail)
      int mst = m;  // row of the output buffer
      if (e.opad) {
        const int im = m / e.o_hw, r = m - im * e.o_hw, oy = r / e.o_w;
        mst = im * e.o_hwp + oy * e.o_wp + (r - oy * e.o_w) + e.o_off;
      }
      const uint32_t t_addr = tmem_base + ((uint32_t)(eq * 32) << 16) + (uint32_t)(acc * BN);
      // one CW-column chunk: requant / bias / post-op / stores
      auto chunk = [&](const int c0, uint32_t (&v)[CW]) {
        const int pc = c0 - col0;  // column within this warp's parameter copy
        if (!mvalid || n0 + c0 >= e.N) return;
        const int nvalid = min(CW, e.N - (n0 + c0));
        if constexpr (EPI == EPI_F32) {
          // bias, residual and post-op for the whole chunk in registers, then
          // the stores (rows are lanes: row-major stores are per-lane float4s,
          // NCHW stores are coalesced across lanes for each column)
          float* y = static_cast<float*>(e.y);
          const bool rowmajor = e.y_layout == 0;
          const bool vec = rowmajor && nvalid == CW && (e.ldy & 3) == 0 && ((reinterpret_cast<uintptr_t>(e.y) & 15) == 0) &&
                           (!e.residual || (reinterpret_cast<uintptr_t>(e.residual) & 15) == 0);
          const size_t base = rowmajor ? (size_t)m * e.ldy + n0 + c0 : ((size_t)img * e.N + n0 + c0) * e.ohw + pix;
          const size_t step = rowmajor ? 1 : (size_t)e.ohw;
          float o[CW];
#pragma unroll
          for (int j = 0; j < CW; j += 4) {
            const float4 b4 = *reinterpret_cast<const float4*>(s_f2 + pc + j);
            o[j + 0] = __uint_as_float(v[j + 0]) + b4.x;
            o[j + 1] = __uint_as_float(v[j + 1]) + b4.y;
            o[j + 2] = __uint_as_float(v[j + 2]) + b4.z;
            o[j + 3] = __uint_as_float(v[j + 3]) + b4.w;
          }
          float r[CW];
          const bool has_res = e.residual != nullptr && e.res_mode != 0;
          if (has_res) {
            if (vec) {
#pragma unroll
              for (int j = 0; j < CW; j += 4) {
                const float4 r4 = *reinterpret_cast<const float4*>(e.residual + base + j);
                r[j] = r4.x; r[j + 1] = r4.y; r[j + 2] = r4.z; r[j + 3] = r4.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < CW; ++j) r[j] = j < nvalid ? e.residual[base + j * step] : 0.0f;
            }
            if (e.res_mode == 1) {
#pragma unroll
              for (int j = 0; j < CW; ++j) o[j] = fmaf(e.res_scale, r[j], o[j]);
            }
          }
          switch (e.act) {
            case ACT_NONE: break;
            case ACT_RELU:
#pragma unroll
              for (int j = 0; j < CW; ++j) o[j] = fmaxf(o[j], 0.0f);
              break;
            case ACT_CLIP:
#pragma unroll
              for (int j = 0; j < CW; ++j) o[j] = fminf(fmaxf(o[j], e.act_a), e.act_b);
              break;
            default:
#pragma unroll
              for (int j = 0; j < CW; ++j) o[j] = apply_act(o[j], e.act, e.act_a, e.act_b);
              break;
          }
          if (has_res && e.res_mode == 2) {
#pragma unroll
            for (int j = 0; j < CW; ++j) o[j] += r[j];
          }
          if (Cfg::OUT_BLOCK > 0 && y_tma) {
            // swizzled staging, as the u8 epilogue (16-byte chunk c of row r at
            // r * SEG + ((c ^ f(r)) << 4)); the TMA store writes whole rows
            constexpr int SEG = Cfg::OUT_SEG;
            const int pb = pc * 4, h = pb / SEG, cc = (pb % SEG) >> 4;
            uint8_t* seg = stg + h * (32 * SEG) + lane * SEG;
#pragma unroll
            for (int k = 0; k < CW / 4; ++k)
              ptx::st_shared_v4(seg + (((cc + k) ^ swz) << 4), __float_as_uint(o[4 * k]), __float_as_uint(o[4 * k + 1]),
                                __float_as_uint(o[4 * k + 2]), __float_as_uint(o[4 * k + 3]));
          } else if (vec) {
#pragma unroll
            for (int j = 0; j < CW; j += 4)
              *reinterpret_cast<float4*>(y + base + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
              if (j < nvalid) y[base + j * step] = o[j];
          }
        } else {
          // q[j]: the requantised value in the low byte
          uint32_t q[CW];
          const bool fused = (EPI == EPI_R2A) || e.qres != nullptr;
          // residual words (4 bytes each) of this row's CW columns
          uint32_t rw[CW / 4];
          if (fused) {
            if constexpr (EPI == EPI_R2A && Cfg::RES_TMA) {
              const int h = pc / SEG, cc = (pc % SEG) >> 4;
              const uint8_t* seg = rstg + h * (32 * SEG) + lane * SEG;
#pragma unroll
              for (int k = 0; k < CW / 16; ++k) {
                const uint4 r0 = *reinterpret_cast<const uint4*>(seg + (((cc + k) ^ swz) << 4));
                rw[4 * k] = r0.x; rw[4 * k + 1] = r0.y; rw[4 * k + 2] = r0.z; rw[4 * k + 3] = r0.w;
              }
            } else {
              const uint8_t* rp = e.qres + (size_t)m * e.ldy + n0 + c0;
              if (nvalid == CW && ((reinterpret_cast<uintptr_t>(rp) & 15) == 0)) {
#pragma unroll
                for (int k = 0; k < CW / 16; ++k) {
                  const uint4 r0 = reinterpret_cast<const uint4*>(rp)[k];
                  rw[4 * k] = r0.x; rw[4 * k + 1] = r0.y; rw[4 * k + 2] = r0.z; rw[4 * k + 3] = r0.w;
                }
              } else {
#pragma unroll
                for (int j = 0; j < CW / 4; ++j) {
                  uint32_t x = 0;
#pragma unroll
                  for (int u = 0; u < 4; ++u)
                    if (4 * j + u < nvalid) x |= (uint32_t)rp[4 * j + u] << (8 * u);
                  rw[j] = x;
                }
              }
            }
          }
          const long long ebase = (long long)m * e.N + n0 + c0;
          bool scalar_add = fused;  // cleared when the vectorised body below covers the chunk
          if (EPI == EPI_R2 || EPI == EPI_R2A) {
            float t[CW];  // RND_MAGIC + rne(f)
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
              const int4 ci4 = *reinterpret_cast<const int4*>(s_ci + pc + j);
              const float4 a4 = *reinterpret_cast<const float4*>(s_f1 + pc + j);
              t[j + 0] = r2_magic((int32_t)v[j + 0], ci4.x, a4.x, e);
              t[j + 1] = r2_magic((int32_t)v[j + 1], ci4.y, a4.y, e);
              t[j + 2] = r2_magic((int32_t)v[j + 2], ci4.z, a4.z, e);
              t[j + 3] = r2_magic((int32_t)v[j + 3], ci4.w, a4.w, e);
            }
            if (fused && ebase + CW <= e.qa_vec_end) {
              // QLinearAdd(q, residual) body (QLinearAdd.cpp:46-104):
              // fma(a, sa, fma(b, sb, fixed)), rne, saturate; a = rne(f) + y_zp
              // is t - (RND_MAGIC - y_zp), exact (integers below 2^24)
              const float sa = e.qa_sa, sb = e.qa_sb, fx = e.qa_fixed;
              const float ca = __fsub_rn(e.yzp_f, RND_MAGIC);
#pragma unroll
              for (int j = 0; j < CW; ++j) {
                const float fa = __fadd_rn(t[j], ca);
                const float fb = byte_to_float(rw[j >> 2], j & 3);
                float r = __fmaf_rn(fa, sa, __fmaf_rn(fb, sb, fx));
                // x86 conversion: values >= 2^31 become INT_MIN, i.e. 0 after the max
                r = r >= 2147483648.0f ? 0.0f : fminf(fmaxf(r, 0.0f), 255.0f);
                q[j] = __float_as_uint(__fadd_rn(r, RND_MAGIC));
              }
              scalar_add = false;
            } else {
#pragma unroll
              for (int j = 0; j < CW; ++j) q[j] = __float_as_uint(t[j]) + (uint32_t)e.yzp;
            }
          } else if constexpr (EPI == EPI_R3N) {
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
              const int4 ci4 = *reinterpret_cast<const int4*>(s_ci + pc + j);
              const float4 a4 = *reinterpret_cast<const float4*>(s_f1 + pc + j);
              const float4 b4 = *reinterpret_cast<const float4*>(s_f2 + pc + j);
              q[j + 0] = requant_r3_row((int32_t)v[j + 0], ci4.x, a4.x, b4.x, r3_add_f, r3_add_i, r3_tail, e);
              q[j + 1] = requant_r3_row((int32_t)v[j + 1], ci4.y, a4.y, b4.y, r3_add_f, r3_add_i, r3_tail, e);
              q[j + 2] = requant_r3_row((int32_t)v[j + 2], ci4.z, a4.z, b4.z, r3_add_f, r3_add_i, r3_tail, e);
              q[j + 3] = requant_r3_row((int32_t)v[j + 3], ci4.w, a4.w, b4.w, r3_add_f, r3_add_i, r3_tail, e);
            }
          } else {
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
              const int4 ci4 = *reinterpret_cast<const int4*>(s_ci + pc + j);
              const float4 a4 = *reinterpret_cast<const float4*>(s_f1 + pc + j);
              const float4 b4 = *reinterpret_cast<const float4*>(s_f2 + pc + j);
              q[j + 0] = requant_u8<EPI>((int32_t)v[j + 0], ci4.x, rowc, a4.x, b4.x, e);
              q[j + 1] = requant_u8<EPI>((int32_t)v[j + 1], ci4.y, rowc, a4.y, b4.y, e);
              q[j + 2] = requant_u8<EPI>((int32_t)v[j + 2], ci4.z, rowc, a4.z, b4.z, e);
              q[j + 3] = requant_u8<EPI>((int32_t)v[j + 3], ci4.w, rowc, a4.w, b4.w, e);
            }
          }
          if (scalar_add) {
              // element-wise QLinearAdd: the 16-wide body for elements below
              // qa_vec_end, nnr's scalar tail formula
              // fma(sa, a - a_zp, sb * (b - b_zp)) + y_zp for the rest
#pragma unroll
              for (int j = 0; j < CW; ++j) {
                const int qa = (int)(q[j] & 0xFFu), qb = (int)((rw[j >> 2] >> (8 * (j & 3))) & 0xFFu);
                int r;
                if (ebase + j < e.qa_vec_end) {
                  r = ptx::cvt_rne_x86(__fmaf_rn((float)qa, e.qa_sa, __fmaf_rn((float)qb, e.qa_sb, e.qa_fixed)));
                } else {
                  const float da = (float)(qa - e.qa_azp), db = (float)(qb - e.qa_bzp);
                  r = ptx::cvt_rne_x86(__fadd_rn(__fmaf_rn(e.qa_sa, da, __fmul_rn(e.qa_sb, db)), (float)e.qa_yzp));
                }
                q[j] = (uint32_t)(r < 0 ? 0 : (r > 255 ? 255 : r));
              }
          }
          uint8_t* y = static_cast<uint8_t*>(e.y);
          uint32_t w[CW / 4];
#pragma unroll
          for (int j = 0; j < CW / 4; ++j) w[j] = pack_low_bytes(q[4 * j], q[4 * j + 1], q[4 * j + 2], q[4 * j + 3]);
          if (y_tma) {
            const int h = pc / SEG, cc = (pc % SEG) >> 4;
            uint8_t* seg = stg + h * (32 * SEG) + lane * SEG;
#pragma unroll
            for (int k = 0; k < CW / 16; ++k)
              ptx::st_shared_v4(seg + (((cc + k) ^ swz) << 4), w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          } else if (e.y_layout == 0) {
            uint8_t* dst = y + (size_t)mst * e.ldy + n0 + c0;
            if (nvalid == CW && (e.ldy & 15) == 0 && (reinterpret_cast<uintptr_t>(e.y) & 15) == 0) {
#pragma unroll
              for (int k = 0; k < CW / 16; ++k)
                reinterpret_cast<uint4*>(dst)[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < CW; ++j)
                if (j < nvalid) dst[j] = (uint8_t)q[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
              if (j < nvalid) y[((size_t)img * e.N + n0 + c0 + j) * e.ohw + pix] = (uint8_t)q[j];
          }
        }
      };
      // Interior tiles of u8 epilogues with a TMA-stored output take a lean
      // path: no row / column / tail checks, one inlined copy in the loop.
      // (A_SHIFT: the lean path stores each row's bytes straight to HBM; rows
      // that are not output pixels are skipped)
      bool fast = false;
      if constexpr (EPI != EPI_F32) {
        if (direct)
          fast = shift_direct && n0 + BN <= e.N && e.qres == nullptr;
        else
          fast = y_tma && (AMODE == A_ROWS || AMODE == A_XROWS || m0 + BM <= e.M) && n0 + BN <= e.N &&
               (EPI == EPI_R2A ? (long long)(m0 + BM) * e.N <= e.qa_vec_end : e.qres == nullptr);
      }
      auto chunk_fast = [&](const int c0, uint32_t (&v)[CW]) {
        if constexpr (EPI != EPI_F32) {
          // Column pairs use the packed fp32 instructions (__fmul2_rn,
          // __fadd2_rn, __ffma2_rn): two IEEE round-to-nearest operations per
          // instruction, each lane bit-identical to the scalar operation.
          const float2 k_magic = make_float2(RND_MAGIC, RND_MAGIC);
          const int pc = c0 - col0;
          uint32_t q[CW];
          // R2A: this row's residual bytes, loaded first so that their
          // latency overlaps the requantisation below
          uint4 rq[CW / 16];
          if constexpr (EPI == EPI_R2A && !Cfg::RES_TMA) {
            const uint4* rp = reinterpret_cast<const uint4*>(e.qres + (size_t)m * e.ldy + n0 + c0);
#pragma unroll
            for (int k = 0; k < CW / 16; ++k) rq[k] = __ldg(rp + k);
          }
          if constexpr (EPI == EPI_R2 || EPI == EPI_R2A) {
            // R2 with y_zp = 0 and the full u8 range (every Relu output):
            // clamp(rne(f), 0, 255) is one saturating conversion
            bool sat_done = false;
            if constexpr (EPI == EPI_R2) {
              if (kp_sat) {
#pragma unroll
                for (int j = 0; j < CW; j += 4) {
                  const int4 ci4 = *reinterpret_cast<const int4*>(s_ci + pc + j);
                  const float4 a4 = *reinterpret_cast<const float4*>(s_f1 + pc + j);
                  const float2 f0 = __fmul2_rn(make_float2(__int2float_rn((int32_t)(v[j + 0] + (uint32_t)ci4.x)),
                                                           __int2float_rn((int32_t)(v[j + 1] + (uint32_t)ci4.y))),
                                               make_float2(a4.x, a4.y));
                  const float2 f1 = __fmul2_rn(make_float2(__int2float_rn((int32_t)(v[j + 2] + (uint32_t)ci4.z)),
                                                           __int2float_rn((int32_t)(v[j + 3] + (uint32_t)ci4.w))),
                                               make_float2(a4.z, a4.w));
                  q[j + 0] = ptx::cvt_rni_sat_u8(f0.x);
                  q[j + 1] = ptx::cvt_rni_sat_u8(f0.y);
                  q[j + 2] = ptx::cvt_rni_sat_u8(f1.x);
                  q[j + 3] = ptx::cvt_rni_sat_u8(f1.y);
                }
                sat_done = true;
              }
            }
            if (!sat_done) {
            float2 t[CW / 2];  // RND_MAGIC + rne(f), f = clamp(float(acc + bias) * os)
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
              const int4 ci4 = *reinterpret_cast<const int4*>(s_ci + pc + j);
              const float4 a4 = *reinterpret_cast<const float4*>(s_f1 + pc + j);
              float2 f0 = __fmul2_rn(make_float2(__int2float_rn((int32_t)(v[j + 0] + (uint32_t)ci4.x)),
                                                 __int2float_rn((int32_t)(v[j + 1] + (uint32_t)ci4.y))),
                                     make_float2(a4.x, a4.y));
              float2 f1 = __fmul2_rn(make_float2(__int2float_rn((int32_t)(v[j + 2] + (uint32_t)ci4.z)),
                                                 __int2float_rn((int32_t)(v[j + 3] + (uint32_t)ci4.w))),
                                     make_float2(a4.z, a4.w));
              f0.x = fminf(fmaxf(f0.x, kp_lo), kp_hi);
              f0.y = fminf(fmaxf(f0.y, kp_lo), kp_hi);
              f1.x = fminf(fmaxf(f1.x, kp_lo), kp_hi);
              f1.y = fminf(fmaxf(f1.y, kp_lo), kp_hi);
              t[j / 2] = __fadd2_rn(f0, k_magic);
              t[j / 2 + 1] = __fadd2_rn(f1, k_magic);
            }
            if constexpr (EPI == EPI_R2A) {
              // QLinearAdd body (QLinearAdd.cpp:46-104): fma(a, sa, fma(b, sb, fixed)),
              // rne, saturate; a = rne(f) + y_zp = t - (RND_MAGIC - y_zp) exactly,
              // b = (2^23 + byte) - 2^23 exactly
              uint32_t rw[CW / 4];
              if constexpr (Cfg::RES_TMA) {
                const int h = pc / SEG, cc = (pc % SEG) >> 4;
                const uint8_t* seg = rstg + h * (32 * SEG) + lane * SEG;
#pragma unroll
                for (int k = 0; k < CW / 16; ++k) rq[k] = *reinterpret_cast<const uint4*>(seg + (((cc + k) ^ swz) << 4));
              }
#pragma unroll
              for (int k = 0; k < CW / 16; ++k) {
                rw[4 * k] = rq[k].x; rw[4 * k + 1] = rq[k].y; rw[4 * k + 2] = rq[k].z; rw[4 * k + 3] = rq[k].w;
              }
              const float2 sa = make_float2(kp_sa, kp_sa), sb = make_float2(kp_sb, kp_sb);
              const float2 fx = make_float2(kp_fx, kp_fx), ca = make_float2(kp_ca, kp_ca);
              const float2 nbm = make_float2(-BYTE_MAGIC, -BYTE_MAGIC);
              auto add_pairs = [&](auto ovf) {
#pragma unroll
                for (int j = 0; j < CW; j += 2) {
                  const float2 fa = __fadd2_rn(t[j / 2], ca);
                  const uint32_t w = rw[j >> 2];
                  const float2 fb = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650 | (j & 3))),
                                                           __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650 | ((j + 1) & 3)))),
                                               nbm);
                  float2 r = __ffma2_rn(fa, sa, __ffma2_rn(fb, sb, fx));
                  if constexpr (!decltype(ovf)::value) {
                    q[j] = ptx::cvt_rni_sat_u8(r.x);
                    q[j + 1] = ptx::cvt_rni_sat_u8(r.y);
                    continue;
                  }
                  if constexpr (decltype(ovf)::value) {
                    // x86 conversion: values >= 2^31 become INT_MIN, i.e. 0 after the max
                    r.x = r.x >= 2147483648.0f ? 0.0f : r.x;
                    r.y = r.y >= 2147483648.0f ? 0.0f : r.y;
                  }
                  r.x = fminf(fmaxf(r.x, 0.0f), 255.0f);
                  r.y = fminf(fmaxf(r.y, 0.0f), 255.0f);
                  r = __fadd2_rn(r, k_magic);
                  q[j] = __float_as_uint(r.x);
                  q[j + 1] = __float_as_uint(r.y);
                }
              };
              // the 2^31 case is possible only when 255 (|sa| + |sb|) + |fixed| reaches it
              if (kp_ovf)
                add_pairs(std::true_type{});
              else
                add_pairs(std::false_type{});
            } else {
#pragma unroll
              for (int j = 0; j < CW; j += 2) {
                q[j] = __float_as_uint(t[j / 2].x) + kp_yzp;
                q[j + 1] = __float_as_uint(t[j / 2].y) + kp_yzp;
              }
            }
            }
          } else if constexpr (EPI == EPI_R3 || EPI == EPI_R3N) {
            // f = fma(float(acc), cs, bias_f); f = fma(f, inv_y, y_zp); clamp; rne
            const float2 iy = make_float2(e.inv_y, e.inv_y), yz = make_float2(e.yzp_f, e.yzp_f);
            const uint32_t qmin_u = (uint32_t)e.qmin_f;
            auto r3_quads = [&](auto has_qmin) {
#pragma unroll
              for (int j = 0; j < CW; j += 4) {
                const int4 ci4 = *reinterpret_cast<const int4*>(s_ci + pc + j);
                const float4 a4 = *reinterpret_cast<const float4*>(s_f1 + pc + j);
                const float4 b4 = *reinterpret_cast<const float4*>(s_f2 + pc + j);
                float2 f0 = __ffma2_rn(make_float2(__int2float_rn((int32_t)(v[j] + (uint32_t)ci4.x)),
                                                   __int2float_rn((int32_t)(v[j + 1] + (uint32_t)ci4.y))),
                                       make_float2(a4.x, a4.y), make_float2(b4.x, b4.y));
                float2 f1 = __ffma2_rn(make_float2(__int2float_rn((int32_t)(v[j + 2] + (uint32_t)ci4.z)),
                                                   __int2float_rn((int32_t)(v[j + 3] + (uint32_t)ci4.w))),
                                       make_float2(a4.z, a4.w), make_float2(b4.z, b4.w));
                f0 = __ffma2_rn(f0, iy, yz);
                f1 = __ffma2_rn(f1, iy, yz);
                // the upper bound is 255: rne + clamp to [0, 255] in one
                // conversion, then the lower bound (y_zp under a fused Relu;
                // nothing to do when it is 0)
                q[j] = ptx::cvt_rni_sat_u8(f0.x);
                q[j + 1] = ptx::cvt_rni_sat_u8(f0.y);
                q[j + 2] = ptx::cvt_rni_sat_u8(f1.x);
                q[j + 3] = ptx::cvt_rni_sat_u8(f1.y);
                if constexpr (decltype(has_qmin)::value) {
                  q[j] = max(q[j], qmin_u);
                  q[j + 1] = max(q[j + 1], qmin_u);
                  q[j + 2] = max(q[j + 2], qmin_u);
                  q[j + 3] = max(q[j + 3], qmin_u);
                }
              }
            };
            if (qmin_u != 0)
              r3_quads(std::true_type{});
            else
              r3_quads(std::false_type{});
          } else {
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
              const int4 ci4 = *reinterpret_cast<const int4*>(s_ci + pc + j);
              const float4 a4 = *reinterpret_cast<const float4*>(s_f1 + pc + j);
              const float4 b4 = *reinterpret_cast<const float4*>(s_f2 + pc + j);
              q[j + 0] = requant_u8<EPI>((int32_t)v[j + 0], ci4.x, rowc, a4.x, b4.x, e);
              q[j + 1] = requant_u8<EPI>((int32_t)v[j + 1], ci4.y, rowc, a4.y, b4.y, e);
              q[j + 2] = requant_u8<EPI>((int32_t)v[j + 2], ci4.z, rowc, a4.z, b4.z, e);
              q[j + 3] = requant_u8<EPI>((int32_t)v[j + 3], ci4.w, rowc, a4.w, b4.w, e);
            }
          }
          if (direct) {
            if (mvalid) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(e.y) + (size_t)mst * e.ldy + n0 + c0);
#pragma unroll
              for (int k = 0; k < CW / 16; ++k)
                dst[k] = make_uint4(pack_low_bytes(q[16 * k], q[16 * k + 1], q[16 * k + 2], q[16 * k + 3]),
                                    pack_low_bytes(q[16 * k + 4], q[16 * k + 5], q[16 * k + 6], q[16 * k + 7]),
                                    pack_low_bytes(q[16 * k + 8], q[16 * k + 9], q[16 * k + 10], q[16 * k + 11]),
                                    pack_low_bytes(q[16 * k + 12], q[16 * k + 13], q[16 * k + 14], q[16 * k + 15]));
            }
            return;
          }
          const int h = pc / SEG, cc = (pc % SEG) >> 4;
          uint8_t* seg = stg + h * (32 * SEG) + lane * SEG;
#pragma unroll
          for (int k = 0; k < CW / 16; ++k)
            ptx::st_shared_v4(seg + (((cc + k) ^ swz) << 4), pack_low_bytes(q[16 * k], q[16 * k + 1], q[16 * k + 2], q[16 * k + 3]),
                              pack_low_bytes(q[16 * k + 4], q[16 * k + 5], q[16 * k + 6], q[16 * k + 7]),
                              pack_low_bytes(q[16 * k + 8], q[16 * k + 9], q[16 * k + 10], q[16 * k + 11]),
                              pack_low_bytes(q[16 * k + 12], q[16 * k + 13], q[16 * k + 14], q[16 * k + 15]));
        }
      };
      uint32_t va[CW], vb[CW];
      int tev = 0;
      bool released = false;
      if (fast && HB == CW) {
        // one chunk per warp: the accumulator goes back to the MMA warp as
        // soon as it is in registers, so the next tiles' MMAs overlap this
        // requantisation
        ptx::tmem_ld_async(t_addr + (uint32_t)col0, va);
        ptx::tmem_wait_ld(va);
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&tempty_bar[acc]);
        released = true;
        chunk_fast(col0, va);
      } else if (fast) {
        // many epilogue warps per SM hide the TMEM load latency: one buffer
#pragma unroll 1
        for (int c0 = col0; c0 < col0 + HB; c0 += CW) {
          ptx::tmem_ld_async(t_addr + (uint32_t)c0, va);
          ptx::tmem_wait_ld(va);
          chunk_fast(c0, va);
          if (lane == 0) NNRCU_TRACE2_AT(warp, lt, tev++);
        }
      } else if (SPLIT == 4) {
#pragma unroll 1
        for (int c0 = col0; c0 < col0 + HB; c0 += CW) {
          ptx::tmem_ld_async(t_addr + (uint32_t)c0, va);
          ptx::tmem_wait_ld(va);
          chunk(c0, va);
        }
      } else {
      // few epilogue warps: TMEM loads double-buffered, chunk i + 1 in flight while i is processed
      ptx::tmem_ld_async(t_addr + (uint32_t)col0, va);
      ptx::tmem_wait_ld(va);
      if (lane == 0) NNRCU_TRACE2_AT(warp, lt, tev++);
#pragma unroll 1
      for (int c0 = col0; c0 < col0 + HB; c0 += 2 * CW) {
        const bool has_b = c0 + CW < col0 + HB;
        if (has_b) ptx::tmem_ld_async(t_addr + (uint32_t)(c0 + CW), vb);
        chunk(c0, va);
        if (lane == 0) NNRCU_TRACE2_AT(warp, lt, tev++);
        if (has_b) {
          ptx::tmem_wait_ld(vb);
          if (lane == 0) NNRCU_TRACE2_AT(warp, lt, tev++);
          const bool has_a = c0 + 2 * CW < col0 + HB;
          if (has_a) ptx::tmem_ld_async(t_addr + (uint32_t)(c0 + 2 * CW), va);
          chunk(c0 + CW, vb);
          if (lane == 0) NNRCU_TRACE2_AT(warp, lt, tev++);
          if (has_a) ptx::tmem_wait_ld(va);
          if (lane == 0) NNRCU_TRACE2_AT(warp, lt, tev++);
        }
      }
      }
      if (lane == 0) NNRCU_TRACE_AT(warp, lt, 3);
      // hand the accumulator back to the MMA warp
      if (!released) {
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&tempty_bar[acc]);
      }
      if (Cfg::OUT_BLOCK > 0 && y_tma) {
        // publish the staged block: rows >= M and columns >= N are clipped by the map
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) NNRCU_TRACE2_AT(warp, lt, 14);
        if (lane == 0) {
          constexpr int SEG = Cfg::OUT_SEG;
          constexpr int SEGE = SEG / Cfg::ESZ;  // elements per segment
          if (eq * 32 < nvr)
            for (int h = 0; h < Cfg::ROW_BYTES / SEG; ++h)
              if (n0 + col0 + h * SEGE < e.N) {
                // A_ROWS: map [rows][OW][N], pixels past OW are clipped
                if (AMODE == A_ROWS || AMODE == A_XROWS)
                  ptx::tma_store_3d(&tmY, stg + h * (32 * SEG), n0 + col0 + h * SEGE, ow0 + eq * 32, orow);
                else
                  ptx::tma_store_2d(&tmY, stg + h * (32 * SEG), n0 + col0 + h * SEGE, m0 + eq * 32);
              }
          ptx::bulk_commit();
          NNRCU_TRACE2_AT(warp, lt, 15);
        }
      }
    }
    if (Cfg::OUT_BLOCK > 0 && y_tma && lane == 0) ptx::bulk_wait0();  // stores complete before smem is released
    if (EPI == EPI_R2A && res_failed) ptx::settle_ns(200000);      // residual loads still in flight land first
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == R::MMA_WARP) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  NNRCU_SPAN_END();
}

}  // namespace nnrcu
