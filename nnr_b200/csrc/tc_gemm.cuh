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
// NPLANE = 2: fp32 emulated as split bf16 (kind::f16, f32 accumulate):
//             a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi with x_hi = bf16(x),
//             x_lo = bf16(x - x_hi); the dropped a_lo*b_lo term is < 2^-16
//             relative per product.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "ptx.cuh"

namespace nnrcu {

enum : int { A_TMA = 0, A_GATHER = 1, A_IM2COL = 2 };
enum : int { EPI_R1 = 1, EPI_R2 = 2, EPI_R3 = 3, EPI_R4 = 4, EPI_F32 = 10 };
enum : int { ACT_NONE = 0, ACT_RELU = 1, ACT_CLIP = 2, ACT_HARDSWISH = 3, ACT_SIGMOID = 4, ACT_LEAKYRELU = 5,
             ACT_TANH = 6 };
enum : int { ST_OK = 0, ST_TIMEOUT_FULL = 1, ST_TIMEOUT_EMPTY = 2, ST_TIMEOUT_ACCUM = 3 };

constexpr int BM = 128;       // rows per tile (TMEM lanes)
constexpr int BKB = 128;      // K bytes per stage per plane (one swizzle row); 64 for the 64-byte-slab variant
constexpr int NUM_THREADS = 320;  // 4 epilogue + 4 gather + TMA + MMA warps

// Geometry of the implicit im2col gather (A_GATHER). All sizes in bytes where noted.
struct GatherGeom {
  const uint8_t* x;      // NHWC activations, plane 0
  const uint8_t* x2;     // plane 1 (bf16 low halves) or null
  int N, H, W;
  int cbytes;            // bytes per pixel (channel stride), multiple of 16
  int OH, OW, KH, KW, sh, sw, ph, pw, dh, dw;
  int kbytes;            // real K in bytes = KH*KW*cbytes
  uint32_t pad_word;     // value written for padding pixels (x_zp replicated, or 0)
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
  // Fused QLinearAdd after the requant (u8 epilogues): y = QLinearAdd(q, qres)
  // with qres laid out like y. Same float sequence as the standalone op.
  const uint8_t* qres;                 // residual operand b, or null
  float qa_sa, qa_sb, qa_fixed;        // a_s / y_s, b_s / y_s, y_zp - fma(sa, a_zp, sb * b_zp)
  int qa_azp, qa_bzp, qa_yzp;
  long long qa_vec_end;                // elements below use the 16-wide body, the rest the scalar tail
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
  int* status;             // device status word (first error wins)
};

template <int BN, int NPLANE, int EPI, int KB = BKB, int SPLIT = 1>
struct TileCfg {
  static constexpr int A_BYTES = BM * KB;              // 16 KB per plane (8 KB with 64-byte slabs)
  static constexpr int B_BYTES = BN * KB;
  static constexpr int STAGE_BYTES = NPLANE * (A_BYTES + B_BYTES);
  // u8 epilogues stage each warp's 32 x BN output block for a TMA store
  static constexpr int OUT_BYTES = (EPI == EPI_F32) ? 0 : 4 * 32 * BN;
  // Epilogue warps: 4 x SPLIT, each covering 32 TMEM lanes x BN / SPLIT columns.
  static constexpr int HB = BN / SPLIT;
  static constexpr int OUT_SEG = HB >= 128 ? 128 : HB;  // bytes per staged row segment (= TMA box width)
  static constexpr int STAGES_RAW = (200 * 1024 - OUT_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 12 ? 12 : STAGES_RAW;
  // Gather producers publish a stage LAG iterations after issuing it: LAG
  // stages of copies in flight, STAGES - 1 - LAG stages of slack for the MMA.
  static constexpr int LAG = (STAGES - 1) / 2 > 1 ? (STAGES - 1) / 2 : 1;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators (power of two)
  static constexpr int PARAM_BYTES = 4 * SPLIT /*epilogue warps*/ * 3 * HB * 4;
  static constexpr int SMEM_BYTES =
      1024 /*align slack*/ + STAGES * STAGE_BYTES + OUT_BYTES + 512 /*barriers*/ + PARAM_BYTES;
  static_assert(STAGES >= 2, "need at least two pipeline stages");
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

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

// Requantise one int32 accumulator to u8 with the formula EPI selects.
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
  } else if constexpr (EPI == EPI_R2) {
    // f = float(acc + bias) * os; max(lo - y_zp) then min(hi - y_zp); rne; + y_zp; saturate
    int32_t v = (int32_t)((uint32_t)raw + (uint32_t)ci);
    float f = __fmul_rn(__int2float_rn(v), f1);
    f = fminf(fmaxf(f, e.rq_lo), e.rq_hi);
    // f lies in [-y_zp, 255 - y_zp] (integral bounds), so rne(f) + y_zp is
    // already in [0, 255]: the unsigned saturation of the reference is a no-op
    return (uint32_t)(__float2int_rn(f) + e.yzp);
  } else if constexpr (EPI == EPI_R3) {
    // f = fma(float(acc), cs, bias_f); f = fma(f, inv_y, y_zp); min(hi) then max(qmin); rne
    int32_t acc = (int32_t)((uint32_t)raw + (uint32_t)ci);
    float f = __fmaf_rn(__int2float_rn(acc), f1, f2);
    f = __fmaf_rn(f, e.inv_y, e.yzp_f);
    f = fmaxf(fminf(f, e.qmax_f), e.qmin_f);
    return (uint32_t)__float2int_rn(f);
  } else {  // EPI_R4
    // val = fma(float(acc), a_s*b_s/y_s, y_zp); nearbyint; clamp [0, 255]
    int32_t acc = (int32_t)((uint32_t)raw + (uint32_t)ci + (uint32_t)rowc);
    float f = __fmaf_rn(__int2float_rn(acc), e.combined, e.yzp_f);
    int32_t q = __float2int_rn(f);
    q = q < 0 ? 0 : (q > 255 ? 255 : q);
    return (uint32_t)q;
  }
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
template <int BN, int NPLANE, int AMODE, int EPI, int KB>
__global__ void __launch_bounds__(NUM_THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
               const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmY,
               const __grid_constant__ CUtensorMap tmR, int y_tma,
               int b_plane_rows, GatherGeom g, EpiParams e, int num_kb, int m_tiles, int n_tiles) {
  // In TMA / im2col modes the gather warps 4-7 are free and join the epilogue:
  // warps w and w + 4 drain the same 32 TMEM lanes, each half of the columns.
  constexpr int SPLIT = (AMODE == A_GATHER) ? 1 : 2;
  constexpr int HB = BN / SPLIT;
  using Cfg = TileCfg<BN, NPLANE, EPI, KB, SPLIT>;
  static_assert(KB == BKB || AMODE != A_GATHER, "the gather producers fill 128-byte slabs");
  constexpr int STAGES = Cfg::STAGES;
  constexpr int A_BYTES = Cfg::A_BYTES;
  constexpr int B_BYTES = Cfg::B_BYTES;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                                        // [STAGES][NPLANE][A_BYTES]
  uint8_t* sB = sA + STAGES * NPLANE * A_BYTES;              // [STAGES][NPLANE][B_BYTES]
  uint8_t* sOut = sB + STAGES * NPLANE * B_BYTES;            // [4 warps][32 rows][BN] (u8 epilogues)
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sOut + Cfg::OUT_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;                  // [2] accumulator ready
  uint64_t* tempty_bar = tfull_bar + 2;                      // [2] accumulator drained
  uint64_t* res_bar = tempty_bar + 2;                        // [8] residual tile landed (per epilogue warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_bar + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = m_tiles * n_tiles;
  // per-column constants, one private copy per epilogue warp (no cross-warp sync)
  int32_t* s_ci = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(full_bar) + 512 +
                                             (warp & (4 * SPLIT - 1)) * (3 * HB * 4));
  float* s_f1 = reinterpret_cast<float*>(s_ci + HB);
  float* s_f2 = s_f1 + HB;

  if (threadIdx.x == 0) {
    const uint32_t full_count = (AMODE == A_GATHER) ? (4u + 1u) : 1u;  // 4 gather warps + TMA
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full_bar[s], full_count);
      ptx::mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 8; ++a) ptx::mbar_init(&res_bar[a], 1);
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull_bar[a], 1);
      ptx::mbar_init(&tempty_bar[a], 4 * SPLIT);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == 8 && lane == 0) {
    ptx::tma_prefetch_desc(&tmB);
    if (AMODE != A_GATHER) {
      ptx::tma_prefetch_desc(&tmA0);
      if (NPLANE == 2) ptx::tma_prefetch_desc(&tmA1);
    }
  }
  if (warp == 9) ptx::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto fail = [&](int code) {
    record_status(e.status, code);
    *abort_flag = 1;
  };

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      constexpr uint32_t tx = (AMODE != A_GATHER ? NPLANE * A_BYTES : 0) + NPLANE * B_BYTES;
      bool aborted = false;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !aborted; tile += gridDim.x) {
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
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!ptx::mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag)) { fail(ST_TIMEOUT_EMPTY); aborted = true; break; }
          ptx::mbar_arrive_expect_tx(&full_bar[s], tx);
          uint8_t* a_st = sA + (size_t)s * NPLANE * A_BYTES;
          uint8_t* b_st = sB + (size_t)s * NPLANE * B_BYTES;
          const int kx = kb * KB / (NPLANE == 2 ? 2 : 1);  // element coordinate along K
          for (int p = 0; p < NPLANE; ++p)
            ptx::tma_load_2d(b_st + p * B_BYTES, &tmB, &full_bar[s], kx, p * b_plane_rows + n0);
          if (AMODE == A_TMA) {
            ptx::tma_load_2d(a_st, &tmA0, &full_bar[s], kx, m0);
            if (NPLANE == 2) ptx::tma_load_2d(a_st + A_BYTES, &tmA1, &full_bar[s], kx, m0);
          } else if (AMODE == A_IM2COL) {
            // one K slab = 128 bytes of channels of a single filter tap
            const int kbyte = kb * KB;
            const int tap = kbyte / g.cbytes;
            const int cc = (kbyte - tap * g.cbytes) / (NPLANE == 2 ? 2 : 1);
            const int kh = tap / g.KW, kw = tap - kh * g.KW;
            const uint16_t ow_off = (uint16_t)(kw * g.dw), oh_off = (uint16_t)(kh * g.dh);
            ptx::tma_load_im2col_4d(a_st, &tmA0, &full_bar[s], cc, i_w, i_h, i_n, ow_off, oh_off);
            if (NPLANE == 2) ptx::tma_load_im2col_4d(a_st + A_BYTES, &tmA1, &full_bar[s], cc, i_w, i_h, i_n, ow_off, oh_off);
          }
        }
      }
      if (aborted) ptx::settle_ns(200000);  // let copies already in flight land before the CTA exits
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = (NPLANE == 1) ? ptx::umma_idesc(2, 0, 1, BM, BN) : ptx::umma_idesc(1, 1, 1, BM, BN);
      bool aborted = false;
      int it = 0, lt = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !aborted; tile += gridDim.x, ++lt) {
        const int acc = lt & 1;
        const uint32_t use_ph = (uint32_t)(lt >> 1) & 1u;
        if (!ptx::mbar_wait(&tempty_bar[acc], use_ph ^ 1u, abort_flag)) { fail(ST_TIMEOUT_ACCUM); aborted = true; break; }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!ptx::mbar_wait(&full_bar[s], ph, abort_flag)) { fail(ST_TIMEOUT_FULL); aborted = true; break; }
          ptx::tc_fence_after();
          ptx::fence_proxy_async_smem();
          const uint32_t a_addr = ptx::smem_u32(sA + (size_t)s * NPLANE * A_BYTES);
          const uint32_t b_addr = ptx::smem_u32(sB + (size_t)s * NPLANE * B_BYTES);
#pragma unroll
          for (int k = 0; k < KB / 32; ++k) {
            const uint32_t koff = k * 32;
            if constexpr (NPLANE == 1) {
              ptx::mma_i8(d_tmem, ptx::umma_desc_sw<KB>(a_addr + koff), ptx::umma_desc_sw<KB>(b_addr + koff), idesc,
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
          ptx::mma_commit(&empty_bar[s]);
        }
        if (!aborted) ptx::mma_commit(&tfull_bar[acc]);  // fires when this tile's MMAs have completed
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
          uint8_t* const row_dst = row_dst0 + (size_t)s * NPLANE * A_BYTES;
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
  } else if (warp < 4 * SPLIT) {
    // ------------------------------------------------------------ epilogue (warps 0-3, and 4-7 when SPLIT = 2)
    const int eq = warp & 3;           // TMEM lane quarter
    const int col0 = (warp >> 2) * HB; // this warp's columns [col0, col0 + HB) of the tile
    const int row = eq * 32 + lane;    // TMEM lane == tile row
    int lt = 0;
    int cached_n0 = -1;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
      const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
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
          if (EPI == EPI_R2) {
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
      uint8_t* const stg = sOut + warp * (32 * HB);
      // fused residual add: the residual block lands in the staging buffer
      // (same box and swizzle as the output store), loaded while the MMAs
      // run, and is combined with the requantised tile in place
      const bool res_tma = EPI != EPI_F32 && y_tma && e.qres != nullptr;
      if (EPI != EPI_F32 && y_tma) {
        if (lane == 0) {
          ptx::bulk_wait_read0();
          if (res_tma) {
            constexpr int SEG = Cfg::OUT_SEG;
            ptx::mbar_arrive_expect_tx(&res_bar[warp], 32 * HB);
            for (int h = 0; h < HB / SEG; ++h)
              ptx::tma_load_2d(stg + h * (32 * SEG), &tmR, &res_bar[warp], n0 + col0 + h * SEG, m0 + eq * 32);
          }
        }
        __syncwarp();
      }
      if (!__all_sync(0xffffffffu, ptx::mbar_wait(&tfull_bar[acc], use_ph, abort_flag))) {
        fail(ST_TIMEOUT_ACCUM);
        break;
      }
      ptx::tc_fence_after();
      if (res_tma && !__all_sync(0xffffffffu, ptx::mbar_wait(&res_bar[warp], (uint32_t)lt & 1u, abort_flag))) {
        fail(ST_TIMEOUT_ACCUM);
        break;
      }
      const int m = m0 + row;
      const bool mvalid = m < e.M;
      int32_t rowc = 0;
      if (EPI == EPI_R4 && e.rowcorr && mvalid) rowc = e.rowcorr[m];
      int img = 0, pix = 0;
      if (e.y_layout == 1 && mvalid) { img = m / e.ohw; pix = m - img * e.ohw; }
      const uint32_t t_addr = tmem_base + ((uint32_t)(eq * 32) << 16) + (uint32_t)(acc * BN);
      // one 32-column chunk: requant / bias / post-op / stores
      auto chunk = [&](const int c0, uint32_t (&v)[32]) {
        const int pc = c0 - col0;  // column within this warp's parameter copy
        if (!mvalid || n0 + c0 >= e.N) return;
        const int nvalid = min(32, e.N - (n0 + c0));
        if constexpr (EPI == EPI_F32) {
          float* y = static_cast<float*>(e.y);
          const bool rowmajor = e.y_layout == 0;
          float* dst = rowmajor ? y + (size_t)m * e.ldy + n0 + c0 : nullptr;
          const float* res = (e.residual && rowmajor) ? e.residual + (size_t)m * e.ldy + n0 + c0 : nullptr;
          if (rowmajor && nvalid == 32 && (e.ldy & 3) == 0 && ((reinterpret_cast<uintptr_t>(e.y) & 15) == 0) &&
              (!e.residual || (reinterpret_cast<uintptr_t>(e.residual) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              float o[4];
              float4 rr = make_float4(0.f, 0.f, 0.f, 0.f);
              if (res) rr = *reinterpret_cast<const float4*>(res + j);
              const float rv[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                float a = __uint_as_float(v[j + u]) + s_f2[pc + j + u];
                if (e.res_mode == 1) a = fmaf(e.res_scale, rv[u], a);
                a = apply_act(a, e.act, e.act_a, e.act_b);
                if (e.res_mode == 2) a += rv[u];
                o[u] = a;
              }
              *reinterpret_cast<float4*>(dst + j) = make_float4(o[0], o[1], o[2], o[3]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j >= nvalid) break;
              const size_t idx = rowmajor ? (size_t)m * e.ldy + n0 + c0 + j
                                          : ((size_t)img * e.N + n0 + c0 + j) * e.ohw + pix;
              const float rr = e.residual ? e.residual[idx] : 0.0f;
              float a = __uint_as_float(v[j]) + s_f2[pc + j];
              if (e.res_mode == 1) a = fmaf(e.res_scale, rr, a);
              a = apply_act(a, e.act, e.act_a, e.act_b);
              if (e.res_mode == 2) a += rr;
              y[idx] = a;
            }
          }
        } else {
          uint32_t q[32];
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const int4 ci4 = *reinterpret_cast<const int4*>(s_ci + pc + j);
            const float4 a4 = *reinterpret_cast<const float4*>(s_f1 + pc + j);
            const float4 b4 = *reinterpret_cast<const float4*>(s_f2 + pc + j);
            q[j + 0] = requant_u8<EPI>((int32_t)v[j + 0], ci4.x, rowc, a4.x, b4.x, e);
            q[j + 1] = requant_u8<EPI>((int32_t)v[j + 1], ci4.y, rowc, a4.y, b4.y, e);
            q[j + 2] = requant_u8<EPI>((int32_t)v[j + 2], ci4.z, rowc, a4.z, b4.z, e);
            q[j + 3] = requant_u8<EPI>((int32_t)v[j + 3], ci4.w, rowc, a4.w, b4.w, e);
          }
          if (e.qres) {
            // QLinearAdd(q, residual) (QLinearAdd.cpp:46-104): body
            // fma(a, sa, fma(b, sb, fixed)), rne, saturate; tail elements
            // fma(sa, a - a_zp, sb * (b - b_zp)) + y_zp.
            const uint8_t* rp = e.qres + (size_t)m * e.ldy + n0 + c0;
            uint8_t rb[32];
            if (res_tma) {
              constexpr int SEG = Cfg::OUT_SEG;
              const int h = pc / SEG, cc = (pc % SEG) >> 4;
              const int f = SEG == 128 ? (lane & 7) : (SEG == 64 ? ((lane >> 1) & 3) : ((lane >> 2) & 1));
              const uint8_t* seg = stg + h * (32 * SEG) + lane * SEG;
              *reinterpret_cast<uint4*>(rb) = *reinterpret_cast<const uint4*>(seg + ((cc ^ f) << 4));
              *reinterpret_cast<uint4*>(rb + 16) = *reinterpret_cast<const uint4*>(seg + (((cc + 1) ^ f) << 4));
            } else if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(rp) & 15) == 0)) {
              *reinterpret_cast<uint4*>(rb) = reinterpret_cast<const uint4*>(rp)[0];
              *reinterpret_cast<uint4*>(rb + 16) = reinterpret_cast<const uint4*>(rp)[1];
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) rb[j] = j < nvalid ? rp[j] : 0;
            }
            const long long ebase = (long long)m * e.N + n0 + c0;
            if (ebase + 32 <= e.qa_vec_end) {  // whole chunk in the 16-wide body (the common case)
              const float sa = e.qa_sa, sb = e.qa_sb, fx = e.qa_fixed;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int r = __float2int_rn(__fmaf_rn((float)q[j], sa, __fmaf_rn((float)rb[j], sb, fx)));
                q[j] = (uint32_t)min(max(r, 0), 255);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float fa = (float)q[j], fb = (float)rb[j];
                int r;
                if (ebase + j < e.qa_vec_end) {
                  r = __float2int_rn(__fmaf_rn(fa, e.qa_sa, __fmaf_rn(fb, e.qa_sb, e.qa_fixed)));
                } else {
                  const float da = (float)((int)q[j] - e.qa_azp), db = (float)((int)rb[j] - e.qa_bzp);
                  r = __float2int_rn(__fadd_rn(__fmaf_rn(e.qa_sa, da, __fmul_rn(e.qa_sb, db)), (float)e.qa_yzp));
                }
                q[j] = (uint32_t)(r < 0 ? 0 : (r > 255 ? 255 : r));
              }
            }
          }
          uint8_t* y = static_cast<uint8_t*>(e.y);
          uint32_t w[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            w[j] = q[4 * j] | (q[4 * j + 1] << 8) | (q[4 * j + 2] << 16) | (q[4 * j + 3] << 24);
          if (y_tma) {
            // swizzled staging (matches the store map's 128B / 64B swizzle):
            // row r, 16-byte chunk c of a segment lives at r*SEG + ((c ^ f(r)) << 4)
            constexpr int SEG = Cfg::OUT_SEG;
            const int h = pc / SEG, cc = (pc % SEG) >> 4;
            const int f = SEG == 128 ? (lane & 7) : (SEG == 64 ? ((lane >> 1) & 3) : ((lane >> 2) & 1));
            uint8_t* seg = stg + h * (32 * SEG) + lane * SEG;
            ptx::st_shared_v4(seg + ((cc ^ f) << 4), w[0], w[1], w[2], w[3]);
            ptx::st_shared_v4(seg + (((cc + 1) ^ f) << 4), w[4], w[5], w[6], w[7]);
          } else if (e.y_layout == 0) {
            uint8_t* dst = y + (size_t)m * e.ldy + n0 + c0;
            if (nvalid == 32 && (e.ldy & 15) == 0 && (reinterpret_cast<uintptr_t>(e.y) & 15) == 0) {
              reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
              reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nvalid) dst[j] = (uint8_t)q[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nvalid) y[((size_t)img * e.N + n0 + c0 + j) * e.ohw + pix] = (uint8_t)q[j];
          }
        }
            };
      // TMEM loads are double-buffered: chunk i + 1 is in flight while i is processed
      uint32_t va[32], vb[32];
      ptx::tmem_ld32_async(t_addr + (uint32_t)col0, va);
      ptx::tmem_wait_ld(va);
#pragma unroll 1
      for (int c0 = col0; c0 < col0 + HB; c0 += 64) {
        const bool has_b = c0 + 32 < col0 + HB;
        if (has_b) ptx::tmem_ld32_async(t_addr + (uint32_t)(c0 + 32), vb);
        chunk(c0, va);
        if (has_b) {
          ptx::tmem_wait_ld(vb);
          const bool has_a = c0 + 64 < col0 + HB;
          if (has_a) ptx::tmem_ld32_async(t_addr + (uint32_t)(c0 + 64), va);
          chunk(c0 + 32, vb);
          if (has_a) ptx::tmem_wait_ld(va);
        }
      }
      // hand the accumulator back to the MMA warp
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&tempty_bar[acc]);
      if (EPI != EPI_F32 && y_tma) {
        // publish the staged block: rows >= M and columns >= N are clipped by the map
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          constexpr int SEG = Cfg::OUT_SEG;
          if (m0 + eq * 32 < e.M)
            for (int h = 0; h < HB / SEG; ++h)
              if (n0 + col0 + h * SEG < e.N)
                ptx::tma_store_2d(&tmY, stg + h * (32 * SEG), n0 + col0 + h * SEG, m0 + eq * 32);
          ptx::bulk_commit();
        }
      }
    }
    if (EPI != EPI_F32 && y_tma && lane == 0) ptx::bulk_wait0();  // stores complete before smem is released
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace nnrcu
