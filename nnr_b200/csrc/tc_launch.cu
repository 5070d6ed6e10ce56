// Instantiations of the tcgen05 engine and the runtime dispatch onto them.
#include <algorithm>

#include "internal.h"
#include "tc_gemm.cuh"

namespace nnrcu {

namespace {

// One (N tile, K slab) box of B per block: loaded by the tensor map (so the
// shared-memory swizzle is exactly the one the engine's loads produce), then
// written out as a contiguous image.
__global__ void pack_b_images_kernel(const __grid_constant__ CUtensorMap tmB, int bn, int kb, int num_kb,
                                     uint8_t* __restrict out, int* status) {
  extern __shared__ uint8_t raw[];
  __shared__ uint64_t bar;
  uint8_t* sm = raw + ((1024u - (ptx::smem_u32(raw) & 1023u)) & 1023u);
  const uint32_t bytes = (uint32_t)(bn * kb);
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ptx::mbar_arrive_expect_tx(&bar, bytes);
    ptx::tma_load_2d(sm, &tmB, &bar, (int)blockIdx.y * kb, (int)blockIdx.x * bn);
  }
  if (!ptx::mbar_wait(&bar, 0u)) {
    if (threadIdx.x == 0) record_status(status, ST_TIMEOUT_FULL);
    ptx::settle_ns(200000);
    return;
  }
  uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)blockIdx.x * num_kb + blockIdx.y) * bytes);
  const uint4* src = reinterpret_cast<const uint4*>(sm);
  for (uint32_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) dst[i] = src[i];
}

template <int BN, int NPLANE, int AMODE, int EPI, int KB = BKB, int NKBR = 0>
int launch_one(const TcLaunch& L, const GatherGeom& g, const EpiParams& e, cudaStream_t stream) {
  using Cfg = KernelCfg<BN, NPLANE, AMODE, EPI, KB, NKBR>;
  auto kern = tc_gemm_kernel<BN, NPLANE, AMODE, EPI, KB, NKBR>;
  // The attribute is per function; setting it is cheap but not free, so do it
  // once per device.
  static unsigned long long configured = 0;
  int dev = 0;
  NNRCU_CUDA(cudaGetDevice(&dev));
  if (!(configured & (1ull << dev))) {
    NNRCU_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    configured |= 1ull << dev;
  }
  const long long tiles = (long long)L.m_tiles * L.n_tiles;
  int grid = (int)std::min<long long>(tiles, (long long)num_sms());
  // resident B: each CTA keeps one N tile's weights, so its tiles must all
  // share that N tile (tile % n_tiles == blockIdx.x % n_tiles)
  if (NKBR > 0) grid = std::max(L.n_tiles, grid / L.n_tiles * L.n_tiles);
  // u8 outputs in row-major [M, ldy] leave through a TMA store of each
  // warp's staged 32 x BN block (coalesced rows instead of per-lane pieces).
  CUtensorMap tmY{};
  int y_tma = 0;
  if ((AMODE == A_ROWS || AMODE == A_XROWS) && EPI != EPI_F32 && e.y_layout == 0 && !e.opad && (reinterpret_cast<uintptr_t>(e.y) & 15) == 0 &&
      (e.ldy & 15) == 0) {
    // [output rows][OW][N]: a warp's 32 pixels of one output row, clipped at OW
    const int seg = Cfg::OUT_SEG;
    const uint64_t dims[3] = {(uint64_t)e.N, (uint64_t)g.OW, (uint64_t)g.N * g.OH};
    const uint64_t strides[2] = {(uint64_t)e.ldy, (uint64_t)e.ldy * g.OW};
    const uint32_t box[3] = {(uint32_t)seg, 32, 1};
    int rc = encode_tmap_3d(&tmY, CU_TENSOR_MAP_DATA_TYPE_UINT8, e.y, dims, strides, box,
                            seg == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                       : (seg == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B));
    if (rc != NNRCU_OK) return rc;
    y_tma = 1;
  } else if (AMODE != A_ROWS && AMODE != A_XROWS && AMODE != A_SHIFT && EPI != EPI_F32 && e.y_layout == 0 && !e.opad && (reinterpret_cast<uintptr_t>(e.y) & 15) == 0 &&
             (e.ldy & 15) == 0) {
    const int seg = Cfg::OUT_SEG;
    int rc = encode_tmap_2d(&tmY, CU_TENSOR_MAP_DATA_TYPE_UINT8, e.y, (uint64_t)e.N, (uint64_t)e.M, (uint64_t)e.ldy,
                            seg, 32,
                            seg == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                       : (seg == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B));
    if (rc != NNRCU_OK) return rc;
    y_tma = 1;
  }
  if (EPI == EPI_F32 && Cfg::OUT_BLOCK > 0 && AMODE != A_ROWS && e.y_layout == 0 &&
      (reinterpret_cast<uintptr_t>(e.y) & 15) == 0 && (e.ldy & 3) == 0) {
    // fp32 rows leave through the staged TMA store too (32-float segments)
    const int seg = Cfg::OUT_SEG;
    int rc = encode_tmap_2d(&tmY, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, e.y, (uint64_t)e.N, (uint64_t)e.M,
                            (uint64_t)e.ldy * 4, seg / 4, 32,
                            seg == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                       : (seg == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B));
    if (rc != NNRCU_OK) return rc;
    y_tma = 1;
  }
  CUtensorMap tmR{};
  if (EPI == EPI_R2A) {
    if (!y_tma) return set_error(NNRCU_ERR_INVALID, "the prefetched residual add needs a TMA-stored output");
    if (reinterpret_cast<uintptr_t>(e.qres) & 15) return set_error(NNRCU_ERR_INVALID, "residual must be 16-byte aligned");
    const int seg = Cfg::OUT_SEG;
    int rc = encode_tmap_2d(&tmR, CU_TENSOR_MAP_DATA_TYPE_UINT8, e.qres, (uint64_t)e.N, (uint64_t)e.M,
                            (uint64_t)e.ldy, seg, 32,
                            seg == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                       : (seg == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B));
    if (rc != NNRCU_OK) return rc;
  }
  // programmatic dependent launch: the prologue of this grid may overlap the
  // tail of the previous kernel on the stream (the kernel waits before its
  // first dependent access)
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Roles<AMODE, BN, EPI>::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NNRCU_CUDA(cudaLaunchKernelEx(&cfg, kern, *L.tmA0, *L.tmA1, *L.tmB, tmY, tmR, y_tma, L.b_plane_rows, g, e, L.num_kb,
                                L.m_tiles, L.n_tiles));
  NNRCU_CUDA(cudaGetLastError());
  return NNRCU_OK;
}

template <int BN>
int dispatch_bn(const TcLaunch& L, const GatherGeom& g, const EpiParams& e, cudaStream_t st) {
  if (L.kb_bytes == 16) {
    // eight 16-byte taps per stage (space-to-depth convs): int8 im2col, N tile <= 128
    if constexpr (BN <= 128) {
      if (L.nplane == 1 && L.amode == A_ROWS) {
        if (L.epi == EPI_R1) return launch_one<BN, 1, A_ROWS, EPI_R1, 16>(L, g, e, st);
        if (L.epi == EPI_R2) return launch_one<BN, 1, A_ROWS, EPI_R2, 16>(L, g, e, st);
        if (L.epi == EPI_R3) return launch_one<BN, 1, A_ROWS, EPI_R3, 16>(L, g, e, st);
        if (L.epi == EPI_R3N) return launch_one<BN, 1, A_ROWS, EPI_R3N, 16>(L, g, e, st);
      }
      if (L.nplane == 1 && L.amode == A_IM2COL) {
        if (L.epi == EPI_R1) return launch_one<BN, 1, A_IM2COL, EPI_R1, 16>(L, g, e, st);
        if (L.epi == EPI_R2) return launch_one<BN, 1, A_IM2COL, EPI_R2, 16>(L, g, e, st);
        if (L.epi == EPI_R3) return launch_one<BN, 1, A_IM2COL, EPI_R3, 16>(L, g, e, st);
        if (L.epi == EPI_R3N) return launch_one<BN, 1, A_IM2COL, EPI_R3N, 16>(L, g, e, st);
      }
    }
    return set_error(NNRCU_ERR_INVALID, "no 16-byte-tap engine instance for bn %d amode %d epilogue %d", BN, L.amode,
                     L.epi);
  }
  if (L.kb_bytes == 64) {
    // 64-byte K slabs (channel strides of 64 bytes): TMA-fed A only; split-bf16
    // fp32 (32 bf16 per slab) with 2-D TMA tiles
    if (L.nplane == 2 && L.amode == A_TMA && L.epi == EPI_F32) {
      if constexpr (BN <= 128) return launch_one<BN, 2, A_TMA, EPI_F32, 64>(L, g, e, st);
    }
    if (L.nplane != 1 || L.amode == A_GATHER)
      return set_error(NNRCU_ERR_INVALID, "64-byte K slabs need int8 or split-bf16 with a TMA-fed A operand");
    if (L.epi == EPI_R2A && L.amode == A_TMA) return launch_one<BN, 1, A_TMA, EPI_R2A, 64>(L, g, e, st);
    if (L.amode == A_XROWS) {
      // space-to-depth convs as 64-byte kernel rows (N tile <= 128)
      if constexpr (BN <= 128) {
        if (L.epi == EPI_R1) return launch_one<BN, 1, A_XROWS, EPI_R1, 64>(L, g, e, st);
        if (L.epi == EPI_R2) return launch_one<BN, 1, A_XROWS, EPI_R2, 64>(L, g, e, st);
        if (L.epi == EPI_R3) return launch_one<BN, 1, A_XROWS, EPI_R3, 64>(L, g, e, st);
        if (L.epi == EPI_R3N) return launch_one<BN, 1, A_XROWS, EPI_R3N, 64>(L, g, e, st);
      }
      return set_error(NNRCU_ERR_INVALID, "no 64-byte-row s2d instance for bn %d epilogue %d", BN, L.epi);
    }
    if (L.amode == A_IM2COL) {
      if (L.epi == EPI_R1) return launch_one<BN, 1, A_IM2COL, EPI_R1, 64>(L, g, e, st);
      if (L.epi == EPI_R2) return launch_one<BN, 1, A_IM2COL, EPI_R2, 64>(L, g, e, st);
    } else {
      if (L.epi == EPI_R1) return launch_one<BN, 1, A_TMA, EPI_R1, 64>(L, g, e, st);
      if (L.epi == EPI_R2) return launch_one<BN, 1, A_TMA, EPI_R2, 64>(L, g, e, st);
      if (L.epi == EPI_R3) return launch_one<BN, 1, A_TMA, EPI_R3, 64>(L, g, e, st);
      if (L.epi == EPI_R3N) return launch_one<BN, 1, A_TMA, EPI_R3N, 64>(L, g, e, st);
      if (L.epi == EPI_R4) return launch_one<BN, 1, A_TMA, EPI_R4, 64>(L, g, e, st);
    }
    return set_error(NNRCU_ERR_INVALID, "no 64-byte-slab engine instance for amode %d epilogue %d", L.amode, L.epi);
  }
  if (L.nplane == 3 || L.nplane == 4) {
    // one bf16 (3) or fp16 (4) plane: 2-D TMA or gathered A, fp32 epilogue
    if (L.epi != EPI_F32) return set_error(NNRCU_ERR_INVALID, "16-bit engine needs the fp32 epilogue");
    if (L.nplane == 3)
      return L.amode == A_TMA ? launch_one<BN, 3, A_TMA, EPI_F32>(L, g, e, st) : launch_one<BN, 3, A_GATHER, EPI_F32>(L, g, e, st);
    return L.amode == A_TMA ? launch_one<BN, 4, A_TMA, EPI_F32>(L, g, e, st) : launch_one<BN, 4, A_GATHER, EPI_F32>(L, g, e, st);
  }
  if (L.nplane == 2) {
    if (L.epi != EPI_F32) return set_error(NNRCU_ERR_INVALID, "split-bf16 engine needs the fp32 epilogue");
    if (L.amode == A_TMA) return launch_one<BN, 2, A_TMA, EPI_F32>(L, g, e, st);
    if (L.amode == A_IM2COL) return launch_one<BN, 2, A_IM2COL, EPI_F32>(L, g, e, st);
    return launch_one<BN, 2, A_GATHER, EPI_F32>(L, g, e, st);
  }
  if (L.amode == A_IM2COL) {
    switch (L.epi) {
      case EPI_R1: return launch_one<BN, 1, A_IM2COL, EPI_R1>(L, g, e, st);
      case EPI_R2: return launch_one<BN, 1, A_IM2COL, EPI_R2>(L, g, e, st);
      default: break;
    }
  } else if (L.amode == A_TMA) {
    switch (L.epi) {
      case EPI_R1: return launch_one<BN, 1, A_TMA, EPI_R1>(L, g, e, st);
      case EPI_R2: return launch_one<BN, 1, A_TMA, EPI_R2>(L, g, e, st);
      case EPI_R2A: return launch_one<BN, 1, A_TMA, EPI_R2A>(L, g, e, st);
      case EPI_R4: return launch_one<BN, 1, A_TMA, EPI_R4>(L, g, e, st);
      default: break;
    }
  } else {
    switch (L.epi) {
      case EPI_R1: return launch_one<BN, 1, A_GATHER, EPI_R1>(L, g, e, st);
      case EPI_R2: return launch_one<BN, 1, A_GATHER, EPI_R2>(L, g, e, st);
      case EPI_R3: return launch_one<BN, 1, A_GATHER, EPI_R3>(L, g, e, st);
      case EPI_R3N: return launch_one<BN, 1, A_GATHER, EPI_R3N>(L, g, e, st);
      case EPI_R4: return launch_one<BN, 1, A_GATHER, EPI_R4>(L, g, e, st);
      default: break;
    }
  }
  return set_error(NNRCU_ERR_INVALID, "no engine instance for amode %d epilogue %d", L.amode, L.epi);
}

}  // namespace

#ifdef NNRCU_TRACE
extern "C" int nnrcu_trace_read(void* host, size_t bytes) {
  NNRCU_CUDA(cudaDeviceSynchronize());
  NNRCU_CUDA(cudaMemcpyFromSymbol(host, g_trace, bytes < sizeof(g_trace) ? bytes : sizeof(g_trace)));
  void* dev = nullptr;
  NNRCU_CUDA(cudaGetSymbolAddress(&dev, g_trace));
  NNRCU_CUDA(cudaMemset(dev, 0, sizeof(g_trace)));
  return NNRCU_OK;
}
extern "C" int nnrcu_trace2_read(void* host, size_t bytes) {
  NNRCU_CUDA(cudaDeviceSynchronize());
  NNRCU_CUDA(cudaMemcpyFromSymbol(host, g_trace2, bytes < sizeof(g_trace2) ? bytes : sizeof(g_trace2)));
  void* dev = nullptr;
  NNRCU_CUDA(cudaGetSymbolAddress(&dev, g_trace2));
  NNRCU_CUDA(cudaMemset(dev, 0, sizeof(g_trace2)));
  return NNRCU_OK;
}
#endif

#ifdef NNRCU_TRACE
static int g_span_next = 0;
extern "C" int nnrcu_span_reset(void) {
  // slots restart at 0 (for the next capture); spans are cleared to (max, 0, max, 0)
  g_span_next = 0;
  static unsigned long long init[256 * 4];
  for (int i = 0; i < 256; ++i) init[i * 4] = init[i * 4 + 2] = ~0ull, init[i * 4 + 1] = init[i * 4 + 3] = 0;
  NNRCU_CUDA(cudaMemcpyToSymbol(g_span, init, sizeof(init)));
  return NNRCU_OK;
}
extern "C" int nnrcu_span_read(void* host, size_t bytes) {
  NNRCU_CUDA(cudaDeviceSynchronize());
  NNRCU_CUDA(cudaMemcpyFromSymbol(host, g_span, bytes < sizeof(g_span) ? bytes : sizeof(g_span)));
  return NNRCU_OK;
}
#endif

int pack_b_images(const CUtensorMap* tmB, int bn, int kb_bytes, int n_tiles, int num_kb, void* out) {
  const int smem = bn * kb_bytes + 1024;
  NNRCU_CUDA(cudaFuncSetAttribute(pack_b_images_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  pack_b_images_kernel<<<dim3(n_tiles, num_kb), 256, smem>>>(*tmB, bn, kb_bytes, num_kb, static_cast<uint8_t*>(out),
                                                              status_ptr());
  NNRCU_CUDA(cudaGetLastError());
  NNRCU_CUDA(cudaDeviceSynchronize());
  int st = 0;
  NNRCU_CUDA(cudaMemcpy(&st, status_ptr(), sizeof(int), cudaMemcpyDeviceToHost));
  if (st) return set_error(NNRCU_ERR_CUDA, "packing the weight images timed out (status %d)", st);
  return NNRCU_OK;
}

int tc_launch(const TcLaunch& L, const GatherGeom& g, const EpiParams& e_in, cudaStream_t stream) {
  EpiParams e = e_in;
#ifdef NNRCU_TRACE
  e.trace_seq = g_span_next++;
#else
  e.trace_seq = -1;
#endif
  if (L.m_tiles <= 0 || L.n_tiles <= 0 || L.num_kb <= 0) return NNRCU_OK;
  if ((long long)L.m_tiles * L.n_tiles > 0x7fffffffLL)
    return set_error(NNRCU_ERR_INVALID, "too many tiles (%d x %d)", L.m_tiles, L.n_tiles);
  if (L.amode == A_GATHER && ((reinterpret_cast<uintptr_t>(g.x) & 15) || (g.x2 && (reinterpret_cast<uintptr_t>(g.x2) & 15)) ||
                              (g.cbytes & 15)))
    return set_error(NNRCU_ERR_INVALID, "gathered operand must be 16-byte aligned with a 16-byte pixel stride");
  // an R2 requant with a fused add whose output and residual can move by
  // TMA (16-byte aligned NHWC rows) runs the residual-prefetching instance
  TcLaunch L2 = L;
  if (L.epi == EPI_R3 && e.y_layout == 1) L2.epi = EPI_R3N;
  // Resident B: a single N tile whose K fits 9 slabs (3x3 convs over 64 or
  // 128 channels), im2col-fed, R2
  if (L.n_tiles == 1 && L.num_kb <= 9 && L.amode == A_IM2COL && L.epi == EPI_R2 && L.nplane == 1 &&
      ((L.bn == 64 && L.kb_bytes == 64) || (L.bn == 128 && L.kb_bytes == 128))) {
    if (L.bn == 64) return launch_one<64, 1, A_IM2COL, EPI_R2, 64, 9>(L, g, e, stream);
    return launch_one<128, 1, A_IM2COL, EPI_R2, 128, 9>(L, g, e, stream);
  }
  if (L.amode == A_SHIFT) {
    // shifted-patch convs: N tile 64 (or 128 over 128-byte slabs), resident B of at most 9 K slabs
    if (!(L.bn == 64 || (L.bn == 128 && L.kb_bytes == 128)) || L.nplane != 1 || L.num_kb > 9 ||
        !(L.n_tiles == 1 || L.n_tiles == 2 || L.n_tiles == 4))
      return set_error(NNRCU_ERR_INVALID, "shifted-patch conv: unsupported tiling (bn %d, %d K slabs, %d N tiles)", L.bn,
                       L.num_kb, L.n_tiles);
    if (L.bn == 128) {
      if (L.epi == EPI_R1) return launch_one<128, 1, A_SHIFT, EPI_R1, 128, 9>(L, g, e, stream);
      if (L.epi == EPI_R2) return launch_one<128, 1, A_SHIFT, EPI_R2, 128, 9>(L, g, e, stream);
    } else if (L.kb_bytes == 64) {
      if (L.epi == EPI_R1) return launch_one<64, 1, A_SHIFT, EPI_R1, 64, 9>(L, g, e, stream);
      if (L.epi == EPI_R2) return launch_one<64, 1, A_SHIFT, EPI_R2, 64, 9>(L, g, e, stream);
    } else if (L.kb_bytes == 128) {
      if (L.epi == EPI_R1) return launch_one<64, 1, A_SHIFT, EPI_R1, 128, 9>(L, g, e, stream);
      if (L.epi == EPI_R2) return launch_one<64, 1, A_SHIFT, EPI_R2, 128, 9>(L, g, e, stream);
    }
    return set_error(NNRCU_ERR_INVALID, "no shifted-patch instance for %d-byte slabs, epilogue %d", L.kb_bytes, L.epi);
  }
  if (L.epi == EPI_R2 && L.amode == A_TMA && e.qres && e.y_layout == 0 && (e.ldy & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(e.y) & 15) == 0 && (reinterpret_cast<uintptr_t>(e.qres) & 15) == 0)
    L2.epi = EPI_R2A;
  switch (L.bn) {
    case 64: return dispatch_bn<64>(L2, g, e, stream);
    case 128: return dispatch_bn<128>(L2, g, e, stream);
    case 256: return dispatch_bn<256>(L2, g, e, stream);
    default: return set_error(NNRCU_ERR_INVALID, "unsupported N tile %d", L.bn);
  }
}

int pick_bn(int M, int N, int nplane, int sms) {
  // Estimated time ~ waves * per-tile cost, with the per-tile cost linear in
  // BN plus a fixed overhead (prologue, epilogue drain) worth ~48 columns.
  const int cands[3] = {256, 128, 64};
  int best = 128;
  double best_cost = 1e30;
  const int mt = (M + BM - 1) / BM;
  for (int bn : cands) {
    if (nplane == 2 && bn == 256) continue;  // two stages only: keep 128 for split-bf16
    const int nt = (N + bn - 1) / bn;
    const long long tiles = (long long)mt * nt;
    const long long waves = (tiles + sms - 1) / sms;
    const double cost = (double)waves * (bn + 48);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

}  // namespace nnrcu
