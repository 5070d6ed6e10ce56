// QLinearMatMul entry point that allocates no device memory.
//
// Who needs it: callers that must not call cudaMalloc at inference time, for
// example a host runtime whose device memory is fully reserved up front by
// another allocator, code that runs while a CUDA graph is being captured by
// someone else, or an embedding that forbids allocation after start-up. The
// regular QLinearMatMul (nnrcu_qlinearmatmul_create/_run) allocates the packed
// weights and zero-point sums when it is created; this variant instead takes
// the raw ONNX inputs on the device and keeps everything it derives from them
// in one file-scope device array of fixed size.
//
// The scratch array lives in every device that loads this library, for the
// life of the process. It is shared by all calls on a device and keeps the
// previous call's contents; each call rewrites every byte it later reads.
// Calls whose kernels overlap on the GPU (two streams, or concurrent host
// threads on one device) race on the array and must be serialised by the
// caller.
#include <mutex>

#include "internal.h"
#include "tc_gemm.cuh"

namespace nnrcu {
namespace {

constexpr size_t kScratchBytes = NNRCU_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDev = 64;
uint8_t* g_scratch_dev[kMaxDev] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array for the current device. The array's
// name in host code is only a stand-in for the symbol, so the address comes
// from cudaGetSymbolAddress, once per device, with that device current.
int scratch_address(uint8_t** out) {
  int dev = 0;
  NNRCU_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDev) return set_error(NNRCU_ERR_INVALID, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_dev[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(NNRCU_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch) failed: %s", cudaGetErrorString(e));
    g_scratch_dev[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch_dev[dev];
  return NNRCU_OK;
}

// bt[j][kk] = b[kk][j] for j < n, kk < k; zero in the padding, so the TMA
// tiles never read a previous call's bytes.
__global__ void noalloc_pack_bt(const int8_t* __restrict b, int k, int n, int kpad, int npad, int8_t* __restrict bt) {
  __shared__ int8_t tile[32][33];
  const int k0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int kk = k0 + i, j = j0 + threadIdx.x;
    tile[i][threadIdx.x] = (kk < k && j < n) ? b[(size_t)kk * n + j] : (int8_t)0;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int j = j0 + i, kk = k0 + threadIdx.x;
    if (j < npad && kk < kpad) bt[(size_t)j * kpad + kk] = tile[threadIdx.x][i];
  }
}

// colcorr[j] = -a_zp * sum_kk b[kk][j] + k * a_zp * b_zp (int32, wrapping).
__global__ void noalloc_colcorr(const int8_t* __restrict b, int k, int n, int a_zp, int b_zp, int32_t* __restrict out) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  int32_t s = 0;
  for (int kk = 0; kk < k; ++kk) s += b[(size_t)kk * n + j];
  out[j] = (int32_t)(0u - (uint32_t)a_zp * (uint32_t)s + (uint32_t)k * (uint32_t)a_zp * (uint32_t)b_zp);
}

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace
}  // namespace nnrcu

using namespace nnrcu;

extern "C" int nnrcu_qlinearmatmul_noalloc(const uint8_t* a, const int8_t* b, uint8_t* y, int m, int k, int n,
                                           float a_scale, uint8_t a_zp, float b_scale, int8_t b_zp, float y_scale,
                                           uint8_t y_zp, void* stream) {
  if (!a || !b || !y) return set_error(NNRCU_ERR_INVALID, "NULL tensor");
  if (m <= 0 || k <= 0 || n <= 0) return set_error(NNRCU_ERR_INVALID, "QLinearMatMul dims must be positive");
  if (k % 16 != 0) return set_error(NNRCU_ERR_INVALID, "no-alloc QLinearMatMul needs k %% 16 == 0 (k = %d)", k);
  if ((reinterpret_cast<uintptr_t>(a) & 15) != 0)
    return set_error(NNRCU_ERR_INVALID, "no-alloc QLinearMatMul needs a 16-byte aligned A");
  const int kpad = (k + BKB - 1) / BKB * BKB;
  const int npad = (n + 255) / 256 * 256;
  const size_t bt_bytes = align256((size_t)npad * kpad);
  const size_t col_bytes = align256((size_t)n * 4);
  const size_t row_bytes = b_zp != 0 ? align256((size_t)m * 4) : 0;
  const size_t need = bt_bytes + col_bytes + row_bytes;
  if (need > kScratchBytes)
    return set_error(NNRCU_ERR_INVALID,
                     "no-alloc QLinearMatMul needs %zu bytes of scratch for m=%d k=%d n=%d; the static limit is %zu "
                     "bytes (use nnrcu_qlinearmatmul_create/_run instead)",
                     need, m, k, n, kScratchBytes);

  // Everything that can fail runs before the first launch, so an error
  // return leaves the caller's stream untouched: the stream's device, the
  // per-device set-up (architecture check, status word), the scratch
  // address and both tensor maps.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (st != nullptr) {
    int cur = 0, sdev = 0;
    NNRCU_CUDA(cudaGetDevice(&cur));
    NNRCU_CUDA(cudaStreamGetDevice(st, &sdev));
    if (sdev != cur)
      return set_error(NNRCU_ERR_INVALID, "no-alloc QLinearMatMul: the stream belongs to device %d, the current device is %d",
                       sdev, cur);
  }
  int* status = status_ptr();
  if (!status) return NNRCU_ERR_CUDA;
  uint8_t* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != NNRCU_OK) return rc;
  int8_t* bt = reinterpret_cast<int8_t*>(scratch);
  int32_t* colcorr = reinterpret_cast<int32_t*>(scratch + bt_bytes);
  int32_t* rowcorr = b_zp != 0 ? reinterpret_cast<int32_t*>(scratch + bt_bytes + col_bytes) : nullptr;

  const int bn = pick_bn(m, n, 1, num_sms());
  const int amode = k >= BKB ? A_TMA : A_GATHER;
  CUtensorMap tmA{}, tmB{};
  rc = encode_tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, bt, kpad, npad, kpad, BKB, bn);
  if (rc != NNRCU_OK) return rc;
  if (amode == A_TMA) {
    rc = encode_tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, k, (uint64_t)m, k, BKB, BM);
    if (rc != NNRCU_OK) return rc;
  }

  dim3 tgrid(kpad / 32, npad / 32), tblock(32, 8);
  noalloc_pack_bt<<<tgrid, tblock, 0, st>>>(b, k, n, kpad, npad, bt);
  NNRCU_CUDA(cudaGetLastError());
  noalloc_colcorr<<<(n + 255) / 256, 256, 0, st>>>(b, k, n, a_zp, b_zp, colcorr);
  NNRCU_CUDA(cudaGetLastError());
  if (rowcorr) {
    rc = launch_rowcorr_u8(a, m, k, k, b_zp, rowcorr, st);
    if (rc != NNRCU_OK) return rc;
  }

  GatherGeom g{};
  g.x = a;
  g.N = 1; g.H = 1; g.W = m;
  g.cbytes = k;
  g.OH = 1; g.OW = m; g.KH = 1; g.KW = 1; g.sh = 1; g.sw = 1; g.ph = 0; g.pw = 0; g.dh = 1; g.dw = 1;
  g.kbytes = k;
  EpiParams e{};
  e.M = m; e.N = n;
  e.colcorr = colcorr;
  e.rowcorr = rowcorr;
  e.combined = a_scale * b_scale / y_scale;  // QLinearMatMul.cpp:134
  e.yzp_f = (float)y_zp;
  e.y = y;
  e.y_layout = 0;
  e.ldy = n;
  e.ohw = 1;
  e.status = status;
  TcLaunch L{};
  L.bn = bn; L.nplane = 1; L.amode = amode; L.epi = EPI_R4;
  L.m_tiles = (m + BM - 1) / BM;
  L.n_tiles = (n + bn - 1) / bn;
  L.tmA0 = &tmA; L.tmA1 = &tmA; L.tmB = &tmB;
  L.b_plane_rows = npad;
  L.num_kb = kpad / BKB;
  return tc_launch(L, g, e, st);
}
