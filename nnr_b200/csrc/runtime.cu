// Runtime part of the C ABI: errors, devices, streams, memory, graphs, the
// device status word and tensor-map encoding.
#include <cstdlib>
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.h"

namespace nnrcu {

namespace {
thread_local char g_err[512] = "";

// Status word that kernels set (first error wins) instead of trapping.
__device__ int g_status_word;

constexpr int kMaxDevices = 64;
int* g_status_addr[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};
std::mutex g_mu;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
PFN_cuTensorMapEncodeIm2col_v12000 g_encode_im2col = nullptr;
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return NNRCU_OK;
  if (e == cudaErrorMemoryAllocation) return set_error(NNRCU_ERR_NOMEM, "%s: %s", what, cudaGetErrorString(e));
  return set_error(NNRCU_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static int device_setup(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return set_error(NNRCU_ERR_INVALID, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status_addr[dev]) return NNRCU_OK;
  void* p = nullptr;
  NNRCU_CUDA(cudaGetSymbolAddress(&p, g_status_word));
  NNRCU_CUDA(cudaMemset(p, 0, sizeof(int)));
  int sms = 0;
  NNRCU_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int major = 0, minor = 0;
  NNRCU_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  NNRCU_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
  if (major != 10 || minor != 0)
    return set_error(NNRCU_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", dev,
                     major, minor);
  if (!g_encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    NNRCU_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn)
      return set_error(NNRCU_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    fn = nullptr;
    NNRCU_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn)
      return set_error(NNRCU_ERR_CUDA, "cuTensorMapEncodeIm2col entry point not found");
    g_encode_im2col = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(fn);
  }
  g_num_sms[dev] = sms;
  g_status_addr[dev] = static_cast<int*>(p);
  return NNRCU_OK;
}

static int current_device(int* dev) {
  NNRCU_CUDA(cudaGetDevice(dev));
  return device_setup(*dev);
}

int* status_ptr() {
  int dev = 0;
  if (current_device(&dev) != NNRCU_OK) return nullptr;
  return g_status_addr[dev];
}

int num_sms() {
  int dev = 0;
  if (current_device(&dev) != NNRCU_OK) return 148;
  return g_num_sms[dev];
}

bool pdl_enabled() {
  // programmatic dependent launch of the engine kernels; NNRCU_PDL=0 turns it off
  static const bool on = [] {
    const char* v = std::getenv("NNRCU_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool shift_enabled() {
  // shifted-patch mode for stride-1 spatial QLinearConvs; NNRCU_SHIFT=0 turns it off
  // (read when an operator is created)
  const char* v = std::getenv("NNRCU_SHIFT");
  return !(v && v[0] == '0');
}

bool xrows_enabled() {
  // space-to-depth convs as 64-byte kernel rows (A_XROWS); NNRCU_XROWS=0 keeps A_ROWS
  const char* v = std::getenv("NNRCU_XROWS");
  return !(v && v[0] == '0');
}

bool xrows_map_ok() {
  // whether the driver encodes a tensor map whose 64-byte rows are 16 bytes
  // apart (checked once per process on a scratch allocation)
  static int ok = -1;
  if (ok < 0) {
    void* p = nullptr;
    ok = 0;
    if (cudaMalloc(&p, 1 << 20) == cudaSuccess) {
      CUtensorMap m{};
      ok = encode_tmap_2d(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, p, 64, (1 << 16) - 3, 16, 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_64B) == NNRCU_OK;
      cudaFree(p);
    }
    (void)cudaGetLastError();
  }
  return ok == 1;
}

bool bimg_enabled() {
  // int8 engine: B from shared-memory images by plain bulk copies; NNRCU_BIMG=0 keeps the tensor-map loads
  const char* v = std::getenv("NNRCU_BIMG");
  return !(v && v[0] == '0');
}

bool r2_sat_enabled() {
  // R2 epilogue with y_zp = 0 as one saturating conversion; NNRCU_R2SAT=0 turns it off
  const char* v = std::getenv("NNRCU_R2SAT");
  return !(v && v[0] == '0');
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NNRCU_OK) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride_bytes & 15) != 0)
    return set_error(NNRCU_ERR_INVALID, "TMA operand must be 16-byte aligned (base %p, row stride %llu)", base,
                     (unsigned long long)row_stride_bytes);
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NNRCU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) dims %llu x %llu box %u x %u", (int)r,
                     (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
  return NNRCU_OK;
}

int encode_tmap_nd(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NNRCU_OK) return rc;
  if (rank < 1 || rank > 5 || (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(NNRCU_ERR_INVALID, "TMA operand: rank %d, base must be 16-byte aligned", rank);
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    estr[i] = 1;
    if (i < rank - 1) {
      if (strides_bytes[i] & 15) return set_error(NNRCU_ERR_INVALID, "TMA stride must be a multiple of 16 bytes");
      st[i] = strides_bytes[i];
    }
  }
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), d, st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(NNRCU_ERR_CUDA, "cuTensorMapEncodeTiled (%d-d) failed (%d)", rank, (int)r);
  return NNRCU_OK;
}

int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
                   const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swizzle) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NNRCU_OK) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (strides_bytes[0] & 15) != 0 || (strides_bytes[1] & 15) != 0)
    return set_error(NNRCU_ERR_INVALID, "TMA operand must be 16-byte aligned");
  const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  const cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
  const cuuint32_t b[3] = {box[0], box[1], box[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), d, st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(NNRCU_ERR_CUDA, "cuTensorMapEncodeTiled (3-d) failed (%d)", (int)r);
  return NNRCU_OK;
}

int encode_tmap_im2col(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, int n, int h,
                       int w, int c, int pt, int pl, int pb, int pr, int kh, int kw, int dh, int dw, int sh, int sw,
                       int kslab) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NNRCU_OK) return rc;
  const uint64_t row = (uint64_t)c * elem_bytes;
  // kslab: bytes of channels per pixel in one copy (128 / 64 with the
  // matching swizzle; 16 = one whole 16-byte pixel, unswizzled)
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (kslab != 128 && kslab != 64 && kslab != 16) || (row % kslab) != 0)
    return set_error(NNRCU_ERR_INVALID, "im2col operand must be 16-byte aligned with a channel stride in whole copies");
  const cuuint64_t dims[4] = {(cuuint64_t)c, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)n};
  const cuuint64_t strides[3] = {row, row * (uint64_t)w, row * (uint64_t)w * (uint64_t)h};
  const int lower[2] = {-pl, -pt};
  const int upper[2] = {pr - (kw - 1) * dw, pb - (kh - 1) * dh};
  const cuuint32_t estr[4] = {1, (cuuint32_t)sw, (cuuint32_t)sh, 1};
  CUresult r = g_encode_im2col(map, dtype, 4, const_cast<void*>(base), dims, strides, lower, upper,
                               (cuuint32_t)(kslab / elem_bytes), 128, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               kslab == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                            : (kslab == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE),
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(NNRCU_ERR_CUDA, "cuTensorMapEncodeIm2col failed (%d) n=%d h=%d w=%d c=%d", (int)r, n, h, w, c);
  return NNRCU_OK;
}

}  // namespace nnrcu

using namespace nnrcu;

extern "C" {

int nnrcu_init(int device) {
  int n = 0;
  NNRCU_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return set_error(NNRCU_ERR_INVALID, "device %d not present (%d devices)", device, n);
  NNRCU_CUDA(cudaSetDevice(device));
  return device_setup(device);
}

int nnrcu_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return NNRCU_ERR_INVALID;
  snprintf(buf, len, "%s", g_err);
  return NNRCU_OK;
}

int nnrcu_device_status(int* status_out) {
  if (!status_out) return set_error(NNRCU_ERR_INVALID, "status_out is NULL");
  int* p = status_ptr();
  if (!p) return NNRCU_ERR_CUDA;
  int v = 0;
  NNRCU_CUDA(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) NNRCU_CUDA(cudaMemset(p, 0, sizeof(int)));
  *status_out = v;
  return NNRCU_OK;
}

int nnrcu_stream_create(void** stream) {
  if (!stream) return set_error(NNRCU_ERR_INVALID, "stream is NULL");
  cudaStream_t s;
  NNRCU_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return NNRCU_OK;
}
int nnrcu_stream_destroy(void* stream) {
  NNRCU_CUDA(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
  return NNRCU_OK;
}
int nnrcu_stream_sync(void* stream) {
  NNRCU_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int st = 0;
  int rc = nnrcu_device_status(&st);
  if (rc != NNRCU_OK) return rc;
  if (st != 0) return set_error(NNRCU_ERR_DEVICE, "kernel reported device status %d", st);
  return NNRCU_OK;
}
int nnrcu_malloc(void** ptr, size_t bytes) {
  if (!ptr) return set_error(NNRCU_ERR_INVALID, "ptr is NULL");
  NNRCU_CUDA(cudaMalloc(ptr, bytes ? bytes : 1));
  return NNRCU_OK;
}
int nnrcu_free(void* ptr) {
  NNRCU_CUDA(cudaFree(ptr));
  return NNRCU_OK;
}
int nnrcu_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  NNRCU_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
  return NNRCU_OK;
}
int nnrcu_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  NNRCU_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
  return NNRCU_OK;
}
int nnrcu_memset(void* dst, int value, size_t bytes, void* stream) {
  NNRCU_CUDA(cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream)));
  return NNRCU_OK;
}
int nnrcu_host_register(void* ptr, size_t bytes) {
  if (!ptr || !bytes) return set_error(NNRCU_ERR_INVALID, "NULL or empty host buffer");
  const cudaError_t e = cudaHostRegister(ptr, bytes, cudaHostRegisterDefault);
  if (e == cudaErrorHostMemoryAlreadyRegistered) {
    (void)cudaGetLastError();
    return NNRCU_OK;
  }
  NNRCU_CUDA(e);
  return NNRCU_OK;
}
int nnrcu_host_unregister(void* ptr) {
  NNRCU_CUDA(cudaHostUnregister(ptr));
  return NNRCU_OK;
}
int nnrcu_graph_begin(void* stream) {
  NNRCU_CUDA(cudaStreamBeginCapture(static_cast<cudaStream_t>(stream), cudaStreamCaptureModeThreadLocal));
  return NNRCU_OK;
}
int nnrcu_graph_end(void* stream, void** graph_exec) {
  if (!graph_exec) return set_error(NNRCU_ERR_INVALID, "graph_exec is NULL");
  cudaGraph_t g;
  NNRCU_CUDA(cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &g));
  cudaGraphExec_t ge;
  cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  NNRCU_CUDA(e);
  *graph_exec = ge;
  return NNRCU_OK;
}
int nnrcu_graph_launch(void* graph_exec, void* stream) {
  NNRCU_CUDA(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), static_cast<cudaStream_t>(stream)));
  return NNRCU_OK;
}
int nnrcu_graph_destroy(void* graph_exec) {
  NNRCU_CUDA(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)));
  return NNRCU_OK;
}

int nnrcu_op_workspace_size(const nnrcu_op* op, size_t* bytes) {
  if (!op || !bytes) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  *bytes = op->ws_bytes;
  return NNRCU_OK;
}
int nnrcu_op_num_ops(const nnrcu_op* op, int64_t* ops) {
  if (!op || !ops) return set_error(NNRCU_ERR_INVALID, "NULL argument");
  *ops = op->num_ops;
  return NNRCU_OK;
}
int nnrcu_op_destroy(nnrcu_op* op) {
  if (!op) return NNRCU_OK;
  void* bufs[] = {op->wB, op->wBimg, op->colcorr, op->bias_i, op->cs_arr, op->bias_f, op->os, op->bias, op->cmat, op->w_dw};
  int rc = NNRCU_OK;
  for (void* b : bufs)
    if (b && cudaFree(b) != cudaSuccess) rc = set_error(NNRCU_ERR_CUDA, "cudaFree failed in nnrcu_op_destroy");
  delete op;
  return rc;
}

}  // extern "C"
