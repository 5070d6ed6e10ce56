// The CUDA operators of nnr's backend_t::CUDA and their registration.
//
// Each class mirrors the attributes and shape rules of nnr's CPU operator of
// the same op_type (cited per class) and runs on the device through
// libnnrcu's C ABI; see cuda_backend.h for residency, layouts and graphs.
#include <cfloat>
#include <cmath>
#include <cstring>

#include "backend/cpu/conv_shape.h"
#include "cpu_features.h"
#include "cuda_backend.h"

namespace nnr::cuda {

namespace {

constexpr uint8_t LAYOUT_DEVICE = LAYOUT_NCHW | LAYOUT_NHWC;

int to_nnrcu(memory_layout_t l) { return l == memory_layout_t::NHWC ? NNRCU_LAYOUT_NHWC : NNRCU_LAYOUT_NCHW; }

// 16-bit tensors: the nnrcu dtype, or 0 for other types
int half_dtype(data_type_t t) {
  return t == NNR_DATA_TYPE_BFLOAT16 ? NNRCU_DT_BF16 : (t == NNR_DATA_TYPE_FLOAT16 ? NNRCU_DT_F16 : 0);
}

bool is_const_tensor(context_t* ctx, const tensor_t* t) {
  if (!t) return false;
  if (ctx->initializer_names.count(t->name)) return true;
  for (auto* nd : ctx->graph->nodes)
    if (nd->folded)
      for (auto* o : nd->outputs)
        if (o == t) return true;
  return false;
}

// The fused post-op of a Conv/Gemm/MatMul (fuse_post_ops.cpp:69-71 sets
// post_fn and fused_op) as the device epilogue's enum and parameters.
bool post_op_of(const operator_t* op, int* kind, float* a, float* b) {
  *kind = NNRCU_POST_NONE;
  *a = 0.0f;
  *b = 0.0f;
  if (!op->post_fn || !op->fused_op) return true;
  operator_t* f = op->fused_op;
  const std::string_view t = f->op_type;
  if (t == "Relu") {
    *kind = NNRCU_POST_RELU;
  } else if (t == "Clip") {  // Clip.cpp:20-40: min/max from inputs 1 and 2, else unbounded
    *kind = NNRCU_POST_CLIP;
    *a = f->inputs.size() > 1 && f->inputs[1] ? scalar_f32(f->inputs[1], -FLT_MAX) : -FLT_MAX;
    *b = f->inputs.size() > 2 && f->inputs[2] ? scalar_f32(f->inputs[2], FLT_MAX) : FLT_MAX;
  } else if (t == "HardSwish") {
    *kind = NNRCU_POST_HARDSWISH;
  } else if (t == "Sigmoid") {
    *kind = NNRCU_POST_SIGMOID;
  } else if (t == "LeakyRelu") {
    *kind = NNRCU_POST_LEAKYRELU;
    *a = f->attribute(attr_key_t::alpha, 0.01f);
  } else if (t == "Tanh") {
    *kind = NNRCU_POST_TANH;
  } else {
    return false;
  }
  return true;
}

// ------------------------------------------------------------------ convolution attributes
// Conv.cpp:124-149 and QLinearConv's init parse the same attributes.
struct conv_attrs_t {
  int auto_pad = 0;
  int group = 1;
  std::vector<int64_t> kernels, dilations, pads, strides;

  void parse(operator_t* op) {
    const std::string_view ap = op->attribute(attr_key_t::auto_pad, "NOTSET");
    auto_pad = ap == "SAME_UPPER" ? 1 : ap == "SAME_LOWER" ? 2 : ap == "VALID" ? 3 : 0;
    group = op->attribute(attr_key_t::group, (int32_t)1);
    ints_attr(op, attr_key_t::kernel_shape, kernels);
    std::vector<int64_t> v;
    ints_attr(op, attr_key_t::dilations, v);
    dilations.assign(2, 1);
    for (size_t i = 0; i < v.size() && i < 2; ++i) dilations[i] = v[i];
    ints_attr(op, attr_key_t::pads, v);
    pads.assign(4, 0);
    for (size_t i = 0; i < v.size() && i < 4; ++i) pads[i] = v[i];
    ints_attr(op, attr_key_t::strides, v);
    strides.assign(2, 1);
    for (size_t i = 0; i < v.size() && i < 2; ++i) strides[i] = v[i];
  }

  // output dims and resolved pads through nnr's own shape helper
  // (backend/cpu/conv_shape.h:21-79)
  bool out_dims(const tensor_t* x, const tensor_t* w, int* dims, int* cpads) {
    if (!x || !w || x->ndim != 4 || w->ndim != 4) return false;
    int k[2] = {w->dims[2], w->dims[3]};
    if (kernels.size() == 2) k[0] = (int)kernels[0], k[1] = (int)kernels[1];
    int d[2] = {(int)dilations[0], (int)dilations[1]};
    int s[2] = {(int)strides[0], (int)strides[1]};
    int p[4] = {(int)pads[0], (int)pads[1], (int)pads[2], (int)pads[3]};
    compute_conv_output_shape(auto_pad, x->dims, 4, w->dims[0], k, 2, d, s, p, cpads, dims);
    return dims[2] > 0 && dims[3] > 0;
  }

  nnrcu_conv_desc desc(const tensor_t* x, const tensor_t* w, const int* cpads) const {
    nnrcu_conv_desc dd{};
    dd.n = x->dims[0];
    dd.c = x->dims[1];
    dd.h = x->dims[2];
    dd.w = x->dims[3];
    dd.oc = w->dims[0];
    dd.kh = w->dims[2];
    dd.kw = w->dims[3];
    dd.group = group;
    dd.stride_h = (int)strides[0];
    dd.stride_w = (int)strides[1];
    dd.pad_top = cpads[0];
    dd.pad_left = cpads[1];
    dd.pad_bottom = cpads[2];
    dd.pad_right = cpads[3];
    dd.dil_h = (int)dilations[0];
    dd.dil_w = (int)dilations[1];
    return dd;
  }
};

// Device layout cost in nnr's "effective bytes" (layout_cost.h): the device
// kernels read and write NHWC natively; an NCHW boundary costs them an
// input and an output reorder, priced like nnr's reorder_cost (2.5x bytes).
float device_layout_cost(memory_layout_t layout, float x_bytes, float w_bytes, float y_bytes) {
  const float base = x_bytes + w_bytes + y_bytes;
  if (layout == memory_layout_t::NHWC) return base;
  if (layout == memory_layout_t::NCHW) return base + 2.5f * (x_bytes + y_bytes);
  return 1e30f;  // channel-blocked layouts are not device layouts
}

struct op_holder_t {
  nnrcu_op* op = nullptr;
  ~op_holder_t() { reset(); }
  void reset() {
    if (op) nnrcu_op_destroy(op);
    op = nullptr;
  }
  size_t ws() const {
    size_t b = 0;
    if (op) nnrcu_op_workspace_size(op, &b);
    return b;
  }
};

// ------------------------------------------------------------------ QLinearConv
// QLinearConv_operator (backend/cpu/QLinearConv.cpp, QLinearConv_reshape.h:
// 18-340): x u8, w s8 (fuse_qdq_compute converts u8 weights), per-tensor or
// per-channel w_scale, zero w_zp, optional int32 bias. The requant formula
// is the one nnr's dispatch picks for the layouts nnr assigned
// (NNRCU_RQ_AUTO: R3 for the stem, R1 for small NCHW outputs, R2 for NHWC).
struct QLinearConv_cuda : cuda_op_t {
  conv_attrs_t a;
  int cpads[4] = {};
  op_holder_t h;

  bool init() override {
    if (inputs.size() < 8 || outputs.size() != 1) return false;
    a.parse(this);
    layout_mask = LAYOUT_DEVICE;
    return true;
  }
  bool infer_shape() override {
    int dims[4];
    if (!a.out_dims(inputs[0], inputs[3], dims, cpads)) return false;
    return outputs[0]->reshape({dims, 4}, NNR_DATA_TYPE_UINT8);
  }
  int64_t num_ops() const override {
    const tensor_t *w = inputs[3], *y = outputs[0];
    return 2LL * y->ndata * w->dims[1] * w->dims[2] * w->dims[3];
  }
  float layout_cost(memory_layout_t layout, bool) const override {
    const tensor_t *x = inputs[0], *w = inputs[3], *y = outputs[0];
    return device_layout_cost(layout, (float)x->ndata, (float)w->ndata, (float)y->ndata);
  }
  bool device_ok() const override {
    // u8 activations, s8 weights, fp32 scales (s8 activations and other
    // scale types are declined: nnr's arithmetic differs there)
    return inputs[0]->type == NNR_DATA_TYPE_UINT8 && inputs[3]->type == NNR_DATA_TYPE_INT8 && inputs[0]->ndim == 4 &&
           inputs[1]->type == NNR_DATA_TYPE_FLOAT32 && inputs[4]->type == NNR_DATA_TYPE_FLOAT32 &&
           inputs[6]->type == NNR_DATA_TYPE_FLOAT32;
  }
  bool prepare_device(device_state_t& s) override {
    tensor_t *x = inputs[0], *w = inputs[3], *y = outputs[0];
    nnrcu_conv_desc d = a.desc(x, w, cpads);
    d.in_layout = to_nnrcu(in_layout(s, x));
    d.out_layout = to_nnrcu(y->format);
    d.post_op = post_fn ? NNRCU_POST_RELU : NNRCU_POST_NONE;  // qmin = max(lo, y_zp), QLinearConv.cpp:419
    d.requant = NNRCU_RQ_AUTO;
    const tensor_t *ws = inputs[4], *wzp = inputs[5];
    const tensor_t* bias = inputs.size() > 8 ? inputs[8] : nullptr;
    if (ws->type != NNR_DATA_TYPE_FLOAT32) return s.fail("QLinearConv: w_scale must be fp32");
    if (wzp && wzp->type != NNR_DATA_TYPE_INT8 && wzp->ndata > 0)
      return s.fail("QLinearConv: w_zp must be int8 (symmetric weights)");
    if (bias && bias->type != NNR_DATA_TYPE_INT32) return s.fail("QLinearConv: bias must be int32");
    h.reset();
    const int rc = nnrcu_qlinearconv_create(
        &d, (const int8_t*)w->data, (const float*)ws->data, (int)ws->ndata, wzp ? (const int8_t*)wzp->data : nullptr,
        wzp ? (int)wzp->ndata : 0, bias ? (const int32_t*)bias->data : nullptr, scalar_f32(inputs[1], 1.0f),
        (uint8_t)scalar_zp(inputs[2]), scalar_f32(inputs[6], 1.0f), (uint8_t)scalar_zp(inputs[7]), &h.op);
    if (!nnrcu_ok(s, rc, "QLinearConv")) return false;
    set_out_layout(s, y, y->format);
    return true;
  }
  size_t device_workspace() const override { return h.ws(); }
  bool run_device(device_state_t& s, void* stream) override {
    return nnrcu_ok(s,
                    nnrcu_qlinearconv_run(h.op, (const uint8_t*)s.dev(inputs[0]), (uint8_t*)s.dev(outputs[0]),
                                          s.workspace, stream),
                    "QLinearConv");
  }
};

// ------------------------------------------------------------------ Conv (fp32, bf16, fp16)
// Conv_operator (backend/cpu/Conv.cpp, Conv_reshape.h:17-380,
// Conv_exec.h:1163-1192): fp32 dense convs as split-bf16 on the tensor cores,
// depthwise on CUDA cores; bias and the fused post-op in the epilogue.
// bf16 / fp16 tensors (Conv_exec_entry.h:188-381: convert, fp32 conv, round
// back) run on one 16-bit plane (dense convs only).
struct Conv_cuda : cuda_op_t {
  conv_attrs_t a;
  int cpads[4] = {};
  op_holder_t h;

  bool init() override {
    if (inputs.size() < 2 || outputs.size() != 1) return false;
    a.parse(this);
    layout_mask = LAYOUT_DEVICE;
    return true;
  }
  bool infer_shape() override {
    int dims[4];
    if (!a.out_dims(inputs[0], inputs[1], dims, cpads)) return false;
    return outputs[0]->reshape({dims, 4}, inputs[0]->type);
  }
  int64_t num_ops() const override {
    const tensor_t *w = inputs[1], *y = outputs[0];
    return 2LL * y->ndata * w->dims[1] * w->dims[2] * w->dims[3];
  }
  float layout_cost(memory_layout_t layout, bool) const override {
    const tensor_t *x = inputs[0], *w = inputs[1], *y = outputs[0];
    return device_layout_cost(layout, 4.0f * x->ndata, 4.0f * w->ndata, 4.0f * y->ndata);
  }
  bool device_ok() const override {
    const data_type_t t = inputs[0]->type;
    const bool half = half_dtype(t) != 0;
    if (!(t == NNR_DATA_TYPE_FLOAT32 || half)) return false;
    return inputs[0]->ndim == 4 && inputs[1]->type == t && is_const_tensor(ctx, inputs[1]) &&
           (inputs.size() < 3 || !inputs[2] || (is_const_tensor(ctx, inputs[2]) && inputs[2]->type == t));
  }
  bool prepare_device(device_state_t& s) override {
    tensor_t *x = inputs[0], *w = inputs[1], *y = outputs[0];
    const tensor_t* b = inputs.size() > 2 ? inputs[2] : nullptr;
    nnrcu_conv_desc d = a.desc(x, w, cpads);
    d.in_layout = to_nnrcu(in_layout(s, x));
    d.out_layout = to_nnrcu(y->format);
    if (!post_op_of(this, &d.post_op, &d.post_a, &d.post_b))
      return s.fail("Conv: fused post-op %.*s has no device epilogue", (int)fused_op->op_type.size(),
                    fused_op->op_type.data());
    h.reset();
    dtype = half_dtype(x->type);
    const int rc = dtype ? nnrcu_conv_half_create(&d, dtype, (const uint16_t*)w->data,
                                                  b ? (const uint16_t*)b->data : nullptr, &h.op)
                         : nnrcu_conv_f32_create(&d, (const float*)w->data, b ? (const float*)b->data : nullptr, &h.op);
    if (!nnrcu_ok(s, rc, "Conv")) return false;
    set_out_layout(s, y, y->format);
    return true;
  }
  size_t device_workspace() const override { return h.ws(); }
  bool run_device(device_state_t& s, void* stream) override {
    if (dtype)
      return nnrcu_ok(s,
                      nnrcu_conv_half_run(h.op, (const uint16_t*)s.dev(inputs[0]), (uint16_t*)s.dev(outputs[0]),
                                          s.workspace, stream),
                      "Conv");
    return nnrcu_ok(s,
                    nnrcu_conv_f32_run(h.op, (const float*)s.dev(inputs[0]), (float*)s.dev(outputs[0]), nullptr,
                                       s.workspace, stream),
                    "Conv");
  }
  int dtype = 0;
};

// ------------------------------------------------------------------ Gemm / MatMul (fp32, bf16, fp16)
// Gemm_operator (backend/cpu/Gemm.cpp:40-294) with B (and C) initializers;
// MatMul_operator (backend/cpu/MatMul.cpp:13-228) with a constant 2-D B, the
// leading dims of A folded into M (:156-172). bf16 / fp16 Gemm/MatMul run on
// one 16-bit plane (Gemm.cpp:297-513; alpha 1). An fp32 MatMul follows the
// precision nnr's own dispatch gives it on this host: with AVX-512 BF16 and a
// constant B, bf16-rounded operands (MatMul.cpp:128-152, :424-428), else
// fp32 (split-bf16). Unlike that nnr path, a fused post-op is applied.
struct Gemm_cuda : cuda_op_t {
  bool matmul = false;
  float alpha = 1.0f, beta = 1.0f;
  int trans_a = 0, trans_b = 0;
  int M = 0, N = 0, K = 0;
  op_holder_t h;

  bool init() override {
    if (inputs.size() < 2 || outputs.size() != 1) return false;
    matmul = op_type == "MatMul";
    if (!matmul) {
      alpha = attribute(attr_key_t::alpha, 1.0f);
      beta = attribute(attr_key_t::beta, 1.0f);
      trans_a = attribute(attr_key_t::transA, (int32_t)0);
      trans_b = attribute(attr_key_t::transB, (int32_t)0);
    }
    layout_mask = LAYOUT_NCHW;
    return true;
  }
  // MatMul whose B is computed at run time (or batched): nnr's shapes and
  // broadcast strides (MatMul.cpp:32-94), one offset pair per output batch
  bool dyn = false;
  int dm = 0, dn = 0, dk = 0;
  std::vector<std::pair<long long, long long>> offs;
  size_t dws = 0;
  int dpost = 0;
  float dpa = 0, dpb = 0;
  bool infer_dynamic() {
    const tensor_t *A = inputs[0], *B = inputs[1];
    std::vector<int> ad(A->dims, A->dims + A->ndim), bd(B->dims, B->dims + B->ndim);
    if (A->ndim == 1) ad = {1, A->dims[0]};
    if (B->ndim == 1) bd = {B->dims[0], 1};
    if (ad.size() < 2 || bd.size() < 2 || ad.back() != bd[bd.size() - 2]) return false;
    const int nd = (int)std::max(ad.size(), bd.size()), nb = nd - 2;
    std::vector<int> dims(nd);
    dm = ad[ad.size() - 2], dk = ad.back(), dn = bd.back();
    dims[nd - 2] = dm, dims[nd - 1] = dn;
    for (int i = 3; i <= nd; ++i) {
      const int ai = (int)ad.size() - i, bi = (int)bd.size() - i;
      const int al = ai < 0 ? 1 : ad[ai], bl = bi < 0 ? 1 : bd[bi];
      if (al != bl && al > 1 && bl > 1) return false;
      dims[nd - i] = std::max(al, bl);
    }
    std::vector<long long> as(nb, 0), bs(nb, 0);
    long long sa = (long long)dm * dk, sb = (long long)dk * dn;
    for (int i = nb - 1; i >= 0; --i) {
      const int ai = i - (nb - ((int)ad.size() - 2)), bi = i - (nb - ((int)bd.size() - 2));
      if (ai >= 0 && ad[ai] > 1) as[i] = sa, sa *= ad[ai];
      if (bi >= 0 && bd[bi] > 1) bs[i] = sb, sb *= bd[bi];
    }
    long long total = 1;
    for (int i = 0; i < nb; ++i) total *= dims[i];
    offs.clear();
    std::vector<int> idx(nb, 0);
    for (long long t = 0; t < total; ++t) {
      long long ao = 0, bo = 0;
      for (int i = 0; i < nb; ++i) ao += idx[i] * as[i], bo += idx[i] * bs[i];
      offs.emplace_back(ao, bo);
      for (int i = nb - 1; i >= 0; --i) {
        if (++idx[i] < dims[i]) break;
        idx[i] = 0;
      }
    }
    M = dm, N = dn, K = dk;
    return outputs[0]->reshape({dims.data(), (size_t)nd}, A->type);
  }
  bool device_input(int idx) const override { return idx == 0 || (dyn && idx == 1); }
  bool infer_shape() override {
    const tensor_t *A = inputs[0], *B = inputs[1];
    dyn = matmul && !(B->ndim == 2 && A->ndim >= 2 && is_const_tensor(ctx, B));
    if (dyn) return infer_dynamic();
    if (B->ndim != 2 || A->ndim < 2) return false;
    if (matmul) {
      K = A->dims[A->ndim - 1];
      M = (int)(A->ndata / std::max(K, 1));
      N = B->dims[1];
      if (B->dims[0] != K) return false;
      int dims[MAX_NDIM];
      for (int i = 0; i < A->ndim - 1; ++i) dims[i] = A->dims[i];
      dims[A->ndim - 1] = N;
      return outputs[0]->reshape({dims, (size_t)A->ndim}, A->type);
    }
    if (A->ndim != 2) return false;
    M = trans_a ? A->dims[1] : A->dims[0];
    K = trans_a ? A->dims[0] : A->dims[1];
    N = trans_b ? B->dims[0] : B->dims[1];
    const int dims[2] = {M, N};
    return outputs[0]->reshape({dims, 2}, A->type);
  }
  int64_t num_ops() const override { return 2LL * M * N * K * (dyn ? (int64_t)offs.size() : 1); }
  bool device_ok() const override {
    const data_type_t t = inputs[0]->type;
    if (dyn) return (t == NNR_DATA_TYPE_FLOAT32 || half_dtype(t) != 0) && inputs[1]->type == t;
    const bool half = half_dtype(t) != 0;
    if (!(t == NNR_DATA_TYPE_FLOAT32 || (half && alpha == 1.0f && !trans_a)) || inputs[1]->type != t ||
        !is_const_tensor(ctx, inputs[1]))
      return false;
    if (!matmul && inputs.size() > 2 && inputs[2] && (!is_const_tensor(ctx, inputs[2]) || inputs[2]->type != t))
      return false;
    return true;
  }
  bool prepare_device(device_state_t& s) override {
    if (dyn) {
      if (!post_op_of(this, &dpost, &dpa, &dpb)) return s.fail("MatMul: fused post-op has no device epilogue");
      dtype = half_dtype(inputs[0]->type);
      if (!nnrcu_ok(s, dtype ? nnrcu_matmul_half_workspace(dm, dn, dk, &dws) : nnrcu_matmul_f32_workspace(dm, dn, dk, &dws),
                    "MatMul"))
        return false;
      set_out_layout(s, outputs[0], memory_layout_t::NCHW);
      return true;
    }
    const tensor_t* C = !matmul && inputs.size() > 2 ? inputs[2] : nullptr;
    std::vector<float> crow;
    const float* c = nullptr;
    int c_rows = 0;
    if (C && C->ndata > 0 && !half_dtype(inputs[0]->type)) {  // (16-bit C is handled below)
      if (C->ndata == (size_t)N) {
        c = (const float*)C->data, c_rows = 1;
      } else if (C->ndata == (size_t)M * N) {
        c = (const float*)C->data, c_rows = M;
      } else if (C->ndata == 1) {
        crow.assign(N, *(const float*)C->data);
        c = crow.data(), c_rows = 1;
      } else {
        return s.fail("Gemm: C of %zu elements does not broadcast to [%d, %d]", C->ndata, M, N);
      }
    }
    int post = 0;
    float pa = 0, pb = 0;
    if (!post_op_of(this, &post, &pa, &pb)) return s.fail("Gemm/MatMul: fused post-op has no device epilogue");
    h.reset();
    dtype = half_dtype(inputs[0]->type);
    if (dtype) {
      const tensor_t* Ch = !matmul && inputs.size() > 2 ? inputs[2] : nullptr;
      int rows = 0;
      if (Ch && Ch->ndata > 0) rows = Ch->ndata == (size_t)N ? 1 : (Ch->ndata == (size_t)M * N ? M : -1);
      if (rows < 0) return s.fail("Gemm: 16-bit C must be a [n] row or a full [m, n] matrix");
      if (!nnrcu_ok(s,
                    nnrcu_gemm_half_create(M, N, K, trans_a, trans_b, 1.0f, rows ? beta : 0.0f, dtype,
                                           (const uint16_t*)inputs[1]->data,
                                           rows ? (const uint16_t*)Ch->data : nullptr, rows, post, pa, pb, &h.op),
                    "Gemm"))
        return false;
      set_out_layout(s, outputs[0], memory_layout_t::NCHW);
      return true;
    }
    const int prec = matmul && has_avx512_bf16() ? NNRCU_PREC_BF16 : NNRCU_PREC_SPLIT_BF16;
    if (!nnrcu_ok(s,
                  nnrcu_gemm_f32_create_ex(M, N, K, trans_a, trans_b, alpha, c ? beta : 0.0f,
                                           (const float*)inputs[1]->data, c, c_rows, post, pa, pb, prec, &h.op),
                  "Gemm"))
      return false;
    set_out_layout(s, outputs[0], memory_layout_t::NCHW);
    return true;
  }
  size_t device_workspace() const override { return dyn ? dws : h.ws(); }
  bool run_device(device_state_t& s, void* stream) override {
    if (dyn) {
      // runs of output batches whose A and B offsets advance by fixed strides: one call each
      const float* a = (const float*)s.dev(inputs[0]);
      const float* b = (const float*)s.dev(inputs[1]);
      float* y = (float*)s.dev(outputs[0]);
      size_t i = 0;
      while (i < offs.size()) {
        size_t j = i + 1;
        const long long sa = j < offs.size() ? offs[j].first - offs[i].first : 0;
        const long long sb = j < offs.size() ? offs[j].second - offs[i].second : 0;
        while (j < offs.size() && sa >= 0 && sb >= 0 && offs[j].first - offs[j - 1].first == sa &&
               offs[j].second - offs[j - 1].second == sb)
          ++j;
        int rc;
        if (dtype) {
          const uint16_t* ah = (const uint16_t*)s.dev(inputs[0]);
          const uint16_t* bh = (const uint16_t*)s.dev(inputs[1]);
          rc = nnrcu_matmul_half_run(ah + offs[i].first, bh + offs[i].second,
                                     (uint16_t*)s.dev(outputs[0]) + i * (size_t)dm * dn, (int)(j - i), dm, dn, dk, sa,
                                     sb, dtype, dpost, dpa, dpb, s.workspace, dws, stream);
        } else {
          rc = nnrcu_matmul_f32_run(a + offs[i].first, b + offs[i].second, y + i * (size_t)dm * dn, (int)(j - i), dm,
                                    dn, dk, sa, sb, dpost, dpa, dpb, s.workspace, dws, stream);
        }
        if (!nnrcu_ok(s, rc, "MatMul")) return false;
        i = j;
      }
      return true;
    }
    if (dtype)
      return nnrcu_ok(s,
                      nnrcu_gemm_half_run(h.op, (const uint16_t*)s.dev(inputs[0]), (uint16_t*)s.dev(outputs[0]),
                                          s.workspace, stream),
                      "Gemm");
    return nnrcu_ok(s,
                    nnrcu_gemm_f32_run(h.op, (const float*)s.dev(inputs[0]), (float*)s.dev(outputs[0]),
                                       s.workspace, stream),
                    "Gemm");
  }
  int dtype = 0;
};

// ------------------------------------------------------------------ QLinearMatMul
// QLinearMatMul_operator (backend/cpu/QLinearMatMul.cpp:33-232): a u8
// [..., k], a constant s8 B [k, n] with a per-tensor scale, R4 requant.
struct QLinearMatMul_cuda : cuda_op_t {
  int M = 0, K = 0, N = 0;
  op_holder_t h;

  bool init() override {
    if (inputs.size() != 8 || outputs.size() != 1) return false;
    layout_mask = LAYOUT_NCHW;
    return true;
  }
  bool infer_shape() override {
    const tensor_t *A = inputs[0], *B = inputs[3];
    if (B->ndim != 2 || A->ndim < 1) return false;
    K = A->dims[A->ndim - 1];
    if (B->dims[0] != K) return false;
    N = B->dims[1];
    M = (int)(A->ndata / std::max(K, 1));
    int dims[MAX_NDIM];
    for (int i = 0; i < A->ndim - 1; ++i) dims[i] = A->dims[i];
    dims[A->ndim - 1] = N;
    return outputs[0]->reshape({dims, (size_t)A->ndim}, NNR_DATA_TYPE_UINT8);
  }
  int64_t num_ops() const override { return 2LL * M * N * K; }
  bool device_ok() const override {
    // u8 output from u8 x s8 with fp32 scales: the R4 path. nnr computes the
    // combined scale in fp16 for fp16 scales (QLinearMatMul.cpp:123-133) and
    // has an s8-output branch (:185-196); both are declined.
    return inputs[0]->type == NNR_DATA_TYPE_UINT8 && inputs[3]->type == NNR_DATA_TYPE_INT8 &&
           is_const_tensor(ctx, inputs[3]) && inputs[4]->ndata == 1 && inputs[1]->type == NNR_DATA_TYPE_FLOAT32 &&
           inputs[4]->type == NNR_DATA_TYPE_FLOAT32 && inputs[6]->type == NNR_DATA_TYPE_FLOAT32 &&
           outputs[0]->type == NNR_DATA_TYPE_UINT8;
  }
  bool prepare_device(device_state_t& s) override {
    h.reset();
    const int rc = nnrcu_qlinearmatmul_create(M, K, N, scalar_f32(inputs[1], 1.0f), (uint8_t)scalar_zp(inputs[2]),
                                              (const int8_t*)inputs[3]->data, scalar_f32(inputs[4], 1.0f),
                                              (int8_t)scalar_zp(inputs[5]), scalar_f32(inputs[6], 1.0f),
                                              (uint8_t)scalar_zp(inputs[7]), &h.op);
    if (!nnrcu_ok(s, rc, "QLinearMatMul")) return false;
    set_out_layout(s, outputs[0], memory_layout_t::NCHW);
    return true;
  }
  size_t device_workspace() const override { return h.ws(); }
  bool run_device(device_state_t& s, void* stream) override {
    return nnrcu_ok(s,
                    nnrcu_qlinearmatmul_run(h.op, (const uint8_t*)s.dev(inputs[0]), (uint8_t*)s.dev(outputs[0]),
                                            s.workspace, stream),
                    "QLinearMatMul");
  }
};

// ------------------------------------------------------------------ elementwise glue
// Elementwise operators keep their input's layout (memory order), as nnr's
// LAYOUT_ALL operators do on the host; they may fall back to nnr's CPU
// operator for variants the device kernels do not cover.

// QuantizeLinear (backend/cpu/QuantizeLinear.cpp:128-161): fp32 -> u8,
// per-tensor scale and zero point; the 16-wide body / scalar tail split is by
// flat index, so the kernel walks the tensor in memory order.
struct QuantizeLinear_cuda : cuda_op_t {
  bool init() override {
    if (inputs.size() < 2 || outputs.size() != 1) return false;
    layout_mask = LAYOUT_ALL;
    return true;
  }
  bool infer_shape() override {
    const tensor_t* zp = inputs.size() > 2 ? inputs[2] : nullptr;
    const data_type_t t = zp && zp->type == NNR_DATA_TYPE_INT8 ? NNR_DATA_TYPE_INT8 : NNR_DATA_TYPE_UINT8;
    return outputs[0]->reshape_identity(inputs[0], t);
  }
  bool host_allowed() const override { return true; }
  bool device_ok() const override {
    const tensor_t* zp = inputs.size() > 2 ? inputs[2] : nullptr;
    return inputs[0]->type == NNR_DATA_TYPE_FLOAT32 && inputs[1]->ndata == 1 &&
           (!zp || (zp->type == NNR_DATA_TYPE_UINT8 && zp->ndata == 1)) && inputs[0]->ndata < (1u << 31);
  }
  bool prepare_device(device_state_t& s) override {
    set_out_layout(s, outputs[0], in_layout(s, inputs[0]));
    return true;
  }
  bool run_device(device_state_t& s, void* stream) override {
    const int total = (int)inputs[0]->ndata;
    const tensor_t* zp = inputs.size() > 2 ? inputs[2] : nullptr;
    return nnrcu_ok(s,
                    nnrcu_quantize_linear_u8((const float*)s.dev(inputs[0]), (uint8_t*)s.dev(outputs[0]), 1, 1, 1,
                                             total, scalar_f32(inputs[1], 1.0f), (uint8_t)scalar_zp(zp),
                                             NNRCU_LAYOUT_NCHW, 0, stream),
                    "QuantizeLinear");
  }
};

// DequantizeLinear (backend/cpu/DequantizeLinear.cpp:135-160) of a u8
// activation with a per-tensor scale. Weight and bias DequantizeLinear
// nodes are constant-folded at load time on the host.
struct DequantizeLinear_cuda : cuda_op_t {
  bool init() override {
    if (inputs.size() < 2 || outputs.size() != 1) return false;
    layout_mask = LAYOUT_ALL;
    return true;
  }
  bool infer_shape() override { return outputs[0]->reshape_identity(inputs[0], NNR_DATA_TYPE_FLOAT32); }
  bool host_allowed() const override { return true; }
  bool device_ok() const override {
    return inputs[0]->type == NNR_DATA_TYPE_UINT8 && inputs[1]->ndata == 1 &&
           (inputs.size() < 3 || !inputs[2] || inputs[2]->ndata == 1) && inputs[0]->ndata < (1u << 31);
  }
  bool prepare_device(device_state_t& s) override {
    set_out_layout(s, outputs[0], in_layout(s, inputs[0]));
    return true;
  }
  bool run_device(device_state_t& s, void* stream) override {
    const tensor_t* zp = inputs.size() > 2 ? inputs[2] : nullptr;
    return nnrcu_ok(s,
                    nnrcu_dequantize_linear_u8((const uint8_t*)s.dev(inputs[0]), scalar_f32(inputs[1], 1.0f),
                                               (uint8_t)scalar_zp(zp), nullptr, 1, (int)inputs[0]->ndata,
                                               (float*)s.dev(outputs[0]), stream),
                    "DequantizeLinear");
  }
};

// QLinearAdd (backend/cpu/QLinearAdd.cpp:46-104) of two same-shape u8
// tensors, as fuse_qdq_compute builds it from DQ, DQ -> Add [-> Relu] -> Q.
struct QLinearAdd_cuda : cuda_op_t {
  bool init() override {
    if (inputs.size() < 7 || outputs.size() != 1) return false;
    layout_mask = LAYOUT_ALL;
    return true;
  }
  bool device_input(int idx) const override { return idx == 0 || idx == 3; }
  bool infer_shape() override { return outputs[0]->reshape_identity(inputs[0], inputs[0]->type); }
  bool host_allowed() const override { return true; }
  bool device_ok() const override {
    const tensor_t *A = inputs[0], *B = inputs[3];
    if (A->type != NNR_DATA_TYPE_UINT8 || B->type != NNR_DATA_TYPE_UINT8 || A->ndata != B->ndata) return false;
    if (A->ndim != B->ndim) return false;
    for (int i = 0; i < A->ndim; ++i)
      if (A->dims[i] != B->dims[i]) return false;
    return true;
  }
  bool prepare_device(device_state_t& s) override {
    if (in_layout(s, inputs[0]) != in_layout(s, inputs[3]))
      return s.fail("QLinearAdd: inputs in different layouts");
    set_out_layout(s, outputs[0], in_layout(s, inputs[0]));
    return true;
  }
  bool run_device(device_state_t& s, void* stream) override {
    const tensor_t* yzp = inputs.size() > 7 ? inputs[7] : nullptr;
    return nnrcu_ok(
        s,
        nnrcu_qlinearadd_u8((const uint8_t*)s.dev(inputs[0]), scalar_f32(inputs[1], 1.0f),
                            (uint8_t)scalar_zp(inputs[2]), (const uint8_t*)s.dev(inputs[3]),
                            scalar_f32(inputs[4], 1.0f), (uint8_t)scalar_zp(inputs[5]), scalar_f32(inputs[6], 1.0f),
                            (uint8_t)scalar_zp(yzp), (uint8_t*)s.dev(outputs[0]), inputs[0]->ndata, stream),
        "QLinearAdd");
  }
};

// fp32 Add (backend/cpu/binary_math.cpp:57-77): same shapes, or B a
// trailing-row broadcast of an NCHW / 2-D A (a bias row).
struct Add_cuda : cuda_op_t {
  bool init() override {
    if (inputs.size() != 2 || outputs.size() != 1) return false;
    layout_mask = LAYOUT_ALL;
    return true;
  }
  bool device_input(int idx) const override { return idx == 0 || idx == 1; }
  bool infer_shape() override { return outputs[0]->reshape_multi_broadcast(inputs[0], inputs[1], inputs[0]->type); }
  bool host_allowed() const override { return true; }
  bool same_shape() const {
    const tensor_t *A = inputs[0], *B = inputs[1];
    if (A->ndim != B->ndim) return false;
    for (int i = 0; i < A->ndim; ++i)
      if (A->dims[i] != B->dims[i]) return false;
    return true;
  }
  bool row_broadcast() const {
    const tensor_t *A = inputs[0], *B = inputs[1];
    if (B->ndim > A->ndim || B->ndata == 0 || A->ndata % B->ndata) return false;
    for (int i = 1; i <= B->ndim; ++i)
      if (B->dims[B->ndim - i] != A->dims[A->ndim - i]) return false;
    return A->ndim <= 2 || A->format == memory_layout_t::NCHW;
  }
  bool device_ok() const override {
    return inputs[0]->type == NNR_DATA_TYPE_FLOAT32 && inputs[1]->type == NNR_DATA_TYPE_FLOAT32 &&
           outputs[0]->ndata == inputs[0]->ndata && (same_shape() || row_broadcast());
  }
  bool prepare_device(device_state_t& s) override {
    if (same_shape() && in_layout(s, inputs[0]) != in_layout(s, inputs[1]) && inputs[0]->ndim == 4 &&
        inputs[0]->dims[2] * inputs[0]->dims[3] > 1)
      return s.fail("Add: inputs in different layouts");
    set_out_layout(s, outputs[0], in_layout(s, inputs[0]));
    return true;
  }
  bool run_device(device_state_t& s, void* stream) override {
    const size_t total = inputs[0]->ndata;
    const size_t period = same_shape() ? total : inputs[1]->ndata;
    return nnrcu_ok(s,
                    nnrcu_add_f32((const float*)s.dev(inputs[0]), (const float*)s.dev(inputs[1]),
                                  (float*)s.dev(outputs[0]), total, period, stream),
                    "Add");
  }
};

// ------------------------------------------------------------------ pooling
// Both run on NHWC data; an NCHW input or output is reordered on the device
// in the workspace.
void* ws_at(device_state_t& s, size_t off) { return static_cast<uint8_t*>(s.workspace) + off; }

// MaxPool (backend/cpu/MaxPool.cpp:279) on u8 (fuse_qdq rewires a
// DQ -> MaxPool -> Q onto the quantised tensor), dilation 1.
struct MaxPool_cuda : cuda_op_t {
  std::vector<int64_t> k, s_, p;
  int ceil_mode = 0;
  bool init() override {
    if (inputs.size() != 1 || outputs.empty()) return false;
    std::vector<int64_t> v;
    ints_attr(this, attr_key_t::kernel_shape, k);
    ints_attr(this, attr_key_t::strides, v);
    s_.assign(2, 1);
    for (size_t i = 0; i < v.size() && i < 2; ++i) s_[i] = v[i];
    ints_attr(this, attr_key_t::pads, v);
    p.assign(4, 0);
    for (size_t i = 0; i < v.size() && i < 4; ++i) p[i] = v[i];
    ceil_mode = attribute(attr_key_t::ceil_mode, (int32_t)0);
    layout_mask = LAYOUT_DEVICE;
    return true;
  }
  bool infer_shape() override {
    const tensor_t* x = inputs[0];
    if (x->ndim != 4 || k.size() != 2) return false;
    int dims[4] = {x->dims[0], x->dims[1], 0, 0};
    for (int i = 0; i < 2; ++i) {
      const int num = x->dims[2 + i] + (int)p[i] + (int)p[i + 2] - (int)k[i];
      dims[2 + i] = (ceil_mode ? (num + (int)s_[i] - 1) / (int)s_[i] : num / (int)s_[i]) + 1;
    }
    return outputs[0]->reshape({dims, 4}, x->type);
  }
  bool host_allowed() const override { return true; }
  bool device_ok() const override {
    std::vector<int64_t> dil;
    ints_attr(const_cast<MaxPool_cuda*>(this), attr_key_t::dilations, dil);
    for (auto d : dil)
      if (d != 1) return false;
    return inputs[0]->type == NNR_DATA_TYPE_UINT8 && outputs.size() == 1 && !ceil_mode;
  }
  size_t device_workspace() const override { return inputs[0]->ndata + outputs[0]->ndata; }
  bool prepare_device(device_state_t& s) override {
    set_out_layout(s, outputs[0], outputs[0]->format);
    return true;
  }
  bool run_device(device_state_t& s, void* stream) override {
    const tensor_t *x = inputs[0], *y = outputs[0];
    const int N = x->dims[0], C = x->dims[1], H = x->dims[2], W = x->dims[3];
    const void* xin = s.dev(inputs[0]);
    if (in_layout(s, inputs[0]) != memory_layout_t::NHWC) {
      if (!nnrcu_ok(s, nnrcu_nchw_to_nhwc(xin, ws_at(s, 0), N, C, H, W, 1, stream), "MaxPool")) return false;
      xin = ws_at(s, 0);
    }
    const bool out_nhwc = y->format == memory_layout_t::NHWC;
    void* yout = out_nhwc ? s.dev(outputs[0]) : ws_at(s, x->ndata);
    if (!nnrcu_ok(s,
                  nnrcu_maxpool_u8_nhwc((const uint8_t*)xin, (uint8_t*)yout, N, H, W, C, (int)k[0], (int)k[1],
                                        (int)s_[0], (int)s_[1], (int)p[0], (int)p[1], (int)p[2], (int)p[3], stream),
                  "MaxPool"))
      return false;
    if (!out_nhwc)
      return nnrcu_ok(s, nnrcu_nhwc_to_nchw(yout, s.dev(outputs[0]), N, C, y->dims[2], y->dims[3], 1, stream),
                      "MaxPool");
    return true;
  }
};

// GlobalAveragePool (kernel/pool.h:109-125) on fp32: per channel a
// sequential sum over the positions times 1/spatial.
struct GlobalAveragePool_cuda : cuda_op_t {
  bool init() override {
    if (inputs.size() != 1 || outputs.size() != 1) return false;
    layout_mask = LAYOUT_DEVICE;
    return true;
  }
  bool infer_shape() override {
    const tensor_t* x = inputs[0];
    if (x->ndim != 4) return false;
    const int dims[4] = {x->dims[0], x->dims[1], 1, 1};
    return outputs[0]->reshape({dims, 4}, x->type);
  }
  bool host_allowed() const override { return true; }
  bool device_ok() const override { return inputs[0]->type == NNR_DATA_TYPE_FLOAT32 && inputs[0]->ndim == 4; }
  size_t device_workspace() const override { return inputs[0]->ndata * 4; }
  bool prepare_device(device_state_t& s) override {
    set_out_layout(s, outputs[0], outputs[0]->format);  // [N, C, 1, 1]: both layouts are the same bytes
    return true;
  }
  bool run_device(device_state_t& s, void* stream) override {
    const tensor_t* x = inputs[0];
    const int N = x->dims[0], C = x->dims[1], H = x->dims[2], W = x->dims[3];
    const void* xin = s.dev(inputs[0]);
    if (in_layout(s, inputs[0]) != memory_layout_t::NHWC && H * W > 1) {
      if (!nnrcu_ok(s, nnrcu_nchw_to_nhwc(xin, s.workspace, N, C, H, W, 4, stream), "GlobalAveragePool"))
        return false;
      xin = s.workspace;
    }
    return nnrcu_ok(s, nnrcu_gap_f32_nhwc((const float*)xin, N, H * W, C, (float*)s.dev(outputs[0]), stream),
                    "GlobalAveragePool");
  }
};

template <typename T>
operator_t* make(int, pool_t& pool) {
  return pool_new<T>(pool);
}

// Static registration under backend_t::CUDA, like the CPU backend's
// registrar (backend/cpu/solve_operator.cpp:18-31); cuda_backend_anchor()
// keeps this file linked from a static library.
struct cuda_registrar {
  cuda_registrar() {
    auto& r = global_registry();
    r.register_op("QLinearConv", backend_t::CUDA, make<QLinearConv_cuda>);
    r.register_op("QLinearMatMul", backend_t::CUDA, make<QLinearMatMul_cuda>);
    r.register_op("Conv", backend_t::CUDA, make<Conv_cuda>);
    r.register_op("Gemm", backend_t::CUDA, make<Gemm_cuda>);
    r.register_op("MatMul", backend_t::CUDA, make<Gemm_cuda>);
    r.register_op("QuantizeLinear", backend_t::CUDA, make<QuantizeLinear_cuda>);
    r.register_op("DequantizeLinear", backend_t::CUDA, make<DequantizeLinear_cuda>);
    r.register_op("QLinearAdd", backend_t::CUDA, make<QLinearAdd_cuda>);
    r.register_op("Add", backend_t::CUDA, make<Add_cuda>);
    r.register_op("MaxPool", backend_t::CUDA, make<MaxPool_cuda>);
    r.register_op("GlobalAveragePool", backend_t::CUDA, make<GlobalAveragePool_cuda>);
  }
} cuda_registrar_instance;

}  // namespace

int cuda_backend_anchor() { return 1; }

}  // namespace nnr::cuda
