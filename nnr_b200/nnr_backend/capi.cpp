// C entry points of an nnr build with the CUDA backend (libnnr_cuda.so):
// what an application does with nnr (nnr.h:482-590) — load an ONNX model,
// prepare, fill inputs, run, read outputs — with preferred_backend = CUDA,
// plus read-outs of what the backend did (device and host operators,
// arena size, copies, graph replays) for tests and the benchmark.
#include <cstdio>
#include <cstring>
#include <new>

#include "cuda_backend.h"

using namespace nnr;

namespace nnr::cuda {
int cuda_backend_anchor();
}

extern "C" {

// Loads an ONNX ModelProto, selects the CUDA backend on `device` and runs
// nnr's preparation (fold_run, fusion passes including fuse_qdq_compute,
// layout assignment, memory planning); this part needs no GPU. The device
// is first used by the first run(). graphs: capture/replay the run in a CUDA
// graph when every operator is on the device. Returns a context or NULL.
void* nnrcuda_load(const void* buf, size_t len, int device, int memory_planning, int graphs) {
  nnr::cuda::cuda_backend_anchor();
  auto* ctx = new (std::nothrow) context_t();
  if (!ctx) return nullptr;
  ctx->preferred_backend = (uint8_t)backend_t::CUDA;
  if (!ctx->load(buf, len)) {
    delete ctx;
    return nullptr;
  }
  if (memory_planning) ctx->enable_memory_planning(true);
  if (!ctx->prepare()) {
    delete ctx;
    return nullptr;
  }
  auto* s = nnr::cuda::state_of(ctx);
  s->use_graph = graphs != 0;
  s->device = device;
  return ctx;
}

void nnrcuda_free(void* h) {
  auto* ctx = static_cast<context_t*>(h);
  delete ctx;                       // operators free their device objects
  nnr::cuda::release_state(ctx);    // then the arena, workspace and stream
}

int nnrcuda_set_input(void* h, const char* name, const void* data, size_t bytes) {
  tensor_t* t = static_cast<context_t*>(h)->search_tensor(name);
  if (!t || !t->data || t->ndata * data_type_sizeof(t) != bytes) return -1;
  memcpy(t->data, data, bytes);
  return 0;
}

// A graph input's own host buffer (nnr's tensor_t::data) and its size: an
// application may fill it in place instead of passing a copy to
// nnrcuda_set_input (nnr's own applications write tensor data directly).
int nnrcuda_input_buffer(void* h, const char* name, void** data, size_t* bytes) {
  tensor_t* t = static_cast<context_t*>(h)->search_tensor(name);
  if (!t || !t->data || !data || !bytes) return -1;
  *data = t->data;
  *bytes = t->ndata * data_type_sizeof(t);
  return 0;
}

int nnrcuda_run(void* h) { return static_cast<context_t*>(h)->run() ? 0 : -1; }

int nnrcuda_tensor_info(void* h, const char* name, int* dims, int* ndim, int* type, int* format) {
  tensor_t* t = static_cast<context_t*>(h)->search_tensor(name);
  if (!t) return -1;
  *ndim = t->ndim;
  for (int i = 0; i < t->ndim; ++i) dims[i] = t->dims[i];
  *type = (int)t->type;
  *format = (int)t->format;
  return 0;
}

int nnrcuda_get(void* h, const char* name, void* out, size_t bytes) {
  tensor_t* t = static_cast<context_t*>(h)->search_tensor(name);
  if (!t || !t->data || t->ndata * data_type_sizeof(t) != bytes) return -1;
  memcpy(out, t->data, bytes);
  return 0;
}

// Node i after nnr's passes: op_type, flags (bit 0 skip, bit 1 folded,
// bit 2 a CUDA operator running on the device), its output's layout.
int nnrcuda_node(void* h, int i, char* op_type, size_t len, int* flags, int* out_format) {
  auto* ctx = static_cast<context_t*>(h);
  if (!ctx->graph || i < 0 || i >= (int)ctx->graph->nodes.size()) return -1;
  operator_t* n = ctx->graph->nodes[i];
  snprintf(op_type, len, "%.*s", (int)n->op_type.size(), n->op_type.data());
  auto* c = dynamic_cast<nnr::cuda::cuda_op_t*>(n);
  *flags = (n->skip ? 1 : 0) | (n->folded ? 2 : 0) | (c && !c->on_host ? 4 : 0);
  *out_format = (!n->outputs.empty() && n->outputs[0]) ? (int)n->outputs[0]->format : -1;
  return 0;
}

int nnrcuda_num_nodes(void* h) {
  auto* ctx = static_cast<context_t*>(h);
  return ctx->graph ? (int)ctx->graph->nodes.size() : 0;
}

// out[0..9]: runs, graph replays, H2D bytes, D2H bytes, device operators,
// host operators, host-run glue operators, arena bytes, constant bytes,
// arena slots.
int nnrcuda_stats(void* h, int64_t* out) {
  auto* s = nnr::cuda::find_state(static_cast<context_t*>(h));
  if (!s) return -1;
  const auto& st = s->stats;
  const int64_t v[10] = {st.runs,     st.graph_replays, st.h2d_bytes,   st.d2h_bytes,   st.device_ops,
                         st.host_ops, st.host_glue,     st.arena_bytes, st.const_bytes, st.slots};
  memcpy(out, v, sizeof(v));
  return 0;
}

int nnrcuda_last_error(void* h, char* buf, size_t len) {
  auto* s = h ? nnr::cuda::find_state(static_cast<context_t*>(h)) : nullptr;
  snprintf(buf, len, "%s", s ? s->error.c_str() : "");
  return 0;
}

}  // extern "C"
