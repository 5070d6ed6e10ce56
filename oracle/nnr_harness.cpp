// C entry points around nnr's own CPU runtime (context_t), compiled with the
// nnr library into oracle/_ref/libnnr_cpu.so by oracle/Makefile (`make nnr`).
// TEST INFRASTRUCTURE ONLY: tests use it to pin the C restatement in
// nnr_oracle.c (fp32 Conv/Gemm/MatMul, post-ops, the QDQ glue operators) and
// bench.py uses it as the reference CPU timing. Nothing in nnr_b200/ links or
// loads it.
//
// The calls follow nnr's public API (nnr.h:482-590): load() an ONNX byte
// stream, prepare() (fold_run, the optimizer passes including Conv+BN and
// post-op fusion, memory planning), fill graph inputs, run(), read outputs.
#include <cstdio>
#include <cstring>
#include <string>

#include "nnr.h"
#include "registry.h"

using namespace nnr;

extern "C" {

void nnrh_set_threads(int n) { context_t::set_num_threads(n); }

// Loads an ONNX ModelProto (bytes). backend: 0 = CPU. options: bit 0 turns
// nnr's channel-blocked (nChw16c) layout off (context_t::set_no_blocked).
// Returns an opaque context, or NULL.
void* nnrh_load(const void* buf, size_t len, int backend, int memory_planning, int options) {
  auto* ctx = new (std::nothrow) context_t();
  if (!ctx) return nullptr;
  ctx->preferred_backend = (uint8_t)backend;
  if (!ctx->load(buf, len)) {
    fprintf(stderr, "nnrh_load: load failed\n");
    delete ctx;
    return nullptr;
  }
  if (memory_planning) ctx->enable_memory_planning(true);
  if (options & 1) ctx->set_no_blocked(true);
  return ctx;
}

int nnrh_prepare(void* h) { return static_cast<context_t*>(h)->prepare() ? 0 : -1; }

void nnrh_free(void* h) { delete static_cast<context_t*>(h); }

// Copies `bytes` bytes into the named tensor (a graph input).
int nnrh_set_input(void* h, const char* name, const void* data, size_t bytes) {
  auto* ctx = static_cast<context_t*>(h);
  tensor_t* t = ctx->search_tensor(name);
  if (!t || !t->data) return -1;
  const size_t have = t->ndata * data_type_sizeof(t);
  if (have != bytes) {
    fprintf(stderr, "nnrh_set_input(%s): %zu bytes given, tensor holds %zu\n", name, bytes, have);
    return -2;
  }
  memcpy(t->data, data, bytes);
  return 0;
}

int nnrh_run(void* h) { return static_cast<context_t*>(h)->run() ? 0 : -1; }

// Shape, element type (data_type_t) and layout (memory_layout_t) of a tensor.
int nnrh_tensor_info(void* h, const char* name, int* dims, int* ndim, int* type, int* format) {
  tensor_t* t = static_cast<context_t*>(h)->search_tensor(name);
  if (!t) return -1;
  *ndim = t->ndim;
  for (int i = 0; i < t->ndim; ++i) dims[i] = t->dims[i];
  *type = (int)t->type;
  *format = (int)t->format;
  return 0;
}

// Copies the named tensor's bytes out, as stored (nnrh_tensor_info gives the
// layout).
int nnrh_get(void* h, const char* name, void* out, size_t bytes) {
  tensor_t* t = static_cast<context_t*>(h)->search_tensor(name);
  if (!t || !t->data) return -1;
  const size_t have = t->ndata * data_type_sizeof(t);
  if (have != bytes) return -2;
  memcpy(out, t->data, bytes);
  return 0;
}

// Copies `bytes` bytes from the start of the named tensor's buffer, whatever
// its logical size (a channel-blocked tensor holds padded channels).
int nnrh_get_raw(void* h, const char* name, void* out, size_t bytes) {
  tensor_t* t = static_cast<context_t*>(h)->search_tensor(name);
  if (!t || !t->data) return -1;
  memcpy(out, t->data, bytes);
  return 0;
}

// Number of graph nodes and, per node, its op_type and flags (bit 0 skip,
// bit 1 folded): shows what fusion produced.
int nnrh_num_nodes(void* h) {
  auto* ctx = static_cast<context_t*>(h);
  return ctx->graph ? (int)ctx->graph->nodes.size() : 0;
}

int nnrh_node(void* h, int i, char* op_type, size_t len, int* flags) {
  auto* ctx = static_cast<context_t*>(h);
  if (!ctx->graph || i < 0 || i >= (int)ctx->graph->nodes.size()) return -1;
  operator_t* n = ctx->graph->nodes[i];
  snprintf(op_type, len, "%.*s", (int)n->op_type.size(), n->op_type.data());
  *flags = (n->skip ? 1 : 0) | (n->folded ? 2 : 0);
  return 0;
}

}  // extern "C"
