// Device state of nnr's CUDA backend: roles of every tensor, the device
// arena that mirrors nnr's memory plan, uploads and downloads, and the
// per-run control of eager, captured and replayed execution.
#include "cuda_backend.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

namespace nnr::cuda {

namespace {
std::mutex g_states_mu;
std::unordered_map<context_t*, device_state_t*> g_states;

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

size_t tensor_bytes(const tensor_t* t) { return t->ndata * data_type_sizeof(t->type); }

bool is_device_op(operator_t* n) {
  auto* c = dynamic_cast<cuda_op_t*>(n);
  return c && !c->on_host;
}

bool is_view(operator_t* n) {
  const int vi = n->view_input_index();
  return vi >= 0 && vi < (int)n->inputs.size() && n->inputs[vi] && !n->outputs.empty() && n->outputs[0];
}
}  // namespace

bool nnrcu_ok(device_state_t& s, int rc, const char* what) {
  if (rc == NNRCU_OK) return true;
  char msg[512];
  nnrcu_last_error(msg, sizeof(msg));
  return s.fail("%s: %s (code %d)", what, msg, rc);
}

bool device_state_t::fail(const char* fmt, ...) {
  char buf[768];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  error = buf;
  fprintf(stderr, "nnr cuda: %s\n", buf);
  return false;
}

device_state_t* state_of(context_t* ctx) {
  std::lock_guard<std::mutex> lk(g_states_mu);
  auto it = g_states.find(ctx);
  if (it != g_states.end()) return it->second;
  auto* s = new device_state_t();
  s->ctx = ctx;
  g_states[ctx] = s;
  return s;
}

device_state_t* find_state(context_t* ctx) {
  std::lock_guard<std::mutex> lk(g_states_mu);
  auto it = g_states.find(ctx);
  return it == g_states.end() ? nullptr : it->second;
}

void release_state(context_t* ctx) {
  device_state_t* s = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_states_mu);
    auto it = g_states.find(ctx);
    if (it == g_states.end()) return;
    s = it->second;
    g_states.erase(it);
  }
  delete s;
}

void device_state_t::invalidate() {
  if (graph_exec) {
    nnrcu_graph_destroy(graph_exec);
    graph_exec = nullptr;
  }
  if (arena) nnrcu_free(arena);
  if (workspace) nnrcu_free(workspace);
  for (void* p : pinned) nnrcu_host_unregister(p);
  pinned.clear();
  for (auto& [t, p] : consts) nnrcu_free(p);
  arena = workspace = nullptr;
  arena_bytes = workspace_bytes = 0;
  consts.clear();
  slot_of_host.clear();
  canon.clear();
  dev_layout.clear();
  device_produced.clear();
  uploads.clear();
  downloads.clear();
  order.clear();
  all_device = false;
  run_index = 0;
  phase = 0;
  ready = false;
}

device_state_t::~device_state_t() {
  invalidate();
  if (stream) nnrcu_stream_destroy(stream);
}

tensor_t* device_state_t::resolve(tensor_t* t) const {
  for (int guard = 0; t && guard < 1024; ++guard) {
    auto it = canon.find(t);
    if (it == canon.end()) return t;
    t = it->second;
  }
  return t;
}

void* device_state_t::dev(tensor_t* t) {
  t = resolve(t);
  auto c = consts.find(t);
  if (c != consts.end()) return c->second;
  const void* key = t->data ? t->data : (const void*)t;
  auto it = slot_of_host.find(key);
  if (it == slot_of_host.end()) return nullptr;
  return static_cast<uint8_t*>(arena) + it->second;
}

// Builds the roles of every tensor for the prepared graph, the arena and the
// operators' device objects. Runs at the first exec() of a CUDA operator
// after prepare() (formats and the memory plan are final by then).
bool device_state_t::setup() {
  invalidate();
  if (!nnrcu_ok(*this, nnrcu_init(device), "device")) return false;
  if (!stream) {
    if (!nnrcu_ok(*this, nnrcu_stream_create(&stream), "stream")) return false;
  }
  auto& nodes = ctx->graph->nodes;
  const int n = (int)nodes.size();

  // aliases: view outputs and skipped (fused-away) nodes forward their input
  for (auto* nd : nodes) {
    if (nd->folded) continue;
    if (nd->skip && !nd->inputs.empty() && nd->inputs[0] && !nd->outputs.empty() && nd->outputs[0])
      canon[nd->outputs[0]] = nd->inputs[0];
    else if (!nd->skip && is_view(nd))
      canon[nd->outputs[0]] = nd->inputs[nd->view_input_index()];
  }

  std::unordered_map<const tensor_t*, operator_t*> producer;
  std::unordered_set<const tensor_t*> graph_in, graph_out;
  for (auto& name : ctx->graph_inputs)
    if (tensor_t* t = ctx->search_tensor(name)) graph_in.insert(resolve(t));
  for (auto& name : ctx->graph_outputs)
    if (tensor_t* t = ctx->search_tensor(name)) graph_out.insert(resolve(t));

  stats.device_ops = stats.host_ops = stats.host_glue = 0;
  for (int i = 0; i < n; ++i) {
    operator_t* nd = nodes[i];
    if (nd->skip || nd->folded) continue;
    auto* cop = dynamic_cast<cuda_op_t*>(nd);
    if (cop) {
      cop->on_host = !cop->device_ok();
      if (cop->on_host && !cop->host_allowed())
        return fail("%.*s (%.*s): this variant is not supported on the device", (int)nd->op_type.size(),
                    nd->op_type.data(), (int)nd->node_name.size(), nd->node_name.data());
      if (cop->on_host) {
        stats.host_ops++;
        stats.host_glue++;
        cop = nullptr;
      }
    }
    if (cop) {
      order.push_back(cop);
      stats.device_ops++;
    } else if (!is_view(nd)) {
      stats.host_ops++;
    }
    if (!is_view(nd))
      for (auto* t : nd->outputs)
        if (t) producer[resolve(t)] = nd;
  }
  if (order.empty()) return fail("no CUDA operator in the graph");
  all_device = stats.host_ops == 0;

  auto is_constant = [&](tensor_t* c) {
    if (ctx->initializer_names.count(c->name)) return true;
    auto it = producer.find(c);
    if (it != producer.end()) return false;
    return !graph_in.count(c);  // produced by a folded node (or never written)
  };

  // per CUDA op: which inputs are device data, who uploads, what is produced
  std::unordered_set<const tensor_t*> uploaded;
  std::vector<tensor_t*> slots;  // canonical tensors that need an arena slot
  auto want_slot = [&](tensor_t* c) { slots.push_back(c); };
  for (auto* op : order) {
    for (size_t k = 0; k < op->inputs.size(); ++k) {
      tensor_t* t = op->inputs[k];
      if (!t || t->ndata == 0) continue;
      if (!op->device_input((int)k)) continue;
      tensor_t* c = resolve(t);
      if (is_constant(c)) {
        if (!consts.count(c)) {
          void* p = nullptr;
          const size_t b = tensor_bytes(c);
          if (!nnrcu_ok(*this, nnrcu_malloc(&p, std::max<size_t>(b, 256)), "constant upload")) return false;
          if (!nnrcu_ok(*this, nnrcu_memcpy_h2d(p, c->data, b, stream), "constant upload")) return false;
          consts[c] = p;
          dev_layout[c] = c->format;
          stats.const_bytes += (int64_t)b;
        }
        continue;
      }
      auto pit = producer.find(c);
      const bool on_device = pit != producer.end() && is_device_op(pit->second);
      if (!on_device && !uploaded.count(c)) {
        uploaded.insert(c);
        uploads[op].push_back(c);
        dev_layout[c] = c->format;
        want_slot(c);
      }
    }
    for (auto* t : op->outputs) {
      if (!t) continue;
      tensor_t* c = resolve(t);
      device_produced.insert(c);
      want_slot(c);
    }
  }

  // downloads: device-produced tensors that the host reads
  for (const tensor_t* cc : device_produced) {
    tensor_t* c = const_cast<tensor_t*>(cc);
    bool host_reads = graph_out.count(c) > 0;
    for (int i = 0; i < n && !host_reads; ++i) {
      operator_t* nd = nodes[i];
      if (nd->skip || nd->folded || is_view(nd) || is_device_op(nd)) continue;
      for (auto* t : nd->inputs)
        if (t && resolve(t) == c) host_reads = true;
    }
    if (host_reads) downloads[producer[c]].push_back(c);
  }

  // graph inputs uploaded and graph outputs downloaded every run: page-lock
  // their host buffers (nnr's own allocations), so that those copies run at
  // the link's rate instead of through pageable staging
  auto pin = [&](tensor_t* c) {
    const size_t b = tensor_bytes(c);
    if (!c->data || b < (1u << 16)) return;  // (small buffers gain nothing)
    if (std::find(pinned.begin(), pinned.end(), c->data) != pinned.end()) return;
    if (nnrcu_host_register(c->data, b) == NNRCU_OK) pinned.push_back(c->data);
  };
  for (auto& [op, list] : uploads)
    for (auto* c : list)
      if (graph_in.count(c)) pin(c);
  for (auto& [op, list] : downloads)
    for (auto* c : list)
      if (graph_out.count(c)) pin(c);

  // arena: one slot per distinct host buffer (nnr's memory plan), the
  // largest tensor that uses it deciding its size
  std::unordered_map<const void*, size_t> slot_size;
  std::vector<const void*> keys;
  for (auto* c : slots) {
    const void* key = c->data ? c->data : (const void*)c;
    auto it = slot_size.find(key);
    if (it == slot_size.end()) {
      slot_size[key] = tensor_bytes(c);
      keys.push_back(key);
    } else {
      it->second = std::max(it->second, tensor_bytes(c));
    }
  }
  size_t off = 0;
  for (auto* k : keys) {
    slot_of_host[k] = off;
    off += align256(std::max<size_t>(slot_size[k], 1));
  }
  arena_bytes = std::max<size_t>(off, 256);
  if (!nnrcu_ok(*this, nnrcu_malloc(&arena, arena_bytes), "device arena")) return false;
  stats.arena_bytes = (int64_t)arena_bytes;
  stats.slots = (int64_t)keys.size();

  // operators: layouts in execution order, then their device objects
  size_t ws = 0;
  for (auto* op : order) {
    if (!op->prepare_device(*this)) return false;
    ws = std::max(ws, op->device_workspace());
  }
  for (auto& [op, list] : downloads)
    for (auto* c : list) ws = std::max(ws, tensor_bytes(c));  // reorder scratch
  workspace_bytes = std::max<size_t>(ws, 256);
  if (!nnrcu_ok(*this, nnrcu_malloc(&workspace, workspace_bytes), "device workspace")) return false;
  if (!nnrcu_ok(*this, nnrcu_stream_sync(stream), "set-up")) return false;
  ready = true;
  return true;
}

// ------------------------------------------------------------------ operator base
bool cuda_op_t::inputs_constant() const {
  for (auto* t : inputs) {
    if (!t) continue;
    if (!ctx->initializer_names.count(t->name)) {
      // outputs of nodes folded earlier in fold_run are constants too
      bool folded_src = false;
      for (auto* nd : ctx->graph->nodes)
        if (nd->folded)
          for (auto* o : nd->outputs)
            if (o == t) folded_src = true;
      if (!folded_src) return false;
    }
  }
  return true;
}

// Constant folding at load time (fold_run, nnr.cpp:1341-1366) is host work:
// it runs nnr's own CPU operator for this node on the constant inputs.
bool cuda_op_t::fold_on_host() {
  if (!host_twin) {
    host_twin = global_registry().solve(op_type, opset, ctx->attr_pool, backend_t::CPU);
    if (!host_twin) return false;
    host_twin->ctx = ctx;
    host_twin->opset = opset;
    host_twin->op_type = op_type;
    host_twin->node_name = node_name;
    host_twin->domain = domain;
    host_twin->inputs = inputs;
    host_twin->outputs = outputs;
    host_twin->attrs = attrs;
    if (!host_twin->init()) return false;
  }
  return host_twin->reshape() && host_twin->exec();
}

bool cuda_op_t::reshape() {
  if (auto* s = find_state(ctx)) s->ready = false;  // shapes may change: rebuild at the next exec
  return infer_shape();
}

bool cuda_op_t::exec() {
  // Before the plan exists nnr is still loading: fold_run executes constant
  // nodes (fold on the host) and cheap nodes on garbage for shape
  // propagation (nothing to do on the device).
  if (!ctx->optimizer->plan_built) return inputs_constant() ? fold_on_host() : true;
  device_state_t& s = *st();
  if (!s.ready && !s.setup()) return false;
  if (on_host) return fold_on_host();
  void* stream = s.stream;
  const bool first = this == s.order.front();
  const bool last = this == s.order.back();

  auto upload = [&](tensor_t* c) {
    const size_t b = c->ndata * data_type_sizeof(c->type);
    s.dev_layout[c] = c->format;
    s.stats.h2d_bytes += (int64_t)b;
    return nnrcu_ok(s, nnrcu_memcpy_h2d(s.dev(c), c->data, b, stream), "upload");
  };
  auto download = [&](tensor_t* c) {
    const size_t b = c->ndata * data_type_sizeof(c->type);
    const void* src = s.dev(c);
    // the host copy is in the layout nnr has flagged; the device copy may be
    // in the other one (an elementwise op keeps its input's layout)
    const memory_layout_t dl = s.dev_layout[c];
    if (c->ndim == 4 && dl != c->format && c->dims[2] * c->dims[3] > 1) {
      const int es = (int)data_type_sizeof(c->type);
      const int N = c->dims[0], C = c->dims[1], H = c->dims[2], W = c->dims[3];
      const int rc = dl == memory_layout_t::NHWC ? nnrcu_nhwc_to_nchw(src, s.workspace, N, C, H, W, es, stream)
                                                 : nnrcu_nchw_to_nhwc(src, s.workspace, N, C, H, W, es, stream);
      if (!nnrcu_ok(s, rc, "download reorder")) return false;
      src = s.workspace;
    }
    s.stats.d2h_bytes += (int64_t)b;
    return nnrcu_ok(s, nnrcu_memcpy_d2h(c->data, src, b, stream), "download");
  };

  if (first) {
    s.run_index++;
    s.stats.runs++;
    s.phase = 0;
    if (s.use_graph && s.all_device) s.phase = s.graph_exec ? 2 : (s.run_index >= 2 ? 1 : 0);
    if (s.phase != 0) {
      for (auto* op : s.order)
        for (auto* c : s.uploads[op])
          if (!upload(c)) return false;
      if (s.phase == 1 && !nnrcu_ok(s, nnrcu_graph_begin(stream), "graph capture")) return false;
      if (s.phase == 2) {
        if (!nnrcu_ok(s, nnrcu_graph_launch(s.graph_exec, stream), "graph launch")) return false;
        s.stats.graph_replays++;
      }
    }
  }
  if (s.phase == 0)
    for (auto* c : s.uploads[this])
      if (!upload(c)) return false;
  if (s.phase != 2 && !run_device(s, stream)) {
    if (s.phase == 1) {
      void* g = nullptr;
      nnrcu_graph_end(stream, &g);
      if (g) nnrcu_graph_destroy(g);
      s.use_graph = false;
    }
    return false;
  }
  if (s.phase == 0) {
    auto& dl = s.downloads[this];
    for (auto* c : dl)
      if (!download(c)) return false;
    if (!dl.empty() || last)
      if (!nnrcu_ok(s, nnrcu_stream_sync(stream), "sync")) return false;
  }
  if (last && s.phase != 0) {
    if (s.phase == 1) {
      if (!nnrcu_ok(s, nnrcu_graph_end(stream, &s.graph_exec), "graph capture")) return false;
      if (!nnrcu_ok(s, nnrcu_graph_launch(s.graph_exec, stream), "graph launch")) return false;
    }
    for (auto* op : s.order)
      for (auto* c : s.downloads[op])
        if (!download(c)) return false;
    if (!nnrcu_ok(s, nnrcu_stream_sync(stream), "sync")) return false;
  }
  if (last) {
    int status = 0;
    if (!nnrcu_ok(s, nnrcu_device_status(&status), "device status")) return false;
    if (status != 0) return s.fail("a kernel reported device status %d", status);
  }
  return true;
}

// ------------------------------------------------------------------ helpers
int64_t ints_attr(operator_t* op, attr_key_t key, std::vector<int64_t>& out) {
  int64_t* ints = nullptr;
  const int n = op->attribute(key, ints);
  out.assign(ints, ints + std::max(n, 0));
  return n;
}

float scalar_f32(const tensor_t* t, float def) {
  if (!t || !t->data || t->ndata < 1) return def;
  if (t->type == NNR_DATA_TYPE_FLOAT32) return *(const float*)t->data;
  if (t->type == NNR_DATA_TYPE_FLOAT16) return float16_to_float32(*(const uint16_t*)t->data);
  return def;
}

int scalar_zp(const tensor_t* t) {
  if (!t || !t->data || t->ndata < 1) return 0;
  switch (t->type) {
    case NNR_DATA_TYPE_UINT8: return *(const uint8_t*)t->data;
    case NNR_DATA_TYPE_INT8: return *(const int8_t*)t->data;
    case NNR_DATA_TYPE_INT32: return *(const int32_t*)t->data;
    default: return 0;
  }
}

}  // namespace nnr::cuda
