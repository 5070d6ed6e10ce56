// nnr's backend_t::CUDA: operator_t subclasses that run the conv/GEMM hot
// path and its QDQ glue on a B200 through libnnrcu's C ABI (include/nnrcu.h).
// These files are meant to sit in nnr's tree as src/backend/cuda/ and be
// compiled with it; registering them makes registry_t::solve() return them
// when context_t::preferred_backend is CUDA (registry.cpp:10-27), including
// for the QLinearConv/QLinearMatMul/QLinearAdd nodes that fuse_qdq_compute
// builds (fuse_qdq_compute.cpp:142, :304).
//
// Device residency. nnr's tensors keep host buffers (tensor_t::data); the
// backend keeps one device copy per buffer, in one device arena per context:
//  * one slot per distinct host buffer, so tensors that nnr's memory planner
//    put into the same pool slot (memory_planner.cpp:109-337) share a device
//    slot too: the device arena reuses memory exactly where the host plan
//    does, with the same lifetime analysis;
//  * a tensor produced by a CUDA operator lives only on the device; it is
//    copied to its host buffer only when a host (CPU) operator reads it or
//    it is a graph output;
//  * a tensor produced on the host (a graph input, a CPU operator's output)
//    is uploaded before the first CUDA operator that reads it, every run;
//    initializers are uploaded once.
// Views (Flatten/Reshape aliases, skipped fused nodes) resolve to the
// tensor they alias.
//
// Layouts. The device stores each tensor in the layout nnr assigned to it
// (tensor_t::format, NCHW or NHWC): the CUDA operators advertise NHWC with a
// device cost (layout_cost), so assign_layouts keeps int8 and depthwise
// chains NHWC, and no host reorder ever touches device-resident data.
//
// Execution. Every operator enqueues on the context's stream. When the whole
// graph runs on the device, the second run() is captured into one CUDA
// graph and later runs replay it: the first CUDA operator uploads the inputs
// and launches the graph, the others only record, and the last one copies
// the graph outputs back and waits.
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "nnr.h"
#include "nnrcu.h"
#include "registry.h"

namespace nnr::cuda {

struct cuda_op_t;

struct backend_stats_t {
  int64_t runs = 0;
  int64_t graph_replays = 0;
  int64_t h2d_bytes = 0;
  int64_t d2h_bytes = 0;
  int64_t device_ops = 0;   // CUDA operators in the graph
  int64_t host_ops = 0;     // other active operators (views excluded)
  int64_t host_glue = 0;    // CUDA glue operators that ran nnr's CPU code (unsupported variant)
  int64_t arena_bytes = 0;  // device arena (activations)
  int64_t const_bytes = 0;  // uploaded initializers
  int64_t slots = 0;        // distinct activation slots
};

// Per-context device state (one stream, arena, workspace, graph).
struct device_state_t {
  context_t* ctx = nullptr;
  int device = 0;              // CUDA device of this context
  void* stream = nullptr;
  bool ready = false;          // roles and arena built for the current shapes
  bool use_graph = true;       // capture/replay when the whole graph is on the device
  std::string error;

  // arena
  void* arena = nullptr;
  size_t arena_bytes = 0;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  std::unordered_map<const void*, size_t> slot_of_host;  // host buffer -> arena offset
  std::unordered_map<const tensor_t*, void*> consts;     // uploaded initializers (own allocations)

  // roles (built by setup())
  std::unordered_map<const tensor_t*, tensor_t*> canon;       // alias -> tensor it views
  std::unordered_map<const tensor_t*, memory_layout_t> dev_layout;
  std::unordered_set<const tensor_t*> device_produced;        // canonical tensors
  std::unordered_map<const operator_t*, std::vector<tensor_t*>> uploads;  // H2D before an op
  std::unordered_map<const operator_t*, std::vector<tensor_t*>> downloads; // D2H after an op
  std::vector<cuda_op_t*> order;  // CUDA operators in execution order
  std::vector<void*> pinned;      // page-locked host buffers of graph inputs / outputs
  bool all_device = false;

  // graph mode
  int run_index = 0;
  int phase = 0;  // 0 eager, 1 capturing, 2 replaying
  void* graph_exec = nullptr;

  backend_stats_t stats;

  ~device_state_t();
  tensor_t* resolve(tensor_t* t) const;
  void* dev(tensor_t* t);  // device pointer of a tensor (after setup)
  bool setup();
  void invalidate();
  bool fail(const char* fmt, ...);
};

device_state_t* state_of(context_t* ctx);   // creates on first use
device_state_t* find_state(context_t* ctx); // or nullptr
void release_state(context_t* ctx);

// Base of every CUDA operator.
struct cuda_op_t : operator_t {
  device_state_t* st() const { return state_of(ctx); }
  bool exec() final;
  bool reshape() final;
  // shape inference (host-side, no device work)
  virtual bool infer_shape() = 0;
  // device work for one run; the base class did the uploads and does the
  // downloads. Layout of inputs: st()->dev_layout; outputs must be written
  // in the layout the op records with set_out_layout().
  virtual bool run_device(device_state_t& s, void* stream) = 0;
  // whether input idx is read on the device (others, such as scales and
  // weights, are read on the host when the op prepares)
  virtual bool device_input(int idx) const { return idx == 0; }
  // device workspace this op needs (after prepare_device)
  virtual size_t device_workspace() const { return 0; }
  // one-time device preparation once layouts are final (weight packing and
  // upload). Called by setup(), in execution order.
  virtual bool prepare_device(device_state_t& s) { return true; }
  // whether this instance (its types, shapes, attributes) runs on the device
  virtual bool device_ok() const { return true; }
  // glue operators whose variant the device does not handle (an fp32
  // MaxPool, a broadcasting Add, ...) run nnr's CPU operator instead; the
  // conv/GEMM operators never do: their exec() fails with a message
  virtual bool host_allowed() const { return false; }
  bool on_host = false;  // decided by setup()
  // true when every input is a constant: nnr is folding this node at load
  // time (fold_run), which runs on the host through nnr's own CPU operator
  bool inputs_constant() const;
  bool fold_on_host();  // also runs host_allowed variants
  void set_out_layout(device_state_t& s, tensor_t* t, memory_layout_t l) { s.dev_layout[s.resolve(t)] = l; }
  memory_layout_t in_layout(device_state_t& s, tensor_t* t) const { return s.dev_layout[s.resolve(t)]; }
  operator_t* host_twin = nullptr;  // nnr's CPU operator, for constant folding only
};

// attribute helpers
int64_t ints_attr(operator_t* op, attr_key_t key, std::vector<int64_t>& out);
float scalar_f32(const tensor_t* t, float def);
int scalar_zp(const tensor_t* t);

bool nnrcu_ok(device_state_t& s, int rc, const char* what);

}  // namespace nnr::cuda
