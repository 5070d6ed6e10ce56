// nnr's CPU QLinearConv, QLinearMatMul and MatMulInteger are built on the
// Xbyak JIT, which this build does not have; their CPU resolvers decline
// (nullptr, registry.cpp's "not available" answer). With preferred_backend
// CUDA the CUDA operators of this backend are chosen first anyway
// (registry.cpp:14-20); these stand-ins only satisfy the CPU registrar's
// references (backend/cpu/solve_operator.cpp:9-11).
#include "nnr.h"

namespace nnr {
operator_t* resolver_default_op_QLinearConv(int, pool_t&) { return nullptr; }
operator_t* resolver_default_op_QLinearMatMul(int, pool_t&) { return nullptr; }
operator_t* resolver_default_op_MatMulInteger(int, pool_t&) { return nullptr; }
}  // namespace nnr
