// Stand-ins for the three nnr CPU operators that cannot be compiled without
// the Xbyak JIT (absent from the nnr checkout): QLinearConv, QLinearMatMul
// and MatMulInteger. Returning nullptr is nnr's own "decline" (registry.cpp:
// solve returns nullptr; fuse_qdq_compute.cpp:143-144 then keeps the float
// DQ -> Conv/MatMul -> Q subgraph). Test infrastructure only.
#include "nnr.h"

namespace nnr {
operator_t* resolver_default_op_QLinearConv(int, pool_t&) { return nullptr; }
operator_t* resolver_default_op_QLinearMatMul(int, pool_t&) { return nullptr; }
operator_t* resolver_default_op_MatMulInteger(int, pool_t&) { return nullptr; }
}  // namespace nnr
