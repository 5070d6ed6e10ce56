"""MatMul with both operands computed at run time (nnr's MatMul_operator with
a non-initializer B: MatMul.cpp:32-94 shapes and broadcast strides, :194-228
exec), through nnrcu_matmul_f32_run and through nnr's own run loop on the
device. fp32 results must be within 1e-5 relative L2 of the fp64 product
(split-bf16 drops only the lo x lo term)."""
import numpy as np
import pytest

from nnr_b200 import ops

SHAPES = [
    # a shape, b shape
    ((33, 40), (40, 50)),                 # plain 2-D
    ((2, 3, 17, 64), (2, 3, 64, 24)),     # batched, same batch dims
    ((4, 1, 17, 24), (3, 24, 9)),         # broadcast both ways
    ((5, 70, 96), (96, 130)),             # 2-D B under a batched A
    ((64,), (64, 20)),                    # 1-D A
    ((3, 12, 40), (40,)),                 # 1-D B
    ((1, 12, 128, 64), (1, 12, 64, 128)), # attention scores shape
]


def _ref(a, b):
    return np.matmul(a.astype(np.float64), b.astype(np.float64))


@pytest.mark.parametrize("shapes", SHAPES)
def test_broadcast_shapes_follow_nnr(shapes):
    a_shape, b_shape = shapes
    shape, m, n, k, offs = ops.matmul_broadcast(a_shape, b_shape)
    a = np.arange(np.prod(a_shape), dtype=np.float64).reshape(a_shape) % 7 - 3
    b = np.arange(np.prod(b_shape), dtype=np.float64).reshape(b_shape) % 5 - 2
    # nnr keeps the unit dims of 1-D operands: compare on the element set
    want = np.matmul(a.reshape((1,) + a_shape) if len(a_shape) == 1 else a,
                     b.reshape(b_shape + (1,)) if len(b_shape) == 1 else b)
    assert int(np.prod(shape)) == want.size
    af, bf = a.ravel(), b.ravel()
    got = np.stack([af[ao:ao + m * k].reshape(m, k) @ bf[bo:bo + k * n].reshape(k, n) for ao, bo in offs])
    assert np.array_equal(got.ravel(), want.ravel())


@pytest.mark.gpu
@pytest.mark.parametrize("shapes", SHAPES)
@pytest.mark.parametrize("post", [None, "Relu"])
def test_matmul_dynamic_device(cuda_dev, shapes, post):
    import torch
    a_shape, b_shape = shapes
    rng = np.random.default_rng(sum(a_shape) + sum(b_shape))
    a = rng.normal(0, 1, a_shape).astype(np.float32)
    b = rng.normal(0, 0.2, b_shape).astype(np.float32)
    y = ops.matmul_f32(torch.from_numpy(a).to(cuda_dev), torch.from_numpy(b).to(cuda_dev), post=post)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    want = _ref(a.reshape((1,) + a_shape) if len(a_shape) == 1 else a,
                b.reshape(b_shape + (1,)) if len(b_shape) == 1 else b)
    if post == "Relu":
        want = np.maximum(want, 0)
    got = y.cpu().numpy().astype(np.float64).ravel()
    assert np.linalg.norm(got - want.ravel()) <= 1e-5 * np.linalg.norm(want)


@pytest.mark.gpu
@pytest.mark.parametrize("shapes", [SHAPES[1], SHAPES[2], SHAPES[6]])
def test_matmul_dynamic_through_nnr(cuda_dev, shapes):
    """nnr's loader and run loop with the CUDA backend: a MatMul of two graph
    inputs (+ fused Relu) runs on the device and matches nnr's CPU runtime."""
    from nnr_b200 import nnr_cuda as NC, onnx_models as M
    from oracle import nnr_ref as R
    if not NC.available():
        pytest.skip("libnnr_cuda.so not built")
    a_shape, b_shape = shapes
    y_shape, *_ = ops.matmul_broadcast(a_shape, b_shape)
    rng = np.random.default_rng(7)
    a = rng.normal(0, 1, a_shape).astype(np.float32)
    b = rng.normal(0, 0.2, b_shape).astype(np.float32)
    model = M.matmul_dynamic(a_shape, b_shape, y_shape, post="Relu")
    net = NC.NnrCudaModel(model)
    try:
        assert any(o == "MatMul" and dev for o, _, _, dev, _ in net.nodes())
        net.set("a", a)
        net.set("b", b)
        net.run()
        got = net.get("y").astype(np.float64)
    finally:
        net.close()
    want = np.maximum(_ref(a, b), 0)
    assert np.linalg.norm(got - want) <= 1e-5 * np.linalg.norm(want)
    if R.available():
        cpu = R.NnrModel(model)
        cpu.set("a", a)
        cpu.set("b", b)
        cpu.run()
        nn = cpu.get("y").astype(np.float64)
        assert np.linalg.norm(got - nn) <= 2e-5 * np.linalg.norm(nn)


def _bits(x, dtype):
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("mng", Path(__file__).parent / "golden" / "make_nnr_golden.py")
    g = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(g)
    return g


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("shapes", [SHAPES[1], SHAPES[2], SHAPES[6]])
def test_matmul_dynamic_half(cuda_dev, dtype, shapes):
    """16-bit run-time MatMul: every result within one unit in the last place
    of the fp64 product rounded to the type, plus the fp32 summation error
    (1e-5 of the sum of |terms|), as nnr's 16-bit paths (fp32 compute)."""
    import torch
    G = _bits(None, None)
    et = 16 if dtype == "bf16" else 10
    a_shape, b_shape = shapes
    rng = np.random.default_rng(sum(a_shape))
    ab = G.to_bits16(rng.normal(0, 1, a_shape), et)
    bb = G.to_bits16(rng.normal(0, 0.2, b_shape), et)
    af, bf = G.bits16_to_f32(ab, et).astype(np.float64), G.bits16_to_f32(bb, et).astype(np.float64)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    at = torch.from_numpy(ab.view(np.int16)).to(cuda_dev).view(tdt)
    bt = torch.from_numpy(bb.view(np.int16)).to(cuda_dev).view(tdt)
    y = ops.matmul_half(at, bt, post="Relu")
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    got = G.bits16_to_f32(y.contiguous().view(torch.int16).cpu().numpy().view(np.uint16), et).astype(np.float64)
    want = np.maximum(np.matmul(af, bf), 0)
    abs_sum = np.matmul(np.abs(af), np.abs(bf))
    wb = G.bits16_to_f32(G.to_bits16(want, et), et).astype(np.float64)
    mant = 10 if et == 10 else 7
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(wb), 1e-30))) - mant)
    assert int((np.abs(got - wb) > ulp * 1.0001 + 1e-5 * abs_sum).sum()) == 0


@pytest.mark.gpu
def test_matmul_dynamic_half_through_nnr(cuda_dev):
    """An fp16 MatMul of two graph inputs through nnr's run loop on the device,
    against nnr's own CPU runtime (fp32 compute, rounded to fp16): within one
    fp16 ulp plus the fp32 summation error."""
    from nnr_b200 import nnr_cuda as NC, onnx_models as M, onnx_pb as P
    from oracle import nnr_ref as R
    if not (NC.available() and R.available()):
        pytest.skip("nnr libraries not built")
    G = _bits(None, None)
    a_shape, b_shape = (2, 3, 17, 64), (2, 3, 64, 24)
    y_shape, *_ = ops.matmul_broadcast(a_shape, b_shape)
    rng = np.random.default_rng(9)
    a = rng.normal(0, 1, a_shape).astype(np.float16)
    b = rng.normal(0, 0.2, b_shape).astype(np.float16)
    model = M.matmul_dynamic(a_shape, b_shape, y_shape, elem=P.FLOAT16)
    net = NC.NnrCudaModel(model)
    try:
        assert any(o == "MatMul" and dev for o, _, _, dev, _ in net.nodes())
        net.set("a", a)
        net.set("b", b)
        net.run()
        got = G.bits16_to_f32(net.get("y"), 10).astype(np.float64)
    finally:
        net.close()
    cpu = R.NnrModel(model)
    cpu.set("a", a)
    cpu.set("b", b)
    cpu.run()
    nn = G.bits16_to_f32(np.asarray(cpu.get("y")).view(np.uint16), 10).astype(np.float64)
    abs_sum = np.matmul(np.abs(a.astype(np.float64)), np.abs(b.astype(np.float64)))
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(nn), 1e-30))) - 10)
    assert int((np.abs(got - nn) > ulp * 1.0001 + 1e-5 * abs_sum).sum()) == 0
