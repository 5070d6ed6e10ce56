"""nnr's own loader, passes and run loop driving the CUDA backend
(nnr_b200/nnr_backend, built with nnr into libnnr_cuda.so).

CPU part (no GPU needed: nnr's load and prepare do no device work):
- config 4 written as a QDQ ONNX graph goes through nnr's fuse_qdq_compute
  and fuse_qdq: 53 QLinearConv, 16 QLinearAdd, one QLinearMatMul, MaxPool on
  u8, every active operator a CUDA operator (only the Flatten view on the
  host);
- layout assignment with the backend's device cost keeps the int8 chain NHWC
  (assign_layouts.cpp): every QLinearConv, QLinearAdd and MaxPool output is
  NHWC, so no host reorder can touch device data.
GPU part (marked gpu):
- config 4 through nnr's context_t on the device, bit-exact against the
  oracle's QDQ network (every layer's formula follows from the layouts nnr
  assigned), eager, captured and replayed runs, batch 2 and 32;
- config 5 (MobileNetV2) through nnr on the device within the fp32 bound;
- config 1 and a config-3 Gemm slice through nnr on the device.
"""
import collections

import numpy as np
import pytest

from nnr_b200 import nnr_cuda as NC

pytestmark = pytest.mark.skipif(not NC.available(), reason="libnnr_cuda.so not built (needs the nnr sources)")


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def r50_small():
    from nnr_b200 import resnet50
    return resnet50.build(batch=2)


def test_resnet50_qdq_fusion_and_layouts(r50_small):
    from nnr_b200 import onnx_models as M
    net = NC.NnrCudaModel(M.resnet50_qdq(r50_small))
    try:
        act = net.active()
        ops = collections.Counter(o for o, *_ in act)
        assert ops["QLinearConv"] == 53 and ops["QLinearAdd"] == 16 and ops["QLinearMatMul"] == 1
        assert ops["MaxPool"] == 1 and "Conv" not in ops and "MatMul" not in ops
        host = [o for o, s, f, dev, fmt in act if not dev]
        assert host == ["Flatten"], host
        for o, s, f, dev, fmt in act:
            if o in ("QLinearConv", "QLinearAdd", "MaxPool"):
                assert fmt == NC.NHWC, f"{o} output left NCHW"
    finally:
        net.close()


def test_mobilenetv2_graph_on_device():
    from nnr_b200 import mobilenetv2 as MB
    from nnr_b200 import onnx_models as M
    net = NC.NnrCudaModel(M.mobilenetv2(MB.build(batch=1)))
    try:
        act = net.active()
        ops = collections.Counter(o for o, *_ in act)
        assert ops["Conv"] == 52 and "Clip" not in ops  # Clip(0, 6) fused as the conv epilogue
        assert [o for o, s, f, dev, fmt in act if not dev] == ["Flatten"]
    finally:
        net.close()


# ------------------------------------------------------------------ on the device
@pytest.mark.gpu
@pytest.mark.parametrize("batch,planning", [(2, True), (32, True), (32, False)])
def test_resnet50_through_nnr_bit_exact(cuda_dev, batch, planning):
    """nnr's run loop on the device gives the oracle's logits exactly, in the
    eager first run, the captured second run and replayed runs, with nnr's
    memory planner (device slots keyed by its planned host buffers) and
    without it."""
    from nnr_b200 import onnx_models as M
    from nnr_b200 import resnet50
    from oracle import oracle as O
    model = resnet50.build(batch=batch)
    net = NC.NnrCudaModel(M.resnet50_qdq(model), memory_planning=planning)
    try:
        for i in range(4):
            x = resnet50.input_batch(batch * i, batch)
            net.set("input", x)
            net.run()
            got = net.get("logits")
            want = O.run_qmodel(model, x)
            assert np.array_equal(got, want), f"run {i}: {(got != want).sum()} logits differ"
        st = net.stats()
        assert st["host_ops"] == 0 and st["host_glue"] == 0  # (the Flatten view is not an operator run)
        assert st["graph_replays"] == 2
        assert st["h2d_bytes"] == 4 * x.nbytes and st["d2h_bytes"] == 4 * batch * 1000 * 4
    finally:
        net.close()


@pytest.mark.gpu
def test_mobilenetv2_through_nnr(cuda_dev):
    from nnr_b200 import mobilenetv2 as MB
    from nnr_b200 import onnx_models as M
    from oracle import oracle as O
    model = MB.build(batch=4)
    x = MB.input_batch(0, 4)
    net = NC.NnrCudaModel(M.mobilenetv2(model))
    try:
        ref = O.run_fmodel(model, x)
        for _ in range(3):
            net.set("input", x)
            net.run()
            assert rel(net.get("logits"), ref) <= 1e-3
        assert net.stats()["graph_replays"] == 1
    finally:
        net.close()


@pytest.mark.gpu
def test_config1_and_gemm_through_nnr(cuda_dev):
    from nnr_b200 import onnx_models as M
    from nnr_b200 import workloads as W
    from oracle import oracle as O
    c = W.config1_conv_relu()
    net = NC.NnrCudaModel(M.conv(c.x.shape, c.w, c.bias, pads=c.pads, post="Relu"))
    try:
        net.set("x", c.x)
        net.run()
        assert rel(net.get("y"), O.conv_f32(c.x, c.w, c.bias, pads=c.pads, post=1)) <= 1e-4
    finally:
        net.close()
    c3 = W.config3_matmul()
    a = c3.a_f32[:256]
    net = NC.NnrCudaModel(M.gemm(256, 768, 3072, c3.b_f32, c3.c_f32))
    try:
        net.set("a", a)
        net.run()
        assert rel(net.get("y"), O.gemm_f32(a, c3.b_f32, c3.c_f32)) <= 1e-4
    finally:
        net.close()


@pytest.mark.gpu
def test_unsupported_variant_fails_loudly(cuda_dev):
    """A QLinearConv with non-zero weight zero points has no device path; the
    run fails with a message instead of running elsewhere."""
    from nnr_b200 import onnx_pb as P
    g = P.Graph("qconv_wzp")
    g.input("x", P.UINT8, (1, 8, 6, 6))
    xs, xz = g.scalar(np.float32(0.1)), g.scalar(np.uint8(3))
    g.node("DequantizeLinear", ["x", xs, xz], ["xd"])
    g.init("w", np.ones((8, 8, 3, 3), np.int8))
    g.init("ws", np.float32(0.01))
    g.init("wz", np.int8(5))
    g.node("DequantizeLinear", ["w", "ws", "wz"], ["wd"])
    g.node("Conv", ["xd", "wd"], ["c"], kernel_shape=[3, 3], pads=[1, 1, 1, 1])
    g.node("QuantizeLinear", ["c", g.scalar(np.float32(0.2)), g.scalar(np.uint8(0))], ["y"])
    g.output("y", P.UINT8, (1, 8, 6, 6))
    net = NC.NnrCudaModel(g.model())
    try:
        net.set("x", np.zeros((1, 8, 6, 6), np.uint8))
        with pytest.raises(RuntimeError):
            net.run()
        assert net.error()
    finally:
        net.close()


@pytest.mark.gpu
def test_16bit_and_matmul_through_nnr(cuda_dev):
    """bf16 / fp16 Conv and Gemm graphs through nnr on the device (nnr's
    16-bit paths: fp32 compute, rounded back; within one ulp of the oracle
    plus fp32 summation error), and an fp32 MatMul that follows nnr's own
    precision on this host (bf16-rounded operands with AVX-512 BF16)."""
    import importlib.util
    from pathlib import Path

    from nnr_b200 import onnx_models as M
    from oracle import oracle as O
    spec = importlib.util.spec_from_file_location("g", Path(__file__).parent / "golden" / "make_nnr_golden.py")
    G = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(G)
    rng = np.random.default_rng(11)
    for et in (16, 10):
        xb = G.to_bits16(rng.uniform(-1, 1, (2, 32, 10, 10)), et)
        wb = G.to_bits16(rng.normal(0, 0.2, (48, 32, 3, 3)), et)
        bb = G.to_bits16(rng.normal(0, 0.1, 48), et)
        net = NC.NnrCudaModel(M.conv_half(xb.shape, wb, bb, et, pads=(1, 1, 1, 1), post="Relu"))
        try:
            assert [o for o, s, f, dev, fmt in net.active() if not dev] == []
            net.set("x", xb)
            net.run()
            got = G.bits16_to_f32(net.get("y").view(np.uint16), et)
            f = {k: G.bits16_to_f32(v, et) for k, v in (("x", xb), ("w", wb), ("b", bb))}
            ref = G.bits16_to_f32(G.to_bits16(O.conv_f32(f["x"], f["w"], f["b"], pads=(1, 1, 1, 1), post=1), et), et)
            tol = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - (10 if et == 10 else 7))
            absum = O.conv_f32(np.abs(f["x"]), np.abs(f["w"]), np.abs(f["b"]), pads=(1, 1, 1, 1))
            assert np.all(np.abs(got - ref) <= tol * 1.0001 + 1e-5 * absum)
        finally:
            net.close()
    a = rng.normal(0, 1, (40, 96)).astype(np.float32)
    b = rng.normal(0, 0.1, (96, 70)).astype(np.float32)
    net = NC.NnrCudaModel(M.matmul(a.shape, b))
    try:
        net.set("a", a)
        net.run()
        got = net.get("y")
        want = O.matmul_f32_bf16_host(a, b) if "avx512_bf16" in Path("/proc/cpuinfo").read_text() \
            else O.gemm_f32(a, b, None, beta=0.0)
        assert rel(got, want) <= 1e-5
    finally:
        net.close()


@pytest.mark.gpu
def test_s8_activation_qlinearconv_declined_loudly(cuda_dev):
    """A QDQ Conv on s8 activations fuses to a QLinearConv that the device
    does not implement (its requant and padding differ from the u8 path):
    the run fails with a message instead of computing something else."""
    from nnr_b200 import onnx_pb as P
    g = P.Graph("qconv_s8")
    g.input("x", P.INT8, (1, 8, 6, 6))
    g.node("DequantizeLinear", ["x", g.scalar(np.float32(0.1)), g.scalar(np.int8(0))], ["xd"])
    g.init("w", np.ones((8, 8, 3, 3), np.int8))
    g.node("DequantizeLinear", ["w", g.scalar(np.float32(0.01)), g.scalar(np.int8(0))], ["wd"])
    g.node("Conv", ["xd", "wd"], ["c"], kernel_shape=[3, 3], pads=[1, 1, 1, 1])
    g.node("QuantizeLinear", ["c", g.scalar(np.float32(0.2)), g.scalar(np.int8(0))], ["y"])
    g.output("y", P.INT8, (1, 8, 6, 6))
    net = NC.NnrCudaModel(g.model())
    try:
        assert [n[0] for n in net.active()] == ["QLinearConv"]
        net.set("x", np.zeros((1, 8, 6, 6), np.int8))
        with pytest.raises(RuntimeError):
            net.run()
        assert "not supported on the device" in net.error()
    finally:
        net.close()
