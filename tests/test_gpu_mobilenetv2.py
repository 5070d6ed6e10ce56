"""MobileNetV2 fp32 on the device vs the CPU oracle.

Each operator alone meets the north star's fp32 bound (1e-4 L2-normalised
relative error, test_gpu_fp32.py). Through the 52 convs of the network the
split-bf16 errors compound, so whole-network tensors are held to 1e-3 (the
measured figure is printed; it is a few 1e-5 for most tensors).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

NET_TOL = 1e-3


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def net_and_ref():
    from nnr_b200 import fgraph, mobilenetv2 as M
    model = M.build(batch=2)
    x = M.input_batch(0, 2)
    net = fgraph.FloatNetwork(model, 0, reuse=False, split_links=False)
    net.view("input").copy_(torch.from_numpy(x))
    net.run()
    torch.cuda.synchronize()
    logits, ref = O.run_fmodel(model, x, keep=True)
    yield model, net, x, ref
    net.close()


def test_every_tensor_close(net_and_ref):
    from nnr_b200 import ops
    model, net, _, ref = net_and_ref
    assert ops.device_status() == 0
    worst = (0.0, None)
    for nd in model.nodes:
        if nd.output in net.fused_away:
            continue
        e = rel(net.view(nd.output).cpu().numpy(), ref[nd.output])
        worst = max(worst, (e, nd.output))
    print(f"worst relative L2 error {worst[0]:.2e} at {worst[1]}")
    assert worst[0] <= NET_TOL, worst


def test_split_links_bit_identical(net_and_ref):
    """The network with its depthwise -> projection pairs linked through
    split-bf16 planes computes every remaining tensor bit-identically."""
    from nnr_b200 import fgraph, ops
    model, net, x, _ = net_and_ref
    n2 = fgraph.FloatNetwork(model, 0, reuse=False)
    try:
        assert len(n2.plane_links) == 17  # one per inverted-residual block
        n2.view("input").copy_(torch.from_numpy(x))
        n2.run()
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        for nd in model.nodes:
            if nd.output in net.fused_away or nd.output in n2.plane_links:
                continue
            a = n2.view(nd.output).cpu().numpy()
            b = net.view(nd.output).cpu().numpy()
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), nd.output
    finally:
        n2.close()


def test_graph_replay_and_host_path(net_and_ref):
    from nnr_b200 import fgraph, mobilenetv2 as M
    model, net, x, ref = net_and_ref
    n2 = fgraph.FloatNetwork(model, 0)
    try:
        n2.capture()
        out = n2.forward(torch.from_numpy(x).pin_memory())
        n2.stream.synchronize()
        assert rel(out.numpy(), ref["logits"]) <= NET_TOL
        assert np.array_equal(out.numpy(), net.view("logits").cpu().numpy())
    finally:
        n2.close()


OP_TOL = 1e-4  # the north star's fp32 bound, per operator


@pytest.fixture(scope="module")
def bench_net_and_ref():
    """The configuration bench.py times: batch 128 (rank 0's shard)."""
    from nnr_b200 import fgraph, mobilenetv2 as M
    model = M.build(batch=128)
    x = M.input_batch(0, 128)
    logits, ref = O.run_fmodel(model, x, keep=True)
    net = fgraph.FloatNetwork(model, 0, reuse=False, split_links=False)
    yield model, net, x, ref
    net.close()


def test_bench_batch_every_op_within_1e4(bench_net_and_ref):
    """Each device step (Conv, Conv + fused residual Add, GlobalAveragePool,
    Gemm) is fed the oracle's own input tensors and must reproduce the
    oracle's output within 1e-4 relative L2: per-operator error, without the
    compounding of 52 layers."""
    from nnr_b200 import ops
    model, net, _, ref = bench_net_and_ref
    worst = (0.0, None)
    for t, (kind, j, ins, out, i) in enumerate(net.steps):
        for name in ins:
            net.view(name).copy_(torch.from_numpy(ref[name]))
        net.run_step(t)
        net.stream.synchronize()
        e = rel(net.view(out).cpu().numpy(), ref[out])
        worst = max(worst, (e, f"{kind} {out}"))
        assert e <= OP_TOL, (kind, out, e)
    assert ops.device_status() == 0
    print(f"worst per-op relative L2 error {worst[0]:.2e} at {worst[1]}")


def test_bench_batch_whole_network(bench_net_and_ref):
    """The same batch end to end through the captured graph (the bench's
    launch path): every tensor within the compounded-network bound."""
    from nnr_b200 import fgraph, ops
    model, net, x, ref = bench_net_and_ref
    net.view("input").copy_(torch.from_numpy(x))
    net.run()
    torch.cuda.synchronize()
    worst = (0.0, None)
    for nd in model.nodes:
        if nd.output in net.fused_away:
            continue
        worst = max(worst, (rel(net.view(nd.output).cpu().numpy(), ref[nd.output]), nd.output))
    print(f"batch 128: worst relative L2 error {worst[0]:.2e} at {worst[1]}")
    assert worst[0] <= NET_TOL, worst
    n2 = fgraph.FloatNetwork(model, 0)
    try:
        n2.capture()
        out = n2.forward(torch.from_numpy(x).pin_memory())
        n2.stream.synchronize()
        assert ops.device_status() == 0
        assert np.array_equal(out.numpy(), net.view("logits").cpu().numpy())
    finally:
        n2.close()
