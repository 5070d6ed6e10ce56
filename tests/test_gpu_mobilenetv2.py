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
    net = fgraph.FloatNetwork(model, 0, reuse=False)
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
