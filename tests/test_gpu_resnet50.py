"""ResNet-50 v1 QDQ int8 end to end on the device vs the
CPU oracle: the fp32 logits after the last DequantizeLinear + Add must be
identical (every op on the path is integer or performs nnr's float
operations in nnr's order), and so must every intermediate u8 tensor."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model4():
    from nnr_b200 import resnet50
    return resnet50.build(batch=4)


def test_resnet50_qdq_bit_exact(cuda_dev, model4):
    from nnr_b200 import graph, ops, resnet50
    x = resnet50.input_batch(0, 4)
    ref, tensors = O.run_qmodel(model4, x, keep=True)
    net = graph.DeviceNetwork(model4, 0, reuse=False)
    net.view("input").copy_(torch.from_numpy(x))
    net.run()
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for nd in model4.nodes:  # first divergent layer, if any
        if nd.output == "logits" or nd.output in net.fused_away:
            continue
        got = net.view(nd.output).cpu().numpy()
        want = tensors[nd.output]
        assert np.array_equal(got, want), f"{nd.op} {nd.output}: {(got != want).sum()} of {want.size} differ"
    got = net.view("logits").cpu().numpy()
    assert np.array_equal(got, ref)


def test_resnet50_unfused_add_path(cuda_dev, model4):
    """Without the conv+add fusion (separate QLinearAdd kernels) the logits are the same."""
    from nnr_b200 import graph, resnet50
    x = resnet50.input_batch(0, 4)
    ref = O.run_qmodel(model4, x)
    net = graph.DeviceNetwork(model4, 0, fuse_add=False)
    net.view("input").copy_(torch.from_numpy(x))
    net.run()
    torch.cuda.synchronize()
    assert not net.fused_away
    assert np.array_equal(net.view("logits").cpu().numpy(), ref)


def test_resnet50_graph_replay_and_host_path(cuda_dev, model4):
    """Captured CUDA graph + host input/output path give the same logits."""
    from nnr_b200 import graph, resnet50
    x = resnet50.input_batch(4, 4)
    ref = O.run_qmodel(model4, x)
    net = graph.DeviceNetwork(model4, 0)
    net.capture()
    xh = torch.from_numpy(x).pin_memory()
    for _ in range(2):
        out = net.forward(xh)
        net.stream.synchronize()
        assert np.array_equal(out.numpy(), ref)
    net.close()


def test_resnet50_pipelined_forwards(cuda_dev, model4):
    """DeviceNetwork.forward_many (input copies overlapped with the previous
    forward) gives each batch the same logits as a lone forward."""
    from nnr_b200 import graph, resnet50
    net = graph.DeviceNetwork(model4, 0)
    try:
        net.capture()
        xs = [torch.from_numpy(resnet50.input_batch(4 * i, 4)).pin_memory() for i in range(3)]
        outs = [torch.empty(model4.shapes["logits"], dtype=torch.float32).pin_memory() for _ in range(3)]
        net.forward_many(xs, outs)
        net.stream.synchronize()
        for x, o in zip(xs, outs):
            ref = net.forward(x)
            net.stream.synchronize()
            assert torch.equal(o, ref)
    finally:
        net.close()


@pytest.fixture(scope="module")
def model32():
    from nnr_b200 import resnet50
    return resnet50.build(batch=32)


def test_resnet50_bench_configuration_bit_exact(cuda_dev, model32):
    """The configuration bench.py times: batch 32 (rank 0's shard of the
    256-image batch), the planned arena with reuse, the captured CUDA graph.
    Every intermediate tensor (arena without reuse, so each stays readable)
    and the logits of the captured, reusing network are bit-exact against the
    oracle."""
    from nnr_b200 import graph, ops, resnet50
    x = resnet50.input_batch(0, 32)
    ref, tensors = O.run_qmodel(model32, x, keep=True)
    net = graph.DeviceNetwork(model32, 0, reuse=False)
    try:
        net.view("input").copy_(torch.from_numpy(x))
        net.run()
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        for nd in model32.nodes:
            if nd.output == "logits" or nd.output in net.fused_away:
                continue
            got = net.view(nd.output).cpu().numpy()
            want = tensors[nd.output]
            assert np.array_equal(got, want), f"{nd.op} {nd.output}: {(got != want).sum()} of {want.size} differ"
        assert np.array_equal(net.view("logits").cpu().numpy(), ref)
    finally:
        net.close()
    bench_net = graph.DeviceNetwork(model32, 0)
    try:
        bench_net.capture()
        out = bench_net.forward(torch.from_numpy(x).pin_memory())
        bench_net.stream.synchronize()
        assert ops.device_status() == 0
        assert np.array_equal(out.numpy(), ref)
    finally:
        bench_net.close()
