"""Host logic of the device arena (lifetime-based slot packing), no GPU."""
import numpy as np
import pytest

from nnr_b200.graph import Interval, check_plan, plan_arena


def test_disjoint_lifetimes_share_memory():
    items = [Interval("a", 1000, 0, 1), Interval("b", 1000, 2, 3), Interval("c", 1000, 4, 5)]
    offs, total = plan_arena(items)
    check_plan(items, offs)
    assert total == 1024  # all three reuse one slot


def test_overlapping_lifetimes_do_not_overlap_in_memory():
    items = [Interval("a", 1000, 0, 2), Interval("b", 500, 1, 3), Interval("c", 300, 2, 2)]
    offs, total = plan_arena(items)
    check_plan(items, offs)
    assert total >= 1024 + 512 + 512


@pytest.mark.parametrize("seed", range(20))
def test_random_plans_are_valid_and_not_worse_than_peak_x2(seed):
    rng = np.random.default_rng(seed)
    items = []
    for i in range(60):
        a = int(rng.integers(0, 40))
        items.append(Interval(f"t{i}", int(rng.integers(1, 5000)), a, a + int(rng.integers(0, 8))))
    offs, total = plan_arena(items)
    check_plan(items, offs)
    peak = max(sum((it.nbytes + 255) // 256 * 256 for it in items if it.first <= s <= it.last) for s in range(50))
    assert peak <= total <= 2 * peak


def test_resnet50_arena_is_far_below_sum_of_tensors():
    """The planned ResNet-50 (batch 32) arena reuses memory across layers."""
    from nnr_b200 import resnet50
    m = resnet50.build(batch=32)
    first, last = {"input": -1}, {}
    for i, nd in enumerate(m.nodes):
        first.setdefault(nd.output, i)
        for x in nd.inputs:
            last[x] = i
    last["logits"] = len(m.nodes)
    def nb(n):
        return int(np.prod(m.shapes[n])) * (4 if n in ("input", "logits") else 1)
    items = [Interval(n, nb(n), first[n], last.get(n, first[n])) for n in first]
    offs, total = plan_arena(items)
    check_plan(items, offs)
    assert total < 0.3 * sum(nb(n) for n in first)
