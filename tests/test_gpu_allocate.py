"""dkv_allocate_rungs (the per-token rung allocator on the GPU) against the reference's own counts
(tests/golden/allocator.npz) and against the reference's sort-based arithmetic (the host path of
dimmerkv.kvtc.allocate_rungs) on random cases with many ties, at several level counts and budgets."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dimmerkv.allocate import allocate_rungs_gpu
from dimmerkv.kvtc import allocate_rungs

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def test_allocator_matches_reference_fixture(golden):
    g = golden("allocator")
    errors = torch.from_numpy(g["errors"])
    got = allocate_rungs_gpu(errors.to(DEV), torch.from_numpy(g["level_bytes"]), int(g["middle"]), int(g["budget"]))
    assert np.array_equal(got.cpu().numpy(), g["chosen"])
    # The drop-in dispatches CUDA float32 errors to the kernel.
    again = allocate_rungs(errors.to(DEV), torch.from_numpy(g["level_bytes"]).to(DEV), int(g["middle"]), int(g["budget"]))
    assert np.array_equal(again.cpu().numpy(), g["chosen"])


@pytest.mark.parametrize("slots,levels,ties", [(200, 2, False), (1000, 6, True), (40000, 12, True),
                                                (7002, 33, False), (5000, 12, "flat")])
def test_allocator_matches_host_arithmetic(slots, levels, ties):
    rng = np.random.default_rng(slots + levels)
    middle = slots // 2  # keys then values, middle slots each (the reference's layout)
    e = rng.random((slots, levels)).astype(np.float32)
    if ties is True:
        e = np.round(e * 8) / 8  # few distinct gains: large tie groups
    e = -np.sort(-e, axis=1)
    if ties == "flat":
        e[: slots // 3] = e[: slots // 3, :1]  # no gain at all: value 0 for a third of the slots
    sizes_k = np.cumsum(rng.integers(1, 40, size=levels))
    sizes_v = np.cumsum(rng.integers(1, 40, size=levels))
    level_bytes = torch.tensor(np.concatenate([sizes_k, sizes_v]), dtype=torch.int64)
    base = middle * int(sizes_k[0]) + (slots - middle) * int(sizes_v[0])
    full = middle * int(sizes_k[-1]) + (slots - middle) * int(sizes_v[-1])
    errors = torch.from_numpy(e)
    for budget in (base, base + 1, base + (full - base) // 3, (base + full) // 2, full - 1, full, full + 1000):
        want = allocate_rungs(errors, level_bytes, middle, budget)  # host: the reference's sort and cumsum
        got = allocate_rungs_gpu(errors.to(DEV), level_bytes, middle, budget)
        assert torch.equal(got.cpu(), want), budget


def test_allocator_rejects_budget_below_the_coarsest_rungs():
    errors = torch.rand(10, 4, device=DEV)
    with pytest.raises(ValueError, match="coarsest"):
        allocate_rungs_gpu(errors, torch.tensor([10, 20, 30, 40, 10, 20, 30, 40]), 5, 99)


def test_allocator_reports_non_growing_levels():
    errors = torch.rand(10, 3, device=DEV)
    with pytest.raises(Exception, match="descriptor"):
        allocate_rungs_gpu(errors, torch.tensor([10, 10, 30, 10, 20, 30]), 5, 1000)
