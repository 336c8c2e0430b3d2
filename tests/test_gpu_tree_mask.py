"""build_tree_mask on the GPU against the reference's masks (golden)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import projectgorgon_b200 as G
from conftest import load_golden
from oracle import gorgon_oracle as O

pytestmark = pytest.mark.gpu
MASKS = load_golden("tree_mask")


@pytest.mark.parametrize("name", list(MASKS["names"]))
@pytest.mark.parametrize("depth", [None, 1, 2, 3, 5])
def test_tree_mask_bit_exact(name, depth):
    par = [int(x) for x in MASKS[f"{name}_parents"]]
    key = "none" if depth is None else str(depth)
    got = G.build_tree_mask(par, depth)
    assert got.is_cuda and got.dtype == torch.bool
    np.testing.assert_array_equal(got.cpu().numpy(), MASKS[f"{name}_mask_{key}"])


def test_reference_small_case():
    mask = G.build_tree_mask([-1, 0, 0])
    assert bool(mask[1, 2]) is False
    assert bool(mask[1, 0]) is True


def test_best_first_256_and_batched_rows():
    par = torch.tensor(MASKS["bestfirst256_parents"], dtype=torch.int32, device="cuda")
    np.testing.assert_array_equal(G.build_tree_mask(par).cpu().numpy(), MASKS["bestfirst256_mask_none"])
    import random
    from projectgorgon_b200.trees import random_tree
    rows = [random_tree(64, random.Random(s), 5) for s in range(5)]
    got = G.build_tree_mask(torch.tensor(rows, device="cuda"), 5).cpu().numpy()
    for b, r in enumerate(rows):
        np.testing.assert_array_equal(got[b], O.build_tree_mask(r, 5))


def test_bad_parent_sets_device_error_without_faulting():
    G.device_error(clear=True)
    got = G.build_tree_mask([-1, 0, 9], None)
    torch.cuda.synchronize()
    assert G.device_error(clear=True) & 1
    assert bool(got[2, 2]) and not bool(got[2, 0])
