"""Input generators: the reference generator restated bit-for-bit (CPU)."""
import numpy as np
import pytest
import torch

from fastqr import inputs


def test_generate_input_matches_reference_bit_for_bit(golden):
    """Same seeded draws as official/reference.py:125-142 on the CPU generator."""
    data, meta = golden
    for name, m in meta["cases"].items():
        a = inputs.generate_input(device="cpu", **m["spec"])
        assert a.is_contiguous()
        np.testing.assert_array_equal(a.numpy(), data[f"{name}.A"], err_msg=name)
    for name, m in meta["blocked"].items():
        a = inputs.generate_input(device="cpu", **m["spec"])
        np.testing.assert_array_equal(a.numpy(), data[f"{name}.A"], err_msg=name)


def test_generate_input_rejects_bad_args():
    with pytest.raises(ValueError):
        inputs.generate_input(0, 8, 0, 1, device="cpu")
    with pytest.raises(ValueError):
        inputs.generate_input(2, 8, 0, 1, case="nope", device="cpu")


def test_c2_is_graded_generate_input():
    a = inputs.baseline_input("C2", seed=5, device="cpu", batch=2)
    b = inputs.generate_input(2, 256, 6, 5, device="cpu")
    assert torch.equal(a, b)
    norms = a[0].norm(dim=0)
    assert norms[0] / norms[-1] > 1e5


def test_c3_labels_are_shuffled_and_balanced():
    lab = inputs.c3_labels(512, 0)
    assert int((lab == inputs.C3_DENSE).sum()) == 256
    assert int((lab == inputs.C3_LOWRANK).sum()) == 128
    assert int((lab == inputs.C3_UPPER).sum()) == 128
    # every contiguous 1/8 shard holds a mix
    for r in range(8):
        assert len(set(lab[r * 64:(r + 1) * 64].tolist())) == 3


def test_c3_structures():
    a = inputs.baseline_input("C3", seed=1, device="cpu", batch=12)
    lab = inputs.c3_labels(512, 1)[:12]
    for i in range(12):
        s = torch.linalg.svdvals(a[i].double())
        if lab[i] == inputs.C3_LOWRANK:
            assert s[256] / s[0] < 1e-5
        elif lab[i] == inputs.C3_UPPER:
            assert torch.equal(a[i], torch.triu(a[i]))
        else:
            assert s[-1] / s[0] > 1e-7


def test_c3_shard_is_slice_of_global_batch():
    full = inputs.baseline_input("C3", seed=3, device="cpu", batch=6)
    part = inputs.baseline_input("C3", seed=3, device="cpu", batch=3, first=3)
    assert torch.equal(full[3:], part)


def test_c4_near_rank_deficient():
    a = inputs.baseline_input("C4", seed=2, device="cpu", batch=1)
    s = torch.linalg.svdvals(a[0].double())
    assert s[767] / s[0] > 1e-4
    assert s[768] / s[0] < 1e-5


def test_well_conditioned_mask():
    assert inputs.well_conditioned_mask("C1", 4).all()
    assert not inputs.well_conditioned_mask("C2", 4).any()
    m = inputs.well_conditioned_mask("C3", 512, seed=0)
    assert int(m.sum()) == 256
