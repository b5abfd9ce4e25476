"""The pretokenized batch loader (unifiedlm_c_b200.data) against the reference's iterator restated
in oracle/data.py (tinystories.py:175-251): same batches, same order, for several ranks, on the host
path here and on the device path under the gpu marker."""
import numpy as np
import pytest
import torch

from oracle import data as OD
from unifiedlm_c_b200.data import PretokBatches


def write_shards(tmp_path, sizes, seed=0):
    rng = np.random.default_rng(seed)
    for i, n in enumerate(sizes):
        rng.integers(0, 65536, size=n, dtype=np.uint16).tofile(str(tmp_path / f"data{i:02d}.bin"))
    return str(tmp_path)


@pytest.mark.parametrize("rank", [0, 1])
@pytest.mark.parametrize("split", ["train", "val"])
def test_batches_match_reference_order(tmp_path, rank, split):
    d = write_shards(tmp_path, [4000, 3000, 5200, 2600])
    ref = OD.reference_batches(d, split, 64, 8, 40, rank=rank)  # several passes over the shards
    it = PretokBatches(d, split, 64, 8, device="cpu", rank=rank)
    for xr, yr in ref:
        x, y = next(it)
        assert x.dtype == torch.int64 and x.shape == (8, 64)
        assert np.array_equal(x.numpy(), xr) and np.array_equal(y.numpy(), yr)


@pytest.mark.gpu
def test_device_batches_match_reference(tmp_path):
    d = write_shards(tmp_path, [9000, 7000, 8000], seed=3)
    ref = OD.reference_batches(d, "train", 256, 16, 12)
    it = PretokBatches(d, "train", 256, 16, device="cuda")
    for xr, yr in ref:
        x, y = next(it)
        assert x.is_cuda and x.dtype == torch.int64
        assert np.array_equal(x.cpu().numpy(), xr) and np.array_equal(y.cpu().numpy(), yr)
