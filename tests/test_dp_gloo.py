"""The data-parallel gradient exchange on CPU: two gloo ranks, different gradients, one all-reduce;
every rank must end with the same average, and a single rank must be left untouched."""
import os
import sys

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, out):
    sys.path.insert(0, ROOT)
    from __graft_entry__ import load_package
    load_package()
    from unifiedlm_c_b200.dp import GradBucket
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shapes = [(8, 3), (5,), (), (2, 2, 2)]
        g = torch.Generator().manual_seed(100 + rank)
        grads = [torch.randn(s, generator=g) for s in shapes]
        bucket = GradBucket(shapes, device="cpu")
        bucket.pack(grads)
        avg = bucket.all_reduce(average=True)
        torch.save([a.clone() for a in avg], os.path.join(out, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_all_reduce_two_gloo_ranks(tmp_path):
    port = 29500 + os.getpid() % 1000
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    r0 = torch.load(tmp_path / "r0.pt")
    r1 = torch.load(tmp_path / "r1.pt")
    shapes = [(8, 3), (5,), (), (2, 2, 2)]
    g0 = torch.Generator().manual_seed(100)
    g1 = torch.Generator().manual_seed(101)
    ga = [torch.randn(s, generator=g0) for s in shapes]
    gb = [torch.randn(s, generator=g1) for s in shapes]
    for a, b, x, y in zip(r0, r1, ga, gb):
        assert torch.equal(a, b)
        assert torch.allclose(a, (x + y) / 2, atol=1e-6)


def test_single_process_is_a_no_op():
    sys.path.insert(0, ROOT)
    from unifiedlm_c_b200.dp import GradBucket
    b = GradBucket([(3,), (2, 2)], device="cpu")
    b.pack([torch.ones(3), torch.full((2, 2), 2.0)])
    v = b.all_reduce()
    assert torch.equal(v[0], torch.ones(3)) and torch.equal(v[1], torch.full((2, 2), 2.0))
