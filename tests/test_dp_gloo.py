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
        # the same tensors twice over, as two segments started one by one (in reverse order, as a
        # backward produces them) and finished together
        seg = GradBucket(shapes * 2, device="cpu", segments=2)
        for i in (1, 0):
            seg.pack_segment(i, grads)
            seg.start_segment(i)
        avg2 = seg.finish(average=True)
        torch.save([a.clone() for a in avg2], os.path.join(out, f"s{rank}.pt"))
        # one segment started alone: only it is summed and divided
        one = GradBucket(shapes * 2, device="cpu", segments=2)
        one.pack_segment(0, grads)
        one.pack_segment(1, grads)
        one.start_segment(1)
        avg3 = one.finish(average=True)
        torch.save([a.clone() for a in avg3], os.path.join(out, f"o{rank}.pt"))
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
    s0 = torch.load(tmp_path / "s0.pt")
    s1 = torch.load(tmp_path / "s1.pt")
    assert len(s0) == 2 * len(shapes)
    for a, b, ref in zip(s0, s1, r0 * 2):
        assert torch.equal(a, b) and torch.equal(a, ref)
    o0 = torch.load(tmp_path / "o0.pt")
    o1 = torch.load(tmp_path / "o1.pt")
    n = len(shapes)
    for a, x in zip(o0[:n], ga):
        assert torch.equal(a, x)
    for a, x in zip(o1[:n], gb):
        assert torch.equal(a, x)
    for a, b, ref in zip(o0[n:], o1[n:], r0):
        assert torch.equal(a, b) and torch.equal(a, ref)


def test_single_process_is_a_no_op():
    sys.path.insert(0, ROOT)
    from unifiedlm_c_b200.dp import GradBucket
    b = GradBucket([(3,), (2, 2)], device="cpu")
    b.pack([torch.ones(3), torch.full((2, 2), 2.0)])
    v = b.all_reduce()
    assert torch.equal(v[0], torch.ones(3)) and torch.equal(v[1], torch.full((2, 2), 2.0))
    s = GradBucket([(3,), (2, 2)] * 3, device="cpu", segments=3)
    for i in range(3):
        s.pack_segment(i, [torch.full((3,), float(i)), torch.full((2, 2), -float(i))])
        s.start_segment(i)
    v = s.finish()
    for i in range(3):
        assert torch.equal(v[2 * i], torch.full((3,), float(i)))
        assert torch.equal(v[2 * i + 1], torch.full((2, 2), -float(i)))


def test_segment_arguments_are_checked():
    sys.path.insert(0, ROOT)
    import pytest
    from unifiedlm_c_b200.dp import GradBucket
    with pytest.raises(ValueError):
        GradBucket([(3,), (2,), (1,)], device="cpu", segments=2)
    b = GradBucket([(3,), (2,)], device="cpu", segments=2)
    with pytest.raises(IndexError):
        b.pack_segment(2, [torch.ones(3)])
    with pytest.raises(ValueError):
        b.pack_segment(0, [torch.ones(3), torch.ones(2)])
