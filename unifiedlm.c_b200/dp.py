"""Data-parallel gradient exchange for the fast-memory path (the reference trains with DDP,
train.py:87-98, 182-183: one process per GPU, NCCL all-reduce of every parameter gradient).

Sequences are independent, so the only collective is the sum (or mean) of parameter gradients over
ranks. `GradBucket` packs a list of gradient tensors into one flat fp32 buffer, all-reduces it in a
single call (one NCCL launch instead of one per tensor) and unpacks it. Works with any
torch.distributed backend (NCCL on GPUs, gloo on CPU for tests).
"""
import torch
import torch.distributed as dist


class GradBucket:
    def __init__(self, shapes, device, dtype=torch.float32):
        self.shapes = [tuple(s) for s in shapes]
        self.numels = [int(torch.Size(s).numel()) for s in self.shapes]
        self.offsets = [0]
        for n in self.numels:
            self.offsets.append(self.offsets[-1] + n)
        self.flat = torch.zeros(self.offsets[-1], device=device, dtype=dtype)

    def views(self):
        return [self.flat[a:b].view(s) for a, b, s in zip(self.offsets, self.offsets[1:], self.shapes)]

    def pack(self, grads):
        """Copy the gradients into the bucket (one multi-tensor copy launch for same-dtype inputs)."""
        views = self.views()
        if all(g.dtype == self.flat.dtype and tuple(g.shape) == v.shape for g, v in zip(grads, views)):
            torch._foreach_copy_(views, list(grads))
        else:
            torch.cat([g.reshape(-1).to(self.flat.dtype) for g in grads], out=self.flat)
        return self.flat

    def all_reduce(self, average=True, group=None):
        """Sum over ranks (then divide by the world size if `average`). No-op without a process group."""
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, group=group)
            if average:
                self.flat.div_(dist.get_world_size(group))
        return self.views()
