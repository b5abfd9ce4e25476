"""Data-parallel gradient exchange for the fast-memory path (the reference trains with DDP,
train.py:87-98, 182-183: one process per GPU, NCCL all-reduce of every parameter gradient).

Sequences are independent, so the only collective is the sum (or mean) of parameter gradients over
ranks. `GradBucket` packs a list of gradient tensors into one flat fp32 buffer, all-reduces it in a
single call (one NCCL launch instead of one per tensor) and unpacks it. Works with any
torch.distributed backend (NCCL on GPUs, gloo on CPU for tests).

The buffer can also be cut into consecutive segments (one per block of the model, say) whose
all-reduces start as soon as their gradients exist (`pack_segment` + `start_segment`, then
`finish`): like DDP's gradient buckets, the exchange of the later blocks' gradients runs on NCCL's
stream while the earlier blocks' backward still computes. The result is the same sum as the
one-shot `all_reduce`.
"""
import torch
import torch.distributed as dist


class GradBucket:
    def __init__(self, shapes, device, dtype=torch.float32, segments=1):
        self.shapes = [tuple(s) for s in shapes]
        self.numels = [int(torch.Size(s).numel()) for s in self.shapes]
        self.offsets = [0]
        for n in self.numels:
            self.offsets.append(self.offsets[-1] + n)
        self.flat = torch.zeros(self.offsets[-1], device=device, dtype=dtype)
        if segments < 1 or len(self.shapes) % segments:
            raise ValueError(f"{len(self.shapes)} tensors do not split into {segments} equal segments")
        self.per_segment = len(self.shapes) // segments
        self.segments = segments
        self._pending = []

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

    def _segment_range(self, i):
        if not 0 <= i < self.segments:
            raise IndexError(f"segment {i} of {self.segments}")
        return i * self.per_segment, (i + 1) * self.per_segment

    def segment(self, i):
        """The slice of the flat buffer that holds segment `i`."""
        a, b = self._segment_range(i)
        return self.flat[self.offsets[a]:self.offsets[b]]

    def pack_segment(self, i, grads):
        """Copy the gradients of segment `i` (its tensors, in order) into the bucket."""
        a, b = self._segment_range(i)
        grads = list(grads)
        if len(grads) != b - a:
            raise ValueError(f"segment {i} holds {b - a} tensors, got {len(grads)}")
        views = self.views()[a:b]
        if all(g.dtype == self.flat.dtype and tuple(g.shape) == v.shape for g, v in zip(grads, views)):
            torch._foreach_copy_(views, grads)
        else:
            for v, g in zip(views, grads):
                v.copy_(g.reshape(v.shape))
        return self.segment(i)

    def start_segment(self, i, group=None):
        """Start the sum over ranks of segment `i` without waiting for it. With NCCL the collective
        is queued behind the work already issued on the current stream and runs on NCCL's own
        stream; `finish` makes the current stream wait for it. No-op without a process group."""
        if _world(group) > 1:
            self._pending.append((i, dist.all_reduce(self.segment(i), group=group, async_op=True)))

    def finish(self, average=True, group=None):
        """Wait for every started segment (then divide those by the world size if `average`)."""
        pending, self._pending = self._pending, []
        for _, work in pending:
            work.wait()
        world = _world(group)
        if average and world > 1 and pending:
            started = sorted(i for i, _ in pending)
            if started == list(range(self.segments)):
                self.flat.div_(world)
            else:
                for i in started:
                    self.segment(i).div_(world)
        return self.views()

    def all_reduce(self, average=True, group=None):
        """Sum over ranks (then divide by the world size if `average`). No-op without a process group."""
        world = _world(group)
        if world > 1:
            dist.all_reduce(self.flat, group=group)
            if average:
                self.flat.div_(world)
        return self.views()


def _world(group=None):
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group)
    return 1
