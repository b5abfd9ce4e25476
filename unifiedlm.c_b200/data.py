"""Pretokenized training batches for the GPU: the reference's uint16 shard loader
(tinystories.py:175-251, PretokDataset + Task.iter_batches) with the same chunk order, staged as
uint16 in pinned host memory and widened to int64 on the device.

The reference reads one (max_seq_len + 1)-token chunk per example from a memory-mapped shard,
converts it to int64 on the host, and lets a DataLoader batch and pin it. Here a batch is gathered
straight from the memory maps into a pinned uint16 buffer (a quarter of the bytes), copied to the
device on a side stream while the previous batch is in use (two buffers), and widened there.

Order: shards sorted by name; "train" uses all but the first, "val" the first; a
`random.Random(42 + worker_id + 1337 * rank)` shuffles the shard list each pass and, per shard, the
chunk indices 0 .. len // max_seq_len - 2; consecutive chunks form a batch, as the reference's
single-worker DataLoader does. x = chunk[:-1], y = chunk[1:].
"""
import glob
import os
import random

import numpy as np
import torch


def shard_files(bin_dir, split):
    files = sorted(glob.glob(os.path.join(bin_dir, "*.bin")))
    files = files[1:] if split == "train" else files[:1]
    if not files:
        raise FileNotFoundError(f"no .bin shards for split {split!r} in {bin_dir}")
    return files


def chunk_stream(files, max_seq_len, seed):
    """(shard path, start token) of every example, in the reference's order, forever."""
    rng = random.Random(seed)
    files = list(files)
    maps = {}
    while True:
        rng.shuffle(files)
        for shard in files:
            m = maps.get(shard)
            if m is None:
                m = maps[shard] = np.memmap(shard, dtype=np.uint16, mode="r")
            num = len(m) // max_seq_len - 1  # the last partial chunk is dropped
            if num <= 0:
                raise ValueError(f"shard {shard} holds fewer than two chunks of {max_seq_len} tokens")
            ixs = list(range(num))
            rng.shuffle(ixs)
            for ix in ixs:
                yield m, ix * max_seq_len


class PretokBatches:
    """Iterator of (x, y) int64 (batch, max_seq_len) device tensors."""

    def __init__(self, bin_dir, split, max_seq_len, batch_size, device="cuda", rank=None, worker_id=0):
        if rank is None:
            import torch.distributed as dist
            rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
        self.files = shard_files(bin_dir, split)
        self.T = int(max_seq_len)
        self.B = int(batch_size)
        self.dev = torch.device(device)
        self.seed = 42 + worker_id + 1337 * rank
        self._stream = chunk_stream(self.files, self.T, self.seed)
        on_gpu = self.dev.type == "cuda"
        self._host = [torch.empty(self.B, self.T + 1, dtype=torch.int16, pin_memory=on_gpu) for _ in range(2)]
        self._copy_stream = torch.cuda.Stream(self.dev) if on_gpu else None
        self._events = [None, None]
        self._k = 0

    def _fill(self, buf):
        view = buf.numpy().view(np.uint16)
        for i in range(self.B):
            m, start = next(self._stream)
            view[i] = m[start:start + self.T + 1]

    def __iter__(self):
        return self

    def __next__(self):
        slot = self._k & 1
        self._k += 1
        buf = self._host[slot]
        if self._events[slot] is not None:
            self._events[slot].synchronize()  # the copy that last read this buffer has finished
        self._fill(buf)
        if self._copy_stream is None:
            tok = buf.view(torch.int16).to(torch.int64) & 0xFFFF
        else:
            with torch.cuda.stream(self._copy_stream):
                dev16 = buf.to(self.dev, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self._copy_stream)
                self._events[slot] = ev
            torch.cuda.current_stream(self.dev).wait_stream(self._copy_stream)
            dev16.record_stream(torch.cuda.current_stream(self.dev))
            tok = dev16.to(torch.int64) & 0xFFFF  # uint16 tokens held as int16 bits
        return tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
