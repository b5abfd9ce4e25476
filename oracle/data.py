"""TEST INFRASTRUCTURE ONLY — a CPU restatement of the reference's pretokenized data iterator
(tinystories.py:175-226 PretokDataset.__iter__ with Task.iter_batches' single-worker DataLoader,
tinystories.py:242-251) to check unifiedlm_c_b200.data against. Nothing in the library imports it."""
import glob
import os
import random

import numpy as np


def reference_batches(bin_dir, split, max_seq_len, batch_size, n_batches, rank=0, worker_id=0):
    """The first n_batches (x, y) int64 numpy batches the reference would yield."""
    rng = random.Random(42 + worker_id + 1337 * rank)
    files = sorted(glob.glob(os.path.join(bin_dir, "*.bin")))
    files = files[1:] if split == "train" else files[:1]
    xs, ys, out = [], [], []
    while True:
        rng.shuffle(files)
        for shard in files:
            m = np.memmap(shard, dtype=np.uint16, mode="r")
            num = len(m) // max_seq_len - 1
            ixs = list(range(num))
            rng.shuffle(ixs)
            for ix in ixs:
                chunk = m[ix * max_seq_len: ix * max_seq_len + max_seq_len + 1].astype(np.int64)
                xs.append(chunk[:-1])
                ys.append(chunk[1:])
                if len(xs) == batch_size:
                    out.append((np.stack(xs), np.stack(ys)))
                    xs, ys = [], []
                    if len(out) == n_batches:
                        return out
