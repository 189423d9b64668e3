"""Pure-Python restatement of the reference's BOS-aligned best-fit packing loop
(atlas_jax/data.py:54-121), TEST INFRASTRUCTURE ONLY: the checker of the native
packer (include/atlas_data.h).  ``docs`` is an iterator of token lists standing in
for tokenizer.encode over the parquet document stream; the refill cadence (one
tokenizer batch of ``refill_size`` documents whenever the buffer is below
buffer_size, data.py:85-95) is kept."""

import numpy as np


def pack_batches(docs, batch_size, seq_len, n_batches, buffer_size=1000, refill_size=128):
    docs = iter(docs)
    cap = seq_len + 1                                   # data.py:82
    buf = []

    def refill():                                       # data.py:85-89
        for _ in range(refill_size):
            buf.append(next(docs))
    rows = np.zeros((batch_size, cap), dtype=np.int32)
    out = []
    for _ in range(n_batches):
        for r in range(batch_size):
            pos = 0
            while pos < cap:
                while len(buf) < buffer_size:            # data.py:94-95
                    refill()
                remaining = cap - pos
                best, best_len = -1, 0                   # data.py:100-106
                for i, d in enumerate(buf):
                    if len(d) <= remaining and len(d) > best_len:
                        best, best_len = i, len(d)
                if best >= 0:                            # data.py:108-111
                    d = buf.pop(best)
                    rows[r, pos:pos + len(d)] = d
                    pos += len(d)
                else:                                    # data.py:113-117
                    j = min(range(len(buf)), key=lambda i: len(buf[i]))
                    d = buf.pop(j)
                    rows[r, pos:pos + remaining] = d[:remaining]
                    pos += remaining
        out.append((rows[:, :-1].copy(), rows[:, 1:].copy()))   # data.py:119-121
    return out
