"""Native BOS-aligned best-fit packer (include/atlas_data.h) against the restated
reference loop (oracle/packing.py, atlas_jax/data.py:54-121): identical batches on
the same document stream, bit for bit."""
import itertools

import numpy as np
import pytest

from oracle import packing as OP

BOS = 7


def _docs(seed, max_len):
    rng = np.random.default_rng(seed)
    while True:  # many equal lengths, so tie-breaking by arrival order matters
        n = int(rng.integers(1, max_len + 1)) if rng.random() < 0.7 else int(rng.choice([3, 5, 8]))
        yield [BOS] + rng.integers(100, 30000, n - 1).tolist() if n > 1 else [BOS]


def _native(docs, B, T, n_batches, buffer_size, refill_size):
    from atlas_b200.data import Packer
    it = iter(docs)
    pk = Packer(B, T, buffer_size)
    refill = lambda: [next(it) for _ in range(refill_size)]  # noqa: E731
    return [tuple(x.numpy() for x in pk.next_batch(refill)) for _ in range(n_batches)]


@pytest.mark.parametrize("B,T,buf,refill,max_len", [(2, 16, 10, 4, 12), (4, 64, 50, 16, 90), (3, 7, 5, 1, 30),
                                                    (8, 256, 1000, 128, 400)])
def test_packer_matches_reference_loop(B, T, buf, refill, max_len):
    n = 6
    ref = OP.pack_batches(_docs(1, max_len), B, T, n, buf, refill)
    got = _native(_docs(1, max_len), B, T, n, buf, refill)
    for (ri, rt), (gi, gt) in zip(ref, got):
        np.testing.assert_array_equal(gi, ri)
        np.testing.assert_array_equal(gt, rt)
        assert (gi[:, 0] == BOS).all()
        np.testing.assert_array_equal(gi[:, 1:], gt[:, :-1])


def test_packer_rejects_bad_input():
    from atlas_b200.data import Packer
    with pytest.raises(ValueError):
        Packer(0, 8)
    pk = Packer(1, 4, 2)
    with pytest.raises(ValueError):
        pk.push([[BOS], []])
    assert pk.buffered == 0
    pk.push([[BOS, 1], [BOS, 2, 3]])
    assert pk.buffered == 2


def test_data_loader_reads_parquet_like_the_reference(tmp_path):
    """data_loader over parquet files (last file = validation split) and a toy
    tokenizer, against the restated loop on the same document stream."""
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    from atlas_b200.data import data_loader
    rng = np.random.default_rng(0)
    texts = [" ".join(str(int(x)) for x in rng.integers(1, 99, int(rng.integers(1, 40)))) for _ in range(900)]
    for f in range(3):
        pq.write_table(pa.table({"text": texts[f * 300:(f + 1) * 300]}), tmp_path / f"shard_{f:02d}.parquet",
                       row_group_size=50)

    class Tok:
        def get_bos_token_id(self):
            return BOS

        def encode(self, batch, prepend=None):
            return [[prepend] + [int(w) + 10 for w in t.split()] for t in batch]
    B, T = 2, 32
    got = list(itertools.islice(data_loader(str(tmp_path), Tok(), B, T, buffer_size=40), 5))
    stream = (d for _ in itertools.count() for d in Tok().encode(texts[:600], prepend=BOS))
    ref = OP.pack_batches(stream, B, T, 5, buffer_size=40, refill_size=50)  # one row group per refill
    for (gi, gt), (ri, rt) in zip(got, ref):
        np.testing.assert_array_equal(gi.numpy(), ri)
        np.testing.assert_array_equal(gt.numpy(), rt)
