"""BOS-aligned best-fit packing data loader (atlas_jax/data.py:24-121), with the
packing loop in native code (include/atlas_data.h).

``data_loader`` keeps the reference's signature and yields (inputs, targets) int32
tensors of shape (batch_size, seq_len); parquet reading (pyarrow) and tokenisation
(the caller's tokenizer: ``encode(texts, prepend=bos)`` and ``get_bos_token_id()``)
stay on the Python side exactly as in the reference.
"""

import ctypes
import os

import numpy as np
import torch

from . import _lib as L

ATLAS_PACK_NEED_DOCS = 6
_bound = False


def _lib():
    global _bound
    lib = L.load()
    if not _bound:
        lib.atlas_packer_create.restype = ctypes.c_void_p
        lib.atlas_packer_create.argtypes = [ctypes.c_int32] * 3
        lib.atlas_packer_destroy.restype = None
        lib.atlas_packer_destroy.argtypes = [ctypes.c_void_p]
        lib.atlas_packer_push.restype = ctypes.c_int
        lib.atlas_packer_push.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        lib.atlas_packer_buffered.restype = ctypes.c_int64
        lib.atlas_packer_buffered.argtypes = [ctypes.c_void_p]
        lib.atlas_packer_next_batch.restype = ctypes.c_int
        lib.atlas_packer_next_batch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _bound = True
    return lib


class Packer:
    """Native best-fit row packer: push tokenised documents, pull (inputs, targets)."""

    def __init__(self, batch_size, seq_len, buffer_size=1000):
        self.lib = _lib()
        self.h = self.lib.atlas_packer_create(batch_size, seq_len, buffer_size)
        if not self.h:
            raise ValueError("batch_size, seq_len and buffer_size must be positive")
        self.B, self.T = batch_size, seq_len

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.atlas_packer_destroy(self.h)
            self.h = None

    def push(self, docs):
        """docs: a list of token sequences (each non-empty)."""
        if not docs:
            return
        lens = np.fromiter((len(d) for d in docs), dtype=np.int64, count=len(docs))
        offsets = np.zeros(len(docs) + 1, dtype=np.int64)
        np.cumsum(lens, out=offsets[1:])
        toks = np.concatenate([np.asarray(d, dtype=np.int32) for d in docs])
        rc = self.lib.atlas_packer_push(self.h, toks.ctypes.data, offsets.ctypes.data, len(docs))
        if rc != L.ATLAS_OK:
            raise ValueError("documents must be non-empty")

    @property
    def buffered(self):
        return self.lib.atlas_packer_buffered(self.h)

    def next_batch(self, refill):
        """The next (inputs, targets) batch; ``refill()`` returns more documents when
        the packer needs them (the reference's refill_buffer, data.py:85-89)."""
        inputs = torch.empty(self.B, self.T, dtype=torch.int32)
        targets = torch.empty(self.B, self.T, dtype=torch.int32)
        while True:
            rc = self.lib.atlas_packer_next_batch(self.h, inputs.data_ptr(), targets.data_ptr())
            if rc == L.ATLAS_OK:
                return inputs, targets
            if rc != ATLAS_PACK_NEED_DOCS:
                raise RuntimeError(f"packer error {rc}")
            self.push(refill())


def list_parquet_files(data_dir):
    """All .parquet files in data_dir, sorted by name (data.py:24-31)."""
    return [os.path.join(data_dir, f) for f in sorted(os.listdir(data_dir))
            if f.endswith(".parquet") and not f.endswith(".tmp")]


def _document_batches(parquet_paths, tokenizer_batch_size=128, rank=0, world_size=1):
    """Endless (texts, file index) batches; row groups sharded by rank (data.py:34-51)."""
    import pyarrow.parquet as pq
    while True:
        for pq_idx, path in enumerate(parquet_paths):
            pf = pq.ParquetFile(path)
            for rg_idx in range(rank, pf.num_row_groups, world_size):
                texts = pf.read_row_group(rg_idx).column("text").to_pylist()
                for i in range(0, len(texts), tokenizer_batch_size):
                    yield texts[i:i + tokenizer_batch_size], pq_idx


def data_loader(data_dir, tokenizer, batch_size, seq_len, split="train", buffer_size=1000, rank=0, world_size=1):
    """BOS-aligned best-fit packing loader (data.py:54-121): yields (inputs, targets)."""
    paths = list_parquet_files(data_dir)
    assert len(paths) > 0, f"No parquet files found in {data_dir}"
    paths = paths[:-1] if split == "train" else paths[-1:]
    bos = tokenizer.get_bos_token_id()
    batches = _document_batches(paths, rank=rank, world_size=world_size)

    def refill():
        texts, _ = next(batches)
        return tokenizer.encode(texts, prepend=bos)
    packer = Packer(batch_size, seq_len, buffer_size)
    while True:
        yield packer.next_batch(refill)
