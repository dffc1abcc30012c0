"""The on-disk token cache of cdl's training script, format 1
(cdl/dataset/token_cache.py:1-14, 60-134, 268-438), read and written
without the Hugging Face download and tokenizer steps.

Layout of a cache directory::

    tokens.u16   [test blocks][train blocks ...]   raw little-endian token ids
    meta.json    CacheMeta (sorted keys, indent 2)
    cache.lock   flock'ed while the cache is opened or appended

Each block is ``seq_len`` tokens of ``meta.dtype`` (uint16, or uint32 for a
vocabulary above 65535).  The test blocks come first and never change; train
blocks are appended in place, the tokens that do not fill a block kept in
``meta.tail``.  A crash between the token write and the meta write leaves
bytes past the committed block count, which opening truncates away.

Building a cache from text (tokenize, split the last ``num_test_blocks``
blocks off as the test set) and appending need the token ids from the caller:
``build_from_tokens`` / ``TokenCache.append_tokens`` take them as an array,
where cdl fetches and tokenizes the Hub streams itself.

``DeviceBlockLoader`` is the B200 side: it copies a batch of blocks in the
file's dtype from pinned host memory (a quarter of the bytes of the int64
blocks cdl's ``BlockDataset`` yields) and widens it to int64 on the device.
"""

from __future__ import annotations

import fcntl
import json
import os
from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import asdict, dataclass, field
from pathlib import Path

import numpy as np
import torch

CACHE_FORMAT = 1


@dataclass
class CacheMeta:
    """meta.json (token_cache.py:60-88): the same keys and meaning."""

    format: int
    model_id: str
    tokenizer: str
    tokenizer_revision: str | None
    eos_token_id: int
    seq_len: int
    dtype: str
    ratios: dict[str, float]
    seed: int
    num_test_blocks: int
    num_calib_blocks: int
    n_train_blocks: int
    n_test_blocks: int
    tail: list[int] = field(default_factory=list)
    docs_consumed: dict[str, int] = field(default_factory=dict)

    @classmethod
    def load(cls, path: Path) -> "CacheMeta":
        return cls(**json.loads(Path(path).read_text(encoding="utf-8")))

    def save(self, path: Path) -> None:
        path = Path(path)
        tmp = path.with_suffix(path.suffix + ".tmp")
        with open(tmp, "w", encoding="utf-8") as f:
            f.write(json.dumps(asdict(self), indent=2, sort_keys=True))
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)


class BlockDataset(torch.utils.data.Dataset):
    """Fixed-length blocks of a memory-mapped token file as int64 tensors
    (token_cache.py:91-134)."""

    def __init__(self, path: Path, dtype, offset_blocks: int, n_blocks: int, seq_len: int):
        self.path = Path(path)
        self.dtype = np.dtype(dtype)
        self.offset_blocks, self.n_blocks, self.seq_len = offset_blocks, n_blocks, seq_len
        self._mmap = None

    def blocks(self) -> np.ndarray:
        """The blocks in the file's dtype, ``[n_blocks, seq_len]`` (a memmap)."""
        if self._mmap is None:
            if self.n_blocks == 0:
                self._mmap = np.empty((0, self.seq_len), dtype=self.dtype)
            else:
                self._mmap = np.memmap(self.path, dtype=self.dtype, mode="r",
                                       offset=self.offset_blocks * self.seq_len * self.dtype.itemsize,
                                       shape=(self.n_blocks, self.seq_len))
        return self._mmap

    def __len__(self) -> int:
        return self.n_blocks

    def __getitem__(self, index: int) -> torch.Tensor:
        return torch.from_numpy(np.asarray(self.blocks()[index], dtype=np.int64))

    def __getstate__(self) -> dict:
        state = self.__dict__.copy()
        state["_mmap"] = None  # not pickled into DataLoader workers
        return state


@contextmanager
def _lock(path: Path) -> Iterator[None]:
    with open(path, "w", encoding="utf-8") as f:
        fcntl.flock(f.fileno(), fcntl.LOCK_EX)
        try:
            yield
        finally:
            fcntl.flock(f.fileno(), fcntl.LOCK_UN)


def token_dtype(tokens: np.ndarray) -> np.dtype:
    """uint16 when every id fits, else uint32 (token_cache.py:370-379)."""
    top = int(tokens.max()) if tokens.size else 0
    if top <= np.iinfo(np.uint16).max:
        return np.dtype(np.uint16)
    if top <= np.iinfo(np.uint32).max:
        return np.dtype(np.uint32)
    raise ValueError(f"token id {top} does not fit in uint32")


def _check_size(path: Path, meta: CacheMeta) -> None:
    """A short file is an error; bytes past the committed blocks (a crashed
    append) are cut off (token_cache.py:420-438)."""
    if not path.exists():
        raise ValueError(f"token cache is missing {path}; rebuild the cache")
    want = (meta.n_test_blocks + meta.n_train_blocks) * meta.seq_len * np.dtype(meta.dtype).itemsize
    have = path.stat().st_size
    if have < want:
        raise ValueError(f"token cache {path} is truncated: {have} < {want} bytes")
    if have > want:
        with open(path, "r+b") as f:
            f.truncate(want)


def build_from_tokens(directory: str | Path, tokens: np.ndarray, *, seq_len: int, num_test_blocks: int,
                      num_calib_blocks: int = 0, model_id: str = "", tokenizer: str = "",
                      tokenizer_revision: str | None = None, eos_token_id: int = 0,
                      ratios: dict[str, float] | None = None, seed: int = 0,
                      docs_consumed: dict[str, int] | None = None) -> "TokenCache":
    """A new cache from a token stream, split as cdl's first build splits it
    (token_cache.py:298-345): whole blocks only, the last ``num_test_blocks``
    of them the test set, written first; the partial block is dropped."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    tokens = np.asarray(tokens)
    tokens = tokens.astype(token_dtype(tokens), copy=False)
    n_blocks = len(tokens) // seq_len
    if n_blocks <= num_test_blocks:
        raise ValueError(f"only {n_blocks} blocks of seq_len={seq_len}; need more than "
                         f"num_test_blocks={num_test_blocks}")
    test_start = n_blocks - num_test_blocks
    with _lock(directory / "cache.lock"):
        tmp = directory / "tokens.u16.tmp"
        with open(tmp, "wb") as f:
            tokens[test_start * seq_len: n_blocks * seq_len].tofile(f)
            tokens[: test_start * seq_len].tofile(f)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, directory / "tokens.u16")
        meta = CacheMeta(CACHE_FORMAT, model_id, tokenizer, tokenizer_revision, eos_token_id, seq_len,
                         tokens.dtype.name, dict(ratios or {}), seed, num_test_blocks, num_calib_blocks,
                         test_start, num_test_blocks, [], dict(docs_consumed or {}))
        meta.save(directory / "meta.json")
    return TokenCache(directory, meta)


class TokenCache:
    """An existing cache directory: its train / test splits, the calibration
    blocks (the first train blocks) and in-place appends."""

    def __init__(self, directory: str | Path, meta: CacheMeta):
        self.directory = Path(directory)
        self.meta = meta
        self.tokens_path = self.directory / "tokens.u16"
        self.meta_path = self.directory / "meta.json"
        self.dtype = np.dtype(meta.dtype)
        self._refresh()

    @classmethod
    def open(cls, directory: str | Path, expect: dict | None = None) -> "TokenCache":
        """Open a cache; ``expect`` maps meta fields to required values (cdl
        checks format, model, tokenizer, eos, seq_len, ratios, seed and the
        test split against its config, token_cache.py:391-417)."""
        directory = Path(directory)
        with _lock(directory / "cache.lock"):
            meta = CacheMeta.load(directory / "meta.json")
            if meta.format != CACHE_FORMAT:
                raise ValueError(f"token cache format {meta.format}, expected {CACHE_FORMAT}")
            for name, want in (expect or {}).items():
                have = getattr(meta, name)
                if have != want:
                    raise ValueError(f"token cache mismatch for {name}: cache has {have!r}, config wants {want!r}")
            _check_size(directory / "tokens.u16", meta)
        return cls(directory, meta)

    def _refresh(self) -> None:
        m = self.meta
        self.train_dataset = BlockDataset(self.tokens_path, self.dtype, m.n_test_blocks, m.n_train_blocks, m.seq_len)
        self.test_dataset = BlockDataset(self.tokens_path, self.dtype, 0, m.n_test_blocks, m.seq_len)

    @property
    def n_train_blocks(self) -> int:
        return self.meta.n_train_blocks

    def calib_blocks(self, n_blocks: int) -> torch.Tensor:
        """The first ``n_blocks`` train blocks, int64 (token_cache.py:175-181)."""
        n = min(n_blocks, self.meta.n_train_blocks)
        if n <= 0:
            return torch.empty((0, self.meta.seq_len), dtype=torch.long)
        return torch.from_numpy(np.asarray(self.train_dataset.blocks()[:n], dtype=np.int64))

    def append_tokens(self, tokens: np.ndarray, docs_consumed: dict[str, int] | None = None) -> None:
        """Append a token stream to the train split: the stored tail first,
        whole blocks written, the rest kept as the new tail; the token file
        is cut back to its committed size before writing (token_cache.py:245-267)."""
        tokens = np.asarray(tokens)
        if tokens.size and int(tokens.max()) > np.iinfo(self.dtype).max:
            raise ValueError(f"new token id {int(tokens.max())} does not fit {self.dtype}")
        m = self.meta
        with _lock(self.directory / "cache.lock"):
            stream = np.concatenate([np.asarray(m.tail, dtype=self.dtype), tokens.astype(self.dtype, copy=False)])
            n_full = len(stream) // m.seq_len
            if n_full:
                committed = (m.n_test_blocks + m.n_train_blocks) * m.seq_len * self.dtype.itemsize
                with open(self.tokens_path, "r+b") as f:
                    f.seek(committed)
                    f.truncate()
                    f.seek(0, os.SEEK_END)
                    stream[: n_full * m.seq_len].tofile(f)
                    f.flush()
                    os.fsync(f.fileno())
                m.n_train_blocks += n_full
            m.tail = stream[n_full * m.seq_len:].tolist()
            for name, count in (docs_consumed or {}).items():
                m.docs_consumed[name] = m.docs_consumed.get(name, 0) + count
            m.save(self.meta_path)
        self._refresh()


class DeviceBlockLoader:
    """Batches of blocks on a CUDA device, in the order of cdl's train loader
    (``DataLoader(train_dataset, batch_size, shuffle=True, drop_last=True)``,
    smollm2.py:540-546): with ``shuffle`` each epoch is one ``randperm`` whose
    generator is seeded, as torch's DataLoader and RandomSampler seed it, from
    the global torch RNG (or is ``generator``).  Each batch is gathered from
    the memmap into one of two pinned buffers in the file's dtype, copied
    asynchronously and widened to int64 on the device; a buffer is refilled
    only after its previous copy finished."""

    def __init__(self, dataset: BlockDataset, batch_size: int, device, *, shuffle: bool = True,
                 drop_last: bool = True, generator: torch.Generator | None = None):
        if dataset.dtype not in (np.dtype(np.uint16), np.dtype(np.uint32)):
            raise ValueError(f"unsupported token dtype {dataset.dtype}")
        self.dataset, self.batch_size, self.device = dataset, batch_size, torch.device(device)
        self.shuffle, self.drop_last, self.generator = shuffle, drop_last, generator
        # ids travel as int16 / int32 bit patterns and are widened unsigned on the device
        self._wire = torch.int16 if dataset.dtype == np.uint16 else torch.int32
        self._mask = 0xFFFF if self._wire == torch.int16 else 0xFFFFFFFF
        pin = self.device.type == "cuda"
        self._host = [torch.empty((batch_size, dataset.seq_len), dtype=self._wire, pin_memory=pin)
                      for _ in range(2)]
        self._done = [None, None]

    def __len__(self) -> int:
        n = len(self.dataset)
        return n // self.batch_size if self.drop_last else -(-n // self.batch_size)

    def _order(self) -> list[int]:
        n = len(self.dataset)
        if not self.shuffle:
            return list(range(n))
        # the DataLoader iterator first draws its workers' base seed, then the
        # sampler draws its own seed (both from the global RNG without a generator)
        g = self.generator
        torch.empty((), dtype=torch.int64).random_(generator=g)
        if g is None:
            g = torch.Generator()
            g.manual_seed(int(torch.empty((), dtype=torch.int64).random_().item()))
        return torch.randperm(n, generator=g).tolist()

    def __iter__(self) -> Iterator[torch.Tensor]:
        order, blocks = self._order(), self.dataset.blocks()
        cuda = self.device.type == "cuda"
        for i in range(len(self)):
            idx = order[i * self.batch_size:(i + 1) * self.batch_size]
            j = i & 1
            if self._done[j] is not None:
                self._done[j].synchronize()
            host = self._host[j][: len(idx)]
            host.numpy().view(self.dataset.dtype)[:] = blocks[idx]
            out = host.to(self.device, non_blocking=cuda).to(torch.int64) & self._mask
            if cuda:
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream(self.device))
                self._done[j] = ev
            yield out
