"""Data: byte tokenizer, seeded synthetic token batches, EOS packing and a
bounded background-prefetch iterator (data.py / grain_data.py of the reference).

The reference streams parquet shards through Grain; this box has no network, so
the production loader is a seeded synthetic token source (uniform random
tokens, per-rank seed) with the same background prefetch and pinned-memory
staging.  ``ParquetLoader`` keeps the reference's local-parquet pipeline
(read -> tokenize + EOS -> drop empty docs -> concat-then-split packing ->
batch) for users with data on disk.
"""
from __future__ import annotations

import itertools
import queue
import threading
from typing import Iterator, Optional, Sequence

import numpy as np


class ByteTokenizer:
    """Byte-level tokenizer (data.py:28-43): ids 0..255, EOS = vocab - 1."""

    def __init__(self, vocab_size: int = 256):
        self.vocab_size = vocab_size
        self.eos_id = vocab_size - 1

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))[: self.vocab_size - 1]

    def decode(self, ids) -> str:
        return bytes([i for i in ids if 0 <= i < 256]).decode("utf-8", errors="replace")


def get_tokenizer(config):
    """Byte tokenizer, or a local HF tokenizer path if it loads (no network)."""
    if config.tokenizer in ("byte",):
        return ByteTokenizer(vocab_size=min(config.vocab_size, 256) if config.vocab_size < 256
                             else config.vocab_size)
    try:
        from transformers import AutoTokenizer
        return AutoTokenizer.from_pretrained(config.tokenizer, local_files_only=True)
    except Exception as e:
        print(f"[data] tokenizer {config.tokenizer!r} unavailable offline ({str(e)[:60]}); "
              f"using bytes")
        return ByteTokenizer(vocab_size=config.vocab_size)


def random_batches(config, batch_size: int, seq_len: int, seed: int = 0) -> Iterator[np.ndarray]:
    """Uniform random tokens (data.py:205-209): ``integers(0, V, (B, S), int32)``."""
    rng = np.random.default_rng(seed)
    while True:
        yield rng.integers(0, config.vocab_size, size=(batch_size, seq_len), dtype=np.int32)


def pack_sequences(token_iter, seq_len: int, eos_id: int) -> Iterator[np.ndarray]:
    """Concat-then-split packing with EOS between documents (data.py:142-151)."""
    buf: list[int] = []
    for tokens in token_iter:
        if len(tokens) == 0:
            continue
        buf.extend(tokens)
        buf.append(eos_id)
        while len(buf) >= seq_len:
            chunk = buf[:seq_len]
            del buf[:seq_len]
            yield np.asarray(chunk, dtype=np.int32)


def prefetch(it: Iterator, depth: int = 8) -> Iterator:
    """Run ``it`` on a daemon thread with a bounded queue; producer exceptions
    are re-raised in the consumer (data.py:154-173)."""
    q: queue.Queue = queue.Queue(maxsize=depth)
    sentinel = object()

    def worker():
        try:
            for item in it:
                q.put(item)
        except BaseException as e:  # surfaced downstream
            q.put(e)
        finally:
            q.put(sentinel)

    threading.Thread(target=worker, daemon=True).start()
    while True:
        item = q.get()
        if item is sentinel:
            return
        if isinstance(item, BaseException):
            raise item
        yield item


class SyntheticLoader:
    """Seeded synthetic token batches for one data-parallel rank.

    Batches are drawn on a background thread into pinned host memory so the
    host->device copy of step i+1 overlaps step i.  ``state_dict`` /
    ``load_state_dict`` capture the RNG so a resumed run continues the stream.
    """

    def __init__(self, vocab_size: int, batch_size: int, seq_len: int, seed: int = 0,
                 rank: int = 0, pin: bool = True, depth: int = 4):
        self.vocab_size, self.batch_size, self.seq_len = vocab_size, batch_size, seq_len
        self.seed, self.rank, self.pin, self.depth = seed, rank, pin, depth
        self.rng = np.random.default_rng([seed, rank])
        self.produced = 0

    def _gen(self):
        import torch
        while True:
            a = self.rng.integers(0, self.vocab_size, size=(self.batch_size, self.seq_len),
                                  dtype=np.int32)
            t = torch.from_numpy(a).long()
            if self.pin and torch.cuda.is_available():
                t = t.pin_memory()
            self.produced += 1
            yield t

    def __iter__(self):
        return prefetch(self._gen(), self.depth)

    def state_dict(self):
        return {"bit_generator": self.rng.bit_generator.state, "produced": self.produced}

    def load_state_dict(self, st):
        self.rng.bit_generator.state = st["bit_generator"]
        self.produced = st["produced"]


class ParquetLoader:
    """Local parquet documents -> packed ``[batch, seq_len]`` int32 batches.

    Same stages as grain_data.py:91-150: shuffled (seeded) file order, a
    round-robin interleave of ``interleave`` files, tokenize + EOS, drop empty
    documents, concat-then-split packing, batching, background prefetch.
    """

    TEXT_FIELDS = ("content", "text", "raw_content", "document")

    def __init__(self, files: Sequence[str], tokenizer, seq_len: int, batch_size: int,
                 eos_id: Optional[int] = None, interleave: int = 4, shuffle_files: bool = True,
                 seed: int = 0, buffer: int = 8, repeat: bool = True):
        self.files = list(files)
        self.tok = tokenizer
        self.seq_len, self.batch_size = seq_len, batch_size
        self.eos = eos_id if eos_id is not None else getattr(tokenizer, "eos_id", 0)
        self.interleave, self.shuffle, self.seed = interleave, shuffle_files, seed
        self.buffer, self.repeat = buffer, repeat

    def _file_order(self):
        epoch = 0
        while True:
            files = list(self.files)
            if self.shuffle:
                np.random.default_rng([self.seed, epoch]).shuffle(files)
            yield from files
            epoch += 1
            if not self.repeat:
                return

    def _docs(self, path):
        import pyarrow.parquet as pq
        pf = pq.ParquetFile(path)
        for rg in range(pf.num_row_groups):
            tab = pf.read_row_group(rg)
            field = next((f for f in self.TEXT_FIELDS if f in tab.column_names), None)
            if field is None:
                raise KeyError(f"no text field in {path}; columns={tab.column_names}")
            docs = tab.column(field).to_pylist()
            if self.shuffle:  # seeded within-row-group shuffle (file = its index in `files`)
                fi = self.files.index(path)
                order = np.random.default_rng([self.seed, fi, rg]).permutation(len(docs))
                docs = [docs[i] for i in order]
            for text in docs:
                yield text or ""

    def _interleaved_docs(self):
        """Round-robin over ``interleave`` open files; a finished file is
        replaced by the next one in the (shuffled, repeated) order."""
        from collections import deque
        files = self._file_order()
        iters = deque(self._docs(f) for f in itertools.islice(files, self.interleave))
        while iters:
            it = iters.popleft()
            try:
                doc = next(it)
            except StopIteration:
                f = next(files, None)
                if f is not None:
                    iters.append(self._docs(f))
                continue
            iters.append(it)
            yield doc

    def _tokens(self):
        for doc in self._interleaved_docs():
            if not doc:
                continue
            yield self.tok.encode(doc)

    def _batches(self):
        packed = pack_sequences(self._tokens(), self.seq_len, self.eos)
        while True:
            rows = list(itertools.islice(packed, self.batch_size))
            if len(rows) < self.batch_size:
                return
            yield np.stack(rows)

    def __iter__(self):
        return prefetch(self._batches(), self.buffer)
