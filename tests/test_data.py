"""Loader tests on synthetic local parquet (mirrors the reference's test_grain_data.py)."""
import itertools

import numpy as np
import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from hanuman_b200.data import ByteTokenizer, ParquetLoader, SyntheticLoader, prefetch


def _write(path, docs, field="content"):
    pq.write_table(pa.table({field: docs}), path, row_group_size=8)


@pytest.fixture
def shards(tmp_path):
    rng = np.random.default_rng(0)

    def make(n):
        return ["".join(chr(int(c)) for c in rng.integers(97, 123, size=int(rng.integers(20, 120))))
                for _ in range(n)]
    f0, f1 = tmp_path / "a.parquet", tmp_path / "b.parquet"
    _write(f0, make(40) + [""])
    _write(f1, make(40))
    return [str(f0), str(f1)]


def _loader(shards, seq_len=32, batch_size=4, **kw):
    tok = ByteTokenizer(256)
    return ParquetLoader(shards, tok, seq_len, batch_size, eos_id=tok.eos_id,
                         interleave=kw.pop("interleave", 2), buffer=2, **kw)


def test_batch_shape_dtype_and_range(shards):
    bs = list(itertools.islice(iter(_loader(shards)), 5))
    assert len(bs) == 5
    for b in bs:
        assert b.shape == (4, 32) and b.dtype == np.int32
        assert b.min() >= 0 and b.max() < 256


def test_packing_is_dense(shards):
    b = next(iter(_loader(shards, seq_len=16, batch_size=2)))
    assert b.shape == (2, 16) and (b >= 0).all()


def test_deterministic_given_seed(shards):
    a = next(iter(_loader(shards, seed=7)))
    b = next(iter(_loader(shards, seed=7)))
    np.testing.assert_array_equal(a, b)


def test_shuffle_seed_changes_order(shards):
    a = np.stack(list(itertools.islice(iter(_loader(shards, seed=1)), 3)))
    b = np.stack(list(itertools.islice(iter(_loader(shards, seed=2)), 3)))
    assert not np.array_equal(a, b)


def test_empty_documents_are_filtered(shards):
    bs = list(itertools.islice(iter(_loader(shards, seq_len=24, batch_size=3)), 3))
    assert len(bs) == 3 and all(b.shape == (3, 24) for b in bs)


def test_synthetic_loader_resumes_stream():
    a = SyntheticLoader(100, 2, 8, seed=3, rank=1, pin=False)
    it = iter(a)
    first = next(it)
    st = a.state_dict()  # state after the producer thread ran ahead is fine to restore
    b = SyntheticLoader(100, 2, 8, seed=3, rank=1, pin=False)
    c = SyntheticLoader(100, 2, 8, seed=3, rank=1, pin=False)
    assert (next(iter(b)) == first).all()
    c.load_state_dict(st)
    assert c.produced == st["produced"]


def test_prefetch_propagates_producer_errors():
    def gen():
        yield 1
        raise ValueError("boom")
    it = prefetch(gen(), 2)
    assert next(it) == 1
    with pytest.raises(ValueError):
        next(it)
