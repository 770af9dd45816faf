"""Data path: corpora, native window gather, resumable loader, TinyStories tools (CPU).

Reference counterparts: tests/unit/test_data_corpus.py, test_mmap_corpus.py,
test_data_loader_resume.py, test_tinystories.py.
"""

from __future__ import annotations

import importlib.util
import io
import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

TEXTS = [f"story number {i}: the cat sat on the mat and looked at bird {i % 7}." for i in
         range(60)]


@pytest.fixture(scope="module")
def tok(tmp_path_factory):
    from nano_megatron_b200.tokenizer import ByteBPETrainingConfig, ByteLevelBPETokenizer

    d = tmp_path_factory.mktemp("tok") / "t"
    ByteLevelBPETokenizer.train(TEXTS, ByteBPETrainingConfig(vocab_size=300)).save(d)
    return ByteLevelBPETokenizer.load(d)


def test_pt_and_mmap_corpus_share_fingerprint(tmp_path, tok):
    from nano_megatron_b200.data import MMapTokenCorpus, TokenCorpus, preprocess_texts_mmap

    c = TokenCorpus.from_texts(TEXTS, tok)
    c.save(tmp_path / "c.pt")
    c2 = TokenCorpus.load(tmp_path / "c.pt")
    assert c2 == c and c2.fingerprint == c.fingerprint
    m = preprocess_texts_mmap(TEXTS, tmp_path / "mm", tok, encoding_batch_size=7)
    assert m.fingerprint == c.fingerprint
    assert m.token_dtype == np.dtype("<u2")
    np.testing.assert_array_equal(np.asarray(m.tokens, dtype=np.int64), c.tokens.numpy())
    assert MMapTokenCorpus.load(tmp_path / "mm").fingerprint == c.fingerprint
    with pytest.raises(FileExistsError):
        preprocess_texts_mmap(TEXTS, tmp_path / "mm", tok)
    ref = Path(__file__).parents[1] / "baseline" / "_ref"
    if (ref / "nano_megatron").is_dir():
        sys.path.insert(0, str(ref))
        try:
            from nano_megatron.data import MMapTokenCorpus as RM, TokenCorpus as RT

            assert RM.load(tmp_path / "mm").fingerprint == c.fingerprint
            assert RT.load(tmp_path / "c.pt").fingerprint == c.fingerprint
        finally:
            sys.path.remove(str(ref))


def test_native_gather_matches_python_windows(tmp_path, tok):
    from nano_megatron_b200.data import FixedLengthTokenDataset, MMapTokenDataset, TokenCorpus
    from nano_megatron_b200.data.mmap_corpus import preprocess_texts_mmap
    from nano_megatron_b200.native import native

    c = TokenCorpus.from_texts(TEXTS, tok)
    preprocess_texts_mmap(TEXTS, tmp_path / "mm", tok)
    S = 16
    for ds in (FixedLengthTokenDataset(c.tokens, S), MMapTokenDataset(tmp_path / "mm", S)):
        assert len(ds) == (c.tokens.numel() - 1) // S
        idx = torch.randperm(len(ds))[:33]
        out = torch.empty(33, S + 1, dtype=torch.int64)
        ds.native_source().gather(ds.window_starts(idx), S + 1, out, 3)
        for r, i in enumerate(idx.tolist()):
            torch.testing.assert_close(out[r], c.tokens[i * S:i * S + S + 1])
        s = ds[5]
        torch.testing.assert_close(s["input_ids"], c.tokens[80:96])
        torch.testing.assert_close(s["labels"], c.tokens[81:97])
    src = native().TokenSource(c.tokens)
    with pytest.raises(IndexError):
        src.gather(torch.tensor([c.tokens.numel() - 3]), 8, torch.empty(1, 8, dtype=torch.int64))
    # uint32 storage path (vocab > 65536)
    big = torch.randint(0, 70000, (4097,))
    (tmp_path / "u4.bin").write_bytes(big.numpy().astype("<u4").tobytes())
    s4 = native().TokenSource(str(tmp_path / "u4.bin"), 4, 4097)
    o = torch.empty(2, 9, dtype=torch.int64)
    s4.gather(torch.tensor([0, 4000]), 9, o, 2)
    torch.testing.assert_close(o[1], big[4000:4009])


def _reference_order(n, replicas, rank, seed, epoch, shuffle=True):
    from torch.utils.data import DistributedSampler

    s = DistributedSampler(range(n), num_replicas=replicas, rank=rank, shuffle=shuffle, seed=seed,
                           drop_last=True)
    s.set_epoch(epoch)
    return list(s)


def test_loader_order_resume_and_reshard(tmp_path, tok):
    from nano_megatron_b200.data import StatefulDataLoader, TokenCorpus
    from nano_megatron_b200.data.datasets import FixedLengthTokenDataset

    c = TokenCorpus.from_texts(TEXTS * 4, tok)
    ds = FixedLengthTokenDataset(c.tokens, 8)
    n = len(ds)

    def make(replicas, rank):
        return StatefulDataLoader(ds, local_batch_size=4, replica_count=replicas,
                                  replica_index=rank, shuffle=True, shuffle_seed=11,
                                  data_fingerprint=ds.fingerprint)

    # replica order equals torch's DistributedSampler order, epoch after epoch
    ld = make(2, 1)
    spe = ld.samples_per_epoch
    seen = []
    for _ in range(2 * ld.batches_per_epoch):
        seen.append(next(ld)["input_ids"])
    want = []
    for ep in range(2):
        o = _reference_order(n, 2, 1, 11, ep)[:spe // 2]
        want += o
    got_rows = torch.cat(seen)
    for r, i in enumerate(want):
        torch.testing.assert_close(got_rows[r], c.tokens[i * 8:i * 8 + 8])
    # exact resume mid-epoch
    a = make(2, 0)
    for _ in range(3):
        next(a)
    st = a.state_dict()
    nxt = next(a)["labels"]
    b = make(2, 0)
    b.load_state_dict(st)
    torch.testing.assert_close(next(b)["labels"], nxt)
    # reshard DP2 -> DP1: the global prefix continues with the DP1 order
    one = make(1, 0)
    one.load_state_dict({"epoch": st["epoch"], "shuffle_seed": 11,
                         "sample_offset": st["sample_offset"]})
    o1 = _reference_order(n, 1, 0, 11, st["epoch"])
    first = next(one)["input_ids"]
    i0 = o1[st["sample_offset"]]
    torch.testing.assert_close(first[0], c.tokens[i0 * 8:i0 * 8 + 8])
    with pytest.raises(RuntimeError):
        b.load_state_dict({**st, "shuffle_seed": 12})
    a.close()
    b.close()


def test_random_dataset_matches_reference_generator():
    from nano_megatron_b200.data import RandomTokenDataset

    ds = RandomTokenDataset(num_samples=10, sequence_length=7, vocab_size=50, seed=3)
    g = torch.Generator().manual_seed(3 + 4)
    w = torch.randint(50, (8,), generator=g)
    torch.testing.assert_close(ds[4]["input_ids"], w[:-1])


class _FakeResponse(io.BytesIO):
    def __init__(self, body: bytes, status: int, headers=None) -> None:
        super().__init__(body)
        self.status = status
        self.headers = headers or {}

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def test_tinystories_download_sample_and_corpus(tmp_path, tok):
    import hashlib

    from nano_megatron_b200.data import tinystories as ts
    from nano_megatron_b200.data.tinystories_corpus import (build_tinystories_corpus,
                                                            validate_tinystories_corpus)
    from nano_megatron_b200.tokenizer import ByteBPETrainingConfig, ByteLevelBPETokenizer

    stories = [f"Once upon a time {i} there was a fox." for i in range(40)]
    body = b"".join(s.encode() + b"\n<|endoftext|>\n" for s in stories) + b"  <|endoftext|>"
    sha = hashlib.sha256(body).hexdigest()
    calls = []

    def opener(req):
        calls.append(req.headers.get("Range"))
        rng = req.headers.get("Range")
        if len(calls) == 1:                       # first attempt: truncated body
            return _FakeResponse(body[:100], 200)
        start = int(rng.split("=")[1].rstrip("-"))
        return _FakeResponse(body[start:], 206, {"Content-Range": f"bytes {start}-"})

    dst = tmp_path / "train.txt"
    v = ts.download_pinned_file(dst, urls=["http://mirror/a"], expected_size=len(body),
                                expected_sha256=sha, opener=opener, retries=2)
    assert v.sha256 == sha and dst.read_bytes() == body and calls[1] == "bytes=100-"
    assert list(ts.iter_delimited_stories(dst, chunk_size=17)) == stories
    chosen, total = ts.select_story_indices(dst, sample_size=10, seed=5,
                                            expected_source_records=40)
    scores = sorted(range(40), key=lambda i: ts.selection_score(5, i))[:10]
    assert chosen == frozenset(scores) and total == 40
    meta = ts.create_exact_sample(dst, tmp_path / "s.jsonl", tmp_path / "s.json",
                                  source_verification=v, sample_size=10, seed=5,
                                  expected_source_records=40)
    assert meta["reused"] is False and meta["artifact"]["records"] == 10
    again = ts.create_exact_sample(dst, tmp_path / "s.jsonl", tmp_path / "s.json",
                                   source_verification=v, sample_size=10, seed=5,
                                   expected_source_records=40)
    assert again["reused"] is True
    val = tmp_path / "valid.txt"
    val.write_bytes(b"<|endoftext|>".join(f"A short tale {i}.".encode() for i in range(12)))
    vv = ts.verify_file(val, expected_size=val.stat().st_size,
                        expected_sha256=hashlib.sha256(val.read_bytes()).hexdigest())
    tdir = tmp_path / "tok8"
    ByteLevelBPETokenizer.train(stories, ByteBPETrainingConfig(vocab_size=280)).save(tdir)
    out = build_tinystories_corpus(dst, val, tdir, tmp_path / "corpus", train_verification=v,
                                   validation_verification=vv, expected_train_stories=40,
                                   expected_validation_stories=12,
                                   expected_vocab_size=ByteLevelBPETokenizer.load(tdir).vocab_size)
    assert out["reused"] is False
    m = validate_tinystories_corpus(tmp_path / "corpus", tokenizer_path=tdir)
    assert m["corpora"]["train"]["documents"] == 40
