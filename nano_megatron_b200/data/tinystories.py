"""Pinned TinyStories sources: verified resumable download, story splitting, exact sampling.

The pinned revisions, byte sizes, sha256 digests and record counts identify the
upstream files (same pins as the reference,
src/nano_megatron/data/tinystories.py:17-43). Downloads try each mirror in
turn, resume a ``.part`` file with an HTTP Range request, verify size and
digest, and publish by rename. The 500k sample keeps the ``k`` stories with the
smallest blake2b-128 score of ``"<algorithm>\\0<seed>\\0<index>"`` (a bottom-k
selection in bounded memory, order preserved), so every builder picks the same
stories.
"""

from __future__ import annotations

import hashlib
import heapq
import json
import os
import uuid
from collections.abc import Callable, Iterator, Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any
from urllib.request import Request, urlopen

TINYSTORIES_CANONICAL_REVISION = "f54c09fd23315a6f9c86f9dc80f725de7d8f9c64"
TINYSTORIES_MIRROR_REVISION = "d71d0182cc67962186d395b75b2c180340904e00"
TINYSTORIES_TRAIN_BYTES = 1_924_281_556
TINYSTORIES_TRAIN_SHA256 = "c5cf5e22ff13614e830afbe61a99fbcbe8bcb7dd72252b989fa1117a368d401f"
TINYSTORIES_TRAIN_RECORDS = 2_119_719
TINYSTORIES_EMPTY_RECORDS = 230
TINYSTORIES_TRAIN_STORIES = TINYSTORIES_TRAIN_RECORDS - TINYSTORIES_EMPTY_RECORDS
TINYSTORIES_SAMPLE_STORIES = 500_000
TINYSTORIES_SAMPLE_SEED = 1234
TINYSTORIES_DELIMITER = b"<|endoftext|>"
TINYSTORIES_VALIDATION_BYTES = 19_447_282
TINYSTORIES_VALIDATION_SHA256 = "94e431816c4cce81ff71e4408ff8d3bda9a42e8d2663986697c3954288cb38b4"
TINYSTORIES_VALIDATION_STORIES = 21_990


def _urls(filename: str) -> tuple[str, str]:
    return ("https://www.modelscope.cn/api/v1/datasets/AI-ModelScope/TinyStories/repo?"
            f"Revision={TINYSTORIES_MIRROR_REVISION}&FilePath={filename}",
            "https://huggingface.co/datasets/roneneldan/TinyStories/resolve/"
            f"{TINYSTORIES_CANONICAL_REVISION}/{filename}?download=true")


TINYSTORIES_TRAIN_URLS = _urls("TinyStories-train.txt")
TINYSTORIES_VALIDATION_URLS = _urls("TinyStories-valid.txt")

SAMPLE_FORMAT = "nano-megatron-tinystories-sample"
SAMPLE_VERSION = 1
SELECTION_ALGORITHM = "blake2b-index-bottom-k-v1"

ProgressCallback = Callable[[int, int], None]


@dataclass(frozen=True, slots=True)
class FileVerification:
    path: Path
    size_bytes: int
    sha256: str


def _pos(name: str, v) -> int:
    if isinstance(v, bool) or not isinstance(v, int):
        raise TypeError(f"{name} must be an integer")
    if v < 1:
        raise ValueError(f"{name} must be positive")
    return v


def _nonneg(name: str, v) -> int:
    if isinstance(v, bool) or not isinstance(v, int):
        raise TypeError(f"{name} must be an integer")
    if v < 0:
        raise ValueError(f"{name} must be non-negative")
    return v


def _sha(v) -> str:
    if not isinstance(v, str) or len(v) != 64:
        raise ValueError("expected_sha256 must be a 64-character hexadecimal digest")
    try:
        bytes.fromhex(v)
    except ValueError as e:
        raise ValueError("expected_sha256 must be hexadecimal") from e
    return v.lower()


def sha256_file(path, *, chunk_size: int = 8 << 20) -> str:
    _pos("chunk_size", chunk_size)
    h = hashlib.sha256()
    with Path(path).open("rb") as f:
        for block in iter(lambda: f.read(chunk_size), b""):
            h.update(block)
    return h.hexdigest()


def verify_file(path, *, expected_size: int, expected_sha256: str) -> FileVerification:
    p = Path(path)
    size, want = _pos("expected_size", expected_size), _sha(expected_sha256)
    if not p.is_file():
        raise FileNotFoundError(f"expected file does not exist: {p}")
    if p.stat().st_size != size:
        raise ValueError(f"file size does not match pinned source: {p}: {p.stat().st_size} != "
                         f"{size}")
    got = sha256_file(p)
    if got != want:
        raise ValueError(f"file SHA256 does not match pinned source: {p}: {got} != {want}")
    return FileVerification(p.resolve(), size, got)


def _status(resp) -> int:
    s = getattr(resp, "status", None)
    if s is None:
        s = resp.getcode()
    if isinstance(s, bool) or not isinstance(s, int):
        raise RuntimeError(f"download response returned invalid HTTP status {s!r}")
    return s


def _fetch(url: str, dest: Path, *, size: int, sha: str, chunk: int, opener,
           progress) -> FileVerification:
    part = dest.with_name(dest.name + ".part")
    have = part.stat().st_size if part.exists() else 0
    if have > size:
        raise ValueError(f"partial download is larger than the pinned source: {part}: {have} > "
                         f"{size}")
    if have == size:
        try:
            v = verify_file(part, expected_size=size, expected_sha256=sha)
        except ValueError:
            part.unlink()
            raise
        part.replace(dest)
        return FileVerification(dest.resolve(), v.size_bytes, v.sha256)
    headers = {"User-Agent": "nano-megatron-tinystories/1"}
    if have:
        headers["Range"] = f"bytes={have}-"
    h = hashlib.sha256()
    if have:
        with part.open("rb") as f:
            for block in iter(lambda: f.read(chunk), b""):
                h.update(block)
    with opener(Request(url, headers=headers)) as resp:
        st = _status(resp)
        append = have > 0 and st == 206
        if append:
            cr = resp.headers.get("Content-Range", "")
            if not cr.startswith(f"bytes {have}-"):
                raise RuntimeError("download server returned an incompatible Content-Range for "
                                   f"resume: {cr!r}")
        elif st in (200, 206):
            have, h = 0, hashlib.sha256()       # server ignored Range: restart the .part file
        else:
            raise RuntimeError(f"download server returned HTTP status {st} for {url}")
        got = have
        with part.open("ab" if append else "wb") as f:
            if progress is not None:
                progress(got, size)
            for block in iter(lambda: resp.read(chunk), b""):
                f.write(block)
                h.update(block)
                got += len(block)
                if got > size:
                    f.close()
                    part.unlink(missing_ok=True)
                    raise ValueError(f"download exceeded pinned source size: {got} > {size}")
                if progress is not None:
                    progress(got, size)
            f.flush()
            os.fsync(f.fileno())
    if got != size:
        raise EOFError(f"download ended before the pinned source size: {got} != {size}; rerun to "
                       f"resume {part}")
    if h.hexdigest() != sha:
        part.unlink(missing_ok=True)
        raise ValueError("downloaded TinyStories source failed SHA256 verification: "
                         f"{h.hexdigest()} != {sha}")
    part.replace(dest)
    return FileVerification(dest.resolve(), got, h.hexdigest())


def download_pinned_file(destination, *, urls: Sequence[str] = TINYSTORIES_TRAIN_URLS,
                         expected_size: int = TINYSTORIES_TRAIN_BYTES,
                         expected_sha256: str = TINYSTORIES_TRAIN_SHA256,
                         chunk_size: int = 8 << 20, retries: int = 3, opener=urlopen,
                         progress: ProgressCallback | None = None) -> FileVerification:
    """Mirror fallback + Range resume + verification + atomic publish."""
    dest = Path(destination)
    size, sha = _pos("expected_size", expected_size), _sha(expected_sha256)
    chunk, tries = _pos("chunk_size", chunk_size), _pos("retries", retries)
    urls = tuple(urls)
    if not urls or any(not isinstance(u, str) or not u for u in urls):
        raise ValueError("urls must contain at least one non-empty URL")
    if dest.exists():
        return verify_file(dest, expected_size=size, expected_sha256=sha)
    dest.parent.mkdir(parents=True, exist_ok=True)
    failures = []
    for attempt in range(1, tries + 1):
        for url in urls:
            try:
                return _fetch(url, dest, size=size, sha=sha, chunk=chunk, opener=opener,
                              progress=progress)
            except (EOFError, OSError, RuntimeError, ValueError) as e:
                failures.append(f"attempt {attempt} {url}: {type(e).__name__}: {e}")
    raise RuntimeError("could not download pinned TinyStories source: " + "; ".join(failures))


def _story_bytes(path, *, delimiter: bytes = TINYSTORIES_DELIMITER,
                 chunk_size: int = 8 << 20) -> Iterator[bytes]:
    if not isinstance(delimiter, bytes) or not delimiter:
        raise ValueError("delimiter must be non-empty bytes")
    _pos("chunk_size", chunk_size)
    tail = b""
    with Path(path).open("rb") as f:
        for block in iter(lambda: f.read(chunk_size), b""):
            pieces = (tail + block).split(delimiter)
            tail = pieces.pop()
            for p in pieces:
                p = p.strip()
                if p:
                    yield p
    tail = tail.strip()
    if tail:
        yield tail


def iter_delimited_stories(path, *, delimiter: bytes = TINYSTORIES_DELIMITER,
                           chunk_size: int = 8 << 20) -> Iterator[str]:
    for s in _story_bytes(path, delimiter=delimiter, chunk_size=chunk_size):
        yield s.decode("utf-8")


def selection_score(seed: int, index: int) -> int:
    msg = f"{SELECTION_ALGORITHM}\0{seed}\0{index}".encode("ascii")
    return int.from_bytes(hashlib.blake2b(msg, digest_size=16).digest(), "big")


def select_story_indices(source, *, sample_size: int, seed: int,
                         expected_source_records: int | None,
                         progress: ProgressCallback | None = None) -> tuple[frozenset, int]:
    k, seed = _pos("sample_size", sample_size), _nonneg("seed", seed)
    if expected_source_records is not None:
        _pos("expected_source_records", expected_source_records)
        if k > expected_source_records:
            raise ValueError("sample_size cannot exceed expected_source_records")
    heap: list[tuple[int, int]] = []     # max-heap on (score, index) via negation
    total = 0
    for i, _ in enumerate(_story_bytes(source)):
        item = (-selection_score(seed, i), -i)
        if len(heap) < k:
            heapq.heappush(heap, item)
        elif item > heap[0]:
            heapq.heapreplace(heap, item)
        total = i + 1
        if progress is not None and total % 100_000 == 0:
            progress(total, expected_source_records or k)
    if total < k:
        raise ValueError(f"source contains only {total} stories; cannot select {k}")
    if expected_source_records is not None and total != expected_source_records:
        raise ValueError(f"TinyStories source record count changed: {total} != "
                         f"{expected_source_records}")
    if progress is not None:
        progress(total, expected_source_records or k)
    return frozenset(-ni for _, ni in heap), total


def _json(path: Path) -> dict:
    try:
        v = json.loads(path.read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError) as e:
        raise ValueError(f"could not read TinyStories metadata {path}: {e}") from e
    if not isinstance(v, dict):
        raise ValueError(f"TinyStories metadata must contain a JSON object: {path}")
    return v


def validate_sample_artifact(sample_path, metadata_path, *, sample_size: int, seed: int,
                             expected_source_records: int, expected_source_sha256: str) -> dict:
    sample, mfile = Path(sample_path), Path(metadata_path)
    if not sample.is_file() or not mfile.is_file():
        raise FileNotFoundError("TinyStories sample requires both JSONL and metadata files")
    meta = _json(mfile)
    sel, src, art = meta.get("selection"), meta.get("source"), meta.get("artifact")
    if meta.get("format") != SAMPLE_FORMAT or meta.get("version") != SAMPLE_VERSION:
        raise ValueError("TinyStories sample metadata format/version is unsupported")
    if not all(isinstance(x, dict) for x in (sel, src, art)):
        raise ValueError("TinyStories sample metadata sections are invalid")
    want = {"algorithm": SELECTION_ALGORITHM, "records": sample_size, "seed": seed,
            "source_records": expected_source_records}
    if sel != want:
        raise ValueError(f"TinyStories sample selection metadata does not match: {sel!r} != "
                         f"{want!r}")
    if src.get("sha256") != _sha(expected_source_sha256):
        raise ValueError("TinyStories sample was built from a different source digest")
    if art.get("records") != sample_size or art.get("size_bytes") != sample.stat().st_size:
        raise ValueError("TinyStories sample artifact count/size metadata does not match")
    if art.get("sha256") != sha256_file(sample):
        raise ValueError("TinyStories sample JSONL failed SHA256 verification")
    return meta


def create_exact_sample(source_path, sample_path, metadata_path, *,
                        source_verification: FileVerification,
                        sample_size: int = TINYSTORIES_SAMPLE_STORIES,
                        seed: int = TINYSTORIES_SAMPLE_SEED,
                        expected_source_records: int = TINYSTORIES_TRAIN_STORIES,
                        progress: ProgressCallback | None = None) -> dict[str, Any]:
    """Create (or validate and reuse) the deterministic JSONL sample."""
    src = Path(source_path).resolve()
    out = Path(sample_path).resolve()
    mfile = Path(metadata_path).resolve()
    if src != source_verification.path.resolve():
        raise ValueError("source_verification does not describe source_path")
    if not src.is_file() or src.stat().st_size != source_verification.size_bytes:
        raise ValueError("source_path size changed after source verification")
    if out == mfile or src in (out, mfile):
        raise ValueError("source, sample, and metadata paths must be distinct")
    if out.exists() or mfile.exists():
        if not out.is_file() or not mfile.is_file():
            raise FileExistsError("refusing to replace an incomplete TinyStories sample "
                                  f"artifact; remove both {out} and {mfile} to rebuild")
        meta = validate_sample_artifact(out, mfile, sample_size=sample_size, seed=seed,
                                        expected_source_records=expected_source_records,
                                        expected_source_sha256=source_verification.sha256)
        return {**meta, "reused": True}
    out.parent.mkdir(parents=True, exist_ok=True)
    mfile.parent.mkdir(parents=True, exist_ok=True)
    chosen, total = select_story_indices(src, sample_size=sample_size, seed=seed,
                                         expected_source_records=expected_source_records,
                                         progress=progress)
    tag = uuid.uuid4().hex
    otmp = out.with_name(f".{out.name}.{tag}.tmp")
    mtmp = mfile.with_name(f".{mfile.name}.{tag}.tmp")
    h = hashlib.sha256()
    written = records = 0
    published = False
    try:
        with otmp.open("xb") as f:
            for i, story in enumerate(_story_bytes(src)):
                records = i + 1
                if i not in chosen:
                    continue
                line = (json.dumps({"text": story.decode("utf-8")}, ensure_ascii=False,
                                   separators=(",", ":")) + "\n").encode("utf-8")
                f.write(line)
                h.update(line)
                written += 1
                if progress is not None and written % 100_000 == 0:
                    progress(written, sample_size)
            f.flush()
            os.fsync(f.fileno())
        if written != sample_size:
            raise RuntimeError(f"sample writer emitted {written} stories, expected {sample_size}")
        if records != expected_source_records:
            raise RuntimeError("TinyStories source record count changed between sample passes: "
                               f"{records} != {expected_source_records}")
        if progress is not None:
            progress(written, sample_size)
        pinned = source_verification.sha256 == TINYSTORIES_TRAIN_SHA256
        meta = {
            "artifact": {"format": "jsonl", "path": str(out), "records": written,
                         "sha256": h.hexdigest(), "size_bytes": otmp.stat().st_size,
                         "text_key": "text"},
            "format": SAMPLE_FORMAT,
            "selection": {"algorithm": SELECTION_ALGORITHM, "records": sample_size, "seed": seed,
                          "source_records": total},
            "source": {"canonical_revision": TINYSTORIES_CANONICAL_REVISION,
                       "empty_records_excluded": TINYSTORIES_EMPTY_RECORDS if pinned else None,
                       "mirror_revision": TINYSTORIES_MIRROR_REVISION,
                       "non_empty_stories": total, "path": str(src),
                       "records_including_empty": TINYSTORIES_TRAIN_RECORDS if pinned else None,
                       "sha256": source_verification.sha256,
                       "size_bytes": source_verification.size_bytes,
                       "story_delimiter": TINYSTORIES_DELIMITER.decode("ascii")},
            "version": SAMPLE_VERSION}
        mtmp.write_text(json.dumps(meta, ensure_ascii=False, indent=2, sort_keys=True) + "\n",
                        encoding="utf-8")
        otmp.replace(out)
        published = True
        mtmp.replace(mfile)
    except BaseException:
        otmp.unlink(missing_ok=True)
        mtmp.unlink(missing_ok=True)
        if published:
            out.unlink(missing_ok=True)
        raise
    return {**meta, "reused": False}


def prepare_tinystories_500k(data_dir=Path("data/raw/tinystories"), *,
                             urls: Sequence[str] = TINYSTORIES_TRAIN_URLS,
                             progress: ProgressCallback | None = None) -> dict[str, Any]:
    d = Path(data_dir)
    src, sample, meta = d / "TinyStories-train.txt", d / "train_500k.jsonl", \
        d / "train_500k.metadata.json"
    v = download_pinned_file(src, urls=urls, progress=progress)
    m = create_exact_sample(src, sample, meta, source_verification=v, progress=progress)
    return {"command": "prepare-tinystories-500k", "sample": m,
            "sample_metadata": str(meta.resolve()), "sample_output": str(sample.resolve()),
            "source": {"path": str(v.path), "sha256": v.sha256, "size_bytes": v.size_bytes}}
