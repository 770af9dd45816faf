"""TinyStories, pinned: download with resume and verification, story splitting, and the
deterministic 500k-story training sample.

Sources. Each upstream file is pinned by revision, byte size, SHA-256 and story count
(:data:`TRAIN`, :data:`VALIDATION`); a download tries each mirror in turn, resumes a
``<name>.part`` file with an HTTP ``Range`` request, hashes while it writes, and appears
under its final name (a rename) only once size and digest match.

Stories. The raw files are stories separated by ``<|endoftext|>``; a story is the text
between two separators with surrounding whitespace removed, and blank stories are
skipped (the pinned train file has 230 of them).

Sample. The training sample keeps the ``k`` stories with the smallest score
``blake2b-128("<algorithm>\\0<seed>\\0<story index>")`` (read as a big-endian integer),
written in their original order. Any builder that hashes the same way picks the same
stories, in one pass and with memory for ``k`` entries only. A metadata JSON next to the
JSONL sample records the selection, the source and the sample's own digest; a sample whose
metadata does not verify is rebuilt by nobody silently.

The pins, URLs, the score recipe and the metadata layout are the reference's
(src/nano_megatron/data/tinystories.py), so both frameworks build byte-identical samples.
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
TINYSTORIES_DELIMITER = b"<|endoftext|>"


def _mirrors(filename: str) -> tuple[str, str]:
    """ModelScope mirror first, the Hugging Face original second."""
    return (f"https://www.modelscope.cn/api/v1/datasets/AI-ModelScope/TinyStories/repo?"
            f"Revision={TINYSTORIES_MIRROR_REVISION}&FilePath={filename}",
            f"https://huggingface.co/datasets/roneneldan/TinyStories/resolve/"
            f"{TINYSTORIES_CANONICAL_REVISION}/{filename}?download=true")


@dataclass(frozen=True)
class PinnedFile:
    filename: str
    size: int
    sha256: str
    stories: int              # non-empty stories

    @property
    def urls(self) -> tuple[str, str]:
        return _mirrors(self.filename)


TRAIN = PinnedFile("TinyStories-train.txt", 1_924_281_556,
                   "c5cf5e22ff13614e830afbe61a99fbcbe8bcb7dd72252b989fa1117a368d401f",
                   2_119_719 - 230)
VALIDATION = PinnedFile("TinyStories-valid.txt", 19_447_282,
                        "94e431816c4cce81ff71e4408ff8d3bda9a42e8d2663986697c3954288cb38b4",
                        21_990)

TINYSTORIES_TRAIN_BYTES = TRAIN.size
TINYSTORIES_TRAIN_SHA256 = TRAIN.sha256
TINYSTORIES_TRAIN_RECORDS = 2_119_719           # separator-delimited records, blanks included
TINYSTORIES_EMPTY_RECORDS = 230
TINYSTORIES_TRAIN_STORIES = TRAIN.stories
TINYSTORIES_TRAIN_URLS = TRAIN.urls
TINYSTORIES_VALIDATION_BYTES = VALIDATION.size
TINYSTORIES_VALIDATION_SHA256 = VALIDATION.sha256
TINYSTORIES_VALIDATION_STORIES = VALIDATION.stories
TINYSTORIES_VALIDATION_URLS = VALIDATION.urls
TINYSTORIES_SAMPLE_STORIES = 500_000
TINYSTORIES_SAMPLE_SEED = 1234

SAMPLE_FORMAT = "nano-megatron-tinystories-sample"
SAMPLE_VERSION = 1
SELECTION_ALGORITHM = "blake2b-index-bottom-k-v1"
_CHUNK = 8 << 20

ProgressCallback = Callable[[int, int], None]


@dataclass(frozen=True, slots=True)
class FileVerification:
    path: Path
    size_bytes: int
    sha256: str


# ---------------------------------------------------------------------- small checks
def _int_at_least(name: str, v, low: int) -> int:
    if isinstance(v, bool) or not isinstance(v, int):
        raise TypeError(f"{name} must be an int, got {v!r}")
    if v < low:
        raise ValueError(f"{name} must be >= {low}, got {v}")
    return v


def _digest(v) -> str:
    ok = isinstance(v, str) and len(v) == 64 and all(c in "0123456789abcdefABCDEF" for c in v)
    if not ok:
        raise ValueError(f"{v!r} is not a SHA-256 hex digest (64 hex characters)")
    return v.lower()


def sha256_file(path, *, chunk_size: int = _CHUNK) -> str:
    _int_at_least("chunk_size", chunk_size, 1)
    h = hashlib.sha256()
    with Path(path).open("rb") as f:
        while block := f.read(chunk_size):
            h.update(block)
    return h.hexdigest()


def verify_file(path, *, expected_size: int, expected_sha256: str) -> FileVerification:
    """Size and SHA-256 of ``path`` against the pins (size first: it is free)."""
    p = Path(path)
    size = _int_at_least("expected_size", expected_size, 1)
    want = _digest(expected_sha256)
    if not p.is_file():
        raise FileNotFoundError(f"{p} does not exist")
    have = p.stat().st_size
    if have != size:
        raise ValueError(f"{p} is {have} bytes; the pinned source is {size}")
    got = sha256_file(p)
    if got != want:
        raise ValueError(f"{p} has SHA-256 {got}; the pinned source has {want}")
    return FileVerification(p.resolve(), size, got)


# ---------------------------------------------------------------------- download
class _Transfer:
    """One attempt at one URL: continue ``<dest>.part`` and publish it when complete."""

    def __init__(self, dest: Path, size: int, sha: str, chunk: int, opener, progress) -> None:
        self.dest, self.part = dest, dest.with_name(dest.name + ".part")
        self.size, self.sha, self.chunk = size, sha, chunk
        self.opener, self.progress = opener, progress

    def _publish(self, digest: str) -> FileVerification:
        self.part.replace(self.dest)
        return FileVerification(self.dest.resolve(), self.size, digest)

    def _hash_of_part(self) -> "hashlib._Hash":
        h = hashlib.sha256()
        with self.part.open("rb") as f:
            while block := f.read(self.chunk):
                h.update(block)
        return h

    def run(self, url: str) -> FileVerification:
        start = self.part.stat().st_size if self.part.exists() else 0
        if start > self.size:
            raise ValueError(f"{self.part} holds {start} bytes, more than the pinned "
                             f"{self.size}")
        if start == self.size:                       # finished earlier, never published
            try:
                v = verify_file(self.part, expected_size=self.size, expected_sha256=self.sha)
            except ValueError:
                self.part.unlink()
                raise
            return self._publish(v.sha256)
        headers = {"User-Agent": "nano-megatron-tinystories/1"}
        if start:
            headers["Range"] = f"bytes={start}-"
        with self.opener(Request(url, headers=headers)) as resp:
            status = getattr(resp, "status", None)
            status = resp.getcode() if status is None else status
            if isinstance(status, bool) or not isinstance(status, int):
                raise RuntimeError(f"{url}: unusable HTTP status {status!r}")
            if status not in (200, 206):
                raise RuntimeError(f"{url}: HTTP status {status}")
            resumed = start > 0 and status == 206
            if resumed:
                span = resp.headers.get("Content-Range", "")
                if not span.startswith(f"bytes {start}-"):
                    raise RuntimeError(f"{url}: asked to resume at byte {start}, server sent "
                                       f"Content-Range {span!r}")
                h = self._hash_of_part()
            else:                                     # full body (Range ignored or no .part)
                start, h = 0, hashlib.sha256()
            got = self._stream(resp, h, start, append=resumed)
        if got != self.size:
            raise EOFError(f"{url}: stream ended at byte {got} of {self.size}; run again to "
                           f"resume {self.part}")
        digest = h.hexdigest()
        if digest != self.sha:
            self.part.unlink(missing_ok=True)
            raise ValueError(f"{url}: downloaded file has SHA-256 {digest}, pinned {self.sha}")
        return self._publish(digest)

    def _stream(self, resp, h, got: int, *, append: bool) -> int:
        with self.part.open("ab" if append else "wb") as f:
            if self.progress is not None:
                self.progress(got, self.size)
            while block := resp.read(self.chunk):
                got += len(block)
                if got > self.size:
                    f.close()
                    self.part.unlink(missing_ok=True)
                    raise ValueError(f"server sent more than the pinned {self.size} bytes")
                f.write(block)
                h.update(block)
                if self.progress is not None:
                    self.progress(got, self.size)
            f.flush()
            os.fsync(f.fileno())
        return got


def download_pinned_file(destination, *, urls: Sequence[str] = TINYSTORIES_TRAIN_URLS,
                         expected_size: int = TINYSTORIES_TRAIN_BYTES,
                         expected_sha256: str = TINYSTORIES_TRAIN_SHA256,
                         chunk_size: int = _CHUNK, retries: int = 3, opener=urlopen,
                         progress: ProgressCallback | None = None) -> FileVerification:
    """Verified copy of a pinned file at ``destination`` (an existing file is verified,
    not fetched again). Up to ``retries`` rounds over ``urls``; every failure is named in
    the final error."""
    dest = Path(destination)
    size = _int_at_least("expected_size", expected_size, 1)
    sha = _digest(expected_sha256)
    chunk = _int_at_least("chunk_size", chunk_size, 1)
    rounds = _int_at_least("retries", retries, 1)
    urls = tuple(urls)
    if not urls or not all(isinstance(u, str) and u for u in urls):
        raise ValueError("urls must be one or more non-empty strings")
    if dest.exists():
        return verify_file(dest, expected_size=size, expected_sha256=sha)
    dest.parent.mkdir(parents=True, exist_ok=True)
    transfer = _Transfer(dest, size, sha, chunk, opener, progress)
    errors = []
    for r in range(rounds):
        for url in urls:
            try:
                return transfer.run(url)
            except (EOFError, OSError, RuntimeError, ValueError) as e:
                errors.append(f"[round {r + 1}] {url}: {type(e).__name__}: {e}")
    raise RuntimeError("download failed on every mirror: " + " | ".join(errors))


# ---------------------------------------------------------------------- stories
def _story_bytes(path, *, delimiter: bytes = TINYSTORIES_DELIMITER,
                 chunk_size: int = _CHUNK) -> Iterator[bytes]:
    """Stripped, non-blank byte strings between separators, streamed in chunks."""
    if not isinstance(delimiter, bytes) or not delimiter:
        raise ValueError("the story delimiter must be non-empty bytes")
    _int_at_least("chunk_size", chunk_size, 1)
    buf = bytearray()
    with Path(path).open("rb") as f:
        while block := f.read(chunk_size):
            buf += block
            begin = 0
            while (cut := buf.find(delimiter, begin)) >= 0:
                story = bytes(buf[begin:cut]).strip()
                if story:
                    yield story
                begin = cut + len(delimiter)
            del buf[:begin]
    last = bytes(buf).strip()
    if last:
        yield last


def iter_delimited_stories(path, *, delimiter: bytes = TINYSTORIES_DELIMITER,
                           chunk_size: int = _CHUNK) -> Iterator[str]:
    return (s.decode("utf-8") for s in _story_bytes(path, delimiter=delimiter,
                                                    chunk_size=chunk_size))


def selection_score(seed: int, index: int) -> int:
    key = f"{SELECTION_ALGORITHM}\0{seed}\0{index}".encode("ascii")
    return int.from_bytes(hashlib.blake2b(key, digest_size=16).digest(), "big")


def select_story_indices(source, *, sample_size: int, seed: int,
                         expected_source_records: int | None,
                         progress: ProgressCallback | None = None) -> tuple[frozenset, int]:
    """Indices of the ``sample_size`` lowest-scoring stories, and the story count."""
    k = _int_at_least("sample_size", sample_size, 1)
    seed = _int_at_least("seed", seed, 0)
    if expected_source_records is not None:
        _int_at_least("expected_source_records", expected_source_records, 1)
        if k > expected_source_records:
            raise ValueError(f"cannot sample {k} of {expected_source_records} stories")
    count = 0
    total_hint = expected_source_records or k

    def scored():
        nonlocal count
        for i, _ in enumerate(_story_bytes(source)):
            count = i + 1
            if progress is not None and count % 100_000 == 0:
                progress(count, total_hint)
            yield selection_score(seed, i), i

    best = heapq.nsmallest(k, scored())          # keeps a k-entry heap while streaming
    if count < k:
        raise ValueError(f"{source} has {count} stories, fewer than the {k} requested")
    if expected_source_records is not None and count != expected_source_records:
        raise ValueError(f"{source} has {count} stories; the pinned source has "
                         f"{expected_source_records}")
    if progress is not None:
        progress(count, total_hint)
    return frozenset(i for _, i in best), count


# ---------------------------------------------------------------------- the sample
def _read_json_object(path: Path) -> dict:
    try:
        obj = json.loads(path.read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError) as e:
        raise ValueError(f"unreadable sample metadata {path}: {e}") from e
    if not isinstance(obj, dict):
        raise ValueError(f"sample metadata {path} is not a JSON object")
    return obj


def validate_sample_artifact(sample_path, metadata_path, *, sample_size: int, seed: int,
                             expected_source_records: int, expected_source_sha256: str) -> dict:
    """Check an existing sample against its metadata and the requested selection."""
    sample, mpath = Path(sample_path), Path(metadata_path)
    if not (sample.is_file() and mpath.is_file()):
        raise FileNotFoundError(f"a sample is the pair {sample} + {mpath}; one is missing")
    meta = _read_json_object(mpath)
    if (meta.get("format"), meta.get("version")) != (SAMPLE_FORMAT, SAMPLE_VERSION):
        raise ValueError(f"{mpath}: format/version {meta.get('format')!r}/"
                         f"{meta.get('version')!r} is not {SAMPLE_FORMAT!r}/{SAMPLE_VERSION}")
    parts = {k: meta.get(k) for k in ("selection", "source", "artifact")}
    bad = [k for k, v in parts.items() if not isinstance(v, dict)]
    if bad:
        raise ValueError(f"{mpath}: sections {bad} are not objects")
    want = {"algorithm": SELECTION_ALGORITHM, "records": sample_size, "seed": seed,
            "source_records": expected_source_records}
    if parts["selection"] != want:
        raise ValueError(f"{mpath}: selection {parts['selection']!r} differs from the "
                         f"requested {want!r}")
    if parts["source"].get("sha256") != _digest(expected_source_sha256):
        raise ValueError(f"{mpath}: sample was drawn from another source file")
    art = parts["artifact"]
    if (art.get("records"), art.get("size_bytes")) != (sample_size, sample.stat().st_size):
        raise ValueError(f"{mpath}: the sample's story count or byte size changed")
    if art.get("sha256") != sha256_file(sample):
        raise ValueError(f"{sample}: content does not match the SHA-256 in {mpath}")
    return meta


def _sample_metadata(out: Path, src: Path, v: FileVerification, *, written: int,
                     digest: str, size: int, sample_size: int, seed: int,
                     total: int) -> dict[str, Any]:
    pinned = v.sha256 == TINYSTORIES_TRAIN_SHA256
    return {
        "artifact": {"format": "jsonl", "path": str(out), "records": written, "sha256": digest,
                     "size_bytes": size, "text_key": "text"},
        "format": SAMPLE_FORMAT,
        "selection": {"algorithm": SELECTION_ALGORITHM, "records": sample_size, "seed": seed,
                      "source_records": total},
        "source": {"canonical_revision": TINYSTORIES_CANONICAL_REVISION,
                   "empty_records_excluded": TINYSTORIES_EMPTY_RECORDS if pinned else None,
                   "mirror_revision": TINYSTORIES_MIRROR_REVISION, "non_empty_stories": total,
                   "path": str(src),
                   "records_including_empty": TINYSTORIES_TRAIN_RECORDS if pinned else None,
                   "sha256": v.sha256, "size_bytes": v.size_bytes,
                   "story_delimiter": TINYSTORIES_DELIMITER.decode("ascii")},
        "version": SAMPLE_VERSION}


def create_exact_sample(source_path, sample_path, metadata_path, *,
                        source_verification: FileVerification,
                        sample_size: int = TINYSTORIES_SAMPLE_STORIES,
                        seed: int = TINYSTORIES_SAMPLE_SEED,
                        expected_source_records: int = TINYSTORIES_TRAIN_STORIES,
                        progress: ProgressCallback | None = None) -> dict[str, Any]:
    """Write the sample JSONL + metadata (two passes over the source: select, then write),
    or verify and reuse an existing pair. Both files appear by rename, sample first."""
    src, out, mpath = (Path(p).resolve() for p in (source_path, sample_path, metadata_path))
    if src != source_verification.path.resolve():
        raise ValueError(f"the verification is for {source_verification.path}, not {src}")
    if not src.is_file() or src.stat().st_size != source_verification.size_bytes:
        raise ValueError(f"{src} changed since it was verified")
    if len({src, out, mpath}) != 3:
        raise ValueError("source, sample and metadata must be three different paths")
    if out.exists() or mpath.exists():
        if not (out.is_file() and mpath.is_file()):
            raise FileExistsError(f"half a sample exists ({out}, {mpath}); delete both to "
                                  "rebuild it")
        meta = validate_sample_artifact(out, mpath, sample_size=sample_size, seed=seed,
                                        expected_source_records=expected_source_records,
                                        expected_source_sha256=source_verification.sha256)
        return dict(meta, reused=True)
    for d in {out.parent, mpath.parent}:
        d.mkdir(parents=True, exist_ok=True)
    keep, total = select_story_indices(src, sample_size=sample_size, seed=seed,
                                       expected_source_records=expected_source_records,
                                       progress=progress)
    tag = uuid.uuid4().hex
    out_tmp = out.with_name(f".{out.name}.{tag}.tmp")
    meta_tmp = mpath.with_name(f".{mpath.name}.{tag}.tmp")
    h = hashlib.sha256()
    written = seen = 0
    sample_published = False
    try:
        with out_tmp.open("xb") as f:
            for i, story in enumerate(_story_bytes(src)):
                seen = i + 1
                if i in keep:
                    row = json.dumps({"text": story.decode("utf-8")}, ensure_ascii=False,
                                     separators=(",", ":")).encode("utf-8") + b"\n"
                    f.write(row)
                    h.update(row)
                    written += 1
                    if progress is not None and written % 100_000 == 0:
                        progress(written, sample_size)
            f.flush()
            os.fsync(f.fileno())
        if written != sample_size:
            raise RuntimeError(f"wrote {written} stories instead of {sample_size}")
        if seen != expected_source_records:
            raise RuntimeError(f"{src} changed between the two passes ({seen} stories, "
                               f"expected {expected_source_records})")
        if progress is not None:
            progress(written, sample_size)
        meta = _sample_metadata(out, src, source_verification, written=written,
                                digest=h.hexdigest(), size=out_tmp.stat().st_size,
                                sample_size=sample_size, seed=seed, total=total)
        meta_tmp.write_text(json.dumps(meta, ensure_ascii=False, indent=2, sort_keys=True)
                            + "\n", encoding="utf-8")
        out_tmp.replace(out)
        sample_published = True
        meta_tmp.replace(mpath)
    except BaseException:
        for p in (out_tmp, meta_tmp) + ((out,) if sample_published else ()):
            p.unlink(missing_ok=True)
        raise
    return dict(meta, reused=False)


def prepare_tinystories_500k(data_dir=Path("data/raw/tinystories"), *,
                             urls: Sequence[str] = TINYSTORIES_TRAIN_URLS,
                             progress: ProgressCallback | None = None) -> dict[str, Any]:
    """Download the pinned train file into ``data_dir`` and build the 500k sample."""
    d = Path(data_dir)
    src = d / TRAIN.filename
    sample, mpath = d / "train_500k.jsonl", d / "train_500k.metadata.json"
    v = download_pinned_file(src, urls=urls, progress=progress)
    meta = create_exact_sample(src, sample, mpath, source_verification=v, progress=progress)
    return {"command": "prepare-tinystories-500k", "sample": meta,
            "sample_metadata": str(mpath.resolve()), "sample_output": str(sample.resolve()),
            "source": {"path": str(v.path), "sha256": v.sha256, "size_bytes": v.size_bytes}}
