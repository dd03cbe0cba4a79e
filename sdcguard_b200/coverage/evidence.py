"""Bounded, strict evidence IO for recorded runs: canonical JSON bytes, SHA-256 digests, strict JSON parsing
(no duplicate keys, no NaN/Inf, bounded depth and node count, no lone surrogates), safe relative member names,
no-follow regular-file reads, bounded zip archives, and a lexical node allowance across many members.

Hashes establish local consistency of a recording, not its authenticity.

The bounds and the canonical encoding are an interface shared with the reference's recordings and verdict files
(src/sdcguard/evidence_io.py:15-49, evidence_json_budget.py:14-118, required_gate.py:26-57): recordings valid
there are valid here, so the limits are the same numbers.
"""
from __future__ import annotations

import hashlib
import io as _io
import json
import math
import os
import re
import stat
import zipfile
import zlib
from pathlib import Path

MAX_FILE_BYTES = 64 * 1024 * 1024
MAX_JSON_NODES = 1_000_000
MAX_TOTAL_JSON_NODES = 2_000_000
MAX_DEPTH = 64
ARCHIVE_MAX_MEMBERS = 1024
ARCHIVE_MAX_MEMBER_BYTES = 32 * 1024 * 1024
ARCHIVE_MAX_TOTAL_BYTES = 128 * 1024 * 1024


class EvidenceError(ValueError):
    """Evidence that cannot be read within the supported contract."""


# ------------------------------------------------------------------------------------------ JSON
def _check_tree(value, max_nodes: int) -> None:
    """Iterative walk: bounded depth and node count, JSON-only types, finite numbers, no lone surrogates."""
    count = 0
    stack = [(value, 0)]
    pop, push = stack.pop, stack.append
    while stack:
        v, depth = pop()
        count += 1
        if depth > MAX_DEPTH or count > max_nodes:
            raise ValueError("JSON structure exceeds supported bounds")
        t = type(v)
        if t is str:
            if not v.isascii():
                try:
                    v.encode("utf-8")
                except UnicodeEncodeError:
                    raise ValueError("JSON contains an unpaired Unicode surrogate") from None
        elif t is dict:
            d1 = depth + 1
            for k, item in v.items():
                if type(k) is not str:
                    raise ValueError("JSON object keys must be strings")
                push((item, d1))
                push((k, d1))
        elif t is list:
            d1 = depth + 1
            for item in v:
                push((item, d1))
        elif t is float:
            if not math.isfinite(v):
                raise ValueError("JSON contains a non-finite number")
        elif v is not None and t is not bool and t is not int:
            raise ValueError("value is not supported JSON")


def json_bytes(value) -> bytes:
    """Canonical encoding: sorted keys, two-space indent, no NaN, trailing newline, UTF-8."""
    _check_tree(value, MAX_JSON_NODES)
    return (json.dumps(value, sort_keys=True, indent=2, allow_nan=False) + "\n").encode("utf-8")


def same(a, b) -> bool:
    """Typed JSON equality (true, 1 and 1.0 differ). Values here come from strictly parsed evidence or from this
    package, so the canonical encoding is compared without a second bounds walk."""
    try:
        return (json.dumps(a, sort_keys=True, allow_nan=False, check_circular=False)
                == json.dumps(b, sort_keys=True, allow_nan=False, check_circular=False))
    except TypeError:
        return json_bytes(a) == json_bytes(b)   # raises the canonical error for an unsupported value


def digest(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def _object_without_duplicates(pairs):
    """JSON object hook: the keys of one object must be distinct (the first repeated key is named)."""
    obj = dict(pairs)
    if len(obj) != len(pairs):
        seen = set()
        dup = next(k for k, _ in pairs if k in seen or seen.add(k))
        raise ValueError(f"duplicate JSON key: {dup}")
    return obj


def _refuse_constant(name):
    raise ValueError(f"non-finite JSON value: {name}")


_STRICT = json.JSONDecoder(object_pairs_hook=_object_without_duplicates, parse_constant=_refuse_constant)


def parse_json(raw: bytes, *, max_nodes: int = MAX_JSON_NODES):
    """Strict JSON of at most MAX_FILE_BYTES: UTF-8, no duplicate keys, no NaN/Infinity, bounded depth and node
    count (the whole document must be one value)."""
    if not isinstance(raw, bytes) or len(raw) > MAX_FILE_BYTES:
        raise EvidenceError("JSON input exceeds the bounded regular-file contract")
    try:
        value = _STRICT.decode(raw.decode("utf-8"))
        _check_tree(value, max_nodes)
    except (ValueError, UnicodeError, TypeError, RecursionError) as e:
        raise EvidenceError("malformed strict JSON: " + str(e)) from e
    return value


# ------------------------------------------------------------------------------------------ files
_UNSAFE_PART = re.compile(r"^(|\.|\.\.)$|:")


def relative(name) -> list[str]:
    """The parts of a safe relative member name: a non-empty string of '/'-separated parts, none empty, '.',
    '..' or holding ':' (a drive letter), and no backslash, NUL or leading '/'."""
    ok = isinstance(name, str) and name and not name.startswith("/") and "\\" not in name and "\x00" not in name
    parts = name.split("/") if ok else []
    if not ok or any(_UNSAFE_PART.search(part) for part in parts):
        raise EvidenceError("unsafe relative evidence path")
    return parts


def _open_dir(path: Path) -> int:
    if not hasattr(os, "O_NOFOLLOW"):
        raise ValueError("no-follow reads are unavailable on this platform")
    p = Path(path).absolute()
    fd = os.open(p.anchor, os.O_RDONLY | os.O_DIRECTORY)
    try:
        for part in p.parts[1:]:
            if part in ("", ".", ".."):
                raise ValueError("directory traversal is not supported")
            nxt = os.open(part, os.O_RDONLY | os.O_DIRECTORY | os.O_NOFOLLOW, dir_fd=fd)
            os.close(fd)
            fd = nxt
        return fd
    except BaseException:
        os.close(fd)
        raise


def read_file(root, name: str, limit: int = MAX_FILE_BYTES) -> bytes:
    """Read a regular file below root without following links, at most `limit` bytes, and check that it did
    not change while it was read."""
    parts = relative(name)
    try:
        d = _open_dir(Path(root))
        fd = None
        try:
            for part in parts[:-1]:
                nxt = os.open(part, os.O_RDONLY | os.O_DIRECTORY | os.O_NOFOLLOW, dir_fd=d)
                os.close(d)
                d = nxt
            fd = os.open(parts[-1], os.O_RDONLY | os.O_NOFOLLOW | os.O_NONBLOCK, dir_fd=d)
            before = os.fstat(fd)
            if not stat.S_ISREG(before.st_mode):
                raise ValueError("input must be a regular file")
            if before.st_size > limit:
                raise ValueError(f"input exceeds {limit}-byte limit")
            chunks, total = [], 0
            while True:
                block = os.read(fd, min(1 << 16, limit + 1 - total))
                if not block:
                    break
                chunks.append(block)
                total += len(block)
                if total > limit:
                    raise ValueError(f"input exceeds {limit}-byte limit")
            after = os.fstat(fd)
            named = os.stat(parts[-1], dir_fd=d, follow_symlinks=False)
            sig = lambda s: (s.st_dev, s.st_ino, s.st_size, s.st_mtime_ns, s.st_ctime_ns)  # noqa: E731
            if not stat.S_ISREG(named.st_mode) or sig(before) != sig(after) or sig(after) != sig(named) \
                    or total != after.st_size:
                raise ValueError("input changed while it was read")
            return b"".join(chunks)
        finally:
            if fd is not None:
                os.close(fd)
            os.close(d)
    except (OSError, ValueError) as e:
        raise EvidenceError("cannot read captured file " + str(name) + ": " + str(e)) from e


def read_archive(raw: bytes) -> dict[str, bytes]:
    """All members of a recorded zip archive, within member-count, member-size and expanded-size bounds; no
    directories, links, encryption or unusual compression; no member whose parent path is also a file."""
    if type(raw) is not bytes or len(raw) > MAX_FILE_BYTES:
        raise EvidenceError("owner archive exceeds the input bound")
    files: dict[str, bytes] = {}
    total = 0
    try:
        with zipfile.ZipFile(_io.BytesIO(raw)) as z:
            items = z.infolist()
            if len(items) > ARCHIVE_MAX_MEMBERS:
                raise EvidenceError("owner archive exceeds 1024 files")
            for it in items:
                relative(it.filename)
                if (it.filename in files or it.is_dir() or it.flag_bits & 1
                        or stat.S_IFMT(it.external_attr >> 16) not in (0, stat.S_IFREG)
                        or it.compress_type not in (zipfile.ZIP_DEFLATED, zipfile.ZIP_STORED)
                        or it.file_size > ARCHIVE_MAX_MEMBER_BYTES):
                    raise EvidenceError("unsafe or unsupported owner archive member")
                total += it.file_size
                if total > ARCHIVE_MAX_TOTAL_BYTES:
                    raise EvidenceError("owner archive exceeds 128 MiB expanded bytes")
                files[it.filename] = z.read(it)
                if len(files[it.filename]) != it.file_size:
                    raise EvidenceError("owner member size differs")
    except (zipfile.BadZipFile, OSError, EOFError, RuntimeError, NotImplementedError, zlib.error) as e:
        raise EvidenceError("unreadable owner archive: " + str(e)) from e
    for name in files:
        parts = name.split("/")
        if any("/".join(parts[:i]) in files for i in range(1, len(parts))):
            raise EvidenceError("owner archive parent path overlaps a file")
    return files


def object_at(files: dict, name: str) -> dict:
    value = parse_json(files[name])
    if type(value) is not dict:
        raise EvidenceError("expected object: " + name)
    return value


# ------------------------------------------------------------------------------------------ node allowance
_BOMS = (b"\xef\xbb\xbf", b"\xff\xfe", b"\xfe\xff", b"\x00\x00\xfe\xff", b"\xff\xfe\x00\x00")


def _utf8_ok(raw: bytes) -> bool:
    if b"\x00" in raw:
        return False
    try:
        raw.decode("utf-8", errors="strict")
    except UnicodeDecodeError:
        return False
    return True


def _lexical_nodes(raw: bytes, jsonl: bool, allowance: int) -> int:
    """One node per string (object keys included), per container opening and per other atom; JSONL lexical
    state resets at every CR/LF. Counts without decoding a tree."""
    if not _utf8_ok(raw):
        raise EvidenceError("unsupported structured encoding; NUL-free UTF8 without a leading BOM is required")
    records = raw.splitlines() if jsonl else [raw]
    for rec in records:
        if rec.startswith(_BOMS):
            raise EvidenceError("unsupported structured encoding; NUL-free UTF8 without a leading BOM is required")
    nodes = 0
    for rec in records:
        in_str = esc = atom = False
        for b in rec:
            if in_str:
                if esc:
                    esc = False
                elif b == 0x5C:
                    esc = True
                elif b == 0x22:
                    in_str = False
                continue
            if b == 0x22:
                nodes += 1
                in_str, esc, atom = True, False, False
            elif b in (0x5B, 0x7B):
                nodes += 1
                atom = False
            elif b in (9, 10, 13, 32, 0x2C, 0x3A, 0x5D, 0x7D):
                atom = False
            elif not atom:
                nodes += 1
                atom = True
            if nodes > allowance:
                raise EvidenceError("raw structured-input node allowance exceeded")
    return nodes


def count_nodes(files: dict, *, max_nodes: int = MAX_JSON_NODES) -> int:
    """Lexical node count of every .json / .jsonl member against one shared allowance."""
    if type(max_nodes) is not int or not 0 <= max_nodes <= MAX_TOTAL_JSON_NODES:
        raise EvidenceError("raw structured-input node allowance must be a bounded nonnegative integer")
    if type(files) is not dict:
        raise EvidenceError("raw structured-input members must be an exact dictionary")
    nodes = 0
    for name, raw in files.items():
        if type(name) is not str or type(raw) is not bytes:
            raise EvidenceError("raw structured-input names and bytes have unsupported types")
        relative(name)
        if name.endswith((".json", ".jsonl")):
            nodes += _lexical_nodes(raw, name.endswith(".jsonl"), max_nodes - nodes)
    return nodes
