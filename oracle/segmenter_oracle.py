"""Pure-Python restatement of marian-edge's long-text splitter.

TEST INFRASTRUCTURE ONLY: the checker for the C++ splitter behind
``mc_segment_text`` (marian-edge_b200/csrc/segmenter.cpp).  Only tests/ may
import it; the product never does.

Restates ``segment_text`` of crates/marian-core/src/segmenter.rs (v0.7.0)
over the UTF-8 bytes of the input, so every range is a byte range exactly as
the reference's ``Range<usize>`` over a ``&str``.  Pinned by the reference's
own cases (crates/marian-cpu/tests/segmenter.rs), restated in
tests/test_segmenter.py.
"""
from __future__ import annotations

from dataclasses import dataclass

MAX_SEGMENTER_INPUT_BYTES = 4 * 1024 * 1024   # segmenter.rs:14
MAX_SEGMENTS = 4096                           # segmenter.rs:16
MAX_ENCODING_CALLS = 32768                    # segmenter.rs:18
MAX_ENCODING_BYTES = 64 * 1024 * 1024         # segmenter.rs:20
MAX_COUNTED_PIECES = 8 * 1024 * 1024          # segmenter.rs:22

# Unicode White_Space (Rust char::is_whitespace)
_WHITE = set(range(0x09, 0x0E)) | {0x20, 0x85, 0xA0, 0x1680, 0x2028, 0x2029, 0x202F, 0x205F, 0x3000} \
    | set(range(0x2000, 0x200B))
_TERMINATORS = {ord("."), ord("!"), ord("?"), 0x3002, 0xFF01, 0xFF1F, 0x2026}          # segmenter.rs:594
_CLOSING = {ord('"'), ord("'"), 0x2019, 0x201D, 0x00BB, ord(")"), ord("]"), ord("}"),  # segmenter.rs:550
            0x3009, 0x300B, 0x300D, 0x300F, 0x3011, 0x3015, 0x3017, 0x3019, 0x301B}
_TITLE = {"capt.", "col.", "dr.", "gen.", "gov.", "lt.", "mr.", "mrs.", "ms.", "prof.", "rep.",   # :643
          "rev.", "sen.", "sgt.", "sr.", "st."}
_NON_TERMINAL = {"e.g.", "i.e.", "fig.", "no.", "vs.", "jan.", "feb.", "mar.", "apr.", "jun.",   # :648
                 "jul.", "aug.", "sep.", "sept.", "oct.", "nov.", "dec."}
_COMMON = {"approx.", "co.", "corp.", "dept.", "ed.", "eds.", "est.", "etc.", "inc.", "ltd.",     # :653
           "misc.", "p.", "pp.", "vol."}


class SegmentError(Exception):
    """SegmentError (segmenter.rs:48-72): kind plus the variant's fields."""

    def __init__(self, kind: str, **fields):
        super().__init__(kind, fields)
        self.kind = kind
        self.fields = fields


@dataclass
class Segment:
    content: tuple[int, int]
    separator: tuple[int, int]
    source_pieces: int


def _scalar(b: bytes, i: int) -> tuple[int, int]:
    """(code point, next index) of the scalar starting at byte i."""
    lead = b[i]
    n = 1 if lead < 0x80 else 2 if lead < 0xE0 else 3 if lead < 0xF0 else 4
    return ord(b[i:i + n].decode("utf-8")), i + n


def _scalar_before(b: bytes, end: int) -> tuple[int, int]:
    """(start, code point) of the scalar ending at byte end."""
    s = end - 1
    while s > 0 and (b[s] & 0xC0) == 0x80:
        s -= 1
    return s, _scalar(b, s)[0]


def _boundary(b: bytes, i: int) -> bool:
    return i == 0 or i >= len(b) or (b[i] & 0xC0) != 0x80


def _skip(b: bytes, i: int, end: int, member) -> int:
    while i < end:
        c, n = _scalar(b, i)
        if not member(c):
            break
        i = n
    return i


def _ws(c: int) -> bool:
    return c in _WHITE


class _Counter:
    """PieceCounter (segmenter.rs:186-265): memoized and bounded."""

    def __init__(self, b: bytes, fn):
        self.b, self.fn, self.cache = b, fn, {}
        self.calls = self.nbytes = self.pieces = 0

    def __call__(self, start: int, end: int) -> int:
        if (start, end) in self.cache:
            return self.cache[(start, end)]
        self.calls += 1
        if self.calls > MAX_ENCODING_CALLS:
            raise SegmentError("encoding_work_limit", resource="tokenizer calls", maximum=MAX_ENCODING_CALLS)
        self.nbytes += end - start
        if self.nbytes > MAX_ENCODING_BYTES:
            raise SegmentError("encoding_work_limit", resource="encoded bytes", maximum=MAX_ENCODING_BYTES)
        try:
            n = self.fn(self.b[start:end].decode("utf-8"))
        except Exception as e:  # the closure's Err(message)
            raise SegmentError("encoding", start=start, end=end, message=str(e)) from None
        self.pieces += n
        if self.pieces > MAX_COUNTED_PIECES:
            raise SegmentError("encoding_work_limit", resource="counted pieces", maximum=MAX_COUNTED_PIECES)
        self.cache[(start, end)] = n
        return n


def _period_ends_sentence(b: bytes, index: int, quoted_end: int) -> bool:
    """segmenter.rs:601-641"""
    prev = _scalar_before(b, index)[1] if index > 0 else None
    nxt = _scalar(b, index + 1)[0] if index + 1 < len(b) else None
    digit = lambda c: c is not None and ord("0") <= c <= ord("9")
    if digit(prev) and digit(nxt):
        return False
    start = 0
    e = index
    while e > 0:
        s, c = _scalar_before(b, e)
        if _ws(c) or c in (ord("("), ord("["), ord("{"), ord('"'), 0x201C):
            start = e
            break
        e = s
    raw = b[start:index + 1].decode("utf-8")
    # to_ascii_lowercase + retain(ASCII alphanumeric or '.'): filter first, so
    # that no non-ASCII letter lowercases into ASCII (as str.lower() can).
    token = "".join(ch.lower() for ch in raw if ch.isascii() and (ch.isalnum() or ch == "."))
    f = _skip(b, quoted_end, len(b), _ws)
    following = _scalar(b, f)[0] if f < len(b) else None
    if token in _TITLE and following is not None:
        return False
    if token in _NON_TERMINAL and following is not None:
        return False
    if token in _COMMON and following is not None and (
            ord("a") <= following <= ord("z") or ord("0") <= following <= ord("9")):
        return False
    parts = token.rstrip(".").split(".")
    acronym = len(parts) <= 8 and all(len(p) == 1 and p.isascii() and p.isalpha() for p in parts)
    if acronym and following is not None and ord("A") <= following <= ord("Z"):
        return False
    return True


def _units(b: bytes, content_end: int):
    """sentence_units, segmenter.rs:267-320: [(content, separator)]."""
    units, cursor, i = [], 0, 0
    while i < content_end:
        c, n = _scalar(b, i)
        if c in _TERMINATORS:
            pe = _skip(b, i, content_end, lambda x: x in _TERMINATORS)
            qe = _skip(b, pe, content_end, lambda x: x in _CLOSING)
            follows = qe == content_end or (qe < content_end and _ws(_scalar(b, qe)[0]))
            if follows and (c != ord(".") or _period_ends_sentence(b, i, qe)):
                se = _skip(b, qe, content_end, _ws)
                units.append([(cursor, qe), (qe, se)])
                cursor = i = se
                continue
            i = max(pe, n)
            continue
        if _ws(c):
            we = _skip(b, i, content_end, _ws)
            if b"\n" in b[i:we] or b"\r" in b[i:we]:
                units.append([(cursor, i), (i, we)])
                cursor = we
            i = we
            continue
        i = n
    if cursor < content_end:
        units.append([(cursor, content_end), (content_end, len(b))])
    elif units:
        units[-1][1] = (units[-1][1][0], len(b))
    return units


def _break_points(b: bytes, start: int, end: int):
    """fallback_break_points, segmenter.rs:475-516: [(content_end, next_start, priority)]."""
    pts, i = [], start
    while i < end:
        c, n = _scalar(b, i)
        if _ws(c):
            we = _skip(b, i, end, _ws)
            pts.append((i, we, 2))
            i = we
            continue
        prio = None
        if c in (ord(";"), 0xFF1B, ord(":"), 0xFF1A, ord("/"), 0x2013, 0x2014):
            prio = 0
        elif c in (ord(","), 0xFF0C):
            prio = 1
        elif c == ord("-"):
            repeated = i + 1 < end and b[i + 1] == ord("-")
            before = i == start or _ws(_scalar_before(b, i)[1])
            after = i + 1 >= end or _ws(_scalar(b, i + 1)[0])
            if repeated or before or after:
                prio = 0
        if prio is not None:
            pe = n
            if c == ord("-"):
                while pe < end and b[pe] == ord("-"):
                    pe += 1
            pts.append((pe, _skip(b, pe, end, _ws), prio))
            i = pe
            continue
        i = n
    return pts


def segment_text(text: str, max_pieces: int, count_pieces) -> list[Segment]:
    """segmenter.rs:122-175 (count_pieces(str) -> int, raising on failure)."""
    b = text.encode("utf-8")
    if max_pieces == 0:
        raise SegmentError("zero_piece_limit")
    if len(b) > MAX_SEGMENTER_INPUT_BYTES:
        raise SegmentError("input_too_large", bytes=len(b), maximum=MAX_SEGMENTER_INPUT_BYTES)
    count = _Counter(b, count_pieces)
    out: list[Segment] = []

    def push(seg: Segment):
        if len(out) >= MAX_SEGMENTS:
            raise SegmentError("too_many_segments", maximum=MAX_SEGMENTS)
        out.append(seg)

    content_end = len(b)
    while content_end > 0:
        s, c = _scalar_before(b, content_end)
        if not _ws(c):
            break
        content_end = s
    whole = count(0, content_end)
    units = _units(b, content_end)
    if whole <= max_pieces and len(units) <= 1:
        return [Segment((0, content_end), (content_end, len(b)), whole)]
    for (cs, ce), sep in units:
        n = count(cs, ce)
        if n <= max_pieces:
            push(Segment((cs, ce), sep, n))
            continue
        # split_oversize_unit, segmenter.rs:322-390
        pts = _break_points(b, cs, ce)
        start, done = cs, False
        while start < ce:
            rem = count(start, ce)
            if rem <= max_pieces:
                push(Segment((start, ce), sep, rem))
                done = True
                break
            chosen = None
            for prio in range(3):  # rightmost_fitting_break, segmenter.rs:392-432
                cands = [p for p in pts if p[2] == prio and p[0] > start and p[1] > start and p[1] < ce]
                lo, hi = 0, len(cands)
                while lo < hi:
                    mid = lo + (hi - lo) // 2
                    k = count(start, cands[mid][0])
                    if k <= max_pieces:
                        chosen, lo = (cands[mid], k), mid + 1
                    else:
                        hi = mid
                if chosen is not None:
                    break
            if chosen is not None:
                (c_end, nxt, _), k = chosen
            else:  # largest_fitting_scalar_prefix, segmenter.rs:434-473
                first_end = _scalar(b, start)[1]
                k = count(start, first_end)
                if k > max_pieces:
                    raise SegmentError("unsplitable_scalar", start=start, end=first_end, pieces=k,
                                       maximum=max_pieces)
                lo, hi, best = first_end, ce, (first_end, k)
                while lo < hi:
                    mid = lo + (hi - lo + 1) // 2
                    while mid > start and not _boundary(b, mid):
                        mid -= 1
                    if mid <= best[0]:
                        break
                    kk = count(start, mid)
                    if kk <= max_pieces:
                        best, lo = (mid, kk), mid
                    else:
                        if mid <= start:
                            hi = start
                        else:
                            hi = mid - 1
                            while hi > start and not _boundary(b, hi):
                                hi -= 1
                c_end = nxt = best[0]
                k = best[1]
            push(Segment((start, c_end), (c_end, nxt), k))
            start = nxt
        if not done and sep[0] < sep[1] and out:
            out[-1].separator = (out[-1].separator[0], sep[1])
    return out
