"""Long-text splitting for the text backend (marian_core::segment_text).

The splitting runs in the C++ library (``mc_segment_text``,
csrc/segmenter.cpp); this module adapts a Python piece counter -- for
example ``lambda s: len(sentencepiece.encode(s))`` -- to its callback.
Ranges are byte ranges of the UTF-8 encoding, as the reference's
``Range<usize>`` over a ``&str`` (crates/marian-core/src/segmenter.rs:26-46).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _lib as L

MAX_SEGMENTS = 4096  # segmenter.rs:16

KINDS = {1: "zero_piece_limit", 2: "input_too_large", 3: "encoding", 4: "encoding_work_limit",
         5: "too_many_segments", 6: "unsplitable_scalar", 7: "invalid_utf8", 8: "invalid_argument"}


@dataclass(frozen=True)
class TextSegment:
    content_range: tuple[int, int]
    separator_range: tuple[int, int]
    source_pieces: int

    def content(self, text: str | bytes) -> str:
        b = text.encode("utf-8") if isinstance(text, str) else text
        return b[self.content_range[0]:self.content_range[1]].decode("utf-8")

    def separator(self, text: str | bytes) -> str:
        b = text.encode("utf-8") if isinstance(text, str) else text
        return b[self.separator_range[0]:self.separator_range[1]].decode("utf-8")

    def full_range(self) -> tuple[int, int]:
        return (self.content_range[0], self.separator_range[1])


class SegmentError(ValueError):
    """A SegmentError of the reference (segmenter.rs:48-72): kind and fields."""

    def __init__(self, err: L.SegmentError):
        self.kind = KINDS.get(err.kind, str(err.kind))
        self.start, self.end = int(err.start), int(err.end)
        self.pieces, self.maximum = int(err.pieces), int(err.maximum)
        super().__init__(err.message.decode("utf-8", "replace"))


def segment_text(text: str, max_pieces: int, count_pieces) -> list[TextSegment]:
    """Splits text into lossless segments whose content fits max_pieces.

    count_pieces(str) -> int must return the exact source-piece count; an
    exception it raises becomes an ``encoding`` SegmentError carrying its
    message (the reference closure's Err).
    """
    lib = L.load()
    data = text.encode("utf-8")

    def _count(_ctx, ptr, n, out, msg, cap):
        try:
            out[0] = int(count_pieces(C.string_at(ptr, n).decode("utf-8")))
            return 0
        except Exception as e:  # reported through the message buffer
            m = str(e).encode("utf-8")[:max(0, cap - 1)]
            C.memmove(msg, m, len(m))
            msg[len(m)] = b"\0"
            return 1

    fn = L.PIECE_COUNT_FN(_count)
    segs = (L.TextSegment * MAX_SEGMENTS)()
    n = C.c_size_t(0)
    err = L.SegmentError()
    rc = lib.mc_segment_text(data, len(data), int(max_pieces), fn, None, segs, MAX_SEGMENTS, C.byref(n),
                             C.byref(err))
    if rc != L.MC_OK:
        raise SegmentError(err)
    return [TextSegment((s.content_start, s.content_end), (s.separator_start, s.separator_end),
                        int(s.source_pieces)) for s in segs[:n.value]]
