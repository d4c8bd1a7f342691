"""Long-text splitter: the C++ library (mc_segment_text) against the reference.

The cases restate crates/marian-cpu/tests/segmenter.rs (marian-edge v0.7.0)
with its two piece counters; each runs against the library and against the
pure-Python restatement in oracle/segmenter_oracle.py, which a seeded differential
test then compares with the library on random mixed-script texts.
"""
import random

import pytest

from marian_cuda import segmenter as S
import segmenter_oracle as O


def word_pieces(text):  # tests/segmenter.rs:5-7
    return len(text.split())


def scalar_pieces(text):  # tests/segmenter.rs:9-14 (Rust whitespace set)
    return sum(1 for ch in text if ord(ch) not in O._WHITE)


def _lib(text, limit, fn):
    return [(s.content_range, s.separator_range, s.source_pieces) for s in S.segment_text(text, limit, fn)]


def _oracle(text, limit, fn):
    return [(s.content, s.separator, s.source_pieces) for s in O.segment_text(text, limit, fn)]


IMPLS = {"library": _lib, "oracle": _oracle}


def _kind(exc):
    return exc.kind


def _content(text, seg):
    return text.encode()[seg[0][0]:seg[0][1]].decode()


def _sep(text, seg):
    return text.encode()[seg[1][0]:seg[1][1]].decode()


def reconstructed(text, segs):
    return "".join(_content(text, s) + _sep(text, s) for s in segs)


@pytest.fixture(params=list(IMPLS))
def seg(request):
    return IMPLS[request.param]


def test_short_text_stays_in_one_lossless_segment(seg):
    text = "Hello world.  \r\n"
    s = seg(text, 255, word_pieces)
    assert len(s) == 1
    assert _content(text, s[0]) == "Hello world."
    assert _sep(text, s[0]) == "  \r\n"
    assert (s[0][0][0], s[0][1][1]) == (0, len(text.encode()))
    assert reconstructed(text, s) == text


def test_abbreviation_decimal_version_domain_and_email_do_not_make_false_boundaries(seg):
    prefix = "Dr. Smith used e.g. version 1.2.3 at example.com and a.b@example.org. "
    text = prefix + "word " * 260 + " End."
    s = seg(text, 255, word_pieces)
    assert _content(text, s[0]) == prefix.rstrip()
    assert not any(_content(text, x) in ("Dr.", "e.g.", "version 1.2.", "example.", "a.b@example.") for x in s)
    assert reconstructed(text, s) == text
    assert all(x[2] <= 255 for x in s)


def test_sentence_quotes_cjk_terminators_crlf_and_blank_lines_are_preserved(seg):
    text = "word " * 256 + " \r\n\r\nHe asked, \"Ready?!\"  中文句子。\n下一句！  Final…”"
    s = seg(text, 255, word_pieces)
    assert reconstructed(text, s) == text
    assert all(x[2] <= 255 for x in s)
    assert any(_sep(text, x) == "  \r\n\r\n" for x in s)
    assert any(_content(text, x).endswith("Ready?!\"") for x in s)
    assert any(_content(text, x).endswith("中文句子。") for x in s)


def test_short_multiline_text_keeps_each_separator_outside_the_model(seg):
    text = "Line one.\nLine two?\r\nLine three!"
    s = seg(text, 255, word_pieces)
    assert len(s) == 3
    assert [_sep(text, x) for x in s] == ["\n", "\r\n", ""]
    assert reconstructed(text, s) == text


def test_seven_hundred_tokens_split_at_preferred_boundaries(seg):
    text = " ".join(f"token{i}" for i in range(700))
    s = seg(text, 255, word_pieces)
    assert [x[2] for x in s] == [255, 255, 190]
    assert reconstructed(text, s) == text


@pytest.mark.parametrize("delimiter", [";", ":", "/", " —", " --", ","])
def test_falls_back_through_punctuation(seg, delimiter):
    text = f"{'a' * 140}{delimiter} {'b' * 140}{delimiter} {'c' * 40}"
    s = seg(text, 150, scalar_pieces)
    assert reconstructed(text, s) == text
    assert _content(text, s[0]).endswith(delimiter.lstrip())


def test_falls_back_to_utf8_scalars(seg):
    text = "界" * 260 + "🙂" * 260 + "文" * 180
    s = seg(text, 255, scalar_pieces)
    assert len(s) == 3
    assert reconstructed(text, s) == text
    b = text.encode()
    boundary = lambda i: i == len(b) or (b[i] & 0xC0) != 0x80
    assert all(x[2] <= 255 and boundary(x[0][0]) and boundary(x[0][1]) for x in s)


def test_leading_period_and_leading_newline_remain_lossless(seg):
    text = "\r\n. Hidden start. " + "x" * 300
    s = seg(text, 100, scalar_pieces)
    assert reconstructed(text, s) == text
    assert all(x[2] <= 100 for x in s)


@pytest.mark.parametrize("pieces,expected", [(254, 1), (255, 1), (256, 2)])
def test_exact_piece_limit_boundaries_are_not_off_by_one(seg, pieces, expected):
    text = " ".join(["x"] * pieces)
    s = seg(text, 255, word_pieces)
    assert len(s) == expected
    assert all(x[2] <= 255 for x in s)
    assert reconstructed(text, s) == text


def test_whitespace_only_input_is_one_separator_only_segment(seg):
    text = " \t\r\n\n "
    s = seg(text, 255, word_pieces)
    assert len(s) == 1
    assert _content(text, s[0]) == ""
    assert _sep(text, s[0]) == text
    assert s[0][2] == 0


def test_rejects_zero_limit_encoder_failure_and_unsplitable_scalar(seg):
    with pytest.raises((S.SegmentError, O.SegmentError)) as e:
        seg("text", 0, word_pieces)
    assert _kind(e.value) == "zero_piece_limit"

    def broken(_):
        raise RuntimeError("broken model")

    with pytest.raises((S.SegmentError, O.SegmentError)) as e:
        seg("bad", 3, broken)
    assert _kind(e.value) == "encoding"
    fields = e.value.fields if isinstance(e.value, O.SegmentError) else vars(e.value)
    assert (fields["start"], fields["end"]) == (0, 3)

    with pytest.raises((S.SegmentError, O.SegmentError)) as e:
        seg("🙂🙂", 1, lambda t: len(t) * 2)
    assert _kind(e.value) == "unsplitable_scalar"
    fields = e.value.fields if isinstance(e.value, O.SegmentError) else vars(e.value)
    assert (fields["start"], fields["end"], fields["pieces"], fields["maximum"]) == (0, 4, 2, 1)


def test_library_error_messages_follow_the_reference_display():
    with pytest.raises(S.SegmentError, match="^source piece limit must be non-zero$"):
        S.segment_text("text", 0, word_pieces)
    with pytest.raises(S.SegmentError, match=r"^source tokenizer failed for byte range 0\.\.3: broken model$"):
        S.segment_text("bad", 3, lambda t: (_ for _ in ()).throw(RuntimeError("broken model")))
    with pytest.raises(S.SegmentError,
                       match=r"^UTF-8 scalar at byte range 0\.\.4 encodes to 2 pieces; maximum is 1$"):
        S.segment_text("🙂🙂", 1, lambda t: len(t) * 2)


def test_enforces_input_and_segment_safety_limits(seg):
    with pytest.raises((S.SegmentError, O.SegmentError)) as e:
        seg("x" * (O.MAX_SEGMENTER_INPUT_BYTES + 1), 255, scalar_pieces)
    assert _kind(e.value) == "input_too_large"
    with pytest.raises((S.SegmentError, O.SegmentError)) as e:
        seg("x" * (O.MAX_SEGMENTS + 1), 1, scalar_pieces)
    assert _kind(e.value) in ("too_many_segments", "encoding_work_limit")


def test_invalid_utf8_is_an_input_error():
    # Only a C caller can pass bytes that are not UTF-8.
    import ctypes as C
    from marian_cuda import _lib as L
    lib = L.load()
    data = b"abc\xff\xfe"
    segs = (L.TextSegment * 4)()
    n = C.c_size_t()
    err = L.SegmentError()
    fn = L.PIECE_COUNT_FN(lambda *a: 0)
    assert lib.mc_segment_text(data, len(data), 10, fn, None, segs, 4, C.byref(n), C.byref(err)) == L.MC_INVALID_INPUT
    assert err.kind == 7


_ALPHABET = ["word", "Dr.", "e.g.", "U.S.", "etc.", "no.", "J.", "1.5", "v2.0.1", "a.b@c.org", "x", "Smith",
             ".", "!", "?", "?!", "...", "…", "。", "！", "？", ";", ":", "/", ",", "，", "；", "-", "--",
             "—", "–", "\"", "'", ")", "”", "’", "」", "』", "(", "“", "中文", "界", "🙂", "é", "Zoë",
             " ", " ", " ", "  ", "\n", "\r\n", "\t", " ", " ", "　", "\n\n"]


def _random_text(rng, n):
    return "".join(rng.choice(_ALPHABET) + (" " if rng.random() < 0.5 else "") for _ in range(n))


def test_library_matches_the_oracle_on_random_texts():
    rng = random.Random(1234)
    counters = [word_pieces, scalar_pieces, lambda t: (len(t.encode()) + 2) // 3]
    checked = 0
    for case in range(400):
        text = _random_text(rng, rng.randint(0, 120))
        limit = rng.choice([1, 2, 3, 5, 8, 13, 40, 255])
        fn = counters[case % len(counters)]
        try:
            want = _oracle(text, limit, fn)
        except O.SegmentError as e:
            with pytest.raises(S.SegmentError) as got:
                _lib(text, limit, fn)
            assert got.value.kind == e.kind, (text, limit)
            continue
        got = _lib(text, limit, fn)
        assert got == want, (text, limit)
        assert reconstructed(text, got) == text
        assert all(p <= limit for _, _, p in got)
        checked += 1
    assert checked > 200


def test_longtext_workload_segments_fit_and_partition_over_replicas():
    # The long-text benchmark stream: documents split by the library into
    # segments of at most 128 tokens (EOS included), dealt over replicas.
    import numpy as np
    from marian_cuda import workloads as W
    full = W.longtext_batch(40, seed=3)
    lens = np.diff(full.offsets.astype(np.int64))
    assert lens.max() <= 128 and lens.min() >= 2
    assert all(full.tokens[o - 1] == W.EOS for o in full.offsets[1:])
    parts = [W.longtext_batch(40, seed=3, rank=r, world=3) for r in range(3)]
    assert sum(p.size for p in parts) == full.size
    assert sorted(np.concatenate([np.diff(p.offsets.astype(np.int64)) for p in parts])) == sorted(lens)
    assert np.array_equal(full.force_len, W.force_lengths(lens - 1))
