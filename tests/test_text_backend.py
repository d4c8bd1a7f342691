"""Text translation: long-text splitting and the shared output budget.

translate_texts restates translate_with_engine
(crates/marian-cpu/src/backend.rs:107-346).  The CPU tests pin its planning
and budget rules with a word-level tokenizer and a deterministic fake engine;
the GPU test runs CudaBackend.translate on the CUDA engine against the same
loop driven by the CPU oracle engine.
"""
import zlib

import numpy as np
import pytest

from marian_cuda import backend as B
from marian_cuda import workloads as W
import oracle as O


class WordTokenizer:
    """One piece per whitespace-separated word; ids 2..vocab-1 (0 = EOS, 1 = UNK)."""

    def __init__(self, vocab=512):
        self.vocab = vocab

    def vocabulary_size(self):
        return self.vocab

    def encode(self, text):
        return [2 + zlib.crc32(w.encode()) % (self.vocab - 2) for w in text.split()]

    def decode(self, ids):
        return " ".join(f"w{i}" for i in ids)


class FakeEngine:
    """Row output: the source ids reversed (EOS dropped), cut at the row's
    limit, then EOS if the limit leaves room.  Records every call's limits."""

    def __init__(self):
        self.calls = []

    def __call__(self, tokens, offsets, limits):
        self.calls.append(list(map(int, limits)))
        out, off = [], [0]
        for r in range(len(limits)):
            src = [int(t) for t in tokens[offsets[r]:offsets[r + 1]] if t != 0][::-1]
            row = src[:int(limits[r])]
            if len(row) < int(limits[r]):
                row.append(0)
            out += row
            off.append(len(out))
        return np.array(out, np.int32), np.array(off, np.uint32)


def _translate(inputs, engine=None):
    tok = WordTokenizer()
    return B.translate_texts(inputs, engine or FakeEngine(), tok, tok, "en", "zh")


def _inp(text, budget=512):
    return B.TranslationInput(text, "en", "zh", budget)


def test_budget_is_shared_across_an_inputs_segments():
    tok = WordTokenizer()
    text = "one two three four.\nfive six seven eight.\nnine ten eleven twelve."
    eng = FakeEngine()
    out, = B.translate_texts([_inp(text, 9)], eng, tok, tok, "en", "zh")
    # segment 1: limit 9 -> 4 words + EOS (5 used); segment 2: limit 4 -> 4
    # words, no room for EOS; segment 3: budget spent -> empty, never sent
    assert eng.calls == [[9], [4]]
    s1 = tok.decode(tok.encode("one two three four.")[::-1])
    s2 = tok.decode(tok.encode("five six seven eight.")[::-1])
    assert out.text == s1 + "\n" + s2 + "\n" + ""
    assert out.input_tokens == 15 and out.output_tokens == 8 and out.score is None


def test_rounds_send_the_next_segment_of_every_input():
    eng = FakeEngine()
    outs = _translate([_inp("a b. c d e.", 100), _inp("f.", 7), _inp("", 5), _inp("g h i j k l m n o p", 3)], eng)
    assert eng.calls == [[100, 7, 3], [97]]
    assert outs[2].text == "" and outs[2].input_tokens == 0
    assert outs[3].output_tokens == 3  # cut at its budget
    tok = WordTokenizer()
    assert outs[0].text == tok.decode(tok.encode("a b.")[::-1]) + " " + tok.decode(tok.encode("c d e.")[::-1])


def test_separators_survive_verbatim_and_long_inputs_split_under_the_source_limit():
    text = "  " + " ".join(f"t{i}" for i in range(600)) + " \r\n\r\n"
    eng = FakeEngine()
    out, = _translate([_inp(text, 10_000)], eng)
    assert len(eng.calls) == 3  # 255 + 255 + 90 words, one segment per round
    assert out.input_tokens == 600 + 3  # pieces + one EOS per segment
    assert not out.text.startswith(" ")  # leading blanks are content (tokenized away), not a separator
    assert out.text.endswith(" \r\n\r\n")


def test_errors_follow_the_reference_kinds():
    with pytest.raises(B.BackendError) as e:
        _translate([B.TranslationInput("x", "de", "zh", 5)])
    assert e.value.kind == "unsupported_direction"

    class BadVocab(WordTokenizer):
        def encode(self, text):
            return [self.vocab + 5 for _ in text.split()]

    with pytest.raises(B.BackendError) as e:
        B.translate_texts([_inp("x y")], FakeEngine(), BadVocab(), WordTokenizer(), "en", "zh")
    assert e.value.kind == "invalid_input" and "outside vocabulary" in str(e.value)

    class Broken(WordTokenizer):
        def encode(self, text):
            raise RuntimeError("no model")

    with pytest.raises(B.BackendError) as e:
        B.translate_texts([_inp("x")], FakeEngine(), Broken(), WordTokenizer(), "en", "zh")
    assert e.value.kind == "invalid_input" and "source tokenizer failed" in str(e.value)

    def greedy_engine(tokens, offsets, limits):
        out, off = FakeEngine()(tokens, offsets, limits)
        return np.concatenate([out, [5, 5]]).astype(np.int32), np.concatenate([off[:-1], [off[-1] + 2]])

    with pytest.raises(B.BackendError) as e:
        _translate([_inp("a b c", 2)], greedy_engine)
    assert e.value.kind == "inference"
    assert _translate([]) == []


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny_self", "tiny_ssru"])
def test_text_translation_on_the_gpu_matches_the_oracle_engine(name):
    mb = W.synthetic_model(W.SHAPES[name], seed=3)
    tok = WordTokenizer(vocab=W.SHAPES[name].vocab)
    rng = np.random.default_rng(7)
    words = [f"w{i}" for i in range(300)]
    texts = []
    for n in (3, 12, 40, 300, 700):
        sent = lambda k: " ".join(rng.choice(words, k)) + rng.choice([".", "!", "?"])
        texts.append("\n".join(sent(int(rng.integers(1, 30))) for _ in range(max(1, n // 20))) + " " +
                     " ".join(rng.choice(words, n)))
    inputs = [_inp(t, b) for t, b in zip(texts, (512, 40, 7, 1000, 90))]
    om = O.OracleModel(mb)
    want = B.translate_texts(inputs, lambda t, o, m: om.translate(t, o, m, None), tok, tok, "en", "zh")
    backend = B.CudaBackend(mb, source_tokenizer=tok, target_tokenizer=tok, source_lang="en", target_lang="zh",
                            max_inflight=32)
    try:
        got = backend.translate(inputs)
    finally:
        backend.engine.close()
    assert got == want


def test_text_path_with_the_oracle_engine_respects_budgets_and_separators():
    # The planning and budget loop over real greedy outputs (the CPU oracle
    # engine on a tiny model): each input's generated tokens fit its budget,
    # every separator survives, and an input whose budget runs out before its
    # last segment gets empty text there.
    mb = W.synthetic_model(W.SHAPES["tiny_self"], seed=5)
    om = O.OracleModel(mb)
    tok = WordTokenizer(vocab=W.SHAPES["tiny_self"].vocab)
    engine = lambda t, o, m: om.translate(t, o, m, None)
    texts = ["a b c.\nd e f g.\r\n", "one two three four five six seven. eight nine.  ", "x"]
    budgets = [40, 3, 5]
    outs = B.translate_texts([_inp(t, b) for t, b in zip(texts, budgets)], engine, tok, tok, "en", "zh")
    for text, budget, out in zip(texts, budgets, outs):
        assert out.output_tokens <= budget
        assert out.input_tokens == len(text.split()) + len(
            [s for s in _segments(text) if s.strip()])  # pieces + one EOS per non-empty segment
    assert outs[0].text.endswith("\r\n") and "\n" in outs[0].text
    assert outs[1].text.endswith("  ")
    again = B.translate_texts([_inp(t, b) for t, b in zip(texts, budgets)], engine, tok, tok, "en", "zh")
    assert again == outs  # greedy decoding is deterministic


def _segments(text):
    from marian_cuda import segmenter as S
    return [sg.content(text) for sg in S.segment_text(text, 255, lambda t: len(t.split()))]


def test_backend_entry_points_follow_the_trait():
    # TranslationBackend's batch calls (marian-core/src/backend.rs:7-38) on a
    # CudaBackend whose engine is the CPU oracle, so the test needs no GPU.
    class OracleEngine:
        def __init__(self, mb):
            self.om = O.OracleModel(mb)

        def translate_token_ids(self, t, o, m, force_len=None):
            return self.om.translate(t, o, m, None)

    mb = W.synthetic_model(W.SHAPES["tiny_self"], seed=5)
    tok = WordTokenizer(vocab=W.SHAPES["tiny_self"].vocab)
    be = object.__new__(B.CudaBackend)
    be.engine = OracleEngine(mb)
    be.source_tokenizer = be.target_tokenizer = tok
    be.source_lang, be.target_lang, be.eos_id = "en", "zh", 0
    inputs = [_inp("a b c. d e.", 30), _inp("f g", 4)]
    outs = be.translate_batch(inputs)
    assert be.translate(inputs) == outs
    assert be.translate_batch_with_repetitions(inputs, [3, 1]) == outs  # one output per logical input
    with pytest.raises(B.BackendError) as e:
        be.translate_batch_with_repetitions(inputs, [1])
    assert e.value.kind == "invalid_input"
    ids = be.translate_token_batch([tok.encode("f g") + [0]], max_output_tokens=4)
    assert tok.decode([int(t) for t in ids[0] if t != 0]) == outs[1].text
    be.source_tokenizer = None
    with pytest.raises(B.BackendError):
        be.translate_batch(inputs)
