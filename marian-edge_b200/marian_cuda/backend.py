"""Host-side mirror of marian-edge's backend seams over libmarian_cuda.so.

* :class:`CudaEngine` is the ``CpuTokenEngine`` seam
  (``crates/marian-cpu/src/backend.rs:48-57``): ``translate_token_ids(tokens,
  offsets, max_output_tokens)`` returns ``(tokens, offsets)`` exactly like
  ``BatchOutput`` (``engine.rs:82``), plus the streaming calls of the device
  continuous batcher (``submit`` / ``step`` / ``poll``).
* :class:`CudaBackend` is the ``TranslationBackend`` contract
  (``crates/marian-core/src/backend.rs:7-38``): ``info()``, ``is_ready()``,
  ``translate_batch`` / ``translate_batch_with_repetitions`` over text
  through the caller's source and target tokenizers (``translate`` is the
  same call; ``translate_token_batch`` serves token-id callers).  The text
  calls split long inputs (``segment_text``) and share each input's output
  budget across its segments exactly as the reference's CPU backend does
  (``crates/marian-cpu/src/backend.rs:107-346``, :func:`translate_texts`).

Errors map to the reference's ``BackendError`` kinds
(``marian-core/src/types.rs:61-70``) through :class:`MarianCudaError.status`.
There is no CPU path: every call runs the CUDA library or raises.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from . import segmenter as _seg


def _ptr(a):
    return None if a is None else a.ctypes.data


@dataclass
class BackendInfo:
    name: str
    device: str
    model: str
    precision: str
    attention: str
    supports_batching: bool = True


class CudaEngine:
    def __init__(self, model_bytes: bytes, device: int = 0, max_inflight: int = 1024,
                 max_encode_tokens: int = 65536, page_tokens: int = 16, kv_pages: int = 0,
                 max_length_factor: int = 3, lanes: int = 0, shortlist: bytes | None = None):
        self._lib = L.load()
        cfg = L.Config()
        self._lib.mc_config_default(C.byref(cfg))
        cfg.device, cfg.max_inflight, cfg.max_encode_tokens = device, max_inflight, max_encode_tokens
        cfg.page_tokens, cfg.kv_pages, cfg.max_length_factor = page_tokens, kv_pages, max_length_factor
        if lanes:
            cfg.lanes = lanes
        h = C.c_void_p()
        L.check(self._lib.mc_create(C.byref(cfg), C.byref(h)))
        self._h = h
        self.device = device
        L.check(self._lib.mc_load_marian_bin(h, model_bytes, len(model_bytes)), h)
        if shortlist is not None:
            L.check(self._lib.mc_load_shortlist(h, shortlist, len(shortlist)), h)
        info = L.ModelInfo()
        L.check(self._lib.mc_model_info_get(h, C.byref(info)), h)
        self.info = info

    # -- lifecycle ------------------------------------------------------------
    def close(self):
        if getattr(self, "_h", None):
            self._lib.mc_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self):
        return self._h

    def is_ready(self) -> bool:
        return bool(self._lib.mc_is_ready(self._h))

    def stream(self) -> int:
        return self._lib.mc_stream(self._h) or 0

    # -- CpuTokenEngine::translate_token_ids ------------------------------------
    def translate_token_ids(self, tokens, offsets, max_output_tokens, force_len=None):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint32)
        batch = len(offsets) - 1
        mo = np.ascontiguousarray(max_output_tokens, dtype=np.uint32)
        if len(mo) != batch:
            raise L.MarianCudaError(L.MC_INVALID_INPUT, "max_output_tokens does not match packed batch")
        fl = None if force_len is None else np.ascontiguousarray(force_len, dtype=np.uint32)
        cap = max(1, batch * 256)
        out = np.empty(cap, dtype=np.int32)
        out_off = np.zeros(batch + 1, dtype=np.uint32)
        L.check(self._lib.mc_translate_token_ids(self._h, _ptr(tokens), tokens.size, _ptr(offsets),
                                                 batch, _ptr(mo), _ptr(fl), _ptr(out), cap,
                                                 _ptr(out_off)), self._h)
        return out[:out_off[-1]].copy(), out_off

    # -- continuous batching ------------------------------------------------------
    def submit(self, request_id: int, tokens, max_output_tokens: int, force_len: int = 0):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        L.check(self._lib.mc_submit(self._h, request_id, _ptr(t), t.size, max_output_tokens,
                                    force_len), self._h)

    def step(self):
        a, q = C.c_uint32(), C.c_uint32()
        L.check(self._lib.mc_step(self._h, C.byref(a), C.byref(q)), self._h)
        return a.value, q.value

    def poll(self, max_results: int = 4096, token_capacity: int = 1 << 20):
        ids = np.empty(max_results, dtype=np.uint64)
        lens = np.empty(max_results, dtype=np.uint32)
        toks = np.empty(token_capacity, dtype=np.int32)
        n = C.c_uint32()
        L.check(self._lib.mc_poll(self._h, _ptr(ids), _ptr(lens), max_results, _ptr(toks),
                                  token_capacity, C.byref(n)), self._h)
        out, pos = [], 0
        for i in range(n.value):
            out.append((int(ids[i]), toks[pos:pos + lens[i]].copy()))
            pos += int(lens[i])
        return out

    # -- encoder pass only (Q8CpuEngine::encode, q8_engine.rs:511-574) ----------
    def encode_token_ids(self, tokens, offsets, want_output: bool = False):
        """One packed encoder pass over a static batch (cross keys/values
        written, slots released); returns the packed [tokens, dim] encoder
        output when want_output."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint32)
        out = np.empty((tokens.size, self.info.dim), np.float32) if want_output else None
        L.check(self._lib.mc_encode_token_ids(self._h, _ptr(tokens), tokens.size, _ptr(offsets),
                                              len(offsets) - 1, _ptr(out)), self._h)
        return out

    # -- arrival-schedule replay (measurement) -----------------------------------
    def replay(self, tokens, offsets, max_output_tokens, force_len, arrival_s):
        """Submits row b at arrival_s[b] seconds (host clock) and steps until
        every request is done; returns each request's latency in seconds."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint32)
        mo = np.ascontiguousarray(max_output_tokens, dtype=np.uint32)
        fl = None if force_len is None else np.ascontiguousarray(force_len, dtype=np.uint32)
        arr = np.ascontiguousarray(arrival_s, dtype=np.float64)
        lat = np.full(len(offsets) - 1, np.nan, np.float64)
        L.check(self._lib.mc_replay(self._h, _ptr(tokens), tokens.size, _ptr(offsets), len(offsets) - 1,
                                    _ptr(mo), _ptr(fl), _ptr(arr), _ptr(lat)), self._h)
        return lat

    # -- per-layer capture for parity tests ------------------------------------
    def trace_first_step(self, tokens, offsets):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint32)
        batch = len(offsets) - 1
        lmax = int(np.diff(offsets.astype(np.int64)).max())
        d, nl = self.info.dim, self.info.decoder_layers
        enc = np.zeros((batch * lmax, d), np.float32)
        ck = np.zeros((nl, batch * lmax, d), np.float32)
        cv = np.zeros((nl, batch * lmax, d), np.float32)
        st = np.zeros((batch, d), np.float32)
        L.check(self._lib.mc_trace_first_step(self._h, _ptr(tokens), tokens.size, _ptr(offsets), batch,
                                              _ptr(enc), _ptr(ck), _ptr(cv), _ptr(st)), self._h)
        return {"encoder_output": enc, "cross_key": ck, "cross_value": cv, "decoder_state_step0": st}


# ---- text translation (crates/marian-cpu/src/backend.rs:107-346) ------------
MAXIMUM_SOURCE_TOKENS = 256          # marian-cpu/src/limits.rs:3
MAXIMUM_TRANSLATION_SEGMENTS = 4096  # marian-cpu/src/limits.rs:7


@dataclass
class TranslationInput:
    """marian-core/src/types.rs:7-12"""
    text: str
    source_lang: str
    target_lang: str
    max_output_tokens: int = 512


@dataclass
class TranslationOutput:
    """marian-core/src/types.rs:41-47"""
    text: str
    score: float | None
    input_tokens: int
    output_tokens: int


class BackendError(Exception):
    """BackendError (marian-core/src/types.rs:61-70); kind is one of
    ``invalid_input``, ``unsupported_direction``, ``inference``."""

    def __init__(self, kind: str, message: str):
        super().__init__(message)
        self.kind = kind


def translate_texts(inputs, engine_fn, source, target, source_lang: str, target_lang: str,
                    eos_id: int = 0):
    """translate_with_engine (marian-cpu/src/backend.rs:107-346).

    Each input is split by :func:`segmenter.segment_text` under
    MAXIMUM_SOURCE_TOKENS - 1 source pieces; its non-empty segments are
    tokenized, EOS-terminated and translated in order, every segment
    limited to what the input's max_output_tokens budget has left after the
    segments before it (an input whose budget is spent gets empty text for
    its remaining segments); translations are joined with the original
    separators.  ``source``/``target`` are the tokenizers
    (``encode(str) -> list[int]``, ``decode(list[int]) -> str``,
    ``vocabulary_size() -> int``, backend.rs:26-32); ``engine_fn(tokens,
    offsets, max_output_tokens) -> (tokens, offsets)`` is the token engine.
    Each round sends the next segment of every input with work left: the
    engine batches any number of rows of any length, so the CPU engine's
    batch bounds (backend.rs:222-240) have no counterpart, and the results
    are the same because each row's greedy decode is independent of its
    batch.
    """
    if not inputs:
        return []
    for inp in inputs:
        if inp.source_lang != source_lang or inp.target_lang != target_lang:
            raise BackendError("unsupported_direction",
                               f"{inp.source_lang} -> {inp.target_lang}; loaded model is "
                               f"{source_lang} -> {target_lang}")
    vocab = source.vocabulary_size()
    planned = []   # per input: [translated or None, separator, input_tokens, output_tokens]
    work = []      # per input: [(planned index, tokens)]
    total = 0
    for inp in inputs:
        try:
            segments = _seg.segment_text(inp.text, MAXIMUM_SOURCE_TOKENS - 1,
                                         lambda t: len(source.encode(t)))
        except _seg.SegmentError as e:
            raise BackendError("invalid_input", str(e)) from None
        text = inp.text.encode("utf-8")
        plan, todo = [], []
        for sg in segments:
            content, separator = sg.content(text), sg.separator(text)
            if not content:
                plan.append(["", separator, 0, 0])
                continue
            if total >= MAXIMUM_TRANSLATION_SEGMENTS:
                raise BackendError("invalid_input", f"batch requires more than "
                                                    f"{MAXIMUM_TRANSLATION_SEGMENTS} translated segments")
            pieces = list(source.encode(content))
            if len(pieces) != sg.source_pieces:
                raise BackendError("inference", f"source tokenizer returned {len(pieces)} pieces after "
                                                f"sizing the segment as {sg.source_pieces}")
            bad = next((t for t in pieces if t < 0 or t >= vocab), None)
            if bad is not None:
                raise BackendError("invalid_input",
                                   f"tokenizer returned source token {bad} outside vocabulary {vocab}")
            pieces.append(eos_id)
            if len(pieces) > MAXIMUM_SOURCE_TOKENS:
                raise BackendError("inference", f"segmented source has {len(pieces)} tokens including EOS; "
                                                f"maximum is {MAXIMUM_SOURCE_TOKENS}")
            todo.append((len(plan), pieces))
            plan.append([None, separator, len(pieces), 0])
            total += 1
        planned.append(plan)
        work.append(todo)

    positions = [0] * len(inputs)
    remaining = [int(inp.max_output_tokens) for inp in inputs]
    while True:
        for i, todo in enumerate(work):
            if remaining[i] == 0:  # the budget is spent: the rest translate to nothing
                while positions[i] < len(todo):
                    planned[i][todo[positions[i]][0]][0] = ""
                    positions[i] += 1
        batch = [(i, todo[positions[i]]) for i, todo in enumerate(work) if positions[i] < len(todo)]
        if not batch:
            break
        offsets = np.zeros(len(batch) + 1, np.uint32)
        offsets[1:] = np.cumsum([len(t) for _, (_, t) in batch])
        tokens = np.concatenate([np.asarray(t, np.int32) for _, (_, t) in batch])
        limits = np.array([remaining[i] for i, _ in batch], np.uint32)
        out, out_off = engine_fn(tokens, offsets, limits)
        if len(out_off) != len(batch) + 1:
            raise BackendError("inference", "engine returned malformed batch offsets")
        for row, (i, (pi, _)) in enumerate(batch):
            start, end = int(out_off[row]), int(out_off[row + 1])
            if end < start or end > len(out):
                raise BackendError("inference", "engine returned out-of-range token offsets")
            if end - start > remaining[i]:
                raise BackendError("inference", "engine exceeded the original max_output_tokens budget")
            remaining[i] -= end - start
            ids = [int(t) for t in out[start:end] if t != eos_id]
            planned[i][pi][0] = target.decode(ids)
            planned[i][pi][3] = len(ids)
            positions[i] += 1

    return [TranslationOutput("".join(p[0] + p[1] for p in plan), None, sum(p[2] for p in plan),
                              sum(p[3] for p in plan)) for plan in planned]


class CudaBackend:
    """TranslationBackend: token ids directly, or text through the caller's
    tokenizers (translate)."""

    def __init__(self, model_bytes: bytes, device: int = 0, source_tokenizer=None, target_tokenizer=None,
                 source_lang: str = "", target_lang: str = "", eos_id: int = 0, **kw):
        self.engine = CudaEngine(model_bytes, device=device, **kw)
        self.source_tokenizer, self.target_tokenizer = source_tokenizer, target_tokenizer
        self.source_lang, self.target_lang, self.eos_id = source_lang, target_lang, eos_id

    def translate_batch(self, inputs):
        """TranslationBackend::translate_batch (marian-core/src/backend.rs:20-23):
        list of TranslationInput (text) -> list of TranslationOutput, through the
        caller's tokenizers, long-text splitting and the shared output budget."""
        if self.source_tokenizer is None or self.target_tokenizer is None:
            raise BackendError("invalid_input", "text translation needs source and target tokenizers")
        return translate_texts(inputs, self.engine.translate_token_ids, self.source_tokenizer,
                               self.target_tokenizer, self.source_lang, self.target_lang, self.eos_id)

    translate = translate_batch

    def translate_batch_with_repetitions(self, inputs, repetitions):
        """marian-core/src/backend.rs:25-37: one output per logical input.  The
        repetition counts (admitted requests per row) are not needed to fill
        the GPU, so the rows are translated once, as the trait's default does."""
        if len(inputs) != len(repetitions):
            raise BackendError("invalid_input", f"{len(inputs)} inputs but {len(repetitions)} repetition counts")
        return self.translate_batch(inputs)

    def info(self) -> BackendInfo:
        i = self.engine.info
        kind = "ssru" if i.decoder_kind == 0 else "self-attention"
        return BackendInfo("cuda", f"NVIDIA B200 (cuda:{self.engine.device})",
                           f"transformer-{kind} d{i.dim} e{i.encoder_layers} d{i.decoder_layers}",
                           "q8", "varlen-paged")

    def is_ready(self) -> bool:
        return self.engine.is_ready()

    def translate_token_batch(self, sources, max_output_tokens=512):
        """Token-id callers: list of token-id sequences each ending in EOS -> the
        generated ids per sequence (EOS included when generated)."""
        offsets = np.zeros(len(sources) + 1, np.uint32)
        offsets[1:] = np.cumsum([len(s) for s in sources])
        toks = np.concatenate([np.asarray(s, np.int32) for s in sources]) if sources else np.zeros(0, np.int32)
        out, off = self.engine.translate_token_ids(toks, offsets, np.full(len(sources), max_output_tokens, np.uint32))
        return [out[off[i]:off[i + 1]] for i in range(len(sources))]
