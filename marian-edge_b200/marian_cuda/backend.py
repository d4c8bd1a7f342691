"""Host-side mirror of marian-edge's backend seams over libmarian_cuda.so.

* :class:`CudaEngine` is the ``CpuTokenEngine`` seam
  (``crates/marian-cpu/src/backend.rs:48-57``): ``translate_token_ids(tokens,
  offsets, max_output_tokens)`` returns ``(tokens, offsets)`` exactly like
  ``BatchOutput`` (``engine.rs:82``), plus the streaming calls of the device
  continuous batcher (``submit`` / ``step`` / ``poll``).
* :class:`CudaBackend` is the ``TranslationBackend`` contract
  (``crates/marian-core/src/backend.rs:7-38``) for callers that already hold
  token ids: ``info()``, ``is_ready()``, ``translate_batch``.

Errors map to the reference's ``BackendError`` kinds
(``marian-core/src/types.rs:61-70``) through :class:`MarianCudaError.status`.
There is no CPU path: every call runs the CUDA library or raises.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L


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


class CudaBackend:
    """TranslationBackend over token ids (the tokenizer stays with the caller)."""

    def __init__(self, model_bytes: bytes, device: int = 0, **kw):
        self.engine = CudaEngine(model_bytes, device=device, **kw)

    def info(self) -> BackendInfo:
        i = self.engine.info
        kind = "ssru" if i.decoder_kind == 0 else "self-attention"
        return BackendInfo("cuda", f"NVIDIA B200 (cuda:{self.engine.device})",
                           f"transformer-{kind} d{i.dim} e{i.encoder_layers} d{i.decoder_layers}",
                           "q8", "varlen-paged")

    def is_ready(self) -> bool:
        return self.engine.is_ready()

    def translate_batch(self, sources, max_output_tokens=512):
        """sources: list of token-id sequences each ending in EOS."""
        offsets = np.zeros(len(sources) + 1, np.uint32)
        offsets[1:] = np.cumsum([len(s) for s in sources])
        toks = np.concatenate([np.asarray(s, np.int32) for s in sources]) if sources else np.zeros(0, np.int32)
        out, off = self.engine.translate_token_ids(toks, offsets, np.full(len(sources), max_output_tokens, np.uint32))
        return [out[off[i]:off[i + 1]] for i in range(len(sources))]

    def translate_batch_with_repetitions(self, sources, repetitions, max_output_tokens=512):
        # one output per logical input (marian-core/src/backend.rs:26-37)
        assert len(sources) == len(repetitions)
        return self.translate_batch(sources, max_output_tokens)
