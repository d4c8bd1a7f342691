"""ctypes binding of the CPU oracle (liboq.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs as the checker.  The product path
(marian_cuda) never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboq.so")
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "marian-edge_b200"))
from marian_cuda import marian_bin as mb  # noqa: E402

MAX_LAYERS = 16
MAX_GEN = 256


def build(force=False):
    src = os.path.join(HERE, "q8_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(
            os.path.getmtime(src), os.path.getmtime(os.path.join(HERE, "q8_oracle.h"))):
        subprocess.run(["make", "-s", "-C", HERE], check=True)


class Linear(C.Structure):
    _fields_ = [("weights", C.c_void_p), ("activation_mult", C.c_float),
                ("weight_mult", C.c_float), ("bias", C.c_void_p),
                ("in_dim", C.c_int32), ("out_dim", C.c_int32), ("weight_row_mults", C.c_void_p)]


class AttentionBlock(C.Structure):
    _fields_ = [("wq", Linear), ("wk", Linear), ("wv", Linear), ("wo", Linear),
                ("ln_scale", C.c_void_p), ("ln_bias", C.c_void_p)]


class FfnBlock(C.Structure):
    _fields_ = [("w1", Linear), ("w2", Linear), ("ln_scale", C.c_void_p), ("ln_bias", C.c_void_p)]


class SsruBlock(C.Structure):
    _fields_ = [("w", Linear), ("wf", Linear), ("ln_scale", C.c_void_p), ("ln_bias", C.c_void_p)]


class Shortlist(C.Structure):
    _fields_ = [("first_num", C.c_uint64), ("offsets", C.c_void_p), ("targets", C.c_void_p)]


class Model(C.Structure):
    _fields_ = [("dim", C.c_int32), ("heads", C.c_int32), ("ffn_dim", C.c_int32),
                ("encoder_layers", C.c_int32), ("decoder_layers", C.c_int32),
                ("decoder_kind", C.c_int32), ("source_vocab", C.c_int32),
                ("target_vocab", C.c_int32), ("max_length_factor", C.c_int32),
                ("encoder_embedding", C.c_void_p), ("encoder_embedding_mult", C.c_float),
                ("decoder_embedding", C.c_void_p), ("decoder_embedding_mult", C.c_float),
                ("decoder_output_activation_mult", C.c_float), ("output_bias", C.c_void_p),
                ("encoder_attention", AttentionBlock * MAX_LAYERS),
                ("encoder_ffn", FfnBlock * MAX_LAYERS),
                ("decoder_ssru", SsruBlock * MAX_LAYERS),
                ("decoder_self", AttentionBlock * MAX_LAYERS),
                ("decoder_context", AttentionBlock * MAX_LAYERS),
                ("decoder_ffn", FfnBlock * MAX_LAYERS),
                ("shortlist", Shortlist)]


class Trace(C.Structure):
    _fields_ = [("encoder_output", C.c_void_p), ("cross_key", C.c_void_p),
                ("cross_value", C.c_void_p), ("decoder_state_step0", C.c_void_p),
                ("top2_gap", C.c_void_p)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(LIB_PATH)
        _lib.oq_quantize_u8.restype = C.c_int64
        _lib.oq_quantize_u8.argtypes = [C.c_void_p, C.c_size_t, C.c_float, C.c_void_p]
        _lib.oq_gemm_u8_i8.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p]
        _lib.oq_linear_run.argtypes = [C.POINTER(Linear), C.c_void_p, C.c_size_t, C.c_void_p]
        _lib.oq_epilogue.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        _lib.oq_residual_layer_norm.argtypes = [C.c_void_p] * 4 + [C.c_size_t, C.c_size_t, C.c_void_p]
        _lib.oq_ssru_update_layer_norm.argtypes = [C.c_void_p] * 6 + [C.c_size_t, C.c_size_t, C.c_void_p]
        _lib.oq_attention.argtypes = [C.c_void_p] * 4 + [C.c_size_t] * 5 + [C.c_void_p]
        _lib.oq_sinusoidal_positions.argtypes = [C.c_size_t, C.c_void_p]
        _lib.oq_full_vocab_candidates.restype = C.c_size_t
        _lib.oq_full_vocab_candidates.argtypes = [C.c_size_t, C.c_void_p]
        _lib.oq_select_token.restype = C.c_int64
        _lib.oq_select_token.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_float, C.c_float,
                                         C.c_void_p, C.c_void_p, C.c_size_t]
        _lib.oq_shortlist_candidates.restype = C.c_int64
        _lib.oq_shortlist_candidates.argtypes = [C.POINTER(Shortlist), C.c_size_t, C.c_size_t, C.c_void_p,
                                                 C.c_size_t, C.c_void_p]
        _lib.oq_translate.argtypes = [C.POINTER(Model), C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                      C.POINTER(Trace), C.c_char_p, C.c_size_t]
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


# ---- thin numpy wrappers -----------------------------------------------------

def quantize_u8(x, mult):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size, dtype=np.uint8)
    rc = lib().oq_quantize_u8(_p(x), x.size, mult, _p(out))
    if rc != 0:
        raise ValueError(f"quantization failed ({rc})")
    return out.reshape(x.shape)


def gemm_u8_i8(a_u8, w_i8):
    a = np.ascontiguousarray(a_u8, dtype=np.uint8)
    w = np.ascontiguousarray(w_i8, dtype=np.int8)
    rows, k = a.shape
    n = w.shape[0]
    acc = np.empty((rows, n), dtype=np.int32)
    lib().oq_gemm_u8_i8(_p(a), _p(w), rows, k, n, _p(acc))
    return acc


def epilogue(acc, col_scale, bias=None, row_scale=None, relu=False, residual=None):
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    rows, n = acc.shape
    out = np.empty((rows, n), dtype=np.float32)
    cs = np.ascontiguousarray(col_scale, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rs = None if row_scale is None else np.ascontiguousarray(row_scale, dtype=np.float32)
    r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
    lib().oq_epilogue(_p(acc), rows, n, _p(rs), _p(cs), _p(b), int(relu), _p(r), _p(out))
    return out


def make_linear(weights, activation_mult, weight_mult, bias=None, row_mults=None):
    w = np.ascontiguousarray(weights, dtype=np.int8)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rm = None if row_mults is None else np.ascontiguousarray(row_mults, dtype=np.float32)
    lin = Linear(w.ctypes.data, float(activation_mult), float(weight_mult), _p(b), w.shape[1], w.shape[0],
                 _p(rm))
    lin._keep = (w, b, rm)
    return lin


def linear_run(lin, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.shape[0]
    out = np.empty((rows, lin.out_dim), dtype=np.float32)
    rc = lib().oq_linear_run(C.byref(lin), _p(x), rows, _p(out))
    if rc != 0:
        raise ValueError(f"linear failed ({rc})")
    return out


def residual_layer_norm(x, r, scale, bias):
    x = np.ascontiguousarray(x, dtype=np.float32)
    r = np.ascontiguousarray(r, dtype=np.float32)
    s = np.ascontiguousarray(scale, dtype=np.float32)
    b = np.ascontiguousarray(bias, dtype=np.float32)
    rows, dim = x.shape
    out = np.empty_like(x)
    lib().oq_residual_layer_norm(_p(x), _p(r), _p(s), _p(b), rows, dim, _p(out))
    return out


def ssru_update_layer_norm(cand, forget, state, residual, scale, bias):
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (cand, forget)]
    st = np.ascontiguousarray(state, dtype=np.float32).copy()
    res = np.ascontiguousarray(residual, dtype=np.float32)
    s = np.ascontiguousarray(scale, dtype=np.float32)
    b = np.ascontiguousarray(bias, dtype=np.float32)
    rows, dim = arrs[0].shape
    out = np.empty_like(arrs[0])
    lib().oq_ssru_update_layer_norm(_p(arrs[0]), _p(arrs[1]), _p(st), _p(res), _p(s), _p(b),
                                    rows, dim, _p(out))
    return out, st


def attention(q, k, v, lengths, batch, q_len, k_len, dim, heads):
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    ln = np.ascontiguousarray(lengths, dtype=np.int32)
    out = np.empty(batch * q_len * dim, dtype=np.float32)
    rc = lib().oq_attention(_p(q), _p(k), _p(v), _p(ln), batch, q_len, k_len, dim, heads, _p(out))
    if rc != 0:
        raise ValueError(f"attention failed ({rc})")
    return out


def positions(dim):
    out = np.empty(4096 * dim, dtype=np.float32)
    if lib().oq_sinusoidal_positions(dim, _p(out)) != 0:
        raise ValueError("positional embedding dimension must be even and at least 4")
    return out


def full_vocab_candidates(vocab):
    out = np.empty(vocab, dtype=np.uint32)
    n = lib().oq_full_vocab_candidates(vocab, _p(out))
    return out[:n].copy()


# ---- lexical shortlist (marian-model/src/shortlist.rs) -----------------------

SHORTLIST_MAGIC = 17_373_278_592_220_534_773       # shortlist.rs:3
SHORTLIST_MAX_TARGET_ENTRIES = 4_000_000           # shortlist.rs:4


def parse_shortlist(data: bytes, source_vocab: int, target_vocab: int):
    """LexicalShortlist::from_bytes (shortlist.rs:59-148): a 48-byte header of
    six little-endian u64 (magic, -, firstNum, -, offset count, target count),
    the u64 offsets (source_vocab + 1, from 0 up to the target count) and the
    u32 target ids.  Returns (first_num, offsets, targets); raises ValueError
    with the reference's messages."""
    maximum = 48 + (source_vocab + 1) * 8 + SHORTLIST_MAX_TARGET_ENTRIES * 4
    if len(data) > maximum:
        raise ValueError(f"lexical shortlist has {len(data)} bytes; maximum is {maximum}")
    if len(data) < 48:
        raise ValueError("truncated lexical shortlist header")
    magic, _, first_num, _, offset_count, target_count = struct.unpack_from("<6Q", data, 0)
    if (magic != SHORTLIST_MAGIC or offset_count != source_vocab + 1 or first_num > target_vocab
            or target_count > SHORTLIST_MAX_TARGET_ENTRIES):
        raise ValueError("unsupported lexical shortlist format")
    expected = 48 + offset_count * 8 + target_count * 4
    if len(data) != expected:
        raise ValueError(f"lexical shortlist has {len(data)} bytes, expected {expected}")
    offsets = np.frombuffer(data, "<u8", offset_count, 48).astype(np.uint64)
    if (offsets[0] != 0 or offsets[-1] != target_count or np.any(offsets[1:] < offsets[:-1])
            or np.any(offsets > target_count)):
        raise ValueError("lexical shortlist offsets are invalid")
    targets = np.frombuffer(data, "<u4", target_count, 48 + offset_count * 8).astype(np.uint32)
    bad = np.nonzero(targets >= target_vocab)[0]
    if bad.size:
        raise ValueError(f"lexical shortlist target {targets[bad[0]]} exceeds vocabulary {target_vocab}")
    return int(first_num), offsets, targets


def _shortlist_struct(parsed, keep):
    if parsed is None:
        return Shortlist(0, None, None)
    first_num, offsets, targets = parsed
    keep.extend([offsets, targets])
    return Shortlist(first_num, offsets.ctypes.data, targets.ctypes.data)


def shortlist_candidates(parsed, source_vocab, target_vocab, tokens):
    """LexicalShortlist::candidates (shortlist.rs:150-198) for one sentence;
    parsed is parse_shortlist's result or None (no shortlist file)."""
    keep = []
    sl = _shortlist_struct(parsed, keep)
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.empty(max(1, target_vocab), dtype=np.uint32)
    n = lib().oq_shortlist_candidates(C.byref(sl), source_vocab, target_vocab, _p(t), t.size, _p(out))
    messages = {-1: "source token ID is negative", -2: "source token exceeds vocabulary",
                -3: "lexical shortlist produced no candidates",
                -4: "lexical shortlist does not contain EOS token 0"}
    if n < 0:
        raise ValueError(messages[n])
    return out[:n].copy()


def select_token(state, embedding, embedding_mult, activation_mult, output_bias, candidates):
    st = np.ascontiguousarray(state, dtype=np.float32)
    e = np.ascontiguousarray(embedding, dtype=np.int8)
    b = np.ascontiguousarray(output_bias, dtype=np.float32)
    c = np.ascontiguousarray(candidates, dtype=np.uint32)
    return lib().oq_select_token(_p(st), st.size, _p(e), embedding_mult, activation_mult, _p(b),
                                 _p(c), c.size)


# ---- model -------------------------------------------------------------------

class OracleModel:
    """A parsed Marian binary v1 model bound to the oracle's C structs."""

    def __init__(self, model_bytes: bytes, max_length_factor: int = 3, shortlist: bytes | None = None):
        t = mb.parse(model_bytes)
        self.tensors = t
        self._keep = []
        m = Model()
        ew, eq = t["encoder_Wemb"].data
        dw, dq = t["decoder_Wemb"].data
        vocab, dim = t["encoder_Wemb"].shape
        m.dim = dim
        enc_layers = sum(1 for n in t if n.startswith("encoder_l") and n.endswith("_self_Wq"))
        dec_self = sum(1 for n in t if n.startswith("decoder_l") and n.endswith("_self_Wq"))
        dec_ssru = sum(1 for n in t if n.startswith("decoder_l") and n.endswith("_rnn_W"))
        m.decoder_kind = 1 if dec_self else 0
        m.decoder_layers = dec_self or dec_ssru
        m.encoder_layers = enc_layers
        m.ffn_dim = t["encoder_l1_ffn_W1"].shape[1]
        yml = bytes(t["special:model.yml"].data.astype(np.uint8)).decode(errors="replace")
        heads = 8
        for line in yml.splitlines():
            if line.startswith("transformer-heads:"):
                heads = int(line.split(":")[1])
        m.heads = heads
        m.source_vocab = vocab
        m.target_vocab = t["decoder_Wemb"].shape[0]
        m.max_length_factor = max_length_factor
        m.encoder_embedding = self._hold(ew)
        m.encoder_embedding_mult = float(eq)
        m.decoder_embedding = self._hold(dw)
        m.decoder_embedding_mult = float(dq)
        m.decoder_output_activation_mult = float(mb.activation_scale(t, "decoder_Wemb"))
        m.output_bias = self._hold(t["decoder_ff_logit_out_b"].data)
        for i in range(enc_layers):
            self._attn(m.encoder_attention[i], f"encoder_l{i + 1}_self")
            self._ffn(m.encoder_ffn[i], f"encoder_l{i + 1}_ffn")
        for i in range(m.decoder_layers):
            p = f"decoder_l{i + 1}"
            if m.decoder_kind == 0:
                s = m.decoder_ssru[i]
                s.w = self._linear(p + "_rnn_W", None)
                s.wf = self._linear(p + "_rnn_Wf", p + "_rnn_bf")
                s.ln_scale = self._hold(t[p + "_rnn_ffn_ln_scale"].data)
                s.ln_bias = self._hold(t[p + "_rnn_ffn_ln_bias"].data)
            else:
                self._attn(m.decoder_self[i], p + "_self")
            self._attn(m.decoder_context[i], p + "_context")
            self._ffn(m.decoder_ffn[i], p + "_ffn")
        self.shortlist = None
        if shortlist is not None:
            self.shortlist = parse_shortlist(shortlist, m.source_vocab, m.target_vocab)
        m.shortlist = _shortlist_struct(self.shortlist, self._keep)
        self.model = m
        self.dim = dim
        self.heads = heads
        self.positions = positions(dim)

    def _hold(self, arr):
        arr = np.ascontiguousarray(arr)
        self._keep.append(arr)
        return arr.ctypes.data

    def _linear(self, wname, bname):
        t = self.tensors
        w, qm = t[wname].data
        in_dim, out_dim = t[wname].shape
        alpha = mb.activation_scale(t, wname)
        b = self._hold(t[bname].data) if bname else None
        rows = t.get(wname + "_QuantMultRows")  # per-row extension
        rm = self._hold(np.asarray(rows.data, np.float32).reshape(-1)) if rows is not None else None
        return Linear(self._hold(w), float(alpha), float(qm), b, in_dim, out_dim, rm)

    def _attn(self, blk, prefix):
        blk.wq = self._linear(prefix + "_Wq", prefix + "_bq")
        blk.wk = self._linear(prefix + "_Wk", prefix + "_bk")
        blk.wv = self._linear(prefix + "_Wv", prefix + "_bv")
        blk.wo = self._linear(prefix + "_Wo", prefix + "_bo")
        blk.ln_scale = self._hold(self.tensors[prefix + "_Wo_ln_scale"].data)
        blk.ln_bias = self._hold(self.tensors[prefix + "_Wo_ln_bias"].data)

    def _ffn(self, blk, prefix):
        blk.w1 = self._linear(prefix + "_W1", prefix + "_b1")
        blk.w2 = self._linear(prefix + "_W2", prefix + "_b2")
        blk.ln_scale = self._hold(self.tensors[prefix + "_ffn_ln_scale"].data)
        blk.ln_bias = self._hold(self.tensors[prefix + "_ffn_ln_bias"].data)

    def translate(self, tokens, offsets, max_out, force_len=None, trace=False):
        """Returns (out_tokens, out_offsets[, trace dict])."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.uint32)
        batch = len(offsets) - 1
        mo = np.ascontiguousarray(max_out, dtype=np.uint32)
        fl = None if force_len is None else np.ascontiguousarray(force_len, dtype=np.uint32)
        cap = batch * MAX_GEN
        out_tokens = np.empty(cap, dtype=np.int32)
        out_offsets = np.empty(batch + 1, dtype=np.uint32)
        err = C.create_string_buffer(512)
        tr = None
        bufs = {}
        if trace:
            lmax = int(np.diff(offsets.astype(np.int64)).max())
            L = self.model.decoder_layers
            bufs = {
                "encoder_output": np.zeros((batch * lmax, self.dim), np.float32),
                "cross_key": np.zeros((L, batch * lmax, self.dim), np.float32),
                "cross_value": np.zeros((L, batch * lmax, self.dim), np.float32),
                "decoder_state_step0": np.zeros((batch, self.dim), np.float32),
                "top2_gap": np.full((batch, MAX_GEN), np.nan, np.float32),
            }
            tr = Trace(*(bufs[k].ctypes.data for k in
                         ("encoder_output", "cross_key", "cross_value", "decoder_state_step0", "top2_gap")))
        rc = lib().oq_translate(C.byref(self.model), _p(self.positions), _p(tokens), _p(offsets), batch,
                                _p(mo), _p(fl), _p(out_tokens), _p(out_offsets), cap,
                                C.byref(tr) if tr is not None else None, err, 512)
        if rc != 0:
            raise ValueError(err.value.decode())
        toks = out_tokens[:out_offsets[-1]].copy()
        if trace:
            return toks, out_offsets, bufs
        return toks, out_offsets
