"""Seeded synthetic models and request streams for tests and benchmarks.

No real model, vocabulary or corpus is available to this build, so parity and
throughput are measured on random-init models written in Marian binary v1 and
on token-id streams drawn from fixed distributions:

* ids: Zipf(s=1.1) over 3..V-1 (rejection sampled), EOS=0 appended;
* short batches: source length uniform 8..64 (EOS excluded);
* streams: source length lognormal(ln 24, 0.8) clipped to 4..256 tokens
  including EOS;
* output length: the harness rule ``force_len = round_half_even(1.2 * src)``
  (src excludes EOS) masks EOS until the last step so the work is fixed.

Model shapes: ``graph_r`` is the reference's shipped Transformer-SSRU
(d=384, 8 heads, 6 encoder layers, 4 SSRU decoder layers, FFN 1536,
``marian-model/src/manifest.rs:27-36``); ``graph_b`` is the benchmark shape
(d=512, 8 heads, 6 encoder layers, 2 self+cross-attention decoder layers,
FFN 2048).  Both have a 32000 vocabulary and tensor names following
``q8_engine.rs:1050-1101``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import marian_bin as mb

EOS = 0


@dataclass(frozen=True)
class ModelShape:
    dim: int
    heads: int
    ffn: int
    encoder_layers: int
    decoder_layers: int
    decoder_kind: str  # "ssru" or "selfattn"
    vocab: int = 32000
    max_length_factor: int = 3


GRAPH_R = ModelShape(384, 8, 1536, 6, 4, "ssru")
GRAPH_B = ModelShape(512, 8, 2048, 6, 2, "selfattn")
# Small shapes keep CPU-only tests fast; they exercise every code path.
TINY_SSRU = ModelShape(128, 4, 256, 2, 2, "ssru", vocab=512)
TINY_SELF = ModelShape(128, 4, 256, 2, 2, "selfattn", vocab=512)
# FFN 4d at d = 128 and d = 256: the fused kernel's FFN variant at its other
# two widths (clusters of 4 and 8 CTAs of 32 columns).
TINY_SELF_FFN4 = ModelShape(128, 4, 512, 2, 2, "selfattn", vocab=512)
MID_SELF = ModelShape(256, 4, 1024, 2, 2, "selfattn", vocab=1024)

SHAPES = {"graph_r": GRAPH_R, "graph_b": GRAPH_B, "tiny_ssru": TINY_SSRU, "tiny_self": TINY_SELF,
          "tiny_self_ffn4": TINY_SELF_FFN4, "mid_self": MID_SELF}

_Q8_STD = float(np.sqrt((255.0 ** 2 - 1.0) / 12.0))  # std of U{-127..127}


def _q8_weight(rng, out_dim, in_dim, gain=1.0):
    values = rng.integers(-127, 128, size=(out_dim, in_dim), dtype=np.int16).astype(np.int8)
    # real weight = q / quant_mult with std ~ gain/sqrt(in_dim)
    quant_mult = np.float32(_Q8_STD * np.sqrt(in_dim) / gain)
    return values, quant_mult


def _alpha(rng):
    # Static activation alpha: inputs have std ~1, clip at ~5 sigma.
    return np.float32(25.0 * rng.uniform(0.9, 1.1))


# Random post-norm stacks drift toward one shared direction per row; zero-sum
# W2 rows remove the common-mode output the ReLU's positive mean would add.
_BRANCH_GAIN = 1.0
_ZERO_SUM = True
# A small decoder embedding weakens the tied-embedding self-loop (the previous
# token's embedding re-selecting itself), so outputs are less repetitive.
_DECODER_EMB_GAIN = 0.1


def _zero_sum_rows(values):
    """Shift each int8 row so it sums to ~0 (removes the common-mode output
    a ReLU's positive mean would otherwise add to every row)."""
    v = values.astype(np.int32)
    v -= np.rint(v.mean(axis=1, keepdims=True)).astype(np.int32)
    return np.clip(v, -127, 127).astype(np.int8)


def _dense(tensors, rng, name, in_dim, out_dim, bias_name=None, per_row=False):
    gain = _BRANCH_GAIN if name.endswith(("_Wo", "_W2")) else 1.0
    w, qm = _q8_weight(rng, out_dim, in_dim, gain)
    if _ZERO_SUM and name.endswith("_W2"):
        w = _zero_sum_rows(w)
    tensors.append(mb.q8(name, w, qm, (in_dim, out_dim)))
    tensors.append(mb.f32(name + "_QuantMultA", [_alpha(rng)], (1, 1)))
    if per_row:
        # per-output-row multipliers (the loader's _QuantMultRows extension):
        # row n's real weights are w[n] / mult[n]
        mult = (qm * rng.uniform(0.5, 2.0, out_dim)).astype(np.float32)
        tensors.append(mb.f32(name + "_QuantMultRows", mult, (1, out_dim)))
    if bias_name:
        tensors.append(mb.f32(bias_name, rng.uniform(-0.1, 0.1, out_dim), (1, out_dim)))


def _ln(tensors, rng, prefix, dim):
    tensors.append(mb.f32(prefix + "_scale", 1.0 + rng.uniform(-0.1, 0.1, dim), (1, dim)))
    tensors.append(mb.f32(prefix + "_bias", rng.uniform(-0.1, 0.1, dim), (1, dim)))


def _attention(tensors, rng, prefix, d, per_row=False):
    for w, b in (("Wq", "bq"), ("Wk", "bk"), ("Wv", "bv"), ("Wo", "bo")):
        _dense(tensors, rng, f"{prefix}_{w}", d, d, f"{prefix}_{b}", per_row)
    _ln(tensors, rng, f"{prefix}_Wo_ln", d)


def _ffn(tensors, rng, prefix, d, f, per_row=False):
    _dense(tensors, rng, f"{prefix}_W1", d, f, f"{prefix}_b1", per_row)
    _dense(tensors, rng, f"{prefix}_W2", f, d, f"{prefix}_b2", per_row)
    _ln(tensors, rng, f"{prefix}_ffn_ln", d)


def synthetic_model(shape: ModelShape, seed: int = 0, per_row: bool = False) -> bytes:
    """Random-init Q8 model of the given shape, as Marian binary v1 bytes.

    per_row: every dense linear also carries per-output-row weight
    multipliers (``<W>_QuantMultRows``, the per-row scale extension);
    embeddings keep their per-tensor multiplier."""
    rng = np.random.Generator(np.random.PCG64(seed))
    d, f, v = shape.dim, shape.ffn, shape.vocab
    t: list = []
    emb_qm = np.float32(_Q8_STD * np.sqrt(d))
    t.append(mb.q8("encoder_Wemb", _q8_weight(rng, v, d)[0], emb_qm, (v, d)))
    t.append(mb.q8("decoder_Wemb", _q8_weight(rng, v, d)[0], np.float32(emb_qm / _DECODER_EMB_GAIN), (v, d)))
    t.append(mb.f32("decoder_Wemb_QuantMultA", [_alpha(rng)], (1, 1)))
    t.append(mb.f32("decoder_ff_logit_out_b", rng.uniform(-0.1, 0.1, v), (1, v)))
    yml = (f"# synthetic marian-cuda test model\ndim-emb: {d}\ntransformer-heads: {shape.heads}\n"
           f"enc-depth: {shape.encoder_layers}\ndec-depth: {shape.decoder_layers}\n"
           f"transformer-dim-ffn: {f}\ndec-cell: {shape.decoder_kind}\n"
           f"max-length-factor: {shape.max_length_factor}\n").encode()
    t.append(mb.raw_int8("special:model.yml", yml))
    for layer in range(1, shape.encoder_layers + 1):
        _attention(t, rng, f"encoder_l{layer}_self", d, per_row)
        _ffn(t, rng, f"encoder_l{layer}_ffn", d, f, per_row)
    for layer in range(1, shape.decoder_layers + 1):
        if shape.decoder_kind == "ssru":
            p = f"decoder_l{layer}_rnn"
            _dense(t, rng, p + "_W", d, d, None, per_row)
            _dense(t, rng, p + "_Wf", d, d, p + "_bf", per_row)
            _ln(t, rng, p + "_ffn_ln", d)
        else:
            _attention(t, rng, f"decoder_l{layer}_self", d, per_row)
        _attention(t, rng, f"decoder_l{layer}_context", d, per_row)
        _ffn(t, rng, f"decoder_l{layer}_ffn", d, f, per_row)
    return mb.write(t)


# ---- token streams ---------------------------------------------------------

def zipf_ids(rng, n, vocab, s=1.1):
    """n ids ~ Zipf(s) shifted to start at 3, rejection-sampled into [3, vocab)."""
    out = np.empty(n, dtype=np.int32)
    filled = 0
    while filled < n:
        z = rng.zipf(s, size=2 * (n - filled) + 16) + 2
        z = z[z < vocab]
        take = min(len(z), n - filled)
        out[filled:filled + take] = z[:take]
        filled += take
    return out


def force_lengths(src_lens):
    """Harness output length: round_half_even(1.2 * src_len), src excludes EOS."""
    return np.rint(1.2 * np.asarray(src_lens, dtype=np.float64)).astype(np.uint32)


@dataclass
class Batch:
    tokens: np.ndarray      # int32, packed, each source ends in EOS
    offsets: np.ndarray     # uint32 [B+1]
    max_out: np.ndarray     # uint32 [B]
    force_len: np.ndarray   # uint32 [B]

    @property
    def size(self):
        return len(self.offsets) - 1


def pack(sources, max_out=None, force=True) -> Batch:
    tokens = np.concatenate([np.append(np.asarray(s, dtype=np.int32), EOS) for s in sources]).astype(np.int32)
    lens = np.array([len(s) + 1 for s in sources], dtype=np.uint32)
    offsets = np.zeros(len(sources) + 1, dtype=np.uint32)
    offsets[1:] = np.cumsum(lens)
    fl = force_lengths([len(s) for s in sources])
    fl = np.maximum(fl, 1).astype(np.uint32)
    if max_out is None:
        max_out = fl.copy() if force else np.full(len(sources), 512, dtype=np.uint32)
    return Batch(tokens, offsets, np.asarray(max_out, dtype=np.uint32), fl if force else None)


def short_batch(n=16, vocab=32000, seed=0, lo=8, hi=64) -> Batch:
    """Static batch: lengths uniform lo..hi (EOS excluded), Zipf ids."""
    rng = np.random.Generator(np.random.PCG64(seed))
    lens = rng.integers(lo, hi + 1, size=n)
    return pack([zipf_ids(rng, int(l), vocab) for l in lens])


def lognormal_lengths(rng, n, median=24.0, sigma=0.8, lo=4, hi=256):
    """Source lengths including EOS."""
    lens = np.rint(rng.lognormal(np.log(median), sigma, size=n)).astype(np.int64)
    return np.clip(lens, lo, hi)


def stream_batch(n=256, vocab=32000, seed=0) -> Batch:
    """Ragged batch with lognormal lengths (encoder and stream workloads)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    lens = lognormal_lengths(rng, n)
    return pack([zipf_ids(rng, int(l) - 1, vocab) for l in lens])


class WordIds:
    """Tokenizer of the synthetic documents: the word "w<id>" (a trailing
    '.' marks a pseudo-sentence end) is the piece <id>."""

    def __init__(self, vocab=32000):
        self.vocab = vocab

    def vocabulary_size(self):
        return self.vocab

    def encode(self, text):
        return [int(w.rstrip(".")[1:]) for w in text.split()]

    def decode(self, ids):
        return " ".join(f"w{i}" for i in ids)


def longtext_document(rng, vocab=32000, lo=200, hi=2000, s_lo=8, s_hi=64) -> str:
    """One long-text document: lo..hi Zipf ids as words, with a pseudo-sentence
    end ('.') every s_lo..s_hi tokens."""
    n = int(rng.integers(lo, hi + 1))
    ids = zipf_ids(rng, n, vocab)
    parts, k = [], 0
    while k < n:
        m = min(int(rng.integers(s_lo, s_hi + 1)), n - k)
        parts.append(" ".join(f"w{i}" for i in ids[k:k + m]) + ".")
        k += m
    return " ".join(parts)


def longtext_batch(n_docs, vocab=32000, seed=0, rank=0, world=1, max_tokens=128) -> Batch:
    """The long-text stream: n_docs documents split by the library's
    segment_text into segments of at most max_tokens tokens with EOS, sorted
    by length and dealt round-robin over `world` replicas (this one takes
    every world-th from `rank`); output length rule as the other workloads."""
    from . import segmenter
    rng = np.random.Generator(np.random.PCG64(seed))
    tok = WordIds(vocab)
    sources = []
    for _ in range(n_docs):
        doc = longtext_document(rng, vocab)
        for sg in segmenter.segment_text(doc, max_tokens - 1, lambda t: len(t.split())):
            ids = tok.encode(sg.content(doc))
            if ids:
                sources.append(ids)
    order = sorted(range(len(sources)), key=lambda i: (len(sources[i]), i))
    return pack([sources[i] for i in order[rank::world]])


def poisson_arrivals(n, rate, seed=0):
    rng = np.random.Generator(np.random.PCG64(seed + 7919))
    return np.cumsum(rng.exponential(1.0 / rate, size=n))


def legal_cpu_batches(batch: Batch, max_batch=256, max_cells=65536):
    """Split a batch into reference-legal engine batches.

    First-fit in input order as marian-cpu/src/backend.rs:223-243: each pass
    scans the remaining rows and adds every row that keeps the batch at most
    256 rows and batch * Lmax^2 at most 65536 cells.
    """
    lens = [int(l) for l in np.diff(batch.offsets.astype(np.int64))]
    remaining = list(range(len(lens)))
    groups = []
    while remaining:
        cur, lmax, rest = [], 0, []
        for i in remaining:
            if len(cur) >= max_batch:
                rest.append(i)
                continue
            cand = max(lmax, lens[i])
            if (len(cur) + 1) * cand * cand > max_cells:
                rest.append(i)
                continue
            cur.append(i)
            lmax = cand
        if not cur:
            raise ValueError("unable to construct a bounded CPU inference batch")
        groups.append(cur)
        remaining = rest
    return groups


def subset(batch: Batch, rows) -> Batch:
    rows = list(rows)
    srcs = [batch.tokens[batch.offsets[r]:batch.offsets[r + 1] - 1] for r in rows]
    b = pack(srcs, max_out=batch.max_out[rows], force=batch.force_len is not None)
    return b


# ---- lexical shortlist files (marian-model/src/shortlist.rs:59-148 format) ---
SHORTLIST_MAGIC = 17_373_278_592_220_534_773


def shortlist_bytes(first_num: int, offsets, targets) -> bytes:
    """A Marian lexical shortlist file: six little-endian u64 header fields
    (magic, 0, firstNum, 0, offset count, target count), u64 offsets, u32
    targets -- the layout the reference's test fixture writes
    (shortlist.rs:239-257)."""
    offsets = np.asarray(offsets, dtype="<u8")
    targets = np.asarray(targets, dtype="<u4")
    head = np.array([SHORTLIST_MAGIC, 0, first_num, 0, offsets.size, targets.size], dtype="<u8")
    return head.tobytes() + offsets.tobytes() + targets.tobytes()


def synthetic_shortlist(source_vocab: int, target_vocab: int, seed: int = 0, first_num: int = 100,
                        max_per_token: int = 40) -> bytes:
    """Seeded random shortlist: each source id gets 0..max_per_token distinct
    uniformly drawn target ids in [2, target_vocab); ids below first_num (EOS
    among them when first_num > 0) are always candidates."""
    rng = np.random.Generator(np.random.PCG64(seed))
    offsets = [0]
    targets = []
    for _ in range(source_vocab):
        k = int(rng.integers(0, max_per_token + 1))
        ids = np.unique(rng.integers(2, target_vocab, size=k)) if k else np.zeros(0, np.int64)
        targets.extend(int(t) for t in ids)
        offsets.append(len(targets))
    return shortlist_bytes(first_num, offsets, targets)
