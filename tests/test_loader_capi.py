"""The library's own Marian binary v1 reader (csrc/model_loader.cpp) through
the C ABI, on the host (mc_inspect_marian_bin needs no device).

The fixtures restate legacy_q8.rs's tests (crates/marian-cpu/src/
legacy_q8.rs:851-995): the valid item set, truncation, trailing data, wrong
version, invalid shapes, non-finite multipliers, -128, duplicate names, and
missing or orphan activation scales; plus the alpha normalisation golden
8.279258 (legacy_q8.rs:931-942).  The per-row weight-multiplier extension
(<W>_QuantMultRows) is checked the same way.  Every case is also given to
the Python reader (marian_bin.py), which must agree.
"""
import ctypes as C
import struct

import numpy as np
import pytest

from marian_cuda import _lib as L
from marian_cuda import marian_bin as mb
from marian_cuda import workloads as W


def inspect(data: bytes):
    lib = L.load()
    rep = L.ModelReport()
    msg = C.create_string_buffer(512)
    st = lib.mc_inspect_marian_bin(data, len(data), C.byref(rep), msg, 512)
    return st, rep, msg.value.decode()


def python_accepts(data: bytes):
    try:
        t = mb.parse(data)
    except mb.MarianFormatError:
        return False
    # validate_q8's scale relationships (legacy_q8.rs:497-542)
    try:
        for name, tensor in t.items():
            if name.endswith("_QuantMultA"):
                weight = name[: -len("_QuantMultA")]
                mb.activation_scale(t, weight)
                if t[weight].tensor_type != mb.TYPE_INTGEMM8:
                    return False
            elif tensor.tensor_type == mb.TYPE_INTGEMM8 and not name.endswith("_Wemb"):
                mb.activation_scale(t, name)
    except (KeyError, mb.MarianFormatError, ValueError):
        return False
    return True


def valid_items():
    # legacy_q8.rs:851-903
    return [
        mb.q8("encoder_l1_self_Wq", [2, -3, 5, 7, -11, 13], 8.0, (2, 3)),
        mb.f32("encoder_l1_self_Wq_QuantMultA", [4.0], (1, 1)),
        mb.f32("encoder_l1_self_bq", [0.25, -0.5, 1.0], (1, 3)),
        mb.q8("encoder_Wemb", [8, -8, 4, -4], 4.0, (2, 2)),
        mb.q8("decoder_Wemb", [1, 2, 3, 4, 5, 6], 2.0, (3, 2)),
        mb.q8("decoder_Wemb_QuantMultA", [127], 15.33954, (1, 1)),
        mb.f32("decoder_ff_logit_out_b", [0.0, 0.25, -0.25], (1, 3)),
        mb.raw_int8("special:model.yml", b"abc"),
    ]


def test_valid_fixture_parses_with_the_references_inventory():
    st, rep, msg = inspect(mb.write(valid_items()))
    assert st == L.MC_OK, msg
    assert (rep.tensors, rep.dense_linears, rep.embeddings, rep.activation_scales) == (8, 1, 2, 2)
    assert abs(rep.decoder_output_alpha - 8.279258) < 1e-5  # legacy_q8.rs:931-942
    assert rep.engine_graph == 0 and msg  # a valid Q8 file, but not an engine graph


def _bad_cases():
    data = mb.write(valid_items())
    cases = {
        "truncated": data[:-1],
        "trailing byte": data + b"\0",
        "version 2": struct.pack("<Q", 2) + data[8:],
        "empty": b"",
    }
    items = valid_items()
    items[0] = mb.Tensor("encoder_l1_self_Wq", mb.TYPE_INTGEMM8, (-1, 3), items[0].data)
    cases["negative shape"] = mb.write(items)
    items = valid_items()
    items[0] = mb.q8("encoder_l1_self_Wq", [2, -3, 5, 7, -11, 13], float("nan"), (2, 3))
    cases["nan multiplier"] = mb.write(items)
    items = valid_items()
    items[0] = mb.q8("encoder_l1_self_Wq", [-128, -3, 5, 7, -11, 13], 8.0, (2, 3))
    cases["-128"] = mb.write(items)
    cases["duplicate"] = mb.write([valid_items()[0], valid_items()[0]])
    items = valid_items()
    del items[1]
    cases["missing activation scale"] = mb.write(items)  # legacy_q8.rs:985-990
    items = valid_items()
    items[1] = mb.f32("absent_W_QuantMultA", [4.0], (1, 1))
    cases["orphan activation scale"] = mb.write(items)  # legacy_q8.rs:992-995
    items = valid_items()
    items[1] = mb.f32("encoder_l1_self_Wq_QuantMultA", [-4.0], (1, 1))
    cases["negative activation scale"] = mb.write(items)
    items = valid_items()
    items[1] = mb.f32("encoder_l1_self_Wq_QuantMultA", [4.0, 4.0], (1, 2))
    cases["vector activation scale"] = mb.write(items)
    padded = bytearray(data)
    padded[-4] = 1  # the zero padding of the float32 record before the 3-byte raw one
    cases["non-zero record padding"] = bytes(padded)
    return cases


@pytest.mark.parametrize("case", sorted(_bad_cases()))
def test_invalid_files_are_rejected_as_model_errors(case):
    data = _bad_cases()[case]
    st, _, msg = inspect(data)
    assert st == L.MC_MODEL, (case, st)
    assert msg
    assert not python_accepts(data), case


def test_engine_graphs_are_recognised():
    for name, kind in (("graph_b", 1), ("graph_r", 0), ("tiny_ssru", 0)):
        shape = W.SHAPES[name]
        st, rep, msg = inspect(W.synthetic_model(shape, seed=0))
        assert st == L.MC_OK, msg
        assert rep.engine_graph == 1 and rep.decoder_kind == kind
        assert (rep.dim, rep.heads, rep.encoder_layers, rep.decoder_layers) == (
            shape.dim, shape.heads, shape.encoder_layers, shape.decoder_layers)
        assert rep.row_scaled_linears == 0


def _per_row_model():
    return W.synthetic_model(W.TINY_SELF, seed=1, per_row=True)


def test_per_row_extension_is_accepted():
    st, rep, msg = inspect(_per_row_model())
    assert st == L.MC_OK, msg
    assert rep.engine_graph == 1
    assert rep.row_scaled_linears == rep.dense_linears > 0


def _replace(data: bytes, name: str, tensor):
    t = mb.parse(data)
    items = [tensor if n == name else t[n] for n in t]
    return mb.write(items)


@pytest.mark.parametrize("bad", ["nan", "zero", "shape", "embedding"])
def test_per_row_extension_rejects_bad_multipliers(bad):
    data = _per_row_model()
    name = "encoder_l1_self_Wq_QuantMultRows"
    out = W.TINY_SELF.dim
    good = np.asarray(mb.parse(data)[name].data, np.float32)
    if bad == "nan":
        v = good.copy()
        v[3] = np.nan
        data = _replace(data, name, mb.f32(name, v, (1, out)))
    elif bad == "zero":
        v = good.copy()
        v[0] = 0.0
        data = _replace(data, name, mb.f32(name, v, (1, out)))
    elif bad == "shape":
        data = _replace(data, name, mb.f32(name, good[:-1], (1, out - 1)))
    else:  # multipliers for an embedding table are not part of the extension
        t = mb.parse(data)
        items = list(t.values()) + [mb.f32("encoder_Wemb_QuantMultRows", np.ones(W.TINY_SELF.vocab),
                                           (1, W.TINY_SELF.vocab))]
        data = mb.write(items)
    st, _, msg = inspect(data)
    assert st == L.MC_MODEL, (bad, st, msg)
