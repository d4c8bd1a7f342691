"""Marian binary v1 reader/writer against legacy_q8.rs's own fixtures
(crates/marian-cpu/src/legacy_q8.rs:796-1000)."""
import struct

import numpy as np
import pytest

from marian_cuda import marian_bin as mb


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


def test_parses_v1_and_q8_roles():
    # legacy_q8.rs:905-929
    t = mb.parse(mb.write(valid_items()))
    assert len(t) == 8
    w = t["encoder_l1_self_Wq"]
    assert w.shape == (2, 3)
    assert len(w.payload()) == 256
    values, qm = w.data
    assert values.tolist() == [2, -3, 5, 7, -11, 13] and qm == 8.0
    assert t["special:model.yml"].data.tolist() == [97, 98, 99]


def test_normalizes_accidentally_quantized_decoder_alpha():
    # legacy_q8.rs:931-942
    t = mb.parse(mb.write(valid_items()))
    assert abs(mb.activation_scale(t, "decoder_Wemb") - 8.279258) < 1e-5


def test_embedding_row_dequantizes_one_row():
    # legacy_q8.rs:944-952
    t = mb.parse(mb.write(valid_items()))
    values, qm = t["encoder_Wemb"].data
    row = values.reshape(2, 2)[1].astype(np.float32) / np.float32(qm)
    assert row.tolist() == [1.0, -1.0]


def test_rejects_truncation_trailing_data_and_wrong_version():
    # legacy_q8.rs:954-964
    data = mb.write(valid_items())
    with pytest.raises(mb.MarianFormatError):
        mb.parse(data[:-1])
    with pytest.raises(mb.MarianFormatError):
        mb.parse(data + b"\0")
    with pytest.raises(mb.MarianFormatError):
        mb.parse(struct.pack("<Q", 2) + data[8:])


def test_rejects_invalid_shapes_scales_and_q8_range():
    # legacy_q8.rs:966-980
    items = valid_items()
    items[0] = mb.Tensor("encoder_l1_self_Wq", mb.TYPE_INTGEMM8, (-1, 3), items[0].data)
    with pytest.raises(mb.MarianFormatError):
        mb.parse(mb.write(items))
    items = valid_items()
    items[0] = mb.q8("encoder_l1_self_Wq", [2, -3, 5, 7, -11, 13], float("nan"), (2, 3))
    with pytest.raises(mb.MarianFormatError):
        mb.parse(mb.write(items))
    items = valid_items()
    items[0] = mb.q8("encoder_l1_self_Wq", [-128, -3, 5, 7, -11, 13], 8.0, (2, 3))
    with pytest.raises(mb.MarianFormatError):
        mb.parse(mb.write(items))
    with pytest.raises(mb.MarianFormatError):
        mb.parse(mb.write([valid_items()[0], valid_items()[0]]))
