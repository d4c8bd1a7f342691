"""Pin the CPU oracle to the reference's own unit vectors.

Each test restates one reference test (file:line given) against the oracle
library; the expected values are the reference's literals.
"""
import math

import numpy as np
import pytest

import oracle as O
from marian_cuda import workloads as W


def test_quantization_ties_to_even_and_saturation():
    # crates/marian-cpu/src/q8_gemm.rs:609-617
    x = np.array([-200.0, -127.6, -126.5, -1.5, -0.5, 0.5, 1.5, 126.5, 127.6, 200.0], np.float32)
    assert O.quantize_u8(x, 1.0).tolist() == [0, 0, 1, 125, 127, 127, 129, 253, 254, 254]
    with pytest.raises(ValueError):
        O.quantize_u8(np.array([np.nan], np.float32), 1.0)
    with pytest.raises(ValueError):
        O.quantize_u8(np.array([0.0], np.float32), 0.0)


LINEAR_W = np.array([2, -3, 5, 7, -11, 13, -17, 19], np.int8).reshape(2, 4)
LINEAR_INPUTS = [
    ([0.0, 0.25, -0.5, 1.0], 1),
    ([0.0, 0.25, -0.5, 1.0, 1.25, -1.0, 0.5, -0.25], 2),
    ([0.0, 0.25, -0.5, 1.0, 1.25, -1.0, 0.5, -0.25, -2.0, 0.75, 1.5, 0.0], 3),
    ([0.0, 0.25, -0.5, 1.0, 1.25, -1.0, 0.5, -0.25, -2.0, 0.75, 1.5, 0.0, 0.5, 0.5, -0.5, -0.5], 4),
]


@pytest.mark.parametrize("values,rows", LINEAR_INPUTS)
def test_linear_matches_integer_oracle(values, rows):
    # crates/marian-cpu/src/q8_gemm.rs:620-668
    lin = O.make_linear(LINEAR_W, 4.0, 8.0, np.array([0.25, -0.5], np.float32))
    x = np.array(values, np.float32).reshape(rows, 4)
    q = O.quantize_u8(x, 4.0).astype(np.int32)
    expected = np.empty((rows, 2), np.float32)
    for r in range(rows):
        for c in range(2):
            acc = int(((q[r] - 127) * LINEAR_W[c].astype(np.int32)).sum())
            expected[r, c] = np.float32(np.float32(acc) / np.float32(32.0)) + np.float32([0.25, -0.5][c])
    np.testing.assert_array_equal(O.linear_run(lin, x), expected)


def test_full_range_weights_are_exact():
    # crates/marian-cpu/src/q8_gemm.rs:671-693
    lin = O.make_linear(np.array([[127, 127, -127, -127]], np.int8), 1.0, 1.0)
    out = O.linear_run(lin, np.array([[127.0, 127.0, -127.0, -127.0]], np.float32))
    assert out.tolist() == [[64516.0]]


def _value_at(index):
    # crates/marian-cpu/src/q8_avx2.rs:375-382
    acts = [0, 1, 126, 127, 128, 253, 254, 255, 42]
    wts = [-128, -127, -64, -1, 0, 1, 63, 126, 127]
    return acts[index % 9], wts[(index * 7 + 3) % 9]


@pytest.mark.parametrize("length", [1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 383, 384, 385, 1536, 1537])
def test_every_tail_length_is_exact(length):
    # crates/marian-cpu/src/q8_avx2.rs:428-452
    pairs = [_value_at(i) for i in range(length)]
    a = np.array([p[0] for p in pairs], np.uint8).reshape(1, length)
    w = np.array([p[1] for p in pairs], np.int8).reshape(1, length)
    expected = sum((int(x) - 127) * int(y) for x, y in pairs)
    assert int(O.gemm_u8_i8(a, w)[0, 0]) == expected


def test_saturation_hazard_pairs_are_exact():
    # crates/marian-cpu/src/q8_avx2.rs:444-451
    a = np.full((1, 31), 254, np.uint8)
    w = np.full((1, 31), 127, np.int8)
    assert int(O.gemm_u8_i8(a, w)[0, 0]) == 127 * 127 * 31


def test_tiled_gemm_matches_scalar_oracle():
    # crates/marian-cpu/src/q8_avx2.rs:454-476
    rows, k, n = 3, 37, 7
    a = np.array([_value_at(i)[0] for i in range(rows * k)], np.uint8).reshape(rows, k)
    w = np.array([_value_at(i + 11)[1] for i in range(n * k)], np.int8).reshape(n, k)
    expected = (a.astype(np.int64) - 127) @ w.astype(np.int64).T
    np.testing.assert_array_equal(O.gemm_u8_i8(a, w), expected.astype(np.int32))


def test_residual_norm_is_per_row():
    # crates/marian-cpu/src/tensor.rs:919-930
    x = np.array([1.0, 2.0, 3.0, 4.0, 4.0, 3.0, 2.0, 1.0], np.float32).reshape(2, 4)
    out = O.residual_layer_norm(x, np.ones((2, 4), np.float32), np.ones(4, np.float32),
                                np.zeros(4, np.float32)).ravel()
    assert abs(out[0] + out[4]) < 1e-6
    assert abs(out[3] + out[7]) < 1e-6
    assert abs(out[:4].sum()) < 1e-6
    assert abs(out[4:].sum()) < 1e-6


def test_attention_masks_padded_keys():
    # crates/marian-cpu/src/tensor.rs:932-941
    out = O.attention([1.0, 0.0], [1.0, 0.0, 100.0, 0.0], [3.0, 4.0, 99.0, 99.0], [1], 1, 1, 2, 2, 1)
    assert out.tolist() == [3.0, 4.0]


def test_ssru_updates_state_before_normalizing():
    # crates/marian-cpu/src/tensor.rs:943-962
    out, state = O.ssru_update_layer_norm([[2.0, -2.0]], [[0.0, 0.0]], [[0.0, 2.0]], [[0.0, 0.0]],
                                          [1.0, 1.0], [0.0, 0.0])
    assert state.ravel().tolist() == [1.0, 0.0]
    assert abs(out[0, 0] - 0.999998) < 1e-5
    assert abs(out[0, 1] + 0.999998) < 1e-5


def test_argmax_is_stable_on_equal_logits():
    # crates/marian-cpu/src/tensor.rs:964-970 (restated for the Q8 selector,
    # q8_engine.rs:749-790): equal logits keep the earliest candidate.
    emb = np.array([[1, 0], [1, 0]], np.int8)
    tok = O.select_token(np.array([1.0, 2.0], np.float32), emb, 1.0, 1.0,
                         np.zeros(2, np.float32), np.array([1, 0], np.uint32))
    assert tok == 1


def test_positions_are_grouped_sin_then_cos():
    # crates/marian-model/src/position.rs:27-38
    p = O.positions(384)
    assert p[0] == 0.0 and p[191] == 0.0
    assert p[192] == 1.0 and p[383] == 1.0
    assert abs(p[384] - math.sin(1.0)) < 1e-7
    assert abs(p[384 + 192] - math.cos(1.0)) < 1e-7
    with pytest.raises(ValueError):
        O.positions(3)


def test_full_vocabulary_masks_control_tokens():
    # crates/marian-model/src/shortlist.rs:261-270
    c = O.full_vocab_candidates(64).tolist()
    assert 1 not in c
    assert all(i not in c for i in range(7, 39))
    assert 0 in c and 63 in c
    # 32000-token vocabulary: everything but 1 and 7..38
    assert len(O.full_vocab_candidates(32000)) == 32000 - 1 - 32


# ---- lexical shortlist (marian-model/src/shortlist.rs) ------------------------

def test_shortlist_full_vocabulary_masks_control_tokens():
    # shortlist.rs:259-266: no file, 64-id vocabulary, sentence [0, 63]
    c = O.shortlist_candidates(None, 64, 64, [0, 63])
    assert 1 not in c and not any(i in c for i in range(7, 39))
    assert 0 in c and 63 in c


def test_shortlist_must_supply_eos():
    # shortlist.rs:268-277: firstNum 0, source id 0 -> target 2 only
    sl = O.parse_shortlist(W.shortlist_bytes(0, [0, 1], [2]), 1, 64)
    with pytest.raises(ValueError, match="lexical shortlist does not contain EOS token 0"):
        O.shortlist_candidates(sl, 1, 64, [0])


def test_shortlist_entry_count_is_bounded():
    # shortlist.rs:279-291: a target count of MAX_TARGET_ENTRIES + 1 is rejected
    b = bytearray(W.shortlist_bytes(0, [0, 0], []))
    b[40:48] = (O.SHORTLIST_MAX_TARGET_ENTRIES + 1).to_bytes(8, "little")
    with pytest.raises(ValueError):
        O.parse_shortlist(bytes(b), 1, 64)


def test_shortlist_candidates_are_padded_to_multiples_of_eight():
    # shortlist.rs:185-192: 3 candidates {0, 2, 3} gain the first 5 absent ids from 50
    sl = O.parse_shortlist(W.shortlist_bytes(0, [0, 3], [0, 2, 3]), 1, 64)
    assert O.shortlist_candidates(sl, 1, 64, [0]).tolist() == [0, 2, 3, 50, 51, 52, 53, 54]
    # firstNum 10 marks 0..9; 1 and 7..9 are masked, 40 and 60 come from the token
    sl = O.parse_shortlist(W.shortlist_bytes(10, [0, 0, 2], [40, 60]), 2, 64)
    assert O.shortlist_candidates(sl, 2, 64, [1, 0]).tolist() == [0, 2, 3, 4, 5, 6, 40, 60]


def test_shortlist_parser_rejects_malformed_files():
    good = W.shortlist_bytes(0, [0, 1, 2], [0, 5])
    O.parse_shortlist(good, 2, 64)
    for bad, msg in ((good[:40], "truncated"), (good + b"\0", "expected"),
                     (W.shortlist_bytes(0, [0, 2, 1], [0, 5]), "offsets are invalid"),
                     (W.shortlist_bytes(0, [0, 1, 2], [0, 64]), "exceeds vocabulary"),
                     (W.shortlist_bytes(65, [0, 1, 2], [0, 5]), "unsupported")):
        with pytest.raises(ValueError, match=msg):
            O.parse_shortlist(bad, 2, 64)


def test_synthetic_shortlist_round_trips():
    raw = W.synthetic_shortlist(300, 512, seed=4, first_num=16, max_per_token=8)
    first, offs, tg = O.parse_shortlist(raw, 300, 512)
    assert first == 16 and offs.size == 301 and tg.size == int(offs[-1])
    c = O.shortlist_candidates((first, offs, tg), 300, 512, [5, 17, 0])
    assert c[0] == 0 and c.size % 8 == 0 and np.all(np.diff(c.astype(np.int64)) > 0)
