"""mc_q8_linear (Q8Linear::run_into on the device) against the oracle's
linear: quantization, exact int32 GEMM and the two-rounding epilogue make
the f32 outputs bit-exact (q8_gemm.rs:380-448)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from marian_cuda import _lib as L  # noqa: E402


def run_linear(x, w, a_mult, w_mult, bias=None):
    lib = L.load()
    m, k = x.shape
    n = w.shape[0]
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    wd = torch.from_numpy(np.ascontiguousarray(w, np.int8)).cuda()
    bd = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias, np.float32)).cuda()
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    st = lib.mc_q8_linear(xd.data_ptr(), m, k, wd.data_ptr(), n, a_mult, w_mult,
                          None if bd is None else bd.data_ptr(), y.data_ptr(), None)
    assert st == L.MC_OK
    bits = C.c_uint32(0)
    assert lib.mc_op_status(C.byref(bits)) == L.MC_OK
    return y.cpu().numpy(), bits.value


def pad_k(x, w, k16):
    xp = np.zeros((x.shape[0], k16), np.float32)
    xp[:, :x.shape[1]] = x
    wp = np.zeros((w.shape[0], k16), np.int8)
    wp[:, :w.shape[1]] = w
    return xp, wp


@pytest.mark.parametrize("rows", [1, 2, 3, 4])
def test_reference_linear_vectors(rows):
    # q8_gemm.rs:620-668 (weights [2,-3,5,7,-11,13,-17,19], alpha 4, w 8,
    # bias [0.25, -0.5]); K padded 4 -> 16 with zeros, which quantize to 0.
    w = np.array([2, -3, 5, 7, -11, 13, -17, 19], np.int8).reshape(2, 4)
    vals = [0.0, 0.25, -0.5, 1.0, 1.25, -1.0, 0.5, -0.25, -2.0, 0.75, 1.5, 0.0, 0.5, 0.5, -0.5, -0.5]
    x = np.array(vals[:4 * rows], np.float32).reshape(rows, 4)
    bias = np.array([0.25, -0.5], np.float32)
    xp, wp = pad_k(x, w, 16)
    got, bits = run_linear(xp, wp, 4.0, 8.0, bias)
    assert bits == 0
    np.testing.assert_array_equal(got, O.linear_run(O.make_linear(w, 4.0, 8.0, bias), x))


@pytest.mark.parametrize("m,k,n", [(333, 512, 1536), (7, 2048, 512), (64, 512, 2048), (5, 512, 32000)])
def test_random_linears_bit_exact(m, k, n):
    rng = np.random.default_rng(m + k + n)
    x = rng.normal(0, 1.0, size=(m, k)).astype(np.float32)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    a_mult, w_mult = np.float32(25.3), np.float32(1700.5)
    got, bits = run_linear(x, w, a_mult, w_mult, bias)
    assert bits == 0
    np.testing.assert_array_equal(got, O.linear_run(O.make_linear(w, a_mult, w_mult, bias), x))


def test_non_finite_activation_is_reported():
    x = np.zeros((4, 16), np.float32)
    x[2, 5] = np.nan
    w = np.ones((3, 16), np.int8)
    _, bits = run_linear(x, w, 1.0, 1.0)
    assert bits & 1


def test_quantization_ties_and_clamps_reference_vector():
    # q8_gemm.rs:609-617: multiplier 1 quantizes
    # [-200, -127.6, -126.5, -1.5, -0.5, 0.5, 1.5, 126.5, 127.6, 200] to the u8
    # values [0, 0, 1, 125, 127, 127, 129, 253, 254, 254] (ties to even,
    # clamped to +-127 around the zero point 127).  An identity weight matrix
    # with both multipliers 1 returns the centred integers as the outputs.
    x = np.zeros((1, 16), np.float32)
    x[0, :10] = [-200.0, -127.6, -126.5, -1.5, -0.5, 0.5, 1.5, 126.5, 127.6, 200.0]
    w = np.eye(16, dtype=np.int8)
    got, bits = run_linear(x, w, 1.0, 1.0)
    assert bits == 0
    u8 = np.array([0, 0, 1, 125, 127, 127, 129, 253, 254, 254], np.float32)
    np.testing.assert_array_equal(got[0, :10], u8 - 127.0)
    np.testing.assert_array_equal(got[0, 10:], 0.0)
    np.testing.assert_array_equal(O.quantize_u8(x[0, :10], 1.0), u8.astype(np.uint8))
