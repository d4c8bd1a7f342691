"""mc_q8_linear_noalloc: the Q8 linear for callers that cannot allocate
device memory (a host whose memory manager owns the GPU's memory, or a
latency-critical path that cannot take an allocation).  Its scratch is a
fixed device array; its results must equal the oracle's Q8 linear and
mc_q8_linear's (which allocates its scratch per call) bit for bit, on
consecutive calls that reuse the same array.  This file runs last so a
failure here leaves every other test run.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from marian_cuda import _lib as L  # noqa: E402


def _linear(lib, fn, x, w, bias, a_mult, w_mult, want_bits=True):
    m, k = x.shape
    n = w.shape[0]
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    if fn == "alloc":
        st = lib.mc_q8_linear(x.data_ptr(), m, k, w.data_ptr(), n, a_mult, w_mult, bias.data_ptr(),
                              y.data_ptr(), None)
        assert st == L.MC_OK
        bits = C.c_uint32(0)
        assert lib.mc_op_status(C.byref(bits)) == L.MC_OK
        value = bits.value
    else:
        bits = C.c_uint32(0xFFFF)
        st = lib.mc_q8_linear_noalloc(x.data_ptr(), m, k, w.data_ptr(), n, a_mult, w_mult,
                                      bias.data_ptr(), y.data_ptr(), None,
                                      C.byref(bits) if want_bits else None)
        assert st == L.MC_OK
        value = bits.value if want_bits else None
    torch.cuda.synchronize()
    return y.cpu().numpy(), value


def _operands(rng, m, k, n):
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    return x, w, bias


def test_noalloc_linear_matches_oracle_and_allocating_linear_on_consecutive_calls():
    lib = L.load()
    rng = np.random.default_rng(2024)
    shapes = [(333, 512, 1536), (1024, 2048, 512)]  # two calls in a row, different sizes
    a_mult, w_mult = np.float32(25.0), np.float32(1700.0)
    for m, k, n in shapes:
        x, w, bias = _operands(rng, m, k, n)
        xd, wd, bd = (torch.from_numpy(v).cuda() for v in (x, w, bias))
        ref, ref_bits = _linear(lib, "alloc", xd, wd, bd, a_mult, w_mult)
        got, got_bits = _linear(lib, "noalloc", xd, wd, bd, a_mult, w_mult)
        assert ref_bits == 0 and got_bits == 0
        assert np.isfinite(got).all()
        np.testing.assert_array_equal(got, ref)  # the Q8 linear is bit-exact
        # and the CPU restatement of Q8Linear::run_into (q8_gemm.rs:380-448)
        np.testing.assert_array_equal(got, O.linear_run(O.make_linear(w, a_mult, w_mult, bias), x))


def test_noalloc_linear_accepts_exactly_its_maximum():
    lib = L.load()
    rng = np.random.default_rng(7)
    k = 2048
    m = L.NOALLOC_MAX_ACTIVATIONS // k  # m * k == the scratch size
    assert m * k == L.NOALLOC_MAX_ACTIVATIONS
    x, w, bias = _operands(rng, m, k, 48)
    xd, wd, bd = (torch.from_numpy(v).cuda() for v in (x, w, bias))
    got, bits = _linear(lib, "noalloc", xd, wd, bd, np.float32(25.0), np.float32(1700.0))
    assert bits == 0
    ref, _ = _linear(lib, "alloc", xd, wd, bd, np.float32(25.0), np.float32(1700.0))
    np.testing.assert_array_equal(got, ref)
    rows = rng.choice(m, size=64, replace=False)  # the oracle on a sample of the rows
    np.testing.assert_array_equal(
        got[rows], O.linear_run(O.make_linear(w, np.float32(25.0), np.float32(1700.0), bias), x[rows]))


def test_noalloc_status_bits_report_clear_and_accumulate():
    lib = L.load()
    rng = np.random.default_rng(11)
    x, w, bias = _operands(rng, 8, 64, 32)
    bad = x.copy()
    bad[3, 7] = np.nan
    args = [torch.from_numpy(v).cuda() for v in (x, bad, w, bias)]
    xd, badd, wd, bd = args
    _, bits = _linear(lib, "noalloc", badd, wd, bd, 25.0, 1700.0)
    assert bits & 1  # non-finite activation, reported
    _, bits = _linear(lib, "noalloc", xd, wd, bd, 25.0, 1700.0)
    assert bits == 0  # ... and cleared by that report
    _linear(lib, "noalloc", badd, wd, bd, 25.0, 1700.0, want_bits=False)
    _, bits = _linear(lib, "noalloc", xd, wd, bd, 25.0, 1700.0)
    assert bits & 1  # without a report the bit accumulates into the next one
    _, bits = _linear(lib, "noalloc", xd, wd, bd, 25.0, 1700.0)
    assert bits == 0


def test_noalloc_linear_rejects_sizes_beyond_its_scratch():
    lib = L.load()
    k = 2048
    m = L.NOALLOC_MAX_ACTIVATIONS // k + 1  # one row past the fixed scratch
    x = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    w = torch.zeros((16, k), dtype=torch.int8, device="cuda")
    y = torch.zeros((m, 16), dtype=torch.float32, device="cuda")
    st = lib.mc_q8_linear_noalloc(x.data_ptr(), m, k, w.data_ptr(), 16, 1.0, 1.0, None, y.data_ptr(),
                                  None, None)
    assert st == L.MC_INVALID_INPUT
