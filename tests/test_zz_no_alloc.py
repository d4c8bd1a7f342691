"""mc_q8_linear_noalloc: the Q8 linear for callers that cannot allocate
device memory (a host whose memory manager owns the GPU's memory, or a
latency-critical path that cannot take an allocation).  Its scratch is a
fixed device array; its results must equal mc_q8_linear's (which allocates
its scratch per call) bit for bit, on consecutive calls that reuse the same
array.  This file runs last so a failure here leaves every other test run.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from marian_cuda import _lib as L  # noqa: E402


def _linear(lib, fn, x, w, bias, a_mult, w_mult):
    m, k = x.shape
    n = w.shape[0]
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    if fn == "alloc":
        st = lib.mc_q8_linear(x.data_ptr(), m, k, w.data_ptr(), n, a_mult, w_mult, bias.data_ptr(),
                              y.data_ptr(), None)
        assert st == L.MC_OK
        bits = C.c_uint32(0)
        assert lib.mc_op_status(C.byref(bits)) == L.MC_OK
    else:
        bits = C.c_uint32(0xFFFF)
        st = lib.mc_q8_linear_noalloc(x.data_ptr(), m, k, w.data_ptr(), n, a_mult, w_mult,
                                      bias.data_ptr(), y.data_ptr(), None, C.byref(bits))
        assert st == L.MC_OK
    torch.cuda.synchronize()
    return y.cpu().numpy(), bits.value


def test_noalloc_linear_matches_allocating_linear_on_consecutive_calls():
    lib = L.load()
    rng = np.random.default_rng(2024)
    shapes = [(333, 512, 1536), (1024, 2048, 512)]  # two calls in a row, different sizes
    for m, k, n in shapes:
        x = torch.from_numpy(rng.normal(0, 1, size=(m, k)).astype(np.float32)).cuda()
        w = torch.from_numpy(rng.integers(-127, 128, size=(n, k), dtype=np.int8)).cuda()
        bias = torch.from_numpy(rng.uniform(-0.1, 0.1, n).astype(np.float32)).cuda()
        ref, ref_bits = _linear(lib, "alloc", x, w, bias, 25.0, 1700.0)
        got, got_bits = _linear(lib, "noalloc", x, w, bias, 25.0, 1700.0)
        assert ref_bits == 0 and got_bits == 0
        assert np.isfinite(got).all()
        np.testing.assert_array_equal(got, ref)  # the Q8 linear is bit-exact


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
