"""tcgen05 int8 GEMM through the C ABI against exact integer arithmetic and
the oracle's epilogue (q8_gemm.rs:380-448 semantics).

The (K, N) x M grid is the GEMM microbenchmark's: K, N in {(512,1536),
(512,2048), (2048,512), (512,32000)} and ragged M in {1, 7, 64, 333, 1024,
4096}.  Accumulators must be bit-exact; the f32 epilogue must be bit-exact as
well because it is the same two IEEE roundings (acc*scale, +bias).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _lib():
    from marian_cuda import _lib as L
    return L.load(), L


def _exact_acc(a, w):
    # float64 BLAS is exact here: |sum| <= 2048 * 127 * 127 < 2^53
    return (a.astype(np.float64) @ w.astype(np.float64).T).astype(np.int64).astype(np.int32)


def _run(lib, a_d, w_d, m, n, k, mode, out, col_scale=None, row_scale=None, bias=None, residual=None, relu=0):
    ptr = lambda t: None if t is None else t.data_ptr()
    st = lib.mc_q8_gemm(ptr(a_d), ptr(w_d), m, n, k, ptr(row_scale), ptr(col_scale), ptr(bias),
                        ptr(residual), relu, mode, ptr(out), None)
    assert st == 0
    bits = C.c_uint32(0)
    assert lib.mc_op_status(C.byref(bits)) == 0
    assert bits.value == 0


SHAPES = [(512, 1536), (512, 2048), (2048, 512), (512, 32000)]
MS = [1, 7, 64, 333, 1024, 4096]


@pytest.mark.parametrize("k,n", SHAPES)
def test_accumulators_bit_exact(k, n):
    lib, _ = _lib()
    rng = np.random.default_rng(k * 7 + n)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    w_d = torch.from_numpy(w).cuda()
    for m in MS:
        a = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
        a_d = torch.from_numpy(a).cuda()
        out = torch.empty((m, n), dtype=torch.int32, device="cuda")
        _run(lib, a_d, w_d, m, n, k, 0, out)
        got = out.cpu().numpy()
        np.testing.assert_array_equal(got, _exact_acc(a, w), err_msg=f"m={m} k={k} n={n}")


@pytest.mark.parametrize("k,n", [(512, 1536), (2048, 512)])
def test_f32_epilogue_bit_exact_vs_oracle(k, n):
    import oracle as O
    lib, _ = _lib()
    rng = np.random.default_rng(11)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    w_d = torch.from_numpy(w).cuda()
    col_scale = (1.0 / (rng.uniform(0.001, 0.02, n) * 3.0)).astype(np.float32) * np.float32(1e-4)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    for m in (7, 333):
        a = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
        row_scale = rng.uniform(0.001, 0.02, m).astype(np.float32)
        residual = rng.normal(size=(m, n)).astype(np.float32)
        acc = _exact_acc(a, w)
        for relu, rs, res in ((0, None, None), (1, row_scale, None), (0, row_scale, residual)):
            out = torch.empty((m, n), dtype=torch.float32, device="cuda")
            t = lambda x: None if x is None else torch.from_numpy(x).cuda()
            _run(lib, torch.from_numpy(a).cuda(), w_d, m, n, k, 1, out, t(col_scale), t(rs), t(bias),
                 t(res), relu)
            expected = O.epilogue(acc, col_scale, bias, rs, bool(relu), res)
            np.testing.assert_array_equal(out.cpu().numpy(), expected)


def test_reference_linear_golden_padded_k():
    # q8_gemm.rs:620-668 vectors; K padded from 4 to 16 with zeros (zero
    # columns leave every integer dot product unchanged).
    import oracle as O
    lib, _ = _lib()
    w4 = np.array([2, -3, 5, 7, -11, 13, -17, 19], np.int8).reshape(2, 4)
    x = np.array([0.0, 0.25, -0.5, 1.0, 1.25, -1.0, 0.5, -0.25, -2.0, 0.75, 1.5, 0.0,
                  0.5, 0.5, -0.5, -0.5], np.float32).reshape(4, 4)
    q = (O.quantize_u8(x, 4.0).astype(np.int16) - 127).astype(np.int8)
    a = np.zeros((4, 16), np.int8); a[:, :4] = q
    w = np.zeros((2, 16), np.int8); w[:, :4] = w4
    out = torch.empty((4, 2), dtype=torch.float32, device="cuda")
    cs = torch.full((2,), 1.0 / 32.0, dtype=torch.float32, device="cuda")
    b = torch.tensor([0.25, -0.5], dtype=torch.float32, device="cuda")
    _run(lib, torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(), 4, 2, 16, 1, out, cs, None, b)
    lin = O.make_linear(w4, 4.0, 8.0, np.array([0.25, -0.5], np.float32))
    np.testing.assert_array_equal(out.cpu().numpy(), O.linear_run(lin, x))


def test_full_range_is_exact():
    # q8_gemm.rs:671-693: [127,127,-127,-127] . [127,127,-127,-127] = 64516
    lib, _ = _lib()
    a = np.zeros((1, 16), np.int8); a[0, :4] = [127, 127, -127, -127]
    w = np.zeros((1, 16), np.int8); w[0, :4] = [127, 127, -127, -127]
    out = torch.empty((1, 1), dtype=torch.int32, device="cuda")
    _run(lib, torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(), 1, 1, 16, 0, out)
    assert int(out.item()) == 64516


def test_rejects_bad_shapes():
    lib, L = _lib()
    a = torch.zeros((4, 16), dtype=torch.int8, device="cuda")
    out = torch.empty((4, 4), dtype=torch.int32, device="cuda")
    assert lib.mc_q8_gemm(a.data_ptr(), a.data_ptr(), 4, 4, 15, None, None, None, None, 0, 0,
                          out.data_ptr(), None) == L.MC_INVALID_INPUT
