"""The fused linear + residual + LayerNorm kernel (csrc/linear_ln.cu).

mc_q8_linear_ln must equal the oracle's Q8Linear::run_into followed by its
residual_layer_norm_into (q8_gemm.rs:380-448, tensor.rs:132-155) bit for
bit: the int32 GEMM is exact, the dequantization keeps two roundings, the
mean and the variance are the reference's left-to-right sums, and the
quantized copy is quantize_symmetric_u8_into's (q8_gemm.rs:609-617).  Row
counts cover partial 128-row blocks, one row, and the decode capacity;
widths are every one the kernel supports (the cluster splits columns 4 or
8 ways); K covers the attention output (K = d) and FFN W2 (K = 4 d).

Inside the engine, decode steps use the kernel for the three sub-layer
ends; MARIAN_CUDA_FUSED_LN=0 selects the separate GEMM and LayerNorm
kernels, and the two engines must agree bit for bit.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from marian_cuda import _lib as L  # noqa: E402
from marian_cuda import workloads as W  # noqa: E402
from marian_cuda.backend import CudaEngine  # noqa: E402


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_fused(x, w, a_mult, w_mult, bias, residual, gamma, beta, y_alpha=None):
    lib = L.load()
    m, k = x.shape
    d = w.shape[0]
    xd, wd, rd, gd, btd = (_dev(v) for v in (x, w, residual, gamma, beta))
    bd = None if bias is None else _dev(bias)
    y = torch.full((m, d), float("nan"), dtype=torch.float32, device="cuda")
    yq = None if y_alpha is None else torch.zeros((m, d), dtype=torch.int8, device="cuda")
    st = lib.mc_q8_linear_ln(xd.data_ptr(), m, k, wd.data_ptr(), d, a_mult, w_mult,
                             None if bd is None else bd.data_ptr(), rd.data_ptr(), gd.data_ptr(),
                             btd.data_ptr(), y.data_ptr(), None if yq is None else yq.data_ptr(),
                             0.0 if y_alpha is None else y_alpha, None)
    assert st == L.MC_OK
    bits = C.c_uint32(0)
    assert lib.mc_op_status(C.byref(bits)) == L.MC_OK
    return y.cpu().numpy(), None if yq is None else yq.cpu().numpy(), bits.value


def oracle_linear_ln(x, w, a_mult, w_mult, bias, residual, gamma, beta):
    lin = O.linear_run(O.make_linear(w, a_mult, w_mult, bias), x)
    return O.residual_layer_norm(lin, residual, gamma, beta)


def operands(rng, m, k, d, bias=True):
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    w = rng.integers(-127, 128, size=(d, k), dtype=np.int8)
    b = rng.uniform(-0.5, 0.5, d).astype(np.float32) if bias else None
    r = rng.normal(0, 2, size=(m, d)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, d).astype(np.float32)
    be = rng.uniform(-0.2, 0.2, d).astype(np.float32)
    return x, w, b, r, g, be


@pytest.mark.parametrize("d", [512, 384, 256, 128])
@pytest.mark.parametrize("m", [1, 77, 128, 129, 1024])
@pytest.mark.parametrize("kf", [1, 4])
def test_fused_linear_ln_matches_oracle(d, m, kf):
    rng = np.random.default_rng(1000 * d + 10 * m + kf)
    k = kf * d
    x, w, b, r, g, be = operands(rng, m, k, d)
    a_mult, w_mult, y_alpha = np.float32(23.5), np.float32(1650.25), np.float32(31.0)
    got, got_q, bits = run_fused(x, w, a_mult, w_mult, b, r, g, be, y_alpha)
    assert bits == 0
    ref = oracle_linear_ln(x, w, a_mult, w_mult, b, r, g, be)
    np.testing.assert_array_equal(got, ref)
    ref_q = O.quantize_u8(ref, y_alpha).astype(np.int16) - 127  # centred, as the kernels store it
    np.testing.assert_array_equal(got_q.astype(np.int16), ref_q)


def test_fused_linear_ln_without_bias_and_copies():
    rng = np.random.default_rng(5)
    x, w, _, r, g, be = operands(rng, 300, 512, 512, bias=False)
    got, _, bits = run_fused(x, w, 30.0, 1000.0, None, r, g, be)
    assert bits == 0
    np.testing.assert_array_equal(got, oracle_linear_ln(x, w, 30.0, 1000.0, None, r, g, be))


def test_fused_linear_ln_reports_non_finite_rows():
    rng = np.random.default_rng(9)
    x, w, b, r, g, be = operands(rng, 200, 512, 512)
    r[150, 3] = np.inf  # row 150 normalizes to NaN: its quantized copy is an error
    got, _, bits = run_fused(x, w, 30.0, 1000.0, b, r, g, be, y_alpha=10.0)
    assert bits & 1
    ok = np.arange(200) != 150
    np.testing.assert_array_equal(got[ok], oracle_linear_ln(x[ok], w, 30.0, 1000.0, b, r[ok], g, be))


def test_fused_linear_ln_rejects_unsupported_widths():
    lib = L.load()
    x = torch.zeros((4, 640), dtype=torch.float32, device="cuda")
    w = torch.zeros((640, 640), dtype=torch.int8, device="cuda")
    v = torch.zeros(640, dtype=torch.float32, device="cuda")
    st = lib.mc_q8_linear_ln(x.data_ptr(), 4, 640, w.data_ptr(), 640, 1.0, 1.0, None, x.data_ptr(),
                             v.data_ptr(), v.data_ptr(), x.data_ptr(), None, 0.0, None)
    assert st == L.MC_INVALID_INPUT


def _engine_run(mb, batch, fused):
    old = os.environ.get("MARIAN_CUDA_FUSED_LN")
    os.environ["MARIAN_CUDA_FUSED_LN"] = "1" if fused else "0"
    try:
        with CudaEngine(mb, max_inflight=256, max_encode_tokens=8192) as eng:
            got, off = eng.translate_token_ids(batch.tokens, batch.offsets, batch.max_out, batch.force_len)
            head = W.subset(batch, list(range(64)))  # one encoder pass
            tr = eng.trace_first_step(head.tokens, head.offsets)
    finally:
        if old is None:
            del os.environ["MARIAN_CUDA_FUSED_LN"]
        else:
            os.environ["MARIAN_CUDA_FUSED_LN"] = old
    return got, off, tr


@pytest.mark.parametrize("name", ["graph_b", "graph_r", "tiny_self", "tiny_self_ffn4", "mid_self"])
def test_engine_fused_and_separate_layernorm_agree_bit_for_bit(name):
    mb = W.synthetic_model(W.SHAPES[name], seed=3)
    rng = np.random.Generator(np.random.PCG64(44))
    lens = W.lognormal_lengths(rng, 300)
    batch = W.pack([W.zipf_ids(rng, int(n) - 1, W.SHAPES[name].vocab) for n in lens])
    a_tok, a_off, a_tr = _engine_run(mb, batch, fused=True)
    b_tok, b_off, b_tr = _engine_run(mb, batch, fused=False)
    np.testing.assert_array_equal(a_off, b_off)
    np.testing.assert_array_equal(a_tok, b_tok)
    np.testing.assert_array_equal(a_tr["decoder_state_step0"], b_tr["decoder_state_step0"])


@pytest.mark.parametrize("name", ["tiny_self_ffn4", "mid_self"])
def test_engine_with_fused_second_linears_matches_oracle(name):
    # d = 128 (clusters of 4) and d = 256 (clusters of 8) with FFN 4d: every
    # decoder sub-layer end runs fused, two of them with a second linear.
    # The oracle runs reference-legal sub-batches (limits.rs:3-7).
    mb = W.synthetic_model(W.SHAPES[name], seed=5)
    om = O.OracleModel(mb)
    full = W.short_batch(n=48, vocab=W.SHAPES[name].vocab, seed=9)
    with CudaEngine(mb, max_inflight=256, max_encode_tokens=8192) as eng:
        got, got_off = eng.translate_token_ids(full.tokens, full.offsets, full.max_out, full.force_len)
    for grp in W.legal_cpu_batches(full):
        b = W.subset(full, grp)
        ref, ref_off, tr = om.translate(b.tokens, b.offsets, b.max_out, b.force_len, trace=True)
        for j, row in enumerate(grp):
            g, r = got[got_off[row]:got_off[row + 1]], ref[ref_off[j]:ref_off[j + 1]]
            if len(g) == len(r) and np.array_equal(g, r):
                continue
            m = min(len(g), len(r))
            k = next(i for i in range(m + 1) if i == m or g[i] != r[i])
            assert k < 256 and tr["top2_gap"][j, k] < 1e-3, f"row {row} diverges at step {k}"
