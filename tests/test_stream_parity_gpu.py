"""Parity on the benchmark's own request distribution.

The throughput workloads draw lognormal(ln 24, 0.8) source lengths clipped to
4..256 tokens, so the engine spends its time in encoder-attention launches of
the <=128 and <=256 length buckets and in decode attention over up to 256
cross keys and 256 cached self keys -- at head_dim 64 (graph_b) and 48
(graph_r).  These tests run exactly those kernel configurations against the
CPU oracle (the reference's Q8 engine restated, q8_engine.rs:353-466):

* a seeded sample of the benchmark stream with sources forced into the
  65..128 and 129..256 buckets and rows that generate more than 200 tokens,
  served by the continuous batcher with 256 slots (several admissions, slot
  and page reuse); every sentence is compared with the oracle run on
  reference-legal sub-batches (limits.rs:3-7: B <= 256, B * Lmax^2 <= 65,536;
  a sentence's result does not depend on its batch);
* a config-3-shaped encoder pass: 256 lognormal sentences in one packed
  pass, whose encoder output and cross keys/values must be bit-identical to
  the oracle's.

Tokens must be identical, or differ only where the oracle's top-2 logit gap
at the first divergence is below 1e-3, in at most 1% of sentences.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

import oracle as O  # noqa: E402
from marian_cuda import workloads as W  # noqa: E402
from marian_cuda.backend import CudaEngine  # noqa: E402

NEAR_TIE = 1e-3
# source lengths (EOS included) planted into every sample: both long
# encoder buckets, their edges, and rows whose generation exceeds 200 steps
# (src 179 -> round(1.2 * 179) = 215 steps; src 255 -> the 256-step cap)
PLANTED = [65, 66, 100, 128, 129, 150, 180, 200, 230, 255, 256, 256]

_models = {}


def model(name):
    if name not in _models:
        _models[name] = W.synthetic_model(W.SHAPES[name], seed=0)
    return _models[name]


def bench_sample(n, seed, vocab=32000):
    rng = np.random.Generator(np.random.PCG64(seed))
    lens = W.lognormal_lengths(rng, n)
    lens[:len(PLANTED)] = PLANTED
    lens = lens[rng.permutation(n)]
    return W.pack([W.zipf_ids(rng, int(l) - 1, vocab) for l in lens])


def oracle_by_row(om, batch, trace):
    """Translates every reference-legal sub-batch on the host's cores (the
    oracle is reentrant; ctypes releases the GIL).  Returns per-row token
    arrays, per-row top-2 gaps, and the per-group traces."""
    groups = W.legal_cpu_batches(batch)

    def run(grp):
        sb = W.subset(batch, grp)
        return grp, om.translate(sb.tokens, sb.offsets, sb.max_out, sb.force_len, trace=True)

    rows, gaps, traces = {}, {}, []
    with ThreadPoolExecutor(max_workers=max(1, min(32, os.cpu_count() or 1))) as ex:
        for grp, (toks, offs, tr) in ex.map(run, groups):
            for j, r in enumerate(grp):
                rows[r] = toks[offs[j]:offs[j + 1]]
                gaps[r] = tr["top2_gap"][j]
            if trace:
                traces.append((grp, tr))
    return rows, gaps, traces


def compare(batch, got, got_off, rows, gaps):
    identical, ties = 0, []
    for b in range(batch.size):
        g, r = got[got_off[b]:got_off[b + 1]], rows[b]
        if len(g) == len(r) and np.array_equal(g, r):
            identical += 1
            continue
        m = min(len(g), len(r))
        k = next(i for i in range(m + 1) if i == m or g[i] != r[i])
        assert k < 256 and gaps[b][k] < NEAR_TIE, f"row {b} diverges at step {k} (gap {gaps[b][k]})"
        ties.append(b)
    assert len(ties) <= batch.size // 100, f"{len(ties)} near-tie divergences in {batch.size} rows"
    return identical


@pytest.mark.parametrize("name", ["graph_b", "graph_r"])
def test_benchmark_stream_sample_matches_oracle(name):
    batch = bench_sample(n=320, seed=20260 + len(name))
    lens = np.diff(batch.offsets.astype(np.int64))
    assert ((lens > 64) & (lens <= 128)).sum() >= 3 and (lens > 128).sum() >= 6
    limits = np.minimum(np.minimum(batch.force_len, 3 * lens), 256)
    assert (limits > 200).sum() >= 4
    mb = model(name)
    with CudaEngine(mb, max_inflight=256, max_encode_tokens=8192) as eng:
        got, got_off = eng.translate_token_ids(batch.tokens, batch.offsets, batch.max_out, batch.force_len)
    rows, gaps, _ = oracle_by_row(O.OracleModel(mb), batch, trace=False)
    out_lens = np.diff(got_off.astype(np.int64))
    assert out_lens.max() == 256  # the 256-step cap was reached
    compare(batch, got, got_off, rows, gaps)


@pytest.mark.parametrize("name", ["graph_b", "graph_r"])
def test_ragged_encoder_pass_of_256_sentences_is_bit_exact(name):
    # config 3's shape: 256 lognormal sentences packed into one encoder pass
    batch = bench_sample(n=256, seed=777 + len(name))
    batch.max_out[:] = 1  # the oracle only needs the encoder and step 0
    batch.force_len[:] = 1
    mb = model(name)
    with CudaEngine(mb, max_inflight=256, max_encode_tokens=16384) as eng:
        gtr = eng.trace_first_step(batch.tokens, batch.offsets)
    _, _, traces = oracle_by_row(O.OracleModel(mb), batch, trace=True)
    lens = np.diff(batch.offsets.astype(np.int64))
    lmax = int(lens.max())
    checked = 0
    for grp, tr in traces:
        sl = int(max(lens[r] for r in grp))
        for j, row in enumerate(grp):
            n = int(lens[row])
            g_rows = slice(row * lmax, row * lmax + n)
            r_rows = slice(j * sl, j * sl + n)
            np.testing.assert_array_equal(gtr["encoder_output"][g_rows], tr["encoder_output"][r_rows])
            np.testing.assert_array_equal(gtr["cross_key"][:, g_rows], tr["cross_key"][:, r_rows])
            np.testing.assert_array_equal(gtr["cross_value"][:, g_rows], tr["cross_value"][:, r_rows])
            st, rs = gtr["decoder_state_step0"][row], tr["decoder_state_step0"][j]
            assert np.abs(st - rs).max() <= 1e-6 * np.abs(rs).max()
            checked += 1
    assert checked == batch.size
