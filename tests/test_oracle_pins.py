"""CPU: the oracle against the golden fixtures (tests/golden/make_golden.py,
tests/golden/make_q81_pin.py) and the reference's own relative properties."""
import os
import sys

import numpy as np
import pytest

import oracle
from malaga_b200 import convert as C
from malaga_b200 import gguf_io as G

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_oracle_matches_transformers_m2m100_on_tiny_model(model):
    """f32 semantics pin: identical greedy ids over 16 steps for the 6 sentences of
    pipeline.rs:132-134, logits within 5e-3 (f16 KV rounding of the fused path)."""
    g = np.load(os.path.join(GOLDEN, "tiny_hf_greedy.npz"))
    src = [list(map(int, r[:l])) for r, l in zip(g["src_ids"], g["src_lens"])]
    orc = oracle.Oracle(model("tiny", "f32"))
    ids, logits = orc.greedy(src, int(g["tgt"]), g["tokens"].shape[1], force=True, logits=True)
    np.testing.assert_array_equal(ids, g["tokens"])
    np.testing.assert_allclose(logits, g["logits"], atol=5e-3, rtol=1e-3)


def test_dequantization_matches_gguf_py(tmp_path):
    """Block layouts pin: our quantizer is deterministic, and the oracle dequantizes
    its Q8_0 / Q4_K / Q6_K blocks exactly as gguf-py does."""
    g = np.load(os.path.join(GOLDEN, "dequant_golden.npz"))
    x = g["x"]
    plans = []
    for t, name in ((G.Q8_0, "Q8_0"), (G.Q4_K, "Q4_K"), (G.Q6_K, "Q6_K")):
        q = C.quantize(x, t).reshape(x.shape[0], -1)
        np.testing.assert_array_equal(q, g[f"{name}_bytes"])
        plans.append(G.TensorPlan(f"t.{name}", x.shape, t, lambda q=q: q))
    path = str(tmp_path / "blocks.gguf")
    G.write_gguf(path, [("general.architecture", "nllb")], plans)
    lib = oracle.lib()
    h = lib.orc_load(path.encode())
    try:
        for name in ("Q8_0", "Q4_K", "Q6_K"):
            want = g[f"{name}_deq"]
            got = np.array([[lib.orc_dequant(h, f"t.{name}".encode(), r, j) for j in range(x.shape[1])]
                            for r in range(x.shape[0])], np.float32)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name
    finally:
        lib.orc_free(h)


def test_exp_and_log_accuracy():
    L = oracle.lib()
    rng = np.random.default_rng(0)
    xs = np.concatenate([-np.abs(rng.standard_normal(4000) * 20), np.linspace(-87, 0, 2000)]).astype(np.float32)
    e = np.array([L.orc_exp(float(v)) for v in xs], np.float32)
    ref = np.exp(xs.astype(np.float64))
    assert (np.abs(e - ref) / np.spacing(ref.astype(np.float32))).max() <= 1.0
    assert L.orc_exp(float("-inf")) == 0.0
    ys = np.exp(rng.uniform(-80, 80, 4000)).astype(np.float32)
    lg = np.array([L.orc_log(float(v)) for v in ys], np.float32)
    rl = np.log(ys.astype(np.float64))
    assert (np.abs(lg - rl) / np.spacing(np.abs(rl).astype(np.float32))).max() <= 2.0


def test_log_softmax_topk_semantics():
    """translator.rs:343-358: k argmax passes -- larger value first, lower index
    on ties, each index once; log_softmax values match float64 to a few ulp."""
    rng = np.random.default_rng(5)
    x = np.stack([rng.integers(-2, 3, 1000).astype(np.float32), rng.standard_normal(1000).astype(np.float32)])
    vals, idx = oracle.log_softmax_topk(x, 6)
    for r in range(2):
        want = sorted(range(1000), key=lambda i: (-x[r, i], i))[:6]
        assert list(idx[r]) == want
        ref = x[r].astype(np.float64) - x[r].max()
        ref = ref - np.log(np.exp(ref).sum())
        np.testing.assert_allclose(vals[r], ref[want], rtol=0, atol=1e-5)
    v, i = oracle.log_softmax_topk(np.array([[3.0, 1.0]], np.float32), 4)  # fewer values than k
    assert list(i[0]) == [0, 1, 0, 0] and np.isneginf(v[0, 2:]).all()


def _tiny_src():
    return [[254] + C.tiny_sentence(3 + 4 * i, i) + [2] for i in range(6)]


def test_batching_does_not_change_outputs(model):
    """pipeline.rs:45-57 (batch == single, f32 preset). Quantized presets are not
    batch-invariant in the reference (MMVQ below 9 rows, MMQ above, different
    warp counts: docs/performance.md:51-54) and not here either."""
    orc = oracle.Oracle(model("tiny", "f32"))
    src = _tiny_src()
    batched = orc.greedy(src, 256, 12)
    for i, s in enumerate(src):
        np.testing.assert_array_equal(orc.greedy([s], 256, 12)[0], batched[i])


def test_beam_one_is_greedy_and_beam_is_deterministic(model):
    """pipeline.rs:60-69."""
    orc = oracle.Oracle(model("tiny", "f32"))
    src = [[254] + C.tiny_sentence(8, 3) + [2]]
    greedy = oracle.strip_eos(orc.greedy(src, 256, 20)[0], 2)
    assert [int(t) for t in orc.beam(src, 256, 1, 20)[0]] == greedy
    assert orc.beam(src, 256, 3, 20) == orc.beam(src, 256, 3, 20)


def _pin_cases():
    g = np.load(os.path.join(GOLDEN, "q81_pin.npz"))
    return g, [tuple(int(v) for v in c) for c in g["cases"]], [int(r) for r in g["rows"]]


def test_q81_matmuls_match_an_independent_build_of_the_published_kernels():
    """Quantized-arithmetic pin: the oracle's restatement of the reference's q8_1
    matmuls (candle-kernels 0.11.0 quantize_q8_1, MMVQ, MMQ) against vLLM's
    compiled port of the same llama.cpp kernels, run on a B200 by
    tests/golden/make_q81_pin.py: bit-identical outputs for Q8_0 / Q4_K / Q6_K,
    K = 1024 and 4096, 1-64 activation rows, quantizer edge cases included.
    vLLM launches MMVQ with one warp per row, i.e. the oracle's nw = 1; candle's
    launch (4 warps up to 4 rows, 2 up to 8) only regroups the same per-thread
    sums."""
    sys.path.insert(0, GOLDEN)
    import make_q81_pin as M

    g, cases, rows_list = _pin_cases()
    for ci, (t, n, k) in enumerate(cases):
        w = g[f"w{ci}"]
        for rows in rows_list:
            x = M.activations(rows, k, 1000 * ci + rows)
            np.testing.assert_allclose(g[f"xsum{ci}_{rows}"], [x.astype(np.float64).sum(),
                                                               np.abs(x).astype(np.float64).sum()])
            if f"vec{ci}_{rows}" in g:
                y = oracle.matmul(t, w, n, k, x, "mmvq", nw=1)
                want = g[f"vec{ci}_{rows}"]
                assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), ("mmvq", t, k, rows)
            y = oracle.matmul(t, w, n, k, x, "mmq")
            want = g[f"mmq{ci}_{rows}"]
            assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), ("mmq", t, k, rows)


def test_q81_quantizer_edge_cases():
    """quantize_q8_1: d = amax/127, q = roundf(x/d) (halves away from zero), all-zero
    blocks give q = 0 and d = 0, d and the block sum rounded to f16."""
    x = np.zeros((1, 128), np.float32)
    x[0, 32:64] = np.float32(0.5) * np.arange(-16, 16, dtype=np.float32)
    x[0, 64] = 127.0
    x[0, 65:96] = 2.5
    x[0, 96] = -3.0
    q, d, s = oracle.quantize_q81(x)
    assert not q[0, :32].any() and d[0, 0] == 0.0
    assert d[0, 2] == 1.0 and q[0, 64] == 127 and (q[0, 65:96] == 3).all()
    assert q[0, 96] == -127 and np.float16(d[0, 3]) == np.float16(3.0 / 127)
    assert s[0, 1] == np.float16(x[0, 32:64].sum())
